"""B200-native paged latent-cache decode (sm_100a) behind the call surface of
tatavishnurao/LatentPagedAttention-rs ``python_ref/latent_paged_attention``.

The directory name contains a hyphen, so import it with
``importlib.import_module("latentpagedattention-rs_b200")`` (the repository
root on ``sys.path``).  All computation runs in ``libplkv_b200.so`` (C ABI in
``include/plkv_b200.h``); importing the operations fails if it is not built.
"""

from . import block_table, memory_model, workloads  # noqa: F401  (pure host modules)
from .block_table import PagedBlockTable, logical_blocks_for_seq_len  # noqa: F401

__all__ = ["PagedBlockTable", "logical_blocks_for_seq_len", "block_table", "memory_model",
           "workloads", "ops"]


def __getattr__(name):
    # The CUDA-backed operations load libplkv_b200.so on first use.
    if name == "ops":
        import importlib

        mod = importlib.import_module(__name__ + ".ops")
        globals()["ops"] = mod
        return mod
    raise AttributeError(name)
