"""CPU oracle for the paged latent-cache decode path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of ``bench.py`` may import this package; the product
(``latentpagedattention-rs_b200``) never does, and fails loudly without its
CUDA library instead of falling back here.

Two restatements of tatavishnurao/LatentPagedAttention-rs live here:

* ``oracle.np_ref`` -- NumPy restatement of the Python oracle
  (python_ref/latent_paged_attention/attention_ref.py, cache_ref.py,
  block_table.py), pinned against the reference's golden JSON fixtures in
  ``tests/golden/reference``.
* ``oracle.c_ref`` -- ctypes binding of ``plkv_oracle.c``, a C restatement of
  the Rust CPU reference (crates/plkv-core/src/lib.rs) with FP32 ("faithful")
  and FP64 accumulation, and an OpenMP batch driver used as the timed CPU
  baseline.
"""

from . import c_ref, np_ref  # noqa: F401
