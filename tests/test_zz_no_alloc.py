"""plkv_latent_decode_noalloc: the decode entry point for callers that cannot
allocate device memory (a plugin host that owns every device byte and passes
only inputs and outputs, or a binding with no CUDA allocator).  Its split-K
scratch is the library's fixed device array instead of a caller workspace.

Checked through the C ABI against plkv_latent_decode with a caller workspace,
on two calls in a row with different inputs (the shared array keeps the first
call's contents), in exact mode at the exact-mode tolerance of the other GPU
tests and in tensor-core mode (whose FP16 copy of the query also lives in the
shared array) at the tensor-core tolerance.  This
file is collected last so that a run stopping at the first failure has run
every other test first; it also passes on its own in a fresh process.
"""

import ctypes
import importlib
import math

import numpy as np
import pytest
import torch

from conftest import PACKAGE
from tests_support import rel_err

pytestmark = pytest.mark.gpu

EXACT_REL = 1e-5
TC_REL = 2e-3
SCRATCH_LIMIT = 32 * 1024 * 1024  # PLKV_NOALLOC_SCRATCH_BYTES in include/plkv_b200.h


def _case(seed, lens, Hq=128, L=576, Lv=512, D=128, bs=64):
    rng = np.random.default_rng(seed)
    nb = [(n + bs - 1) // bs for n in lens]
    P = sum(nb) + 2
    perm = rng.permutation(P).astype(np.int32)
    tables = np.full((len(lens), max(nb)), -1, np.int32)
    k = 0
    for b, c in enumerate(nb):
        tables[b, :c] = perm[k:k + c]
        k += c
    dev = "cuda"
    return dict(
        cache=torch.as_tensor((rng.standard_normal((P, bs, L), dtype=np.float32) * 0.5)
                              .astype(np.float16), device=dev),
        q_lat=torch.as_tensor(rng.standard_normal((len(lens), Hq, L), dtype=np.float32), device=dev),
        w_v=torch.as_tensor(rng.standard_normal((Hq, Lv, D), dtype=np.float32)
                            / np.float32(math.sqrt(Lv)), device=dev),
        tables=torch.as_tensor(tables, device=dev),
        lens_host=np.asarray(lens, np.int32), lens=torch.as_tensor(np.asarray(lens, np.int32),
                                                                   device=dev),
        Hq=Hq, L=L, Lv=Lv, D=D, bs=bs)


def _args(_lib, c, plan, ctx, lse, workspace, mode=None):
    B = len(c["lens_host"])
    return _lib.LatentDecodeArgs(
        q_lat=c["q_lat"].data_ptr(), cache=c["cache"].data_ptr(), num_physical=c["cache"].shape[0],
        block_size=c["bs"], latent_dim=c["L"], value_dim=c["Lv"], batch=B, q_heads=c["Hq"],
        scale=1.0 / math.sqrt(c["D"]), block_tables=c["tables"].data_ptr(),
        max_blocks=c["tables"].shape[1], seq_lens=c["lens"].data_ptr(),
        items=plan.items.data_ptr(), seq_item_begin=plan.seq_item_begin.data_ptr(),
        n_items=plan.n_items, worker_item_begin=(None if plan.worker_item_begin is None
                                                 else plan.worker_item_begin.data_ptr()),
        n_workers=plan.n_workers, allow_empty=0, w_v=c["w_v"].data_ptr(), proj_heads=c["Hq"],
        head_dim=c["D"], ctx=ctx.data_ptr(), lse=lse.data_ptr(), scores=None, probs=None,
        max_seq_len=0, mode=_lib.MODE_EXACT_F32 if mode is None else mode,
        workspace=None if workspace is None else workspace.data_ptr(),
        workspace_bytes=0 if workspace is None else workspace.numel(), err_flags=None)


def _run_both(ops, _lib, c, target_items, mode=None, workers=None):
    B, Hq, D = len(c["lens_host"]), c["Hq"], c["D"]
    plan = (ops.plan_workers(c["lens_host"], c["bs"], n_workers=workers) if workers
            else ops.plan_splits(c["lens_host"], c["bs"], target_items=target_items))
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    ref_ctx = torch.empty((B, Hq, D), dtype=torch.float32, device="cuda")
    ref_lse = torch.empty((B, Hq), dtype=torch.float32, device="cuda")
    ws = torch.empty(ops.latent_workspace_bytes(plan.n_items, B, Hq, c["L"], c["Lv"]),
                     dtype=torch.uint8, device="cuda")
    a = _args(_lib, c, plan, ref_ctx, ref_lse, ws, mode)
    assert L.plkv_latent_decode(ctypes.byref(a), stream) == _lib.PLKV_OK
    ctx = torch.full((B, Hq, D), float("nan"), dtype=torch.float32, device="cuda")
    lse = torch.full((B, Hq), float("nan"), dtype=torch.float32, device="cuda")
    n = _args(_lib, c, plan, ctx, lse, None, mode)
    assert L.plkv_latent_decode_noalloc(ctypes.byref(n), stream) == _lib.PLKV_OK
    torch.cuda.synchronize()
    return ctx.cpu(), lse.cpu(), ref_ctx.cpu(), ref_lse.cpu(), plan


def test_noalloc_decode_matches_workspace_decode_twice():
    ops = importlib.import_module(PACKAGE + ".ops")
    _lib = importlib.import_module(PACKAGE + "._lib")
    first = _case(21, [4000, 37, 1500])
    ctx, lse, ref_ctx, ref_lse, plan = _run_both(ops, _lib, first, target_items=40)
    assert ops.latent_workspace_bytes(plan.n_items, 3, 128, 576, 512) <= SCRATCH_LIMIT
    assert torch.isfinite(ctx).all()
    assert rel_err(ctx, ref_ctx) <= EXACT_REL
    assert rel_err(lse, ref_lse) <= EXACT_REL
    # Second call in a row: other inputs and a different cut into work items;
    # the shared scratch still holds the first call's partial results.
    second = _case(22, [129, 2500], Hq=128)
    ctx2, lse2, ref_ctx2, ref_lse2, _ = _run_both(ops, _lib, second, target_items=17)
    assert torch.isfinite(ctx2).all()
    assert rel_err(ctx2, ref_ctx2) <= EXACT_REL
    assert rel_err(lse2, ref_lse2) <= EXACT_REL


def test_noalloc_tensor_core_matches_workspace_decode_twice():
    ops = importlib.import_module(PACKAGE + ".ops")
    _lib = importlib.import_module(PACKAGE + "._lib")
    first = _case(31, [3000, 64, 777])
    ctx, lse, ref_ctx, ref_lse, _ = _run_both(ops, _lib, first, 0, _lib.MODE_TC_F16, workers=5)
    assert torch.isfinite(ctx).all()
    assert rel_err(ctx, ref_ctx) <= TC_REL
    assert rel_err(lse, ref_lse) <= TC_REL
    second = _case(32, [1300, 4100])
    ctx2, lse2, ref_ctx2, ref_lse2, _ = _run_both(ops, _lib, second, 0, _lib.MODE_TC_F16,
                                                  workers=3)
    assert torch.isfinite(ctx2).all()
    assert rel_err(ctx2, ref_ctx2) <= TC_REL
    assert rel_err(lse2, ref_lse2) <= TC_REL


def test_noalloc_rejects_requests_beyond_the_scratch_array():
    ops = importlib.import_module(PACKAGE + ".ops")
    _lib = importlib.import_module(PACKAGE + "._lib")
    c = _case(23, [64 * 200])
    plan = ops.plan_splits(c["lens_host"], c["bs"], target_items=200)
    assert ops.latent_workspace_bytes(plan.n_items, 1, 128, 576, 512) > SCRATCH_LIMIT
    ctx = torch.zeros((1, 128, 128), dtype=torch.float32, device="cuda")
    lse = torch.zeros((1, 128), dtype=torch.float32, device="cuda")
    a = _args(_lib, c, plan, ctx, lse, None)
    st = _lib.lib().plkv_latent_decode_noalloc(ctypes.byref(a),
                                               torch.cuda.current_stream().cuda_stream)
    assert st == _lib.PLKV_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert torch.count_nonzero(ctx) == 0   # nothing was launched
