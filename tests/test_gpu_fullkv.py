"""FP16 full-KV paged GQA decode (lib.rs:1147-1269, attention_ref.py:172-224):
the tensor-core pass (head_dim 128, up to 16 query heads per KV head, no
intermediates) against the FP64 oracle at the exact-mode bar (1e-5
normwise) and against the CUDA-core pass (taken when scores are requested)."""

import importlib
import math

import numpy as np
import pytest
import torch

from conftest import PACKAGE
from oracle import c_ref
from tests_support import rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"
EXACT_REL = 1e-5


def _ops():
    return importlib.import_module(PACKAGE + ".ops")


def _case(seed, lens, Hq, KV, bs, D=128, poison=True):
    """Head-major FP16 pools [P, KV, bs, D] with every slot no sequence
    covers set to NaN / Inf, tables of randomly placed blocks, FP32 query."""
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, np.int32)
    nb = (lens + bs - 1) // bs
    P = int(nb.sum()) + 3
    perm = rng.permutation(P).astype(np.int32)
    tables = np.full((lens.size, max(1, int(nb.max()))), -1, np.int32)
    k = 0
    for b in range(lens.size):
        tables[b, :nb[b]] = perm[k:k + nb[b]]
        k += nb[b]
    kc = (rng.standard_normal((P, KV, bs, D), dtype=np.float32) * 0.7).astype(np.float16)
    vc = rng.standard_normal((P, KV, bs, D), dtype=np.float32).astype(np.float16)
    if poison:
        used = np.zeros((P, bs), bool)
        for b, n in enumerate(lens):
            for t in range(n):
                used[tables[b, t // bs], t % bs] = True
        pb, pt = np.nonzero(~used)
        kc[pb[0::2], :, pt[0::2]] = np.float16(np.nan)
        vc[pb[1::2], :, pt[1::2]] = np.float16(np.inf)
        kc[pb[1::2], :, pt[1::2]] = np.float16(np.inf)
        vc[pb[0::2], :, pt[0::2]] = np.float16(np.nan)
    q = rng.standard_normal((lens.size, Hq, D), dtype=np.float32)
    return dict(lens=lens, tables=tables, kc=kc, vc=vc, q=q, bs=bs, scale=1 / math.sqrt(D))


def _oracle(c):
    kb = c["kc"].view(np.uint16)
    vb = c["vc"].view(np.uint16)
    # the oracle reads only covered slots; give it the same bits
    return c_ref.fullkv_decode_batch(c["q"], kb, vb, c["tables"], c["lens"], c["scale"],
                                     acc64=True)


def _run(c, target=None, scores=False):
    ops = _ops()
    t = lambda a: torch.as_tensor(np.ascontiguousarray(a), device=DEV)
    plan = (ops.plan_splits(c["lens"], c["bs"], target_items=target) if target
            else ops.plan_splits(c["lens"], c["bs"]))
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    kw = dict(scale=c["scale"], want_lse=True, flags=flags)
    if scores:
        kw.update(want_scores=True, max_seq_len=int(c["lens"].max()))
    r = ops.fullkv_decode(t(c["q"]), t(c["kc"]), t(c["vc"]), t(c["tables"]), t(c["lens"]), plan,
                          **kw)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    return r


@pytest.mark.parametrize("Hq,KV,bs", [(32, 8, 16), (8, 8, 16), (16, 1, 64), (64, 8, 32)])
@pytest.mark.parametrize("target", [None, 200])
def test_fullkv_tensor_cores_vs_oracle(Hq, KV, bs, target):
    """Lengths around the 128-token tile (1, 127, 128, 129), long sequences
    cut into several work items, unused slots holding NaN / Inf: the
    tensor-core pass equals the FP64 restatement to 1e-5."""
    c = _case(11 + Hq + bs, [1, 127, 128, 129, 1000, 3001], Hq, KV, bs)
    r = _run(c, target)
    exp = _oracle(c)
    got = r["ctx"].cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_err(got, exp) <= EXACT_REL


def test_fullkv_tensor_cores_match_cuda_core_pass():
    """Same inputs through both passes (scores requested -> CUDA cores):
    contexts and log-sum-exps agree to 1e-5."""
    c = _case(5, [17, 300, 2048, 4097], 32, 8, 16)
    tc = _run(c, target=50)
    cc = _run(c, target=50, scores=True)
    assert rel_err(tc["ctx"].cpu(), cc["ctx"].cpu()) <= EXACT_REL
    assert rel_err(tc["lse"].cpu(), cc["lse"].cpu()) <= EXACT_REL


def test_fullkv_large_scores_rescale():
    """Scores that grow along the sequence force the lazily updated running
    max to move many times (O rescaled in tensor memory)."""
    c = _case(7, [2000, 700], 32, 8, 16, poison=False)
    ramp = np.linspace(0.1, 6.0, c["kc"].shape[0] * c["bs"], dtype=np.float32)
    kc = c["kc"].astype(np.float32)
    # rows of physical block p scaled by a ramp: positions far apart differ a lot
    kc *= ramp.reshape(c["kc"].shape[0], 1, c["bs"], 1)
    c["kc"] = kc.astype(np.float16)
    c["q"] *= 4
    r = _run(c)
    assert rel_err(r["ctx"].cpu().numpy(), _oracle(c)) <= EXACT_REL


def test_fullkv_long_items_from_the_fullkv_planner():
    """Items of the full-KV planner (at least 2048 tokens each: 16 tiles and
    more per CTA) against the FP64 oracle."""
    c = _case(23, [20000, 36001, 300, 16384], 32, 8, 16)
    ops = _ops()
    t = lambda a: torch.as_tensor(np.ascontiguousarray(a), device=DEV)
    plan = ops.plan_fullkv(c["lens"], c["bs"], 8)
    sizes = plan.items_host[:, 2] - plan.items_host[:, 1]
    assert plan.n_items <= 40 and np.sort(sizes)[1] * 16 >= 1024
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    r = ops.fullkv_decode(t(c["q"]), t(c["kc"]), t(c["vc"]), t(c["tables"]), t(c["lens"]), plan,
                          scale=c["scale"], flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    got = r["ctx"].cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_err(got, _oracle(c)) <= EXACT_REL
