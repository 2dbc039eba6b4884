"""GPU parity of the decode at the latent widths and sizes the workloads use,
against the FP64 oracle (oracle/plkv_oracle.c, lib.rs:941-1145 with FP64
accumulation) on the identical FP16 inputs.

Bars, written per test: exact FP32 mode <= 1e-5 and tensor-core mode <=
2e-3 normwise relative error (max|a - e| / max|e|) per sequence.

* GQA-latent shapes of the write-then-attend workload (Hq 32, KV 8, D 128,
  block 16) at latent widths 256 (the workload's), 320, 576/512 and 600,
  which select every instantiation of the exact partial pass.
* Tensor-core mode on the full long-context (8 x 131072 tokens) and MLA-batch
  (64 sequences, lengths U[1024, 32768]) workloads, sampled heads of sampled
  sequences straight against the oracle.
* A caller error word that already holds a timeout bit does not end a later
  tensor-core call (the kernel's abort word is per launch).
"""

import math

import numpy as np
import pytest
import torch

from oracle import c_ref
from tests_support import rel_err

pytestmark = pytest.mark.gpu

EXACT_REL = 1e-5
TC_REL = 2e-3
DEV = "cuda"


def t(x, dtype=None):
    return torch.as_tensor(np.ascontiguousarray(x), device=DEV, dtype=dtype)


def f16_to_bits(x):
    return x.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _gqa_case(seed, lens, L, Lv, Hq=32, KV=8, D=128, bs=16):
    rng = np.random.default_rng(seed)
    nb = [(n + bs - 1) // bs for n in lens]
    P = sum(nb) + 5
    perm = rng.permutation(P).astype(np.int32)
    tables = np.full((len(lens), max(nb)), -1, np.int32)
    k = 0
    for b, c in enumerate(nb):
        tables[b, :c] = perm[k:k + c]
        k += c
    return dict(
        cache=rng.standard_normal((P, bs, L), dtype=np.float32).astype(np.float16),
        q=rng.standard_normal((len(lens), Hq, D), dtype=np.float32),
        w_k=rng.standard_normal((L, KV * D), dtype=np.float32) / np.float32(math.sqrt(D)),
        w_v=rng.standard_normal((Lv, KV * D), dtype=np.float32) / np.float32(math.sqrt(Lv)),
        tables=tables, lens=np.asarray(lens, np.int32), L=L, Lv=Lv, Hq=Hq, KV=KV, D=D, bs=bs)


def _head_major(w, heads, D):
    return t(w.reshape(w.shape[0], heads, D).transpose(1, 0, 2))


@pytest.mark.parametrize("L,Lv", [(256, 256), (320, 320), (576, 512), (600, 600)])
def test_gqa_latent_exact_widths_vs_oracle(ops, L, Lv):
    """Query projected through W_k, direct latent decode, W_v projection, at
    the write-then-attend shapes; every instantiation of the exact pass."""
    c = _gqa_case(40 + L, [512, 1001, 4096], L, Lv)
    KV, D, bs = c["KV"], c["D"], c["bs"]
    cache = t(c["cache"])
    q_lat = ops.project_query(t(c["q"]), _head_major(c["w_k"], KV, D))
    plan = ops.plan_splits(c["lens"], bs)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    r = ops.latent_decode(q_lat, cache, t(c["tables"]), t(c["lens"]), plan,
                          scale=1 / math.sqrt(D), value_dim=Lv, w_v=_head_major(c["w_v"], KV, D),
                          want_lse=True, flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    ctx = r["ctx"].cpu().numpy()
    bits = c["cache"].view(np.uint16)
    for b, n in enumerate(c["lens"]):
        ql = c_ref.project_query(c["q"][b], c["w_k"], KV)
        _, _, _, ec = c_ref.latent_decode_seq(ql, bits, c["tables"][b], int(n), int(n), bs,
                                              1 / math.sqrt(D), value_dim=Lv,
                                              w_v_canonical=c["w_v"], proj_heads=KV,
                                              head_dim=D, acc64=True, want_intermediates=False)
        assert rel_err(ctx[b], ec) <= EXACT_REL, (L, b, rel_err(ctx[b], ec))


def _tc_vs_oracle(ops, pkg, name, seqs, heads):
    s = pkg.workloads.spec(name)
    x = pkg.workloads.device_inputs(s, DEV, with_out_proj=False)
    lens = t(x["lens"])
    plan = ops.plan_workers(x["lens"], s.block_size)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    r = ops.latent_decode(x["q_lat"], x["cache"], x["tables"], lens, plan, scale=s.scale,
                          value_dim=s.value_dim, w_v=x["w_v"], mode="tc", want_lse=True,
                          flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    ctx = r["ctx"].cpu().numpy()
    lse = r["lse"].cpu().numpy()
    q_lat = x["q_lat"].cpu().numpy()
    w_can = x["w_v"].cpu().numpy().transpose(1, 0, 2).reshape(s.value_dim, -1)
    tables = x["tables"].cpu().numpy()
    for b in seqs:
        n = int(x["lens"][b])
        nb = (n + s.block_size - 1) // s.block_size
        # the sequence's blocks only, compacted (the pool is gigabytes)
        bits = f16_to_bits(x["cache"][torch.as_tensor(tables[b, :nb], device=DEV).long()])
        local = np.arange(nb, dtype=np.int32)
        for h0, h1 in heads:
            es, _, _, ec = c_ref.latent_decode_seq(q_lat[b], bits, local, n, n, s.block_size,
                                                   s.scale, value_dim=s.value_dim,
                                                   w_v_canonical=w_can, proj_heads=s.proj_heads,
                                                   head_dim=s.head_dim, heads=(h0, h1),
                                                   acc64=True)
            got = ctx[b, h0:h1]
            assert rel_err(got, ec[h0:h1]) <= TC_REL, (name, b, h0, rel_err(got, ec[h0:h1]))
            for h in range(h0, h1):
                srow = es[h, :n].astype(np.float64)
                mx = srow.max()
                e_lse = mx + math.log(np.exp(srow - mx).sum())
                assert abs(lse[b, h] - e_lse) <= TC_REL * max(1.0, abs(e_lse))


def test_long_context_tensor_core_vs_oracle(ops, pkg):
    """The headline workload at full size, tensor-core mode, against the
    oracle directly: heads from both CTAs of a pair, first and last sequence."""
    _tc_vs_oracle(ops, pkg, "long_context", seqs=(0, 7), heads=((0, 2), (63, 65), (126, 128)))


def test_mla_batch_tensor_core_vs_oracle(ops, pkg):
    """The 64-sequence MLA batch (lengths U[1024, 32768]) at full size."""
    s = pkg.workloads.spec("mla_batch")
    lens = pkg.workloads.initial_lens(s)
    seqs = (int(np.argmin(lens)), int(np.argmax(lens)), 31)
    _tc_vs_oracle(ops, pkg, "mla_batch", seqs=seqs, heads=((0, 4), (60, 68), (124, 128)))


def _mla_small(seed, lens, bs=64):
    rng = np.random.default_rng(seed)
    L, Lv, Hq, D = 576, 512, 128, 128
    nb = [(n + bs - 1) // bs for n in lens]
    P = sum(nb) + 3
    perm = rng.permutation(P).astype(np.int32)
    tables = np.full((len(lens), max(nb)), -1, np.int32)
    k = 0
    for b, c in enumerate(nb):
        tables[b, :c] = perm[k:k + c]
        k += c
    return dict(cache=(rng.standard_normal((P, bs, L), dtype=np.float32) * 0.5).astype(np.float16),
                q_lat=rng.standard_normal((len(lens), Hq, L), dtype=np.float32),
                w_uv=rng.standard_normal((Hq, Lv, D), dtype=np.float32) / np.float32(math.sqrt(Lv)),
                tables=tables, lens=np.asarray(lens, np.int32), bs=bs, Lv=Lv, D=D)


def test_stale_timeout_bit_does_not_end_a_later_call(ops):
    """A caller error word that still holds PLKV_FLAG_TIMEOUT from an earlier
    call (or a shared word that another kernel set) is only reported into:
    the tensor-core pass learns of failures from its own per-launch word, so
    a later call with the same word computes the full result."""
    m = _mla_small(5, [3000, 700])
    plan = ops.plan_workers(m["lens"], m["bs"], n_workers=4)
    args = (t(m["q_lat"]), t(m["cache"]), t(m["tables"]), t(m["lens"]), plan)
    kw = dict(scale=1 / math.sqrt(m["D"]), value_dim=m["Lv"], w_v=t(m["w_uv"]), mode="tc")
    clean = ops.latent_decode(*args, **kw)["ctx"].cpu()
    flags = torch.full((1,), 0x20, dtype=torch.int32, device=DEV)   # PLKV_FLAG_TIMEOUT
    for _ in range(2):
        got = ops.latent_decode(*args, flags=flags, **kw)["ctx"].cpu()
        torch.cuda.synchronize()
        assert torch.count_nonzero(got) == got.numel()
        assert torch.equal(got, clean)
    assert int(flags.item()) == 0x20                                 # reported bits are kept


@pytest.mark.parametrize("L,Hq,bs,target", [(256, 32, 16, None), (256, 32, 16, 40),
                                            (128, 32, 64, None), (256, 8, 32, 17)])
def test_gqa_latent_tensor_core_pass_vs_oracle(ops, L, Hq, bs, target):
    """The exact mode's tensor-core pass (latent = value width 128 / 256, up
    to 32 heads, no intermediates): lengths around the 128-token tile, several
    work items per sequence, unused pool slots holding NaN / Inf; equal to the
    FP64 restatement at 1e-5, and to the CUDA-core pass (taken when scores
    are requested) in context and log-sum-exp."""
    KV = 8 if Hq >= 8 else Hq
    lens = [1, 127, 128, 129, 1000, 3001]
    c = _gqa_case(70 + L + Hq, lens, L, L, Hq=Hq, KV=KV, bs=bs)
    used = np.zeros(c["cache"].shape[:2], bool)
    for b, n in enumerate(c["lens"]):
        for tok in range(n):
            used[c["tables"][b, tok // bs], tok % bs] = True
    pb, pt = np.nonzero(~used)
    c["cache"][pb[0::2], pt[0::2]] = np.float16(np.nan)
    c["cache"][pb[1::2], pt[1::2]] = np.float16(np.inf)
    D = c["D"]
    cache = t(c["cache"])
    q_lat = ops.project_query(t(c["q"]), _head_major(c["w_k"], KV, D))
    plan = (ops.plan_splits(c["lens"], bs, target_items=target) if target
            else ops.plan_splits(c["lens"], bs))
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    kw = dict(scale=1 / math.sqrt(D), value_dim=L, w_v=_head_major(c["w_v"], KV, D),
              want_lse=True, flags=flags)
    r = ops.latent_decode(q_lat, cache, t(c["tables"]), t(c["lens"]), plan, **kw)
    rc = ops.latent_decode(q_lat, cache, t(c["tables"]), t(c["lens"]), plan, want_scores=True,
                           max_seq_len=int(c["lens"].max()), **kw)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    ctx = r["ctx"].cpu().numpy()
    assert np.isfinite(ctx).all()
    assert rel_err(ctx, rc["ctx"].cpu().numpy()) <= EXACT_REL
    assert rel_err(r["lse"].cpu().numpy(), rc["lse"].cpu().numpy()) <= EXACT_REL
    bits = c["cache"].view(np.uint16)
    for b, n in enumerate(c["lens"]):
        ql = c_ref.project_query(c["q"][b], c["w_k"], KV)
        _, _, _, ec = c_ref.latent_decode_seq(ql, bits, c["tables"][b], int(n), int(n), bs,
                                              1 / math.sqrt(D), value_dim=L,
                                              w_v_canonical=c["w_v"], proj_heads=KV,
                                              head_dim=D, acc64=True, want_intermediates=False)
        assert rel_err(ctx[b], ec) <= EXACT_REL, (L, b, rel_err(ctx[b], ec))


def test_gqa_projections_batched_gemm_vs_oracle(ops):
    """40 sequences x 4 query heads per KV head = 160 rows per head: both the
    query projection (W_k) and the value projection (W_v) run as the batched
    FP32 GEMM (64 x 64 tiles, partial edge tiles: 160 rows, 128 / 256
    columns). Query rows and contexts equal the FP64 restatement at 1e-5."""
    rng = np.random.default_rng(91)
    lens = list(rng.integers(1, 300, 40))
    c = _gqa_case(91, lens, 256, 256)
    KV, D = c["KV"], c["D"]
    q_lat = ops.project_query(t(c["q"]), _head_major(c["w_k"], KV, D))
    plan = ops.plan_splits(c["lens"], c["bs"], target_items=64)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    r = ops.latent_decode(q_lat, t(c["cache"]), t(c["tables"]), t(c["lens"]), plan,
                          scale=1 / math.sqrt(D), value_dim=256,
                          w_v=_head_major(c["w_v"], KV, D), flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    ql_gpu = q_lat.cpu().numpy()
    ctx = r["ctx"].cpu().numpy()
    bits = c["cache"].view(np.uint16)
    for b, n in enumerate(c["lens"]):
        ql = c_ref.project_query(c["q"][b], c["w_k"], KV)
        assert rel_err(ql_gpu[b], ql) <= EXACT_REL
        _, _, _, ec = c_ref.latent_decode_seq(ql, bits, c["tables"][b], int(n), int(n), c["bs"],
                                              1 / math.sqrt(D), value_dim=256,
                                              w_v_canonical=c["w_v"], proj_heads=KV,
                                              head_dim=D, acc64=True, want_intermediates=False)
        assert rel_err(ctx[b], ec) <= EXACT_REL, (b, rel_err(ctx[b], ec))
