"""Materialised latent -> K/V reconstruction (plkv_reconstruct_kv) against the
reference's fixture and the oracle, and the materialised decode built on it.

Bars: the fixture at the reference's GPU tolerances (atol 2e-5, rtol 1e-5,
latent_kv_reconstruction_gpu.rs:12-13); FP32 output normwise relative error
<= 1e-6 against the FP64-accumulating oracle; FP16 output within one FP16
ulp (2^-10 relative) of the FP64 result plus 2e-6 of its largest magnitude
(FP32 accumulation error of cancelling sums); rows outside the slot list
untouched; the decode over the rebuilt K/V <= 1e-5 against the oracle's
full-KV decode of the same FP16 bits."""

import importlib
import math

import numpy as np
import pytest
import torch

from conftest import PACKAGE, load_reference_fixture
from oracle import c_ref
from tests_support import rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ops():
    return importlib.import_module(PACKAGE + ".ops")


@pytest.mark.parametrize("case", [0, 1])
def test_reconstruction_fixture(case):
    ops = _ops()
    fx = load_reference_fixture("latent_kv_reconstruction_f32.json")
    c = fx["cases"][case]
    KV, D = fx["kv_heads"], fx["head_dim"]
    lat = np.asarray(c["latent_cache"], np.float32)[None]
    k, v = ops.latent_kv_reconstruction(lat, np.asarray(c["k_projection"], np.float32),
                                        np.asarray(c["v_projection"], np.float32),
                                        kv_heads=KV, head_dim=D)
    k, v = k.cpu().numpy()[0], v.cpu().numpy()[0]
    for got, key in ((k, "expected_k_token_major"), (v, "expected_v_token_major")):
        np.testing.assert_allclose(got, np.asarray(c[key], np.float32), rtol=1e-5, atol=2e-5)
    np.testing.assert_allclose(k.transpose(1, 0, 2), np.asarray(c["expected_k_head_major"]),
                               rtol=1e-5, atol=2e-5)
    np.testing.assert_allclose(v.transpose(1, 0, 2), np.asarray(c["expected_v_head_major"]),
                               rtol=1e-5, atol=2e-5)


def test_reconstruction_rejections():
    ops = _ops()
    lat = np.zeros((1, 8, 8), np.float32)
    proj = np.zeros((8, 16), np.float32)
    with pytest.raises(ValueError):
        ops.latent_kv_reconstruction(lat[0], proj, proj, kv_heads=2, head_dim=8)
    with pytest.raises(ValueError):
        ops.latent_kv_reconstruction(lat, proj, proj[:, :8], kv_heads=2, head_dim=8)
    with pytest.raises(ValueError):
        ops.latent_kv_reconstruction(lat, proj[:, :15], proj[:, :15], kv_heads=2, head_dim=8)
    with pytest.raises(ValueError):
        ops.latent_kv_reconstruction(lat, proj, proj, kv_heads=0, head_dim=8)
    bad = lat.copy()
    bad[0, 3, 5] = np.nan
    with pytest.raises(ValueError):
        ops.latent_kv_reconstruction(bad, proj, proj, kv_heads=2, head_dim=8)


def _paged_case(seed=4, B=5, bs=16, L=256, KV=8, D=128, extra=3):
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 90, B).astype(np.int32)
    nb = (lens + bs - 1) // bs
    P = int(nb.sum()) + extra
    perm = rng.permutation(P).astype(np.int32)
    tables = np.full((B, int(nb.max())), -1, np.int32)
    k = 0
    for b in range(B):
        tables[b, :nb[b]] = perm[k:k + nb[b]]
        k += nb[b]
    cache = rng.standard_normal((P, bs, L), dtype=np.float32).astype(np.float16)
    w_k = rng.standard_normal((L, KV * D), dtype=np.float32) / np.float32(math.sqrt(D))
    w_v = rng.standard_normal((L, KV * D), dtype=np.float32) / np.float32(math.sqrt(L))
    slots = np.concatenate([tables[b, np.arange(lens[b]) // bs] * bs + np.arange(lens[b]) % bs
                            for b in range(B)]).astype(np.int64)
    return dict(lens=lens, tables=tables, cache=cache, w_k=w_k, w_v=w_v, slots=slots, P=P, bs=bs,
                L=L, KV=KV, D=D)


def _hm(w, KV, D):
    return torch.as_tensor(np.ascontiguousarray(w.reshape(w.shape[0], KV, D).transpose(1, 0, 2)),
                           device=DEV)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_paged_reconstruction_matches_oracle(out_dtype):
    ops = _ops()
    c = _paged_case()
    P, bs, KV, D = c["P"], c["bs"], c["KV"], c["D"]
    sentinel = 7.0
    k_out = torch.full((P, KV, bs, D), sentinel, dtype=out_dtype, device=DEV)
    v_out = torch.full_like(k_out, sentinel)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.reconstruct_kv(torch.as_tensor(c["cache"], device=DEV), _hm(c["w_k"], KV, D),
                       _hm(c["w_v"], KV, D), slots=torch.as_tensor(c["slots"], device=DEV),
                       block_size=bs, out_dtype=out_dtype, k_out=k_out, v_out=v_out, flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    rows = c["cache"].reshape(-1, c["L"]).astype(np.float32)[c["slots"]]
    ek, ev = c_ref.reconstruct_kv(rows, c["w_k"], c["w_v"], acc64=True)
    gk = k_out.float().cpu().numpy().transpose(0, 2, 1, 3).reshape(P * bs, KV * D)
    gv = v_out.float().cpu().numpy().transpose(0, 2, 1, 3).reshape(P * bs, KV * D)
    for got, exp in ((gk, ek), (gv, ev)):
        g = got[c["slots"]]
        if out_dtype == torch.float32:
            assert rel_err(g, exp) <= 1e-6
        else:
            # one FP16 ulp of the value plus the FP32 accumulation error, which
            # scales with the size of the terms, not of a cancelled result
            np.testing.assert_allclose(g, exp, rtol=2.0 ** -10,
                                       atol=2e-6 * float(np.max(np.abs(exp))))
        untouched = np.setdiff1d(np.arange(P * bs), c["slots"])
        assert np.all(got[untouched] == sentinel)


def test_materialised_decode_matches_oracle_and_direct_path():
    """Rebuild FP16 K/V for the active slots, decode them with the full-KV
    decode, and compare with the oracle's full-KV decode of the same bits; the
    direct latent decode of the same query agrees to FP16 rounding of K / V."""
    ops = _ops()
    c = _paged_case(seed=9)
    P, bs, KV, D, L = c["P"], c["bs"], c["KV"], c["D"], c["L"]
    Hq = 32
    rng = np.random.default_rng(1)
    q = rng.standard_normal((c["lens"].size, Hq, D), dtype=np.float32)
    scale = 1 / math.sqrt(D)
    k16 = torch.zeros((P, KV, bs, D), dtype=torch.float16, device=DEV)
    v16 = torch.zeros_like(k16)
    ops.reconstruct_kv(torch.as_tensor(c["cache"], device=DEV), _hm(c["w_k"], KV, D),
                       _hm(c["w_v"], KV, D), slots=torch.as_tensor(c["slots"], device=DEV),
                       block_size=bs, k_out=k16, v_out=v16)
    tables = torch.as_tensor(c["tables"], device=DEV)
    lens = torch.as_tensor(c["lens"], device=DEV)
    plan = ops.plan_splits(c["lens"], bs)
    ctx = ops.fullkv_decode(torch.as_tensor(q, device=DEV), k16, v16, tables, lens, plan,
                            scale=scale)["ctx"].cpu().numpy()
    kb = k16.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    vb = v16.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    exp = c_ref.fullkv_decode_batch(q, kb, vb, c["tables"], c["lens"], scale, acc64=True)
    assert rel_err(ctx, exp) <= 1e-5
    q_lat = torch.as_tensor(np.stack([c_ref.project_query(q[b], c["w_k"], KV)
                                      for b in range(q.shape[0])]), device=DEV)
    direct = ops.latent_decode(q_lat, torch.as_tensor(c["cache"], device=DEV), tables, lens,
                               plan, scale=scale, value_dim=L, w_v=_hm(c["w_v"], KV, D))
    assert rel_err(ctx, direct["ctx"].cpu().numpy()) <= 2e-2


@pytest.mark.parametrize("B,K,N", [(64, 16384, 7168), (1, 4096, 4096), (2, 64, 64), (200, 512, 320)])
def test_out_proj_tensor_cores_vs_oracle(B, K, N):
    """W_o on the tensor cores (TF32 operands, FP32 accumulation) against the
    FP64 oracle at 2e-3 normwise, and against the FP32 CUDA-core product."""
    ops = _ops()
    rng = np.random.default_rng(B + N)
    x = rng.standard_normal((B, K), dtype=np.float32)
    w = (rng.standard_normal((K, N), dtype=np.float32) / np.float32(math.sqrt(K)))
    xt, wt = torch.as_tensor(x, device=DEV), torch.as_tensor(w, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    got = ops.out_proj_tc(xt, wt, flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    g = got.cpu().numpy()
    rows = np.unique(np.array([0, B // 2, B - 1]))
    exp = c_ref.out_proj(x[rows], w, acc64=True)
    assert rel_err(g[rows], exp) <= 2e-3
    if B <= 64:
        ref32 = ops.out_proj(xt, wt).cpu().numpy()
        assert rel_err(g, ref32) <= 2e-3
