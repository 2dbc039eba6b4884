"""GPU parity of libplkv_b200 against the oracle and the reference's golden vectors.

Bars (written per test):
* FP16 cache bits and block addressing: bit-exact.
* Exact FP32 mode: the reference's GPU tolerances (tiny: 2e-4 / 1e-4 / 2e-4,
  paged_latent_write_attention_fp16_gpu.rs:18-23; model_small: 5e-3 / 2e-4 /
  2e-3, model_profile_gpu.rs:157-165) against the golden vectors, and a
  normwise relative error max|a-e|/max|e| <= 1e-5 against the FP64 oracle on
  the identical FP16 inputs.
"""

import math

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_golden_json, load_reference_fixture
from oracle import c_ref
from tests_support import assert_close, model_shaped_inputs, regenerate, rel_err

pytestmark = pytest.mark.gpu

EXACT_REL = 1e-5
TC_REL = 2e-3     # tensor-core mode: FP16 query and probabilities, FP32 accumulation
DEV = "cuda"


def t(x, dtype=None):
    return torch.as_tensor(np.ascontiguousarray(x), device=DEV, dtype=dtype)


def bits_to_f16(bits):
    return t(np.asarray(bits, np.uint16).view(np.float16))


def f16_to_bits(x):
    return x.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


# -------------------------------------------------------------- FP16 storage

def test_quantize_bit_exact(ops):
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 100,
                           rng.standard_normal(10000).astype(np.float32) * 1e-6,
                           (np.arange(1024, 2048, dtype=np.float32) + 0.5) / 1024,
                           np.array([65504, 65519, -65519, 6e-8, 3e-8, 0.0, -0.0], np.float32)])
    got = ops.fp16_storage_bits(t(vals)).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, c_ref.f32_to_f16_bits(vals))
    with pytest.raises(ValueError, match="overflowed"):
        ops.fp16_storage_bits(t(np.array([70000.0], np.float32)))
    with pytest.raises(ValueError, match="finite"):
        ops.fp16_storage_bits(t(np.array([1.0, np.inf], np.float32)))


@pytest.mark.parametrize("case", [0, 1])
def test_latent_write_matches_fixture_bits(ops, case):
    fx = load_reference_fixture("paged_latent_write_attention_fp16_storage.json")
    c = fx["cases"][case]
    cache = bits_to_f16(c["initial_latent_fp16_bits"])
    before = cache.clone()
    out = ops.paged_latent_write_fp16_storage(cache, fx["block_table"], c["token_position"],
                                              t(c["new_latent_source_f32"], torch.float32))
    np.testing.assert_array_equal(f16_to_bits(out),
                                  np.asarray(c["expected_updated_latent_fp16_bits"], np.uint16))
    assert torch.equal(cache, before)  # copy semantics (cache_ref.py:98-100)
    # In place, through the batched append with a length counter.
    lens = t(np.array([c["token_position"]], np.int32))
    ops.latent_append(t(c["new_latent_source_f32"], torch.float32).reshape(1, -1), cache,
                      t(np.array([fx["block_table"]], np.int32)), seq_lens=lens)
    np.testing.assert_array_equal(f16_to_bits(cache), f16_to_bits(out))
    assert int(lens.item()) == c["token_position"] + 1


def test_latent_write_rejections(ops):
    fx = load_reference_fixture("paged_latent_write_attention_fp16_storage.json")
    c = fx["cases"][0]
    cache = bits_to_f16(c["initial_latent_fp16_bits"])
    with pytest.raises(IndexError):
        ops.paged_latent_write_fp16_storage(cache, [2, 0, 3, 1], 8, t(np.zeros(8, np.float32)))
    with pytest.raises(IndexError):
        ops.paged_latent_write_fp16_storage(cache, [4, 0, 3, 1], 0, t(np.zeros(8, np.float32)))
    with pytest.raises(ValueError):
        ops.paged_latent_write_fp16_storage(cache, [2, 0, 3, 1], 0, t(np.zeros(7, np.float32)))
    bad = np.zeros(8, np.float32)
    bad[3] = 70000.0
    with pytest.raises(ValueError, match="overflowed"):
        ops.paged_latent_write_fp16_storage(cache, [2, 0, 3, 1], 0, t(bad))
    # Batched: a rejected row is not written at all, the others are.
    before = cache.clone()
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    rows = np.ones((2, 8), np.float32)
    rows[0, 5] = np.nan
    ops.latent_append(t(rows), cache, t(np.array([[2, 0, 3, 1], [2, 0, 3, 1]], np.int32)),
                      positions=t(np.array([0, 5], np.int32)), flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) & 1
    got, ref = f16_to_bits(cache), f16_to_bits(before)
    assert np.array_equal(got[2, 0], ref[2, 0])          # NaN row untouched
    assert np.all(got[3, 1] == np.float16(1).view(np.uint16))  # position 5 -> block 3, offset 1


def test_slot_append_bit_exact(ops):
    rng = np.random.default_rng(2)
    cache = torch.zeros((6, 4, 16), dtype=torch.float16, device=DEV)
    rows = rng.standard_normal((3, 16)).astype(np.float32)
    slots = np.array([5, -1, 22], np.int64)
    ops.latent_append_slots(t(rows), cache, t(slots))
    got = f16_to_bits(cache).reshape(24, 16)
    np.testing.assert_array_equal(got[5], c_ref.quantize_f16(rows[0]))
    np.testing.assert_array_equal(got[22], c_ref.quantize_f16(rows[2]))
    assert np.count_nonzero(got) == np.count_nonzero(got[[5, 22]])


@pytest.mark.parametrize("case", [0, 1])
def test_kv_append_matches_fixture(ops, case):
    fx = load_reference_fixture("paged_kv_write_f32.json")
    c = fx["cases"][case]
    P, bs, KV, D = fx["num_physical_blocks"], fx["block_size"], fx["kv_heads"], fx["head_dim"]

    def hm(tok):
        return c_ref.quantize_f16(np.asarray(tok, np.float32).reshape(P, bs, KV, D)
                                  .transpose(0, 2, 1, 3))

    k, v = bits_to_f16(hm(c["initial_k_cache"])), bits_to_f16(hm(c["initial_v_cache"]))
    ops.kv_append(t(np.asarray(c["new_k"], np.float32)[None]),
                  t(np.asarray(c["new_v"], np.float32)[None]), k, v,
                  t(np.array([fx["gpu_padded_block_table"]], np.int32)),
                  positions=t(np.array([c["token_position"]], np.int32)))
    np.testing.assert_array_equal(f16_to_bits(k), hm(c["expected_k_cache"]))
    np.testing.assert_array_equal(f16_to_bits(v), hm(c["expected_v_cache"]))


# -------------------------------------------------------- drop-in decode

@pytest.mark.parametrize("phase", ["pre", "post"])
@pytest.mark.parametrize("case", [0, 1])
def test_write_then_attend_fixture(ops, case, phase):
    fx = load_reference_fixture("paged_latent_write_attention_fp16_storage.json")
    c = fx["cases"][case]
    cache = bits_to_f16(c["initial_latent_fp16_bits"])
    if phase == "post":
        cache = ops.paged_latent_write_fp16_storage(
            cache, fx["block_table"], c["token_position"],
            t(c["new_latent_source_f32"], torch.float32), inplace=True)
    s, p, ctx = ops.direct_paged_latent_gqa_fp16_storage_runtime_intermediates(
        t(np.asarray(c["q"], np.float32)[None]), cache, fx["block_table"], 8, 8, 2,
        t(c["k_projection"], torch.float32), t(c["v_projection"], torch.float32), q_heads=4,
        kv_heads=2, head_dim=8, group_size=2)
    pre = f"fp16_storage_{phase}_write_"
    assert_close(s.cpu()[0], c[pre + "scores"], 2e-4, 1e-5, "scores")
    assert_close(p.cpu()[0], c[pre + "probabilities"], 1e-4, 1e-5, "probs")
    assert_close(ctx.cpu()[0], c[pre + "context"], 2e-4, 1e-5, "context")
    # FP16 storage differs from FP32 storage while staying close to it
    # (paged_latent_write_attention_fp16_gpu.rs:24-26).
    f32 = f"fp32_{phase}_write_"
    assert_close(ctx.cpu()[0], c[f32 + "context"], 2e-3, 0, "fp16 vs fp32 context")


@pytest.mark.parametrize("case", [0, 1])
def test_runtime_active_lengths_fixture(ops, case):
    fx = load_reference_fixture("runtime_sequence_tiny_fp16_storage.json")
    c = fx["cases"][case]
    cache = bits_to_f16(c["initial_latent_fp16_bits"])
    for rc in c["runtime_cases"]:
        n = rc["active_seq_len"]
        s, p, ctx = ops.direct_paged_latent_gqa_fp16_storage_runtime_intermediates(
            t(np.asarray(c["q"], np.float32)[None]), cache, fx["block_table"],
            fx["max_seq_len"], n, fx["block_size"], t(c["k_projection"], torch.float32),
            t(c["v_projection"], torch.float32), q_heads=4, kv_heads=2, head_dim=8,
            group_size=2)
        s, p = s.cpu().numpy()[0], p.cpu().numpy()[0]
        es = np.asarray(rc["scores"], np.float32)
        assert_close(s[:, :n], es[:, :n], 2e-4, 1e-5, f"scores n={n}")
        assert np.all(s[:, n:] == np.float32(-3.4028234663852886e38))
        assert_close(p, rc["probabilities"], 1e-4, 1e-5, f"probs n={n}")
        assert np.all(p[:, n:] == 0.0)
        assert np.max(np.abs(p.sum(-1) - 1.0)) <= 1e-4
        assert_close(ctx.cpu()[0], rc["context"], 2e-4, 1e-5, f"context n={n}")


def test_identity_table_negative_control(ops):
    fx = load_reference_fixture("runtime_sequence_tiny_fp16_storage.json")
    c = fx["cases"][0]
    cache = bits_to_f16(c["initial_latent_fp16_bits"])
    args = (t(np.asarray(c["q"], np.float32)[None]), cache)
    kw = dict(q_heads=4, kv_heads=2, head_dim=8, group_size=2)
    kp, vp = t(c["k_projection"], torch.float32), t(c["v_projection"], torch.float32)
    s1, _, _ = ops.direct_paged_latent_gqa_fp16_storage_runtime_intermediates(
        *args, [2, 0, 3, 1], 8, 8, 2, kp, vp, **kw)
    s2, _, _ = ops.direct_paged_latent_gqa_fp16_storage_runtime_intermediates(
        *args, [0, 1, 2, 3], 8, 8, 2, kp, vp, **kw)
    assert float((s1 - s2).abs().max()) > 1e-5


def test_tiny_workload_golden(ops, pkg):
    g = load_golden_json("tiny_workload.json")
    s = pkg.workloads.spec("tiny")
    cache = bits_to_f16(g["cache_f16_bits"])
    B, Hq, KV, D = s.batch, s.q_heads, s.kv_heads, s.head_dim
    lens_host = np.asarray(g["lens"], np.int32)
    tables = t(np.asarray(g["tables"], np.int32))
    lens = t(lens_host)
    q = t(np.asarray(g["q"], np.float32))
    wk = ops.projection_to_head_major(t(g["w_k"], torch.float32), KV, D)
    wv = ops.projection_to_head_major(t(g["w_v"], torch.float32), KV, D)
    q_lat = ops.project_query(q, wk)
    for target in (1, 3, 64):
        plan = ops.plan_splits(lens_host, s.block_size, target_items=target)
        r = ops.latent_decode(q_lat, cache, tables, lens, plan, scale=s.scale, w_v=wv,
                              want_scores=True, want_probs=True, max_seq_len=g["max_seq_len"])
        for b, n in enumerate(lens_host):
            assert_close(r["scores"][b].cpu()[:, :n], np.asarray(g["scores"][b])[:, :n], 2e-4,
                         1e-5, "scores")
            assert_close(r["probs"][b].cpu(), g["probs"][b], 1e-4, 1e-5, "probs")
            assert_close(r["ctx"][b].cpu(), g["ctx"][b], 2e-4, 1e-5, "ctx")
        out = ops.out_proj(r["ctx"].reshape(B, -1), t(g["w_o"], torch.float32))
        assert_close(out.cpu(), g["out_f64"], 1e-4, 1e-5, "W_o")
    # Full-KV baseline on the same shapes (K = fp16(L W_k), V = fp16(L W_v)).
    khm = bits_to_f16(np.asarray(g["k_tok_f16_bits"], np.uint16).transpose(0, 2, 1, 3))
    vhm = bits_to_f16(np.asarray(g["v_tok_f16_bits"], np.uint16).transpose(0, 2, 1, 3))
    plan = ops.plan_splits(lens_host, s.block_size, target_items=4)
    r = ops.fullkv_decode(q, khm, vhm, tables, lens, plan, scale=s.scale, want_scores=True,
                          want_probs=True, max_seq_len=g["max_seq_len"])
    for b, n in enumerate(lens_host):
        assert_close(r["scores"][b].cpu()[:, :n], np.asarray(g["fullkv_scores"][b])[:, :n], 2e-4,
                     1e-5, "fullkv scores")
        assert_close(r["probs"][b].cpu()[:, :n], np.asarray(g["fullkv_probs"][b])[:, :n], 1e-4,
                     1e-5, "fullkv probs")
        assert_close(r["ctx"][b].cpu(), g["fullkv_ctx"][b], 2e-4, 1e-5, "fullkv ctx")


def test_fullkv_dropin_matches_reference_layout(ops):
    fx = load_reference_fixture("paged_gqa_decode_f32.json")
    c = fx["cases"][0]
    k32 = np.asarray(c["k_physical_token_major"], np.float32)
    v32 = np.asarray(c["v_physical_token_major"], np.float32)
    s, p, ctx = ops.paged_gqa_decode_attention_intermediates(
        t(np.asarray(c["q"], np.float32)[None]), t(k32), t(v32), fx["block_table"], 8, 2,
        group_size=2)
    kb = c_ref.quantize_f16(k32.transpose(0, 2, 1, 3))
    vb = c_ref.quantize_f16(v32.transpose(0, 2, 1, 3))
    es, ep, ec = c_ref.fullkv_decode_seq(np.asarray(c["q"], np.float32), kb, vb,
                                         fx["block_table"], 8, 8, 1 / math.sqrt(8), acc64=True)
    assert rel_err(s.cpu()[0], es) <= EXACT_REL
    assert rel_err(p.cpu()[0], ep) <= EXACT_REL
    assert rel_err(ctx.cpu()[0], ec) <= EXACT_REL
    assert_close(ctx.cpu()[0], c["expected_context"], 2e-3, 1e-2, "fp16 vs fp32 fixture")


def test_model_small_kat(ops):
    d = np.load(f"{GOLDEN}/model_small_kat.npz")
    for n in d["active_lens"]:
        n = int(n)
        s, p, ctx = ops.direct_paged_latent_gqa_fp16_storage_runtime_intermediates(
            t(d["q"]), t(d["latent_f32"]), d["table"], 1024, n, 16, t(d["k_proj"]),
            t(d["v_proj"]), q_heads=16, kv_heads=4, head_dim=64, group_size=4)
        assert_close(s.cpu()[0][:, :n], d[f"scores_{n}"][:, :n], 5e-3, 1e-5, f"scores {n}")
        assert_close(p.cpu()[0], d[f"probs_{n}"], 2e-4, 1e-5, f"probs {n}")
        assert_close(ctx.cpu()[0], d[f"ctx_{n}"], 2e-3, 1e-5, f"ctx {n}")
        pn = p.cpu().numpy()[0]
        assert np.all(pn[:, n:] == 0) and np.max(np.abs(pn.sum(-1) - 1)) <= 1e-4


def test_model_shaped_workload(ops, pkg):
    d = np.load(f"{GOLDEN}/model_shaped.npz")
    x, s = model_shaped_inputs(pkg, str(d["inputs_sha256"]))
    cache = t(x["cache_f16"])
    tables = t(x["tables"])
    lens_host = x["lens"].copy()
    lens = t(lens_host - 1)               # 255 rows before the append
    ops.latent_append(t(x["new_rows"][0]), cache, tables, seq_lens=lens)
    n = int(lens_host[0])
    assert int(lens.item()) == n
    phys = x["tables"][0, (n - 1) // s.block_size]
    np.testing.assert_array_equal(f16_to_bits(cache)[phys, (n - 1) % s.block_size],
                                  d["updated_row_bits"])
    wk = t(pkg.workloads.head_major(x["w_k"], s.kv_heads, s.head_dim))
    wv = t(pkg.workloads.head_major(x["w_v"], s.proj_heads, s.head_dim))
    q_lat = ops.project_query(t(x["q"]), wk)
    plan = ops.plan_splits(lens_host, s.block_size)
    r = ops.latent_decode(q_lat, cache, tables, lens, plan, scale=s.scale, w_v=wv,
                          want_scores=True, want_probs=True, max_seq_len=n)
    assert_close(r["scores"].cpu()[0], d["scores"], 5e-3, 1e-5, "scores")
    assert_close(r["probs"].cpu()[0], d["probs"], 2e-4, 1e-5, "probs")
    assert_close(r["ctx"].cpu()[0], d["ctx"], 2e-3, 1e-5, "ctx")
    # Against the FP64 oracle on the identical FP16 inputs: 1e-5 normwise.
    bits = f16_to_bits(cache)
    q_lat_h = q_lat.cpu().numpy()[0]
    es, ep, _, ec = c_ref.latent_decode_seq(q_lat_h, bits, x["tables"][0], n, n, s.block_size,
                                            s.scale, w_v_canonical=x["w_v"],
                                            proj_heads=s.proj_heads, head_dim=s.head_dim,
                                            acc64=True)
    assert rel_err(r["scores"].cpu()[0], es) <= EXACT_REL
    assert rel_err(r["probs"].cpu()[0], ep) <= EXACT_REL
    assert rel_err(r["ctx"].cpu()[0], ec) <= EXACT_REL
    out = ops.out_proj(r["ctx"].reshape(1, -1), t(x["w_o"]))
    assert rel_err(out.cpu()[0], d["out_f64"]) <= 1e-4   # golden ctx is the FP32 oracle's
    ref_out = c_ref.out_proj(r["ctx"].cpu().numpy().reshape(1, -1), x["w_o"], acc64=True)
    assert rel_err(out.cpu(), ref_out) <= EXACT_REL


# ---------------------------------------------- larger shapes vs FP64 oracle

def _mla_case(pkg, batch, lens, seed=5, bs=64):
    """Absorbed-MLA shapes (Hq=128, L=576, Lv=512, D=128, bs=64), small batch."""
    rng = np.random.default_rng(seed)
    L, Lv, Hq, D = 576, 512, 128, 128
    nb = [(n + bs - 1) // bs for n in lens]
    P = sum(nb) + 3
    perm = rng.permutation(P).astype(np.int32)
    tables = np.full((batch, max(nb)), -1, np.int32)
    k = 0
    for b in range(batch):
        tables[b, :nb[b]] = perm[k:k + nb[b]]
        k += nb[b]
    cache = (rng.standard_normal((P, bs, L), dtype=np.float32) * 0.5).astype(np.float16)
    q_lat = rng.standard_normal((batch, Hq, L), dtype=np.float32)
    w_uv = rng.standard_normal((Hq, Lv, D), dtype=np.float32) / np.float32(math.sqrt(Lv))
    return dict(tables=tables, cache=cache, q_lat=q_lat, w_uv=w_uv, lens=np.asarray(lens, np.int32),
                bs=bs, L=L, Lv=Lv, Hq=Hq, D=D, scale=1 / math.sqrt(D))


def _check_mla(ops, m, mode, rel, heads=(0, 37, 127), target=None, lse_tol=1e-4, workers=None):
    lens_host = m["lens"]
    plan = (ops.plan_workers(lens_host, m["bs"], n_workers=workers) if workers
            else ops.plan_splits(lens_host, m["bs"], target_items=target))
    r = ops.latent_decode(t(m["q_lat"]), t(m["cache"]), t(m["tables"]), t(lens_host), plan,
                          scale=m["scale"], value_dim=m["Lv"], w_v=t(m["w_uv"]), mode=mode,
                          want_lse=True)
    ctx = r["ctx"].cpu().numpy()
    lse = r["lse"].cpu().numpy()
    w_can = m["w_uv"].transpose(1, 0, 2).reshape(m["Lv"], -1)   # canonical [Lv, Hq*D]
    bits = m["cache"].view(np.uint16)
    for b in range(len(lens_host)):
        n = int(lens_host[b])
        for h in heads:
            es, _, _, ec = c_ref.latent_decode_seq(
                m["q_lat"][b], bits, m["tables"][b], n, n, m["bs"], m["scale"],
                value_dim=m["Lv"], w_v_canonical=w_can, proj_heads=m["Hq"], head_dim=m["D"],
                heads=(h, h + 1), acc64=True)
            assert rel_err(ctx[b, h], ec[h]) <= rel, f"b={b} h={h} err={rel_err(ctx[b, h], ec[h])}"
            srow = es[h, :n].astype(np.float64)
            mx = srow.max()
            e_lse = mx + math.log(np.exp(srow - mx).sum())
            assert abs(lse[b, h] - e_lse) <= lse_tol * max(1.0, abs(e_lse))
    return r


def test_mla_exact_small_batch(ops, pkg):
    m = _mla_case(pkg, 3, [1, 777, 4096])
    _check_mla(ops, m, "exact", EXACT_REL)
    _check_mla(ops, m, "exact", EXACT_REL, target=1000)   # many splits, same answer


@pytest.mark.parametrize("lens", [[1, 777, 4096], [64, 65, 3000], [32, 5000]])
def test_mla_tensor_core_small_batch(ops, pkg, lens):
    m = _mla_case(pkg, len(lens), lens, seed=7)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    plan = ops.plan_splits(m["lens"], m["bs"])
    ops.latent_decode(t(m["q_lat"]), t(m["cache"]), t(m["tables"]), t(m["lens"]), plan,
                      scale=m["scale"], value_dim=m["Lv"], w_v=t(m["w_uv"]), mode="tc",
                      flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    _check_mla(ops, m, "tc", TC_REL, heads=(0, 63, 64, 127), lse_tol=2e-3)
    _check_mla(ops, m, "tc", TC_REL, heads=(5, 100), target=3, lse_tol=2e-3)
    # Persistent CTA pairs: several items per worker, items crossing sequences.
    _check_mla(ops, m, "tc", TC_REL, heads=(1, 66), lse_tol=2e-3, workers=2)
    _check_mla(ops, m, "tc", TC_REL, heads=(2, 127), lse_tol=2e-3, workers=5)


@pytest.mark.parametrize("workers", [0, 1, 7, 74])
def test_tensor_core_matches_exact_mode(ops, pkg, workers):
    m = _mla_case(pkg, 5, [900, 2048, 0, 131, 6000], seed=13)
    outs = {}
    for mode in ("exact", "tc"):
        plan = (ops.plan_workers(m["lens"], m["bs"], n_workers=workers) if mode == "tc" and workers
                else ops.plan_splits(m["lens"], m["bs"]))
        outs[mode] = ops.latent_decode(t(m["q_lat"]), t(m["cache"]), t(m["tables"]),
                                       t(m["lens"]), plan, scale=m["scale"], value_dim=m["Lv"],
                                       w_v=t(m["w_uv"]), mode=mode, want_lse=True,
                                       allow_empty=True)
    assert rel_err(outs["tc"]["ctx"].cpu(), outs["exact"]["ctx"].cpu()) <= TC_REL
    le, lt = outs["exact"]["lse"].cpu(), outs["tc"]["lse"].cpu()
    fin = torch.isfinite(le)
    assert torch.equal(fin, torch.isfinite(lt))
    assert rel_err(lt[fin], le[fin]) <= TC_REL


@pytest.mark.parametrize("workers,bs", [(0, 64), (3, 64), (3, 256), (5, 128), (4, 32)])
def test_tensor_core_ignores_nonfinite_slots_past_the_end(ops, pkg, workers, bs):
    """Pool slots past a sequence's length (the rest of its last block, and
    blocks no table names) hold NaN and Inf: the tensor-core pass reads whole
    row groups there but must weigh them by exactly zero, as the exact pass,
    which never reads them, does.  Block sizes 32 / 64 / 128 / 256 place a
    tile's pages at every offset inside a block (32: a 64-token tile spans
    two blocks)."""
    lens = [777, 131, 4101, 64, 33, 320]
    m = _mla_case(pkg, len(lens), lens, seed=17, bs=bs)
    cache = m["cache"].reshape(-1, m["L"])          # [P * bs, L] view
    used = np.zeros(cache.shape[0], bool)
    for b, n in enumerate(lens):
        for tok in range(n):
            used[m["tables"][b, tok // m["bs"]] * m["bs"] + tok % m["bs"]] = True
    bad = np.nonzero(~used)[0]
    cache[bad[0::2]] = np.float16(np.nan)
    cache[bad[1::2]] = np.float16(np.inf)
    outs = {}
    for mode in ("exact", "tc"):
        plan = (ops.plan_workers(m["lens"], m["bs"], n_workers=workers) if mode == "tc" and workers
                else ops.plan_splits(m["lens"], m["bs"]))
        outs[mode] = ops.latent_decode(t(m["q_lat"]), t(m["cache"]), t(m["tables"]),
                                       t(m["lens"]), plan, scale=m["scale"], value_dim=m["Lv"],
                                       w_v=t(m["w_uv"]), mode=mode, want_lse=True)
    assert torch.isfinite(outs["tc"]["ctx"]).all() and torch.isfinite(outs["tc"]["lse"]).all()
    assert rel_err(outs["tc"]["ctx"].cpu(), outs["exact"]["ctx"].cpu()) <= TC_REL
    assert rel_err(outs["tc"]["lse"].cpu(), outs["exact"]["lse"].cpu()) <= TC_REL


def test_tensor_core_rejects_block_size_16(ops, pkg):
    """The tensor-core pass loads whole 32-row halves of a block per TMA box."""
    m = _mla_case(pkg, 1, [100], seed=3, bs=16)
    plan = ops.plan_workers(m["lens"], m["bs"])
    with pytest.raises(Exception, match="unsupported"):
        ops.latent_decode(t(m["q_lat"]), t(m["cache"]), t(m["tables"]), t(m["lens"]), plan,
                          scale=m["scale"], value_dim=m["Lv"], w_v=t(m["w_uv"]), mode="tc")


def test_tensor_core_rejects_intermediates(ops, pkg):
    m = _mla_case(pkg, 1, [100], seed=3)
    plan = ops.plan_splits(m["lens"], m["bs"])
    with pytest.raises(Exception):
        ops.latent_decode(t(m["q_lat"]), t(m["cache"]), t(m["tables"]), t(m["lens"]), plan,
                          scale=m["scale"], value_dim=m["Lv"], w_v=t(m["w_uv"]), mode="tc",
                          want_scores=True, max_seq_len=100)


def test_split_invariance_and_empty_sequences(ops, pkg):
    m = _mla_case(pkg, 4, [0, 64, 3000, 1], seed=9)
    lens_host = m["lens"]
    outs = []
    for target in (4, 37, 500):
        plan = ops.plan_splits(lens_host, m["bs"], target_items=target)
        r = ops.latent_decode(t(m["q_lat"]), t(m["cache"]), t(m["tables"]), t(lens_host), plan,
                              scale=m["scale"], value_dim=m["Lv"], w_v=t(m["w_uv"]),
                              want_lse=True, allow_empty=True)
        outs.append(r)
    for r in outs[1:]:
        assert rel_err(r["ctx"].cpu(), outs[0]["ctx"].cpu()) <= 1e-6
    ctx0 = outs[0]["ctx"].cpu().numpy()
    assert np.all(ctx0[0] == 0) and np.all(np.isneginf(outs[0]["lse"].cpu().numpy()[0]))


def test_lse_merge_equals_unsplit_decode(ops, pkg):
    """Split-K across shards: decode each shard's block range, merge with LSE."""
    m = _mla_case(pkg, 2, [5000, 1300], seed=11)
    lens_host = m["lens"]
    full = ops.latent_decode(t(m["q_lat"]), t(m["cache"]), t(m["tables"]), t(lens_host),
                             ops.plan_splits(lens_host, m["bs"]), scale=m["scale"],
                             value_dim=m["Lv"], w_v=t(m["w_uv"]), want_lse=True)
    shards = 3
    nb = (lens_host + m["bs"] - 1) // m["bs"]
    ctxs, lses = [], []
    for r in range(shards):
        lo, hi = nb * r // shards, nb * (r + 1) // shards
        tab = np.full_like(m["tables"], -1)
        local = np.zeros_like(lens_host)
        for b in range(2):
            tab[b, :hi[b] - lo[b]] = m["tables"][b, lo[b]:hi[b]]
            local[b] = max(0, min(lens_host[b], hi[b] * m["bs"]) - lo[b] * m["bs"])
        rr = ops.latent_decode(t(m["q_lat"]), t(m["cache"]), t(tab), t(local),
                               ops.plan_splits(local, m["bs"]), scale=m["scale"],
                               value_dim=m["Lv"], w_v=t(m["w_uv"]), want_lse=True,
                               allow_empty=True)
        ctxs.append(rr["ctx"])
        lses.append(rr["lse"])
    merged, lse = ops.lse_merge(torch.stack(ctxs), torch.stack(lses))
    assert rel_err(merged.cpu(), full["ctx"].cpu()) <= 1e-5
    assert rel_err(lse.cpu(), full["lse"].cpu()) <= 1e-5


def test_long_context_full_size_sampled(ops, pkg):
    """The long-context workload at full size (8 x 131072 tokens): FP64 oracle
    on sampled (sequence, head) rows."""
    s = pkg.workloads.spec("long_context")
    x = pkg.workloads.device_inputs(s, DEV)
    plan = ops.plan_splits(x["lens"], s.block_size)
    lens = t(x["lens"])
    r = ops.latent_decode(x["q_lat"], x["cache"], x["tables"], lens, plan, scale=s.scale,
                          value_dim=s.value_dim, w_v=x["w_v"], want_lse=True)
    torch.cuda.synchronize()
    ctx = r["ctx"].cpu().numpy()
    bits = f16_to_bits(x["cache"])
    q_lat = x["q_lat"].cpu().numpy()
    w_can = x["w_v"].cpu().numpy().transpose(1, 0, 2).reshape(s.value_dim, -1)
    tables = x["tables"].cpu().numpy()
    for b, h in ((0, 0), (3, 77), (7, 127)):
        n = int(x["lens"][b])
        _, _, _, ec = c_ref.latent_decode_seq(q_lat[b], bits, tables[b], n, n, s.block_size,
                                              s.scale, value_dim=s.value_dim, w_v_canonical=w_can,
                                              proj_heads=s.proj_heads, head_dim=s.head_dim,
                                              heads=(h, h + 1), acc64=True,
                                              want_intermediates=False)
        assert rel_err(ctx[b, h], ec[h]) <= EXACT_REL, (b, h, rel_err(ctx[b, h], ec[h]))
    assert np.all(np.isfinite(ctx))


def test_long_context_tensor_core_full_size(ops, pkg):
    """Tensor-core mode on the full long-context workload against exact mode."""
    s = pkg.workloads.spec("long_context")
    x = pkg.workloads.device_inputs(s, DEV)
    lens = t(x["lens"])
    res = {}
    for mode in ("exact", "tc"):
        plan = (ops.plan_workers(x["lens"], s.block_size) if mode == "tc"
                else ops.plan_splits(x["lens"], s.block_size))
        res[mode] = ops.latent_decode(x["q_lat"], x["cache"], x["tables"], lens, plan,
                                      scale=s.scale, value_dim=s.value_dim, w_v=x["w_v"],
                                      mode=mode)["ctx"].cpu()
    assert rel_err(res["tc"], res["exact"]) <= TC_REL


def test_write_attend_fullkv_matches_latent(ops, pkg):
    """Full-KV baseline on K/V derived from the same latent rows agrees with
    the latent path up to FP16 rounding of K and V (2e-3)."""
    s = pkg.workloads.spec("tiny")
    x, _ = regenerate(pkg, "tiny")
    g = load_golden_json("tiny_workload.json")
    khm = bits_to_f16(np.asarray(g["k_tok_f16_bits"], np.uint16).transpose(0, 2, 1, 3))
    vhm = bits_to_f16(np.asarray(g["v_tok_f16_bits"], np.uint16).transpose(0, 2, 1, 3))
    plan = ops.plan_splits(x["lens"], s.block_size)
    r = ops.fullkv_decode(t(x["q"]), khm, vhm, t(x["tables"]), t(x["lens"]), plan, scale=s.scale)
    assert_close(r["ctx"].cpu(), np.asarray(g["ctx"]), 2e-2, 2e-2, "full-KV vs latent")
