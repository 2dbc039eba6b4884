"""Pin the CPU oracle (C restatement of lib.rs + NumPy restatement of
attention_ref.py) against the reference's golden vectors.

Tolerances are the reference's own CPU-vs-Python ones
(crates/plkv-core/src/lib.rs:2272-2274: scores 5e-5, probabilities 5e-5,
context 1e-4, each + 1e-5 relative); FP16 storage bits are bit-exact.
"""

import numpy as np
import pytest

from conftest import GOLDEN, load_golden_json, load_reference_fixture
from oracle import c_ref, np_ref

SCORE_TOL = (5e-5, 1e-5)
PROB_TOL = (5e-5, 1e-5)
CTX_TOL = (1e-4, 1e-5)


def assert_close(actual, expected, tol, label=""):
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    assert actual.shape == expected.shape, label
    atol, rtol = tol
    bad = np.abs(actual - expected) > atol + rtol * np.abs(expected)
    assert not bad.any(), (f"{label}: {bad.sum()} mismatches, max abs err "
                           f"{np.max(np.abs(actual - expected)):.3g}")


# ------------------------------------------------------------------- FP16

def test_f16_conversion_matches_numpy_round_to_nearest_even():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10,
        rng.standard_normal(5000).astype(np.float32) * 1e-5,      # subnormal range
        rng.standard_normal(5000).astype(np.float32) * 3e4,
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, -65520.0, 5.96e-8, 2.98e-8,
                  2.9802322e-08, 6.1035156e-05, 1.0009765625, 1.00048828125,
                  1.00146484375], dtype=np.float32),
    ])
    # Exact ties: halfway between representable halves.
    ties = (np.arange(1024, 2048, dtype=np.float32) + np.float32(0.5)) / np.float32(1024)
    vals = np.concatenate([vals, ties, -ties]).astype(np.float32)
    with np.errstate(over="ignore"):
        expected = vals.astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(c_ref.f32_to_f16_bits(vals), expected)


def test_quantize_rejects_non_finite_and_overflow():
    # test_attention_shapes.py:120-124 / lib.rs:307-316
    with pytest.raises(c_ref.OracleError) as e:
        c_ref.quantize_f16(np.array([70000.0], dtype=np.float32))
    assert e.value.status == 7
    with pytest.raises(c_ref.OracleError) as e:
        c_ref.quantize_f16(np.array([np.inf], dtype=np.float32))
    assert e.value.status == 6
    with pytest.raises(ValueError):
        np_ref.fp16_storage_roundtrip_f32(np.array([70000.0], dtype=np.float32))
    with pytest.raises(ValueError):
        np_ref.fp16_storage_roundtrip_f32(np.array([np.nan], dtype=np.float32))


@pytest.mark.parametrize("case", [0, 1])
def test_fp16_fixture_bits(case):
    fx = load_reference_fixture("paged_latent_write_attention_fp16_storage.json")
    c = fx["cases"][case]
    init = np.asarray(c["initial_latent_source_f32"], dtype=np.float32)
    new = np.asarray(c["new_latent_source_f32"], dtype=np.float32)
    np.testing.assert_array_equal(c_ref.quantize_f16(init),
                                  np.asarray(c["initial_latent_fp16_bits"], dtype=np.uint16))
    np.testing.assert_array_equal(c_ref.quantize_f16(new),
                                  np.asarray(c["new_latent_fp16_bits"], dtype=np.uint16))
    np.testing.assert_array_equal(np_ref.fp16_storage_bits(init),
                                  np.asarray(c["initial_latent_fp16_bits"], dtype=np.uint16))


# -------------------------------------------------------------- addressing

@pytest.mark.parametrize(("pos", "expected"), [(3, (1, 0, 1)), (4, (2, 1, 0))])
def test_resolve_location(pos, expected):
    # tests/test_cache_ref.py:16-19 of the reference
    table = np.array([2, 0, 1])
    assert np_ref.resolve_paged_token_location(table, pos, 2) == expected
    assert c_ref.resolve_location(table, pos, 2, 4) == expected


def test_resolve_location_errors():
    table = np.array([2, 0, 1])
    with pytest.raises(ValueError):
        np_ref.resolve_paged_token_location(table, 0, 0)
    with pytest.raises(IndexError):
        np_ref.resolve_paged_token_location(table, 6, 2)
    with pytest.raises(c_ref.OracleError):
        c_ref.resolve_location(table, 6, 2, 4)
    with pytest.raises(c_ref.OracleError):
        c_ref.resolve_location(np.array([4, 0, 1]), 0, 2, 4)


def test_block_table_fixtures():
    for name in ("block_table_seq5_block2.json", "block_table_seq128_block16.json"):
        fx = load_reference_fixture(name)
        t = np_ref.PagedBlockTable(fx["block_size"])
        t.allocate_token_positions(fx["seq_len"])
        assert t.to_list() == fx["logical_blocks"]
        for loc in fx["token_locations"]:
            assert t.translate(loc["token"]) == (loc["physical_block"], loc["offset"])


def test_paged_lookup_fixture():
    fx = load_reference_fixture("paged_lookup_f32_seq5_block2_width4.json")
    out = np_ref.paged_lookup_ref(np.asarray(fx["physical_blocks"], dtype=np.float32),
                                  np.asarray(fx["block_table"]), fx["seq_len"], fx["block_size"])
    np.testing.assert_array_equal(out, np.asarray(fx["expected_logical_output"], np.float32))


# ------------------------------------------------------------------ writes

@pytest.mark.parametrize("case", [0, 1])
def test_latent_write_fp16_bit_exact(case):
    fx = load_reference_fixture("paged_latent_write_attention_fp16_storage.json")
    c = fx["cases"][case]
    init_bits = np.asarray(c["initial_latent_fp16_bits"], dtype=np.uint16)
    updated = c_ref.latent_write_f16(init_bits, fx["block_table"], c["token_position"],
                                     c["new_latent_source_f32"])
    np.testing.assert_array_equal(updated, np.asarray(c["expected_updated_latent_fp16_bits"],
                                                      dtype=np.uint16))
    ref = np_ref.paged_latent_write_fp16_storage_ref(
        np.asarray(c["initial_latent_source_f32"], np.float32), np.asarray(fx["block_table"]),
        c["token_position"], np.asarray(c["new_latent_source_f32"], np.float32))
    np.testing.assert_array_equal(ref, np.asarray(c["expected_updated_latent_fp16_as_f32"],
                                                  np.float32))
    # exactly one row changed
    changed = np.any(updated != init_bits, axis=-1)
    assert changed.sum() <= 1


def test_latent_write_rejects_bad_inputs():
    cache = np.zeros((4, 2, 8), np.uint16)
    for table, pos, row in (([2, 0, 3, 1], 8, [0.0] * 8), ([4, 0, 3, 1], 0, [0.0] * 8)):
        with pytest.raises(c_ref.OracleError):
            c_ref.latent_write_f16(cache, table, pos, row)
    with pytest.raises(c_ref.OracleError):
        c_ref.latent_write_f16(cache, [2, 0, 3, 1], 0, [np.inf] + [0.0] * 7)


@pytest.mark.parametrize("case", [0, 1])
def test_kv_write_fixture(case):
    fx = load_reference_fixture("paged_kv_write_f32.json")
    c = fx["cases"][case]
    P, bs, KV, D = fx["num_physical_blocks"], fx["block_size"], fx["kv_heads"], fx["head_dim"]

    def to_hm_bits(tok):  # token-major [P, bs, KV*D] -> head-major bits [P, KV, bs, D]
        a = np.asarray(tok, np.float32).reshape(P, bs, KV, D).transpose(0, 2, 1, 3)
        return c_ref.quantize_f16(a)

    k, v = c_ref.kv_write_f16(to_hm_bits(c["initial_k_cache"]), to_hm_bits(c["initial_v_cache"]),
                              fx["block_table"], c["token_position"], c["new_k"], c["new_v"])
    np.testing.assert_array_equal(k, to_hm_bits(c["expected_k_cache"]))
    np.testing.assert_array_equal(v, to_hm_bits(c["expected_v_cache"]))
    ek, ev = np_ref.paged_kv_write_ref(
        np.asarray(c["initial_k_cache"], np.float32), np.asarray(c["initial_v_cache"], np.float32),
        np.asarray(fx["block_table"]), c["token_position"], np.asarray(c["new_k"], np.float32),
        np.asarray(c["new_v"], np.float32))
    np.testing.assert_array_equal(ek, np.asarray(c["expected_k_cache"], np.float32))
    np.testing.assert_array_equal(ev, np.asarray(c["expected_v_cache"], np.float32))


# ------------------------------------------------------------------ decode

def _c_decode(q, cache_bits, table, active, max_len, bs, kp, vp, KV, D, acc64=False):
    """C oracle on one sequence through the reference's argument convention."""
    q = np.asarray(q, np.float32).reshape(-1, D)
    q_lat = c_ref.project_query(q, kp, KV)
    Hq = q.shape[0]
    return c_ref.latent_decode_seq(q_lat, cache_bits, table, active, max_len, bs,
                                   1.0 / np.sqrt(D), w_v_canonical=vp, proj_heads=KV,
                                   head_dim=D, acc64=acc64)


@pytest.mark.parametrize("acc64", [False, True])
@pytest.mark.parametrize("phase", ["pre", "post"])
@pytest.mark.parametrize("case", [0, 1])
def test_fp16_write_then_attend_fixture(case, phase, acc64):
    fx = load_reference_fixture("paged_latent_write_attention_fp16_storage.json")
    c = fx["cases"][case]
    bits = np.asarray(c["initial_latent_fp16_bits"], np.uint16)
    if phase == "post":
        bits = c_ref.latent_write_f16(bits, fx["block_table"], c["token_position"],
                                      c["new_latent_source_f32"])
    kp = np.asarray(c["k_projection"], np.float32)
    vp = np.asarray(c["v_projection"], np.float32)
    s, p, _, ctx = _c_decode(c["q"], bits, fx["block_table"], 8, 8, 2, kp, vp, 2, 8, acc64)
    pre = f"fp16_storage_{phase}_write_"
    assert_close(s, c[pre + "scores"], SCORE_TOL, "scores")
    assert_close(p, c[pre + "probabilities"], PROB_TOL, "probabilities")
    assert_close(ctx, c[pre + "context"], CTX_TOL, "context")


@pytest.mark.parametrize("case", [0, 1])
def test_runtime_active_lengths_fixture(case):
    fx = load_reference_fixture("runtime_sequence_tiny_fp16_storage.json")
    c = fx["cases"][case]
    bits = np.asarray(c["initial_latent_fp16_bits"], np.uint16)
    kp = np.asarray(c["k_projection"], np.float32)
    vp = np.asarray(c["v_projection"], np.float32)
    for rc in c["runtime_cases"]:
        n = rc["active_seq_len"]
        s, p, _, ctx = _c_decode(c["q"], bits, fx["block_table"], n, fx["max_seq_len"],
                                 fx["block_size"], kp, vp, fx["kv_heads"], fx["head_dim"])
        es = np.asarray(rc["scores"], np.float32)
        ep = np.asarray(rc["probabilities"], np.float32)
        assert_close(s[:, :n], es[:, :n], SCORE_TOL, f"scores n={n}")
        assert np.all(s[:, n:] == np.float32(-3.4028234663852886e38))
        assert np.all(es[:, n:] == s[:, n:])
        assert_close(p, ep, PROB_TOL, f"probs n={n}")
        assert np.all(p[:, n:] == 0.0) and rc["inactive_probabilities_zero"]
        assert np.max(np.abs(p.sum(axis=-1) - 1.0)) <= 1e-6
        assert_close(ctx, rc["context"], CTX_TOL, f"context n={n}")


@pytest.mark.parametrize("case", [0, 1])
def test_np_oracle_direct_paged_fixture(case):
    fx = load_reference_fixture("direct_paged_latent_gqa_decode_f32.json")
    c = fx["cases"][case]
    q = np.asarray(c["q"], np.float32)[None]
    s, p, ctx = np_ref.direct_paged_latent_gqa_decode_attention_intermediates_ref(
        q, np.asarray(c["latent_physical_blocks"], np.float32), np.asarray(fx["block_table"]),
        fx["seq_len"], fx["block_size"], np.asarray(c["k_projection"], np.float32),
        np.asarray(c["v_projection"], np.float32), q_heads=4, kv_heads=2, head_dim=8,
        group_size=2)
    assert_close(s[0], c["expected_scores"], SCORE_TOL, "scores")
    assert_close(p[0], c["expected_probabilities"], PROB_TOL, "probs")
    assert_close(ctx[0], c["expected_context"], CTX_TOL, "context")


@pytest.mark.parametrize("case", [0, 1])
def test_np_oracle_paged_gqa_fixture(case):
    fx = load_reference_fixture("paged_gqa_decode_f32.json")
    c = fx["cases"][case]
    s, p, ctx = np_ref.paged_gqa_decode_attention_intermediates_ref(
        np.asarray(c["q"], np.float32)[None], np.asarray(c["k_physical_token_major"], np.float32),
        np.asarray(c["v_physical_token_major"], np.float32), np.asarray(fx["block_table"]),
        fx["seq_len"], fx["block_size"], group_size=fx["group_size"])
    assert_close(s[0], c["expected_scores"], (1e-5, 1e-5), "scores")
    assert_close(p[0], c["expected_probabilities"], (1e-5, 1e-5), "probs")
    assert_close(ctx[0], c["expected_context"], (1e-5, 1e-5), "context")


@pytest.mark.parametrize("case", [0, 1])
def test_c_oracle_fullkv_on_gpu_head_major_fixture(case):
    # paged_gqa_decode_f32.json carries the GPU head-major physical layout
    # (fixtures.py:188-190); its values are FP32, so compare against the FP16
    # rounding through the NumPy oracle and the fixture with the FP16 ladder.
    fx = load_reference_fixture("paged_gqa_decode_f32.json")
    c = fx["cases"][case]
    k32 = np.asarray(c["k_physical_gpu_head_major"], np.float32)
    v32 = np.asarray(c["v_physical_gpu_head_major"], np.float32)
    kb, vb = c_ref.quantize_f16(k32), c_ref.quantize_f16(v32)
    q = np.asarray(c["q"], np.float32)
    s, p, ctx = c_ref.fullkv_decode_seq(q, kb, vb, fx["block_table"], 8, 8, 1 / np.sqrt(8))
    k16 = kb.view(np.float16).astype(np.float32).transpose(0, 2, 1, 3)
    v16 = vb.view(np.float16).astype(np.float32).transpose(0, 2, 1, 3)
    es, ep, ec = np_ref.paged_gqa_decode_attention_intermediates_ref(
        q[None], k16, v16, np.asarray(fx["block_table"]), 8, 2, group_size=2)
    assert_close(s, es[0], SCORE_TOL, "scores")
    assert_close(p, ep[0], PROB_TOL, "probs")
    assert_close(ctx, ec[0], CTX_TOL, "context")
    assert_close(ctx, c["expected_context"], (2e-3, 1e-2), "context vs fp32 fixture")


def test_tiny_workload_golden():
    g = load_golden_json("tiny_workload.json")
    bits = np.asarray(g["cache_f16_bits"], np.uint16)
    kp = np.asarray(g["w_k"], np.float32)
    vp = np.asarray(g["w_v"], np.float32)
    q = np.asarray(g["q"], np.float32)
    ktok = np.asarray(g["k_tok_f16_bits"], np.uint16)
    vtok = np.asarray(g["v_tok_f16_bits"], np.uint16)
    khm, vhm = ktok.transpose(0, 2, 1, 3).copy(), vtok.transpose(0, 2, 1, 3).copy()
    for b, n in enumerate(g["lens"]):
        table = np.asarray(g["tables"][b])
        s, p, _, ctx = _c_decode(q[b], bits, table, n, g["max_seq_len"], 4, kp, vp, 2, 16)
        assert_close(s[:, :n], np.asarray(g["scores"][b])[:, :n], SCORE_TOL, "scores")
        assert_close(p, g["probs"][b], PROB_TOL, "probs")
        assert_close(ctx, g["ctx"][b], CTX_TOL, "ctx")
        fs, fp, fc = c_ref.fullkv_decode_seq(q[b], khm, vhm, table, n, n, 0.25)
        assert_close(fs, g["fullkv_scores"][b], SCORE_TOL, "fullkv scores")
        assert_close(fp, g["fullkv_probs"][b], PROB_TOL, "fullkv probs")
        assert_close(fc, g["fullkv_ctx"][b], CTX_TOL, "fullkv ctx")
    ctx = np.asarray(g["ctx"], np.float32).reshape(2, -1)
    out = c_ref.out_proj(ctx, np.asarray(g["w_o"], np.float32), acc64=True)
    assert_close(out, g["out_f64"], (1e-5, 1e-5), "W_o")


def test_model_small_kat():
    d = np.load(f"{GOLDEN}/model_small_kat.npz")
    bits = c_ref.quantize_f16(d["latent_f32"])
    q = d["q"][0]
    q_lat = c_ref.project_query(q, d["k_proj"], 4)
    for n in d["active_lens"]:
        n = int(n)
        s, p, _, ctx = c_ref.latent_decode_seq(q_lat, bits, d["table"], n, 1024, 16, 1 / 8.0,
                                               w_v_canonical=d["v_proj"], proj_heads=4,
                                               head_dim=64)
        assert_close(s[:, :n], d[f"scores_{n}"][:, :n], SCORE_TOL, f"scores {n}")
        assert_close(p, d[f"probs_{n}"], PROB_TOL, f"probs {n}")
        assert_close(ctx, d[f"ctx_{n}"], CTX_TOL, f"ctx {n}")


def test_model_shaped_golden(pkg):
    from tests_support import model_shaped_inputs

    d = np.load(f"{GOLDEN}/model_shaped.npz")
    x, s = model_shaped_inputs(pkg, str(d["inputs_sha256"]))
    n = int(x["lens"][0])
    table = x["tables"][0]
    bits = c_ref.latent_write_f16(x["cache_f16"].view(np.uint16), table, n - 1, x["new_rows"][0, 0])
    phys = table[(n - 1) // s.block_size]
    np.testing.assert_array_equal(bits[phys, (n - 1) % s.block_size], d["updated_row_bits"])
    q_lat = c_ref.project_query(x["q"][0], x["w_k"], s.kv_heads)
    sc, p, _, ctx = c_ref.latent_decode_seq(q_lat, bits, table, n, n, s.block_size, s.scale,
                                            w_v_canonical=x["w_v"], proj_heads=s.kv_heads,
                                            head_dim=s.head_dim)
    assert_close(sc, d["scores"], SCORE_TOL, "scores")
    assert_close(p, d["probs"], PROB_TOL, "probs")
    assert_close(ctx, d["ctx"], CTX_TOL, "ctx")


@pytest.mark.parametrize("case", [0, 1])
def test_reconstruction_fixture(case):
    """latent_kv_reconstruction_f32.json: the C restatement of
    reconstruct_latent_kv_f32 (lib.rs:517-580) and the NumPy restatement of
    latent_kv_reconstruction_ref (attention_ref.py:227-274) at the reference's
    CPU tolerances (latent_kv_reconstruction_gpu.rs:10-11: 1e-5 / 1e-5)."""
    from oracle import np_ref

    fx = load_reference_fixture("latent_kv_reconstruction_f32.json")
    c = fx["cases"][case]
    KV, D = fx["kv_heads"], fx["head_dim"]
    lat = np.asarray(c["latent_cache"], np.float32)
    kp = np.asarray(c["k_projection"], np.float32)
    vp = np.asarray(c["v_projection"], np.float32)
    ek = np.asarray(c["expected_k_token_major"], np.float32)
    ev = np.asarray(c["expected_v_token_major"], np.float32)
    k, v = c_ref.reconstruct_kv(lat, kp, vp)
    for got, exp in ((k, ek), (v, ev)):
        np.testing.assert_allclose(got.reshape(exp.shape), exp, rtol=1e-5, atol=1e-5)
    k_hm = k.reshape(-1, KV, D).transpose(1, 0, 2)
    np.testing.assert_allclose(k_hm, np.asarray(c["expected_k_head_major"]), rtol=1e-5, atol=1e-5)
    nk, nv = np_ref.latent_kv_reconstruction_ref(lat[None], kp, vp, kv_heads=KV, head_dim=D)
    np.testing.assert_allclose(nk[0], ek, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(nv[0], ev, rtol=1e-5, atol=1e-5)


def test_reconstruction_rejections():
    """lib.rs:2156-2176 and attention_ref.py:246-272: bad shapes and
    non-finite inputs are rejected."""
    from oracle import np_ref

    lat = np.zeros((8, 8), np.float32)
    proj = np.zeros((8, 16), np.float32)
    bad = lat.copy()
    bad[0, 0] = np.nan
    with pytest.raises(RuntimeError):
        c_ref.reconstruct_kv(bad, proj, proj)
    with pytest.raises(ValueError):
        np_ref.latent_kv_reconstruction_ref(lat, proj, proj, kv_heads=2, head_dim=8)
    with pytest.raises(ValueError):
        np_ref.latent_kv_reconstruction_ref(lat[None], proj[:, :15], proj[:, :15], kv_heads=2,
                                            head_dim=8)
    with pytest.raises(ValueError):
        np_ref.latent_kv_reconstruction_ref(lat[None], proj, proj[:, :8], kv_heads=2, head_dim=8)
    with pytest.raises(ValueError):
        np_ref.latent_kv_reconstruction_ref(lat[None], proj, proj, kv_heads=0, head_dim=8)
    huge = np.full((1, 1, 8), 3e38, np.float32)
    with pytest.raises(ValueError):
        np_ref.latent_kv_reconstruction_ref(huge, np.full((8, 16), 3e38, np.float32),
                                            np.full((8, 16), 3e38, np.float32), kv_heads=2,
                                            head_dim=8)
