"""Generate the golden vectors under tests/golden from the reference's own Python.

Run in a checkout that has tatavishnurao/LatentPagedAttention-rs next to it:

    python tests/golden/make_golden.py --reference <reference checkout>

It imports ``python_ref/latent_paged_attention`` and writes

* ``reference/*.json``  -- the reference's committed golden fixture files for
  the hot path (fixtures/reference/, written by fixtures.py:850-878), copied
  as data, and ``reference/regeneration_check.json`` -- the largest
  difference between them and a fresh run of the reference's generator
  functions here (ULP-level, from BLAS summation order);
* ``tiny_workload.json`` -- the tiny workload (B=2, per-sequence tables,
  lengths [7, 13]) through attention_ref.py:617-648 per sequence, the FP16
  full-KV baseline through attention_ref.py:172-224 and W_o in float64;
* ``model_small_kat.npz`` -- the deterministic model_small inputs of
  crates/plkv-kernels/examples/model_profile_gpu.rs:210-245 at active lengths
  17 / 129 / 513 / 1024 through attention_ref.py:617-648;
* ``model_shaped.npz`` -- the model-shaped workload (255 rows + one row
  written with cache_ref.py:103-114, then read at length 256).

Only this script reads the reference; tests read the files it writes.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

REFERENCE_FIXTURES = [
    "paged_latent_write_attention_fp16_storage.json",
    "runtime_sequence_tiny_fp16_storage.json",
    "direct_paged_latent_gqa_decode_f32.json",
    "paged_latent_write_attention_f32.json",
    "paged_gqa_decode_f32.json",
    "paged_kv_write_f32.json",
    "block_table_seq5_block2.json",
    "block_table_seq128_block16.json",
    "paged_lookup_f32_seq5_block2_width4.json",
    "latent_kv_reconstruction_f32.json",
]


def inputs_digest(arrays: dict) -> str:
    h = hashlib.sha256()
    for k in sorted(arrays):
        a = np.ascontiguousarray(arrays[k])
        h.update(k.encode())
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def _load_reference(path: str):
    sys.path.insert(0, os.path.join(path, "python_ref"))
    ar = importlib.import_module("latent_paged_attention.attention_ref")
    cr = importlib.import_module("latent_paged_attention.cache_ref")
    fx = importlib.import_module("latent_paged_attention.fixtures")
    return ar, cr, fx


def _load_workloads():
    sys.path.insert(0, ROOT)
    return importlib.import_module("latentpagedattention-rs_b200.workloads")


def _max_diff(a, b) -> float:
    if isinstance(a, dict):
        return max((_max_diff(a[k], b[k]) for k in a), default=0.0)
    if isinstance(a, list):
        try:
            x = np.asarray(a, dtype=np.float64)
            y = np.asarray(b, dtype=np.float64)
            return float(np.max(np.abs(x - y))) if x.size else 0.0
        except (ValueError, TypeError):
            return max((_max_diff(u, v) for u, v in zip(a, b)), default=0.0)
    if isinstance(a, (int, float)) and isinstance(b, (int, float)):
        return abs(float(a) - float(b))
    return 0.0 if a == b else float("inf")


def write_reference_fixtures(fx, ref_root: str, out_dir: str) -> None:
    os.makedirs(out_dir, exist_ok=True)
    makers = {
        "paged_latent_write_attention_fp16_storage.json":
            fx.paged_latent_write_attention_fp16_storage_fixture,
        "runtime_sequence_tiny_fp16_storage.json": fx.runtime_sequence_tiny_fp16_storage_fixture,
        "direct_paged_latent_gqa_decode_f32.json": fx.direct_paged_latent_gqa_decode_f32_fixture,
        "paged_latent_write_attention_f32.json": fx.paged_latent_write_attention_f32_fixture,
        "paged_gqa_decode_f32.json": fx.paged_gqa_decode_f32_fixture,
        "paged_kv_write_f32.json": fx.paged_kv_write_fixture,
        "block_table_seq5_block2.json": lambda: fx.block_table_fixture(5, 2),
        "block_table_seq128_block16.json": lambda: fx.block_table_fixture(128, 16),
        "paged_lookup_f32_seq5_block2_width4.json": fx.paged_lookup_f32_fixture,
        "latent_kv_reconstruction_f32.json": fx.latent_kv_reconstruction_f32_fixture,
    }
    drift = {}
    for name in REFERENCE_FIXTURES:
        with open(os.path.join(ref_root, "fixtures", "reference", name), encoding="utf-8") as f:
            committed_text = f.read()
        committed = json.loads(committed_text)
        drift[name] = _max_diff(committed, json.loads(json.dumps(makers[name]())))
        with open(os.path.join(out_dir, name), "w", encoding="utf-8") as f:
            f.write(committed_text)
    with open(os.path.join(out_dir, "regeneration_check.json"), "w", encoding="utf-8") as f:
        json.dump({"max_abs_difference_committed_vs_regenerated": drift}, f, indent=2)
        f.write("\n")


def tiny_workload(ar, wl) -> dict:
    s = wl.spec("tiny")
    x = wl.host_inputs(s)
    B, Hq, KV, D, L, bs = s.batch, s.q_heads, s.kv_heads, s.head_dim, s.latent_dim, s.block_size
    G = Hq // KV
    lens = x["lens"]
    max_len = int(lens.max())
    cache32 = x["cache_f16"].astype(np.float32)
    # Full-KV baseline storage derived from the same latent rows:
    # K = fp16(L W_k), V = fp16(L W_v), token-major [P, bs, KV, D].
    k_tok = (cache32.reshape(-1, L) @ x["w_k"]).reshape(-1, bs, KV, D).astype(np.float16)
    v_tok = (cache32.reshape(-1, L) @ x["w_v"]).reshape(-1, bs, KV, D).astype(np.float16)
    out = {"lens": lens.tolist(), "tables": x["tables"].tolist(), "max_seq_len": max_len,
           "q": x["q"].tolist(), "w_k": x["w_k"].tolist(), "w_v": x["w_v"].tolist(),
           "w_o": x["w_o"].tolist(),
           "cache_f16_bits": x["cache_f16"].view(np.uint16).tolist(),
           "k_tok_f16_bits": k_tok.view(np.uint16).tolist(),
           "v_tok_f16_bits": v_tok.view(np.uint16).tolist(),
           "scores": [], "probs": [], "ctx": [], "fullkv_scores": [], "fullkv_probs": [],
           "fullkv_ctx": []}
    for b in range(B):
        nb = (int(lens[b]) + bs - 1) // bs
        table = x["tables"][b, :nb].astype(np.int64)
        sc, pr, cx = ar.direct_paged_latent_gqa_fp16_storage_runtime_intermediates_ref(
            x["q"][b:b + 1], cache32, table, max_len, int(lens[b]), bs, x["w_k"], x["w_v"],
            q_heads=Hq, kv_heads=KV, head_dim=D, group_size=G)
        out["scores"].append(sc[0].tolist())
        out["probs"].append(pr[0].tolist())
        out["ctx"].append(cx[0].tolist())
        fs, fp, fc = ar.paged_gqa_decode_attention_intermediates_ref(
            x["q"][b:b + 1], k_tok.astype(np.float32), v_tok.astype(np.float32), table,
            int(lens[b]), bs, group_size=G)
        out["fullkv_scores"].append(fs[0].tolist())
        out["fullkv_probs"].append(fp[0].tolist())
        out["fullkv_ctx"].append(fc[0].tolist())
    ctx = np.asarray(out["ctx"], dtype=np.float64).reshape(B, Hq * D)
    out["out_f64"] = (ctx @ x["w_o"].astype(np.float64)).tolist()
    out["inputs_sha256"] = inputs_digest({k: v for k, v in x.items() if isinstance(v, np.ndarray)})
    return out


def _deterministic_values(n: int, step: float, offset: float) -> np.ndarray:
    """model_profile_gpu.rs:215-222, evaluated in float64 then rounded to float32."""
    idx = np.arange(n)
    lane = (idx % 257).astype(np.float64)
    vals = np.array([math.sin(v) for v in (lane * step + offset)]) * 0.75
    return (vals + ((idx % 13) - 6.0) * 0.01).astype(np.float32)


def model_small_kat(ar) -> dict:
    Hq, KV, G, D, L, bs, max_len, P = 16, 4, 4, 64, 32, 16, 1024, 64
    table = np.array([(l * 17 + 11) % P for l in range(P)], dtype=np.int64)
    q = _deterministic_values(Hq * D, 0.011, -0.4).reshape(1, Hq, D)
    logical = _deterministic_values(max_len * L, 0.007, -1.2).reshape(P, bs, L)
    physical = np.empty_like(logical)
    physical[table] = logical
    k_proj = _deterministic_values(L * KV * D, 0.005, -0.7).reshape(L, KV * D)
    v_proj = _deterministic_values(L * KV * D, 0.006, 0.3).reshape(L, KV * D)
    out = {"q": q, "latent_f32": physical, "table": table.astype(np.int32), "k_proj": k_proj,
           "v_proj": v_proj, "active_lens": np.array([17, 129, 513, 1024], dtype=np.int32)}
    for n in (17, 129, 513, 1024):
        sc, pr, cx = ar.direct_paged_latent_gqa_fp16_storage_runtime_intermediates_ref(
            q, physical, table, max_len, n, bs, k_proj, v_proj, q_heads=Hq, kv_heads=KV,
            head_dim=D, group_size=G)
        out[f"scores_{n}"] = sc[0]
        out[f"probs_{n}"] = pr[0]
        out[f"ctx_{n}"] = cx[0]
    return out


def model_shaped(ar, cr, wl) -> dict:
    s = wl.spec("model_shaped")
    x = wl.host_inputs(s)
    Hq, KV, D, bs = s.q_heads, s.kv_heads, s.head_dim, s.block_size
    n = int(x["lens"][0])
    nb = (n + bs - 1) // bs
    table = x["tables"][0, :nb].astype(np.int64)
    updated = cr.paged_latent_write_fp16_storage_ref(x["cache_f16"].astype(np.float32), table,
                                                     n - 1, x["new_rows"][0, 0])
    sc, pr, cx = ar.direct_paged_latent_gqa_fp16_storage_runtime_intermediates_ref(
        x["q"], updated, table, n, n, bs, x["w_k"], x["w_v"], q_heads=Hq, kv_heads=KV,
        head_dim=D, group_size=Hq // KV)
    out_f64 = cx.reshape(1, -1).astype(np.float64) @ x["w_o"].astype(np.float64)
    return {"scores": sc[0], "probs": pr[0], "ctx": cx[0], "out_f64": out_f64[0],
            "updated_row_bits": updated[table[(n - 1) // bs], (n - 1) % bs].astype(
                np.float16).view(np.uint16),
            "inputs_sha256": np.array(inputs_digest(
                {k: v for k, v in x.items() if isinstance(v, np.ndarray)}))}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=os.environ.get("PLKV_REFERENCE"), required=
                    os.environ.get("PLKV_REFERENCE") is None,
                    help="root of a checkout of the reference project (or set PLKV_REFERENCE)")
    args = ap.parse_args()
    ar, cr, fx = _load_reference(args.reference)
    wl = _load_workloads()
    write_reference_fixtures(fx, args.reference, os.path.join(HERE, "reference"))
    with open(os.path.join(HERE, "tiny_workload.json"), "w", encoding="utf-8") as f:
        json.dump(tiny_workload(ar, wl), f)
        f.write("\n")
    np.savez_compressed(os.path.join(HERE, "model_small_kat.npz"), **model_small_kat(ar))
    np.savez_compressed(os.path.join(HERE, "model_shaped.npz"), **model_shaped(ar, cr, wl))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
