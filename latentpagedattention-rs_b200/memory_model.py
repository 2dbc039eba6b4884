"""KV-cache memory accounting: bytes per token and per cache for a full GQA
KV cache and for a latent cache, and their ratio.

Restates python_ref/latent_paged_attention/memory_model.py:11-52 (and the
checked-arithmetic Rust mirror, crates/plkv-core/src/lib.rs:52-102): the same
function names, argument meaning and errors (TypeError for non-int arguments,
ValueError for values <= 0).  `estimate` mirrors the reference CLI
(cli.py:21-53) with argparse in place of typer:

    python -m latentpagedattention-rs_b200.memory_model --layers 28 --seq-len 4096 \\
        --batch-size 1 --kv-heads 8 --head-dim 128 --latent-dim 512 --dtype-bytes 2
"""

from __future__ import annotations

import argparse


def _validate_positive_int(name: str, value: int) -> None:
    if not isinstance(value, int) or isinstance(value, bool):
        raise TypeError(f"{name} must be an int, got {type(value).__name__}")
    if value <= 0:
        raise ValueError(f"{name} must be > 0, got {value}")


def kv_bytes_per_token_gqa(n_kv_heads: int, head_dim: int, dtype_bytes: int, *,
                           include_k_and_v: bool = True) -> int:
    """Bytes per token per layer of a GQA KV cache (K and V, or one of them)."""
    _validate_positive_int("n_kv_heads", n_kv_heads)
    _validate_positive_int("head_dim", head_dim)
    _validate_positive_int("dtype_bytes", dtype_bytes)
    return n_kv_heads * head_dim * dtype_bytes * (2 if include_k_and_v else 1)


def kv_bytes_per_token_latent(latent_dim: int, dtype_bytes: int) -> int:
    """Bytes per token per layer of a latent KV cache."""
    _validate_positive_int("latent_dim", latent_dim)
    _validate_positive_int("dtype_bytes", dtype_bytes)
    return latent_dim * dtype_bytes


def compression_ratio(full_kv_bytes: int, latent_kv_bytes: int) -> float:
    """full_kv_bytes / latent_kv_bytes."""
    _validate_positive_int("full_kv_bytes", full_kv_bytes)
    _validate_positive_int("latent_kv_bytes", latent_kv_bytes)
    return full_kv_bytes / latent_kv_bytes


def estimate_total_kv_cache_bytes(num_layers: int, seq_len: int, batch_size: int,
                                  bytes_per_token_per_layer: int) -> int:
    """Total cache bytes over layers, sequence length and batch."""
    _validate_positive_int("num_layers", num_layers)
    _validate_positive_int("seq_len", seq_len)
    _validate_positive_int("batch_size", batch_size)
    _validate_positive_int("bytes_per_token_per_layer", bytes_per_token_per_layer)
    return num_layers * seq_len * batch_size * bytes_per_token_per_layer


def cache_bytes_report(*, tokens: int, kv_heads: int, head_dim: int, latent_dim: int,
                       dtype_bytes: int = 2, num_layers: int = 1) -> dict:
    """Persistent cache bytes of `tokens` cached tokens (summed over the batch)
    for the full-KV and the latent layouts, and their ratio."""
    full = kv_bytes_per_token_gqa(kv_heads, head_dim, dtype_bytes)
    latent = kv_bytes_per_token_latent(latent_dim, dtype_bytes)
    return {"tokens": tokens, "layers": num_layers,
            "full_kv_bytes_per_token": full, "latent_bytes_per_token": latent,
            "full_kv_bytes": estimate_total_kv_cache_bytes(num_layers, tokens, 1, full),
            "latent_bytes": estimate_total_kv_cache_bytes(num_layers, tokens, 1, latent),
            "compression_ratio": compression_ratio(full, latent)}


def _format_mib(num_bytes: int) -> str:
    return f"{num_bytes / (1024 ** 2):.2f} MiB"


def estimate(layers: int, seq_len: int, batch_size: int, kv_heads: int, head_dim: int,
             latent_dim: int, dtype_bytes: int) -> str:
    """The reference CLI's table (cli.py:21-53) as text."""
    gqa = kv_bytes_per_token_gqa(kv_heads, head_dim, dtype_bytes)
    lat = kv_bytes_per_token_latent(latent_dim, dtype_bytes)
    gqa_total = estimate_total_kv_cache_bytes(layers, seq_len, batch_size, gqa)
    lat_total = estimate_total_kv_cache_bytes(layers, seq_len, batch_size, lat)
    rows = [("Variant", "KV bytes/token/layer", "Total KV cache bytes", "Total KV cache MiB"),
            ("GQA KV", str(gqa), str(gqa_total), _format_mib(gqa_total)),
            ("Latent KV", str(lat), str(lat_total), _format_mib(lat_total))]
    widths = [max(len(r[i]) for r in rows) for i in range(4)]
    lines = ["KV Cache Estimate"]
    for r in rows:
        lines.append("  ".join(c.ljust(w) if i == 0 else c.rjust(w)
                               for i, (c, w) in enumerate(zip(r, widths))))
    lines.append("Compression ratio (GQA bytes/token/layer / latent bytes/token/layer): "
                 f"{compression_ratio(gqa, lat):.3f}x")
    return "\n".join(lines)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="Print GQA KV vs latent KV memory estimates.")
    for name in ("layers", "seq-len", "batch-size", "kv-heads", "head-dim", "latent-dim",
                 "dtype-bytes"):
        ap.add_argument(f"--{name}", type=int, required=True)
    a = ap.parse_args(argv)
    print(estimate(a.layers, a.seq_len, a.batch_size, a.kv_heads, a.head_dim, a.latent_dim,
                   a.dtype_bytes))


if __name__ == "__main__":
    main()
