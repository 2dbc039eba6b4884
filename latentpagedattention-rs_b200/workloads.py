"""Seeded synthetic workloads for the paged latent decode path.

Five workloads, in the order of the benchmark definition (seed =
20260710 + index, the reference's seed base of bench_ref.py:102):

  0 tiny          B=2, Hq=4, KV=2, D=16, L=8, bs=4, lens [7, 13]
  1 model_shaped  B=1, Hq=32, KV=8, D=128, L=128, bs=16, 255 prefilled + 1 appended
  2 mla_batch     B=64, Hq=128 absorbed, L=576 (512 value + 64 RoPE), bs=64,
                  lens U[1024, 32768], W_uv [128, 512, 128], W_o [16384, 7168]
  3 write_attend  B=256, Hq=32, KV=8, L=256, D=128, bs=16, lens U[512, 8192],
                  pool 2^18 blocks, 100 append+attend steps, full-KV baseline
  4 long_context  B=8 x 131072 tokens, absorbed MLA shapes, blocks split
                  across GPUs

Distributions: latent cache N(0, 1) (N(0, 0.5) for the MLA shapes) rounded to
FP16; query / absorbed query N(0, 1); W_k N(0, 1/sqrt(head_dim)); W_v / W_uv
N(0, 1/sqrt(value_dim)); W_o N(0, 1/sqrt(q_heads*head_dim)).  Block tables
are drawn from a random permutation of the physical pool.  Small workloads
are generated on the host with NumPy (bit-reproducible); the large ones on the
device with a seeded torch generator.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

SEED_BASE = 20260710


@dataclass(frozen=True)
class WorkloadSpec:
    name: str
    index: int
    batch: int
    q_heads: int
    kv_heads: int          # heads of W_k (GQA); equals q_heads for absorbed MLA
    head_dim: int
    latent_dim: int
    value_dim: int
    block_size: int
    absorbed: bool         # the query arrives already projected (q_lat)
    proj_heads: int        # heads of W_v / W_uv
    out_dim: int           # W_o width (0: none)
    cache_std: float
    lens: tuple = field(default=())          # fixed active lengths, or ()
    len_range: tuple = field(default=())     # (lo, hi) inclusive, drawn per sequence
    pool_blocks: int = 0                     # 0: exactly what the tables need
    steps: int = 1                           # append+attend steps of the workload
    appended: bool = True                    # one row appended before the read

    @property
    def seed(self) -> int:
        return SEED_BASE + self.index

    @property
    def group(self) -> int:
        return self.q_heads // self.proj_heads

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(float(self.head_dim))


WORKLOADS = {
    "tiny": WorkloadSpec("tiny", 0, 2, 4, 2, 16, 8, 8, 4, False, 2, 64, 1.0, lens=(7, 13),
                         appended=False),
    "model_shaped": WorkloadSpec("model_shaped", 1, 1, 32, 8, 128, 128, 128, 16, False, 8, 4096,
                                 1.0, lens=(256,)),
    "mla_batch": WorkloadSpec("mla_batch", 2, 64, 128, 128, 128, 576, 512, 64, True, 128, 7168,
                              0.5, len_range=(1024, 32768)),
    "write_attend": WorkloadSpec("write_attend", 3, 256, 32, 8, 128, 256, 256, 16, False, 8, 0,
                                 1.0, len_range=(512, 8192), pool_blocks=1 << 18, steps=100),
    "long_context": WorkloadSpec("long_context", 4, 8, 128, 128, 128, 576, 512, 64, True, 128, 0,
                                 0.5, lens=(131072,) * 8),
}


def spec(name: str) -> WorkloadSpec:
    return WORKLOADS[name]


def initial_lens(s: WorkloadSpec) -> np.ndarray:
    """Active lengths at the first decode read (after its appended row)."""
    if s.lens:
        return np.asarray(s.lens, dtype=np.int32)
    rng = np.random.default_rng(s.seed)
    lo, hi = s.len_range
    return rng.integers(lo, hi + 1, size=s.batch, dtype=np.int64).astype(np.int32)


def build_tables(s: WorkloadSpec, lens: np.ndarray, *, shards: int = 1,
                 shard: int = 0) -> tuple[np.ndarray, int, np.ndarray]:
    """Block tables drawn from a random permutation of the physical pool.

    Every sequence gets blocks for ``lens + steps - 1`` tokens (room for the
    appends of the whole run).  With ``shards > 1`` each sequence's logical
    blocks are cut into ``shards`` contiguous ranges and the table of shard
    ``shard`` covers only its range (split-K across GPUs): returns that
    shard's tables, pool size and per-sequence first logical block.
    """
    rng = np.random.default_rng(s.seed + 7919 * (shard + 1) if shards > 1 else s.seed + 1)
    cap = lens.astype(np.int64) + (s.steps - 1)
    nblocks = (cap + s.block_size - 1) // s.block_size
    first = (nblocks * shard) // shards
    last = (nblocks * (shard + 1)) // shards
    counts = last - first
    need = int(counts.sum())
    pool = max(need, s.pool_blocks // shards if s.pool_blocks else 0, 1)
    perm = rng.permutation(pool)[:need].astype(np.int32)
    max_blocks = max(int(counts.max()), 1)
    tables = np.full((s.batch, max_blocks), -1, dtype=np.int32)
    k = 0
    for b in range(s.batch):
        tables[b, :counts[b]] = perm[k:k + counts[b]]
        k += counts[b]
    return tables, pool, first.astype(np.int64)


def host_inputs(s: WorkloadSpec) -> dict:
    """All inputs of a small workload as NumPy arrays (bit-reproducible)."""
    rng = np.random.default_rng(s.seed + 2)
    lens = initial_lens(s)
    tables, pool, _ = build_tables(s, lens)
    L, Lv, D, Hq = s.latent_dim, s.value_dim, s.head_dim, s.q_heads
    cache_src = (rng.standard_normal((pool, s.block_size, L), dtype=np.float32)
                 * np.float32(s.cache_std))
    out = {"lens": lens, "tables": tables, "pool": pool,
           "cache_f16": cache_src.astype(np.float16)}
    if s.absorbed:
        out["q_lat"] = rng.standard_normal((s.batch, Hq, L), dtype=np.float32)
    else:
        out["q"] = rng.standard_normal((s.batch, Hq, D), dtype=np.float32)
        out["w_k"] = (rng.standard_normal((L, s.kv_heads * D), dtype=np.float32)
                      * np.float32(1.0 / math.sqrt(D)))
    out["w_v"] = (rng.standard_normal((Lv, s.proj_heads * D), dtype=np.float32)
                  * np.float32(1.0 / math.sqrt(Lv)))
    if s.out_dim:
        out["w_o"] = (rng.standard_normal((Hq * D, s.out_dim), dtype=np.float32)
                      * np.float32(1.0 / math.sqrt(Hq * D)))
    out["new_rows"] = (rng.standard_normal((s.steps, s.batch, L), dtype=np.float32)
                       * np.float32(s.cache_std))
    return out


def head_major(w_canonical: np.ndarray, heads: int, head_dim: int) -> np.ndarray:
    """[rows, heads*head_dim] -> [heads, rows, head_dim] (fixtures.py:418-432 layout)."""
    r = w_canonical.shape[0]
    return np.ascontiguousarray(w_canonical.reshape(r, heads, head_dim).transpose(1, 0, 2))


def device_inputs(s: WorkloadSpec, device, *, shards: int = 1, shard: int = 0,
                  with_out_proj: bool = True, with_fullkv: bool = False,
                  extra_blocks: int = 0) -> dict:
    """Inputs of any workload generated on a CUDA device (torch generator).

    With ``shards > 1`` the cache holds only shard ``shard``'s blocks of every
    sequence; ``lens`` are then the shard-local lengths and ``global_lens``
    the full ones.  The query and the weights are identical on every shard.
    ``extra_blocks`` free blocks follow the ``pool`` blocks the tables draw
    from (ids pool .. pool + extra_blocks - 1), for a loop that allocates.
    """
    import torch

    dev = torch.device(device)
    lens = initial_lens(s)
    tables, pool, first_block = build_tables(s, lens, shards=shards, shard=shard)
    L, Lv, D, Hq = s.latent_dim, s.value_dim, s.head_dim, s.q_heads
    g = torch.Generator(device=dev)
    g.manual_seed(s.seed * 1000 + 17 * shard + 3)
    total = pool + int(extra_blocks)
    cache = torch.empty((total, s.block_size, L), dtype=torch.float16, device=dev)
    chunk = max(1, (1 << 26) // (s.block_size * L))
    for i in range(0, total, chunk):
        j = min(total, i + chunk)
        cache[i:j] = (torch.randn((j - i, s.block_size, L), generator=g, device=dev)
                      * s.cache_std).half()
    gw = torch.Generator(device=dev)
    gw.manual_seed(s.seed * 1000 + 999)  # shared by all shards
    out = {"tables": torch.as_tensor(tables, device=dev), "pool": pool, "cache": cache,
           "global_lens": lens}
    if s.absorbed:
        out["q_lat"] = torch.randn((s.batch, Hq, L), generator=gw, device=dev)
    else:
        out["q"] = torch.randn((s.batch, Hq, D), generator=gw, device=dev)
        out["w_k"] = torch.randn((s.kv_heads, L, D), generator=gw, device=dev) / math.sqrt(D)
    out["w_v"] = torch.randn((s.proj_heads, Lv, D), generator=gw, device=dev) / math.sqrt(Lv)
    if s.out_dim and with_out_proj:
        out["w_o"] = torch.randn((Hq * D, s.out_dim), generator=gw, device=dev) / math.sqrt(Hq * D)
    out["new_rows"] = torch.randn((s.batch, L), generator=gw, device=dev) * s.cache_std
    if shards > 1:
        from .multigpu import split_k_ranges

        _, _, local = split_k_ranges(lens, s.block_size, shards, shard, s.steps - 1)
        out["lens"] = local
        out["token_offset"] = first_block * s.block_size
    else:
        out["lens"] = lens.copy()
        out["token_offset"] = np.zeros(s.batch, dtype=np.int64)
    if with_fullkv:
        out.update(fullkv_from_latent(s, out, dev))
    return out


def fullkv_from_latent(s: WorkloadSpec, inputs: dict, device) -> dict:
    """Full-KV baseline caches K = fp16(L W_k), V = fp16(L W_v) for the blocks
    the tables use (as fp16_full_kv_baseline_gpu.rs:483-507 derives them),
    head-major [P, KV, bs, D]."""
    import torch

    cache = inputs["cache"]
    tables = inputs["tables"]
    P, bs, L = cache.shape
    KV, D = s.kv_heads, s.head_dim
    wk = inputs["w_k"].permute(1, 0, 2).reshape(L, KV * D)       # canonical [L, KV*D]
    wv = inputs["w_v"].permute(1, 0, 2).reshape(s.value_dim, KV * D)
    k = torch.zeros((P, KV, bs, D), dtype=torch.float16, device=device)
    v = torch.zeros((P, KV, bs, D), dtype=torch.float16, device=device)
    used = torch.unique(tables[tables >= 0])
    for i in range(0, used.numel(), 4096):
        blk = used[i:i + 4096]
        rows = cache[blk].float()                                  # [n, bs, L]
        kk = (rows @ wk).reshape(-1, bs, KV, D).permute(0, 2, 1, 3)
        vv = (rows[..., :s.value_dim] @ wv).reshape(-1, bs, KV, D).permute(0, 2, 1, 3)
        k[blk] = kk.half()
        v[blk] = vv.half()
    return {"k_cache": k, "v_cache": v}


def algorithmic_bytes(s: WorkloadSpec, lens: np.ndarray, *, with_out_proj: bool,
                      fullkv: bool = False, n_items: int = 0) -> int:
    """Bytes a decode step must move at minimum: latent rows attended (FP16),
    weights read once as stored (FP32), query, output, appended rows (FP32 in,
    FP16 out) and the block-table entries walked."""
    B, Hq, D, L = s.batch, s.q_heads, s.head_dim, s.latent_dim
    toks = int(np.sum(lens, dtype=np.int64))
    if fullkv:
        cache = toks * s.kv_heads * D * 2 * 2
        weights = 0
        q_bytes = B * Hq * D * 4
        append = B * s.kv_heads * D * (4 + 2) * 2
    else:
        cache = toks * L * 2
        weights = s.proj_heads * s.value_dim * D * 4
        if not s.absorbed:
            weights += s.kv_heads * L * D * 4
        q_bytes = B * Hq * (L if s.absorbed else D) * 4
        append = B * L * (4 + 2)
    if with_out_proj and s.out_dim:
        weights += Hq * D * s.out_dim * 4
        out_bytes = B * s.out_dim * 4
    else:
        out_bytes = B * Hq * D * 4
    tables = int(np.sum((lens.astype(np.int64) + s.block_size - 1) // s.block_size)) * 4
    return cache + weights + q_bytes + out_bytes + append + tables


def algorithmic_flops(s: WorkloadSpec, lens: np.ndarray, *, with_out_proj: bool) -> int:
    toks = int(np.sum(lens, dtype=np.int64))
    f = toks * s.q_heads * 2 * (s.latent_dim + s.value_dim)
    f += s.batch * s.q_heads * s.value_dim * s.head_dim * 2
    if not s.absorbed:
        f += s.batch * s.q_heads * s.latent_dim * s.head_dim * 2
    if with_out_proj and s.out_dim:
        f += s.batch * s.q_heads * s.head_dim * s.out_dim * 2
    return f
