"""NumPy restatement of the reference's Python oracle for the hot path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Each function restates one function of tatavishnurao/LatentPagedAttention-rs
``python_ref/latent_paged_attention`` with the same arguments, results and
exceptions; the cited lines are the ones it follows.  The per-sequence batch
helpers at the end are extensions (the reference shares one block table
across the batch) built as loops over the restated single-table functions.
"""

from __future__ import annotations

import numpy as np

MASKED_SCORE = np.float32(-3.4028234663852886e38)


# --------------------------------------------------------------- cache_ref.py

def fp16_storage_roundtrip_f32(values: np.ndarray) -> np.ndarray:
    """cache_ref.py:6-14 -- FP32 -> FP16 (round to nearest even) -> FP32."""
    values = np.asarray(values)
    if not np.isfinite(values).all():
        raise ValueError("FP16 storage input must be finite")
    with np.errstate(over="ignore"):
        stored = values.astype(np.float16)
    if not np.isfinite(stored).all():
        raise ValueError("FP16 storage conversion overflowed")
    return stored.astype(np.float32)


def fp16_storage_bits(values: np.ndarray) -> np.ndarray:
    """cache_ref.py:17-19 -- IEEE FP16 storage bit patterns as uint16."""
    return fp16_storage_roundtrip_f32(values).astype(np.float16).view(np.uint16)


def resolve_paged_token_location(block_table: np.ndarray, token_position: int,
                                 block_size: int) -> tuple[int, int, int]:
    """cache_ref.py:22-40 -- (logical block, physical block, in-block offset)."""
    block_table = np.asarray(block_table)
    if block_table.ndim != 1:
        raise ValueError("block_table must be 1D")
    if block_size <= 0:
        raise ValueError(f"block_size must be > 0, got {block_size}")
    if token_position < 0:
        raise ValueError(f"token_position must be >= 0, got {token_position}")
    logical = token_position // block_size
    if logical >= block_table.size:
        raise IndexError("block_table does not cover token_position")
    physical = int(block_table[logical])
    if physical < 0:
        raise ValueError("block_table contains a negative physical block")
    return logical, physical, token_position % block_size


def paged_latent_write_ref(latent_cache: np.ndarray, block_table: np.ndarray,
                           token_position: int, new_latent: np.ndarray) -> np.ndarray:
    """cache_ref.py:76-100 -- write one latent row into a copy of the cache."""
    if latent_cache.ndim != 3:
        raise ValueError("latent_cache must have shape [blocks, block_size, latent_dim]")
    if np.asarray(block_table).ndim != 1:
        raise ValueError("block_table must be 1D")
    if new_latent.ndim != 1:
        raise ValueError("new_latent must be 1D")
    if new_latent.shape[0] != latent_cache.shape[2]:
        raise ValueError("new_latent width must match latent_dim")
    if not np.isfinite(latent_cache).all() or not np.isfinite(new_latent).all():
        raise ValueError("latent cache and replacement must be finite")
    _, physical, offset = resolve_paged_token_location(block_table, token_position,
                                                       latent_cache.shape[1])
    if physical >= latent_cache.shape[0]:
        raise IndexError("block_table contains an out-of-range physical block")
    updated = np.array(latent_cache, copy=True)
    updated[physical, offset, :] = new_latent
    return updated


def paged_latent_write_fp16_storage_ref(latent_cache_f32: np.ndarray, block_table: np.ndarray,
                                        token_position: int,
                                        new_latent_f32: np.ndarray) -> np.ndarray:
    """cache_ref.py:103-114 -- FP16-stored latent write, returned as FP32."""
    return paged_latent_write_ref(fp16_storage_roundtrip_f32(latent_cache_f32), block_table,
                                  token_position, fp16_storage_roundtrip_f32(new_latent_f32))


def paged_kv_write_ref(k_cache: np.ndarray, v_cache: np.ndarray, block_table: np.ndarray,
                       token_position: int, new_k: np.ndarray,
                       new_v: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """cache_ref.py:43-73 -- write one K/V row into copies of the caches."""
    if k_cache.ndim != 3 or v_cache.ndim != 3:
        raise ValueError("K and V caches must have shape [blocks, block_size, width]")
    if k_cache.shape != v_cache.shape:
        raise ValueError("K and V cache shapes must match")
    if np.asarray(block_table).ndim != 1:
        raise ValueError("block_table must be 1D")
    if new_k.ndim != 1 or new_v.ndim != 1:
        raise ValueError("new_k and new_v must be 1D")
    if new_k.shape != new_v.shape or new_k.shape[0] != k_cache.shape[2]:
        raise ValueError("new K/V vectors must have the cache width")
    _, physical, offset = resolve_paged_token_location(block_table, token_position,
                                                       k_cache.shape[1])
    if physical >= k_cache.shape[0]:
        raise IndexError("block_table contains an out-of-range physical block")
    k_out = np.array(k_cache, copy=True)
    v_out = np.array(v_cache, copy=True)
    k_out[physical, offset, :] = new_k
    v_out[physical, offset, :] = new_v
    return k_out, v_out


# ------------------------------------------------- materialised reconstruction

def latent_kv_reconstruction_ref(latent_cache: np.ndarray, k_proj: np.ndarray,
                                 v_proj: np.ndarray, *, kv_heads: int,
                                 head_dim: int) -> tuple[np.ndarray, np.ndarray]:
    """attention_ref.py:227-274 -- K, V [batch, seq, kv_heads, head_dim] from a
    latent cache [batch, seq, latent] and projections [latent, kv_heads*head_dim]."""
    if latent_cache.ndim != 3:
        raise ValueError("latent_cache must have shape [batch, seq_len, latent_dim]")
    if k_proj.ndim != 2 or v_proj.ndim != 2:
        raise ValueError("k_proj and v_proj must have shape [latent_dim, kv_heads * head_dim]")
    if k_proj.shape != v_proj.shape:
        raise ValueError("k_proj and v_proj shapes must match")
    if kv_heads <= 0:
        raise ValueError(f"kv_heads must be > 0, got {kv_heads}")
    if head_dim <= 0:
        raise ValueError(f"head_dim must be > 0, got {head_dim}")
    batch, seq_len, latent_dim = latent_cache.shape
    if batch <= 0 or seq_len <= 0 or latent_dim <= 0:
        raise ValueError("latent_cache dimensions must be > 0")
    if k_proj.shape[0] != latent_dim:
        raise ValueError("latent_dim mismatch between cache and projections")
    if k_proj.shape[1] != kv_heads * head_dim:
        raise ValueError("projection width must equal kv_heads * head_dim")
    k = np.asarray(latent_cache @ k_proj, dtype=np.float32).reshape(batch, seq_len, kv_heads,
                                                                      head_dim)
    v = np.asarray(latent_cache @ v_proj, dtype=np.float32).reshape(batch, seq_len, kv_heads,
                                                                      head_dim)
    if not np.all(np.isfinite(k)):
        raise ValueError("reconstructed K cache must be finite")
    if not np.all(np.isfinite(v)):
        raise ValueError("reconstructed V cache must be finite")
    return k, v


# ------------------------------------------------------------ block_table.py

class PagedBlockTable:
    """block_table.py:14-61 -- bump allocator of logical -> physical blocks."""

    def __init__(self, block_size: int) -> None:
        if not isinstance(block_size, int):
            raise TypeError(f"block_size must be an int, got {type(block_size).__name__}")
        if block_size <= 0:
            raise ValueError(f"block_size must be > 0, got {block_size}")
        self.block_size = block_size
        self.logical_to_physical: list[int] = []
        self.next_physical_block = 0
        self.num_tokens = 0

    def allocate_token_positions(self, num_tokens: int) -> list[tuple[int, int, int]]:
        if not isinstance(num_tokens, int):
            raise TypeError(f"num_tokens must be an int, got {type(num_tokens).__name__}")
        if num_tokens <= 0:
            raise ValueError(f"num_tokens must be > 0, got {num_tokens}")
        out = []
        for _ in range(num_tokens):
            pos = self.num_tokens
            if pos // self.block_size == len(self.logical_to_physical):
                self.logical_to_physical.append(self.next_physical_block)
                self.next_physical_block += 1
            self.num_tokens += 1
            out.append((pos, *self.translate(pos)))
        return out

    def translate(self, token_pos: int) -> tuple[int, int]:
        if not isinstance(token_pos, int):
            raise TypeError(f"token_pos must be an int, got {type(token_pos).__name__}")
        if token_pos < 0:
            raise ValueError(f"token_pos must be >= 0, got {token_pos}")
        if token_pos >= self.num_tokens:
            raise IndexError(f"token_pos {token_pos} is out of range for "
                             f"{self.num_tokens} allocated tokens")
        return self.logical_to_physical[token_pos // self.block_size], token_pos % self.block_size

    def to_list(self) -> list[int]:
        return list(self.logical_to_physical)


# --------------------------------------------------------- attention_ref.py

def softmax_stable(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """attention_ref.py:6-10."""
    e = np.exp(x - np.max(x, axis=axis, keepdims=True))
    return e / np.sum(e, axis=axis, keepdims=True)


def _check_group(q_heads: int, kv_heads: int, group_size: int) -> None:
    """attention_ref.py:13-20."""
    if group_size <= 0:
        raise ValueError(f"group_size must be > 0, got {group_size}")
    if q_heads != kv_heads * group_size:
        raise ValueError("expected q_heads == kv_heads * group_size, "
                         f"got q_heads={q_heads}, kv_heads={kv_heads}, group_size={group_size}")


def paged_lookup_ref(cache_blocks: np.ndarray, block_table: np.ndarray, seq_len: int,
                     block_size: int) -> np.ndarray:
    """attention_ref.py:23-63 -- token-major gather through the block table."""
    if cache_blocks.ndim < 3:
        raise ValueError("cache_blocks must have shape [num_blocks, block_size, ...] with ndim >= 3")
    if block_table.ndim != 1:
        raise ValueError("block_table must be 1D")
    if block_size <= 0:
        raise ValueError(f"block_size must be > 0, got {block_size}")
    if seq_len <= 0:
        raise ValueError(f"seq_len must be > 0, got {seq_len}")
    if cache_blocks.shape[1] != block_size:
        raise ValueError(f"block_size mismatch: cache has {cache_blocks.shape[1]}, "
                         f"argument was {block_size}")
    if block_table.size == 0:
        raise ValueError("block_table must not be empty")
    if np.any(block_table < 0) or np.any(block_table >= cache_blocks.shape[0]):
        raise ValueError("block_table contains out-of-range physical block indices")
    if block_table.size * block_size < seq_len:
        raise ValueError("block_table does not cover the requested seq_len")
    return cache_blocks[block_table].reshape(-1, *cache_blocks.shape[2:])[:seq_len]


def gqa_decode_attention_intermediates_ref(q, k_cache, v_cache, *, group_size):
    """attention_ref.py:90-141 -- dense GQA decode with intermediates."""
    if q.ndim != 3 or k_cache.ndim != 4 or v_cache.ndim != 4:
        raise ValueError("expected q [batch, q_heads, head_dim], "
                         "k_cache/v_cache [batch, seq_len, kv_heads, head_dim]")
    if k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache must share the same shape")
    if q.shape[0] != k_cache.shape[0]:
        raise ValueError("batch size mismatch between q and cache tensors")
    if q.shape[2] != k_cache.shape[3]:
        raise ValueError("head_dim mismatch between q and cache tensors")
    q_heads, head_dim = q.shape[1], q.shape[2]
    _check_group(q_heads, k_cache.shape[2], group_size)
    kv_of = np.arange(q_heads) // group_size
    k_sel = k_cache[:, :, kv_of, :]
    v_sel = v_cache[:, :, kv_of, :]
    scores = np.einsum("bqh,btqh->bqt", q, k_sel) / np.sqrt(float(head_dim))
    probs = softmax_stable(scores, axis=-1)
    context = np.einsum("bqt,btqh->bqh", probs, v_sel)
    if not np.all(np.isfinite(scores)):
        raise ValueError("scores must be finite")
    if not np.all(np.isfinite(probs)):
        raise ValueError("probabilities must be finite")
    if not np.allclose(np.sum(probs, axis=-1), 1.0, atol=1e-6):
        raise ValueError("probability rows must sum to one")
    return scores, probs, context


def paged_gqa_decode_attention_intermediates_ref(q, k_blocks, v_blocks, block_table, seq_len,
                                                 block_size, *, group_size):
    """attention_ref.py:172-224 -- paged full-KV GQA (token-major blocks)."""
    if q.ndim != 3:
        raise ValueError("q must have shape [batch, q_heads, head_dim]")
    if k_blocks.ndim != 4 or v_blocks.ndim != 4:
        raise ValueError("k_blocks and v_blocks must have shape "
                         "[num_physical_blocks, block_size, kv_heads, head_dim]")
    if k_blocks.shape != v_blocks.shape:
        raise ValueError("k_blocks and v_blocks must share the same shape")
    if block_table.ndim != 1:
        raise ValueError("block_table must be 1D")
    if seq_len <= 0:
        raise ValueError(f"seq_len must be > 0, got {seq_len}")
    if block_size <= 0:
        raise ValueError(f"block_size must be > 0, got {block_size}")
    if k_blocks.shape[1] != block_size:
        raise ValueError(f"block_size mismatch: cache has {k_blocks.shape[1]}, "
                         f"argument was {block_size}")
    if q.shape[2] != k_blocks.shape[3]:
        raise ValueError("head_dim mismatch between q and paged cache tensors")
    if block_table.size * block_size < seq_len:
        raise ValueError("block_table does not cover the requested seq_len")
    k = paged_lookup_ref(k_blocks, block_table, seq_len, block_size)
    v = paged_lookup_ref(v_blocks, block_table, seq_len, block_size)
    batch = q.shape[0]
    return gqa_decode_attention_intermediates_ref(
        q, np.broadcast_to(k[None], (batch, *k.shape)),
        np.broadcast_to(v[None], (batch, *v.shape)), group_size=group_size)


def direct_paged_latent_gqa_decode_attention_intermediates_ref(
        q, latent_blocks, block_table, seq_len, block_size, k_proj, v_proj, *,
        q_heads, kv_heads, head_dim, group_size):
    """attention_ref.py:478-535 -- direct latent-space decode through the table."""
    if q.ndim != 3 or q.shape[0] <= 0 or q.shape[1:] != (q_heads, head_dim):
        raise ValueError("q must have shape [batch, q_heads, head_dim]")
    if latent_blocks.ndim != 3 or latent_blocks.shape[1] != block_size:
        raise ValueError("latent_blocks must have shape [physical_blocks, block_size, latent_dim]")
    if block_table.ndim != 1 or block_table.size * block_size < seq_len:
        raise ValueError("block_table must cover seq_len and be 1D")
    if seq_len <= 0 or block_size <= 0 or kv_heads <= 0 or head_dim <= 0:
        raise ValueError("dimensions must be positive")
    _check_group(q_heads, kv_heads, group_size)
    if k_proj.ndim != 2 or v_proj.shape != k_proj.shape:
        raise ValueError("K/V projections must share a 2D shape")
    latent_dim = latent_blocks.shape[2]
    if k_proj.shape != (latent_dim, kv_heads * head_dim):
        raise ValueError("projection shape does not match latent dimensions")
    if np.any(block_table < 0) or np.any(block_table >= latent_blocks.shape[0]):
        raise ValueError("block_table contains out-of-range physical block indices")
    if not all(np.isfinite(x).all() for x in (q, latent_blocks, k_proj, v_proj)):
        raise ValueError("inputs must be finite")
    batch = q.shape[0]
    scores = np.empty((batch, q_heads, seq_len), dtype=np.float32)
    probs = np.empty_like(scores)
    context = np.empty((batch, q_heads, head_dim), dtype=np.float32)
    wk = k_proj.reshape(latent_dim, kv_heads, head_dim)
    wv = v_proj.reshape(latent_dim, kv_heads, head_dim)
    scale = np.float32(1.0 / np.sqrt(float(head_dim)))
    nblocks = (seq_len + block_size - 1) // block_size
    for b in range(batch):
        for h in range(q_heads):
            kv = h // group_size
            projected = wk[:, kv, :] @ q[b, h]
            for lb in range(nblocks):
                phys = int(block_table[lb])
                lo, hi = lb * block_size, min((lb + 1) * block_size, seq_len)
                scores[b, h, lo:hi] = latent_blocks[phys, : hi - lo] @ projected * scale
            probs[b, h] = softmax_stable(scores[b, h])
            lat_ctx = np.zeros(latent_dim, dtype=np.float32)
            for lb in range(nblocks):
                phys = int(block_table[lb])
                lo, hi = lb * block_size, min((lb + 1) * block_size, seq_len)
                lat_ctx += probs[b, h, lo:hi] @ latent_blocks[phys, : hi - lo]
            context[b, h] = lat_ctx @ wv[:, kv, :]
    if not all(np.isfinite(x).all() for x in (scores, probs, context)):
        raise ValueError("outputs must be finite")
    if not np.allclose(probs.sum(axis=-1), 1.0, atol=1e-6):
        raise ValueError("probability rows must sum to one")
    return scores, probs, context


def direct_paged_latent_gqa_fp16_storage_intermediates_ref(
        q, latent_blocks_f32, block_table, seq_len, block_size, k_proj, v_proj, *,
        q_heads, kv_heads, head_dim, group_size):
    """attention_ref.py:538-568 -- as above on FP16-rounded storage."""
    return direct_paged_latent_gqa_decode_attention_intermediates_ref(
        q, fp16_storage_roundtrip_f32(latent_blocks_f32), block_table, seq_len, block_size,
        k_proj, v_proj, q_heads=q_heads, kv_heads=kv_heads, head_dim=head_dim,
        group_size=group_size)


def direct_paged_latent_gqa_decode_attention_runtime_intermediates_ref(
        q, latent_blocks, block_table, max_seq_len, active_seq_len, block_size, k_proj, v_proj,
        *, q_heads, kv_heads, head_dim, group_size):
    """attention_ref.py:571-614 -- runtime active length, padded intermediates."""
    if active_seq_len <= 0 or active_seq_len > max_seq_len:
        raise ValueError("active_seq_len must satisfy 1 <= active_seq_len <= max_seq_len")
    scores, probs, context = direct_paged_latent_gqa_decode_attention_intermediates_ref(
        q, latent_blocks, block_table, active_seq_len, block_size, k_proj, v_proj,
        q_heads=q_heads, kv_heads=kv_heads, head_dim=head_dim, group_size=group_size)
    if max_seq_len == active_seq_len:
        return scores, probs, context
    padded_scores = np.full((q.shape[0], q_heads, max_seq_len), MASKED_SCORE)
    padded_probs = np.zeros((q.shape[0], q_heads, max_seq_len), dtype=np.float32)
    padded_scores[:, :, :active_seq_len] = scores
    padded_probs[:, :, :active_seq_len] = probs
    if not np.all(padded_probs[:, :, active_seq_len:] == 0.0):
        raise ValueError("inactive probabilities must be zero")
    if not np.allclose(padded_probs.sum(axis=-1), 1.0, atol=1e-6):
        raise ValueError("active probability rows must sum to one")
    return padded_scores, padded_probs, context


def direct_paged_latent_gqa_fp16_storage_runtime_intermediates_ref(
        q, latent_blocks_f32, block_table, max_seq_len, active_seq_len, block_size, k_proj,
        v_proj, *, q_heads, kv_heads, head_dim, group_size):
    """attention_ref.py:617-648 -- runtime active length on FP16 storage."""
    return direct_paged_latent_gqa_decode_attention_runtime_intermediates_ref(
        q, fp16_storage_roundtrip_f32(latent_blocks_f32), block_table, max_seq_len,
        active_seq_len, block_size, k_proj, v_proj, q_heads=q_heads, kv_heads=kv_heads,
        head_dim=head_dim, group_size=group_size)


# ---------------------------------------------------- batch extensions (f64)

def latent_decode_batch_f64(q_lat, cache_f16, tables, lens, block_size, value_dim, scale,
                            w_v_head_major=None, group=1):
    """Per-sequence-table direct latent decode in float64.

    Extension of attention_ref.py:510-530 to one block table and one active
    length per sequence and to an absorbed query ``q_lat [B, Hq, L]``;
    ``w_v_head_major`` is ``[proj_heads, value_dim, head_dim]`` with query
    head ``h`` using projection head ``h // group``.  Returns
    ``(scores list, probs list, ctx_lat [B,Hq,Lv], ctx [B,Hq,D] or None)``.
    """
    cache = np.asarray(cache_f16).astype(np.float64)
    q_lat = np.asarray(q_lat, dtype=np.float64)
    batch, q_heads, _ = q_lat.shape
    scores, probs = [], []
    ctx_lat = np.zeros((batch, q_heads, value_dim))
    for b in range(batch):
        n = int(lens[b])
        nblocks = (n + block_size - 1) // block_size
        rows = cache[np.asarray(tables[b][:nblocks], dtype=np.int64)].reshape(-1, cache.shape[2])[:n]
        s = (q_lat[b] @ rows.T) * scale
        p = np.exp(s - s.max(axis=1, keepdims=True))
        p /= p.sum(axis=1, keepdims=True)
        scores.append(s)
        probs.append(p)
        ctx_lat[b] = p @ rows[:, :value_dim]
    ctx = None
    if w_v_head_major is not None:
        w = np.asarray(w_v_head_major, dtype=np.float64)
        heads = np.arange(q_heads) // group
        ctx = np.einsum("bhl,hld->bhd", ctx_lat, w[heads])
    return scores, probs, ctx_lat, ctx


def fullkv_decode_batch_f64(q, k_f16, v_f16, tables, lens, block_size, scale, group):
    """Per-sequence-table FP16 full-KV paged GQA decode in float64.

    Extension of lib.rs:1147-1269 (head-major ``[P, KV, bs, D]`` storage) to
    a table and an active length per sequence.
    """
    k = np.asarray(k_f16).astype(np.float64)
    v = np.asarray(v_f16).astype(np.float64)
    q = np.asarray(q, dtype=np.float64)
    batch, q_heads, head_dim = q.shape
    ctx = np.zeros((batch, q_heads, head_dim))
    scores, probs = [], []
    for b in range(batch):
        n = int(lens[b])
        nblocks = (n + block_size - 1) // block_size
        tb = np.asarray(tables[b][:nblocks], dtype=np.int64)
        kr = k[tb].transpose(1, 0, 2, 3).reshape(k.shape[1], -1, head_dim)[:, :n]
        vr = v[tb].transpose(1, 0, 2, 3).reshape(v.shape[1], -1, head_dim)[:, :n]
        kh = kr[np.arange(q_heads) // group]
        vh = vr[np.arange(q_heads) // group]
        s = np.einsum("hd,htd->ht", q[b], kh) * scale
        p = np.exp(s - s.max(axis=1, keepdims=True))
        p /= p.sum(axis=1, keepdims=True)
        scores.append(s)
        probs.append(p)
        ctx[b] = np.einsum("ht,htd->hd", p, vh)
    return scores, probs, ctx


# ------------------------------------------------- materialised reconstruction

def latent_kv_reconstruction_ref(latent_cache: np.ndarray, k_proj: np.ndarray,
                                 v_proj: np.ndarray, *, kv_heads: int,
                                 head_dim: int) -> tuple[np.ndarray, np.ndarray]:
    """attention_ref.py:227-274 -- K, V [batch, seq, kv_heads, head_dim] from a
    latent cache [batch, seq, latent] and projections [latent, kv_heads*head_dim]."""
    if latent_cache.ndim != 3:
        raise ValueError("latent_cache must have shape [batch, seq_len, latent_dim]")
    if k_proj.ndim != 2 or v_proj.ndim != 2:
        raise ValueError("k_proj and v_proj must have shape [latent_dim, kv_heads * head_dim]")
    if k_proj.shape != v_proj.shape:
        raise ValueError("k_proj and v_proj shapes must match")
    if kv_heads <= 0:
        raise ValueError(f"kv_heads must be > 0, got {kv_heads}")
    if head_dim <= 0:
        raise ValueError(f"head_dim must be > 0, got {head_dim}")
    batch, seq_len, latent_dim = latent_cache.shape
    if batch <= 0 or seq_len <= 0 or latent_dim <= 0:
        raise ValueError("latent_cache dimensions must be > 0")
    if k_proj.shape[0] != latent_dim:
        raise ValueError("latent_dim mismatch between cache and projections")
    if k_proj.shape[1] != kv_heads * head_dim:
        raise ValueError("projection width must equal kv_heads * head_dim")
    k = np.asarray(latent_cache @ k_proj, dtype=np.float32).reshape(batch, seq_len, kv_heads,
                                                                      head_dim)
    v = np.asarray(latent_cache @ v_proj, dtype=np.float32).reshape(batch, seq_len, kv_heads,
                                                                      head_dim)
    if not np.all(np.isfinite(k)):
        raise ValueError("reconstructed K cache must be finite")
    if not np.all(np.isfinite(v)):
        raise ValueError("reconstructed V cache must be finite")
    return k, v


# ------------------------------------------------------------ block_table.py

def allocate_token_positions_batch(tables: np.ndarray, lens: np.ndarray, counts: np.ndarray,
                                   next_block: int, block_size: int, num_physical: int):
    """Batched form of PagedBlockTable.allocate_token_positions
    (block_table.py:26-38): sequences in batch order, each taking ``counts[b]``
    new positions; a logical block without a physical block (entry < 0) takes
    the pool's next block id (one counter shared by the batch, where the
    reference keeps one per table).  Ids at or past ``num_physical`` are not
    stored (pool exhausted) and positions that land in no valid block get slot
    -1.  Returns (tables, lens, slots, next_block); slot = physical * bs + offset.
    """
    tables = np.array(tables, dtype=np.int32, copy=True)
    lens = np.array(lens, dtype=np.int32, copy=True)
    max_blocks = tables.shape[1]
    slots = []
    nb = int(next_block)
    for b in range(lens.size):
        c = int(counts[b])
        if c <= 0:
            continue
        first, last = int(lens[b]) // block_size, (int(lens[b]) + c - 1) // block_size
        for lb in range(first, last + 1):
            if lb < max_blocks and tables[b, lb] < 0:
                if nb < num_physical:
                    tables[b, lb] = nb
                nb += 1
        for i in range(c):
            pos = int(lens[b]) + i
            lb = pos // block_size
            phys = int(tables[b, lb]) if lb < max_blocks else -1
            ok = 0 <= phys < num_physical
            slots.append(phys * block_size + pos % block_size if ok else -1)
        lens[b] += c
    return tables, lens, np.asarray(slots, dtype=np.int64), nb
