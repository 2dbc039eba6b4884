"""Host operations over libplkv_b200 with PyTorch CUDA tensors.

Two layers:

* Drop-in functions that keep the names, arguments, results and exceptions of
  tatavishnurao/LatentPagedAttention-rs ``python_ref/latent_paged_attention``
  (cache_ref.py, attention_ref.py) but run on the GPU: the FP16 storage
  conversion, the latent-row write, the runtime-length direct paged latent
  decode and the paged full-KV GQA baseline.
* The batched serving API (``DecodePlan``, ``latent_decode``,
  ``fullkv_decode``, ``latent_append``, ``kv_append``, ``out_proj``,
  ``lse_merge``) with a block table and an active length per sequence, used
  by the benchmark and the multi-GPU runner.

Every computation is a kernel of libplkv_b200.so; nothing here falls back to
a CPU or PyTorch implementation.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import check, lib

MASKED_SCORE = -3.4028234663852886e38


# ------------------------------------------------------------------ helpers

def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _need_cuda(name: str, t: torch.Tensor, dtype: torch.dtype | None = None) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must have dtype {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _to_cuda(x, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x.to(device=device, dtype=dtype).contiguous()
    return torch.as_tensor(np.asarray(x), dtype=dtype, device=device).contiguous()


def _flags_tensor(device: torch.device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def raise_for_flags(flags: int, where: str) -> None:
    """Turn device error flags into the reference's exceptions."""
    if flags & _lib.FLAG_NON_FINITE_INPUT:
        raise ValueError("FP16 storage input must be finite")
    if flags & _lib.FLAG_FP16_OVERFLOW:
        raise ValueError("FP16 storage conversion overflowed")
    if flags & _lib.FLAG_BAD_POSITION:
        raise IndexError("block_table does not cover token_position")
    if flags & _lib.FLAG_BAD_BLOCK:
        raise IndexError("block_table contains an out-of-range physical block")
    if flags & _lib.FLAG_BAD_LENGTH:
        raise ValueError("active sequence length exceeds the block table")
    if flags:
        raise RuntimeError(f"{where}: device error flags 0x{flags:x}")


# ------------------------------------------------------------- FP16 storage

def fp16_storage_bits(values: torch.Tensor) -> torch.Tensor:
    """cache_ref.py:17-19 / lib.rs:302-319 on the GPU.

    Returns the FP16 storage as an int16 tensor of IEEE binary16 bit patterns;
    raises ValueError for non-finite input or overflow like the reference.
    """
    _need_cuda("values", values, torch.float32)
    out = torch.empty(values.shape, dtype=torch.float16, device=values.device)
    flags = _flags_tensor(values.device)
    check(lib().plkv_quantize_f16(_ptr(values), _ptr(out), values.numel(), _ptr(flags),
                                  _stream(values.device)), "plkv_quantize_f16")
    raise_for_flags(int(flags.item()), "fp16_storage_bits")
    return out.view(torch.int16)


def fp16_storage_roundtrip_f32(values: torch.Tensor) -> torch.Tensor:
    """cache_ref.py:6-14 on the GPU: FP32 -> FP16 storage -> FP32."""
    return fp16_storage_bits(values).view(torch.float16).float()


def to_fp16_storage(values: torch.Tensor) -> torch.Tensor:
    """FP32 tensor -> FP16 storage tensor (same checks as fp16_storage_bits)."""
    return fp16_storage_bits(values).view(torch.float16)


# --------------------------------------------------------------- addressing

def resolve_paged_token_location(block_table, token_position: int,
                                 block_size: int) -> tuple[int, int, int]:
    """cache_ref.py:22-40 -- (logical block, physical block, in-block offset)."""
    table = np.asarray(block_table.cpu() if isinstance(block_table, torch.Tensor) else block_table)
    if table.ndim != 1:
        raise ValueError("block_table must be 1D")
    if block_size <= 0:
        raise ValueError(f"block_size must be > 0, got {block_size}")
    if token_position < 0:
        raise ValueError(f"token_position must be >= 0, got {token_position}")
    logical = token_position // block_size
    if logical >= table.size:
        raise IndexError("block_table does not cover token_position")
    physical = int(table[logical])
    if physical < 0:
        raise ValueError("block_table contains a negative physical block")
    return logical, physical, token_position % block_size


def projection_to_head_major(projection: torch.Tensor, heads: int, head_dim: int) -> torch.Tensor:
    """Canonical [latent, heads*head_dim] -> head-major [heads, latent, head_dim]
    (the GPU layout of fixtures.py:418-432)."""
    if projection.ndim != 2 or projection.shape[1] != heads * head_dim:
        raise ValueError("projection width must equal kv_heads * head_dim")
    return projection.reshape(projection.shape[0], heads, head_dim).permute(1, 0, 2).contiguous()


# ------------------------------------------------------------------ appends

def latent_append(rows: torch.Tensor, cache: torch.Tensor, block_tables: torch.Tensor, *,
                  positions: torch.Tensor | None = None, seq_lens: torch.Tensor | None = None,
                  seq_ids: torch.Tensor | None = None, flags: torch.Tensor | None = None) -> None:
    """Batched in-place FP16 latent-row write (lib.rs:889-939 per row).

    ``rows [n, L]`` FP32; ``cache [P, bs, L]`` FP16; ``block_tables [B, max_blocks]``
    int32.  Row i goes to sequence ``seq_ids[i]`` (default i) at ``positions[i]``;
    with ``seq_lens`` (int32, updated in place) the row is appended at the
    sequence's current length instead.
    """
    _need_cuda("rows", rows, torch.float32)
    _need_cuda("cache", cache, torch.float16)
    _need_cuda("block_tables", block_tables, torch.int32)
    P, bs, L = cache.shape
    if rows.ndim != 2 or rows.shape[1] != L:
        raise ValueError("new_latent width must match latent_dim")
    check(lib().plkv_latent_append_f16(
        _ptr(rows), _ptr(block_tables), block_tables.shape[1], _ptr(seq_ids), _ptr(positions),
        _ptr(seq_lens), rows.shape[0], _ptr(cache), P, bs, L, _ptr(flags),
        _stream(rows.device)), "plkv_latent_append_f16")


def latent_append_slots(rows: torch.Tensor, cache: torch.Tensor, slots: torch.Tensor,
                        flags: torch.Tensor | None = None) -> None:
    """Slot-mapped FP16 latent-row write (slot = physical * bs + offset)."""
    _need_cuda("rows", rows, torch.float32)
    _need_cuda("cache", cache, torch.float16)
    _need_cuda("slots", slots, torch.int64)
    P, bs, L = cache.shape
    check(lib().plkv_latent_append_slots_f16(_ptr(rows), _ptr(slots), rows.shape[0], _ptr(cache),
                                             P * bs, L, _ptr(flags), _stream(rows.device)),
          "plkv_latent_append_slots_f16")


def allocate_slots(block_tables: torch.Tensor, seq_lens: torch.Tensor, next_block: torch.Tensor,
                   num_physical: int, block_size: int, *, counts: torch.Tensor | None = None,
                   n_new: int | None = None, slots: torch.Tensor | None = None,
                   flags: torch.Tensor | None = None) -> torch.Tensor:
    """Device-side bump allocation of new token positions for a batch
    (PagedBlockTable.allocate_token_positions, block_table.py:26-38, on the
    GPU): advances `seq_lens` in place, stores new blocks in `block_tables`
    (entries < 0 are "no block yet") and the pool counter `next_block` ([1]
    int32), and returns the slot of every new token (int64, sequence order).
    `counts` ([B] int32, default one token per sequence) needs `n_new` (their
    sum) so that nothing synchronises with the host."""
    _need_cuda("block_tables", block_tables, torch.int32)
    _need_cuda("seq_lens", seq_lens, torch.int32)
    _need_cuda("next_block", next_block, torch.int32)
    B = seq_lens.shape[0]
    if counts is not None:
        _need_cuda("counts", counts, torch.int32)
        if n_new is None:
            raise ValueError("n_new (the sum of counts) is required with counts")
    total = B if counts is None else int(n_new)
    if slots is None:
        slots = torch.empty(max(total, 1), dtype=torch.int64, device=seq_lens.device)
    _need_cuda("slots", slots, torch.int64)
    if slots.numel() < total:
        raise ValueError(f"slots holds {slots.numel()} entries, {total} tokens are allocated")
    check(lib().plkv_allocate_slots(_ptr(block_tables), block_tables.shape[1], _ptr(seq_lens),
                                    _ptr(counts), B, block_size, _ptr(next_block), num_physical,
                                    _ptr(slots), slots.numel(), _ptr(flags),
                                    _stream(seq_lens.device)),
          "plkv_allocate_slots")
    return slots[:total]


def kv_append(k_rows: torch.Tensor, v_rows: torch.Tensor, k_cache: torch.Tensor,
              v_cache: torch.Tensor, block_tables: torch.Tensor, *,
              positions: torch.Tensor | None = None, seq_lens: torch.Tensor | None = None,
              seq_ids: torch.Tensor | None = None, flags: torch.Tensor | None = None) -> None:
    """Batched in-place FP16 K/V row write into head-major [P, KV, bs, D] caches."""
    for n, t in (("k_rows", k_rows), ("v_rows", v_rows)):
        _need_cuda(n, t, torch.float32)
    for n, t in (("k_cache", k_cache), ("v_cache", v_cache)):
        _need_cuda(n, t, torch.float16)
    _need_cuda("block_tables", block_tables, torch.int32)
    P, KV, bs, D = k_cache.shape
    check(lib().plkv_kv_append_f16(
        _ptr(k_rows), _ptr(v_rows), _ptr(block_tables), block_tables.shape[1], _ptr(seq_ids),
        _ptr(positions), _ptr(seq_lens), k_rows.shape[0], _ptr(k_cache), _ptr(v_cache), P, KV,
        bs, D, _ptr(flags), _stream(k_rows.device)), "plkv_kv_append_f16")


def paged_latent_write_fp16_storage(latent_cache: torch.Tensor, block_table, token_position: int,
                                    new_latent_f32: torch.Tensor, *,
                                    inplace: bool = False) -> torch.Tensor:
    """cache_ref.py:103-114 / lib.rs:889-939 on the GPU.

    ``latent_cache`` is the FP16 storage ``[blocks, block_size, latent_dim]``
    (an FP32 tensor is first converted with the FP16 storage checks).  The
    write goes into a copy unless ``inplace``; the FP16 cache is returned.
    """
    if latent_cache.ndim != 3:
        raise ValueError("latent_cache must have shape [blocks, block_size, latent_dim]")
    table = torch.as_tensor(np.asarray(block_table.cpu() if isinstance(block_table, torch.Tensor)
                                       else block_table))
    if table.ndim != 1:
        raise ValueError("block_table must be 1D")
    if new_latent_f32.ndim != 1:
        raise ValueError("new_latent must be 1D")
    if new_latent_f32.shape[0] != latent_cache.shape[2]:
        raise ValueError("new_latent width must match latent_dim")
    device = latent_cache.device
    cache = latent_cache if latent_cache.dtype == torch.float16 else to_fp16_storage(
        latent_cache.contiguous())
    if not bool(torch.isfinite(cache).all()):
        raise ValueError("latent cache and replacement must be finite")
    _, physical, _ = resolve_paged_token_location(table, token_position, cache.shape[1])
    if physical >= cache.shape[0]:
        raise IndexError("block_table contains an out-of-range physical block")
    if not inplace and cache is latent_cache:
        cache = cache.clone()
    flags = _flags_tensor(device)
    latent_append(_to_cuda(new_latent_f32, torch.float32, device).reshape(1, -1), cache,
                  _to_cuda(table, torch.int32, device).reshape(1, -1),
                  positions=torch.tensor([token_position], dtype=torch.int32, device=device),
                  flags=flags)
    raise_for_flags(int(flags.item()), "paged_latent_write_fp16_storage")
    return cache


# ------------------------------------------------------------------ planning

@dataclass
class DecodePlan:
    """Split-K work items on the device (from plkv_plan_splits / plkv_plan_workers)."""

    items: torch.Tensor           # [n_items, 4] int32 (seq, block_begin, block_end, 0)
    seq_item_begin: torch.Tensor  # [batch + 1] int32
    n_items: int
    batch: int
    items_host: np.ndarray
    seq_item_begin_host: np.ndarray
    worker_item_begin: torch.Tensor | None = None  # [n_workers + 1] int32
    n_workers: int = 0


def default_target_items(device: torch.device | None = None) -> int:
    if device is not None and torch.cuda.is_available():
        sms = torch.cuda.get_device_properties(device).multi_processor_count
    else:
        sms = 148
    return 2 * sms


def plan_splits(seq_lens_host, block_size: int, *, target_items: int | None = None,
                min_blocks: int = 1, device: torch.device | str = "cuda") -> DecodePlan:
    """Cut every sequence into contiguous split-K items (host planner of the C ABI)."""
    lens = np.ascontiguousarray(np.asarray(seq_lens_host, dtype=np.int32))
    batch = int(lens.size)
    device = torch.device(device)
    if target_items is None:
        target_items = default_target_items(device if device.type == "cuda" else None)
    n = ctypes.c_int32(0)
    L = lib()
    st = L.plkv_plan_splits(lens.ctypes.data, batch, block_size, target_items, min_blocks, None, 0,
                            None, ctypes.byref(n))
    if st not in (_lib.PLKV_OK, _lib.PLKV_ERR_WORKSPACE):
        check(st, "plkv_plan_splits")
    items = np.zeros((n.value, 4), dtype=np.int32)
    begin = np.zeros(batch + 1, dtype=np.int32)
    check(L.plkv_plan_splits(lens.ctypes.data, batch, block_size, target_items, min_blocks,
                             items.ctypes.data, n.value, begin.ctypes.data, ctypes.byref(n)),
          "plkv_plan_splits")
    return DecodePlan(torch.as_tensor(items, device=device), torch.as_tensor(begin, device=device),
                      n.value, batch, items, begin)


def plan_workers(seq_lens_host, block_size: int, *, n_workers: int | None = None,
                 device: torch.device | str = "cuda") -> DecodePlan:
    """Balanced plan for the persistent tensor-core decode: the blocks of all
    sequences are cut into `n_workers` equal contiguous ranges (default: one
    per CTA pair of the device)."""
    lens = np.ascontiguousarray(np.asarray(seq_lens_host, dtype=np.int32))
    batch = int(lens.size)
    device = torch.device(device)
    if n_workers is None:
        n_workers = default_target_items(device if device.type == "cuda" else None) // 4
    n = ctypes.c_int32(0)
    L = lib()
    st = L.plkv_plan_workers(lens.ctypes.data, batch, block_size, n_workers, None, 0, None, None,
                             ctypes.byref(n))
    if st not in (_lib.PLKV_OK, _lib.PLKV_ERR_WORKSPACE):
        check(st, "plkv_plan_workers")
    items = np.zeros((max(n.value, 1), 4), dtype=np.int32)
    begin = np.zeros(batch + 1, dtype=np.int32)
    wbegin = np.zeros(n_workers + 1, dtype=np.int32)
    check(L.plkv_plan_workers(lens.ctypes.data, batch, block_size, n_workers, items.ctypes.data,
                              n.value, begin.ctypes.data, wbegin.ctypes.data, ctypes.byref(n)),
          "plkv_plan_workers")
    items = items[:n.value]
    return DecodePlan(torch.as_tensor(items, device=device), torch.as_tensor(begin, device=device),
                      n.value, batch, items, begin, torch.as_tensor(wbegin, device=device),
                      n_workers)


FULLKV_MIN_ITEM_TOKENS = 2048


def plan_fullkv(seq_lens_host, block_size: int, kv_heads: int, *,
                device: torch.device | str = "cuda") -> DecodePlan:
    """Split-K plan for the full-KV decode, whose grid is items x KV heads.

    Items hold at least 2048 tokens (16 tiles of the tensor-core pass, which
    spends about two tiles' time filling its pipeline), unless the grid would
    then leave SMs idle.  On a B200, 16 x 4096 tokens (8 KV heads) take 74 us
    in 32 items against 171 us in the 304 of the default split, and
    64 x 4096 tokens take 241 us against 323 us."""
    lens = np.asarray(seq_lens_host, dtype=np.int64)
    device = torch.device(device)
    sms = default_target_items(device if device.type == "cuda" else None) // 2
    total = int(lens.sum())
    min_tokens = min(FULLKV_MIN_ITEM_TOKENS, max(1, total * max(1, kv_heads) // sms))
    return plan_splits(lens.astype(np.int32), block_size,
                       min_blocks=max(1, min_tokens // block_size), device=device)


# ------------------------------------------------------------------- decode

def project_query(q: torch.Tensor, w_k_head_major: torch.Tensor, *,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """q_lat[b, h] = W_k[kv(h)] q[b, h] (lib.rs:1026-1032), W_k [KV, L, D]."""
    _need_cuda("q", q, torch.float32)
    _need_cuda("w_k", w_k_head_major, torch.float32)
    B, Hq, D = q.shape
    KV, L, D2 = w_k_head_major.shape
    if D2 != D:
        raise ValueError("head_dim mismatch between q and W_k")
    if out is None:
        out = torch.empty((B, Hq, L), dtype=torch.float32, device=q.device)
    _need_cuda("out", out, torch.float32)
    if tuple(out.shape) != (B, Hq, L):
        raise ValueError(f"out must have shape {(B, Hq, L)}")
    q_lat = out
    check(lib().plkv_project_query(_ptr(q), _ptr(w_k_head_major), _ptr(q_lat), B, Hq, KV, D, L,
                                   _stream(q.device)), "plkv_project_query")
    return q_lat


def latent_workspace_bytes(n_items: int, batch: int, q_heads: int, latent_dim: int,
                           value_dim: int) -> int:
    return int(lib().plkv_latent_decode_workspace_size(n_items, batch, q_heads, latent_dim,
                                                       value_dim))


def latent_decode(q_lat: torch.Tensor, cache: torch.Tensor, block_tables: torch.Tensor,
                  seq_lens: torch.Tensor, plan: DecodePlan, *, scale: float,
                  value_dim: int | None = None, w_v: torch.Tensor | None = None,
                  mode: str = "exact", out: torch.Tensor | None = None,
                  want_lse: bool = False, want_scores: bool = False, want_probs: bool = False,
                  max_seq_len: int | None = None, workspace: torch.Tensor | None = None,
                  allow_empty: bool = False, flags: torch.Tensor | None = None,
                  phase: str = "all") -> dict:
    """Batched direct paged latent decode (lib.rs:941-1145 per sequence).

    ``q_lat [B, Hq, L]`` FP32; ``cache [P, bs, L]`` FP16; ``block_tables
    [B, max_blocks]`` and ``seq_lens [B]`` int32; ``w_v`` head-major
    ``[proj_heads, value_dim, head_dim]`` (query head h uses
    ``h // (Hq // proj_heads)``) or None for the latent context.
    ``phase`` runs both passes ("all"), only the split-K partial pass
    ("partial") or only the combine ("combine", same arguments and workspace).
    Returns a dict with ``ctx`` and, on request, ``lse``, ``scores``, ``probs``.
    """
    _need_cuda("q_lat", q_lat, torch.float32)
    _need_cuda("cache", cache, torch.float16)
    _need_cuda("block_tables", block_tables, torch.int32)
    _need_cuda("seq_lens", seq_lens, torch.int32)
    B, Hq, L = q_lat.shape
    P, bs, L2 = cache.shape
    if L2 != L:
        raise ValueError("latent_dim mismatch between q_lat and cache")
    Lv = L if value_dim is None else int(value_dim)
    dev = q_lat.device
    if w_v is not None:
        _need_cuda("w_v", w_v, torch.float32)
        PH, Lv2, D = w_v.shape
        if Lv2 != Lv:
            raise ValueError("W_v rows must equal value_dim")
    else:
        PH, D = Hq, Lv
    if out is None:
        out = torch.empty((B, Hq, D), dtype=torch.float32, device=dev)
    lse = torch.empty((B, Hq), dtype=torch.float32, device=dev) if want_lse else None
    if (want_scores or want_probs) and max_seq_len is None:
        raise ValueError("max_seq_len is required for scores / probabilities")
    scores = (torch.empty((B, Hq, max_seq_len), dtype=torch.float32, device=dev)
              if (want_scores or want_probs) else None)
    probs = torch.empty_like(scores) if want_probs else None
    need = latent_workspace_bytes(plan.n_items, B, Hq, L, Lv)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    a = _lib.LatentDecodeArgs(
        q_lat=_ptr(q_lat), cache=_ptr(cache), num_physical=P, block_size=bs, latent_dim=L,
        value_dim=Lv, batch=B, q_heads=Hq, scale=float(scale), block_tables=_ptr(block_tables),
        max_blocks=block_tables.shape[1], seq_lens=_ptr(seq_lens), items=_ptr(plan.items),
        seq_item_begin=_ptr(plan.seq_item_begin), n_items=plan.n_items,
        worker_item_begin=_ptr(plan.worker_item_begin), n_workers=plan.n_workers,
        allow_empty=int(allow_empty), w_v=_ptr(w_v), proj_heads=PH, head_dim=D, ctx=_ptr(out),
        lse=_ptr(lse), scores=_ptr(scores), probs=_ptr(probs),
        max_seq_len=int(max_seq_len or 0),
        mode=_lib.MODE_TC_F16 if mode == "tc" else _lib.MODE_EXACT_F32,
        workspace=_ptr(workspace), workspace_bytes=workspace.numel(), err_flags=_ptr(flags))
    fn = {"all": lib().plkv_latent_decode, "partial": lib().plkv_latent_decode_partial,
          "combine": lib().plkv_latent_decode_combine}[phase]
    check(fn(ctypes.byref(a), _stream(dev)), "plkv_latent_decode")
    return {"ctx": out, "lse": lse, "scores": scores, "probs": probs, "workspace": workspace,
            "args": a}


def fullkv_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  block_tables: torch.Tensor, seq_lens: torch.Tensor, plan: DecodePlan, *,
                  scale: float, out: torch.Tensor | None = None, want_lse: bool = False,
                  want_scores: bool = False, want_probs: bool = False,
                  max_seq_len: int | None = None, workspace: torch.Tensor | None = None,
                  allow_empty: bool = False, flags: torch.Tensor | None = None) -> dict:
    """Batched FP16 full-KV paged GQA decode (lib.rs:1147-1269 per sequence).

    ``q [B, Hq, D]`` FP32; ``k_cache``/``v_cache`` head-major ``[P, KV, bs, D]`` FP16.
    """
    _need_cuda("q", q, torch.float32)
    _need_cuda("k_cache", k_cache, torch.float16)
    _need_cuda("v_cache", v_cache, torch.float16)
    _need_cuda("block_tables", block_tables, torch.int32)
    _need_cuda("seq_lens", seq_lens, torch.int32)
    B, Hq, D = q.shape
    P, KV, bs, D2 = k_cache.shape
    if D2 != D or v_cache.shape != k_cache.shape:
        raise ValueError("head_dim mismatch between q and paged cache tensors")
    dev = q.device
    if out is None:
        out = torch.empty((B, Hq, D), dtype=torch.float32, device=dev)
    lse = torch.empty((B, Hq), dtype=torch.float32, device=dev) if want_lse else None
    if (want_scores or want_probs) and max_seq_len is None:
        raise ValueError("max_seq_len is required for scores / probabilities")
    scores = (torch.empty((B, Hq, max_seq_len), dtype=torch.float32, device=dev)
              if (want_scores or want_probs) else None)
    probs = torch.empty_like(scores) if want_probs else None
    need = int(lib().plkv_fullkv_decode_workspace_size(plan.n_items, B, Hq, D))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    a = _lib.FullKVDecodeArgs(
        q=_ptr(q), k_cache=_ptr(k_cache), v_cache=_ptr(v_cache), num_physical=P, kv_heads=KV,
        block_size=bs, head_dim=D, batch=B, q_heads=Hq, scale=float(scale),
        block_tables=_ptr(block_tables), max_blocks=block_tables.shape[1],
        seq_lens=_ptr(seq_lens), items=_ptr(plan.items), seq_item_begin=_ptr(plan.seq_item_begin),
        n_items=plan.n_items, allow_empty=int(allow_empty), ctx=_ptr(out), lse=_ptr(lse),
        scores=_ptr(scores), probs=_ptr(probs), max_seq_len=int(max_seq_len or 0),
        workspace=_ptr(workspace), workspace_bytes=workspace.numel(), err_flags=_ptr(flags))
    check(lib().plkv_fullkv_decode(ctypes.byref(a), _stream(dev)), "plkv_fullkv_decode")
    return {"ctx": out, "lse": lse, "scores": scores, "probs": probs, "workspace": workspace}


def lse_merge(ctx_shards: torch.Tensor, lse_shards: torch.Tensor,
              out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """LSE merge of per-shard contexts ``[S, rows..., width]`` / ``[S, rows...]``."""
    _need_cuda("ctx_shards", ctx_shards, torch.float32)
    _need_cuda("lse_shards", lse_shards, torch.float32)
    S = ctx_shards.shape[0]
    width = ctx_shards.shape[-1]
    rows = lse_shards[0].numel()
    if out is None:
        out = torch.empty(ctx_shards.shape[1:], dtype=torch.float32, device=ctx_shards.device)
    lse_out = torch.empty(lse_shards.shape[1:], dtype=torch.float32, device=ctx_shards.device)
    check(lib().plkv_lse_merge(_ptr(ctx_shards), _ptr(lse_shards), S, rows, width, _ptr(out),
                               _ptr(lse_out), _stream(ctx_shards.device)), "plkv_lse_merge")
    return out, lse_out


def default_out_proj_splits(in_dim: int, out_dim: int, device: torch.device | None = None) -> int:
    """Split of the contracted dimension of the W_o GEMM: about four CTAs per
    SM over the 128-column tiles, at least 64 rows of W_o per split."""
    tiles = (out_dim + 127) // 128
    k_splits = max(1, min(64, (2 * default_target_items(device)) // max(tiles, 1)))
    return min(k_splits, max(1, in_dim // 64))


def out_proj_workspace_bytes(batch: int, out_dim: int, k_splits: int) -> int:
    return int(lib().plkv_out_proj_workspace_size(batch, out_dim, k_splits))


def out_proj(x: torch.Tensor, w_o: torch.Tensor, *, out: torch.Tensor | None = None,
             k_splits: int | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """W_o output projection ``out = x @ w_o`` in FP32 (x [B, in], w_o [in, out])."""
    _need_cuda("x", x, torch.float32)
    _need_cuda("w_o", w_o, torch.float32)
    B, K = x.shape
    K2, N = w_o.shape
    if K2 != K:
        raise ValueError("W_o rows must equal the concatenated head width")
    if k_splits is None:
        k_splits = default_out_proj_splits(K, N, x.device)
    if out is None:
        out = torch.empty((B, N), dtype=torch.float32, device=x.device)
    need = int(lib().plkv_out_proj_workspace_size(B, N, k_splits))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    check(lib().plkv_out_proj(_ptr(x), _ptr(w_o), _ptr(out), B, K, N, k_splits, _ptr(workspace),
                              workspace.numel(), _stream(x.device)), "plkv_out_proj")
    return out


def default_out_proj_tc_splits(in_dim: int, out_dim: int, batch: int,
                               device: torch.device | None = None) -> int:
    """K splits of the tensor-core W_o product: enough CTAs (256 output
    columns x 128 batch rows x a K range each) to cover every SM once."""
    sms = default_target_items(device) // 2
    tiles = ((out_dim + 255) // 256) * ((batch + 127) // 128)
    return max(1, min(in_dim // 32, sms // max(tiles, 1)))


def out_proj_tc(x: torch.Tensor, w_o: torch.Tensor, *, out: torch.Tensor | None = None,
                k_splits: int | None = None, workspace: torch.Tensor | None = None,
                flags: torch.Tensor | None = None) -> torch.Tensor:
    """W_o output projection ``out = x @ w_o`` on the tensor cores (TF32
    operands, FP32 accumulation; ~1e-3 normwise relative error)."""
    _need_cuda("x", x, torch.float32)
    _need_cuda("w_o", w_o, torch.float32)
    B, K = x.shape
    K2, N = w_o.shape
    if K2 != K:
        raise ValueError("W_o rows must equal the concatenated head width")
    if k_splits is None:
        k_splits = default_out_proj_tc_splits(K, N, B, x.device)
    if out is None:
        out = torch.empty((B, N), dtype=torch.float32, device=x.device)
    need = int(lib().plkv_out_proj_tc_workspace_size(B, N, k_splits))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    check(lib().plkv_out_proj_tc(_ptr(x), _ptr(w_o), _ptr(out), B, K, N, k_splits,
                                 _ptr(workspace), workspace.numel(), _ptr(flags),
                                 _stream(x.device)), "plkv_out_proj_tc")
    return out


# ------------------------------------------------- materialised reconstruction

def reconstruct_kv(latent: torch.Tensor, w_k: torch.Tensor, w_v: torch.Tensor, *,
                   slots: torch.Tensor | None = None, n_rows: int | None = None,
                   block_size: int = 1, value_dim: int | None = None,
                   out_dtype: torch.dtype = torch.float16, k_out: torch.Tensor | None = None,
                   v_out: torch.Tensor | None = None,
                   flags: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Materialised K / V from latent rows (reconstruct_latent_kv_f32,
    lib.rs:517-580) into the head-major paged layout
    ``[num_slots // block_size, KV, block_size, D]``.

    ``latent`` is the latent pool viewed as rows ``[num_slots, L]`` (FP32 or
    FP16; a paged cache ``[P, bs, L]`` is accepted as is); ``w_k`` / ``w_v``
    head-major ``[KV, L, D]`` / ``[KV, Lv, D]`` FP32; ``slots`` (int64) picks
    the rows to rebuild (default: the first ``n_rows``, else all)."""
    if latent.dtype not in (torch.float32, torch.float16):
        raise TypeError("latent must be FP32 or FP16")
    _need_cuda("latent", latent)
    _need_cuda("w_k", w_k, torch.float32)
    _need_cuda("w_v", w_v, torch.float32)
    L = latent.shape[-1]
    rows = latent.reshape(-1, L)
    num_slots = rows.shape[0]
    KV, L2, D = w_k.shape
    if L2 != L:
        raise ValueError("latent_dim mismatch between latent rows and W_k")
    Lv = w_v.shape[1] if value_dim is None else int(value_dim)
    if tuple(w_v.shape) != (KV, Lv, D):
        raise ValueError("W_v must be [kv_heads, value_dim, head_dim]")
    if out_dtype not in (torch.float32, torch.float16):
        raise TypeError("out_dtype must be FP32 or FP16")
    if num_slots % block_size:
        raise ValueError("the number of latent rows must be a multiple of block_size")
    shape = (num_slots // block_size, KV, block_size, D)
    if k_out is None:
        k_out = torch.empty(shape, dtype=out_dtype, device=latent.device)
    if v_out is None:
        v_out = torch.empty(shape, dtype=out_dtype, device=latent.device)
    for name, t in (("k_out", k_out), ("v_out", v_out)):
        _need_cuda(name, t, out_dtype)
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {shape}")
    if slots is not None:
        _need_cuda("slots", slots, torch.int64)
        n = slots.numel() if n_rows is None else int(n_rows)
        if n > slots.numel():
            raise ValueError("n_rows exceeds the slot list")
    else:
        n = num_slots if n_rows is None else int(n_rows)
    check(lib().plkv_reconstruct_kv(_ptr(rows), int(rows.dtype == torch.float16), num_slots, L,
                                    Lv, _ptr(slots), n, _ptr(w_k), _ptr(w_v), KV, D, block_size,
                                    _ptr(k_out), _ptr(v_out), int(out_dtype == torch.float16),
                                    _ptr(flags), _stream(latent.device)), "plkv_reconstruct_kv")
    return k_out, v_out


def latent_kv_reconstruction(latent_cache, k_proj, v_proj, *, kv_heads: int,
                             head_dim: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Drop-in for latent_kv_reconstruction_ref (attention_ref.py:227-274) on
    the GPU: ``latent_cache [batch, seq, latent]``, ``k_proj`` / ``v_proj``
    ``[latent, kv_heads * head_dim]`` -> K, V ``[batch, seq, kv_heads,
    head_dim]`` FP32, with the reference's argument checks and messages."""
    dev = torch.device("cuda")
    lat = _to_cuda(latent_cache, torch.float32, dev)
    kp = _to_cuda(k_proj, torch.float32, dev)
    vp = _to_cuda(v_proj, torch.float32, dev)
    if lat.ndim != 3:
        raise ValueError("latent_cache must have shape [batch, seq_len, latent_dim]")
    if kp.ndim != 2 or vp.ndim != 2:
        raise ValueError("k_proj and v_proj must have shape [latent_dim, kv_heads * head_dim]")
    if kp.shape != vp.shape:
        raise ValueError("k_proj and v_proj shapes must match")
    if kv_heads <= 0:
        raise ValueError(f"kv_heads must be > 0, got {kv_heads}")
    if head_dim <= 0:
        raise ValueError(f"head_dim must be > 0, got {head_dim}")
    batch, seq_len, latent_dim = lat.shape
    if batch <= 0 or seq_len <= 0 or latent_dim <= 0:
        raise ValueError("latent_cache dimensions must be > 0")
    if kp.shape[0] != latent_dim:
        raise ValueError("latent_dim mismatch between cache and projections")
    if kp.shape[1] != kv_heads * head_dim:
        raise ValueError("projection width must equal kv_heads * head_dim")
    flags = _flags_tensor(dev)
    k, v = reconstruct_kv(lat, projection_to_head_major(kp, kv_heads, head_dim),
                          projection_to_head_major(vp, kv_heads, head_dim), block_size=1,
                          out_dtype=torch.float32, flags=flags)
    f = int(flags.item())
    if f & (_lib.FLAG_NON_FINITE_INPUT | _lib.FLAG_FP16_OVERFLOW):
        raise ValueError("reconstructed K cache must be finite")
    raise_for_flags(f, "latent_kv_reconstruction")
    return (k.reshape(batch, seq_len, kv_heads, head_dim),
            v.reshape(batch, seq_len, kv_heads, head_dim))


# ------------------------------------------- drop-ins for attention_ref.py

def _check_group(q_heads: int, kv_heads: int, group_size: int) -> None:
    """attention_ref.py:13-20."""
    if group_size <= 0:
        raise ValueError(f"group_size must be > 0, got {group_size}")
    if q_heads != kv_heads * group_size:
        raise ValueError("expected q_heads == kv_heads * group_size, "
                         f"got q_heads={q_heads}, kv_heads={kv_heads}, group_size={group_size}")


def direct_paged_latent_gqa_fp16_storage_runtime_intermediates(
        q, latent_blocks, block_table, max_seq_len: int, active_seq_len: int, block_size: int,
        k_proj, v_proj, *, q_heads: int, kv_heads: int, head_dim: int, group_size: int,
        mode: str = "exact"):
    """attention_ref.py:617-648 / lib.rs:1090-1145 on the GPU.

    Same arguments as the reference: ``q [batch, q_heads, head_dim]``,
    ``latent_blocks [physical_blocks, block_size, latent_dim]`` (FP32 source
    values, rounded to FP16 storage here, or an FP16 storage tensor), one
    ``block_table`` shared by the batch, canonical ``k_proj``/``v_proj``
    ``[latent_dim, kv_heads*head_dim]``.  Returns ``(scores, probabilities,
    context)`` as CUDA tensors, scores/probabilities padded to max_seq_len.
    """
    if active_seq_len <= 0 or active_seq_len > max_seq_len:
        raise ValueError("active_seq_len must satisfy 1 <= active_seq_len <= max_seq_len")
    device = q.device if isinstance(q, torch.Tensor) and q.is_cuda else torch.device("cuda")
    q = _to_cuda(q, torch.float32, device)
    if q.ndim != 3 or q.shape[0] <= 0 or tuple(q.shape[1:]) != (q_heads, head_dim):
        raise ValueError("q must have shape [batch, q_heads, head_dim]")
    lb = latent_blocks if isinstance(latent_blocks, torch.Tensor) else torch.as_tensor(
        np.asarray(latent_blocks))
    if lb.ndim != 3 or lb.shape[1] != block_size:
        raise ValueError("latent_blocks must have shape [physical_blocks, block_size, latent_dim]")
    table = np.asarray(block_table.cpu() if isinstance(block_table, torch.Tensor) else block_table)
    if table.ndim != 1 or table.size * block_size < active_seq_len:
        raise ValueError("block_table must cover seq_len and be 1D")
    if block_size <= 0 or kv_heads <= 0 or head_dim <= 0:
        raise ValueError("dimensions must be positive")
    _check_group(q_heads, kv_heads, group_size)
    kp = _to_cuda(k_proj, torch.float32, device)
    vp = _to_cuda(v_proj, torch.float32, device)
    if kp.ndim != 2 or tuple(vp.shape) != tuple(kp.shape):
        raise ValueError("K/V projections must share a 2D shape")
    latent_dim = lb.shape[2]
    if tuple(kp.shape) != (latent_dim, kv_heads * head_dim):
        raise ValueError("projection shape does not match latent dimensions")
    if np.any(table < 0) or np.any(table >= lb.shape[0]):
        raise ValueError("block_table contains out-of-range physical block indices")
    if not (bool(torch.isfinite(q).all()) and bool(torch.isfinite(kp).all())
            and bool(torch.isfinite(vp).all())):
        raise ValueError("inputs must be finite")
    if lb.dtype == torch.float16:
        cache = lb.to(device).contiguous()
        if not bool(torch.isfinite(cache).all()):
            raise ValueError("inputs must be finite")
    else:
        cache = to_fp16_storage(_to_cuda(lb, torch.float32, device))
    batch = q.shape[0]
    wk = projection_to_head_major(kp, kv_heads, head_dim)
    wv = projection_to_head_major(vp, kv_heads, head_dim)
    q_lat = project_query(q, wk)
    tables = _to_cuda(np.broadcast_to(table.astype(np.int32), (batch, table.size)), torch.int32,
                      device)
    lens_host = np.full(batch, active_seq_len, dtype=np.int32)
    lens = _to_cuda(lens_host, torch.int32, device)
    plan = plan_splits(lens_host, block_size, device=device)
    flags = _flags_tensor(device)
    r = latent_decode(q_lat, cache, tables, lens, plan, scale=1.0 / math.sqrt(float(head_dim)),
                      w_v=wv, mode=mode, want_scores=True, want_probs=True,
                      max_seq_len=max_seq_len, flags=flags)
    raise_for_flags(int(flags.item()), "direct_paged_latent_gqa_fp16_storage_runtime")
    return r["scores"], r["probs"], r["ctx"]


def paged_full_kv_gqa_decode_fp16_storage_runtime(
        q, k_head_major, v_head_major, block_table, max_seq_len: int, active_seq_len: int, *,
        group_size: int):
    """lib.rs:1147-1269 on the GPU.

    ``k_head_major``/``v_head_major`` are FP16 storage ``[P, kv_heads,
    block_size, head_dim]`` (FP32 sources are rounded to FP16 first); one
    ``block_table`` shared by the batch.  Returns ``(scores, probabilities,
    context)`` padded to ``max_seq_len``.
    """
    device = q.device if isinstance(q, torch.Tensor) and q.is_cuda else torch.device("cuda")
    q = _to_cuda(q, torch.float32, device)
    if q.ndim != 3:
        raise ValueError("q must have shape [batch, q_heads, head_dim]")
    if max_seq_len <= 0 or active_seq_len <= 0:
        raise ValueError("sequence lengths must be > 0")
    if active_seq_len > max_seq_len:
        raise ValueError("active sequence length exceeds max sequence length")
    kk = k_head_major if isinstance(k_head_major, torch.Tensor) else torch.as_tensor(
        np.asarray(k_head_major))
    vv = v_head_major if isinstance(v_head_major, torch.Tensor) else torch.as_tensor(
        np.asarray(v_head_major))
    if kk.ndim != 4 or tuple(kk.shape) != tuple(vv.shape):
        raise ValueError("k/v must have shape [num_physical_blocks, kv_heads, block_size, head_dim]")
    P, KV, bs, D = kk.shape
    if q.shape[2] != D:
        raise ValueError("head_dim mismatch between q and paged cache tensors")
    _check_group(q.shape[1], KV, group_size)
    table = np.asarray(block_table.cpu() if isinstance(block_table, torch.Tensor) else block_table)
    if table.ndim != 1 or table.size * bs < max_seq_len:
        raise ValueError("block table does not cover max sequence")
    if np.any(table < 0) or np.any(table >= P):
        raise ValueError("block table index out of range")
    k16 = kk.to(device).contiguous() if kk.dtype == torch.float16 else to_fp16_storage(
        _to_cuda(kk, torch.float32, device))
    v16 = vv.to(device).contiguous() if vv.dtype == torch.float16 else to_fp16_storage(
        _to_cuda(vv, torch.float32, device))
    batch = q.shape[0]
    tables = _to_cuda(np.broadcast_to(table.astype(np.int32), (batch, table.size)), torch.int32,
                      device)
    lens_host = np.full(batch, active_seq_len, dtype=np.int32)
    lens = _to_cuda(lens_host, torch.int32, device)
    plan = plan_splits(lens_host, bs, device=device)
    flags = _flags_tensor(device)
    r = fullkv_decode(q, k16, v16, tables, lens, plan, scale=1.0 / math.sqrt(float(D)),
                      want_scores=True, want_probs=True, max_seq_len=max_seq_len, flags=flags)
    raise_for_flags(int(flags.item()), "paged_full_kv_gqa_decode_fp16_storage_runtime")
    return r["scores"], r["probs"], r["ctx"]


def paged_gqa_decode_attention_intermediates(q, k_blocks, v_blocks, block_table, seq_len: int,
                                             block_size: int, *, group_size: int):
    """attention_ref.py:172-224 with FP16 storage, on the GPU.

    Takes the reference's token-major blocks ``[P, block_size, kv_heads,
    head_dim]`` and converts them once to the head-major GPU layout.
    """
    kb = k_blocks if isinstance(k_blocks, torch.Tensor) else torch.as_tensor(np.asarray(k_blocks))
    vb = v_blocks if isinstance(v_blocks, torch.Tensor) else torch.as_tensor(np.asarray(v_blocks))
    if kb.ndim != 4 or vb.ndim != 4:
        raise ValueError("k_blocks and v_blocks must have shape "
                         "[num_physical_blocks, block_size, kv_heads, head_dim]")
    if kb.shape[1] != block_size:
        raise ValueError(f"block_size mismatch: cache has {kb.shape[1]}, argument was {block_size}")
    if seq_len <= 0:
        raise ValueError(f"seq_len must be > 0, got {seq_len}")
    table = np.asarray(block_table.cpu() if isinstance(block_table, torch.Tensor) else block_table)
    if table.ndim != 1:
        raise ValueError("block_table must be 1D")
    if table.size * block_size < seq_len:
        raise ValueError("block_table does not cover the requested seq_len")
    return paged_full_kv_gqa_decode_fp16_storage_runtime(
        q, kb.permute(0, 2, 1, 3).contiguous(), vb.permute(0, 2, 1, 3).contiguous(), table,
        seq_len, seq_len, group_size=group_size)


def tc_available(spec) -> bool:
    """Whether the tcgen05 decode kernel covers this workload's shapes
    (absorbed MLA: 128 query heads, latent 576 = 512 value + 64 RoPE,
    block size a multiple of 32)."""
    return (spec.q_heads == 128 and spec.latent_dim == 576 and spec.value_dim == 512
            and spec.block_size % 32 == 0)
