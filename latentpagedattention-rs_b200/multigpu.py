"""Multi-GPU plumbing of the decode path (one process per GPU).

Two partitionings, both strong scaling of one global batch:

* split-K: every sequence's logical blocks are cut into `world` contiguous
  ranges; rank r holds only its range's blocks (its own pool and tables) and
  decodes them into a normalised context plus log-sum-exp per (sequence,
  head).  The per-rank results are all-gathered and merged with the LSE rule
  (``gather_and_merge``).  The value projection is linear, so it is applied
  before the exchange, which then carries head_dim floats per head.
* sequence sharding: sequences go to ranks by longest-processing-time on
  their lengths (``lpt_assign``); no collective on the data path.

With a W_o output projection, W_o is column-sharded: rank r holds columns
``column_range(out_dim, world, r)``.  The rows to project (the merged
contexts under split-K, every rank's sequences under sequence sharding,
gathered with ``gather_rows``) are multiplied by the local slice and the
column slices are all-gathered (``sharded_out_proj``): each rank reads 1/world
of W_o instead of all of it.

The functions take the decode / merge callables as arguments so that the
same host logic runs with the CUDA kernels on GPUs and, in tests, with
CPU stand-ins over a ``gloo`` process group.
"""

from __future__ import annotations

import numpy as np


def lpt_assign(lens, world: int) -> np.ndarray:
    """Owner rank of every sequence: longest first onto the least-loaded rank."""
    lens = np.asarray(lens, dtype=np.int64)
    owner = np.zeros(lens.size, dtype=np.int64)
    load = np.zeros(world, dtype=np.int64)
    for b in np.argsort(-lens, kind="stable"):
        r = int(np.argmin(load))
        owner[b] = r
        load[r] += int(lens[b])
    return owner


def split_k_ranges(global_lens, block_size: int, world: int, rank: int,
                   extra_tokens: int = 0) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Rank `rank`'s share of every sequence under split-K.

    Returns (first_block, block_count, local_len): the first global logical
    block it holds, how many, and how many active tokens fall in them.
    ``extra_tokens`` reserves room for appends (blocks are counted on
    ``len + extra_tokens``)."""
    lens = np.asarray(global_lens, dtype=np.int64)
    nblocks = (lens + extra_tokens + block_size - 1) // block_size
    first = (nblocks * rank) // world
    last = (nblocks * (rank + 1)) // world
    lo = first * block_size
    hi = np.minimum(last * block_size, lens)
    local = np.clip(hi - lo, 0, None)
    return first, last - first, local.astype(np.int32)


def append_slots(global_positions, tables_local: np.ndarray, first_block: np.ndarray,
                 block_size: int) -> np.ndarray:
    """Slot (physical * block_size + offset) of each sequence's appended row
    in this rank's pool, or -1 when another rank holds that position."""
    pos = np.asarray(global_positions, dtype=np.int64)
    slots = np.full(pos.size, -1, dtype=np.int64)
    for b, p in enumerate(pos):
        lb = p // block_size - int(first_block[b])
        if 0 <= lb < tables_local.shape[1] and tables_local[b, lb] >= 0:
            slots[b] = int(tables_local[b, lb]) * block_size + int(p % block_size)
    return slots


def gather_and_merge(ctx, lse, world: int, merge_fn, gathered_ctx=None, gathered_lse=None,
                     group=None):
    """All-gather every rank's (ctx [B, H, D], lse [B, H]) and merge them.

    ``merge_fn(stacked_ctx [world, B, H, D], stacked_lse [world, B, H])``
    returns the merged context.  Every rank ends with the same result."""
    import torch
    import torch.distributed as dist

    if gathered_ctx is None:
        gathered_ctx = torch.empty((world, *ctx.shape), dtype=ctx.dtype, device=ctx.device)
    if gathered_lse is None:
        gathered_lse = torch.empty((world, *lse.shape), dtype=lse.dtype, device=lse.device)
    if ctx.device.type == "cuda":
        dist.all_gather_into_tensor(gathered_ctx, ctx.contiguous(), group=group)
        dist.all_gather_into_tensor(gathered_lse, lse.contiguous(), group=group)
    else:  # gloo has no all_gather_into_tensor
        dist.all_gather(list(gathered_ctx.unbind(0)), ctx.contiguous(), group=group)
        dist.all_gather(list(gathered_lse.unbind(0)), lse.contiguous(), group=group)
    return merge_fn(gathered_ctx, gathered_lse)


# ---------------------------------------------------- W_o column sharding

def column_range(out_dim: int, world: int, rank: int) -> tuple[int, int]:
    """Columns [c0, c1) of W_o that `rank` holds: equal contiguous slices
    (``out_dim`` must be a multiple of ``world``)."""
    if out_dim % world:
        raise ValueError(f"out_dim {out_dim} is not a multiple of the world size {world}")
    w = out_dim // world
    return rank * w, (rank + 1) * w


def gather_rows(x_local, world: int, max_rows: int, gathered=None, group=None):
    """All-gather every rank's row block ``x_local [n_r, K]`` (n_r <= max_rows)
    into ``gathered [world, max_rows, K]``; rows past n_r of a block are
    left as they were (the caller ignores them)."""
    import torch
    import torch.distributed as dist

    n, K = x_local.shape
    if n > max_rows:
        raise ValueError("x_local has more rows than max_rows")
    if gathered is None:
        gathered = torch.zeros((world, max_rows, K), dtype=x_local.dtype, device=x_local.device)
    send = x_local
    if n < max_rows:
        send = torch.zeros((max_rows, K), dtype=x_local.dtype, device=x_local.device)
        send[:n] = x_local
    if x_local.device.type == "cuda":
        dist.all_gather_into_tensor(gathered, send.contiguous(), group=group)
    else:
        dist.all_gather(list(gathered.unbind(0)), send.contiguous(), group=group)
    return gathered


def sharded_out_proj(x_full, w_o_slice, world: int, proj_fn, gathered=None, group=None):
    """Column-sharded W_o: every rank computes ``x_full @ w_o_slice`` (its
    ``out_dim / world`` columns, ``proj_fn(x, w)``) and the slices are
    all-gathered into ``gathered [world, rows, out_dim / world]``, so every
    rank holds ``out = concat(gathered[0], ..., gathered[world-1], dim=1)``
    while reading only 1/world of W_o."""
    import torch
    import torch.distributed as dist

    y = proj_fn(x_full, w_o_slice)
    if gathered is None:
        gathered = torch.empty((world, *y.shape), dtype=y.dtype, device=y.device)
    if y.device.type == "cuda":
        dist.all_gather_into_tensor(gathered, y.contiguous(), group=group)
    else:
        dist.all_gather(list(gathered.unbind(0)), y.contiguous(), group=group)
    return gathered


def assemble_columns(gathered):
    """[world, rows, cols] slices -> [rows, world * cols] (for checking)."""
    return gathered.permute(1, 0, 2).reshape(gathered.shape[1], -1)
