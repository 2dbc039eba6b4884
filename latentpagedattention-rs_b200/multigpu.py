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


# ------------------------------------------ peer-memory split-K exchange

class PeerExchange:
    """Split-K result exchange through peer memory (``plkv_peer_*``).

    Rank r publishes its (ctx [rows, width], lse [rows]) in a buffer of its
    own that every rank of the node has mapped; each rank's merge reads the W
    ranks' rows over NVLink and applies the LSE rule, so every rank ends with
    the merged rows.  Replaces ``gather_and_merge`` (two all-gathers and a
    merge kernel) with two kernels and no collective on the data path; the
    one collective is the handle swap at construction.  Every rank must call
    ``publish`` and ``merge`` once per step, in the same order, and ``close``
    only after its last merge (it synchronises the ranks first)."""

    def __init__(self, rows: int, width: int, world: int, rank: int, device, group=None,
                 _local_ptrs=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _lib

        self._lib = _lib
        L = _lib.lib()
        self.rows, self.width, self.world, self.rank = int(rows), int(width), world, rank
        self.device = torch.device(device)
        self.group = group
        self.opened, self.own = [], None
        if _local_ptrs is not None:
            ptrs = list(_local_ptrs)
        else:
            nbytes = self._buffer_bytes()
            own = ctypes.c_void_p()
            handle = (ctypes.c_char * 64)()
            _lib.check(L.plkv_peer_alloc(nbytes, ctypes.byref(own), handle), "plkv_peer_alloc")
            self.own = own.value
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            ptrs = []
            for s in range(world):
                if s == rank:
                    ptrs.append(self.own)
                    continue
                h = (ctypes.c_char * 64).from_buffer_copy(handles[s])
                p = ctypes.c_void_p()
                _lib.check(L.plkv_peer_open(h, ctypes.byref(p)), "plkv_peer_open")
                self.opened.append(p.value)
                ptrs.append(p.value)
        self.bufs = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.ctrl = torch.zeros(4, dtype=torch.int64, device=self.device)

    def _buffer_bytes(self) -> int:
        return int(self._lib.lib().plkv_peer_buffer_bytes(self.rows, self.width))

    @classmethod
    def local_group(cls, world: int, rows: int, width: int, device):
        """`world` exchanges over plain buffers of one device (a single-process
        stand-in for the ranks, for tests): publishes must all precede the
        merges in stream order.  Returns (exchanges, buffers)."""
        import torch

        from . import _lib

        L = _lib.lib()
        nbytes = int(L.plkv_peer_buffer_bytes(rows, width))
        bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=device) for _ in range(world)]
        stream = torch.cuda.current_stream(torch.device(device)).cuda_stream
        for b in bufs:
            _lib.check(L.plkv_peer_init_buffer(b.data_ptr(), nbytes, stream),
                       "plkv_peer_init_buffer")
        ptrs = [b.data_ptr() for b in bufs]
        return [cls(rows, width, world, r, device, _local_ptrs=ptrs) for r in range(world)], bufs

    def _stream(self):
        import torch

        return torch.cuda.current_stream(self.device).cuda_stream

    def publish(self, ctx, lse, flags=None) -> None:
        import torch

        for n, t in (("ctx", ctx), ("lse", lse)):
            if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float32
                    and t.is_contiguous()):
                raise TypeError(f"{n} must be a contiguous FP32 CUDA tensor")
        if ctx.numel() != self.rows * self.width or lse.numel() != self.rows:
            raise ValueError("ctx / lse do not match the exchange's rows x width")
        L = self._lib.lib()
        self._lib.check(L.plkv_peer_publish(ctx.data_ptr(), lse.data_ptr(), self.rows, self.width,
                                            self.bufs.data_ptr(), self.world, self.rank,
                                            self.ctrl.data_ptr(),
                                            None if flags is None else flags.data_ptr(),
                                            self._stream()),
                        "plkv_peer_publish")

    def merge(self, out, lse_out=None, flags=None):
        import torch

        if not (isinstance(out, torch.Tensor) and out.is_cuda and out.dtype == torch.float32
                and out.is_contiguous() and out.numel() == self.rows * self.width):
            raise TypeError("out must be a contiguous FP32 CUDA tensor of rows x width")
        L = self._lib.lib()
        self._lib.check(L.plkv_peer_merge(self.rows, self.width, self.bufs.data_ptr(), self.world,
                                          self.rank, self.ctrl.data_ptr(), out.data_ptr(),
                                          None if lse_out is None else lse_out.data_ptr(),
                                          None if flags is None else flags.data_ptr(),
                                          self._stream()),
                        "plkv_peer_merge")
        return out

    def close(self) -> None:
        """Synchronise the ranks, then unmap the peers' buffers and free this
        rank's (no rank may still read it)."""
        import torch
        import torch.distributed as dist

        if self.own is None and not self.opened:
            return
        torch.cuda.synchronize(self.device)
        if dist.is_initialized():
            dist.barrier(group=self.group)
        L = self._lib.lib()
        for p in self.opened:
            L.plkv_peer_close(p)
        if self.own is not None:
            L.plkv_peer_free(self.own)
        self.opened, self.own = [], None


# ------------------------------------- head-sharded split-K merge (peer memory)

class ShardExchange(PeerExchange):
    """Head-sharded merge of split-K results (``plkv_shard_publish`` /
    ``plkv_shard_merge``).

    Rank r owns query heads ``[r * H / W, (r + 1) * H / W)``.  After the
    partial pass, ``publish(args)`` merges the rank's work items per
    (sequence, head) and stores the normalised latent context and its
    log-sum-exp into the owner's buffer over NVLink; ``merge(out)`` waits for
    every rank's publish of the step, merges the W sources and applies W_uv of
    the owned heads.  Every rank reads W_uv for H / W heads only, and the
    result stays sharded by heads (``out [B, H / W, D]``), the layout a
    row-sharded W_o consumes.  Same lifetime rules as ``PeerExchange``."""

    def __init__(self, batch: int, q_heads: int, value_dim: int, world: int, rank: int, device,
                 group=None, _local_ptrs=None):
        from . import _lib

        if q_heads % world:
            raise ValueError(f"q_heads {q_heads} is not a multiple of the world size {world}")
        self.batch, self.q_heads, self.value_dim = int(batch), int(q_heads), int(value_dim)
        self._nbytes = int(_lib.lib().plkv_shard_buffer_bytes(batch, q_heads, value_dim))
        super().__init__(1, 1, world, rank, device, group=group, _local_ptrs=_local_ptrs)

    def _buffer_bytes(self) -> int:
        return self._nbytes

    @property
    def heads_per_rank(self) -> int:
        return self.q_heads // self.world

    @classmethod
    def local_group(cls, world: int, batch: int, q_heads: int, value_dim: int, device):
        """`world` exchanges over plain buffers of one device (a single-process
        stand-in for the ranks, for tests): publishes must all precede the
        merges in stream order.  Returns (exchanges, buffers)."""
        import torch

        from . import _lib

        L = _lib.lib()
        nbytes = int(L.plkv_shard_buffer_bytes(batch, q_heads, value_dim))
        bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=device) for _ in range(world)]
        stream = torch.cuda.current_stream(torch.device(device)).cuda_stream
        for b in bufs:
            _lib.check(L.plkv_peer_init_buffer(b.data_ptr(), nbytes, stream),
                       "plkv_peer_init_buffer")
        ptrs = [b.data_ptr() for b in bufs]
        return [cls(batch, q_heads, value_dim, world, r, device, _local_ptrs=ptrs)
                for r in range(world)], bufs

    def publish(self, decode_args) -> None:
        """``decode_args``: the ``LatentDecodeArgs`` of the rank's partial pass
        (its workspace holds the work items' results)."""
        import ctypes

        L = self._lib.lib()
        self._lib.check(L.plkv_shard_publish(ctypes.byref(decode_args), self.bufs.data_ptr(),
                                             self.world, self.rank, self.ctrl.data_ptr(),
                                             self._stream()), "plkv_shard_publish")

    def merge(self, out, w_v=None, lse_out=None, flags=None):
        import torch

        hpr = self.heads_per_rank
        width = self.value_dim if w_v is None else int(w_v.shape[2])
        if not (isinstance(out, torch.Tensor) and out.is_cuda and out.dtype == torch.float32
                and out.is_contiguous() and out.numel() == self.batch * hpr * width):
            raise TypeError("out must be a contiguous FP32 CUDA tensor of batch x heads/world x "
                            "width")
        L = self._lib.lib()
        self._lib.check(L.plkv_shard_merge(
            self.bufs.data_ptr(), self.world, self.rank, self.ctrl.data_ptr(), self.batch,
            self.q_heads, self.value_dim, None if w_v is None else w_v.data_ptr(),
            0 if w_v is None else int(w_v.shape[2]), out.data_ptr(),
            None if lse_out is None else lse_out.data_ptr(),
            None if flags is None else flags.data_ptr(), self._stream()), "plkv_shard_merge")
        return out
