"""Device-resident multi-step decode over a paged latent pool, replayable as a
CUDA graph.

One step runs entirely on the GPU, stream-ordered, with no host round trip:

1. one new token position per sequence (``plkv_allocate_slots``: the bump
   rule of PagedBlockTable.allocate_token_positions, block_table.py:26-38,
   over the pool's shared block counter);
2. the step's FP32 latent rows stored as FP16 at those slots
   (``plkv_latent_append_slots_f16``; paged_latent_write_fp16_storage_ref,
   cache_ref.py:103-114, one row per sequence);
3. the query projected into the latent space (attention_ref.py:513) unless it
   arrives absorbed;
4. the decode over the grown lengths: split-K partial pass and LSE combine
   with the value projection (lib.rs:1090-1145 per sequence);
5. optionally the W_o output projection.

The split plan is made once, for the lengths the loop can reach (lengths at
construction + ``max_new_tokens``).  Work items past a sequence's current
length are empty (the partial pass writes m = -inf for them and the combine
skips them), so one plan stays valid while the lengths grow on the device.
Every buffer is allocated up front, so ``capture()`` can record
``steps_per_replay`` steps into one CUDA graph and ``step()`` replays it: one
host call for all of their launches.

The loop updates the caller's ``block_tables``, ``seq_lens`` and
``next_block`` tensors in place, as the reference's table grows in place.
Device-side errors (pool exhausted, table too short, non-finite rows) set bits
in ``flags``; ``check()`` reads them.
"""

from __future__ import annotations

import numpy as np
import torch

from . import ops


class PagedLatentDecodeLoop:
    def __init__(self, cache: torch.Tensor, block_tables: torch.Tensor, seq_lens: torch.Tensor,
                 next_block: torch.Tensor, *, q_heads: int, scale: float,
                 max_new_tokens: int, w_v: torch.Tensor | None = None,
                 value_dim: int | None = None, w_k: torch.Tensor | None = None,
                 w_o: torch.Tensor | None = None, mode: str = "exact",
                 steps_per_replay: int = 1, seq_lens_host=None,
                 n_workers: int | None = None) -> None:
        """``cache [P, bs, L]`` FP16; ``block_tables [B, max_blocks]`` int32
        (entries < 0: no block yet); ``seq_lens [B]`` int32 (tokens stored);
        ``next_block [1]`` int32 (the pool's next free block); ``w_k`` head-major
        ``[KV, L, D]`` when the query is not absorbed (then ``q [B, Hq, D]``,
        else ``q_lat [B, Hq, L]``); ``w_v`` head-major ``[proj_heads, Lv, D]``;
        ``w_o [Hq * D, N]``; ``mode`` "exact" or "tc"."""
        ops._need_cuda("cache", cache, torch.float16)
        ops._need_cuda("block_tables", block_tables, torch.int32)
        ops._need_cuda("seq_lens", seq_lens, torch.int32)
        ops._need_cuda("next_block", next_block, torch.int32)
        if max_new_tokens <= 0 or steps_per_replay <= 0:
            raise ValueError("max_new_tokens and steps_per_replay must be > 0")
        if mode not in ("exact", "tc"):
            raise ValueError("mode must be 'exact' or 'tc'")
        dev = cache.device
        P, bs, L = cache.shape
        B = seq_lens.shape[0]
        if block_tables.shape[0] != B:
            raise ValueError("block_tables and seq_lens disagree on the batch")
        lens = np.asarray(seq_lens.cpu() if seq_lens_host is None else seq_lens_host, np.int64)
        cap = lens + max_new_tokens
        if int(cap.max()) > block_tables.shape[1] * bs:
            raise ValueError("block_tables cannot hold max_new_tokens more tokens")
        if int(cap.max()) >= 1 << 31:
            raise ValueError("sequence lengths must stay below 2^31")
        Lv = L if value_dim is None else int(value_dim)
        D_in = L if w_k is None else w_k.shape[2]
        D = w_v.shape[2] if w_v is not None else Lv
        self.cache, self.tables, self.seq_lens, self.next_block = cache, block_tables, seq_lens, next_block
        self.q_heads, self.scale, self.value_dim, self.mode = q_heads, float(scale), Lv, mode
        self.w_k, self.w_v, self.w_o = w_k, w_v, w_o
        self.max_new_tokens = int(max_new_tokens)
        self.steps_per_replay = int(steps_per_replay)
        self.steps_taken = 0
        self.plan = (ops.plan_workers(cap, bs, n_workers=n_workers, device=dev) if mode == "tc"
                     else ops.plan_splits(cap, bs, device=dev))
        S = self.steps_per_replay
        f32 = dict(dtype=torch.float32, device=dev)
        # Static inputs and outputs, one slice per step of a replay.
        self.q = torch.zeros((S, B, q_heads, D_in), **f32)
        self.rows = torch.zeros((S, B, L), **f32)
        self.ctx = torch.zeros((S, B, q_heads, D), **f32)
        self.out = torch.zeros((S, B, w_o.shape[1]), **f32) if w_o is not None else None
        self.q_lat = torch.empty((B, q_heads, L), **f32) if w_k is not None else None
        self.slots = torch.empty(B, dtype=torch.int64, device=dev)
        self.flags = torch.zeros(1, dtype=torch.int32, device=dev)
        self.workspace = torch.empty(
            ops.latent_workspace_bytes(self.plan.n_items, B, q_heads, L, Lv), dtype=torch.uint8,
            device=dev)
        if w_o is not None and mode == "tc":
            # tensor-core mode: W_o on the tensor cores too (TF32 operands)
            self.wo_splits = ops.default_out_proj_tc_splits(w_o.shape[0], w_o.shape[1], B, dev)
            self.wo_workspace = torch.empty(
                int(ops.lib().plkv_out_proj_tc_workspace_size(B, w_o.shape[1], self.wo_splits)),
                dtype=torch.uint8, device=dev)
        elif w_o is not None:
            self.wo_splits = ops.default_out_proj_splits(w_o.shape[0], w_o.shape[1], dev)
            self.wo_workspace = torch.empty(
                max(1, ops.out_proj_workspace_bytes(B, w_o.shape[1], self.wo_splits)),
                dtype=torch.uint8, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        # Optional CUDA events recorded around the decode's partial pass of
        # each step (eager steps only): (start, end) pairs.
        self.partial_events: list | None = None

    # ----------------------------------------------------------- launches
    def _launch_step(self, i: int) -> None:
        P, bs, _ = self.cache.shape
        ops.allocate_slots(self.tables, self.seq_lens, self.next_block, P, bs, slots=self.slots,
                           flags=self.flags)
        ops.latent_append_slots(self.rows[i], self.cache, self.slots, flags=self.flags)
        q_lat = self.q[i] if self.w_k is None else ops.project_query(self.q[i], self.w_k,
                                                                     out=self.q_lat)
        kw = dict(scale=self.scale, value_dim=self.value_dim, w_v=self.w_v, mode=self.mode,
                  out=self.ctx[i], workspace=self.workspace, flags=self.flags)
        ev = self.partial_events.pop(0) if self.partial_events else None
        if ev is not None:
            ev[0].record()
        ops.latent_decode(q_lat, self.cache, self.tables, self.seq_lens, self.plan,
                          phase="partial", **kw)
        if ev is not None:
            ev[1].record()
        ops.latent_decode(q_lat, self.cache, self.tables, self.seq_lens, self.plan,
                          phase="combine", **kw)
        if self.w_o is not None and self.mode == "tc":
            ops.out_proj_tc(self.ctx[i].reshape(self.ctx.shape[1], -1), self.w_o,
                            out=self.out[i], k_splits=self.wo_splits,
                            workspace=self.wo_workspace, flags=self.flags)
        elif self.w_o is not None:
            ops.out_proj(self.ctx[i].reshape(self.ctx.shape[1], -1), self.w_o, out=self.out[i],
                         k_splits=self.wo_splits, workspace=self.wo_workspace)

    def _launch_replay(self) -> None:
        for i in range(self.steps_per_replay):
            self._launch_step(i)

    @property
    def launches_per_step(self) -> int:
        """Kernels of one step: allocation, append, query projection (when not
        absorbed), partial pass (+ FP16 query staging in tensor-core mode),
        combine, W_o (GEMM + split reduction)."""
        return (4 + (self.w_k is not None) + (self.mode == "tc")
                + (2 if self.w_o is not None else 0))

    # ---------------------------------------------------------------- API
    def step(self, q: torch.Tensor | None = None, rows: torch.Tensor | None = None):
        """Advance ``steps_per_replay`` steps.  ``q`` / ``rows`` (shaped like
        the static ``self.q`` / ``self.rows``, host or device) are copied into
        the static inputs first when given.  Returns the step outputs (``out``
        with W_o, else ``ctx``), valid until the next call."""
        if self.steps_taken + self.steps_per_replay > self.max_new_tokens:
            raise RuntimeError(f"the loop was sized for {self.max_new_tokens} new tokens")
        if q is not None:
            self.q.copy_(q.reshape(self.q.shape), non_blocking=True)
        if rows is not None:
            self.rows.copy_(rows.reshape(self.rows.shape), non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._launch_replay()
        self.steps_taken += self.steps_per_replay
        return self.out if self.out is not None else self.ctx

    def capture(self) -> None:
        """Record one replay (``steps_per_replay`` steps) into a CUDA graph.

        The kernels are first run once on the real buffers, so that module
        loading and the one-time setup of the library happen outside the
        capture; the tables, lengths, pool counter and flags are then put back."""
        dev = self.cache.device
        saved = (self.tables.clone(), self.seq_lens.clone(), self.next_block.clone())
        if self.steps_taken + self.steps_per_replay > self.max_new_tokens:
            raise RuntimeError("no room left for the warm-up replay of the capture")
        self._launch_replay()
        self.tables.copy_(saved[0])
        self.seq_lens.copy_(saved[1])
        self.next_block.copy_(saved[2])
        self.flags.zero_()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            self._launch_replay()
        torch.cuda.synchronize(dev)
        self.graph = g

    def release(self) -> None:
        self.graph = None

    def check(self) -> None:
        """Raise the reference's exception for any device error flag (synchronises)."""
        ops.raise_for_flags(int(self.flags.item()), "paged latent decode loop")
