#!/usr/bin/env python
"""Benchmark of the paged latent-cache decode step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--mode exact|tc] [--impl ours|reference] [--with-wo]
                    [--no-graph] [--grow]

A step is one append + decode pass over the whole batch: one FP32 latent row
per sequence is written into the FP16 cache through its block table (the
same slot every step, so the attended length stays fixed), then the split-K
decode (scores, mask, online softmax, latent context) and the log-sum-exp
combine with the W_uv / W_v projection run; `--with-wo` adds the W_o output
projection.  `--grow` makes every step append a new token per sequence
instead: its position is allocated on the device (block table, length and
pool counter advance there), as in the reference's write-then-attend loop.
The step is recorded once into a CUDA graph and replayed, the NCCL
all-gather of the split-K shards included (`--no-graph` launches it eagerly);
the partial pass's kernel time always comes from CUDA events around it in the
eager steps that precede the replays.  The default workload is the long-context
one (8 sequences of 131072 tokens, absorbed-MLA shapes: 128 heads, latent
512 + 64, block 64).

Metric: achieved HBM TB/s = algorithmic bytes of the step / step time (the
step time is reported as ms_per_step).  With N > 1 (torchrun) each sequence's
blocks are split across the ranks and the per-rank (context, log-sum-exp)
results are all-gathered over NCCL and merged; the time is the max over ranks.

`--impl reference` times the reference's CPU implementation of the path (the
C restatement of crates/plkv-core/src/lib.rs:941-1145 in oracle/, OpenMP over
(sequence, head) on every host core) on a bounded sample of the same workload
and reports the same metric.
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PACKAGE = "latentpagedattention-rs_b200"
METRIC = "paged latent decode µs/step and achieved HBM TB/s vs peak at 1/2/4/8 B200"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
SPLIT_K_WORKLOADS = {"long_context"}      # sequences' blocks split across ranks
BATCH_SHARD_WORKLOADS = {"mla_batch", "write_attend"}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="long_context")
    ap.add_argument("--mode", default="auto", choices=["auto", "exact", "tc"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--with-wo", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="target CPU work of the bounded CPU-baseline sample")
    ap.add_argument("--graph", dest="graph", action="store_true", default=None,
                    help="replay the step from a CUDA graph (default on one GPU; the kernel "
                         "time comes from the eager steps)")
    ap.add_argument("--no-graph", dest="graph", action="store_false")
    ap.add_argument("--grow", action="store_true",
                    help="append a new token per sequence each step (device allocator)")
    ap.add_argument("--path", default="latent", choices=["latent", "fullkv", "materialised"],
                    help="latent: the direct latent decode; fullkv: stored FP16 K/V; "
                         "materialised: K/V rebuilt from the latent pool every step")
    ap.add_argument("--exchange", default="shard", choices=["shard", "peer", "nccl"],
                    help="split-K result exchange: head-sharded merge over peer memory (each "
                         "rank ends with its heads' rows), all heads over peer memory (two "
                         "kernels) or "
                         "NCCL all-gathers and a merge kernel")
    ap.add_argument("--kernel-suite", action="store_true",
                    help="time every kernel of the library on one synthetic case each")
    ap.add_argument("--suite-reps", type=int, default=5,
                    help="timed calls per kernel in --kernel-suite (after up to 2 warm-up calls)")
    ap.add_argument("--suite-only", default="",
                    help="--kernel-suite: run only the operations whose name contains one of "
                         "these comma-separated texts (profiling a kernel on its suite case)")
    ap.add_argument("--seqs", type=int, default=0,
                    help="keep only the first N sequences (small profiling cases)")
    return ap.parse_args()


def profiled_traffic(mode: str, s, toks_local: int) -> int | None:
    """DRAM bytes (read + write) of one partial-pass launch as captured by ncu
    (profiles/latent_partial_<mode>_<workload>.md, line
    `traffic_bytes_per_launch: N` for the full workload), scaled to the tokens
    this rank's launch processes; None when no capture exists."""
    path = os.path.join(ROOT, "profiles", f"latent_partial_{mode}_{s.name}.md")
    try:
        text = open(path, encoding="utf-8").read()
    except OSError:
        return None
    m = re.search(r"^traffic_bytes_per_launch:\s*(\d+)", text, flags=re.M)
    if not m:
        return None
    wl = importlib.import_module(PACKAGE + ".workloads")
    full_tokens = int(np.sum(wl.initial_lens(s), dtype=np.int64))
    return int(int(m.group(1)) * toks_local / max(full_tokens, 1))


def load_peaks() -> tuple[dict, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path, encoding="utf-8") as f:
            return json.load(f), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    QUERY = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            cmd = ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                   "-lms", "100"]
            if self.uuid:
                cmd[1:1] = ["-i", self.uuid]
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path, encoding="utf-8") as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 10:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        busy = [v for v in sm if v > 0.5 * max(sm)] if sm else []
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[6:10]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(busy) if busy else None,
                "sm_max_mhz": float(rows[0][3]) if rows[0][3].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# ---------------------------------------------------------------- helpers

def host_cores() -> int:
    """Host cores this process may run on (torchrun's OMP_NUM_THREADS=1 does
    not limit the CPU baseline: it passes its thread count explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def host_compact(s, x: dict, seqs, lens) -> dict:
    """Host copies of what the CPU path reads for sequences `seqs` (lengths
    `lens`): their blocks gathered into a compact pool with renumbered tables,
    the query and the weights."""
    import torch

    tables = x["tables"].cpu().numpy()
    nbs = [int((int(n) + s.block_size - 1) // s.block_size) for n in lens]
    blocks = np.concatenate([tables[b, :nb] for b, nb in zip(seqs, nbs)]).astype(np.int64)
    out = {"lens": np.asarray(lens, np.int32), "seqs": np.asarray(seqs)}
    local = np.full((len(seqs), max(max(nbs), 1)), -1, np.int32)
    k = 0
    for i, nb in enumerate(nbs):
        local[i, :nb] = np.arange(k, k + nb, dtype=np.int32)
        k += nb
    out["tables"] = local
    sel = torch.as_tensor(blocks, device=x["cache"].device)
    cache = x["cache"][sel].contiguous()
    out["cache_bits"] = cache.view(torch.int16).cpu().numpy().view(np.uint16)
    del cache
    if "k_cache" in x:
        for name in ("k_cache", "v_cache"):
            kv = x[name][sel].contiguous()
            out[name + "_bits"] = kv.view(torch.int16).cpu().numpy().view(np.uint16)
    idx = torch.as_tensor(np.asarray(seqs), device=x["cache"].device)
    if s.absorbed:
        out["q_lat"] = x["q_lat"][idx].cpu().numpy()
    else:
        out["q"] = x["q"][idx].cpu().numpy()
        wk = x["w_k"].cpu().numpy()
        out["w_k_canonical"] = wk.transpose(1, 0, 2).reshape(wk.shape[1], -1)
    wv = x["w_v"].cpu().numpy()
    out["w_v_canonical"] = np.ascontiguousarray(wv.transpose(1, 0, 2).reshape(s.value_dim, -1))
    return out


def cpu_decode(s, h: dict, path: str, threads: int) -> None:
    """The reference's CPU path for the compacted sequences of `h`: the C
    restatement of crates/plkv-core/src/lib.rs:1090-1145 (direct latent
    decode) or lib.rs:1147-1269 (full-KV baseline), OpenMP over (sequence,
    head) on `threads` host cores."""
    from oracle import c_ref

    if path == "fullkv":
        c_ref.fullkv_decode_batch(h["q"], h["k_cache_bits"], h["v_cache_bits"], h["tables"],
                                  h["lens"], s.scale, threads=threads)
        return
    if s.absorbed:
        q_lat = h["q_lat"]
    else:
        q_lat = np.stack([c_ref.project_query(q, h["w_k_canonical"], s.kv_heads)
                          for q in h["q"]])
    c_ref.latent_decode_batch(q_lat, h["cache_bits"], h["tables"], h["lens"], s.block_size,
                              s.scale, s.value_dim, h["w_v_canonical"], s.proj_heads,
                              s.head_dim, threads=threads)


class CpuSample:
    """A bounded sample of the workload for the CPU path: sequence 0 (all
    query heads) cut to its first `tokens` tokens, sized so that one run
    takes about `seconds`.  The work is linear in the tokens attended, so its
    throughput is the full step's; `full_step()` times the whole workload
    once to check that."""

    def __init__(self, s, x: dict, path: str, threads: int, seconds: float):
        self.s, self.x, self.path, self.threads = s, x, path, threads
        self.n0 = int(x["global_lens"][0])
        tokens = min(self.n0, 8 * s.block_size)
        while True:
            h = host_compact(s, x, [0], [tokens])
            t0 = time.perf_counter()
            cpu_decode(s, h, path, threads)
            dt = time.perf_counter() - t0
            if tokens >= self.n0 or dt >= 0.2 * seconds:
                break
            tokens = min(self.n0, tokens * 4)
        want = int(tokens * seconds / max(dt, 1e-6))
        tokens = int(np.clip(want // s.block_size * s.block_size, s.block_size, self.n0))
        self.tokens = tokens
        self.h = host_compact(s, x, [0], [tokens])
        self.tokens_full = int(np.sum(x["global_lens"].astype(np.int64)))
        self.desc = (f"sequence 0, all {s.q_heads} query heads, its first {tokens} of "
                     f"{self.n0} tokens ({tokens / self.tokens_full:.3%} of the step's "
                     f"{self.tokens_full} tokens)")

    def run(self) -> float:
        t0 = time.perf_counter()
        cpu_decode(self.s, self.h, self.path, self.threads)
        return time.perf_counter() - t0

    def full_step(self, limit_s: float, sample_s: float) -> float | None:
        """Seconds of one full step of the workload, or None when the sample
        (`sample_s` per run) predicts more than `limit_s`."""
        if sample_s * self.tokens_full / self.tokens > limit_s:
            return None
        s, x = self.s, self.x
        h = host_compact(s, x, list(range(s.batch)), [int(n) for n in x["global_lens"]])
        t0 = time.perf_counter()
        cpu_decode(s, h, self.path, self.threads)
        return time.perf_counter() - t0


# -------------------------------------------------------------- reference arm

def workload_config(s, args, tokens: int, w_o: bool, algo: int) -> dict:
    """The workload a line measures; identical in both arms."""
    return {"workload": s.name, "path": args.path, "batch": s.batch, "q_heads": s.q_heads,
            "kv_heads": s.kv_heads, "latent_dim": s.latent_dim, "value_dim": s.value_dim,
            "head_dim": s.head_dim, "block_size": s.block_size, "tokens": tokens, "w_o": w_o,
            "l2": ("inputs larger than L2 (no flush)" if algo > 126e6
                   else "inputs smaller than L2")}


def run_reference(args, s, rank: int, world: int):
    """The reference's CPU implementation of the path on the host cores.

    Rank 0 alone runs it (other ranks of a torchrun launch exit), with every
    host core it may use, on the same bounded sample at every N."""
    if rank != 0:
        return
    import torch

    dev = torch.device("cuda:0") if torch.cuda.is_available() else torch.device("cpu")
    from oracle import c_ref

    c_ref.build()
    threads = host_cores()
    wl = importlib.import_module(PACKAGE + ".workloads")
    # Inputs are generated exactly as our arm generates them (device generator).
    x = wl.device_inputs(s, dev, with_out_proj=False, with_fullkv=args.path == "fullkv")
    per_step_target = min(2.5, 60.0 / max(1, args.steps + args.warmup))
    sample = CpuSample(s, x, args.path, threads, per_step_target)
    for _ in range(args.warmup):
        sample.run()
    t_run0 = time.perf_counter()
    per_step = [sample.run() for _ in range(args.steps)]
    timed_s = time.perf_counter() - t_run0
    t = statistics.median(per_step)
    full_s = sample.full_step(limit_s=60.0, sample_s=t)
    del x
    torch.cuda.empty_cache()
    lens = wl.initial_lens(s)
    algo = wl.algorithmic_bytes(s, lens, with_out_proj=args.with_wo, fullkv=args.path == "fullkv")
    frac = sample.tokens / sample.tokens_full
    value = algo * frac / t / 1e12
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t * 1e3, "us_per_step": t * 1e6, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(s, args, int(lens.sum()),
                                      bool(args.with_wo and s.out_dim), algo),
            "run": {"mode": "exact FP32 (CPU)", "path": args.path, "threads": threads},
            "step_is_sample": True,
            "timed_seconds": timed_s,
            "full_step_ms_from_sample": t / frac * 1e3,
            "full_step_ms_measured": None if full_s is None else full_s * 1e3,
            "cpu_baseline": {"value": value, "unit": "TB/s", "cores": threads,
                             "kind": "port", "sample": sample.desc},
            "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    if full_s is not None:
        line["full_step_value_measured"] = algo / full_s / 1e12
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm

def run_ours(args, s, rank: int, world: int):
    import torch
    import torch.distributed as dist

    ops = importlib.import_module(PACKAGE + ".ops")
    wl = importlib.import_module(PACKAGE + ".workloads")
    mg = importlib.import_module(PACKAGE + ".multigpu")
    dl = importlib.import_module(PACKAGE + ".decode_loop")
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    mode = args.mode
    if mode == "auto":
        mode = "tc" if (s.absorbed and ops.tc_available(s)) else "exact"
    split_k = world > 1 and s.name in SPLIT_K_WORKLOADS
    if args.graph is None:
        args.graph = True
    if split_k and args.grow:
        raise SystemExit("--grow: not with the split-K shards of this workload")
    if args.path != "latent" and (s.absorbed or split_k or args.grow):
        raise SystemExit("--path fullkv / materialised: one-GPU GQA workloads with W_k, no --grow")
    D = s.head_dim
    flags = torch.zeros(1, dtype=torch.int32, device=dev)   # device error word of every step
    last = {}                                               # attention-level result of a step
    # --grow: every step allocates one new token per sequence on the device;
    # room for all the steps this run takes (warm-up, eager, graph, e2e).
    # warm-up, eager, graph and end-to-end steps (the latter at least 30), and
    # the parity step
    grow_steps = args.warmup + 3 * args.steps + max(30, args.steps) + 16 if args.grow else 0
    extra_blocks = s.batch * (grow_steps // s.block_size + 2) if args.grow else 0
    x = wl.device_inputs(s, dev, shards=world if split_k else 1, shard=rank if split_k else 0,
                         with_out_proj=args.with_wo, extra_blocks=extra_blocks)
    global_lens = x["global_lens"]
    B = s.batch
    seqs = np.arange(B)
    if world > 1 and not split_k and s.name in BATCH_SHARD_WORKLOADS:
        seqs = np.nonzero(mg.lpt_assign(global_lens, world) == rank)[0]
    sel = torch.as_tensor(seqs, device=dev)
    tables = x["tables"][sel].contiguous()
    lens_host = np.asarray(x["lens"])[seqs].astype(np.int32)
    lens = torch.as_tensor(lens_host, device=dev)
    nb_local = len(seqs)
    q_in = (x["q_lat"] if s.absorbed else x["q"])[sel].contiguous()
    new_rows = x["new_rows"][sel].contiguous()
    # The appended row lands on the last token (same slot every step).
    gpos = global_lens[seqs].astype(np.int64) - 1
    if split_k:
        first, _, _ = mg.split_k_ranges(global_lens, s.block_size, world, rank, s.steps - 1)
        slots = mg.append_slots(gpos, x["tables"].cpu().numpy(), first, s.block_size)
        slots_d = torch.as_tensor(slots, device=dev)
        positions = None
    else:
        positions = torch.as_tensor(gpos.astype(np.int32), device=dev)
    w_o = x.get("w_o")
    # Head-sharded split-K results: W_o row-sharded, this rank keeps the rows
    # of its heads and the partial outputs are summed.  Otherwise W_o is
    # column-sharded: this rank keeps out_dim / world columns.
    shard_x_on = split_k and args.exchange == "shard"
    wo_sharded = w_o is not None and world > 1
    if wo_sharded:
        if args.grow:
            raise SystemExit("--with-wo on several GPUs: not with --grow")
        if shard_x_on:
            hpr_d = s.q_heads // world * D
            w_o = w_o[rank * hpr_d:(rank + 1) * hpr_d].contiguous()
        else:
            c0, c1 = mg.column_range(s.out_dim, world, rank)
            w_o = w_o[:, c0:c1].contiguous()
        x["w_o"] = None
        torch.cuda.empty_cache()
    if args.grow:
        lens0 = lens_host.astype(np.int64) - 1     # tokens stored before the first step
        cap = lens0 + grow_steps
        width = int((cap.max() + s.block_size - 1) // s.block_size)
        keep = (lens0 + s.block_size - 1) // s.block_size
        tab = tables.cpu().numpy()
        t_host = np.full((nb_local, width), -1, np.int32)
        for i in range(nb_local):
            t_host[i, :keep[i]] = tab[i, :keep[i]]
        g_lens = torch.as_tensor(lens0.astype(np.int32), device=dev)
        # new blocks come from the free ids that follow the pre-filled pool
        g_next = torch.tensor([x["pool"]], dtype=torch.int32, device=dev)
        loop = dl.PagedLatentDecodeLoop(
            x["cache"], torch.as_tensor(t_host, device=dev), g_lens, g_next, q_heads=s.q_heads,
            scale=s.scale, max_new_tokens=grow_steps, w_v=x["w_v"], value_dim=s.value_dim,
            w_k=None if s.absorbed else x["w_k"], w_o=w_o, mode=mode, seq_lens_host=lens0)
        loop.q[0].copy_(q_in)
        loop.rows[0].copy_(new_rows)
        q_buf, rows_buf = loop.q[0], loop.rows[0]
        plan = loop.plan
        launches_per_step = loop.launches_per_step

        flags = loop.flags

        def run_step(ev=None, marks=None):
            if ev is not None:
                loop.partial_events = [ev]
            r = loop.step()[0]
            last["ctx"] = loop.ctx[0]
            return r
    elif args.path != "latent":
        # Comparison points on the same shapes: stored FP16 K/V ("fullkv": the
        # step appends K/V rows and decodes them) and K/V rebuilt from the
        # latent pool every step ("materialised": latent append, then K/V of
        # every active token, then the same full-KV decode).
        KV, bs = s.kv_heads, s.block_size
        P = x["cache"].shape[0]
        plan = ops.plan_fullkv(lens_host, bs, KV, device=dev)
        ctx = torch.empty((nb_local, s.q_heads, D), dtype=torch.float32, device=dev)
        fws = torch.empty(int(ops.lib().plkv_fullkv_decode_workspace_size(
            plan.n_items, nb_local, s.q_heads, D)), dtype=torch.uint8, device=dev)
        if args.path == "fullkv":
            kv = wl.fullkv_from_latent(s, x, dev)
            k_cache, v_cache = kv["k_cache"], kv["v_cache"]
            gk = torch.Generator(device=dev)
            gk.manual_seed(s.seed * 1000 + 5)
            k_rows = torch.randn((nb_local, KV, D), generator=gk, device=dev)
            v_rows = torch.randn((nb_local, KV, D), generator=gk, device=dev)
        else:
            k_cache = torch.zeros((P, KV, bs, D), dtype=torch.float16, device=dev)
            v_cache = torch.zeros_like(k_cache)
            tab = tables.cpu().numpy()
            act = np.concatenate([tab[i, np.arange(n) // bs].astype(np.int64) * bs
                                  + np.arange(n) % bs for i, n in enumerate(lens_host)])
            act_slots = torch.as_tensor(act, device=dev)
        out = (torch.empty((nb_local, s.out_dim), dtype=torch.float32, device=dev)
               if w_o is not None else None)
        wo_splits = wo_ws = None
        if w_o is not None:
            wo_splits = ops.default_out_proj_splits(w_o.shape[0], w_o.shape[1], dev)
            wo_ws = torch.empty(max(1, ops.out_proj_workspace_bytes(nb_local, w_o.shape[1],
                                                                    wo_splits)),
                                dtype=torch.uint8, device=dev)
        rec_events = []

        def step(q_src, rows_src, ev=None):
            if args.path == "fullkv":
                ops.kv_append(k_rows, v_rows, k_cache, v_cache, tables, positions=positions,
                              flags=flags)
            else:
                ops.latent_append(rows_src, x["cache"], tables, positions=positions, flags=flags)
                rev = None
                if ev is not None:
                    rev = (torch.cuda.Event(enable_timing=True),
                           torch.cuda.Event(enable_timing=True))
                    rec_events.append(rev)
                    rev[0].record()
                ops.reconstruct_kv(x["cache"], x["w_k"], x["w_v"], slots=act_slots,
                                   block_size=bs, k_out=k_cache, v_out=v_cache, flags=flags)
                if rev is not None:
                    rev[1].record()
            if ev is not None:
                ev[0].record()
            ops.fullkv_decode(q_src, k_cache, v_cache, tables, lens, plan, scale=s.scale,
                              out=ctx, workspace=fws, flags=flags)
            if ev is not None:
                ev[1].record()
            res = ctx
            last["ctx"] = ctx
            if w_o is not None:
                res = ops.out_proj(res.reshape(nb_local, -1), w_o, out=out, k_splits=wo_splits,
                                   workspace=wo_ws)
            return res

        q_buf, rows_buf = q_in, new_rows

        def run_step(ev=None, marks=None):
            return step(q_buf, rows_buf, ev)

        # append, (reconstruction), full-KV partial + combine, W_o GEMM + reduction
        launches_per_step = 3 + (args.path == "materialised") + (2 if w_o is not None else 0)
    else:
        plan = (ops.plan_workers(lens_host, s.block_size, device=dev) if mode == "tc"
                else ops.plan_splits(lens_host, s.block_size, device=dev))
        ctx = torch.empty((nb_local, s.q_heads, D), dtype=torch.float32, device=dev)
        ws = torch.empty(ops.latent_workspace_bytes(plan.n_items, nb_local, s.q_heads,
                                                    s.latent_dim, s.value_dim),
                         dtype=torch.uint8, device=dev)
        want_lse = split_k
        shard_x = (mg.ShardExchange(nb_local, s.q_heads, s.value_dim, world, rank, dev)
                   if shard_x_on else None)
        res_shard = (torch.empty((nb_local, s.q_heads // world, D), dtype=torch.float32,
                                 device=dev) if shard_x is not None else None)
        peer_x = (mg.PeerExchange(nb_local * s.q_heads, D, world, rank, dev)
                  if split_k and args.exchange == "peer" else None)
        merged = (torch.empty((nb_local, s.q_heads, D), dtype=torch.float32, device=dev)
                  if peer_x is not None else None)
        nccl_x = split_k and args.exchange == "nccl"
        gathered_ctx = torch.empty((world, nb_local, s.q_heads, D), dtype=torch.float32,
                                   device=dev) if nccl_x else None
        gathered_lse = torch.empty((world, nb_local, s.q_heads), dtype=torch.float32,
                                   device=dev) if nccl_x else None
        merged_nccl = (torch.empty((nb_local, s.q_heads, D), dtype=torch.float32, device=dev)
                       if nccl_x else None)
        K_o = s.q_heads * D
        max_rows = 0
        if wo_sharded and shard_x is not None:
            out = torch.empty((nb_local, s.out_dim), dtype=torch.float32, device=dev)
        elif wo_sharded:
            # rows projected on every rank: the merged contexts (split-K) or
            # every rank's sequences, gathered into equal padded blocks
            max_rows = (B if split_k else
                        int(np.bincount(mg.lpt_assign(global_lens, world), minlength=world).max()))
            proj_rows = B if split_k else world * max_rows
            g_rows = (None if split_k else
                      torch.zeros((world, max_rows, K_o), dtype=torch.float32, device=dev))
            g_out = torch.empty((world, proj_rows, w_o.shape[1]), dtype=torch.float32, device=dev)
            out = torch.empty((proj_rows, w_o.shape[1]), dtype=torch.float32, device=dev)
        else:
            out = (torch.empty((nb_local, s.out_dim), dtype=torch.float32, device=dev)
                   if w_o is not None else None)
        q_lat_buf = (None if s.absorbed else
                     torch.empty((nb_local, s.q_heads, s.latent_dim), dtype=torch.float32,
                                 device=dev))
        wo_splits = wo_ws = None
        if w_o is not None:
            if mode == "tc":
                # tensor-core mode: W_o on the tensor cores (TF32 operands)
                wo_splits = ops.default_out_proj_tc_splits(w_o.shape[0], w_o.shape[1],
                                                           out.shape[0], dev)
                wo_ws = torch.empty(int(ops.lib().plkv_out_proj_tc_workspace_size(
                    out.shape[0], w_o.shape[1], wo_splits)), dtype=torch.uint8, device=dev)
            else:
                wo_splits = ops.default_out_proj_splits(w_o.shape[0], w_o.shape[1], dev)
                wo_ws = torch.empty(max(1, ops.out_proj_workspace_bytes(
                    out.shape[0], w_o.shape[1], wo_splits)), dtype=torch.uint8, device=dev)

        def project(a, w):
            if mode == "tc":
                return ops.out_proj_tc(a, w, out=out, k_splits=wo_splits, workspace=wo_ws,
                                       flags=flags)
            return ops.out_proj(a, w, out=out, k_splits=wo_splits, workspace=wo_ws)

        def step(q_src, rows_src, ev=None, marks=None):
            def mark(name):
                # phase boundaries of the eager steps (CUDA events on the stream)
                if marks is not None:
                    e = torch.cuda.Event(enable_timing=True)
                    e.record()
                    marks.append((name, e))

            mark("start")
            if split_k:
                ops.latent_append_slots(rows_src, x["cache"], slots_d, flags=flags)
            else:
                ops.latent_append(rows_src, x["cache"], tables, positions=positions, flags=flags)
            mark("append")
            q_lat = q_src if s.absorbed else ops.project_query(q_src, x["w_k"], out=q_lat_buf)
            if not s.absorbed:
                mark("project_query")
            if ev is not None:
                ev[0].record()
            r = ops.latent_decode(q_lat, x["cache"], tables, lens, plan, scale=s.scale,
                                  value_dim=s.value_dim, w_v=x["w_v"], mode=mode, out=ctx,
                                  want_lse=want_lse, workspace=ws, allow_empty=split_k,
                                  flags=flags, phase="partial")
            if ev is not None:
                ev[1].record()
            mark("partial (q staging + decode)")
            if shard_x is not None:
                # head-sharded merge: this rank's heads only, W_uv of those heads
                shard_x.publish(r["args"])
                mark("shard publish")
                res = shard_x.merge(res_shard, w_v=x["w_v"], flags=flags)
                mark("shard merge + W_uv")
                last["ctx"] = res
                if w_o is not None:
                    res = project(res.reshape(nb_local, -1), w_o)
                    mark("W_o (row shard)")
                    dist.all_reduce(res)
                    mark("W_o all-reduce")
                return res
            r = ops.latent_decode(q_lat, x["cache"], tables, lens, plan, scale=s.scale,
                                  value_dim=s.value_dim, w_v=x["w_v"], mode=mode, out=ctx,
                                  want_lse=want_lse, workspace=ws, allow_empty=split_k,
                                  flags=flags, phase="combine")
            mark("combine + W_uv")
            res = ctx
            if split_k and peer_x is not None:
                peer_x.publish(ctx, r["lse"], flags=flags)
                res = peer_x.merge(merged, flags=flags)
                mark("peer exchange")
            elif split_k:
                res = mg.gather_and_merge(ctx, r["lse"], world,
                                          lambda c, l: ops.lse_merge(c, l, out=merged_nccl)[0],
                                          gathered_ctx, gathered_lse)
                mark("NCCL exchange")
            last["ctx"] = res
            if w_o is not None and wo_sharded:
                rows = (res.reshape(B, -1) if split_k else
                        mg.gather_rows(res.reshape(nb_local, -1), world, max_rows,
                                       gathered=g_rows).reshape(-1, K_o))
                res = mg.sharded_out_proj(rows, w_o, world, project, gathered=g_out)
                mark("W_o (sharded)")
            elif w_o is not None:
                res = project(res.reshape(nb_local, -1), w_o)
                mark("W_o")
            return res

        q_buf, rows_buf = q_in, new_rows

        def run_step(ev=None, marks=None):
            return step(q_buf, rows_buf, ev, marks)

        # append, partial pass (+ FP16 query staging in tensor-core mode),
        # combine, query projection, shard merge (peer exchange: publish +
        # merge), W_o GEMM + split reduction
        launches_per_step = (3 + (mode == "tc") + (0 if s.absorbed else 1)
                             + ((2 if peer_x is not None or shard_x is not None else 1)
                                if split_k else 0)
                             - (1 if shard_x is not None else 0)
                             + (2 if w_o is not None else 0))

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[dev.index])
        torch.cuda.synchronize(dev)

    steps_done = 0
    for _ in range(args.warmup):
        run_step()
    steps_done += args.warmup
    barrier()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        uuid = None
    clocks = ClockSampler(uuid) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    barrier()
    # Eager steps, with CUDA events around the partial pass of each one.
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    timed_from = steps_done
    step_marks = [[] for _ in range(args.steps)]
    start.record()
    for i in range(args.steps):
        run_step(kev[i], step_marks[i])
    end.record()
    barrier()
    steps_done += args.steps
    eager_ms = start.elapsed_time(end)
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    # Mean device time of each phase of the eager steps (between consecutive
    # marks); the max over ranks is taken below.
    phase_names = [n for n, _ in step_marks[0][1:]] if step_marks[0] else []
    phase_us = [statistics.mean(m[k][1].elapsed_time(m[k + 1][1]) * 1e3 for m in step_marks)
                for k in range(len(phase_names))]
    elapsed_ms = eager_ms
    stepper = run_step
    graph = None
    if args.graph:
        # The same step recorded once into a CUDA graph and replayed.
        if args.grow:
            loop.capture()

            def stepper():
                r = loop.step()[0]
                last["ctx"] = loop.ctx[0]
                return r
        else:
            # With split-K the step holds the exchange of the shards' (context,
            # lse); every rank captures the same sequence, after the eager
            # steps above have set up the communicator.
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, capture_error_mode="thread_local"):
                g_res = step(q_buf, rows_buf)
            g_ctx = last["ctx"]
            barrier()

            def stepper():
                graph.replay()
                last["ctx"] = g_ctx
                return g_res
        for _ in range(3):
            stepper()
        steps_done += 3
        barrier()
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        timed_from = steps_done
        g0.record()
        for _ in range(args.steps):
            stepper()
        g1.record()
        barrier()
        steps_done += args.steps
        elapsed_ms = g0.elapsed_time(g1)
    clock_info = clocks.stop() if clocks else None
    t = torch.tensor([elapsed_ms, kern_ms, eager_ms] + phase_us, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, kern_ms, eager_ms = float(t[0]), float(t[1]), float(t[2])
    phases = {n: round(float(v), 1) for n, v in zip(phase_names, t[3:].tolist())}
    ms_per_step = elapsed_ms / args.steps
    # Lengths attended in the middle of the timed steps (they grow by one a
    # step with --grow).
    attended = (lens_host.astype(np.int64) + (timed_from + args.steps // 2 if args.grow else 0))
    attended_global = (global_lens.astype(np.int64)
                       + (timed_from + args.steps // 2 if args.grow else 0))

    # End to end with host buffers: every step copies its query and new rows
    # from pinned host memory and reads its result back; the next step's
    # host-to-device copy and this step's device-to-host copy run on a copy
    # stream beside the step.
    e2e = None
    if not args.no_e2e:
        barrier()
        # the first step's host-to-device copy has nothing to overlap (the
        # pipeline fills); enough steps that it does not dominate
        n_e2e = max(30, args.steps)
        e2e_ms, h2d, d2h = e2e_pipelined(stepper, q_buf, rows_buf, n_e2e, dev)
        steps_done += n_e2e + 3
        te = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        hb = torch.tensor([h2d, d2h], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
            dist.all_reduce(hb)
        e2e = {"ms_per_step": float(te[0]), "h2d_bytes_per_step": int(hb[0]),
               "d2h_bytes_per_step": int(hb[1])}

    # Parity of the last step's result against an FP64 restatement of the
    # path (torch, on the device) over the attended rows of sampled
    # sequences, gathered from every rank under split-K.  Outside timing.
    res_last = stepper()
    torch.cuda.synchronize(dev)
    parity = check_parity(s, x, mode, world, rank, dev, split_k, seqs, global_lens,
                          lens_host, tables, last["ctx"], res_last, w_o, wo_sharded,
                          loop if args.grow else None,
                          (k_cache, v_cache) if args.path != "latent" else None,
                          max_rows if (wo_sharded and not split_k) else 0,
                          (rank * (s.q_heads // world), (rank + 1) * (s.q_heads // world))
                          if (args.path == "latent" and not args.grow and shard_x is not None)
                          else None)
    err = torch.tensor([float(int(flags.item()))], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
    err_flags = int(err.item())

    if graph is not None:
        # A graph that holds NCCL calls must be released before the process
        # group is destroyed.
        torch.cuda.synchronize(dev)
        graph.reset()
        graph = None
    if not args.grow and args.path == "latent":
        for ex in (peer_x, shard_x):
            if ex is not None:
                ex.close()
    if rank != 0:
        return None
    peaks, peak_kind = load_peaks()
    algo = wl.algorithmic_bytes(s, attended_global, with_out_proj=w_o is not None,
                                fullkv=args.path == "fullkv")
    value = algo / (ms_per_step * 1e-3) / 1e12
    # Roofline of the dominant kernel (split-K partial pass on rank 0):
    # latent rows attended x L x 2 bytes + query + table entries, per launch.
    toks_local = int(np.sum(attended, dtype=np.int64))
    tables_bytes = int(np.sum((attended + s.block_size - 1) // s.block_size)) * 4
    if args.path == "latent":
        kern_bytes = (toks_local * s.latent_dim * 2 + nb_local * s.q_heads * s.latent_dim * 4
                      + tables_bytes)
        kern_name = f"latent partial ({mode})"
        traffic = profiled_traffic(mode, s, toks_local)
    else:
        # full-KV decode (partial + combine): K and V rows attended + query + tables
        kern_bytes = (toks_local * s.kv_heads * D * 2 * 2 + nb_local * s.q_heads * D * 4
                      + tables_bytes)
        kern_name = "full-KV decode (partial + combine)"
        traffic = None
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    achieved = kern_bytes / (kern_ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "traffic": traffic, "kernel": kern_name,
                "kernel_ms": kern_ms, "bytes_per_launch": kern_bytes,
                "peak_source": f"{peak_kind} hbm_gbs"}
    flops = wl.algorithmic_flops(s, attended, with_out_proj=False)
    if args.path == "latent":
        roofline["achieved_tflops"] = flops / (kern_ms * 1e-3) / 1e12
    path_info = {"path": args.path}
    if args.path == "materialised" and rec_events:
        rec_ms = statistics.mean(a.elapsed_time(b) for a, b in rec_events)
        rec_flops = 2 * toks_local * s.kv_heads * D * (s.latent_dim + s.value_dim)
        path_info.update(reconstruct_ms=rec_ms,
                         reconstruct_tflops_fp32=rec_flops / (rec_ms * 1e-3) / 1e12)
    line = {"metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "us_per_step": ms_per_step * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "f32" if mode == "exact" else "f16",
            "data": "synthetic (seeded, device-generated)",
            "config": workload_config(s, args, int(attended_global.sum()), w_o is not None,
                                      algo),
            "run": {"mode": mode, **path_info, "cuda_graph": bool(args.graph),
                    "ms_per_step_eager": eager_ms / args.steps,
                    "growing": ("one token per sequence allocated on the device each step"
                                if args.grow else "no: the append rewrites the last token"),
                    "exchange": (args.exchange if split_k else None),
                    "parallelism": (f"split-k{world}" if split_k else
                                    (f"dp{world}" if world > 1 else "single")),
                    "work_items": plan.n_items,
                    # device time of each phase of an eager step, max over ranks
                    "phases_us_eager": phases},
            "roofline": roofline, "gpu_launches": launches_per_step * args.steps,
            "clocks": clock_info, "parity": parity, "err_flags": err_flags,
            # persistent cache of the attended tokens: the latent pool against the
            # FP16 K/V pool the same heads would need (memory_model.py)
            "cache_bytes": importlib.import_module(PACKAGE + ".memory_model").cache_bytes_report(
                tokens=int(global_lens.sum()), kv_heads=s.kv_heads, head_dim=D,
                latent_dim=s.latent_dim)}
    if e2e:
        line["e2e"] = {"value": algo / (e2e["ms_per_step"] * 1e-3) / 1e12, "unit": "TB/s",
                       "ms_per_step": e2e["ms_per_step"],
                       "h2d_bytes_per_step": e2e["h2d_bytes_per_step"],
                       "d2h_bytes_per_step": e2e["d2h_bytes_per_step"],
                       "copies": "pinned host buffers; the next step's H2D and this step's "
                                 "D2H overlap the step on a copy stream"}
    if world == 1 and not args.no_cpu_baseline:
        from oracle import c_ref

        c_ref.build()
        threads = host_cores()
        xs = dict(x)
        xs["global_lens"] = global_lens
        if args.path == "fullkv":
            xs["k_cache"], xs["v_cache"] = k_cache, v_cache
        sample = CpuSample(s, xs, "fullkv" if args.path == "fullkv" else "latent", threads,
                           min(10.0, args.cpu_seconds))
        t_cpu = statistics.median(sample.run() for _ in range(2))
        frac = sample.tokens / sample.tokens_full
        line["cpu_baseline"] = {"value": algo * frac / t_cpu / 1e12, "unit": "TB/s",
                                "cores": threads, "kind": "port", "sample": sample.desc,
                                "full_step_ms_from_sample": t_cpu / frac * 1e3}
    return line


def e2e_pipelined(stepper, q_dst, rows_dst, n_steps: int, dev):
    """Times `n_steps` steps end to end: each step's query and new rows come
    from pinned host memory and its result goes back to pinned host memory.
    The inputs are double-buffered on the device, so step i+1's host-to-device
    copy and step i's device-to-host copy run on a copy stream while step i
    computes; the step copies its staged inputs into the static buffers it
    reads.  Returns (ms per step, H2D bytes, D2H bytes per step)."""
    import torch

    comp = torch.cuda.current_stream(dev)
    cs = torch.cuda.Stream(dev)
    q_host = [q_dst.cpu().pin_memory() for _ in range(2)]
    r_host = [rows_dst.cpu().pin_memory() for _ in range(2)]
    q_stage = [torch.empty_like(q_dst) for _ in range(2)]
    r_stage = [torch.empty_like(rows_dst) for _ in range(2)]
    res0 = stepper()
    res_stage = [torch.empty_like(res0) for _ in range(2)]
    res_host = [torch.empty(tuple(res0.shape), dtype=res0.dtype).pin_memory() for _ in range(2)]
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    out_ready = [torch.cuda.Event() for _ in range(2)]
    d2h_done = [torch.cuda.Event() for _ in range(2)]

    def h2d(k):
        with torch.cuda.stream(cs):
            q_stage[k].copy_(q_host[k], non_blocking=True)
            r_stage[k].copy_(r_host[k], non_blocking=True)
            h2d_done[k].record(cs)

    def run(n):
        cs.wait_stream(comp)
        h2d(0)
        for i in range(n):
            k = i & 1
            if i + 1 < n:
                if i >= 1:
                    cs.wait_event(consumed[1 - k])   # step i-1 has read that stage
                h2d(1 - k)
            comp.wait_event(h2d_done[k])
            q_dst.copy_(q_stage[k], non_blocking=True)
            rows_dst.copy_(r_stage[k], non_blocking=True)
            consumed[k].record(comp)
            res = stepper()
            if i >= 2:
                comp.wait_event(d2h_done[k])         # step i-2's result has left that stage
            res_stage[k].copy_(res, non_blocking=True)
            out_ready[k].record(comp)
            cs.wait_event(out_ready[k])
            with torch.cuda.stream(cs):
                res_host[k].copy_(res_stage[k], non_blocking=True)
                d2h_done[k].record(cs)
        comp.wait_stream(cs)

    run(2)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    run(n_steps)
    e1.record(comp)
    torch.cuda.synchronize(dev)
    h2d_bytes = q_dst.numel() * q_dst.element_size() + rows_dst.numel() * rows_dst.element_size()
    d2h_bytes = res0.numel() * res0.element_size()
    return e0.elapsed_time(e1) / n_steps, h2d_bytes, d2h_bytes


def _ref_latent_ctx(s, q_lat64, rows16, w_v):
    """FP64 restatement of the direct latent decode of one sequence
    (attention_ref.py:617-648): scores of the attended rows, softmax,
    latent context, per-head value projection."""
    import torch

    r = rows16.double()
    sc = (q_lat64 @ r.T) * s.scale
    p = torch.softmax(sc, dim=1)
    c = p @ r[:, :s.value_dim]
    w = w_v.double()
    group = s.q_heads // w.shape[0]
    if group > 1:
        w = w.repeat_interleave(group, dim=0)
    return torch.einsum("hl,hld->hd", c, w)


def _ref_fullkv_ctx(s, q64, k16, v16):
    """FP64 restatement of the full-KV paged GQA decode of one sequence
    (lib.rs:1147-1269): k16 / v16 token-major [n, KV, D]."""
    import torch

    KV, D = k16.shape[1], k16.shape[2]
    G = s.q_heads // KV
    q = q64.view(KV, G, D)
    sc = torch.einsum("kgd,tkd->kgt", q, k16.double()) * s.scale
    p = torch.softmax(sc, dim=2)
    return torch.einsum("kgt,tkd->kgd", p, v16.double()).reshape(s.q_heads, D)


def check_parity(s, x, mode, world, rank, dev, split_k, seqs, global_lens, lens_host,
                 tables, ctx_res, res, w_o, wo_sharded, loop, kv, max_rows, head_range=None):
    """Normwise relative error max|a - e| / max|e| of sampled sequences'
    results against the FP64 restatement; max over ranks."""
    import torch
    import torch.distributed as dist

    mg = importlib.import_module(PACKAGE + ".multigpu")
    tol = 2e-3 if mode == "tc" else 1e-5
    bs = s.block_size
    cur_tables = loop.tables if loop is not None else tables
    cur_lens = (loop.seq_lens.cpu().numpy() if loop is not None else lens_host).astype(np.int64)
    errs, errs_wo, checked = [], [], []
    if split_k:
        # every rank holds a range of every sequence's blocks: gather them
        counts = np.stack([mg.split_k_ranges(global_lens, bs, world, r, s.steps - 1)[1]
                           for r in range(world)])                 # [world, B]
        sample = sorted({0, s.batch - 1})
    else:
        sample = sorted({0, len(seqs) - 1}) if len(seqs) else []
    for i in sample:
        if split_k:
            cnt = counts[:, i]
            mx = int(cnt.max())
            send = torch.zeros((mx, bs, s.latent_dim), dtype=torch.float16, device=dev)
            mine = int(cnt[rank])
            if mine:
                send[:mine] = x["cache"][tables[i, :mine].long()]
            got = torch.empty((world, mx, bs, s.latent_dim), dtype=torch.float16, device=dev)
            dist.all_gather_into_tensor(got, send)
            rows = torch.cat([got[r, :int(cnt[r])] for r in range(world)]).reshape(-1, s.latent_dim)
            n = int(global_lens[i])
            b_global = i
        else:
            n = int(cur_lens[i])
            nb = (n + bs - 1) // bs
            blk = cur_tables[i, :nb].long()
            b_global = int(seqs[i])
            if kv is None:
                rows = x["cache"][blk].reshape(-1, s.latent_dim)
        if kv is not None:
            kc, vc = kv
            k16 = kc[blk].permute(0, 2, 1, 3).reshape(-1, s.kv_heads, s.head_dim)[:n]
            v16 = vc[blk].permute(0, 2, 1, 3).reshape(-1, s.kv_heads, s.head_dim)[:n]
            q_src = (loop.q[0] if loop is not None else x["q"][torch.as_tensor(seqs, device=dev)])
            ref = _ref_fullkv_ctx(s, q_src[i].double(), k16, v16)
        else:
            rows = rows[:n]
            if s.absorbed:
                q_src = loop.q[0] if loop is not None else x["q_lat"]
                q64 = q_src[i if loop is not None else b_global].double()
            else:
                q_src = loop.q[0] if loop is not None else x["q"]
                wk = x["w_k"].double().repeat_interleave(s.q_heads // s.kv_heads, dim=0)
                q64 = torch.einsum("hd,hld->hl",
                                   q_src[i if loop is not None else b_global].double(), wk)
            ref = _ref_latent_ctx(s, q64, rows, x["w_v"])
        got_ctx = ctx_res[i].double()
        if head_range is not None:
            # this rank holds the merged rows of its heads only
            h0, h1 = head_range
            errs.append(float((got_ctx - ref[h0:h1]).abs().max() / ref.abs().max()))
        else:
            errs.append(float((got_ctx - ref).abs().max() / ref.abs().max()))
        checked.append(int(b_global))
        if w_o is not None and head_range is not None:
            # W_o row-sharded by heads: the reference output is the sum of the
            # ranks' partial products
            ref_out = ref[h0:h1].reshape(1, -1) @ w_o.double()
            dist.all_reduce(ref_out)
            errs_wo.append(float((res[i].double() - ref_out[0]).abs().max()
                                 / ref_out.abs().max()))
        elif w_o is not None:
            ref_out = ref.reshape(1, -1) @ w_o.double()
            if wo_sharded:
                row = i if split_k else rank * max_rows + i
                got_out = res[rank, row].double()
            else:
                got_out = res[i].double()
            errs_wo.append(float((got_out - ref_out[0]).abs().max() / ref_out.abs().max()))
    e = torch.tensor([max(errs, default=0.0), max(errs_wo, default=0.0)], dtype=torch.float64,
                     device=dev)
    if world > 1:
        dist.all_reduce(e, op=dist.ReduceOp.MAX)
    out = {"ref": "FP64 restatement of the path (torch) over the attended rows"
                  + (", gathered from every rank" if split_k else ""),
           "sequences": checked, "max_rel_err": float(e[0]), "tol": tol,
           "ok": bool(float(e[0]) <= tol)}
    if w_o is not None:
        out["w_o_max_rel_err"] = float(e[1])
        out["ok"] = out["ok"] and float(e[1]) <= tol
    return out


def run_kernel_suite(args) -> dict:
    """Every kernel of the library on one synthetic case each, sized so that
    its inputs exceed the 126 MB L2 where the operation is bandwidth-bound:
    CUDA-event time per call (mean of 5 after 2 warm-up calls), algorithmic
    bytes per call (what the operation must read and write at minimum) and
    the achieved fraction of the measured HBM bandwidth.  Run under ncu
    (``-k regex:plkv|tc::``) it gives each kernel's DRAM traffic."""
    import torch

    ops = importlib.import_module(PACKAGE + ".ops")
    wl = importlib.import_module(PACKAGE + ".workloads")
    mg = importlib.import_module(PACKAGE + ".multigpu")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(20260710)
    peaks, peak_kind = load_peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    f32 = dict(dtype=torch.float32, device=dev)

    def randn(*shape, scale=1.0):
        return torch.randn(shape, generator=g, device=dev) * scale

    def paged(B, n_tok, bs, per_row_elems, rng_seed):
        """Block tables of B sequences of n_tok tokens drawn from a permuted pool."""
        nb = (n_tok + bs - 1) // bs
        perm = np.random.default_rng(rng_seed).permutation(B * nb).astype(np.int32)
        tables = torch.as_tensor(perm.reshape(B, nb), device=dev)
        lens_h = np.full(B, n_tok, np.int32)
        return tables, lens_h, torch.as_tensor(lens_h, device=dev), B * nb

    results = []

    reps = max(1, args.suite_reps)

    def timed(name, kernels, fn, nbytes, note="", per_call=1):
        """Device time per call: `reps` calls recorded into a CUDA graph and
        replayed (launched from Python, calls of a few microseconds would
        time the host); eager when the call cannot be captured."""
        if args.suite_only and not any(w in name for w in args.suite_only.split(",")):
            return
        for _ in range(min(2, reps)):
            fn()
        torch.cuda.synchronize(dev)
        graph, how = None, "graph"
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(reps):
                    fn()
            graph.replay()
            torch.cuda.synchronize(dev)
        except Exception:
            graph, how = None, "eager"
            torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if graph is not None:
            graph.replay()
        else:
            for _ in range(reps):
                fn()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / reps / per_call
        gbs = nbytes / (ms * 1e-3) / 1e9
        results.append({"op": name, "kernels": kernels, "us": round(ms * 1e3, 2),
                        "algorithmic_bytes": int(nbytes), "GB/s": round(gbs, 1),
                        "frac_of_hbm": round(gbs / hbm, 3), "timing": how, "note": note})
        del graph

    # FP32 -> FP16 storage conversion
    x = randn(64 << 20)
    y = torch.empty(64 << 20, dtype=torch.int16, device=dev)
    timed("quantize_f16 (64 Mi values)", ["quantize_f16_kernel"],
          lambda: ops.lib().plkv_quantize_f16(x.data_ptr(), y.data_ptr(), x.numel(), None,
                                              torch.cuda.current_stream(dev).cuda_stream),
          x.numel() * 6)
    del x, y
    # latent append through the block tables (long-context batch) and by slot
    L = 576
    tables, lens_h, lens, P = paged(8, 131072, 64, L, 1)
    cache = torch.zeros((P, 64, L), dtype=torch.float16, device=dev)
    rows = randn(8, L)
    pos = torch.as_tensor(lens_h - 1, device=dev)
    timed("latent_append (8 rows, block tables)", ["latent_append_kernel"],
          lambda: ops.latent_append(rows, cache, tables, positions=pos), 8 * L * 6 + 8 * 4,
          "launch-bound: 8 rows")
    n_rows = 65536
    slots = torch.as_tensor(np.random.default_rng(2).permutation(P * 64)[:n_rows].astype(np.int64),
                            device=dev)
    rows_many = randn(n_rows, L)
    timed("latent_append_slots (65536 rows)", ["latent_append_slots_kernel"],
          lambda: ops.latent_append_slots(rows_many, cache, slots), n_rows * (L * 6 + 8))
    del rows_many
    # tensor-core decode of two long sequences: FP16 query staging, partial pass, combine
    s = wl.spec("long_context")
    t2 = tables[:2].contiguous()
    l2 = lens[:2].contiguous()
    q_lat = randn(2, 128, L)
    w_uv = randn(128, 512, 128, scale=1 / math.sqrt(512))
    plan = ops.plan_workers(lens_h[:2], 64, device=dev)
    ws = torch.empty(ops.latent_workspace_bytes(plan.n_items, 2, 128, L, 512), dtype=torch.uint8,
                     device=dev)
    ctx = torch.empty((2, 128, 128), **f32)
    kw = dict(scale=s.scale, value_dim=512, w_v=w_uv, mode="tc", out=ctx, workspace=ws)
    tok = 2 * 131072
    timed("latent decode, tensor-core partial pass (2 x 131072 tokens)",
          ["q_prep_kernel", "latent_partial_tc_kernel"],
          lambda: ops.latent_decode(q_lat, cache, t2, l2, plan, phase="partial", **kw),
          tok * L * 2 + 2 * 128 * L * 4 + 2 * 2048 * 4)
    timed("latent decode, combine + W_uv (2 sequences)", ["merge_rows_kernel", "project_rows_kernel"],
          lambda: ops.latent_decode(q_lat, cache, t2, l2, plan, phase="combine", **kw),
          plan.n_items * 128 * (512 + 2) * 4 + w_uv.numel() * 4 + 2 * 128 * 128 * 4)
    del cache, ws
    # exact FP32 decode of GQA shapes (write-then-attend sizes), latent and full-KV
    B, n_tok, bs, Hq, KV, D, Lg = 64, 4096, 16, 32, 8, 128, 256
    tables, lens_h, lens, P = paged(B, n_tok, bs, Lg, 3)
    cache = (randn(P, bs, Lg)).half()
    qg = randn(B, Hq, D)
    w_k = randn(KV, Lg, D, scale=1 / math.sqrt(D))
    w_v = randn(KV, Lg, D, scale=1 / math.sqrt(Lg))
    qlat_buf = torch.empty((B, Hq, Lg), **f32)
    timed("project_query (64 x 32 heads, L = 256)", ["project_query_kernel"],
          lambda: ops.project_query(qg, w_k, out=qlat_buf),
          qg.numel() * 4 + w_k.numel() * 4 + qlat_buf.numel() * 4)
    plan = ops.plan_splits(lens_h, bs, device=dev)
    ws = torch.empty(ops.latent_workspace_bytes(plan.n_items, B, Hq, Lg, Lg), dtype=torch.uint8,
                     device=dev)
    ctx = torch.empty((B, Hq, D), **f32)
    kw = dict(scale=1 / math.sqrt(D), value_dim=Lg, w_v=w_v, mode="exact", out=ctx, workspace=ws)
    timed("latent decode, exact-mode partial pass (64 x 4096 tokens, GQA, L = 256)",
          ["latent_gqa_tc_kernel"],
          lambda: ops.latent_decode(qlat_buf, cache, tables, lens, plan, phase="partial", **kw),
          B * n_tok * Lg * 2 + B * Hq * Lg * 4,
          "tensor cores, FP16 hi + lo query and probabilities (FP32-accurate)")
    timed("latent decode, exact combine + W_v", ["merge_rows_kernel", "project_rows_kernel"],
          lambda: ops.latent_decode(qlat_buf, cache, tables, lens, plan, phase="combine", **kw),
          plan.n_items * Hq * (Lg + 2) * 4 + w_v.numel() * 4 + ctx.numel() * 4)
    # materialised reconstruction of every active token's K / V, then the full-KV decode
    k16 = torch.zeros((P, KV, bs, D), dtype=torch.float16, device=dev)
    v16 = torch.zeros_like(k16)
    tab = tables.cpu().numpy()
    act = torch.as_tensor(np.concatenate([tab[i, np.arange(n_tok) // bs].astype(np.int64) * bs
                                          + np.arange(n_tok) % bs for i in range(B)]), device=dev)
    n_act = act.numel()
    timed("reconstruct_kv (262144 rows, L = 256 -> 8 x 128, FP16 out)", ["reconstruct_kv_kernel"],
          lambda: ops.reconstruct_kv(cache, w_k, w_v, slots=act, block_size=bs, k_out=k16,
                                     v_out=v16),
          n_act * (Lg * 2 + 8 + 2 * KV * D * 2) + (w_k.numel() + w_v.numel()) * 4,
          "FP32 CUDA-core bound (2 x 256 x 2048 FLOP per row)")
    fplan = ops.plan_fullkv(lens_h, bs, KV, device=dev)
    fws = torch.empty(int(ops.lib().plkv_fullkv_decode_workspace_size(fplan.n_items, B, Hq, D)),
                      dtype=torch.uint8, device=dev)
    timed("full-KV decode (64 x 4096 tokens, 8 KV heads, FP16)",
          ["fullkv_partial_tc_kernel", "merge_rows_kernel"],
          lambda: ops.fullkv_decode(qg, k16, v16, tables, lens, fplan, scale=1 / math.sqrt(D),
                                    out=ctx, workspace=fws),
          B * n_tok * KV * D * 2 * 2 + qg.numel() * 4 + ctx.numel() * 4)
    kr, vr = randn(B, KV, D), randn(B, KV, D)
    posg = torch.as_tensor(lens_h - 1, device=dev)
    timed("kv_append (64 rows)", ["kv_append_kernel"],
          lambda: ops.kv_append(kr, vr, k16, v16, tables, positions=posg),
          B * KV * D * 2 * 6, "launch-bound")
    del cache, k16, v16, fws, ws
    # token allocation for 65536 sequences
    nseq = 65536
    tab_a = torch.full((nseq, 4), -1, dtype=torch.int32, device=dev)
    lens_a = torch.zeros(nseq, dtype=torch.int32, device=dev)
    nb = torch.zeros(1, dtype=torch.int32, device=dev)
    slots_a = torch.empty(nseq, dtype=torch.int64, device=dev)

    def alloc():
        lens_a.zero_()
        ops.allocate_slots(tab_a, lens_a, nb, 1 << 30, 64, slots=slots_a)
    timed("allocate_slots (65536 sequences, one token each)", ["allocate_slots_kernel"], alloc,
          nseq * (4 + 4 + 4 + 8), "one CTA: a scan over the batch (includes a 256 KB memset)")
    # W_o output projection, LSE merge of 8 shards, peer-memory exchange (2 stand-in ranks)
    w_o = randn(16384, 7168, scale=1 / math.sqrt(16384))
    xo = randn(64, 16384)
    oo = torch.empty((64, 7168), **f32)
    timed("out_proj W_o (64 x 16384 x 7168, FP32)", ["out_proj_partial_kernel", "out_proj_reduce_kernel"],
          lambda: ops.out_proj(xo, w_o, out=oo), w_o.numel() * 4 + xo.numel() * 4 + oo.numel() * 4,
          "FP32 CUDA-core bound (15 GFLOP)")
    wo_tc_ws = torch.empty(int(ops.lib().plkv_out_proj_tc_workspace_size(
        64, 7168, ops.default_out_proj_tc_splits(16384, 7168, 64, dev))), dtype=torch.uint8,
        device=dev)
    timed("out_proj_tc W_o (64 x 16384 x 7168, TF32 tensor cores)",
          ["out_proj_tf32_kernel", "out_proj_reduce_kernel"],
          lambda: ops.out_proj_tc(xo, w_o, out=oo, workspace=wo_tc_ws),
          w_o.numel() * 4 + xo.numel() * 4 + oo.numel() * 4)
    del w_o
    cs, ls = randn(8, 1024, 128), randn(8, 1024)
    timed("lse_merge (8 shards x 1024 rows x 128)", ["lse_merge_kernel"],
          lambda: ops.lse_merge(cs, ls), cs.numel() * 4 + ls.numel() * 4 + 1024 * 129 * 4)
    exch, _bufs = mg.PeerExchange.local_group(2, 1024, 128, dev)
    mo = torch.empty((1024, 128), **f32)

    def peer_step():
        exch[0].publish(cs[0].contiguous(), ls[0].contiguous())
        exch[1].publish(cs[1].contiguous(), ls[1].contiguous())
        exch[0].merge(mo)
        exch[1].merge(mo)
    timed("peer exchange: 2 publishes + 2 merges (1024 rows x 128)",
          ["publish_kernel", "merge_kernel"], peer_step, 2 * (1024 * 129 * 4) * 3,
          "one GPU standing in for two ranks")
    for e in exch:
        e.close()
    del exch, _bufs
    # Split-K at 8 GPUs, one rank's share of the long-context step (8 x 16384
    # tokens), with one GPU standing in for the 8 ranks: partial pass, the
    # head-sharded publish of one rank, and the per-rank cost of publish +
    # merge + W_uv of 16 heads (all 8 stand-in ranks' calls / 8).
    W = 8
    tables, lens_h, lens, P = paged(8, 131072 // W, 64, L, 5)
    cache = (randn(P, 64, L, scale=0.5)).half()
    q8 = randn(8, 128, L)
    plan = ops.plan_workers(lens_h, 64, device=dev)
    ws = torch.empty(ops.latent_workspace_bytes(plan.n_items, 8, 128, L, 512), dtype=torch.uint8,
                     device=dev)
    ctx8 = torch.empty((8, 128, 128), **f32)
    kw = dict(scale=s.scale, value_dim=512, w_v=w_uv, mode="tc", out=ctx8, workspace=ws,
              want_lse=True, allow_empty=True)
    tok8 = 8 * (131072 // W)
    timed("split-K rank share at 8 GPUs: tensor-core partial pass (8 x 16384 tokens)",
          ["q_prep_kernel", "latent_partial_tc_kernel"],
          lambda: ops.latent_decode(q8, cache, tables, lens, plan, phase="partial", **kw),
          tok8 * L * 2 + 8 * 128 * L * 4)
    rr = ops.latent_decode(q8, cache, tables, lens, plan, phase="partial", **kw)
    sx, _sb = mg.ShardExchange.local_group(W, 8, 128, 512, dev)
    so = torch.empty((8, 128 // W, 128), **f32)
    item_bytes = plan.n_items * 128 * (512 + 2) * 4
    timed("split-K at 8 GPUs: head-sharded publish of one rank (8 x 128 rows)",
          ["shard_publish_kernel"], lambda: sx[0].publish(rr["args"]),
          item_bytes + 8 * 128 * 516 * 4, "one GPU standing in for the ranks")

    def shard_step():
        for e in sx:
            e.publish(rr["args"])
        for e in sx:
            e.merge(so, w_v=w_uv)
    timed("split-K at 8 GPUs: publish + merge + W_uv of 16 heads, per rank",
          ["shard_publish_kernel", "shard_merge_rows_kernel", "project_rows_kernel"], shard_step,
          item_bytes + 2 * 8 * 128 * 516 * 4 + w_uv.numel() * 4 // W,
          "one GPU standing in for the 8 ranks (no NVLink): all ranks' calls / 8", per_call=W)
    for e in sx:
        e.close()
    return {"kernel_suite": results, "peak_GB/s": hbm, "peak_source": f"{peak_kind} hbm_gbs"}

def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    wl = importlib.import_module(PACKAGE + ".workloads")
    s = wl.spec(args.workload)
    if args.seqs:
        import dataclasses

        s = dataclasses.replace(s, batch=args.seqs, lens=s.lens[:args.seqs])
    if args.impl == "reference":
        run_reference(args, s, rank, world)
        return
    if args.kernel_suite:
        print(json.dumps(run_kernel_suite(args)), flush=True)
        return
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    saved_stdout = None
    if world > 1:
        # Library banners (NCCL prints its version on rank 0) go to stderr, so
        # that rank 0's standard output is the one JSON line.
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    line = None
    try:
        line = run_ours(args, s, rank, world)
    finally:
        if world > 1:
            dist.destroy_process_group()
        if saved_stdout is not None:
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
        if line.get("err_flags") or not line.get("parity", {}).get("ok", True):
            print(f"bench: the step's result failed its checks (device error flags "
                  f"0x{line.get('err_flags', 0):x}, parity {line.get('parity')})", file=sys.stderr)
            sys.exit(3)


if __name__ == "__main__":
    main()
