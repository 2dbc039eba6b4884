"""Split-K result exchange through peer memory (plkv_peer_publish /
plkv_peer_merge) against the LSE merge rule.

Bars: merged rows within 1e-5 normwise relative error of an FP64 LSE merge of
the same FP32 inputs (FP32 accumulation in the kernel); every rank's result
bitwise identical (same order of sources); the step counter and the slot
parity advance across steps; no error flags.

On one GPU the ranks are stand-ins in one process over plain buffers (all
publishes precede the merges in stream order, so no wait is outstanding).
With two or more GPUs a second test runs one process per GPU over cudaIpc
mappings."""

import importlib
import json
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import PACKAGE, ROOT
from tests_support import rel_err

pytestmark = pytest.mark.gpu


def _mg():
    return importlib.import_module(PACKAGE + ".multigpu")


def _inputs(rng, world, rows, width):
    ctx = rng.standard_normal((world, rows, width)).astype(np.float32)
    lse = (rng.standard_normal((world, rows)) * 3).astype(np.float32)
    lse[rng.random((world, rows)) < 0.2] = -np.inf      # empty shards
    lse[:, 0] = -np.inf                                  # a row empty on every rank
    return ctx, lse


def _expected(ctx, lse):
    c = ctx.astype(np.float64)
    l = lse.astype(np.float64)
    m = l.max(axis=0)
    finite = np.isfinite(m)
    w = np.where(np.isfinite(l), np.exp(l - np.where(finite, m, 0.0)), 0.0)
    den = w.sum(axis=0)
    out = np.where(den[:, None] > 0, (w[..., None] * c).sum(axis=0) / np.maximum(den, 1e-300)[:, None],
                   0.0)
    lse_out = np.where(den > 0, m + np.log(np.maximum(den, 1e-300)), -np.inf)
    return out, lse_out


@pytest.mark.parametrize("world", [1, 2, 3])
def test_local_exchange_matches_lse_merge(world):
    mg = _mg()
    dev = torch.device("cuda")
    rows, width = 37, 24
    exch, bufs = mg.PeerExchange.local_group(world, rows, width, dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    rng = np.random.default_rng(world)
    for step in range(3):
        ctx, lse = _inputs(rng, world, rows, width)
        tc = [torch.as_tensor(ctx[r], device=dev) for r in range(world)]
        tl = [torch.as_tensor(lse[r], device=dev) for r in range(world)]
        for r in range(world):
            exch[r].publish(tc[r], tl[r])
        outs, lses = [], []
        for r in range(world):
            o = torch.empty((rows, width), dtype=torch.float32, device=dev)
            lo = torch.empty(rows, dtype=torch.float32, device=dev)
            exch[r].merge(o, lo, flags=flags)
            outs.append(o)
            lses.append(lo)
        torch.cuda.synchronize()
        exp_out, exp_lse = _expected(ctx, lse)
        for r in range(world):
            assert rel_err(outs[r].cpu().numpy(), exp_out) <= 1e-5, (step, r)
            got_l = lses[r].cpu().numpy()
            fin = np.isfinite(exp_lse)
            np.testing.assert_array_equal(np.isfinite(got_l), fin)
            np.testing.assert_allclose(got_l[fin], exp_lse[fin], rtol=0, atol=1e-5)
            assert torch.equal(outs[r], outs[0])
            assert int(exch[r].ctrl[0].item()) == step + 1
    assert int(flags.item()) == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ipc_worker(rank, world, port, out_path):
    import sys

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    mg = importlib.import_module(PACKAGE + ".multigpu")
    dev = torch.device("cuda", rank)
    rows, width = 300, 128
    ex = mg.PeerExchange(rows, width, world, rank, dev)
    try:
        flags = torch.zeros(1, dtype=torch.int32, device=dev)
        worst = 0.0
        for step in range(4):
            rng = np.random.default_rng(100 + step)      # same inputs on every rank
            ctx, lse = _inputs(rng, world, rows, width)
            o = torch.empty((rows, width), dtype=torch.float32, device=dev)
            ex.publish(torch.as_tensor(ctx[rank], device=dev), torch.as_tensor(lse[rank], device=dev))
            ex.merge(o, flags=flags)
            torch.cuda.synchronize()
            worst = max(worst, rel_err(o.cpu().numpy(), _expected(ctx, lse)[0]))
        res = torch.tensor([worst, float(flags.item())], dtype=torch.float64, device=dev)
        dist.all_reduce(res, op=dist.ReduceOp.MAX)
        if rank == 0:
            with open(out_path, "w") as f:
                json.dump({"err": float(res[0]), "flags": int(res[1])}, f)
    finally:
        ex.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs of one node")
def test_ipc_exchange_two_processes(tmp_path):
    world = min(torch.cuda.device_count(), 4)
    out = tmp_path / "peer.json"
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_ipc_worker, args=(r, world, port, str(out))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    res = json.loads(out.read_text())
    assert res["err"] <= 1e-5 and res["flags"] == 0


def _mla_shards(seed, lens, world, bs=64):
    """Absorbed-MLA inputs and each stand-in rank's share of every sequence's
    blocks (contiguous ranges, as the split-K runner cuts them)."""
    rng = np.random.default_rng(seed)
    L, Lv, Hq, D = 576, 512, 128, 128
    nb = [(n + bs - 1) // bs for n in lens]
    P = sum(nb) + 2
    perm = rng.permutation(P).astype(np.int32)
    tables = np.full((len(lens), max(nb)), -1, np.int32)
    k = 0
    for b, c in enumerate(nb):
        tables[b, :c] = perm[k:k + c]
        k += c
    lens = np.asarray(lens, np.int32)
    shards = []
    nbv = np.asarray(nb)
    for r in range(world):
        lo, hi = nbv * r // world, nbv * (r + 1) // world
        tab = np.full_like(tables, -1)
        local = np.zeros_like(lens)
        for b in range(len(lens)):
            tab[b, :hi[b] - lo[b]] = tables[b, lo[b]:hi[b]]
            local[b] = max(0, min(lens[b], hi[b] * bs) - lo[b] * bs)
        shards.append((tab, local))
    return dict(cache=(rng.standard_normal((P, bs, L), dtype=np.float32) * 0.5).astype(np.float16),
                q_lat=rng.standard_normal((len(lens), Hq, L), dtype=np.float32),
                w_uv=(rng.standard_normal((Hq, Lv, D), dtype=np.float32)
                      / np.float32(np.sqrt(Lv))),
                tables=tables, lens=lens, shards=shards, bs=bs, Lv=Lv, Hq=Hq, D=D)


@pytest.mark.parametrize("world,mode", [(2, "exact"), (4, "exact"), (8, "exact"), (4, "tc")])
def test_head_sharded_merge_equals_unsplit_decode(world, mode):
    """Split-K over `world` stand-in ranks on one GPU: each rank's partial pass
    over its block ranges, head-sharded publish into the owners' buffers,
    merge + W_uv of the owned heads; the heads concatenated equal the
    unsplit decode (exact: 1e-5, tensor-core: 2e-3) over two steps."""
    ops = importlib.import_module(PACKAGE + ".ops")
    mg = _mg()
    dev = torch.device("cuda")
    m = _mla_shards(7 + world, [5000, 1300, 64, 2049], world)
    t = lambda a: torch.as_tensor(np.ascontiguousarray(a), device=dev)
    q, cache, w = t(m["q_lat"]), t(m["cache"]), t(m["w_uv"])
    scale = 1 / np.sqrt(m["D"])
    full = ops.latent_decode(q, cache, t(m["tables"]), t(m["lens"]),
                             ops.plan_splits(m["lens"], m["bs"]), scale=scale, value_dim=m["Lv"],
                             w_v=w, want_lse=True)
    B, Hq, D = len(m["lens"]), m["Hq"], m["D"]
    exch, _bufs = mg.ShardExchange.local_group(world, B, Hq, m["Lv"], dev)
    hpr = Hq // world
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    for _step in range(2):
        parts = []
        for r, (tab, local) in enumerate(m["shards"]):
            plan = (ops.plan_workers(local, m["bs"], n_workers=3) if mode == "tc"
                    else ops.plan_splits(local, m["bs"]))
            rr = ops.latent_decode(q, cache, t(tab), t(local), plan, scale=scale,
                                   value_dim=m["Lv"], w_v=w, mode=mode, allow_empty=True,
                                   flags=flags, phase="partial")
            parts.append(rr)
            exch[r].publish(rr["args"])
        outs, lses = [], []
        for r in range(world):
            o = torch.empty((B, hpr, D), dtype=torch.float32, device=dev)
            ls = torch.empty((B, hpr), dtype=torch.float32, device=dev)
            exch[r].merge(o, w_v=w, lse_out=ls, flags=flags)
            outs.append(o)
            lses.append(ls)
        torch.cuda.synchronize()
        assert int(flags.item()) == 0
        got = torch.cat(outs, dim=1).cpu()
        got_lse = torch.cat(lses, dim=1).cpu()
        tol = 2e-3 if mode == "tc" else 1e-5
        assert rel_err(got, full["ctx"].cpu()) <= tol
        assert rel_err(got_lse, full["lse"].cpu()) <= tol


def _shard_worker(rank, world, port, out_path, mode):
    import sys

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    ops = importlib.import_module(PACKAGE + ".ops")
    mg = importlib.import_module(PACKAGE + ".multigpu")
    dev = torch.device("cuda", rank)
    m = _mla_shards(31 + world, [5000, 1300, 64, 2049, 777], world)   # same inputs on every rank
    t = lambda a: torch.as_tensor(np.ascontiguousarray(a), device=dev)
    q, cache, w = t(m["q_lat"]), t(m["cache"]), t(m["w_uv"])
    scale = 1 / np.sqrt(m["D"])
    full = ops.latent_decode(q, cache, t(m["tables"]), t(m["lens"]),
                             ops.plan_splits(m["lens"], m["bs"]), scale=scale, value_dim=m["Lv"],
                             w_v=w, want_lse=True)
    B, Hq, D = len(m["lens"]), m["Hq"], m["D"]
    hpr = Hq // world
    ex = mg.ShardExchange(B, Hq, m["Lv"], world, rank, dev)
    try:
        flags = torch.zeros(1, dtype=torch.int32, device=dev)
        tab, local = m["shards"][rank]
        worst = 0.0
        for _step in range(3):
            plan = (ops.plan_workers(local, m["bs"], n_workers=5) if mode == "tc"
                    else ops.plan_splits(local, m["bs"]))
            rr = ops.latent_decode(q, cache, t(tab), t(local), plan, scale=scale,
                                   value_dim=m["Lv"], w_v=w, mode=mode, allow_empty=True,
                                   flags=flags, phase="partial")
            ex.publish(rr["args"])
            o = torch.empty((B, hpr, D), dtype=torch.float32, device=dev)
            ls = torch.empty((B, hpr), dtype=torch.float32, device=dev)
            ex.merge(o, w_v=w, lse_out=ls, flags=flags)
            torch.cuda.synchronize()
            heads = slice(rank * hpr, (rank + 1) * hpr)
            worst = max(worst, rel_err(o.cpu(), full["ctx"][:, heads].cpu()),
                        rel_err(ls.cpu(), full["lse"][:, heads].cpu()))
        res = torch.tensor([worst, float(flags.item())], dtype=torch.float64, device=dev)
        dist.all_reduce(res, op=dist.ReduceOp.MAX)
        if rank == 0:
            with open(out_path, "w") as f:
                json.dump({"err": float(res[0]), "flags": int(res[1])}, f)
    finally:
        ex.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs of one node")
@pytest.mark.parametrize("mode", ["exact", "tc"])
def test_shard_exchange_processes(tmp_path, mode):
    """One process per GPU: each rank's partial pass over its block ranges,
    the head-sharded publish into the owners' buffers over peer memory and
    the owner's merge + W_uv equal, head for head, the unsplit decode of the
    whole batch (exact 1e-5, tensor-core 2e-3) over three steps."""
    world = min(torch.cuda.device_count(), 8)
    out = tmp_path / "shard.json"
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_shard_worker, args=(r, world, port, str(out), mode))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    res = json.loads(out.read_text())
    tol = 2e-3 if mode == "tc" else 1e-5
    assert res["err"] <= tol and res["flags"] == 0
