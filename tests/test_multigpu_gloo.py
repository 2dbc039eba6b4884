"""Multi-GPU host logic on CPU: world-size-2 ``gloo`` process groups.

Each rank decodes only its split-K share of every sequence (with the FP64
oracle standing in for the CUDA kernel), the shares are all-gathered and
LSE-merged through ``multigpu.gather_and_merge``, and the merged context must
equal the oracle's decode of the whole sequences.  Also checks sequence
sharding (LPT) and the slot of the appended row on the owning rank.
"""

import importlib
import json
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import PACKAGE, ROOT
from oracle import np_ref


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    rng = np.random.default_rng(99)
    B, Hq, L, Lv, D, bs = 3, 8, 64, 48, 16, 8
    lens = np.array([37, 64, 5], np.int32)
    nb = (lens + bs - 1) // bs
    P = int(nb.sum()) + 2
    perm = rng.permutation(P).astype(np.int32)
    tables = np.full((B, nb.max()), -1, np.int32)
    k = 0
    for b in range(B):
        tables[b, :nb[b]] = perm[k:k + nb[b]]
        k += nb[b]
    cache = (rng.standard_normal((P, bs, L)) * 0.7).astype(np.float16)
    q_lat = rng.standard_normal((B, Hq, L)).astype(np.float32)
    w = (rng.standard_normal((Hq, Lv, D)) / math.sqrt(Lv)).astype(np.float32)
    return dict(B=B, Hq=Hq, L=L, Lv=Lv, D=D, bs=bs, lens=lens, tables=tables, cache=cache,
                q_lat=q_lat, w=w, scale=0.25)


def _merge_f64(ctx, lse):
    m = lse.max(dim=0).values
    wts = torch.where(torch.isinf(lse), torch.zeros_like(lse), torch.exp(lse - m))
    num = (wts[..., None] * ctx).sum(dim=0)
    den = wts.sum(dim=0)
    return num / den[..., None]


def _worker(rank, world, port, out_path):
    import sys

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mg = importlib.import_module(PACKAGE + ".multigpu")
        p = _problem()
        first, count, local = mg.split_k_ranges(p["lens"], p["bs"], world, rank)
        tables = np.full_like(p["tables"], -1)
        for b in range(p["B"]):
            tables[b, :count[b]] = p["tables"][b, first[b]:first[b] + count[b]]
        ctx = np.zeros((p["B"], p["Hq"], p["D"]))
        lse = np.full((p["B"], p["Hq"]), -np.inf)
        for b in range(p["B"]):
            if local[b] == 0:
                continue
            s, _, _, c = np_ref.latent_decode_batch_f64(
                p["q_lat"][b:b + 1], p["cache"], tables[b:b + 1], local[b:b + 1], p["bs"],
                p["Lv"], p["scale"], w_v_head_major=p["w"], group=1)
            ctx[b] = c[0]
            sc = s[0]
            mx = sc.max(axis=1)
            lse[b] = mx + np.log(np.exp(sc - mx[:, None]).sum(axis=1))
        merged = mg.gather_and_merge(torch.as_tensor(ctx), torch.as_tensor(lse), world, _merge_f64)
        # Slot of the appended row (position len-1) exists on exactly one rank.
        slots = mg.append_slots(p["lens"] - 1, tables, first, p["bs"])
        owned = torch.as_tensor((slots >= 0).astype(np.int64))
        dist.all_reduce(owned)
        if rank == 0:
            _, _, _, full = np_ref.latent_decode_batch_f64(
                p["q_lat"], p["cache"], p["tables"], p["lens"], p["bs"], p["Lv"], p["scale"],
                w_v_head_major=p["w"], group=1)
            err = float(np.max(np.abs(merged.numpy() - full)) / np.max(np.abs(full)))
            with open(out_path, "w") as f:
                json.dump({"err": err, "owned": owned.tolist(),
                           "local_total": int(dist.get_world_size())}, f)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_split_k_gather_merge_over_gloo(tmp_path, world):
    out = tmp_path / "result.json"
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(out))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    res = json.loads(out.read_text())
    assert res["err"] <= 1e-12
    assert res["owned"] == [1, 1, 1]


def test_lpt_assign_balances_tokens(pkg):
    mg = importlib.import_module(PACKAGE + ".multigpu")
    lens = pkg.workloads.initial_lens(pkg.workloads.spec("mla_batch"))
    for world in (2, 4, 8):
        owner = mg.lpt_assign(lens, world)
        load = np.bincount(owner, weights=lens, minlength=world)
        assert set(owner.tolist()) == set(range(world))
        assert load.max() - load.min() <= lens.max()
        assert load.max() / load.mean() < 1.1


def test_split_k_ranges_cover_each_sequence(pkg):
    mg = importlib.import_module(PACKAGE + ".multigpu")
    lens = np.array([131072, 5, 0, 700], np.int64)
    for world in (1, 2, 4, 8):
        tot = np.zeros(4, np.int64)
        blocks = np.zeros(4, np.int64)
        for r in range(world):
            first, count, local = mg.split_k_ranges(lens, 64, world, r)
            tot += local
            blocks += count
        np.testing.assert_array_equal(tot, lens)
        np.testing.assert_array_equal(blocks, (lens + 63) // 64)


def _wo_worker(rank, world, port, out_path):
    import sys

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mg = importlib.import_module(PACKAGE + ".multigpu")
        rng = np.random.default_rng(7)
        K, N = 48, 40
        w_full = torch.as_tensor(rng.standard_normal((K, N)))
        c0, c1 = mg.column_range(N, world, rank)
        w_slice = w_full[:, c0:c1].contiguous()
        proj = lambda x, w: x @ w
        # split-K: every rank holds the same merged rows
        x_all = torch.as_tensor(rng.standard_normal((5, K)))
        out_k = mg.assemble_columns(mg.sharded_out_proj(x_all, w_slice, world, proj))
        err_k = float((out_k - x_all @ w_full).abs().max())
        # sequence sharding: rank r holds rows of its own sequences (uneven counts)
        owner = np.array([0, 1, 1, 0, 1, 1, 1])
        rows = torch.as_tensor(rng.standard_normal((owner.size, K)))
        mine = rows[torch.as_tensor(np.nonzero(owner == rank)[0])]
        max_rows = int(np.bincount(owner, minlength=world).max())
        g = mg.gather_rows(mine, world, max_rows)
        out_s = mg.assemble_columns(mg.sharded_out_proj(g.reshape(-1, K), w_slice, world, proj))
        err_s = 0.0
        for r in range(world):
            idx = np.nonzero(owner == r)[0]
            got = out_s.reshape(world, max_rows, N)[r, :idx.size]
            err_s = max(err_s, float((got - rows[idx] @ w_full).abs().max()))
        if rank == 0:
            with open(out_path, "w") as f:
                json.dump({"err_k": err_k, "err_s": err_s, "cols": [c0, c1]}, f)
    finally:
        dist.destroy_process_group()


def test_wo_column_sharding_over_gloo(tmp_path):
    out = tmp_path / "wo.json"
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_wo_worker, args=(r, 2, port, str(out))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    res = json.loads(out.read_text())
    assert res["err_k"] <= 1e-12 and res["err_s"] <= 1e-12
    assert res["cols"] == [0, 20]


def test_column_range_rejects_uneven(pkg):
    mg = importlib.import_module(PACKAGE + ".multigpu")
    assert mg.column_range(7168, 8, 3) == (2688, 3584)
    with pytest.raises(ValueError):
        mg.column_range(7168, 3, 0)
