"""The device-resident decode loop (allocate -> append -> project -> decode ->
combine -> W_o): every step against the oracle, and CUDA-graph replays against
eager steps bit for bit.

Bars: exact mode normwise relative error <= 1e-5 against the FP64-accumulating
oracle on the identical FP16 cache; tensor-core mode <= 2e-3; cache bits,
tables, lengths and the pool counter bit-exact; graph vs eager bit-exact
(same kernels, same plan, same order)."""

import importlib
import math

import numpy as np
import pytest
import torch

from conftest import PACKAGE
from oracle import c_ref
from oracle.np_ref import allocate_token_positions_batch as host_alloc
from tests_support import rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"
EXACT_REL = 1e-5
TC_REL = 2e-3


def _mods():
    return (importlib.import_module(PACKAGE + ".ops"),
            importlib.import_module(PACKAGE + ".decode_loop"))


def _state(rng, B, bs, L, lens, max_blocks, extra_blocks, std=1.0):
    """Pre-filled tables from a permutation of the first blocks of the pool;
    new blocks come from the counter, which starts after them."""
    nb = (lens + bs - 1) // bs
    used = int(nb.sum())
    perm = rng.permutation(used).astype(np.int32)
    tables = np.full((B, max_blocks), -1, np.int32)
    k = 0
    for b in range(B):
        tables[b, :nb[b]] = perm[k:k + nb[b]]
        k += nb[b]
    P = used + extra_blocks
    cache = (rng.standard_normal((P, bs, L), dtype=np.float32) * std).astype(np.float16)
    return tables, cache, used


def _gqa_setup(seed=11, B=6, steps=12):
    rng = np.random.default_rng(seed)
    Hq, KV, D, L, bs, N = 8, 2, 16, 32, 8, 48
    lens = rng.integers(1, 40, B).astype(np.int32)
    tables, cache, used = _state(rng, B, bs, L, lens, 12, 40)
    w_k = (rng.standard_normal((L, KV * D), dtype=np.float32) / np.float32(math.sqrt(D)))
    w_v = (rng.standard_normal((L, KV * D), dtype=np.float32) / np.float32(math.sqrt(L)))
    w_o = (rng.standard_normal((Hq * D, N), dtype=np.float32) / np.float32(math.sqrt(Hq * D)))
    q = rng.standard_normal((steps, B, Hq, D), dtype=np.float32)
    rows = rng.standard_normal((steps, B, L), dtype=np.float32)
    return dict(Hq=Hq, KV=KV, D=D, L=L, bs=bs, lens=lens, tables=tables, cache=cache,
                used=used, w_k=w_k, w_v=w_v, w_o=w_o, q=q, rows=rows, scale=1 / math.sqrt(D))


def _head_major(w, heads, d):
    return np.ascontiguousarray(w.reshape(w.shape[0], heads, d).transpose(1, 0, 2))


def _gqa_loop(dl, c, steps_per_replay=1, max_new=12):
    dev_state = (torch.as_tensor(c["cache"], device=DEV), torch.as_tensor(c["tables"], device=DEV),
                 torch.as_tensor(c["lens"], device=DEV),
                 torch.tensor([c["used"]], dtype=torch.int32, device=DEV))
    loop = dl.PagedLatentDecodeLoop(
        *dev_state, q_heads=c["Hq"], scale=c["scale"], max_new_tokens=max_new,
        w_v=torch.as_tensor(_head_major(c["w_v"], c["KV"], c["D"]), device=DEV),
        w_k=torch.as_tensor(_head_major(c["w_k"], c["KV"], c["D"]), device=DEV),
        w_o=torch.as_tensor(c["w_o"], device=DEV), steps_per_replay=steps_per_replay)
    return loop, dev_state


def test_loop_steps_match_oracle_exact():
    ops, dl = _mods()
    c = _gqa_setup()
    loop, (cache, tables, lens, nb) = _gqa_loop(dl, c)
    B, bs = c["lens"].size, c["bs"]
    h_tables, h_lens, h_nb = c["tables"], c["lens"], c["used"]
    P = c["cache"].shape[0]
    for step in range(12):
        out = loop.step(torch.as_tensor(c["q"][step]), torch.as_tensor(c["rows"][step]))
        torch.cuda.synchronize()
        h_tables, h_lens, slots, h_nb = host_alloc(h_tables, h_lens, np.ones(B, np.int32), h_nb,
                                                   bs, P)
        np.testing.assert_array_equal(tables.cpu().numpy(), h_tables)
        np.testing.assert_array_equal(lens.cpu().numpy(), h_lens)
        assert int(nb.item()) == h_nb
        bits = cache.cpu().numpy().view(np.uint16)
        flat = bits.reshape(-1, c["L"])
        for b in range(B):
            np.testing.assert_array_equal(flat[slots[b]], c_ref.quantize_f16(c["rows"][step, b]))
        q_lat = np.stack([c_ref.project_query(c["q"][step, b], c["w_k"], c["KV"])
                          for b in range(B)])
        ctx = c_ref.latent_decode_batch(q_lat, bits, h_tables, h_lens, bs, c["scale"], c["L"],
                                        c["w_v"], c["KV"], c["D"], acc64=True)
        exp = c_ref.out_proj(ctx.reshape(B, -1), c["w_o"], acc64=True)
        assert rel_err(loop.ctx[0].cpu().numpy(), ctx) <= EXACT_REL
        assert rel_err(out[0].cpu().numpy(), exp) <= EXACT_REL
    loop.check()


@pytest.mark.parametrize("steps_per_replay", [1, 3])
def test_graph_replay_equals_eager_exact(steps_per_replay):
    ops, dl = _mods()
    c = _gqa_setup(seed=12)
    eager, se = _gqa_loop(dl, c)
    graph, sg = _gqa_loop(dl, c, steps_per_replay=steps_per_replay, max_new=12 + steps_per_replay)
    graph.capture()
    S = steps_per_replay
    for r in range(9 // S):
        outs = []
        for i in range(S):
            outs.append(eager.step(torch.as_tensor(c["q"][r * S + i]),
                                   torch.as_tensor(c["rows"][r * S + i])).clone())
        got = graph.step(torch.as_tensor(c["q"][r * S:(r + 1) * S]),
                         torch.as_tensor(c["rows"][r * S:(r + 1) * S]))
        torch.cuda.synchronize()
        for i in range(S):
            assert torch.equal(got[i], outs[i][0]), f"replay {r} step {i}"
    for a, b in zip(se, sg):
        assert torch.equal(a, b)
    graph.check()
    graph.release()


def test_graph_replay_tensor_core_mla():
    """Absorbed MLA shapes in tensor-core mode: graph replays equal eager steps
    bit for bit, and the last step matches the oracle within the TC bar."""
    ops, dl = _mods()
    rng = np.random.default_rng(21)
    B, Hq, L, Lv, D, bs, steps = 3, 128, 576, 512, 128, 64, 5
    lens = np.array([100, 700, 64], np.int32)
    tables, cache, used = _state(rng, B, bs, L, lens, 16, 8, std=0.5)
    w_uv = rng.standard_normal((Hq, Lv, D), dtype=np.float32) / np.float32(math.sqrt(Lv))
    q = rng.standard_normal((steps, B, Hq, L), dtype=np.float32)
    rows = rng.standard_normal((steps, B, L), dtype=np.float32) * np.float32(0.5)
    loops = []
    for _ in range(2):
        st = (torch.as_tensor(cache, device=DEV), torch.as_tensor(tables, device=DEV),
              torch.as_tensor(lens, device=DEV), torch.tensor([used], dtype=torch.int32,
                                                              device=DEV))
        loops.append((dl.PagedLatentDecodeLoop(
            *st, q_heads=Hq, scale=1 / math.sqrt(D), max_new_tokens=steps + 1,
            w_v=torch.as_tensor(w_uv, device=DEV), value_dim=Lv, mode="tc",
            n_workers=4), st))
    (eager, se), (graph, sg) = loops
    graph.capture()
    for i in range(steps):
        a = eager.step(torch.as_tensor(q[i]), torch.as_tensor(rows[i]))[0].clone()
        g = graph.step(torch.as_tensor(q[i]), torch.as_tensor(rows[i]))[0]
        torch.cuda.synchronize()
        assert torch.equal(a, g), f"step {i}"
    for x, y in zip(se, sg):
        assert torch.equal(x, y)
    bits = se[0].cpu().numpy().view(np.uint16)
    h_tables, h_lens = se[1].cpu().numpy(), se[2].cpu().numpy()
    np.testing.assert_array_equal(h_lens, lens + steps)
    w_can = w_uv.transpose(1, 0, 2).reshape(Lv, -1)
    ctx = eager.ctx[0].cpu().numpy()
    for b in range(B):
        for h in (0, 77, 127):
            _, _, _, ec = c_ref.latent_decode_seq(
                q[-1, b], bits, h_tables[b], int(h_lens[b]), int(h_lens[b]), bs, 1 / math.sqrt(D),
                value_dim=Lv, w_v_canonical=w_can, proj_heads=Hq, head_dim=D, heads=(h, h + 1),
                acc64=True, want_intermediates=False)
            assert rel_err(ctx[b, h], ec[h]) <= TC_REL
    eager.check()
    graph.check()
    graph.release()


def test_loop_rejects_short_tables():
    ops, dl = _mods()
    c = _gqa_setup()
    with pytest.raises(ValueError):
        _gqa_loop(dl, c, max_new=1000)
