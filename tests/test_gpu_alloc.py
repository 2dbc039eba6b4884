"""Device-side token allocation (plkv_allocate_slots) against the reference's
bump allocator (block_table.py:26-38, mirrored by block_table.PagedBlockTable)
and the oracle's batched, shared-counter form of it."""

import importlib

import numpy as np
import pytest
import torch

from conftest import PACKAGE
from oracle import c_ref
from oracle.np_ref import allocate_token_positions_batch as host_alloc

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ops():
    return importlib.import_module(PACKAGE + ".ops")


def _bt():
    return importlib.import_module(PACKAGE + ".block_table")


def _run(tables, lens, counts, next_block, bs, num_physical):
    ops = _ops()
    t = torch.as_tensor(tables, device=DEV)
    sl = torch.as_tensor(lens, device=DEV)
    nb = torch.tensor([next_block], dtype=torch.int32, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    cnt = None if counts is None else torch.as_tensor(counts, device=DEV)
    n_new = len(lens) if counts is None else int(np.sum(counts))
    slots = ops.allocate_slots(t, sl, nb, num_physical, bs, counts=cnt, n_new=n_new, flags=flags)
    torch.cuda.synchronize()
    return (t.cpu().numpy(), sl.cpu().numpy(), slots.cpu().numpy(), int(nb.item()),
            int(flags.item()))


def test_reference_case_block_size_4():
    """tests/test_block_table.py:5-13 of the reference: six tokens, block size 4."""
    ref = _bt().PagedBlockTable(4)
    alloc = ref.allocate_token_positions(6)
    tables = np.full((1, 8), -1, np.int32)
    t, sl, slots, nb, flags = _run(tables, np.zeros(1, np.int32), np.array([6], np.int32), 0, 4,
                                   64)
    assert flags == 0
    assert [s for s in slots] == [blk * 4 + off for _, blk, off in alloc]
    assert list(t[0, :2]) == ref.to_list() and np.all(t[0, 2:] == -1)
    assert sl[0] == 6 and nb == ref.next_physical_block == 2
    assert alloc[4] == (4, 1, 0)


def test_one_token_per_step_matches_reference_per_sequence():
    """A single sequence decoding step by step gets the reference's blocks."""
    ref = _bt().PagedBlockTable(16)
    tables = np.full((1, 16), -1, np.int32)
    lens = np.zeros(1, np.int32)
    nb = 0
    for _ in range(40):
        (pos, blk, off), = ref.allocate_token_positions(1)
        tables, lens, slots, nb, flags = _run(tables, lens, None, nb, 16, 1000)
        assert flags == 0 and slots[0] == blk * 16 + off and lens[0] == pos + 1
    assert nb == ref.next_physical_block


@pytest.mark.parametrize("seed,bs", [(1, 16), (2, 64), (3, 32)])
def test_batched_allocation_matches_host_rule(seed, bs):
    rng = np.random.default_rng(seed)
    B, max_blocks = 1500, 40          # more than one 1024-sequence chunk
    lens = rng.integers(0, bs * 30, B).astype(np.int32)
    tables = np.full((B, max_blocks), -1, np.int32)
    pre = 100000
    for b in range(B):                # blocks of existing tokens: ids far from the counter
        n = (lens[b] + bs - 1) // bs
        tables[b, :n] = pre + np.arange(n)
        pre += n
    counts = rng.integers(0, 3 * bs, B).astype(np.int32)
    counts[::7] = 0
    counts[::11] = 1
    num_physical = 10 ** 7
    exp = host_alloc(tables, lens, counts, 5, bs, num_physical)
    got = _run(tables, lens, counts, 5, bs, num_physical)
    assert got[4] == 0
    np.testing.assert_array_equal(got[0], exp[0])
    np.testing.assert_array_equal(got[1], exp[1])
    np.testing.assert_array_equal(got[2], exp[2])
    assert got[3] == exp[3]


def test_pool_exhaustion_and_table_end_are_flagged():
    tables = np.full((3, 2), -1, np.int32)
    lens = np.array([0, 0, 7], np.int32)
    counts = np.array([5, 4, 2], np.int32)
    exp = host_alloc(tables, lens, counts, 0, 4, 3)
    t, sl, slots, nb, flags = _run(tables, lens, counts, 0, 4, 3)
    np.testing.assert_array_equal(slots, exp[2])
    assert (slots == -1).any() and flags != 0
    np.testing.assert_array_equal(t, exp[0])


def test_allocate_then_append_writes_the_new_rows():
    ops = _ops()
    rng = np.random.default_rng(9)
    B, bs, L, P = 5, 8, 16, 64
    lens = np.array([0, 3, 8, 15, 1], np.int32)
    tables = np.full((B, 6), -1, np.int32)
    perm = rng.permutation(np.arange(32, P)).astype(np.int32)
    k = 0
    for b in range(B):
        n = (lens[b] + bs - 1) // bs
        tables[b, :n] = perm[k:k + n]
        k += n
    cache = torch.zeros((P, bs, L), dtype=torch.float16, device=DEV)
    t = torch.as_tensor(tables, device=DEV)
    sl = torch.as_tensor(lens, device=DEV)
    nb = torch.tensor([0], dtype=torch.int32, device=DEV)
    rows = rng.standard_normal((B, L)).astype(np.float32)
    slots = ops.allocate_slots(t, sl, nb, P, bs)
    ops.latent_append_slots(torch.as_tensor(rows, device=DEV), cache, slots)
    torch.cuda.synchronize()
    flat = cache.view(-1, L).cpu().numpy().view(np.uint16)
    exp_t, exp_l, exp_slots, _ = host_alloc(tables, lens, np.ones(B, np.int32), 0, bs, P)
    for b in range(B):
        np.testing.assert_array_equal(flat[exp_slots[b]], c_ref.quantize_f16(rows[b]))
    np.testing.assert_array_equal(sl.cpu().numpy(), exp_l)
