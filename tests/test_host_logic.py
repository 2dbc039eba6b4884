"""Host-side logic without a GPU: the block-table model keeps the reference's
semantics (block_table.py / test_block_table.py), workloads are seeded and
shaped as specified, and the algorithmic byte model is consistent."""

import numpy as np
import pytest

from conftest import load_reference_fixture


def test_block_table_matches_reference_fixture(pkg):
    for name in ("block_table_seq5_block2.json", "block_table_seq128_block16.json"):
        fx = load_reference_fixture(name)
        t = pkg.PagedBlockTable(fx["block_size"])
        got = t.allocate_token_positions(fx["seq_len"])
        assert t.to_numpy() == fx["logical_blocks"]
        assert [g[0] for g in got] == list(range(fx["seq_len"]))
        for loc in fx["token_locations"]:
            assert t.translate(loc["token"]) == (loc["physical_block"], loc["offset"])
            assert t.slot(loc["token"]) == loc["physical_block"] * fx["block_size"] + loc["offset"]


def test_block_table_errors(pkg):
    with pytest.raises(TypeError):
        pkg.PagedBlockTable(2.0)
    with pytest.raises(ValueError):
        pkg.PagedBlockTable(0)
    t = pkg.PagedBlockTable(2)
    t.allocate_token_positions(3)
    with pytest.raises(IndexError):
        t.translate(3)
    with pytest.raises(ValueError):
        t.translate(-1)
    with pytest.raises(TypeError):
        t.translate(1.0)
    with pytest.raises(ValueError):
        t.allocate_token_positions(0)
    assert pkg.logical_blocks_for_seq_len(5, 2) == 3
    with pytest.raises(ValueError):
        pkg.logical_blocks_for_seq_len(0, 2)


def test_stack_tables(pkg):
    out = pkg.block_table.stack_tables([[2, 0], [3, 1, 5]])
    np.testing.assert_array_equal(out, [[2, 0, -1], [3, 1, 5]])
    assert out.dtype == np.int32


@pytest.mark.parametrize("name", ["tiny", "model_shaped"])
def test_small_workloads_are_deterministic(pkg, name):
    s = pkg.workloads.spec(name)
    a = pkg.workloads.host_inputs(s)
    b = pkg.workloads.host_inputs(s)
    for k, v in a.items():
        if isinstance(v, np.ndarray):
            np.testing.assert_array_equal(v, b[k])


def test_tiny_workload_shape(pkg):
    s = pkg.workloads.spec("tiny")
    x = pkg.workloads.host_inputs(s)
    assert list(x["lens"]) == [7, 13]
    assert x["pool"] == 6
    used = np.concatenate([x["tables"][0, :2], x["tables"][1, :4]])
    assert sorted(used.tolist()) == list(range(6))     # a permutation of 6 physical blocks
    assert x["cache_f16"].shape == (6, 4, 8)
    assert x["w_o"].shape == (64, 64)


@pytest.mark.parametrize("name", ["mla_batch", "write_attend", "long_context"])
def test_large_workload_tables(pkg, name):
    s = pkg.workloads.spec(name)
    lens = pkg.workloads.initial_lens(s)
    tables, pool, first = pkg.workloads.build_tables(s, lens)
    need = (lens.astype(np.int64) + s.steps - 1 + s.block_size - 1) // s.block_size
    used = np.concatenate([tables[b, :need[b]] for b in range(s.batch)])
    assert len(np.unique(used)) == used.size                  # no aliasing
    assert used.min() >= 0 and used.max() < pool
    if s.len_range:
        assert lens.min() >= s.len_range[0] and lens.max() <= s.len_range[1]


@pytest.mark.parametrize("shards", [2, 4, 8])
def test_split_k_shards_partition_every_sequence(pkg, shards):
    s = pkg.workloads.spec("long_context")
    lens = pkg.workloads.initial_lens(s)
    nb = (lens + s.block_size - 1) // s.block_size
    counts = np.zeros_like(nb)
    for r in range(shards):
        tables, pool, first = pkg.workloads.build_tables(s, lens, shards=shards, shard=r)
        c = (tables >= 0).sum(axis=1)
        np.testing.assert_array_equal(first, (nb * r) // shards)
        counts += c
    np.testing.assert_array_equal(counts, nb)


def test_algorithmic_bytes_long_context(pkg):
    s = pkg.workloads.spec("long_context")
    lens = pkg.workloads.initial_lens(s)
    b = pkg.workloads.algorithmic_bytes(s, lens, with_out_proj=False)
    latent = 8 * 131072 * 576 * 2
    assert latent == 1_207_959_552
    assert b - latent == (128 * 512 * 128 * 4 + 8 * 128 * 576 * 4 + 8 * 128 * 128 * 4
                          + 8 * 576 * 6 + 8 * 2048 * 4)


def test_batched_allocation_oracle_matches_block_table(pkg):
    """oracle.np_ref.allocate_token_positions_batch against the reference's
    fixtures and, sequence by sequence, PagedBlockTable with the counter the
    earlier sequences left (block_table.py:26-38)."""
    from oracle.np_ref import allocate_token_positions_batch as alloc

    for name in ("block_table_seq5_block2.json", "block_table_seq128_block16.json"):
        fx = load_reference_fixture(name)
        bs, n = fx["block_size"], fx["seq_len"]
        tables, lens, slots, nb = alloc(np.full((1, 64), -1, np.int32), np.zeros(1, np.int32),
                                        np.array([n], np.int32), 0, bs, 1 << 20)
        assert list(tables[0, :len(fx["logical_blocks"])]) == fx["logical_blocks"]
        for loc in fx["token_locations"]:
            assert slots[loc["token"]] == loc["physical_block"] * bs + loc["offset"]
        assert lens[0] == n and nb == len(fx["logical_blocks"])

    rng = np.random.default_rng(3)
    bs, B = 8, 9
    tables = np.full((B, 12), -1, np.int32)
    lens = np.zeros(B, np.int32)
    refs = [None] * B
    nb = 0
    for _ in range(4):                                   # four rounds of uneven appends
        counts = rng.integers(0, 20, B).astype(np.int32)
        tables, lens, slots, nb2 = alloc(tables, lens, counts, nb, bs, 1 << 20)
        k = 0
        for b in range(B):
            if counts[b] == 0:
                continue
            if refs[b] is None:
                refs[b] = pkg.PagedBlockTable(bs, first_physical_block=nb)
            refs[b].next_physical_block = nb             # the shared counter
            got = refs[b].allocate_token_positions(int(counts[b]))
            nb = refs[b].next_physical_block
            assert list(slots[k:k + counts[b]]) == [p * bs + o for _, p, o in got]
            k += counts[b]
            assert list(tables[b, :refs[b].num_blocks]) == refs[b].to_list()
        assert nb == nb2 and k == slots.size
    # pool exhaustion: ids at or past num_physical are not stored, slots are -1
    t2, _, s2, nb3 = alloc(np.full((1, 4), -1, np.int32), np.zeros(1, np.int32),
                           np.array([10], np.int32), 0, 4, 2)
    assert list(t2[0]) == [0, 1, -1, -1] and list(s2[8:]) == [-1, -1] and nb3 == 3
