"""C ABI of libplkv_b200.so without a GPU: every symbol of include/plkv_b200.h
is exported and bound, host-side validation returns the reference's error
codes before anything is launched, and the split planner's contract holds."""

import ctypes
import os
import re

import numpy as np
import pytest

from conftest import PACKAGE, ROOT

HEADER = os.path.join(ROOT, "include", "plkv_b200.h")


def _lib_mod():
    import importlib

    return importlib.import_module(PACKAGE + "._lib")


def header_functions() -> list[str]:
    text = open(HEADER, encoding="utf-8").read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(plkv_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    m = _lib_mod()
    lib = m.lib()
    names = header_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(m.SIGNATURES), "ctypes bindings must cover the header exactly"
    assert lib.plkv_version() >= 100
    assert lib.plkv_status_string(3) == b"invalid paged lookup"


def test_status_codes_match_header():
    m = _lib_mod()
    text = open(HEADER, encoding="utf-8").read()
    for name in ("ZERO_VALUE", "ARITHMETIC_OVERFLOW", "INVALID_PAGED_LOOKUP", "NON_FINITE",
                 "FP16_OVERFLOW", "WORKSPACE", "UNSUPPORTED"):
        v = int(re.search(rf"PLKV_ERR_{name} = (\d+)", text).group(1))
        assert getattr(m, f"PLKV_ERR_{name}") == v


def _plan(lens, bs, target, min_blocks=1):
    m = _lib_mod()
    lens = np.ascontiguousarray(np.asarray(lens, np.int32))
    n = ctypes.c_int32(0)
    st = m.lib().plkv_plan_splits(lens.ctypes.data, lens.size, bs, target, min_blocks, None, 0,
                                  None, ctypes.byref(n))
    assert st == m.PLKV_ERR_WORKSPACE
    items = np.zeros((n.value, 4), np.int32)
    begin = np.zeros(lens.size + 1, np.int32)
    st = m.lib().plkv_plan_splits(lens.ctypes.data, lens.size, bs, target, min_blocks,
                                  items.ctypes.data, n.value, begin.ctypes.data, ctypes.byref(n))
    assert st == m.PLKV_OK
    return items, begin


@pytest.mark.parametrize("lens,bs,target", [
    ([7, 13], 4, 296), ([256], 16, 296), ([131072] * 8, 64, 296), ([0, 5, 0], 4, 10),
    (list(np.random.default_rng(3).integers(1024, 32769, 64)), 64, 296), ([1], 1, 1)])
def test_plan_covers_every_block_once(lens, bs, target):
    items, begin = _plan(lens, bs, target)
    assert begin[0] == 0 and begin[-1] == len(items)
    for b, n in enumerate(lens):
        its = items[begin[b]:begin[b + 1]]
        assert len(its) >= 1 and np.all(its[:, 0] == b)
        nb = (n + bs - 1) // bs
        covered = np.concatenate([np.arange(i[1], i[2]) for i in its]) if nb else np.array([])
        np.testing.assert_array_equal(covered, np.arange(nb))
    sizes = items[:, 2] - items[:, 1]
    per = -(-sum((n + bs - 1) // bs for n in lens) // max(target, len(lens)))
    assert sizes.max() <= max(per, 1)


def test_plan_rejects_bad_arguments():
    m = _lib_mod()
    n = ctypes.c_int32(0)
    lens = np.array([-1], np.int32)
    assert m.lib().plkv_plan_splits(lens.ctypes.data, 1, 4, 4, 1, None, 0, None,
                                    ctypes.byref(n)) == m.PLKV_ERR_INVALID_ARGUMENT
    assert m.lib().plkv_plan_splits(lens.ctypes.data, 0, 4, 4, 1, None, 0, None,
                                    ctypes.byref(n)) == m.PLKV_ERR_ZERO_VALUE


def test_host_validation_before_launch():
    """Argument errors return a status without touching the GPU."""
    m = _lib_mod()
    L = m.lib()
    a = m.LatentDecodeArgs(batch=0, q_heads=4, latent_dim=8, value_dim=8, block_size=4,
                           num_physical=6, max_blocks=4, n_items=1)
    assert L.plkv_latent_decode(ctypes.byref(a), None) == m.PLKV_ERR_ZERO_VALUE
    a.batch = 2
    assert L.plkv_latent_decode(ctypes.byref(a), None) == m.PLKV_ERR_INVALID_ARGUMENT
    fake = 256  # never dereferenced: validation fails first
    a.q_lat = a.cache = a.block_tables = a.seq_lens = a.items = a.seq_item_begin = fake
    a.ctx = a.workspace = fake
    a.w_v, a.proj_heads, a.head_dim = fake, 3, 16   # 4 heads cannot map onto 3
    assert L.plkv_latent_decode(ctypes.byref(a), None) == m.PLKV_ERR_INVALID_PAGED_LOOKUP
    a.proj_heads = 2
    a.latent_dim, a.value_dim = 12, 12               # rows must be 16-byte multiples
    assert L.plkv_latent_decode(ctypes.byref(a), None) == m.PLKV_ERR_UNSUPPORTED
    a.latent_dim, a.value_dim = 8, 8
    a.workspace_bytes = 1
    assert L.plkv_latent_decode(ctypes.byref(a), None) == m.PLKV_ERR_WORKSPACE
    a.workspace_bytes, a.workspace = 1 << 30, fake + 16   # scratch must be 256-byte aligned
    assert L.plkv_latent_decode(ctypes.byref(a), None) == m.PLKV_ERR_INVALID_ARGUMENT
    a.workspace = fake
    assert L.plkv_project_query(fake, fake, fake, 1, 6, 4, 16, 8, None) == \
        m.PLKV_ERR_INVALID_PAGED_LOOKUP
    assert L.plkv_latent_append_f16(fake, fake, 4, None, fake, None, 1, fake, 6, 0, 8, None,
                                    None) == m.PLKV_ERR_ZERO_VALUE
    assert L.plkv_latent_append_f16(fake, fake, 4, None, fake, None, 0, fake, 6, 4, 8, None,
                                    None) == m.PLKV_OK
    f = m.FullKVDecodeArgs(batch=1, q_heads=6, kv_heads=4, head_dim=16, block_size=4,
                           num_physical=6, max_blocks=4, n_items=1)
    assert L.plkv_fullkv_decode(ctypes.byref(f), None) == m.PLKV_ERR_INVALID_PAGED_LOOKUP
    assert L.plkv_out_proj(fake, fake, fake, 65, 16, 16, 1, fake, 1 << 20, None) == \
        m.PLKV_ERR_UNSUPPORTED
    assert L.plkv_latent_decode_workspace_size(10, 2, 4, 8, 8) > 10 * 4 * 8 * 4
    assert L.plkv_allocate_slots(fake, 4, fake, None, 0, 16, fake, 64, fake, 4, None, None) == \
        m.PLKV_ERR_ZERO_VALUE
    assert L.plkv_allocate_slots(None, 4, fake, None, 2, 16, fake, 64, fake, 4, None, None) == \
        m.PLKV_ERR_INVALID_ARGUMENT
    assert L.plkv_allocate_slots(fake, 4, fake, None, 2, 16, fake, 1 << 40, fake, 4, None, None) == \
        m.PLKV_ERR_ARITHMETIC_OVERFLOW
    assert L.plkv_allocate_slots(fake, 4, fake, None, 2, 16, fake, 64, fake, 0, None, None) == \
        m.PLKV_ERR_ZERO_VALUE
    # peer exchange: buffer size, argument checks before any launch
    assert L.plkv_peer_buffer_bytes(0, 8) == 0
    assert L.plkv_peer_buffer_bytes(10, 8) == 512 + 2 * 512  # 360-byte slots padded to 512
    assert L.plkv_peer_publish(fake, fake, 0, 8, fake, 2, 0, fake, None, None) == \
        m.PLKV_ERR_ZERO_VALUE
    assert L.plkv_peer_publish(fake, fake, 4, 8, fake, 2, 2, fake, None, None) == \
        m.PLKV_ERR_INVALID_ARGUMENT
    assert L.plkv_peer_publish(fake, fake, 4, 8, fake, 33, 0, fake, None, None) == \
        m.PLKV_ERR_INVALID_ARGUMENT
    assert L.plkv_peer_init_buffer(None, 4096, None) == m.PLKV_ERR_INVALID_ARGUMENT
    assert L.plkv_peer_init_buffer(fake, 64, None) == m.PLKV_ERR_INVALID_ARGUMENT
    assert L.plkv_peer_merge(4, 8, None, 2, 0, fake, fake, None, None, None) == \
        m.PLKV_ERR_INVALID_ARGUMENT
    assert L.plkv_peer_alloc(0, None, None) == m.PLKV_ERR_INVALID_ARGUMENT


def test_product_never_imports_the_oracle():
    pkg_dir = os.path.join(ROOT, PACKAGE)
    for dirpath, _, files in os.walk(pkg_dir):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                text = open(os.path.join(dirpath, f), encoding="utf-8").read()
                assert "import oracle" not in text and "from oracle" not in text, f
                assert "plkv_oracle" not in text, f


def _plan_workers(lens, bs, workers):
    m = _lib_mod()
    lens = np.ascontiguousarray(np.asarray(lens, np.int32))
    n = ctypes.c_int32(0)
    st = m.lib().plkv_plan_workers(lens.ctypes.data, lens.size, bs, workers, None, 0, None, None,
                                   ctypes.byref(n))
    assert st == m.PLKV_ERR_WORKSPACE
    items = np.zeros((n.value, 4), np.int32)
    begin = np.zeros(lens.size + 1, np.int32)
    wbegin = np.zeros(workers + 1, np.int32)
    st = m.lib().plkv_plan_workers(lens.ctypes.data, lens.size, bs, workers, items.ctypes.data,
                                   n.value, begin.ctypes.data, wbegin.ctypes.data, ctypes.byref(n))
    assert st == m.PLKV_OK
    return items, begin, wbegin


@pytest.mark.parametrize("lens,bs,workers", [
    ([131072] * 8, 64, 74), ([7, 13], 4, 74), ([0, 5000, 0, 3], 64, 3), ([1], 64, 1),
    (list(np.random.default_rng(3).integers(1024, 32769, 64)), 64, 74), ([640] * 3, 64, 40)])
def test_worker_plan_balances_and_covers(lens, bs, workers):
    items, begin, wbegin = _plan_workers(lens, bs, workers)
    assert begin[0] == 0 and begin[-1] == len(items)
    assert wbegin[0] == 0 and wbegin[-1] == len(items) and np.all(np.diff(wbegin) >= 0)
    for b, n in enumerate(lens):
        its = items[begin[b]:begin[b + 1]]
        assert len(its) >= 1 and np.all(its[:, 0] == b)
        nb = (n + bs - 1) // bs
        covered = np.concatenate([np.arange(i[1], i[2]) for i in its])
        np.testing.assert_array_equal(covered, np.arange(nb))
    total = sum((n + bs - 1) // bs for n in lens)
    per_worker = [int(np.sum(items[wbegin[w]:wbegin[w + 1], 2] - items[wbegin[w]:wbegin[w + 1], 1]))
                  for w in range(workers)]
    assert sum(per_worker) == total
    # worker cost = blocks + per-item cost; the plan is never worse than an
    # equal split of the blocks (whose workers may hold two items)
    c = max(1, (256 + bs - 1) // bs)
    cost = [per_worker[w] + c * int(wbegin[w + 1] - wbegin[w]) for w in range(workers)]
    nb = np.array([(n + bs - 1) // bs for n in lens])
    start = np.concatenate([[0], np.cumsum(nb)])
    eq = []
    for w in range(workers):
        a, b = total * w // workers, total * (w + 1) // workers
        n_it = sum(1 for s in range(len(lens)) if (nb[s] == 0 and a <= start[s] < max(b, a + 1))
                   or (min(b, start[s + 1]) > max(a, start[s])))
        eq.append((b - a) + c * n_it)
    assert max(cost) <= max(eq)
    assert max(cost) <= -(-(total + c * len(lens)) // workers) + 2 * c


@pytest.mark.parametrize("lens,bs,kv,min_tokens", [
    ([4096] * 16, 16, 8, 2048), ([4096] * 64, 16, 8, 2048), ([256], 16, 8, 16),
    ([100, 20000, 7], 32, 1, 20107 // 148)])
def test_fullkv_plan_item_sizes(lens, bs, kv, min_tokens):
    """The full-KV planner keeps every item at least `min_tokens` long
    (except a sequence's whole remainder) and still covers every block once."""
    import importlib

    ops = importlib.import_module(PACKAGE + ".ops")
    plan = ops.plan_fullkv(lens, bs, kv, device="cpu")
    items, begin = plan.items_host, plan.seq_item_begin_host
    for b, n in enumerate(lens):
        its = items[begin[b]:begin[b + 1]]
        nb = (n + bs - 1) // bs
        covered = np.concatenate([np.arange(i[1], i[2]) for i in its])
        np.testing.assert_array_equal(covered, np.arange(nb))
        if len(its) > 1:
            assert (its[:, 2] - its[:, 1]).min() * bs >= min_tokens // 2
    if lens == [4096] * 16:
        assert plan.n_items == 32
