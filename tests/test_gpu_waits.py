"""Failure paths of the bounded device waits, driven to their limits in the
form this hardware pool allows: a wait on something that never happens (a
barrier with no arrival, a peer that never publishes) runs out its 1 s limit,
records PLKV_FLAG_TIMEOUT in the caller's error word and returns; no fault,
trap or endless loop is involved, and the context stays usable."""

import importlib

import numpy as np
import pytest
import torch

from conftest import PACKAGE

pytestmark = pytest.mark.gpu

FLAG_TIMEOUT = 0x20


def _lib():
    return importlib.import_module(PACKAGE + "._lib")


def _selftest(ctl):
    L = _lib()
    elapsed = torch.zeros(2, dtype=torch.int64, device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(L.lib().plkv_selftest_bounded_wait(ctl.data_ptr(), elapsed.data_ptr(),
                                               flags.data_ptr(),
                                               torch.cuda.current_stream().cuda_stream),
            "plkv_selftest_bounded_wait")
    torch.cuda.synchronize()
    return elapsed.cpu().numpy() / 1e9, int(flags.item())


def test_wait_gives_up_and_the_other_cta_follows():
    """CTA 0 waits out its 1 s limit and reports; CTA 1, which started 0.5 s
    later, gives up through the launch's abort word after about 0.5 s instead
    of its own 1 s."""
    ctl = torch.zeros(1, dtype=torch.int32, device="cuda")
    e, flags = _selftest(ctl)
    assert flags == FLAG_TIMEOUT
    assert int(ctl.item()) == 1
    assert 0.99 <= e[0] <= 1.2, e
    assert 0.4 <= e[1] <= 0.6, e
    x = torch.arange(10, device="cuda", dtype=torch.float32)   # the context is still usable
    assert float((x * 2).sum().item()) == 90.0


def test_wait_with_abort_already_set_ends_at_once_without_reporting():
    ctl = torch.ones(1, dtype=torch.int32, device="cuda")
    e, flags = _selftest(ctl)
    assert flags == 0
    assert np.all(e >= 0) and np.all(e < 1e-3), e


def test_peer_merge_times_out_when_a_peer_never_publishes():
    """Two stand-in ranks on one GPU: rank 0 publishes and merges, rank 1
    never publishes.  Rank 0's merge gives up after its 1 s limit, reports
    PLKV_FLAG_TIMEOUT, reads no peer rows and writes 0 / -inf; the exchange
    works again once rank 1 catches up."""
    mg = importlib.import_module(PACKAGE + ".multigpu")
    dev = torch.device("cuda")
    rows, width = 16, 8
    exch, _bufs = mg.PeerExchange.local_group(2, rows, width, dev)
    ctx = torch.randn((rows, width), device=dev)
    lse = torch.randn(rows, device=dev)
    out = torch.full((rows, width), float("nan"), device=dev)
    lse_out = torch.full((rows,), float("nan"), device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    exch[0].publish(ctx, lse, flags=flags)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    exch[0].merge(out, lse_out, flags=flags)
    t1.record()
    torch.cuda.synchronize()
    assert int(flags.item()) == FLAG_TIMEOUT
    assert 990 <= t0.elapsed_time(t1) <= 1300
    assert torch.count_nonzero(out) == 0
    assert torch.all(torch.isneginf(lse_out))
    # Rank 1 publishes and merges the step it missed; then both ranks run the
    # next step and rank 0's merge of it completes.
    exch[1].publish(ctx, lse)
    exch[1].merge(out, lse_out)
    flags.zero_()
    exch[0].publish(ctx, lse, flags=flags)
    exch[1].publish(ctx, lse, flags=flags)
    exch[0].merge(out, lse_out, flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    assert torch.allclose(out, ctx, rtol=1e-6, atol=1e-6)
