"""Failure detection on the GPU without a fault: a kernel's bounded wait on a barrier that nothing
releases gives up, the device error word reports it at the next sync (the reference surfaces GPU
errors at read/sync, device.js:224-231), and the context keeps working."""

import ctypes as C

import pytest
import torch

from tests._util import rel_l2
from tests.conftest import pkg

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_the_context_survives():
    dev, ops = pkg("device"), pkg("ops")
    ctx = dev.Context.get(0)
    res = (C.c_int * 2)()
    ctx.call("anima_selftest_wait_timeout", C.c_uint(50000), res)  # 50 ms
    assert res[0] == 0 and res[1] == 1  # the wait gave up and raised the abort flag
    with pytest.raises(dev.AnimaError, match="data wait timed out"):
        ctx.sync()
    ctx.sync()  # the error was reported once and cleared
    # the context still runs the pipeline kernels
    x = torch.randn(64, 2048, device="cuda")
    y = ops.rotate(x)
    z = ops.rotate(y)  # the Hadamard is its own inverse
    assert rel_l2(z.cpu().numpy(), x.cpu().numpy()) < 1e-6
    ctx.sync()


def test_peer_barrier_without_the_other_rank_times_out():
    """The sequence-parallel barrier as rank 0 of a two-rank group whose second rank never
    arrives (its flag words are a second local array that nothing writes): after the 50 ms limit
    the kernel records the timeout and returns; a one-rank barrier completes."""
    dev = pkg("device")
    ctx = dev.Context.get(0)
    addrs = []
    for _ in range(2):
        a, h = C.c_void_p(), C.create_string_buffer(64)
        ctx.call("anima_ipc_alloc", 64, C.byref(a), h)
        addrs.append(a.value)
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    try:
        g = dev.PeerGroup()
        g.rank, g.world, g.timeout_us = 0, 1, 50000
        g.flags[0] = addrs[0]
        g.counter = counter.data_ptr()
        ctx.call("anima_peer_barrier", C.byref(g))
        ctx.sync()                       # alone, every rank has arrived
        assert int(counter.item()) == 1
        g.world = 2
        g.flags[1] = addrs[1]            # "rank 1": its own flags get this rank's epoch, its word in ours never
        ctx.call("anima_peer_barrier", C.byref(g))
        with pytest.raises(dev.AnimaError, match="cross-GPU barrier timed out"):
            ctx.sync()
        ctx.sync()
        assert int(counter.item()) == 2
    finally:
        for a in addrs:
            ctx.call("anima_ipc_free", a)
