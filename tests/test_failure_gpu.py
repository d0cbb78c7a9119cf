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
