"""One host process driving contexts on several GPUs through the C ABI (the N-API host of the
reference's engine is such a process): every entry point runs on its context's device whatever
device the calling thread has current, and leaves the caller's current device as it was.

The GPU test needs two devices (skipped on one). The CPU test is ctypes-only: on a machine
without a usable device, context creation fails with a status and a message instead of crashing.
"""

import ctypes

import numpy as np
import pytest
import torch

from tests.conftest import pkg


def test_ctx_create_without_device_fails_cleanly():
    if torch.cuda.is_available():
        pytest.skip("a device is present: the negative case needs a machine without one")
    lib = ctypes.CDLL(pkg("build").build())
    lib.anima_ctx_create.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
    lib.anima_last_error.restype = ctypes.c_char_p
    h = ctypes.c_void_p()
    st = lib.anima_ctx_create(1, ctypes.byref(h))
    assert st != 0 and not h.value
    assert lib.anima_last_error()


def _linear_and_attention(ops, wts, dev):
    torch.manual_seed(3)
    x = torch.randn(512, 2048).to(dev)
    w = wts.Linear("i8", 1024, 2048, torch.randint(-127, 128, (1024, 2048), dtype=torch.int8).to(dev),
                   torch.full((1024,), 1e-3).to(dev))
    qa = ops.rotate_quant(x, 2)
    y = ops.linear(qa, w, out=torch.empty(512, 1024, device=dev))
    qkv = torch.randn(1024, 6144).to(torch.bfloat16).to(dev)
    a = ops.attention(qkv, qkv, qkv, Lq=1024, Lk=1024, H=16, ldq=6144, ldk=6144, ldv=6144, q_off=0, k_off=2048,
                      v_off=4096, out_dtype=torch.float32)
    return y, a


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_contexts_on_two_devices_in_one_process():
    ops, wts, dev = pkg("ops"), pkg("weights"), pkg("device")
    torch.cuda.set_device(0)
    y0, a0 = _linear_and_attention(ops, wts, "cuda:0")
    # device 0 stays current while the library runs the same work on device 1
    y1, a1 = _linear_and_attention(ops, wts, "cuda:1")
    assert torch.cuda.current_device() == 0
    dev.Context.get(0).sync()
    dev.Context.get(1).sync()
    assert torch.cuda.current_device() == 0
    np.testing.assert_array_equal(y0.cpu().numpy(), y1.cpu().numpy())
    np.testing.assert_array_equal(a0.cpu().numpy(), a1.cpu().numpy())
