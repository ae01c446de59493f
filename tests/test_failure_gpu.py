"""Failure detection without a GPU fault: bounded device waits, host-side
error paths, and the context staying usable afterwards."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(gpu):
    rb = gpu
    ctx = rb.get_context(0)
    assert ctx.device_error() == 0
    rb.call("rtb_debug_wait_probe", ctx.handle, 5_000_000, None)  # 5 ms
    st = rb.lib().rtb_stream_synchronize(ctx.handle, None)
    assert st == rb._lib.RTB_E_TIMEOUT
    assert "code 8" in rb._lib.last_error()
    assert ctx.device_error() == 0  # reported once, then cleared
    # the context (and the GPU) still work
    a = torch.randn(300, 200, device="cuda")
    b = torch.randn(200, 100, device="cuda")
    c = rb.sgemm(a, b)
    torch.cuda.synchronize()
    ref = a.double() @ b.double()
    assert float((c.double() - ref).norm() / ref.norm()) < 1e-5


def test_host_side_errors(gpu):
    rb = gpu
    L = rb.lib()
    ctx = rb.get_context(0)
    # allocation failure is a status, not an abort
    p = ctypes.c_void_p()
    st = L.rtb_malloc(ctx.handle, ctypes.byref(p), 1 << 50, None)
    assert st == rb._lib.RTB_E_OOM and not p.value
    assert "rtb_malloc" in rb._lib.last_error()
    # bad shapes / arguments
    assert L.rtb_sgemm(ctx.handle, -1, 2, 2, None, 2, 0, None, 2, 0, None, 0, None, 2, 0,
                       None) == rb._lib.RTB_E_INVALID
    assert L.rtb_sgemm(ctx.handle, 2, 2, 2, None, 2, 2, None, 2, 0, None, 0, None, 2, 0,
                       None) == rb._lib.RTB_E_INVALID
    assert L.rtb_set_timeout_ns(ctx.handle, 10) == rb._lib.RTB_E_INVALID
    h = ctypes.c_void_p()
    assert L.rtb_nccl_comm_init(ctx.handle, None, 2, 0, ctypes.byref(h)) == rb._lib.RTB_E_INVALID
    assert L.rtb_nccl_comm_init(ctx.handle, b"x" * 128, 2, 5, ctypes.byref(h)) == \
        rb._lib.RTB_E_INVALID
    # and the context is still healthy
    assert ctx.device_error() == 0
