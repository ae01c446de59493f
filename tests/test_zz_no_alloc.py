"""The allocation-free conv entry point (rtb_conv2d_fwd_noalloc).

It exists for callers that cannot allocate device memory on the conv path (a
host framework whose own allocator owns the GPU memory budget, or a
latency-critical loop where an allocation may synchronise the device): its
scratch is a fixed 16 MiB array inside the library.  This file is named so
that pytest collects it last; it passes both alone in a fresh process and
after the rest of the suite."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-5  # the 3xTF32 relative Frobenius tolerance used by the conv tests


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _call(rb, name, x, w, b, stride, pad, act, x_layout, y_layout):
    if x_layout == rb.LAYOUT_NCHW:
        N, Ci, H, W = x.shape
    else:
        N, H, W, Ci = x.shape
    Co, _, kh, kw = w.shape
    Ho = (H + 2 * pad - kh) // stride + 1
    Wo = (W + 2 * pad - kw) // stride + 1
    shape = (N, Co, Ho, Wo) if y_layout == rb.LAYOUT_NCHW else (N, Ho, Wo, Co)
    y = torch.empty(shape, device="cuda")
    ctx = rb.get_context(0)
    st = getattr(rb.lib(), name)(ctx.handle, N, Ci, H, W, Co, kh, kw, stride, stride, pad, pad,
                                _p(x), x_layout, _p(w), _p(b), None, act, _p(y), y_layout,
                                rb.PREC_3XTF32, None)
    return st, y


def _rel(a, b):
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm())


def test_noalloc_matches_conv2d_fwd_twice(gpu):
    rb = gpu
    g = torch.Generator(device="cuda").manual_seed(11)
    cases = [  # (x shape, layout, w shape, stride, pad)
        ((8, 64, 28, 28), rb.LAYOUT_NCHW, (96, 64, 3, 3), 1, 1),
        ((4, 14, 14, 128), rb.LAYOUT_NHWC, (64, 128, 3, 3), 2, 1),
    ]
    for xs, xl, ws, stride, pad in cases:  # two calls in a row, different shapes
        x = torch.randn(xs, device="cuda", generator=g)
        w = torch.randn(ws, device="cuda", generator=g) * 0.05
        b = torch.randn(ws[0], device="cuda", generator=g) * 0.1
        st_ref, y_ref = _call(rb, "rtb_conv2d_fwd", x, w, b, stride, pad, rb.ACT_RELU, xl,
                              rb.LAYOUT_NCHW)
        st, y = _call(rb, "rtb_conv2d_fwd_noalloc", x, w, b, stride, pad, rb.ACT_RELU, xl,
                      rb.LAYOUT_NCHW)
        torch.cuda.synchronize()
        assert st_ref == 0 and st == 0, rb._lib.last_error()
        assert _rel(y, y_ref) <= TOL
    assert rb.get_context(0).device_error() == 0


def test_noalloc_rejects_oversized(gpu):
    rb = gpu
    x = torch.empty((64, 64, 56, 56), device="cuda")      # 51 MiB padded input > 16 MiB
    w = torch.empty((64, 64, 3, 3), device="cuda")
    st, _ = _call(rb, "rtb_conv2d_fwd_noalloc", x, w, None, 1, 1, rb.ACT_NONE, rb.LAYOUT_NCHW,
                  rb.LAYOUT_NCHW)
    assert st == rb._lib.RTB_E_INVALID
    assert "16 MiB" in rb._lib.last_error()
