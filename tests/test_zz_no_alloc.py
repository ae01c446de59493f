"""The allocation-free conv entry point (rtb_conv2d_fwd_noalloc).

It exists for callers that cannot allocate device memory on the conv path (a
host framework whose own allocator owns the GPU memory budget, or a
latency-critical loop where an allocation may synchronise the device): its
scratch is a fixed 16 MiB array inside the library, shared by every call on a
device and holding the previous call's data.  So each case here runs right
after a call that filled the scratch with NaN, checks the result against the
float64 oracle and against rtb_conv2d_fwd, and the allocation check watches
the stream-ordered pool and the device's free memory across a call.

This file is named so that pytest collects it last; it passes both alone in a
fresh process and after the rest of the suite."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-5  # the 3xTF32 relative Frobenius tolerance used by the conv tests


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _out_shape(rb, x, x_layout, w, stride, pad, y_layout):
    if x_layout == rb.LAYOUT_NCHW:
        N, Ci, H, W = x.shape
    else:
        N, H, W, Ci = x.shape
    Co, _, kh, kw = w.shape
    Ho = (H + 2 * pad - kh) // stride + 1
    Wo = (W + 2 * pad - kw) // stride + 1
    return (N, Co, Ho, Wo) if y_layout == rb.LAYOUT_NCHW else (N, Ho, Wo, Co)


def _call(rb, name, x, w, b, stride, pad, act, x_layout, y_layout, y=None):
    if x_layout == rb.LAYOUT_NCHW:
        N, Ci, H, W = x.shape
    else:
        N, H, W, Ci = x.shape
    Co, _, kh, kw = w.shape
    if y is None:
        y = torch.empty(_out_shape(rb, x, x_layout, w, stride, pad, y_layout), device="cuda")
    ctx = rb.get_context(0)
    st = getattr(rb.lib(), name)(ctx.handle, N, Ci, H, W, Co, kh, kw, stride, stride, pad, pad,
                                _p(x), x_layout, _p(w), _p(b), None, act, _p(y), y_layout,
                                rb.PREC_3XTF32, None)
    return st, y


def _rel(a, b):
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm())


def _fill_scratch_with_nan(rb):
    """A call whose padded NHWC input copy covers the first 12.8 MiB of the
    scratch with NaN (its output is NaN as well and is not used)."""
    x = torch.full((4, 64, 112, 112), float("nan"), device="cuda")
    w = torch.full((8, 64, 1, 1), float("nan"), device="cuda")
    st, _ = _call(rb, "rtb_conv2d_fwd_noalloc", x, w, None, 1, 0, rb.ACT_NONE, rb.LAYOUT_NCHW,
                  rb.LAYOUT_NCHW)
    assert st == 0, rb._lib.last_error()


CASES = [  # (x shape, x layout, w shape, stride, pad)
    ((8, 64, 28, 28), "NCHW", (96, 64, 3, 3), 1, 1),    # TMA im2col producer
    ((4, 5, 30, 30), "NCHW", (16, 5, 3, 3), 1, 1),      # Ci=5 -> Cp=8: zero padding channels
    ((3, 17, 17, 6), "NHWC", (24, 6, 3, 3), 2, 1),      # unaligned NHWC rows repacked (Cp=8)
    ((4, 14, 14, 128), "NHWC", (64, 128, 3, 3), 2, 1),  # aligned NHWC read in place
    ((2, 3, 64, 64), "NCHW", (64, 3, 7, 7), 2, 3),      # stem-shaped: Ci=3 (Cp=4), 7x7 stride 2
]


@pytest.mark.parametrize("xs,xl,ws,stride,pad", CASES)
def test_noalloc_matches_oracle_and_conv2d_fwd_after_stale_scratch(gpu, orc, xs, xl, ws, stride,
                                                                   pad):
    rb = gpu
    layout = rb.LAYOUT_NCHW if xl == "NCHW" else rb.LAYOUT_NHWC
    x = orc.normal(xs, 21, 1)
    w = orc.normal(ws, 21, 2, 0.0, float(np.sqrt(2.0 / np.prod(ws[1:]))))
    b = orc.uniform((ws[0],), 21, 3, -0.1, 0.1)
    xn = x if xl == "NCHW" else np.ascontiguousarray(x.transpose(0, 3, 1, 2))
    pre = (orc.conv2d_f64(xn, w, (stride, stride), (pad, pad))
           + b.astype(np.float64)[None, :, None, None])
    ref = torch.from_numpy(np.maximum(pre, 0.0))
    xd, wd, bd = (torch.from_numpy(np.ascontiguousarray(t)).cuda() for t in (x, w, b))
    st_ref, y_ref = _call(rb, "rtb_conv2d_fwd", xd, wd, bd, stride, pad, rb.ACT_RELU, layout,
                          rb.LAYOUT_NCHW)
    for _ in range(2):  # two calls in a row, each after the scratch was filled with NaN
        _fill_scratch_with_nan(rb)
        st, y = _call(rb, "rtb_conv2d_fwd_noalloc", xd, wd, bd, stride, pad, rb.ACT_RELU, layout,
                      rb.LAYOUT_NCHW)
        torch.cuda.synchronize()
        assert st_ref == 0 and st == 0, rb._lib.last_error()
        assert torch.isfinite(y).all()
        assert _rel(y.cpu(), ref) <= TOL
        assert _rel(y, y_ref) <= TOL
    assert rb.get_context(0).device_error() == 0


def test_noalloc_call_allocates_nothing(gpu):
    """Across a call (after one identical call, so every kernel is loaded):
    the stream-ordered pool's in-use high watermark and reserved size, and the
    device's free memory, stay exactly where they were."""
    rb = gpu
    rt = pytest.importorskip("cuda.bindings.runtime")
    drv = pytest.importorskip("cuda.bindings.driver")
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn((8, 64, 28, 28), device="cuda", generator=g)
    w = torch.randn((96, 64, 3, 3), device="cuda", generator=g) * 0.05
    b = torch.randn(96, device="cuda", generator=g) * 0.1
    y = torch.empty((8, 96, 28, 28), device="cuda")
    st, _ = _call(rb, "rtb_conv2d_fwd_noalloc", x, w, b, 1, 1, rb.ACT_RELU, rb.LAYOUT_NCHW,
                  rb.LAYOUT_NCHW, y)
    assert st == 0, rb._lib.last_error()
    torch.cuda.synchronize()

    err, pool = rt.cudaDeviceGetDefaultMemPool(0)
    assert err == rt.cudaError_t.cudaSuccess

    def attr(a):
        e, v = rt.cudaMemPoolGetAttribute(pool, a)
        assert e == rt.cudaError_t.cudaSuccess
        return int(v)

    A = rt.cudaMemPoolAttr
    e, = rt.cudaMemPoolSetAttribute(pool, A.cudaMemPoolAttrUsedMemHigh, drv.cuuint64_t(0))
    assert e == rt.cudaError_t.cudaSuccess
    used0 = attr(A.cudaMemPoolAttrUsedMemCurrent)
    reserved0 = attr(A.cudaMemPoolAttrReservedMemCurrent)
    e, free0, _ = rt.cudaMemGetInfo()
    assert e == rt.cudaError_t.cudaSuccess
    st, _ = _call(rb, "rtb_conv2d_fwd_noalloc", x, w, b, 1, 1, rb.ACT_RELU, rb.LAYOUT_NCHW,
                  rb.LAYOUT_NCHW, y)
    assert st == 0, rb._lib.last_error()
    torch.cuda.synchronize()
    e, free1, _ = rt.cudaMemGetInfo()
    assert e == rt.cudaError_t.cudaSuccess
    assert attr(A.cudaMemPoolAttrUsedMemHigh) <= used0
    assert attr(A.cudaMemPoolAttrUsedMemCurrent) == used0
    assert attr(A.cudaMemPoolAttrReservedMemCurrent) == reserved0
    assert free1 == free0
    # and the allocating entry point does use the pool (the check can see it)
    e, = rt.cudaMemPoolSetAttribute(pool, A.cudaMemPoolAttrUsedMemHigh, drv.cuuint64_t(0))
    st, _ = _call(rb, "rtb_conv2d_fwd", x, w, b, 1, 1, rb.ACT_RELU, rb.LAYOUT_NCHW,
                  rb.LAYOUT_NCHW, y)
    torch.cuda.synchronize()
    assert st == 0 and attr(A.cudaMemPoolAttrUsedMemHigh) > used0


def test_noalloc_rejects_oversized_and_bad_arguments_without_touching_scratch(gpu):
    rb = gpu
    x = torch.empty((64, 64, 56, 56), device="cuda")      # 51 MiB padded input > 16 MiB
    w = torch.empty((64, 64, 3, 3), device="cuda")
    st, _ = _call(rb, "rtb_conv2d_fwd_noalloc", x, w, None, 1, 1, rb.ACT_NONE, rb.LAYOUT_NCHW,
                  rb.LAYOUT_NCHW)
    assert st == rb._lib.RTB_E_INVALID
    assert "16 MiB" in rb._lib.last_error()
    # invalid y layout / activation / precision: rejected before any launch
    xs = torch.ones((1, 4, 8, 8), device="cuda")
    ws = torch.ones((4, 4, 3, 3), device="cuda")
    y = torch.empty((1, 4, 8, 8), device="cuda")
    ctx = rb.get_context(0)
    L = rb.lib()
    args = (ctx.handle, 1, 4, 8, 8, 4, 3, 3, 1, 1, 1, 1, _p(xs), rb.LAYOUT_NCHW, _p(ws), None,
            None)
    assert L.rtb_conv2d_fwd_noalloc(*args, 0, _p(y), 7, rb.PREC_3XTF32, None) == rb._lib.RTB_E_INVALID
    assert L.rtb_conv2d_fwd_noalloc(*args, 9, _p(y), rb.LAYOUT_NCHW, rb.PREC_3XTF32,
                                    None) == rb._lib.RTB_E_INVALID
    assert L.rtb_conv2d_fwd_noalloc(*args, 0, _p(y), rb.LAYOUT_NCHW, 5, None) == rb._lib.RTB_E_INVALID
