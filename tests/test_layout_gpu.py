"""The conv path's data-layout kernels through the C ABI, bit-exact against
numpy: NCHW -> NHWC with channels padded to a multiple of 4 (the implicit
GEMM's input layout) and the weight repack [Co, Ci, kh, kw] -> [Co, kh*kw*Cp]
with k = (r*kw + s)*Cp + ci (the im2col column order of
rustorch-core/src/ops/conv.rs, taps outermost so a k-block is one tap)."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ptr(t, offset_elems=0):
    return ctypes.c_void_p(t.data_ptr() + 4 * offset_elems)


@pytest.mark.parametrize("shape", [(2, 128, 28, 28), (3, 5, 9, 11), (1, 3, 7, 7), (2, 37, 13, 13),
                                   (1, 64, 1, 130), (4, 36, 5, 5)])
@pytest.mark.parametrize("y_offset", [0, 1])
def test_nchw_to_nhwc_padded(gpu, shape, y_offset):
    import rustorch_b200 as rb
    n, c, h, w = shape
    cp = (c + 3) // 4 * 4
    x = torch.randn(shape, device="cuda")
    # y_offset = 1 shifts the output by 4 bytes: the kernel must not assume
    # 16-byte alignment of a caller's buffer
    y = torch.full((n * h * w * cp + y_offset,), 7.0, device="cuda")
    rb.call("rtb_nchw_to_nhwc_padded", gpu.get_context(0).handle, n, c, h, w, _ptr(x),
            _ptr(y, y_offset), None)
    torch.cuda.synchronize()
    got = y[y_offset:].cpu().numpy().reshape(n, h, w, cp)
    ref = np.zeros((n, h, w, cp), np.float32)
    ref[..., :c] = x.cpu().numpy().transpose(0, 2, 3, 1)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("co,ci,kh,kw", [(128, 128, 3, 3), (64, 3, 7, 7), (10, 36, 5, 5),
                                         (7, 5, 3, 2), (256, 512, 3, 3), (16, 2048, 1, 1)])
def test_prepack_weight(gpu, co, ci, kh, kw):
    import rustorch_b200 as rb
    cp = (ci + 3) // 4 * 4
    w = torch.randn((co, ci, kh, kw), device="cuda")
    wp = torch.full((co * kh * kw * cp,), 7.0, device="cuda")
    rb.call("rtb_conv2d_prepack_weight", gpu.get_context(0).handle, co, ci, kh, kw, _ptr(w),
            _ptr(wp), None)
    torch.cuda.synchronize()
    got = wp.cpu().numpy().reshape(co, kh * kw, cp)
    ref = np.zeros((co, kh * kw, cp), np.float32)
    ref[:, :, :ci] = w.cpu().numpy().reshape(co, ci, kh * kw).transpose(0, 2, 1)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("co,ci,kh,kw", [(128, 128, 3, 3), (7, 5, 3, 2), (64, 16, 4, 4)])
def test_prepack_weight_lo(gpu, co, ci, kh, kw):
    """rtb_conv2d_prepack_weight_lo: the same packed weight as
    rtb_conv2d_prepack_weight, and its 3xTF32 low part x - trunc_tf32(x)
    (low 13 mantissa bits of the fp32 pattern cleared) bit for bit."""
    import rustorch_b200 as rb
    cp = (ci + 3) // 4 * 4
    n = co * kh * kw * cp
    w = torch.randn((co, ci, kh, kw), device="cuda")
    wp = torch.full((n,), 7.0, device="cuda")
    wl = torch.full((n,), 7.0, device="cuda")
    ref_p = torch.empty((n,), device="cuda")
    h = gpu.get_context(0).handle
    rb.call("rtb_conv2d_prepack_weight_lo", h, co, ci, kh, kw, _ptr(w), _ptr(wp), _ptr(wl), None)
    rb.call("rtb_conv2d_prepack_weight", h, co, ci, kh, kw, _ptr(w), _ptr(ref_p), None)
    torch.cuda.synchronize()
    p = wp.cpu().numpy()
    np.testing.assert_array_equal(p, ref_p.cpu().numpy())
    hi = (p.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    np.testing.assert_array_equal(wl.cpu().numpy(), p - hi)


@pytest.mark.parametrize("prec", [0, 1])
def test_conv_packed_lo_matches_packed(gpu, prec):
    """A conv through rtb_conv2d_fwd_packed_lo (the weight's low part given)
    gives bit-identical results to rtb_conv2d_fwd_packed (low part computed
    by the call), in both precisions (TF32 ignores it)."""
    import rustorch_b200 as rb
    n, ci, hw, co, k = 16, 64, 28, 128, 3
    cp = ci
    h = gpu.get_context(0).handle
    x = torch.randn((n, hw, hw, cp), device="cuda")
    w = torch.randn((co, ci, k, k), device="cuda") * 0.05
    b = torch.randn((co,), device="cuda") * 0.1
    sz = co * k * k * cp
    wp = torch.empty((sz,), device="cuda")
    wl = torch.empty((sz,), device="cuda")
    rb.call("rtb_conv2d_prepack_weight_lo", h, co, ci, k, k, _ptr(w), _ptr(wp), _ptr(wl), None)
    y0 = torch.empty((n, hw, hw, co), device="cuda")
    y1 = torch.empty((n, hw, hw, co), device="cuda")
    rb.call("rtb_conv2d_fwd_packed", h, n, ci, hw, hw, co, k, k, 1, 1, 1, 1, _ptr(x), _ptr(wp),
            _ptr(b), None, rb.ACT_RELU, _ptr(y0), rb.LAYOUT_NHWC, prec, None)
    rb.call("rtb_conv2d_fwd_packed_lo", h, n, ci, hw, hw, co, k, k, 1, 1, 1, 1, _ptr(x), _ptr(wp),
            _ptr(wl), _ptr(b), None, rb.ACT_RELU, _ptr(y1), rb.LAYOUT_NHWC, prec, None)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)
