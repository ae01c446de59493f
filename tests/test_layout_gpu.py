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
