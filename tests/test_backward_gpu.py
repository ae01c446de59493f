"""Backward contractions on the B200 (MatmulBackward, rustorch-core/src/ops.rs:
529-570; Conv2dBackward, ops/conv.rs:336-736) against the oracle's f64
restatements, which are pinned by the reference's matmul-backward test and by
the adjoint identity with the pinned forward conv (tests/test_oracle.py).
Tolerances as for the forward path: 3xTF32 <= 1e-5, TF32 <= 5e-3."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {0: 1e-5, 1: 5e-3}


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def test_kat_matmul_backward(gpu, kats):
    k = kats["matmul_backward_2x2"]
    a = _dev(np.array(k["a"], np.float32).reshape(k["a_shape"]))
    b = _dev(np.array(k["b"], np.float32).reshape(k["b_shape"]))
    g = torch.ones((a.shape[0], b.shape[1]), device="cuda")
    for prec in (0, 1):
        da, db = gpu.matmul_backward(a, b, g, precision=prec)
        assert np.max(np.abs(_host(da).reshape(-1) - k["expected_grad_a"])) < k["abs_tol"]
        assert np.max(np.abs(_host(db).reshape(-1) - k["expected_grad_b"])) < k["abs_tol"]


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (7, 33, 65), (256, 300, 129), (1024, 512, 768),
                                   (2048, 64, 4096)])
@pytest.mark.parametrize("prec", [0, 1])
def test_matmul_backward(gpu, orc, m, n, k, prec):
    a = orc.normal((m, k), 11, 1)
    b = orc.normal((k, n), 11, 2)
    g = orc.normal((m, n), 11, 3)
    ra, rb_ = orc.matmul_backward_f64(a, b, g)
    da, db = gpu.matmul_backward(_dev(a), _dev(b), _dev(g), precision=prec)
    assert orc.rel_frob(_host(da), ra) <= TOL[prec]
    assert orc.rel_frob(_host(db), rb_) <= TOL[prec]


def test_matmul_backward_accumulate(gpu, orc):
    """accumulate adds to existing gradients (the reference's accumulate_grad)."""
    a = orc.normal((96, 80), 12, 1)
    b = orc.normal((80, 40), 12, 2)
    g = orc.normal((96, 40), 12, 3)
    ra, rb_ = orc.matmul_backward_f64(a, b, g)
    prev_a = orc.normal((96, 80), 12, 4)
    prev_b = orc.normal((80, 40), 12, 5)
    da, db = _dev(prev_a), _dev(prev_b)
    gpu.matmul_backward(_dev(a), _dev(b), _dev(g), out_a=da, out_b=db, accumulate=True)
    assert orc.rel_frob(_host(da), ra + prev_a) <= 1e-5
    assert orc.rel_frob(_host(db), rb_ + prev_b) <= 1e-5


@pytest.mark.parametrize("xshape,wshape,stride,pad", [
    ((2, 3, 9, 11), (4, 3, 3, 2), (1, 1), (1, 0)),
    ((2, 5, 12, 10), (7, 5, 3, 3), (2, 2), (1, 1)),
    ((1, 4, 11, 13), (6, 4, 5, 3), (2, 1), (0, 2)),
    ((4, 64, 28, 28), (64, 64, 3, 3), (1, 1), (1, 1)),      # Cp = 64: TMA im2col producer
    ((4, 64, 56, 56), (128, 64, 3, 3), (2, 2), (1, 1)),     # ResNet downsampling 3x3
    ((4, 64, 56, 56), (128, 64, 1, 1), (2, 2), (0, 0)),     # 1x1 stride 2
    ((2, 3, 64, 64), (16, 3, 7, 7), (2, 2), (3, 3)),        # stem-like
])
@pytest.mark.parametrize("prec", [0, 1])
def test_conv2d_backward(gpu, orc, xshape, wshape, stride, pad, prec):
    x = orc.normal(xshape, 13, 1)
    w = orc.normal(wshape, 13, 2, 0.0, float(np.sqrt(2.0 / np.prod(wshape[1:]))))
    ho = (xshape[2] + 2 * pad[0] - wshape[2]) // stride[0] + 1
    wo = (xshape[3] + 2 * pad[1] - wshape[3]) // stride[1] + 1
    g = orc.normal((xshape[0], wshape[0], ho, wo), 13, 3)
    rx = orc.conv2d_grad_input_f64(g, w, xshape, stride, pad)
    rw = orc.conv2d_grad_weight_f64(x, g, wshape, stride, pad)
    dx, dw = gpu.conv2d_backward(_dev(x), _dev(w), _dev(g), stride, pad, precision=prec)
    assert orc.rel_frob(_host(dx), rx) <= TOL[prec]
    assert orc.rel_frob(_host(dw), rw) <= TOL[prec]


def test_conv2d_backward_unsupported_padding(gpu):
    x = torch.ones((1, 2, 5, 5), device="cuda")
    w = torch.ones((3, 2, 3, 3), device="cuda")
    g = torch.ones((1, 3, 7, 7), device="cuda")
    with pytest.raises(gpu.RtbError) as e:
        gpu.conv2d_backward(x, w, g, (1, 1), (3, 3))
    assert e.value.status == 5
    # grad_weight alone has no such restriction
    dx, dw = gpu.conv2d_backward(x, w, g, (1, 1), (3, 3), need_x=False)
    assert dx is None and torch.isfinite(dw).all()
