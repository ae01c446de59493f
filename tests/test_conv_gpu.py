"""Conv2d (+bias, +residual, +ReLU) parity on the B200: the implicit-GEMM
tcgen05 kernels against the oracle's restatement of ops::conv2d /
nn::Conv2d::forward, and the pooling kernels against ops::max_pool2d."""
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


def test_kat_conv2d(gpu, kats):
    k = kats["conv2d_3x3_k2"]
    x = np.array(k["x"], np.float32).reshape(k["x_shape"])
    w = np.array(k["w"], np.float32).reshape(k["w_shape"])
    for prec in (0, 1):
        y = _host(gpu.conv2d_fwd(_dev(x), _dev(w), stride=tuple(k["stride"]),
                                 padding=tuple(k["padding"]), precision=prec))
        assert np.max(np.abs(y.reshape(-1) - np.array(k["expected"]))) < k["abs_tol"]


def test_kat_jit_conv_relu_ones(gpu, kats):
    k = kats["jit_conv2d_relu_ones"]
    x = torch.full(k["x_shape"], k["x_fill"], device="cuda")
    w = torch.full(k["w_shape"], k["w_fill"], device="cuda")
    y = _host(gpu.conv2d_fwd(x, w, act=gpu.ACT_RELU))
    assert list(y.shape) == k["out_shape"]
    assert abs(y.reshape(-1)[0] - k["expected_first"]) < k["abs_tol"]


def test_kat_bench_conv_fill(gpu, kats):
    k = kats["bench_conv2d_fill"]
    x = torch.full(k["x_shape"], k["x_fill"], device="cuda")
    w = torch.full(k["w_shape"], k["w_fill"], device="cuda")
    y = _host(gpu.conv2d_fwd(x, w, stride=tuple(k["stride"]), padding=tuple(k["padding"])))
    interior = y[:, :, 1:-1, 1:-1]
    assert np.max(np.abs(interior / k["expected_interior"] - 1.0)) < k["rel_tol"]


def _cfg2_inputs(orc):
    """Conv2d+bias+ReLU, ResNet-50 stage-2 3x3 layer: x [32,128,28,28] ~ N(0,1),
    w Kaiming-normal std sqrt(2/1152), b ~ U(-0.1, 0.1), seed 1."""
    x = orc.normal((32, 128, 28, 28), 1, 0)
    w = orc.normal((128, 128, 3, 3), 1, 1, 0.0, float(np.sqrt(2.0 / (128 * 9))))
    b = orc.uniform((128,), 1, 2, -0.1, 0.1)
    return x, w, b


@pytest.mark.parametrize("prec", [0, 1])
def test_conv_bias_relu_resnet50_layer(gpu, orc, prec):
    x, w, b = _cfg2_inputs(orc)
    pre = orc.conv2d_f64(x, w, (1, 1), (1, 1)) + b.astype(np.float64)[None, :, None, None]
    y = _host(gpu.conv2d_fwd(_dev(x), _dev(w), _dev(b), (1, 1), (1, 1), act=gpu.ACT_RELU,
                             precision=prec))
    assert orc.rel_frob(y, np.maximum(pre, 0)) <= TOL[prec]
    # ReLU zero pattern: exact outside |pre| < 1e-5 in 3xTF32; in TF32 mode the
    # exemption band scales with that mode's 5e-3 tolerance (1e-2 of rms(pre)).
    band = 1e-5 if prec == 0 else 1e-2 * float(np.sqrt(np.mean(pre * pre)))
    mask = np.abs(pre) >= band
    assert np.array_equal((y > 0)[mask], (pre > 0)[mask])
    if prec == 0:
        # the reference's own CPU path (im2col + parallel core, f32) on the same inputs
        y32, _ = orc.conv2d_bias_relu(x, w, b, (1, 1), (1, 1))
        assert orc.rel_frob(y, y32.astype(np.float64)) <= 2e-5


@pytest.mark.parametrize("stage,c,hw", [(1, 64, 56), (3, 256, 14), (4, 512, 7)])
@pytest.mark.parametrize("prec", [0, 1])
def test_conv_bias_relu_resnet50_other_stages(gpu, orc, stage, c, hw, prec):
    """The other ResNet-50 3x3 layers at batch 32 (stage 1: 64 channels at
    56x56, stage 3: 256 at 14x14, stage 4: 512 at 7x7), Conv2d+bias+ReLU with
    the inputs generated like the stage-2 workload (seed 1 + stage)."""
    x = orc.normal((32, c, hw, hw), 1 + stage, 0)
    w = orc.normal((c, c, 3, 3), 1 + stage, 1, 0.0, float(np.sqrt(2.0 / (c * 9))))
    b = orc.uniform((c,), 1 + stage, 2, -0.1, 0.1)
    pre = orc.conv2d_f64(x, w, (1, 1), (1, 1)) + b.astype(np.float64)[None, :, None, None]
    y = _host(gpu.conv2d_fwd(_dev(x), _dev(w), _dev(b), (1, 1), (1, 1), act=gpu.ACT_RELU,
                             precision=prec))
    assert orc.rel_frob(y, np.maximum(pre, 0)) <= TOL[prec]
    band = 1e-5 if prec == 0 else 1e-2 * float(np.sqrt(np.mean(pre * pre)))
    mask = np.abs(pre) >= band
    assert np.array_equal((y > 0)[mask], (pre > 0)[mask])


@pytest.mark.parametrize("shape,wshape,stride,pad", [
    ((2, 3, 224, 224), (64, 3, 7, 7), (2, 2), (3, 3)),      # ResNet stem, Ci=3 -> padded to 4
    ((4, 64, 56, 56), (64, 64, 3, 3), (1, 1), (1, 1)),
    ((4, 64, 56, 56), (128, 64, 3, 3), (2, 2), (1, 1)),
    ((4, 64, 56, 56), (128, 64, 1, 1), (2, 2), (0, 0)),     # downsample 1x1 s2
    ((2, 256, 14, 14), (256, 256, 3, 3), (1, 1), (1, 1)),
    ((2, 512, 7, 7), (512, 512, 3, 3), (1, 1), (1, 1)),
    ((3, 5, 9, 11), (7, 5, 3, 2), (1, 2), (2, 0)),          # odd everything
    ((1, 36, 5, 5), (10, 36, 5, 5), (1, 1), (0, 0)),        # K-blocks straddle taps
    ((8, 7, 40, 40), (16, 7, 3, 3), (1, 1), (1, 1)),        # Cp=8: 4 taps per k-block
    ((4, 13, 48, 48), (32, 13, 5, 5), (2, 2), (2, 2)),      # Cp=16: 2 taps per k-block
    # stride 2 over <= 4 channels: 3xTF32 runs these as stride-1 convs of the
    # 16-channel space-to-depth input (odd sizes, even and odd kernels)
    ((2, 1, 33, 30), (8, 1, 4, 5), (2, 2), (1, 2)),
    ((3, 4, 17, 19), (16, 4, 3, 3), (2, 2), (1, 1)),
    ((2, 2, 64, 64), (24, 2, 2, 2), (2, 2), (0, 0)),
    ((4, 3, 100, 90), (32, 3, 5, 5), (2, 2), (2, 2)),       # large enough for TMA im2col
])
@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("producer", ["auto", "gather"])
def test_conv_shapes(gpu, orc, shape, wshape, stride, pad, prec, producer, monkeypatch):
    """producer=auto uses the TMA im2col path where Ci % 32 == 0, the multi-tap
    TMA im2col path (32 / Cp taps per k-block) for Cp in {8, 16} in 3xTF32
    mode, and the cp.async gather otherwise; producer=gather forces the
    cp.async gather everywhere."""
    if producer == "gather":
        monkeypatch.setenv("RTB_CONV_GATHER", "1")
    x = orc.normal(shape, 5, 1)
    w = orc.normal(wshape, 5, 2, 0.0, float(np.sqrt(2.0 / np.prod(wshape[1:]))))
    ref = orc.conv2d_f64(x, w, stride, pad)
    y = _host(gpu.conv2d_fwd(_dev(x), _dev(w), None, stride, pad, precision=prec))
    assert y.shape == ref.shape
    assert orc.rel_frob(y, ref) <= TOL[prec]


def test_conv_nhwc_residual(gpu, orc):
    """NHWC in/out with a residual and ReLU (a ResNet basic-block tail)."""
    x = orc.normal((2, 16, 16, 64), 6, 1)       # NHWC
    w = orc.normal((64, 64, 3, 3), 6, 2, 0.0, 0.06)
    b = orc.uniform((64,), 6, 3, -0.1, 0.1)
    r = orc.normal((2, 16, 16, 64), 6, 4)       # NHWC residual
    xn = np.ascontiguousarray(x.transpose(0, 3, 1, 2))
    pre = orc.conv2d_f64(xn, w, (1, 1), (1, 1)) + b.astype(np.float64)[None, :, None, None]
    pre = pre.transpose(0, 2, 3, 1) + r.astype(np.float64)
    y = _host(gpu.conv2d_fwd(_dev(x), _dev(w), _dev(b), (1, 1), (1, 1), residual=_dev(r),
                             act=gpu.ACT_RELU, x_layout=gpu.LAYOUT_NHWC, y_layout=gpu.LAYOUT_NHWC))
    assert orc.rel_frob(y, np.maximum(pre, 0)) <= 1e-5


@pytest.mark.parametrize("shape", [(2, 64, 32, 32), (3, 48, 28, 28), (2, 40, 9, 9)])
def test_conv_nchw_residual(gpu, orc, shape):
    """NCHW in/out with a residual and ReLU: 1024-pixel images (every tile
    inside one image: 3-D TMA stores), 784-pixel images (tiles across image
    boundaries take the direct stores) and 81-pixel images (hw % 4 != 0)."""
    n, c, h, w_ = shape
    x = orc.normal(shape, 9, 1)
    w = orc.normal((c + 8, c, 3, 3), 9, 2, 0.0, float(np.sqrt(2.0 / (9 * c))))
    b = orc.uniform((c + 8,), 9, 3, -0.1, 0.1)
    r = orc.normal((n, c + 8, h, w_), 9, 4)
    pre = (orc.conv2d_f64(x, w, (1, 1), (1, 1)) + b.astype(np.float64)[None, :, None, None]
           + r.astype(np.float64))
    for prec, tol in ((0, 1e-5), (1, 5e-3)):
        y = _host(gpu.conv2d_fwd(_dev(x), _dev(w), _dev(b), (1, 1), (1, 1), residual=_dev(r),
                                 act=gpu.ACT_RELU, precision=prec))
        assert orc.rel_frob(y, np.maximum(pre, 0)) <= tol


def test_conv_errors(gpu):
    x = torch.ones((1, 3, 8, 8), device="cuda")
    with pytest.raises(ValueError, match="must match input channels"):
        gpu.conv2d_fwd(x, torch.ones((4, 2, 3, 3), device="cuda"))
    with pytest.raises(gpu.RtbError) as e:
        gpu.conv2d_fwd(x, torch.ones((4, 3, 9, 9), device="cuda"))
    assert e.value.status == 1


def test_max_pool_bit_exact(gpu, orc):
    x = orc.normal((2, 64, 112, 112), 8, 1)
    ref = orc.max_pool2d(x, (3, 3), (2, 2), (1, 1))
    y = _host(gpu.max_pool2d(_dev(x)))
    np.testing.assert_array_equal(y, ref)
    yh = _host(gpu.max_pool2d(_dev(x.transpose(0, 2, 3, 1)), layout=gpu.LAYOUT_NHWC))
    np.testing.assert_array_equal(yh.transpose(0, 3, 1, 2), ref)


@pytest.mark.parametrize("n,c,h,w,pad", [(3, 4, 13, 9, 1), (2, 12, 33, 34, 0), (1, 8, 14, 15, 1),
                                          (2, 64, 112, 112, 1)])
def test_max_pool_nhwc_3x3s2_bit_exact(gpu, orc, n, c, h, w, pad):
    """The 3x3 stride-2 NHWC kernel (row maxima carried between output rows)
    against ops::max_pool2d bit for bit: odd sizes, strips of 8 output rows
    cut at 7 and 17 rows, ties between +0 and -0 (the first in window order
    wins), NaN (never wins) and -inf inputs."""
    x = orc.normal((n, c, h, w), 8, 3)
    rng = np.random.default_rng(8)
    special = np.array([0.0, -0.0, np.nan, -np.inf, 0.0, -0.0], np.float32)
    mask = rng.random(x.shape) < 0.3
    x[mask] = special[rng.integers(0, len(special), int(mask.sum()))]
    x[0, 0, :, :] = rng.choice(np.array([0.0, -0.0], np.float32), (h, w))  # a plane of ties
    ref = orc.max_pool2d(x, (3, 3), (2, 2), (pad, pad))
    yh = _host(gpu.max_pool2d(_dev(x.transpose(0, 2, 3, 1)), padding=(pad, pad),
                              layout=gpu.LAYOUT_NHWC))
    got = np.ascontiguousarray(yh.transpose(0, 3, 1, 2))
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_global_avg_pool(gpu, orc):
    x = orc.normal((4, 512, 7, 7), 8, 2)
    ref = orc.global_avg_pool(x)
    np.testing.assert_allclose(_host(gpu.global_avg_pool(_dev(x))), ref, rtol=1e-6, atol=1e-7)
    yh = _host(gpu.global_avg_pool(_dev(x.transpose(0, 2, 3, 1)), layout=gpu.LAYOUT_NHWC))
    np.testing.assert_allclose(yh, ref, rtol=1e-6, atol=1e-7)


def test_add_relu(gpu, orc):
    a = orc.normal((1000,), 9, 1)
    b = orc.normal((1000,), 9, 2)
    np.testing.assert_array_equal(_host(gpu.add(_dev(a), _dev(b))), a + b)
    np.testing.assert_array_equal(_host(gpu.relu(_dev(a))), orc.relu(a))
