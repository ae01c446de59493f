"""matmul_bias_norm_activation on the B200 (rustorch-core/src/ops.rs:1815-1886:
matmul + bias, layer_norm over N, activation) against the oracle's f64
restatement, which is pinned by the 2x2 known answer and by torch's layer_norm
(tests/test_oracle.py).

Tolerance: the contraction's bound (3xTF32 1e-5, TF32 5e-3, relative Frobenius)
carried through the normalisation.  A row's GEMM error is relative to the
row's product A.B, and the normalisation divides by the row's standard
deviation, so the bound is scaled by cond = max over rows of
rms(A.B row) / std(row) (1 for zero-centred rows), times 2 for the LayerNorm's
own fp32 rounding and the affine parameters."""
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


def _cond(orc, a, b, bias):
    ab = orc.matmul_f64(a, b)
    c = ab + (np.asarray(bias, np.float64)[None, :] if bias is not None else 0.0)
    std = c.std(axis=1)
    rms = np.sqrt((ab ** 2).mean(axis=1))
    ok = std > 0
    return max(1.0, float((rms[ok] / std[ok]).max())) if ok.any() else 1.0


def _check(gpu, orc, a, b, bias, g, beta, eps, act, prec, transB=False):
    ref = orc.matmul_bias_norm_activation_f64(a, b, bias, g, beta, eps, act)
    bd = _dev(b.T.copy()).t() if transB else _dev(b)
    y = gpu.matmul_bias_norm_activation(_dev(a), bd, None if bias is None else _dev(bias),
                                        None if g is None else _dev(g),
                                        None if beta is None else _dev(beta), eps, act, prec)
    got = _host(y)
    assert np.isfinite(got).all()
    tol = 2 * TOL[prec] * _cond(orc, a, b, bias)
    err = orc.rel_frob(got, ref) if np.abs(ref).max() > 0 else float(np.abs(got).max())
    assert err <= tol, (err, tol)
    return got, ref


def test_kat_2x2(gpu):
    a = _dev(np.array([[1, 2], [3, 4]], np.float32))
    eye = _dev(np.eye(2, dtype=np.float32))
    for prec in (0, 1):
        y = _host(gpu.matmul_bias_norm_activation(a, eye, eps=0.0, act=gpu.ACT_RELU,
                                                  precision=prec))
        np.testing.assert_array_equal(y, [[0, 1], [0, 1]])
        g = _dev(np.array([2, 3], np.float32))
        b = _dev(np.array([0.5, -0.5], np.float32))
        t = _host(gpu.matmul_bias_norm_activation(a, eye, None, g, b, 0.0, gpu.ACT_TANH, prec))
        np.testing.assert_allclose(t, np.tanh([[-1.5, 2.5], [-1.5, 2.5]]), rtol=0, atol=1e-6)


# (m, n, k): ragged and scalar paths (n % 4 != 0), the reference's Auto
# threshold for its fused order (m >= 128, k >= 128, n >= 32), rows kept on
# chip and rows re-read (n > 16384), the small-M contraction path (m <= 16)
SHAPES = [(1, 1, 1), (7, 33, 19), (128, 256, 128), (300, 1000, 257), (16, 512, 4096),
          (64, 2048, 64), (33, 4096, 32), (17, 8192, 16), (40, 12000, 48), (50, 16385, 32),
          (64, 20000, 64), (2048, 1024, 1024)]


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("prec", [0, 1])
def test_shapes_affine_relu(gpu, orc, m, n, k, prec):
    a = orc.normal((m, k), 31, 1)
    b = orc.normal((k, n), 31, 2)
    bias = orc.normal((n,), 31, 3)
    g = orc.normal((n,), 31, 4)
    beta = orc.normal((n,), 31, 5)
    got, ref = _check(gpu, orc, a, b, bias, g, beta, 1e-5, 1, prec)
    # zero pattern: disagreements only where the exact pre-activation is within
    # the tolerance band of 0
    pre = orc.matmul_bias_norm_activation_f64(a, b, bias, g, beta, 1e-5, 0)
    band = 2 * TOL[prec] * _cond(orc, a, b, bias) * max(1.0, float(np.abs(g).max()))
    bad = (got > 0) != (ref > 0)
    assert not (bad & (np.abs(pre) > band)).any()


@pytest.mark.parametrize("act", [0, 1, 2, 3])
@pytest.mark.parametrize("affine", [False, True])
def test_activations(gpu, orc, act, affine):
    m, n, k = 200, 384, 160
    a = orc.normal((m, k), 32, 1)
    b = orc.normal((k, n), 32, 2)
    bias = orc.normal((n,), 32, 3) if affine else None
    g = orc.normal((n,), 32, 4) if affine else None
    beta = orc.normal((n,), 32, 5) if affine else None
    _check(gpu, orc, a, b, bias, g, beta, 1e-5, act, 0)


def test_linear_weight_layout(gpu, orc):
    """nn::Linear::forward_fused_norm_activation (rustorch-nn/src/linear.rs:53-71)
    passes weight.t(): B arrives as a transposed [N, K] view."""
    a = orc.normal((256, 512), 33, 1)
    w = orc.normal((768, 512), 33, 2)
    bias = orc.normal((768,), 33, 3)
    for prec in (0, 1):
        _check(gpu, orc, a, np.ascontiguousarray(w.T), bias, None, None, 1e-5, 3, prec,
               transB=True)


def test_large_offset_rows(gpu, orc):
    """Rows whose mean is 1000x their spread: the two-pass variance keeps them
    exact where the one-pass E[x^2] - E[x]^2 in f32 loses them."""
    m, n, k = 64, 1024, 64
    a = orc.normal((m, k), 34, 1)
    b = orc.normal((k, n), 34, 2)
    bias = (orc.normal((n,), 34, 3) + 8000.0).astype(np.float32)
    # fp32 storage of C (values near 8000, ulp 2^-10) is the floor here
    ref = orc.matmul_bias_norm_activation_f64(a, b, bias, None, None, 1e-5, 0)
    y = _host(gpu.matmul_bias_norm_activation(_dev(a), _dev(b), _dev(bias), eps=1e-5,
                                              precision=0))
    assert np.isfinite(y).all()
    assert orc.rel_frob(y, ref) <= 1e-4


def test_k_zero_and_empty(gpu, orc):
    """K = 0 gives C = bias (the reference's matmul of empty inner dims), then
    the normalisation; M = 0 / N = 0 give empty results without a launch."""
    bias = orc.normal((40,), 35, 1)
    a = torch.empty((3, 0), device="cuda")
    b = torch.empty((0, 40), device="cuda")
    y = _host(gpu.matmul_bias_norm_activation(a, b, _dev(bias), act=gpu.ACT_NONE))
    ref = orc.layer_norm(np.tile(bias, (3, 1)), None, None, 1e-5)
    np.testing.assert_allclose(y, ref, rtol=0, atol=1e-5)
    e = gpu.matmul_bias_norm_activation(torch.empty((0, 8), device="cuda"),
                                        torch.zeros((8, 5), device="cuda"))
    assert tuple(e.shape) == (0, 5)
    e2 = gpu.matmul_bias_norm_activation(torch.zeros((4, 8), device="cuda"),
                                         torch.zeros((8, 0), device="cuda"))
    assert tuple(e2.shape) == (4, 0)


def test_rejects_bad_parameters(gpu):
    a = torch.zeros((4, 8), device="cuda")
    b = torch.zeros((8, 5), device="cuda")
    with pytest.raises(ValueError):
        gpu.matmul_bias_norm_activation(a, b, norm_weight=torch.zeros(4, device="cuda"))
    with pytest.raises(gpu.RtbError):
        gpu.matmul_bias_norm_activation(a, b, act=7)


# d picks the kernel: one warp per row (<= 1024, scalar <= 512), 64/128/256
# threads per row in registers (<= 2048/4096/8192), the bulk-copy ring
# (<= 16384), plain staged rows (unaligned), rows re-read beyond 16384
@pytest.mark.parametrize("rows,d", [(1, 1), (3, 5), (9, 500), (1000, 768), (5, 1500), (7, 3000),
                                    (300, 4096), (3, 6000), (37, 4097), (8, 16384), (4, 16388),
                                    (2, 40000)])
@pytest.mark.parametrize("act", [0, 2])
def test_layer_norm(gpu, orc, rows, d, act):
    """ops::layer_norm alone against the f64 restatement: only fp32 rounding is
    left, so the bound is 1e-6 relative Frobenius."""
    x = orc.normal((rows, d), 36, 1) * 3 + 0.5
    g = orc.normal((d,), 36, 2)
    b = orc.normal((d,), 36, 3)
    ref = orc.matmul_bias_norm_activation_f64(x, np.eye(d, dtype=np.float32), None, g, b, 1e-5,
                                              act) if d <= 4097 else None
    if ref is None:  # avoid a d x d identity: normalise in numpy f64
        x64 = x.astype(np.float64)
        mu = x64.mean(1, keepdims=True)
        ref = (x64 - mu) / np.sqrt(((x64 - mu) ** 2).mean(1, keepdims=True) + 1e-5) * g + b
        if act == 2:
            ref = 1 / (1 + np.exp(-ref))
    y = _host(gpu.layer_norm(_dev(x), _dev(g), _dev(b), 1e-5, act))
    assert orc.rel_frob(y, ref) <= 1e-6


def test_layer_norm_in_place_strided_3d(gpu, orc):
    x = orc.normal((4, 6, 520), 37, 1)
    ref = orc.layer_norm(x.reshape(-1, 520), None, None, 1e-5).reshape(x.shape)
    t = _dev(x)
    gpu.layer_norm(t, out=t)
    np.testing.assert_allclose(_host(t), ref, rtol=0, atol=2e-5)
    # rows of a wider matrix (leading dimension 600 > d = 520)
    wide = _dev(np.pad(x.reshape(-1, 520), ((0, 0), (0, 80))))
    y = gpu.layer_norm(wide[:, :520])
    np.testing.assert_allclose(_host(y), ref.reshape(-1, 520), rtol=0, atol=2e-5)
