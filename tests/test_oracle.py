"""The oracle pinned to the reference's own known-answer tests and checked
against an independent float64 computation (CPU only)."""
import numpy as np
import pytest
import torch


def test_kat_matmul_2x2(orc, kats):
    k = kats["matmul_2x2"]
    a = np.array(k["a"], np.float32).reshape(k["a_shape"])
    b = np.array(k["b"], np.float32).reshape(k["b_shape"])
    c, choice = orc.matmul(a, b)
    assert choice == 0  # 2x2 is below the parallel-core thresholds -> sgemm
    assert np.max(np.abs(c.reshape(-1) - np.array(k["expected"]))) < k["abs_tol"]
    pc = orc.matmul_parallel_core(a, b)
    assert np.max(np.abs(pc.reshape(-1) - np.array(k["expected"]))) < k["abs_tol"]


def test_kat_conv2d(orc, kats):
    k = kats["conv2d_3x3_k2"]
    x = np.array(k["x"], np.float32).reshape(k["x_shape"])
    w = np.array(k["w"], np.float32).reshape(k["w_shape"])
    y, choice = orc.conv2d(x, w, tuple(k["stride"]), tuple(k["padding"]))
    assert choice == 0  # work < 65536 -> direct f64 path
    assert np.max(np.abs(y.reshape(-1) - np.array(k["expected"]))) < k["abs_tol"]
    yi = np.empty_like(y)
    # the im2col path must agree on the same case
    yi = orc.conv2d_direct(x, w, tuple(k["stride"]), tuple(k["padding"]))
    np.testing.assert_array_equal(yi, y)


def test_kat_jit_conv_relu(orc, kats):
    k = kats["jit_conv2d_relu_ones"]
    x = np.full(k["x_shape"], k["x_fill"], np.float32)
    w = np.full(k["w_shape"], k["w_fill"], np.float32)
    y, _ = orc.conv2d_bias_relu(x, w, None, tuple(k["stride"]), tuple(k["padding"]))
    assert list(y.shape) == k["out_shape"]
    assert abs(y.reshape(-1)[0] - k["expected_first"]) < k["abs_tol"]


def test_kat_bench_matmul_ones(orc, kats):
    k = kats["bench_matmul_ones"]
    a = np.full((k["m"], k["k"]), k["a_fill"], np.float32)
    b = np.full((k["k"], k["n"]), k["b_fill"], np.float32)
    c, _ = orc.matmul(a, b)
    assert np.all(c == k["expected_all"])


def test_kat_bench_conv_fill(orc, kats):
    k = kats["bench_conv2d_fill"]
    x = np.full(k["x_shape"], k["x_fill"], np.float32)
    w = np.full(k["w_shape"], k["w_fill"], np.float32)
    y, choice = orc.conv2d(x, w, tuple(k["stride"]), tuple(k["padding"]))
    assert choice == 1  # im2col; k = 144 < 256 -> sgemm
    interior = y[:, :, 1:-1, 1:-1]
    assert np.max(np.abs(interior / k["expected_interior"] - 1.0)) < k["rel_tol"]


def test_kat_deterministic_unit(orc, kats):
    k = kats["deterministic_unit"]
    got = [orc.unit(i, k["seed"]) for i in k["idx"]]
    assert got == [np.float32(v) for v in k["expected"]]


def test_auto_dispatch_rule(orc):
    # should_use_parallel_auto: m >= 128 && k >= 256 && n <= 128
    assert orc.lib().orc_matmul_auto_parallel(25088, 1152, 128) == 1  # conv cfg im2col GEMM
    assert orc.lib().orc_matmul_auto_parallel(1024, 1024, 1024) == 0
    assert orc.lib().orc_matmul_auto_parallel(127, 1024, 64) == 0
    assert orc.lib().orc_matmul_auto_parallel(128, 255, 64) == 0


def _np_parallel_core(a, b, bias=None):
    """Independent restatement of matmul_cpu_parallel_core in numpy float32
    (separate multiply and add, sequential over k, unrolled by 8 like the
    reference: the order of additions is identical)."""
    m, k = a.shape
    n = b.shape[1]
    s = np.tile(bias.astype(np.float32), (m, 1)) if bias is not None else np.zeros((m, n), np.float32)
    for p in range(k):
        s = (s + (a[:, p:p + 1] * b[p:p + 1, :]).astype(np.float32)).astype(np.float32)
    return s


def test_parallel_core_bit_exact(orc):
    rng = np.random.default_rng(5)
    a = rng.standard_normal((9, 37)).astype(np.float32)
    b = rng.standard_normal((37, 11)).astype(np.float32)
    bias = rng.standard_normal(11).astype(np.float32)
    np.testing.assert_array_equal(orc.matmul_parallel_core(a, b), _np_parallel_core(a, b))
    np.testing.assert_array_equal(orc.matmul_parallel_core(a, b, bias), _np_parallel_core(a, b, bias))


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (7, 300, 5), (130, 257, 64), (64, 600, 200)])
def test_matmul_vs_f64(orc, m, k, n):
    a = orc.normal((m, k), 11, 1)
    b = orc.normal((k, n), 11, 2)
    ref = torch.from_numpy(a).double() @ torch.from_numpy(b).double()
    c, _ = orc.matmul(a, b)
    assert orc.rel_frob(c, ref.numpy()) < 1e-6
    c64 = orc.matmul_f64(a, b)
    np.testing.assert_allclose(c64, ref.numpy(), rtol=1e-12, atol=1e-12)
    rows = np.array([0, m - 1]), np.array([n - 1, 0])
    np.testing.assert_allclose(orc.matmul_f64_sampled(a, b, *rows), ref.numpy()[rows], rtol=1e-12)


@pytest.mark.parametrize("shape,wshape,stride,pad", [
    ((2, 3, 9, 7), (4, 3, 3, 3), (1, 1), (1, 1)),
    ((1, 5, 11, 11), (6, 5, 3, 3), (2, 2), (1, 1)),
    ((2, 4, 8, 8), (3, 4, 1, 1), (2, 2), (0, 0)),
    ((1, 3, 15, 13), (2, 3, 7, 7), (2, 2), (3, 3)),
    ((2, 16, 6, 6), (8, 16, 3, 3), (1, 1), (0, 2)),
])
def test_conv_vs_torch_f64(orc, shape, wshape, stride, pad):
    x = orc.normal(shape, 3, 1)
    w = orc.normal(wshape, 3, 2)
    ref = torch.nn.functional.conv2d(torch.from_numpy(x).double(), torch.from_numpy(w).double(),
                                     stride=stride, padding=pad).numpy()
    y, _ = orc.conv2d(x, w, stride, pad)
    assert orc.rel_frob(y, ref) < 1e-6
    np.testing.assert_allclose(orc.conv2d_f64(x, w, stride, pad), ref, rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(orc.conv2d_direct(x, w, stride, pad), ref, rtol=1e-6, atol=1e-6)


def test_pooling_vs_torch(orc):
    x = orc.normal((2, 3, 13, 11), 4, 1)
    y = orc.max_pool2d(x, (3, 3), (2, 2), (1, 1))
    ref = torch.nn.functional.max_pool2d(torch.from_numpy(x), 3, 2, 1).numpy()
    np.testing.assert_array_equal(y, ref)
    g = orc.global_avg_pool(x)
    np.testing.assert_allclose(g, x.astype(np.float64).mean(axis=(2, 3)), rtol=1e-6)


def test_relu_nan_and_bias(orc):
    x = np.array([-1.0, 0.0, 2.0, np.nan], np.float32)
    np.testing.assert_array_equal(orc.relu(x), np.array([0, 0, 2, 0], np.float32))
    y = np.zeros((1, 2, 2, 2), np.float32)
    out = orc.add_bias_nchw(y, np.array([1.0, -2.0], np.float32))
    assert np.all(out[0, 0] == 1.0) and np.all(out[0, 1] == -2.0)


def test_prng_distribution(orc):
    z = orc.normal((200000,), 0, 0)
    assert abs(float(z.mean())) < 0.01 and abs(float(z.std()) - 1.0) < 0.01
    u = orc.uniform((200000,), 1, 3, -0.1, 0.1)
    assert u.min() >= -0.1 and u.max() <= 0.1 and abs(float(u.mean())) < 1e-3
    # deterministic and keyed by (seed, tensor id)
    np.testing.assert_array_equal(orc.normal((17,), 4, 2), orc.normal((17,), 4, 2))
    assert not np.array_equal(orc.normal((17,), 4, 2), orc.normal((17,), 4, 3))


def test_matmul_backward_kat(orc, kats):
    """MatmulBackward restated (ops.rs:529-570) against the reference's test
    (loss = sum(a . b), so the incoming gradient is all ones)."""
    k = kats["matmul_backward_2x2"]
    a = np.array(k["a"], np.float32).reshape(k["a_shape"])
    b = np.array(k["b"], np.float32).reshape(k["b_shape"])
    ga, gb = orc.matmul_backward_f64(a, b, np.ones((a.shape[0], b.shape[1])))
    assert np.max(np.abs(ga.reshape(-1) - k["expected_grad_a"])) < k["abs_tol"]
    assert np.max(np.abs(gb.reshape(-1) - k["expected_grad_b"])) < k["abs_tol"]


@pytest.mark.parametrize("stride,pad", [((1, 1), (1, 0)), ((2, 2), (1, 1)), ((2, 1), (0, 2))])
def test_conv_backward_adjoint(orc, stride, pad):
    """The Conv2dBackward restatements (conv.rs:336-502) are the adjoints of the
    pinned forward conv: <conv(x, w), g> = <x, grad_input(g, w)> = <w, grad_weight(x, g)>."""
    x = orc.normal((2, 3, 9, 11), 1, 1)
    w = orc.normal((4, 3, 3, 2), 1, 2)
    y = orc.conv2d_f64(x, w, stride, pad)
    g = orc.normal(y.shape, 1, 3)
    gx = orc.conv2d_grad_input_f64(g, w, x.shape, stride, pad)
    gw = orc.conv2d_grad_weight_f64(x, g, w.shape, stride, pad)
    lhs = float((y * g.astype(np.float64)).sum())
    assert abs(float((x.astype(np.float64) * gx).sum()) - lhs) <= 1e-10 * max(1.0, abs(lhs))
    assert abs(float((w.astype(np.float64) * gw).sum()) - lhs) <= 1e-10 * max(1.0, abs(lhs))


def test_layer_norm_kat_2x2(orc):
    """matmul_bias_norm_activation on [[1,2],[3,4]] . I: each row has mean m and
    variance 1/4 under the reference's formula (rustorch-core/src/ops/norm.rs:
    660-667), so with eps 0 it normalises to [-1, 1] exactly."""
    a = np.array([[1, 2], [3, 4]], np.float32)
    eye = np.eye(2, dtype=np.float32)
    y = orc.matmul_bias_norm_activation(a, eye, eps=0.0, act=0)
    np.testing.assert_array_equal(y, [[-1, 1], [-1, 1]])
    np.testing.assert_array_equal(orc.matmul_bias_norm_activation(a, eye, eps=0.0, act=1),
                                  [[0, 1], [0, 1]])
    g = np.array([2, 3], np.float32)
    b = np.array([0.5, -0.5], np.float32)
    t = orc.matmul_bias_norm_activation(a, eye, None, g, b, eps=0.0, act=3)
    np.testing.assert_allclose(t, np.tanh([[-1.5, 2.5], [-1.5, 2.5]]), rtol=0, atol=1e-7)
    s = orc.matmul_bias_norm_activation(a, eye, eps=0.0, act=2)
    np.testing.assert_allclose(s, 1 / (1 + np.exp([[1.0, -1.0], [1.0, -1.0]])), rtol=0, atol=1e-7)
    f = orc.matmul_bias_norm_activation_f64(a, eye, None, g, b, eps=0.0, act=3)
    np.testing.assert_allclose(f, np.tanh([[-1.5, 2.5], [-1.5, 2.5]]), rtol=0, atol=1e-15)


@pytest.mark.parametrize("rows,d", [(1, 1), (5, 7), (64, 1000), (33, 4096)])
def test_layer_norm_ref_vs_torch_and_f64(orc, rows, d):
    """The reference formula (f32, one pass) against torch's layer_norm and the
    f64 two-pass restatement on zero-centred rows, where E[x^2] - E[x]^2 does
    not cancel."""
    x = orc.normal((rows, d), 21, 1)
    g = orc.normal((d,), 21, 2)
    b = orc.normal((d,), 21, 3)
    y = orc.layer_norm(x, g, b, 1e-5)
    t = torch.nn.functional.layer_norm(torch.from_numpy(x), (d,), torch.from_numpy(g),
                                       torch.from_numpy(b), 1e-5).numpy()
    x64 = x.astype(np.float64)
    mu = x64.mean(1, keepdims=True)
    ref = (x64 - mu) / np.sqrt(((x64 - mu) ** 2).mean(1, keepdims=True) + 1e-5) * g + b
    assert np.abs(y - t).max() < 1e-4
    assert orc.rel_frob(y, ref) < 1e-5
    f = orc.matmul_bias_norm_activation_f64(x, np.eye(d, dtype=np.float32), None, g, b, 1e-5, 0)
    assert np.abs(f - ref).max() < 1e-9


def test_layer_norm_reference_cancellation(orc):
    """Rows with |mean| >> std: the reference's E[x^2] - E[x]^2 in f32 loses the
    variance (ops/norm.rs:665) -- here it comes out negative and the rows turn
    to NaN -- while the f64 two-pass value stays exact.  The CUDA path is held
    to the exact value."""
    x = (orc.normal((16, 1024), 22, 1) + 1000.0).astype(np.float32)
    x64 = x.astype(np.float64)
    mu = x64.mean(1, keepdims=True)
    ref = (x64 - mu) / np.sqrt(((x64 - mu) ** 2).mean(1, keepdims=True) + 1e-5)
    y = orc.layer_norm(x, None, None, 1e-5)
    f = orc.matmul_bias_norm_activation_f64(x, np.eye(1024, dtype=np.float32), None, None, None,
                                            1e-5, 0)
    assert np.abs(f - ref).max() < 1e-9
    assert not np.isfinite(y).all() or orc.rel_frob(y, ref) > 1e-3


def test_activation_restatement(orc):
    x = orc.normal((4096,), 23, 1) * 4
    x[:3] = [np.nan, 0.0, -0.0]
    np.testing.assert_array_equal(orc.activation(x, 1)[3:], np.maximum(x[3:], 0))
    assert orc.activation(x, 1)[0] == 0.0  # f32::max(NaN, 0) = 0
    np.testing.assert_allclose(orc.activation(x, 2)[1:], 1 / (1 + np.exp(-x[1:].astype(np.float64))),
                               rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(orc.activation(x, 3)[1:], np.tanh(x[1:].astype(np.float64)),
                               rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("N,C,H,W,Co,kh,kw,ph,pw", [
    (2, 3, 23, 20, 5, 7, 7, 3, 3),   # the ResNet stem's form, odd sizes
    (1, 1, 9, 9, 4, 4, 5, 1, 2),     # even and odd kernel extents
    (2, 4, 10, 11, 3, 3, 3, 1, 1),
    (1, 2, 8, 8, 2, 2, 2, 0, 0),
])
def test_space_to_depth_identity(orc, N, C, H, W, Co, kh, kw, ph, pw):
    """The identity behind the CUDA path for stride-2 convs over <= 4 channels:
    conv(x, w, stride 2, pad p) equals the stride-1, unpadded conv of the
    16-channel space-to-depth input x2[n][(pr*2+pc)*4+c][hs][ws] =
    x[n][c][2hs+pr-ph][2ws+pc-pw] with the kernel w2[co][(pr*2+pc)*4+c][R][S] =
    w[co][c][2R+pr][2S+pc] (zero outside), Hs = Ho + ceil(kh/2) - 1."""
    x = orc.normal((N, C, H, W), 41, 1)
    w = orc.normal((Co, C, kh, kw), 41, 2)
    ref = orc.conv2d_f64(x, w, (2, 2), (ph, pw))
    Ho, Wo = ref.shape[2:]
    kh2, kw2 = (kh + 1) // 2, (kw + 1) // 2
    Hs, Ws = Ho + kh2 - 1, Wo + kw2 - 1
    xp = np.zeros((N, C, 2 * Hs + 2, 2 * Ws + 2), np.float32)
    hh, ww = min(H, 2 * Hs + 2 - ph), min(W, 2 * Ws + 2 - pw)
    xp[:, :, ph:ph + hh, pw:pw + ww] = x[:, :, :hh, :ww]
    x2 = np.zeros((N, 16, Hs, Ws), np.float32)
    w2 = np.zeros((Co, 16, kh2, kw2), np.float32)
    for pr in range(2):
        for pc in range(2):
            ch = (pr * 2 + pc) * 4
            x2[:, ch:ch + C] = xp[:, :, pr:pr + 2 * Hs:2, pc:pc + 2 * Ws:2]
            sub = w[:, :, pr::2, pc::2]
            w2[:, ch:ch + C, :sub.shape[2], :sub.shape[3]] = sub
    got = orc.conv2d_f64(x2, w2, (1, 1), (0, 0))
    assert got.shape == ref.shape
    np.testing.assert_allclose(got, ref, rtol=0, atol=1e-9)
