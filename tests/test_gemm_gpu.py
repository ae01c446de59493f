"""GEMM parity on the B200: the tcgen05 kernels (through the C ABI) against the
oracle's restatement of the reference's CPU matmul, on seeded inputs.

Tolerances (relative Frobenius error against the f64-accumulated oracle):
3xTF32 <= 1e-5, TF32 <= 5e-3.  ReLU zero patterns must agree wherever the
f64 pre-activation satisfies |x| >= 1e-5."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {0: 1e-5, 1: 5e-3}  # PREC_3XTF32, PREC_TF32


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def _relu_pattern_ok(y, pre64, prec=0):
    band = 1e-5 if prec == 0 else 1e-2 * float(np.sqrt(np.mean(pre64 * pre64)))
    mask = np.abs(pre64) >= band
    return np.array_equal((y > 0)[mask], (pre64 > 0)[mask])


def test_kat_matmul_2x2(gpu, kats):
    k = kats["matmul_2x2"]
    a = np.array(k["a"], np.float32).reshape(k["a_shape"])
    b = np.array(k["b"], np.float32).reshape(k["b_shape"])
    for prec in (0, 1):
        c = _host(gpu.sgemm(_dev(a), _dev(b), precision=prec))
        assert np.max(np.abs(c.reshape(-1) - np.array(k["expected"]))) < k["abs_tol"]


def test_kat_bench_ones(gpu, kats):
    k = kats["bench_matmul_ones"]
    a = torch.ones((k["m"], k["k"]), device="cuda")
    b = torch.ones((k["k"], k["n"]), device="cuda")
    for prec in (0, 1):
        c = _host(gpu.sgemm(a, b, precision=prec))
        assert np.all(c == k["expected_all"])


@pytest.mark.parametrize("prec", [0, 1])
def test_gemm_1024_seed0(gpu, orc, prec):
    """The 1024^3 f32 matmul workload (A, B ~ N(0,1), seed 0)."""
    a = orc.normal((1024, 1024), 0, 0)
    b = orc.normal((1024, 1024), 0, 1)
    ref = orc.matmul_f64(a, b)
    c = _host(gpu.sgemm(_dev(a), _dev(b), precision=prec))
    err = orc.rel_frob(c, ref)
    assert err <= TOL[prec], err
    # and against the f32 restatement of the reference's own kernel
    c32, choice = orc.matmul(a, b)
    assert choice == 0
    assert orc.rel_frob(c, c32.astype(np.float64)) <= 2 * TOL[prec]


@pytest.mark.parametrize("m,n,k", [
    (1, 1, 1), (3, 5, 7), (17, 33, 65), (128, 128, 32), (129, 257, 31), (200, 1000, 512),
    (64, 64, 2048), (300, 96, 100), (1, 4096, 256), (2048, 8, 64), (513, 130, 1027)])
@pytest.mark.parametrize("prec", [0, 1])
def test_gemm_shapes(gpu, orc, m, n, k, prec):
    a = orc.normal((m, k), 7, 1)
    b = orc.normal((k, n), 7, 2)
    ref = orc.matmul_f64(a, b)
    c = _host(gpu.sgemm(_dev(a), _dev(b), precision=prec))
    assert c.shape == (m, n)
    assert orc.rel_frob(c, ref) <= TOL[prec]


@pytest.mark.parametrize("prec", [0, 1])
def test_linear_transposed_weight_bias_relu(gpu, orc, prec):
    """nn::Linear: x.matmul(w.t()) + b with ReLU; w.t() is passed as a
    transposed view (K-major B) without a copy."""
    x = orc.normal((333, 256), 2, 1)
    w = orc.uniform((500, 256), 2, 2, -0.1, 0.1)
    b = orc.uniform((500,), 2, 3, -0.1, 0.1)
    pre = orc.matmul_f64(x, np.ascontiguousarray(w.T)) + b.astype(np.float64)
    wt = _dev(w).t()
    assert wt.stride(0) == 1
    y = _host(gpu.sgemm(_dev(x), wt, bias=_dev(b), act=gpu.ACT_RELU, precision=prec))
    assert orc.rel_frob(y, np.maximum(pre, 0)) <= TOL[prec]
    assert _relu_pattern_ok(y, pre, prec)
    ref32 = orc.linear(x, w, b, relu=True)
    assert orc.rel_frob(y, ref32.astype(np.float64)) <= 2 * TOL[prec] + 1e-6


def test_matmul_fused_none_bias(gpu, orc):
    a = orc.normal((100, 70), 3, 1)
    b = orc.normal((70, 60), 3, 2)
    bias = orc.normal((60,), 3, 3)
    ref = orc.matmul_f64(a, b) + bias.astype(np.float64)
    y = _host(gpu.sgemm(_dev(a), _dev(b), bias=_dev(bias)))
    assert orc.rel_frob(y, ref) <= 1e-5
    y32 = orc.matmul_fused(a, b, bias, 0)
    assert orc.rel_frob(y32, ref) <= 1e-6


def test_transposed_a_and_strided(gpu, orc):
    a = orc.normal((96, 80), 9, 1)
    b = orc.normal((80, 72), 9, 2)
    ref = orc.matmul_f64(a, b)
    at = _dev(np.ascontiguousarray(a.T)).t()          # stride (1, 96): transA path
    c = _host(gpu.sgemm(at, _dev(b)))
    assert orc.rel_frob(c, ref) <= 1e-5
    big = _dev(np.pad(a, ((0, 0), (0, 3))))[:, :80]   # lda = 83: unaligned -> packed
    c = _host(gpu.sgemm(big, _dev(b)))
    assert orc.rel_frob(c, ref) <= 1e-5


def test_k_zero_gives_bias(gpu):
    a = torch.empty((5, 0), device="cuda")
    b = torch.empty((0, 7), device="cuda")
    bias = torch.arange(7, dtype=torch.float32, device="cuda") - 3
    c = _host(gpu.sgemm(a, b, bias=bias, act=gpu.ACT_RELU))
    assert np.array_equal(c, np.tile(np.maximum(np.arange(7) - 3, 0), (5, 1)).astype(np.float32))
    c = _host(gpu.sgemm(a, b))
    assert np.all(c == 0)


def test_empty_m_n(gpu):
    a = torch.empty((0, 4), device="cuda")
    b = torch.ones((4, 3), device="cuda")
    assert gpu.sgemm(a, b).shape == (0, 3)


def test_errors(gpu):
    a = torch.ones((4, 3), device="cuda")
    with pytest.raises(ValueError, match="Matmul dimension mismatch"):
        gpu.sgemm(a, torch.ones((4, 3), device="cuda"))
    with pytest.raises(ValueError, match="Matmul only supports 2D"):
        gpu.sgemm(torch.ones((2, 2, 2), device="cuda"), a)
    with pytest.raises(gpu.RtbError) as e:
        gpu.sgemm(a, torch.ones((3, 4), device="cuda"), act=7)
    assert e.value.status == 1  # unknown activation: RTB_E_INVALID


def _act64(pre, act):
    if act == 2:
        return 1.0 / (1.0 + np.exp(-pre))
    if act == 3:
        return np.tanh(pre)
    return np.maximum(pre, 0.0) if act == 1 else pre


@pytest.mark.parametrize("act", [2, 3])
@pytest.mark.parametrize("prec", [0, 1])
@pytest.mark.parametrize("m,n,k,trans_b", [
    (4096, 4096, 1024, 1),   # the MLP's first Linear (W^T view, K-major B)
    (4096, 1024, 4096, 1),   # its last Linear
    (333, 500, 256, 0),      # ragged tiles, row-major rhs
    (16, 1000, 777, 0),      # the small-M path
    (5, 7, 0, 0),            # K = 0: act(bias)
])
def test_matmul_fused_sigmoid_tanh(gpu, orc, act, prec, m, n, k, trans_b):
    """ops::matmul_fused with Activation::Sigmoid / Tanh (rustorch-core/src/
    ops.rs:1703-1708): act(A.B + bias) in the GEMM epilogue.  Sigmoid and tanh
    have slopes <= 1/4 and <= 1, so the contraction's error bound carries
    over: relative Frobenius error <= 1e-5 (3xTF32) / 5e-3 (TF32) against
    float64, with 1/(1+exp(-x)) and tanh(x) evaluated in float64."""
    a = orc.normal((m, k), 12, 1, 0.0, 1.0 / np.sqrt(max(k, 1)))
    w = orc.normal((n, k) if trans_b else (k, n), 12, 2)
    b = w.T if trans_b else w
    bias = orc.uniform((n,), 12, 3, -0.5, 0.5)
    rows = np.arange(m) if m <= 512 else np.r_[0:40, m // 2:m // 2 + 24, m - 40:m]
    pre = (orc.matmul_f64(a[rows], np.ascontiguousarray(b)) if k else
           np.zeros((len(rows), n))) + bias.astype(np.float64)
    bd = _dev(w).t() if trans_b else _dev(w)
    y = _host(gpu.sgemm(_dev(a), bd, bias=_dev(bias), act=act, precision=prec))
    tol = TOL[0] if (m <= 16 or k == 0) else TOL[prec]  # small-M / K=0: exact fp32 in both modes
    assert orc.rel_frob(y[rows], _act64(pre, act)) <= tol
    if k and m <= 512:
        # and the reference's own staged f32 path (matmul -> add bias -> act)
        y32 = orc.matmul_fused(a, np.ascontiguousarray(b), bias, act)
        assert orc.rel_frob(y, y32.astype(np.float64)) <= 2 * tol


@pytest.mark.parametrize("act", [2, 3])
def test_conv_sigmoid_tanh_epilogue(gpu, orc, act):
    """The conv epilogue (NCHW and NHWC stores) applies the same activations."""
    x = orc.normal((4, 64, 20, 20), 13, 1)
    w = orc.normal((96, 64, 3, 3), 13, 2, 0.0, float(np.sqrt(2.0 / 576)))
    bias = orc.uniform((96,), 13, 3, -0.2, 0.2)
    pre = orc.conv2d_f64(x, w, (1, 1), (1, 1)) + bias.astype(np.float64)[None, :, None, None]
    y = _host(gpu.conv2d_fwd(_dev(x), _dev(w), _dev(bias), (1, 1), (1, 1), act=act))
    assert orc.rel_frob(y, _act64(pre, act)) <= TOL[0]
    yh = _host(gpu.conv2d_fwd(_dev(x), _dev(w), _dev(bias), (1, 1), (1, 1), act=act,
                              y_layout=gpu.LAYOUT_NHWC))
    assert orc.rel_frob(yh.transpose(0, 3, 1, 2), _act64(pre, act)) <= TOL[0]


@pytest.mark.parametrize("prec", [0, 1])
def test_batched(gpu, orc, prec):
    a = orc.normal((3, 65, 40), 5, 1)
    b = orc.normal((3, 40, 33), 5, 2)
    c = _host(gpu.sgemm_batched(_dev(a), _dev(b), precision=prec))
    for i in range(3):
        assert orc.rel_frob(c[i], orc.matmul_f64(a[i], b[i])) <= TOL[prec]


@pytest.mark.parametrize("prec", [0, 1])
def test_batched_many_and_transposed_b(gpu, orc, prec):
    """rtb_sgemm_batched with 48 problems of ragged size, B given row-major
    [K,N] per batch and as Linear-style [N,K] per batch (transB=1, strided),
    a shared bias and ReLU, against looped 2-D float64 products (the
    reference's matmul is 2-D; its oracle for a batch is the loop)."""
    import ctypes
    bt, m, n, k = 48, 150, 72, 200
    a = orc.normal((bt, m, k), 14, 1)
    w = orc.normal((bt, n, k), 14, 2)          # [N,K] per batch (transposed operand)
    bias = orc.uniform((n,), 14, 3, -0.5, 0.5)
    pre = np.stack([orc.matmul_f64(a[i], np.ascontiguousarray(w[i].T)) for i in range(bt)])
    pre += bias.astype(np.float64)
    ref = np.maximum(pre, 0.0)
    da, dw, dbias = _dev(a), _dev(w), _dev(bias)
    ctx = gpu.get_context(0)

    def run(bptr, ldb, stride_b, trans_b):
        c = torch.empty((bt, m, n), device="cuda")
        gpu.call("rtb_sgemm_batched", ctx.handle, bt, m, n, k, ctypes.c_void_p(da.data_ptr()), k,
                 m * k, 0, ctypes.c_void_p(bptr), ldb, stride_b, trans_b,
                 ctypes.c_void_p(dbias.data_ptr()), gpu.ACT_RELU, ctypes.c_void_p(c.data_ptr()),
                 n, m * n, prec, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        return _host(c)

    ct = run(dw.data_ptr(), k, n * k, 1)
    assert orc.rel_frob(ct, ref) <= TOL[prec]
    bkn = _dev(np.ascontiguousarray(w.transpose(0, 2, 1)))   # [K,N] per batch
    cn = run(bkn.data_ptr(), n, k * n, 0)
    assert orc.rel_frob(cn, ref) <= TOL[prec]


def test_skinny_8192_sampled(gpu, orc):
    """Skinny M=16 with N=K=8192 at full size; checked on sampled entries
    against f64 dot products (a full f64 GEMM would take minutes on the CPU)."""
    a = orc.normal((16, 8192), 4, 1)
    b = orc.normal((8192, 8192), 4, 2)
    c = _host(gpu.sgemm(_dev(a), _dev(b)))
    rng = np.random.default_rng(0)
    rows = rng.integers(0, 16, 4096)
    cols = rng.integers(0, 8192, 4096)
    ref = orc.matmul_f64_sampled(a, b, rows, cols)
    assert orc.rel_frob(c[rows, cols], ref) <= 1e-5


def test_square_4096_sampled_and_linearity(gpu, orc):
    a = orc.normal((4096, 4096), 4, 3)
    b = orc.normal((4096, 4096), 4, 4)
    da, db = _dev(a), _dev(b)
    c = gpu.sgemm(da, db)
    rng = np.random.default_rng(1)
    rows = rng.integers(0, 4096, 4096)
    cols = rng.integers(0, 4096, 4096)
    ref = orc.matmul_f64_sampled(a, b, rows, cols)
    assert orc.rel_frob(_host(c)[rows, cols], ref) <= 1e-5
    # linearity: A.(2B) == 2(A.B) exactly (scaling by 2 is exact in every split)
    c2 = gpu.sgemm(da, db * 2)
    assert torch.equal(c2, c * 2)


@pytest.mark.parametrize("prec", [0, 1])
def test_square_2048_k_split_schedule(gpu, orc, prec):
    """2048^3 (256 tiles on 148 SMs): the scheduler cuts the last 108 tiles
    into K pieces, several per CTA, whose fix-ups run while the CTA's next
    piece is in flight; sampled entries against float64."""
    a = orc.normal((2048, 2048), 4, 5)
    b = orc.normal((2048, 2048), 4, 6)
    c = _host(gpu.sgemm(_dev(a), _dev(b), precision=prec))
    rng = np.random.default_rng(7)
    rows = rng.integers(0, 2048, 8192)
    cols = rng.integers(0, 2048, 8192)
    ref = orc.matmul_f64_sampled(a, b, rows, cols)
    assert orc.rel_frob(c[rows, cols], ref) <= TOL[prec]


@pytest.mark.parametrize("n", [8192, 16384])
def test_square_large_sampled_and_linearity(gpu, orc, n):
    """The large square f32 matmuls of the sweep (8192^3, 16384^3; A, B ~ N(0,1),
    seed 4 as the bench uses them) at full size: 4096 sampled entries against
    float64 dot products, plus the exact identity A.(2B) == 2(A.B) over the
    whole of C (scaling by 2 is exact in every split and every sum)."""
    a = orc.normal((n, n), 4, 0)
    b = orc.normal((n, n), 4, 1)
    da, db = _dev(a), _dev(b)
    c = gpu.sgemm(da, db)
    rng = np.random.default_rng(n)
    rows = rng.integers(0, n, 4096)
    cols = rng.integers(0, n, 4096)
    ref = orc.matmul_f64_sampled(a, b, rows, cols)
    torch.cuda.synchronize()
    got = c[torch.from_numpy(rows).cuda(), torch.from_numpy(cols).cuda()].cpu().numpy()
    assert orc.rel_frob(got, ref) <= 1e-5
    del a
    db.mul_(2.0)
    c2 = gpu.sgemm(da, db)
    assert torch.equal(c2, c * 2)
    assert gpu.get_context(0).device_error() == 0


@pytest.mark.parametrize("k", [1024, 16384])
def test_all_positive_long_k(gpu, orc, k):
    """All-positive operands (no cancellation) are the hardest case for the
    tensor core's accumulation: the 3xTF32 error must stay under 1e-5 and must
    not grow with K (the accumulator is promoted to fp32 at a fixed interval)."""
    a = orc.uniform((256, k), 6, 1, 0.0, 1.0)
    b = orc.uniform((k, 256), 6, 2, 0.0, 1.0)
    ref = orc.matmul_f64(a, b)
    c = _host(gpu.sgemm(_dev(a), _dev(b), precision=0))
    assert orc.rel_frob(c, ref) <= 1e-5


def test_tf32_operand_truncation(gpu):
    """The 3xTF32 split relies on how the tensor core turns an fp32 operand
    into TF32: it keeps the top 10 explicit mantissa bits and drops the low 13
    (round toward zero).  x = 1 + 0.75 * 2^-10 is 1.0 truncated, 1 + 2^-10
    rounded; the product with 1.0 shows which one the hardware used."""
    x = 1.0 + 2.0 ** -11 + 2.0 ** -12
    # 128 rows: above the small-M threshold, so the tensor-core path runs
    for sign in (1.0, -1.0):
        a = torch.full((128, 1), sign * x, device="cuda")
        one = torch.ones((1, 1), device="cuda")
        ca = _host(gpu.sgemm(a, one, precision=gpu.PREC_TF32))
        cb = _host(gpu.sgemm(torch.ones((128, 1), device="cuda"), a[:1], precision=gpu.PREC_TF32))
        assert np.all(ca == sign * 1.0) and np.all(cb == sign * 1.0), (ca[0], cb[0])
        # and 3xTF32 recovers the full fp32 value
        c3 = _host(gpu.sgemm(a, one, precision=gpu.PREC_3XTF32))
        assert np.all(c3 == np.float32(sign * x)), c3[0]


@pytest.mark.parametrize("m", [1, 7, 8, 9, 16, 17, 32, 64])
@pytest.mark.parametrize("n,k", [(1, 1), (100, 31), (257, 1000), (1024, 4096), (300, 8192)])
@pytest.mark.parametrize("trans_b", [0, 1])
def test_small_m_path(gpu, orc, m, n, k, trans_b):
    """M <= 16 runs the CUDA-core small-M path (exact fp32 FMAs, B streamed
    once, the chunk sequence shared out to the CTAs with an ordered fix-up
    of blocks several CTAs touch; (300, 8192): two blocks shared by all 148
    CTAs); 17..64 check the switch to the tensor-core path: both B layouts
    (the matmul rhs [K,N] and Linear's transposed weight view of [N,K]), bias
    and ReLU, ragged N and K."""
    a = orc.normal((m, k), 9, 1)
    w = orc.normal((n, k), 9, 2) if trans_b else orc.normal((k, n), 9, 2)
    b = w.T if trans_b else w
    bias = orc.uniform((n,), 9, 3, -0.5, 0.5)
    pre = orc.matmul_f64(a, np.ascontiguousarray(b)) + bias.astype(np.float64)
    bd = _dev(w).t() if trans_b else _dev(w)
    for prec in (0, 1):
        y = _host(gpu.sgemm(_dev(a), bd, bias=_dev(bias), act=gpu.ACT_RELU, precision=prec))
        ref = np.maximum(pre, 0.0)
        tol_prec = 0 if m <= 16 else prec  # the small-M path is exact fp32 in both modes
        assert orc.rel_frob(y, ref) <= TOL[tol_prec]
        # outputs here are ~sqrt(K) in size: the 1e-5 zero band is scaled by
        # their rms (it is written for the O(1) outputs of the workloads)
        scale = max(1.0, float(np.sqrt(np.mean(pre * pre))))
        assert _relu_pattern_ok(y / scale, pre / scale, tol_prec)


@pytest.mark.parametrize("m", [16, 64, 256])
def test_small_m_skinny_8192(gpu, orc, m):
    """The skinny M x 8192 x 8192 workloads (M=16 on the small-M path, M=64
    and M=256 on the tensor cores) against float64 on a sample of columns."""
    a = orc.normal((m, 8192), 4, 0)
    b = orc.normal((8192, 8192), 4, 1)
    c = _host(gpu.sgemm(_dev(a), _dev(b)))
    cols = np.random.default_rng(2).integers(0, 8192, 256)
    ref = a.astype(np.float64) @ b[:, cols].astype(np.float64)
    assert orc.rel_frob(c[:, cols], ref) <= TOL[0]


def test_split_counters_across_launches_and_streams(gpu, orc):
    """Tail-split GEMMs (1024^3: 64 tiles cut into K pieces) and small-M split-K
    GEMMs count piece arrivals in per-stream, generation-tagged words that are
    never cleared: launches repeated on one stream and interleaved on two
    streams give bit-identical results."""
    a = orc.normal((1024, 1024), 40, 1)
    b = orc.normal((1024, 1024), 40, 2)
    s_m = orc.normal((8, 4096), 40, 3)
    s_b = orc.normal((4096, 2048), 40, 4)
    da, db, dsm, dsb = (torch.from_numpy(t).cuda() for t in (a, b, s_m, s_b))
    ref = gpu.sgemm(da, db).cpu().numpy()
    ref_s = gpu.sgemm(dsm, dsb).cpu().numpy()
    assert orc.rel_frob(ref, orc.matmul_f64(a, b)) <= 1e-5
    assert orc.rel_frob(ref_s, orc.matmul_f64(s_m, s_b)) <= 1e-5
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = []
    for i in range(6):
        with torch.cuda.stream(streams[i % 2]):
            outs.append((gpu.sgemm(da, db), gpu.sgemm(dsm, dsb)))
    torch.cuda.synchronize()
    for c, cs in outs:
        np.testing.assert_array_equal(c.cpu().numpy(), ref)
        np.testing.assert_array_equal(cs.cpu().numpy(), ref_s)
    assert gpu.get_context(0).device_error() == 0


def test_split_counters_per_thread_streams(gpu, orc):
    """Tail-split GEMMs (1024^3) and small-M split-K GEMMs launched from two
    host threads on cudaStreamPerThread (one handle, a different stream per
    thread, so launches may overlap): each launch counts its pieces in
    counters of its own, and every result is bit-identical to the same GEMM
    on an ordinary stream.  Also a stream made by rtb_stream_create and
    destroyed between uses (its counter block is released with it)."""
    import ctypes
    import threading
    a = orc.normal((1024, 1024), 41, 1)
    b = orc.normal((1024, 1024), 41, 2)
    s_m = orc.normal((8, 4096), 41, 3)
    s_b = orc.normal((4096, 2048), 41, 4)
    da, db, dsm, dsb = (torch.from_numpy(t).cuda() for t in (a, b, s_m, s_b))
    ref = gpu.sgemm(da, db).cpu().numpy()
    ref_s = gpu.sgemm(dsm, dsb).cpu().numpy()
    ctx = gpu.get_context(0)
    per_thread = ctypes.c_void_p(2)  # cudaStreamPerThread
    outs = [[torch.empty((1024, 1024), device="cuda") for _ in range(4)] for _ in range(2)]
    outs_s = [[torch.empty((8, 2048), device="cuda") for _ in range(4)] for _ in range(2)]
    torch.cuda.synchronize()
    errors = []

    def p(t):
        return ctypes.c_void_p(t.data_ptr())

    def work(t):
        try:
            for i in range(4):
                gpu.call("rtb_sgemm", ctx.handle, 1024, 1024, 1024, p(da), 1024, 0, p(db), 1024, 0,
                         None, 0, p(outs[t][i]), 1024, 0, per_thread)
                gpu.call("rtb_sgemm", ctx.handle, 8, 2048, 4096, p(dsm), 4096, 0, p(dsb), 2048, 0,
                         None, 0, p(outs_s[t][i]), 2048, 0, per_thread)
            gpu.call("rtb_stream_synchronize", ctx.handle, per_thread)
        except Exception as e:  # reported by the main thread
            errors.append(e)

    th = [threading.Thread(target=work, args=(t,)) for t in range(2)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    torch.cuda.synchronize()
    assert not errors, errors
    for t in range(2):
        for i in range(4):
            np.testing.assert_array_equal(outs[t][i].cpu().numpy(), ref)
            np.testing.assert_array_equal(outs_s[t][i].cpu().numpy(), ref_s)
    for _ in range(3):  # created, used, destroyed: a reused handle gets a fresh block
        h = ctypes.c_void_p()
        gpu.call("rtb_stream_create", ctx.handle, ctypes.byref(h))
        c = torch.empty((1024, 1024), device="cuda")
        gpu.call("rtb_sgemm", ctx.handle, 1024, 1024, 1024, p(da), 1024, 0, p(db), 1024, 0, None,
                 0, p(c), 1024, 0, h)
        gpu.call("rtb_stream_synchronize", ctx.handle, h)
        gpu.call("rtb_stream_destroy", ctx.handle, h)
        np.testing.assert_array_equal(c.cpu().numpy(), ref)
    assert ctx.device_error() == 0


def test_inputs_written_by_the_previous_kernel(gpu, orc):
    """The contraction, LayerNorm and small-M kernels are launched with
    programmatic stream serialization and wait (griddepcontrol.wait) for the
    previous kernel before reading: inputs that a torch kernel writes right
    before each call must be seen complete, every time."""
    torch.manual_seed(7)
    x = torch.randn(1024, 1024, device="cuda")
    y = torch.randn(1024, 1024, device="cuda")
    s = torch.randn(16, 4096, device="cuda")
    t = torch.randn(4096, 4096, device="cuda")
    for i in range(4):
        a = x * (i + 1.0)            # written by a torch kernel just before the call
        c = gpu.sgemm(a, y)
        ln = gpu.layer_norm(c * 0.5 + i)
        cs = gpu.sgemm(s * (i + 2.0), t)   # small-M path
        ref = (a.double() @ y.double())
        assert float((c.double() - ref).norm() / ref.norm()) <= 1e-5
        lref = torch.nn.functional.layer_norm((ref * 0.5 + i).float(), (1024,))
        assert float((ln - lref).norm() / lref.norm()) <= 1e-5
        sref = (s.double() * (i + 2.0)) @ t.double()
        assert float((cs.double() - sref).norm() / sref.norm()) <= 1e-5


def test_cuda_graph_capture_and_replay(gpu, orc):
    """A tail-split GEMM (1024^3), a small-M split-K GEMM and a conv captured
    into one CUDA graph and replayed with new inputs: under capture the split
    counters are the launch's own, zeroed by a memset node, so every replay
    elects its fix-up pieces afresh."""
    torch.manual_seed(11)
    a = torch.randn(1024, 1024, device="cuda")
    b = torch.randn(1024, 1024, device="cuda")
    sm = torch.randn(8, 4096, device="cuda")
    sb = torch.randn(4096, 2048, device="cuda")
    x = torch.randn(32, 128, 28, 28, device="cuda")
    w = torch.randn(128, 128, 3, 3, device="cuda") * 0.03
    bias = torch.randn(128, device="cuda") * 0.1
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up outside the capture
        for _ in range(2):
            gpu.sgemm(a, b)
            gpu.sgemm(sm, sb)
            gpu.conv2d_fwd(x, w, bias, (1, 1), (1, 1), act=gpu.ACT_RELU)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        c = gpu.sgemm(a, b)
        cs = gpu.sgemm(sm, sb)
        y = gpu.conv2d_fwd(x, w, bias, (1, 1), (1, 1), act=gpu.ACT_RELU)
    for i in range(3):
        a.mul_(-1.0 if i % 2 else 2.0)
        sm.add_(0.5)
        x.mul_(1.5)
        g.replay()
        torch.cuda.synchronize()
        ref = a.double() @ b.double()
        assert float((c.double() - ref).norm() / ref.norm()) <= 1e-5
        sref = sm.double() @ sb.double()
        assert float((cs.double() - sref).norm() / sref.norm()) <= 1e-5
        yref = torch.relu(torch.nn.functional.conv2d(x.double(), w.double(), bias.double(),
                                                     padding=1))
        assert float((y.double() - yref).norm() / yref.norm()) <= 1e-5
    assert gpu.get_context(0).device_error() == 0


@pytest.mark.parametrize("trans_b", [False, True])
@pytest.mark.parametrize("n,k", [(333, 517), (70, 1031), (1000, 96)])
def test_prepass_low_part_ragged(gpu, orc, n, k, trans_b):
    """GEMMs of >= 16 M-tiles get B's 3xTF32 low part from the once-per-call
    prepass (TMA-loaded beside B) instead of the converters: ragged N and K
    (the prepass pads its rows to a multiple of 4 floats), B as a [K,N]
    matrix or as the [N,K] Linear-weight view, 128- and 64-column tiles,
    bias + ReLU, against float64."""
    m = 2048 + 17
    a = orc.normal((m, k), 7, 0)
    w = orc.normal((n, k), 7, 1) if trans_b else orc.normal((k, n), 7, 1)
    bias = orc.uniform((n,), 7, 2, -0.5, 0.5)
    bm = w.T if trans_b else w
    pre = orc.matmul_f64(a, np.ascontiguousarray(bm)) + bias.astype(np.float64)
    bd = _dev(w).t() if trans_b else _dev(w)
    c = _host(gpu.sgemm(_dev(a), bd, bias=_dev(bias), act=gpu.ACT_RELU, precision=0))
    ref = np.maximum(pre, 0.0)
    assert orc.rel_frob(c, ref) <= TOL[0]
    assert _relu_pattern_ok(c, pre)


@pytest.mark.parametrize("m", [17, 33, 64, 65, 100, 128])
@pytest.mark.parametrize("n,k", [(2052, 300), (2051, 257), (4096, 1000)])
@pytest.mark.parametrize("trans_b", [0, 1])
def test_skinny_transposed_path(gpu, orc, m, n, k, trans_b):
    """3xTF32 products of 17..128 rows against >= 2048 columns (K >= 256) run
    as C^T = B^T . A^T: B's [K,N] storage read as an MN-major A operand (or
    the Linear weight's [N,K] as a K-major one; N or K not a multiple of 4
    packs it first), A as the narrow operand (64 columns up to 64 rows, else
    128), the tile transposed on the way out and the bias added per row of
    C^T.  Ragged N (a partial last 128-row tile) and K, bias + ReLU, against
    float64."""
    a = orc.normal((m, k), 11, 1)
    w = orc.normal((n, k), 11, 2) if trans_b else orc.normal((k, n), 11, 2)
    bm = w.T if trans_b else w
    bias = orc.uniform((n,), 11, 3, -0.5, 0.5)
    pre = orc.matmul_f64(a, np.ascontiguousarray(bm)) + bias.astype(np.float64)
    bd = _dev(w).t() if trans_b else _dev(w)
    y = _host(gpu.sgemm(_dev(a), bd, bias=_dev(bias), act=gpu.ACT_RELU, precision=0))
    ref = np.maximum(pre, 0.0)
    assert orc.rel_frob(y, ref) <= TOL[0]
    scale = max(1.0, float(np.sqrt(np.mean(pre * pre))))
    assert _relu_pattern_ok(y / scale, pre / scale)


@pytest.mark.parametrize("pad", [4, 3])
@pytest.mark.parametrize("act", [0, 2, 3])
def test_skinny_transposed_strided_output(gpu, orc, pad, act):
    """The transposed skinny path writing into a view of a wider buffer
    (ldc = N + 4: 16-byte stores; ldc = N + 3: the element-wise stores),
    no bias or sigmoid / tanh; the padding columns stay untouched."""
    m, n, k = 48, 2304, 512
    a = orc.normal((m, k), 12, 1)
    b = orc.normal((k, n), 12, 2)
    bias = orc.uniform((n,), 12, 3, -0.5, 0.5) if act else None
    pre = orc.matmul_f64(a, b) + (bias.astype(np.float64) if act else 0.0)
    buf = torch.full((m, n + pad), 7.0, device="cuda")
    out = buf[:, :n]
    gpu.sgemm(_dev(a), _dev(b), bias=_dev(bias) if act else None, act=act, out=out)
    got = _host(buf)
    ref = {0: pre, 2: 1.0 / (1.0 + np.exp(-pre)), 3: np.tanh(pre)}[act]
    assert orc.rel_frob(got[:, :n], ref) <= TOL[0]
    assert np.all(got[:, n:] == 7.0)
