"""ORACLE — test infrastructure only.

ctypes wrapper over ``oracle/liboracle.so``, the plain-C restatement of
RusTorch's CPU dense-contraction path (see ``oracle/oracle.c`` for the
reference file:line each function follows).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm use
this module, and only as the checker or the timed CPU baseline; the product
package ``rustorch_b200`` never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_p = ctypes.c_void_p


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_stream_key.restype = _u64
        L.orc_stream_key.argtypes = [_u64, _u64]
        L.orc_unit.restype = ctypes.c_float
        L.orc_unit.argtypes = [_u64, _u64]
        L.orc_fill_uniform.argtypes = [_p, _i64, _u64, _u64, ctypes.c_float, ctypes.c_float]
        L.orc_fill_normal.argtypes = [_p, _i64, _u64, _u64, ctypes.c_float, ctypes.c_float]
        L.orc_max_threads.restype = ctypes.c_int
        L.orc_sgemm_mm.argtypes = [_i64] * 3 + [_p, _i64, _i64, _p, _i64, _i64, _p, ctypes.c_int]
        L.orc_matmul_parallel_core.argtypes = [_i64] * 3 + [_p, _p, _p, _p, ctypes.c_int]
        L.orc_matmul_auto_parallel.restype = ctypes.c_int
        L.orc_matmul_auto_parallel.argtypes = [_i64] * 3
        L.orc_matmul.restype = ctypes.c_int
        L.orc_matmul.argtypes = [_i64] * 3 + [_p, _i64, _i64, _p, _i64, _i64, _p, _p, ctypes.c_int]
        L.orc_matmul_f64.argtypes = [_i64] * 3 + [_p, _i64, _i64, _p, _i64, _i64, _p, ctypes.c_int]
        L.orc_matmul_f64_sampled.argtypes = [_i64, _p, _i64, _i64, _p, _i64, _i64, _p, _p, _i64, _p,
                                             ctypes.c_int]
        L.orc_relu.argtypes = [_p, _i64]
        L.orc_add_bias_nchw.argtypes = [_p, _p, _i64, _i64, _i64]
        L.orc_add_bias_rows.argtypes = [_p, _p, _i64, _i64]
        L.orc_add.argtypes = [_p, _p, _p, _i64]
        conv_args = [_i64] * 11 + [_p, _p, _p, ctypes.c_int]
        L.orc_conv2d_direct.argtypes = conv_args
        L.orc_conv2d_im2col.restype = ctypes.c_int
        L.orc_conv2d_im2col.argtypes = conv_args
        L.orc_conv2d.restype = ctypes.c_int
        L.orc_conv2d.argtypes = conv_args
        L.orc_conv2d_f64.argtypes = conv_args
        L.orc_conv2d_grad_input_f64.argtypes = conv_args
        L.orc_conv2d_grad_weight_f64.argtypes = conv_args
        L.orc_max_pool2d.argtypes = [_i64] * 10 + [_p, _p]
        L.orc_global_avg_pool.argtypes = [_i64] * 3 + [_p, _p]
        L.orc_layer_norm_ref.argtypes = [_p, _i64, _i64, _p, _p, ctypes.c_float]
        L.orc_layer_norm_f64.argtypes = [_p, _i64, _i64, _p, _p, ctypes.c_double]
        L.orc_activation.argtypes = [_p, _i64, ctypes.c_int]
        L.orc_activation_f64.argtypes = [_p, _i64, ctypes.c_int]
        L.orc_rel_frob.restype = ctypes.c_double
        L.orc_rel_frob.argtypes = [_p, _p, _i64]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"] or a.ndim == 0
    return a.ctypes.data


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def max_threads() -> int:
    return lib().orc_max_threads()


# ---------------------------------------------------------------- PRNG
def stream_key(seed: int, tensor_id: int) -> int:
    return lib().orc_stream_key(seed, tensor_id)


def unit(idx: int, seed: int) -> float:
    """The reference's deterministic_unit(idx, seed)."""
    return lib().orc_unit(idx, seed)


def normal(shape, seed: int, tensor_id: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(shape, dtype=np.float32)
    lib().orc_fill_normal(_ptr(out), out.size, seed, tensor_id, mean, std)
    return out


def uniform(shape, seed: int, tensor_id: int, lo: float, hi: float) -> np.ndarray:
    out = np.empty(shape, dtype=np.float32)
    lib().orc_fill_uniform(_ptr(out), out.size, seed, tensor_id, lo, hi)
    return out


# ---------------------------------------------------------------- GEMM
def matmul(a: np.ndarray, b: np.ndarray, bias=None, threads: int = 0):
    """ops::matmul (auto dispatch) -> (C, choice) ; choice 0 = sgemm, 1 = parallel."""
    a = _f32(a)
    b = _f32(b)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    c = np.empty((m, n), dtype=np.float32)
    bias_keep = _f32(bias) if bias is not None else None
    bp = _ptr(bias_keep) if bias_keep is not None else None
    ch = lib().orc_matmul(m, k, n, _ptr(a), k, 1, _ptr(b), n, 1, bp, _ptr(c), threads)
    if ch < 0:
        raise MemoryError("oracle matmul allocation failed")
    return c, ch


def sgemm_mm(a: np.ndarray, b: np.ndarray, threads: int = 1) -> np.ndarray:
    a = _f32(a)
    b = _f32(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), dtype=np.float32)
    lib().orc_sgemm_mm(m, k, n, _ptr(a), k, 1, _ptr(b), n, 1, _ptr(c), threads)
    return c


def matmul_parallel_core(a: np.ndarray, b: np.ndarray, bias=None, threads: int = 0) -> np.ndarray:
    a = _f32(a)
    b = _f32(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), dtype=np.float32)
    bias_keep = _f32(bias) if bias is not None else None
    lib().orc_matmul_parallel_core(m, k, n, _ptr(a), _ptr(b),
                                   _ptr(bias_keep) if bias_keep is not None else None, _ptr(c),
                                   threads)
    return c


def matmul_f64(a: np.ndarray, b: np.ndarray, threads: int = 0) -> np.ndarray:
    a = _f32(a)
    b = _f32(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), dtype=np.float64)
    lib().orc_matmul_f64(m, k, n, _ptr(a), k, 1, _ptr(b), n, 1, _ptr(c), threads)
    return c


def matmul_f64_sampled(a: np.ndarray, b: np.ndarray, rows, cols, threads: int = 0) -> np.ndarray:
    a = _f32(a)
    b = _f32(b)
    k = a.shape[1]
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    cols = np.ascontiguousarray(cols, dtype=np.int64)
    out = np.empty(rows.shape[0], dtype=np.float64)
    lib().orc_matmul_f64_sampled(k, _ptr(a), k, 1, _ptr(b), b.shape[1], 1, _ptr(rows), _ptr(cols),
                                 rows.shape[0], _ptr(out), threads)
    return out


def matmul_fused(a, b, bias=None, act: int = 0, threads: int = 0) -> np.ndarray:
    """ops::matmul_fused CPU path (rustorch-core/src/ops.rs:1543-1710): bias
    inside the GEMM for Activation::None, else staged matmul -> add -> act."""
    if act == 0:
        return matmul(a, b, bias, threads)[0]
    c, _ = matmul(a, b, None, threads)
    if bias is not None:
        bias_keep = _f32(bias)
        lib().orc_add_bias_rows(_ptr(c), _ptr(bias_keep), c.shape[0], c.shape[1])
    if act == 1:
        lib().orc_relu(_ptr(c), c.size)
    elif act in (2, 3):  # ops/activations.rs:47-50 (sigmoid), :213 (tanh)
        lib().orc_activation(_ptr(c), c.size, act)
    else:
        raise ValueError(f"unknown activation {act}")
    return c


def linear(x, w, b=None, relu: bool = False, threads: int = 0) -> np.ndarray:
    """nn::Linear::forward (rustorch-nn/src/linear.rs:75-95): x.matmul(w.t()) + b."""
    x = _f32(x)
    w = _f32(w)
    m, k = x.shape
    n = w.shape[0]
    c = np.empty((m, n), dtype=np.float32)
    ch = lib().orc_matmul(m, k, n, _ptr(x), k, 1, _ptr(w), 1, k, None, _ptr(c), threads)
    if ch < 0:
        raise MemoryError
    if b is not None:
        bk = _f32(b)
        lib().orc_add_bias_rows(_ptr(c), _ptr(bk), m, n)
    if relu:
        lib().orc_relu(_ptr(c), c.size)
    return c


# ---------------------------------------------------------------- elementwise
def relu(x: np.ndarray) -> np.ndarray:
    y = _f32(x).copy()
    lib().orc_relu(_ptr(y), y.size)
    return y


def add_bias_nchw(y: np.ndarray, bias: np.ndarray) -> np.ndarray:
    y = _f32(y).copy()
    b = _f32(bias).reshape(-1)
    n, c = y.shape[0], y.shape[1]
    lib().orc_add_bias_nchw(_ptr(y), _ptr(b), n, c, y.size // (n * c))
    return y


# ---------------------------------------------------------------- conv
def _conv_dims(x, w, stride, padding):
    n, ci, h, wd = x.shape
    co, ci2, kh, kw = w.shape
    assert ci == ci2
    sh, sw = stride
    ph, pw = padding
    ho = (h + 2 * ph - kh) // sh + 1
    wo = (wd + 2 * pw - kw) // sw + 1
    return n, ci, h, wd, co, kh, kw, sh, sw, ph, pw, ho, wo


def conv2d(x, w, stride=(1, 1), padding=(0, 0), threads: int = 0):
    """ops::conv2d auto dispatch -> (y NCHW, choice); choice 0 direct, 1 im2col+sgemm,
    2 im2col+parallel core."""
    x = _f32(x)
    w = _f32(w)
    n, ci, h, wd, co, kh, kw, sh, sw, ph, pw, ho, wo = _conv_dims(x, w, stride, padding)
    y = np.empty((n, co, ho, wo), dtype=np.float32)
    ch = lib().orc_conv2d(n, ci, h, wd, co, kh, kw, sh, sw, ph, pw, _ptr(x), _ptr(w), _ptr(y),
                          threads)
    if ch < 0:
        raise MemoryError("oracle conv allocation failed")
    return y, ch


def conv2d_direct(x, w, stride=(1, 1), padding=(0, 0), threads: int = 0) -> np.ndarray:
    x = _f32(x)
    w = _f32(w)
    n, ci, h, wd, co, kh, kw, sh, sw, ph, pw, ho, wo = _conv_dims(x, w, stride, padding)
    y = np.empty((n, co, ho, wo), dtype=np.float32)
    lib().orc_conv2d_direct(n, ci, h, wd, co, kh, kw, sh, sw, ph, pw, _ptr(x), _ptr(w), _ptr(y),
                            threads)
    return y


def conv2d_f64(x, w, stride=(1, 1), padding=(0, 0), threads: int = 0) -> np.ndarray:
    x = _f32(x)
    w = _f32(w)
    n, ci, h, wd, co, kh, kw, sh, sw, ph, pw, ho, wo = _conv_dims(x, w, stride, padding)
    y = np.empty((n, co, ho, wo), dtype=np.float64)
    lib().orc_conv2d_f64(n, ci, h, wd, co, kh, kw, sh, sw, ph, pw, _ptr(x), _ptr(w), _ptr(y),
                         threads)
    return y


def conv2d_grad_input_f64(gy, w, x_shape, stride=(1, 1), padding=(0, 0), threads: int = 0):
    """Conv2dBackward grad_input (rustorch-core/src/ops/conv.rs:336-389, the f64
    direct core), float64 result; gy [N,Co,Ho,Wo], w [Co,Ci,kh,kw]."""
    gy = _f32(gy)
    w = _f32(w)
    n, ci, h, wd = x_shape
    co, _, kh, kw = w.shape
    gx = np.empty((n, ci, h, wd), dtype=np.float64)
    lib().orc_conv2d_grad_input_f64(n, ci, h, wd, co, kh, kw, stride[0], stride[1], padding[0],
                                    padding[1], _ptr(gy), _ptr(w), _ptr(gx), threads)
    return gx


def conv2d_grad_weight_f64(x, gy, w_shape, stride=(1, 1), padding=(0, 0), threads: int = 0):
    """Conv2dBackward grad_weight (rustorch-core/src/ops/conv.rs:455-502, the f64
    direct core), float64 result; x [N,Ci,H,W], gy [N,Co,Ho,Wo]."""
    x = _f32(x)
    gy = _f32(gy)
    n, ci, h, wd = x.shape
    co, _, kh, kw = w_shape
    gw = np.empty((co, ci, kh, kw), dtype=np.float64)
    lib().orc_conv2d_grad_weight_f64(n, ci, h, wd, co, kh, kw, stride[0], stride[1], padding[0],
                                     padding[1], _ptr(x), _ptr(gy), _ptr(gw), threads)
    return gw


def layer_norm(x, g=None, b=None, eps: float = 1e-5) -> np.ndarray:
    """ops::layer_norm over the last dimension, f32, the reference's one-pass
    formula (rustorch-core/src/ops/norm.rs:613-700)."""
    y = _f32(x).copy()
    gk = _f32(g) if g is not None else None
    bk = _f32(b) if b is not None else None
    d = y.shape[-1]
    lib().orc_layer_norm_ref(_ptr(y), y.size // d if d else 0, d,
                             _ptr(gk) if gk is not None else None,
                             _ptr(bk) if bk is not None else None, eps)
    return y


def activation(x, act: int) -> np.ndarray:
    """apply_activation (rustorch-core/src/ops.rs:1773-1780), f32."""
    y = _f32(x).copy()
    lib().orc_activation(_ptr(y), y.size, act)
    return y


def matmul_bias_norm_activation(a, b, bias=None, g=None, beta=None, eps: float = 1e-5,
                                act: int = 0, threads: int = 0) -> np.ndarray:
    """ops::matmul_bias_norm_activation (rustorch-core/src/ops.rs:1815-1886),
    f32: matmul_fused(a, b, bias) (the pipeline_fused order, ops.rs:1801-1813),
    layer_norm over N, then the activation."""
    c = matmul(a, b, bias, threads)[0]
    return activation(layer_norm(c, g, beta, eps), act)


def matmul_bias_norm_activation_f64(a, b, bias=None, g=None, beta=None, eps: float = 1e-5,
                                    act: int = 0, threads: int = 0) -> np.ndarray:
    """The same pipeline in float64 with a two-pass variance: the exact value
    the CUDA path is checked against."""
    c = matmul_f64(a, b, threads)
    if bias is not None:
        c += np.asarray(bias, np.float64)[None, :]
    c = np.ascontiguousarray(c)
    gk = _f32(g) if g is not None else None
    bk = _f32(beta) if beta is not None else None
    d = c.shape[-1]
    lib().orc_layer_norm_f64(_ptr(c), c.size // d if d else 0, d,
                             _ptr(gk) if gk is not None else None,
                             _ptr(bk) if bk is not None else None, eps)
    lib().orc_activation_f64(_ptr(c), c.size, act)
    return c


def matmul_backward_f64(a, b, gc):
    """MatmulBackward (rustorch-core/src/ops.rs:529-570): grad_lhs = grad . rhs^T,
    grad_rhs = lhs^T . grad, in float64."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    gc = np.asarray(gc, np.float64)
    return gc @ b.T, a.T @ gc


def conv2d_bias_relu(x, w, b, stride=(1, 1), padding=(0, 0), relu_: bool = True, threads: int = 0):
    """nn::Conv2d::forward + ReLU (rustorch-nn/src/conv.rs:52-63, ops.rs:449-491):
    conv (auto path), broadcast bias add, relu.  Returns (y, pre_activation)."""
    y, _ = conv2d(x, w, stride, padding, threads)
    if b is not None:
        y = add_bias_nchw(y, b)
    pre = y
    if relu_:
        y = relu(y)
    return y, pre


def max_pool2d(x, kernel=(3, 3), stride=(2, 2), padding=(1, 1)) -> np.ndarray:
    x = _f32(x)
    n, c, h, w = x.shape
    kh, kw = kernel
    sh, sw = stride
    ph, pw = padding
    ho = (h + 2 * ph - kh) // sh + 1
    wo = (w + 2 * pw - kw) // sw + 1
    y = np.empty((n, c, ho, wo), dtype=np.float32)
    lib().orc_max_pool2d(n, c, h, w, kh, kw, sh, sw, ph, pw, _ptr(x), _ptr(y))
    return y


def global_avg_pool(x) -> np.ndarray:
    x = _f32(x)
    n, c = x.shape[0], x.shape[1]
    y = np.empty((n, c), dtype=np.float32)
    lib().orc_global_avg_pool(n, c, x.size // (n * c), _ptr(x), _ptr(y))
    return y


def rel_frob(x, ref) -> float:
    x = _f32(x)
    ref = np.ascontiguousarray(ref, dtype=np.float64)
    assert x.size == ref.size
    return lib().orc_rel_frob(_ptr(x), _ptr(ref), x.size)
