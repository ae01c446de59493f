"""rustorch_b200 — B200-native (sm_100a) dense-contraction backend for RusTorch.

Host-side mirror of the reference's operator interface for this path, over the
C ABI in include/rustorch_b200.h:

    ops.matmul(lhs, rhs)                         rustorch-core/src/ops.rs:1888
    ops.matmul_fused(lhs, rhs, bias, activation) rustorch-core/src/ops.rs:1543
    ops.conv2d(input, weight, stride, padding)   rustorch-core/src/ops/conv.rs:738
    nn.Linear / nn.Conv2d                        rustorch-nn/src/{linear,conv}.rs
    jit.Graph / NodeType / Optimizer / Executor  rustorch-core/src/jit.rs

Tensors are torch CUDA float32 tensors (torch provides device memory and
streams only; all arithmetic runs in this library's kernels).  Calls are
ordered on torch's current stream of the tensor's device.
"""
from __future__ import annotations

import ctypes
import threading

from . import _lib
from ._lib import (ACT_NONE, ACT_RELU, ACT_SIGMOID, ACT_TANH, LAYOUT_NCHW, LAYOUT_NHWC,
                   PREC_3XTF32, PREC_DEFAULT, PREC_TF32, RtbError, call, lib)

__all__ = ["Context", "get_context", "sgemm", "sgemm_batched", "matmul_bias_norm_activation",
           "layer_norm",
           "conv2d_fwd", "matmul_backward",
           "conv2d_backward", "max_pool2d",
           "global_avg_pool", "add", "relu", "fill_normal", "fill_uniform", "RtbError",
           "ACT_NONE", "ACT_RELU", "ACT_SIGMOID", "ACT_TANH", "PREC_3XTF32", "PREC_TF32",
           "PREC_DEFAULT", "LAYOUT_NCHW", "LAYOUT_NHWC", "lib"]


class Context:
    """An rtb_ctx on one device (stream, error word, workspace pool)."""

    def __init__(self, device: int = 0):
        self.device = device
        h = ctypes.c_void_p()
        call("rtb_init", device, ctypes.byref(h))
        self.handle = h

    def close(self) -> None:
        if self.handle:
            call("rtb_destroy", self.handle)
            self.handle = None

    def info(self):
        sm, ma, mi = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        mem = ctypes.c_size_t()
        call("rtb_get_device_info", self.handle, ctypes.byref(sm), ctypes.byref(ma),
             ctypes.byref(mi), ctypes.byref(mem))
        return {"sm_count": sm.value, "cc": (ma.value, mi.value), "total_mem": mem.value}

    def set_timeout_ns(self, ns: int) -> None:
        call("rtb_set_timeout_ns", self.handle, int(ns))

    def device_error(self) -> int:
        """Synchronise and read/clear the device error word (0 = none)."""
        code = ctypes.c_int()
        st = lib().rtb_device_error(self.handle, ctypes.byref(code))
        if st not in (_lib.RTB_OK, _lib.RTB_E_TIMEOUT):
            _lib.check(st, "rtb_device_error")
        return code.value

    def synchronize(self, stream=None) -> None:
        call("rtb_stream_synchronize", self.handle, stream)


_ctx_lock = threading.Lock()
_contexts: dict = {}


def get_context(device: int = 0) -> Context:
    with _ctx_lock:
        c = _contexts.get(device)
        if c is None:
            c = Context(device)
            _contexts[device] = c
        return c


def _torch():
    import torch
    return torch


def _stream_of(t):
    torch = _torch()
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _dev(t) -> int:
    return t.device.index if t.device.index is not None else 0


def _check_f32_cuda(*ts):
    torch = _torch()
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda or t.dtype != torch.float32:
            raise ValueError("rustorch_b200 expects float32 CUDA tensors")


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _operand_2d(t):
    """(tensor, leading dim, trans) for a 2-D strided view without copying when
    one dimension is unit-stride; trans=1 means stored as the transpose."""
    if t.stride(1) == 1 and t.stride(0) >= max(t.shape[1], 1):
        return t, t.stride(0), 0
    if t.stride(0) == 1 and t.stride(1) >= max(t.shape[0], 1):
        return t, t.stride(1), 1
    t = t.contiguous()
    return t, t.shape[1], 0


def sgemm(a, b, bias=None, act: int = ACT_NONE, precision: int = PREC_DEFAULT, out=None):
    """C = act(a @ b + bias) for 2-D float32 CUDA tensors a [M,K], b [K,N]."""
    torch = _torch()
    _check_f32_cuda(a, b, bias, out)
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("Matmul only supports 2D")
    M, K = a.shape
    K2, N = b.shape
    if K != K2:
        raise ValueError("Matmul dimension mismatch")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=a.device)
    a_, lda, ta = _operand_2d(a)
    b_, ldb, tb = _operand_2d(b)
    if bias is not None:
        bias = bias.contiguous()
    ctx = get_context(_dev(a))
    call("rtb_sgemm", ctx.handle, M, N, K, _ptr(a_), lda, ta, _ptr(b_), ldb, tb, _ptr(bias), act,
         _ptr(out), out.stride(0), precision, _stream_of(a))
    return out


def matmul_bias_norm_activation(a, b, bias=None, norm_weight=None, norm_bias=None,
                                eps: float = 1e-5, act: int = ACT_NONE,
                                precision: int = PREC_DEFAULT, out=None):
    """ops::matmul_bias_norm_activation: act(layer_norm(a @ b + bias) * norm_weight
    + norm_bias), the LayerNorm over the last dimension (N), for 2-D float32
    CUDA tensors a [M,K], b [K,N]; act is any ACT_*."""
    torch = _torch()
    _check_f32_cuda(a, b, bias, norm_weight, norm_bias, out)
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("Matmul only supports 2D")
    M, K = a.shape
    K2, N = b.shape
    if K != K2:
        raise ValueError("Matmul dimension mismatch")
    for t in (bias, norm_weight, norm_bias):
        if t is not None and t.numel() != N:
            raise ValueError("bias / norm parameters must have N elements")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=a.device)
    a_, lda, ta = _operand_2d(a)
    b_, ldb, tb = _operand_2d(b)
    bias, norm_weight, norm_bias = (t.contiguous() if t is not None else None
                                    for t in (bias, norm_weight, norm_bias))
    ctx = get_context(_dev(a))
    call("rtb_matmul_bias_norm_act", ctx.handle, M, N, K, _ptr(a_), lda, ta, _ptr(b_), ldb, tb,
         _ptr(bias), _ptr(norm_weight), _ptr(norm_bias), float(eps), act, _ptr(out),
         out.stride(0), precision, _stream_of(a))
    return out


def layer_norm(x, norm_weight=None, norm_bias=None, eps: float = 1e-5, act: int = ACT_NONE,
               out=None):
    """ops::layer_norm over the last dimension (+ an optional activation) for a
    float32 CUDA tensor whose rows are contiguous; out may be x (in place)."""
    torch = _torch()
    _check_f32_cuda(x, norm_weight, norm_bias, out)
    if x.dim() == 0:
        raise ValueError("LayerNorm: Input shape smaller than normalized shape")
    d = x.shape[-1]
    x2 = x.reshape(-1, d) if d else x.reshape(-1, 0)
    if x2.numel() and x2.stride(1) != 1:
        x2 = x2.contiguous()
    for t in (norm_weight, norm_bias):
        if t is not None and t.numel() != d:
            raise ValueError("LayerNorm: Input shape does not match normalized shape")
    if out is None:
        out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    y2 = out.view(-1, d) if d else out.reshape(-1, 0)
    norm_weight, norm_bias = (t.contiguous() if t is not None else None
                              for t in (norm_weight, norm_bias))
    ctx = get_context(_dev(x))
    call("rtb_layer_norm", ctx.handle, x2.shape[0], d, _ptr(x2), max(x2.stride(0), d),
         _ptr(norm_weight), _ptr(norm_bias), float(eps), act, _ptr(y2), max(y2.stride(0), d),
         _stream_of(x))
    return out


def sgemm_batched(a, b, bias=None, act: int = ACT_NONE, precision: int = PREC_DEFAULT):
    """Batched C[i] = act(a[i] @ b[i] + bias) for contiguous 3-D tensors."""
    torch = _torch()
    _check_f32_cuda(a, b, bias)
    a = a.contiguous()
    b = b.contiguous()
    Bt, M, K = a.shape
    _, K2, N = b.shape
    if K != K2 or b.shape[0] != Bt:
        raise ValueError("batched matmul dimension mismatch")
    out = torch.empty((Bt, M, N), dtype=torch.float32, device=a.device)
    ctx = get_context(_dev(a))
    call("rtb_sgemm_batched", ctx.handle, Bt, M, N, K, _ptr(a), K, M * K, 0, _ptr(b), N, K * N, 0,
         _ptr(bias.contiguous() if bias is not None else None), act, _ptr(out), N, M * N,
         precision, _stream_of(a))
    return out


def conv_out_hw(h, w, kh, kw, stride, padding):
    return (h + 2 * padding[0] - kh) // stride[0] + 1, (w + 2 * padding[1] - kw) // stride[1] + 1


def conv2d_fwd(x, w, bias=None, stride=(1, 1), padding=(0, 0), residual=None, act: int = ACT_NONE,
               x_layout: int = LAYOUT_NCHW, y_layout: int = LAYOUT_NCHW,
               precision: int = PREC_DEFAULT):
    """y = act(conv2d(x, w) + bias + residual); w is [Co, Ci, kh, kw]."""
    torch = _torch()
    _check_f32_cuda(x, w, bias, residual)
    x = x.contiguous()
    w = w.contiguous()
    if x_layout == LAYOUT_NCHW:
        N, Ci, H, W = x.shape
    else:
        N, H, W, Ci = x.shape
    Co, Ci2, kh, kw = w.shape
    if Ci2 != Ci:
        raise ValueError(f"Weight input channels {Ci2} must match input channels {Ci}")
    Ho, Wo = conv_out_hw(H, W, kh, kw, stride, padding)
    shape = (N, Co, Ho, Wo) if y_layout == LAYOUT_NCHW else (N, Ho, Wo, Co)
    y = torch.empty(shape, dtype=torch.float32, device=x.device)
    if residual is not None:
        residual = residual.contiguous()
    ctx = get_context(_dev(x))
    call("rtb_conv2d_fwd", ctx.handle, N, Ci, H, W, Co, kh, kw, stride[0], stride[1], padding[0],
         padding[1], _ptr(x), x_layout, _ptr(w), _ptr(bias.contiguous() if bias is not None else None),
         _ptr(residual), act, _ptr(y), y_layout, precision, _stream_of(x))
    return y


def matmul_backward(a, b, grad, need_a: bool = True, need_b: bool = True, out_a=None, out_b=None,
                    accumulate: bool = False, precision: int = PREC_DEFAULT):
    """MatmulBackward of c = a @ b: (grad @ b.T, a.T @ grad) for contiguous 2-D
    float32 CUDA tensors; with accumulate the results are added to out_a/out_b."""
    torch = _torch()
    _check_f32_cuda(a, b, grad)
    a, b, grad = a.contiguous(), b.contiguous(), grad.contiguous()
    M, K = a.shape
    N = b.shape[1]
    if b.shape[0] != K or tuple(grad.shape) != (M, N):
        raise ValueError("matmul_backward: shape mismatch")
    da = (out_a if out_a is not None else torch.empty((M, K), dtype=torch.float32,
                                                      device=a.device)) if need_a else None
    db = (out_b if out_b is not None else torch.empty((K, N), dtype=torch.float32,
                                                      device=a.device)) if need_b else None
    ctx = get_context(_dev(a))
    call("rtb_matmul_backward", ctx.handle, M, N, K, _ptr(a), _ptr(b), _ptr(grad), _ptr(da),
         _ptr(db), int(accumulate), precision, _stream_of(a))
    return da, db


def conv2d_backward(x, w, grad, stride=(1, 1), padding=(0, 0), need_x: bool = True,
                    need_w: bool = True, precision: int = PREC_DEFAULT):
    """Conv2dBackward (NCHW): (grad wrt x, grad wrt w) of y = conv2d(x, w)."""
    torch = _torch()
    _check_f32_cuda(x, w, grad)
    x, w, grad = x.contiguous(), w.contiguous(), grad.contiguous()
    N, Ci, H, W = x.shape
    Co, _, kh, kw = w.shape
    dx = torch.empty_like(x) if need_x else None
    dw = torch.empty_like(w) if need_w else None
    ctx = get_context(_dev(x))
    call("rtb_conv2d_backward", ctx.handle, N, Ci, H, W, Co, kh, kw, stride[0], stride[1],
         padding[0], padding[1], _ptr(x), _ptr(w), _ptr(grad), _ptr(dx), _ptr(dw), 0, precision,
         _stream_of(x))
    return dx, dw


def max_pool2d(x, kernel=(3, 3), stride=(2, 2), padding=(1, 1), layout: int = LAYOUT_NCHW):
    torch = _torch()
    _check_f32_cuda(x)
    x = x.contiguous()
    if layout == LAYOUT_NCHW:
        N, C, H, W = x.shape
    else:
        N, H, W, C = x.shape
    Ho, Wo = conv_out_hw(H, W, kernel[0], kernel[1], stride, padding)
    shape = (N, C, Ho, Wo) if layout == LAYOUT_NCHW else (N, Ho, Wo, C)
    y = torch.empty(shape, dtype=torch.float32, device=x.device)
    ctx = get_context(_dev(x))
    call("rtb_max_pool2d", ctx.handle, N, C, H, W, kernel[0], kernel[1], stride[0], stride[1],
         padding[0], padding[1], _ptr(x), _ptr(y), layout, _stream_of(x))
    return y


def global_avg_pool(x, layout: int = LAYOUT_NCHW):
    torch = _torch()
    _check_f32_cuda(x)
    x = x.contiguous()
    if layout == LAYOUT_NCHW:
        N, C, H, W = x.shape
    else:
        N, H, W, C = x.shape
    y = torch.empty((N, C), dtype=torch.float32, device=x.device)
    ctx = get_context(_dev(x))
    call("rtb_global_avg_pool", ctx.handle, N, C, H, W, _ptr(x), _ptr(y), layout, _stream_of(x))
    return y


def add(a, b):
    torch = _torch()
    _check_f32_cuda(a, b)
    if a.shape != b.shape:
        raise ValueError("add: shapes differ")
    a = a.contiguous()
    b = b.contiguous()
    y = torch.empty_like(a)
    call("rtb_add", get_context(_dev(a)).handle, a.numel(), _ptr(a), _ptr(b), _ptr(y),
         _stream_of(a))
    return y


def relu(x):
    torch = _torch()
    _check_f32_cuda(x)
    x = x.contiguous()
    y = torch.empty_like(x)
    call("rtb_relu", get_context(_dev(x)).handle, x.numel(), _ptr(x), _ptr(y), _stream_of(x))
    return y


def fill_normal(shape, seed: int, tensor_id: int, mean: float = 0.0, std: float = 1.0):
    """Host numpy array from the documented SplitMix64/Box-Muller generator."""
    import numpy as np
    out = np.empty(shape, dtype=np.float32)
    call("rtb_fill_normal_host", out.ctypes.data_as(ctypes.c_void_p), out.size, seed, tensor_id,
         mean, std)
    return out


def fill_uniform(shape, seed: int, tensor_id: int, lo: float, hi: float):
    import numpy as np
    out = np.empty(shape, dtype=np.float32)
    call("rtb_fill_uniform_host", out.ctypes.data_as(ctypes.c_void_p), out.size, seed, tensor_id,
         lo, hi)
    return out
