"""ctypes binding of librustorch_b200.so (the C ABI in include/rustorch_b200.h).

There is no fallback: if the shared library is missing or fails to load, every
entry point raises.  Build it with ``python -m rustorch_b200.build``.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "librustorch_b200.so")

RTB_OK = 0
RTB_E_INVALID = 1
RTB_E_OOM = 2
RTB_E_CUDA = 3
RTB_E_TIMEOUT = 4
RTB_E_UNSUPPORTED = 5
RTB_E_NCCL = 6

ACT_NONE, ACT_RELU, ACT_SIGMOID, ACT_TANH = 0, 1, 2, 3
PREC_3XTF32, PREC_TF32, PREC_DEFAULT = 0, 1, -1
LAYOUT_NCHW, LAYOUT_NHWC = 0, 1

# Every symbol the header declares, with (restype, argtypes).
_i = ctypes.c_int
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_sz = ctypes.c_size_t
_p = ctypes.c_void_p
_pp = ctypes.POINTER(ctypes.c_void_p)
_f = ctypes.c_float

SIGNATURES = {
    "rtb_init": (_i, [_i, _pp]),
    "rtb_destroy": (_i, [_p]),
    "rtb_device_count": (_i, [ctypes.POINTER(_i)]),
    "rtb_get_device_info": (_i, [_p, ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i),
                                 ctypes.POINTER(_sz)]),
    "rtb_status_string": (ctypes.c_char_p, [_i]),
    "rtb_last_error": (_i, [ctypes.c_char_p, _sz]),
    "rtb_set_timeout_ns": (_i, [_p, _u64]),
    "rtb_device_error": (_i, [_p, ctypes.POINTER(_i)]),
    "rtb_set_kernel_trace": (_i, [_p, _p, _i64]),
    "rtb_debug_wait_probe": (_i, [_p, _u64, _p]),
    "rtb_malloc": (_i, [_p, _pp, _sz, _p]),
    "rtb_free": (_i, [_p, _p, _p]),
    "rtb_host_alloc": (_i, [_p, _pp, _sz]),
    "rtb_host_free": (_i, [_p, _p]),
    "rtb_memcpy_h2d": (_i, [_p, _p, _p, _sz, _p]),
    "rtb_memcpy_d2h": (_i, [_p, _p, _p, _sz, _p]),
    "rtb_memcpy_d2d": (_i, [_p, _p, _p, _sz, _p]),
    "rtb_memset_zero": (_i, [_p, _p, _sz, _p]),
    "rtb_context_stream": (_i, [_p, _pp]),
    "rtb_stream_create": (_i, [_p, _pp]),
    "rtb_stream_destroy": (_i, [_p, _p]),
    "rtb_stream_synchronize": (_i, [_p, _p]),
    "rtb_sgemm": (_i, [_p, _i64, _i64, _i64, _p, _i64, _i, _p, _i64, _i, _p, _i, _p, _i64, _i, _p]),
    "rtb_sgemm_batched": (_i, [_p, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i, _p, _i64, _i64, _i,
                               _p, _i, _p, _i64, _i64, _i, _p]),
    "rtb_conv2d_fwd": (_i, [_p] + [_i64] * 11 + [_p, _i, _p, _p, _p, _i, _p, _i, _i, _p]),
    "rtb_conv2d_fwd_noalloc": (_i, [_p] + [_i64] * 11 + [_p, _i, _p, _p, _p, _i, _p, _i, _i, _p]),
    "rtb_matmul_bias_norm_act": (_i, [_p, _i64, _i64, _i64, _p, _i64, _i, _p, _i64, _i, _p, _p, _p,
                                      ctypes.c_float, _i, _p, _i64, _i, _p]),
    "rtb_layer_norm": (_i, [_p, _i64, _i64, _p, _i64, _p, _p, ctypes.c_float, _i, _p, _i64, _p]),
    "rtb_matmul_backward": (_i, [_p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i, _i, _p]),
    "rtb_peer_buffer_create": (_i, [_p, _p, _sz, _p]),
    "rtb_peer_buffer_local": (_i, [_p, _p]),
    "rtb_peer_buffer_destroy": (_i, [_p, _p]),
    "rtb_sgemm_nsplit_p2p": (_i, [_p, _p, _p, _i64, _i64, _i64, _p, _p, _i, _p]),
    "rtb_conv2d_backward": (_i, [_p] + [_i64] * 11 + [_p, _p, _p, _p, _p, _i, _i, _p]),
    "rtb_conv2d_packed_weight_size": (_i64, [_i64] * 4),
    "rtb_conv2d_prepack_weight": (_i, [_p, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "rtb_conv2d_fwd_packed": (_i, [_p] + [_i64] * 11 + [_p, _p, _p, _p, _i, _p, _i, _i, _p]),
    "rtb_conv2d_prepack_weight_lo": (_i, [_p, _i64, _i64, _i64, _i64, _p, _p, _p, _p]),
    "rtb_conv2d_fwd_packed_lo": (_i, [_p] + [_i64] * 11 + [_p, _p, _p, _p, _p, _i, _p, _i, _i, _p]),
    "rtb_nchw_to_nhwc_padded": (_i, [_p, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "rtb_max_pool2d": (_i, [_p] + [_i64] * 10 + [_p, _p, _i, _p]),
    "rtb_global_avg_pool": (_i, [_p] + [_i64] * 4 + [_p, _p, _i, _p]),
    "rtb_add": (_i, [_p, _i64, _p, _p, _p, _p]),
    "rtb_relu": (_i, [_p, _i64, _p, _p, _p]),
    "rtb_elementwise_broadcast": (_i, [_p, _i, _i, _p, _p, _p, _p, _p, _p, _p]),
    "rtb_fill_normal_host": (_i, [_p, _i64, _u64, _u64, _f, _f]),
    "rtb_fill_uniform_host": (_i, [_p, _i64, _u64, _u64, _f, _f]),
    "rtb_nccl_unique_id": (_i, [_p]),
    "rtb_nccl_comm_init": (_i, [_p, _p, _i, _i, _pp]),
    "rtb_nccl_comm_destroy": (_i, [_p]),
    "rtb_sgemm_nsplit_allgather": (_i, [_p, _p, _i64, _i64, _i64, _p, _p, _p, _p, _i, _p]),
    # include/rustorch_b200_vision.h
    "rtb_resnet18_create": (_i, [_i, _u64, _i, _pp]),
    "rtb_resnet18_destroy": (_i, [_p]),
    "rtb_resnet18_forward": (_i, [_p, _i64, _p, _p, _p]),
    "rtb_resnet18_num_params": (_i64, [_p]),
    "rtb_resnet18_get_param": (_i, [_p, _i64, _p, ctypes.POINTER(_i64)]),
    "rtb_resnet18_flops_per_image": (_i64, [_p]),
}

_lib = None


class RtbError(RuntimeError):
    def __init__(self, status: int, where: str, msg: str):
        super().__init__(f"{where}: status {status} ({STATUS.get(status, '?')}): {msg}")
        self.status = status


STATUS = {0: "ok", 1: "invalid", 2: "oom", 3: "cuda", 4: "timeout", 5: "unsupported", 6: "nccl"}


def lib() -> ctypes.CDLL:
    """Load the library (raises if it is absent: there is no CPU fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing; build it with `python -m rustorch_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().rtb_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(status: int, where: str) -> None:
    if status != RTB_OK:
        raise RtbError(status, where, last_error())


def call(name: str, *args) -> int:
    """Call an rtb_* entry point and raise RtbError on a non-zero status."""
    st = getattr(lib(), name)(*args)
    check(st, name)
    return st
