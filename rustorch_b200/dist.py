"""Multi-GPU plumbing for the two natural shardings of the contraction path.

- Batch-sharded conv / ResNet forward: every rank runs its own batch; there is
  no exchange step (see bench.py's resnet18 workload).
- N-split GEMM: every rank holds A [M,K] and the column block B[:, cols(rank)],
  computes its block of C on the tensor cores and the blocks are all-gathered
  over NVLink/NVSwitch with NCCL (rtb_sgemm_nsplit_allgather).

One process per GPU.  The library's NCCL communicator is bootstrapped by
broadcasting its 128-byte unique id over an existing torch.distributed group
(any backend, e.g. gloo), so no second rendezvous is needed.
"""
from __future__ import annotations

import ctypes

from . import _lib
from ._lib import call, lib


def shard_columns(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of the columns rank `rank` owns in an N-split of n columns
    over `world` ranks (equal blocks; n must be divisible by world)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    if n % world:
        raise ValueError(f"N-split needs N divisible by the rank count ({n} % {world} != 0)")
    w = n // world
    return rank * w, (rank + 1) * w


def broadcast_id(group=None, make_id=None) -> bytes:
    """Rank 0 creates an id (NCCL's by default) and every rank returns it."""
    import torch
    import torch.distributed as dist

    rank = dist.get_rank(group)
    # an NCCL group moves CUDA tensors only
    dev = (torch.device("cuda", torch.cuda.current_device())
           if dist.get_backend(group) == "nccl" else torch.device("cpu"))
    buf = torch.zeros(128, dtype=torch.uint8, device=dev)
    if rank == 0:
        raw = make_id() if make_id else _nccl_unique_id()
        buf.copy_(torch.frombuffer(bytearray(raw), dtype=torch.uint8))
    dist.broadcast(buf, src=0, group=group)
    return bytes(buf.cpu().tolist())


def _nccl_unique_id() -> bytes:
    out = ctypes.create_string_buffer(128)
    call("rtb_nccl_unique_id", out)
    return out.raw


class NsplitGemm:
    """C = A . B with B's columns split across ranks and C all-gathered."""

    def __init__(self, ctx, world: int, rank: int, group=None):
        self.ctx = ctx
        self.world, self.rank = world, rank
        uid = broadcast_id(group)
        comm = ctypes.c_void_p()
        call("rtb_nccl_comm_init", ctx.handle, ctypes.c_char_p(uid), world, rank,
             ctypes.byref(comm))
        self.comm = comm

    def close(self) -> None:
        if self.comm:
            call("rtb_nccl_comm_destroy", self.comm)
            self.comm = None

    def __call__(self, a, b_local, precision: int = _lib.PREC_DEFAULT, out=None, parts=None):
        """a: [M,K] (replicated), b_local: [K, N/world] (this rank's columns),
        both contiguous float32 CUDA tensors; returns C [M, N] on every rank
        (in `out` when given; `parts` is the [world, M, N/world] gather buffer)."""
        import torch
        M, K = a.shape
        nl = b_local.shape[1]
        N = nl * self.world
        if parts is None:
            parts = torch.empty((self.world, M, nl), dtype=torch.float32, device=a.device)
        c = out if out is not None else torch.empty((M, N), dtype=torch.float32, device=a.device)
        stream = ctypes.c_void_p(torch.cuda.current_stream(a.device).cuda_stream)
        call("rtb_sgemm_nsplit_allgather", self.ctx.handle, self.comm, M, N, K,
             ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b_local.data_ptr()),
             ctypes.c_void_p(parts.data_ptr()), ctypes.c_void_p(c.data_ptr()), precision, stream)
        return c


class _DeviceArray:
    """A device pointer with __cuda_array_interface__ (zero-copy torch view)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4",
                                         "data": (ptr, False), "version": 3, "strides": None}


class NsplitGemmP2P:
    """C = A . B with B's columns split across ranks, fused with the exchange:
    the GEMM epilogue writes every tile into all ranks' C over NVLink
    (rtb_sgemm_nsplit_p2p).  C is a library-owned peer buffer of [M, N]; `c`
    is this rank's copy as a torch tensor (valid until the next call)."""

    def __init__(self, ctx, world: int, rank: int, M: int, N: int, group=None):
        import torch
        self.ctx = ctx
        self.world, self.rank = world, rank
        self.M, self.N = M, N
        uid = broadcast_id(group)
        comm = ctypes.c_void_p()
        call("rtb_nccl_comm_init", ctx.handle, ctypes.c_char_p(uid), world, rank,
             ctypes.byref(comm))
        self.comm = comm
        pb = ctypes.c_void_p()
        call("rtb_peer_buffer_create", ctx.handle, comm, M * N * 4, ctypes.byref(pb))
        self.pbuf = pb
        local = ctypes.c_void_p()
        call("rtb_peer_buffer_local", pb, ctypes.byref(local))
        self.c = torch.as_tensor(_DeviceArray(local.value, (M, N)),
                                 device=torch.device("cuda", torch.cuda.current_device()))

    def close(self) -> None:
        if self.pbuf:
            call("rtb_peer_buffer_destroy", self.pbuf, self.comm)
            self.pbuf = None
        if self.comm:
            call("rtb_nccl_comm_destroy", self.comm)
            self.comm = None

    def __call__(self, a, b_local, precision: int = _lib.PREC_DEFAULT):
        """a: [M,K] (replicated), b_local: [K, N/world]; returns C [M, N]."""
        import torch
        K = a.shape[1]
        stream = ctypes.c_void_p(torch.cuda.current_stream(a.device).cuda_stream)
        call("rtb_sgemm_nsplit_p2p", self.ctx.handle, self.comm, self.pbuf, self.M, self.N, K,
             ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b_local.data_ptr()), precision, stream)
        return self.c


__all__ = ["shard_columns", "broadcast_id", "NsplitGemm", "NsplitGemmP2P", "lib"]
