"""N-split GEMM on 2 GPUs (one process per GPU): GEMM then NCCL all-gather of
C, and the fused form whose epilogue writes every tile into both ranks' C over
NVLink.  Skipped on a single-GPU box."""
import multiprocessing as mp
import os
import socket

import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        import rustorch_b200 as rb
        from rustorch_b200 import dist as rdist
        ctx = rb.get_context(rank)
        g = torch.Generator().manual_seed(4)
        M, K, N = 1024, 2048, 4096
        a = torch.randn(M, K, generator=g)
        b = torch.randn(K, N, generator=g)
        lo, hi = rdist.shard_columns(N, world, rank)
        ns = rdist.NsplitGemm(ctx, world, rank)
        da, db = a.cuda(), b[:, lo:hi].contiguous().cuda()
        c = ns(da, db)
        torch.cuda.synchronize()
        ref = a.double() @ b.double()
        err = float((c.cpu().double() - ref).norm() / ref.norm())
        ns.close()
        # fused GEMM + exchange over NVLink: the same local GEMM, so the same
        # bits as GEMM-then-all-gather; twice, the second with other inputs
        fused = rdist.NsplitGemmP2P(ctx, world, rank, M, N)
        c2 = fused(da, db).clone()
        same = bool(torch.equal(c2, c))
        a3 = torch.randn(M, K, generator=g)
        c3 = fused(a3.cuda(), db).cpu().double()
        ref3 = a3.double() @ b.double()
        err3 = float((c3 - ref3).norm() / ref3.norm())
        fused.close()
        q.put((rank, err, ctx.device_error(), same, err3))
    finally:
        dist.destroy_process_group()


def test_nsplit_allgather_two_gpus(gpu):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    for rank, err, code, same, err3 in res:
        assert err <= 1e-5 and code == 0, res
        assert same and err3 <= 1e-5, res
