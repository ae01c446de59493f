"""Host-side multi-GPU orchestration on CPU ranks (gloo, world_size 2): the
NCCL-id broadcast, the N-split column partition, and the [P][M][N/P] gather
layout that rtb_sgemm_nsplit_allgather repacks into C [M][N] (gloo stands in
for NCCL; the per-rank block product is a plain matmul)."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest


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
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from rustorch_b200 import dist as rdist
        uid = rdist.broadcast_id(make_id=lambda: bytes(range(128)))
        M, K, N = 33, 20, 24
        rng = np.random.default_rng(7)
        a = rng.standard_normal((M, K))
        b = rng.standard_normal((K, N))
        lo, hi = rdist.shard_columns(N, world, rank)
        c_local = torch.from_numpy(a @ b[:, lo:hi]).contiguous()
        parts = [torch.empty_like(c_local) for _ in range(world)]
        dist.all_gather(parts, c_local)
        stacked = torch.stack(parts)                       # [P, M, N/P]
        c = stacked.permute(1, 0, 2).reshape(M, N)         # the repack the kernel does
        q.put((rank, uid == bytes(range(128)), bool(np.allclose(c.numpy(), a @ b)),
               (lo, hi)))
    finally:
        dist.destroy_process_group()


def test_nsplit_orchestration_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert all(r[1] and r[2] for r in res), res
    assert [r[3] for r in res] == [(0, 12), (12, 24)]


def test_shard_columns_rules():
    from rustorch_b200.dist import shard_columns
    assert shard_columns(16384, 8, 7) == (14336, 16384)
    with pytest.raises(ValueError):
        shard_columns(10, 4, 0)
    with pytest.raises(ValueError):
        shard_columns(8, 2, 2)
