"""3-layer MLP forward (batch 4096, 1024->4096->4096->1024, Linear+ReLU after
the first two layers, Kaiming-uniform weights, zero biases, seed 2) against
nn::Linear's CPU path.  Rows are independent, so a 64-row sample through the
oracle is an exact restatement of those rows of the full-size forward."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("prec,tol", [(0, 1e-5), (1, 5e-3)])
def test_mlp_forward_rows(gpu, orc, prec, tol):
    rb = gpu
    dims = [1024, 4096, 4096, 1024]
    x = orc.normal((4096, 1024), 2, 0)
    ws = []
    for i in range(3):
        bound = math.sqrt(3.0) * math.sqrt(2.0) / math.sqrt(dims[i])
        ws.append(orc.uniform((dims[i + 1], dims[i]), 2, 1 + i, -bound, bound))
    a = torch.from_numpy(x).cuda()
    for i in range(3):
        w = torch.from_numpy(ws[i]).cuda()
        a = rb.sgemm(a, w.t(), bias=torch.zeros(dims[i + 1], device="cuda"),
                     act=rb.ACT_RELU if i < 2 else rb.ACT_NONE, precision=prec)
    torch.cuda.synchronize()
    got = a.cpu().numpy()
    rows = np.array([0, 1, 777, 2048, 4095] + list(range(100, 159)))
    r = x[rows]
    r64 = r.astype(np.float64)
    for i in range(3):
        r = orc.linear(r, ws[i], np.zeros(dims[i + 1], np.float32), relu=i < 2)
        r64 = r64 @ ws[i].T.astype(np.float64)
        if i < 2:
            r64 = np.maximum(r64, 0.0)
    assert orc.rel_frob(got[rows], r64) <= tol
    assert orc.rel_frob(got[rows], r.astype(np.float64)) <= 2 * tol
