"""3xTF32 split modes beyond the parity suite's defaults:

- the round-to-nearest hi part (RTB_SPLIT_TRUNC=0, read once per process,
  hence a subprocess) instead of the tensor core's own truncation, for every
  A producer of the 64-column (wide) mode: tiled TMA, one-tap and multi-tap
  TMA im2col, cp.async gather;
- non-finite input pixels in convs whose last k-block holds fewer filter taps
  than it has room for (multi-tap im2col, Cp = 8 and 16): the converters
  zero the k columns past the last tap, so outputs whose window misses the
  non-finite pixels stay finite and exact, as in the reference."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("ci,k", [(6, 3), (16, 3), (13, 5)])
def test_multitap_partial_last_kblock_nonfinite_pixels(gpu, orc, ci, k):
    """Cp = 8 (4 taps per k-block) and Cp = 16 (2 taps): 9 or 25 taps leave the
    last k-block partly empty, and the tile's other tap slots hold an earlier
    k-block's pixels.  About 0.5% of the input pixels are +inf or NaN; every
    output whose window misses them must be finite and match float64, the
    others must be non-finite, as in the reference."""
    n, h, w, co = 8, 32, 32, 64
    x = orc.normal((n, ci, h, w), 13, 1)
    rng = np.random.default_rng(13)
    bad = rng.random((n, h, w)) < 0.005
    idx = np.argwhere(bad)
    for j, (b, i, jj) in enumerate(idx):
        x[b, :, i, jj] = np.inf if j % 2 == 0 else np.nan
    wt = orc.normal((co, ci, k, k), 13, 2, 0.0, float(np.sqrt(2.0 / (ci * k * k))))
    pad = (k // 2, k // 2)
    y = _host(gpu.conv2d_fwd(_dev(x), _dev(wt), None, (1, 1), pad, precision=0))
    # windows that touch a non-finite pixel (any channel)
    flag = bad.astype(np.float32)[:, None, :, :]
    touched = orc.conv2d_f64(flag, np.ones((1, 1, k, k), np.float32), (1, 1), pad)[:, 0] > 0
    clean = np.broadcast_to(~touched[:, None], y.shape)
    assert clean.mean() > 0.8
    assert np.all(np.isfinite(y[clean]))
    assert not np.any(np.isfinite(y[~clean]))
    xc = np.where(np.isfinite(x), x, 0.0).astype(np.float32)
    ref = orc.conv2d_f64(xc, wt, (1, 1), pad)
    assert orc.rel_frob(y[clean], ref[clean]) <= 1e-5


_RNA_SCRIPT = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
import rustorch_b200 as rb
from oracle import oracle as orc
orc.build()
dev = torch.device("cuda", 0)
def d(a): return torch.from_numpy(np.ascontiguousarray(a)).to(dev)
errs = {}
# GEMM on 64-column tiles (tiled TMA A)
a = orc.normal((2048 + 37, 300), 21, 1); b = orc.normal((300, 64), 21, 2)
c = rb.sgemm(d(a), d(b), precision=0); torch.cuda.synchronize()
errs["gemm_n64"] = orc.rel_frob(c.cpu().numpy(), orc.matmul_f64(a, b))
# convs: one-tap TMA im2col (Cp = 64), multi-tap (Cp = 8, 16), gather (Cp = 4)
for name, xs, ws in [("im2col_cp64", (4, 64, 20, 20), (64, 64, 3, 3)),
                     ("multitap_cp8", (8, 6, 32, 32), (64, 6, 3, 3)),
                     ("multitap_cp16", (8, 13, 32, 32), (64, 13, 5, 5)),
                     ("gather_cp4", (2, 3, 21, 17), (64, 3, 3, 3))]:
    x = orc.normal(xs, 22, 1)
    w = orc.normal(ws, 22, 2, 0.0, float(np.sqrt(2.0 / np.prod(ws[1:]))))
    pad = (ws[2] // 2, ws[3] // 2)
    y = rb.conv2d_fwd(d(x), d(w), None, (1, 1), pad, precision=0); torch.cuda.synchronize()
    errs[name] = orc.rel_frob(y.cpu().numpy(), orc.conv2d_f64(x, w, (1, 1), pad))
print(repr(errs))
"""


def test_round_to_nearest_hi_written_back(gpu):
    """RTB_SPLIT_TRUNC=0: the hi part is TF32 rounded to nearest (lo = x - hi
    exactly), every producer of the wide mode within the 3xTF32 bound."""
    env = dict(os.environ, RTB_SPLIT_TRUNC="0")
    r = subprocess.run([sys.executable, "-c", _RNA_SCRIPT, ROOT], env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    errs = eval(r.stdout.strip().splitlines()[-1])
    assert len(errs) == 5
    for name, e in errs.items():
        assert e <= 1e-5, (name, e)
