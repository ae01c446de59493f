"""ResNet-18 forward (inference, BatchNorm folded) on the B200 against the
oracle composition of the reference's CPU ops on the same parameters.

The model's parameters are read back through the C shim so both sides use
identical weights; the input is the documented seeded N(0,1) batch.  Each of
the 20 convs carries the 3xTF32 contraction error (<= 1e-5 relative); the
logits are checked at 1e-4 relative Frobenius after 21 chained contractions."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _params(rb, h):
    L = rb.lib()
    n = L.rtb_resnet18_num_params(h)
    out = []
    for i in range(n):
        shape = (ctypes.c_int64 * 4)()
        rb.call("rtb_resnet18_get_param", h, i, None, shape)
        sh = [shape[k] for k in range(4)]
        arr = np.empty(int(np.prod(sh)), np.float32)
        rb.call("rtb_resnet18_get_param", h, i, ctypes.c_void_p(arr.ctypes.data), shape)
        out.append(arr.reshape(sh))
    convs = [(out[2 * i], out[2 * i + 1].reshape(-1)) for i in range(20)]
    fc_w = out[40].reshape(1000, 512)
    fc_b = out[41].reshape(-1)
    return convs, fc_w, fc_b


def _oracle_forward(orc, x, convs, fc_w, fc_b):
    def conv(t, i, stride, pad, relu, residual=None):
        w, b = convs[i]
        y, _ = orc.conv2d(t, w, stride, pad)
        y = orc.add_bias_nchw(y, b)
        if residual is not None:
            y = y + residual
        return orc.relu(y) if relu else y

    t = conv(x, 0, (2, 2), (3, 3), True)
    stem = t
    t = orc.max_pool2d(t, (3, 3), (2, 2), (1, 1))
    i = 1
    for st in range(4):
        for blk in range(2):
            down = st > 0 and blk == 0
            s = 2 if down else 1
            a = conv(t, i, (s, s), (1, 1), True)
            ident = conv(t, i + 2, (2, 2), (0, 0), False) if down else t
            t = conv(a, i + 1, (1, 1), (1, 1), True, ident)
            i += 3 if down else 2
    pooled = orc.global_avg_pool(t)
    return orc.linear(pooled, fc_w, fc_b), stem


def test_resnet18_forward_matches_oracle(gpu, orc):
    rb = gpu
    h = ctypes.c_void_p()
    rb.call("rtb_resnet18_create", 0, 3, rb.PREC_3XTF32, ctypes.byref(h))
    try:
        assert rb.lib().rtb_resnet18_flops_per_image(h) == 3628146688  # 3.628 GFLOP / image
        convs, fc_w, fc_b = _params(rb, h)
        assert convs[0][0].shape == (64, 3, 7, 7) and fc_w.shape == (1000, 512)
        x = orc.normal((2, 3, 224, 224), 3, 1000)
        xd = torch.from_numpy(x).cuda()
        logits = torch.empty((2, 1000), device="cuda")
        rb.call("rtb_resnet18_forward", h, 2, ctypes.c_void_p(xd.data_ptr()),
                ctypes.c_void_p(logits.data_ptr()), None)
        torch.cuda.synchronize()
        got = logits.cpu().numpy()
        ref, _ = _oracle_forward(orc, x, convs, fc_w, fc_b)
        err = orc.rel_frob(got, ref.astype(np.float64))
        assert err <= 1e-4, err
        assert np.array_equal(got.argmax(1), ref.argmax(1))
        # a second call at a smaller batch reuses the buffers
        rb.call("rtb_resnet18_forward", h, 1, ctypes.c_void_p(xd.data_ptr()),
                ctypes.c_void_p(logits.data_ptr()), None)
        torch.cuda.synchronize()
        assert orc.rel_frob(logits[:1].cpu().numpy(), ref[:1].astype(np.float64)) <= 1e-4
        assert rb.get_context(0).device_error() == 0
    finally:
        rb.call("rtb_resnet18_destroy", h)


def test_resnet18_forward_full_batch_256(gpu, orc):
    """The benchmarked configuration: the whole B=256 batch in one forward
    (M reaches 3.2M rows on the stem, so other tile, split and grid-stride
    paths run than at B=2); images 0, 127 and 255 are checked against the
    oracle composition of the reference's CPU ops, and the rest of the batch
    must be finite."""
    rb = gpu
    h = ctypes.c_void_p()
    rb.call("rtb_resnet18_create", 0, 3, rb.PREC_3XTF32, ctypes.byref(h))
    try:
        convs, fc_w, fc_b = _params(rb, h)
        x = orc.normal((256, 3, 224, 224), 3, 1000)
        xd = torch.from_numpy(x).cuda()
        logits = torch.empty((256, 1000), device="cuda")
        rb.call("rtb_resnet18_forward", h, 256, ctypes.c_void_p(xd.data_ptr()),
                ctypes.c_void_p(logits.data_ptr()), None)
        torch.cuda.synchronize()
        got = logits.cpu().numpy()
        assert np.isfinite(got).all()
        pick = [0, 127, 255]
        ref, _ = _oracle_forward(orc, np.ascontiguousarray(x[pick]), convs, fc_w, fc_b)
        err = orc.rel_frob(got[pick], ref.astype(np.float64))
        assert err <= 1e-4, err
        assert np.array_equal(got[pick].argmax(1), ref.argmax(1))
        assert rb.get_context(0).device_error() == 0
    finally:
        rb.call("rtb_resnet18_destroy", h)
