"""Run ResNet-18 forwards on one GPU (for timing and profiling a whole forward).

    python -m rustorch_b200.resnet18_run [BATCH] [FORWARDS]

Creates the model (seed 3, 3xTF32) with rtb_resnet18_create, then runs
FORWARDS forwards (default 3) of a seeded [BATCH, 3, 224, 224] batch (default
64 images) through rtb_resnet18_forward on cuda:0, checks the device error
word and prints the sum of |logits|.  Each forward is 24 launches (space-to-
depth stem prologue, 20 convolutions, max pool, average pool, fc), after the
20 weight-prepack launches of the model's construction.
"""
from __future__ import annotations

import ctypes
import sys

import torch

from . import call, fill_normal, get_context, PREC_3XTF32


def main(argv) -> int:
    batch = int(argv[1]) if len(argv) > 1 else 64
    forwards = int(argv[2]) if len(argv) > 2 else 3
    h = ctypes.c_void_p()
    call("rtb_resnet18_create", 0, 3, PREC_3XTF32, ctypes.byref(h))
    try:
        x = torch.from_numpy(fill_normal((batch, 3, 224, 224), 3, 1000)).cuda()
        y = torch.empty((batch, 1000), device="cuda")
        for _ in range(forwards):
            call("rtb_resnet18_forward", h, batch, ctypes.c_void_p(x.data_ptr()),
                 ctypes.c_void_p(y.data_ptr()), None)
        torch.cuda.synchronize()
        if get_context(0).device_error():
            print("device error word set", file=sys.stderr)
            return 1
        print(f"resnet18 batch {batch} x {forwards} forwards: sum |logits| = "
              f"{float(y.abs().sum()):.6g}")
    finally:
        call("rtb_resnet18_destroy", h)
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
