"""Benchmark of the B200 dense-contraction path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Workloads (default: resnet18):
  resnet18  ResNet-18 forward (BatchNorm folded), B=256 images per GPU, x ~ N(0,1), seed 3.
            Batch-sharded at N>1 (no collective).  The line also carries `gemm`: the
            device-timed f32 matmul 1024^3 (replicas) and 8192^3 (N-split at N>1).
  conv      Conv2d+bias+ReLU, ResNet-50 stage-2 3x3 layer: x [32,128,28,28] ~ N(0,1),
            w [128,128,3,3] Kaiming-normal, b ~ U(-0.1,0.1), stride 1, pad 1, seed 1.
            One step = one reference-facing conv call (NCHW in/out).  Replicas at N>1.
  conv_r50s1, conv_r50s3, conv_r50s4
            the same call on ResNet-50's other 3x3 layers at batch 32: 64 channels at
            56x56, 256 at 14x14, 512 at 7x7 (seed 1 + stage).
  gemm1024  f32 matmul 1024^3, A, B ~ N(0,1), seed 0.  Replicas at N>1.
  gemm2048, gemm4096, gemm8192, gemm16384
            square f32 matmul sweep, seed 4.  2048/4096 replicas at N>1;
            8192/16384 N-split across the GPUs, the GEMM epilogue storing every
            tile into all ranks' C over NVLink (RTB_NSPLIT_NCCL=1: GEMM then NCCL
            all-gather instead); strong scaling: one problem per job.
  gemm_m16, gemm_m32, gemm_m64, gemm_m128, gemm_m256
            skinny f32 matmul M x 8192 x 8192, seed 4 (HBM-bound for M < 128:
            roofline in GB/s).  Replicas at N>1.
  mlp       3-layer MLP forward, batch 4096, 1024->4096->4096->1024, seed 2.  Replicas.
  conv_bwd  Conv2dBackward (grad_input + grad_weight) of the conv layer above, dy ~ N(0,1).

Timing: W warm-up steps, then K steps between barrier + synchronize, CUDA
events on the launching stream, max over ranks.  Inputs/outputs rotate over
enough copies to exceed the 126 MB L2 so no step reads the previous step's
data from L2.  `value` is the whole-job throughput (sum over ranks of the
algorithmic FLOPs / max time).  `e2e` times the same call through the C ABI
with host buffers (pinned H2D of the step's inputs, D2H of its output), steps
pipelined over 2-3 streams so one step's copies overlap another's call.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024

# DRAM bytes (read + write) per launch of each workload's dominant kernel, from
# one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum); the capture and
# its command are summarised in the named profiles/ file.
TRAFFIC = {
    "resnet18": (5.061e9, "profiles/resnet18_fwd_launches.md"),
    "conv": (14.16e6, "profiles/conv2d_bias_relu_r50s2_3x3.md"),
    "conv_r50s4": (22.20e6, "profiles/kernel_counters_gemm_conv.md"),
    "gemm1024": (8.48e6, "profiles/kernel_counters_gemm_conv.md"),
    "gemm8192": (5.228e9, "profiles/sgemm_8192_3xtf32.md"),
    "gemm_m16": (272.7e6, "profiles/sgemm_small_m16_8192.md"),
    "gemm_m64": (277.7e6, "profiles/sgemm_skinny_m64_transposed.md"),
    "gemm_m256": (280.6e6, "profiles/kernel_counters_gemm_conv.md"),
    "mlp": (910.7e6, "profiles/kernel_counters_gemm_conv.md"),
    "linear_norm": (208.1e6, "profiles/linear_norm_relu_8192x1024x4096.md"),
}
# Tensor-pipe activity of each workload's dominant kernel(s) as ncu counts it
# (sm__pipe_tensor_cycles_active, % of elapsed cycles), from the named capture.
TENSOR_PIPE = {
    "resnet18": (0.488, "profiles/resnet18_fwd_launches.md"),
    "conv": (0.338, "profiles/conv2d_bias_relu_r50s2_3x3.md"),
    "conv_r50s4": (0.302, "profiles/kernel_counters_gemm_conv.md"),
    "gemm1024": (0.2015, "profiles/kernel_counters_gemm_conv.md"),
    "gemm8192": (0.747, "profiles/sgemm_8192_3xtf32.md"),
    "gemm_m64": (0.289, "profiles/sgemm_skinny_m64_transposed.md"),
    "gemm_m256": (0.504, "profiles/kernel_counters_gemm_conv.md"),
    "mlp": (0.677, "profiles/kernel_counters_gemm_conv.md"),
    "linear_norm": (0.685, "profiles/linear_norm_relu_8192x1024x4096.md"),
}
# DRAM bytes per launch of a workload's second kernel (roofline.secondary)
TRAFFIC_SECONDARY = {
    "linear_norm": (211.2e6, "profiles/linear_norm_relu_8192x1024x4096.md"),
}
PRECISION = [0]  # rtb precision enum used by every workload call (0 = 3xTF32, 1 = TF32)
MMAS_PER_MAC = [3]


# ------------------------------------------------------------------ helpers
def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "basis": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "basis": "fallback"}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML every
    ~1 ms by a background thread while the timed region runs (the timed
    regions here are milliseconds long, below nvidia-smi's 200 ms cadence)."""

    REASONS = {"hw_slowdown": 0x8, "sw_power_cap": 0x4, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, torch_dev):
        self.rows = []
        self.h = None
        self.stop = threading.Event()
        try:
            import pynvml
            self.nv = pynvml
            pynvml.nvmlInit()
            import torch
            pr = torch.cuda.get_device_properties(torch_dev)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            try:
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(torch_dev.index or 0)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # NVML unavailable: report unsampled
            self.err = str(e)
            self.h = None

    def sample(self):
        if self.h is None:
            return
        try:
            sm = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
            try:
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except AttributeError:
                rs = self.nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
            self.rows.append((sm, rs))
        except Exception:
            pass

    def _run(self):
        while not self.stop.is_set():
            self.sample()
            time.sleep(0.001)

    def __enter__(self):
        self.sample()
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()
        return self

    def __exit__(self, *a):
        self.stop.set()
        self.t.join(timeout=2)
        self.sample()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        reasons = sorted({n for _, rs in self.rows for n, bit in self.REASONS.items() if rs & bit})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.rows), "source": "nvml"}


def _host_threads():
    """Host threads this process may really use: its CPU affinity, capped by a
    cgroup CPU quota when one is set (os.cpu_count() reports the machine)."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    try:
        quota, period = open("/sys/fs/cgroup/cpu.max").read().split()[:2]
        if quota != "max":
            n = max(1, min(n, int(int(quota) // int(period))))
    except (OSError, ValueError):
        pass
    return n


def _dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


class E2EPipeline:
    """End-to-end steps on three streams: uploads (H2D) on one, the calls on
    one, downloads (D2H) on one, so each copy engine moves step after step
    back to back while the calls run between them (PCIe is full duplex).
    `depth` slots of device and pinned host buffers rotate; events keep a
    slot's upload behind the previous call that read it and its call behind
    the previous download of its result.  Every step still moves its own
    inputs and result.  Per step:
        k = pipe.next()            # then the H2D copies on pipe.h_in
        pipe.compute(k)            # then the call(s) on pipe.h_c / pipe.s_c
        pipe.download(k)           # then the D2H copies on pipe.h_out
        pipe.finish(k)
    """

    def __init__(self, torch, dev, depth):
        self.torch, self.dev, self.depth = torch, dev, depth
        self.s_in, self.s_c, self.s_out = (torch.cuda.Stream(dev) for _ in range(3))
        self.h_in, self.h_c, self.h_out = (ctypes.c_void_p(st.cuda_stream)
                                           for st in (self.s_in, self.s_c, self.s_out))
        self.ev_in = [torch.cuda.Event() for _ in range(depth)]
        self.ev_comp = [torch.cuda.Event() for _ in range(depth)]
        self.ev_out = [torch.cuda.Event() for _ in range(depth)]
        self.used = [False] * depth
        self.i = 0

    def next(self):
        k = self.i % self.depth
        self.i += 1
        if self.used[k]:  # the slot's inputs were read by its previous call
            self.s_in.wait_event(self.ev_comp[k])
        return k

    def compute(self, k):
        self.ev_in[k].record(self.s_in)
        self.s_c.wait_event(self.ev_in[k])
        if self.used[k]:  # the slot's result buffer was read by its previous download
            self.s_c.wait_event(self.ev_out[k])

    def download(self, k):
        self.ev_comp[k].record(self.s_c)
        self.s_out.wait_event(self.ev_comp[k])

    def finish(self, k):
        self.ev_out[k].record(self.s_out)
        self.used[k] = True

    def begin(self, ev):
        for st in (self.s_in, self.s_c, self.s_out):
            st.wait_event(ev)

    def join(self, cur):
        for st in (self.s_in, self.s_c, self.s_out):
            e = self.torch.cuda.Event()
            e.record(st)
            cur.wait_event(e)


def _pinned_copy(rb, ctx, arr):
    p = ctypes.c_void_p()
    rb.call("rtb_host_alloc", ctx.handle, ctypes.byref(p), arr.nbytes)
    ctypes.memmove(p, arr.ctypes.data, arr.nbytes)
    return p


def _pinned_empty(rb, ctx, nbytes):
    p = ctypes.c_void_p()
    rb.call("rtb_host_alloc", ctx.handle, ctypes.byref(p), nbytes)
    return p


# ------------------------------------------------------------------ workloads
# ResNet-50's 3x3 layers at batch 32: stage -> (channels, image side).  Stage 2
# is the conv workload (seed 1); the other stages draw their inputs with seed
# 1 + stage, as their GPU parity tests do.
R50_STAGES = {1: (64, 56), 2: (128, 28), 3: (256, 14), 4: (512, 7)}


def _r50_seed(stage):
    return 1 if stage == 2 else 1 + stage


class ConvWorkload:
    name = "conv2d_bias_relu_resnet50_3x3"

    def _shape(self, stage):
        c, hw = R50_STAGES[stage]
        self.stage = stage
        self.seed = _r50_seed(stage)
        self.N, self.C, self.H, self.W, self.Co = 32, c, hw, hw, c
        self.flops = 2.0 * self.N * self.H * self.W * self.Co * self.C * 9
        if stage != 2:
            self.name = f"conv2d_bias_relu_resnet50_s{stage}_3x3"

    def __init__(self, rb, torch, dev, stage=2):
        self.rb, self.torch, self.dev = rb, torch, dev
        self._shape(stage)
        n = self.N * self.C * self.H * self.W
        x = rb.fill_normal((self.N, self.C, self.H, self.W), self.seed, 0)
        w = rb.fill_normal((self.Co, self.C, 3, 3), self.seed, 1, 0.0,
                           math.sqrt(2.0 / (self.C * 9)))
        b = rb.fill_uniform((self.Co,), self.seed, 2, -0.1, 0.1)
        self.host = {"x": x, "w": w, "b": b}
        bytes_per_set = 2 * n * 4
        self.nsets = max(2, int(math.ceil(2 * L2_BYTES / bytes_per_set)))
        self.xs = [torch.from_numpy(x).to(dev) for _ in range(self.nsets)]
        self.ys = [torch.empty((self.N, self.Co, self.H, self.W), device=dev)
                   for _ in range(self.nsets)]
        self.w = torch.from_numpy(w).to(dev)
        self.b = torch.from_numpy(b).to(dev)
        self.i = 0
        self.config = {"workload": f"conv2d+bias+relu ResNet-50 stage-{stage} 3x3",
                       "input": [32, self.C, self.H, self.W],
                       "weight": [self.Co, self.C, 3, 3], "stride": 1,
                       "pad": 1, "seed": self.seed, "layout": "NCHW in/out",
                       "l2": f"rotating {self.nsets} input/output sets "
                             f"({self.nsets * bytes_per_set / 2**20:.0f} MiB > 126 MiB L2)"}
        self.launches_per_step = 2  # NCHW->NHWC + weight prepack (one launch), implicit-GEMM conv

    def step(self):
        rb = self.rb
        k = self.i % self.nsets
        self.i += 1
        x, y = self.xs[k], self.ys[k]
        ctx = rb.get_context(self.dev.index or 0)
        stream = ctypes.c_void_p(self.torch.cuda.current_stream(self.dev).cuda_stream)
        rb.call("rtb_conv2d_fwd", ctx.handle, self.N, self.C, self.H, self.W, self.Co, 3, 3, 1, 1, 1,
                1, ctypes.c_void_p(x.data_ptr()), rb.LAYOUT_NCHW,
                ctypes.c_void_p(self.w.data_ptr()), ctypes.c_void_p(self.b.data_ptr()), None,
                rb.ACT_RELU, ctypes.c_void_p(y.data_ptr()), rb.LAYOUT_NCHW, PRECISION[0], stream)

    # dominant kernel alone (NHWC input + prepacked weight), for the roofline
    def kernel_setup(self):
        torch, rb = self.torch, self.rb
        ctx = rb.get_context(self.dev.index or 0)
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)
        self.xh = [torch.empty((self.N, self.H, self.W, self.C), device=self.dev)
                   for _ in range(self.nsets)]
        for k in range(self.nsets):
            rb.call("rtb_nchw_to_nhwc_padded", ctx.handle, self.N, self.C, self.H, self.W,
                    ctypes.c_void_p(self.xs[k].data_ptr()), ctypes.c_void_p(self.xh[k].data_ptr()),
                    stream)
        self.wp = torch.empty((self.Co * 9 * self.C,), device=self.dev)
        rb.call("rtb_conv2d_prepack_weight", ctx.handle, self.Co, self.C, 3, 3,
                ctypes.c_void_p(self.w.data_ptr()), ctypes.c_void_p(self.wp.data_ptr()), stream)

    def kernel_step(self):
        rb = self.rb
        k = self.i % self.nsets
        self.i += 1
        ctx = rb.get_context(self.dev.index or 0)
        stream = ctypes.c_void_p(self.torch.cuda.current_stream(self.dev).cuda_stream)
        rb.call("rtb_conv2d_fwd_packed", ctx.handle, self.N, self.C, self.H, self.W, self.Co, 3, 3,
                1, 1, 1, 1, ctypes.c_void_p(self.xh[k].data_ptr()),
                ctypes.c_void_p(self.wp.data_ptr()), ctypes.c_void_p(self.b.data_ptr()), None,
                rb.ACT_RELU, ctypes.c_void_p(self.ys[k].data_ptr()), rb.LAYOUT_NCHW,
                PRECISION[0], stream)

    def e2e_setup(self):
        rb, torch = self.rb, self.torch
        ctx = rb.get_context(self.dev.index or 0)
        self.pipe = E2EPipeline(torch, self.dev, 3)
        ybytes = self.N * self.Co * self.H * self.W * 4
        self.slots = []
        for _ in range(self.pipe.depth):
            slot = {key: (_pinned_copy(rb, ctx, arr), arr.nbytes) for key, arr in self.host.items()}
            slot["y"] = (_pinned_empty(rb, ctx, ybytes), ybytes)
            slot["dx"] = torch.empty((self.N, self.C, self.H, self.W), device=self.dev)
            slot["dw"] = torch.empty_like(self.w)
            slot["db"] = torch.empty_like(self.b)
            slot["dy"] = torch.empty((self.N, self.Co, self.H, self.W), device=self.dev)
            self.slots.append(slot)
        self.h2d_bytes = sum(arr.nbytes for arr in self.host.values())
        self.d2h_bytes = ybytes

    def e2e_step(self):
        rb = self.rb
        ctx = rb.get_context(self.dev.index or 0)
        pipe = self.pipe
        k = pipe.next()
        slot = self.slots[k]
        for key, dst in (("x", slot["dx"]), ("w", slot["dw"]), ("b", slot["db"])):
            p, nb = slot[key]
            rb.call("rtb_memcpy_h2d", ctx.handle, ctypes.c_void_p(dst.data_ptr()), p, nb, pipe.h_in)
        pipe.compute(k)
        y = slot["dy"]
        rb.call("rtb_conv2d_fwd", ctx.handle, self.N, self.C, self.H, self.W, self.Co, 3, 3, 1, 1, 1,
                1, ctypes.c_void_p(slot["dx"].data_ptr()), rb.LAYOUT_NCHW,
                ctypes.c_void_p(slot["dw"].data_ptr()), ctypes.c_void_p(slot["db"].data_ptr()),
                None, rb.ACT_RELU, ctypes.c_void_p(y.data_ptr()), rb.LAYOUT_NCHW, PRECISION[0],
                pipe.h_c)
        pipe.download(k)
        p, nb = slot["y"]
        rb.call("rtb_memcpy_d2h", ctx.handle, p, ctypes.c_void_p(y.data_ptr()), nb, pipe.h_out)
        pipe.finish(k)

    def e2e_teardown(self):
        ctx = self.rb.get_context(self.dev.index or 0)
        for slot in self.slots:
            for key in ("x", "w", "b", "y"):
                self.rb.call("rtb_host_free", ctx.handle, slot[key][0])
        self.slots = []

    # CPU baseline: the reference's own CPU path (oracle restatement) on a sample
    def cpu_sample(self, threads):
        from oracle import oracle as orc
        x = orc.normal((self.N, self.C, self.H, self.W), self.seed, 0)
        w = orc.normal((self.Co, self.C, 3, 3), self.seed, 1, 0.0, math.sqrt(2.0 / (self.C * 9)))
        b = orc.uniform((self.Co,), self.seed, 2, -0.1, 0.1)
        nimg = 2
        xs = x[:nimg].copy()
        orc.conv2d_bias_relu(xs[:1], w, b, (1, 1), (1, 1), threads=threads)  # warm
        t0 = time.perf_counter()
        reps = 0
        while True:
            orc.conv2d_bias_relu(xs, w, b, (1, 1), (1, 1), threads=threads)
            reps += 1
            if time.perf_counter() - t0 > 10.0 or reps >= 20:
                break
        dt = (time.perf_counter() - t0) / reps
        flops = self.flops * nimg / self.N
        return flops / dt / 1e12, (f"{nimg} of 32 images per call (im2col + row-parallel core, "
                                   f"bias, ReLU), {reps} calls")


class ConvBwdWorkload:
    """Conv2dBackward of the ResNet-50 stage-2 3x3 layer: grad_input and
    grad_weight for x [32,128,28,28], w [128,128,3,3], dy ~ N(0,1), NCHW."""
    name = "conv2d_backward_resnet50_3x3"

    def __init__(self, rb, torch, dev):
        self.rb, self.torch, self.dev = rb, torch, dev
        self.N, self.C, self.H, self.W, self.Co = 32, 128, 28, 28, 128
        self.flops = 2 * 2.0 * self.N * self.H * self.W * self.Co * self.C * 9  # dx and dw
        x = rb.fill_normal((self.N, self.C, self.H, self.W), 1, 0)
        w = rb.fill_normal((self.Co, self.C, 3, 3), 1, 1, 0.0, math.sqrt(2.0 / (self.C * 9)))
        dy = rb.fill_normal((self.N, self.Co, self.H, self.W), 1, 3)
        self.host = {"x": x, "w": w, "dy": dy}
        per_set = (x.nbytes + dy.nbytes + x.nbytes)
        self.nsets = max(2, int(math.ceil(2 * L2_BYTES / per_set)))
        self.xs = [torch.from_numpy(x).to(dev) for _ in range(self.nsets)]
        self.dys = [torch.from_numpy(dy).to(dev) for _ in range(self.nsets)]
        self.dxs = [torch.empty_like(self.xs[0]) for _ in range(self.nsets)]
        self.w = torch.from_numpy(w).to(dev)
        self.dw = torch.empty_like(self.w)
        self.i = 0
        self.config = {"workload": "conv2d backward (grad_input + grad_weight), ResNet-50 "
                                   "stage-2 3x3", "input": [32, 128, 28, 28],
                       "weight": [128, 128, 3, 3], "stride": 1, "pad": 1, "seed": 1,
                       "layout": "NCHW", "roofline_note": "achieved = the whole backward call",
                       "l2": f"rotating {self.nsets} x/dy/dx sets"}
        # dx: dilate, flip-pack, conv; dw: layout, im2col, transpose, GEMM, unpack
        self.launches_per_step = 8

    def _call(self, x, dy, dx, dw, stream, w=None):
        rb = self.rb
        ctx = rb.get_context(self.dev.index or 0)
        w = self.w if w is None else w
        rb.call("rtb_conv2d_backward", ctx.handle, self.N, self.C, self.H, self.W, self.Co, 3, 3,
                1, 1, 1, 1, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                ctypes.c_void_p(dy.data_ptr()), ctypes.c_void_p(dx.data_ptr()),
                ctypes.c_void_p(dw.data_ptr()), 0, PRECISION[0], stream)

    def step(self):
        k = self.i % self.nsets
        self.i += 1
        stream = ctypes.c_void_p(self.torch.cuda.current_stream(self.dev).cuda_stream)
        self._call(self.xs[k], self.dys[k], self.dxs[k], self.dw, stream)

    def kernel_setup(self):
        pass

    def kernel_step(self):
        self.step()

    def e2e_setup(self):
        rb, torch = self.rb, self.torch
        ctx = rb.get_context(self.dev.index or 0)
        self.pipe = E2EPipeline(torch, self.dev, 2)
        self.slots = []
        for _ in range(self.pipe.depth):
            slot = {key: _pinned_copy(rb, ctx, arr) for key, arr in self.host.items()}
            slot["pdx"] = _pinned_empty(rb, ctx, self.host["x"].nbytes)
            slot["pdw"] = _pinned_empty(rb, ctx, self.host["w"].nbytes)
            slot["dx_"] = torch.empty_like(self.xs[0])
            slot["dy_"] = torch.empty_like(self.dys[0])
            slot["x_"] = torch.empty_like(self.xs[0])
            slot["ddx"] = torch.empty_like(self.xs[0])
            slot["ddw"] = torch.empty_like(self.w)
            slot["w_"] = torch.empty_like(self.w)
            self.slots.append(slot)
        self.h2d_bytes = sum(a.nbytes for a in self.host.values())
        self.d2h_bytes = self.host["x"].nbytes + self.host["w"].nbytes

    def e2e_step(self):
        rb = self.rb
        ctx = rb.get_context(self.dev.index or 0)
        pipe = self.pipe
        k = pipe.next()
        sl = self.slots[k]
        for key, dst in (("x", sl["x_"]), ("dy", sl["dy_"])):
            rb.call("rtb_memcpy_h2d", ctx.handle, ctypes.c_void_p(dst.data_ptr()), sl[key],
                    self.host[key].nbytes, pipe.h_in)
        rb.call("rtb_memcpy_h2d", ctx.handle, ctypes.c_void_p(sl["w_"].data_ptr()), sl["w"],
                self.host["w"].nbytes, pipe.h_in)
        pipe.compute(k)
        self._call(sl["x_"], sl["dy_"], sl["ddx"], sl["ddw"], pipe.h_c, sl["w_"])
        pipe.download(k)
        rb.call("rtb_memcpy_d2h", ctx.handle, sl["pdx"], ctypes.c_void_p(sl["ddx"].data_ptr()),
                self.host["x"].nbytes, pipe.h_out)
        rb.call("rtb_memcpy_d2h", ctx.handle, sl["pdw"], ctypes.c_void_p(sl["ddw"].data_ptr()),
                self.host["w"].nbytes, pipe.h_out)
        pipe.finish(k)

    def e2e_teardown(self):
        ctx = self.rb.get_context(self.dev.index or 0)
        for sl in self.slots:
            for key in ("x", "w", "dy", "pdx", "pdw"):
                self.rb.call("rtb_host_free", ctx.handle, sl[key])
        self.slots = []

    def cpu_sample(self, threads):
        """The reference's Conv2dBackward direct cores (f64 accumulation,
        conv.rs:336-502) restated, on one image of the batch."""
        from oracle import oracle as orc
        x = orc.normal((1, self.C, self.H, self.W), 1, 0)
        w = orc.normal((self.Co, self.C, 3, 3), 1, 1, 0.0, math.sqrt(2.0 / (self.C * 9)))
        dy = orc.normal((1, self.Co, self.H, self.W), 1, 3)
        t0 = time.perf_counter()
        reps = 0
        while True:
            orc.conv2d_grad_input_f64(dy, w, x.shape, (1, 1), (1, 1), threads=threads)
            orc.conv2d_grad_weight_f64(x, dy, w.shape, (1, 1), (1, 1), threads=threads)
            reps += 1
            if time.perf_counter() - t0 > 10.0 or reps >= 20:
                break
        dt = (time.perf_counter() - t0) / reps
        return self.flops / self.N / dt / 1e12, (f"1 of 32 images per call (direct f64 grad_input "
                                                 f"and grad_weight cores), {reps} calls")


# f32 matmul shapes (M, N, K, seed): the 1024^3 workload and the large-GEMM
# sweep (square 2048..16384, skinny M = 16/32/64/128/256 with N = K = 8192).
GEMM_SHAPES = {
    "gemm1024": (1024, 1024, 1024, 0),
    "gemm2048": (2048, 2048, 2048, 4),
    "gemm4096": (4096, 4096, 4096, 4),
    "gemm8192": (8192, 8192, 8192, 4),
    "gemm16384": (16384, 16384, 16384, 4),
    "gemm_m16": (16, 8192, 8192, 4),
    "gemm_m32": (32, 8192, 8192, 4),
    "gemm_m64": (64, 8192, 8192, 4),
    "gemm_m128": (128, 8192, 8192, 4),
    "gemm_m256": (256, 8192, 8192, 4),
}


class GemmWorkload:
    """C = A . B, A [M,K] and B [K,N] ~ N(0,1).  Replicas at N>1, except square
    problems of 8192 and up, which are N-split: every rank holds A and its
    N/P columns of B, computes its block of C on the tensor cores, and the
    blocks are all-gathered over NCCL (strong scaling, one problem per job)."""

    def __init__(self, rb, torch, dev, m, n, k, seed, world=1, rank=0):
        self.rb, self.torch, self.dev = rb, torch, dev
        self.m, self.n, self.k, self.seed = m, n, k, seed
        self.name = f"sgemm_{n}" if m == n == k else f"sgemm_{m}x{n}x{k}"
        self.nsplit = world > 1 and m == n == k and n >= 8192 and n % world == 0
        self.world, self.rank = world, rank
        self.scaling = "strong" if self.nsplit else "weak"
        self.flops = 2.0 * m * n * k                      # one step of the whole job
        self.n_local = n // world if self.nsplit else n
        self.kernel_flops = 2.0 * m * self.n_local * k    # the dominant kernel, per GPU
        self.bytes = 4.0 * (m * k + k * n + m * n)        # algorithmic HBM bytes
        # HBM-bound where the arithmetic intensity is below the 3xTF32 ridge
        self.bound = "hbm" if self.flops / self.bytes < 46 else "tensor"
        a = rb.fill_normal((m, k), seed, 0)
        b = rb.fill_normal((k, n), seed, 1)
        if self.nsplit:
            c0 = rank * self.n_local
            b = np.ascontiguousarray(b[:, c0:c0 + self.n_local])
        self.host = {"a": a, "b": b}
        per = 4 * (m * k + k * self.n_local + m * n)
        self.nsets = 1 if (self.nsplit or per >= 2 * L2_BYTES) else min(
            24, int(math.ceil(2 * L2_BYTES / per)))
        self.as_ = [torch.from_numpy(a).to(dev) for _ in range(self.nsets)]
        self.bs = [torch.from_numpy(b).to(dev) for _ in range(self.nsets)]
        self.cs = [torch.empty((m, n), device=dev) for _ in range(self.nsets)]
        self.i = 0
        # N-split: fused GEMM + exchange (epilogue P2P stores into every rank's C
        # over NVLink) unless RTB_NSPLIT_NCCL=1 asks for GEMM then NCCL all-gather
        self.fused = self.nsplit and os.environ.get("RTB_NSPLIT_NCCL", "0") != "1"
        if self.nsplit:
            from rustorch_b200.dist import NsplitGemm, NsplitGemmP2P
            ctx = rb.get_context(dev.index or 0)
            self.gemm = (NsplitGemmP2P(ctx, world, rank, m, n) if self.fused
                         else NsplitGemm(ctx, world, rank))
            self.parts = torch.empty((world, m, self.n_local), device=dev)
            self.c_local = torch.empty((m, self.n_local), device=dev)
        par = None
        if self.nsplit:
            par = (f"N-split x{world}: A . B[:, cols(rank)] per GPU, epilogue stores every tile "
                   f"into all ranks' C over NVLink (fused exchange)" if self.fused else
                   f"N-split x{world}: A . B[:, cols(rank)] per GPU + NCCL all-gather of C")
        self.config = {"workload": f"f32 matmul {m}x{n}x{k}", "seed": seed,
                       "layout": "row-major A[M,K], B[K,N]",
                       "l2": (f"rotating {self.nsets} operand sets" if self.nsets > 1 else
                              "operands larger than L2")}
        if par:
            self.config["parallelism_detail"] = par
        # GEMM-then-all-gather adds the repack kernel (NCCL's own launches not counted)
        self.launches_per_step = 2 if (self.nsplit and not self.fused) else 1

    def step(self):
        k = self.i % self.nsets
        self.i += 1
        if self.fused:
            self.gemm(self.as_[k], self.bs[k], precision=PRECISION[0])
        elif self.nsplit:
            self.gemm(self.as_[k], self.bs[k], precision=PRECISION[0], out=self.cs[k],
                      parts=self.parts)
        else:
            self.rb.sgemm(self.as_[k], self.bs[k], out=self.cs[k], precision=PRECISION[0])

    def kernel_setup(self):
        pass

    def kernel_step(self):
        k = self.i % self.nsets
        self.i += 1
        out = self.c_local if self.nsplit else self.cs[k]
        self.rb.sgemm(self.as_[k], self.bs[k], out=out, precision=PRECISION[0])

    def e2e_setup(self):
        rb, torch = self.rb, self.torch
        ctx = rb.get_context(self.dev.index or 0)
        sizes = {"a": self.m * self.k * 4, "b": self.k * self.n_local * 4,
                 "c": self.m * self.n * 4}
        per_slot = sum(sizes.values())
        # the N-split step holds NCCL calls, which stay on one stream in issue order
        depth = 1 if self.nsplit else (3 if per_slot <= 256 * 2**20 else 2)
        self.pipe = E2EPipeline(torch, self.dev, depth)
        self.slots = []
        for k in range(depth):
            slot = {"a": (_pinned_copy(rb, ctx, self.host["a"]), sizes["a"]),
                    "b": (_pinned_copy(rb, ctx, self.host["b"]), sizes["b"]),
                    "c": (_pinned_empty(rb, ctx, sizes["c"]), sizes["c"])}
            if k < self.nsets:  # device operands: reuse the rotating sets where they exist
                slot["da"], slot["db"], slot["dc"] = self.as_[k], self.bs[k], self.cs[k]
            else:
                slot["da"] = torch.empty_like(self.as_[0])
                slot["db"] = torch.empty_like(self.bs[0])
                slot["dc"] = torch.empty_like(self.cs[0])
            self.slots.append(slot)
        self.h2d_bytes = sizes["a"] + sizes["b"]
        self.d2h_bytes = sizes["c"]

    def e2e_step(self):
        rb = self.rb
        ctx = rb.get_context(self.dev.index or 0)
        pipe = self.pipe
        k = pipe.next()
        slot = self.slots[k]
        a, b, c = slot["da"], slot["db"], slot["dc"]
        for key, dst in (("a", a), ("b", b)):
            p, nb = slot[key]
            rb.call("rtb_memcpy_h2d", ctx.handle, ctypes.c_void_p(dst.data_ptr()), p, nb, pipe.h_in)
        pipe.compute(k)
        if self.fused:
            with self.torch.cuda.stream(pipe.s_c):
                c = self.gemm(a, b, precision=PRECISION[0])
        elif self.nsplit:
            with self.torch.cuda.stream(pipe.s_c):
                self.gemm(a, b, precision=PRECISION[0], out=c, parts=self.parts)
        else:
            rb.call("rtb_sgemm", ctx.handle, self.m, self.n, self.k,
                    ctypes.c_void_p(a.data_ptr()), self.k, 0, ctypes.c_void_p(b.data_ptr()),
                    self.n_local, 0, None, rb.ACT_NONE, ctypes.c_void_p(c.data_ptr()), self.n,
                    PRECISION[0], pipe.h_c)
        pipe.download(k)
        p, nb = slot["c"]
        rb.call("rtb_memcpy_d2h", ctx.handle, p, ctypes.c_void_p(c.data_ptr()), nb, pipe.h_out)
        pipe.finish(k)

    def e2e_teardown(self):
        ctx = self.rb.get_context(self.dev.index or 0)
        for slot in self.slots:
            for key in ("a", "b", "c"):
                self.rb.call("rtb_host_free", ctx.handle, slot[key][0])
        self.slots = []

    def close(self):
        if self.nsplit:
            self.gemm.close()

    def cpu_sample(self, threads):
        """matrixmultiply restatement (single-threaded, as the reference builds
        it) on a row sample of the same product."""
        from oracle import oracle as orc
        m, n, k = self.m, self.n, self.k
        rows = max(1, min(m, int(2e9 / (2 * n * k))))
        a = orc.normal((rows, k), self.seed, 0)   # the first rows of A
        b = orc.normal((k, n), self.seed, 1)
        t0 = time.perf_counter()
        reps = 0
        while True:
            orc.sgemm_mm(a, b, threads=1)
            reps += 1
            if time.perf_counter() - t0 > 10.0 or reps >= 10:
                break
        dt = (time.perf_counter() - t0) / reps
        return 2.0 * rows * n * k / dt / 1e12, (f"{rows} of {m} rows of A per call, "
                                                f"single-threaded blocked sgemm, {reps} calls")

    def cpu_sample_all_cores(self, threads):
        """The same blocked sgemm on every host core (64-row panels in parallel):
        what the CPU does when it is not held to the reference's one thread."""
        from oracle import oracle as orc
        m, n, k = self.m, self.n, self.k
        rows = max(1, min(m, max(64 * threads, int(2e9 * threads / (2 * n * k)))))
        a = orc.normal((rows, k), self.seed, 0)
        b = orc.normal((k, n), self.seed, 1)
        t0 = time.perf_counter()
        reps = 0
        while True:
            orc.sgemm_mm(a, b, threads=threads)
            reps += 1
            if time.perf_counter() - t0 > 10.0 or reps >= 10:
                break
        dt = (time.perf_counter() - t0) / reps
        return 2.0 * rows * n * k / dt / 1e12, (f"{rows} of {m} rows of A per call, blocked "
                                                f"sgemm on {threads} threads, {reps} calls")


class ResNet18Workload:
    """ResNet-18 forward, B=256 images per GPU (batch-sharded, no communication)."""
    name = "resnet18_fwd"

    def __init__(self, rb, torch, dev, batch=256):
        self.rb, self.torch, self.dev = rb, torch, dev
        self.B = batch
        self.h = ctypes.c_void_p()
        rb.call("rtb_resnet18_create", dev.index or 0, 3, PRECISION[0], ctypes.byref(self.h))
        self.flops_img = rb.lib().rtb_resnet18_flops_per_image(self.h)
        self.flops = float(self.flops_img * self.B)
        x = rb.fill_normal((self.B, 3, 224, 224), 3, 1000)
        self.host = {"x": x}
        self.x = torch.from_numpy(x).to(dev)          # 154 MB > L2
        self.logits = torch.empty((self.B, 1000), device=dev)
        self.config = {"workload": "ResNet-18 forward (BN folded), fp32",
                       "batch_per_gpu": self.B, "input": [self.B, 3, 224, 224], "seed": 3,
                       "flops_per_image": self.flops_img,
                       "l2": "inputs larger than L2 (154 MB per batch)"}
        self.launches_per_step = 24  # stem prologue, 20 convs, max pool, avg pool, fc
        self.unit = "img/s"
        self.gemm_extras = True
        self.kernel_desc = ("the whole forward timed alone: 20 implicit-GEMM conv launches, "
                            "the fc GEMM, the stem prologue and the two pools")

    def release(self):
        """Free the model and its buffers before the GEMM sub-benchmarks run."""
        if self.h:
            self.rb.call("rtb_resnet18_destroy", self.h)
            self.h = None
        self.x = self.logits = None

    def _fwd(self, x):
        stream = ctypes.c_void_p(self.torch.cuda.current_stream(self.dev).cuda_stream)
        self.rb.call("rtb_resnet18_forward", self.h, self.B, ctypes.c_void_p(x.data_ptr()),
                     ctypes.c_void_p(self.logits.data_ptr()), stream)

    def step(self):
        self._fwd(self.x)

    def kernel_setup(self):
        pass

    def kernel_step(self):
        self._fwd(self.x)

    def e2e_setup(self):
        rb, torch = self.rb, self.torch
        ctx = rb.get_context(self.dev.index or 0)
        x = self.host["x"]
        # two slots, each with its own model instance (a forward's activation
        # buffers belong to its instance), same seed: identical weights
        self.pipe = E2EPipeline(torch, self.dev, 2)
        self.slots = []
        for k in range(self.pipe.depth):
            h = self.h
            if k > 0:
                h = ctypes.c_void_p()
                rb.call("rtb_resnet18_create", self.dev.index or 0, 3, PRECISION[0],
                        ctypes.byref(h))
            self.slots.append({"h": h, "px": _pinned_copy(rb, ctx, x),
                               "py": _pinned_empty(rb, ctx, self.B * 1000 * 4),
                               "dx": torch.empty_like(self.x),
                               "dy": torch.empty_like(self.logits)})
        self.h2d_bytes = x.nbytes
        self.d2h_bytes = self.B * 1000 * 4

    def e2e_step(self):
        rb = self.rb
        ctx = rb.get_context(self.dev.index or 0)
        pipe = self.pipe
        k = pipe.next()
        slot = self.slots[k]
        rb.call("rtb_memcpy_h2d", ctx.handle, ctypes.c_void_p(slot["dx"].data_ptr()), slot["px"],
                self.h2d_bytes, pipe.h_in)
        pipe.compute(k)
        rb.call("rtb_resnet18_forward", slot["h"], self.B, ctypes.c_void_p(slot["dx"].data_ptr()),
                ctypes.c_void_p(slot["dy"].data_ptr()), pipe.h_c)
        pipe.download(k)
        rb.call("rtb_memcpy_d2h", ctx.handle, slot["py"], ctypes.c_void_p(slot["dy"].data_ptr()),
                self.d2h_bytes, pipe.h_out)
        pipe.finish(k)

    def e2e_teardown(self):
        ctx = self.rb.get_context(self.dev.index or 0)
        for k, slot in enumerate(self.slots):
            self.rb.call("rtb_host_free", ctx.handle, slot["px"])
            self.rb.call("rtb_host_free", ctx.handle, slot["py"])
            if k > 0:
                self.rb.call("rtb_resnet18_destroy", slot["h"])
        self.slots = []

    def cpu_sample(self, threads):
        """The reference's CPU ops (conv2d auto path, bias, relu, max_pool2d,
        add, avg pool, Linear) composed into ResNet-18, on one image."""
        from oracle import oracle as orc
        convs = []
        specs = [(3, 64, 7, 2, 3)]
        cin = 64
        for st, co in enumerate([64, 128, 256, 512]):
            for blk in range(2):
                down = st > 0 and blk == 0
                specs += [(cin, co, 3, 2 if down else 1, 1), (co, co, 3, 1, 1)]
                if down:
                    specs.append((cin, co, 1, 2, 0))
                cin = co
        for i, (ci, co, k, s, p) in enumerate(specs):
            convs.append((orc.normal((co, ci, k, k), 3, i, 0.0, math.sqrt(2.0 / (ci * k * k))),
                          np.zeros(co, np.float32), s, p))
        fc_w = orc.uniform((1000, 512), 3, 100, -1 / math.sqrt(512), 1 / math.sqrt(512))
        fc_b = orc.uniform((1000,), 3, 101, -1 / math.sqrt(512), 1 / math.sqrt(512))
        x = orc.normal((1, 3, 224, 224), 3, 1000)

        def conv(t, i, relu, res=None):
            w, b, s, p = convs[i]
            y, _ = orc.conv2d(t, w, (s, s), (p, p), threads)
            y = orc.add_bias_nchw(y, b)
            if res is not None:
                y = y + res
            return orc.relu(y) if relu else y

        def forward(t):
            t = orc.max_pool2d(conv(t, 0, True), (3, 3), (2, 2), (1, 1))
            i = 1
            for st in range(4):
                for blk in range(2):
                    down = st > 0 and blk == 0
                    a = conv(t, i, True)
                    ident = conv(t, i + 2, False) if down else t
                    t = conv(a, i + 1, True, ident)
                    i += 3 if down else 2
            return orc.linear(orc.global_avg_pool(t), fc_w, fc_b)

        t0 = time.perf_counter()
        reps = 0
        while reps < 1 or (time.perf_counter() - t0 < 10.0 and reps < 5):
            forward(x)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        return 1.0 / dt, f"1 image per forward (reference CPU ops composed), {reps} forwards"


class MlpWorkload:
    """3-layer MLP forward: X [4096,1024] -> 4096 -> 4096 -> 1024, Linear+ReLU
    after the first two layers (bias and ReLU fused in the GEMM epilogue)."""
    name = "mlp3_fwd"

    def __init__(self, rb, torch, dev):
        self.rb, self.torch, self.dev = rb, torch, dev
        self.dims = [1024, 4096, 4096, 1024]
        self.M = 4096
        self.flops = float(sum(2 * self.M * self.dims[i] * self.dims[i + 1] for i in range(3)))
        gain = math.sqrt(2.0)
        self.host = {"x": rb.fill_normal((self.M, 1024), 2, 0)}
        self.ws, self.bs = [], []
        for i in range(3):
            fan_in = self.dims[i]
            bound = math.sqrt(3.0) * gain / math.sqrt(fan_in)
            w = rb.fill_uniform((self.dims[i + 1], fan_in), 2, 1 + i, -bound, bound)
            self.host[f"w{i}"] = w
            self.ws.append(torch.from_numpy(w).to(dev))
            self.bs.append(torch.zeros(self.dims[i + 1], device=dev))
        self.x = torch.from_numpy(self.host["x"]).to(dev)
        self.h = [torch.empty((self.M, d), device=dev) for d in self.dims[1:]]
        self.config = {"workload": "3-layer MLP forward 4096x(1024->4096->4096->1024)",
                       "seed": 2, "l2": "operands + activations larger than L2 (~370 MB)"}
        self.launches_per_step = 3
        self.unit = "TFLOP/s"

    def _fwd(self, x, h=None):
        rb = self.rb
        h = self.h if h is None else h
        a = x
        for i in range(3):
            rb.sgemm(a, self.ws[i].t(), bias=self.bs[i], act=rb.ACT_RELU if i < 2 else rb.ACT_NONE,
                     precision=PRECISION[0], out=h[i])
            a = h[i]

    def step(self):
        self._fwd(self.x)

    def kernel_setup(self):
        pass

    def kernel_step(self):
        self._fwd(self.x)

    def e2e_setup(self):
        rb, torch = self.rb, self.torch
        ctx = rb.get_context(self.dev.index or 0)
        x = self.host["x"]
        self.pipe = E2EPipeline(torch, self.dev, 2)
        self.slots = []
        for k in range(self.pipe.depth):
            h = self.h if k == 0 else [torch.empty_like(t) for t in self.h]
            self.slots.append({"px": _pinned_copy(rb, ctx, x),
                               "py": _pinned_empty(rb, ctx, self.M * 1024 * 4),
                               "dx": torch.empty_like(self.x), "h": h})
        self.h2d_bytes = x.nbytes
        self.d2h_bytes = self.M * 1024 * 4

    def e2e_step(self):
        rb = self.rb
        ctx = rb.get_context(self.dev.index or 0)
        pipe = self.pipe
        k = pipe.next()
        slot = self.slots[k]
        rb.call("rtb_memcpy_h2d", ctx.handle, ctypes.c_void_p(slot["dx"].data_ptr()), slot["px"],
                self.h2d_bytes, pipe.h_in)
        pipe.compute(k)
        with self.torch.cuda.stream(pipe.s_c):  # rb.sgemm launches on torch's current stream
            self._fwd(slot["dx"], slot["h"])
        pipe.download(k)
        rb.call("rtb_memcpy_d2h", ctx.handle, slot["py"], ctypes.c_void_p(slot["h"][2].data_ptr()),
                self.d2h_bytes, pipe.h_out)
        pipe.finish(k)

    def e2e_teardown(self):
        ctx = self.rb.get_context(self.dev.index or 0)
        for slot in self.slots:
            self.rb.call("rtb_host_free", ctx.handle, slot["px"])
            self.rb.call("rtb_host_free", ctx.handle, slot["py"])
        self.slots = []

    def cpu_sample(self, threads):
        """nn::Linear x3 on the reference's CPU path for a 64-row sample."""
        from oracle import oracle as orc
        rows = 64
        x = orc.normal((self.M, 1024), 2, 0)[:rows]
        ws = []
        for i in range(3):
            bound = math.sqrt(3.0) * math.sqrt(2.0) / math.sqrt(self.dims[i])
            ws.append(orc.uniform((self.dims[i + 1], self.dims[i]), 2, 1 + i, -bound, bound))
        t0 = time.perf_counter()
        reps = 0
        while reps < 1 or (time.perf_counter() - t0 < 10.0 and reps < 10):
            a = x
            for i in range(3):
                a = orc.linear(a, ws[i], np.zeros(self.dims[i + 1], np.float32), relu=i < 2,
                               threads=threads)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        return self.flops * rows / self.M / dt / 1e12, f"{rows} of 4096 rows, {reps} passes"


class LinearNormWorkload:
    """nn::Linear::forward_fused_norm_activation (rustorch-nn/src/linear.rs:53-71
    -> ops::matmul_bias_norm_activation, rustorch-core/src/ops.rs:1815-1886):
    X [8192, 1024] . W^T (W [4096, 1024]) + bias, LayerNorm over the 4096
    features (weight, bias, eps 1e-5), ReLU.  Two launches: the tcgen05 GEMM
    with the bias in its epilogue, then the row-wise LayerNorm + ReLU."""
    name = "linear_norm_relu"

    def __init__(self, rb, torch, dev):
        self.rb, self.torch, self.dev = rb, torch, dev
        self.M, self.K, self.N = 8192, 1024, 4096
        self.flops = 2.0 * self.M * self.K * self.N   # GEMM FLOPs (LayerNorm's ~9 per element omitted)
        bound = 1.0 / math.sqrt(self.K)
        self.host = {"x": rb.fill_normal((self.M, self.K), 4, 0),
                     "w": rb.fill_uniform((self.N, self.K), 4, 1, -bound, bound),
                     "b": rb.fill_uniform((self.N,), 4, 2, -bound, bound),
                     "g": rb.fill_normal((self.N,), 4, 3, 1.0, 0.1),
                     "beta": rb.fill_normal((self.N,), 4, 4, 0.0, 0.1)}
        t = {k: torch.from_numpy(v).to(dev) for k, v in self.host.items()}
        self.x, self.w, self.b, self.g, self.beta = t["x"], t["w"], t["b"], t["g"], t["beta"]
        self.y = torch.empty((self.M, self.N), device=dev)
        self.config = {"workload": "Linear 1024->4096 + bias, LayerNorm(4096) + ReLU over 8192 rows",
                       "seed": 4, "l2": "operands + output larger than L2 (~180 MB)"}
        self.launches_per_step = 2
        self.unit = "TFLOP/s"
        self.ln_bytes = 2.0 * 4 * self.M * self.N     # LayerNorm pass: read C, write Y

    def _fwd(self, x, y):
        self.rb.matmul_bias_norm_activation(x, self.w.t(), self.b, self.g, self.beta, 1e-5,
                                            self.rb.ACT_RELU, PRECISION[0], out=y)

    def step(self):
        self._fwd(self.x, self.y)

    def kernel_setup(self):
        pass

    def kernel_step(self):  # the dominant kernel: the GEMM with its bias epilogue
        self.rb.sgemm(self.x, self.w.t(), bias=self.b, precision=PRECISION[0], out=self.y)

    def secondary_step(self):  # the LayerNorm + ReLU pass alone, in place on C
        self.rb.layer_norm(self.y, self.g, self.beta, 1e-5, self.rb.ACT_RELU, out=self.y)

    def e2e_setup(self):
        rb, torch = self.rb, self.torch
        ctx = rb.get_context(self.dev.index or 0)
        self.pipe = E2EPipeline(torch, self.dev, 2)
        self.slots = []
        for k in range(self.pipe.depth):
            self.slots.append({"px": _pinned_copy(rb, ctx, self.host["x"]),
                               "py": _pinned_empty(rb, ctx, self.M * self.N * 4),
                               "dx": self.x if k == 0 else torch.empty_like(self.x),
                               "dy": self.y if k == 0 else torch.empty_like(self.y)})
        self.h2d_bytes = self.M * self.K * 4
        self.d2h_bytes = self.M * self.N * 4

    def e2e_step(self):
        rb = self.rb
        ctx = rb.get_context(self.dev.index or 0)
        pipe = self.pipe
        k = pipe.next()
        slot = self.slots[k]
        rb.call("rtb_memcpy_h2d", ctx.handle, ctypes.c_void_p(slot["dx"].data_ptr()), slot["px"],
                self.h2d_bytes, pipe.h_in)
        pipe.compute(k)
        with self.torch.cuda.stream(pipe.s_c):
            self._fwd(slot["dx"], slot["dy"])
        pipe.download(k)
        rb.call("rtb_memcpy_d2h", ctx.handle, slot["py"], ctypes.c_void_p(slot["dy"].data_ptr()),
                self.d2h_bytes, pipe.h_out)
        pipe.finish(k)

    def e2e_teardown(self):
        ctx = self.rb.get_context(self.dev.index or 0)
        for slot in self.slots:
            self.rb.call("rtb_host_free", ctx.handle, slot["px"])
            self.rb.call("rtb_host_free", ctx.handle, slot["py"])
        self.slots = []

    def cpu_sample(self, threads):
        """The reference's CPU pipeline (matmul + bias, one-pass f32 layer_norm,
        ReLU) on a 64-row sample."""
        return linear_norm_cpu_sample(self.M, self.K, self.N, threads)


def linear_norm_cpu_sample(M, K, N, threads, rows=64):
    from oracle import oracle as orc
    bound = 1.0 / math.sqrt(K)
    x = orc.normal((M, K), 4, 0)[:rows]
    w = orc.uniform((N, K), 4, 1, -bound, bound)
    b = orc.uniform((N,), 4, 2, -bound, bound)
    g = orc.normal((N,), 4, 3, 1.0, 0.1)
    beta = orc.normal((N,), 4, 4, 0.0, 0.1)
    wt = np.ascontiguousarray(w.T)
    t0 = time.perf_counter()
    reps = 0
    while reps < 1 or (time.perf_counter() - t0 < 10.0 and reps < 10):
        orc.matmul_bias_norm_activation(x, wt, b, g, beta, 1e-5, 1, threads)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    return 2.0 * rows * K * N / dt / 1e12, f"{rows} of {M} rows, {reps} passes"


WORKLOADS = {
    "conv": lambda rb, torch, dev: ConvWorkload(rb, torch, dev),
    "conv_r50s1": lambda rb, torch, dev: ConvWorkload(rb, torch, dev, 1),
    "conv_r50s3": lambda rb, torch, dev: ConvWorkload(rb, torch, dev, 3),
    "conv_r50s4": lambda rb, torch, dev: ConvWorkload(rb, torch, dev, 4),
    "conv_bwd": lambda rb, torch, dev: ConvBwdWorkload(rb, torch, dev),
    "resnet18": lambda rb, torch, dev: ResNet18Workload(rb, torch, dev),
    "mlp": lambda rb, torch, dev: MlpWorkload(rb, torch, dev),
    "linear_norm": lambda rb, torch, dev: LinearNormWorkload(rb, torch, dev),
}


def _gemm_factory(m, n, k, seed):
    def make(rb, torch, dev):
        rank, world, _ = _dist_env()
        return GemmWorkload(rb, torch, dev, m, n, k, seed, world, rank)
    return make


for _name, (_m, _n, _k, _seed) in GEMM_SHAPES.items():
    WORKLOADS[_name] = _gemm_factory(_m, _n, _k, _seed)


# ------------------------------------------------------------------ timing
def _time_steps(torch, fn, steps, warmup, dev, dist=None, min_warm_s=0.3, pipe=None):
    # At least `warmup` steps, and at least min_warm_s of work so the SM
    # clocks have left their idle state before the timed region starts.  With
    # several ranks every rank runs the same number of steps (a step may hold
    # collectives, which must match across ranks): the extra count is agreed
    # with a max all-reduce.
    t0 = time.perf_counter()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    elapsed = time.perf_counter() - t0
    extra = 0
    if elapsed < min_warm_s:
        per_step = max(elapsed / max(1, warmup), 1e-6)
        extra = int(math.ceil((min_warm_s - elapsed) / per_step))
    if dist is not None:
        t = torch.tensor([extra], device=dev, dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        extra = int(t.item())
    for i in range(extra):
        fn()
        if (i + 1) % 16 == 0:
            torch.cuda.synchronize(dev)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    s = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s)
    if pipe is not None:   # multi-stream steps start after e0 and finish before e1
        pipe.begin(e0)
    for _ in range(steps):
        fn()
    if pipe is not None:
        pipe.join(s)
    e1.record(s)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    return ms


def _time_graph_steps(torch, fn, steps, warmup, dev, dist=None):
    """Device time of `steps` calls of fn issued from one CUDA graph: the
    calls (the same kernels on the same rotated operands) are captured once,
    and the timed region replays the graph, so the host's launch rate (one
    Python call per 25-us GEMM, eight processes sharing the host at N=8) is
    not what is measured."""
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    # thread-local capture: other host threads (the process group's watchdog
    # at N > 1) keep using CUDA while this thread captures
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        for _ in range(steps):
            fn()
    torch.cuda.synchronize(dev)
    ms = _time_steps(torch, g.replay, 1, max(1, warmup // 3), dev, dist)
    del g
    torch.cuda.synchronize(dev)
    return ms


def _gemm_extras(rb, torch, dev, args, dist, world, roof_peak):
    """The GEMM half of the headline metric beside the ResNet-18 line: f32
    matmul 1024^3 (replicas) and 8192^3 (N-split across the ranks at N>1),
    A, B ~ N(0,1), device-timed like the main workload (CUDA events between
    barrier + synchronize, max over ranks, operands rotated past L2)."""
    out = {}
    for name in ("gemm1024", "gemm8192"):
        wl = WORKLOADS[name](rb, torch, dev)
        if wl.nsplit:
            ms = _time_steps(torch, wl.step, args.steps, args.warmup, dev, dist)
            launch = "one call per step"
        else:
            try:
                ms = _time_graph_steps(torch, wl.step, args.steps, args.warmup, dev, dist)
                launch = "the K steps captured in one CUDA graph, replayed once per timed pass"
            except RuntimeError as e:  # same collectives either way: ranks stay in step
                torch.cuda.synchronize(dev)
                ms = _time_steps(torch, wl.step, args.steps, args.warmup, dev, dist)
                launch = f"one call per step (graph capture failed: {str(e)[:80]})"
        jobs = 1 if wl.scaling == "strong" else world
        v = jobs * wl.flops * args.steps / (ms / 1e3) / 1e12
        out[name] = {"value": round(v, 3), "unit": "TFLOP/s", "ms_per_step": round(ms / args.steps, 5),
                     "scaling": wl.scaling,
                     "parallelism": wl.config.get("parallelism_detail", f"replicas x{world}"),
                     "frac_of_roof": round(v / (world * roof_peak), 4),
                     "l2": wl.config["l2"], "launch": launch}
        if hasattr(wl, "close"):
            wl.close()
        del wl
        torch.cuda.synchronize(dev)
        torch.cuda.empty_cache()
    return out


def run_ours(args):
    import torch
    import rustorch_b200 as rb

    rank, world, local = _dist_env()
    dist = None
    if world > 1:
        import torch.distributed as tdist
        from datetime import timedelta
        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                 device_id=torch.device("cuda", local))
        dist = tdist
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    rb.get_context(local)
    wl = WORKLOADS[args.workload](rb, torch, dev)
    peaks = _peaks()

    unit = getattr(wl, "unit", "TFLOP/s")
    scaling = getattr(wl, "scaling", "weak")

    def rate(total_ms, ranks):
        # whole-job throughput in the workload's unit over `ranks` GPUs; with
        # strong scaling one step is one problem for the whole job
        jobs = 1 if scaling == "strong" else ranks
        if unit == "img/s":
            return jobs * wl.B * args.steps / (total_ms / 1e3)
        return jobs * wl.flops * args.steps / (total_ms / 1e3) / 1e12

    with ClockSampler(dev) as clk:
        ms = _time_steps(torch, wl.step, args.steps, args.warmup, dev, dist)
    ms_per_step = ms / args.steps
    value = rate(ms, world)

    # dominant kernel alone, CUDA events on its launch stream
    wl.kernel_setup()
    kms = _time_steps(torch, wl.kernel_step, args.steps, max(3, args.warmup), dev, None)
    kflops = getattr(wl, "kernel_flops", wl.flops)
    k_tflops = kflops * args.steps / (kms / 1e3) / 1e12
    tf32_peak = peaks["bf16_tflops"] / 2.0
    # captures are per precision (3xTF32 unless the key names TF32)
    tp_key = f"{args.workload}:tf32" if args.precision == "tf32" else args.workload
    roof_peak = tf32_peak / MMAS_PER_MAC[0]  # 3xTF32: three tensor-core MMAs per algorithmic MAC
    if getattr(wl, "bound", "tensor") == "hbm":
        # below the ridge: bytes that must cross HBM per launch / launch time
        k_gbs = wl.bytes * args.steps / (kms / 1e3) / 1e9
        roofline = {"bound": "hbm", "achieved": round(k_gbs, 1), "peak": peaks["hbm_gbs"],
                    "unit": "GB/s", "frac": round(k_gbs / peaks["hbm_gbs"], 4),
                    "traffic": TRAFFIC.get(args.workload, (None,))[0],
                    "traffic_source": TRAFFIC.get(args.workload, (None, None))[1],
                    "peak_basis": f"{peaks['basis']} HBM copy {peaks['hbm_gbs']} GB/s",
                    "algorithmic_bytes": wl.bytes, "kernel_tflops": round(k_tflops, 3),
                    "kernel_ms": round(kms / args.steps, 5)}
    else:
        roofline = {"bound": "tensor", "achieved": round(k_tflops, 3),
                    "peak": round(roof_peak, 3), "unit": "TFLOP/s",
                    "frac": round(k_tflops / roof_peak, 4),
                    "traffic": TRAFFIC.get(args.workload, (None,))[0],
                    "traffic_source": TRAFFIC.get(args.workload, (None, None))[1],
                    "peak_basis": f"{peaks['basis']} bf16 {peaks['bf16_tflops']} TFLOP/s "
                                  f"/ 2 (TF32 rate) / {MMAS_PER_MAC[0]} (MMAs per MAC)",
                    "tensor_pipe_frac": TENSOR_PIPE.get(tp_key, (None,))[0],
                    "tensor_pipe_source": TENSOR_PIPE.get(tp_key, (None, None))[1],
                    "tensor_pipe_basis": "ncu sm__pipe_tensor_cycles_active, fraction of "
                                         "elapsed cycles, from the named capture",
                    "mma_rate_implied": round(MMAS_PER_MAC[0] * k_tflops / tf32_peak, 4),
                    "kernel_ms": round(kms / args.steps, 5)}
        if hasattr(wl, "kernel_desc"):
            roofline["kernel"] = wl.kernel_desc

    if hasattr(wl, "secondary_step"):
        # the second launch of a two-kernel step (HBM-bound), timed alone
        sms = _time_steps(torch, wl.secondary_step, args.steps, max(3, args.warmup), dev, None)
        s_gbs = wl.ln_bytes * args.steps / (sms / 1e3) / 1e9
        roofline["secondary"] = {"kernel": "layernorm_act", "bound": "hbm",
                                 "achieved": round(s_gbs, 1), "peak": peaks["hbm_gbs"],
                                 "unit": "GB/s", "frac": round(s_gbs / peaks["hbm_gbs"], 4),
                                 "algorithmic_bytes": wl.ln_bytes,
                                 "traffic": TRAFFIC_SECONDARY.get(args.workload, (None,))[0],
                                 "traffic_source": TRAFFIC_SECONDARY.get(args.workload,
                                                                         (None, None))[1],
                                 "kernel_ms": round(sms / args.steps, 5)}

    # end to end through the C ABI with host buffers
    wl.e2e_setup()
    ems = _time_steps(torch, wl.e2e_step, args.steps, max(3, args.warmup), dev, dist,
                      pipe=getattr(wl, "pipe", None))
    wl.e2e_teardown()
    e2e = rate(ems, world)

    err = rb.get_context(local).device_error()
    if err:
        raise RuntimeError(f"device error word set: {err}")

    gemm_extra = None
    if getattr(wl, "gemm_extras", False) and not args.no_gemm_extras:
        wl.release()
        gemm_extra = _gemm_extras(rb, torch, dev, args, dist, world, roof_peak)

    if rank == 0:
        threads = _host_threads()
        if world == 1:
            cpu_val, sample = wl.cpu_sample(threads)
            cpu_line = {"value": round(cpu_val, 6), "unit": unit, "cores": threads,
                        "kind": "port", "sample": sample}
            if hasattr(wl, "cpu_sample_all_cores") and scaling != "strong":
                v_all, s_all = wl.cpu_sample_all_cores(threads)
                cpu_line["all_cores"] = {"value": round(v_all, 6), "cores": threads,
                                         "sample": s_all}
        else:  # the CPU baseline is a one-GPU figure (the N=1 line carries it)
            cpu_line = {"value": None, "unit": unit, "cores": threads, "kind": "port",
                        "sample": "measured on the N=1 line only"}
        if scaling == "strong":
            par = f"N-split x{world} + NCCL all-gather"
        elif unit == "img/s":
            par = f"batch-sharded x{world} (no collective)"
        else:
            par = f"replicas x{world}"
        line = {
            "metric": f"{wl.name} {unit} ({args.precision.upper()}, fp32 in/out)",
            "value": round(value, 3), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None,
            "dtype": "f32 (3xTF32 tensor-core split)" if PRECISION[0] == 0 else "f32 (TF32 tensor core)",
            "data": "synthetic (SplitMix64/Box-Muller, seeded)",
            "config": dict(wl.config, parallelism=par),
            "roofline": roofline,
            "cpu_baseline": cpu_line,
            "e2e": {"value": round(e2e, 3), "unit": unit,
                    "h2d_bytes_per_step": wl.h2d_bytes, "d2h_bytes_per_step": wl.d2h_bytes},
            "gpu_launches": wl.launches_per_step * args.steps,
            "clocks": clk.summary(),
        }
        if gemm_extra is not None:
            line["gemm"] = gemm_extra
        print(json.dumps(line), flush=True)
    if hasattr(wl, "close"):
        wl.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args):
    """The reference's CPU path (oracle restatement; the Rust reference cannot
    be built here) on the box's host cores, on a bounded sample per step."""
    rank, world, _ = _dist_env()
    if rank != 0:
        return
    threads = _host_threads()
    # Workload descriptions only (no GPU): cpu_sample needs the sizes.
    if args.workload == "conv" or args.workload.startswith("conv_r50s"):
        stage = 2 if args.workload == "conv" else int(args.workload[-1])
        wl = ConvWorkload.__new__(ConvWorkload)
        wl._shape(stage)
        cfg = {"workload": f"conv2d+bias+relu ResNet-50 stage-{stage} 3x3",
               "input": [32, wl.C, wl.H, wl.W], "weight": [wl.Co, wl.C, 3, 3], "stride": 1,
               "pad": 1, "seed": wl.seed}
        unit = "TFLOP/s"
    elif args.workload == "conv_bwd":
        wl = ConvBwdWorkload.__new__(ConvBwdWorkload)
        wl.N, wl.C, wl.H, wl.W, wl.Co = 32, 128, 28, 28, 128
        wl.flops = 2 * 2.0 * wl.N * wl.H * wl.W * wl.Co * wl.C * 9
        cfg = {"workload": "conv2d backward (grad_input + grad_weight), ResNet-50 stage-2 3x3",
               "input": [32, 128, 28, 28], "weight": [128, 128, 3, 3], "stride": 1, "pad": 1,
               "seed": 1}
        unit = "TFLOP/s"
    elif args.workload == "resnet18":
        wl = ResNet18Workload.__new__(ResNet18Workload)
        wl.B = 256
        cfg = {"workload": "ResNet-18 forward (BN folded), fp32", "batch_per_gpu": 256,
               "input": [256, 3, 224, 224], "seed": 3, "flops_per_image": 3628146688}
        unit = "img/s"
    elif args.workload == "mlp":
        wl = MlpWorkload.__new__(MlpWorkload)
        wl.dims, wl.M = [1024, 4096, 4096, 1024], 4096
        wl.flops = float(sum(2 * wl.M * wl.dims[i] * wl.dims[i + 1] for i in range(3)))
        cfg = {"workload": "3-layer MLP forward 4096x(1024->4096->4096->1024)", "seed": 2}
        unit = "TFLOP/s"
    elif args.workload == "linear_norm":
        wl = LinearNormWorkload.__new__(LinearNormWorkload)
        wl.M, wl.K, wl.N = 8192, 1024, 4096
        wl.flops = 2.0 * wl.M * wl.K * wl.N
        wl.cpu_sample = lambda threads: linear_norm_cpu_sample(wl.M, wl.K, wl.N, threads)
        cfg = {"workload": "Linear 1024->4096 + bias, LayerNorm(4096) + ReLU over 8192 rows",
               "seed": 4}
        unit = "TFLOP/s"
    else:
        m, n, k, seed = GEMM_SHAPES[args.workload]
        wl = GemmWorkload.__new__(GemmWorkload)
        wl.m, wl.n, wl.k, wl.seed, wl.flops = m, n, k, seed, 2.0 * m * n * k
        wl.name = f"sgemm_{n}" if m == n == k else f"sgemm_{m}x{n}x{k}"
        cfg = {"workload": f"f32 matmul {m}x{n}x{k}", "seed": seed}
        unit = "TFLOP/s"
    name = getattr(wl, "name", args.workload)
    vals, samples = [], []
    t0 = time.perf_counter()
    for _ in range(max(1, args.steps)):
        v, smp = wl.cpu_sample(threads)
        vals.append(v)
        samples.append(smp)
        if time.perf_counter() - t0 > 120:
            break
    v = statistics.median(vals)
    line = {"impl": "reference",
            "metric": f"{name} {unit} ({args.precision.upper()}, fp32 in/out)",
            "value": round(v, 6), "unit": unit, "n_gpus": world, "steps": len(vals),
            "warmup": args.warmup, "higher_is_better": True, "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (SplitMix64/Box-Muller, seeded)", "config": cfg,
            "cpu_baseline": {"value": round(v, 6), "unit": unit, "cores": threads,
                             "kind": "port", "sample": samples[0]},
            "e2e": {"value": round(v, 6), "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "reference CPU path restated in C (no Rust toolchain to build the reference)"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="resnet18", choices=sorted(WORKLOADS))
    ap.add_argument("--no-gemm-extras", action="store_true",
                    help="resnet18: leave out the f32 matmul 1024^3 / 8192^3 sub-object")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="3xtf32", choices=["3xtf32", "tf32"])
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    PRECISION[0] = 1 if args.precision == "tf32" else 0
    MMAS_PER_MAC[0] = 1 if args.precision == "tf32" else 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
