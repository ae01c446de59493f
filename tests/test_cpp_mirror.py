"""The C++ mirror of the reference API (include/rustorch_b200.hpp), exercised
by tests/cpp/test_reference_api.cpp — the reference's own tests restated in
C++ — compiled against librustorch_b200.so."""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "test_reference_api.cpp")
BIN = os.path.join(ROOT, "_build", "test_reference_api")


@pytest.fixture(scope="module")
def binary():
    from rustorch_b200 import build
    build.build()
    os.makedirs(os.path.dirname(BIN), exist_ok=True)
    libdir = os.path.join(ROOT, "rustorch_b200")
    cmd = ["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"), SRC, "-o", BIN,
           "-L", libdir, "-lrustorch_b200", f"-Wl,-rpath,{libdir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return BIN


def _run(binary, *args):
    r = subprocess.run([binary, *args], capture_output=True, text=True, timeout=300)
    return r.returncode, r.stdout + r.stderr


def test_graph_rewrites_and_panics_cpu(binary):
    rc, out = _run(binary, "--cpu-only")
    assert rc == 0, out
    for name in ("jit_fuse_conv_relu_rewrite", "jit_fuse_conv_bias_relu_rewrite",
                 "jit_no_fusion_when_relu_not_next", "panics_without_device_work"):
        assert f"PASS {name}" in out, out


@pytest.mark.gpu
def test_reference_tests_on_device(binary, kats, gpu):
    rc, out = _run(binary)
    assert rc == 0, out
    got = {}
    for line in out.splitlines():
        if line.startswith("KAT "):
            parts = line.split()
            got[parts[1]] = np.array([float(v) for v in parts[2:]])
    np.testing.assert_allclose(got["matmul_2x2"], kats["matmul_2x2"]["expected"],
                               atol=kats["matmul_2x2"]["abs_tol"], rtol=0)
    np.testing.assert_allclose(got["conv2d_3x3_k2"], kats["conv2d_3x3_k2"]["expected"],
                               atol=kats["conv2d_3x3_k2"]["abs_tol"], rtol=0)
    kb = kats["matmul_backward_2x2"]
    np.testing.assert_allclose(got["matmul_backward_2x2_a"], kb["expected_grad_a"],
                               atol=kb["abs_tol"], rtol=0)
    np.testing.assert_allclose(got["matmul_backward_2x2_b"], kb["expected_grad_b"],
                               atol=kb["abs_tol"], rtol=0)
    k = kats["jit_conv2d_relu_ones"]
    assert abs(got["jit_conv2d_relu_ones"][0] - k["expected_first"]) < k["abs_tol"]
