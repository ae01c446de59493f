"""Generate tests/golden/reference_kat.json from the reference's own tests.

Run where the RusTorch sources are checked out, passing their root
directory.  The reference is Rust and cannot be built
here, so its known-answer tests are read as text: the literal input and
expected-output arrays are extracted from the test sources and written out with
their file:line.  The committed JSON is what the tests use; this script is only
needed to regenerate it.

    python tests/golden/make_golden.py /path/to/RusTorch
"""
from __future__ import annotations

import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def _floats(txt: str):
    txt = re.sub(r"(?<=\d)(f32|f64|usize)", "", txt)  # Rust literal suffixes
    return [float(v) for v in re.findall(r"-?\d+\.\d+|-?\d+", txt)]


def _fn_body(src: str, name: str):
    i = src.index("fn " + name)
    line = src[:i].count("\n") + 1
    j = src.index("\n}\n", i)
    return src[i:j], line


def _tensor_new(body: str, var: str):
    """`let var = Tensor::new(&[...], &[...])` -> (data, shape)."""
    m = re.search(var + r"\s*=\s*Tensor::new\(\s*&\[(.*?)\]\s*,\s*&\[(.*?)\]\s*,?\s*\)", body, re.S)
    return _floats(m.group(1)), [int(v) for v in _floats(m.group(2))]


def main(root: str) -> None:
    kats = []
    rel = "rustorch-core/tests/autograd_test.rs"
    src = open(os.path.join(root, rel)).read()

    body, line = _fn_body(src, "test_matmul_forward_precision_under_1e6")
    a, ash = _tensor_new(body, "a")
    b, bsh = _tensor_new(body, "b")
    exp = _floats(re.search(r"expected\s*=\s*\[(.*?)\]", body, re.S).group(1))
    tol = float(re.search(r"err < ([0-9e\.\-]+)", body).group(1))
    kats.append({"name": "matmul_2x2", "op": "matmul", "source": f"{rel}:{line}",
                 "a": a, "a_shape": ash, "b": b, "b_shape": bsh,
                 "expected": exp, "abs_tol": tol})

    # MatmulBackward through loss = sum(a . b): grad_a = 1 . b^T, grad_b = a^T . 1
    body, line = _fn_body(src, "test_matmul_backward_precision_under_1e6")
    a, ash = _tensor_new(body, "a")
    b, bsh = _tensor_new(body, "b")
    exp_a = _floats(re.search(r"expected_a\s*=\s*\[(.*?)\]", body, re.S).group(1))
    exp_b = _floats(re.search(r"expected_b\s*=\s*\[(.*?)\]", body, re.S).group(1))
    tol = float(re.search(r"err < ([0-9e\.\-]+)", body).group(1))
    kats.append({"name": "matmul_backward_2x2", "op": "matmul_backward",
                 "source": f"{rel}:{line}", "a": a, "a_shape": ash, "b": b, "b_shape": bsh,
                 "grad_out": "ones (loss = sum of the product)",
                 "expected_grad_a": exp_a, "expected_grad_b": exp_b, "abs_tol": tol})

    body, line = _fn_body(src, "test_conv2d_forward_precision_under_1e6")
    x, xsh = _tensor_new(body, "input")
    w, wsh = _tensor_new(body, "weight")
    m = re.search(r"conv2d\(&input, &weight, \((\d+), (\d+)\), \((\d+), (\d+)\)\)", body)
    exp = _floats(re.search(r"expected\s*=\s*\[(.*?)\]", body, re.S).group(1))
    tol = float(re.search(r"err < ([0-9e\.\-]+)", body).group(1))
    kats.append({"name": "conv2d_3x3_k2", "op": "conv2d", "source": f"{rel}:{line}",
                 "x": x, "x_shape": xsh, "w": w, "w_shape": wsh,
                 "stride": [int(m.group(1)), int(m.group(2))],
                 "padding": [int(m.group(3)), int(m.group(4))],
                 "expected": exp, "abs_tol": tol})

    rel = "rustorch-core/examples/jit_demo.rs"
    src = open(os.path.join(root, rel)).read()
    line = src[:src.index("Tensor::ones(&[1, 1, 4, 4])")].count("\n") + 1
    ish = [int(v) for v in _floats(re.search(r"input_shape = vec!\[(.*?)\]", src).group(1))]
    wsh = [int(v) for v in _floats(re.search(r"weight_shape = vec!\[(.*?)\]", src).group(1))]
    osh = [int(v) for v in _floats(re.search(r"conv_out_shape = vec!\[(.*?)\]", src).group(1))]
    m = re.search(r"assert!\(\(output\.data\(\)\[0\] - ([0-9\.]+)\)\.abs\(\) < ([0-9e\.\-]+)\)", src)
    kats.append({"name": "jit_conv2d_relu_ones", "op": "jit_conv2d_relu", "source": f"{rel}:{line}",
                 "x_fill": 1.0, "x_shape": ish, "w_fill": 1.0, "w_shape": wsh,
                 "stride": [1, 1], "padding": [0, 0], "out_shape": osh,
                 "expected_first": float(m.group(1)), "abs_tol": float(m.group(2)),
                 "fused_node": "Conv2dRelu"})

    rel = "rustorch-core/benches/matmul_bench.rs"
    src = open(os.path.join(root, rel)).read()
    line = src.index("let size = 256usize")
    line = src[:line].count("\n") + 1
    size = int(re.search(r"let size = (\d+)usize", src).group(1))
    kats.append({"name": "bench_matmul_ones", "op": "matmul", "source": f"{rel}:{line}",
                 "m": size, "k": size, "n": size, "a_fill": 1.0, "b_fill": 1.0,
                 "expected_all": float(size), "abs_tol": 0.0})
    line = src[:src.index("let n = 8usize")].count("\n") + 1
    dims = {k: int(v) for k, v in re.findall(r"let (n|c_in|c_out|h|w|k) = (\d+)usize", src)}
    fill = _floats(re.search(r"vec!\[(0\.\d+)f32; n \* c_in", src).group(1))[0]
    m = re.search(r"conv2d\(&input, &weight, \((\d+), (\d+)\), \((\d+), (\d+)\)\)", src)
    kats.append({"name": "bench_conv2d_fill", "op": "conv2d", "source": f"{rel}:{line}",
                 "x_shape": [dims["n"], dims["c_in"], dims["h"], dims["w"]],
                 "w_shape": [dims["c_out"], dims["c_in"], dims["k"], dims["k"]],
                 "x_fill": fill, "w_fill": fill,
                 "stride": [int(m.group(1)), int(m.group(2))],
                 "padding": [int(m.group(3)), int(m.group(4))],
                 "expected_interior": fill * fill * dims["c_in"] * dims["k"] * dims["k"],
                 "rel_tol": 1e-5})

    # The reference's deterministic data generator, first values for seed 7
    # (demo_visual/src/bin/bench_alignment_ci.rs:12-20): computed here with a
    # direct restatement so the oracle's orc_unit can be pinned to it.
    rel = "demo_visual/src/bin/bench_alignment_ci.rs"
    src = open(os.path.join(root, rel)).read()
    line = src[:src.index("fn deterministic_unit")].count("\n") + 1
    consts = [int(c, 16) for c in re.findall(r"0x([0-9A-Fa-f]{16})", src[src.index("fn deterministic_unit"):][:600])]
    mask = (1 << 64) - 1

    def unit(idx, seed):
        x = (idx + seed * consts[0]) & mask
        x ^= x >> 30
        x = (x * consts[1]) & mask
        x ^= x >> 27
        x = (x * consts[2]) & mask
        x ^= x >> 31
        import numpy as np
        return float(np.float32(np.float32(x & 0xFFFFFFFF) / np.float32(4294967295.0)))

    kats.append({"name": "deterministic_unit", "op": "prng", "source": f"{rel}:{line}",
                 "seed": 7, "idx": list(range(8)), "expected": [unit(i, 7) for i in range(8)]})

    out = os.path.join(HERE, "reference_kat.json")
    with open(out, "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "kats": kats}, f, indent=1)
    print("wrote", out, len(kats), "known-answer tests")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/RusTorch")
    main(sys.argv[1])
