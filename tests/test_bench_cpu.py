"""bench.py's reference arm (the reference's CPU path restated, timed on the
host cores) runs without a GPU and prints the contract's JSON line."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_gemm1024():
    d = _run("--impl", "reference", "--workload", "gemm1024", "--steps", "1", "--warmup", "3")
    assert d["impl"] == "reference"
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["config"]["workload"].startswith("f32 matmul 1024x1024x1024")


def test_reference_arm_skinny_names_shape():
    d = _run("--impl", "reference", "--workload", "gemm_m16", "--steps", "1")
    assert d["metric"].startswith("sgemm_16x8192x8192")
    assert d["value"] > 0


def test_reference_arm_linear_norm_matches_our_config():
    """The Linear + LayerNorm + ReLU workload's reference arm names the same
    metric and workload as our arm (the driver pairs the two lines)."""
    d = _run("--impl", "reference", "--workload", "linear_norm", "--steps", "1")
    assert d["metric"].startswith("linear_norm_relu TFLOP/s")
    assert d["config"]["workload"] == "Linear 1024->4096 + bias, LayerNorm(4096) + ReLU over 8192 rows"
    assert d["value"] > 0 and d["cpu_baseline"]["sample"].startswith("64 of 8192 rows")


def test_reference_arm_default_is_resnet18():
    """With no --workload the bench measures ResNet-18 forward img/s (B=256 per
    GPU); the reference arm names the same metric and configuration."""
    d = _run("--impl", "reference", "--steps", "1")
    assert d["metric"].startswith("resnet18_fwd img/s")
    assert d["unit"] == "img/s" and d["value"] > 0
    assert d["config"]["workload"] == "ResNet-18 forward (BN folded), fp32"
    assert d["config"]["batch_per_gpu"] == 256 and d["config"]["seed"] == 3


def test_reference_arm_r50_stage_names():
    d = _run("--impl", "reference", "--workload", "conv_r50s4", "--steps", "1")
    assert d["metric"].startswith("conv2d_bias_relu_resnet50_s4_3x3 TFLOP/s")
    assert d["config"]["input"] == [32, 512, 7, 7] and d["config"]["seed"] == 5
