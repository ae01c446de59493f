"""C-ABI checks that need no GPU: the library builds/loads, exports every
symbol the header declares, validates arguments, and its host data generator
matches the oracle's bit for bit."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def rb():
    from rustorch_b200 import build
    build.build()
    import rustorch_b200
    rustorch_b200.lib()
    return rustorch_b200


def _header_functions():
    """Every rtb_* function declared in the C headers include/*.h."""
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in sorted(os.listdir(inc)):
        if f.endswith(".h"):
            src = re.sub(r"/\*.*?\*/", "", open(os.path.join(inc, f)).read(), flags=re.S)
            names |= set(re.findall(r"\b(rtb_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_header_symbols_exported(rb):
    from rustorch_b200 import _lib
    names = _header_functions()
    assert len(names) >= 30
    L = rb.lib()
    for n in names:
        assert hasattr(L, n), f"{n} declared in the header but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_no_oracle_in_product():
    """The product package never imports or links the oracle."""
    pkg = os.path.join(ROOT, "rustorch_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                txt = open(os.path.join(dirpath, f), errors="replace").read()
                assert "oracle" not in txt.lower() or f == "build.py" and False, \
                    f"{f} references the oracle"


def test_status_strings(rb):
    L = rb.lib()
    for code, word in [(0, b"ok"), (1, b"invalid"), (4, b"timed out"), (5, b"unsupported")]:
        assert word in L.rtb_status_string(code)


def test_null_context_rejected(rb):
    L = rb.lib()
    st = L.rtb_sgemm(None, 2, 2, 2, None, 2, 0, None, 2, 0, None, 0, None, 2, 0, None)
    assert st == rb._lib.RTB_E_INVALID
    assert "rtb_ctx" in rb._lib.last_error()
    assert L.rtb_conv2d_fwd(None, *([1] * 11), None, 0, None, None, None, 0, None, 0, 0,
                            None) == rb._lib.RTB_E_INVALID
    assert L.rtb_matmul_bias_norm_act(None, 2, 2, 2, None, 2, 0, None, 2, 0, None, None, None,
                                      1e-5, 0, None, 2, 0, None) == rb._lib.RTB_E_INVALID
    assert L.rtb_layer_norm(None, 2, 2, None, 2, None, None, 1e-5, 0, None, 2,
                            None) == rb._lib.RTB_E_INVALID
    assert "rtb_ctx" in rb._lib.last_error()


def test_init_without_gpu_fails_cleanly(rb):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    h = ctypes.c_void_p()
    st = rb.lib().rtb_init(0, ctypes.byref(h))
    assert st != 0 and not h.value
    assert rb._lib.last_error()


@pytest.mark.parametrize("n,seed,tid", [(1, 0, 0), (17, 3, 1), (100003, 2, 5)])
def test_host_generator_matches_oracle(rb, orc, n, seed, tid):
    a = rb.fill_normal((n,), seed, tid, 0.5, 2.0)
    b = orc.normal((n,), seed, tid, 0.5, 2.0)
    np.testing.assert_array_equal(a, b)
    a = rb.fill_uniform((n,), seed, tid, -0.1, 0.1)
    b = orc.uniform((n,), seed, tid, -0.1, 0.1)
    np.testing.assert_array_equal(a, b)


def test_packed_weight_size(rb):
    L = rb.lib()
    assert L.rtb_conv2d_packed_weight_size(64, 3, 7, 7) == 64 * 49 * 4
    assert L.rtb_conv2d_packed_weight_size(128, 128, 3, 3) == 128 * 9 * 128
