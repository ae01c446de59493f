import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def kats():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "reference_kat.json")) as f:
        return {k["name"]: k for k in json.load(f)["kats"]}


@pytest.fixture(scope="session")
def gpu():
    """Skip cleanly where torch sees no CUDA device (the -m gpu suite runs on a B200)."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import rustorch_b200 as rb
    rb.lib()
    return rb
