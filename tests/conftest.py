import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the CUDA kernels through the C ABI")


@pytest.fixture(scope="session")
def golden():
    """Golden fixtures written from the reference run (tests/golden/make_golden.py).
    Returns {case: {key: array}}."""
    data = np.load(GOLDEN)
    cases = {}
    for name in data.files:
        case, key = name.split("/", 1)
        cases.setdefault(case, {})[key] = data[name]
    return cases


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.build()
    return oracle
