import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a); run with -m gpu")
    # the oracle (CPU checker) and the product library are built in-tree when missing
    if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True, capture_output=True)
    if not os.path.exists(os.path.join(ROOT, "syrinx_b200", "libsyrinx_b200.so")):
        subprocess.run(["make", "-j8", "-C", os.path.join(ROOT, "syrinx_b200", "csrc")], check=True,
                       capture_output=True)


@pytest.fixture(scope="session")
def kats():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "parity_kat.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def quant_golden():
    import numpy as np
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "quant_golden.npz")))


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(ROOT, "tests", "golden")
