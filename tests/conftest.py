import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "dispatcher-hybrid-2_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: takes more than ~20 s on the CPU")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(GOLDEN)
