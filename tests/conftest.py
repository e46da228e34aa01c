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


def reference_package():
    """Import the reference package (dispatcher_hybrid) when its source tree
    is available: from $DISPATCHER_REFERENCE, or a `reference` directory next
    to this repository.  Returns None otherwise (the GPU box never has it)."""
    import importlib
    for d in (os.environ.get("DISPATCHER_REFERENCE", ""),
              os.path.join(os.path.dirname(ROOT), "reference")):
        if d and os.path.isdir(os.path.join(d, "dispatcher_hybrid")):
            if d not in sys.path:
                sys.path.append(d)
            break
    try:
        return importlib.import_module("dispatcher_hybrid")
    except Exception:
        return None
