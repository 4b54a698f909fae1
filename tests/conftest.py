"""Shared test set-up: import paths and the `gpu` marker.

`-m "not gpu"` runs here without a GPU: the oracle against the golden
vectors, the host-side planner and ABI refusals through the built C library,
the Python API with fake backends, and world_size-2 gloo runs of the
sharding logic. `-m gpu` runs the CUDA parity tests through the C ABI.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE_ROOT = ROOT / "alelyon-compute-kit_b200"
for path in (PACKAGE_ROOT, ROOT / "oracle", ROOT):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        return np.load(GOLDEN / f"{name}.npz")
    return load
