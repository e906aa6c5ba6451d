import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "mrl-index-rust-vector_b200")
for p in (ROOT, PKG_DIR, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; runs the CUDA product path")


@pytest.fixture(scope="session")
def ora():
    import ora as _ora  # the CPU oracle (test infrastructure)

    _ora.lib()
    return _ora


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(os.path.join(ROOT, "tests", "golden", "golden_small.npz"))


@pytest.fixture(scope="session")
def dev():
    import mrl_b200

    d = mrl_b200.Device(0)
    yield d
    d.close()
