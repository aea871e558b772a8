"""pytest configuration: the ``gpu`` marker and import paths.

Tests marked ``gpu`` need a B200 and call the CUDA library through its C ABI; the rest run
on CPU (the oracle against the reference's golden vectors, host logic, library loading).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "kimi-k3-in-c_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the CUDA kernels)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        d = np.load(os.path.join(GOLDEN, name + ".npz"))
        return {k: d[k] for k in d.files}
    return load


@pytest.fixture(scope="session")
def ctx():
    """One libk3cuda context on device 0 for the whole GPU session."""
    import k3cuda
    c = k3cuda.Context(int(os.environ.get("K3CUDA_DEVICE", "0")))
    yield c
    c.close()
