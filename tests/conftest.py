"""Test configuration: the `gpu` marker, import paths, and the shared library fixture.

CPU runs (`-m "not gpu"`) cover the oracle against the golden fixtures and gguf-py, the host logic and the C ABI's
exports; GPU runs (`-m gpu`) are the parity tests proper and call the CUDA kernels through the C ABI.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "faie2-flashnext_b200")
for p in (ROOT, os.path.join(PKG, "flashnext"), PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); the parity tests proper")


@pytest.fixture(scope="session")
def libpath():
    """Path of the built C-ABI library (built here if missing; the GPU box receives the prebuilt file)."""
    from fn import DLL
    if not os.path.exists(DLL):
        import build
        build.build(verbose=False)
    return DLL


@pytest.fixture(scope="session")
def fn(libpath):
    from fn import FN
    f = FN(libpath)
    f.set_device(int(os.environ.get("FN_DEVICE", "0")))
    return f


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "dequant_golden.npz"))
