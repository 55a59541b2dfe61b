import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels of libp0mm.so)")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """the oracle and the CUDA library are built in-tree before any test (nvcc cross-compiles without a GPU)"""
    from oracle import ref
    ref.build()
    from p0pc0rn_b200 import build
    build.build()


@pytest.fixture(scope="session")
def g():
    """one device context for the GPU tests; the CUDA library must load (no fallback exists)"""
    import p0pc0rn_b200 as p0
    gpu = p0.Gpu(0)
    yield gpu
    gpu.close()
