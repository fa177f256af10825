import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and libmans_cuda.so")
    config.addinivalue_line("markers", "slow: long-running parity case at full benchmark size")


@pytest.fixture(scope="session")
def ctx():
    """One CUDA context for the GPU tests (the library must load: no fallback)."""
    import meltan_b200 as mb
    c = mb.Context(0)
    yield c
    c.close()
