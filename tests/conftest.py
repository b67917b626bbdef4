import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.lib()
    return o


@pytest.fixture(scope="session")
def backend_module():
    """The product package; fails loudly if the CUDA library is not built."""
    import kernrt_b200

    kernrt_b200.load()
    return kernrt_b200


@pytest.fixture(scope="module")
def gpu():
    """A CUDA backend on device 0 (the test is marked gpu; no fallback)."""
    import kernrt_b200

    b = kernrt_b200.CudaBackend(0)
    yield b
    b.close()
