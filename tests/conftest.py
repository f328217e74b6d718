import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libllmdot_cuda.so")
    config.addinivalue_line("markers", "slow: multi-minute case (large synthetic model)")


def _have_gpu() -> bool:
    try:
        from dotllm_b200 import native
        return native.device_count() > 0
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    # GPU tests fail loudly (not skip) when selected on a machine whose library or device is
    # missing: the product path has no fallback, and a silent skip would hide that.
    pass


@pytest.fixture(scope="session")
def gpu():
    from dotllm_b200 import native
    n = native.device_count()
    if n == 0:
        raise RuntimeError("no CUDA device visible: GPU tests need a B200")
    return n


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    O.set_threads(max(1, O.max_threads()))
    return O


@pytest.fixture(scope="session")
def backend(gpu):
    from dotllm_b200.backend import CudaBackend
    b = CudaBackend(0)
    yield b
    b.dispose()
