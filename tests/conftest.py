import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200 / sm_100a)")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from h3_engine_b200 import _lib
    _lib.lib()          # fail loudly if the library is missing
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _no_device_error(request):
    """Every GPU test ends with a clean device error word."""
    yield
    if request.node.get_closest_marker("gpu") is not None and has_gpu():
        from h3_engine_b200 import _lib
        assert _lib.device_error(clear=True) == 0, "a kernel recorded a device-side error"
