import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the CUDA extension")


@pytest.fixture(scope="session")
def cuda_lib():
    """Builds libosam.so if it is out of date and loads it; GPU tests fail (not skip) without a GPU."""
    import torch
    from objectsam_b200 import build
    build.build()
    from objectsam_b200._lib import lib
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    major, minor = torch.cuda.get_device_capability()
    assert (major, minor) == (10, 0), f"needs sm_100 (B200), got sm_{major}{minor}"
    return lib()


@pytest.fixture(autouse=True)
def _no_device_error(request):
    """Every GPU test must leave the library's device error word clean (no timed-out waits)."""
    yield
    if request.node.get_closest_marker("gpu") is not None:
        from objectsam_b200._lib import device_error
        assert device_error() == 0, "a kernel reported a device-side error"
