import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built libsaf.so")
    config.addinivalue_line("markers", "expects_device_status: the test sets and checks the device status flags")


@pytest.fixture(scope="session")
def cuda_device():
    """The GPU tests' device.  A GPU test that runs without a usable B200
    fails (it does not skip): the driver runs `-m gpu` on a B200 box only."""
    import torch

    assert torch.cuda.is_available(), "GPU tests need CUDA"
    from sparseattnfunctions_b200 import _lib

    lib = _lib.load()
    assert lib.saf_device_check(0) == 0, "device 0 is not an sm_100 GPU"
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _check_device_status(request):
    """After every GPU test, the device status word must be clear (no wait
    timed out, no CSR index was out of range) unless the test expects it."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    if request.node.get_closest_marker("expects_device_status") is not None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from sparseattnfunctions_b200 import _lib

    flags = _lib.read_device_status(0, clear=True)
    assert flags == 0, f"device status flags set: {flags:#x}"
