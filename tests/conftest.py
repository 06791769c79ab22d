import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def dev():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mlz_b200
    mlz_b200.init(0)
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name))
    return load


@pytest.fixture(autouse=True)
def _device_error_word(request):
    """After every GPU test the kernel error word must be clear (no bounded wait expired)."""
    yield
    if request.node.get_closest_marker("gpu") is None or not cuda_available():
        return
    import mlz_b200
    assert mlz_b200.device_errors(0) == 0
