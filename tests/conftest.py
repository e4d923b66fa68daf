import os
import sys

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda_device():
    """The CUDA device for GPU tests.  GPU tests fail (never skip) when no
    device is usable: a silent skip would hide a missing native path."""
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)
