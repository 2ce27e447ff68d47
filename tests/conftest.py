"""Shared fixtures. `-m gpu` tests need a B200 and the built kernel library; everything else runs on CPU."""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built libfoidfinder_b200.so")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability()
    if major != 10:
        pytest.fail(f"GPU tests need an sm_100 device, got compute capability {torch.cuda.get_device_capability()}")
    return torch.device("cuda", 0)


@pytest.fixture()
def no_device_error(cuda_device):
    """Asserts, after the test body, that no kernel reported a bounded-wait timeout."""
    from foidfinder_b200 import ops

    ops.device_error(cuda_device.index or 0, clear=True)
    yield
    assert ops.device_error(cuda_device.index or 0, clear=True) == 0, "a kernel reported a device-side timeout"
