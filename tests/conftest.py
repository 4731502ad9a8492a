import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long CPU oracle runs")


@pytest.fixture(scope="session")
def cuda_lib():
    """The built library on a CUDA device; GPU tests fail (never skip) if it is missing."""
    import torch

    from dsa_b200 import _native

    assert torch.cuda.is_available(), "gpu-marked test needs a CUDA device"
    return _native.load()
