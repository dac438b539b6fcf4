"""Shared pytest configuration.

``gpu`` marks tests that need a CUDA device and the built ``libgdn2_b200.so``;
the CPU suite runs with ``-m "not gpu"``.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and libgdn2_b200.so")
    config.addinivalue_line("markers", "slow: long-running test")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device not available")
    return torch.device("cuda:0")
