"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on any machine (oracle vs golden vectors, host logic, the
C ABI's exports).  `-m gpu` tests need a B200 and call the CUDA path through
the C ABI (libspider_b200.so).
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (B200)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
