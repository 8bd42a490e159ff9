"""pytest configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs on any CPU host (oracle, golden vectors, host logic, the
C-ABI export table); `-m gpu` runs the parity tests through the CUDA kernels.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libnl_ops.so")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
