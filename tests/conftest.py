"""Test configuration: import paths and the ``gpu`` marker.

``-m "not gpu"`` runs on any host (oracle vs golden vectors, host logic,
C-ABI exports); ``-m gpu`` runs the parity tests on a B200 through the
C ABI of libw4a8.so.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "lsq-lowbit-optimization_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
