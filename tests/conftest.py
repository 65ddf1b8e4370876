"""Shared test configuration.

``-m "not gpu"`` runs on any machine; ``-m gpu`` needs a CUDA device and the
in-tree native library.  GPU tests never fall back to the CPU: a missing
device or library is a failure, not a skip, when they are selected.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests" / "golden"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the native library")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is unavailable")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def golden():
    import torch

    def load(name):
        return torch.load(ROOT / "tests" / "golden" / name, weights_only=False)
    return load
