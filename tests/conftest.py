"""Shared pytest configuration: the ``gpu`` marker and common fixtures."""
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built libtilemix_b200.so")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.fixture
def exact_numerics(monkeypatch):
    """Run the library in exact numerics (IEEE divisions, fp32-accumulated scores): the
    arithmetic of the CPU oracle and of the reference's interpreter fixtures, so comparisons
    against them are tight. The default numerics reproduce the reference's GPU run instead
    (tests/test_gpu_reference_triton.py)."""
    monkeypatch.setenv("TILEMIX_B200_NUMERICS", "exact")
