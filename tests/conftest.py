"""Shared pytest setup: import paths, the ``gpu`` marker and common fixtures."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for path in (REPO / "drama3-studio_b200", REPO, REPO / "tests"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a host without CUDA; run with -m 'not gpu'")
    from drama_b200 import _lib

    _lib.library().device_check(torch.cuda.current_device())
    return torch.device("cuda", torch.cuda.current_device())
