"""Shared pytest set-up: import paths, the ``gpu`` marker, golden-fixture loading."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
PKG_ROOT = REPO / "triton-muonadamw_b200"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str):
    return torch.load(GOLDEN / name, weights_only=False)


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
