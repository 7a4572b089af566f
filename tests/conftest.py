"""Shared test set-up: the ``gpu`` marker, repo-root imports and golden-file loaders."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


def cuda_ok() -> bool:
    import torch

    return torch.cuda.is_available()


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN
