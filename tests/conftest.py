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


def ideal_linear(a, w, b, epi_name: str):
    """The Linear and its epilogue in fp64 with no intermediate rounding: a [M, K] and the decoded weight
    w [N, K] as given (bf16 values), bias b. The gated residual uses the x and gate of the decoding-GEMM
    tests (x = sin(1e-4 * index), gate = linspace(-2, 2, N) in bf16)."""
    import math

    import torch

    f64 = torch.float64
    acc = a.to(f64) @ w.to(f64).T
    if b is not None:
        acc = acc + b.to(f64)
    if epi_name == "gelu":
        return 0.5 * acc * (1 + torch.tanh(math.sqrt(2 / math.pi) * (acc + 0.044715 * acc ** 3)))
    if epi_name == "resid":
        m, n = acc.shape
        x = torch.arange(m * n, device=acc.device, dtype=torch.float32).reshape(m, n).mul_(1e-4).sin_().to(f64)
        gate = torch.linspace(-2, 2, n, device=acc.device).to(torch.bfloat16).to(f64).reshape(1, n)
        return x + gate * acc
    return acc


def assert_no_further(got, ref, ideal):
    """``got`` (a launch that accumulates K in another order, e.g. split-K) is no further from the fp64
    result than ``ref`` (the unsplit GEMM on the same operands): the two differ only by fp32 accumulation
    order, which moves a few bf16 roundings by one ulp."""
    import torch

    eg = (got.to(torch.float64) - ideal).abs()
    er = (ref.to(torch.float64) - ideal).abs()
    assert eg.mean().item() <= 1.25 * er.mean().item() + 1e-9, (eg.mean().item(), er.mean().item())
    assert eg.max().item() <= 2.0 * er.max().item() + 1e-6, (eg.max().item(), er.max().item())
