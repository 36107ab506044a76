"""Shared pytest setup: import paths, the `gpu` marker and library fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "foundation-pose-inference-library_b200"
for p in (str(PKG / "python"), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def fpk():
    from fp_b200.kernels import FpkLibrary

    return FpkLibrary()


@pytest.fixture(scope="session")
def oracle():
    from oracle_lib import Oracle

    return Oracle()
