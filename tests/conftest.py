"""Shared pytest setup: the `gpu` marker and import paths.

Tests marked ``gpu`` need a CUDA (B200) device and run the libebx kernels;
everything else runs on CPU.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and runs libebx kernels")


@pytest.fixture(scope="session")
def cuda_ok():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True
