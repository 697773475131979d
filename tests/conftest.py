"""Shared pytest configuration.

* ``gpu`` marks tests that need a B200; the CPU suite runs ``-m "not gpu"``.
* The repository root is put on ``sys.path`` (for ``bysj_b200`` and
  ``oracle``), and ``oracle/`` itself so the oracle reads as the reference's
  ``reference`` package in tests.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for path in (ROOT, ROOT / "oracle"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built extension")


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {k: data[k] for k in data.files}


@pytest.fixture
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")
