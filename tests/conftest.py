"""Shared pytest setup: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs on a CPU-only host: oracle-vs-golden pins, host-side API
logic, the C-ABI symbol check and the gloo multi-process tests.  ``-m gpu``
tests need a CUDA device and are the parity tests proper (CUDA kernels called
through the C-ABI, compared with the CPU oracle).
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_ROOT = ROOT / "bayes-ssm_b200"
for path in (ROOT, PKG_ROOT):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run with -m gpu)")


def cuda_available() -> bool:
    try:
        import torch
        return bool(torch.cuda.is_available())
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN
