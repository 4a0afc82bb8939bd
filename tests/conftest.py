"""pytest configuration shared by the CPU and GPU suites.

* ``-m "not gpu"`` -- the oracle against the golden vectors, host logic, the
  C-ABI library's symbol table, and multi-rank host logic over gloo; runs here.
* ``-m gpu``       -- parity of the CUDA kernels (through the C-ABI) against
  the oracle on a B200.
"""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mini-cuda-kernel-engine_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden_dir() -> str:
    return os.path.join(ROOT, "tests", "golden")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False
