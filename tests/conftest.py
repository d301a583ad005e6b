"""Shared test configuration.

* registers the ``gpu`` marker (tests that need a B200; run with ``-m gpu``);
* puts the repository root (for ``oracle``) and the package directory
  ``specdiff-ae_b200`` (for ``specverify``) on ``sys.path``;
* loads golden fixtures from ``tests/golden``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "specdiff-ae_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def load_golden(name):
    return np.load(GOLDEN / name, allow_pickle=False)


def bf16_from_bits(bits):
    """uint16 bf16 bit patterns -> float32 numpy (exact)."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


@pytest.fixture(scope="session")
def golden():
    return load_golden


def cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
