"""Shared pytest setup: import paths, the `gpu` marker, and common helpers."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "latent-weight-lab_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden" / "golden_block_fht.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity tests of the CUDA path")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN, allow_pickle=False)


@pytest.fixture(scope="session")
def native_lib():
    """liblwl_b200.so, built in-tree if it is missing (nvcc cross-compiles without a GPU)."""
    import build as lwl_build  # latent-weight-lab_b200/build.py

    if not lwl_build.LIB.exists():
        lwl_build.build()
    from latent_weight_lab import _native

    return _native.load()


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64).reshape(-1)
    b = np.asarray(b, dtype=np.float64).reshape(-1)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a - b))
