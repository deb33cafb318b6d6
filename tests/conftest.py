"""Shared test setup: import paths, the `gpu` marker, and fixtures for the engine and oracle.

Tests marked `gpu` need a B200 (they run the engine's kernels); everything else runs on a
CPU-only machine.  The oracle (oracle/) is the checker, never the thing under test.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "chroma-radiance_b200"
for p in (str(PKG), str(REPO), str(REPO / "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the engine's CUDA kernels)")


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def engine():
    import b2g

    b2g.init()
    return b2g


@pytest.fixture(scope="session")
def ref():
    """The reference's own cuBLASLt path (built from its sources); skipped when not built."""
    from oracle import REF_PATH, Ref

    if not REF_PATH.exists():
        pytest.skip("oracle/_ref/libref_cublaslt.so not built (needs the reference sources at build time)")
    return Ref()


def rel_err(got, want) -> float:
    """max|got - want| / max|want| in float64."""
    g = np.asarray(got, dtype=np.float64)
    w = np.asarray(want, dtype=np.float64)
    denom = np.abs(w).max()
    return float(np.abs(g - w).max() / (denom if denom > 0 else 1.0))
