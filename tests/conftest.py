"""Shared fixtures.  `-m "not gpu"` runs on any host; `-m gpu` needs a B200."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def lib():
    import cubutterfly_b200 as cb
    from cubutterfly_b200 import _build

    if not cb.DEFAULT_LIBRARY.exists():
        _build.build()
    return cb.Library()


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference

    if not Reference.available():
        pytest.skip("oracle/_ref (the reference's compiled CPU oracles) is not built on this host")
    return Reference()


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(ROOT / "tests" / "golden" / "golden.npz"))


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a host without a CUDA device")
    return torch.device("cuda:0")


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.complex128 if np.iscomplexobj(a) or np.iscomplexobj(b) else np.float64)
    b = np.asarray(b, dtype=a.dtype)
    den = np.linalg.norm(b.ravel())
    return float(np.linalg.norm((a - b).ravel()) / (den if den else 1.0))
