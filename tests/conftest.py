"""Shared fixtures. GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
from __future__ import annotations

import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def all_signatures(min_dim: int = 1, max_dim: int = 6):
    """(dimension, negative count, signature) for every canonical signature."""
    from geometricelementaryoperators_b200 import canonical_signature

    for n in range(min_dim, max_dim + 1):
        for q in range(n + 1):
            yield n, q, canonical_signature(n, q)


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def reference():
    """The reference compiled from its own sources; built on demand where the tree exists."""
    from oracle import oracle as orc

    if not orc.ensure_reference_built():
        pytest.skip("reference build not available (golden fixtures still pin the oracle)")
    return orc.Reference()


def tol_close(a, b, tol: float) -> bool:
    """The reference's mixed form |a-b| <= tol (1 + |a| + |b|) (tests/test_batch_gp.c:23-25)."""
    import numpy as np

    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return bool(np.all(np.abs(a - b) <= tol * (1.0 + np.abs(a) + np.abs(b))))


def max_violation(a, b, tol: float) -> float:
    import numpy as np

    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b) / (tol * (1.0 + np.abs(a) + np.abs(b)))))
