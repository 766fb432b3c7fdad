"""B200-native batched geometric-product path of GEO (Geometric Elementary Operators).

The product is the C-ABI shared library ``libgeo_b200.so`` built from ``csrc/``
(sm_100a CUDA kernels + the reference's ``geo_batch_gp_*``, ``geo_batch_gp_cuda_*``,
``geo_hand_cuda_*`` and ``geo_operator_*`` entry points, plus the additive
``geo_b200_*`` trainer / data-parallel / pairwise / sparse calls declared in
``include/geo/geo_b200.h``). This module is a thin ctypes mirror of that ABI for
Python callers (tests, bench); it adds no arithmetic of its own and raises if
the library is missing rather than falling back to anything.
"""
from __future__ import annotations

import ctypes
import pathlib

from . import abi
from .abi import (  # noqa: F401  (re-exported)
    GEO_BATCH_GP_ABI_VERSION,
    GEO_BATCH_GP_CUDA_ABI_VERSION,
    GEO_B200_ABI_VERSION,
    BatchGpPlan,
    CudaPlan,
    OperatorPlanI32,
    OperatorTermI32,
    OptimizerConfig,
    lib,
    library_path,
)

__all__ = [
    "abi", "lib", "library_path", "BatchGpPlan", "CudaPlan", "OperatorPlanI32", "OperatorTermI32",
    "OptimizerConfig", "canonical_signature",
]


def canonical_signature(dimension: int, negative: int) -> list[int]:
    """First dimension-negative axes square to +1, the last `negative` to -1.

    This is the signature convention of the reference tests
    (tests/test_batch_gp.c:44), so Cl(3,3) = [1, 1, 1, -1, -1, -1].
    """
    return [1 if a < dimension - negative else -1 for a in range(dimension)]
