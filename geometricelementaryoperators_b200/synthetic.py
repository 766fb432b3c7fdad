"""Seeded synthetic workloads (host, numpy) for tests and benchmarks.

* ``splitmix_uniform``: counter-based splitmix64 -> uniform[-1, 1) with 53-bit
  resolution (exact in float64), the generator family the reference benchmarks
  use (benchmarks/bench_v8_batch_gp.c:16-25, there quantised to 1/1000).
* ``reference_fill``: the reference benchmark's own fill_vector values,
  ((x % 2001) - 1000) / 1000, for reproducing its inputs exactly.
* ``normal``: Box-Muller on two splitmix streams.

No dataset is involved anywhere: every benchmark shape is synthetic.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, count: int, offset: int = 0) -> np.ndarray:
    """x_i = mix(seed + golden * (offset + i + 1)) for i < count (uint64, wrapping)."""
    i = np.arange(offset + 1, offset + count + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        x = np.uint64(seed) + _GOLDEN * i
        x ^= x >> np.uint64(30)
        x *= _M1
        x ^= x >> np.uint64(27)
        x *= _M2
        x ^= x >> np.uint64(31)
    return x


def splitmix_uniform(seed: int, shape, offset: int = 0) -> np.ndarray:
    n = int(np.prod(shape))
    x = splitmix64(seed, n, offset)
    u = (x >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    return (2.0 * u - 1.0).reshape(shape)


def reference_fill(seed: int, count: int) -> np.ndarray:
    """Values of the reference benchmark's fill_vector(values, count, seed)."""
    x = splitmix64(seed, count)
    return ((x % np.uint64(2001)).astype(np.int64).astype(np.float64) - 1000.0) / 1000.0


def normal(seed: int, shape, std: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    u1 = (splitmix64(seed, n) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    u2 = (splitmix64(seed ^ 0x5DEECE66D, n) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    r = np.sqrt(-2.0 * np.log1p(-u1))
    return (std * r * np.cos(2.0 * np.pi * u2)).reshape(shape)
