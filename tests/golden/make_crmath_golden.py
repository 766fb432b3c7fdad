"""Generate tests/golden/crmath_golden.npz: arguments and the correctly rounded
exp and tanh of each (mpmath at 300 bits, rounded to binary64 by exact integer
arithmetic, so subnormal results are rounded once), plus this machine's C
library values of both (the reference evaluates its graph nonlinearities with
those: full_cycle_v8.c tanh node and sigmoid).

Arguments: normal and uniform samples over the ranges the graphs see and the
whole domain of exp, powers of two down to the thresholds of the short cuts,
the overflow and underflow edges, and arguments whose double-double evaluation
cannot decide the rounding (the fixed-point path then decides; found by
searching the fast path's rounding test over ~10^8 random arguments).

Usage: python tests/golden/make_crmath_golden.py
"""
from __future__ import annotations

import ctypes
import math
import pathlib

import mpmath
import numpy as np

OUT = pathlib.Path(__file__).resolve().parent / "crmath_golden.npz"

HARD = [  # the fast path's rounding test fails on these (exp: E, tanh: T)
    ("E", "0x1.ece5869f268p+5"), ("E", "-0x1.18671c71f0b74p+9"), ("E", "0x1.c78fd5aa7d2e6p+7"),
    ("E", "-0x1.5c8fedce2056dp+9"),
    ("T", "-0x1.09f3fc9059ebbp+3"), ("T", "-0x1.43c572aa6ecc2p+3"), ("T", "-0x1.0bc0c9a151d38p+4"),
    ("T", "0x1.3738082ef370ap+3"), ("T", "0x1.5ca99f1dcbe1cp+2"), ("T", "0x1.1dcd357b1b28bp+4"),
]


def round_binary64(v: mpmath.mpf) -> float:
    """Nearest binary64 to v (ties to even; v not a tie for these functions)."""
    if v == 0:
        return 0.0
    sign = -1.0 if v < 0 else 1.0
    a = abs(v)
    if a >= mpmath.mpf(2) ** 1024:
        return sign * math.inf
    e = int(mpmath.floor(mpmath.log(a, 2)))
    while mpmath.mpf(2) ** e > a:
        e -= 1
    while mpmath.mpf(2) ** (e + 1) <= a:
        e += 1
    ulp_e = max(e, -1022) - 52
    n = int(mpmath.nint(a / mpmath.mpf(2) ** ulp_e))
    if n >= 2 ** 53 and e >= 1023:
        return sign * math.inf
    return sign * math.ldexp(float(n), ulp_e)


def main() -> None:
    mpmath.mp.prec = 300
    rng = np.random.default_rng(2024)
    parts = [
        rng.normal(0.0, 3.0, 1200),
        rng.normal(0.0, 0.05, 300),
        rng.uniform(-745.5, 709.9, 400),
        rng.uniform(-20.0, 20.0, 400),
        np.exp2(rng.uniform(-60.0, 5.0, 400)) * rng.choice([-1.0, 1.0], 400),
        np.array([0.0, -0.0, 1e-300, -1e-300, 2.0 ** -54, -(2.0 ** -54), 2.0 ** -53, 2.0 ** -27, -(2.0 ** -27),
                  2.0 ** -26, 19.0, 19.1, -19.1, 19.06, 708.0, 709.78, 709.79, 710.0, -708.0, -708.5, -745.0,
                  -745.13, -745.2, -746.0, 1.0, -1.0, 0.5, 1e-8, math.inf, -math.inf, 2.0 ** -1074]),
        np.array([float.fromhex(h) for _, h in HARD]),
    ]
    x = np.concatenate(parts).astype(np.float64)
    exp_cr = np.empty_like(x)
    tanh_cr = np.empty_like(x)
    for i, v in enumerate(x):
        v = float(v)
        if math.isinf(v):
            exp_cr[i] = math.inf if v > 0 else 0.0
            tanh_cr[i] = math.copysign(1.0, v)
            continue
        exp_cr[i] = round_binary64(mpmath.exp(mpmath.mpf(v)))
        t = round_binary64(mpmath.tanh(mpmath.mpf(v)))
        tanh_cr[i] = math.copysign(abs(t), v)  # tanh(-0) = -0
    libm = ctypes.CDLL("libm.so.6")
    for name in ("exp", "tanh"):
        getattr(libm, name).restype = ctypes.c_double
        getattr(libm, name).argtypes = [ctypes.c_double]
    exp_libc = np.array([libm.exp(float(v)) for v in x])
    tanh_libc = np.array([libm.tanh(float(v)) for v in x])
    np.savez_compressed(OUT, x=x, exp=exp_cr, tanh=tanh_cr, exp_libc=exp_libc, tanh_libc=tanh_libc)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {x.size} arguments)")
    for name, cr, lc in (("exp", exp_cr, exp_libc), ("tanh", tanh_cr, tanh_libc)):
        diff = int(np.sum(cr.view(np.uint64) != lc.view(np.uint64)))
        print(f"C library {name} differs from the correctly rounded value on {diff} of {x.size}")


if __name__ == "__main__":
    main()
