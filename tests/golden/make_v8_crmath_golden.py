"""Generate tests/golden/v8_crmath_golden.npz: the all-node-kinds V8 graph trained
per sample (3 SGD and 3 Adam steps over 9 samples, the v8cb_* cases of
make_golden.py) by the reference's own CPU code built with its exp and tanh
bound to the runtime's correctly rounded functions (oracle/_ref/
libgeo_ref_crmath.so, `make -C oracle ref`). Against these the GPU graph
runtime, which uses the same functions, is held to the float64 parity bar after
Adam too; against the C-library build (batch_gp_golden.npz) the remaining gap is
the C library's rounding of tanh and exp.

Usage: python tests/golden/make_v8_crmath_golden.py
"""
from __future__ import annotations

import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests" / "golden"))

from make_golden import composed_batch_cases  # noqa: E402
from oracle import oracle as orc  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent / "v8_crmath_golden.npz"
LIB = ROOT / "oracle" / "_ref" / "libgeo_ref_crmath.so"


def main() -> None:
    if not LIB.exists():
        raise SystemExit(f"{LIB} is missing: build it with `make -C oracle ref REF=<reference tree>`")
    data: dict = {}
    composed_batch_cases(orc.Reference(LIB), data)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(data)} arrays)")
    glibc = np.load(ROOT / "tests" / "golden" / "batch_gp_golden.npz")
    for key in sorted(k for k in data if k.endswith("_w1")):
        d = np.max(np.abs(data[key] - glibc[key]))
        print(f"{key}: max |crmath build - C library build| = {d:.3g}")


if __name__ == "__main__":
    main()
