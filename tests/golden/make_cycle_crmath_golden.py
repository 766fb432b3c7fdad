"""Checkpoints of the reference's own geo_cycle runner built with exp and tanh
bound to the runtime's correctly rounded functions (oracle/_ref/geo_cycle_crmath,
`make -C oracle ref`), for the models trained with Adam: written next to the
C-library fixtures as tests/golden/cycle/<name>.crmath.checkpoint and
<name>.crmath.train.txt, from the same IR and CSV files (make_cycle_golden.py).

Usage: python tests/golden/make_cycle_crmath_golden.py
"""
from __future__ import annotations

import pathlib
import subprocess

ROOT = pathlib.Path(__file__).resolve().parents[2]
RUNNER = ROOT / "oracle" / "_ref" / "geo_cycle_crmath"
OUT = pathlib.Path(__file__).resolve().parent / "cycle"
MODELS = ["mlp", "all_ops", "constraint", "resume1", "resume2"]


def main() -> None:
    if not RUNNER.exists():
        raise SystemExit(f"{RUNNER} is missing: build it with `make -C oracle ref REF=<reference tree>`")
    for name in MODELS:
        base = "resume" if name.startswith("resume") else name
        ckpt = OUT / f"{name}.crmath.checkpoint"
        res = subprocess.run([str(RUNNER), "train", str(OUT / f"{name}.geoir"), str(OUT / f"{base}.csv"), str(ckpt)],
                             capture_output=True, text=True, check=True)
        (OUT / f"{name}.crmath.train.txt").write_text(res.stdout.replace(str(ckpt), f"{name}.crmath.checkpoint"))
        print(name, res.stdout.strip())


if __name__ == "__main__":
    main()
