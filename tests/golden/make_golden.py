"""Generate tests/golden/batch_gp_golden.npz from the reference itself.

Runs the reference CPU code compiled from its own sources (oracle/_ref, built
by `make -C oracle ref` where the reference tree is present) on seeded inputs
and stores inputs and outputs as exact float64 arrays:

* batch path (reference src/batch_gp.c): for every canonical signature of
  dimension 1..6 and both sides, forward, parameter VJP and one MSE-SGD step
  (lr 0.01) on a batch of 3 samples;
* sign tables (reference src/operator_kernel.c:111-135) for every canonical
  signature, packed as int8 [4^n];
* dense pairwise GP / VJP / JVP (src/operator_kernel.c:412-539) per signature;
* sparse plans (src/operator_kernel.c:191-334) with terms {0:+1, 1:-2, top:+1};
* the V8 per-sample loop (src/full_cycle_v8.c) with SGD and Adam, 3 steps on
  3 samples, for a handful of signatures and both sides;
* the all-node-kinds V8 graph of the reference test (tests/test_full_cycle_v8.c:
  158-181): loss and the gradients of both parameters, every signature.

Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from geometricelementaryoperators_b200 import canonical_signature  # noqa: E402
from geometricelementaryoperators_b200.synthetic import splitmix_uniform  # noqa: E402
from oracle import oracle as orc  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent / "batch_gp_golden.npz"
V8_CASES = [(2, 0), (3, 0), (4, 1), (5, 1), (6, 0), (6, 3)]


def composed_batch_cases(ref, data: dict) -> None:
    """v8cb_*: 3 SGD and 3 Adam steps of the all-node-kinds graph over 9 samples."""
    for n, q in [(2, 0), (3, 1), (4, 0), (5, 2), (6, 0), (6, 3)]:
        sig = canonical_signature(n, q)
        N = 1 << n
        values = {"input": orc.v8_mv_fill(n, 3 + n + q), "target": orc.v8_mv_fill(n, 11 + 2 * n + q),
                  "w1": orc.v8_mv_fill(n, 19 + n + q), "w2": orc.v8_mv_fill(n, 29 + n + q)}
        xs = splitmix_uniform(91 + n + q, (9, N))
        ts = splitmix_uniform(92 + n + q, (9, N))
        data[f"v8cb_n{n}q{q}_x"], data[f"v8cb_n{n}q{q}_t"] = xs, ts
        for opt in (1, 2):
            w1s, w2s, losses = ref.v8_composed_train(sig, values, xs, ts, opt, 1e-2, steps=3)
            data[f"v8cb_n{n}q{q}_opt{opt}_w1"] = w1s
            data[f"v8cb_n{n}q{q}_opt{opt}_w2"] = w2s
            data[f"v8cb_n{n}q{q}_opt{opt}_loss"] = losses


def main() -> None:
    if not orc.ensure_reference_built():
        raise SystemExit("the reference build (oracle/_ref) is required to make golden vectors")
    ref = orc.Reference()
    data: dict[str, np.ndarray] = {}
    for n in range(1, 7):
        for q in range(n + 1):
            sig = canonical_signature(n, q)
            N = 1 << n
            key = f"n{n}q{q}"
            seed = 1000 + 10 * n + q
            x = splitmix_uniform(seed, (3, N))
            w = splitmix_uniform(seed + 1, (N,))
            t = splitmix_uniform(seed + 2, (3, N))
            data[f"{key}_x"], data[f"{key}_w"], data[f"{key}_t"] = x, w, t
            data[f"{key}_signs"] = np.array([ref.sign(l, r, sig) for l in range(N) for r in range(N)], np.int8)
            for side, left in (("R", False), ("L", True)):
                st, y = ref.forward(sig, x, w, left)
                assert st == 0
                st, g = ref.vjp(sig, x, t, left)
                assert st == 0
                st, w2, loss = ref.sgd_step(sig, x, t, 0.01, w, left)
                assert st == 0
                data[f"{key}{side}_y"], data[f"{key}{side}_g"] = y, g
                data[f"{key}{side}_sgd_w"], data[f"{key}{side}_sgd_loss"] = w2, np.array([loss])
            a, b, c, ta, tb = x[0], x[1], t[0], t[1], t[2]
            data[f"{key}_gp"] = ref.gp(sig, a, b)
            la, rb = ref.gp_vjp(sig, a, b, c)
            data[f"{key}_gp_vjp_l"], data[f"{key}_gp_vjp_r"] = la, rb
            data[f"{key}_gp_jvp"] = ref.gp_jvp(sig, a, b, ta, tb)
            if n >= 2:
                blades, coeffs, params = [0, 1, N - 1], [1, -2, 1], [0.5, -1.25, 2.0]
                for side in (0, 1):
                    data[f"{key}_sp{side}_apply"] = ref.sparse_apply(sig, side, blades, coeffs, a)
                    data[f"{key}_sp{side}_param"] = ref.sparse_apply_parametric(sig, side, blades, params, a)
                    data[f"{key}_sp{side}_vjp"] = ref.sparse_apply_vjp(sig, side, blades, coeffs, c)
                    ic, pc = ref.sparse_apply_parametric_vjp(sig, side, blades, params, a, c)
                    data[f"{key}_sp{side}_pvjp_in"], data[f"{key}_sp{side}_pvjp_par"] = ic, pc
    for n, q in V8_CASES:
        sig = canonical_signature(n, q)
        N = 1 << n
        xs = splitmix_uniform(77 + n, (3, N))
        ts = splitmix_uniform(78 + n, (3, N))
        w0 = splitmix_uniform(79 + n, (N,))
        data[f"v8_n{n}q{q}_x"], data[f"v8_n{n}q{q}_t"], data[f"v8_n{n}q{q}_w0"] = xs, ts, w0
        for opt in (1, 2):
            for side, left in (("R", False), ("L", True)):
                params, losses = ref.v8_train(sig, left, xs, ts, w0, opt, 1e-2, 0.9, 0.999, 1e-8, steps=3)
                data[f"v8_n{n}q{q}{side}_opt{opt}_w"] = params
                data[f"v8_n{n}q{q}{side}_opt{opt}_loss"] = losses
    for n in range(1, 7):
        for q in range(n + 1):
            sig = canonical_signature(n, q)
            values = {"input": orc.v8_mv_fill(n, 3 + n + q), "target": orc.v8_mv_fill(n, 11 + 2 * n + q),
                      "w1": orc.v8_mv_fill(n, 19 + n + q), "w2": orc.v8_mv_fill(n, 29 + n + q)}
            loss, g1, g2 = ref.v8_composed(sig, values)
            data[f"v8c_n{n}q{q}_loss"] = np.array([loss])
            data[f"v8c_n{n}q{q}_g1"], data[f"v8c_n{n}q{q}_g2"] = g1, g2
    # Per-sample training of the all-node-kinds graph over a small batch (the
    # general path of the batched V8 step is checked against these).
    composed_batch_cases(ref, data)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(data)} arrays)")


if __name__ == "__main__":
    main()
