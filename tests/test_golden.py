"""The oracle reproduces the committed golden vectors (made by the reference
itself, tests/golden/make_golden.py) bit for bit. Runs anywhere: no reference
tree and no GPU needed."""
from __future__ import annotations

import pathlib

import numpy as np
import pytest

from tests.conftest import all_signatures

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "batch_gp_golden.npz"
V8_CASES = [(2, 0), (3, 0), (4, 1), (5, 1), (6, 0), (6, 3)]


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_golden_signs(oracle, golden):
    for n, q, sig in all_signatures():
        N = 1 << n
        mine = np.array([oracle.sign(l, r, sig) for l in range(N) for r in range(N)], np.int8)
        assert np.array_equal(mine, golden[f"n{n}q{q}_signs"])


def test_golden_batch(oracle, golden):
    for n, q, sig in all_signatures():
        key = f"n{n}q{q}"
        x, w, t = golden[f"{key}_x"], golden[f"{key}_w"], golden[f"{key}_t"]
        for side, left in (("R", False), ("L", True)):
            assert np.array_equal(oracle.forward(sig, x, w, left)[1], golden[f"{key}{side}_y"])
            assert np.array_equal(oracle.vjp(sig, x, t, left)[1], golden[f"{key}{side}_g"])
            st, w2, loss = oracle.sgd_step(sig, x, t, 0.01, w, left)
            assert st == 0 and np.array_equal(w2, golden[f"{key}{side}_sgd_w"])
            assert loss == golden[f"{key}{side}_sgd_loss"][0]


def test_golden_operators(oracle, golden):
    for n, q, sig in all_signatures():
        key = f"n{n}q{q}"
        x, t = golden[f"{key}_x"], golden[f"{key}_t"]
        a, b, c, ta, tb = x[0], x[1], t[0], t[1], t[2]
        assert np.array_equal(oracle.gp(sig, a, b), golden[f"{key}_gp"])
        la, rb = oracle.gp_vjp(sig, a, b, c)
        assert np.array_equal(la, golden[f"{key}_gp_vjp_l"]) and np.array_equal(rb, golden[f"{key}_gp_vjp_r"])
        assert np.array_equal(oracle.gp_jvp(sig, a, b, ta, tb), golden[f"{key}_gp_jvp"])
        if n < 2:
            continue
        N = 1 << n
        blades, coeffs, params = [0, 1, N - 1], [1, -2, 1], [0.5, -1.25, 2.0]
        for side in (0, 1):
            assert np.array_equal(oracle.sparse_apply(sig, side, blades, coeffs, a), golden[f"{key}_sp{side}_apply"])
            assert np.array_equal(oracle.sparse_apply_parametric(sig, side, blades, params, a),
                                  golden[f"{key}_sp{side}_param"])
            assert np.array_equal(oracle.sparse_apply_vjp(sig, side, blades, coeffs, c), golden[f"{key}_sp{side}_vjp"])
            ic, pc = oracle.sparse_apply_parametric_vjp(sig, side, blades, params, a, c)
            assert np.array_equal(ic, golden[f"{key}_sp{side}_pvjp_in"])
            assert np.array_equal(pc, golden[f"{key}_sp{side}_pvjp_par"])


def test_golden_v8(oracle, golden):
    from geometricelementaryoperators_b200 import canonical_signature

    for n, q in V8_CASES:
        sig = canonical_signature(n, q)
        xs, ts, w0 = golden[f"v8_n{n}q{q}_x"], golden[f"v8_n{n}q{q}_t"], golden[f"v8_n{n}q{q}_w0"]
        for opt in (1, 2):
            for side, left in (("R", False), ("L", True)):
                want = golden[f"v8_n{n}q{q}{side}_opt{opt}_w"]
                w, m, v = w0.copy(), np.zeros_like(w0), np.zeros_like(w0)
                for step in range(1, 4):
                    gsum = np.zeros_like(w0)
                    for j in range(xs.shape[0]):
                        a, b = (w, xs[j]) if left else (xs[j], w)
                        r = oracle.gp(sig, a, b) + (-1.0 * ts[j])
                        la, rb = oracle.gp_vjp(sig, a, b, r)
                        gsum = gsum + (la if left else rb) * 1.0
                    st, w, m, v = oracle.v8_update(opt, 1e-2, 0.9, 0.999, 1e-8, 1.0 / xs.shape[0], step, gsum, w, m, v)
                    assert st == 0 and np.array_equal(w, want[step - 1])


def test_known_answers(oracle):
    """Cl(2,0) basis products (reference tests/test_cl20.c:74-75)."""
    sig = [1, 1]
    e = np.eye(4)
    one, e1, e2, e12 = e[0], e[1], e[2], e[3]
    assert np.array_equal(oracle.gp(sig, e1, e1), one)
    assert np.array_equal(oracle.gp(sig, e2, e2), one)
    assert np.array_equal(oracle.gp(sig, e12, e12), -one)
    assert np.array_equal(oracle.gp(sig, e1, e2), e12)
    assert np.array_equal(oracle.gp(sig, e2, e1), -e12)
