"""Pin the CPU oracle against the reference compiled from its own sources.

The oracle (oracle/geo_oracle.c) restates the reference CPU algorithm; here it
must agree with oracle/_ref (reference src/batch_gp.c, src/operator_kernel.c,
src/full_cycle_v8.c built unmodified) BIT FOR BIT on every canonical
signature, both sides and several batch sizes, including the status codes of
the edge cases the reference tests exercise. The product's host-side plan
logic (geo_batch_gp_plan_init, geo_operator_gp_sign, sparse plan builders in
libgeo_b200.so, no GPU needed) is checked the same way.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from geometricelementaryoperators_b200 import abi, canonical_signature
from geometricelementaryoperators_b200.synthetic import splitmix_uniform
from tests.conftest import all_signatures


def _data(n: int, batch: int, seed: int):
    N = 1 << n
    x = splitmix_uniform(seed, (batch, N))
    w = splitmix_uniform(seed + 1, (N,))
    t = splitmix_uniform(seed + 2, (batch, N))
    return x, w, t


def test_sign_table_exhaustive(oracle, reference):
    """Every (left, right) pair of every signature of dimension 1..6 (also non-canonical)."""
    lib = abi.lib()
    rng = np.random.default_rng(7)
    sigs = [s for _, _, s in all_signatures()]
    sigs += [list(rng.choice([-1, 1], size=n)) for n in range(1, 7) for _ in range(4)]
    for sig in sigs:
        n = len(sig)
        arr = abi.sig_array(sig)
        for l in range(1 << n):
            for r in range(1 << n):
                s_ref = reference.sign(l, r, sig)
                assert oracle.sign(l, r, sig) == s_ref
                assert lib.geo_operator_gp_sign(l, r, arr, n) == s_ref
    # invalid signatures give 0 (reference src/operator_kernel.c:119)
    assert lib.geo_operator_gp_sign(1, 1, abi.sig_array([1, 0]), 2) == 0
    assert reference.sign(1, 1, [1, 0]) == 0


def test_plan_bytes_identical(oracle, reference):
    """geo_batch_gp_plan_init of the product == reference, byte for byte."""
    lib = abi.lib()
    for n, q, sig in all_signatures():
        plan = abi.BatchGpPlan()
        assert lib.geo_batch_gp_plan_init(ctypes.byref(plan), n, abi.sig_array(sig)) == 0
        mine = bytes(ctypes.string_at(ctypes.addressof(plan), ctypes.sizeof(plan)))
        assert mine == bytes(reference.plan(sig))
        assert mine == bytes(oracle.plan(sig))
    plan = abi.BatchGpPlan()
    assert lib.geo_batch_gp_plan_init(ctypes.byref(plan), 0, abi.sig_array([1])) == 2
    assert lib.geo_batch_gp_plan_init(ctypes.byref(plan), 7, abi.sig_array([1] * 6)) == 2
    assert lib.geo_batch_gp_plan_init(ctypes.byref(plan), 2, abi.sig_array([1, 2])) == 1
    assert lib.geo_batch_gp_plan_init(None, 2, abi.sig_array([1, 1])) == 1


@pytest.mark.parametrize("batch", [1, 3, 8, 17])
def test_batch_paths_bit_exact(oracle, reference, batch):
    for n, q, sig in all_signatures():
        x, w, t = _data(n, batch, 100 * n + 10 * q + batch)
        for left in (False, True):
            st_o, y_o = oracle.forward(sig, x, w, left)
            st_r, y_r = reference.forward(sig, x, w, left)
            assert st_o == st_r == 0 and np.array_equal(y_o, y_r)
            st_o, g_o = oracle.vjp(sig, x, t, left)
            st_r, g_r = reference.vjp(sig, x, t, left)
            assert st_o == st_r == 0 and np.array_equal(g_o, g_r)
            st_o, w_o, l_o = oracle.sgd_step(sig, x, t, 0.01, w, left)
            st_r, w_r, l_r = reference.sgd_step(sig, x, t, 0.01, w, left)
            assert st_o == st_r == 0 and np.array_equal(w_o, w_r) and l_o == l_r


def test_batch_status_edges(oracle, reference):
    sig = canonical_signature(3, 1)
    x, w, t = _data(3, 4, 5)
    bad = x.copy()
    bad[2, 3] = np.nan
    for impl in (oracle, reference):
        assert impl.forward(sig, bad, w, False)[0] == 1
        assert impl.vjp(sig, x, np.where(np.isfinite(bad), t, np.inf), True)[0] == 1
        assert impl.sgd_step(sig, x, t, 0.0, w, False)[0] == 1
        assert impl.sgd_step(sig, x, t, -1.0, w, False)[0] == 1
        huge = np.full_like(x, 1e200)
        st, _ = impl.forward(sig, huge, np.full(8, 1e200), False)
        assert st == 3  # overflow -> NUMERIC_FAILURE
    # targets = outputs -> loss 0 and parameter unchanged (reference tests/test_batch_gp.c:83-98)
    for left in (False, True):
        y = oracle.forward(sig, x, w, left)[1]
        st, w2, loss = oracle.sgd_step(sig, x, y, 0.01, w, left)
        assert st == 0 and loss == 0.0 and np.array_equal(w2, w)


def test_operator_paths_bit_exact(oracle, reference):
    rng = np.random.default_rng(3)
    for n, q, sig in all_signatures():
        N = 1 << n
        a, b, c, ta, tb = (rng.uniform(-1, 1, N) for _ in range(5))
        a[rng.integers(0, N)] = 0.0  # exercise the zero-left skip
        assert np.array_equal(oracle.gp(sig, a, b), reference.gp(sig, a, b))
        for u, v in zip(oracle.gp_vjp(sig, a, b, c), reference.gp_vjp(sig, a, b, c)):
            assert np.array_equal(u, v)
        assert np.array_equal(oracle.gp_jvp(sig, a, b, ta, tb), reference.gp_jvp(sig, a, b, ta, tb))
        for side in (0, 1):
            k = min(N, 5)
            blades = rng.choice(N, size=k, replace=False)
            coeffs = rng.integers(1, 4, size=k) * rng.choice([-1, 1], size=k)
            params = rng.uniform(-2, 2, k)
            assert np.array_equal(oracle.sparse_apply(sig, side, blades, coeffs, a),
                                  reference.sparse_apply(sig, side, blades, coeffs, a))
            assert np.array_equal(oracle.sparse_apply_parametric(sig, side, blades, params, a),
                                  reference.sparse_apply_parametric(sig, side, blades, params, a))
            assert np.array_equal(oracle.sparse_apply_vjp(sig, side, blades, coeffs, c),
                                  reference.sparse_apply_vjp(sig, side, blades, coeffs, c))
            for u, v in zip(oracle.sparse_apply_parametric_vjp(sig, side, blades, params, a, c),
                            reference.sparse_apply_parametric_vjp(sig, side, blades, params, a, c)):
                assert np.array_equal(u, v)


def test_sparse_plan_builder_matches_reference(reference):
    lib = abi.lib()
    for n, q, sig in all_signatures(2, 6):
        N = 1 << n
        terms = [(0, 1), (1, -2), (N - 1, 1)]
        for side in (0, 1):
            mine = abi.OperatorPlanI32()
            arr = (abi.OperatorTermI32 * 3)(*[abi.OperatorTermI32(b, c) for b, c in terms])
            st = lib.geo_operator_plan_sparse_i32(ctypes.byref(mine), n, abi.sig_array(sig), side, arr, 3)
            st_r, ref = reference.sparse_plan(sig, side, [b for b, _ in terms], [c for _, c in terms])
            assert st == st_r == 0
            assert bytes(ctypes.string_at(ctypes.addressof(mine), ctypes.sizeof(mine))) == bytes(ref)
    # duplicate blades and zero coefficients are rejected, plan zeroed
    mine = abi.OperatorPlanI32()
    dup = (abi.OperatorTermI32 * 2)(abi.OperatorTermI32(1, 1), abi.OperatorTermI32(1, 2))
    assert lib.geo_operator_plan_sparse_i32(ctypes.byref(mine), 2, abi.sig_array([1, 1]), 0, dup, 2) == 1
    assert lib.geo_operator_plan_sparse_i32(ctypes.byref(mine), 2, abi.sig_array([1, 1]), 0, dup, 0) == 3


@pytest.mark.parametrize("optimizer", [1, 2])
@pytest.mark.parametrize("left", [False, True])
def test_v8_optimizer_composite_bit_exact(oracle, reference, optimizer, left):
    """Oracle composite (per-sample GP VJP summed in sample order + V8 update)
    == the reference per-sample V8 loop, bit for bit, over several steps."""
    for n, q in [(2, 0), (3, 1), (5, 1), (6, 3)]:
        sig = canonical_signature(n, q)
        N = 1 << n
        batch = 3
        xs = splitmix_uniform(11 + n, (batch, N))
        ts = splitmix_uniform(12 + n, (batch, N))
        w0 = splitmix_uniform(13 + n, (N,))
        lr, b1, b2, eps = 1e-2, 0.9, 0.999, 1e-8
        params_ref, losses_ref = reference.v8_train(sig, left, xs, ts, w0, optimizer, lr, b1, b2, eps, steps=3)
        w, m, v = w0.copy(), np.zeros(N), np.zeros(N)
        for step in range(1, 4):
            gsum = np.zeros(N)
            for j in range(batch):
                a, b = (w, xs[j]) if left else (xs[j], w)
                y = oracle.gp(sig, a, b)
                r = y + (-1.0 * ts[j])
                la, rb = oracle.gp_vjp(sig, a, b, r)
                gsum = gsum + (la if left else rb) * 1.0
            st, w, m, v = oracle.v8_update(optimizer, lr, b1, b2, eps, 1.0 / batch, step, gsum, w, m, v)
            assert st == 0
            assert np.array_equal(w, params_ref[step - 1]), (n, q, step)
