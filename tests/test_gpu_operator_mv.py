"""The reference's per-multivector float64 calls under their own names
(geo_operator_gp_f64 / _jvp / _vjp, geo_operator_apply_*_f64 and VJPs; reference
src/operator_kernel.c:191-334, 412-539), computed on the GPU by libgeo_b200.so.

Every output struct (dimension, signature, all 64 coefficient slots) must be
byte-identical to the reference's own CPU code (oracle/_ref, compiled from its
sources), including the reference's skips (a zero left coefficient of the
product, a zero input coefficient of apply) with non-finite values on the
other operand; where the reference build is absent the coefficients are
compared bit for bit with the oracle. Statuses follow the reference's rules and
precedence.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from geometricelementaryoperators_b200 import abi
from geometricelementaryoperators_b200.synthetic import splitmix_uniform
from tests.conftest import all_signatures

pytestmark = pytest.mark.gpu

OK, INVALID, UNSUPPORTED, BAD_PLAN = 0, 1, 2, 6


def mv(sig, coeffs=None) -> abi.MvF64:
    v = abi.MvF64()
    v.dimension = len(sig)
    for i, s in enumerate(sig):
        v.signature[i] = int(s)
    if coeffs is not None:
        for i, c in enumerate(coeffs):
            v.coefficients[i] = float(c)
    return v


def raw(v) -> bytes:
    return bytes(memoryview(v).cast("B"))


def operands(n, seed):
    """Four finite operands; the first has a zero and a -0.0 coefficient."""
    N = 1 << n
    vals = [splitmix_uniform(seed + k, (N,)) for k in range(4)]
    vals[0][0] = 0.0
    vals[0][N - 1] = -0.0
    return vals


def skip_operands(n, seed):
    """A left operand that is zero except on two blades and a right operand with
    an infinity: the reference skips the zero left coefficients, so only the
    outputs those two blades reach become infinite (no NaN is formed)."""
    N = 1 << n
    a = np.zeros(N)
    a[0] = 0.75
    a[N - 1] = -1.5
    b = splitmix_uniform(seed, (N,))
    b[N // 2] = np.inf
    return a, b


def ref_lib():
    """The reference's CPU code (oracle/_ref), with untyped pointer arguments for
    the per-multivector calls (this module passes abi.MvF64 structs)."""
    from oracle import oracle as orc

    if not orc.REF_SO.exists():
        return None
    L = ctypes.CDLL(str(orc.REF_SO))
    P, SZ = ctypes.c_void_p, ctypes.c_size_t
    for name, args in (("geo_operator_gp_f64", [P] * 3), ("geo_operator_gp_f64_jvp", [P] * 5),
                       ("geo_operator_gp_f64_vjp", [P] * 5), ("geo_operator_apply_f64", [P] * 3),
                       ("geo_operator_apply_parametric_f64", [P, P, SZ, P, P]),
                       ("geo_operator_apply_f64_vjp", [P] * 3),
                       ("geo_operator_apply_parametric_f64_vjp", [P, P, SZ, P, P, P, P, SZ])):
        fn = getattr(L, name)
        fn.argtypes, fn.restype = args, ctypes.c_int
    return L


def byref(v):
    return ctypes.addressof(v)


def test_products_match_reference_bytes(oracle):
    L, R = abi.lib(), ref_lib()
    for n, q, sig in all_signatures():
        N = 1 << n
        a, b, c, d = operands(n, 100 * n + q)
        A, Bv, C, D = mv(sig, a), mv(sig, b), mv(sig, c), mv(sig, d)
        got, want = abi.MvF64(), abi.MvF64()
        sa, sb = skip_operands(n, 50 * n + q)
        skip, skip_ref = abi.MvF64(), abi.MvF64()
        assert L.geo_operator_gp_f64(mv(sig, sa), mv(sig, sb), skip) == OK
        assert np.isinf(np.array(skip.coefficients[:N])).sum() == (2 if N > 1 else 1)
        assert not np.isnan(np.array(skip.coefficients[:N])).any()
        assert L.geo_operator_gp_f64(A, Bv, got) == OK
        gl, gr, wl, wr = abi.MvF64(), abi.MvF64(), abi.MvF64(), abi.MvF64()
        assert L.geo_operator_gp_f64_vjp(A, C, D, gl, gr) == OK
        jt, wj = abi.MvF64(), abi.MvF64()
        assert L.geo_operator_gp_f64_jvp(A, C, D, A, jt) == OK
        if R is not None:
            assert R.geo_operator_gp_f64(byref(A), byref(Bv), byref(want)) == OK
            assert raw(got) == raw(want), (n, q)
            ma, mb = mv(sig, sa), mv(sig, sb)
            assert R.geo_operator_gp_f64(byref(ma), byref(mb), byref(skip_ref)) == OK
            assert raw(skip) == raw(skip_ref), (n, q)
            assert R.geo_operator_gp_f64_vjp(byref(A), byref(C), byref(D), byref(wl), byref(wr)) == OK
            assert raw(gl) == raw(wl) and raw(gr) == raw(wr), (n, q)
            assert R.geo_operator_gp_f64_jvp(byref(A), byref(C), byref(D), byref(A), byref(wj)) == OK
            assert raw(jt) == raw(wj), (n, q)
        else:
            assert np.array_equal(np.array(got.coefficients[:N]), oracle.gp(sig, a, b), equal_nan=True)
        assert np.array_equal(np.array(got.coefficients[:N]), oracle.gp(sig, a, b), equal_nan=True)
        la, lb = oracle.gp_vjp(sig, a, c, d)
        assert np.array_equal(np.array(gl.coefficients[:N]), la) and np.array_equal(np.array(gr.coefficients[:N]), lb)
        assert np.array_equal(np.array(jt.coefficients[:N]), oracle.gp_jvp(sig, a, c, d, a))


def _plan(sig, side, blades, coeffs):
    plan = abi.OperatorPlanI32()
    terms = (abi.OperatorTermI32 * len(blades))(*[abi.OperatorTermI32(int(b), int(c)) for b, c in zip(blades, coeffs)])
    assert abi.lib().geo_operator_plan_sparse_i32(ctypes.byref(plan), len(sig), abi.sig_array(sig), side, terms,
                                                  len(blades)) == OK
    return plan


def test_apply_family_matches_reference_bytes(oracle):
    L, R = abi.lib(), ref_lib()
    rng = np.random.default_rng(5)
    for n, q, sig in all_signatures():
        N = 1 << n
        for side in (0, 1):
            for count in sorted({1, min(3, N), min(N, 40)}):
                blades = rng.permutation(N)[:count]
                coeffs = rng.integers(-5, 6, count)
                coeffs[coeffs == 0] = 7
                if count >= 3:
                    coeffs[2] = -2**31  # the reference's int product wraps for sign -1
                params = splitmix_uniform(900 + n + count, (count,))
                params[0] = np.inf  # reaches only outputs whose source coefficient is not zero
                plan = _plan(sig, side, blades, coeffs)
                x, cot, _, _ = operands(n, 300 * n + q + side)
                x[1 % N] = 0.0
                X, Cv = mv(sig, x), mv(sig, cot)
                outs = {k: abi.MvF64() for k in ("apply", "param", "vjp", "pvjp")}
                pc = np.zeros(count)
                pp = np.ascontiguousarray(params)
                assert L.geo_operator_apply_f64(plan, X, outs["apply"]) == OK
                assert L.geo_operator_apply_parametric_f64(plan, pp.ctypes.data_as(ctypes.c_void_p), count, X,
                                                           outs["param"]) == OK
                xf = mv(sig, splitmix_uniform(77 + n, (N,)))
                assert L.geo_operator_apply_f64_vjp(plan, Cv, outs["vjp"]) == OK
                pv = np.ascontiguousarray(np.where(np.isinf(pp), 0.5, pp))  # finite parameters for the VJP
                assert L.geo_operator_apply_parametric_f64_vjp(plan, pv.ctypes.data_as(ctypes.c_void_p), count, xf,
                                                               mv(sig, splitmix_uniform(78 + n, (N,))), outs["pvjp"],
                                                               pc.ctypes.data_as(ctypes.c_void_p), count) == OK
                if R is not None:
                    ref = {k: abi.MvF64() for k in outs}
                    rpc = np.zeros(count)
                    pb = byref(plan)
                    cf = mv(sig, splitmix_uniform(78 + n, (N,)))
                    assert R.geo_operator_apply_f64(pb, byref(X), byref(ref["apply"])) == OK
                    assert R.geo_operator_apply_parametric_f64(pb, pp.ctypes.data, count, byref(X),
                                                               byref(ref["param"])) == OK
                    assert R.geo_operator_apply_f64_vjp(pb, byref(Cv), byref(ref["vjp"])) == OK
                    assert R.geo_operator_apply_parametric_f64_vjp(pb, pv.ctypes.data, count, byref(xf), byref(cf),
                                                                   byref(ref["pvjp"]), rpc.ctypes.data, count) == OK
                    for k in outs:
                        assert raw(outs[k]) == raw(ref[k]), (n, q, side, count, k)
                    assert rpc.tobytes() == pc.tobytes()
                want = oracle.sparse_apply_vjp(sig, side, blades, coeffs, cot)
                assert np.array_equal(np.array(outs["vjp"].coefficients[:N]), want, equal_nan=True)


def test_status_rules():
    L = abi.lib()
    sig = [1, 1, -1]
    a, b, out, out2 = mv(sig, np.ones(8)), mv(sig, np.ones(8)), abi.MvF64(), abi.MvF64()
    assert L.geo_operator_gp_f64(None, b, out) == INVALID
    bad_dim = mv([1] * 6, np.ones(64))
    assert L.geo_operator_gp_f64(a, bad_dim, out) == UNSUPPORTED          # dimensions differ
    other = mv([1, 1, 1], np.ones(8))
    assert L.geo_operator_gp_f64(a, other, out) == INVALID                # metrics differ
    zero_dim = abi.MvF64()
    assert L.geo_operator_gp_f64(zero_dim, zero_dim, out) == UNSUPPORTED
    assert L.geo_operator_gp_f64_vjp(a, b, a, out, out) == INVALID         # aliased outputs
    assert L.geo_operator_gp_f64_jvp(a, b, other, a, out) == INVALID       # tangent metric
    plan = _plan(sig, 0, [1, 2], [3, -1])
    assert L.geo_operator_apply_f64(plan, other, out) == INVALID
    p = np.ones(2)
    assert L.geo_operator_apply_parametric_f64(plan, p.ctypes.data_as(ctypes.c_void_p), 1, a, out) == INVALID
    assert L.geo_operator_apply_parametric_f64_vjp(plan, p.ctypes.data_as(ctypes.c_void_p), 2, a, a, out,
                                                   p.ctypes.data_as(ctypes.c_void_p), 1) == INVALID
    broken = abi.OperatorPlanI32()
    ctypes.memmove(ctypes.byref(broken), ctypes.byref(plan), ctypes.sizeof(plan))
    broken.abi_version = 0
    assert L.geo_operator_apply_f64(broken, a, out) == BAD_PLAN
    ctypes.memmove(ctypes.byref(broken), ctypes.byref(plan), ctypes.sizeof(plan))
    broken.terms[1].coefficient = 0
    assert L.geo_operator_apply_f64_vjp(broken, a, out) == BAD_PLAN
    assert L.geo_operator_apply_f64(None, a, out) == INVALID
    # a failed call leaves the output untouched
    out2.coefficients[0] = 42.0
    assert L.geo_operator_gp_f64(a, other, out2) == INVALID and out2.coefficients[0] == 42.0
