"""GPU parity of the sparse fixed-multivector plans over a batch
(geo_b200_sparse_*) against the oracle (the reference's geo_operator_apply_f64,
_apply_parametric_f64 and their VJPs, src/operator_kernel.c:191-334), on both
kernel routes: the streaming per-term kernel (every n; fewer than 5 terms at
n = 5, 6) and the dense route on the representation kernels (5 terms or more
at n = 5, 6, 16-byte aligned rows).

Tolerance: |a-b| <= 1e-12 (1+|a|+|b|) per element; parameter cotangents are
batch sums and use the same bar.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from geometricelementaryoperators_b200 import abi, canonical_signature
from geometricelementaryoperators_b200.synthetic import splitmix_uniform
from tests.conftest import all_signatures, max_violation, tol_close
from tests.gpu_helpers import TOL, dev, host, ptr, stream, sync

pytestmark = pytest.mark.gpu
RIGHT, LEFT = 0, 1


def _plan(sig, side, blades, coeffs):
    L = abi.lib()
    plan = abi.OperatorPlanI32()
    k = len(blades)
    terms = (abi.OperatorTermI32 * k)(*[abi.OperatorTermI32(int(b), int(c)) for b, c in zip(blades, coeffs)])
    assert L.geo_operator_plan_sparse_i32(ctypes.byref(plan), len(sig), abi.sig_array(sig), side, terms, k) == 0
    return plan


def _terms(n, k, seed):
    rng = np.random.default_rng(seed)
    blades = rng.choice(1 << n, size=k, replace=False)
    coeffs = rng.integers(1, 5, size=k) * rng.choice([-1, 1], size=k)
    params = rng.uniform(-2, 2, k)
    return blades, coeffs, params


def _run_all(plan, dx, dc, dp, B, N, k):
    L = abi.lib()
    o1, o2, o3, o4 = (dev(np.full((B, N), 7.0)) for _ in range(4))
    pc = dev(np.zeros(k))
    assert L.geo_b200_sparse_apply_f64(ctypes.byref(plan), ptr(dx), ptr(o1), B, stream()) == 0
    assert L.geo_b200_sparse_apply_parametric_f64(ctypes.byref(plan), ptr(dp), ptr(dx), ptr(o2), B, stream()) == 0
    assert L.geo_b200_sparse_apply_vjp_f64(ctypes.byref(plan), ptr(dc), ptr(o3), B, stream()) == 0
    assert L.geo_b200_sparse_apply_parametric_vjp_f64(ctypes.byref(plan), ptr(dp), ptr(dx), ptr(dc), ptr(o4),
                                                      ptr(pc), B, stream()) == 0
    sync()
    return host(o1), host(o2), host(o3), host(o4), host(pc)


def _expect(oracle, sig, side, blades, coeffs, params, x, c):
    B = x.shape[0]
    e1 = np.stack([oracle.sparse_apply(sig, side, blades, coeffs, x[i]) for i in range(B)])
    e2 = np.stack([oracle.sparse_apply_parametric(sig, side, blades, params, x[i]) for i in range(B)])
    e3 = np.stack([oracle.sparse_apply_vjp(sig, side, blades, coeffs, c[i]) for i in range(B)])
    pv = [oracle.sparse_apply_parametric_vjp(sig, side, blades, params, x[i], c[i]) for i in range(B)]
    return e1, e2, e3, np.stack([u for u, _ in pv]), np.sum(np.stack([v for _, v in pv]), axis=0)


@pytest.mark.parametrize("k", [1, 2, 4, 5, 13])
def test_sparse_routes_all_signatures(oracle, k):
    """Every canonical signature, both sides, term counts on both sides of the
    route switch (5 terms), a batch that is not a multiple of any tile."""
    B = 133
    for n, q, sig in all_signatures(2, 6):
        N = 1 << n
        kk = min(k, N)
        blades, coeffs, params = _terms(n, kk, 97 * n + 7 * q + kk)
        x = splitmix_uniform(800 + n + q + kk, (B, N))
        c = splitmix_uniform(900 + n + q + kk, (B, N))
        dx, dc, dp = dev(x), dev(c), dev(params)
        for side in (RIGHT, LEFT):
            plan = _plan(sig, side, blades, coeffs)
            got = _run_all(plan, dx, dc, dp, B, N, kk)
            want = _expect(oracle, sig, side, blades, coeffs, params, x, c)
            for name, g, w in zip(("apply", "parametric", "vjp", "param_vjp_in", "param_vjp_params"), got, want):
                assert tol_close(g, w, TOL), (n, q, side, kk, name, max_violation(g, w, TOL))


@pytest.mark.parametrize("k", [1, 3, 32, 64])
def test_sparse_n6_unaligned_and_in_place(oracle, k):
    """8-byte aligned rows take the streaming kernel at any term count; outputs
    equal to inputs work in place on both routes."""
    sig = canonical_signature(6, 2)
    B, N = 201, 64
    blades, coeffs, params = _terms(6, k, 31 + k)
    x = splitmix_uniform(40 + k, (B, N))
    c = splitmix_uniform(50 + k, (B, N))
    L = abi.lib()
    for side in (RIGHT, LEFT):
        plan = _plan(sig, side, blades, coeffs)
        e1, e2, e3, e4, e5 = _expect(oracle, sig, side, blades, coeffs, params, x, c)
        big_x = dev(np.concatenate([[0.0], x.ravel()]))
        big_c = dev(np.concatenate([[0.0], c.ravel()]))
        out = dev(np.zeros(x.size + 1))
        xo, co, oo = (ctypes.c_void_p(t.data_ptr() + 8) for t in (big_x, big_c, out))
        dp = dev(params)
        pc = dev(np.zeros(k))
        assert L.geo_b200_sparse_apply_f64(ctypes.byref(plan), xo, oo, B, stream()) == 0
        sync()
        assert tol_close(host(out)[1:].reshape(B, N), e1, TOL)
        assert L.geo_b200_sparse_apply_vjp_f64(ctypes.byref(plan), co, oo, B, stream()) == 0
        sync()
        assert tol_close(host(out)[1:].reshape(B, N), e3, TOL)
        assert L.geo_b200_sparse_apply_parametric_vjp_f64(ctypes.byref(plan), ptr(dp), xo, co, oo, ptr(pc), B,
                                                          stream()) == 0
        sync()
        assert tol_close(host(out)[1:].reshape(B, N), e4, TOL) and tol_close(host(pc), e5, TOL)
        inplace = dev(x)
        assert L.geo_b200_sparse_apply_parametric_f64(ctypes.byref(plan), ptr(dp), ptr(inplace), ptr(inplace), B,
                                                      stream()) == 0
        sync()
        assert tol_close(host(inplace), e2, TOL)


def test_sparse_stream_non_finite_reaches_only_its_targets(oracle):
    """On the streaming route a non-finite input reaches exactly the outputs
    its terms reach, as in the reference's per-term loop."""
    sig = canonical_signature(6, 0)
    B, N = 8, 64
    blades, coeffs = [0b000011, 0b101000], [3, -2]
    x = splitmix_uniform(61, (B, N))
    x[2, 5] = np.inf
    x[6, 40] = np.nan
    plan = _plan(sig, RIGHT, blades, coeffs)
    y = dev(np.zeros((B, N)))
    assert abi.lib().geo_b200_sparse_apply_f64(ctypes.byref(plan), ptr(dev(x)), ptr(y), B, stream()) == 0
    sync()
    got = host(y)
    bad2 = {5 ^ b for b in blades}
    bad6 = {40 ^ b for b in blades}
    for r, bad in ((2, bad2), (6, bad6)):
        assert {o for o in range(N) if not np.isfinite(got[r, o])} == bad
    xf = x.copy()
    xf[2, 5] = xf[6, 40] = 0.0
    want = np.stack([oracle.sparse_apply(sig, RIGHT, blades, coeffs, xf[i]) for i in range(B)])
    mask = np.isfinite(got)
    assert tol_close(got[mask], want[mask], TOL)


@pytest.mark.parametrize("k", [1, 32])
def test_sparse_full_size(oracle, k):
    """2^22 + 3 rows of Cl(6,0) (the operator bench shape with a ragged tail):
    spot rows against the oracle, and the parameter cotangents are additive
    over a split of the batch."""
    import torch

    sig = canonical_signature(6, 0)
    B, N = (1 << 22) + 3, 64
    blades, coeffs, params = _terms(6, k, 500 + k)
    gen = torch.Generator(device="cuda").manual_seed(70 + k)
    X = torch.rand((B, N), dtype=torch.float64, device="cuda", generator=gen) * 2 - 1
    C = torch.rand((B, N), dtype=torch.float64, device="cuda", generator=gen) * 2 - 1
    Y = torch.empty_like(X)
    dp = dev(params)
    L = abi.lib()
    plan = _plan(sig, RIGHT, blades, coeffs)
    assert L.geo_b200_sparse_apply_f64(ctypes.byref(plan), ptr(X), ptr(Y), B, stream()) == 0
    sync()
    rows = np.concatenate([np.random.default_rng(k).integers(0, B, 256), np.arange(B - 20, B)])
    idx = torch.as_tensor(rows, device="cuda")
    xr, yr = host(X[idx]), host(Y[idx])
    want = np.stack([oracle.sparse_apply(sig, RIGHT, blades, coeffs, xr[i]) for i in range(len(rows))])
    assert tol_close(yr, want, TOL)
    pcs = [dev(np.zeros(k)) for _ in range(3)]
    half = B // 2 + 77
    for (xs, cs, b, pc) in ((X, C, B, pcs[0]), (X[:half], C[:half], half, pcs[1]), (X[half:], C[half:], B - half, pcs[2])):
        assert L.geo_b200_sparse_apply_parametric_vjp_f64(ctypes.byref(plan), ptr(dp), ptr(xs), ptr(cs), None,
                                                          ptr(pc), b, stream()) == 0
    sync()
    assert tol_close(host(pcs[0]), host(pcs[1]) + host(pcs[2]), TOL)
