"""GPU parity of pairwise products (both operands vary) and sparse plans."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from geometricelementaryoperators_b200 import abi, canonical_signature
from geometricelementaryoperators_b200.synthetic import normal, splitmix_uniform
from tests.conftest import all_signatures, max_violation, tol_close
from tests.gpu_helpers import TOL, TOL_F32, dev, host, ptr, stream, sync

pytestmark = pytest.mark.gpu


def test_pairwise_f64_all_signatures(oracle):
    L = abi.lib()
    B = 37
    for n, q, sig in all_signatures():
        N = 1 << n
        a, b, c, ta, tb = (splitmix_uniform(300 + 7 * n + q + k, (B, N)) for k in range(5))
        da, db, dc, dta, dtb = (dev(v) for v in (a, b, c, ta, tb))
        out, lb, rb, jt = (dev(np.zeros((B, N))) for _ in range(4))
        s = abi.sig_array(sig)
        assert L.geo_b200_pairwise_gp_f64(n, s, ptr(da), ptr(db), ptr(out), B, stream()) == 0
        assert L.geo_b200_pairwise_gp_vjp_f64(n, s, ptr(da), ptr(db), ptr(dc), ptr(lb), ptr(rb), B, stream()) == 0
        assert L.geo_b200_pairwise_gp_jvp_f64(n, s, ptr(da), ptr(db), ptr(dta), ptr(dtb), ptr(jt), B, stream()) == 0
        sync()
        want = np.stack([oracle.gp(sig, a[i], b[i]) for i in range(B)])
        assert tol_close(host(out), want, TOL), max_violation(host(out), want, TOL)
        vj = [oracle.gp_vjp(sig, a[i], b[i], c[i]) for i in range(B)]
        assert tol_close(host(lb), np.stack([u for u, _ in vj]), TOL)
        assert tol_close(host(rb), np.stack([v for _, v in vj]), TOL)
        jv = np.stack([oracle.gp_jvp(sig, a[i], b[i], ta[i], tb[i]) for i in range(B)])
        assert tol_close(host(jt), jv, TOL)


def test_pairwise_f64_n6_tma_path(oracle):
    """n = 6 float64 forward on the TMA kernel (16-byte aligned operands): every
    canonical signature plus non-canonical ones (the kernel is specialised on the
    metric of axes 0..3), a batch ending inside a 32-row tile (rows past it stay
    untouched), and the 8-byte aligned fallback."""
    import torch

    L = abi.lib()
    B = 1000 + 17
    sigs = [canonical_signature(6, q) for q in range(7)] + [[-1, 1, -1, 1, 1, -1], [1, -1, 1, 1, -1, 1]]
    for k, sig in enumerate(sigs):
        a, b = splitmix_uniform(710 + k, (B, 64)), splitmix_uniform(720 + k, (B, 64))
        da, db = dev(a), dev(b)
        out = torch.full((B + 40, 64), 7.0, dtype=torch.float64, device="cuda")
        assert L.geo_b200_pairwise_gp_f64(6, abi.sig_array(sig), ptr(da), ptr(db), ptr(out), B, stream()) == 0
        sync()
        want = np.stack([oracle.gp(sig, a[i], b[i]) for i in range(B)])
        got = host(out)
        assert tol_close(got[:B], want, TOL), (sig, max_violation(got[:B], want, TOL))
        assert np.all(got[B:] == 7.0)
        # VJP: two forward products with sign-flipped operands; each output on its own too.
        c = splitmix_uniform(730 + k, (B, 64))
        vj = [oracle.gp_vjp(sig, a[i], b[i], c[i]) for i in range(B)]
        want_l, want_r = np.stack([u for u, _ in vj]), np.stack([v for _, v in vj])
        dc = dev(c)
        for which in ("both", "left", "right"):
            lb = dev(np.zeros((B, 64))) if which != "right" else None
            rb = dev(np.zeros((B, 64))) if which != "left" else None
            assert L.geo_b200_pairwise_gp_vjp_f64(6, abi.sig_array(sig), ptr(da), ptr(db), ptr(dc),
                                                  ptr(lb) if lb is not None else None,
                                                  ptr(rb) if rb is not None else None, B, stream()) == 0
            sync()
            if lb is not None:
                assert tol_close(host(lb), want_l, TOL), (sig, which, max_violation(host(lb), want_l, TOL))
            if rb is not None:
                assert tol_close(host(rb), want_r, TOL), (sig, which, max_violation(host(rb), want_r, TOL))
        # JVP: a_dot b + a b_dot in one pass (the ring alternates the two operand pairs of each tile);
        # rows past the batch untouched.
        ta, tb = splitmix_uniform(740 + k, (B, 64)), splitmix_uniform(750 + k, (B, 64))
        jt = torch.full((B + 40, 64), 7.0, dtype=torch.float64, device="cuda")
        assert L.geo_b200_pairwise_gp_jvp_f64(6, abi.sig_array(sig), ptr(da), ptr(db), ptr(dev(ta)), ptr(dev(tb)),
                                              ptr(jt), B, stream()) == 0
        sync()
        want_j = np.stack([oracle.gp_jvp(sig, a[i], b[i], ta[i], tb[i]) for i in range(B)])
        got_j = host(jt)
        assert tol_close(got_j[:B], want_j, TOL), (sig, max_violation(got_j[:B], want_j, TOL))
        assert np.all(got_j[B:] == 7.0)
        if k in (0, 3):
            big = dev(np.concatenate([[0.0], a.ravel()]))
            o8 = dev(np.zeros(a.size + 1))
            assert L.geo_b200_pairwise_gp_f64(6, abi.sig_array(sig), ctypes.c_void_p(big.data_ptr() + 8), ptr(db),
                                              ctypes.c_void_p(o8.data_ptr() + 8), B, stream()) == 0
            sync()
            assert tol_close(host(o8)[1:].reshape(B, 64), want, TOL)


def test_pairwise_f64_full_size_spot_rows(oracle):
    """2^22 + 9 pairs of Cl(6,0) (the operator bench shape with a ragged tail): spot rows,
    first and last tiles included."""
    import torch

    L = abi.lib()
    sig = canonical_signature(6, 0)
    B = (1 << 22) + 9
    gen = torch.Generator(device="cuda").manual_seed(8)
    da = torch.rand((B, 64), dtype=torch.float64, device="cuda", generator=gen).mul_(2).sub_(1)
    db = torch.rand((B, 64), dtype=torch.float64, device="cuda", generator=gen).mul_(2).sub_(1)
    out = torch.empty_like(da)
    assert L.geo_b200_pairwise_gp_f64(6, abi.sig_array(sig), ptr(da), ptr(db), ptr(out), B, stream()) == 0
    sync()
    rows = np.unique(np.concatenate([np.arange(40), np.arange(B - 40, B),
                                     np.random.default_rng(4).integers(0, B, 300)]))
    idx = torch.as_tensor(rows, device="cuda")
    a, b, got = host(da[idx]), host(db[idx]), host(out[idx])
    want = np.stack([oracle.gp(sig, a[i], b[i]) for i in range(len(rows))])
    assert tol_close(got, want, TOL), max_violation(got, want, TOL)


@pytest.mark.parametrize("q", [0, 3, 6])
@pytest.mark.parametrize("compact", [0, 1])
def test_pairwise_f32_even_operand(oracle, compact, q):
    """Cl(6-q,q) float32 build: even-grade left operand (32 blades, N(0,1)), dense right U[-1,1];
    float64 oracle at 1e-5. The batch ends inside a 64-row tile; rows past it stay untouched."""
    import torch

    L = abi.lib()
    sig = canonical_signature(6, q)
    B = 3001
    even = np.array([b for b in range(64) if bin(b).count("1") % 2 == 0])
    a = np.zeros((B, 64))
    a[:, even] = normal(61 + q, (B, 32))
    b = splitmix_uniform(62 + q, (B, 64))
    a32 = a.astype(np.float32)
    b32 = b.astype(np.float32)
    left = a32[:, even] if compact else a32
    dl = torch.from_numpy(np.ascontiguousarray(left)).cuda()
    dr = torch.from_numpy(b32).cuda()
    out = torch.full((B + 64, 64), 7.0, dtype=torch.float32, device="cuda")
    assert L.geo_b200_pairwise_gp_f32(6, abi.sig_array(sig), ptr(dl), compact, ptr(dr), ptr(out), B, stream()) == 0
    sync()
    want = np.stack([oracle.gp(sig, a32[i].astype(np.float64), b32[i].astype(np.float64)) for i in range(B)])
    got = host(out).astype(np.float64)
    assert tol_close(got[:B], want, TOL_F32), max_violation(got[:B], want, TOL_F32)
    assert np.all(got[B:] == 7.0)


def test_pairwise_f32_full_size_spot_rows(oracle):
    """Float32 sweep shape (compact even left, 2^22 + 5 pairs): spot rows, first and last tiles included."""
    import torch

    L = abi.lib()
    sig = canonical_signature(6, 0)
    B = (1 << 22) + 5
    gen = torch.Generator(device="cuda").manual_seed(5)
    dl = torch.randn((B, 32), dtype=torch.float32, device="cuda", generator=gen)
    dr = torch.rand((B, 64), dtype=torch.float32, device="cuda", generator=gen).mul_(2).sub_(1)
    out = torch.full((B + 3, 64), 7.0, dtype=torch.float32, device="cuda")
    assert L.geo_b200_pairwise_gp_f32(6, abi.sig_array(sig), ptr(dl), 1, ptr(dr), ptr(out), B, stream()) == 0
    sync()
    rows = np.unique(np.concatenate([np.arange(70), np.arange(B - 70, B),
                                     np.random.default_rng(3).integers(0, B, 500)]))
    even = np.array([b for b in range(64) if bin(b).count("1") % 2 == 0])
    al = host(dl[rows]).astype(np.float64)
    br = host(dr[rows]).astype(np.float64)
    got = host(out[rows]).astype(np.float64)
    for i in range(len(rows)):
        a = np.zeros(64)
        a[even] = al[i]
        want = oracle.gp(sig, a, br[i])
        assert tol_close(got[i], want, TOL_F32), (rows[i], max_violation(got[i], want, TOL_F32))
    assert np.all(host(out[B:]) == 7.0)


def test_sparse_plans(oracle):
    L = abi.lib()
    B = 129
    for n, q, sig in all_signatures(2, 6):
        N = 1 << n
        rng = np.random.default_rng(n * 10 + q)
        k = min(N, 6)
        blades = rng.choice(N, size=k, replace=False)
        coeffs = rng.integers(1, 4, size=k) * rng.choice([-1, 1], size=k)
        params = rng.uniform(-2, 2, k)
        x = splitmix_uniform(500 + n + q, (B, N))
        c = splitmix_uniform(600 + n + q, (B, N))
        dx, dc, dp = dev(x), dev(c), dev(params)
        for side in (0, 1):
            plan = abi.OperatorPlanI32()
            terms = (abi.OperatorTermI32 * k)(*[abi.OperatorTermI32(int(b), int(cf)) for b, cf in zip(blades, coeffs)])
            assert L.geo_operator_plan_sparse_i32(ctypes.byref(plan), n, abi.sig_array(sig), side, terms, k) == 0
            o1, o2, o3, o4 = (dev(np.zeros((B, N))) for _ in range(4))
            pc = dev(np.zeros(k))
            assert L.geo_b200_sparse_apply_f64(ctypes.byref(plan), ptr(dx), ptr(o1), B, stream()) == 0
            assert L.geo_b200_sparse_apply_parametric_f64(ctypes.byref(plan), ptr(dp), ptr(dx), ptr(o2), B,
                                                          stream()) == 0
            assert L.geo_b200_sparse_apply_vjp_f64(ctypes.byref(plan), ptr(dc), ptr(o3), B, stream()) == 0
            assert L.geo_b200_sparse_apply_parametric_vjp_f64(ctypes.byref(plan), ptr(dp), ptr(dx), ptr(dc), ptr(o4),
                                                              ptr(pc), B, stream()) == 0
            sync()
            assert tol_close(host(o1), np.stack([oracle.sparse_apply(sig, side, blades, coeffs, x[i])
                                                 for i in range(B)]), TOL)
            assert tol_close(host(o2), np.stack([oracle.sparse_apply_parametric(sig, side, blades, params, x[i])
                                                 for i in range(B)]), TOL)
            assert tol_close(host(o3), np.stack([oracle.sparse_apply_vjp(sig, side, blades, coeffs, c[i])
                                                 for i in range(B)]), TOL)
            pv = [oracle.sparse_apply_parametric_vjp(sig, side, blades, params, x[i], c[i]) for i in range(B)]
            assert tol_close(host(o4), np.stack([u for u, _ in pv]), TOL)
            assert tol_close(host(pc), np.sum(np.stack([v for _, v in pv]), axis=0), TOL)


@pytest.mark.parametrize("precision", [64, 32])
def test_tma_wait_gives_up_with_status(precision, oracle):
    """A bounded wait of the TMA pairwise kernels that runs out is reported: the
    self-test launches the kernel with no load issued (nothing in flight), so
    every CTA's first wait gives up after a few polls; the call returns
    GEO_B200_TIMEOUT, every output row holds NaN, and the context stays usable
    (a normal product right after matches the oracle)."""
    import torch

    L = abi.lib()
    B = 1000 + 17
    dtype = torch.float64 if precision == 64 else torch.float32
    out = torch.zeros((B, 64), dtype=dtype, device="cuda")
    count = ctypes.c_uint(0)
    assert L.geo_b200_pairwise_wait_failures(ctypes.byref(count), 1) in (0, 7)
    st = L.geo_b200_pairwise_wait_selftest(precision, ptr(out), B, 64, stream())
    assert st == 7, abi.lib().geo_b200_status_string(st)  # GEO_B200_TIMEOUT
    assert bool(torch.isnan(out).all())
    assert L.geo_b200_pairwise_wait_failures(ctypes.byref(count), 1) == 0 and count.value == 0
    sig = canonical_signature(6, 0)
    a, b = splitmix_uniform(901, (B, 64)), splitmix_uniform(902, (B, 64))
    s = abi.sig_array(sig)
    if precision == 64:
        da, db = dev(a), dev(b)
        assert L.geo_b200_pairwise_gp_f64(6, s, ptr(da), ptr(db), ptr(out), B, stream()) == 0
        sync()
        want = np.stack([oracle.gp(sig, a[i], b[i]) for i in range(B)])
        assert tol_close(host(out), want, TOL)
    else:
        da, db = dev(a.astype(np.float32)), dev(b.astype(np.float32))
        assert L.geo_b200_pairwise_gp_f32(6, s, ptr(da), 0, ptr(db), ptr(out), B, stream()) == 0
        sync()
        want = np.stack([oracle.gp(sig, a[i].astype(np.float32).astype(np.float64),
                                   b[i].astype(np.float32).astype(np.float64)) for i in range(B)])
        assert tol_close(host(out).astype(np.float64), want, TOL_F32)
    assert L.geo_b200_pairwise_wait_failures(ctypes.byref(count), 0) == 0 and count.value == 0
