"""GPU parity of the batch_gp paths (device ABI, host ABI, hand control)
against the CPU oracle, the committed golden vectors, and full-size properties.

Tolerance: float64 results within |a-b| <= 1e-12 (1+|a|+|b|) of the oracle
(the float64 parity bar; the reference's own CUDA test uses 1e-10,
tests/test_batch_gp_cuda.cu:35). Routing and signs are bit-exact (test_oracle).
"""
from __future__ import annotations

import ctypes
import pathlib

import numpy as np
import pytest

from geometricelementaryoperators_b200 import abi, canonical_signature
from geometricelementaryoperators_b200.synthetic import splitmix_uniform
from tests.conftest import all_signatures, max_violation, tol_close
from tests.gpu_helpers import TOL, CudaPlan, dev, host, make_plan, np_ptr, ptr, stream, sync

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "batch_gp_golden.npz"
BATCHES = [1, 3, 16, 64, 256, 1000, 1024]  # 1024: the Cl(2,0) inference shape


def _lib():
    return abi.lib()


def _case(n, batch, seed):
    N = 1 << n
    return (splitmix_uniform(seed, (batch, N)), splitmix_uniform(seed + 1, (N,)),
            splitmix_uniform(seed + 2, (batch, N)))


@pytest.mark.parametrize("batch", BATCHES)
def test_device_api_all_signatures(oracle, batch):
    L = _lib()
    for n, q, sig in all_signatures():
        plan = CudaPlan(sig)
        x, w, t = _case(n, batch, 31 * n + q + batch)
        dx, dw, dt = dev(x), dev(w), dev(t)
        for left in (0, 1):
            y_ref = oracle.forward(sig, x, w, bool(left))[1]
            g_ref = oracle.vjp(sig, x, t, bool(left))[1]
            st, w_ref, mean_loss = oracle.sgd_step(sig, x, t, 1e-3, w, bool(left))
            assert st == 0
            out = dev(np.zeros_like(x))
            for fn in (L.geo_batch_gp_cuda_reference_forward_f64, L.geo_batch_gp_cuda_planned_forward_f64,
                       L.geo_hand_cuda_forward_f64):
                out.zero_()
                assert fn(ctypes.byref(plan.dev), ptr(dx), batch, ptr(dw), left, ptr(out), stream()) == 0
                sync()
                assert tol_close(host(out), y_ref, TOL), (n, q, left, max_violation(host(out), y_ref, TOL))
            grad = dev(np.zeros(1 << n))
            for fn in (L.geo_batch_gp_cuda_reference_parameter_vjp_f64, L.geo_batch_gp_cuda_parameter_vjp_f64,
                       L.geo_hand_cuda_parameter_vjp_f64):
                grad.zero_()
                assert fn(ctypes.byref(plan.dev), ptr(dx), ptr(dt), batch, left, ptr(grad), stream()) == 0
                sync()
                assert tol_close(host(grad), g_ref, TOL), (n, q, left, max_violation(host(grad), g_ref, TOL))
            for fn in (L.geo_batch_gp_cuda_reference_mse_sgd_step_f64, L.geo_batch_gp_cuda_mse_sgd_step_f64,
                       L.geo_hand_cuda_mse_sgd_step_f64):
                dparam = dev(w.copy())
                res = dev(np.zeros_like(x))
                dgrad = dev(np.zeros(1 << n))
                dloss = dev(np.zeros(1))
                assert fn(ctypes.byref(plan.dev), ptr(dx), ptr(dt), batch, 1e-3, left, ptr(dparam), ptr(res),
                          ptr(dgrad), ptr(dloss), stream()) == 0
                sync()
                # residuals, gradient of the residual loss, loss SUM, updated parameter
                r_ref = y_ref - t
                assert tol_close(host(res), r_ref, TOL)
                g_r = oracle.vjp(sig, x, r_ref, bool(left))[1]
                assert tol_close(host(dgrad), g_r, TOL)
                assert tol_close(host(dloss)[0] / batch, mean_loss, TOL)
                assert tol_close(host(dparam), w_ref, TOL), (n, q, left, max_violation(host(dparam), w_ref, TOL))


def test_host_api_all_signatures(oracle):
    L = _lib()
    for n, q, sig in all_signatures():
        plan = make_plan(sig)
        for batch in (1, 7, 300):
            x, w, t = _case(n, batch, 77 * n + q + batch)
            for left in (False, True):
                out = np.zeros_like(x)
                if left:
                    st = L.geo_batch_gp_left_forward_f64(ctypes.byref(plan), np_ptr(w), np_ptr(x), batch, np_ptr(out))
                else:
                    st = L.geo_batch_gp_right_forward_f64(ctypes.byref(plan), np_ptr(x), batch, np_ptr(w), np_ptr(out))
                assert st == 0
                assert tol_close(out, oracle.forward(sig, x, w, left)[1], TOL)
                g = np.zeros(1 << n)
                fn = L.geo_batch_gp_left_vjp_parameter_f64 if left else L.geo_batch_gp_right_vjp_parameter_f64
                assert fn(ctypes.byref(plan), np_ptr(x), np_ptr(t), batch, np_ptr(g)) == 0
                assert tol_close(g, oracle.vjp(sig, x, t, left)[1], TOL)
                w2 = w.copy()
                loss = ctypes.c_double(-1.0)
                fn = L.geo_batch_gp_left_mse_sgd_step_f64 if left else L.geo_batch_gp_right_mse_sgd_step_f64
                assert fn(ctypes.byref(plan), np_ptr(x), np_ptr(t), batch, 0.01, np_ptr(w2), ctypes.byref(loss)) == 0
                st, w_ref, l_ref = oracle.sgd_step(sig, x, t, 0.01, w, left)
                assert tol_close(w2, w_ref, TOL) and tol_close(loss.value, l_ref, TOL)


def test_host_api_golden():
    """The GPU reproduces the reference's own outputs (golden vectors) at 1e-12."""
    L = _lib()
    golden = np.load(GOLDEN)
    for n, q, sig in all_signatures():
        key = f"n{n}q{q}"
        plan = make_plan(sig)
        x, w, t = golden[f"{key}_x"], golden[f"{key}_w"], golden[f"{key}_t"]
        B = x.shape[0]
        for side, left in (("R", False), ("L", True)):
            out = np.zeros_like(x)
            if left:
                assert L.geo_batch_gp_left_forward_f64(ctypes.byref(plan), np_ptr(w), np_ptr(x), B, np_ptr(out)) == 0
            else:
                assert L.geo_batch_gp_right_forward_f64(ctypes.byref(plan), np_ptr(x), B, np_ptr(w), np_ptr(out)) == 0
            assert tol_close(out, golden[f"{key}{side}_y"], TOL)
            g = np.zeros(1 << n)
            fn = L.geo_batch_gp_left_vjp_parameter_f64 if left else L.geo_batch_gp_right_vjp_parameter_f64
            assert fn(ctypes.byref(plan), np_ptr(x), np_ptr(t), B, np_ptr(g)) == 0
            assert tol_close(g, golden[f"{key}{side}_g"], TOL)
            w2 = w.copy()
            loss = ctypes.c_double()
            fn = L.geo_batch_gp_left_mse_sgd_step_f64 if left else L.geo_batch_gp_right_mse_sgd_step_f64
            assert fn(ctypes.byref(plan), np_ptr(x), np_ptr(t), B, 0.01, np_ptr(w2), ctypes.byref(loss)) == 0
            assert tol_close(w2, golden[f"{key}{side}_sgd_w"], TOL)
            assert tol_close(loss.value, golden[f"{key}{side}_sgd_loss"][0], TOL)


def test_host_api_status_edges(oracle):
    """Same status codes as the reference on non-finite and invalid inputs."""
    L = _lib()
    sig = canonical_signature(4, 1)
    plan = make_plan(sig)
    x, w, t = _case(4, 33, 5)
    out = np.full_like(x, 7.0)
    bad = x.copy()
    bad[5, 3] = np.nan
    # non-finite input -> INVALID_ARGUMENT, outputs untouched
    assert L.geo_batch_gp_right_forward_f64(ctypes.byref(plan), np_ptr(bad), 33, np_ptr(w), np_ptr(out)) == 1
    assert np.all(out == 7.0)
    wbad = w.copy()
    wbad[2] = np.inf
    assert L.geo_batch_gp_left_forward_f64(ctypes.byref(plan), np_ptr(wbad), np_ptr(x), 33, np_ptr(out)) == 1
    # overflow -> NUMERIC_FAILURE with outputs written
    huge = np.full_like(x, 1e200)
    assert L.geo_batch_gp_right_forward_f64(ctypes.byref(plan), np_ptr(huge), 33, np_ptr(np.full(16, 1e200)),
                                            np_ptr(out)) == 3
    assert not np.all(np.isfinite(out))
    # batch 0 / null pointers / bad lr
    assert L.geo_batch_gp_right_forward_f64(ctypes.byref(plan), np_ptr(x), 0, np_ptr(w), np_ptr(out)) == 1
    g = np.zeros(16)
    tbad = t.copy()
    tbad[0, 0] = np.inf
    assert L.geo_batch_gp_right_vjp_parameter_f64(ctypes.byref(plan), np_ptr(x), np_ptr(tbad), 33, np_ptr(g)) == 1
    w2 = w.copy()
    loss = ctypes.c_double(5.0)
    for lr in (0.0, -1.0, float("nan")):
        assert L.geo_batch_gp_right_mse_sgd_step_f64(ctypes.byref(plan), np_ptr(x), np_ptr(t), 33, lr, np_ptr(w2),
                                                     ctypes.byref(loss)) == 1
    # non-finite target -> INVALID_ARGUMENT, parameter unchanged
    assert L.geo_batch_gp_right_mse_sgd_step_f64(ctypes.byref(plan), np_ptr(x), np_ptr(tbad), 33, 0.01, np_ptr(w2),
                                                 ctypes.byref(loss)) == 1
    assert np.array_equal(w2, w)
    # candidate overflow -> NUMERIC_FAILURE, parameter unchanged (transactional)
    big_t = np.full_like(x, -1e300)
    st_ref, _, _ = oracle.sgd_step(sig, x, big_t, 1e10, w, False)
    st = L.geo_batch_gp_right_mse_sgd_step_f64(ctypes.byref(plan), np_ptr(x), np_ptr(big_t), 33, 1e10, np_ptr(w2),
                                               ctypes.byref(loss))
    assert st == st_ref
    if st != 0:
        assert np.array_equal(w2, w)
    # fixed point: targets = outputs -> loss 0, parameter unchanged
    y = np.zeros_like(x)
    assert L.geo_batch_gp_right_forward_f64(ctypes.byref(plan), np_ptr(x), 33, np_ptr(w), np_ptr(y)) == 0
    w3 = w.copy()
    assert L.geo_batch_gp_right_mse_sgd_step_f64(ctypes.byref(plan), np_ptr(x), np_ptr(y), 33, 0.01, np_ptr(w3),
                                                 ctypes.byref(loss)) == 0
    assert loss.value == 0.0 and np.array_equal(w3, w)


def test_device_api_rejections():
    L = _lib()
    plan = CudaPlan(canonical_signature(3, 0))
    x = dev(np.zeros((4, 8)))
    assert L.geo_batch_gp_cuda_planned_forward_f64(ctypes.byref(plan.dev), ptr(x), 0, ptr(x), 0, ptr(x), stream()) == 1
    assert L.geo_batch_gp_cuda_planned_forward_f64(None, ptr(x), 4, ptr(x), 0, ptr(x), stream()) == 1
    bogus = abi.CudaPlan()
    ctypes.memmove(ctypes.byref(bogus), ctypes.byref(plan.dev), ctypes.sizeof(bogus))
    bogus.device_left_blade = None
    assert L.geo_batch_gp_cuda_planned_forward_f64(ctypes.byref(bogus), ptr(x), 4, ptr(x), 0, ptr(x), stream()) == 1
    assert L.geo_batch_gp_cuda_mse_sgd_step_f64(ctypes.byref(plan.dev), ptr(x), ptr(x), 4, 0.0, 0, ptr(x), ptr(x),
                                                ptr(x), ptr(x), stream()) == 1
    assert L.geo_batch_gp_cuda_status_string(2) == b"allocation_failure"


def test_unaligned_device_pointers(oracle):
    """Pointers that are 8- but not 16-byte aligned take the 8-byte staging path."""
    L = _lib()
    for n in (3, 4, 6):
        sig = canonical_signature(n, 1)
        plan = CudaPlan(sig)
        N = 1 << n
        x, w, t = _case(n, 200, 9 + n)
        big = dev(np.concatenate([[0.0], x.ravel()]))
        big_t = dev(np.concatenate([[0.0], t.ravel()]))
        xo = ctypes.c_void_p(big.data_ptr() + 8)
        to = ctypes.c_void_p(big_t.data_ptr() + 8)
        out = dev(np.zeros(x.size + 1))
        oo = ctypes.c_void_p(out.data_ptr() + 8)
        dw = dev(w)
        assert L.geo_batch_gp_cuda_planned_forward_f64(ctypes.byref(plan.dev), xo, 200, ptr(dw), 0, oo, stream()) == 0
        g = dev(np.zeros(N))
        assert L.geo_batch_gp_cuda_parameter_vjp_f64(ctypes.byref(plan.dev), xo, to, 200, 1, ptr(g), stream()) == 0
        sync()
        assert tol_close(host(out)[1:].reshape(200, N), oracle.forward(sig, x, w, False)[1], TOL)
        assert tol_close(host(g), oracle.vjp(sig, x, t, True)[1], TOL)
        # MSE-SGD step with 8-byte aligned residuals (the Cayley cycle kernel at every n)
        res = dev(np.zeros(x.size + 1))
        ro = ctypes.c_void_p(res.data_ptr() + 8)
        dparam, dgrad, dloss = dev(w.copy()), dev(np.zeros(N)), dev(np.zeros(1))
        assert L.geo_batch_gp_cuda_mse_sgd_step_f64(ctypes.byref(plan.dev), ptr(dev(x)), ptr(dev(t)), 200, 1e-3, 0,
                                                    ptr(dparam), ro, ptr(dgrad), ptr(dloss), stream()) == 0
        sync()
        st, w_ref, mean_loss = oracle.sgd_step(sig, x, t, 1e-3, w, False)
        assert st == 0
        assert tol_close(host(res)[1:].reshape(200, N), oracle.forward(sig, x, w, False)[1] - t, TOL)
        assert tol_close(host(dparam), w_ref, TOL) and tol_close(host(dloss)[0] / 200, mean_loss, TOL)


@pytest.mark.parametrize("q", [0, 3])
def test_full_size_n6_properties(oracle, q):
    """At 2^22 samples (the Cl(6,0)/Cl(3,3) training shape): spot rows of the
    forward match the oracle, the VJP is additive over a split of the batch,
    and targets equal to the outputs give exactly zero loss and gradient."""
    import torch

    L = _lib()
    sig = canonical_signature(6, q)
    plan = CudaPlan(sig)
    B, N = 1 << 22, 64
    gen = torch.Generator(device="cuda").manual_seed(5 + q)
    X = torch.rand((B, N), dtype=torch.float64, device="cuda", generator=gen) * 2 - 1
    T = torch.rand((B, N), dtype=torch.float64, device="cuda", generator=gen) * 2 - 1
    w = splitmix_uniform(3 + q, (N,)) * 0.35
    dw = dev(w)
    Y = torch.empty_like(X)
    for left in (0, 1):
        assert L.geo_batch_gp_cuda_planned_forward_f64(ctypes.byref(plan.dev), ptr(X), B, ptr(dw), left, ptr(Y),
                                                       stream()) == 0
        sync()
        rows = np.random.default_rng(q).integers(0, B, 512)
        xr = host(X[torch.as_tensor(rows, device="cuda")])
        assert tol_close(host(Y[torch.as_tensor(rows, device="cuda")]), oracle.forward(sig, xr, w, bool(left))[1], TOL)
        g_all, g_a, g_b = (dev(np.zeros(N)) for _ in range(3))
        half = B // 2 + 123
        for (xp, tp, b, g) in ((X, T, B, g_all), (X[:half], T[:half], half, g_a), (X[half:], T[half:], B - half, g_b)):
            assert L.geo_batch_gp_cuda_parameter_vjp_f64(ctypes.byref(plan.dev), ptr(xp), ptr(tp), b, left, ptr(g),
                                                         stream()) == 0
        sync()
        assert tol_close(host(g_all), host(g_a) + host(g_b), TOL)
        # fixed point: T := Y exactly -> zero loss and zero gradient
        res = torch.empty_like(X)
        dgrad, dloss = dev(np.ones(N)), dev(np.ones(1))
        dparam = dev(w.copy())
        assert L.geo_batch_gp_cuda_mse_sgd_step_f64(ctypes.byref(plan.dev), ptr(X), ptr(Y), B, 1e-3, left,
                                                    ptr(dparam), ptr(res), ptr(dgrad), ptr(dloss), stream()) == 0
        sync()
        assert host(dloss)[0] == 0.0 and np.all(host(dgrad) == 0.0) and np.array_equal(host(dparam), w)


@pytest.mark.parametrize("batch", [1, 17, 33, 1000, 4099, 296 * 16 * 3 + 5, (1 << 22) + 5])
def test_sgd_step_is_residual_then_vjp(oracle, batch):
    """The device MSE-SGD step at n = 5, 6 (one fused pass): its residuals are
    bitwise the planned forward's outputs minus the targets (one IEEE
    subtraction each), its gradient is bitwise the parameter VJP entry point
    applied to those residuals, and loss and update match the oracle (small
    batches: the whole batch; the full-size batch: spot rows, the loss of the
    stored residuals and the update rule)."""
    import torch

    L = _lib()
    big = batch > 1 << 20
    cases = [(6, 0), (6, 3)] if big else [(n, q) for n in (5, 6) for q in range(n + 1)]
    for n, q in cases:
        sig = canonical_signature(n, q)
        plan = CudaPlan(sig)
        N = 1 << n
        gen = torch.Generator(device="cuda").manual_seed(77 * n + q + batch)
        X = torch.rand((batch, N), dtype=torch.float64, device="cuda", generator=gen) * 2 - 1
        T = torch.rand((batch, N), dtype=torch.float64, device="cuda", generator=gen) * 2 - 1
        w = splitmix_uniform(600 + 7 * n + q, (N,)) * 0.35
        dw = dev(w)
        for left in ((q % 2,) if big else (0, 1)):
            Y = torch.empty_like(X)
            assert L.geo_batch_gp_cuda_planned_forward_f64(ctypes.byref(plan.dev), ptr(X), batch, ptr(dw), left,
                                                           ptr(Y), stream()) == 0
            res = torch.full_like(X, 3.0)
            dparam, dgrad, dloss = dev(w.copy()), dev(np.zeros(N)), dev(np.zeros(1))
            assert L.geo_batch_gp_cuda_mse_sgd_step_f64(ctypes.byref(plan.dev), ptr(X), ptr(T), batch, 1e-3, left,
                                                        ptr(dparam), ptr(res), ptr(dgrad), ptr(dloss), stream()) == 0
            g_vjp = dev(np.zeros(N))
            assert L.geo_batch_gp_cuda_parameter_vjp_f64(ctypes.byref(plan.dev), ptr(X), ptr(res), batch, left,
                                                         ptr(g_vjp), stream()) == 0
            sync()
            assert torch.equal(res, Y - T), (n, q, left)
            assert np.array_equal(host(dgrad), host(g_vjp)), (n, q, left)
            if not big:
                st, w_ref, mean_loss = oracle.sgd_step(sig, host(X), host(T), 1e-3, w, bool(left))
                assert st == 0
                assert tol_close(host(dloss)[0] / batch, mean_loss, TOL)
                assert tol_close(host(dparam), w_ref, TOL), (n, q, left, max_violation(host(dparam), w_ref, TOL))
            else:
                rows = np.concatenate([np.random.default_rng(batch + q).integers(0, batch, 256),
                                       np.arange(batch - 20, batch)])
                idx = torch.as_tensor(rows, device="cuda")
                y_ref = oracle.forward(sig, host(X[idx]), w, bool(left))[1]
                assert tol_close(host(res[idx]), y_ref - host(T[idx]), TOL)
                assert tol_close(host(dloss)[0], 0.5 * float((res * res).sum()), TOL)
                assert np.array_equal(host(dparam), w - (1e-3 / batch) * host(dgrad))


def accurate_vjp(oracle, sig, x, cot, left: bool) -> np.ndarray:
    """g_p = sum_i sigma(i,p) (X^T C)[i][i^p] with X^T C formed per 1024-sample chunk in
    float64 and accumulated across chunks in extended precision (about 1e-15
    relative to the result): a summation far more accurate than either the
    reference's sequential sum or the GPU's tree."""
    n = int(np.log2(x.shape[1]))
    N = 1 << n
    acc = np.zeros((N, N), dtype=np.longdouble)
    for a in range(0, x.shape[0], 1024):
        acc += (x[a:a + 1024].T @ cot[a:a + 1024]).astype(np.longdouble)
    g = np.zeros(N, dtype=np.longdouble)
    for p in range(N):
        for i in range(N):
            s = oracle.sign(p, i, sig) if left else oracle.sign(i, p, sig)
            g[p] += s * acc[i, i ^ p]
    return g.astype(np.float64)


def test_n6_oracle_at_scale(oracle):
    """2^16 samples of Cl(6,0) and Cl(3,3): the VJP (65536-sample sums) is within
    1e-12 of an accurate re-summation, at least as close as the reference's own
    sequential sum (which loses ~1e-10 on cancelled components at this size)."""
    L = _lib()
    B = 1 << 16
    for q in (0, 3):
        sig = canonical_signature(6, q)
        plan = CudaPlan(sig)
        x, w, t = _case(6, B, 900 + q)
        dx, dt, dw = dev(x), dev(t), dev(w)
        for left in (0, 1):
            g = dev(np.zeros(64))
            assert L.geo_batch_gp_cuda_parameter_vjp_f64(ctypes.byref(plan.dev), ptr(dx), ptr(dt), B, left, ptr(g),
                                                         stream()) == 0
            sync()
            exact = accurate_vjp(oracle, sig, x, t, bool(left))
            seq = oracle.vjp(sig, x, t, bool(left))[1]
            assert tol_close(host(g), exact, TOL), max_violation(host(g), exact, TOL)
            assert np.max(np.abs(host(g) - exact)) <= np.max(np.abs(seq - exact)) + 1e-12
            assert tol_close(seq, exact, 1e-9)
