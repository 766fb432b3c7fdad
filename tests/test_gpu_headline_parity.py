"""Parity at the stated shapes of the two training configurations the bench
and the scaling runs measure, against the oracle over the whole batch:

* Cl(6,0) and Cl(3,3), 2^22 samples (the headline step): one full-cycle Adam
  step of the trainer (representation kernel, as the bench runs it) from seeded
  splitmix inputs, against the oracle's forward on every row and its gradient
  summed in extended precision. Parameters, moments and loss within 1e-12, and
  the GPU's gradient at least as close to that accurate sum as the reference's
  own sequential per-term sum (src/batch_gp.c:163-201), which is computed too.
* Cl(4,1), 65536 samples, Adam lr 1e-3 (0.9/0.999) for the full 100 steps,
  parameter on either side, both kernel families, against the oracle run for
  the same 100 steps.

The oracle runs over a spawn-started process pool (tests/oracle_pool.py);
reference semantics: src/batch_gp.c:107-235 (forward, parameter VJP),
src/full_cycle_v8.c:976-1013 (the Adam update, restated in oracle/geo_oracle.c
and pinned bit for bit to the reference by tests/test_oracle.py).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from geometricelementaryoperators_b200 import abi, canonical_signature
from geometricelementaryoperators_b200.synthetic import normal, splitmix_uniform
from tests.conftest import max_violation, tol_close
from tests.gpu_helpers import TOL, CudaPlan, np_ptr, ptr, stream, sync
from tests.oracle_pool import PooledOracle, gradient_from_gram

pytestmark = pytest.mark.gpu

ADAM, LR, B1, B2, EPS = 2, 1e-3, 0.9, 0.999, 1e-8
CAYLEY, REPRESENTATION = 1, 2


class Trainer:
    def __init__(self, sig, left, w0, algorithm=0):
        self.L = abi.lib()
        self.h = ctypes.c_void_p()
        cfg = abi.OptimizerConfig(ADAM, LR, B1, B2, EPS)
        w0 = np.ascontiguousarray(w0, np.float64)
        assert self.L.geo_b200_trainer_create(ctypes.byref(self.h), len(sig), abi.sig_array(sig), int(left),
                                              np_ptr(w0), ctypes.byref(cfg)) == 0
        if algorithm:
            assert self.L.geo_b200_trainer_set_algorithm(self.h, algorithm) == 0
        self.n = 1 << len(sig)

    def step(self, X, T, batch):
        return self.L.geo_b200_trainer_step_device(self.h, ptr(X), ptr(T), batch, 1.0 / batch, stream())

    def sync(self):
        loss = ctypes.c_double()
        st = self.L.geo_b200_trainer_sync(self.h, ctypes.byref(loss))
        return st, loss.value

    def state(self):
        w, m, v = np.zeros(self.n), np.zeros(self.n), np.zeros(self.n)
        k = ctypes.c_uint64()
        assert self.L.geo_b200_trainer_get_state(self.h, np_ptr(w), np_ptr(m), np_ptr(v), ctypes.byref(k)) == 0
        return w, m, v, k.value

    def __del__(self):
        try:
            self.L.geo_b200_trainer_destroy(self.h)
        except Exception:
            pass


def _fill_inputs(po: PooledOracle, sig, left: bool, seed: int):
    """X ~ U[-1,1] (splitmix, written in slices); T = x W* (or W* x) + N(0, 1e-3),
    W* ~ N(0, 1), made on the device; both copied into the pool's shared arrays.
    Returns the device copies."""
    import torch

    B, N = po.shape
    rows = 1 << 16
    for a in range(0, B, rows):
        b = min(a + rows, B)
        po.X[a:b] = splitmix_uniform(seed, (b - a, N), offset=a * N)
    X = torch.from_numpy(po.X).cuda()
    plan = CudaPlan(sig)
    w_star = torch.from_numpy(normal(seed + 1, (N,), 1.0)).cuda()
    T = torch.empty_like(X)
    assert abi.lib().geo_batch_gp_cuda_planned_forward_f64(ctypes.byref(plan.dev), ptr(X), B, ptr(w_star),
                                                           int(left), ptr(T), stream()) == 0
    gen = torch.Generator(device="cuda").manual_seed(seed + 2)
    T.add_(torch.randn(T.shape, dtype=torch.float64, device="cuda", generator=gen), alpha=1e-3)
    sync()
    po.T[:] = T.cpu().numpy()
    return X, T


@pytest.mark.parametrize("q", [0, 3])
def test_headline_adam_step_2p22_vs_oracle(oracle, q):
    B, N = 1 << 22, 64
    sig = canonical_signature(6, q)
    po = PooledOracle(B, N)
    try:
        X, T = _fill_inputs(po, sig, False, 7100 + q)
        w0 = normal(7200 + q, (N,), 0.125)
        tr = Trainer(sig, False, w0)
        assert tr.L.geo_b200_trainer_algorithm(tr.h) == REPRESENTATION
        assert tr.step(X, T, B) == 0
        st, loss = tr.sync()
        assert st == 0
        w, m, v, k = tr.state()
        del X, T

        loss_acc, gram = po.residual_gram(sig, False, w0)
        g_acc = gradient_from_gram(oracle, sig, False, gram)
        st, w_ref, m_ref, v_ref = oracle.v8_update(ADAM, LR, B1, B2, EPS, 1.0 / B, 1, g_acc, w0, np.zeros(N),
                                                   np.zeros(N))
        assert st == 0 and k == 1
        assert tol_close(loss, float(loss_acc), TOL), (loss, float(loss_acc))
        assert tol_close(w, w_ref, TOL), max_violation(w, w_ref, TOL)
        assert tol_close(m, m_ref, TOL), max_violation(m, m_ref, TOL)
        assert tol_close(v, v_ref, TOL), max_violation(v, v_ref, TOL)

        # The reference's own sequential sum over the same residuals, through the
        # same update: the GPU's first moment (0.1 times its mean gradient) is at
        # least as close to the accurate value as the reference's.
        g_seq = po.sequential_vjp(oracle, sig, False)
        st, _, m_seq, _ = oracle.v8_update(ADAM, LR, B1, B2, EPS, 1.0 / B, 1, g_seq, w0, np.zeros(N), np.zeros(N))
        assert st == 0
        err_gpu = np.max(np.abs(m - m_ref))
        err_seq = np.max(np.abs(m_seq - m_ref))
        assert err_gpu <= err_seq + 4 * np.finfo(np.float64).eps * np.max(np.abs(m_ref)), (err_gpu, err_seq)
    finally:
        po.close()


_CFG3_ORACLE: dict = {}


def _cfg3_oracle(oracle, po, sig, left, w0, steps):
    """The oracle's 100-step Adam trajectory on the pool's batch (final w, m, v, loss)."""
    B, N = po.shape
    w, m, v = w0.copy(), np.zeros(N), np.zeros(N)
    loss = None
    for k in range(1, steps + 1):
        loss, gram = po.residual_gram(sig, left, w, call_rows=256)
        g = gradient_from_gram(oracle, sig, left, gram)
        st, w, m, v = oracle.v8_update(ADAM, LR, B1, B2, EPS, 1.0 / B, k, g, w, m, v)
        assert st == 0
    return w, m, v, float(loss)


@pytest.mark.parametrize("left", [False, True])
def test_cfg3_cl41_adam_100_steps_vs_oracle(oracle, left):
    """Cl(4,1), 65536 samples, the full 100 Adam steps, both kernel families."""
    B, N, steps = 65536, 32, 100
    sig = canonical_signature(5, 1)
    po = PooledOracle(B, N)
    try:
        X, T = _fill_inputs(po, sig, left, 7300 + left)
        w0 = normal(7400 + left, (N,), 0.1)
        w_ref, m_ref, v_ref, loss_ref = _cfg3_oracle(oracle, po, sig, left, w0, steps)
        for algorithm in (CAYLEY, REPRESENTATION):
            tr = Trainer(sig, left, w0, algorithm)
            for _ in range(steps):
                assert tr.step(X, T, B) == 0
            st, loss = tr.sync()
            assert st == 0
            w, m, v, k = tr.state()
            assert k == steps
            assert tol_close(w, w_ref, TOL), (algorithm, max_violation(w, w_ref, TOL))
            assert tol_close(m, m_ref, TOL) and tol_close(v, v_ref, TOL), algorithm
            # the trainer's loss is the last step's, taken before its update
            assert tol_close(loss, loss_ref, TOL), (algorithm, loss, loss_ref)
    finally:
        po.close()
