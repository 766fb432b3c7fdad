"""GPU parity of the fused full-cycle trainer (geo_b200_trainer_*) against the
oracle composite of the reference V8 loop (batch VJP for the summed gradient,
then the V8 SGD/Adam update restated in oracle/geo_oracle.c, which
test_oracle pins bit-exactly to the reference's per-sample V8 loop)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from geometricelementaryoperators_b200 import abi, canonical_signature
from geometricelementaryoperators_b200.synthetic import normal, splitmix_uniform
from tests.conftest import max_violation, tol_close
from tests.gpu_helpers import TOL, dev, host, np_ptr, ptr, stream, sync

pytestmark = pytest.mark.gpu


CAYLEY, REPRESENTATION = 1, 2


class Trainer:
    def __init__(self, sig, left, w0, optimizer, lr, b1=0.9, b2=0.999, eps=1e-8, algorithm=0):
        self.L = abi.lib()
        self.h = ctypes.c_void_p()
        cfg = abi.OptimizerConfig(optimizer, lr, b1, b2, eps)
        w0 = np.ascontiguousarray(w0, np.float64)
        st = self.L.geo_b200_trainer_create(ctypes.byref(self.h), len(sig), abi.sig_array(sig), int(left),
                                            np_ptr(w0), ctypes.byref(cfg))
        assert st == 0, st
        self.n = 1 << len(sig)
        if algorithm:
            assert self.L.geo_b200_trainer_set_algorithm(self.h, algorithm) == 0

    def step(self, dx, dt, batch, scale):
        return self.L.geo_b200_trainer_step_device(self.h, ptr(dx), ptr(dt), batch, scale, stream())

    def sync(self):
        loss = ctypes.c_double()
        st = self.L.geo_b200_trainer_sync(self.h, ctypes.byref(loss))
        return st, loss.value

    def state(self):
        w, m, v = np.zeros(self.n), np.zeros(self.n), np.zeros(self.n)
        steps = ctypes.c_uint64()
        assert self.L.geo_b200_trainer_get_state(self.h, np_ptr(w), np_ptr(m), np_ptr(v), ctypes.byref(steps)) == 0
        return w, m, v, steps.value

    def __del__(self):
        try:
            self.L.geo_b200_trainer_destroy(self.h)
        except Exception:
            pass


def _oracle_train(oracle, sig, left, x, t, w0, optimizer, lr, steps, b1=0.9, b2=0.999, eps=1e-8):
    w, m, v = w0.copy(), np.zeros_like(w0), np.zeros_like(w0)
    losses = []
    B = x.shape[0]
    for k in range(1, steps + 1):
        st, y = oracle.forward(sig, x, w, left)
        assert st == 0
        r = y - t
        losses.append(float(np.sum(0.5 * r * r)))
        st, g = oracle.vjp(sig, x, r, left)
        assert st == 0
        st, w, m, v = oracle.v8_update(optimizer, lr, b1, b2, eps, 1.0 / B, k, g, w, m, v)
        assert st == 0
    return w, m, v, losses


def _targets(oracle, sig, left, x, seed):
    """Y = W* x (or x W*) + N(0, 1e-3) noise with W* ~ N(0, 1)."""
    N = x.shape[1]
    w_star = normal(seed, (N,), 1.0)
    y = oracle.forward(sig, x, w_star, left)[1]
    return y + normal(seed + 1, y.shape, 1e-3)


def test_trainer_sgd_cfg2_cl30(oracle):
    """Cl(3,0), batch 256, SGD lr 1e-2, 200 steps, parameter on the left (Y = W* X)."""
    sig = canonical_signature(3, 0)
    x = splitmix_uniform(21, (256, 8))
    t = _targets(oracle, sig, True, x, 22)
    w0 = normal(23, (8,), 0.1)
    tr = Trainer(sig, True, w0, 1, 1e-2)
    dx, dt = dev(x), dev(t)
    for _ in range(200):
        assert tr.step(dx, dt, 256, 1.0 / 256) == 0
    st, loss = tr.sync()
    assert st == 0
    w, m, v, steps = tr.state()
    w_ref, _, _, losses = _oracle_train(oracle, sig, True, x, t, w0, 1, 1e-2, 200)
    assert steps == 200
    assert tol_close(w, w_ref, TOL), max_violation(w, w_ref, TOL)
    assert tol_close(loss, losses[-1], TOL)


@pytest.mark.parametrize("algorithm", [CAYLEY, REPRESENTATION])
@pytest.mark.parametrize("left,B,steps", [(True, 65536, 6), (False, 65536, 4), (True, 4096, 100),
                                          (False, 4096, 100)])
def test_trainer_adam_cfg3_cl41(oracle, left, B, steps, algorithm):
    """Cl(4,1) Adam lr 1e-3, 0.9/0.999 on both sides: the batch-65536 shape for a
    few steps and the full 100-step schedule at batch 4096 (oracle cost bound)."""
    sig = canonical_signature(5, 1)
    N = 32
    x = splitmix_uniform(31 + left, (B, N))
    t = _targets(oracle, sig, left, x, 32 + left)
    w0 = normal(33, (N,), 0.1)
    tr = Trainer(sig, left, w0, 2, 1e-3, algorithm=algorithm)
    assert tr.L.geo_b200_trainer_algorithm(tr.h) == algorithm
    dx, dt = dev(x), dev(t)
    for _ in range(steps):
        assert tr.step(dx, dt, B, 1.0 / B) == 0
    st, loss = tr.sync()
    assert st == 0
    w, m, v, count = tr.state()
    w_ref, m_ref, v_ref, losses = _oracle_train(oracle, sig, left, x, t, w0, 2, 1e-3, steps)
    assert count == steps
    assert tol_close(w, w_ref, TOL), max_violation(w, w_ref, TOL)
    assert tol_close(m, m_ref, TOL) and tol_close(v, v_ref, TOL)
    assert tol_close(loss, losses[-1], TOL)


@pytest.mark.parametrize("algorithm", [0, CAYLEY])
def test_trainer_matches_golden_v8(algorithm):
    """Golden vectors of the reference's per-sample V8 loop (SGD and Adam, both sides)."""
    import pathlib

    golden = np.load(pathlib.Path(__file__).resolve().parent / "golden" / "batch_gp_golden.npz")
    for n, q in [(2, 0), (3, 0), (4, 1), (5, 1), (6, 0), (6, 3)]:
        sig = canonical_signature(n, q)
        xs, ts, w0 = golden[f"v8_n{n}q{q}_x"], golden[f"v8_n{n}q{q}_t"], golden[f"v8_n{n}q{q}_w0"]
        dx, dt = dev(xs), dev(ts)
        for opt in (1, 2):
            for side, left in (("R", False), ("L", True)):
                tr = Trainer(sig, left, w0, opt, 1e-2, algorithm=algorithm)
                want = golden[f"v8_n{n}q{q}{side}_opt{opt}_w"]
                losses = golden[f"v8_n{n}q{q}{side}_opt{opt}_loss"]
                for k in range(3):
                    assert tr.step(dx, dt, xs.shape[0], 1.0 / xs.shape[0]) == 0
                    st, loss = tr.sync()
                    assert st == 0
                    w = tr.state()[0]
                    assert tol_close(w, want[k], TOL), (n, q, side, opt, k)
                    assert tol_close(loss, losses[k], TOL)


def test_trainer_host_buffers_and_state_roundtrip(oracle):
    sig = canonical_signature(4, 2)
    x = splitmix_uniform(41, (999, 16))
    t = splitmix_uniform(42, (999, 16))
    w0 = splitmix_uniform(43, (16,))
    tr = Trainer(sig, False, w0, 2, 1e-3)
    loss = ctypes.c_double()
    for _ in range(3):
        assert tr.L.geo_b200_trainer_step_host(tr.h, np_ptr(x), np_ptr(t), 999, 1.0 / 999, ctypes.byref(loss)) == 0
    w, m, v, steps = tr.state()
    w_ref, m_ref, v_ref, losses = _oracle_train(oracle, sig, False, x, t, w0, 2, 1e-3, 3)
    assert steps == 3 and tol_close(w, w_ref, TOL) and tol_close(loss.value, losses[-1], TOL)
    # checkpoint/resume: restore state into a fresh trainer, continue, compare to an uninterrupted run
    tr2 = Trainer(sig, False, w0, 2, 1e-3)
    assert tr2.L.geo_b200_trainer_set_state(tr2.h, np_ptr(w), np_ptr(m), np_ptr(v), 3) == 0
    for h in (tr.h, tr2.h):
        assert tr.L.geo_b200_trainer_step_host(h, np_ptr(x), np_ptr(t), 999, 1.0 / 999, ctypes.byref(loss)) == 0
    a, b = tr.state(), tr2.state()
    assert all(np.array_equal(u, v) for u, v in zip(a[:3], b[:3])) and a[3] == b[3] == 4


def test_trainer_transactional_failure():
    """A non-finite target makes the step fail at sync with the state untouched;
    later steps are blocked until the status is read."""
    sig = canonical_signature(3, 1)
    x = splitmix_uniform(51, (64, 8))
    t = splitmix_uniform(52, (64, 8))
    w0 = splitmix_uniform(53, (8,))
    tr = Trainer(sig, False, w0, 2, 1e-2)
    dx, dt = dev(x), dev(t)
    assert tr.step(dx, dt, 64, 1 / 64) == 0
    assert tr.sync()[0] == 0
    before = tr.state()
    tbad = t.copy()
    tbad[3, 3] = np.nan
    dbad = dev(tbad)
    assert tr.step(dx, dbad, 64, 1 / 64) == 0
    assert tr.step(dx, dt, 64, 1 / 64) == 0  # blocked by the earlier failure
    assert tr.sync()[0] == 3
    after = tr.state()
    assert all(np.array_equal(u, v) for u, v in zip(before[:3], after[:3])) and after[3] == before[3]
    assert tr.step(dx, dt, 64, 1 / 64) == 0
    assert tr.sync()[0] == 0 and tr.state()[3] == before[3] + 1


@pytest.mark.parametrize("n", [5, 6])
def test_representation_all_signatures(oracle, n):
    """The tensor-core representation path on every Cl(p,q) with p+q = n, both sides:
    three Adam steps on 3000 samples (ragged last tile) against the oracle."""
    from tests.conftest import all_signatures

    N = 1 << n
    B = 3000
    for _, q, sig in all_signatures(n, n):
        for left in (False, True):
            x = splitmix_uniform(700 + 10 * q + left, (B, N))
            t = _targets(oracle, sig, left, x, 800 + q)
            w0 = normal(900 + q, (N,), 0.125)
            tr = Trainer(sig, left, w0, 2, 1e-3, algorithm=REPRESENTATION)
            dx, dt = dev(x), dev(t)
            losses = []
            for _ in range(3):
                assert tr.step(dx, dt, B, 1.0 / B) == 0
                st, loss = tr.sync()
                assert st == 0
                losses.append(loss)
            w, m, v, count = tr.state()
            w_ref, m_ref, v_ref, l_ref = _oracle_train(oracle, sig, left, x, t, w0, 2, 1e-3, 3)
            assert count == 3
            assert tol_close(w, w_ref, TOL), (n, q, left, max_violation(w, w_ref, TOL))
            assert tol_close(m, m_ref, TOL) and tol_close(v, v_ref, TOL)
            assert tol_close(losses, l_ref, TOL), (losses, l_ref)


@pytest.mark.parametrize("q", [0, 3])
def test_representation_matches_cayley_full_size(q):
    """At the full 2^22-sample Cl(6,0) / Cl(3,3) shape the two independent kernel
    families give the same gradient record: one Adam step from the same state
    lands on the same parameters and loss (1e-12)."""
    import torch

    sig = canonical_signature(6, q)
    B = 1 << 22
    gen = torch.Generator(device="cuda").manual_seed(40 + q)
    X = torch.rand((B, 64), dtype=torch.float64, device="cuda", generator=gen) * 2 - 1
    T = torch.rand((B, 64), dtype=torch.float64, device="cuda", generator=gen) * 2 - 1
    w0 = normal(41 + q, (64,), 0.125)
    results = []
    for algorithm in (CAYLEY, REPRESENTATION):
        tr = Trainer(sig, False, w0, 2, 1e-3, algorithm=algorithm)
        assert tr.step(X, T, B, 1.0 / B) == 0
        st, loss = tr.sync()
        assert st == 0
        results.append((tr.state(), loss))
    (s1, l1), (s2, l2) = results
    assert tol_close(l1, l2, TOL)
    for a, b in zip(s1[:3], s2[:3]):
        assert tol_close(a, b, TOL), max_violation(a, b, TOL)


def test_large_batch_step_is_additive():
    """2^25 + 7 Cl(6,0) samples (32 GiB resident, eight times the headline
    batch; tile and record indexing far past 2^31 bytes): one whole-batch SGD
    step equals two half-batch accumulations followed by one update, and the
    reported loss sums agree (1e-12)."""
    import torch

    L = abi.lib()
    sig = canonical_signature(6, 0)
    B = (1 << 25) + 7
    gen = torch.Generator(device="cuda").manual_seed(77)
    X = torch.rand((B, 64), dtype=torch.float64, device="cuda", generator=gen).mul_(2).sub_(1)
    T = torch.rand((B, 64), dtype=torch.float64, device="cuda", generator=gen).mul_(2).sub_(1)
    w0 = normal(78, (64,), 0.125)
    whole = Trainer(sig, False, w0, 1, 1e-2)
    assert whole.step(X, T, B, 1.0 / B) == 0
    st, loss_whole = whole.sync()
    assert st == 0
    split = Trainer(sig, False, w0, 1, 1e-2)
    half = B // 2 + 13
    for xs, ts, b in ((X[:half], T[:half], half), (X[half:], T[half:], B - half)):
        assert L.geo_b200_trainer_accumulate_device(split.h, ptr(xs), ptr(ts), b, stream()) == 0
    assert L.geo_b200_trainer_apply(split.h, 1.0 / B, stream()) == 0
    st, loss_split = split.sync()
    assert st == 0
    assert tol_close(loss_whole, loss_split, TOL)
    w1, _, _, n1 = whole.state()
    w2, _, _, n2 = split.state()
    assert n1 == n2 == 1
    assert tol_close(w1, w2, TOL), max_violation(w1, w2, TOL)
    assert not np.array_equal(w1, w0)
