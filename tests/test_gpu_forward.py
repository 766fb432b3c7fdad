"""GPU parity of geo_b200_forward_f64, the fixed-parameter batched forward on a
chosen kernel family, against the CPU oracle (the reference's batch_gp
forward, src/batch_gp.c:107-161) and against the device ABI's forward.

Tolerance: float64 within |a-b| <= 1e-12 (1+|a|+|b|) of the oracle. AUTO must
be bit-identical to the device ABI's forward (the same kernel: Cayley below
n = 5, the representation at n = 5, 6); the families differ by rounding only.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from geometricelementaryoperators_b200 import abi, canonical_signature
from geometricelementaryoperators_b200.synthetic import splitmix_uniform
from tests.conftest import all_signatures, max_violation, tol_close
from tests.gpu_helpers import TOL, CudaPlan, dev, host, ptr, stream, sync

pytestmark = pytest.mark.gpu
AUTO, CAYLEY, REPRESENTATION = 0, 1, 2
# Batches around the tile sizes (16 or 32 samples) and the grid (2 CTAs per SM).
BATCHES = [1, 3, 16, 17, 33, 1000, 4099, 300 * 32 + 7]


def _forward(sig, left, algorithm, x, w, y, batch):
    return abi.lib().geo_b200_forward_f64(len(sig), abi.sig_array(sig), left, algorithm, ptr(x), ptr(w), ptr(y),
                                          batch, stream())


@pytest.mark.parametrize("batch", BATCHES)
def test_forward_all_signatures(oracle, batch):
    L = abi.lib()
    for n, q, sig in all_signatures():
        N = 1 << n
        x = splitmix_uniform(41 * n + q + batch, (batch, N))
        w = splitmix_uniform(43 * n + q + batch, (N,))
        dx, dw = dev(x), dev(w)
        plan = CudaPlan(sig)
        for left in (0, 1):
            y_ref = oracle.forward(sig, x, w, bool(left))[1]
            planned = dev(np.zeros_like(x))
            assert L.geo_batch_gp_cuda_planned_forward_f64(ctypes.byref(plan.dev), ptr(dx), batch, ptr(dw), left,
                                                           ptr(planned), stream()) == 0
            for algorithm in (AUTO, CAYLEY, REPRESENTATION):
                y = dev(np.full_like(x, 7.0))
                st = _forward(sig, left, algorithm, dx, dw, y, batch)
                if algorithm == REPRESENTATION and n < 5:
                    assert st == 1  # no representation kernel below n = 5
                    continue
                assert st == 0, (n, q, left, algorithm)
                sync()
                got = host(y)
                assert tol_close(got, y_ref, TOL), (n, q, left, algorithm, max_violation(got, y_ref, TOL))
                # the device ABI's forward runs the same kernel as AUTO: Cayley below n = 5,
                # the representation at n = 5, 6 (aligned operands)
                if algorithm != CAYLEY or n < 5:
                    assert np.array_equal(got, host(planned)), (n, q, left, algorithm)


def test_forward_rejections():
    L = abi.lib()
    sig = canonical_signature(6, 0)
    x = dev(np.zeros((4, 64)))
    s = abi.sig_array(sig)
    assert L.geo_b200_forward_f64(7, s, 0, AUTO, ptr(x), ptr(x), ptr(x), 4, stream()) == 2
    assert L.geo_b200_forward_f64(6, s, 0, AUTO, ptr(x), ptr(x), ptr(x), 0, stream()) == 1
    assert L.geo_b200_forward_f64(6, s, 0, AUTO, None, ptr(x), ptr(x), 4, stream()) == 1
    assert L.geo_b200_forward_f64(6, s, 0, 9, ptr(x), ptr(x), ptr(x), 4, stream()) == 1
    bad = abi.sig_array([1, 1, 2, 1, 1, 1])
    assert L.geo_b200_forward_f64(6, bad, 0, AUTO, ptr(x), ptr(x), ptr(x), 4, stream()) == 1


def test_forward_unaligned_and_in_place(oracle):
    """8-byte aligned pointers: AUTO falls back to the Cayley kernel and an
    explicit REPRESENTATION is refused; outputs equal to inputs work in place."""
    for q in (0, 3):
        sig = canonical_signature(6, q)
        B = 777
        x = splitmix_uniform(70 + q, (B, 64))
        w = splitmix_uniform(71 + q, (64,))
        y_ref = oracle.forward(sig, x, w, False)[1]
        big = dev(np.concatenate([[0.0], x.ravel()]))
        out = dev(np.zeros(x.size + 1))
        xo = ctypes.c_void_p(big.data_ptr() + 8)
        oo = ctypes.c_void_p(out.data_ptr() + 8)
        dw = dev(w)
        L = abi.lib()
        s = abi.sig_array(sig)
        assert L.geo_b200_forward_f64(6, s, 0, REPRESENTATION, xo, ptr(dw), oo, B, stream()) == 1
        assert L.geo_b200_forward_f64(6, s, 0, AUTO, xo, ptr(dw), oo, B, stream()) == 0
        sync()
        assert tol_close(host(out)[1:].reshape(B, 64), y_ref, TOL)
        inplace = dev(x)
        assert _forward(sig, 0, REPRESENTATION, inplace, dw, inplace, B) == 0
        sync()
        assert tol_close(host(inplace), y_ref, TOL)


def test_forward_non_finite_rows(oracle):
    """A non-finite input coefficient makes every output coefficient of its
    sample non-finite (every output blade takes a term of every input blade,
    src/batch_gp.c:127-137, and the reference's device forward does not check
    its inputs); other samples are unaffected. The oracle (the host API, which
    rejects non-finite inputs) gives the expected values of the finite rows."""
    sig = canonical_signature(6, 0)
    B = 100
    x = splitmix_uniform(90, (B, 64))
    w = splitmix_uniform(91, (64,))
    y_ref = oracle.forward(sig, x, w, False)[1]
    x[7, 5] = np.nan
    x[50, 63] = np.inf
    dx, dw = dev(x), dev(w)
    for algorithm in (CAYLEY, REPRESENTATION):
        y = dev(np.zeros_like(x))
        assert _forward(sig, 0, algorithm, dx, dw, y, B) == 0
        sync()
        got = host(y)
        assert not np.any(np.isfinite(got[7])) and not np.any(np.isfinite(got[50]))
        keep = np.ones(B, dtype=bool)
        keep[[7, 50]] = False
        assert tol_close(got[keep], y_ref[keep], TOL)


@pytest.mark.parametrize("q", [0, 3])
def test_forward_full_size(oracle, q):
    """2^22 + 5 samples (the headline shape plus a ragged tail): spot rows
    against the oracle, and the two kernel families agree everywhere."""
    import torch

    sig = canonical_signature(6, q)
    B = (1 << 22) + 5
    gen = torch.Generator(device="cuda").manual_seed(40 + q)
    X = torch.rand((B, 64), dtype=torch.float64, device="cuda", generator=gen) * 2 - 1
    w = splitmix_uniform(44 + q, (64,))
    dw = dev(w)
    for left in (0, 1):
        Yr = torch.empty_like(X)
        Yc = torch.empty_like(X)
        assert _forward(sig, left, REPRESENTATION, X, dw, Yr, B) == 0
        assert _forward(sig, left, CAYLEY, X, dw, Yc, B) == 0
        sync()
        rows = np.concatenate([np.random.default_rng(q + 2 * left).integers(0, B, 512), np.arange(B - 40, B)])
        idx = torch.as_tensor(rows, device="cuda")
        y_ref = oracle.forward(sig, host(X[idx]), w, bool(left))[1]
        assert tol_close(host(Yr[idx]), y_ref, TOL)
        diff = (Yr - Yc).abs() - TOL * (1 + Yr.abs() + Yc.abs())
        assert float(diff.max()) <= 0.0
