"""The allocation-free parameter VJP (geo_b200_parameter_vjp_noalloc_f64).

Callers that cannot allocate device memory (a host allocator that already owns
the device memory, a loop that must not take cudaMalloc's device-wide
synchronisation, a plugin host that forbids allocation after start-up) use this
variant: its reduction scratch is a fixed array inside the library, so the call
needs no plan upload and no cudaMalloc. This file checks, through the C-ABI,
that two calls in a row each reproduce the ordinary entry point
(geo_batch_gp_cuda_parameter_vjp_f64) within the float64 tolerance of the other
GPU tests, and that batches beyond the array's capacity are refused before any
launch. It is named to be collected last and depends on no earlier test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from geometricelementaryoperators_b200 import abi, canonical_signature
from geometricelementaryoperators_b200.synthetic import splitmix_uniform
from tests.conftest import max_violation, tol_close
from tests.gpu_helpers import TOL, CudaPlan, dev, host, ptr, stream, sync

pytestmark = pytest.mark.gpu

MAX_BATCH = 131072  # GEO_B200_NOALLOC_MAX_BATCH


@pytest.mark.parametrize("n,q,left,batch", [(6, 0, 0, MAX_BATCH), (6, 3, 1, 4099), (5, 1, 1, 65536),
                                            (3, 0, 0, 1000), (2, 1, 1, 77), (1, 0, 0, 5)])
def test_noalloc_vjp_matches_planned_vjp_twice(n, q, left, batch):
    L = abi.lib()
    sig = canonical_signature(n, q)
    N = 1 << n
    plan = CudaPlan(sig)
    for call in range(2):
        x = splitmix_uniform(4000 + 10 * n + call, (batch, N))
        c = splitmix_uniform(5000 + 10 * n + call, (batch, N))
        dx, dc = dev(x), dev(c)
        g_new, g_ref = dev(np.full(N, np.nan)), dev(np.full(N, np.nan))
        assert L.geo_b200_parameter_vjp_noalloc_f64(n, abi.sig_array(sig), left, ptr(dx), ptr(dc), batch,
                                                    ptr(g_new), stream()) == 0
        assert L.geo_batch_gp_cuda_parameter_vjp_f64(ctypes.byref(plan.dev), ptr(dx), ptr(dc), batch, left,
                                                     ptr(g_ref), stream()) == 0
        sync()
        assert tol_close(host(g_new), host(g_ref), TOL), (call, max_violation(host(g_new), host(g_ref), TOL))


@pytest.mark.parametrize("n,q,left", [(6, 0, 0), (4, 1, 1)])
def test_noalloc_vjp_unaligned_rows_and_oracle(n, q, left, oracle):
    """Rows that start 8 bytes past a 16-byte boundary take the tiled kernel's
    8-byte-aligned variant, still with the fixed array; two calls in a row match
    the ordinary entry point and the CPU oracle."""
    import torch

    L = abi.lib()
    sig = canonical_signature(n, q)
    N = 1 << n
    batch = 3001
    plan = CudaPlan(sig)
    for call in range(2):
        x = splitmix_uniform(6100 + 10 * n + call, (batch, N))
        c = splitmix_uniform(6200 + 10 * n + call, (batch, N))
        bx = torch.zeros(batch * N + 1, dtype=torch.float64, device="cuda")
        bc = torch.zeros(batch * N + 1, dtype=torch.float64, device="cuda")
        bx[1:] = torch.from_numpy(x.reshape(-1)).cuda()
        bc[1:] = torch.from_numpy(c.reshape(-1)).cuda()
        px, pc = ctypes.c_void_p(bx.data_ptr() + 8), ctypes.c_void_p(bc.data_ptr() + 8)
        g_new, g_ref = dev(np.full(N, np.nan)), dev(np.full(N, np.nan))
        assert L.geo_b200_parameter_vjp_noalloc_f64(n, abi.sig_array(sig), left, px, pc, batch, ptr(g_new),
                                                    stream()) == 0
        assert L.geo_batch_gp_cuda_parameter_vjp_f64(ctypes.byref(plan.dev), px, pc, batch, left, ptr(g_ref),
                                                     stream()) == 0
        sync()
        assert tol_close(host(g_new), host(g_ref), TOL), (call, max_violation(host(g_new), host(g_ref), TOL))
        st, want = oracle.vjp(sig, x, c, bool(left))
        assert st == 0
        assert tol_close(host(g_new), want, TOL), (call, max_violation(host(g_new), want, TOL))


def test_noalloc_vjp_rejects_batches_beyond_capacity():
    L = abi.lib()
    sig = canonical_signature(6, 0)
    x = dev(np.zeros((4, 64)))
    g = dev(np.full(64, 7.0))
    assert L.geo_b200_parameter_vjp_noalloc_f64(6, abi.sig_array(sig), 0, ptr(x), ptr(x), MAX_BATCH + 1, ptr(g),
                                                stream()) == 1
    assert L.geo_b200_parameter_vjp_noalloc_f64(6, abi.sig_array(sig), 0, ptr(x), ptr(x), 0, ptr(g), stream()) == 1
    assert L.geo_b200_parameter_vjp_noalloc_f64(7, abi.sig_array([1] * 6), 0, ptr(x), ptr(x), 4, ptr(g),
                                                stream()) == 2
    sync()
    assert np.all(host(g) == 7.0)
