"""Data-parallel trainer on two GPUs (one process per GPU, NCCL record exchange).

Each rank trains on its shard of one global batch through
geo_b200_trainer_step_device with a communicator attached; the replicas must
stay bit-identical and match the oracle run of the reference V8 loop over the
whole batch (src/full_cycle_v8.c:942-1041) within 1e-12. Skipped on a box with
fewer than two GPUs.
"""
from __future__ import annotations

import ctypes
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORLD = 2
STEPS = 3
ADAM = 2
LR = 1e-2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(n, q, batch):
    from geometricelementaryoperators_b200 import canonical_signature
    from geometricelementaryoperators_b200.synthetic import normal, splitmix_uniform

    sig = canonical_signature(n, q)
    x = splitmix_uniform(11 + n + q, (batch, 1 << n))
    t = splitmix_uniform(23 + n + q, (batch, 1 << n))
    w0 = normal(5 + n, (1 << n,), 0.125)
    return sig, x, t, w0


def _shards(batch):
    # ragged on purpose: rank 0 gets one sample more
    cut = batch // 2 + 1
    return [(0, cut), (cut, batch)]


def _rank_main(rank, port, n, q, batch, algorithm, queue):
    import torch
    import torch.distributed as dist

    from geometricelementaryoperators_b200 import abi

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    L = abi.lib()
    tr = ctypes.c_void_p()
    comm = ctypes.c_void_p()
    try:
        sig, x, t, w0 = _data(n, q, batch)
        lo, hi = _shards(batch)[rank]
        dx = torch.from_numpy(np.ascontiguousarray(x[lo:hi])).cuda()
        dt = torch.from_numpy(np.ascontiguousarray(t[lo:hi])).cuda()
        uid = (ctypes.c_ubyte * 128)()
        if rank == 0:
            assert L.geo_b200_comm_unique_id(uid) == 0
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, src=0)
        uid = (ctypes.c_ubyte * 128).from_buffer_copy(obj[0])
        assert L.geo_b200_comm_create(ctypes.byref(comm), rank, WORLD, uid, 60000) == 0
        cfg = abi.OptimizerConfig(ADAM, LR, 0.9, 0.999, 1e-8)
        w0c = np.ascontiguousarray(w0)
        assert L.geo_b200_trainer_create(ctypes.byref(tr), n, abi.sig_array(sig), 0,
                                         w0c.ctypes.data_as(ctypes.c_void_p), ctypes.byref(cfg)) == 0
        if algorithm:
            assert L.geo_b200_trainer_set_algorithm(tr, algorithm) == 0
        assert L.geo_b200_trainer_attach_comm(tr, comm) == 0
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        losses = []
        for _ in range(STEPS):
            st = L.geo_b200_trainer_step_device(tr, ctypes.c_void_p(dx.data_ptr()), ctypes.c_void_p(dt.data_ptr()),
                                                hi - lo, 1.0 / batch, s)
            assert st == 0, st
            loss = ctypes.c_double()
            assert L.geo_b200_trainer_sync(tr, ctypes.byref(loss)) == 0
            losses.append(loss.value)
        w = np.zeros(1 << n)
        steps = ctypes.c_uint64()
        assert L.geo_b200_trainer_get_state(tr, w.ctypes.data_as(ctypes.c_void_p), None, None,
                                            ctypes.byref(steps)) == 0
        queue.put((rank, w.tolist(), losses, steps.value, L.geo_b200_trainer_algorithm(tr)))
    except BaseException as exc:  # report instead of leaving the parent waiting
        queue.put((rank, None, repr(exc), 0, 0))
        raise
    finally:
        if tr:
            L.geo_b200_trainer_destroy(tr)
        if comm:
            L.geo_b200_comm_destroy(comm)
        dist.destroy_process_group()


def _oracle_whole_batch(oracle, sig, x, t, w0):
    w, m, v = w0.copy(), np.zeros_like(w0), np.zeros_like(w0)
    losses = []
    B = x.shape[0]
    for k in range(1, STEPS + 1):
        st, y = oracle.forward(sig, x, w, False)
        assert st == 0
        r = y - t
        losses.append(float(np.sum(0.5 * r * r)))
        st, g = oracle.vjp(sig, x, r, False)
        assert st == 0
        st, w, m, v = oracle.v8_update(ADAM, LR, 0.9, 0.999, 1e-8, 1.0 / B, k, g, w, m, v)
        assert st == 0
    return w, losses


@pytest.mark.parametrize("n,q,batch,algorithm", [(4, 1, 3001, 0), (6, 0, 8193, 0), (6, 3, 4097, 1)])
def test_two_gpu_data_parallel_matches_whole_batch(oracle, n, q, batch, algorithm):
    import torch

    from tests.conftest import max_violation, tol_close

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, n, q, batch, algorithm, queue)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            rank, w, losses, steps, alg = queue.get(timeout=300)
            assert w is not None, f"rank {rank} failed: {losses}"
            res[rank] = (np.array(w), losses, steps, alg)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    w0r, l0, s0, a0 = res[0]
    w1r, l1, s1, a1 = res[1]
    assert s0 == s1 == STEPS
    assert np.array_equal(w0r, w1r), "replicas diverged"
    assert l0 == l1
    sig, x, t, w0 = _data(n, q, batch)
    w_ref, l_ref = _oracle_whole_batch(oracle, sig, x, t, w0)
    assert tol_close(w0r, w_ref, 1e-12), max_violation(w0r, w_ref, 1e-12)
    assert tol_close(l0, l_ref, 1e-12), max_violation(l0, l_ref, 1e-12)
