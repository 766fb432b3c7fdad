"""Failure detection of the data-parallel communicator, without a GPU fault.

A rank that never joins: rank 0 of a world of two creates its communicator
alone. geo_b200_comm_create must give up after its timeout with
GEO_B200_TIMEOUT (the non-blocking NCCL initialisation is aborted on the host;
no kernel is launched), instead of waiting forever. Runs on one GPU in a child
process; NVLS is off as for every failure test on this hardware.
"""
from __future__ import annotations

import multiprocessing as mp

import pytest

pytestmark = pytest.mark.gpu

GEO_B200_TIMEOUT = 7


def _create_alone(queue) -> None:
    import ctypes
    import os
    import time

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    from geometricelementaryoperators_b200 import abi

    torch.cuda.set_device(0)
    L = abi.lib()
    uid = (ctypes.c_ubyte * 128)()
    assert L.geo_b200_comm_unique_id(uid) == 0
    comm = ctypes.c_void_p()
    t0 = time.perf_counter()
    st = L.geo_b200_comm_create(ctypes.byref(comm), 0, 2, uid, 2000)
    queue.put((st, time.perf_counter() - t0, comm.value))


def test_comm_create_times_out_when_a_rank_never_joins():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    proc = ctx.Process(target=_create_alone, args=(queue,))
    proc.start()
    try:
        st, elapsed, handle = queue.get(timeout=180)
    finally:
        proc.join(timeout=60)
        if proc.is_alive():
            proc.kill()
    assert st == GEO_B200_TIMEOUT
    assert 1.9 < elapsed < 60.0
    assert not handle
