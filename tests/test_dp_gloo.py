"""Data-parallel protocol on CPU: two gloo ranks, no GPU.

The trainer's multi-GPU step (csrc/api_trainer.cu) shards the batch across
ranks; each rank reduces its shard to one record (parameter gradient sum and
loss sum), the records of all ranks are gathered, every rank sums them in rank
order and applies the same update with gradient scale 1/(global batch). This
file runs that protocol with the oracle's arithmetic on two gloo processes and
checks (1) the replicas stay bit-identical, (2) they match a single process
that trains on the whole batch (the reference's per-sample V8 loop with the
optimizer of src/full_cycle_v8.c:942-1041) to the summation-order tolerance,
and (3) the bench's max-over-ranks timing reduction.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

WORLD = 2
DIM = 4
SIGNATURE = [1, 1, 1, -1]
GLOBAL_BATCH = 96
STEPS = 3
ADAM = 2
LR, B1, B2, EPS = 1e-2, 0.9, 0.999, 1e-8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data():
    rng = np.random.default_rng(7)
    x = rng.uniform(-1, 1, (GLOBAL_BATCH, 1 << DIM))
    t = rng.uniform(-1, 1, (GLOBAL_BATCH, 1 << DIM))
    w0 = rng.normal(0, 0.125, 1 << DIM)
    return x, t, w0


def _shard_record(orc, x, t, w):
    """One rank's record: gradient sum of 0.5|xW - t|^2 over its shard, then the loss sum."""
    st, y = orc.forward(SIGNATURE, x, w, False)
    assert st == 0
    r = y - t
    st, g = orc.vjp(SIGNATURE, x, r, False)
    assert st == 0
    loss = float(np.sum(0.5 * r * r))
    return np.concatenate([g, [loss]])


def _rank_main(rank: int, port: int, queue) -> None:
    import torch
    import torch.distributed as dist

    from oracle.oracle import Oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        orc = Oracle()
        x, t, w = _data()
        per = GLOBAL_BATCH // WORLD
        xs, ts = x[rank * per:(rank + 1) * per], t[rank * per:(rank + 1) * per]
        m = np.zeros_like(w)
        v = np.zeros_like(w)
        losses = []
        for step in range(1, STEPS + 1):
            rec = torch.from_numpy(_shard_record(orc, xs, ts, w))
            gathered = [torch.empty_like(rec) for _ in range(WORLD)]
            dist.all_gather(gathered, rec)
            total = gathered[0].numpy().copy()
            for g in gathered[1:]:
                total = total + g.numpy()  # rank order, as the trainer sums records
            losses.append(total[-1] / GLOBAL_BATCH)
            st, w, m, v = orc.v8_update(ADAM, LR, B1, B2, EPS, 1.0 / GLOBAL_BATCH, step, total[:-1], w, m, v)
            assert st == 0
        finals = [torch.empty(len(w), dtype=torch.float64) for _ in range(WORLD)]
        dist.all_gather(finals, torch.from_numpy(w))

        import bench

        timing = bench.max_over_ranks(float(rank + 1) * 1.5, WORLD)
        queue.put((rank, w.tolist(), [f.tolist() for f in finals], losses, timing))
    finally:
        dist.destroy_process_group()


def _single_process(orc):
    x, t, w = _data()
    m = np.zeros_like(w)
    v = np.zeros_like(w)
    losses = []
    for step in range(1, STEPS + 1):
        rec = _shard_record(orc, x, t, w)
        losses.append(rec[-1] / GLOBAL_BATCH)
        st, w, m, v = orc.v8_update(ADAM, LR, B1, B2, EPS, 1.0 / GLOBAL_BATCH, step, rec[:-1], w, m, v)
        assert st == 0
    return w, losses


def test_two_rank_protocol_matches_single_process(oracle):
    from conftest import tol_close

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, queue)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(WORLD):
            rank, w, finals, losses, timing = queue.get(timeout=240)
            results[rank] = (np.array(w), finals, losses, timing)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)

    w0, finals0, losses0, _ = results[0]
    w1, _, losses1, _ = results[1]
    # identical replicas, bit for bit
    assert np.array_equal(w0, w1)
    assert np.array_equal(np.array(finals0[0]), np.array(finals0[1]))
    assert losses0 == losses1
    # the sharded sum differs from one process's sequential sum only by rounding
    w_ref, losses_ref = _single_process(oracle)
    assert tol_close(w0, w_ref, 1e-12)
    assert tol_close(losses0, losses_ref, 1e-12)
    # the bench reports the slowest rank
    assert results[0][3] == results[1][3] == 1.5 * WORLD


def test_record_split_is_additive(oracle):
    """Summing shard records equals the whole-batch record up to rounding (any split)."""
    from conftest import tol_close

    x, t, w = _data()
    whole = _shard_record(oracle, x, t, w)
    for cut in (1, 17, GLOBAL_BATCH // 2, GLOBAL_BATCH - 1):
        parts = _shard_record(oracle, x[:cut], t[:cut], w) + _shard_record(oracle, x[cut:], t[cut:], w)
        assert tol_close(parts, whole, 1e-12)


if __name__ == "__main__":
    pytest.main([__file__, "-q"])
