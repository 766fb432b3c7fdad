"""The oracle at full batch sizes, spread over a spawn-started process pool
(TEST INFRASTRUCTURE ONLY: the checker for the headline-shape parity tests).

The batch lives in shared memory (X, T and the residuals R, [B][2^n] float64).
Each worker runs the C restatement of the reference (oracle/liboracle.so) on
chunks of rows:

* ``residual_gram``: y = forward(x, w) with the reference's term-major loop
  (reference src/batch_gp.c:107-161, per sample, so chunking changes nothing),
  r = y - t written to R, the chunk's loss sum 0.5 sum r^2 and its Gram block
  X^T R (float64). The caller sums the chunks in extended precision, so the
  gradient g_p = sum_i sigma(i, p) (X^T R)[i][i ^ p] and the loss are accurate
  to about 1e-15 relative: far closer to the true sums than either the
  reference's sequential sum or the GPU's tree.
* ``sequential_vjp``: the reference's own summation, exactly
  (src/batch_gp.c:163-201): per plan term a sequential batch sum from 0 of
  x[s, in] * r[s, out] in sample order (workers take disjoint term ranges; the
  per-term sums are independent), then g[param] += sign * sum in term order.

The pool is started with `spawn` (never fork after CUDA is initialised); a
worker that dies makes the call raise instead of waiting.
"""
from __future__ import annotations

import multiprocessing as mp
import os
from concurrent.futures import ProcessPoolExecutor
from multiprocessing import shared_memory

import numpy as np

_W: dict = {}  # per-worker cache: shared-memory handles and the oracle


def _attach(names, shape):
    key = (tuple(names), tuple(shape))
    if _W.get("key") != key:
        for shm in _W.get("shms", []):
            shm.close()
        shms = [shared_memory.SharedMemory(name=n) for n in names]
        _W["shms"] = shms
        _W["arrays"] = [np.ndarray(shape, dtype=np.float64, buffer=s.buf) for s in shms]
        _W["key"] = key
    if "oracle" not in _W:
        from oracle.oracle import Oracle

        _W["oracle"] = Oracle()
    return _W["arrays"], _W["oracle"]


def _residual_gram_task(args):
    names, shape, sig, left, w, a, b, call = args
    (X, T, R), orc = _attach(names, shape)
    loss = np.longdouble(0)
    gram = np.zeros((shape[1],) * 2, dtype=np.longdouble)
    for c in range(a, b, call):  # the oracle's forward is fastest on short calls (its loop is term-major)
        x = np.ascontiguousarray(X[c:min(c + call, b)])
        st, y = orc.forward(sig, x, w, left)
        if st != 0:
            return st, None, None
        r = y - T[c:c + x.shape[0]]
        R[c:c + x.shape[0]] = r
        loss += np.sum((0.5 * r * r).astype(np.longdouble))
        gram += (x.T @ r).astype(np.longdouble)
    return 0, loss, gram


def _sequential_task(args):
    names, shape, in_b, out_b, chunk = args
    (X, _, R), _ = _attach(names, shape)
    acc = np.zeros(len(in_b))
    for a in range(0, shape[0], chunk):
        p = X[a:a + chunk][:, in_b] * R[a:a + chunk][:, out_b]
        p[0] += acc  # acc + p_0, then each later row added in sample order
        np.add.accumulate(p, axis=0, out=p)
        acc = p[-1].copy()
    return acc


class PooledOracle:
    """X, T, R in shared memory for `batch` rows of 2^n blades, and a spawn pool."""

    def __init__(self, batch: int, blades: int, workers: int | None = None):
        self.shape = (batch, blades)
        nbytes = batch * blades * 8
        self.shms = [shared_memory.SharedMemory(create=True, size=nbytes) for _ in range(3)]
        self.X, self.T, self.R = (np.ndarray(self.shape, dtype=np.float64, buffer=s.buf) for s in self.shms)
        self.workers = workers or os.cpu_count() or 1
        self.pool = ProcessPoolExecutor(self.workers, mp_context=mp.get_context("spawn"))

    @property
    def names(self):
        return [s.name for s in self.shms]

    def close(self):
        self.pool.shutdown()
        del self.X, self.T, self.R
        for s in self.shms:
            s.close()
            s.unlink()

    def residual_gram(self, sig, left: bool, w, task_rows: int = 16384, call_rows: int = 64):
        """(loss sum, X^T R) over the batch, both in extended precision; R filled.
        Per-chunk Gram blocks are X^T R of call_rows rows (float64)."""
        B = self.shape[0]
        task_rows = min(task_rows, max(call_rows, -(-B // self.workers)))
        tasks = [(self.names, self.shape, list(sig), bool(left), np.asarray(w, np.float64), a, min(a + task_rows, B),
                  call_rows) for a in range(0, B, task_rows)]
        loss = np.longdouble(0)
        gram = np.zeros((self.shape[1],) * 2, dtype=np.longdouble)
        for st, l, g in self.pool.map(_residual_gram_task, tasks):
            assert st == 0
            loss += l
            gram += g
        return loss, gram

    def sequential_vjp(self, oracle, sig, left: bool, chunk: int = 512) -> np.ndarray:
        """The reference's sequential per-term sums of x[s, in] r[s, out] over R, combined in term order."""
        N = self.shape[1]
        terms = [(l, r) for l in range(N) for r in range(N)]  # plan order: left-blade major
        in_b = np.array([r if left else l for l, r in terms])
        par_b = [l if left else r for l, r in terms]
        out_b = np.array([l ^ r for l, r in terms])
        sign = [oracle.sign(l, r, sig) for l, r in terms]
        bounds = np.linspace(0, len(terms), 4 * self.workers + 1).astype(int)
        tasks = [(self.names, self.shape, in_b[a:b], out_b[a:b], chunk) for a, b in zip(bounds[:-1], bounds[1:])
                 if b > a]
        acc = np.concatenate(list(self.pool.map(_sequential_task, tasks)))
        g = [0.0] * N
        for t in range(len(terms)):
            g[par_b[t]] += float(sign[t]) * float(acc[t])
        return np.array(g)


def gradient_from_gram(oracle, sig, left: bool, gram) -> np.ndarray:
    """g_p = sum_i sigma(i, p) G[i][i ^ p] in extended precision, rounded once."""
    N = gram.shape[0]
    g = np.zeros(N, dtype=np.longdouble)
    for p in range(N):
        for i in range(N):
            s = oracle.sign(p, i, sig) if left else oracle.sign(i, p, sig)
            g[p] += s * gram[i, i ^ p]
    return g.astype(np.float64)
