"""GPU parity of the general batched V8 path (any graph): geo_b200_v8_batch_train_step
on graphs that are not the fused GP->MSE pattern, and geo_b200_v8_batch_forward.

Checked against golden vectors made by the reference's own per-sample V8 loop
on the all-node-kinds graph (tests/golden/make_golden.py, v8cb_*), and against
the library's per-sample geo_v8_* loop (which the golden tests pin to the
reference), including a constrained parameter and the status rules."""
from __future__ import annotations

import ctypes
import pathlib

import numpy as np
import pytest

from geometricelementaryoperators_b200 import canonical_signature
from geometricelementaryoperators_b200.synthetic import normal, splitmix_uniform
from oracle.oracle import composed_graph, v8_mv_fill
from tests.conftest import max_violation, tol_close
from tests.gpu_helpers import TOL, dev
from tests.test_gpu_v8 import V8Program, _lib, mv, value

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "batch_gp_golden.npz"
CRMATH_GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "v8_crmath_golden.npz"
CASES = [(2, 0), (3, 1), (4, 0), (5, 2), (6, 0), (6, 3)]


def _values(n, q):
    return {"input": v8_mv_fill(n, 3 + n + q), "target": v8_mv_fill(n, 11 + 2 * n + q),
            "w1": v8_mv_fill(n, 19 + n + q), "w2": v8_mv_fill(n, 29 + n + q)}


def _composed(L, sig, values):
    prog = V8Program()
    ids = composed_graph(L, ctypes.byref(prog), sig, lambda c: mv(sig, c), values)
    return prog, ids


def _batch_step(L, prog, x_id, t_id, dx, dt, B, opt, lr=1e-2):
    loss = ctypes.c_double()
    st = L.geo_b200_v8_batch_train_step(ctypes.byref(prog), x_id, t_id, ctypes.c_void_p(dx.data_ptr()),
                                        ctypes.c_void_p(dt.data_ptr()) if dt is not None else None, B, opt, lr, 0.9,
                                        0.999, 1e-8, 1.0 / B, ctypes.byref(loss))
    return st, loss.value


def _loop_step(L, prog, x_id, t_id, xs, ts, sig, n, loss_id, opt, lr=1e-2):
    assert L.geo_v8_zero_grad(ctypes.byref(prog)) == 0
    total = 0.0
    B = xs.shape[0]
    for j in range(B):
        assert L.geo_v8_set_value(ctypes.byref(prog), x_id, ctypes.byref(mv(sig, xs[j]))) == 0
        if t_id is not None:
            assert L.geo_v8_set_value(ctypes.byref(prog), t_id, ctypes.byref(mv(sig, ts[j]))) == 0
        assert L.geo_v8_forward(ctypes.byref(prog)) == 0
        assert L.geo_v8_backward(ctypes.byref(prog), 1 if j else 0) == 0
        total += value(L, prog, loss_id, n)[0]
    assert L.geo_v8_optimizer_step(ctypes.byref(prog), opt, lr, 0.9, 0.999, 1e-8, 1.0 / B) == 0
    return total


# The graph's tanh and sigmoid are correctly rounded here (csrc/crmath.h); the
# reference calls the C library's, whose tanh misses the correctly rounded value
# on about one argument in eight (exp on a few in ten thousand). SGD steps keep
# those differences at the ulp level (checked at 1e-12), but Adam divides each
# update by the root of its second moment, which amplifies them on gradient
# components that nearly cancel over the batch: after three Adam steps the
# reference and this runtime agree to ~1.3e-11, exactly the distance between the
# reference built against the C library and the reference built against the
# correctly rounded functions (make_v8_crmath_golden.py), which this runtime
# meets at 1e-12 (test_general_batch_step_golden_crmath). The batched path
# itself is bit-identical to the per-sample runtime
# (test_general_batch_step_matches_loop_exact).
ADAM_TOL = 1e-10


@pytest.mark.parametrize("n,q", CASES)
def test_general_batch_step_golden(n, q):
    """All-node-kinds graph, 3 SGD and 3 Adam steps over 9 samples vs the reference's per-sample loop."""
    L = _lib()
    golden = np.load(GOLDEN)
    sig = canonical_signature(n, q)
    xs, ts = golden[f"v8cb_n{n}q{q}_x"], golden[f"v8cb_n{n}q{q}_t"]
    dx, dt = dev(xs), dev(ts)
    for opt in (1, 2):
        prog, ids = _composed(L, sig, _values(n, q))
        for k in range(3):
            st, loss = _batch_step(L, prog, ids["x"], ids["y"], dx, dt, xs.shape[0], opt)
            assert st == 0, st
            w1, w2 = value(L, prog, ids["p1"], n), value(L, prog, ids["p2"], n)
            g1 = golden[f"v8cb_n{n}q{q}_opt{opt}_w1"][k]
            g2 = golden[f"v8cb_n{n}q{q}_opt{opt}_w2"][k]
            tol = TOL if opt == 1 else ADAM_TOL
            assert tol_close(w1, g1, tol), (opt, k, max_violation(w1, g1, tol))
            assert tol_close(w2, g2, tol), (opt, k, max_violation(w2, g2, tol))
            assert tol_close(loss, golden[f"v8cb_n{n}q{q}_opt{opt}_loss"][k], TOL)
            assert prog.optimizer_step == k + 1
        L.geo_v8_program_free(ctypes.byref(prog))


@pytest.mark.parametrize("n,q", CASES)
def test_general_batch_step_golden_crmath(n, q):
    """The same graph and steps against the reference built with exp and tanh bound
    to the runtime's correctly rounded functions (tests/golden/make_v8_crmath_golden.py):
    with the nonlinearities rounded alike, SGD and Adam both meet the float64 bar."""
    L = _lib()
    golden = np.load(CRMATH_GOLDEN)
    sig = canonical_signature(n, q)
    xs, ts = golden[f"v8cb_n{n}q{q}_x"], golden[f"v8cb_n{n}q{q}_t"]
    dx, dt = dev(xs), dev(ts)
    for opt in (1, 2):
        prog, ids = _composed(L, sig, _values(n, q))
        for k in range(3):
            st, loss = _batch_step(L, prog, ids["x"], ids["y"], dx, dt, xs.shape[0], opt)
            assert st == 0, st
            w1, w2 = value(L, prog, ids["p1"], n), value(L, prog, ids["p2"], n)
            g1 = golden[f"v8cb_n{n}q{q}_opt{opt}_w1"][k]
            g2 = golden[f"v8cb_n{n}q{q}_opt{opt}_w2"][k]
            assert tol_close(w1, g1, TOL), (opt, k, max_violation(w1, g1, TOL))
            assert tol_close(w2, g2, TOL), (opt, k, max_violation(w2, g2, TOL))
            assert tol_close(loss, golden[f"v8cb_n{n}q{q}_opt{opt}_loss"][k], TOL)
        L.geo_v8_program_free(ctypes.byref(prog))


@pytest.mark.parametrize("n,q", [(3, 0), (6, 0), (6, 3)])
def test_general_batch_step_matches_loop_exact(n, q):
    """513 samples, one per warp: the batched step sums per-sample gradients in sample order,
    so parameters after two Adam steps equal the per-sample geo_v8_* loop bit for bit."""
    L = _lib()
    sig = canonical_signature(n, q)
    N = 1 << n
    B = 513
    xs = splitmix_uniform(201 + n + q, (B, N))
    ts = splitmix_uniform(202 + n + q, (B, N))
    loop, li = _composed(L, sig, _values(n, q))
    batched, bi = _composed(L, sig, _values(n, q))
    dx, dt = dev(xs), dev(ts)
    for _ in range(2):
        total = _loop_step(L, loop, li["x"], li["y"], xs, ts, sig, n, li["loss"], 2)
        st, loss = _batch_step(L, batched, bi["x"], bi["y"], dx, dt, B, 2)
        assert st == 0
        assert tol_close(loss, total, TOL)
        for key in ("p1", "p2"):
            assert np.array_equal(value(L, batched, bi[key], n), value(L, loop, li[key], n)), key
    L.geo_v8_program_free(ctypes.byref(loop))
    L.geo_v8_program_free(ctypes.byref(batched))


@pytest.mark.parametrize("opt", [1, 2])
def test_general_batch_step_many_samples_per_warp(opt):
    """5000 samples (several per warp, summed per warp then in warp order) vs the per-sample loop."""
    L = _lib()
    n, q = 4, 2
    sig = canonical_signature(n, q)
    N = 1 << n
    B = 5000
    xs = splitmix_uniform(211, (B, N))
    ts = splitmix_uniform(212, (B, N))
    loop, li = _composed(L, sig, _values(n, q))
    batched, bi = _composed(L, sig, _values(n, q))
    total = _loop_step(L, loop, li["x"], li["y"], xs, ts, sig, n, li["loss"], opt)
    st, loss = _batch_step(L, batched, bi["x"], bi["y"], dev(xs), dev(ts), B, opt)
    assert st == 0
    assert tol_close(loss, total, TOL)
    tol = TOL if opt == 1 else ADAM_TOL
    for key in ("p1", "p2"):
        a, b = value(L, batched, bi[key], n), value(L, loop, li[key], n)
        assert tol_close(a, b, tol), (key, max_violation(a, b, tol))
    L.geo_v8_program_free(ctypes.byref(loop))
    L.geo_v8_program_free(ctypes.byref(batched))


@pytest.mark.parametrize("n,q", [(3, 1), (6, 0)])
def test_batch_forward_is_the_per_sample_forward(n, q):
    """geo_b200_v8_batch_forward gives bit-identical node values to per-sample geo_v8_forward."""
    import torch

    L = _lib()
    sig = canonical_signature(n, q)
    N = 1 << n
    B = 300
    xs = splitmix_uniform(301 + n, (B, N))
    prog, ids = _composed(L, sig, _values(n, q))
    out = torch.zeros((B, N), dtype=torch.float64, device="cuda")
    for node in ("norm", "loss"):
        st = L.geo_b200_v8_batch_forward(ctypes.byref(prog), ids["x"], ctypes.c_void_p(dev(xs).data_ptr()), B,
                                         ids[node], ctypes.c_void_p(out.data_ptr()))
        assert st == 0
        got = out.cpu().numpy()
        for j in (0, 1, 77, B - 1):
            assert L.geo_v8_set_value(ctypes.byref(prog), ids["x"], ctypes.byref(mv(sig, xs[j]))) == 0
            assert L.geo_v8_forward(ctypes.byref(prog)) == 0
            assert np.array_equal(got[j], value(L, prog, ids[node], n)), (node, j)
    L.geo_v8_program_free(ctypes.byref(prog))


def test_batch_forward_golden_loss():
    """The batched forward of the all-node-kinds graph reproduces the reference's loss (golden v8c)."""
    import torch

    L = _lib()
    golden = np.load(GOLDEN)
    for n, q in CASES:
        sig = canonical_signature(n, q)
        values = _values(n, q)
        prog, ids = _composed(L, sig, values)
        xs = np.tile(values["input"], (5, 1))
        out = torch.zeros((5, 1 << n), dtype=torch.float64, device="cuda")
        assert L.geo_b200_v8_batch_forward(ctypes.byref(prog), ids["x"], ctypes.c_void_p(dev(xs).data_ptr()), 5,
                                           ids["loss"], ctypes.c_void_p(out.data_ptr())) == 0
        got = out.cpu().numpy()[:, 0]
        assert tol_close(got, np.full(5, golden[f"v8c_n{n}q{q}_loss"][0]), TOL)
        L.geo_v8_program_free(ctypes.byref(prog))


def _constrained_program(L, sig, w0, constraint):
    """tanh(x * w) -> add(., scale(t, -1)) -> squared_norm with a constrained parameter w."""
    n = len(sig)
    prog = V8Program()
    ids = {k: ctypes.c_uint32() for k in ("x", "t", "w", "gp", "act", "neg", "res", "loss")}
    zero = mv(sig)
    assert L.geo_v8_program_init(ctypes.byref(prog), n, (ctypes.c_int8 * 6)(*sig, *([0] * (6 - n))), 1, 4) == 0
    assert L.geo_v8_add_leaf(ctypes.byref(prog), 1, b"x", ctypes.byref(zero), 0, 0, ctypes.byref(ids["x"])) == 0
    assert L.geo_v8_add_leaf(ctypes.byref(prog), 2, b"t", ctypes.byref(zero), 0, 0, ctypes.byref(ids["t"])) == 0
    assert L.geo_v8_add_leaf(ctypes.byref(prog), 3, b"w", ctypes.byref(mv(sig, w0)), 1, constraint,
                             ctypes.byref(ids["w"])) == 0
    assert L.geo_v8_add_binary(ctypes.byref(prog), 8, b"gp", ids["x"], ids["w"], ctypes.byref(ids["gp"])) == 0
    assert L.geo_v8_add_unary(ctypes.byref(prog), 14, b"act", ids["gp"], 0.0, 0, ctypes.byref(ids["act"])) == 0
    assert L.geo_v8_add_unary(ctypes.byref(prog), 7, b"neg", ids["t"], -1.0, 0, ctypes.byref(ids["neg"])) == 0
    assert L.geo_v8_add_binary(ctypes.byref(prog), 6, b"res", ids["act"], ids["neg"], ctypes.byref(ids["res"])) == 0
    assert L.geo_v8_add_unary(ctypes.byref(prog), 17, b"loss", ids["res"], 0.0, 0, ctypes.byref(ids["loss"])) == 0
    assert L.geo_v8_compile(ctypes.byref(prog), ids["loss"]) == 0
    return prog, ids


def test_constrained_parameter_and_status_rules():
    """UNIT_EUCLIDEAN parameter through the general path; non-finite rows are rejected with no update."""
    L = _lib()
    n, q = 4, 1
    sig = canonical_signature(n, q)
    N = 1 << n
    B = 101
    w0 = normal(401, (N,), 1.0)
    w0 = w0 / np.sqrt(np.sum(w0 * w0))
    xs = splitmix_uniform(402, (B, N))
    ts = splitmix_uniform(403, (B, N))
    loop, li = _constrained_program(L, sig, w0, 1)
    batched, bi = _constrained_program(L, sig, w0, 1)
    dx, dt = dev(xs), dev(ts)
    for _ in range(3):
        total = _loop_step(L, loop, li["x"], li["t"], xs, ts, sig, n, li["loss"], 2, lr=5e-2)
        st, loss = _batch_step(L, batched, bi["x"], bi["t"], dx, dt, B, 2, lr=5e-2)
        assert st == 0
        assert tol_close(loss, total, TOL)
        a, b = value(L, batched, bi["w"], n), value(L, loop, li["w"], n)
        assert tol_close(a, b, TOL), max_violation(a, b, TOL)
        assert abs(np.sum(a * a) - 1.0) < 1e-12
    before = value(L, batched, bi["w"], n)
    bad = xs.copy()
    bad[57, 3] = np.nan
    st, _ = _batch_step(L, batched, bi["x"], bi["t"], dev(bad), dt, B, 2)
    assert st == 1  # GEO_V8_INVALID_ARGUMENT, as geo_v8_set_value would answer
    assert np.array_equal(value(L, batched, bi["w"], n), before)
    assert batched.optimizer_step == 3
    # a huge target row overflows the loss (0.5 r^2 = inf): numeric failure, no update
    huge = ts.copy()
    huge[5] = 1e200
    st, _ = _batch_step(L, batched, bi["x"], bi["t"], dx, dev(huge), B, 2)
    assert st == 11  # GEO_V8_NUMERIC_FAILURE
    assert np.array_equal(value(L, batched, bi["w"], n), before)
    L.geo_v8_program_free(ctypes.byref(loop))
    L.geo_v8_program_free(ctypes.byref(batched))


def test_package_graph_builder_matches_reference_test_graph():
    """geometricelementaryoperators_b200.v8.all_node_kinds_graph builds the reference test's graph:
    same batched losses and one training step as the graph built node by node."""
    import torch

    from geometricelementaryoperators_b200 import v8

    L = _lib()
    n, q = 5, 1
    sig = canonical_signature(n, q)
    values = _values(n, q)
    ref_prog, rids = _composed(L, sig, values)
    prog, ids = v8.all_node_kinds_graph(sig, values["w1"], values["w2"], values["input"], values["target"])
    B = 64
    xs = splitmix_uniform(601, (B, 1 << n))
    ts = splitmix_uniform(602, (B, 1 << n))
    dx, dt = dev(xs), dev(ts)
    a = torch.zeros((B, 1 << n), dtype=torch.float64, device="cuda")
    b = torch.zeros_like(a)
    prog.batch_forward(ids["x"], dx.data_ptr(), B, ids["loss"], a.data_ptr())
    assert L.geo_b200_v8_batch_forward(ctypes.byref(ref_prog), rids["x"], ctypes.c_void_p(dx.data_ptr()), B,
                                       rids["loss"], ctypes.c_void_p(b.data_ptr())) == 0
    assert torch.equal(a, b)
    loss = prog.batch_train_step(ids["x"], ids["y"], dx.data_ptr(), dt.data_ptr(), B, v8.ADAM, 1e-2)
    st, ref_loss = _batch_step(L, ref_prog, rids["x"], rids["y"], dx, dt, B, 2)
    assert st == 0 and loss == ref_loss
    assert np.array_equal(prog.value(ids["w1"]), value(L, ref_prog, rids["p1"], n))
    prog.free()
    L.geo_v8_program_free(ctypes.byref(ref_prog))
