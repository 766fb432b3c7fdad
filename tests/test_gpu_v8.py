"""GPU parity of the V8 graph runtime (geo_v8_*): the per-sample interpreter
kernels and the batched GP->MSE path, against golden vectors made by the
reference's own V8 runtime and against the reference test's properties
(tests/test_full_cycle_v8.c)."""
from __future__ import annotations

import ctypes
import pathlib

import numpy as np
import pytest

from geometricelementaryoperators_b200 import abi, canonical_signature
from geometricelementaryoperators_b200.synthetic import normal, splitmix_uniform
from oracle.oracle import MvF64, composed_graph, v8_mv_fill
from tests.conftest import all_signatures, max_violation, tol_close
from tests.gpu_helpers import TOL, dev

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "batch_gp_golden.npz"


class V8Program(ctypes.Structure):
    """geo_v8_program_t (reference include/geo/full_cycle_v8.h:89-104)."""

    _fields_ = [("abi_version", ctypes.c_uint32), ("dimension", ctypes.c_uint8), ("signature", ctypes.c_int8 * 6),
                ("pairing", ctypes.c_uint8), ("compiled", ctypes.c_uint8), ("forward_valid", ctypes.c_uint8),
                ("backward_valid", ctypes.c_uint8), ("reserved", ctypes.c_uint8), ("node_count", ctypes.c_uint32),
                ("node_capacity", ctypes.c_uint32), ("loss_node", ctypes.c_uint32),
                ("optimizer_step", ctypes.c_uint64), ("gradient_samples", ctypes.c_uint64),
                ("nodes", ctypes.c_void_p)]


def _lib():
    L = abi.lib()
    M = ctypes.POINTER(MvF64)
    P = ctypes.POINTER(V8Program)
    U32 = ctypes.c_uint32
    U32P = ctypes.POINTER(U32)
    L.geo_v8_program_init.argtypes = [P, ctypes.c_uint8, ctypes.POINTER(ctypes.c_int8), ctypes.c_int, ctypes.c_size_t]
    L.geo_v8_program_free.argtypes = [P]
    L.geo_v8_add_leaf.argtypes = [P, ctypes.c_int, ctypes.c_char_p, M, ctypes.c_int, ctypes.c_int, U32P]
    L.geo_v8_add_unary.argtypes = [P, ctypes.c_int, ctypes.c_char_p, U32, ctypes.c_double, ctypes.c_uint8, U32P]
    L.geo_v8_add_binary.argtypes = [P, ctypes.c_int, ctypes.c_char_p, U32, U32, U32P]
    L.geo_v8_bind_state_update.argtypes = [P, U32, U32]
    L.geo_v8_compile.argtypes = [P, U32]
    L.geo_v8_find_node.argtypes = [P, ctypes.c_char_p]
    L.geo_v8_find_node.restype = U32
    L.geo_v8_set_value.argtypes = [P, U32, M]
    L.geo_v8_forward.argtypes = [P]
    L.geo_v8_zero_grad.argtypes = [P]
    L.geo_v8_backward.argtypes = [P, ctypes.c_int]
    L.geo_v8_optimizer_step.argtypes = [P, ctypes.c_int] + [ctypes.c_double] * 5
    L.geo_v8_commit_states.argtypes = [P]
    L.geo_v8_value.argtypes = [P, U32]
    L.geo_v8_value.restype = M
    L.geo_v8_gradient.argtypes = [P, U32]
    L.geo_v8_gradient.restype = M
    return L


def mv(sig, coeffs=None):
    m = MvF64()
    m.dimension = len(sig)
    for i, s in enumerate(sig):
        m.signature[i] = int(s)
    if coeffs is not None:
        for i, v in enumerate(np.asarray(coeffs, np.float64)):
            m.coefficients[i] = float(v)
    return m


def value(L, prog, node, n):
    return np.array(L.geo_v8_value(ctypes.byref(prog), node).contents.coefficients[: 1 << n])


def gradient(L, prog, node, n):
    return np.array(L.geo_v8_gradient(ctypes.byref(prog), node).contents.coefficients[: 1 << n])


def composed(L, sig):
    n = len(sig)
    q = sum(1 for s in sig if s < 0)
    values = {"input": v8_mv_fill(n, 3 + n + q), "target": v8_mv_fill(n, 11 + 2 * n + q),
              "w1": v8_mv_fill(n, 19 + n + q), "w2": v8_mv_fill(n, 29 + n + q)}
    prog = V8Program()
    ids = composed_graph(L, ctypes.byref(prog), sig, lambda c: mv(sig, c), values)
    return prog, ids, values


def test_composed_graph_golden_all_signatures():
    """All 17 node kinds, all 27 signatures: loss and both gradients vs the reference."""
    L = _lib()
    golden = np.load(GOLDEN)
    for n, q, sig in all_signatures():
        prog, ids, _ = composed(L, sig)
        assert L.geo_v8_forward(ctypes.byref(prog)) == 0
        assert L.geo_v8_backward(ctypes.byref(prog), 0) == 0
        loss = value(L, prog, ids["loss"], n)[0]
        assert tol_close(loss, golden[f"v8c_n{n}q{q}_loss"][0], TOL)
        g1, g2 = gradient(L, prog, ids["p1"], n), gradient(L, prog, ids["p2"], n)
        assert tol_close(g1, golden[f"v8c_n{n}q{q}_g1"], TOL), (n, q, max_violation(g1, golden[f"v8c_n{n}q{q}_g1"], TOL))
        assert tol_close(g2, golden[f"v8c_n{n}q{q}_g2"], TOL)
        L.geo_v8_program_free(ctypes.byref(prog))


def test_composed_graph_finite_differences():
    """Central differences along a direction agree with the analytic gradient at 3e-5
    (reference tests/test_full_cycle_v8.c:183-210)."""
    L = _lib()
    eps = 1e-6
    for n, q, sig in all_signatures():
        prog, ids, values = composed(L, sig)
        assert L.geo_v8_forward(ctypes.byref(prog)) == 0
        assert L.geo_v8_backward(ctypes.byref(prog), 0) == 0
        for pname, wname, dseed in (("p1", "w1", 37), ("p2", "w2", 43)):
            g = gradient(L, prog, ids[pname], n)
            direction = v8_mv_fill(n, dseed + n + q)
            losses = []
            for sgn in (1.0, -1.0):
                assert L.geo_v8_set_value(ctypes.byref(prog), ids[pname],
                                          ctypes.byref(mv(sig, values[wname] + sgn * eps * direction))) == 0
                assert L.geo_v8_forward(ctypes.byref(prog)) == 0
                losses.append(value(L, prog, ids["loss"], n)[0])
            numeric = (losses[0] - losses[1]) / (2 * eps)
            analytic = float(np.dot(g, direction))
            assert abs(numeric - analytic) <= 3e-5 * (1 + abs(numeric) + abs(analytic)), (n, q, pname)
            assert L.geo_v8_set_value(ctypes.byref(prog), ids[pname], ctypes.byref(mv(sig, values[wname]))) == 0
            assert L.geo_v8_forward(ctypes.byref(prog)) == 0
            assert L.geo_v8_backward(ctypes.byref(prog), 0) == 0
        L.geo_v8_program_free(ctypes.byref(prog))


def gp_mse_program(L, sig, left=False, w0=None):
    n = len(sig)
    prog = V8Program()
    ids = {k: ctypes.c_uint32() for k in ("x", "t", "w", "pred", "neg", "res", "loss")}
    zero = mv(sig)
    assert L.geo_v8_program_init(ctypes.byref(prog), n, abi.sig_array(sig), 1, 8) == 0
    assert L.geo_v8_add_leaf(ctypes.byref(prog), 1, b"x", ctypes.byref(zero), 0, 0, ctypes.byref(ids["x"])) == 0
    assert L.geo_v8_add_leaf(ctypes.byref(prog), 2, b"y", ctypes.byref(zero), 0, 0, ctypes.byref(ids["t"])) == 0
    w = mv(sig, w0) if w0 is not None else zero
    assert L.geo_v8_add_leaf(ctypes.byref(prog), 3, b"w", ctypes.byref(w), 1, 0, ctypes.byref(ids["w"])) == 0
    a, b = (ids["w"], ids["x"]) if left else (ids["x"], ids["w"])
    assert L.geo_v8_add_binary(ctypes.byref(prog), 8, b"pred", a, b, ctypes.byref(ids["pred"])) == 0
    assert L.geo_v8_add_unary(ctypes.byref(prog), 7, b"neg_y", ids["t"], -1.0, 0, ctypes.byref(ids["neg"])) == 0
    assert L.geo_v8_add_binary(ctypes.byref(prog), 6, b"residual", ids["pred"], ids["neg"],
                               ctypes.byref(ids["res"])) == 0
    assert L.geo_v8_add_unary(ctypes.byref(prog), 17, b"loss", ids["res"], 0.0, 0, ctypes.byref(ids["loss"])) == 0
    assert L.geo_v8_compile(ctypes.byref(prog), ids["loss"]) == 0
    return prog, ids


def test_batch_accumulation_exact():
    """backward(accumulate) sums per-sample gradients (reference tests/test_full_cycle_v8.c:254-295)."""
    L = _lib()
    sig = [1, 1]
    prog, ids = gp_mse_program(L, sig)
    x1, x2, y1, y2 = (v8_mv_fill(2, s) for s in (3, 5, 7, 11))

    def sample(x, y, acc):
        assert L.geo_v8_set_value(ctypes.byref(prog), ids["x"], ctypes.byref(mv(sig, x))) == 0
        assert L.geo_v8_set_value(ctypes.byref(prog), ids["t"], ctypes.byref(mv(sig, y))) == 0
        assert L.geo_v8_forward(ctypes.byref(prog)) == 0
        assert L.geo_v8_backward(ctypes.byref(prog), acc) == 0

    sample(x1, y1, 0)
    g1 = gradient(L, prog, ids["w"], 2)
    sample(x2, y2, 0)
    g2 = gradient(L, prog, ids["w"], 2)
    sample(x1, y1, 0)
    sample(x2, y2, 1)
    assert tol_close(gradient(L, prog, ids["w"], 2), g1 + g2, 1e-12)
    assert prog.gradient_samples == 2
    assert L.geo_v8_optimizer_step(ctypes.byref(prog), 1, 0.01, 0.9, 0.999, 1e-8, 0.5) == 0
    assert prog.gradient_samples == 0 and prog.optimizer_step == 1
    L.geo_v8_program_free(ctypes.byref(prog))


def test_dynamic_graph_602_nodes():
    L = _lib()
    sig = [1]
    prog = V8Program()
    root = ctypes.c_uint32()
    assert L.geo_v8_program_init(ctypes.byref(prog), 1, abi.sig_array(sig), 1, 1) == 0
    assert L.geo_v8_add_leaf(ctypes.byref(prog), 1, b"root", ctypes.byref(mv(sig, [0.25, -0.5])), 1, 0,
                             ctypes.byref(root)) == 0
    cur = root.value
    for i in range(600):
        nxt = ctypes.c_uint32()
        assert L.geo_v8_add_unary(ctypes.byref(prog), 7, f"scale_{i}".encode(), cur, 0.999, 0, ctypes.byref(nxt)) == 0
        cur = nxt.value
    loss = ctypes.c_uint32()
    assert L.geo_v8_add_unary(ctypes.byref(prog), 17, b"large_loss", cur, 0.0, 0, ctypes.byref(loss)) == 0
    assert prog.node_count == 602 and prog.node_capacity >= 602
    assert L.geo_v8_compile(ctypes.byref(prog), loss) == 0
    assert L.geo_v8_forward(ctypes.byref(prog)) == 0
    assert L.geo_v8_backward(ctypes.byref(prog), 0) == 0
    g = gradient(L, prog, root.value, 1)
    # d/dx 0.5 |0.999^600 x|^2 = 0.999^1200 x (repeated products, 1e-12)
    f = 0.999 ** 1200
    assert tol_close(g, [0.25 * f, -0.5 * f], 1e-12)
    assert L.geo_v8_find_node(ctypes.byref(prog), b"scale_599") == cur
    L.geo_v8_program_free(ctypes.byref(prog))


def test_stateful_recurrence_and_adam():
    L = _lib()
    sig = [1, 1]
    prog = V8Program()
    ids = {k: ctypes.c_uint32() for k in ("x", "y", "s", "w", "tr", "pre", "nxt", "neg", "res", "loss")}
    P = ctypes.byref(prog)
    assert L.geo_v8_program_init(P, 2, abi.sig_array(sig), 1, 16) == 0
    assert L.geo_v8_add_leaf(P, 1, b"x", ctypes.byref(mv(sig, v8_mv_fill(2, 3))), 0, 0, ctypes.byref(ids["x"])) == 0
    assert L.geo_v8_add_leaf(P, 2, b"target", ctypes.byref(mv(sig, v8_mv_fill(2, 5))), 0, 0,
                             ctypes.byref(ids["y"])) == 0
    assert L.geo_v8_add_leaf(P, 5, b"memory", ctypes.byref(mv(sig)), 0, 0, ctypes.byref(ids["s"])) == 0
    assert L.geo_v8_add_leaf(P, 3, b"weight", ctypes.byref(mv(sig, v8_mv_fill(2, 7))), 1, 0,
                             ctypes.byref(ids["w"])) == 0
    assert L.geo_v8_add_binary(P, 8, b"transformed", ids["x"], ids["w"], ctypes.byref(ids["tr"])) == 0
    assert L.geo_v8_add_binary(P, 6, b"preactivation", ids["tr"], ids["s"], ctypes.byref(ids["pre"])) == 0
    assert L.geo_v8_add_unary(P, 14, b"next_memory", ids["pre"], 0.0, 0, ctypes.byref(ids["nxt"])) == 0
    assert L.geo_v8_add_unary(P, 7, b"negative_target", ids["y"], -1.0, 0, ctypes.byref(ids["neg"])) == 0
    assert L.geo_v8_add_binary(P, 6, b"residual", ids["nxt"], ids["neg"], ctypes.byref(ids["res"])) == 0
    assert L.geo_v8_add_unary(P, 17, b"loss", ids["res"], 0.0, 0, ctypes.byref(ids["loss"])) == 0
    assert L.geo_v8_bind_state_update(P, ids["s"], ids["nxt"]) == 0
    assert L.geo_v8_compile(P, ids["loss"]) == 0
    before = value(L, prog, ids["s"], 2)
    assert L.geo_v8_forward(P) == 0
    assert L.geo_v8_backward(P, 0) == 0
    assert L.geo_v8_commit_states(P) == 0
    after = value(L, prog, ids["s"], 2)
    assert not np.isclose(np.dot(before, before), np.dot(after, after))
    assert np.array_equal(after, value(L, prog, ids["nxt"], 2))  # committed from next_memory
    assert L.geo_v8_commit_states(P) == 8  # forward required again
    assert L.geo_v8_optimizer_step(P, 2, 0.01, 0.9, 0.999, 1e-8, 1.0) == 0
    L.geo_v8_program_free(P)


def test_constraints_and_transactionality():
    """Unit-Euclidean, unit-vector-metric and even-versor projections; a failing
    constraint leaves the parameter unchanged (reference tests/test_full_cycle_v8.c:370-440)."""
    L = _lib()
    sig = [1, 1]
    prog = V8Program()
    P = ctypes.byref(prog)
    ids = {k: ctypes.c_uint32() for k in ("p1", "p2", "p3", "z1", "z2", "z3", "a1", "a2", "loss")}
    assert L.geo_v8_program_init(P, 2, abi.sig_array(sig), 1, 16) == 0
    assert L.geo_v8_add_leaf(P, 3, b"unit", ctypes.byref(mv(sig, [3.0, 4.0, 0, 0])), 1, 1, ctypes.byref(ids["p1"])) == 0
    assert L.geo_v8_add_leaf(P, 3, b"vector", ctypes.byref(mv(sig, [0, 2.0, 1.0, 0])), 1, 2,
                             ctypes.byref(ids["p2"])) == 0
    assert L.geo_v8_add_leaf(P, 3, b"versor", ctypes.byref(mv(sig, [2.0, 0, 0, 0])), 1, 3,
                             ctypes.byref(ids["p3"])) == 0
    for zn, src in (("z1", "p1"), ("z2", "p2"), ("z3", "p3")):
        assert L.geo_v8_add_unary(P, 7, zn.replace("z", "zero").encode(), ids[src], 0.0, 0, ctypes.byref(ids[zn])) == 0
    assert L.geo_v8_add_binary(P, 6, b"sum1", ids["z1"], ids["z2"], ctypes.byref(ids["a1"])) == 0
    assert L.geo_v8_add_binary(P, 6, b"sum2", ids["a1"], ids["z3"], ctypes.byref(ids["a2"])) == 0
    assert L.geo_v8_add_unary(P, 17, b"constraint_loss", ids["a2"], 0.0, 0, ctypes.byref(ids["loss"])) == 0
    assert L.geo_v8_compile(P, ids["loss"]) == 0
    assert L.geo_v8_forward(P) == 0
    assert L.geo_v8_backward(P, 0) == 0
    assert L.geo_v8_optimizer_step(P, 1, 0.1, 0.9, 0.999, 1e-8, 1.0) == 0
    p1 = value(L, prog, ids["p1"], 2)
    p2 = value(L, prog, ids["p2"], 2)
    p3 = value(L, prog, ids["p3"], 2)
    assert abs(np.dot(p1, p1) - 1.0) <= 1e-12 * 3
    assert abs(p2[1] ** 2 + p2[2] ** 2 - 1.0) <= 1e-12 * 3
    assert abs(abs(p3[0]) - 1.0) <= 1e-12 * 3
    L.geo_v8_program_free(P)

    bad = V8Program()
    B = ctypes.byref(bad)
    pid, sid, lid = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
    assert L.geo_v8_program_init(B, 2, abi.sig_array(sig), 1, 4) == 0
    assert L.geo_v8_add_leaf(B, 3, b"null_vector", ctypes.byref(mv(sig)), 1, 2, ctypes.byref(pid)) == 0
    assert L.geo_v8_add_unary(B, 7, b"zero", pid, 0.0, 0, ctypes.byref(sid)) == 0
    assert L.geo_v8_add_unary(B, 17, b"loss", sid, 0.0, 0, ctypes.byref(lid)) == 0
    assert L.geo_v8_compile(B, lid) == 0
    assert L.geo_v8_forward(B) == 0
    assert L.geo_v8_backward(B, 0) == 0
    preserved = value(L, bad, pid.value, 2)
    assert L.geo_v8_optimizer_step(B, 1, 0.1, 0.9, 0.999, 1e-8, 1.0) == 12
    assert np.array_equal(preserved, value(L, bad, pid.value, 2))
    L.geo_v8_program_free(B)


def test_status_rules():
    L = _lib()
    sig = [1, -1]
    prog = V8Program()
    P = ctypes.byref(prog)
    a, b = ctypes.c_uint32(), ctypes.c_uint32()
    assert L.geo_v8_program_init(P, 7, abi.sig_array([1] * 6), 1, 0) == 2
    assert L.geo_v8_program_init(P, 2, abi.sig_array(sig), 1, 4) == 0
    assert L.geo_v8_add_leaf(P, 1, b"x", ctypes.byref(mv(sig, [1, 2, 3, 4])), 0, 0, ctypes.byref(a)) == 0
    assert L.geo_v8_add_leaf(P, 1, b"x", ctypes.byref(mv(sig)), 0, 0, ctypes.byref(b)) == 6  # duplicate name
    assert L.geo_v8_add_leaf(P, 1, b"c", ctypes.byref(mv(sig)), 0, 1, ctypes.byref(b)) == 1   # constraint on input
    assert L.geo_v8_forward(P) == 7  # not compiled
    assert L.geo_v8_add_unary(P, 17, b"loss", a, 0.0, 0, ctypes.byref(b)) == 0
    assert L.geo_v8_compile(P, b) == 0
    assert L.geo_v8_backward(P, 0) == 8  # forward required
    assert L.geo_v8_add_unary(P, 7, b"late", a, 1.0, 0, ctypes.byref(b)) == 4  # compiled programs are closed
    bad = mv(sig, [1, float("nan"), 0, 0])
    assert L.geo_v8_set_value(P, a, ctypes.byref(bad)) == 1
    assert L.geo_v8_optimizer_step(P, 2, 0.1, 0.9, 0.999, 1e-8, 1.0) == 9  # backward required
    L.geo_v8_program_free(P)


@pytest.mark.parametrize("n,q,left", [(3, 0, True), (4, 1, False), (5, 1, True), (6, 0, False), (6, 3, True)])
def test_batched_step_matches_per_sample_loop(n, q, left):
    """geo_b200_v8_batch_train_step == zero_grad + per-sample forward/backward + optimizer_step."""
    L = _lib()
    sig = canonical_signature(n, q)
    N = 1 << n
    B = 37
    x = splitmix_uniform(61 + n, (B, N))
    t = splitmix_uniform(62 + n, (B, N))
    w0 = normal(63 + n, (N,), 0.2)
    loop, li = gp_mse_program(L, sig, left, w0)
    batched, bi = gp_mse_program(L, sig, left, w0)
    dx, dt = dev(x), dev(t)
    for step in range(3):
        assert L.geo_v8_zero_grad(ctypes.byref(loop)) == 0
        total = 0.0
        for j in range(B):
            assert L.geo_v8_set_value(ctypes.byref(loop), li["x"], ctypes.byref(mv(sig, x[j]))) == 0
            assert L.geo_v8_set_value(ctypes.byref(loop), li["t"], ctypes.byref(mv(sig, t[j]))) == 0
            assert L.geo_v8_forward(ctypes.byref(loop)) == 0
            assert L.geo_v8_backward(ctypes.byref(loop), 1 if j else 0) == 0
            total += value(L, loop, li["loss"], n)[0]
        assert L.geo_v8_optimizer_step(ctypes.byref(loop), 2, 1e-2, 0.9, 0.999, 1e-8, 1.0 / B) == 0
        loss = ctypes.c_double()
        st = L.geo_b200_v8_batch_train_step(ctypes.byref(batched), bi["x"], bi["t"], ctypes.c_void_p(dx.data_ptr()),
                                            ctypes.c_void_p(dt.data_ptr()), B, 2, 1e-2, 0.9, 0.999, 1e-8, 1.0 / B,
                                            ctypes.byref(loss))
        assert st == 0
        assert tol_close(loss.value, total, TOL)
        w_loop = value(L, loop, li["w"], n)
        w_batch = value(L, batched, bi["w"], n)
        assert tol_close(w_batch, w_loop, TOL), (step, max_violation(w_batch, w_loop, TOL))
        assert batched.optimizer_step == loop.optimizer_step == step + 1
    # a graph with a second parameter is not the GP->MSE pattern
    L.geo_v8_program_free(ctypes.byref(loop))
    L.geo_v8_program_free(ctypes.byref(batched))


def test_batched_step_golden_v8():
    """The batched path against the reference's own per-sample V8 loop (golden)."""
    L = _lib()
    golden = np.load(GOLDEN)
    for n, q in [(2, 0), (3, 0), (4, 1), (5, 1), (6, 0), (6, 3)]:
        sig = canonical_signature(n, q)
        xs, ts, w0 = golden[f"v8_n{n}q{q}_x"], golden[f"v8_n{n}q{q}_t"], golden[f"v8_n{n}q{q}_w0"]
        dx, dt = dev(xs), dev(ts)
        for opt in (1, 2):
            for side, left in (("R", False), ("L", True)):
                prog, ids = gp_mse_program(L, sig, left, w0)
                want = golden[f"v8_n{n}q{q}{side}_opt{opt}_w"]
                for k in range(3):
                    assert L.geo_b200_v8_batch_train_step(ctypes.byref(prog), ids["x"], ids["t"],
                                                         ctypes.c_void_p(dx.data_ptr()),
                                                         ctypes.c_void_p(dt.data_ptr()), 3, opt, 1e-2, 0.9, 0.999,
                                                         1e-8, 1.0 / 3, None) == 0
                    assert tol_close(value(L, prog, ids["w"], n), want[k], TOL), (n, q, side, opt, k)
                L.geo_v8_program_free(ctypes.byref(prog))
