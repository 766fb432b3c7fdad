"""ctypes access to the CPU checker (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs import this module. It loads:

* ``oracle/liboracle.so`` -- this project's C restatement of the reference CPU
  path (oracle/geo_oracle.c), and
* ``oracle/_ref/libgeo_ref.so`` -- the reference's own src/batch_gp.c,
  src/operator_kernel.c and src/full_cycle_v8.c compiled unmodified by
  ``make -C oracle ref`` (present only where the reference tree was available
  at build time; the built file travels with the repository snapshot).
"""
from __future__ import annotations

import ctypes
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libgeo_ref.so"
PLAN_BYTES = 16400

_P = ctypes.c_void_p
_D = ctypes.c_double
_SZ = ctypes.c_size_t
_I = ctypes.c_int
_U8 = ctypes.c_uint8
_I8P = ctypes.POINTER(ctypes.c_int8)


def build_oracle() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(_P)


def sig_array(signature) -> ctypes.Array:
    arr = (ctypes.c_int8 * 6)()
    for i, v in enumerate(signature):
        arr[i] = int(v)
    return arr


class Oracle:
    """This project's C restatement of the reference CPU algorithm."""

    def __init__(self, path: pathlib.Path = ORACLE_SO):
        if not path.exists():
            build_oracle()
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        L.orc_gp_sign.argtypes = [_U8, _U8, _I8P, _U8]
        L.orc_batch_plan_init.argtypes = [_P, _U8, _I8P]
        L.orc_batch_forward.argtypes = [_P, _P, _SZ, _P, _I, _P]
        L.orc_batch_vjp.argtypes = [_P, _P, _P, _SZ, _I, _P]
        L.orc_batch_mse_sgd_step.argtypes = [_P, _P, _P, _SZ, _D, _I, _P, _P]
        L.orc_gp_f64.argtypes = [_U8, _I8P, _P, _P, _P]
        L.orc_gp_f64_jvp.argtypes = [_U8, _I8P, _P, _P, _P, _P, _P]
        L.orc_gp_f64_vjp.argtypes = [_U8, _I8P, _P, _P, _P, _P, _P]
        L.orc_sparse_apply.argtypes = [_U8, _I8P, _I, _P, _P, _SZ, _P, _P]
        L.orc_sparse_apply_parametric.argtypes = [_U8, _I8P, _I, _P, _P, _SZ, _P, _P]
        L.orc_sparse_apply_vjp.argtypes = [_U8, _I8P, _I, _P, _P, _SZ, _P, _P]
        L.orc_sparse_apply_parametric_vjp.argtypes = [_U8, _I8P, _I, _P, _P, _SZ, _P, _P, _P, _P]
        L.orc_v8_optimizer_update.argtypes = [_SZ, _I, _D, _D, _D, _D, _D, ctypes.c_uint64, _P, _P, _P, _P]

    def sign(self, left: int, right: int, signature) -> int:
        return self.lib.orc_gp_sign(left, right, sig_array(signature), len(signature))

    def plan(self, signature) -> ctypes.Array:
        buf = (ctypes.c_uint8 * PLAN_BYTES)()
        st = self.lib.orc_batch_plan_init(buf, len(signature), sig_array(signature))
        if st != 0:
            raise ValueError(f"plan init failed: {st}")
        return buf

    def forward(self, signature, x: np.ndarray, w: np.ndarray, left: bool) -> tuple[int, np.ndarray]:
        x = np.ascontiguousarray(x, dtype=np.float64)
        out = np.zeros_like(x)
        st = self.lib.orc_batch_forward(self.plan(signature), _ptr(x), x.shape[0], _ptr(np.ascontiguousarray(w)),
                                        int(left), _ptr(out))
        return st, out

    def vjp(self, signature, x: np.ndarray, cot: np.ndarray, left: bool) -> tuple[int, np.ndarray]:
        x = np.ascontiguousarray(x, dtype=np.float64)
        cot = np.ascontiguousarray(cot, dtype=np.float64)
        g = np.zeros(x.shape[1])
        st = self.lib.orc_batch_vjp(self.plan(signature), _ptr(x), _ptr(cot), x.shape[0], int(left), _ptr(g))
        return st, g

    def sgd_step(self, signature, x, t, lr: float, w: np.ndarray, left: bool) -> tuple[int, np.ndarray, float]:
        x = np.ascontiguousarray(x, dtype=np.float64)
        t = np.ascontiguousarray(t, dtype=np.float64)
        w = np.array(w, dtype=np.float64)
        loss = ctypes.c_double(np.nan)
        st = self.lib.orc_batch_mse_sgd_step(self.plan(signature), _ptr(x), _ptr(t), x.shape[0], lr, int(left),
                                             _ptr(w), ctypes.byref(loss))
        return st, w, loss.value

    def gp(self, signature, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        n = len(signature)
        out = np.zeros(1 << n)
        self.lib.orc_gp_f64(n, sig_array(signature), _ptr(np.ascontiguousarray(a, np.float64)),
                            _ptr(np.ascontiguousarray(b, np.float64)), _ptr(out))
        return out

    def gp_vjp(self, signature, a, b, cot) -> tuple[np.ndarray, np.ndarray]:
        n = len(signature)
        la, rb = np.zeros(1 << n), np.zeros(1 << n)
        self.lib.orc_gp_f64_vjp(n, sig_array(signature), _ptr(np.ascontiguousarray(a, np.float64)),
                                _ptr(np.ascontiguousarray(b, np.float64)), _ptr(np.ascontiguousarray(cot, np.float64)),
                                _ptr(la), _ptr(rb))
        return la, rb

    def gp_jvp(self, signature, a, b, ta, tb) -> np.ndarray:
        n = len(signature)
        out = np.zeros(1 << n)
        self.lib.orc_gp_f64_jvp(n, sig_array(signature), *[_ptr(np.ascontiguousarray(v, np.float64))
                                                          for v in (a, b, ta, tb)], _ptr(out))
        return out

    def sparse_apply(self, signature, side: int, blades, coeffs, x: np.ndarray) -> np.ndarray:
        n = len(signature)
        bl = np.ascontiguousarray(blades, dtype=np.uint8)
        co = np.ascontiguousarray(coeffs, dtype=np.int32)
        out = np.zeros(1 << n)
        st = self.lib.orc_sparse_apply(n, sig_array(signature), side, _ptr(bl), _ptr(co), len(bl),
                                       _ptr(np.ascontiguousarray(x, np.float64)), _ptr(out))
        assert st == 0
        return out

    def sparse_apply_parametric(self, signature, side, blades, params, x) -> np.ndarray:
        n = len(signature)
        bl = np.ascontiguousarray(blades, dtype=np.uint8)
        out = np.zeros(1 << n)
        st = self.lib.orc_sparse_apply_parametric(n, sig_array(signature), side, _ptr(bl),
                                                  _ptr(np.ascontiguousarray(params, np.float64)), len(bl),
                                                  _ptr(np.ascontiguousarray(x, np.float64)), _ptr(out))
        assert st == 0
        return out

    def sparse_apply_vjp(self, signature, side, blades, coeffs, cot) -> np.ndarray:
        n = len(signature)
        bl = np.ascontiguousarray(blades, dtype=np.uint8)
        co = np.ascontiguousarray(coeffs, dtype=np.int32)
        out = np.zeros(1 << n)
        st = self.lib.orc_sparse_apply_vjp(n, sig_array(signature), side, _ptr(bl), _ptr(co), len(bl),
                                           _ptr(np.ascontiguousarray(cot, np.float64)), _ptr(out))
        assert st == 0
        return out

    def sparse_apply_parametric_vjp(self, signature, side, blades, params, x, cot):
        n = len(signature)
        bl = np.ascontiguousarray(blades, dtype=np.uint8)
        ic = np.zeros(1 << n)
        pc = np.zeros(len(bl))
        st = self.lib.orc_sparse_apply_parametric_vjp(
            n, sig_array(signature), side, _ptr(bl), _ptr(np.ascontiguousarray(params, np.float64)), len(bl),
            _ptr(np.ascontiguousarray(x, np.float64)), _ptr(np.ascontiguousarray(cot, np.float64)), _ptr(ic),
            _ptr(pc))
        assert st == 0
        return ic, pc

    def v8_update(self, optimizer: int, lr, b1, b2, eps, scale, step: int, gsum, w, m, v):
        w = np.array(w, np.float64)
        m = np.array(m, np.float64)
        v = np.array(v, np.float64)
        gsum = np.ascontiguousarray(gsum, np.float64)
        st = self.lib.orc_v8_optimizer_update(len(w), optimizer, lr, b1, b2, eps, scale, step, _ptr(gsum),
                                              _ptr(w), _ptr(m), _ptr(v))
        return st, w, m, v


class Reference:
    """The reference's own CPU code compiled from its sources (oracle/_ref)."""

    def __init__(self, path: pathlib.Path = REF_SO):
        if not path.exists():
            raise FileNotFoundError(str(path))
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        L.geo_batch_gp_plan_init.argtypes = [_P, _U8, _I8P]
        for name in ("geo_batch_gp_right_forward_f64",):
            getattr(L, name).argtypes = [_P, _P, _SZ, _P, _P]
        L.geo_batch_gp_left_forward_f64.argtypes = [_P, _P, _P, _SZ, _P]
        L.geo_batch_gp_right_vjp_parameter_f64.argtypes = [_P, _P, _P, _SZ, _P]
        L.geo_batch_gp_left_vjp_parameter_f64.argtypes = [_P, _P, _P, _SZ, _P]
        L.geo_batch_gp_right_mse_sgd_step_f64.argtypes = [_P, _P, _P, _SZ, _D, _P, _P]
        L.geo_batch_gp_left_mse_sgd_step_f64.argtypes = [_P, _P, _P, _SZ, _D, _P, _P]
        L.geo_operator_gp_sign.argtypes = [_U8, _U8, _I8P, _U8]
        _declare_reference_operators(L)

    def plan(self, signature) -> ctypes.Array:
        buf = (ctypes.c_uint8 * PLAN_BYTES)()
        st = self.lib.geo_batch_gp_plan_init(buf, len(signature), sig_array(signature))
        if st != 0:
            raise ValueError(f"reference plan init failed: {st}")
        return buf

    def forward(self, signature, x, w, left: bool) -> tuple[int, np.ndarray]:
        x = np.ascontiguousarray(x, dtype=np.float64)
        w = np.ascontiguousarray(w, dtype=np.float64)
        out = np.zeros_like(x)
        p = self.plan(signature)
        if left:
            st = self.lib.geo_batch_gp_left_forward_f64(p, _ptr(w), _ptr(x), x.shape[0], _ptr(out))
        else:
            st = self.lib.geo_batch_gp_right_forward_f64(p, _ptr(x), x.shape[0], _ptr(w), _ptr(out))
        return st, out

    def vjp(self, signature, x, cot, left: bool) -> tuple[int, np.ndarray]:
        x = np.ascontiguousarray(x, dtype=np.float64)
        cot = np.ascontiguousarray(cot, dtype=np.float64)
        g = np.zeros(x.shape[1])
        fn = self.lib.geo_batch_gp_left_vjp_parameter_f64 if left else self.lib.geo_batch_gp_right_vjp_parameter_f64
        st = fn(self.plan(signature), _ptr(x), _ptr(cot), x.shape[0], _ptr(g))
        return st, g

    def sgd_step(self, signature, x, t, lr, w, left: bool) -> tuple[int, np.ndarray, float]:
        x = np.ascontiguousarray(x, dtype=np.float64)
        t = np.ascontiguousarray(t, dtype=np.float64)
        w = np.array(w, dtype=np.float64)
        loss = ctypes.c_double(np.nan)
        fn = self.lib.geo_batch_gp_left_mse_sgd_step_f64 if left else self.lib.geo_batch_gp_right_mse_sgd_step_f64
        st = fn(self.plan(signature), _ptr(x), _ptr(t), x.shape[0], lr, _ptr(w), ctypes.byref(loss))
        return st, w, loss.value

    def sign(self, left: int, right: int, signature) -> int:
        return self.lib.geo_operator_gp_sign(left, right, sig_array(signature), len(signature))

    # -- per-multivector operators (reference src/operator_kernel.c) ---------
    def _mv(self, signature, coeffs=None):
        mv = MvF64()
        mv.dimension = len(signature)
        for i, v in enumerate(signature):
            mv.signature[i] = int(v)
        if coeffs is not None:
            for i, v in enumerate(np.asarray(coeffs, np.float64)):
                mv.coefficients[i] = float(v)
        return mv

    @staticmethod
    def _coeffs(mv, n):
        return np.array(mv.coefficients[: 1 << n], dtype=np.float64)

    def gp(self, signature, a, b) -> np.ndarray:
        out = MvF64()
        st = self.lib.geo_operator_gp_f64(ctypes.byref(self._mv(signature, a)), ctypes.byref(self._mv(signature, b)),
                                          ctypes.byref(out))
        assert st == 0
        return self._coeffs(out, len(signature))

    def gp_vjp(self, signature, a, b, cot):
        la, rb = MvF64(), MvF64()
        st = self.lib.geo_operator_gp_f64_vjp(ctypes.byref(self._mv(signature, a)),
                                              ctypes.byref(self._mv(signature, b)),
                                              ctypes.byref(self._mv(signature, cot)), ctypes.byref(la),
                                              ctypes.byref(rb))
        assert st == 0
        n = len(signature)
        return self._coeffs(la, n), self._coeffs(rb, n)

    def gp_jvp(self, signature, a, b, ta, tb):
        out = MvF64()
        st = self.lib.geo_operator_gp_f64_jvp(*[ctypes.byref(self._mv(signature, v)) for v in (a, b, ta, tb)],
                                              ctypes.byref(out))
        assert st == 0
        return self._coeffs(out, len(signature))

    def sparse_plan(self, signature, side: int, blades, coeffs):
        plan = (ctypes.c_uint8 * 528)()
        terms = (OperatorTerm * len(blades))()
        for i, (b, c) in enumerate(zip(blades, coeffs)):
            terms[i].blade = int(b)
            terms[i].coefficient = int(c)
        st = self.lib.geo_operator_plan_sparse_i32(plan, len(signature), sig_array(signature), side, terms,
                                                   len(blades))
        return st, plan

    def sparse_apply(self, signature, side, blades, coeffs, x):
        st, plan = self.sparse_plan(signature, side, blades, coeffs)
        assert st == 0
        out = MvF64()
        assert self.lib.geo_operator_apply_f64(plan, ctypes.byref(self._mv(signature, x)), ctypes.byref(out)) == 0
        return self._coeffs(out, len(signature))

    def sparse_apply_parametric(self, signature, side, blades, params, x):
        st, plan = self.sparse_plan(signature, side, blades, [1] * len(blades))
        assert st == 0
        out = MvF64()
        p = np.ascontiguousarray(params, np.float64)
        assert self.lib.geo_operator_apply_parametric_f64(plan, _ptr(p), len(p), ctypes.byref(self._mv(signature, x)),
                                                          ctypes.byref(out)) == 0
        return self._coeffs(out, len(signature))

    def sparse_apply_vjp(self, signature, side, blades, coeffs, cot):
        st, plan = self.sparse_plan(signature, side, blades, coeffs)
        assert st == 0
        out = MvF64()
        assert self.lib.geo_operator_apply_f64_vjp(plan, ctypes.byref(self._mv(signature, cot)),
                                                   ctypes.byref(out)) == 0
        return self._coeffs(out, len(signature))

    def sparse_apply_parametric_vjp(self, signature, side, blades, params, x, cot):
        st, plan = self.sparse_plan(signature, side, blades, [1] * len(blades))
        assert st == 0
        p = np.ascontiguousarray(params, np.float64)
        ic = MvF64()
        pc = np.zeros(len(p))
        assert self.lib.geo_operator_apply_parametric_f64_vjp(
            plan, _ptr(p), len(p), ctypes.byref(self._mv(signature, x)), ctypes.byref(self._mv(signature, cot)),
            ctypes.byref(ic), _ptr(pc), len(pc)) == 0
        return self._coeffs(ic, len(signature)), pc

    # -- V8 graph runtime (reference src/full_cycle_v8.c) --------------------
    def v8_composed(self, signature, values) -> tuple[float, np.ndarray, np.ndarray]:
        """Forward + backward of the all-node-kinds graph: (loss, grad w1, grad w2)."""
        L = self.lib
        n = len(signature)
        prog = (ctypes.c_uint8 * 256)()
        ids = composed_graph(L, prog, signature, lambda c: self._mv(signature, c), values)
        try:
            assert L.geo_v8_forward(prog) == 0
            assert L.geo_v8_backward(prog, 0) == 0
            loss = ctypes.cast(L.geo_v8_value(prog, ids["loss"]), ctypes.POINTER(MvF64)).contents.coefficients[0]
            g1 = self._coeffs(ctypes.cast(L.geo_v8_gradient(prog, ids["p1"]), ctypes.POINTER(MvF64)).contents, n)
            g2 = self._coeffs(ctypes.cast(L.geo_v8_gradient(prog, ids["p2"]), ctypes.POINTER(MvF64)).contents, n)
        finally:
            L.geo_v8_program_free(prog)
        return loss, g1, g2

    def v8_train(self, signature, left: bool, xs, ts, w0, optimizer: int, lr: float, b1: float, b2: float,
                 eps: float, steps: int):
        """Per-sample V8 loop of the graph x*w (or w*x) -> add(., scale(t,-1)) -> squared_norm.

        Follows benchmarks/bench_v8_full_cycle.c:35-56 and :207-219: every step
        zero_grad, then per sample set x and t, forward, backward(accumulate =
        sample != 0), then optimizer_step(gradient_scale = 1/B). xs/ts hold the
        same minibatch for every step. Returns (parameters after each step,
        summed loss of each step)."""
        L = self.lib
        n = len(signature)
        prog = (ctypes.c_uint8 * 256)()
        zero = self._mv(signature)
        ids = {k: ctypes.c_uint32() for k in ("x", "t", "w", "pred", "neg", "res", "loss")}
        assert L.geo_v8_program_init(prog, n, sig_array(signature), 1, 8) == 0
        assert L.geo_v8_add_leaf(prog, 1, b"x", ctypes.byref(zero), 0, 0, ctypes.byref(ids["x"])) == 0
        assert L.geo_v8_add_leaf(prog, 2, b"y", ctypes.byref(zero), 0, 0, ctypes.byref(ids["t"])) == 0
        assert L.geo_v8_add_leaf(prog, 3, b"w", ctypes.byref(self._mv(signature, w0)), 1, 0,
                                 ctypes.byref(ids["w"])) == 0
        a, b = (ids["w"], ids["x"]) if left else (ids["x"], ids["w"])
        assert L.geo_v8_add_binary(prog, 8, b"pred", a, b, ctypes.byref(ids["pred"])) == 0
        assert L.geo_v8_add_unary(prog, 7, b"neg_y", ids["t"], -1.0, 0, ctypes.byref(ids["neg"])) == 0
        assert L.geo_v8_add_binary(prog, 6, b"residual", ids["pred"], ids["neg"], ctypes.byref(ids["res"])) == 0
        assert L.geo_v8_add_unary(prog, 17, b"loss", ids["res"], 0.0, 0, ctypes.byref(ids["loss"])) == 0
        assert L.geo_v8_compile(prog, ids["loss"]) == 0
        params, losses = [], []
        batch = xs.shape[0]
        try:
            for _ in range(steps):
                assert L.geo_v8_zero_grad(prog) == 0
                total = 0.0
                for j in range(batch):
                    assert L.geo_v8_set_value(prog, ids["x"], ctypes.byref(self._mv(signature, xs[j]))) == 0
                    assert L.geo_v8_set_value(prog, ids["t"], ctypes.byref(self._mv(signature, ts[j]))) == 0
                    assert L.geo_v8_forward(prog) == 0
                    assert L.geo_v8_backward(prog, 1 if j else 0) == 0
                    total += ctypes.cast(L.geo_v8_value(prog, ids["loss"]), ctypes.POINTER(MvF64)).contents.coefficients[0]
                st = L.geo_v8_optimizer_step(prog, optimizer, lr, b1, b2, eps, 1.0 / batch)
                assert st == 0, st
                w = ctypes.cast(L.geo_v8_value(prog, ids["w"]), ctypes.POINTER(MvF64)).contents
                params.append(self._coeffs(w, n))
                losses.append(total)
        finally:
            L.geo_v8_program_free(prog)
        return np.array(params), np.array(losses)


    def v8_composed_train(self, signature, values, xs, ts, optimizer: int, lr: float, steps: int,
                          b1: float = 0.9, b2: float = 0.999, eps: float = 1e-8):
        """Per-sample V8 training of the all-node-kinds graph (composed_graph):
        every step zero_grad, then per sample set x and target, forward,
        backward(accumulate = sample != 0), then optimizer_step(gradient_scale =
        1/B) (reference src/full_cycle_v8.c:569-1041). Returns (w1 after each
        step, w2 after each step, summed loss of each step)."""
        L = self.lib
        n = len(signature)
        prog = (ctypes.c_uint8 * 256)()
        ids = composed_graph(L, prog, signature, lambda c: self._mv(signature, c), values)
        w1s, w2s, losses = [], [], []
        try:
            for _ in range(steps):
                assert L.geo_v8_zero_grad(prog) == 0
                total = 0.0
                for j in range(xs.shape[0]):
                    assert L.geo_v8_set_value(prog, ids["x"], ctypes.byref(self._mv(signature, xs[j]))) == 0
                    assert L.geo_v8_set_value(prog, ids["y"], ctypes.byref(self._mv(signature, ts[j]))) == 0
                    assert L.geo_v8_forward(prog) == 0
                    assert L.geo_v8_backward(prog, 1 if j else 0) == 0
                    total += ctypes.cast(L.geo_v8_value(prog, ids["loss"]), ctypes.POINTER(MvF64)).contents.coefficients[0]
                assert L.geo_v8_optimizer_step(prog, optimizer, lr, b1, b2, eps, 1.0 / xs.shape[0]) == 0
                for key, out in (("p1", w1s), ("p2", w2s)):
                    out.append(self._coeffs(ctypes.cast(L.geo_v8_value(prog, ids[key]), ctypes.POINTER(MvF64)).contents, n))
                losses.append(total)
        finally:
            L.geo_v8_program_free(prog)
        return np.array(w1s), np.array(w2s), np.array(losses)

def composed_graph(L, prog, signature, mv, values) -> dict:
    """Build the all-node-kinds graph of the reference test
    (tests/test_full_cycle_v8.c:158-181) through any library exposing the
    geo_v8_* ABI. `mv(coeffs)` builds a geo_operator_mv_f64_t for `signature`;
    `values` holds the input, target, w1, w2 coefficient arrays. Returns node ids."""
    n = len(signature)
    q = sum(1 for s in signature if s < 0)
    ids = {}

    def nid(name):
        ids[name] = ctypes.c_uint32()
        return ctypes.byref(ids[name])

    const = np.zeros(1 << n)
    const[0] = 1.25
    assert L.geo_v8_program_init(prog, n, sig_array(signature), 1, 4) == 0
    assert L.geo_v8_add_leaf(prog, 1, b"x", ctypes.byref(mv(values["input"])), 1, 0, nid("x")) == 0
    assert L.geo_v8_add_leaf(prog, 2, b"target", ctypes.byref(mv(values["target"])), 0, 0, nid("y")) == 0
    assert L.geo_v8_add_leaf(prog, 3, b"w1", ctypes.byref(mv(values["w1"])), 1, 0, nid("p1")) == 0
    assert L.geo_v8_add_leaf(prog, 3, b"w2", ctypes.byref(mv(values["w2"])), 1, 0, nid("p2")) == 0
    assert L.geo_v8_add_leaf(prog, 4, b"bias", ctypes.byref(mv(const)), 0, 0, nid("c0")) == 0
    assert L.geo_v8_add_binary(prog, 8, b"gp", ids["x"], ids["p1"], nid("gp")) == 0
    assert L.geo_v8_add_unary(prog, 14, b"activation", ids["gp"], 0.0, 0, nid("act")) == 0
    assert L.geo_v8_add_unary(prog, 15, b"gate", ids["p2"], 0.0, 0, nid("gate")) == 0
    assert L.geo_v8_add_binary(prog, 13, b"gated", ids["act"], ids["gate"], nid("gated")) == 0
    assert L.geo_v8_add_unary(prog, 9, b"reversed", ids["gated"], 0.0, 0, nid("rev")) == 0
    assert L.geo_v8_add_unary(prog, 11, b"involuted", ids["rev"], 0.0, 0, nid("inv")) == 0
    assert L.geo_v8_add_unary(prog, 12, b"conjugated", ids["inv"], 0.0, 0, nid("conj")) == 0
    assert L.geo_v8_add_unary(prog, 10, b"projected", ids["conj"], 0.0, q % (n + 1), nid("proj")) == 0
    assert L.geo_v8_add_binary(prog, 6, b"shifted", ids["proj"], ids["c0"], nid("shift")) == 0
    assert L.geo_v8_add_unary(prog, 16, b"normalized", ids["shift"], 1e-12, 0, nid("norm")) == 0
    assert L.geo_v8_add_unary(prog, 7, b"negative_target", ids["y"], -1.0, 0, nid("negy")) == 0
    assert L.geo_v8_add_binary(prog, 6, b"residual", ids["norm"], ids["negy"], nid("res")) == 0
    assert L.geo_v8_add_unary(prog, 17, b"loss", ids["res"], 0.0, 0, nid("loss")) == 0
    assert L.geo_v8_compile(prog, ids["loss"]) == 0
    return ids


def v8_mv_fill(n: int, seed: int) -> np.ndarray:
    """Coefficients of mv_fill in the reference test (tests/test_full_cycle_v8.c:29-41)."""
    out = np.zeros(1 << n)
    for blade in range(1 << n):
        mixed = ((blade + 1) * (seed * 31 + 17) + seed * 7) & 0xFFFFFFFF
        out[blade] = float(mixed % 29 - 14) / 23.0
    return out


class MvF64(ctypes.Structure):
    """geo_operator_mv_f64_t (reference include/geo/operator_kernel.h:53-57)."""

    _fields_ = [("dimension", ctypes.c_uint8), ("signature", ctypes.c_int8 * 6),
                ("coefficients", ctypes.c_double * 64)]


class OperatorTerm(ctypes.Structure):
    _fields_ = [("blade", ctypes.c_uint8), ("coefficient", ctypes.c_int32)]


def _declare_reference_operators(L) -> None:
    M = ctypes.POINTER(MvF64)
    L.geo_operator_gp_f64.argtypes = [M, M, M]
    L.geo_operator_gp_f64_vjp.argtypes = [M, M, M, M, M]
    L.geo_operator_gp_f64_jvp.argtypes = [M, M, M, M, M]
    L.geo_operator_plan_sparse_i32.argtypes = [_P, _U8, _I8P, _I, _P, _SZ]
    L.geo_operator_apply_f64.argtypes = [_P, M, M]
    L.geo_operator_apply_parametric_f64.argtypes = [_P, _P, _SZ, M, M]
    L.geo_operator_apply_f64_vjp.argtypes = [_P, M, M]
    L.geo_operator_apply_parametric_f64_vjp.argtypes = [_P, _P, _SZ, M, M, M, _P, _SZ]
    U32 = ctypes.c_uint32
    U32P = ctypes.POINTER(U32)
    L.geo_v8_program_init.argtypes = [_P, _U8, _I8P, _I, _SZ]
    L.geo_v8_program_free.argtypes = [_P]
    L.geo_v8_add_leaf.argtypes = [_P, _I, ctypes.c_char_p, M, _I, _I, U32P]
    L.geo_v8_add_unary.argtypes = [_P, _I, ctypes.c_char_p, U32, _D, _U8, U32P]
    L.geo_v8_add_binary.argtypes = [_P, _I, ctypes.c_char_p, U32, U32, U32P]
    L.geo_v8_compile.argtypes = [_P, U32]
    L.geo_v8_set_value.argtypes = [_P, U32, M]
    L.geo_v8_forward.argtypes = [_P]
    L.geo_v8_zero_grad.argtypes = [_P]
    L.geo_v8_backward.argtypes = [_P, _I]
    L.geo_v8_optimizer_step.argtypes = [_P, _I, _D, _D, _D, _D, _D]
    L.geo_v8_value.argtypes = [_P, U32]
    L.geo_v8_value.restype = _P
    L.geo_v8_gradient.argtypes = [_P, U32]
    L.geo_v8_gradient.restype = _P


def reference_available() -> bool:
    return REF_SO.exists()


def ensure_reference_built() -> bool:
    """Build oracle/_ref with `make -C oracle ref` when the environment names the
    reference tree (GEO_REFERENCE_TREE); otherwise report whether it was built."""
    import os

    tree = os.environ.get("GEO_REFERENCE_TREE")
    if not REF_SO.exists() and tree:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={tree}"], capture_output=True)
    return REF_SO.exists()
