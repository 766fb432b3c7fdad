"""Python host interface to the V8 graph runtime of libgeo_b200.

Mirrors the reference's graph API (include/geo/full_cycle_v8.h; reference
src/full_cycle_v8.c:287-1098): build a program from leaves and unary/binary
nodes, compile it with a loss node, and train it per sample
(``set_value``/``forward``/``backward``/``optimizer_step``) or per minibatch
through the batched entry points of geo/geo_b200.h
(``geo_b200_v8_batch_train_step``, ``geo_b200_v8_batch_forward``). Every call
goes to the CUDA library; there is no host fallback.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import abi

# geo_v8_node_kind_t (reference include/geo/full_cycle_v8.h:70-88)
INPUT, TARGET, PARAMETER, CONSTANT, STATE = 1, 2, 3, 4, 5
ADD, SCALE, GEOMETRIC_PRODUCT, REVERSE, GRADE_PROJECT = 6, 7, 8, 9, 10
GRADE_INVOLUTION, CLIFFORD_CONJUGATE, HADAMARD, TANH, SIGMOID = 11, 12, 13, 14, 15
EUCLIDEAN_NORMALIZE, SQUARED_NORM = 16, 17
SGD, ADAM = 1, 2
INVALID_NODE = 0xFFFFFFFF


class Multivector(ctypes.Structure):
    """geo_operator_mv_f64_t (reference include/geo/operator_kernel.h:53-57)."""

    _fields_ = [("dimension", ctypes.c_uint8), ("signature", ctypes.c_int8 * 6),
                ("coefficients", ctypes.c_double * 64)]


class ProgramStruct(ctypes.Structure):
    """geo_v8_program_t (reference include/geo/full_cycle_v8.h:89-104)."""

    _fields_ = [("abi_version", ctypes.c_uint32), ("dimension", ctypes.c_uint8), ("signature", ctypes.c_int8 * 6),
                ("pairing", ctypes.c_uint8), ("compiled", ctypes.c_uint8), ("forward_valid", ctypes.c_uint8),
                ("backward_valid", ctypes.c_uint8), ("reserved", ctypes.c_uint8), ("node_count", ctypes.c_uint32),
                ("node_capacity", ctypes.c_uint32), ("loss_node", ctypes.c_uint32),
                ("optimizer_step", ctypes.c_uint64), ("gradient_samples", ctypes.c_uint64),
                ("nodes", ctypes.c_void_p)]


_HANDLE: ctypes.CDLL | None = None


def _lib() -> ctypes.CDLL:
    """A private ctypes handle on libgeo_b200 (the same loaded library as
    abi.lib()) whose V8 functions take this module's struct types, so argument
    declarations made elsewhere for the shared handle are not disturbed."""
    global _HANDLE
    if _HANDLE is None:
        L = ctypes.CDLL(str(abi.library_path()))
        abi.lib()  # fails loudly when the CUDA library is missing
        M = ctypes.POINTER(Multivector)
        P = ctypes.POINTER(ProgramStruct)
        U32 = ctypes.c_uint32
        U32P = ctypes.POINTER(U32)
        L.geo_v8_program_init.argtypes = [P, ctypes.c_uint8, ctypes.POINTER(ctypes.c_int8), ctypes.c_int,
                                          ctypes.c_size_t]
        L.geo_v8_program_free.argtypes = [P]
        L.geo_v8_add_leaf.argtypes = [P, ctypes.c_int, ctypes.c_char_p, M, ctypes.c_int, ctypes.c_int, U32P]
        L.geo_v8_add_unary.argtypes = [P, ctypes.c_int, ctypes.c_char_p, U32, ctypes.c_double, ctypes.c_uint8, U32P]
        L.geo_v8_add_binary.argtypes = [P, ctypes.c_int, ctypes.c_char_p, U32, U32, U32P]
        L.geo_v8_compile.argtypes = [P, U32]
        L.geo_v8_set_value.argtypes = [P, U32, M]
        L.geo_v8_forward.argtypes = [P]
        L.geo_v8_zero_grad.argtypes = [P]
        L.geo_v8_backward.argtypes = [P, ctypes.c_int]
        L.geo_v8_optimizer_step.argtypes = [P, ctypes.c_int] + [ctypes.c_double] * 5
        L.geo_v8_value.argtypes = [P, U32]
        L.geo_v8_value.restype = M
        for name in ("geo_b200_v8_batch_train_step", "geo_b200_v8_batch_forward"):
            res, args = abi.SIGNATURES[name]
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _HANDLE = L
    return _HANDLE


class V8Error(RuntimeError):
    def __init__(self, call: str, status: int):
        super().__init__(f"{call} failed with geo_v8 status {status}")
        self.status = status


def _check(call: str, status: int) -> None:
    if status != 0:
        raise V8Error(call, status)


class Program:
    """A V8 program owned by libgeo_b200 (nodes in mapped page-locked memory)."""

    def __init__(self, signature, pairing: int = 1, capacity: int = 16):
        self.L = _lib()
        self.signature = [int(s) for s in signature]
        self.n = len(self.signature)
        self.p = ProgramStruct()
        sig = (ctypes.c_int8 * 6)(*self.signature, *([0] * (6 - self.n)))
        _check("geo_v8_program_init", self.L.geo_v8_program_init(ctypes.byref(self.p), self.n, sig, pairing, capacity))

    def _mv(self, coeffs=None) -> Multivector:
        m = Multivector()
        m.dimension = self.n
        for i, s in enumerate(self.signature):
            m.signature[i] = s
        if coeffs is not None:
            for i, v in enumerate(np.asarray(coeffs, np.float64)):
                m.coefficients[i] = float(v)
        return m

    def leaf(self, kind: int, name: str, coeffs=None, requires_grad: bool = False, constraint: int = 0) -> int:
        out = ctypes.c_uint32()
        _check("geo_v8_add_leaf", self.L.geo_v8_add_leaf(ctypes.byref(self.p), kind, name.encode(),
                                                          ctypes.byref(self._mv(coeffs)), int(requires_grad),
                                                          constraint, ctypes.byref(out)))
        return out.value

    def unary(self, kind: int, name: str, src: int, scalar: float = 0.0, grade: int = 0) -> int:
        out = ctypes.c_uint32()
        _check("geo_v8_add_unary", self.L.geo_v8_add_unary(ctypes.byref(self.p), kind, name.encode(), src, scalar,
                                                            grade, ctypes.byref(out)))
        return out.value

    def binary(self, kind: int, name: str, a: int, b: int) -> int:
        out = ctypes.c_uint32()
        _check("geo_v8_add_binary", self.L.geo_v8_add_binary(ctypes.byref(self.p), kind, name.encode(), a, b,
                                                              ctypes.byref(out)))
        return out.value

    def compile(self, loss: int) -> None:
        _check("geo_v8_compile", self.L.geo_v8_compile(ctypes.byref(self.p), loss))

    def value(self, node: int) -> np.ndarray:
        return np.array(self.L.geo_v8_value(ctypes.byref(self.p), node).contents.coefficients[: 1 << self.n])

    def batch_train_step(self, input_node: int, target_node: int, device_inputs: int, device_targets: int,
                         batch: int, optimizer: int, learning_rate: float, beta1: float = 0.9,
                         beta2: float = 0.999, epsilon: float = 1e-8, gradient_scale: float | None = None) -> float:
        """One optimizer step over `batch` device rows; returns the summed loss."""
        loss = ctypes.c_double()
        scale = 1.0 / batch if gradient_scale is None else gradient_scale
        _check("geo_b200_v8_batch_train_step", self.L.geo_b200_v8_batch_train_step(
            ctypes.byref(self.p), input_node, target_node, ctypes.c_void_p(device_inputs),
            ctypes.c_void_p(device_targets), batch, optimizer, learning_rate, beta1, beta2, epsilon, scale,
            ctypes.byref(loss)))
        return loss.value

    def batch_forward(self, input_node: int, device_inputs: int, batch: int, output_node: int,
                      device_outputs: int) -> None:
        _check("geo_b200_v8_batch_forward", self.L.geo_b200_v8_batch_forward(
            ctypes.byref(self.p), input_node, ctypes.c_void_p(device_inputs), batch, output_node,
            ctypes.c_void_p(device_outputs)))

    def free(self) -> None:
        if self.p.nodes:
            self.L.geo_v8_program_free(ctypes.byref(self.p))


def all_node_kinds_graph(signature, w1, w2, x0=None, y0=None) -> tuple[Program, dict]:
    """The all-node-kinds training graph of the reference's V8 test
    (tests/test_full_cycle_v8.c:158-181): x*w1 -> tanh, gated by sigmoid(w2)
    (Hadamard), reverse, involution, conjugate, grade projection, + 1.25,
    Euclidean normalisation, minus the target, squared norm. x0 / y0 are the
    initial values of the input and target leaves (zero when omitted)."""
    n = len(signature)
    q = sum(1 for s in signature if s < 0)
    prog = Program(signature, capacity=20)
    zero = np.zeros(1 << n)
    bias = np.zeros(1 << n)
    bias[0] = 1.25
    ids = {"x": prog.leaf(INPUT, "x", zero if x0 is None else x0, True),
           "y": prog.leaf(TARGET, "target", zero if y0 is None else y0)}
    ids["w1"] = prog.leaf(PARAMETER, "w1", w1, True)
    ids["w2"] = prog.leaf(PARAMETER, "w2", w2, True)
    ids["bias"] = prog.leaf(CONSTANT, "bias", bias)
    gp = prog.binary(GEOMETRIC_PRODUCT, "gp", ids["x"], ids["w1"])
    act = prog.unary(TANH, "activation", gp)
    gate = prog.unary(SIGMOID, "gate", ids["w2"])
    gated = prog.binary(HADAMARD, "gated", act, gate)
    rev = prog.unary(REVERSE, "reversed", gated)
    inv = prog.unary(GRADE_INVOLUTION, "involuted", rev)
    conj = prog.unary(CLIFFORD_CONJUGATE, "conjugated", inv)
    proj = prog.unary(GRADE_PROJECT, "projected", conj, 0.0, q % (n + 1))
    shifted = prog.binary(ADD, "shifted", proj, ids["bias"])
    norm = prog.unary(EUCLIDEAN_NORMALIZE, "normalized", shifted, 1e-12)
    negy = prog.unary(SCALE, "negative_target", ids["y"], -1.0)
    res = prog.binary(ADD, "residual", norm, negy)
    ids["loss"] = prog.unary(SQUARED_NORM, "loss", res)
    prog.compile(ids["loss"])
    return prog, ids
