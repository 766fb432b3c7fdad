"""ctypes declarations of every symbol libgeo_b200.so exports (include/geo/*.h).

Struct layouts are the reference's (include/geo/batch_gp.h:23-33,
include/geo/batch_gp_cuda.h:23-34, include/geo/operator_kernel.h:37-57);
``tests/test_abi.py`` checks sizes and offsets against the C headers.
"""
from __future__ import annotations

import ctypes
import pathlib

GEO_BATCH_GP_ABI_VERSION = 0x00010000
GEO_BATCH_GP_CUDA_ABI_VERSION = 0x00010001
GEO_OPERATOR_ABI_VERSION = 0x00050100
GEO_B200_ABI_VERSION = 0x00010000
MAX_TERMS = 4096

_PKG = pathlib.Path(__file__).resolve().parent
_LIB: ctypes.CDLL | None = None


def library_path() -> pathlib.Path:
    return _PKG / "libgeo_b200.so"


class BatchGpPlan(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_uint32),
        ("dimension", ctypes.c_uint8),
        ("signature", ctypes.c_int8 * 6),
        ("blade_count", ctypes.c_uint16),
        ("term_count", ctypes.c_uint16),
        ("left_blade", ctypes.c_uint8 * MAX_TERMS),
        ("right_blade", ctypes.c_uint8 * MAX_TERMS),
        ("output_blade", ctypes.c_uint8 * MAX_TERMS),
        ("sign", ctypes.c_int8 * MAX_TERMS),
    ]


class CudaPlan(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_uint32),
        ("blade_count", ctypes.c_uint16),
        ("term_count", ctypes.c_uint16),
        ("dimension", ctypes.c_uint8),
        ("signature", ctypes.c_int8 * 6),
        ("device_signature", ctypes.c_void_p),
        ("device_left_blade", ctypes.c_void_p),
        ("device_right_blade", ctypes.c_void_p),
        ("device_output_blade", ctypes.c_void_p),
        ("device_sign", ctypes.c_void_p),
    ]


class OperatorTermI32(ctypes.Structure):
    _fields_ = [("blade", ctypes.c_uint8), ("coefficient", ctypes.c_int32)]


class OperatorPlanI32(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_uint32),
        ("dimension", ctypes.c_uint8),
        ("signature", ctypes.c_int8 * 6),
        ("kind", ctypes.c_uint8),
        ("side", ctypes.c_uint8),
        ("term_count", ctypes.c_uint8),
        ("reserved", ctypes.c_uint8),
        ("terms", OperatorTermI32 * 64),
    ]


class MvF64(ctypes.Structure):
    """geo_operator_mv_f64_t: a dense multivector with its metric."""

    _fields_ = [("dimension", ctypes.c_uint8), ("signature", ctypes.c_int8 * 6),
                ("coefficients", ctypes.c_double * 64)]


class OptimizerConfig(ctypes.Structure):
    _fields_ = [
        ("optimizer", ctypes.c_uint32),
        ("learning_rate", ctypes.c_double),
        ("beta1", ctypes.c_double),
        ("beta2", ctypes.c_double),
        ("epsilon", ctypes.c_double),
    ]


_P = ctypes.c_void_p
_D = ctypes.c_double
_SZ = ctypes.c_size_t
_I = ctypes.c_int
_U8 = ctypes.c_uint8
_I8P = ctypes.POINTER(ctypes.c_int8)

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    # geo/batch_gp.h
    "geo_batch_gp_abi_version": (ctypes.c_uint32, []),
    "geo_batch_gp_plan_init": (_I, [ctypes.POINTER(BatchGpPlan), _U8, _I8P]),
    "geo_batch_gp_right_forward_f64": (_I, [ctypes.POINTER(BatchGpPlan), _P, _SZ, _P, _P]),
    "geo_batch_gp_left_forward_f64": (_I, [ctypes.POINTER(BatchGpPlan), _P, _P, _SZ, _P]),
    "geo_batch_gp_right_vjp_parameter_f64": (_I, [ctypes.POINTER(BatchGpPlan), _P, _P, _SZ, _P]),
    "geo_batch_gp_left_vjp_parameter_f64": (_I, [ctypes.POINTER(BatchGpPlan), _P, _P, _SZ, _P]),
    "geo_batch_gp_right_mse_sgd_step_f64": (_I, [ctypes.POINTER(BatchGpPlan), _P, _P, _SZ, _D, _P, _P]),
    "geo_batch_gp_left_mse_sgd_step_f64": (_I, [ctypes.POINTER(BatchGpPlan), _P, _P, _SZ, _D, _P, _P]),
    # geo/batch_gp_cuda.h
    "geo_batch_gp_cuda_abi_version": (ctypes.c_uint32, []),
    "geo_batch_gp_cuda_plan_upload": (_I, [ctypes.POINTER(CudaPlan), ctypes.POINTER(BatchGpPlan)]),
    "geo_batch_gp_cuda_plan_destroy": (None, [ctypes.POINTER(CudaPlan)]),
    "geo_batch_gp_cuda_reference_forward_f64": (_I, [ctypes.POINTER(CudaPlan), _P, _SZ, _P, _I, _P, _P]),
    "geo_batch_gp_cuda_planned_forward_f64": (_I, [ctypes.POINTER(CudaPlan), _P, _SZ, _P, _I, _P, _P]),
    "geo_batch_gp_cuda_reference_parameter_vjp_f64": (_I, [ctypes.POINTER(CudaPlan), _P, _P, _SZ, _I, _P, _P]),
    "geo_batch_gp_cuda_parameter_vjp_f64": (_I, [ctypes.POINTER(CudaPlan), _P, _P, _SZ, _I, _P, _P]),
    "geo_batch_gp_cuda_reference_mse_sgd_step_f64": (
        _I, [ctypes.POINTER(CudaPlan), _P, _P, _SZ, _D, _I, _P, _P, _P, _P, _P]),
    "geo_batch_gp_cuda_mse_sgd_step_f64": (
        _I, [ctypes.POINTER(CudaPlan), _P, _P, _SZ, _D, _I, _P, _P, _P, _P, _P]),
    "geo_batch_gp_cuda_status_string": (ctypes.c_char_p, [_I]),
    # geo/hand_cuda_comparator.h
    "geo_hand_cuda_forward_f64": (_I, [ctypes.POINTER(CudaPlan), _P, _SZ, _P, _I, _P, _P]),
    "geo_hand_cuda_parameter_vjp_f64": (_I, [ctypes.POINTER(CudaPlan), _P, _P, _SZ, _I, _P, _P]),
    "geo_hand_cuda_mse_sgd_step_f64": (_I, [ctypes.POINTER(CudaPlan), _P, _P, _SZ, _D, _I, _P, _P, _P, _P, _P]),
    # geo/operator_kernel.h
    "geo_operator_abi_version": (ctypes.c_uint32, []),
    "geo_operator_gradient_abi_version": (ctypes.c_uint32, []),
    "geo_operator_blade_count": (_SZ, [_U8]),
    "geo_operator_gp_sign": (_I, [_U8, _U8, _I8P, _U8]),
    "geo_operator_plan_fixed_blade_i32": (_I, [ctypes.POINTER(OperatorPlanI32), _U8, _I8P, _I, _U8, ctypes.c_int32]),
    "geo_operator_plan_sparse_i32": (
        _I, [ctypes.POINTER(OperatorPlanI32), _U8, _I8P, _I, ctypes.POINTER(OperatorTermI32), _SZ]),
    "geo_operator_apply_f64": (_I, [ctypes.POINTER(OperatorPlanI32), ctypes.POINTER(MvF64), ctypes.POINTER(MvF64)]),
    "geo_operator_apply_parametric_f64": (
        _I, [ctypes.POINTER(OperatorPlanI32), _P, _SZ, ctypes.POINTER(MvF64), ctypes.POINTER(MvF64)]),
    "geo_operator_apply_f64_vjp": (
        _I, [ctypes.POINTER(OperatorPlanI32), ctypes.POINTER(MvF64), ctypes.POINTER(MvF64)]),
    "geo_operator_apply_parametric_f64_vjp": (
        _I, [ctypes.POINTER(OperatorPlanI32), _P, _SZ, ctypes.POINTER(MvF64), ctypes.POINTER(MvF64),
             ctypes.POINTER(MvF64), _P, _SZ]),
    "geo_operator_gp_f64": (_I, [ctypes.POINTER(MvF64)] * 3),
    "geo_operator_gp_f64_jvp": (_I, [ctypes.POINTER(MvF64)] * 5),
    "geo_operator_gp_f64_vjp": (_I, [ctypes.POINTER(MvF64)] * 5),
    # geo/geo_b200.h
    "geo_b200_abi_version": (ctypes.c_uint32, []),
    "geo_b200_status_string": (ctypes.c_char_p, [_I]),
    "geo_b200_trainer_create": (_I, [ctypes.POINTER(_P), _U8, _I8P, _I, _P, ctypes.POINTER(OptimizerConfig)]),
    "geo_b200_trainer_destroy": (None, [_P]),
    "geo_b200_trainer_step_device": (_I, [_P, _P, _P, _SZ, _D, _P]),
    "geo_b200_trainer_step_host": (_I, [_P, _P, _P, _SZ, _D, _P]),
    "geo_b200_trainer_accumulate_device": (_I, [_P, _P, _P, _SZ, _P]),
    "geo_b200_trainer_apply": (_I, [_P, _D, _P]),
    "geo_b200_trainer_sync": (_I, [_P, _P]),
    "geo_b200_trainer_get_state": (_I, [_P, _P, _P, _P, _P]),
    "geo_b200_trainer_set_parameter": (_I, [_P, _P]),
    "geo_b200_trainer_set_state": (_I, [_P, _P, _P, _P, ctypes.c_uint64]),
    "geo_b200_trainer_device_parameter": (_P, [_P]),
    "geo_b200_trainer_set_algorithm": (_I, [_P, _I]),
    "geo_b200_trainer_algorithm": (_I, [_P]),
    "geo_b200_forward_f64": (_I, [_U8, _I8P, _I, _I, _P, _P, _P, _SZ, _P]),
    "geo_b200_comm_unique_id": (_I, [_P]),
    "geo_b200_comm_create": (_I, [ctypes.POINTER(_P), _I, _I, _P, _I]),
    "geo_b200_comm_destroy": (None, [_P]),
    "geo_b200_comm_abort": (None, [_P]),
    "geo_b200_trainer_attach_comm": (_I, [_P, _P]),
    "geo_b200_v8_batch_train_step": (_I, [_P, ctypes.c_uint32, ctypes.c_uint32, _P, _P, _SZ, _I, _D, _D, _D, _D, _D, _P]),
    "geo_b200_v8_batch_forward": (_I, [_P, ctypes.c_uint32, _P, _SZ, ctypes.c_uint32, _P]),
    "geo_b200_cr_math_f64": (_I, [_I, _P, _P, _SZ, _P]),
    "geo_b200_parameter_vjp_noalloc_f64": (_I, [_U8, _I8P, _I, _P, _P, _SZ, _P, _P]),
    "geo_b200_pairwise_gp_f64": (_I, [_U8, _I8P, _P, _P, _P, _SZ, _P]),
    "geo_b200_pairwise_gp_vjp_f64": (_I, [_U8, _I8P, _P, _P, _P, _P, _P, _SZ, _P]),
    "geo_b200_pairwise_gp_jvp_f64": (_I, [_U8, _I8P, _P, _P, _P, _P, _P, _SZ, _P]),
    "geo_b200_pairwise_gp_f32": (_I, [_U8, _I8P, _P, _I, _P, _P, _SZ, _P]),
    "geo_b200_pairwise_wait_failures": (_I, [ctypes.POINTER(ctypes.c_uint), _I]),
    "geo_b200_pairwise_wait_selftest": (_I, [_I, _P, _SZ, ctypes.c_uint32, _P]),
    "geo_b200_sparse_apply_f64": (_I, [ctypes.POINTER(OperatorPlanI32), _P, _P, _SZ, _P]),
    "geo_b200_sparse_apply_parametric_f64": (_I, [ctypes.POINTER(OperatorPlanI32), _P, _P, _P, _SZ, _P]),
    "geo_b200_sparse_apply_vjp_f64": (_I, [ctypes.POINTER(OperatorPlanI32), _P, _P, _SZ, _P]),
    "geo_b200_sparse_apply_parametric_vjp_f64": (
        _I, [ctypes.POINTER(OperatorPlanI32), _P, _P, _P, _P, _P, _SZ, _P]),
}


def lib() -> ctypes.CDLL:
    """Load libgeo_b200.so (fails loudly when it has not been built)."""
    global _LIB
    if _LIB is None:
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"{path} is missing: build it with `python -m geometricelementaryoperators_b200.build` "
                "(there is no CPU fallback)")
        handle = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def sig_array(signature) -> ctypes.Array:
    arr = (ctypes.c_int8 * 6)()
    for i, v in enumerate(signature):
        arr[i] = int(v)
    return arr
