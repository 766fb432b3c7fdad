"""Helpers for the GPU parity tests: device buffers via torch, calls via the C-ABI."""
from __future__ import annotations

import ctypes

import numpy as np

from geometricelementaryoperators_b200 import abi

TOL = 1e-12  # |a-b| <= TOL (1 + |a| + |b|): the float64 parity bar
TOL_F32 = 1e-5


def torch():
    import torch as _t

    return _t


def dev(a: np.ndarray, dtype=None):
    t = torch()
    return t.from_numpy(np.ascontiguousarray(a)).to("cuda")


def host(t) -> np.ndarray:
    return t.detach().cpu().numpy()


def ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch().cuda.current_stream().cuda_stream)


def sync():
    torch().cuda.synchronize()


def make_plan(signature) -> abi.BatchGpPlan:
    plan = abi.BatchGpPlan()
    assert abi.lib().geo_batch_gp_plan_init(ctypes.byref(plan), len(signature), abi.sig_array(signature)) == 0
    return plan


class CudaPlan:
    def __init__(self, signature):
        self.host = make_plan(signature)
        self.dev = abi.CudaPlan()
        assert abi.lib().geo_batch_gp_cuda_plan_upload(ctypes.byref(self.dev), ctypes.byref(self.host)) == 0

    def __del__(self):
        try:
            abi.lib().geo_batch_gp_cuda_plan_destroy(ctypes.byref(self.dev))
        except Exception:
            pass


def np_ptr(a: np.ndarray) -> ctypes.c_void_p:
    return a.ctypes.data_as(ctypes.c_void_p)
