"""The graph runtime's exp and tanh on the GPU (geo_b200_cr_math_f64, the device
build of the functions the TANH and SIGMOID nodes call) against correctly
rounded values from an extended-precision evaluation
(tests/golden/make_crmath_golden.py): bit for bit on every argument, including
the ones whose double-double evaluation hands over to the fixed-point path, and
with that path forced for every argument."""
from __future__ import annotations

import ctypes
import pathlib

import numpy as np
import pytest

from geometricelementaryoperators_b200 import abi
from tests.gpu_helpers import dev, host, ptr, torch

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "crmath_golden.npz"


@pytest.mark.parametrize("fn,name", [(0, "exp"), (1, "tanh"), (2, "exp"), (3, "tanh")])
def test_device_correctly_rounded(fn, name):
    L = abi.lib()
    g = np.load(GOLDEN)
    x = dev(g["x"])
    y = torch().full_like(x, float("nan"))
    assert L.geo_b200_cr_math_f64(fn, ptr(x), ptr(y), x.numel(), None) == 0
    torch().cuda.synchronize()
    got = host(y)
    bad = np.nonzero(got.view(np.uint64) != g[name].view(np.uint64))[0]
    assert bad.size == 0, [(float(g["x"][i]).hex(), float(got[i]).hex(), float(g[name][i]).hex()) for i in bad[:5]]


def test_in_place_and_arguments():
    L = abi.lib()
    g = np.load(GOLDEN)
    x = dev(g["x"])
    assert L.geo_b200_cr_math_f64(1, ptr(x), ptr(x), x.numel(), None) == 0
    torch().cuda.synchronize()
    assert np.array_equal(host(x).view(np.uint64), g["tanh"].view(np.uint64))
    assert L.geo_b200_cr_math_f64(4, ptr(x), ptr(x), x.numel(), None) == 1  # unknown function
    assert L.geo_b200_cr_math_f64(0, None, ptr(x), 1, None) == 1
    assert L.geo_b200_cr_math_f64(0, None, None, 0, None) == 0


def test_device_matches_host_build_random(tmp_path):
    """10^6 random arguments per distribution: the device functions equal the host build of the same
    source (tests/c/crmath_check.cpp) bit for bit, on the combined functions and on the exact path."""
    import shutil
    import subprocess

    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ not found")
    root = pathlib.Path(__file__).resolve().parents[1]
    csrc = root / "geometricelementaryoperators_b200" / "csrc"
    exe = tmp_path / "crmath_check"
    subprocess.run([cxx, "-std=c++17", "-O2", "-ffp-contract=off", "-I", str(csrc),
                    str(root / "tests" / "c" / "crmath_check.cpp"), "-o", str(exe)], check=True)
    rng = np.random.default_rng(77)
    n = 1 << 20
    x = np.concatenate([rng.normal(0.0, 3.0, n), rng.uniform(-20.0, 20.0, n), rng.uniform(-745.5, 709.9, n // 4),
                        np.exp2(rng.uniform(-40.0, 5.0, n)) * rng.choice([-1.0, 1.0], n)])
    x.tofile(tmp_path / "in.bin")
    subprocess.run([str(exe), str(tmp_path / "in.bin"), str(tmp_path / "out.bin")], check=True)
    want = np.fromfile(tmp_path / "out.bin").reshape(-1, 4)
    L = abi.lib()
    dx = dev(x)
    y = torch().empty_like(dx)
    for fn in range(4):
        assert L.geo_b200_cr_math_f64(fn, ptr(dx), ptr(y), dx.numel(), None) == 0
        torch().cuda.synchronize()
        got = host(y)
        bad = np.nonzero(got.view(np.uint64) != want[:, fn].view(np.uint64))[0]
        assert bad.size == 0, (fn, [(float(x[i]).hex(), float(got[i]).hex(), float(want[i, fn]).hex()) for i in bad[:5]])
