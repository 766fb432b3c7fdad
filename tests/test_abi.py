"""The C-ABI library loads, exports every symbol its headers declare, and keeps
the reference's struct layouts. CPU only: no compute call is made here except
the host-side plan builders (pure integer code)."""
from __future__ import annotations

import ctypes
import pathlib
import re
import subprocess

import pytest

from geometricelementaryoperators_b200 import abi

ROOT = pathlib.Path(__file__).resolve().parent.parent
INCLUDE = ROOT / "include"
CUDA_INCLUDE = "/usr/local/cuda/include"


def declared_symbols() -> set[str]:
    names = set()
    for h in sorted((INCLUDE / "geo").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names.update(re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(geo_\w+)\s*\(", text, flags=re.M))
    return names


def exported_symbols() -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(abi.library_path())], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_library_exports_every_declared_symbol():
    declared = declared_symbols()
    assert len(declared) >= 45
    missing = declared - exported_symbols()
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_library_loads_and_binds_every_symbol():
    L = abi.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name
    assert L.geo_batch_gp_abi_version() == abi.GEO_BATCH_GP_ABI_VERSION
    assert L.geo_batch_gp_cuda_abi_version() == abi.GEO_BATCH_GP_CUDA_ABI_VERSION
    assert L.geo_operator_abi_version() == abi.GEO_OPERATOR_ABI_VERSION
    assert L.geo_b200_abi_version() == abi.GEO_B200_ABI_VERSION
    assert [L.geo_operator_blade_count(n) for n in range(8)] == [0, 2, 4, 8, 16, 32, 64, 0]


def test_ctypes_layouts_match_reference():
    assert ctypes.sizeof(abi.BatchGpPlan) == 16400
    assert abi.BatchGpPlan.sign.offset == 12304
    assert ctypes.sizeof(abi.CudaPlan) == 56
    assert abi.CudaPlan.device_signature.offset == 16
    assert ctypes.sizeof(abi.OperatorPlanI32) == 528
    assert abi.OperatorPlanI32.terms.offset == 16
    assert ctypes.sizeof(abi.MvF64) == 520 and abi.MvF64.coefficients.offset == 8


def _gcc(args, tmp_path):
    res = subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-I", str(INCLUDE), "-I", CUDA_INCLUDE, *args],
                         capture_output=True, text=True, cwd=tmp_path)
    assert res.returncode == 0, res.stderr
    return res


def test_c11_layout_pins_compile(tmp_path):
    exe = tmp_path / "abi_layout"
    _gcc([str(ROOT / "tests" / "c" / "abi_layout.c"), "-o", str(exe)], tmp_path)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    assert out == ["16400", "56", "528", "520"]


def test_c11_consumer_links(tmp_path):
    """A C11 caller of the reference headers links against libgeo_b200.so unchanged."""
    exe = tmp_path / "consumer"
    lib_dir = str(abi.library_path().parent)
    _gcc([str(ROOT / "tests" / "c" / "consumer.c"), "-o", str(exe), "-L", lib_dir, "-lgeo_b200",
          f"-Wl,-rpath,{lib_dir}", "-lm"], tmp_path)
    assert exe.exists()


@pytest.mark.gpu
def test_c11_consumer_runs(tmp_path):
    exe = tmp_path / "consumer"
    lib_dir = str(abi.library_path().parent)
    _gcc([str(ROOT / "tests" / "c" / "consumer.c"), "-o", str(exe), "-L", lib_dir, "-lgeo_b200",
          f"-Wl,-rpath,{lib_dir}", "-lm"], tmp_path)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr
    assert "GEO_B200_CONSUMER: PASS" in res.stdout


def _operator_consumer(tmp_path):
    exe = tmp_path / "operator_consumer"
    lib_dir = str(abi.library_path().parent)
    orc_dir = str(ROOT / "oracle")
    _gcc([str(ROOT / "tests" / "c" / "operator_consumer.c"), "-I", orc_dir, "-o", str(exe), "-L", lib_dir,
          "-lgeo_b200", "-L", orc_dir, "-loracle", f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{orc_dir}", "-lm"],
         tmp_path)
    return exe


def test_c11_operator_consumer_links(tmp_path):
    """A C11 caller of every reference per-multivector operator symbol links against libgeo_b200.so."""
    assert _operator_consumer(tmp_path).exists()


@pytest.mark.gpu
def test_c11_operator_consumer_runs(tmp_path):
    res = subprocess.run([str(_operator_consumer(tmp_path))], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr
    assert "GEO_B200_OPERATOR_CONSUMER: PASS" in res.stdout
