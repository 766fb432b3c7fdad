"""CPU check of the Pauli-string representation search behind the tensor-core
path: for every canonical signature with n >= 2 and both sides the search
finds a representation, the Clifford relations hold against the reference sign
rule (checked inside make_rep_plan), and X' W' scattered back reproduces the
direct product to 1e-12 (tests/c/rep_check.cpp)."""
from __future__ import annotations

import pathlib
import subprocess

ROOT = pathlib.Path(__file__).resolve().parent.parent
CSRC = ROOT / "geometricelementaryoperators_b200" / "csrc"


def test_representation_search(tmp_path):
    exe = tmp_path / "rep_check"
    res = subprocess.run(
        ["g++", "-std=c++17", "-O2", "-I", str(ROOT / "include"), "-I", str(CSRC), "-I", "/usr/local/cuda/include",
         str(ROOT / "tests" / "c" / "rep_check.cpp"), str(CSRC / "representation.cpp"), str(CSRC / "plan_host.cpp"),
         "-o", str(exe)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "REP_CHECK: PASS cases=54" in out.stdout
    # The headline algebras get the small representations.
    assert "n=6 q=0 side=0 D=16 S=4" in out.stdout
    assert "n=6 q=3 side=0 D=8 S=8" in out.stdout


def test_pair_tables(tmp_path):
    """The tables of the float64 pairwise representation kernel: the kernel's arithmetic on the host
    (geo::pair_product_host) equals the direct product for every D = 16 signature and operand reversal
    (tests/c/pair_check.cpp), and the compile-time copy the kernel uses (csrc/pair_tables_gen.h) is what
    csrc/gen/gen_pair_tables.cpp writes from them."""
    srcs = [str(CSRC / "representation.cpp"), str(CSRC / "plan_host.cpp")]
    inc = ["-I", str(ROOT / "include"), "-I", str(CSRC), "-I", "/usr/local/cuda/include"]
    exe = tmp_path / "pair_check"
    res = subprocess.run(["g++", "-std=c++17", "-O2", *inc, str(ROOT / "tests" / "c" / "pair_check.cpp"), *srcs,
                          "-o", str(exe)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and "PAIR_CHECK: PASS cases=112" in out.stdout, out.stdout + out.stderr
    gen = tmp_path / "gen_pair_tables"
    res = subprocess.run(["g++", "-std=c++17", "-O2", *inc, str(CSRC / "gen" / "gen_pair_tables.cpp"), *srcs, "-o", str(gen)],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    header = subprocess.run([str(gen)], capture_output=True, text=True, timeout=60)
    assert header.returncode == 0
    assert header.stdout == (CSRC / "pair_tables_gen.h").read_text()
