"""Build libgeo_b200.so in-tree for sm_100a (B200).

Every CUDA/C++ source under csrc/ is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a -lineinfo`` into _build/, then linked
into ``geometricelementaryoperators_b200/libgeo_b200.so`` (static CUDA runtime;
NCCL is opened at run time when a communicator is created). Objects are rebuilt only when a source or header is newer.

Usage: ``python -m geometricelementaryoperators_b200.build [-v] [--force]``.
"""
from __future__ import annotations

import concurrent.futures
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build" / "geo_b200"
LIB = PKG / "libgeo_b200.so"
CLI = PKG / "geo_cycle_b200"  # the geo_cycle command line on the library

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr", "-I", str(ROOT / "include"), "-I", str(CSRC),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libgeo_b200.so")


def _sources() -> list[pathlib.Path]:
    return sorted(p for p in CSRC.iterdir() if p.suffix in (".cu", ".cpp"))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.h")) + list((ROOT / "include" / "geo").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: pathlib.Path, obj: pathlib.Path, verbose: bool) -> None:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-x", "c++", "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr.strip():
        print(res.stderr, flush=True)


def build(verbose: bool = False, force: bool = False, extra_flags: list[str] | None = None) -> pathlib.Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    hdr = _headers_mtime()
    jobs = []
    objs = []
    for src in _sources():
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            jobs.append((src, obj))
    if extra_flags:
        NVCC_FLAGS.extend(extra_flags)
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(lambda j: _compile(j[0], j[1], verbose), jobs))
    if jobs or force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    cli_src = CSRC / "cli" / "geo_cycle_main.cpp"
    if force or not CLI.exists() or CLI.stat().st_mtime < max(LIB.stat().st_mtime, cli_src.stat().st_mtime):
        cmd = [nvcc(), "-std=c++17", "-O2", "-I", str(ROOT / "include"), "-x", "c++", str(cli_src), "-o", str(CLI),
               "-L", str(LIB.parent), "-lgeo_b200", "-Xlinker", "-rpath", "-Xlinker", "$ORIGIN"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"geo_cycle_b200 link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="--force" in sys.argv)
    print(LIB)
