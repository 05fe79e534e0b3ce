"""Build the in-tree C-ABI library `libqmoe_b200.so` for sm_100a.

Every CUDA translation unit is compiled with
`nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3`, the host
quantiser with g++ (OpenMP, no floating-point contraction), and the objects
are linked into one shared library beside this file.  A rebuild happens only
when a source or header is newer than the library.

Usage: python build.py [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB = HERE / "libqmoe_b200.so"
OBJ = HERE / "_build"

CUDA_SOURCES = ["iq4xs_kernels.cu", "route.cu", "experts.cu", "capi.cu", "noalloc.cu", "stack_kernel.cu", "prefill.cu",
                "hc.cu", "formats.cu"]
HOST_SOURCES = ["quant_host.cpp"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]
GXX_FLAGS = ["-O2", "-fPIC", "-fopenmp", "-ffp-contract=off", "-std=c++17"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libqmoe_b200.so")
    return cand


def _inputs() -> list[Path]:
    files = [CSRC / s for s in CUDA_SOURCES + HOST_SOURCES]
    files += sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h")) + [Path(__file__)]
    return files


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(f.stat().st_mtime > t for f in _inputs() if f.exists())


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        if not verbose:
            sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:4])} ...")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library; returns its path."""
    if not force and not needs_build():
        return LIB
    OBJ.mkdir(exist_ok=True)
    nvcc = _nvcc()
    objs: list[str] = []
    from concurrent.futures import ThreadPoolExecutor

    jobs = []
    for src in CUDA_SOURCES:
        obj = OBJ / (src + ".o")
        jobs.append([nvcc, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)])
        objs.append(str(obj))
    for src in HOST_SOURCES:
        obj = OBJ / (src + ".o")
        jobs.append(["g++", *GXX_FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)])
        objs.append(str(obj))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(lambda c: _run(c, verbose), jobs))
    tmp = LIB.with_suffix(".so.tmp")
    _run([nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(tmp), *objs,
          "-Xcompiler", "-fopenmp", "-lgomp"], verbose)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
