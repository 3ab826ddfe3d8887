"""Build libmxfp8.so (sm_100a) in-tree with nvcc.

    python mxfp8-quantizer_b200/build.py [--force] [--ptxas-verbose]

The library links the CUDA runtime statically and exports only the C ABI
of include/mxfp8.h.  nvcc cross-compiles, so this runs without a GPU.
"""

from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libmxfp8.so"
SOURCES = ["capi.cu", "quantize_tma.cu", "quantize_generic.cu", "dequantize.cu", "selftest.cu"]
HEADERS = ["ptx.cuh", "recipe.cuh", "launch.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA extension cannot be built")


def inputs() -> list[pathlib.Path]:
    return [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [ROOT / "include" / "mxfp8.h",
                                                                        pathlib.Path(__file__)]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in inputs())


def build(force: bool = False, verbose_ptxas: bool = False) -> pathlib.Path:
    if not force and up_to_date():
        return LIB
    tmp = LIB.with_name(f".libmxfp8.{os.getpid()}.so")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
           "-Xcompiler", "-Wall", "-I", str(ROOT / "include"), "-o", str(tmp)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    cmd += [str(CSRC / s) for s in SOURCES]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("nvcc failed building libmxfp8.so")
    if verbose_ptxas:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.ptxas_verbose))
