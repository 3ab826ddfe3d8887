"""Build libmxfp8.so and libmxfp8_checked.so (sm_100a) in-tree with nvcc.

    python mxfp8-quantizer_b200/build.py [--force] [--ptxas-verbose]

The library links the CUDA runtime statically and exports only the C ABI
of include/mxfp8.h.  The checked build compiles the same sources with
MXFP8_CHECKED (every global store tested against its output's bytes; see
include/mxfp8_checked.h).  nvcc cross-compiles, so this runs without a GPU.
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
CHECKED_LIB = PKG / "libmxfp8_checked.so"
SOURCES = ["capi.cu", "quantize_tma.cu", "quantize_generic.cu", "dequantize.cu", "selftest.cu"]
HEADERS = ["ptx.cuh", "recipe.cuh", "launch.h", "guard.cuh", "tile.cuh", "row_path.cuh", "stores.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA extension cannot be built")


def inputs() -> list[pathlib.Path]:
    return [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [
        ROOT / "include" / "mxfp8.h", ROOT / "include" / "mxfp8_checked.h", pathlib.Path(__file__)]


def up_to_date(lib: pathlib.Path) -> bool:
    if not lib.exists():
        return False
    t = lib.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in inputs())


def _command(out: pathlib.Path, checked: bool, verbose_ptxas: bool) -> list[str]:
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
           "-Xcompiler", "-Wall", "-I", str(ROOT / "include"), "-o", str(out)]
    if checked:
        cmd.append("-DMXFP8_CHECKED")
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    return cmd + [str(CSRC / s) for s in SOURCES]


def build(force: bool = False, verbose_ptxas: bool = False) -> pathlib.Path:
    """Build both libraries (in parallel) if a source is newer; returns the product library."""
    jobs = []
    for lib, checked in ((LIB, False), (CHECKED_LIB, True)):
        if force or not up_to_date(lib):
            tmp = lib.with_name(f".{lib.stem}.{os.getpid()}.so")
            proc = subprocess.Popen(_command(tmp, checked, verbose_ptxas and not checked), stdout=subprocess.PIPE,
                                    stderr=subprocess.PIPE, text=True)
            jobs.append((lib, tmp, proc))
    failed = []
    for lib, tmp, proc in jobs:
        out, err = proc.communicate()
        if proc.returncode != 0:
            sys.stderr.write(out + err)
            failed.append(lib.name)
            continue
        if verbose_ptxas:
            sys.stderr.write(err)
        os.replace(tmp, lib)
    if failed:
        raise RuntimeError(f"nvcc failed building {', '.join(failed)}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.ptxas_verbose))
