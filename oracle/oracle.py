"""CPU oracle for the MXFP8 quantizer -- TEST INFRASTRUCTURE ONLY.

A ctypes/numpy wrapper over ``mxfp8_oracle.c``, the integer-exact C
restatement of the reference recipe (MXFP8_quantizer.py:170-200, 456-525,
531-539, 610-662).  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg may import this module; the product path in
``mxfp8-quantizer_b200/`` never does.

Parity pin: ``tests/golden/`` holds digests made by running the reference's
own torch restatement (``reference_quantize`` / ``decode_scale_bytes``) on
seeded inputs; ``tests/test_oracle_golden.py`` checks this oracle against
them.  Blocks holding inf/NaN are outside what that restatement gets right
(it returns scale 256 for NaN blocks); for those the oracle follows the
reference kernel's instruction semantics.
"""

from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
SRC = HERE / "mxfp8_oracle.c"
BUILD_DIR = HERE / "_build"
LIB = BUILD_DIR / "libmxfp8_oracle.so"

BF16 = 0
FP16 = 1

SCALE_VEC_SIZE = 32
SCALE_PACK_COLS = 4
SCALE_ROWS_PER_PACK = 128


def build(force: bool = False) -> pathlib.Path:
    """Compile the C restatement with gcc into ``oracle/_build``."""
    if LIB.exists() and not force and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    BUILD_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(f".{os.getpid()}.tmp")
    cmd = ["gcc", "-O2", "-std=c99", "-D_GNU_SOURCE", "-fPIC", "-shared", "-pthread",
           "-fno-fast-math", "-ffp-contract=off", str(SRC), "-o", str(tmp), "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = build() if not LIB.exists() else LIB
        L = ctypes.CDLL(str(path))
        i64, vp, i32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
        L.oracle_quantize.argtypes = [vp, i32, i64, i64, i64, vp, i64, i64, i64, vp, i64, i32]
        L.oracle_quantize.restype = i32
        L.oracle_scale_storage_bytes.argtypes = [i64, i64]
        L.oracle_scale_storage_bytes.restype = i64
        L.oracle_scale_offset.argtypes = [i64, i64, i64]
        L.oracle_scale_offset.restype = i64
        L.oracle_unpack_scales.argtypes = [vp, i64, i64, vp]
        L.oracle_unpack_scales.restype = i32
        L.oracle_dequantize.argtypes = [vp, i64, i64, i64, vp, vp, i64]
        L.oracle_dequantize.restype = i32
        L.oracle_scale_from_amax_bits.argtypes = [ctypes.c_uint16, i32, ctypes.POINTER(ctypes.c_uint32)]
        L.oracle_scale_from_amax_bits.restype = ctypes.c_uint8
        L.oracle_f32_mul_rn.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        L.oracle_f32_mul_rn.restype = ctypes.c_uint32
        L.oracle_e4m3_from_f32_bits.argtypes = [ctypes.c_uint32]
        L.oracle_e4m3_from_f32_bits.restype = ctypes.c_uint8
        _lib = L
    return _lib


def dtype_code(name: str) -> int:
    name = name.lower()
    if name in ("bf16", "bfloat16"):
        return BF16
    if name in ("fp16", "float16", "half"):
        return FP16
    raise ValueError(f"unknown dtype {name!r}")


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


def scale_storage_bytes(rows: int, cols: int) -> int:
    return int(lib().oracle_scale_storage_bytes(rows, cols))


def padded_shape(m: int, k: int, rows_per_cta: int = 8, k_tile: int = 256) -> tuple[int, int]:
    """The reference's launch shape (MXFP8_quantizer.py:766-791)."""
    return ceil_div(m, rows_per_cta) * rows_per_cta, ceil_div(k, k_tile) * k_tile


def quantize(x_bits: np.ndarray, dtype: str, q_rows: int | None = None, q_cols: int | None = None,
             nthreads: int | None = None) -> tuple[np.ndarray, np.ndarray]:
    """Quantize a (m, k) array of uint16 bf16/fp16 bit patterns.

    ``q_rows``/``q_cols`` give the output geometry (default: the reference's
    zero-padded launch shape).  Returns ``(q, s)``: q is (q_rows, q_cols)
    uint8 E4M3 bytes, s the packed UE8M0 storage (uint8, 1-D)."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    assert x_bits.ndim == 2
    m, k = x_bits.shape
    if q_rows is None or q_cols is None:
        pm, pk = padded_shape(max(m, 1), max(k, 1))
        q_rows = pm if q_rows is None else q_rows
        q_cols = pk if q_cols is None else q_cols
    q = np.empty((q_rows, q_cols), dtype=np.uint8)
    s = np.empty((scale_storage_bytes(q_rows, q_cols),), dtype=np.uint8)
    if nthreads is None:
        nthreads = os.cpu_count() or 1
    rc = lib().oracle_quantize(x_bits.ctypes.data, dtype_code(dtype), m, k, k, q.ctypes.data,
                               q_rows, q_cols, q_cols, s.ctypes.data, s.size, nthreads)
    if rc != 0:
        raise ValueError(f"oracle_quantize rejected the arguments (m={m}, k={k}, q_rows={q_rows}, q_cols={q_cols})")
    return q, s


def unpack_scales(s: np.ndarray, rows: int, scale_cols: int) -> np.ndarray:
    s = np.ascontiguousarray(s, dtype=np.uint8)
    out = np.empty((rows, scale_cols), dtype=np.uint8)
    lib().oracle_unpack_scales(s.ctypes.data, rows, scale_cols, out.ctypes.data)
    return out


def dequantize(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    s = np.ascontiguousarray(s, dtype=np.uint8)
    rows, cols = q.shape
    out = np.empty((rows, cols), dtype=np.float32)
    rc = lib().oracle_dequantize(q.ctypes.data, rows, cols, cols, s.ctypes.data, out.ctypes.data, cols)
    if rc != 0:
        raise ValueError("cols must be a multiple of 32")
    return out


def scale_from_amax_bits(amax_bits: int, dtype: str) -> tuple[int, int]:
    inv = ctypes.c_uint32(0)
    b = lib().oracle_scale_from_amax_bits(amax_bits, dtype_code(dtype), ctypes.byref(inv))
    return int(b), int(inv.value)


def e4m3_from_f32_bits(bits: int) -> int:
    return int(lib().oracle_e4m3_from_f32_bits(bits))


def f32_mul_rn(a_bits: int, b_bits: int) -> int:
    return int(lib().oracle_f32_mul_rn(a_bits, b_bits))
