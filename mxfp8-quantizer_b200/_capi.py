"""ctypes binding of libmxfp8.so (the C ABI declared in include/mxfp8.h).

Plain integers cross the boundary: device pointers, sizes and a stream
handle.  Status codes become exceptions with the reference's conventions:
``ValueError`` for argument problems (MXFP8_quantizer.py:544-552, 770-790,
801-807) and ``RuntimeError("CUDA error after <ctx>: <name>")`` for CUDA
failures (MXFP8_quantizer.py:793-799).  There is no fallback: if the library
is missing the import of the quantizer fails loudly.
"""

from __future__ import annotations

import ctypes
import pathlib
import threading

PKG_DIR = pathlib.Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libmxfp8.so"
CHECKED_LIB_PATH = PKG_DIR / "libmxfp8_checked.so"

BF16, FP16, F32 = 0, 1, 2

OK = 0
ERR_NULL_POINTER = -1
ERR_SHAPE = -2
ERR_DTYPE = -3
ERR_ALIGNMENT = -4
ERR_SCALE_BUFFER = -5
ERR_CUDA = -6
ERR_TENSOR_MAP = -7
ERR_DEVICE = -8

EXPORTS = (
    "mxfp8_scale_storage_bytes",
    "mxfp8_launch_shape",
    "mxfp8_quantize",
    "mxfp8_quantize_noalloc",
    "mxfp8_quantize_padded",
    "mxfp8_dequantize",
    "mxfp8_device_status",
    "mxfp8_noalloc_status",
    "mxfp8_selftest_bounded_wait",
    "mxfp8_strerror",
    "mxfp8_last_error",
)

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class ExtensionMissing(RuntimeError):
    pass


def configure(L: ctypes.CDLL) -> ctypes.CDLL:
    """Declare the C ABI's argument and result types on a loaded library."""
    i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    L.mxfp8_scale_storage_bytes.argtypes = [i64, i64]
    L.mxfp8_scale_storage_bytes.restype = i64
    L.mxfp8_launch_shape.argtypes = [i64, i64, ctypes.POINTER(i64), ctypes.POINTER(i64)]
    L.mxfp8_launch_shape.restype = i32
    L.mxfp8_quantize.argtypes = [vp, i32, i64, i64, i64, vp, i64, i64, i64, vp, i64, vp]
    L.mxfp8_quantize.restype = i32
    L.mxfp8_quantize_noalloc.argtypes = [vp, i32, i64, i64, i64, vp, i64, i64, i64, vp, i64, vp]
    L.mxfp8_quantize_noalloc.restype = i32
    L.mxfp8_quantize_padded.argtypes = [vp, vp, vp, i64, i64, i64, i32, vp]
    L.mxfp8_quantize_padded.restype = i32
    L.mxfp8_dequantize.argtypes = [vp, i64, i64, i64, vp, i64, vp, i32, i64, vp]
    L.mxfp8_dequantize.restype = i32
    L.mxfp8_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), i32]
    L.mxfp8_device_status.restype = i32
    L.mxfp8_noalloc_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), i32]
    L.mxfp8_noalloc_status.restype = i32
    L.mxfp8_selftest_bounded_wait.argtypes = [ctypes.c_uint32, vp]
    L.mxfp8_selftest_bounded_wait.restype = i32
    L.mxfp8_strerror.argtypes = [i32]
    L.mxfp8_strerror.restype = ctypes.c_char_p
    L.mxfp8_last_error.argtypes = []
    L.mxfp8_last_error.restype = ctypes.c_char_p
    if hasattr(L, "mxfp8_checked_window_slack"):
        L.mxfp8_checked_window_slack.argtypes = [i64]
        L.mxfp8_checked_window_slack.restype = i32
    return L


def lib() -> ctypes.CDLL:
    """Load libmxfp8.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ExtensionMissing(
                f"{LIB_PATH} is not built; run `python {PKG_DIR.name}/build.py` (or __graft_entry__.build())")
        _lib = configure(ctypes.CDLL(str(LIB_PATH)))
        return _lib


def checked_lib() -> ctypes.CDLL:
    """libmxfp8_checked.so (include/mxfp8_checked.h): the same C ABI with every
    global store tested against its output; for tests, not for production."""
    if not CHECKED_LIB_PATH.exists():
        raise ExtensionMissing(f"{CHECKED_LIB_PATH} is not built; run `python {PKG_DIR.name}/build.py`")
    return configure(ctypes.CDLL(str(CHECKED_LIB_PATH)))


def strerror(code: int) -> str:
    return lib().mxfp8_strerror(code).decode()


def check(code: int, context: str) -> None:
    """Map a status code onto the reference's exception types."""
    if code == OK:
        return
    if code in (ERR_CUDA, ERR_TENSOR_MAP, ERR_DEVICE):
        detail = lib().mxfp8_last_error().decode()
        raise RuntimeError(f"CUDA error after {context}: {detail or strerror(code)}")
    raise ValueError(f"{context}: {strerror(code)} (status {code})")


def scale_storage_bytes(rows: int, cols: int) -> int:
    n = int(lib().mxfp8_scale_storage_bytes(rows, cols))
    if n < 0:
        raise ValueError(f"invalid scale geometry ({rows}, {cols})")
    return n


def launch_shape(m: int, k: int) -> tuple[int, int]:
    km, kk = ctypes.c_int64(0), ctypes.c_int64(0)
    rc = lib().mxfp8_launch_shape(m, k, ctypes.byref(km), ctypes.byref(kk))
    if rc != OK:
        raise ValueError(f"invalid problem shape m={m}, k={k}")
    return km.value, kk.value


def quantize(x_ptr: int, dtype: int, m: int, k: int, ld_x: int, q_ptr: int, q_rows: int, q_cols: int,
             ld_q: int, s_ptr: int, s_bytes: int, stream: int) -> None:
    rc = lib().mxfp8_quantize(x_ptr or None, dtype, m, k, ld_x, q_ptr or None, q_rows, q_cols, ld_q,
                              s_ptr or None, s_bytes, stream or None)
    check(rc, "quantizer launch")


def quantize_noalloc(x_ptr: int, dtype: int, m: int, k: int, ld_x: int, q_ptr: int, q_rows: int, q_cols: int,
                     ld_q: int, s_ptr: int, s_bytes: int, stream: int) -> None:
    """mxfp8_quantize_noalloc: like quantize(), but the library never allocates
    device memory (for callers that may not call cudaMalloc)."""
    rc = lib().mxfp8_quantize_noalloc(x_ptr or None, dtype, m, k, ld_x, q_ptr or None, q_rows, q_cols, ld_q,
                                      s_ptr or None, s_bytes, stream or None)
    check(rc, "quantizer launch (allocation-free)")


def quantize_padded(x_ptr: int, q_ptr: int, s_ptr: int, m: int, k: int, s_word_count: int, dtype: int,
                    stream: int) -> None:
    rc = lib().mxfp8_quantize_padded(x_ptr or None, q_ptr or None, s_ptr or None, m, k, s_word_count, dtype,
                                     stream or None)
    check(rc, "quantizer launch")


def dequantize(q_ptr: int, rows: int, cols: int, ld_q: int, s_ptr: int, s_bytes: int, out_ptr: int,
               out_dtype: int, ld_out: int, stream: int) -> None:
    rc = lib().mxfp8_dequantize(q_ptr or None, rows, cols, ld_q, s_ptr or None, s_bytes, out_ptr or None,
                                out_dtype, ld_out, stream or None)
    check(rc, "dequantizer launch")


def device_status(clear: bool = False) -> int:
    v = ctypes.c_uint32(0)
    check(lib().mxfp8_device_status(ctypes.byref(v), int(clear)), "device status read")
    return int(v.value)


def noalloc_status(clear: bool = False) -> int:
    """Status word of the allocation-free entry on the current device."""
    v = ctypes.c_uint32(0)
    check(lib().mxfp8_noalloc_status(ctypes.byref(v), int(clear)), "allocation-free status read")
    return int(v.value)


def selftest_bounded_wait(limit_us: int, stream: int) -> None:
    """Launch the bounded-wait self-test kernel (see include/mxfp8.h)."""
    check(lib().mxfp8_selftest_bounded_wait(limit_us, stream or None), "bounded-wait self-test launch")
