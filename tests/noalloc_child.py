"""Child process for tests/test_zz_no_alloc.py: does a call of the
allocation-free entry allocate memory?

Runs without torch, so that only this script and the library touch CUDA:
device buffers come from cuda-python's runtime before counting starts.  A
CUPTI subscriber (tests/alloc_probe.c, built by the parent) counts every
driver API call that allocates (cuMemAlloc*, cuMemCreate, ...) from any CUDA
runtime in the process, the static one inside libmxfp8.so included.  The
counts are read around the first and second mxfp8_quantize_noalloc calls, the
status read, and, as a control that the probe sees the library's
allocations at all, around the first mxfp8_quantize call, whose first call
on a device allocates its status word.

Prints one JSON line; Q and S of the first allocation-free call go to the
.npy files named on the command line.
"""

import ctypes
import json
import pathlib
import sys

import numpy as np
from cuda.bindings import runtime as rt

ROOT = pathlib.Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "mxfp8-quantizer_b200"))
import _capi  # noqa: E402  (ctypes binding only: it imports nothing else of the package)


def ok(res):
    """Unpack a cuda-python result tuple (error, *values), raising on error."""
    err, *vals = res
    if err != rt.cudaError_t.cudaSuccess:
        raise SystemExit(f"cuda-python call failed: {err}")
    if not vals:
        return None
    return vals[0] if len(vals) == 1 else tuple(vals)


def free_bytes() -> int:
    ok(rt.cudaDeviceSynchronize())
    free, _total = ok(rt.cudaMemGetInfo())
    return int(free)


def main() -> None:
    bits_path, q_path, s_path = sys.argv[1:4]
    m, k = int(sys.argv[4]), int(sys.argv[5])
    probe = ctypes.CDLL(sys.argv[6])
    probe.alloc_probe_count.restype = ctypes.c_long
    probe.alloc_probe_last_name.restype = ctypes.c_char_p
    if probe.alloc_probe_start() != 0:
        raise SystemExit("CUPTI subscription failed")
    bits = np.load(bits_path)
    ok(rt.cudaSetDevice(0))
    lib = _capi.configure(ctypes.CDLL(str(_capi.LIB_PATH)))
    s_bytes = int(lib.mxfp8_scale_storage_bytes(m, k))
    x = ok(rt.cudaMalloc(bits.nbytes))
    q = ok(rt.cudaMalloc(m * k))
    s = ok(rt.cudaMalloc(s_bytes))
    q2 = ok(rt.cudaMalloc(m * k))
    s2 = ok(rt.cudaMalloc(s_bytes))
    ok(rt.cudaMemcpy(x, bits.ctypes.data, bits.nbytes, rt.cudaMemcpyKind.cudaMemcpyHostToDevice))

    setup_allocs = probe.alloc_probe_count()  # the buffers above: the probe sees cuda-python's allocations
    word = ctypes.c_uint32(0xFFFFFFFF)

    def call(entry, qq, ss):
        return entry(x, 0, m, k, k, qq, m, k, k, ss, s_bytes, None)

    counts, free = [probe.alloc_probe_count()], [free_bytes()]
    rc_status0 = lib.mxfp8_noalloc_status(ctypes.byref(word), 0)
    status0 = int(word.value)
    counts.append(probe.alloc_probe_count())
    rc1 = call(lib.mxfp8_quantize_noalloc, q, s)  # first call: looks up the scratch array
    free.append(free_bytes())
    counts.append(probe.alloc_probe_count())
    rc2 = call(lib.mxfp8_quantize_noalloc, q, s)
    free.append(free_bytes())
    counts.append(probe.alloc_probe_count())
    rc_status1 = lib.mxfp8_noalloc_status(ctypes.byref(word), 1)
    status1 = int(word.value)
    counts.append(probe.alloc_probe_count())
    rc3 = call(lib.mxfp8_quantize, q2, s2)  # control: allocates its status word
    free.append(free_bytes())
    counts.append(probe.alloc_probe_count())
    control_name = probe.alloc_probe_last_name().decode()

    q_host = np.empty((m, k), dtype=np.uint8)
    s_host = np.empty((s_bytes,), dtype=np.uint8)
    ok(rt.cudaMemcpy(q_host.ctypes.data, q, m * k, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost))
    ok(rt.cudaMemcpy(s_host.ctypes.data, s, s_bytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost))
    np.save(q_path, q_host)
    np.save(s_path, s_host)
    print(json.dumps({"rc": [rc_status0, rc1, rc2, rc_status1, rc3], "status": [status0, status1],
                      "setup_allocs": setup_allocs, "alloc_counts": counts, "control_call": control_name,
                      "free": free}), flush=True)


if __name__ == "__main__":
    main()
