"""The allocation-free entry point, mxfp8_quantize_noalloc, through the C ABI.

It exists for callers that may not call cudaMalloc: plugins whose host
application owns every device allocation through its own pool, code that must
make all its allocations up front, and devices whose memory another
allocator has already reserved in full.  mxfp8_quantize allocates a small
status buffer on its first call per device; this entry keeps that word in a
fixed device array of the library and never allocates.

Checked here: its output equals the CPU oracle's, the reference kernel's
digest (config 4 with its inf/NaN/subnormal blocks) and mxfp8_quantize's,
call after call, although every call shares one fixed array that keeps what
the last call left; its status word can be read and cleared
(mxfp8_noalloc_status) and reports a failure (a store the checked build
skipped); and in a fresh process, no allocating CUDA driver call happens
during its first and second calls (a CUPTI subscriber counts them), while the
allocating entry's first call, as a control, is seen making one.

This file sorts last so a stop-at-first-failure run has already run every
other test; it also passes on its own in a fresh process (the allocation-free
call comes first there, before anything else touched the library).
"""

import ctypes
import hashlib
import json
import os
import pathlib
import subprocess
import sys

import numpy as np
import pytest
import torch

import inputs

pytestmark = pytest.mark.gpu

HERE = pathlib.Path(__file__).resolve().parent


def _capi():
    import MXFP8_quantizer

    return MXFP8_quantizer.load_package()._capi


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _run(entry, bits, dtype, q_rows, q_cols):
    capi = _capi()
    m, k = bits.shape
    x = torch.from_numpy(bits.view(np.int16)).cuda()
    s_bytes = capi.scale_storage_bytes(q_rows, q_cols)
    q = torch.full((q_rows, q_cols), 0xA5, dtype=torch.uint8, device="cuda")
    s = torch.full((s_bytes,), 0xA5, dtype=torch.uint8, device="cuda")
    entry(x.data_ptr(), 0 if dtype == "bf16" else 1, m, k, k, q.data_ptr(), q_rows, q_cols, q_cols, s.data_ptr(),
          s_bytes, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return q.cpu().numpy(), s.cpu().numpy()


CASES = [
    # (name, bits generator, dtype, q_rows, q_cols): config 4's special values
    # in the reference's padded geometry, then a different shape and dtype
    ("c4", lambda: inputs.special_values_bf16(), "bf16", 1000, 4096),
    ("fp16_ragged", lambda: inputs.normal(2051, 2080, 14, "fp16"), "fp16", 2056, 2304),
    # odd K: X rows are not 16-byte aligned (the per-phase tensor-map path)
    ("odd_k", lambda: inputs.normal(1001, 4095, 15, "bf16"), "bf16", 1001, 4096),
]


def test_noalloc_matches_oracle_reference_kernel_and_allocating_entry_two_calls_in_a_row(oracle_mod):
    capi = _capi()
    assert torch.cuda.is_available()
    kernel_golden = json.loads((HERE / "golden" / "golden_kernel.json").read_text())["cases"]
    results = []
    for name, gen, dtype, q_rows, q_cols in CASES:
        bits = gen()
        # allocation-free entry first, twice in a row, before the allocating one
        first = _run(capi.quantize_noalloc, bits, dtype, q_rows, q_cols)
        second = _run(capi.quantize_noalloc, bits, dtype, q_rows, q_cols)
        expect = _run(capi.quantize, bits, dtype, q_rows, q_cols)
        oracle = oracle_mod.quantize(bits, dtype, q_rows, q_cols)
        results.append((name, first, second, expect, oracle))
    # bit-exact (tolerance 0), the bar every parity test here uses
    for name, first, second, expect, oracle in results:
        for got in (first, second):
            assert np.array_equal(got[0], oracle[0]) and np.array_equal(got[1], oracle[1]), name
            assert np.array_equal(got[0], expect[0]) and np.array_equal(got[1], expect[1]), name
        if name == "c4":
            rec = kernel_golden["c4"]
            assert (rec["kernel_m"], rec["kernel_k"]) == (1000, 4096)
            assert sha(first[0]) == rec["q_sha256"] and sha(first[1]) == rec["s_sha256"]
    assert capi.noalloc_status(clear=True) == 0
    assert capi.device_status(clear=True) == 0


def test_noalloc_status_reports_and_clears():
    """The checked build skips any store outside its output's bytes and marks
    the status word; with the output window narrowed on purpose, the
    allocation-free entry's word must show that mark, keep it until read
    with clear, and read 0 afterwards.  Nothing faults: the store is skipped."""
    capi = _capi()
    lib = capi.checked_lib()
    bits = inputs.normal(256, 512, 3, "bf16")
    x = torch.from_numpy(bits.view(np.int16)).cuda()
    s_bytes = capi.scale_storage_bytes(256, 512)
    q = torch.zeros((256, 512), dtype=torch.uint8, device="cuda")
    s = torch.zeros((s_bytes,), dtype=torch.uint8, device="cuda")
    word = ctypes.c_uint32(0)
    byref = ctypes.byref
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        return lib.mxfp8_quantize_noalloc(x.data_ptr(), 0, 256, 512, 512, q.data_ptr(), 256, 512, 512, s.data_ptr(),
                                          s_bytes, stream)

    assert lib.mxfp8_noalloc_status(byref(word), 1) == 0  # start clean
    assert call() == 0
    assert lib.mxfp8_noalloc_status(byref(word), 0) == 0 and word.value == 0
    assert lib.mxfp8_checked_window_slack(16) == 0  # the last 16 bytes of each output are out of bounds now
    try:
        assert call() == 0
    finally:
        assert lib.mxfp8_checked_window_slack(0) == 0
    assert lib.mxfp8_noalloc_status(byref(word), 0) == 0 and word.value == 16
    assert call() == 0  # sticky: a clean call does not clear it
    assert lib.mxfp8_noalloc_status(byref(word), 1) == 0 and word.value == 16
    assert lib.mxfp8_noalloc_status(byref(word), 0) == 0 and word.value == 0
    # the allocating entry's word saw none of it
    assert lib.mxfp8_device_status(byref(word), 1) == 0 and word.value == 0


def build_alloc_probe(out_dir: pathlib.Path) -> pathlib.Path:
    """Compile tests/alloc_probe.c against the toolkit's CUPTI."""
    cuda = pathlib.Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "targets" / "x86_64-linux"
    so = out_dir / "alloc_probe.so"
    subprocess.run(["gcc", "-O2", "-shared", "-fPIC", f"-I{cuda / 'include'}", "-o", str(so),
                    str(HERE / "alloc_probe.c"), f"-L{cuda / 'lib'}", "-lcupti", f"-Wl,-rpath,{cuda / 'lib'}"],
                   check=True, capture_output=True, text=True)
    return so


def test_first_noalloc_call_allocates_nothing(tmp_path, oracle_mod):
    """In a fresh process, a CUPTI subscriber counts every allocating CUDA
    driver call: none during the first and second allocation-free calls or
    the status reads; the allocating entry's first call, as a control, makes
    one (its status word), which shows the probe sees the library's calls."""
    m, k = 512, 2048
    bits = inputs.normal(m, k, 21, "bf16")
    np.save(tmp_path / "x.npy", bits)
    probe = build_alloc_probe(tmp_path)
    out = subprocess.run([sys.executable, str(HERE / "noalloc_child.py"), str(tmp_path / "x.npy"),
                          str(tmp_path / "q.npy"), str(tmp_path / "s.npy"), str(m), str(k), str(probe)],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-3000:]
    r = json.loads(out.stdout.strip().splitlines()[-1])
    assert r["rc"] == [0, 0, 0, 0, 0], r
    assert r["status"] == [0, 0], r
    assert r["setup_allocs"] >= 5, f"the probe did not see the child's own buffer allocations: {r}"
    c = r["alloc_counts"]
    assert c[1] == c[0] and c[2] == c[0] and c[3] == c[0] and c[4] == c[0], f"allocation-free calls allocated: {r}"
    assert c[5] > c[4] and r["control_call"].startswith("cuMemAlloc"), f"control saw no allocation: {r}"
    q_ref, s_ref = oracle_mod.quantize(bits, "bf16", m, k)
    assert np.array_equal(np.load(tmp_path / "q.npy"), q_ref)
    assert np.array_equal(np.load(tmp_path / "s.npy"), s_ref)


def test_noalloc_rejects_bad_arguments_like_the_allocating_entry():
    capi = _capi()
    for entry in (capi.quantize, capi.quantize_noalloc):
        with pytest.raises(ValueError):
            entry(0x1000, 0, 16, 256, 256, 0x2000, 16, 250, 256, 0x3000, 1 << 20, 0)
        with pytest.raises(ValueError):
            entry(0x1000, 0, 16, 256, 256, 0x2000, 16, 256, 256, 0x3000, 10, 0)
        with pytest.raises(ValueError):
            entry(0x1000, 5, 16, 256, 256, 0x2000, 16, 256, 256, 0x3000, 1 << 20, 0)
