"""The checked build (libmxfp8_checked.so, include/mxfp8_checked.h) on the GPU.

Every global store of its kernels is tested against the bytes of the output
it belongs to; a store outside them is skipped and sets bit 16 of the device
status word.  Run over a battery of layouts, it must write exactly the bytes
the product library writes (canaries around and between the outputs
included) and report nothing: no kernel store leaves its output.  With the
windows narrowed on purpose, the guards must skip the stores at the end of
each output and report them (the skipped bytes lie inside the test's own
buffers, so no access leaves allocated memory).
"""

import ctypes

import numpy as np
import pytest
import torch

import inputs

pytestmark = pytest.mark.gpu

CANARY = 0x5A
BOUNDS_BIT = 16


@pytest.fixture(scope="module")
def libs():
    import MXFP8_quantizer

    capi = MXFP8_quantizer.load_package()._capi
    return capi, capi.lib(), capi.checked_lib()


def status_of(L):
    v = ctypes.c_uint32(0)
    assert L.mxfp8_device_status(ctypes.byref(v), 1) == 0
    return v.value


def run_quantize(L, capi, bits, dtype, q_rows, q_cols, ld_x=None, x_offset=0, ld_q=None, q_offset=0, s_offset=0):
    m, k = bits.shape
    ld_x = ld_x or max(k, 1)
    ld_q = ld_q or q_cols
    xbuf = torch.zeros(m * ld_x + x_offset + 8, dtype=torch.int16, device="cuda")
    if m and k:
        xbuf[x_offset:x_offset + m * ld_x].view(m, ld_x)[:, :k] = torch.from_numpy(bits.view(np.int16)).cuda()
    s_bytes = capi.scale_storage_bytes(q_rows, q_cols)
    qbuf = torch.full((q_rows * ld_q + q_offset + 64,), CANARY, dtype=torch.uint8, device="cuda")
    sbuf = torch.full((s_bytes + s_offset + 64,), CANARY, dtype=torch.uint8, device="cuda")
    x_ptr = xbuf.data_ptr() + 2 * x_offset if m and k else None
    rc = L.mxfp8_quantize(x_ptr, 0 if dtype == "bf16" else 1, m, k, ld_x, qbuf.data_ptr() + q_offset, q_rows, q_cols,
                          ld_q, sbuf.data_ptr() + s_offset, s_bytes, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    return qbuf.cpu().numpy(), sbuf.cpu().numpy()


CASES = [
    # (m, k, dtype, q_rows, q_cols, layout kwargs)
    (256, 1024, "bf16", 256, 1024, {}),                                    # tensor path
    (1000, 4064, "bf16", 1000, 4096, {}),                                  # reference geometry, ragged K
    (333, 544, "fp16", 336, 544, dict(ld_x=547)),                          # row path, odd stride
    (129, 8191, "bf16", 136, 8192, dict(x_offset=3)),                      # row path, offset, odd K
    (300, 1000, "bf16", 300, 1024, dict(q_offset=3, s_offset=4)),          # any-offset stores, realigned
    (200, 640, "fp16", 200, 640, dict(ld_q=655)),                          # Q rows at every alignment
    (77, 520, "bf16", 77, 544, dict(ld_x=777, q_offset=8, s_offset=12)),   # row path + 8-byte stores
    (0, 0, "bf16", 100, 64, {}),                                           # empty X: plain-load kernel
    (1, 65535 * 256, "bf16", 8, 65535 * 256, {}),                          # the reference's widest launch
]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}x{c[1]}-{c[2]}-{'-'.join(c[5]) or 'plain'}" for c in CASES])
def test_checked_build_writes_the_product_bytes_and_reports_nothing(case, libs):
    capi, prod, checked = libs
    m, k, dtype, q_rows, q_cols, kw = case
    bits = inputs.normal(m, k, m + 7 * k, dtype, sigma=3.0) if m and k else np.zeros((m, k), np.uint16)
    status_of(prod), status_of(checked)
    q_p, s_p = run_quantize(prod, capi, bits, dtype, q_rows, q_cols, **kw)
    q_c, s_c = run_quantize(checked, capi, bits, dtype, q_rows, q_cols, **kw)
    assert np.array_equal(q_p, q_c) and np.array_equal(s_p, s_c)
    assert status_of(prod) == 0
    assert status_of(checked) == 0


@pytest.mark.parametrize("out_dtype,ld_out", [(0, 96), (1, 97), (2, 101)])
def test_checked_build_dequantize(out_dtype, ld_out, libs):
    capi, prod, checked = libs
    m, k = 64, 96
    q = torch.randint(0, 256, (m, k), dtype=torch.uint8, device="cuda")
    q[q == 0x7F] = 0
    q[q == 0xFF] = 0
    s_bytes = capi.scale_storage_bytes(m, k)
    s = torch.randint(100, 150, (s_bytes,), dtype=torch.uint8, device="cuda")
    esize = 4 if out_dtype == 2 else 2
    outs = []
    for L in (prod, checked):
        out = torch.full((m * ld_out * esize + 64,), CANARY, dtype=torch.uint8, device="cuda")
        rc = L.mxfp8_dequantize(q.data_ptr(), m, k, k, s.data_ptr(), s_bytes, out.data_ptr(), out_dtype, ld_out,
                                torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    assert status_of(checked) == 0


@pytest.mark.parametrize("kw,q_rows,q_cols,m,k", [
    ({}, 256, 1024, 256, 1024),                           # tensor path, 16-byte stores
    (dict(q_offset=3, s_offset=4), 128, 512, 128, 512),   # realigned stores and 4-byte scale stores
    ({}, 100, 64, 0, 0),                                  # plain-load kernel (empty X)
])
def test_checked_guards_skip_and_report_stores_outside_a_narrowed_window(kw, q_rows, q_cols, m, k, libs):
    capi, prod, checked = libs
    slack = 24
    bits = inputs.normal(m, k, 11, "bf16") if m and k else np.zeros((m, k), np.uint16)
    q_off, s_off = kw.get("q_offset", 0), kw.get("s_offset", 0)
    q_end = q_off + q_rows * q_cols            # one past Q's last byte in the test buffer
    s_end = s_off + capi.scale_storage_bytes(q_rows, q_cols)
    q_p, s_p = run_quantize(prod, capi, bits, "bf16", q_rows, q_cols, **kw)
    status_of(checked)
    assert checked.mxfp8_checked_window_slack(slack) == 0
    try:
        q_c, s_c = run_quantize(checked, capi, bits, "bf16", q_rows, q_cols, **kw)
        status = status_of(checked)
    finally:
        assert checked.mxfp8_checked_window_slack(0) == 0
    assert status & BOUNDS_BIT
    # the last `slack` bytes of each output were not written; up to one store
    # width (16 bytes) before them may be skipped too; all else is the product's
    assert (q_c[q_end - slack:q_end] == CANARY).all() and (s_c[s_end - slack:s_end] == CANARY).all()
    assert np.array_equal(q_c[:q_end - slack - 16], q_p[:q_end - slack - 16])
    assert np.array_equal(s_c[:s_end - slack - 16], s_p[:s_end - slack - 16])
    assert np.array_equal(q_c[q_end:], q_p[q_end:]) and np.array_equal(s_c[s_end:], s_p[s_end:])
    # with exact windows the checked build reports nothing again
    run_quantize(checked, capi, bits, "bf16", q_rows, q_cols, **kw)
    assert status_of(checked) == 0
