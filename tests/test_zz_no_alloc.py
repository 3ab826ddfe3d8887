"""The allocation-free entry point, mxfp8_quantize_noalloc, through the C ABI.

It exists for callers that may not call cudaMalloc (code inside CUDA graph
capture, plugins whose host owns all device memory, devices whose memory is
fully reserved by another allocator): mxfp8_quantize allocates a small status
buffer on its first call per device, this entry never allocates.  Its output
must be byte-identical to mxfp8_quantize's, call after call, although every
call shares one fixed scratch array that keeps the previous call's contents.

This file sorts last so a stop-at-first-failure run has already run every
other test; it also passes on its own in a fresh process (the allocation-free
call comes first there, before anything else touched the library).
"""

import numpy as np
import pytest
import torch

import inputs

pytestmark = pytest.mark.gpu


def _capi():
    import MXFP8_quantizer

    return MXFP8_quantizer.load_package()._capi


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
    # (bits generator, dtype, q_rows, q_cols): special values in the
    # reference's padded geometry, then a different shape and dtype
    (lambda: inputs.special_values_bf16(), "bf16", 1000, 4096),
    (lambda: inputs.normal(2051, 2080, 14, "fp16"), "fp16", 2056, 2304),
    # odd K: X rows are not 16-byte aligned (the per-phase tensor-map path)
    (lambda: inputs.normal(1001, 4095, 15, "bf16"), "bf16", 1001, 4096),
]


def test_noalloc_matches_allocating_entry_two_calls_in_a_row():
    capi = _capi()
    assert torch.cuda.is_available()
    results = []
    for gen, dtype, q_rows, q_cols in CASES:
        bits = gen()
        # allocation-free entry first, twice in a row, before the allocating one
        first = _run(capi.quantize_noalloc, bits, dtype, q_rows, q_cols)
        second = _run(capi.quantize_noalloc, bits, dtype, q_rows, q_cols)
        expect = _run(capi.quantize, bits, dtype, q_rows, q_cols)
        results.append((first, second, expect))
    for first, second, expect in results:
        # bit-exact, the tolerance every parity test here uses
        assert np.array_equal(first[0], expect[0]) and np.array_equal(first[1], expect[1])
        assert np.array_equal(second[0], expect[0]) and np.array_equal(second[1], expect[1])
    assert capi.device_status(clear=True) == 0


def test_noalloc_rejects_bad_arguments_like_the_allocating_entry():
    capi = _capi()
    with pytest.raises(ValueError):
        capi.quantize_noalloc(0x1000, 0, 16, 256, 256, 0x2000, 16, 250, 256, 0x3000, 1 << 20, 0)
    with pytest.raises(ValueError):
        capi.quantize_noalloc(0x1000, 0, 16, 256, 256, 0x2000, 16, 256, 256, 0x3000, 10, 0)
