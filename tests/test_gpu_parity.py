"""GPU parity: libmxfp8.so (called through its C ABI) against the CPU oracle
and the reference-recipe digests.  Bit-exact on every byte of Q and of the
packed scale storage."""

import hashlib

import numpy as np
import pytest
import torch

import inputs
from make_golden import CASES

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(1234)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def capi():
    import MXFP8_quantizer

    pkg = MXFP8_quantizer.load_package()
    pkg._capi.lib()
    assert torch.cuda.is_available()
    return pkg._capi


def to_dev(bits, pad_ld=None, offset_elems=0):
    """bits (m, k) uint16 -> device tensor view with row stride pad_ld and a
    start offset (for the strided / misaligned layouts)."""
    m, k = bits.shape
    ld = pad_ld or k
    buf = torch.zeros(m * ld + offset_elems + 8, dtype=torch.int16, device="cuda")
    view = buf[offset_elems:offset_elems + m * ld].view(m, ld)
    view[:, :k] = torch.from_numpy(bits.view(np.int16)).cuda()
    return buf, view, ld


def gpu_quantize(capi, bits, dtype, q_rows, q_cols, ld_x=None, x_offset=0, q_offset=0, ld_q=None, garbage=0xAB,
                 s_offset=0):
    m, k = bits.shape
    _, xv, ld = to_dev(bits, ld_x, x_offset)
    ld_q = ld_q or q_cols
    s_bytes = capi.scale_storage_bytes(q_rows, q_cols)
    qbuf = torch.full((q_rows * ld_q + q_offset + 64,), garbage, dtype=torch.uint8, device="cuda")
    sbuf = torch.full((s_bytes + s_offset + 64,), garbage, dtype=torch.uint8, device="cuda")
    code = 0 if dtype == "bf16" else 1
    capi.quantize(xv.data_ptr(), code, m, k, ld, qbuf.data_ptr() + q_offset, q_rows, q_cols, ld_q,
                  sbuf.data_ptr() + s_offset, s_bytes, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert capi.device_status(clear=True) == 0
    qb = qbuf.cpu().numpy()
    sb = sbuf.cpu().numpy()
    # bytes outside the output region must be untouched
    assert (qb[:q_offset] == garbage).all() and (qb[q_offset + q_rows * ld_q:] == garbage).all()
    assert (sb[:s_offset] == garbage).all() and (sb[s_offset + s_bytes:] == garbage).all()
    q = qb[q_offset:q_offset + q_rows * ld_q].reshape(q_rows, ld_q)
    if ld_q > q_cols:
        assert (q[:, q_cols:] == garbage).all()
    return np.ascontiguousarray(q[:, :q_cols]), sb[s_offset:s_offset + s_bytes]


def check_against_oracle(capi, oracle_mod, bits, dtype, q_rows=None, q_cols=None, **kw):
    m, k = bits.shape
    if q_rows is None:
        q_rows, q_cols = oracle_mod.padded_shape(max(m, 1), max(k, 1))
    q_ref, s_ref = oracle_mod.quantize(bits, dtype, q_rows, q_cols)
    q, s = gpu_quantize(capi, bits, dtype, q_rows, q_cols, **kw)
    if not np.array_equal(q, q_ref):
        bad = np.argwhere(q != q_ref)
        r, c = bad[0]
        raise AssertionError(f"payload mismatch at {len(bad)} bytes, first ({r},{c}): gpu {q[r, c]:#x} "
                             f"oracle {q_ref[r, c]:#x}; x block = {bits[r, c // 32 * 32:(c // 32 + 1) * 32] if r < m else 'pad'}")
    if not np.array_equal(s, s_ref):
        bad = np.flatnonzero(s != s_ref)
        raise AssertionError(f"scale mismatch at {len(bad)} bytes, first offset {bad[0]}: gpu {s[bad[0]]} "
                             f"oracle {s_ref[bad[0]]}")
    return q, s


@pytest.mark.parametrize("name", list(CASES))
def test_reference_digests(name, capi, golden):
    rec = golden["cases"][name]
    desc, gen, dtype = CASES[name]
    bits = gen()
    q, s = gpu_quantize(capi, bits, dtype, rec["kernel_m"], rec["kernel_k"])
    assert sha(q) == rec["q_sha256"], f"{name}: payload differs from the reference recipe"
    assert sha(s) == rec["s_sha256"], f"{name}: packed scales differ from the reference recipe"


@pytest.mark.parametrize("name", ["c4", "c4_ragged", "nonfinite_bf16", "nonfinite_fp16", "c1", "c2"])
def test_reference_kernel_digests(name, capi):
    """Bit-exact against the reference's CuTeDSL kernel run on a B200
    (tests/golden/make_kernel_golden.py), special values included."""
    import json
    import pathlib

    from make_kernel_golden import KERNEL_CASES

    rec = json.loads((pathlib.Path(__file__).parent / "golden" / "golden_kernel.json").read_text())["cases"][name]
    desc, gen, dtype = KERNEL_CASES[name]
    q, s = gpu_quantize(capi, gen(), dtype, rec["kernel_m"], rec["kernel_k"])
    assert sha(q) == rec["q_sha256"], f"{name}: payload differs from the reference kernel"
    assert sha(s) == rec["s_sha256"], f"{name}: packed scales differ from the reference kernel"


@pytest.mark.parametrize("geometry", ["reference", "tight"])
def test_special_values_c4(geometry, capi, oracle_mod):
    bits = inputs.special_values_bf16()
    if geometry == "reference":
        check_against_oracle(capi, oracle_mod, bits, "bf16")
    else:
        check_against_oracle(capi, oracle_mod, bits, "bf16", 1000, 4064)


@pytest.mark.parametrize("layout", ["aligned", "unaligned_rows"])
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_special_values_every_nonfinite_pattern(dtype, layout, capi, oracle_mod):
    """Every inf/NaN pattern, through one tensor map (aligned X) and through
    the per-row-phase maps (row stride 37, X 6 bytes past a 16-byte boundary)."""
    kw = {} if layout == "aligned" else dict(ld_x=37, x_offset=3)
    check_against_oracle(capi, oracle_mod, inputs.nonfinite_patterns(dtype), dtype, **kw)


SHAPES = [(1, 1), (1, 32), (2, 64), (7, 33), (8, 256), (9, 255), (127, 129), (128, 128), (129, 4064),
          (300, 8), (17, 1000), (256, 1024), (1000, 4064), (2051, 2080), (640, 4352), (1, 16384)]


@pytest.mark.parametrize("m,k", SHAPES)
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_ragged_shapes_reference_geometry(m, k, dtype, capi, oracle_mod):
    bits = inputs.normal(m, k, m * 7919 + k, dtype, sigma=3.0)
    check_against_oracle(capi, oracle_mod, bits, dtype)


@pytest.mark.parametrize("m,k", SHAPES)
def test_ragged_shapes_tight_geometry(m, k, capi, oracle_mod):
    bits = inputs.special_values_bf16(m, max(32, (k + 31) // 32 * 32), seed=m + k)[:, :k].copy()
    check_against_oracle(capi, oracle_mod, bits, "bf16", m, (k + 31) // 32 * 32)


@pytest.mark.parametrize("layout", ["x_ld_odd", "x_misaligned", "q_misaligned", "s_word_aligned_only",
                                    "x_strided_tma", "q_strided", "q_ld_odd", "q_8_byte_offset"])
def test_layouts(layout, capi, oracle_mod):
    bits = inputs.normal(333, 544, 5, "fp16")
    kw = {}
    if layout == "x_ld_odd":
        kw = dict(ld_x=547)          # row stride not a multiple of 8 -> row path
    elif layout == "x_misaligned":
        kw = dict(x_offset=1)        # 2-byte aligned only -> row path
    elif layout == "q_misaligned":
        kw = dict(q_offset=3)        # Q at an odd offset -> byte stores
    elif layout == "s_word_aligned_only":
        kw = dict(s_offset=4)
    elif layout == "x_strided_tma":
        kw = dict(ld_x=1024)         # TMA with a row stride
    elif layout == "q_strided":
        kw = dict(ld_q=800)
    elif layout == "q_ld_odd":
        kw = dict(ld_q=555)          # Q rows at every byte alignment
    elif layout == "q_8_byte_offset":
        kw = dict(q_offset=8, s_offset=12)
    check_against_oracle(capi, oracle_mod, bits, "fp16", 336, 544, **kw)


@pytest.mark.parametrize("m,k,q_rows,q_cols", [(0, 0, 100, 64), (5, 0, 8, 32), (0, 7, 129, 32), (3, 0, 3, 4096)])
def test_empty_x_writes_padding(m, k, q_rows, q_cols, capi, oracle_mod):
    """Empty X (the plain-load kernel): every Q byte 0, scale 127 inside the
    geometry and 0 beyond it, as the reference's zero-padded launch gives."""
    bits = np.zeros((m, k), dtype=np.uint16)
    q, s = check_against_oracle(capi, oracle_mod, bits, "bf16", q_rows, q_cols)
    assert not q.any()
    assert set(np.unique(s)) <= {0, 127}


def test_padded_entry_point_matches_general(capi, oracle_mod):
    bits = inputs.normal(1024, 2048, 77)
    x = torch.from_numpy(bits.view(np.int16)).cuda()
    s_bytes = capi.scale_storage_bytes(1024, 2048)
    q = torch.empty((1024, 2048), dtype=torch.uint8, device="cuda")
    s = torch.empty((s_bytes // 4,), dtype=torch.int32, device="cuda")
    capi.quantize_padded(x.data_ptr(), q.data_ptr(), s.data_ptr(), 1024, 2048, s_bytes // 4, 0,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    q_ref, s_ref = oracle_mod.quantize(bits, "bf16", 1024, 2048)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy().view(np.uint8), s_ref)
    with pytest.raises(ValueError):
        capi.quantize_padded(x.data_ptr(), q.data_ptr(), s.data_ptr(), 1001, 2048, s_bytes // 4, 0, 0)


@pytest.mark.slow
def test_row_sharded_c5_shape_matches_unsharded(capi, oracle_mod):
    """Config 5's 131072 x 16384 bf16 N(0, 2) matrix, quantized whole and as 8
    row shards of 128-row chunks (one per GPU of an 8-GPU run): the shards'
    Q and S are contiguous slices of the whole result, byte for byte.  A few
    row chunks are also checked against the oracle."""
    m, k = 131072, 16384
    g = torch.Generator(device="cuda").manual_seed(4)
    x = (torch.randn((m, k), generator=g, device="cuda", dtype=torch.float32) * 2.0).to(torch.bfloat16)
    s_bytes = capi.scale_storage_bytes(m, k)
    q = torch.empty((m, k), dtype=torch.uint8, device="cuda")
    s = torch.empty((s_bytes,), dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    capi.quantize(x.data_ptr(), 0, m, k, k, q.data_ptr(), m, k, k, s.data_ptr(), s_bytes, st)
    rows = m // 8
    per_s = capi.scale_storage_bytes(rows, k)
    qs = torch.empty((rows, k), dtype=torch.uint8, device="cuda")
    ss = torch.empty((per_s,), dtype=torch.uint8, device="cuda")
    for r in range(8):
        xr = x[r * rows:(r + 1) * rows]
        capi.quantize(xr.data_ptr(), 0, rows, k, k, qs.data_ptr(), rows, k, k, ss.data_ptr(), per_s, st)
        assert torch.equal(qs, q[r * rows:(r + 1) * rows])
        assert torch.equal(ss, s[r * per_s:(r + 1) * per_s])
    torch.cuda.synchronize()
    chunk_bytes = capi.scale_storage_bytes(128, k)
    for c in (0, 377, 1023):
        xb = x[c * 128:(c + 1) * 128].view(torch.int16).cpu().numpy().view(np.uint16)
        q_ref, s_ref = oracle_mod.quantize(xb, "bf16", 128, k)
        assert np.array_equal(q[c * 128:(c + 1) * 128].cpu().numpy(), q_ref)
        assert np.array_equal(s[c * chunk_bytes:(c + 1) * chunk_bytes].cpu().numpy(), s_ref)
    del x, q, s
    torch.cuda.empty_cache()


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_dequantize_matches_oracle(out_dtype, capi, oracle_mod):
    import MXFP8_quantizer

    pkg = MXFP8_quantizer.load_package()
    bits = inputs.special_values_bf16(256, 1024, seed=8)
    x = inputs.bits_to_torch(bits, "bf16").cuda()
    q, s = pkg.quantize(x, q_rows=256, q_cols=1024)
    y = pkg.dequantize(q, s, out_dtype)
    torch.cuda.synchronize()
    ref = oracle_mod.dequantize(q.view(torch.uint8).cpu().numpy(), s.cpu().numpy())
    ref_t = torch.from_numpy(ref).to(out_dtype).float()
    got = y.float().cpu()
    both_nan = torch.isnan(got) & torch.isnan(ref_t)
    assert torch.equal(torch.where(both_nan, 0.0, got), torch.where(both_nan, 0.0, ref_t))


def test_drop_in_api_small(capi):
    import MXFP8_quantizer

    r = MXFP8_quantizer.run_quantizer(m=2051, k=2080, input_dtype="fp16", warmup_iterations=2, iterations=5,
                                      benchmark_repeats=2)
    assert r["verification_passed"] and r["q_max_byte_diff"] == 0 and r["scale_bytes_exact"]
    assert r["kernel_m"] == 2056 and r["kernel_k"] == 2304 and r["runtime_min_us"] > 0
    res = MXFP8_quantizer.prepare_and_quantize(1000, 4064, "bf16", 3, None)
    assert res["kernel_k"] == 4096 and res["verify"]["q_max_byte_diff"] == 0
    s = res["buffers"]["s_storage_bytes"].cpu().numpy()
    pkg = MXFP8_quantizer.load_package()
    dense = pkg.decode_scale_bytes(torch.from_numpy(s), 1024, 4096).numpy()
    assert (dense[:1000, 127] == 127).all() and (dense[1000:] == 0).all()
    # the returned dicts carry exactly the reference's keys at run time too
    import json
    import pathlib

    keys = json.loads((pathlib.Path(__file__).parent / "golden" / "api_signatures.json").read_text())["return_keys"]
    assert sorted(r) == keys["run_quantizer"]
    assert sorted(res) == keys["prepare_and_quantize"]
    assert sorted(res["buffers"]) == keys["materialize_quantizer_buffers"]
    assert sorted(res["verify"]) == keys["verify_quantizer_outputs"]


def test_cold_l2_benchmark_mode(capi):
    import MXFP8_quantizer

    r = MXFP8_quantizer.run_quantizer(m=4096, k=4096, warmup_iterations=2, iterations=4, benchmark_repeats=1,
                                      cold_l2=True)
    assert r["workspace_count"] > 1 and r["verification_passed"]


@pytest.mark.parametrize("cfg", [(1024, 1024, 2048, "bf16", 0), (1024, 2048, 4096, "fp16", 2)])
def test_e2e_blockscaled_gemm(cfg, capi):
    import MXFP8_quantizer

    m, n, k, dt, seed = cfg
    r = MXFP8_quantizer.run_e2e_verification(m=m, n=n, k=k, input_dtype=dt, seed=seed)
    assert r["e2e_verification_passed"] and r["max_err_ratio"] < 1.0


def test_status_word_clean(capi):
    assert capi.device_status(clear=False) == 0


def test_dependent_back_to_back_launches_on_shared_buffers(capi, oracle_mod):
    """The quantizer starts early (programmatic dependent launch) and prefetches
    X into L2 before waiting for the previous kernel.  Here every step first
    overwrites X in place with another kernel, then quantizes it into the same
    Q/S buffers, then copies Q/S out: each result must match its own input."""
    m, k = 2048, 4096
    srcs = [inputs.normal(m, k, 300 + i, sigma=float(i + 1)) for i in range(4)]
    dev = [torch.from_numpy(b.view(np.int16)).cuda() for b in srcs]
    expect = [oracle_mod.quantize(b, "bf16", m, k) for b in srcs]
    sb = capi.scale_storage_bytes(m, k)
    x = torch.empty_like(dev[0])
    q = torch.empty((m, k), dtype=torch.uint8, device="cuda")
    s = torch.empty((sb,), dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    outs = []
    for step in range(24):
        x.copy_(dev[step % 4])
        capi.quantize(x.data_ptr(), 0, m, k, k, q.data_ptr(), m, k, k, s.data_ptr(), sb, st)
        if step % 3 == 2:  # also chain quantizer -> quantizer on the same buffers
            capi.quantize(x.data_ptr(), 0, m, k, k, q.data_ptr(), m, k, k, s.data_ptr(), sb, st)
        outs.append((q.clone(), s.clone()))
    torch.cuda.synchronize()
    for step, (qq, ss) in enumerate(outs):
        q_ref, s_ref = expect[step % 4]
        assert np.array_equal(qq.cpu().numpy(), q_ref), step
        assert np.array_equal(ss.cpu().numpy(), s_ref), step


def test_bounded_wait_times_out_and_reports(capi, golden):
    """Failure path without a GPU fault: an mbarrier wait that nothing
    completes gives up after its limit, sets the status bit, and the context
    keeps working (a quantization right after is still bit-exact)."""
    import time

    assert capi.device_status(clear=True) == 0
    t0 = time.perf_counter()
    capi.selftest_bounded_wait(50_000, torch.cuda.current_stream().cuda_stream)  # 50 ms
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert capi.device_status(clear=True) == 8
    assert 0.04 < elapsed < 5.0
    assert capi.device_status(clear=False) == 0
    q, s = gpu_quantize(capi, inputs.normal(256, 1024, 0), "bf16", 256, 1024)   # config 1
    assert sha(q) == golden["cases"]["c1"]["q_sha256"] and sha(s) == golden["cases"]["c1"]["s_sha256"]


@pytest.mark.parametrize("use_graph", [True, False])
@pytest.mark.parametrize("m,k,dtype", [(2500, 1000, "fp16"), (1300, 777, "bf16")])
def test_host_quantizer_matches_device_path(m, k, dtype, use_graph, capi, oracle_mod):
    """HostQuantizer (pinned host X in, host Q/S out, row chunks over three
    streams, replayed from a CUDA graph or enqueued eagerly) gives the bytes
    of the device path, for a ragged row count; odd K takes the device's
    per-phase tensor-map path."""
    import MXFP8_quantizer

    pkg = MXFP8_quantizer.load_package()
    bits = inputs.normal(m, k, 55, dtype, sigma=4.0)
    x_host = inputs.bits_to_torch(bits, dtype).pin_memory()
    hq = pkg.HostQuantizer(m, k, torch.float16 if dtype == "fp16" else torch.bfloat16, chunk_rows=512,
                           use_graph=use_graph)
    q_host = torch.empty((m, hq.q_cols), dtype=torch.uint8).pin_memory()
    s_host = torch.empty((hq.s_bytes,), dtype=torch.uint8).pin_memory()
    for _ in range(2):
        hq(x_host, q_host, s_host)
    torch.cuda.synchronize()
    q_ref, s_ref = oracle_mod.quantize(bits, dtype, m, hq.q_cols)
    assert np.array_equal(q_host.numpy(), q_ref)
    assert np.array_equal(s_host.numpy(), s_ref)


def test_host_quantizer_graph_replays_read_the_buffers_anew(capi, oracle_mod):
    """A replayed call copies whatever the pinned X holds now (new values in
    the same buffer give their own Q and S), and new buffers are captured
    afresh."""
    import MXFP8_quantizer

    pkg = MXFP8_quantizer.load_package()
    m, k = 1100, 2048
    hq = pkg.HostQuantizer(m, k, torch.bfloat16, chunk_rows=256)
    x_host = torch.empty((m, k), dtype=torch.bfloat16).pin_memory()
    q_host = torch.empty((m, hq.q_cols), dtype=torch.uint8).pin_memory()
    s_host = torch.empty((hq.s_bytes,), dtype=torch.uint8).pin_memory()
    for seed in (61, 62, 63):  # eager + capture, then two replays with new values
        bits = inputs.normal(m, k, seed, "bf16", sigma=3.0)
        x_host.copy_(inputs.bits_to_torch(bits, "bf16"))
        hq(x_host, q_host, s_host)
        torch.cuda.synchronize()
        q_ref, s_ref = oracle_mod.quantize(bits, "bf16", m, hq.q_cols)
        assert np.array_equal(q_host.numpy(), q_ref) and np.array_equal(s_host.numpy(), s_ref), seed
    bits = inputs.normal(m, k, 64, "bf16")
    x2 = inputs.bits_to_torch(bits, "bf16").pin_memory()
    q2 = torch.zeros_like(q_host).pin_memory()
    s2 = torch.zeros_like(s_host).pin_memory()
    for _ in range(2):
        hq(x2, q2, s2)
    torch.cuda.synchronize()
    q_ref, s_ref = oracle_mod.quantize(bits, "bf16", m, hq.q_cols)
    assert np.array_equal(q2.numpy(), q_ref) and np.array_equal(s2.numpy(), s_ref)
    assert capi.device_status(clear=True) == 0


def test_dequantize_unaligned_output_rows(capi, oracle_mod):
    """Output rows that are not 16-byte aligned take the element-store path."""
    m, k = 64, 96
    bits = inputs.normal(m, k, 17, sigma=5.0)
    q_ref, s_ref = oracle_mod.quantize(bits, "bf16", m, k)
    q = torch.from_numpy(q_ref).cuda()
    s = torch.from_numpy(s_ref).cuda()
    ld = k + 1
    out = torch.full((m * ld + 8,), float("nan"), dtype=torch.float32, device="cuda")
    capi.dequantize(q.data_ptr(), m, k, k, s.data_ptr(), s.numel(), out.data_ptr() + 4, capi.F32, ld,
                    torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = out[1:1 + m * ld].view(m, ld)[:, :k].cpu().numpy()
    np.testing.assert_array_equal(got, oracle_mod.dequantize(q_ref, s_ref))


@pytest.mark.parametrize("layout", ["tensor", "unaligned_rows", "q_any_offset"])
def test_quantize_inside_cuda_graph(layout, capi, oracle_mod):
    """Launches captured in a CUDA graph (dependent-launch edges between them)
    replay bit-exactly; inputs are refreshed in place between replays.  Every
    kernel variant: one tensor map, per-row-phase maps, any-offset stores."""
    m = 1024
    k = 2047 if layout == "unaligned_rows" else 2048
    q_cols, q_off = 2048, (3 if layout == "q_any_offset" else 0)
    srcs = [inputs.normal(m, k, 700 + i) for i in range(3)]
    sb = capi.scale_storage_bytes(m, q_cols)
    x = torch.empty((m, k), dtype=torch.int16, device="cuda")
    q = torch.empty((3, m * q_cols + 64), dtype=torch.uint8, device="cuda")
    s = torch.empty((3, sb), dtype=torch.uint8, device="cuda")
    x.copy_(torch.from_numpy(srcs[0].view(np.int16)))
    capi.quantize(x.data_ptr(), 0, m, k, k, q[0].data_ptr() + q_off, m, q_cols, q_cols, s[0].data_ptr(), sb,
                  torch.cuda.current_stream().cuda_stream)      # first call outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st = torch.cuda.current_stream().cuda_stream
        for i in range(3):
            capi.quantize(x.data_ptr(), 0, m, k, k, q[i].data_ptr() + q_off, m, q_cols, q_cols, s[i].data_ptr(),
                          sb, st)
    for src in srcs:
        x.copy_(torch.from_numpy(src.view(np.int16)))
        g.replay()
        torch.cuda.synchronize()
        q_ref, s_ref = oracle_mod.quantize(src, "bf16", m, q_cols)
        for i in range(3):
            got = q[i].cpu().numpy()[q_off:q_off + m * q_cols].reshape(m, q_cols)
            assert np.array_equal(got, q_ref)
            assert np.array_equal(s[i].cpu().numpy(), s_ref)
    del g


# The reference README's published end-to-end results (README.md:162-169 of the reference): max abs error and
# pass margin of its block-scaled GEMM on its quantizer's outputs, per DEFAULT_E2E_SUITE entry.
PUBLISHED_E2E = [(1.07e-4, 650), (1.07e-4, 420), (3.36e-4, 265), (2.44e-4, 259), (1.07e-4, 440), (9.16e-5, 379)]


def test_e2e_suite_reproduces_the_published_errors(capi):
    """Same seeds, same inputs, bit-identical Q and S: the block-scaled GEMM
    on this library's outputs lands on the reference's published errors and
    margins (5 % allowed for the GEMM libraries' accumulation order)."""
    import MXFP8_quantizer

    r = MXFP8_quantizer.run_e2e_suite()
    for got, (err, margin) in zip(r["configs"], PUBLISHED_E2E):
        assert got["max_abs_err"] == pytest.approx(err, rel=0.05), got
        assert got["pass_margin"] == pytest.approx(margin, rel=0.05), got


def test_e2e_suite_all_configs(capi):
    import MXFP8_quantizer

    r = MXFP8_quantizer.run_e2e_suite()
    assert r["e2e_suite_passed"] and r["num_configs"] == 6
    assert all(c["quantizer_verify_passed"] and c["max_err_ratio"] < 1.0 for c in r["configs"])
    import json
    import pathlib

    keys = json.loads((pathlib.Path(__file__).parent / "golden" / "api_signatures.json").read_text())["return_keys"]
    assert sorted(r) == keys["run_e2e_suite"]
    assert sorted(MXFP8_quantizer.run_e2e_verification()) == keys["run_e2e_verification"]


@pytest.mark.parametrize("m,k,x_offset,dtype", [(1000, 4097, 0, "bf16"), (333, 4064, 1, "bf16"), (129, 8191, 3, "fp16"),
                                                (64, 31, 1, "fp16"), (1, 1, 1, "bf16"), (260, 300, 0, "bf16")])
@pytest.mark.parametrize("q_offset", [0, 8, 3])
def test_odd_layouts_special_values(m, k, x_offset, dtype, q_offset, capi, oracle_mod):
    """Odd K and 2-byte aligned X (the pipelined kernel's row path), with Q
    16-byte aligned, 8 bytes off (8-byte stores) or 3 bytes off (realigned
    line stores).  Special values, both geometries."""
    kk = (k + 31) // 32 * 32
    bits = inputs.special_values_bf16(m, kk, seed=k)[:, :k].copy() if dtype == "bf16" else \
        inputs.normal(m, k, k, "fp16", sigma=30.0)
    check_against_oracle(capi, oracle_mod, bits, dtype, x_offset=x_offset, q_offset=q_offset)
    check_against_oracle(capi, oracle_mod, bits, dtype, m, kk, x_offset=x_offset, q_offset=q_offset)


@pytest.mark.parametrize("m", [1, 2, 3, 7, 8, 9, 15, 17, 130])
def test_row_path_few_rows_every_offset(m, capi, oracle_mod):
    """Row path with fewer than 8 rows (fewer tensor-map phases than 8) and
    around multiples of 8, at every 2-byte offset of X and odd / even-not-8
    row strides."""
    for k, ld in ((33, 35), (300, 301), (130, 134)):
        bits = inputs.normal(m, k, m * 1000 + k, "bf16", sigma=3.0)
        for x_offset in range(8):
            check_against_oracle(capi, oracle_mod, bits, "bf16", ld_x=ld, x_offset=x_offset)


@pytest.mark.parametrize("m,k,dtype,geometry", [
    (1, 65535 * 256, "bf16", "reference"),      # the reference's widest launch (65535 K-tiles), tensor path
    (3, 65535 * 256 - 1, "fp16", "tight"),      # as wide, odd K: per-phase tensor maps, 3 phases
    (1 << 20, 32, "fp16", "reference"),        # one scale block per row, 8192 row tiles
    (100003, 33, "bf16", "tight"),             # tall with odd K: row path, ragged last row tile
])
def test_extreme_aspect_ratios(m, k, dtype, geometry, capi, oracle_mod):
    """Very wide and very tall X against the oracle, byte for byte."""
    bits = inputs.normal(m, k, m + k, dtype, sigma=5.0)
    if geometry == "reference":
        check_against_oracle(capi, oracle_mod, bits, dtype)
    else:
        check_against_oracle(capi, oracle_mod, bits, dtype, m, (k + 31) // 32 * 32)


@pytest.mark.parametrize("m,k,q_offset", [(8192, 8192, 0), (38000, 8192, 0), (38000, 8191, 0), (16384, 16383, 0),
                                          (16384, 16384, 1), (38000, 8192, 8)])
def test_launch_count_matches_bench_accounting(m, k, q_offset, capi):
    """The kernel launches one call makes, counted by the CUDA profiler,
    equal bench.py's gpu_launches rule (the launch split by tile count)."""
    import bench
    from torch.profiler import ProfilerActivity, profile

    q_cols = (k + 31) // 32 * 32
    s_bytes = capi.scale_storage_bytes(m, q_cols)
    x = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
    q = torch.empty((m * q_cols + 16,), dtype=torch.uint8, device="cuda")
    s = torch.empty((s_bytes,), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    args = (x.data_ptr(), 0, m, k, k, q.data_ptr() + q_offset, m, q_cols, q_cols, s.data_ptr(), s_bytes, stream)
    capi.quantize(*args)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA], acc_events=True) as prof:
        capi.quantize(*args)
        torch.cuda.synchronize()
    launches = sum(1 for e in prof.events() if "quantize_tma_kernel" in e.name)
    assert launches == bench.launches_per_call(m, k, k, q_any_offset=q_offset % 16 != 0)


def test_three_paths_agree_across_launch_split(capi):
    """38000 x 8191 bf16 (622 MB): the same X through the row path (row
    stride 8191, three launches of 148 + 148 + 1 row tiles), the tensor path
    (row stride 8192, two launches of 296 + 1 row tiles) and the tensor path
    with Q 8 bytes off 16-byte alignment (narrower stores, three launches
    like the row path) gives identical Q and S bytes, in the reference
    geometry."""
    m, k = 38000, 8191
    q_rows, q_cols = (m + 7) // 8 * 8, (k + 255) // 256 * 256
    s_bytes = capi.scale_storage_bytes(q_rows, q_cols)
    g = torch.Generator(device="cuda").manual_seed(7)
    dense = torch.empty(m, 8192, dtype=torch.bfloat16, device="cuda")
    dense.normal_(generator=g)
    dense[:, :k] *= torch.logspace(-3, 3, m, device="cuda").to(torch.bfloat16)[:, None]
    packed = dense[:, :k].contiguous()
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for x, ld, q_off in ((packed, k, 0), (dense, 8192, 0), (dense, 8192, 8)):
        q = torch.full((q_rows * q_cols + 16,), 0xAB, dtype=torch.uint8, device="cuda")
        s = torch.full((s_bytes,), 0xAB, dtype=torch.uint8, device="cuda")
        capi.quantize(x.data_ptr(), 0, m, k, ld, q.data_ptr() + q_off, q_rows, q_cols, q_cols,
                      s.data_ptr(), s_bytes, stream)
        outs.append((q[q_off:q_off + q_rows * q_cols], s))
    torch.cuda.synchronize()
    for q, s in outs[1:]:
        assert torch.equal(q, outs[0][0]) and torch.equal(s, outs[0][1])
    assert capi.device_status(clear=True) == 0


def test_randomized_unaligned_x(capi, oracle_mod):
    """150 seeded random cases whose X rows are not 16-byte aligned (the
    per-row-phase tensor maps): shape, dtype, row stride, 2-byte offset,
    geometry and value distribution."""
    rng = np.random.default_rng(77)
    for case in range(150):
        m = int(rng.integers(1, 600))
        k = int(rng.integers(1, 2000))
        dtype = "bf16" if rng.random() < 0.5 else "fp16"
        ld = k + int(rng.integers(0, 10))
        x_offset = int(rng.integers(0, 8))
        if ld % 8 == 0 and x_offset == 0:
            ld += 1
        if rng.random() < 0.3 and dtype == "bf16":
            kk = (k + 31) // 32 * 32
            bits = inputs.special_values_bf16(m, kk, seed=case)[:, :k].copy()
        else:
            bits = inputs.normal(m, k, 1000 + case, dtype, sigma=float(10 ** rng.uniform(-2, 2)))
        if rng.random() < 0.5:
            check_against_oracle(capi, oracle_mod, bits, dtype, ld_x=ld, x_offset=x_offset)
        else:
            check_against_oracle(capi, oracle_mod, bits, dtype, m, (k + 31) // 32 * 32, ld_x=ld, x_offset=x_offset)


def test_randomized_output_layouts(capi, oracle_mod):
    """60 seeded random cases of Q at any byte offset and row stride and S
    at any 4-byte offset, over aligned and unaligned X."""
    rng = np.random.default_rng(4242)
    for case in range(60):
        m = int(rng.integers(1, 300))
        k = int(rng.integers(1, 1100))
        dtype = "bf16" if rng.random() < 0.5 else "fp16"
        q_cols = (k + 31) // 32 * 32
        kw = dict(q_offset=int(rng.integers(0, 16)), ld_q=q_cols + int(rng.integers(0, 24)),
                  s_offset=4 * int(rng.integers(0, 4)))
        if rng.random() < 0.5:
            kw.update(ld_x=k + int(rng.integers(0, 9)), x_offset=int(rng.integers(0, 8)))
        bits = inputs.normal(m, k, 5000 + case, dtype, sigma=float(10 ** rng.uniform(-2, 2)))
        check_against_oracle(capi, oracle_mod, bits, dtype, m, q_cols, **kw)


@pytest.mark.parametrize("q_offset", range(16))
def test_every_q_offset_with_rows_in_phase(q_offset, capi, oracle_mod):
    """Q at each byte offset within 16 bytes with ld_q % 16 == 0, so every row
    starts at the same offset: the any-offset kernels with the word offset
    built in (offsets 1-3, 5-7, 9-11, 13-15), the 4-byte-aligned rows (4, 8,
    12) and the aligned path (0), ragged M and K, S at a 4-byte offset."""
    dtype = "bf16" if q_offset % 2 else "fp16"
    bits = inputs.normal(300, 1000, 700 + q_offset, dtype, sigma=7.0)
    check_against_oracle(capi, oracle_mod, bits, dtype, 300, 1024, q_offset=q_offset, ld_q=1024 + 16 * (q_offset % 3),
                         s_offset=4 * (q_offset % 4))


def test_randomized_shapes_layouts_and_values(capi, oracle_mod):
    """40 seeded random cases: shape, dtype, geometry, row stride, base offset
    and value distribution (normal, log-uniform with specials, subnormal-heavy)."""
    rng = np.random.default_rng(2024)
    for case in range(40):
        m = int(rng.integers(1, 400))
        k = int(rng.integers(1, 1500))
        dtype = "bf16" if rng.random() < 0.6 else "fp16"
        kind = rng.integers(0, 3)
        if kind == 0:
            bits = inputs.normal(m, k, case, dtype, sigma=float(10 ** rng.uniform(-3, 3)))
        elif kind == 1 and dtype == "bf16":
            kk = (k + 31) // 32 * 32
            bits = inputs.special_values_bf16(m, kk, seed=case)[:, :k].copy()
        else:
            bits = inputs.normal(m, k, case, dtype)
            sub = rng.random((m, k)) < 0.3
            bits[sub] = rng.integers(0, 0x80 if dtype == "bf16" else 0x400, size=int(sub.sum())).astype(np.uint16)
        kw = {}
        r = rng.random()
        if r < 0.2:
            kw["ld_x"] = k + int(rng.integers(1, 40))
        elif r < 0.35:
            kw["x_offset"] = int(rng.integers(1, 8))
        if rng.random() < 0.5:
            check_against_oracle(capi, oracle_mod, bits, dtype, **kw)
        else:
            check_against_oracle(capi, oracle_mod, bits, dtype, m, (k + 31) // 32 * 32, **kw)


def test_reference_compatible_clis_run(capi):
    """benchmark.py and e2e.py, run as the reference's users run its tools,
    print their JSON summaries with a passing check."""
    import json
    import pathlib
    import subprocess
    import sys

    root = pathlib.Path(__file__).resolve().parent.parent

    def run(*argv):
        out = subprocess.run([sys.executable, *argv], cwd=root, capture_output=True, text=True, timeout=600)
        assert out.returncode == 0, out.stderr[-2000:]
        return json.loads(out.stdout[out.stdout.index("{"):])

    bench = run("benchmark.py", "--m", "1000", "--k", "4064", "--iterations", "5", "--benchmark-repeats", "2",
                "--warmup-iterations", "2")
    assert bench["verification_passed"] and bench["q_max_byte_diff"] == 0 and bench["effective_tb_s"] > 0
    e2e = run("e2e.py", "--m", "256", "--n", "256", "--k", "512", "--input-dtype", "fp16")
    assert e2e["e2e_verification_passed"] and e2e["max_err_ratio"] < 1.0
