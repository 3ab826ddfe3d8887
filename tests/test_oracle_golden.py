"""The CPU oracle against the reference's own recipe (CPU only).

The golden digests in tests/golden/golden.json were produced by the
reference's torch restatement (MXFP8_quantizer.py:610-662); see
tests/golden/make_golden.py.  tests/golden/golden_kernel.json holds digests
of the reference's CuTeDSL kernel itself, run on a B200
(tests/golden/make_kernel_golden.py), which pin the inf/NaN semantics too.
Special-value blocks are also checked against known answers derived from
the PTX definitions of the reference kernel's instructions
(MXFP8_quantizer.py:116-200, 473-501).
"""

import base64
import hashlib
import json
import pathlib
import struct
import zlib
from fractions import Fraction

import numpy as np
import pytest

import inputs
from make_golden import CASES


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


FAST_CASES = [n for n in CASES if n not in ("c2", "c3")]


@pytest.mark.parametrize("name", FAST_CASES)
def test_oracle_matches_reference_digests(name, golden, oracle_mod):
    rec = golden["cases"][name]
    desc, gen, dtype = CASES[name]
    bits = gen()
    q, s = oracle_mod.quantize(bits, dtype, rec["kernel_m"], rec["kernel_k"])
    assert s.size == rec["s_bytes"]
    assert sha(q) == rec["q_sha256"], f"payload differs from the reference recipe on {name}"
    assert sha(s) == rec["s_sha256"], f"packed scales differ from the reference recipe on {name}"


@pytest.mark.slow
@pytest.mark.parametrize("name", ["c2", "c3"])
def test_oracle_matches_reference_digests_full_size(name, golden, oracle_mod):
    test_oracle_matches_reference_digests(name, golden, oracle_mod)


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def f32_val(b: int) -> float:
    return struct.unpack("<f", struct.pack("<I", b))[0]


def exact_scale_byte(amax: Fraction) -> int:
    """MXFP8_quantizer.py:170-200 evaluated in exact rational arithmetic:
    one rounding of amax*c + eps to f32 (RNE), then ceil to a power of 2."""
    c = Fraction(f32_val(0x3B124925))
    eps = Fraction(f32_val(0x2B8CBCCC))
    v = amax * c + eps
    # round v (positive, normal range) to 24 significant bits, nearest-even
    e = v.numerator.bit_length() - v.denominator.bit_length()
    if Fraction(2) ** e > v:
        e -= 1
    q = v / Fraction(2) ** (e - 23)
    n = q.numerator // q.denominator
    rem = q - n
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and n % 2):
        n += 1
    if n == 1 << 24:
        n >>= 1
        e += 1
    biased = e + 127
    return biased + (1 if n != (1 << 23) else 0)


def decode16(b: int, dtype: str) -> Fraction:
    if dtype == "bf16":
        return Fraction(f32_val(b << 16))
    e, m = (b >> 10) & 0x1F, b & 0x3FF
    return Fraction(m, 1 << 24) if e == 0 else Fraction(0x400 | m, 1 << 10) * Fraction(2) ** (e - 15)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_scale_table_matches_reference_and_exact_rule(dtype, golden, oracle_mod):
    table = np.frombuffer(zlib.decompress(base64.b64decode(golden["scale_tables"][dtype])), np.uint8)
    top = 0x7F7F if dtype == "bf16" else inputs.FP16_MAX
    assert table.size == top + 1
    rng = np.random.default_rng(0)
    exact_checks = set(rng.integers(1, top + 1, size=400).tolist()) | {1, 2, 0x7F, 0x80, top}
    for a in range(top + 1):
        byte, inv = oracle_mod.scale_from_amax_bits(a, dtype)
        assert byte == table[a], f"amax {a:#06x}: oracle {byte} vs reference {table[a]}"
        assert inv == ((254 - (byte if a else 127)) << 23) & 0xFFFFFFFF
        if a and a in exact_checks:
            assert byte == exact_scale_byte(decode16(a, dtype))


def test_scale_rule_special_patterns(oracle_mod):
    # zero block: byte 127, inverse 1.0 (MXFP8_quantizer.py:173-175)
    assert oracle_mod.scale_from_amax_bits(0, "bf16") == (127, 0x3F800000)
    # inf amax: exponent 0xFF, mantissa 0 -> 255, inverse bits (254-255)<<23 = -inf
    assert oracle_mod.scale_from_amax_bits(0x7F80, "bf16") == (255, 0xFF800000)
    assert oracle_mod.scale_from_amax_bits(0x7C00, "fp16") == (255, 0xFF800000)
    # NaN amax: exponent 0xFF + 1 = 256 -> byte 0, inverse bits (254-256)<<23 = -2^127
    assert oracle_mod.scale_from_amax_bits(0x7FC0, "bf16") == (0, 0xFF000000)
    assert oracle_mod.scale_from_amax_bits(0x7E00, "fp16") == (0, 0xFF000000)
    # fp16 max 65504: 65504/448 = 146.2 -> 2^8 -> byte 135
    assert oracle_mod.scale_from_amax_bits(0x7BFF, "fp16")[0] == 135
    # smallest bf16 subnormal hits the eps floor
    assert oracle_mod.scale_from_amax_bits(0x0001, "bf16")[0] == 88


E4M3_KAT = [
    (0.0, 0x00), (-0.0, 0x80), (1.0, 0x38), (-1.0, 0xB8), (448.0, 0x7E), (-448.0, 0xFE),
    (464.0, 0x7E), (500.0, 0x7E), (float("inf"), 0x7E), (float("-inf"), 0xFE),
    (2.0 ** -6, 0x08), (2.0 ** -9, 0x01), (2.0 ** -10, 0x00), (1.5 * 2.0 ** -10, 0x01),
    (3 * 2.0 ** -10, 0x02), (1.0625, 0x38), (1.0625 + 2 ** -20, 0x39), (1.1875, 0x3A),
    (240.0, 0x77), (232.0, 0x76), (0.875 * 2.0 ** -6, 0x07), (0.9375 * 2.0 ** -6, 0x08),
    (1e-30, 0x00), (-1e-30, 0x80), (1e-45, 0x00), (-1e-45, 0x80),
]


@pytest.mark.parametrize("v,code", E4M3_KAT)
def test_e4m3_encoding_known_answers(v, code, oracle_mod):
    assert oracle_mod.e4m3_from_f32_bits(f32_bits(v)) == code


def test_e4m3_nan(oracle_mod):
    for b in (0x7FC00000, 0xFFC00000, 0x7F800001, 0xFFFFFFFF):
        assert oracle_mod.e4m3_from_f32_bits(b) == 0x7F


def test_e4m3_matches_torch_cast_on_finite_range(oracle_mod):
    import torch

    rng = np.random.default_rng(5)
    bits = rng.integers(0, 2 ** 32, size=20000, dtype=np.uint64).astype(np.uint32)
    vals = bits.view(np.float32)
    keep = np.isfinite(vals) & (np.abs(vals) <= 448.0)
    vals = vals[keep]
    want = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = np.array([oracle_mod.e4m3_from_f32_bits(int(b)) for b in vals.view(np.uint32)], np.uint8)
    np.testing.assert_array_equal(got, want)


def test_mul_rn_special_products(oracle_mod):
    ninf, n2p127 = 0xFF800000, 0xFF000000
    assert oracle_mod.f32_mul_rn(f32_bits(0.0), ninf) == 0x7FFFFFFF          # 0 * -inf = NaN
    assert oracle_mod.f32_mul_rn(f32_bits(3.0), ninf) == 0xFF800000          # finite * -inf
    assert oracle_mod.f32_mul_rn(f32_bits(-3.0), ninf) == 0x7F800000
    assert oracle_mod.f32_mul_rn(f32_bits(2.0), n2p127) == 0xFF800000        # overflow
    assert oracle_mod.f32_mul_rn(f32_bits(0.0), n2p127) == 0x80000000        # -0
    assert oracle_mod.f32_mul_rn(f32_bits(2.0 ** -126), n2p127) == f32_bits(-2.0)
    # subnormal product, round to nearest even: 3 * 2^-150 -> 2 * 2^-149? (ties to even)
    assert oracle_mod.f32_mul_rn(0x00000003, 0x3F000000) == 0x00000002
    assert oracle_mod.f32_mul_rn(0x00000001, 0x3F000000) == 0x00000000
    rng = np.random.default_rng(3)
    a = rng.standard_normal(5000).astype(np.float32)
    b = np.exp2(rng.integers(-140, 120, size=5000)).astype(np.float32)
    with np.errstate(over="ignore", under="ignore"):
        want = (a * b).view(np.uint32)
    got = np.array([oracle_mod.f32_mul_rn(int(x), int(y)) for x, y in
                    zip(a.view(np.uint32), b.view(np.uint32))], np.uint32)
    np.testing.assert_array_equal(got, want)


def blocks_of(values, dtype="bf16"):
    """One row of 32 values given as floats or raw bit patterns (ints)."""
    row = np.zeros((1, 32), np.uint16)
    for i, v in enumerate(values):
        row[0, i] = v if isinstance(v, int) else inputs.f32_to_bits(np.array([v], np.float32), dtype)[0]
    return row


def test_nan_block_follows_kernel_semantics(oracle_mod):
    # NaN amax: scale byte 0, inverse -2^127: finite x overflow to -sign*448,
    # zeros become -0, tiny values scale exactly, NaN stays NaN.
    vals = [1.0, -3.0, 0.0, 0x7FC0, 2.0 ** -126, 0x8000] + [0.0] * 26
    q, s = oracle_mod.quantize(blocks_of(vals), "bf16", 1, 32)
    assert s[0] == 0
    assert list(q[0, :6]) == [0xFE, 0x7E, 0x80, 0x7F, 0xC0, 0x00]


def test_inf_block_follows_kernel_semantics(oracle_mod):
    # inf amax: scale byte 255, inverse -inf: non-zero x -> -sign*448, 0 -> NaN.
    vals = [1.0, -3.0, 0.0, 0x7F80, 0xFF80, 0x0001] + [0.0] * 26
    q, s = oracle_mod.quantize(blocks_of(vals), "bf16", 1, 32)
    assert s[0] == 255
    assert list(q[0, :6]) == [0xFE, 0x7E, 0x7F, 0xFE, 0x7E, 0xFE]


def test_padding_contract(oracle_mod):
    # reference launch shape of 1000x4064 is 1000x4096: the padded scale
    # column holds 127 (quantized zeros), rows 1000..1023 hold 0.
    bits = inputs.normal(1000, 4064, 21)
    q, s = oracle_mod.quantize(bits, "bf16")
    assert q.shape == (1000, 4096)
    dense = oracle_mod.unpack_scales(s, 1024, 128)
    assert (dense[:1000, 127] == 127).all()
    assert (dense[1000:] == 0).all()
    assert (q[:, 4064:] == 0).all()
    # tight geometry: 127 scale columns, the padding column is 0
    q2, s2 = oracle_mod.quantize(bits, "bf16", 1000, 4064)
    dense2 = oracle_mod.unpack_scales(s2, 1024, 128)
    assert (dense2[:, 127] == 0).all() and (dense2[1000:] == 0).all()
    np.testing.assert_array_equal(dense2[:1000, :127], dense[:1000, :127])
    np.testing.assert_array_equal(q2, q[:, :4064])


def test_row_chunks_are_independent(oracle_mod):
    # quantization is row-local, and the packed storage is row-block major,
    # so 128-row shards concatenate to the unsharded result (multi-GPU split).
    bits = inputs.normal(512, 768, 31)
    q, s = oracle_mod.quantize(bits, "bf16", 512, 768)
    per = oracle_mod.scale_storage_bytes(128, 768)
    for c in range(4):
        qc, sc = oracle_mod.quantize(bits[c * 128:(c + 1) * 128], "bf16", 128, 768)
        np.testing.assert_array_equal(qc, q[c * 128:(c + 1) * 128])
        np.testing.assert_array_equal(sc, s[c * per:(c + 1) * per])


def test_dequantize_roundtrip_bound(oracle_mod):
    bits = inputs.normal(64, 256, 41)
    q, s = oracle_mod.quantize(bits, "bf16", 64, 256)
    x = (bits.astype(np.uint32) << 16).view(np.float32)
    y = oracle_mod.dequantize(q, s)
    # E4M3 keeps 3 mantissa bits: relative error <= 2^-4 for values above the
    # block's subnormal range
    scale = np.repeat(np.exp2(oracle_mod.unpack_scales(s, 64, 8).astype(np.float32) - 127), 32, axis=1)
    err = np.abs(y - x)
    assert (err <= np.maximum(np.abs(x) * 2.0 ** -4, scale * 2.0 ** -10) + 1e-30).all()


KERNEL_GOLDEN = json.loads((pathlib.Path(__file__).resolve().parent / "golden" / "golden_kernel.json").read_text())


@pytest.mark.parametrize("name", [n for n in KERNEL_GOLDEN["cases"] if n not in ("c2", "c3")])
def test_oracle_matches_reference_kernel_digests(name, oracle_mod):
    """The reference's CuTeDSL kernel itself, run on a B200 (make_kernel_golden.py),
    including every inf/NaN pattern and the special-value config."""
    from make_kernel_golden import KERNEL_CASES

    rec = KERNEL_GOLDEN["cases"][name]
    desc, gen, dtype = KERNEL_CASES[name]
    q, s = oracle_mod.quantize(gen(), dtype, rec["kernel_m"], rec["kernel_k"])
    assert sha(q) == rec["q_sha256"], f"payload differs from the reference kernel on {name}"
    assert sha(s) == rec["s_sha256"], f"packed scales differ from the reference kernel on {name}"
