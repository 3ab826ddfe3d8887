// recipe.cuh -- the MXFP8 block recipe on one 1x32 block, shared by every
// quantizer kernel.  It restates, instruction for instruction, the
// reference kernel's per-block math:
//   amax      = max over the block of (bits & 0x7FFF)        MXFP8_quantizer.py:456-468
//   scale     = fma.rn.f32(amax, f32(1/448), f32(1e-12)),
//               byte = exponent + (mantissa != 0), 127 for an all-zero block,
//               inverse = f32 bits ((254 - byte) << 23)      MXFP8_quantizer.py:170-200
//   payload   = cvt.rn.satfinite.e4m3x2.f32(x * inverse)     MXFP8_quantizer.py:116-137, 473-501
// Element j of the block lands in byte j of the payload.  The 32-bit word
// arithmetic wraps exactly as the reference's Uint32 arithmetic does, which
// fixes the inf block (byte 255, inverse -inf) and the NaN block (byte 0,
// inverse -2^127).  No flush-to-zero anywhere (build without fast-math).
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace mxfp8 {

enum InDType : int { kBF16 = 0, kFP16 = 1 };

constexpr uint32_t kInv448Bits = 0x3B124925u;  // Float32(1.0 / 448.0)
constexpr uint32_t kEpsBits = 0x2B8CBCCCu;      // Float32(1.0e-12)

// Block amax of 16 words (32 packed 16-bit values): bit-pattern maximum of
// |x|, so a NaN pattern outranks inf, which outranks every finite value.
__device__ __forceinline__ uint32_t block_amax_bits(const uint32_t (&w)[16]) {
    uint32_t m0 = 0, m1 = 0;
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
        m0 = __vmaxu2(m0, w[i] & 0x7FFF7FFFu);
        m1 = __vmaxu2(m1, w[i + 1] & 0x7FFF7FFFu);
    }
    m0 = __vmaxu2(m0, m1);
    return max(m0 & 0xFFFFu, m0 >> 16);
}

template <int DT>
__device__ __forceinline__ float widen(uint32_t bits16) {
    if constexpr (DT == kBF16) {
        return __uint_as_float(bits16 << 16);
    } else {
        return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
    }
}

// UE8M0 scale byte and inverse scale from the block amax bit pattern.
template <int DT>
__device__ __forceinline__ void scale_from_amax(uint32_t amax_bits, uint32_t& byte, float& inv) {
    const float amax = widen<DT>(amax_bits);
    const float s = __fmaf_rn(amax, __uint_as_float(kInv448Bits), __uint_as_float(kEpsBits));
    const uint32_t b = __float_as_uint(s);
    uint32_t e = ((b >> 23) & 0xFFu) + ((b & 0x7FFFFFu) != 0u ? 1u : 0u);
    e = amax_bits == 0u ? 127u : e;
    byte = e & 0xFFu;
    inv = __uint_as_float((254u - e) << 23);
}

// Two f32 -> two E4M3 bytes; `lo` lands in the low byte.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

// Packed f32x2 multiply, round-to-nearest-even, subnormals kept.
__device__ __forceinline__ void mul2(float a0, float a1, float s, float& r0, float& r1) {
    uint64_t a, b, d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %1};" : "=l"(b) : "f"(s));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r0), "=f"(r1) : "l"(d));
}

// One word of two packed 16-bit inputs -> 16 bits of payload.
template <int DT>
__device__ __forceinline__ uint32_t quantize_pair(uint32_t w, float inv) {
    float x0, x1;
    if constexpr (DT == kBF16) {
        x0 = __uint_as_float(w << 16);
        x1 = __uint_as_float(w & 0xFFFF0000u);
    } else {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
        x0 = f.x;
        x1 = f.y;
    }
    float p0, p1;
    mul2(x0, x1, inv, p0, p1);
    return cvt_e4m3x2(p0, p1);
}

// Quantize one 32-value block held as 16 words; writes 8 payload words
// (32 bytes, element order) and returns the scale byte.
template <int DT>
__device__ __forceinline__ uint32_t quantize_block(const uint32_t (&w)[16], uint32_t (&q)[8]) {
    uint32_t byte;
    float inv;
    scale_from_amax<DT>(block_amax_bits(w), byte, inv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t lo = quantize_pair<DT>(w[2 * i], inv);
        const uint32_t hi = quantize_pair<DT>(w[2 * i + 1], inv);
        q[i] = lo | (hi << 16);
    }
    return byte;
}

// Packed scale storage: 128-row x 4-column chunks of 512 bytes, row-block
// major (MXFP8_quantizer.py:502-525).
__host__ __device__ __forceinline__ int64_t scale_offset(int64_t r, int64_t c, int64_t col_chunks) {
    const int64_t rr = r & 127;
    return ((r >> 7) * col_chunks + (c >> 2)) * 512 + (rr & 31) * 16 + (rr >> 5) * 4 + (c & 3);
}

}  // namespace mxfp8
