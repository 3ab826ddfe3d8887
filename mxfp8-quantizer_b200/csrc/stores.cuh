// stores.cuh -- the pipelined quantizer's global stores of Q and S when the
// outputs are not 16-byte aligned (template flag QU of quantize_tma.cu).
#pragma once
#include <stdint.h>

#include "guard.cuh"

namespace mxfp8 {

// 16 bytes to global memory with streaming stores at a 4-byte aligned
// address, at the widest width the address allows (8 lanes still cover 128
// contiguous bytes per instruction).
template <bool QU>
__device__ __forceinline__ void store16(uint8_t* dst, const uint4& v, const StoreWindow& w, unsigned int* status) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(dst);
    if (!QU || (a & 15) == 0) {
        gstore(reinterpret_cast<uint4*>(dst), v, w, status);
    } else if ((a & 7) == 0) {
        gstore(reinterpret_cast<uint2*>(dst), make_uint2(v.x, v.y), w, status);
        gstore(reinterpret_cast<uint2*>(dst + 8), make_uint2(v.z, v.w), w, status);
    } else {
        gstore(reinterpret_cast<unsigned int*>(dst), v.x, w, status);
        gstore(reinterpret_cast<unsigned int*>(dst + 4), v.y, w, status);
        gstore(reinterpret_cast<unsigned int*>(dst + 8), v.z, w, status);
        gstore(reinterpret_cast<unsigned int*>(dst + 12), v.w, w, status);
    }
}

// The 16 bytes that start at byte h (0 <= h < 16) of the 32 bytes a | b (a
// first, little-endian): words h / 4 .. h / 4 + 4, then a funnel shift by
// the remaining bytes.  QW >= 0: the caller knows h / 4 == QW for every row
// (all Q rows at the same 16-byte phase), so the words are fixed at compile
// time.  QW < 0: the words are picked with two levels of selects (no branch;
// a switch measured 4.65 vs 4.87 TB/s at a 1-byte Q offset).
template <int QW>
__device__ __forceinline__ uint4 bytes_from(const uint4& a, const uint4& b, uint32_t h) {
    const uint32_t sh = 8u * (h & 3u);
    uint32_t w0, w1, w2, w3, w4;
    if constexpr (QW >= 0) {
        const uint32_t W[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        w0 = W[QW]; w1 = W[QW + 1]; w2 = W[QW + 2]; w3 = W[QW + 3]; w4 = W[QW + 4];
    } else {
        const bool b0 = (h & 4u) != 0, b1 = (h & 8u) != 0;
        const uint32_t t0 = b0 ? a.y : a.x, t1 = b0 ? a.z : a.y, t2 = b0 ? a.w : a.z, t3 = b0 ? b.x : a.w,
                       t4 = b0 ? b.y : b.x, t5 = b0 ? b.z : b.y, t6 = b0 ? b.w : b.z;
        w0 = b1 ? t2 : t0; w1 = b1 ? t3 : t1; w2 = b1 ? t4 : t2; w3 = b1 ? t5 : t3; w4 = b1 ? t6 : t4;
    }
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                      __funnelshift_r(w3, w4, sh));
}

// Chunk c + 1 of the staging row, which lane c of the store pass needs for
// store_row_any when its row's destination is not 4-byte aligned (lane 7's
// is never stored: any chunk will do).
__device__ __forceinline__ int next_chunk(int c) { return c < 7 ? c + 1 : 7; }

// QU store of one row segment of the payload tile (seg bytes, a multiple of
// 32) to dst, which may sit at any byte offset.  Lane c (of the row's 8)
// holds the segment's 16-byte chunk c in v.  A 4-byte aligned dst: lane c
// stores v with 16/8/4-byte stores.  Otherwise the 8 lanes write the aligned
// 16-byte chunks of the segment, one each (lane c the one at dst - d + 16 (c +
// 1), built from chunk c and chunk c + 1, vn, by a byte shift that is the same
// for the whole row), so every such store instruction writes whole lines.
// The unaligned head (h = 16 - d bytes) and tail (d bytes) make 16 boundary
// bytes, slot j < h the head's byte j and slot j >= h the tail's byte
// seg - 16 + j; lane c writes slots c and c + 8 with byte stores read from
// the staging row `rowbuf` (16-byte chunks XOR-swizzled by `key`): no branch
// on the lane, two store instructions per row.  No byte outside the segment
// is written.
template <int QW>
__device__ __forceinline__ void store_row_any(uint8_t* dst, const uint4& v, const uint4& vn, const uint8_t* rowbuf,
                                              uint32_t key, int seg, int c, const StoreWindow& w,
                                              unsigned int* status) {
    const uint32_t d = (uint32_t)(reinterpret_cast<uintptr_t>(dst) & 15);
    if ((d & 3) == 0) {  // 4-byte aligned row: each lane's own chunk v, 16/8/4-byte stores
        if (16 * c < seg) store16<true>(dst + 16 * c, v, w, status);
        return;
    }
    const int h = 16 - (int)d;
    if (16 * (c + 1) < seg)  // aligned chunk c + 1 of dst - d: segment bytes [16 c + h, 16 c + h + 16)
        gstore(reinterpret_cast<uint4*>(dst - d + 16 * (c + 1)), bytes_from<QW>(v, vn, (uint32_t)h), w, status);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int j = c + 8 * r;
        const int o = j < h ? j : seg - 16 + j;  // segment byte of boundary slot j
        gstore(dst + o, rowbuf[((((uint32_t)o >> 4) ^ key) << 4) | ((uint32_t)o & 15u)], w, status);
    }
}

}  // namespace mxfp8
