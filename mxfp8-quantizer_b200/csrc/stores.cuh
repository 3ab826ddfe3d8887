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

// QU store of one row segment of the payload tile (seg bytes, a multiple of
// 32) from the staging row `rowbuf` (16-byte chunks XOR-swizzled by `key`) to
// dst, which may sit at any byte offset.  A 4-byte aligned dst: lane c stores
// its own chunk v with 16/8/4-byte stores.  Otherwise the 8 lanes of the row
// (lane c) write the aligned 16-byte chunks of the segment, one each, built
// from 5 words read at word granularity from the staging row and
// funnel-shifted by the remaining byte offset, so every store instruction
// writes whole lines; the unaligned head (16 - d bytes) and tail (d bytes) go
// out as naturally aligned 1/2/4/8-byte pieces, one per bit of their length:
// lanes 0-3 the head's, lanes 4-7 the tail's.  No byte outside the segment is
// written.  Measured at 8192^2 (TB/s): 8- or 4-byte aligned rows 5.6-6.1, 1-
// or 2-byte 3.3-3.7 (byte-wide head/tail stores: 2.8; 1-byte stores at each
// chunk's own address: 1.3).
__device__ __forceinline__ void store_row_any(uint8_t* dst, const uint4& v, const uint8_t* rowbuf, uint32_t key, int seg,
                                              int c, const StoreWindow& w, unsigned int* status) {
    const uint32_t d = (uint32_t)(reinterpret_cast<uintptr_t>(dst) & 15);
    auto word = [&](int i) {  // word i of the segment (i < 32)
        return *reinterpret_cast<const uint32_t*>(rowbuf + ((((uint32_t)i >> 2) ^ key) << 4) + (i & 3) * 4);
    };
    if ((d & 3) == 0) {  // 4-byte aligned row: each lane's own chunk v, 16/8/4-byte stores
        if (16 * c < seg) store16<true>(dst + 16 * c, v, w, status);
        return;
    }
    uint8_t* base = dst - d;  // 16-byte aligned
    if (16 * (c + 1) < seg) {
        // aligned chunk c + 1 holds segment bytes [e, e + 16), e >= 1
        const int e = 16 * (c + 1) - (int)d;
        const int i0 = e >> 2;
        const uint32_t sh = 8u * (uint32_t)(e & 3);
        uint32_t x[5];
#pragma unroll
        for (int k = 0; k < 5; ++k) x[k] = word((i0 + k) & 31);  // word 32 only when sh == 0 (unused)
        gstore(reinterpret_cast<uint4*>(base + 16 * (c + 1)),
               make_uint4(__funnelshift_r(x[0], x[1], sh), __funnelshift_r(x[1], x[2], sh),
                          __funnelshift_r(x[2], x[3], sh), __funnelshift_r(x[3], x[4], sh)),
               w, status);
    }
    // piece k = c % 4 of the head (c < 4) or the tail (c >= 4), if that bit is set
    const int k = c & 3;
    const uint32_t h = 16 - d;
    const bool tail = c >= 4;
    if (((tail ? d : h) >> k) & 1u) {
        // head pieces grow from the start, tail pieces shrink from the boundary
        const int off = tail ? seg - (int)d + (int)(d & ~((2u << k) - 1)) : (int)(h & ((1u << k) - 1));
        const int i = off >> 2;
        const uint32_t sh = 8u * (uint32_t)(off & 3);
        const uint32_t w0 = word(i), w1 = word((i + 1) & 31), w2 = word((i + 2) & 31);
        const uint32_t lo = __funnelshift_r(w0, w1, sh), hi = __funnelshift_r(w1, w2, sh);
        uint8_t* q = dst + off;
        if (k == 0) gstore(q, (unsigned char)lo, w, status);
        else if (k == 1) gstore(reinterpret_cast<unsigned short*>(q), (unsigned short)lo, w, status);
        else if (k == 2) gstore(reinterpret_cast<unsigned int*>(q), lo, w, status);
        else gstore(reinterpret_cast<uint2*>(q), make_uint2(lo, hi), w, status);
    }
}

}  // namespace mxfp8
