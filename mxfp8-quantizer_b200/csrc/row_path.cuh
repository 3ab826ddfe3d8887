// row_path.cuh -- the pipelined quantizer's thread map and, for X rows that
// are not 16-byte aligned, the re-alignment of each thread's elements from
// its per-row-phase tensor-map box (quantize_tma.cu describes the scheme).
#pragma once
#include <stdint.h>

#include "tile.cuh"

namespace mxfp8 {

// Row of the tile that compute thread `tid` handles, and which 64 of its 128
// columns (h).  Tensor path: row tid % 128, h = tid / 128.  Row path: warp w
// takes the 16 rows 8j + w of tensor-map phase w, lane l row j = l % 16 and
// h = l / 16, so a warp shares one misalignment (warp-uniform re-align code)
// and the 8 lanes of a shared-memory phase read 8 consecutive box rows of
// 272 bytes, which start in 8 different 16-byte bank groups: conflict-free.
template <bool ROWS>
__device__ __forceinline__ int tile_row(int tid) {
    return ROWS ? (tid & 15) * kPhases + (tid >> 5) : (tid & (kTileRows - 1));
}
template <bool ROWS>
__device__ __forceinline__ int tile_half(int tid) {
    return ROWS ? (tid >> 4) & 1 : tid >> 7;
}

// XOR key of the payload staging buffer's 128-byte swizzle for tile row r:
// distinct across the 8 rows that one 8-lane phase writes.
template <bool ROWS>
__device__ __forceinline__ uint32_t stage_key(int r) {
    return ROWS ? (uint32_t)((r >> 3) & 7) : (uint32_t)(r & 7);
}

// Words W .. W+32 of v, shifted down by a further 2 bytes when sel says so.
template <int W>
__device__ __forceinline__ void shift_words(const uint32_t (&v)[36], uint32_t sel, uint32_t (&w0)[16],
                                            uint32_t (&w1)[16]) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const uint32_t x = __byte_perm(v[W + i], v[W + i + 1], sel);
        if (i < 16) w0[i] = x; else w1[i - 16] = x;
    }
}

// Row path: this thread's 64 elements (columns c0 + 64h ..) of row `row` from
// its 272-byte box row, re-aligned to 16-bit lanes and zeroed outside (m, k).
// Column c0 sits `off` bytes into the box row (off < 16, even, the same for
// the whole warp).  The thread loads the 9 aligned 16-byte words from byte
// 128h on, then takes 32 words from word off / 4 on, each a byte permute of
// two neighbours (a 2-byte shift when off % 4 == 2).  Warp-uniform branches
// pick the word offset, so no per-word selects are needed.
__device__ __forceinline__ void read_row_words(const TmaParams& p, const uint8_t* slot, int row, int c0, int h,
                                               uint32_t (&w0)[16], uint32_t (&w1)[16]) {
    const int cf = c0 + 64 * h;
    if (row >= p.m || cf >= p.k) {
#pragma unroll
        for (int i = 0; i < 16; ++i) w0[i] = w1[i] = 0u;
        return;
    }
    // low 4 bits of X's address of (row, c0): 32-bit arithmetic suffices
    const uint32_t off = ((uint32_t)reinterpret_cast<uintptr_t>(p.x) +
                          2u * ((uint32_t)row * (uint32_t)p.ld_x + (uint32_t)c0)) & 15u;
    uint32_t v[36];
#pragma unroll
    for (int i = 0; i < 9; ++i) {
        const uint4 t = *reinterpret_cast<const uint4*>(slot + 128 * h + 16 * i);
        v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
    const uint32_t sel = (off & 2u) ? 0x5432u : 0x3210u;
    switch (off >> 2) {
        case 0: shift_words<0>(v, sel, w0, w1); break;
        case 1: shift_words<1>(v, sel, w0, w1); break;
        case 2: shift_words<2>(v, sel, w0, w1); break;
        default: shift_words<3>(v, sel, w0, w1); break;
    }
    if (cf + 64 > p.k) {  // the columns cross K (the same for the whole warp)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int c = cf + 2 * i;
            uint32_t& x = i < 16 ? w0[i] : w1[i - 16];
            if (c >= p.k) x = 0u;
            else if (c + 1 >= p.k) x &= 0xFFFFu;
        }
    }
}

}  // namespace mxfp8
