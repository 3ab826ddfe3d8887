// quantize_generic.cu -- plain-load MXFP8 quantizer for what the pipelined
// kernel (quantize_tma.cu) does not take: empty X (it then writes only the
// padding) and X rows that are neither 16-byte aligned nor less than 2^36
// elements apart (no tensor map can stride them).  Same recipe (recipe.cuh)
// and output contract.
//
// Work item: 4 rows x one 256-column segment (8 scale blocks), one warp.
// Lane l owns columns [8l, 8l + 8) of the segment, so a quad of lanes holds
// one 1x32 block (amax via two xor-shuffles, as in the reference kernel,
// MXFP8_quantizer.py:157-168).  Loads are 4-byte words: a row whose first
// element is 4-byte aligned takes 4 words per lane; a row that starts 2 bytes
// past a word boundary takes the 5 aligned words around its 8 elements and
// re-aligns them with a byte permute.  A word is loaded only if it holds an
// element of the row, and an aligned 4-byte word never crosses a page, so no
// load touches memory outside X's pages; elements outside (m, k) are zeroed.
#include <cuda_runtime.h>

#include "../../include/mxfp8.h"
#include "launch.h"
#include "recipe.cuh"

namespace mxfp8 {

constexpr int kRowsPerItem = 4;

// Eight elements of row `row` starting at column c (c % 8 == 0), zero outside
// [0, k), as four words of two packed elements.
__device__ __forceinline__ void load8(const uint16_t* row, int64_t c, int64_t k, uint32_t (&w)[4]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(row + c);
    if ((a & 3u) == 0) {
        const uint32_t* p = reinterpret_cast<const uint32_t*>(a);
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = (c + 2 * j < k) ? __ldg(p + j) : 0u;
    } else {
        // element c sits in the upper half of the word at a - 2
        const uint32_t* p = reinterpret_cast<const uint32_t*>(a - 2);
        uint32_t v[5];
#pragma unroll
        for (int j = 0; j < 5; ++j) v[j] = (c + 2 * j - 1 < k) ? __ldg(p + j) : 0u;
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = __byte_perm(v[j], v[j + 1], 0x5432);
    }
    // zero the columns at and beyond k (the loaded words may carry neighbours)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if (c + 2 * j >= k) w[j] = 0u;
        else if (c + 2 * j + 1 >= k) w[j] &= 0xFFFFu;
    }
}

template <int DT>
__device__ __forceinline__ uint32_t quad_quantize(const uint32_t (&w)[4], uint2& q) {
    uint32_t m = __vmaxu2(__vmaxu2(w[0] & 0x7FFF7FFFu, w[1] & 0x7FFF7FFFu), __vmaxu2(w[2] & 0x7FFF7FFFu, w[3] & 0x7FFF7FFFu));
    m = max(m & 0xFFFFu, m >> 16);
    m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
    m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
    uint32_t byte;
    float inv;
    scale_from_amax<DT>(m, byte, inv);
    q.x = quantize_pair<DT>(w[0], inv) | (quantize_pair<DT>(w[1], inv) << 16);
    q.y = quantize_pair<DT>(w[2], inv) | (quantize_pair<DT>(w[3], inv) << 16);
    return byte;
}

template <int DT>
__global__ void __launch_bounds__(256) quantize_generic_kernel(const uint16_t* __restrict__ x, int64_t m, int64_t k,
                                                               int64_t ld_x, uint8_t* __restrict__ q,
                                                               int64_t q_rows, int64_t q_cols, int64_t ld_q,
                                                               uint8_t* __restrict__ s, int64_t scale_rows,
                                                               int64_t scale_cols, int64_t col_chunks,
                                                               StoreWindow qw, StoreWindow sw,
                                                               unsigned int* status) {
    const int lane = threadIdx.x & 31;
    const int64_t segs = (col_chunks + 1) / 2;               // 256-column segments
    const int64_t groups = (scale_rows + kRowsPerItem - 1) / kRowsPerItem;
    const int64_t items = segs * groups;
    const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t it = warp0; it < items; it += nwarps) {
        const int64_t g = it / segs;
        const int64_t seg = it - g * segs;
        const int64_t c = seg * 256 + lane * 8;
        uint32_t w[kRowsPerItem][4];
#pragma unroll
        for (int u = 0; u < kRowsPerItem; ++u) {
            const int64_t r = g * kRowsPerItem + u;
            if (r < m && c < k) {
                load8(x + r * ld_x, c, k, w[u]);
            } else {
                w[u][0] = w[u][1] = w[u][2] = w[u][3] = 0u;
            }
        }
#pragma unroll
        for (int u = 0; u < kRowsPerItem; ++u) {
            const int64_t r = g * kRowsPerItem + u;
            if (r >= scale_rows) break;                       // warp-uniform
            uint2 qq;
            uint32_t byte = quad_quantize<DT>(w[u], qq);
            if (r < q_rows && c < q_cols) {
                uint8_t* dst = q + r * ld_q + c;
                if ((reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
                    gstore_plain(reinterpret_cast<uint2*>(dst), qq, qw, status);
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        gstore_plain(dst + e, (unsigned char)((e < 4 ? qq.x : qq.y) >> (8 * (e & 3))), qw, status);
                }
            }
            const int64_t blk = seg * 8 + (lane >> 2);
            if (r >= q_rows || blk >= scale_cols) byte = 0;
            // quads 0-3 -> lane 0, quads 4-7 -> lane 16: one packed word each
            const uint32_t b1 = __shfl_down_sync(0xFFFFFFFFu, byte, 4);
            const uint32_t b2 = __shfl_down_sync(0xFFFFFFFFu, byte, 8);
            const uint32_t b3 = __shfl_down_sync(0xFFFFFFFFu, byte, 12);
            if ((lane & 15) == 0 && (blk >> 2) < col_chunks)
                gstore_plain(reinterpret_cast<unsigned int*>(s + scale_offset(r, blk, col_chunks)),
                       byte | (b1 << 8) | (b2 << 16) | (b3 << 24), sw, status);
        }
    }
}

int launch_quantize_generic(const QuantizeArgs& a, int sm_count, cudaStream_t stream) {
    const int64_t segs = (a.col_chunks + 1) / 2;
    const int64_t items = segs * ((a.scale_rows + kRowsPerItem - 1) / kRowsPerItem);
    int64_t blocks = (items * 32 + 255) / 256;
    const int64_t cap = (int64_t)sm_count * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    const uint16_t* x = static_cast<const uint16_t*>(a.x);
    if (a.dtype == kBF16)
        quantize_generic_kernel<kBF16><<<(int)blocks, 256, 0, stream>>>(
            x, a.m, a.k, a.ld_x, a.q, a.q_rows, a.q_cols, a.ld_q, a.s, a.scale_rows, a.scale_cols, a.col_chunks,
            a.qw, a.sw, a.status);
    else
        quantize_generic_kernel<kFP16><<<(int)blocks, 256, 0, stream>>>(
            x, a.m, a.k, a.ld_x, a.q, a.q_rows, a.q_cols, a.ld_q, a.s, a.scale_rows, a.scale_cols, a.col_chunks,
            a.qw, a.sw, a.status);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error("quantize_generic_kernel launch", (int)e);
        return MXFP8_ERR_CUDA;
    }
    return MXFP8_OK;
}

}  // namespace mxfp8
