// quantize_generic.cu -- plain-load MXFP8 quantizer for layouts the TMA path
// cannot describe (X or Q not 16-byte aligned, row strides that are not
// multiples of 16 bytes, empty X).  Same recipe and output contract as the
// TMA kernel; one thread per (row, 4-block scale word).
#include <cuda_runtime.h>

#include "../../include/mxfp8.h"
#include "launch.h"
#include "recipe.cuh"

namespace mxfp8 {

template <int DT>
__global__ void __launch_bounds__(256) quantize_generic_kernel(const uint16_t* __restrict__ x, int64_t m, int64_t k,
                                                               int64_t ld_x, uint8_t* __restrict__ q,
                                                               int64_t q_rows, int64_t q_cols, int64_t ld_q,
                                                               uint8_t* __restrict__ s, int64_t scale_rows,
                                                               int64_t scale_cols, int64_t col_chunks) {
    const int64_t n = scale_rows * col_chunks;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx / col_chunks;
        const int64_t cc = idx - r * col_chunks;
        uint32_t word = 0;
        if (r < q_rows) {
#pragma unroll 1
            for (int bi = 0; bi < 4; ++bi) {
                const int64_t blk = cc * 4 + bi;
                if (blk >= scale_cols) break;
                const int64_t c0 = blk * 32;
                uint32_t w[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int64_t c = c0 + 2 * e;
                    uint32_t lo = 0, hi = 0;
                    if (r < m) {
                        if (c < k) lo = __ldg(x + r * ld_x + c);
                        if (c + 1 < k) hi = __ldg(x + r * ld_x + c + 1);
                    }
                    w[e] = lo | (hi << 16);
                }
                uint32_t qw[8];
                const uint32_t byte = quantize_block<DT>(w, qw);
                uint8_t* dst = q + r * ld_q + c0;
                if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                    reinterpret_cast<uint4*>(dst)[0] = make_uint4(qw[0], qw[1], qw[2], qw[3]);
                    reinterpret_cast<uint4*>(dst)[1] = make_uint4(qw[4], qw[5], qw[6], qw[7]);
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) dst[e] = (uint8_t)(qw[e >> 2] >> (8 * (e & 3)));
                }
                word |= byte << (8 * bi);
            }
        }
        // the four scale bytes of (r, 4*cc .. 4*cc+3) are one aligned word
        *reinterpret_cast<uint32_t*>(s + scale_offset(r, cc * 4, col_chunks)) = word;
    }
}

int launch_quantize_generic(const QuantizeArgs& a, int sm_count, cudaStream_t stream) {
    const int64_t n = a.scale_rows * a.col_chunks;
    const int threads = 256;
    int64_t blocks = (n + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    const uint16_t* x = static_cast<const uint16_t*>(a.x);
    if (a.dtype == kBF16)
        quantize_generic_kernel<kBF16><<<(int)blocks, threads, 0, stream>>>(
            x, a.m, a.k, a.ld_x, a.q, a.q_rows, a.q_cols, a.ld_q, a.s, a.scale_rows, a.scale_cols, a.col_chunks);
    else
        quantize_generic_kernel<kFP16><<<(int)blocks, threads, 0, stream>>>(
            x, a.m, a.k, a.ld_x, a.q, a.q_rows, a.q_cols, a.ld_q, a.s, a.scale_rows, a.scale_cols, a.col_chunks);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error("quantize_generic_kernel launch", (int)e);
        return MXFP8_ERR_CUDA;
    }
    return MXFP8_OK;
}

}  // namespace mxfp8
