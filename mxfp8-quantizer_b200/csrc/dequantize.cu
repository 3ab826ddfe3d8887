// dequantize.cu -- MXFP8 (E4M3 payload + packed UE8M0 scales) back to
// bf16 / fp16 / f32: out = e4m3(Q) * 2^(S - 127).  This is the decode the
// reference's end-to-end check applies on the host
// (MXFP8_quantizer.py:1179-1187); here it is one streaming kernel.  Scale
// byte 255 is the UE8M0 NaN; byte 0 is 2^-127.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/mxfp8.h"
#include "launch.h"
#include "recipe.cuh"

namespace mxfp8 {

__device__ __forceinline__ float2 e4m3x2_to_float2(uint32_t two_bytes) {
    uint32_t h2;
    asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(h2) : "r"(two_bytes));
    return __half22float2(*reinterpret_cast<const __half2*>(&h2));
}

__device__ __forceinline__ float ue8m0_to_float(uint32_t b) {
    if (b == 255u) return __uint_as_float(0x7FC00000u);
    if (b == 0u) return __uint_as_float(0x00400000u);
    return __uint_as_float(b << 23);
}

template <int OUT>
__device__ __forceinline__ void store_out(void* out, int64_t idx, float v) {
    if constexpr (OUT == MXFP8_F32) {
        static_cast<float*>(out)[idx] = v;
    } else if constexpr (OUT == MXFP8_BF16) {
        static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
    } else {
        static_cast<__half*>(out)[idx] = __float2half_rn(v);
    }
}

// One thread per (row, 32-element block).
template <int OUT>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint8_t* __restrict__ q, int64_t rows, int64_t cols,
                                                         int64_t ld_q, const uint8_t* __restrict__ s, void* out,
                                                         int64_t ld_out) {
    const int64_t nblk = cols / 32;
    const int64_t col_chunks = (nblk + 3) / 4;
    const int64_t n = rows * nblk;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx / nblk;
        const int64_t b = idx - r * nblk;
        const float scale = ue8m0_to_float(s[scale_offset(r, b, col_chunks)]);
        const uint8_t* src = q + r * ld_q + b * 32;
        uint32_t w[8];
        if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
            const uint4 a = reinterpret_cast<const uint4*>(src)[0];
            const uint4 c = reinterpret_cast<const uint4*>(src)[1];
            w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
            w[4] = c.x; w[5] = c.y; w[6] = c.z; w[7] = c.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                w[i] = src[4 * i] | (src[4 * i + 1] << 8) | (src[4 * i + 2] << 16) | ((uint32_t)src[4 * i + 3] << 24);
        }
        const int64_t o = r * ld_out + b * 32;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float2 lo = e4m3x2_to_float2(w[i] & 0xFFFFu);
            const float2 hi = e4m3x2_to_float2(w[i] >> 16);
            store_out<OUT>(out, o + 4 * i + 0, __fmul_rn(lo.x, scale));
            store_out<OUT>(out, o + 4 * i + 1, __fmul_rn(lo.y, scale));
            store_out<OUT>(out, o + 4 * i + 2, __fmul_rn(hi.x, scale));
            store_out<OUT>(out, o + 4 * i + 3, __fmul_rn(hi.y, scale));
        }
    }
}

int launch_dequantize(const uint8_t* q, int64_t rows, int64_t cols, int64_t ld_q, const uint8_t* s, void* out,
                      int out_dtype, int64_t ld_out, cudaStream_t stream) {
    const int64_t n = rows * (cols / 32);
    if (n == 0) return MXFP8_OK;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int64_t blocks = (n + 255) / 256;
    if (blocks > (int64_t)sms * 16) blocks = (int64_t)sms * 16;
    switch (out_dtype) {
        case MXFP8_F32:
            dequantize_kernel<MXFP8_F32><<<(int)blocks, 256, 0, stream>>>(q, rows, cols, ld_q, s, out, ld_out);
            break;
        case MXFP8_BF16:
            dequantize_kernel<MXFP8_BF16><<<(int)blocks, 256, 0, stream>>>(q, rows, cols, ld_q, s, out, ld_out);
            break;
        default:
            dequantize_kernel<MXFP8_FP16><<<(int)blocks, 256, 0, stream>>>(q, rows, cols, ld_q, s, out, ld_out);
            break;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error("dequantize_kernel launch", (int)e);
        return MXFP8_ERR_CUDA;
    }
    return MXFP8_OK;
}

}  // namespace mxfp8
