// dequantize.cu -- MXFP8 (E4M3 payload + packed UE8M0 scales) back to
// bf16 / fp16 / f32: out = e4m3(Q) * 2^(S - 127).  This is the decode the
// reference's end-to-end check applies on the host
// (MXFP8_quantizer.py:1179-1187); here it is one streaming kernel.  Scale
// byte 255 is the UE8M0 NaN; byte 0 is 2^-127.
//
// Thread map: one thread per 16 payload bytes (half a scale block), so a
// warp reads 512 contiguous payload bytes with 16-byte loads and writes
// 1-2 KiB contiguous output with 16-byte streaming stores.  Falls back to byte loads and element stores when a
// row is not 16-byte aligned.  Launched as a programmatic dependent launch.
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

// 16 decoded values -> out (16 contiguous elements at element index o).
template <int OUT>
__device__ __forceinline__ void store16(void* out, int64_t o, const float (&v)[16], bool vec, const StoreWindow& w,
                                        unsigned int* status) {
    if constexpr (OUT == MXFP8_F32) {
        float* p = static_cast<float*>(out) + o;
        if (vec) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                gstore(reinterpret_cast<float4*>(p) + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]),
                       w, status);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) gstore_plain(p + i, v[i], w, status);
        }
    } else {
        uint32_t h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if constexpr (OUT == MXFP8_BF16) {
                const __nv_bfloat162 t = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                h[i] = *reinterpret_cast<const uint32_t*>(&t);
            } else {
                const __half2 t = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
                h[i] = *reinterpret_cast<const uint32_t*>(&t);
            }
        }
        unsigned short* p = static_cast<unsigned short*>(out) + o;
        if (vec) {
            gstore(reinterpret_cast<uint4*>(p), make_uint4(h[0], h[1], h[2], h[3]), w, status);
            gstore(reinterpret_cast<uint4*>(p) + 1, make_uint4(h[4], h[5], h[6], h[7]), w, status);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                gstore_plain(p + 2 * i, (unsigned short)(h[i] & 0xFFFFu), w, status);
                gstore_plain(p + 2 * i + 1, (unsigned short)(h[i] >> 16), w, status);
            }
        }
    }
}

template <int OUT>
__device__ __forceinline__ void decode16(const uint32_t (&w)[4], float scale, float (&v)[16]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 lo = e4m3x2_to_float2(w[i] & 0xFFFFu);
        const float2 hi = e4m3x2_to_float2(w[i] >> 16);
        v[4 * i + 0] = __fmul_rn(lo.x, scale);
        v[4 * i + 1] = __fmul_rn(lo.y, scale);
        v[4 * i + 2] = __fmul_rn(hi.x, scale);
        v[4 * i + 3] = __fmul_rn(hi.y, scale);
    }
}

// Each thread takes kPieces 16-byte pieces spaced one grid-width apart and
// issues all their loads before decoding any.  Measured on B200 at 8192^2
// (bf16 out, TB/s): 1 piece with up to 64 CTAs/SM 6.15-6.30, 1 piece with 32
// 6.00-6.13, 2 pieces 5.98-6.04, 4 pieces 5.32-5.74; without the dependent
// launch 5.52-5.83.
constexpr int kPieces = 1;
constexpr int kMaxCtasPerSm = 64;

template <int OUT>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint8_t* __restrict__ q, int64_t rows, int64_t cols,
                                                         int64_t ld_q, const uint8_t* __restrict__ s, void* out,
                                                         int64_t ld_out, StoreWindow ow, unsigned int* status) {
    // Programmatic dependent launch: start early, touch memory only after
    // the previous kernel in the stream has completed.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int64_t halves = cols / 16;                 // 16-byte payload pieces per row
    const int64_t col_chunks = (cols / 32 + 3) / 4;
    const int64_t n = rows * halves;
    constexpr int kOutBytes = OUT == MXFP8_F32 ? 4 : 2;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < n; base += stride * kPieces) {
        uint32_t w[kPieces][4];
        uint32_t sb[kPieces];
#pragma unroll
        for (int j = 0; j < kPieces; ++j) {
            const int64_t idx = base + j * stride;
            if (idx >= n) continue;
            const int64_t r = idx / halves;
            const int64_t hp = idx - r * halves;
            sb[j] = __ldg(s + scale_offset(r, hp >> 1, col_chunks));
            const uint8_t* src = q + r * ld_q + hp * 16;
            if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
                const uint4 a = __ldcs(reinterpret_cast<const uint4*>(src));
                w[j][0] = a.x; w[j][1] = a.y; w[j][2] = a.z; w[j][3] = a.w;
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    w[j][i] = src[4 * i] | (src[4 * i + 1] << 8) | (src[4 * i + 2] << 16) |
                              ((uint32_t)src[4 * i + 3] << 24);
            }
        }
#pragma unroll
        for (int j = 0; j < kPieces; ++j) {
            const int64_t idx = base + j * stride;
            if (idx >= n) continue;
            const int64_t r = idx / halves;
            const int64_t hp = idx - r * halves;
            float v[16];
            decode16<OUT>(w[j], ue8m0_to_float(sb[j]), v);
            const int64_t o = r * ld_out + hp * 16;
            const bool vec = ((reinterpret_cast<uintptr_t>(out) + (uint64_t)o * kOutBytes) & 15) == 0;
            store16<OUT>(out, o, v, vec, ow, status);
        }
    }
}

int launch_dequantize(const uint8_t* q, int64_t rows, int64_t cols, int64_t ld_q, const uint8_t* s, void* out,
                      int out_dtype, int64_t ld_out, StoreWindow ow, unsigned int* status, cudaStream_t stream) {
    const int64_t n = rows * (cols / 16);
    if (n == 0) return MXFP8_OK;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int64_t blocks = (n + 256 * kPieces - 1) / (256 * kPieces);
    if (blocks > (int64_t)sms * kMaxCtasPerSm) blocks = (int64_t)sms * kMaxCtasPerSm;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    switch (out_dtype) {
        case MXFP8_F32:
            e = cudaLaunchKernelEx(&cfg, dequantize_kernel<MXFP8_F32>, q, rows, cols, ld_q, s, out, ld_out, ow, status);
            break;
        case MXFP8_BF16:
            e = cudaLaunchKernelEx(&cfg, dequantize_kernel<MXFP8_BF16>, q, rows, cols, ld_q, s, out, ld_out, ow,
                                   status);
            break;
        default:
            e = cudaLaunchKernelEx(&cfg, dequantize_kernel<MXFP8_FP16>, q, rows, cols, ld_q, s, out, ld_out, ow,
                                   status);
            break;
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error("dequantize_kernel launch", (int)e);
        return MXFP8_ERR_CUDA;
    }
    return MXFP8_OK;
}

}  // namespace mxfp8
