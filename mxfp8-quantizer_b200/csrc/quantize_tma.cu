// quantize_tma.cu -- persistent, TMA-pipelined MXFP8 quantizer for sm_100a.
//
// Work unit ("tile"): 128 rows x 128 columns of X, i.e. exactly one 512-byte
// chunk of the packed scale layout (128 rows x 4 scale columns).  One CTA per
// SM walks tiles round-robin.  Warp 8 (one elected lane) streams X tiles into
// a 3-deep shared-memory ring with 2-D TMA loads (two 64-column boxes,
// 128-byte swizzle, zero fill outside (m, k)); warps 0-7 compute; finished
// payload tiles and scale chunks leave through a TMA tile store and a bulk
// copy from one of two staging buffers, so global stores are full-line and
// asynchronous.  One reduction barrier per tile among the 256 compute
// threads both publishes the staging buffer and agrees on aborting.
//
// Depth: 3 stages (96 KiB of X in flight per SM, ~14 MB on the GPU) measured
// faster than 4 or 5 on B200 (6.0-6.2 vs 5.6 TB/s at 16384^2): more
// outstanding loads only crowd out the payload write-back.
//
// Launch: programmatic dependent launch.  Each CTA lets the next kernel in
// the stream start its prologue as soon as SMs free up, and itself touches
// global memory only after griddepcontrol.wait, i.e. after the previous
// kernel has completed; back to back this hides ~1.7 us per launch.
//
// Thread map inside a tile: thread t handles row (t % 128) and the two
// scale blocks 2*(t/128) and 2*(t/128)+1, i.e. 64 contiguous input values
// that sit in box (t/128).  Within an 8-lane shared-memory phase the rows
// are consecutive, so the 128-byte swizzle makes every 16-byte access
// conflict-free, for the X reads and for the payload writes alike.
//
// Reference behaviour restated (not its structure): MXFP8_quantizer.py:355-525.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/mxfp8.h"
#include "launch.h"
#include "ptx.cuh"
#include "recipe.cuh"

namespace mxfp8 {

constexpr int kTileRows = 128;
constexpr int kTileCols = 128;
constexpr int kBoxCols = 64;                              // 64 x 16 bit = 128 B swizzle span
constexpr int kStageBytes = kTileRows * kTileCols * 2;    // 32 KiB of X per tile
constexpr int kBoxBytes = kStageBytes / 2;
constexpr int kQTileBytes = kTileRows * kTileCols;        // 16 KiB of payload per tile
constexpr int kSChunkBytes = 512;
constexpr int kComputeWarps = 8;
constexpr int kComputeThreads = kComputeWarps * 32;
constexpr int kThreads = kComputeThreads + 32;            // + producer warp
constexpr int kQBufs = 2;
constexpr uint64_t kWaitLimitNs = 1000000000ull;          // 1 s per pipeline wait
constexpr uint32_t kBarCompute = 1;                       // named barrier id

constexpr unsigned kErrTileWait = 1u, kErrReleaseWait = 2u, kErrDrainWait = 4u;

template <int STAGES>
struct Layout {
    static constexpr int x_off = 0;
    static constexpr int q_off = STAGES * kStageBytes;
    static constexpr int s_off = q_off + kQBufs * kQTileBytes;
    static constexpr int bar_off = s_off + kQBufs * kSChunkBytes;
    static constexpr int ctl_off = bar_off + 2 * STAGES * 8;
    static constexpr int bytes = ctl_off + 16;
    static constexpr int alloc = bytes + 1024;  // slack to align the base to 1024
};

struct TmaParams {
    int n_tiles;
    int n_col_tiles;
    int q_rows;
    int scale_cols;
    int col_chunks;
    uint8_t* s;
    unsigned int* status;
};

__device__ __forceinline__ bool bar_red_or(uint32_t id, uint32_t n, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, %2, %3, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void report(unsigned int* status, unsigned code) {
    if (status) atomicOr(status, code);
}

template <int DT, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    quantize_tma_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap qmap,
                        const TmaParams p) {
    using L = Layout<STAGES>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // Pointer arithmetic on the __shared__ array (not integer casts) keeps the
    // accesses below plain LDS/STS instead of generic loads and stores.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full0 = sbase + L::bar_off;
    const uint32_t empty0 = full0 + STAGES * 8;
    volatile int* ctl = reinterpret_cast<volatile int*>(smem + L::ctl_off);  // [0] abort, [1] consumed

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;

    if (tid == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(full0 + 8 * i, 1);
            mbar_init(empty0 + 8 * i, kComputeWarps);
        }
        ctl[0] = 0;
        ctl[1] = 0;
        fence_mbar_init();
    }
    if (tid == kComputeThreads) {
        prefetch_tensormap(&xmap);
        prefetch_tensormap(&qmap);
    }
    __syncthreads();
    // Nothing above touched global memory; everything below may read X that
    // the previous kernel wrote or overwrite Q/S that it reads.
    grid_launch_dependents();
    grid_wait_prerequisites();

    int issued = 0;
    if (warp == kComputeWarps) {
        // ---------------- producer: one lane streams X tiles ----------------
        if (lane == 0) {
            int it = 0;
            for (int t = blockIdx.x; t < p.n_tiles; t += gridDim.x, ++it) {
                const int stage = it % STAGES;
                if (it >= STAGES) {
                    const uint32_t parity = ((it / STAGES) - 1) & 1;
                    bool ok = mbar_try_wait(empty0 + 8 * stage, parity);
                    if (!ok) {
                        const uint64_t t0 = global_timer_ns();
                        for (uint32_t i = 1; !ok; ++i) {
                            ok = mbar_try_wait(empty0 + 8 * stage, parity);
                            if ((i & 255u) == 0 && (ctl[0] || global_timer_ns() - t0 > kWaitLimitNs)) break;
                        }
                    }
                    if (!ok) {
                        if (!ctl[0]) report(p.status, kErrReleaseWait);
                        ctl[0] = 1;
                        break;
                    }
                }
                const int rt = t / p.n_col_tiles;
                const int ct = t - rt * p.n_col_tiles;
                const uint32_t full = full0 + 8 * stage;
                const uint32_t dst = sbase + L::x_off + stage * kStageBytes;
                mbar_arrive_expect_tx(full, kStageBytes);
                tma_load_2d(dst, &xmap, ct * kTileCols, rt * kTileRows, full);
                tma_load_2d(dst + kBoxBytes, &xmap, ct * kTileCols + kBoxCols, rt * kTileRows, full);
            }
            issued = it;
        }
    } else {
        // ---------------- compute warps ----------------
        const int r = tid & (kTileRows - 1);  // row inside the tile
        const int h = tid >> 7;               // which box / pair of scale blocks
        const uint32_t swz = (uint32_t)(r & 7);
        int it = 0;
        for (int t = blockIdx.x; t < p.n_tiles; t += gridDim.x, ++it) {
            const int stage = it % STAGES;
            const int qb = it % kQBufs;
            const int rt = t / p.n_col_tiles;
            const int ct = t - rt * p.n_col_tiles;
            // warp-uniform verdict, so the __syncwarp below is never divergent
            const bool ok =
                __all_sync(0xFFFFFFFFu, mbar_wait_bounded(full0 + 8 * stage, (it / STAGES) & 1, kWaitLimitNs));
            if (ok) {
                const uint8_t* xrow = smem + L::x_off + stage * kStageBytes + h * kBoxBytes + r * 128;
                uint32_t w0[16], w1[16];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint4 a = *reinterpret_cast<const uint4*>(xrow + ((j ^ swz) << 4));
                    const uint4 b = *reinterpret_cast<const uint4*>(xrow + (((4 + j) ^ swz) << 4));
                    w0[4 * j] = a.x; w0[4 * j + 1] = a.y; w0[4 * j + 2] = a.z; w0[4 * j + 3] = a.w;
                    w1[4 * j] = b.x; w1[4 * j + 1] = b.y; w1[4 * j + 2] = b.z; w1[4 * j + 3] = b.w;
                }
                // X reads of this stage are done: release it to the producer.
                __syncwarp();
                if (lane == 0) mbar_arrive(empty0 + 8 * stage);

                uint32_t q0[8], q1[8];
                uint32_t b0 = quantize_block<DT>(w0, q0);
                uint32_t b1 = quantize_block<DT>(w1, q1);

                uint8_t* qrow = smem + L::q_off + qb * kQTileBytes + r * 128;
                const uint32_t c0 = 4 * h;  // first 16-byte payload chunk of this thread
                *reinterpret_cast<uint4*>(qrow + (((c0 + 0) ^ swz) << 4)) = make_uint4(q0[0], q0[1], q0[2], q0[3]);
                *reinterpret_cast<uint4*>(qrow + (((c0 + 1) ^ swz) << 4)) = make_uint4(q0[4], q0[5], q0[6], q0[7]);
                *reinterpret_cast<uint4*>(qrow + (((c0 + 2) ^ swz) << 4)) = make_uint4(q1[0], q1[1], q1[2], q1[3]);
                *reinterpret_cast<uint4*>(qrow + (((c0 + 3) ^ swz) << 4)) = make_uint4(q1[4], q1[5], q1[6], q1[7]);

                const int grow = rt * kTileRows + r;
                const int sc = ct * 4 + 2 * h;
                if (grow >= p.q_rows) { b0 = 0; b1 = 0; }
                if (sc >= p.scale_cols) b0 = 0;
                if (sc + 1 >= p.scale_cols) b1 = 0;
                *reinterpret_cast<uint16_t*>(smem + L::s_off + qb * kSChunkBytes + (r & 31) * 16 + (r >> 5) * 4 +
                                             2 * h) = static_cast<uint16_t>(b0 | (b1 << 8));
                fence_proxy_async_smem();
            }
            // The store issued one tile ago must have finished reading its
            // staging buffer before anyone writes that buffer next iteration.
            if (tid == 0) bulk_wait_read<kQBufs - 2>();
            if (bar_red_or(kBarCompute, kComputeThreads, !ok)) {
                if (tid == 0) {
                    report(p.status, kErrTileWait);
                    ctl[0] = 1;
                }
                break;
            }
            if (tid == 0) {
                tma_store_2d(&qmap, ct * kTileCols, rt * kTileRows, sbase + L::q_off + qb * kQTileBytes);
                bulk_store(p.s + ((int64_t)rt * p.col_chunks + ct) * kSChunkBytes,
                           sbase + L::s_off + qb * kSChunkBytes, kSChunkBytes);
                bulk_commit();
            }
        }
        if (tid == 0) ctl[1] = it;
    }
    __syncthreads();
    if (tid == 0) bulk_wait_all<0>();
    if (warp == kComputeWarps && lane == 0) {
        // Loads issued but never consumed (only after an abort) still target
        // this CTA's shared memory: wait for them, with a limit, before exit.
        for (int i = ctl[1]; i < issued; ++i) {
            if (!mbar_wait_bounded(full0 + 8 * (i % STAGES), (i / STAGES) & 1, kWaitLimitNs)) {
                report(p.status, kErrDrainWait);
                break;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

constexpr int kStages = 3;

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

static int encode_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t cols, uint64_t rows,
                     uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows) {
    auto encode = get_encode_fn();
    if (!encode) {
        set_last_error("cuTensorMapEncodeTiled entry point unavailable", 0);
        return MXFP8_ERR_TENSOR_MAP;
    }
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, type, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_last_error("cuTensorMapEncodeTiled failed", (int)r);
        return MXFP8_ERR_TENSOR_MAP;
    }
    return MXFP8_OK;
}

template <int DT>
static int launch_tma_typed(const QuantizeArgs& a, int sm_count, cudaStream_t stream) {
    using L = Layout<kStages>;
    auto kernel = quantize_tma_kernel<DT, kStages>;
    // The attribute is per device; set it on every launch path (cheap).
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::alloc);
    if (e != cudaSuccess) {
        set_last_error("cudaFuncSetAttribute", (int)e);
        return MXFP8_ERR_CUDA;
    }
    CUtensorMap xmap, qmap;
    int rc = encode_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, a.x, (uint64_t)a.k, (uint64_t)a.m,
                       (uint64_t)a.ld_x * 2, kBoxCols, kTileRows);
    if (rc) return rc;
    rc = encode_2d(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.q, (uint64_t)a.q_cols, (uint64_t)a.q_rows,
                   (uint64_t)a.ld_q, kTileCols, kTileRows);
    if (rc) return rc;
    TmaParams p;
    const int64_t n_row_tiles = a.scale_rows / kTileRows;
    const int64_t n_tiles = n_row_tiles * a.col_chunks;
    p.n_tiles = (int)n_tiles;
    p.n_col_tiles = (int)a.col_chunks;
    p.q_rows = (int)a.q_rows;
    p.scale_cols = (int)a.scale_cols;
    p.col_chunks = (int)a.col_chunks;
    p.s = a.s;
    p.status = a.status;
    const int grid = (int)(n_tiles < sm_count ? n_tiles : sm_count);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::alloc;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kernel, xmap, qmap, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error("quantize_tma_kernel launch", (int)e);
        return MXFP8_ERR_CUDA;
    }
    return MXFP8_OK;
}

int launch_quantize_tma(const QuantizeArgs& a, int sm_count, cudaStream_t stream) {
    return a.dtype == kBF16 ? launch_tma_typed<kBF16>(a, sm_count, stream)
                            : launch_tma_typed<kFP16>(a, sm_count, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free launch.  The kernel above needs one word of global scratch
// (its status word for bounded-wait timeouts).  mxfp8_quantize keeps that
// word in a buffer it allocates on the first call on each device; this
// variant keeps it in a fixed device array of this file instead, so it never
// allocates.  Every GPU that loads the library holds the array until exit.
// ---------------------------------------------------------------------------

constexpr int kNoAllocScratchWords = 64;  // 256 bytes per device
constexpr int kStatusWordsPerCall = 1;
constexpr int kMaxNoAllocDevices = 64;
static __device__ __align__(256) unsigned int g_noalloc_scratch[kNoAllocScratchWords];

static std::mutex g_noalloc_mu;
static unsigned int* g_noalloc_addr[kMaxNoAllocDevices];

// Device address of g_noalloc_scratch on device `dev` (the current device),
// looked up once per device.  In host code the array's name is only a
// host-side stand-in; the kernel must be given this address.
static int noalloc_scratch(int dev, unsigned int** out) {
    if (dev < 0 || dev >= kMaxNoAllocDevices) {
        set_last_error("device index beyond the allocation-free table", 0);
        return MXFP8_ERR_DEVICE;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr) {
            set_last_error("cudaGetSymbolAddress(g_noalloc_scratch)", (int)e);
            return MXFP8_ERR_CUDA;
        }
        g_noalloc_addr[dev] = static_cast<unsigned int*>(ptr);
    }
    *out = g_noalloc_addr[dev];
    return MXFP8_OK;
}

int launch_quantize_tma_noalloc(const QuantizeArgs& args, int dev, int sm_count, cudaStream_t stream) {
    static_assert(kStatusWordsPerCall <= kNoAllocScratchWords, "scratch array too small");
    unsigned int* scratch = nullptr;
    int rc = noalloc_scratch(dev, &scratch);
    if (rc) return rc;
    // The array keeps the previous call's contents: the status word must
    // start at zero, so clear it in stream order before the kernel runs.
    cudaError_t e = cudaMemsetAsync(scratch, 0, kStatusWordsPerCall * sizeof(unsigned int), stream);
    if (e != cudaSuccess) {
        set_last_error("cudaMemsetAsync(scratch)", (int)e);
        return MXFP8_ERR_CUDA;
    }
    QuantizeArgs a = args;
    a.status = scratch;
    return launch_quantize_tma(a, sm_count, stream);
}

}  // namespace mxfp8
