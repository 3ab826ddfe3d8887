// quantize_tma.cu -- persistent, TMA-pipelined MXFP8 quantizer for sm_100a.
//
// Work unit ("tile"): 128 rows x 128 columns of X, i.e. exactly one 512-byte
// chunk of the packed scale layout (128 rows x 4 scale columns).  One CTA per
// SM (two on the row path below) walks tiles round-robin.  Warp 8 (one
// elected lane) streams X tiles into
// a 3-deep shared-memory ring with 2-D TMA loads (two 64-column boxes,
// 128-byte swizzle, zero fill outside (m, k)); warps 0-7 compute into one of
// two staging buffers (payload tile + 512-byte scale chunk); one reduction
// barrier per tile among the 256 compute threads publishes the buffer and
// agrees on aborting; then each compute warp writes 16 payload rows back with
// 16-byte streaming stores, 8 lanes per 128-byte row, so every store
// instruction writes four whole lines, and warp 0 writes the scale chunk.
//
// Measured on B200 (min over runs, TB/s at 16384^2 / 8192^2): these plain
// coalesced stores beat TMA tile stores of the same staging buffer
// (6.6 vs 6.1-6.4 / 6.19 vs 6.12), and 3 stages (96 KiB of X in flight per
// SM) beat 2, 4 and 5: more outstanding loads crowd out the write-back.
//
// Launch: programmatic dependent launch.  Each CTA lets the next kernel in
// the stream start its prologue as soon as SMs free up, asks L2 to prefetch
// its first two X tiles, and only then waits (griddepcontrol.wait) for the
// previous kernel to complete before any load or store of its own.  The
// prefetch is a hint (no data moves into the CTA before the wait), so it is
// safe even when the previous kernel writes X; it fills the DRAM bubble
// between back-to-back launches: 8192^2 went from 5.83 (plain launch) to
// 6.16 (dependent launch) to 6.63 TB/s (plus the prefetch).
//
// Thread map inside a tile: thread t handles row (t % 128) and the two
// scale blocks 2*(t/128) and 2*(t/128)+1, i.e. 64 contiguous input values
// that sit in box (t/128).  Within an 8-lane shared-memory phase the rows
// are consecutive, so the 128-byte swizzle makes every 16-byte access
// conflict-free, for the X reads and for the payload writes alike; the
// store pass reads the 8 chunks of one row per 8-lane phase, also
// conflict-free.
//
// Row path (template flag ROWS): X rows that are not 16-byte aligned (odd K,
// row strides that are not a multiple of 8 elements, 2-byte aligned views).
// No tensor map describes such rows, but rows r = 8j + f for a fixed phase f
// are 8 * ld_x elements = 16 * ld_x bytes apart, always a multiple of 16.  So
// the host encodes one tensor map per phase f (at most 8): base = the address
// of row f rounded down to 16 bytes, which puts column c of row 8j + f at
// element c + d_f of map row j (d_f < 8), and extent k + d_f columns by the
// rows of that phase.  A tile is then 8 TMA loads of a 136-column x 16-row box
// (272-byte rows, no swizzle) at column ct * 128, an aligned coordinate.
// Every byte a box reads lies in the 16-byte chunks that hold the row's own
// elements; columns past k + d_f and rows past the phase's last are zero
// filled.  Consumers shift their 64 elements down by d_f in registers; the
// thread map changes so that each compute warp holds one phase (tile_row).
//
// Outputs at any offset (template flag QU, when Q, ld_q or S is not 16-byte
// aligned): the store pass writes Q rows through store_row_any and the scale
// chunk with 16/8/4-byte stores (S is at least 4-byte aligned).  Realigning
// rows costs instructions, so these kernels run 2 CTAs per SM with 2 stages
// each, as the row path does, for twice the warps to hide them.
//
// Reference behaviour restated (not its structure): MXFP8_quantizer.py:355-525.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <mutex>

#include "../../include/mxfp8.h"
#include "launch.h"
#include "ptx.cuh"
#include "recipe.cuh"
#include "row_path.cuh"
#include "stores.cuh"
#include "tile.cuh"

namespace mxfp8 {

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

// Issue the TMA loads of tile (rt, ct) into the stage at shared address dst.
template <bool ROWS>
__device__ __forceinline__ void load_tile(const XMaps<ROWS>& xm, const TmaParams& p, uint32_t dst, int rt, int ct,
                                          uint32_t full) {
    if constexpr (ROWS) {
        mbar_arrive_expect_tx(full, (uint32_t)(p.n_phases * kPhaseBoxBytes));
        for (int f = 0; f < p.n_phases; ++f)
            tma_load_2d(dst + f * kPhaseBoxBytes, &xm.map[f], ct * kTileCols, rt * kPhaseRows, full);
    } else {
        mbar_arrive_expect_tx(full, kStageBytes);
        tma_load_2d(dst, &xm.map[0], ct * kTileCols, rt * kTileRows, full);
        tma_load_2d(dst + kBoxBytes, &xm.map[0], ct * kTileCols + kBoxCols, rt * kTileRows, full);
    }
}

template <bool ROWS>
__device__ __forceinline__ void prefetch_tile(const XMaps<ROWS>& xm, const TmaParams& p, int rt, int ct) {
    if constexpr (ROWS) {
        for (int f = 0; f < p.n_phases; ++f) tma_prefetch_l2_2d(&xm.map[f], ct * kTileCols, rt * kPhaseRows);
    } else {
        tma_prefetch_l2_2d(&xm.map[0], ct * kTileCols, rt * kTileRows);
        tma_prefetch_l2_2d(&xm.map[0], ct * kTileCols + kBoxCols, rt * kTileRows);
    }
}

template <int DT, int STAGES, bool ROWS, bool QU, int QW>
__global__ void __launch_bounds__(kThreads, (ROWS || QU) ? kRowCtasPerSm : 1)
    quantize_tma_kernel(const __grid_constant__ XMaps<ROWS> xm, const TmaParams p) {
    using L = Layout<STAGES, ROWS>;
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
        for (int f = 0; f < (ROWS ? p.n_phases : 1); ++f) prefetch_tensormap(&xm.map[f]);
    }
    __syncthreads();
    if (tid == kComputeThreads) {
        for (int i = 0, t = blockIdx.x; i < kPrefetchTiles && t < p.n_tiles; ++i, t += gridDim.x) {
            const int rt_local = t / p.n_col_tiles;
            prefetch_tile<ROWS>(xm, p, rt_local + p.rt_offset, t - rt_local * p.n_col_tiles);
        }
    }
    // Nothing above loaded or stored global data; everything below may read X
    // that the previous kernel wrote or overwrite Q/S that it reads.
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
                const int rt_local = t / p.n_col_tiles;
                const int ct = t - rt_local * p.n_col_tiles;
                load_tile<ROWS>(xm, p, sbase + L::x_off + stage * L::stage_bytes, rt_local + p.rt_offset, ct,
                                full0 + 8 * stage);
            }
            issued = it;
        }
    } else {
        // ---------------- compute warps ----------------
        const int r = tile_row<ROWS>(tid);   // row inside the tile
        const int h = tile_half<ROWS>(tid);  // which 64 columns / pair of scale blocks
        const uint32_t swz = stage_key<ROWS>(r);
        int it = 0;
        for (int t = blockIdx.x; t < p.n_tiles; t += gridDim.x, ++it) {
            const int stage = it % STAGES;
            const int qb = it % kQBufs;
            const int rt_local = t / p.n_col_tiles;
            const int ct = t - rt_local * p.n_col_tiles;
            const int rt = rt_local + p.rt_offset;
            // warp-uniform outcome, so the __syncwarp below is never divergent
            const bool ok =
                __all_sync(0xFFFFFFFFu, mbar_wait_bounded(full0 + 8 * stage, (it / STAGES) & 1, kWaitLimitNs));
            if (ok) {
                uint32_t w0[16], w1[16];
                if constexpr (ROWS) {
                    const uint8_t* slot = smem + L::x_off + stage * L::stage_bytes + (r & 7) * kPhaseBoxBytes +
                                          (r >> 3) * kRowSlot;
                    read_row_words(p, slot, rt * kTileRows + r, ct * kTileCols, h, w0, w1);
                } else {
                    const uint8_t* xrow = smem + L::x_off + stage * kStageBytes + h * kBoxBytes + r * 128;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint4 a = *reinterpret_cast<const uint4*>(xrow + ((j ^ swz) << 4));
                        const uint4 b = *reinterpret_cast<const uint4*>(xrow + (((4 + j) ^ swz) << 4));
                        w0[4 * j] = a.x; w0[4 * j + 1] = a.y; w0[4 * j + 2] = a.z; w0[4 * j + 3] = a.w;
                        w1[4 * j] = b.x; w1[4 * j + 1] = b.y; w1[4 * j + 2] = b.z; w1[4 * j + 3] = b.w;
                    }
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
            }
            // Publishes staging buffer qb.  Buffer qb is written again two
            // tiles later, after the next barrier, which every thread reaches
            // only once its stores below have read the buffer.
            if (bar_red_or(kBarCompute, kComputeThreads, !ok)) {
                if (tid == 0) {
                    report(p.status, kErrTileWait);
                    ctl[0] = 1;
                }
                break;
            }
            const uint8_t* qbuf = smem + L::q_off + qb * kQTileBytes;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int row = warp * 16 + i * 4 + (lane >> 3);
                const int chunk = lane & 7;
                const int grow = rt * kTileRows + row;
                // loaded before any branch, so the loads of all 4 iterations can be in flight together
                const uint8_t* srow = qbuf + row * 128;
                const uint32_t key = stage_key<ROWS>(row);
                const uint4 v = *reinterpret_cast<const uint4*>(srow + ((chunk ^ key) << 4));
                if constexpr (QU) {
                    uint8_t* dst = p.q + (int64_t)grow * p.ld_q + ct * kTileCols;
                    const int seg = p.q_cols - ct * kTileCols < kTileCols ? p.q_cols - ct * kTileCols : kTileCols;
                    uint4 vn = v;
                    if (reinterpret_cast<uintptr_t>(dst) & 3)  // realigned row: the next chunk too
                        vn = *reinterpret_cast<const uint4*>(srow + ((next_chunk(chunk) ^ key) << 4));
                    if (grow < p.q_rows) store_row_any<QW>(dst, v, vn, srow, key, seg, chunk, p.qw, p.status);
                } else {
                    const int col = ct * kTileCols + chunk * 16;  // q_cols % 32 == 0: a chunk is all in or all out
                    if (grow < p.q_rows && col < p.q_cols)
                        gstore(reinterpret_cast<uint4*>(p.q + (int64_t)grow * p.ld_q + col), v, p.qw, p.status);
                }
            }
            if (warp == 0) {
                const uint4 v = *reinterpret_cast<const uint4*>(smem + L::s_off + qb * kSChunkBytes + lane * 16);
                store16<QU>(p.s + ((int64_t)rt * p.col_chunks + ct) * kSChunkBytes + lane * 16, v, p.sw, p.status);
            }
        }
        if (tid == 0) ctl[1] = it;
    }
    __syncthreads();
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
constexpr int64_t kMaxTilesPerLaunch = 148 * 128;  // ~0.94 GB of traffic per launch
// The two-CTA-per-SM kernels (the row path, the any-offset stores) drift
// apart sooner: above ~8k tiles their launch times turned bimodal (16384 x
// 16383: min 6.43, median 5.68 TB/s; 16384^2 with Q 1 byte off: 4.81 or
// 5.51 from call to call); split at 148 x 64 tiles, median 6.40 on the row
// path, no change at 8192 tiles or below.
constexpr int64_t kMaxTilesPerLaunchRows = 148 * 64;

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

static int encode_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t row_stride_bytes,
                     uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
    auto encode = get_encode_fn();
    if (!encode) {
        set_last_error("cuTensorMapEncodeTiled entry point unavailable", 0);
        return MXFP8_ERR_TENSOR_MAP;
    }
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_last_error("cuTensorMapEncodeTiled failed", (int)r);
        return MXFP8_ERR_TENSOR_MAP;
    }
    return MXFP8_OK;
}

#ifdef MXFP8_CHECKED
// Checked build: the bytes a 2-D map can read, [base, base + (rows - 1) *
// stride + 2 * cols), must lie in the 16-byte chunks that hold X's own
// elements (from X's first chunk to the end of the chunk holding its last
// element).  Bounds of whole rows only; the row path's per-row spans are
// checked by construction (each map row starts in its own row's first chunk).
static int check_map_extent(const QuantizeArgs& a, uintptr_t base, uint64_t cols, uint64_t rows, uint64_t stride) {
    const uintptr_t x = reinterpret_cast<uintptr_t>(a.x);
    const uintptr_t lo = x & ~(uintptr_t)15;
    const uintptr_t hi = (x + 2 * (uintptr_t)((a.m - 1) * a.ld_x + a.k) + 15) & ~(uintptr_t)15;
    const uintptr_t end = base + (rows - 1) * stride + 2 * cols;
    if (base < lo || end > hi) {
        set_last_error("checked build: a tensor map of X reaches outside X's bytes", 0);
        return MXFP8_ERR_TENSOR_MAP;
    }
    return MXFP8_OK;
}
#endif

// Tensor maps of X.  Tensor path: one map, 64 x 128 boxes, 128-byte swizzle.
// Row path: one map per phase f < min(m, 8) (see the file comment).
template <bool ROWS>
static int encode_x_maps(const QuantizeArgs& a, XMaps<ROWS>& xm) {
    memset(&xm, 0, sizeof(xm));
    if constexpr (!ROWS) {
#ifdef MXFP8_CHECKED
        if (int rc = check_map_extent(a, reinterpret_cast<uintptr_t>(a.x), (uint64_t)a.k, (uint64_t)a.m,
                                      (uint64_t)a.ld_x * 2))
            return rc;
#endif
        return encode_2d(&xm.map[0], a.x, (uint64_t)a.k, (uint64_t)a.m, (uint64_t)a.ld_x * 2, kBoxCols, kTileRows,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    } else {
        const int64_t phases = a.m < kPhases ? a.m : kPhases;
        for (int64_t f = 0; f < phases; ++f) {
            const uintptr_t row0 = reinterpret_cast<uintptr_t>(a.x) + (uintptr_t)(2 * f * a.ld_x);
            const uintptr_t base = row0 & ~(uintptr_t)15;
            const uint64_t d = (row0 - base) / 2;  // elements of misalignment, < 8
            const uint64_t rows = (uint64_t)((a.m - f + kPhases - 1) / kPhases);
#ifdef MXFP8_CHECKED
            if (int rc = check_map_extent(a, base, (uint64_t)a.k + d, rows, (uint64_t)a.ld_x * 2 * kPhases)) return rc;
#endif
            int rc = encode_2d(&xm.map[f], reinterpret_cast<const void*>(base), (uint64_t)a.k + d, rows,
                               (uint64_t)a.ld_x * 2 * kPhases, kRowBoxCols, kPhaseRows, CU_TENSOR_MAP_SWIZZLE_NONE);
            if (rc) return rc;
        }
        return MXFP8_OK;
    }
}

template <int DT, bool ROWS, bool QU, int QW = -1>
static int launch_tma_typed(const QuantizeArgs& a, int sm_count, cudaStream_t stream) {
    constexpr int kSt = (ROWS || QU) ? kRowStages : kStages;
    constexpr int kCtasPerSm = (ROWS || QU) ? kRowCtasPerSm : 1;
    using L = Layout<kSt, ROWS>;
    auto kernel = quantize_tma_kernel<DT, kSt, ROWS, QU, QW>;
    // The shared-memory opt-in is per device: set it once per device, so that
    // later launches (including ones under stream capture) make no such call.
    static std::atomic<uint64_t> attr_set{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (e == cudaSuccess && !(attr_set.load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::alloc);
        if (e == cudaSuccess && (ROWS || QU))
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared);
        if (e == cudaSuccess) attr_set.fetch_or(bit, std::memory_order_acq_rel);
    }
    if (e != cudaSuccess) {
        set_last_error("cudaFuncSetAttribute", (int)e);
        return MXFP8_ERR_CUDA;
    }
    XMaps<ROWS> xm;
    int rc = encode_x_maps<ROWS>(a, xm);
    if (rc) return rc;
    TmaParams p;
    p.x = static_cast<const uint8_t*>(a.x);
    p.ld_x = a.ld_x;
    p.m = (int)a.m;
    p.k = (int)a.k;
    p.n_phases = (int)(a.m < kPhases ? a.m : kPhases);
    const int64_t n_row_tiles = a.scale_rows / kTileRows;
    p.n_col_tiles = (int)a.col_chunks;
    p.q = a.q;
    p.ld_q = a.ld_q;
    p.q_rows = (int)a.q_rows;
    p.q_cols = (int)a.q_cols;
    p.scale_cols = (int)a.scale_cols;
    p.col_chunks = (int)a.col_chunks;
    p.s = a.s;
    p.status = a.status;
    p.qw = a.qw;
    p.sw = a.sw;
    // Long problems run as several launches of at most kMaxTilesPerLaunch
    // tiles (whole row tiles, i.e. contiguous slices of Q and S), chained by
    // the dependent launch.  Persistent CTAs drift apart over thousands of
    // tiles and the spread-out access front streams worse; restarting them
    // in step every ~0.9 GB measured 6.77 vs 6.35 TB/s at 131072x16384 and
    // changed nothing at 16384^2 or below.
    int64_t rows_per_launch = n_row_tiles;
    const int64_t max_tiles = (ROWS || QU) ? kMaxTilesPerLaunchRows : kMaxTilesPerLaunch;
    if (n_row_tiles * a.col_chunks > max_tiles) {
        rows_per_launch = max_tiles / a.col_chunks;
        if (rows_per_launch < 1) rows_per_launch = 1;
    }
    for (int64_t r0 = 0; r0 < n_row_tiles && e == cudaSuccess; r0 += rows_per_launch) {
        const int64_t nr = n_row_tiles - r0 < rows_per_launch ? n_row_tiles - r0 : rows_per_launch;
        p.rt_offset = (int)r0;
        p.n_tiles = (int)(nr * a.col_chunks);
        const int ctas = sm_count * kCtasPerSm;
        const int grid = p.n_tiles < ctas ? p.n_tiles : ctas;
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
        e = cudaLaunchKernelEx(&cfg, kernel, xm, p);
        if (e == cudaSuccess) e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        set_last_error("quantize_tma_kernel launch", (int)e);
        return MXFP8_ERR_CUDA;
    }
    return MXFP8_OK;
}

// Any-offset stores with X through one tensor map.  When every Q row starts
// at the same byte offset d within 16 bytes (ld_q % 16 == 0) and d is not a
// multiple of 4, every realigned row takes its words from the same place
// (h / 4 with h = 16 - d), so a kernel with that word offset built in runs
// without the per-row selects: 8192^2 bf16 with Q 1 byte off, 5.33 -> 5.51
// TB/s (every offset 1-15 that is not a multiple of 4: 5.49-5.51).
template <int DT>
static int launch_tensor_qu(const QuantizeArgs& a, int sm_count, cudaStream_t stream) {
    const uint32_t d = (uint32_t)(reinterpret_cast<uintptr_t>(a.q) & 15);
    if (a.ld_q % 16 != 0 || (d & 3) == 0) return launch_tma_typed<DT, false, true>(a, sm_count, stream);
    switch ((16 - d) >> 2) {
        case 0: return launch_tma_typed<DT, false, true, 0>(a, sm_count, stream);
        case 1: return launch_tma_typed<DT, false, true, 1>(a, sm_count, stream);
        case 2: return launch_tma_typed<DT, false, true, 2>(a, sm_count, stream);
        default: return launch_tma_typed<DT, false, true, 3>(a, sm_count, stream);
    }
}

int launch_quantize_tma(const QuantizeArgs& a, int sm_count, cudaStream_t stream) {
    // rows a single tensor map can describe: 16-byte aligned base and row stride
    const bool tensor = (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && a.ld_x % 8 == 0;
    // outputs at any byte offset: narrower stores where a 16-byte store cannot go
    const bool qu = (reinterpret_cast<uintptr_t>(a.q) & 15) != 0 || a.ld_q % 16 != 0 ||
                    (reinterpret_cast<uintptr_t>(a.s) & 15) != 0;
    if (a.dtype == kBF16) {
        if (qu)
            return tensor ? launch_tensor_qu<kBF16>(a, sm_count, stream)
                          : launch_tma_typed<kBF16, true, true>(a, sm_count, stream);
        return tensor ? launch_tma_typed<kBF16, false, false>(a, sm_count, stream)
                      : launch_tma_typed<kBF16, true, false>(a, sm_count, stream);
    }
    if (qu)
        return tensor ? launch_tensor_qu<kFP16>(a, sm_count, stream)
                      : launch_tma_typed<kFP16, true, true>(a, sm_count, stream);
    return tensor ? launch_tma_typed<kFP16, false, false>(a, sm_count, stream)
                  : launch_tma_typed<kFP16, true, false>(a, sm_count, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free launch.  The kernel above needs one word of global scratch:
// its status word, which a bounded wait that times out (or, in the checked
// build, a skipped store) marks with atomicOr.  mxfp8_quantize keeps that word
// in a buffer it allocates on its first call on each device; this variant
// keeps it in a fixed device array of this file instead, so it never
// allocates.  Every GPU that loads the library holds the array until exit.
// The word is sticky: calls only set bits; mxfp8_noalloc_status reads it and
// clears it on request.  A static __device__ array starts at zero.
// ---------------------------------------------------------------------------

constexpr int kNoAllocScratchWords = 64;  // 256 bytes per device
constexpr int kStatusWordsPerCall = 1;
constexpr int kMaxNoAllocDevices = 64;
static __device__ __align__(256) unsigned int g_noalloc_scratch[kNoAllocScratchWords];

struct NoAllocSlot {
    uint64_t ctx;        // context_key() the address was looked up in
    unsigned int* addr;  // device address of g_noalloc_scratch there
};
static std::mutex g_noalloc_mu;
static NoAllocSlot g_noalloc_slot[kMaxNoAllocDevices];

// Device address of g_noalloc_scratch on device `dev` (the current device),
// looked up once per device and context: the first call on a device, and the
// first after its context changed (cudaDeviceReset, another driver-API
// context made current), calls cudaGetSymbolAddress, which allocates nothing.
// In host code the array's name is only a host-side stand-in; kernels must be
// given this address.
int noalloc_status_word(int dev, unsigned int** out) {
    static_assert(kStatusWordsPerCall <= kNoAllocScratchWords, "scratch array too small");
    if (dev < 0 || dev >= kMaxNoAllocDevices) {
        set_last_error("device index beyond the allocation-free table", 0);
        return MXFP8_ERR_DEVICE;
    }
    uint64_t ctx = 0;
    if (int rc = bound_context_key(&ctx)) return rc;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocSlot& slot = g_noalloc_slot[dev];
    if (!slot.addr || slot.ctx != ctx) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr) {
            set_last_error("cudaGetSymbolAddress(g_noalloc_scratch)", (int)e);
            return MXFP8_ERR_CUDA;
        }
        slot.addr = static_cast<unsigned int*>(ptr);
        slot.ctx = ctx;
    }
    *out = slot.addr;
    return MXFP8_OK;
}

int launch_quantize_tma_noalloc(const QuantizeArgs& args, int dev, int sm_count, cudaStream_t stream) {
    unsigned int* scratch = nullptr;
    int rc = noalloc_status_word(dev, &scratch);
    if (rc) return rc;
    QuantizeArgs a = args;
    a.status = scratch;
    return launch_quantize_tma(a, sm_count, stream);
}

}  // namespace mxfp8
