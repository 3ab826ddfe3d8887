// tile.cuh -- tile geometry, shared-memory layout and kernel parameters of
// the pipelined quantizer (quantize_tma.cu).
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "guard.cuh"

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
constexpr int kPrefetchTiles = 2;                        // L2 prefetch before the dependency wait
constexpr uint64_t kWaitLimitNs = 1000000000ull;          // 1 s per pipeline wait
constexpr uint32_t kBarCompute = 1;                       // named barrier id

constexpr unsigned kErrTileWait = 1u, kErrReleaseWait = 2u, kErrDrainWait = 4u;

// Row path staging: per phase, a 16-row box of 136 columns (272 bytes: 128
// columns plus up to 7 of misalignment, a multiple of 16 bytes).
constexpr int kPhases = 8;
constexpr int kPhaseRows = kTileRows / kPhases;           // 16 box rows per phase and tile
constexpr int kRowBoxCols = 136;
constexpr int kRowSlot = kRowBoxCols * 2;                 // 272
constexpr int kPhaseBoxBytes = kPhaseRows * kRowSlot;     // 4352 (a multiple of 128)
constexpr int kRowStageBytes = kPhases * kPhaseBoxBytes;  // 34 KiB of X per tile
// The row path's compute warps do more work per tile (the register shift), so
// it runs 2 CTAs per SM with 2 stages each (~105 KiB of shared memory apiece)
// for twice the warps: 8192 x 8191 bf16 6.25 vs 5.99 TB/s with 1 CTA x 3
// stages (1 CTA x 4 or x 2 stages: slower still).  The any-offset store path
// (QU, whose store pass realigns rows) runs the same way: 8192^2 bf16 with Q
// 1 byte off 5.45 vs 4.87 TB/s, 4 bytes off 6.15 vs 5.78.
constexpr int kRowStages = 2;
constexpr int kRowCtasPerSm = 2;

template <bool ROWS>
struct XMaps {
    CUtensorMap map[ROWS ? kPhases : 1];
};

template <int STAGES, bool ROWS>
struct Layout {
    static constexpr int stage_bytes = ROWS ? kRowStageBytes : kStageBytes;
    static constexpr int x_off = 0;
    static constexpr int q_off = STAGES * stage_bytes;
    static constexpr int s_off = q_off + kQBufs * kQTileBytes;
    static constexpr int bar_off = s_off + kQBufs * kSChunkBytes;
    static constexpr int ctl_off = bar_off + 2 * STAGES * 8;
    static constexpr int bytes = ctl_off + 16;
    static constexpr int alloc = bytes + 1024;  // slack to align the base to 1024
};

struct TmaParams {
    int rt_offset;  // first row tile of this launch (long problems are split by row tiles)
    const uint8_t* x;  // row path only: X base and row stride (for each row's misalignment)
    int64_t ld_x;
    int m;
    int k;
    int n_phases;   // row path: tensor maps in use, min(m, 8)
    uint8_t* q;
    int64_t ld_q;
    int q_rows;
    int q_cols;
    int n_tiles;
    int n_col_tiles;
    int scale_cols;
    int col_chunks;
    uint8_t* s;
    unsigned int* status;
    StoreWindow qw, sw;  // what the stores may touch (checked build)
};

}  // namespace mxfp8
