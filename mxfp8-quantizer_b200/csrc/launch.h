// launch.h -- internal host-side launch interface between the C ABI
// (capi.cu) and the kernel translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "guard.cuh"

namespace mxfp8 {

// Problem description after argument validation.
struct QuantizeArgs {
    const void* x;
    int dtype;
    int64_t m, k, ld_x;
    uint8_t* q;
    int64_t q_rows, q_cols, ld_q;
    uint8_t* s;
    int64_t scale_rows;   // q_rows rounded up to 128
    int64_t scale_cols;   // q_cols / 32
    int64_t col_chunks;   // ceil(scale_cols / 4)
    unsigned int* status; // device error word (may be null)
    StoreWindow qw, sw;   // bytes the kernels may write: Q rows, S storage
};

// Returned by launchers: 0, or a negative mxfp8_status.
int launch_quantize_tma(const QuantizeArgs& a, int sm_count, cudaStream_t stream);
int launch_quantize_generic(const QuantizeArgs& a, int sm_count, cudaStream_t stream);
// Same kernel as launch_quantize_tma, scratch in a fixed device array (never allocates).
int launch_quantize_tma_noalloc(const QuantizeArgs& a, int dev, int sm_count, cudaStream_t stream);
int launch_dequantize(const uint8_t* q, int64_t rows, int64_t cols, int64_t ld_q, const uint8_t* s,
                      void* out, int out_dtype, int64_t ld_out, StoreWindow ow, unsigned int* status,
                      cudaStream_t stream);

int launch_bounded_wait_selftest(unsigned int* status, uint32_t limit_us, cudaStream_t stream);

// Records the CUDA error text for mxfp8_last_error() on this host thread.
void set_last_error(const char* what, int code);

// Key of the CUDA context current on this host thread, unique for the
// process's lifetime; 0 if none is current (context_key) or after binding the
// runtime's context to the thread first (bound_context_key, never 0 on
// success).  Per-device caches compare it to notice a new context.
int context_key(uint64_t* key);
int bound_context_key(uint64_t* key);

// Device address of the allocation-free entries' status word (a fixed device
// array of quantize_tma.cu) on device `dev`, the current device.
int noalloc_status_word(int dev, unsigned int** out);

}  // namespace mxfp8
