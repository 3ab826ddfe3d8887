/*
 * mxfp8.h -- C ABI of the B200 MXFP8 quantizer (libmxfp8.so, sm_100a).
 *
 * X (bf16 or fp16, row-major) -> Q (FP8 E4M3 bytes, row-major) plus S (one
 * UE8M0 byte per 1x32 block along K) written straight into the tcgen05
 * block-scaled layout: 128-row x 4-column chunks of 512 bytes, chunk
 * (row_block, col_block) at byte ((row_block * CB + col_block) * 512), scale
 * (r, c) at (r % 32) * 16 + ((r % 128) / 32) * 4 + (c % 4) inside it, with
 * CB = ceil(scale_cols / 4).
 *
 * All pointers are device pointers unless named *_host.  Streams are
 * cudaStream_t / CUstream handles passed as void*.  Functions never
 * synchronise and never allocate, except where stated.  Every function is
 * safe to call from several host threads.  Return values: MXFP8_OK (0) or a
 * negative mxfp8_status; mxfp8_strerror() names it.
 */
#ifndef MXFP8_H_
#define MXFP8_H_

#include <stdint.h>

#if defined(__GNUC__)
#define MXFP8_API __attribute__((visibility("default")))
#else
#define MXFP8_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef void* mxfp8_stream_t; /* cudaStream_t / CUstream */

enum mxfp8_dtype { MXFP8_BF16 = 0, MXFP8_FP16 = 1, MXFP8_F32 = 2 };

enum mxfp8_status {
    MXFP8_OK = 0,
    MXFP8_ERR_NULL_POINTER = -1,   /* a required pointer is NULL */
    MXFP8_ERR_SHAPE = -2,          /* sizes out of range or inconsistent */
    MXFP8_ERR_DTYPE = -3,          /* unsupported dtype code */
    MXFP8_ERR_ALIGNMENT = -4,      /* a pointer or stride breaks the alignment contract */
    MXFP8_ERR_SCALE_BUFFER = -5,   /* the scale buffer is smaller than required */
    MXFP8_ERR_CUDA = -6,           /* a CUDA runtime call failed (launch, attribute, ...) */
    MXFP8_ERR_TENSOR_MAP = -7,     /* the driver rejected a TMA descriptor */
    MXFP8_ERR_DEVICE = -8          /* no usable sm_100 device is current */
};

/* Packed scale storage bytes for a (rows, cols) quantized matrix:
 * ceil(rows/128)*128 * ceil(ceil(cols/32)/4)*4.  Returns -1 if rows or cols
 * is negative.
 * Replaces packed_scale_storage_bytes, MXFP8_quantizer.py:531-539. */
MXFP8_API int64_t mxfp8_scale_storage_bytes(int64_t rows, int64_t cols);

/* The reference's launch shape: kernel_m = ceil(m/8)*8, kernel_k =
 * ceil(k/256)*256, with its limits (m, k >= 1 and <= INT32_MAX, at most
 * 65535 K-tiles).  Returns MXFP8_ERR_SHAPE when the reference would raise.
 * Replaces shape_problem, MXFP8_quantizer.py:766-791. */
MXFP8_API int mxfp8_launch_shape(int64_t m, int64_t k, int64_t* kernel_m, int64_t* kernel_k);

/* General quantizer.
 *   x      : (m, k) input, row stride ld_x elements (ld_x >= k), 2-byte aligned
 *   q      : (q_rows, q_cols) E4M3 output, row stride ld_q bytes
 *   s      : packed scale storage for (q_rows, q_cols), s_bytes >=
 *            mxfp8_scale_storage_bytes(q_rows, q_cols), 4-byte aligned
 * q_rows >= m, q_cols >= k, q_cols % 32 == 0.  Elements outside (m, k) are
 * quantized as zeros, so padded blocks get scale byte 127 and payload 0x00
 * exactly as in the reference's zero-padded launch; scale bytes of rows >=
 * q_rows (up to the next multiple of 128) or of columns >= q_cols/32 (up to
 * the next multiple of 4) are written as 0.  Every byte of
 * Q[0:q_rows, 0:q_cols] and of the first mxfp8_scale_storage_bytes(q_rows,
 * q_cols) bytes of S is written; nothing needs zeroing beforehand.
 * Every non-empty x runs through one persistent TMA-pipelined kernel: it
 * reads x through one tensor map when x is 16-byte aligned and ld_x % 8 ==
 * 0, else through one tensor map per row phase (row % 8), and writes q and s
 * at any offset (16-byte stores when q, ld_q and s allow them, narrower or
 * realigned stores otherwise).  Empty x (m or k == 0) takes a plain-load
 * kernel that writes the padding.
 * The first call on a device (and the first in each new CUDA context of it)
 * allocates that device's 256-byte status word (see mxfp8_device_status), so
 * make it before any stream capture; later calls allocate nothing.
 * Replaces the host pad copy + launch of materialize_quantizer_buffers and
 * the compiled kernel call, MXFP8_quantizer.py:554-608 and 914-922. */
MXFP8_API int mxfp8_quantize(const void* x, int dtype, int64_t m, int64_t k, int64_t ld_x,
                   void* q, int64_t q_rows, int64_t q_cols, int64_t ld_q,
                   void* s, int64_t s_bytes, mxfp8_stream_t stream);

/* Allocation-free variant of mxfp8_quantize: same arguments, checks,
 * kernels and output bytes, but no call ever allocates device memory.
 * No counterpart in the reference.
 * Who needs it: callers that may not call cudaMalloc.  mxfp8_quantize
 * allocates a 256-byte status buffer on its first call on each device, which
 * fails or is forbidden for plugins whose host owns all device memory
 * through its own pool or arena, for code whose allocations must all be made
 * up front (real-time or certified pipelines), and on a device whose memory
 * another allocator has already reserved in full.
 * How: the quantize kernel's only scratch, one 32-bit status word that a
 * pipeline wait which times out marks, lives in a fixed 256-byte device
 * array of the library (64 words; every GPU that loads the library holds it
 * until exit).  A call needs 1 word, so no problem size exceeds the array.
 * The first call on each device (and the first after its CUDA context
 * changed) looks up the array's device address with cudaGetSymbolAddress,
 * which allocates nothing; make that first call before any stream capture.
 * The word is sticky: calls only set bits in it, and
 * mxfp8_noalloc_status reads it (and clears it on request).  All calls on a
 * device share the word, so after calls whose kernels overlap on the GPU
 * (different streams) a set bit cannot be attributed to one of them, and a
 * clear that runs while such a kernel is in flight can lose its report. */
MXFP8_API int mxfp8_quantize_noalloc(const void* x, int dtype, int64_t m, int64_t k, int64_t ld_x,
                                     void* q, int64_t q_rows, int64_t q_cols, int64_t ld_q,
                                     void* s, int64_t s_bytes, mxfp8_stream_t stream);

/* Reference-compatible launch on already padded, contiguous buffers: x and q
 * are (m, k) with m % 8 == 0 and k % 256 == 0 (the reference's launch shape),
 * s holds s_word_count 32-bit words (>= the packed storage of (m, k)).
 * Argument meaning follows the compiled CuTeDSL callable
 * (x_ptr, q_dwords_ptr, s_words_ptr, m, k, s_word_count, stream) plus the
 * input dtype, which the reference bakes into its compile key.
 * Replaces BlackwellMXFP8Quantizer.__call__ / its compiled launch,
 * MXFP8_quantizer.py:266-353 (called at 836-844 and 914-922). */
MXFP8_API int mxfp8_quantize_padded(const void* x, void* q_dwords, void* s_words, int64_t m, int64_t k,
                          int64_t s_word_count, int dtype, mxfp8_stream_t stream);

/* Dequantize Q (rows, cols) with packed scales S (s_bytes >=
 * mxfp8_scale_storage_bytes(rows, cols), else MXFP8_ERR_SCALE_BUFFER) into
 * out (rows, cols) of out_dtype (MXFP8_BF16, MXFP8_FP16 or MXFP8_F32), row
 * stride ld_out elements: out = e4m3(Q) * 2^(S - 127); scale byte 255 decodes
 * to NaN.  cols % 32 == 0.  The inverse used by the reference's end-to-end
 * check, MXFP8_quantizer.py:1179-1187. */
MXFP8_API int mxfp8_dequantize(const void* q, int64_t rows, int64_t cols, int64_t ld_q, const void* s,
                               int64_t s_bytes, void* out, int out_dtype, int64_t ld_out, mxfp8_stream_t stream);

/* Sticky device-side error word of the current device (0 = none).  Kernels
 * never trap: a pipeline wait that exceeds its time limit (about 1 s) sets a
 * bit here and the kernel returns early.  Bits: 1 = payload tile wait,
 * 2 = stage-release wait, 4 = drain wait on exit, 8 = the self-test's wait,
 * 16 = a store outside its output was skipped (only the checked build,
 * include/mxfp8_checked.h, tests stores).  Reading waits for the device
 * (cudaDeviceSynchronize); clear != 0 resets the word.  The word lives in a
 * small device buffer allocated on the first call on each device (and in
 * each new CUDA context of it).  Calls of mxfp8_quantize_noalloc report to
 * their own word instead (mxfp8_noalloc_status).
 * No counterpart in the reference (its kernel waits without a limit). */
MXFP8_API int mxfp8_device_status(uint32_t* status_out, int clear);

/* The status word of mxfp8_quantize_noalloc calls on the current device:
 * same bits and same reading rules as mxfp8_device_status (waits for the
 * device; clear != 0 resets the word), read from the library's fixed device
 * array, so this allocates no device memory either.
 * No counterpart in the reference (its kernel waits without a limit). */
MXFP8_API int mxfp8_noalloc_status(uint32_t* status_out, int clear);

/* Failure-path self-test: launches one CTA that waits, with the same bounded
 * wait the quantizer pipeline uses, on an mbarrier nothing completes; after
 * limit_us (1 .. 10^7) it gives up, sets bit 8 of the device status word and
 * returns.  No fault, no trap: the context stays usable.  Read the result
 * with mxfp8_device_status after synchronising.
 * No counterpart in the reference (its kernel waits without a limit). */
MXFP8_API int mxfp8_selftest_bounded_wait(uint32_t limit_us, mxfp8_stream_t stream);

/* Name of a status code. */
MXFP8_API const char* mxfp8_strerror(int status);

/* Text of the CUDA error behind the last MXFP8_ERR_CUDA / MXFP8_ERR_TENSOR_MAP
 * returned on this host thread ("" if none). */
MXFP8_API const char* mxfp8_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* MXFP8_H_ */
