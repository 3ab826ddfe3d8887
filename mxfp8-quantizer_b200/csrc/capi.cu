// capi.cu -- the extern "C" boundary of libmxfp8.so (declared in
// include/mxfp8.h): argument validation, per-device state, kernel choice.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <string>

#include "../../include/mxfp8.h"
#ifdef MXFP8_CHECKED
#include "../../include/mxfp8_checked.h"
#endif
#include "launch.h"

namespace mxfp8 {

namespace {

constexpr int kMaxDevices = 64;
constexpr int64_t kInt32Max = 2147483647;

struct DeviceState {
    bool ready = false;
    uint64_t ctx = 0;  // context_key() of the context the status word belongs to
    int sm_count = 0;
    int cc_major = 0, cc_minor = 0;
    unsigned int* status = nullptr;  // device error word (see mxfp8_device_status)
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
thread_local std::string g_last_error;

// Lazily fills the state of the current device: its properties, and a status
// word allocated in the context current on this thread.  A context that is
// not the one the word was allocated in (after cudaDeviceReset, or another
// driver-API context made current) gets a word of its own: the old one went
// with its context.  Returns 0 or a negative status.
int current_device(DeviceState** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        set_last_error("cudaGetDevice", (int)e);
        return MXFP8_ERR_DEVICE;
    }
    uint64_t ctx = 0;
    if (int rc = bound_context_key(&ctx)) return rc;
    std::lock_guard<std::mutex> lock(g_mu);
    DeviceState& st = g_dev[dev];
    if (!st.ready) {
        cudaDeviceProp prop;
        e = cudaGetDeviceProperties(&prop, dev);
        if (e != cudaSuccess) {
            set_last_error("cudaGetDeviceProperties", (int)e);
            return MXFP8_ERR_DEVICE;
        }
        st.sm_count = prop.multiProcessorCount;
        st.cc_major = prop.major;
        st.cc_minor = prop.minor;
        st.ready = true;
    }
    if (st.cc_major != 10 || st.cc_minor != 0) {
        set_last_error("libmxfp8 is built for sm_100a (B200); the current device is another architecture", 0);
        return MXFP8_ERR_DEVICE;
    }
    if (!st.status || ctx != st.ctx) {
        unsigned int* word = nullptr;
        e = cudaMalloc(&word, 256);
        if (e == cudaSuccess) e = cudaMemset(word, 0, 256);
        if (e != cudaSuccess) {
            set_last_error("status word allocation", (int)e);
            return MXFP8_ERR_CUDA;
        }
        st.status = word;
        st.ctx = ctx;
    }
    *out = &st;
    return MXFP8_OK;
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Kernel choice, shared by both quantize entries.  The pipelined kernel takes
// every non-empty X: through one tensor map when X's rows are 16-byte aligned
// and through one tensor map per row phase (row % 8) otherwise, and writes Q
// and S at any offset (narrower stores where 16-byte ones cannot go).  Row
// phases are 16 * ld_x bytes apart and a tensor-map stride must stay below
// 2^40 bytes, so larger strides of unaligned rows (only reachable with sparse
// address reservations) take the plain-load kernel, as does empty X.
bool use_pipelined(const void* x, int64_t ld_x, bool has_x) {
    return has_x && ((aligned(x, 16) && ld_x % 8 == 0) || ld_x < (int64_t(1) << 36));
}

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

#ifdef MXFP8_CHECKED
std::atomic<int64_t> g_window_slack{0};
#endif

// The bytes [base, base + bytes) a kernel may write.  The checked build
// narrows it by mxfp8_checked_window_slack bytes, to show that its store
// guards fire; the product build ignores the window.
StoreWindow make_window(void* base, int64_t bytes) {
    uint8_t* lo = static_cast<uint8_t*>(base);
#ifdef MXFP8_CHECKED
    bytes -= g_window_slack.load(std::memory_order_relaxed);
    if (bytes < 0) bytes = 0;
#endif
    return StoreWindow{lo, lo + bytes};
}

// Argument checks and problem description shared by both quantize entries,
// so the two keep one contract.  Returns 0 or a negative status; *launch is
// false when there is nothing to write (q_rows or q_cols == 0).
int make_quantize_args(const void* x, int dtype, int64_t m, int64_t k, int64_t ld_x, void* q, int64_t q_rows,
                       int64_t q_cols, int64_t ld_q, void* s, int64_t s_bytes, QuantizeArgs* a, bool* launch) {
    *launch = false;
    if (dtype != MXFP8_BF16 && dtype != MXFP8_FP16) return MXFP8_ERR_DTYPE;
    if (m < 0 || k < 0 || q_rows < m || q_cols < k || q_cols % 32 != 0 || ld_x < k || ld_q < q_cols ||
        q_rows > kInt32Max || q_cols > kInt32Max || ld_x > (int64_t(1) << 38) || ld_q > (int64_t(1) << 39))
        return MXFP8_ERR_SHAPE;
    if (q_rows == 0 || q_cols == 0) return MXFP8_OK;
    const bool has_x = m > 0 && k > 0;
    if (!q || !s || (has_x && !x)) return MXFP8_ERR_NULL_POINTER;
    if ((has_x && !aligned(x, 2)) || !aligned(s, 4)) return MXFP8_ERR_ALIGNMENT;
    if (s_bytes < mxfp8_scale_storage_bytes(q_rows, q_cols)) return MXFP8_ERR_SCALE_BUFFER;

    a->x = x;
    a->dtype = dtype;
    a->m = m;
    a->k = k;
    a->ld_x = ld_x;
    a->q = static_cast<uint8_t*>(q);
    a->q_rows = q_rows;
    a->q_cols = q_cols;
    a->ld_q = ld_q;
    a->s = static_cast<uint8_t*>(s);
    a->scale_rows = ceil_div(q_rows, 128) * 128;
    a->scale_cols = q_cols / 32;
    a->col_chunks = ceil_div(a->scale_cols, 4);
    a->qw = make_window(q, (q_rows - 1) * ld_q + q_cols);
    a->sw = make_window(s, mxfp8_scale_storage_bytes(q_rows, q_cols));
    a->status = nullptr;
    if ((a->scale_rows / 128) * a->col_chunks > kInt32Max) return MXFP8_ERR_SHAPE;
    *launch = true;
    return MXFP8_OK;
}

}  // namespace

// A key of the CUDA context current on this host thread, unique for the
// process's lifetime (cuCtxGetId: never reused, unlike the handle), or 0 if
// no context is current yet.  Driver entry points come through the runtime,
// so the library needs no link to libcuda.
int context_key(uint64_t* key) {
    static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    static PFN_cuCtxGetId_v12000 get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 4000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(f);
    });
    *key = 0;
    if (!get_current || !get_id) {
        set_last_error("cuCtxGetCurrent / cuCtxGetId entry points unavailable", 0);
        return MXFP8_ERR_DEVICE;
    }
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return MXFP8_OK;
    unsigned long long id = 0;
    if (get_id(ctx, &id) != CUDA_SUCCESS) {
        set_last_error("cuCtxGetId failed", 0);
        return MXFP8_ERR_DEVICE;
    }
    *key = id + 1;  // 0 stays "no context"
    return MXFP8_OK;
}

// context_key() of the context the runtime uses on this thread, binding it
// first if none is current yet (cudaMemGetInfo needs a context and allocates
// nothing).
int bound_context_key(uint64_t* key) {
    if (int rc = context_key(key)) return rc;
    if (*key) return MXFP8_OK;
    size_t free_b = 0, total_b = 0;
    cudaError_t e = cudaMemGetInfo(&free_b, &total_b);
    if (e != cudaSuccess) {
        set_last_error("cudaMemGetInfo", (int)e);
        return MXFP8_ERR_DEVICE;
    }
    if (int rc = context_key(key)) return rc;
    if (!*key) {
        set_last_error("no CUDA context is current", 0);
        return MXFP8_ERR_DEVICE;
    }
    return MXFP8_OK;
}

// Current device and its SM count for the allocation-free entries, from
// attribute queries (no properties cache, nothing allocated); rejects
// devices other than sm_100.
int noalloc_device(int* dev, int* sm_count) {
    int major = 0, minor = 0;
    cudaError_t e = cudaGetDevice(dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(sm_count, cudaDevAttrMultiProcessorCount, *dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, *dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, *dev);
    if (e != cudaSuccess) {
        set_last_error("device query", (int)e);
        return MXFP8_ERR_DEVICE;
    }
    if (major != 10 || minor != 0) {
        set_last_error("libmxfp8 is built for sm_100a (B200); the current device is another architecture", 0);
        return MXFP8_ERR_DEVICE;
    }
    return MXFP8_OK;
}

// Waits for the device, then copies a status word to the host and clears it
// if asked.  Nothing runs on the device in between unless another host
// thread launches work meanwhile.
int read_status_word(unsigned int* word, uint32_t* out, int clear, const char* what) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(out, word, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(word, 0, sizeof(uint32_t));
    if (e == cudaSuccess && clear) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        set_last_error(what, (int)e);
        return MXFP8_ERR_CUDA;
    }
    return MXFP8_OK;
}

void set_last_error(const char* what, int code) {
    g_last_error = what;
    if (code) {
        g_last_error += ": ";
        g_last_error += cudaGetErrorName(static_cast<cudaError_t>(code));
        g_last_error += " (";
        g_last_error += std::to_string(code);
        g_last_error += ")";
    }
}

}  // namespace mxfp8

using namespace mxfp8;

extern "C" MXFP8_API int64_t mxfp8_scale_storage_bytes(int64_t rows, int64_t cols) {
    if (rows < 0 || cols < 0) return -1;
    return ceil_div(rows, 128) * 128 * (ceil_div(ceil_div(cols, 32), 4) * 4);
}

extern "C" MXFP8_API int mxfp8_launch_shape(int64_t m, int64_t k, int64_t* kernel_m, int64_t* kernel_k) {
    if (!kernel_m || !kernel_k) return MXFP8_ERR_NULL_POINTER;
    if (m < 1 || k < 1 || m > kInt32Max || k > kInt32Max) return MXFP8_ERR_SHAPE;
    const int64_t km = ceil_div(m, 8) * 8, kk = ceil_div(k, 256) * 256;
    if (km / 8 > kInt32Max || kk / 256 > 65535) return MXFP8_ERR_SHAPE;
    *kernel_m = km;
    *kernel_k = kk;
    return MXFP8_OK;
}

extern "C" MXFP8_API int mxfp8_quantize(const void* x, int dtype, int64_t m, int64_t k, int64_t ld_x, void* q,
                              int64_t q_rows, int64_t q_cols, int64_t ld_q, void* s, int64_t s_bytes,
                              mxfp8_stream_t stream) {
    QuantizeArgs a;
    bool launch = false;
    int rc = make_quantize_args(x, dtype, m, k, ld_x, q, q_rows, q_cols, ld_q, s, s_bytes, &a, &launch);
    if (rc || !launch) return rc;
    DeviceState* dev = nullptr;
    rc = current_device(&dev);
    if (rc) return rc;
    a.status = dev->status;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return use_pipelined(x, ld_x, a.m > 0 && a.k > 0) ? launch_quantize_tma(a, dev->sm_count, st)
                                                      : launch_quantize_generic(a, dev->sm_count, st);
}

// Allocation-free entry: the same argument checks and kernels as
// mxfp8_quantize, but device properties come from attribute queries and the
// kernel's status word lives in a fixed device array (quantize_tma.cu), so
// no call, first or later, allocates device memory.
extern "C" MXFP8_API int mxfp8_quantize_noalloc(const void* x, int dtype, int64_t m, int64_t k, int64_t ld_x,
                                               void* q, int64_t q_rows, int64_t q_cols, int64_t ld_q, void* s,
                                               int64_t s_bytes, mxfp8_stream_t stream) {
    QuantizeArgs a;
    bool launch = false;
    int rc = make_quantize_args(x, dtype, m, k, ld_x, q, q_rows, q_cols, ld_q, s, s_bytes, &a, &launch);
    if (rc || !launch) return rc;
    int dev = -1, sms = 0;
    if (int drc = noalloc_device(&dev, &sms)) return drc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Same dispatch as mxfp8_quantize; the plain-load kernel uses no scratch.
    return use_pipelined(x, ld_x, a.m > 0 && a.k > 0) ? launch_quantize_tma_noalloc(a, dev, sms, st)
                                                      : launch_quantize_generic(a, sms, st);
}

extern "C" MXFP8_API int mxfp8_quantize_padded(const void* x, void* q_dwords, void* s_words, int64_t m, int64_t k,
                                     int64_t s_word_count, int dtype, mxfp8_stream_t stream) {
    if (m < 1 || k < 1 || m % 8 != 0 || k % 256 != 0 || s_word_count < 0) return MXFP8_ERR_SHAPE;
    if (!x || !q_dwords || !s_words) return MXFP8_ERR_NULL_POINTER;
    return mxfp8_quantize(x, dtype, m, k, k, q_dwords, m, k, k, s_words, s_word_count * 4, stream);
}

extern "C" MXFP8_API int mxfp8_dequantize(const void* q, int64_t rows, int64_t cols, int64_t ld_q, const void* s,
                                          int64_t s_bytes, void* out, int out_dtype, int64_t ld_out,
                                          mxfp8_stream_t stream) {
    if (out_dtype != MXFP8_BF16 && out_dtype != MXFP8_FP16 && out_dtype != MXFP8_F32) return MXFP8_ERR_DTYPE;
    if (rows < 0 || cols < 0 || cols % 32 != 0 || ld_q < cols || ld_out < cols || rows > kInt32Max ||
        cols > kInt32Max)
        return MXFP8_ERR_SHAPE;
    if (rows == 0 || cols == 0) return MXFP8_OK;
    if (!q || !s || !out) return MXFP8_ERR_NULL_POINTER;
    if (s_bytes < mxfp8_scale_storage_bytes(rows, cols)) return MXFP8_ERR_SCALE_BUFFER;
    if (!aligned(out, out_dtype == MXFP8_F32 ? 4 : 2)) return MXFP8_ERR_ALIGNMENT;
    DeviceState* dev = nullptr;
    int rc = current_device(&dev);
    if (rc) return rc;
    const StoreWindow ow = make_window(out, ((rows - 1) * ld_out + cols) * (out_dtype == MXFP8_F32 ? 4 : 2));
    return launch_dequantize(static_cast<const uint8_t*>(q), rows, cols, ld_q, static_cast<const uint8_t*>(s), out,
                             out_dtype, ld_out, ow, dev->status, static_cast<cudaStream_t>(stream));
}

extern "C" MXFP8_API int mxfp8_device_status(uint32_t* status_out, int clear) {
    if (!status_out) return MXFP8_ERR_NULL_POINTER;
    *status_out = 0;
    DeviceState* dev = nullptr;
    int rc = current_device(&dev);
    if (rc) return rc;
    return read_status_word(dev->status, status_out, clear, "mxfp8_device_status");
}

extern "C" MXFP8_API int mxfp8_noalloc_status(uint32_t* status_out, int clear) {
    if (!status_out) return MXFP8_ERR_NULL_POINTER;
    *status_out = 0;
    int dev = -1, sms = 0;
    if (int rc = noalloc_device(&dev, &sms)) return rc;
    unsigned int* word = nullptr;
    if (int rc = noalloc_status_word(dev, &word)) return rc;
    return read_status_word(word, status_out, clear, "mxfp8_noalloc_status");
}

extern "C" MXFP8_API int mxfp8_selftest_bounded_wait(uint32_t limit_us, mxfp8_stream_t stream) {
    if (limit_us == 0 || limit_us > 10000000u) return MXFP8_ERR_SHAPE;
    DeviceState* dev = nullptr;
    int rc = current_device(&dev);
    if (rc) return rc;
    return launch_bounded_wait_selftest(dev->status, limit_us, static_cast<cudaStream_t>(stream));
}

#ifdef MXFP8_CHECKED
extern "C" MXFP8_API int mxfp8_checked_window_slack(int64_t bytes) {
    if (bytes < 0 || bytes > (int64_t(1) << 20)) return MXFP8_ERR_SHAPE;
    g_window_slack.store(bytes, std::memory_order_relaxed);
    return MXFP8_OK;
}
#endif

extern "C" MXFP8_API const char* mxfp8_strerror(int status) {
    switch (status) {
        case MXFP8_OK: return "success";
        case MXFP8_ERR_NULL_POINTER: return "a required pointer is NULL";
        case MXFP8_ERR_SHAPE: return "sizes out of range or inconsistent";
        case MXFP8_ERR_DTYPE: return "unsupported dtype";
        case MXFP8_ERR_ALIGNMENT: return "a pointer or stride breaks the alignment contract";
        case MXFP8_ERR_SCALE_BUFFER: return "the scale buffer is smaller than required";
        case MXFP8_ERR_CUDA: return "a CUDA runtime call failed";
        case MXFP8_ERR_TENSOR_MAP: return "the driver rejected a TMA descriptor";
        case MXFP8_ERR_DEVICE: return "no usable sm_100 device is current";
        default: return "unknown status";
    }
}

extern "C" MXFP8_API const char* mxfp8_last_error(void) { return g_last_error.c_str(); }
