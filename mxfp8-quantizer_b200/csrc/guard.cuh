// guard.cuh -- global stores of every kernel go through gstore() (or gstore_plain()).
//
// Product build: gstore() is the streaming store itself (st.global.cs).
// Checked build (MXFP8_CHECKED, libmxfp8_checked.so): a store happens only
// when it lies entirely inside the window [lo, hi) of the output it belongs
// to and is aligned to its own size; any other store is skipped and sets
// kErrBoundsStore in the device status word.  It never traps, so the checked
// build stands in for a memory checker on a pool where none may run: the test
// suite runs its layout battery through both builds and requires identical
// bytes and a clean status word.
#pragma once
#include <stdint.h>

namespace mxfp8 {

constexpr unsigned kErrBoundsStore = 16u;  // status bit, checked build only

struct StoreWindow {
    uint8_t* lo;
    uint8_t* hi;  // one past the last byte the kernel may write
};

template <typename T>
__device__ __forceinline__ void gstore(T* p, T v, const StoreWindow& w, unsigned int* status) {
#ifdef MXFP8_CHECKED
    const uint8_t* a = reinterpret_cast<const uint8_t*>(p);
    if (a < w.lo || a + sizeof(T) > w.hi || (reinterpret_cast<uintptr_t>(p) & (sizeof(T) - 1)) != 0) {
        if (status) atomicOr(status, kErrBoundsStore);
        return;
    }
#else
    (void)w;
    (void)status;
#endif
    __stcs(p, v);
}

// Same guard, plain (write-back) store: for element-wise fallback paths.  In
// the dequantize kernel, streaming stores in its unaligned-row fallback cost
// 10 % on the aligned path it never leaves (6.25 -> 5.63 TB/s at 8192^2).
template <typename T>
__device__ __forceinline__ void gstore_plain(T* p, T v, const StoreWindow& w, unsigned int* status) {
#ifdef MXFP8_CHECKED
    const uint8_t* a = reinterpret_cast<const uint8_t*>(p);
    if (a < w.lo || a + sizeof(T) > w.hi || (reinterpret_cast<uintptr_t>(p) & (sizeof(T) - 1)) != 0) {
        if (status) atomicOr(status, kErrBoundsStore);
        return;
    }
#else
    (void)w;
    (void)status;
#endif
    *p = v;
}

}  // namespace mxfp8
