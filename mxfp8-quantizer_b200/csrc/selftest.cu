// selftest.cu -- exercises the bounded-wait failure path on the GPU without
// faulting it: one CTA waits on an mbarrier that nothing will ever complete
// (mbar_wait_bounded, the same routine the quantizer's pipeline uses), gives
// up after `limit_ns`, records the timeout in the device status word and
// returns.  The context stays usable.
#include <cuda_runtime.h>

#include "../../include/mxfp8.h"
#include "launch.h"
#include "ptx.cuh"

namespace mxfp8 {

constexpr unsigned kErrSelfTest = 8u;

__global__ void bounded_wait_selftest_kernel(unsigned int* status, uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    const uint32_t addr = smem_u32(&bar);
    if (threadIdx.x == 0) {
        mbar_init(addr, 1);  // expects one arrival that never comes
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0 && !mbar_wait_bounded(addr, 0, limit_ns)) {
        if (status) atomicOr(status, kErrSelfTest);
    }
}

int launch_bounded_wait_selftest(unsigned int* status, uint32_t limit_us, cudaStream_t stream) {
    bounded_wait_selftest_kernel<<<1, 32, 0, stream>>>(status, (uint64_t)limit_us * 1000ull);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error("bounded_wait_selftest_kernel launch", (int)e);
        return MXFP8_ERR_CUDA;
    }
    return MXFP8_OK;
}

}  // namespace mxfp8
