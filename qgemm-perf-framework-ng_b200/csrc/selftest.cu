// selftest.cu -- pfng_b200_selftest_wait: exercises the bounded-wait and
// error-reporting machinery every pipelined kernel of the library relies on,
// so that a test can make a wait run out on purpose without a fault.
//
// One CTA of two warps shares one mbarrier: warp 0 (the producer) arrives on
// it once, unless told to skip that arrive; warp 1 (the consumer) waits for
// the phase with mbar_wait_n -- the helper behind every kernel's waits --
// limited to `attempts` tries of at most ~1 us each.  A wait that gives up
// records kErrWaitFull in the library's device error word and returns, like
// a pipelined kernel's consumer does, and the kernel ends normally: the
// context stays usable and pfng_b200_check_kernel_error() reports
// PFNG_B200_ERR_KERNEL_TIMEOUT (then clears the word).
#include "pfng_b200.h"
#include "pfng_common.cuh"
#include "pfng_internal.h"

namespace pfng {
namespace {

__global__ void __launch_bounds__(64) selftest_wait_kernel(uint32_t attempts, int skip_arrive, int *err,
                                                           int *waited) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    if (warp == 0) {
        if (threadIdx.x == 0 && !skip_arrive) mbar_arrive(&bar);
    } else if (threadIdx.x == 32) {
        const bool ok = mbar_wait_n(&bar, 0, err, kErrWaitFull, attempts);
        if (waited) *waited = ok ? 1 : 0;
    }
}

}  // namespace
}  // namespace pfng

using namespace pfng;

extern "C" int pfng_b200_selftest_wait(unsigned attempts, int skip_arrive, int *completed, void *stream) {
    if (attempts == 0) return PFNG_B200_ERR_INVALID_ARGUMENT;
    int *err = device_error_word();
    if (!err) return PFNG_B200_ERR_DEVICE;
    selftest_wait_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(attempts, skip_arrive, err, completed);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? PFNG_B200_OK : PFNG_B200_ERR_CUDA_BASE - static_cast<int>(e);
}
