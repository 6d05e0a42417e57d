// Bounded-wait self test (include/llmik.h: lik_selftest_bounded_wait).
//
// A one-warp kernel waits on a shared-memory mbarrier that nothing ever
// arrives at, using the same bounded poll loop as the decode kernels, and
// records the error code it would report instead of hanging. Exercises the
// failure path on a real GPU without faulting, trapping or hanging it.
#include <cuda_runtime.h>

#include <string>

#include "lik_device.cuh"
#include "lik_internal.h"
#include "llmik.h"

namespace lik_selftest {

__device__ int g_err;

__global__ void wait_kernel(uint32_t polls) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        lik::mbar_init(&bar, 1);
        lik::fence_barrier_init();
    }
    __syncwarp();
    const bool ok = lik::mbar_wait_bounded(&bar, 0, polls);
    if (threadIdx.x == 0) g_err = ok ? lik::kDevOk : lik::kDevWaitTimeout;
}

}  // namespace lik_selftest

extern "C" lik_status lik_selftest_bounded_wait(int64_t polls, int* device_error, void* stream) {
    if (polls < 1 || polls > (int64_t{1} << 24) || !device_error) {
        lik::set_last_error("polls must be in [1, 2^24] and device_error given");
        return LIK_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    lik_selftest::wait_kernel<<<1, 32, 0, s>>>(static_cast<uint32_t>(polls));
    cudaError_t e = cudaGetLastError();
    int h = -1;
    if (e == cudaSuccess) e = cudaMemcpyFromSymbolAsync(&h, lik_selftest::g_err, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        lik::set_last_error(std::string("selftest: ") + cudaGetErrorString(e));
        return LIK_ERR_CUDA;
    }
    *device_error = h;
    if (h != lik::kDevOk) {
        lik::set_last_error("a bounded device-side wait expired");
        return LIK_ERR_DEVICE_TIMEOUT;
    }
    return LIK_OK;
}
