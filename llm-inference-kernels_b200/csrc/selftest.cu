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

// The same wait, and on expiry what a decode kernel that gave up leaves in
// its scratch: the timeout code in the error word and a unit counter that is
// not back to zero.
__global__ void leave_timeout_kernel(uint32_t polls, int* err_word, unsigned* counter0) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        lik::mbar_init(&bar, 1);
        lik::fence_barrier_init();
    }
    __syncwarp();
    const bool ok = lik::mbar_wait_bounded(&bar, 0, polls);
    if (threadIdx.x == 0 && !ok) {
        atomicExch(err_word, lik::kDevWaitTimeout);
        atomicAdd(counter0, 1u);
    }
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

extern "C" lik_status lik_selftest_leave_timeout(int64_t polls, void* workspace, size_t workspace_bytes,
                                                 void* stream) {
    if (polls < 1 || polls > (int64_t{1} << 24)) {
        lik::set_last_error("polls must be in [1, 2^24]");
        return LIK_ERR_INVALID_ARGUMENT;
    }
    std::string err;
    lik::DeviceInfo di;
    if (!lik::device_info(di, err)) {
        lik::set_last_error(err);
        return LIK_ERR_CUDA;
    }
    if (workspace == nullptr) {
        workspace = lik::noalloc_scratch(&workspace_bytes, err);
        if (workspace == nullptr) {
            lik::set_last_error(err);
            return LIK_ERR_CUDA;
        }
    }
    const size_t coff = lik::decode_counter_offset(di.sm_count);
    if (workspace_bytes < coff + sizeof(unsigned)) {
        lik::set_last_error("workspace smaller than one decode workspace");
        return LIK_ERR_WORKSPACE;
    }
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    lik_selftest::leave_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<uint32_t>(polls), reinterpret_cast<int*>(ws), reinterpret_cast<unsigned*>(ws + coff));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        lik::set_last_error(std::string("selftest: ") + cudaGetErrorString(e));
        return LIK_ERR_CUDA;
    }
    return LIK_OK;
}
