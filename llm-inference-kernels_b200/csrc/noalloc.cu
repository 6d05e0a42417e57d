// Allocation-free fp16 decode attention entry point.
//
// Some callers cannot allocate device memory at the time they launch
// attention: code running inside a memory pool that is already carved up, a
// runtime whose allocator must not be re-entered from the launch path, or a
// host language binding that only holds raw pointers handed to it and has no
// way to call cudaMalloc. For them this file keeps the split-sequence scratch
// (partial results, per-unit completion counters and the device error word)
// in a fixed array that lives inside the library image on every GPU that loads
// it, so the caller passes only inputs and outputs.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "lik_internal.h"
#include "llmik.h"

namespace lik {
namespace {

// Upper bound of the scratch this entry point can use: 4 MiB per device,
// held until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t{4} << 20;

// Zero-initialised at module load; every call leaves the counters zero again.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch for each device ordinal, found once per
// device (host code cannot use the symbol itself: on the host it names a
// stand-in, not device memory). The array needs no clearing here: a
// __device__ array is zero when the module loads, and every call leaves its
// counters zero again (lik_decode_noalloc_check resets it after an error).
void* scratch_address(std::string& err) {
    static std::mutex mu;
    static void* addr[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        err = std::string("cudaGetDevice: ") + cudaGetErrorString(e);
        return nullptr;
    }
    if (dev < 0 || dev >= 64) {
        err = "device ordinal out of range";
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            err = std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e);
            return nullptr;
        }
        addr[dev] = p;
    }
    return addr[dev];
}

}  // namespace

void* noalloc_scratch(size_t* bytes, std::string& err) {
    *bytes = kNoAllocScratchBytes;
    return scratch_address(err);
}

}  // namespace lik

extern "C" lik_status lik_decode_attention_f16_noalloc(const void* q, const void* k, const void* v, void* out,
                                                        int64_t batch, int64_t n_heads, int64_t n_kv_heads,
                                                        int64_t head_dim, int64_t seqlen, int64_t kv_buf_len,
                                                        float softmax_scale, void* stream) {
    using namespace lik;
    if (n_kv_heads > 0 && n_heads > 0 && batch > 0) {
        const size_t need = lik_decode_workspace_bytes(batch, n_heads, n_kv_heads);
        if (need > kNoAllocScratchBytes) {
            // Validation of other arguments is left to the regular entry point;
            // this is the one limit specific to the fixed scratch array.
            set_last_error("lik_decode_attention_f16_noalloc: this shape needs " + std::to_string(need) +
                           " bytes of scratch, above the fixed 4 MiB (4194304 bytes); use "
                           "lik_decode_attention_f16 with a caller-owned workspace");
            return LIK_ERR_WORKSPACE;
        }
    }
    std::string err;
    void* ws = scratch_address(err);
    if (ws == nullptr) {
        set_last_error(err);
        return LIK_ERR_CUDA;
    }
    return lik_decode_attention_f16(q, k, v, out, batch, n_heads, n_kv_heads, head_dim, seqlen, kv_buf_len,
                                    softmax_scale, ws, kNoAllocScratchBytes, stream);
}

extern "C" lik_status lik_decode_noalloc_check(void* stream, int* device_error) {
    using namespace lik;
    if (device_error == nullptr) {
        set_last_error("lik_decode_noalloc_check: device_error must be given");
        return LIK_ERR_INVALID_ARGUMENT;
    }
    std::string err;
    void* ws = scratch_address(err);
    if (ws == nullptr) {
        set_last_error(err);
        return LIK_ERR_CUDA;
    }
    return check_error_word(ws, kNoAllocScratchBytes, static_cast<cudaStream_t>(stream), device_error);
}
