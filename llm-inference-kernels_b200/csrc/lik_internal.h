// Internal host-side interface between the C ABI (cabi.cu) and the kernel
// launchers (decode.cu, quantize.cu). Not installed; the public surface is
// include/llmik.h.
#pragma once

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <string>

#include "llmik.h"

namespace lik {

enum KvFormat : int { kF16 = 0, kI8 = 1, kI4Sym = 2, kI4Asym = 3 };

struct DecodeArgs {
    int fmt = kF16;
    const void* q = nullptr;
    const void* k = nullptr;
    const void* v = nullptr;
    const void* k_scale = nullptr;
    const void* v_scale = nullptr;
    const void* k_zero = nullptr;
    const void* v_zero = nullptr;
    void* out = nullptr;
    int64_t batch = 0, n_heads = 0, n_kv_heads = 0;
    int64_t seqlen = 0, kv_buf_len = 0;
    int64_t group_size = 0, n_groups_buf = 0;
    float softmax_scale = 0.f;
    // paged KV: seqlen is the maximum context length, kv_buf_len unused
    const int* block_tables = nullptr;
    const int* context_lens = nullptr;
    int64_t block_size = 0, max_blocks = 0, num_blocks = 0;
    void* workspace = nullptr;
    size_t workspace_bytes = 0;
};

// Device properties cached per device ordinal.
struct DeviceInfo {
    int sm_count = 0;
    int max_smem_optin = 0;
};
bool device_info(DeviceInfo& info, std::string& err);

// Record the calling thread's lik_last_error() text.
void set_last_error(const std::string& msg);

// Read (and on error reset) the device error word of a decode scratch area.
lik_status check_error_word(void* scratch, size_t scratch_bytes, cudaStream_t stream, int* device_error);

// Heads handled together by one work unit (a divisor of the GQA group size).
int heads_per_unit(int64_t group, int fmt, bool mma);
// Whether the decode of this KV format / K group size runs on the tensor pipe.
bool decode_uses_mma(int fmt, int64_t group_size);

size_t decode_workspace_bytes(int64_t batch, int64_t n_heads, int64_t n_kv_heads, int sm_count);
// Byte offset of the per-unit completion counters inside a decode workspace.
size_t decode_counter_offset(int sm_count);

// Device address and size of the allocation-free path's fixed scratch on the
// current device (looked up once per device; nullptr + err on failure).
void* noalloc_scratch(size_t* bytes, std::string& err);

lik_status launch_decode(const DecodeArgs& a, cudaStream_t stream, std::string& err);

enum QuantTokenMode : int { kTokI8 = 0, kTokI4Sym = 1, kTokI4Asym = 2 };

lik_status launch_quant_token(int mode, const void* x, void* codes, void* scale, void* zero,
                              int64_t n_slabs, int64_t n_tokens, int64_t dst_pos,
                              int64_t dst_buf_len, cudaStream_t stream, std::string& err);

lik_status launch_quant_kgroup(bool asym, const void* x, void* codes, void* scale, void* zero,
                               int64_t n_slabs, int64_t n_tokens, int64_t group_size,
                               int64_t dst_pos, int64_t dst_buf_len, int64_t n_groups_buf,
                               cudaStream_t stream, std::string& err);

lik_status launch_paged_append(int row_format, const void* x, const int64_t* slots, int64_t n_tokens,
                               int64_t n_heads, void* cache, void* scale, void* zero, int64_t num_blocks,
                               int64_t block_size, cudaStream_t stream, std::string& err);
lik_status launch_dequant(int fmt, const void* kq, const void* ks, const void* kz, const void* vq, const void* vs,
                          const void* vz, void* kout, void* vout, int64_t n_slabs, int64_t seqlen,
                          int64_t kv_buf_len, int64_t group_size, int64_t n_groups_buf, cudaStream_t stream,
                          std::string& err);

constexpr int kHeadDim = 128;

// Workspace layout shared by host and device code.
constexpr size_t kWsErrBytes = 256;       // device error word (+ padding)
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace lik
