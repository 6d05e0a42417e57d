// C ABI entry points (include/llmik.h): argument validation, status codes and
// dispatch to the kernel launchers. Nothing here allocates device memory.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "lik_device.cuh"
#include "lik_internal.h"
#include "llmik.h"

namespace lik {

namespace {

thread_local std::string g_last_error;

lik_status fail(lik_status s, const std::string& msg) {
    g_last_error = msg;
    return s;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace

void set_last_error(const std::string& msg) { g_last_error = msg; }

bool device_info(DeviceInfo& info, std::string& err) {
    static std::mutex mu;
    static DeviceInfo cache[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        err = std::string("cudaGetDevice: ") + cudaGetErrorString(e);
        return false;
    }
    std::lock_guard<std::mutex> lock(mu);
    DeviceInfo& c = cache[dev & 63];
    if (c.sm_count == 0) {
        e = cudaDeviceGetAttribute(&c.sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (e == cudaSuccess)
            e = cudaDeviceGetAttribute(&c.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) {
            c.sm_count = 0;
            err = std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e);
            return false;
        }
    }
    info = c;
    return true;
}

}  // namespace lik

using namespace lik;

namespace {

lik_status check_heads(int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim) {
    if (batch < 0 || n_heads <= 0 || n_kv_heads <= 0)
        return fail(LIK_ERR_INVALID_ARGUMENT, "batch must be >= 0 and head counts > 0");
    if (head_dim != kHeadDim) return fail(LIK_ERR_UNSUPPORTED, "only head_dim=128 supported");
    if (n_heads % n_kv_heads != 0)
        return fail(LIK_ERR_INVALID_ARGUMENT, "n_heads must be a multiple of n_kv_heads");
    if (n_heads > (1 << 20) || n_kv_heads > (1 << 20))
        return fail(LIK_ERR_INVALID_ARGUMENT, "head count out of range");
    return LIK_OK;
}

lik_status check_len(int64_t seqlen, int64_t kv_buf_len) {
    if (seqlen < 1) return fail(LIK_ERR_INVALID_ARGUMENT, "seqlen must be >= 1");
    if (kv_buf_len < seqlen) return fail(LIK_ERR_INVALID_ARGUMENT, "seqlen exceeds allocated cache length");
    if (kv_buf_len > (int64_t{1} << 30))
        return fail(LIK_ERR_INVALID_ARGUMENT, "cache length above 2^30 positions is not supported");
    return LIK_OK;
}

lik_status run_decode(DecodeArgs& a, void* stream) {
    if (a.batch == 0) return LIK_OK;
    if (!a.q || !a.k || !a.v || !a.out) return fail(LIK_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || !aligned16(a.out))
        return fail(LIK_ERR_MISALIGNED, "q, k, v and out must be 16-byte aligned");
    std::string err;
    const lik_status s = launch_decode(a, as_stream(stream), err);
    if (s != LIK_OK) return fail(s, err);
    return LIK_OK;
}

}  // namespace

namespace lik {

// Read the device error word at the start of a decode scratch area after the
// work queued on `stream`; on an error, zero the whole area on `stream` (a
// kernel that gave up may have left unit counters behind) and report it.
lik_status check_error_word(void* scratch, size_t scratch_bytes, cudaStream_t stream, int* device_error) {
    int h = 0;
    cudaError_t e = cudaMemcpyAsync(&h, scratch, sizeof(int), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess && h != 0) e = cudaMemsetAsync(scratch, 0, scratch_bytes, stream);
    if (e != cudaSuccess) return fail(LIK_ERR_CUDA, std::string("error-word check: ") + cudaGetErrorString(e));
    *device_error = h;
    if (h == kDevOk) return LIK_OK;
    if (h == kDevBadBlock)
        return fail(LIK_ERR_DEVICE_BAD_BLOCK, "a paged block-table entry was outside [0, num_blocks)");
    return fail(LIK_ERR_DEVICE_TIMEOUT, "a bounded device-side wait expired");
}

}  // namespace lik

namespace {

lik_status check_quant(const void* x, const void* codes, const void* scale, int64_t batch, int64_t n_kv_heads,
                       int64_t n_tokens, int64_t head_dim, int64_t dst_pos, int64_t dst_buf_len) {
    if (batch < 0 || n_kv_heads <= 0 || n_tokens < 0)
        return fail(LIK_ERR_INVALID_ARGUMENT, "batch and n_tokens must be >= 0, n_kv_heads > 0");
    if (head_dim != kHeadDim) return fail(LIK_ERR_UNSUPPORTED, "only head_dim=128 supported");
    if (dst_pos < 0 || dst_buf_len < dst_pos + n_tokens)
        return fail(LIK_ERR_INVALID_ARGUMENT, "destination [dst_pos, dst_pos + n_tokens) exceeds dst_buf_len");
    if (batch * n_kv_heads * n_tokens == 0) return LIK_OK;
    if (!x || !codes || !scale) return fail(LIK_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(x) || !aligned16(codes))
        return fail(LIK_ERR_MISALIGNED, "x and codes must be 16-byte aligned");
    return LIK_OK;
}

}  // namespace

extern "C" {

int lik_abi_version(void) { return LLMIK_ABI_VERSION; }

const char* lik_status_string(lik_status s) {
    switch (s) {
        case LIK_OK: return "ok";
        case LIK_ERR_INVALID_ARGUMENT: return "invalid argument";
        case LIK_ERR_UNSUPPORTED: return "unsupported configuration";
        case LIK_ERR_MISALIGNED: return "misaligned pointer";
        case LIK_ERR_WORKSPACE: return "workspace missing or too small";
        case LIK_ERR_CUDA: return "CUDA error";
        case LIK_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
        case LIK_ERR_DEVICE_BAD_BLOCK: return "block-table entry out of range";
    }
    return "unknown status";
}

const char* lik_last_error(void) { return g_last_error.c_str(); }

size_t lik_decode_workspace_bytes(int64_t batch, int64_t n_heads, int64_t n_kv_heads) {
    DeviceInfo di;
    std::string err;
    const int sms = device_info(di, err) ? di.sm_count : 256;
    if (n_kv_heads <= 0 || n_heads <= 0 || n_heads % n_kv_heads != 0) return kWsErrBytes;
    return decode_workspace_bytes(batch, n_heads, n_kv_heads, sms);
}

lik_status lik_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
    if (!workspace || workspace_bytes < kWsErrBytes)
        return fail(LIK_ERR_WORKSPACE, "workspace missing or smaller than the minimum");
    const cudaError_t e = cudaMemsetAsync(workspace, 0, workspace_bytes, as_stream(stream));
    if (e != cudaSuccess) return fail(LIK_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
    return LIK_OK;
}

lik_status lik_workspace_check(void* workspace, size_t workspace_bytes, void* stream, int* device_error) {
    if (!workspace || workspace_bytes < kWsErrBytes || !device_error)
        return fail(LIK_ERR_INVALID_ARGUMENT, "workspace and device_error must be given");
    return check_error_word(workspace, workspace_bytes, as_stream(stream), device_error);
}

lik_status lik_decode_attention_f16(const void* q, const void* k, const void* v, void* out, int64_t batch,
                                    int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, int64_t seqlen,
                                    int64_t kv_buf_len, float softmax_scale, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    lik_status s = check_heads(batch, n_heads, n_kv_heads, head_dim);
    if (s == LIK_OK) s = check_len(seqlen, kv_buf_len);
    if (s != LIK_OK) return s;
    DecodeArgs a;
    a.fmt = kF16;
    a.q = q; a.k = k; a.v = v; a.out = out;
    a.batch = batch; a.n_heads = n_heads; a.n_kv_heads = n_kv_heads;
    a.seqlen = seqlen; a.kv_buf_len = kv_buf_len;
    a.softmax_scale = softmax_scale;
    a.workspace = workspace; a.workspace_bytes = workspace_bytes;
    return run_decode(a, stream);
}

lik_status lik_decode_attention_int8(const void* q, const int8_t* k_q, const void* k_scale, const int8_t* v_q,
                                     const void* v_scale, void* out, int64_t batch, int64_t n_heads,
                                     int64_t n_kv_heads, int64_t head_dim, int64_t seqlen, int64_t kv_buf_len,
                                     float softmax_scale, void* workspace, size_t workspace_bytes, void* stream) {
    lik_status s = check_heads(batch, n_heads, n_kv_heads, head_dim);
    if (s == LIK_OK) s = check_len(seqlen, kv_buf_len);
    if (s != LIK_OK) return s;
    if (batch > 0 && (!k_scale || !v_scale)) return fail(LIK_ERR_INVALID_ARGUMENT, "null scale pointer");
    DecodeArgs a;
    a.fmt = kI8;
    a.q = q; a.k = k_q; a.v = v_q; a.out = out;
    a.k_scale = k_scale; a.v_scale = v_scale;
    a.batch = batch; a.n_heads = n_heads; a.n_kv_heads = n_kv_heads;
    a.seqlen = seqlen; a.kv_buf_len = kv_buf_len;
    a.softmax_scale = softmax_scale;
    a.workspace = workspace; a.workspace_bytes = workspace_bytes;
    return run_decode(a, stream);
}

static lik_status decode_int4_common(int fmt, const void* q, const int8_t* k_q, const void* k_scale,
                                     const void* k_zero, const int8_t* v_q, const void* v_scale,
                                     const void* v_zero, void* out, int64_t batch, int64_t n_heads,
                                     int64_t n_kv_heads, int64_t head_dim, int64_t seqlen, int64_t kv_buf_len,
                                     int64_t group_size, int64_t n_groups_buf, float softmax_scale,
                                     void* workspace, size_t workspace_bytes, void* stream) {
    lik_status s = check_heads(batch, n_heads, n_kv_heads, head_dim);
    if (s == LIK_OK) s = check_len(seqlen, kv_buf_len);
    if (s != LIK_OK) return s;
    if (group_size <= 0 || group_size > (1 << 30)) return fail(LIK_ERR_INVALID_ARGUMENT, "group_size must be > 0");
    if ((seqlen + group_size - 1) / group_size > n_groups_buf)
        return fail(LIK_ERR_INVALID_ARGUMENT, "k_scale has fewer groups than ceil(seqlen / group_size)");
    if (batch > 0 && (!k_scale || !v_scale)) return fail(LIK_ERR_INVALID_ARGUMENT, "null scale pointer");
    if (batch > 0 && fmt == kI4Asym && (!k_zero || !v_zero))
        return fail(LIK_ERR_INVALID_ARGUMENT, "null zero-point pointer");
    if (batch > 0 && (!aligned16(k_scale) || (fmt == kI4Asym && !aligned16(k_zero))))
        return fail(LIK_ERR_MISALIGNED, "k_scale / k_zero must be 16-byte aligned");
    DecodeArgs a;
    a.fmt = fmt;
    a.q = q; a.k = k_q; a.v = v_q; a.out = out;
    a.k_scale = k_scale; a.v_scale = v_scale; a.k_zero = k_zero; a.v_zero = v_zero;
    a.batch = batch; a.n_heads = n_heads; a.n_kv_heads = n_kv_heads;
    a.seqlen = seqlen; a.kv_buf_len = kv_buf_len;
    a.group_size = group_size; a.n_groups_buf = n_groups_buf;
    a.softmax_scale = softmax_scale;
    a.workspace = workspace; a.workspace_bytes = workspace_bytes;
    return run_decode(a, stream);
}

lik_status lik_decode_attention_int4(const void* q, const int8_t* k_q, const void* k_scale, const int8_t* v_q,
                                     const void* v_scale, void* out, int64_t batch, int64_t n_heads,
                                     int64_t n_kv_heads, int64_t head_dim, int64_t seqlen, int64_t kv_buf_len,
                                     int64_t group_size, int64_t n_groups_buf, float softmax_scale,
                                     void* workspace, size_t workspace_bytes, void* stream) {
    return decode_int4_common(kI4Sym, q, k_q, k_scale, nullptr, v_q, v_scale, nullptr, out, batch, n_heads,
                              n_kv_heads, head_dim, seqlen, kv_buf_len, group_size, n_groups_buf, softmax_scale,
                              workspace, workspace_bytes, stream);
}

lik_status lik_decode_attention_int4_asym(const void* q, const int8_t* k_q, const void* k_scale,
                                          const void* k_zero, const int8_t* v_q, const void* v_scale,
                                          const void* v_zero, void* out, int64_t batch, int64_t n_heads,
                                          int64_t n_kv_heads, int64_t head_dim, int64_t seqlen,
                                          int64_t kv_buf_len, int64_t group_size, int64_t n_groups_buf,
                                          float softmax_scale, void* workspace, size_t workspace_bytes,
                                          void* stream) {
    return decode_int4_common(kI4Asym, q, k_q, k_scale, k_zero, v_q, v_scale, v_zero, out, batch, n_heads,
                              n_kv_heads, head_dim, seqlen, kv_buf_len, group_size, n_groups_buf, softmax_scale,
                              workspace, workspace_bytes, stream);
}

static lik_status quant_token(int mode, const void* x, int8_t* codes, void* scale, void* zero, int64_t batch,
                              int64_t n_kv_heads, int64_t n_tokens, int64_t head_dim, int64_t dst_pos,
                              int64_t dst_buf_len, void* stream) {
    lik_status s = check_quant(x, codes, scale, batch, n_kv_heads, n_tokens, head_dim, dst_pos, dst_buf_len);
    if (s != LIK_OK || batch * n_tokens == 0) return s;
    if (mode == kTokI4Asym && !zero) return fail(LIK_ERR_INVALID_ARGUMENT, "null zero-point pointer");
    std::string err;
    s = launch_quant_token(mode, x, codes, scale, zero, batch * n_kv_heads, n_tokens, dst_pos, dst_buf_len,
                           as_stream(stream), err);
    return s == LIK_OK ? s : fail(s, err);
}

static lik_status quant_kgroup(bool asym, const void* x, int8_t* packed, void* scale, void* zero, int64_t batch,
                               int64_t n_kv_heads, int64_t n_tokens, int64_t head_dim, int64_t group_size,
                               int64_t dst_pos, int64_t dst_buf_len, int64_t n_groups_buf, void* stream) {
    lik_status s = check_quant(x, packed, scale, batch, n_kv_heads, n_tokens, head_dim, dst_pos, dst_buf_len);
    if (s != LIK_OK) return s;
    if (group_size <= 0 || group_size > (1 << 30)) return fail(LIK_ERR_INVALID_ARGUMENT, "group_size must be > 0");
    if (dst_pos % group_size != 0) return fail(LIK_ERR_INVALID_ARGUMENT, "dst_pos must be a multiple of group_size");
    if (dst_pos / group_size + (n_tokens + group_size - 1) / group_size > n_groups_buf)
        return fail(LIK_ERR_INVALID_ARGUMENT, "scale buffer has too few groups");
    if (batch * n_tokens == 0) return LIK_OK;
    if (asym && !zero) return fail(LIK_ERR_INVALID_ARGUMENT, "null zero-point pointer");
    std::string err;
    s = launch_quant_kgroup(asym, x, packed, scale, zero, batch * n_kv_heads, n_tokens, group_size, dst_pos,
                            dst_buf_len, n_groups_buf, as_stream(stream), err);
    return s == LIK_OK ? s : fail(s, err);
}

lik_status lik_quantize_per_token_int8(const void* x, int8_t* codes, void* scale, int64_t batch, int64_t n_kv_heads,
                                       int64_t n_tokens, int64_t head_dim, int64_t dst_pos, int64_t dst_buf_len,
                                       void* stream) {
    return quant_token(kTokI8, x, codes, scale, nullptr, batch, n_kv_heads, n_tokens, head_dim, dst_pos,
                       dst_buf_len, stream);
}

lik_status lik_quantize_v_per_token_int4(const void* x, int8_t* packed, void* scale, int64_t batch,
                                         int64_t n_kv_heads, int64_t n_tokens, int64_t head_dim, int64_t dst_pos,
                                         int64_t dst_buf_len, void* stream) {
    return quant_token(kTokI4Sym, x, packed, scale, nullptr, batch, n_kv_heads, n_tokens, head_dim, dst_pos,
                       dst_buf_len, stream);
}

lik_status lik_quantize_v_per_token_int4_asym(const void* x, int8_t* packed, void* scale, void* zero,
                                              int64_t batch, int64_t n_kv_heads, int64_t n_tokens,
                                              int64_t head_dim, int64_t dst_pos, int64_t dst_buf_len,
                                              void* stream) {
    return quant_token(kTokI4Asym, x, packed, scale, zero, batch, n_kv_heads, n_tokens, head_dim, dst_pos,
                       dst_buf_len, stream);
}

lik_status lik_quantize_k_per_channel_groupwise_int4(const void* x, int8_t* packed, void* scale, int64_t batch,
                                                     int64_t n_kv_heads, int64_t n_tokens, int64_t head_dim,
                                                     int64_t group_size, int64_t dst_pos, int64_t dst_buf_len,
                                                     int64_t n_groups_buf, void* stream) {
    return quant_kgroup(false, x, packed, scale, nullptr, batch, n_kv_heads, n_tokens, head_dim, group_size,
                        dst_pos, dst_buf_len, n_groups_buf, stream);
}

lik_status lik_quantize_k_per_channel_groupwise_int4_asym(const void* x, int8_t* packed, void* scale, void* zero,
                                                          int64_t batch, int64_t n_kv_heads, int64_t n_tokens,
                                                          int64_t head_dim, int64_t group_size, int64_t dst_pos,
                                                          int64_t dst_buf_len, int64_t n_groups_buf,
                                                          void* stream) {
    return quant_kgroup(true, x, packed, scale, zero, batch, n_kv_heads, n_tokens, head_dim, group_size, dst_pos,
                        dst_buf_len, n_groups_buf, stream);
}

lik_status lik_paged_append(int row_format, const void* x, const int64_t* slot_mapping, int64_t n_tokens,
                            int64_t n_kv_heads, int64_t head_dim, void* cache, void* scale, void* zero,
                            int64_t num_blocks, int64_t block_size, void* stream) {
    if (row_format < 0 || row_format > 3) return fail(LIK_ERR_INVALID_ARGUMENT, "unknown row_format");
    if (n_tokens < 0 || n_kv_heads <= 0 || num_blocks < 0 || block_size <= 0 || block_size > (1 << 20))
        return fail(LIK_ERR_INVALID_ARGUMENT, "need n_tokens >= 0, n_kv_heads > 0, num_blocks >= 0, block_size > 0");
    if (head_dim != kHeadDim) return fail(LIK_ERR_UNSUPPORTED, "only head_dim=128 supported");
    if (n_tokens == 0) return LIK_OK;
    if (!x || !slot_mapping || !cache) return fail(LIK_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (row_format != 0 && !scale) return fail(LIK_ERR_INVALID_ARGUMENT, "null scale pointer");
    if (row_format == 3 && !zero) return fail(LIK_ERR_INVALID_ARGUMENT, "null zero-point pointer");
    if (!aligned16(x) || !aligned16(cache)) return fail(LIK_ERR_MISALIGNED, "x and cache must be 16-byte aligned");
    if (n_tokens > (int64_t{1} << 40) / n_kv_heads) return fail(LIK_ERR_INVALID_ARGUMENT, "too many tokens");
    std::string err;
    const lik_status s = launch_paged_append(row_format, x, slot_mapping, n_tokens, n_kv_heads, cache, scale, zero,
                                             num_blocks, block_size, as_stream(stream), err);
    return s == LIK_OK ? s : fail(s, err);
}

static lik_status dequant_common(int fmt, const void* kq, const void* ks, const void* kz, const void* vq,
                                 const void* vs, const void* vz, void* ko, void* vo, int64_t batch, int64_t n_kv_heads,
                                 int64_t seqlen, int64_t kv_buf_len, int64_t head_dim, int64_t group_size,
                                 int64_t n_groups_buf, void* stream) {
    if (batch < 0 || n_kv_heads <= 0 || seqlen < 0 || kv_buf_len < seqlen)
        return fail(LIK_ERR_INVALID_ARGUMENT, "need batch >= 0, n_kv_heads > 0, 0 <= seqlen <= kv_buf_len");
    if (head_dim != kHeadDim) return fail(LIK_ERR_UNSUPPORTED, "only head_dim=128 supported");
    if (batch * seqlen == 0) return LIK_OK;
    if (!kq || !ks || !vq || !vs || !ko || !vo || (fmt == 2 && (!kz || !vz)))
        return fail(LIK_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(kq) || !aligned16(vq) || !aligned16(ko) || !aligned16(vo))
        return fail(LIK_ERR_MISALIGNED, "codes and outputs must be 16-byte aligned");
    if (fmt != 0) {
        if (group_size <= 0) return fail(LIK_ERR_INVALID_ARGUMENT, "group_size must be > 0");
        if ((seqlen + group_size - 1) / group_size > n_groups_buf)
            return fail(LIK_ERR_INVALID_ARGUMENT, "k_scale has fewer groups than ceil(seqlen / group_size)");
    }
    std::string err;
    const lik_status s = launch_dequant(fmt, kq, ks, kz, vq, vs, vz, ko, vo, batch * n_kv_heads, seqlen, kv_buf_len,
                                        group_size, n_groups_buf, as_stream(stream), err);
    return s == LIK_OK ? s : fail(s, err);
}

lik_status lik_dequantize_int8(const int8_t* k_q, const void* k_scale, const int8_t* v_q, const void* v_scale,
                               void* k_out, void* v_out, int64_t batch, int64_t n_kv_heads, int64_t seqlen,
                               int64_t kv_buf_len, int64_t head_dim, void* stream) {
    return dequant_common(0, k_q, k_scale, nullptr, v_q, v_scale, nullptr, k_out, v_out, batch, n_kv_heads, seqlen,
                          kv_buf_len, head_dim, 0, 0, stream);
}

lik_status lik_dequantize_int4(const int8_t* k_q, const void* k_scale, const int8_t* v_q, const void* v_scale,
                               void* k_out, void* v_out, int64_t batch, int64_t n_kv_heads, int64_t seqlen,
                               int64_t kv_buf_len, int64_t head_dim, int64_t group_size, int64_t n_groups_buf,
                               void* stream) {
    return dequant_common(1, k_q, k_scale, nullptr, v_q, v_scale, nullptr, k_out, v_out, batch, n_kv_heads, seqlen,
                          kv_buf_len, head_dim, group_size, n_groups_buf, stream);
}

lik_status lik_dequantize_int4_asym(const int8_t* k_q, const void* k_scale, const void* k_zero, const int8_t* v_q,
                                    const void* v_scale, const void* v_zero, void* k_out, void* v_out, int64_t batch,
                                    int64_t n_kv_heads, int64_t seqlen, int64_t kv_buf_len, int64_t head_dim,
                                    int64_t group_size, int64_t n_groups_buf, void* stream) {
    return dequant_common(2, k_q, k_scale, k_zero, v_q, v_scale, v_zero, k_out, v_out, batch, n_kv_heads, seqlen,
                          kv_buf_len, head_dim, group_size, n_groups_buf, stream);
}

lik_status lik_decode_attention_paged(int kv_format, const void* q, const void* k_cache, const void* v_cache,
                                      const void* k_scale, const void* v_scale, const void* k_zero, const void* v_zero,
                                      const int32_t* block_tables, const int32_t* context_lens, void* out,
                                      int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                                      int64_t num_blocks, int64_t block_size, int64_t max_blocks_per_seq,
                                      int64_t max_context_len,
                                      int64_t group_size, float softmax_scale, void* workspace,
                                      size_t workspace_bytes, void* stream) {
    lik_status s = check_heads(batch, n_heads, n_kv_heads, head_dim);
    if (s != LIK_OK) return s;
    if (kv_format < kF16 || kv_format > kI4Asym) return fail(LIK_ERR_INVALID_ARGUMENT, "unknown kv_format");
    if (block_size <= 0 || block_size % 16 != 0 || block_size > (1 << 20))
        return fail(LIK_ERR_INVALID_ARGUMENT, "block_size must be a positive multiple of 16");
    if (num_blocks < 1) return fail(LIK_ERR_INVALID_ARGUMENT, "num_blocks must be >= 1");
    if (max_blocks_per_seq <= 0 || max_context_len < 1 || max_context_len > block_size * max_blocks_per_seq ||
        max_context_len > (int64_t{1} << 30))
        return fail(LIK_ERR_INVALID_ARGUMENT, "need 1 <= max_context_len <= block_size * max_blocks_per_seq");
    if (batch == 0) return LIK_OK;
    if (!block_tables || !context_lens) return fail(LIK_ERR_INVALID_ARGUMENT, "null block table or lengths");
    const bool quant = kv_format != kF16;
    const bool int4 = kv_format == kI4Sym || kv_format == kI4Asym;
    if (quant && (!k_scale || !v_scale)) return fail(LIK_ERR_INVALID_ARGUMENT, "null scale pointer");
    if (kv_format == kI4Asym && (!k_zero || !v_zero)) return fail(LIK_ERR_INVALID_ARGUMENT, "null zero-point pointer");
    if (quant && (!aligned16(k_scale) || !aligned16(v_scale) ||
                  (kv_format == kI4Asym && (!aligned16(k_zero) || !aligned16(v_zero)))))
        return fail(LIK_ERR_MISALIGNED, "scale / zero pointers must be 16-byte aligned");
    if (int4 && (group_size <= 0 || block_size % group_size != 0))
        return fail(LIK_ERR_INVALID_ARGUMENT, "group_size must divide block_size");
    DecodeArgs a;
    a.fmt = kv_format;
    a.q = q; a.k = k_cache; a.v = v_cache; a.out = out;
    a.k_scale = k_scale; a.v_scale = v_scale; a.k_zero = k_zero; a.v_zero = v_zero;
    a.batch = batch; a.n_heads = n_heads; a.n_kv_heads = n_kv_heads;
    a.seqlen = max_context_len; a.kv_buf_len = max_context_len;
    a.group_size = int4 ? group_size : 0;
    a.n_groups_buf = int4 ? (max_context_len + group_size - 1) / group_size : 0;
    a.block_tables = block_tables; a.context_lens = context_lens;
    a.block_size = block_size; a.max_blocks = max_blocks_per_seq; a.num_blocks = num_blocks;
    a.softmax_scale = softmax_scale;
    a.workspace = workspace; a.workspace_bytes = workspace_bytes;
    return run_decode(a, stream);
}

}  // extern "C"
