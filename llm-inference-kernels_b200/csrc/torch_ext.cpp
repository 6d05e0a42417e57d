// `llmik_cuda._C`: the PyTorch op surface of the reference extension
// (bindings/extension.cpp:476-494), rebuilt on the C ABI of
// libllmik_b200.so (include/llmik.h).
//
// This layer only validates tensors (the reference's TORCH_CHECK
// preconditions, plus head_dim == 128 and n_heads % n_kv_heads == 0 on every
// op), allocates outputs with the caching allocator, picks the current stream
// and turns a lik_status into a Python RuntimeError. All arithmetic is in the
// CUDA library; there is no CPU path.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>
#include <tuple>

#include "llmik.h"

namespace {

void ok_or_throw(lik_status s, const char* op) {
    TORCH_CHECK(s == LIK_OK, op, ": ", lik_status_string(s), ": ", lik_last_error());
}

void* cur_stream() { return static_cast<void*>(at::cuda::getCurrentCUDAStream().stream()); }

// One zero-initialised workspace per (device, stream), grown on demand. Kept
// alive for the life of the process so repeated decode steps (and CUDA-graph
// replays) reuse it; the kernels leave it zeroed after every call.
std::mutex& ws_mutex() {
    static std::mutex mu;
    return mu;
}
std::map<std::pair<int, void*>, at::Tensor>& ws_cache() {
    static std::map<std::pair<int, void*>, at::Tensor> cache;
    return cache;
}

at::Tensor& workspace(const at::Tensor& like, size_t bytes) {
    std::lock_guard<std::mutex> lock(ws_mutex());
    auto key = std::make_pair(static_cast<int>(like.get_device()), cur_stream());
    at::Tensor& t = ws_cache()[key];
    if (!t.defined() || static_cast<size_t>(t.numel()) < bytes) {
        t = torch::empty({static_cast<int64_t>(bytes)}, like.options().dtype(torch::kUInt8));
        ok_or_throw(lik_workspace_init(t.data_ptr(), bytes, cur_stream()), "workspace init");
    }
    return t;
}

// Failure detection for the torch ops: read the device error word of every
// cached workspace of the current device (synchronizing each workspace's
// stream). A kernel whose bounded wait expired, or that met an out-of-range
// block-table entry, left a code there and possibly unit counters that are
// not zero; lik_workspace_check zeroes such a workspace again, and this op
// then raises, so the failed step is reported and the next one starts clean.
void check_device_errors() {
    const int dev = static_cast<int>(c10::cuda::current_device());
    std::string msg;
    std::lock_guard<std::mutex> lock(ws_mutex());
    for (auto& kv : ws_cache()) {
        if (kv.first.first != dev || !kv.second.defined()) continue;
        int code = 0;
        const lik_status st =
            lik_workspace_check(kv.second.data_ptr(), kv.second.numel(), kv.first.second, &code);
        if (st != LIK_OK) msg += std::string(msg.empty() ? "" : "; ") + lik_status_string(st) + ": " + lik_last_error();
    }
    TORCH_CHECK(msg.empty(), "decode kernel reported a device-side error (workspace reset): ", msg);
}

// Test hook for check_device_errors: leave, in the current stream's
// workspace, what a decode kernel whose bounded wait expired leaves (a
// one-warp kernel whose own bounded wait runs out; no GPU fault involved).
void selftest_leave_timeout() {
    const auto like = torch::empty({1}, torch::TensorOptions().device(torch::kCUDA, c10::cuda::current_device()));
    at::Tensor& ws = workspace(like, lik_decode_workspace_bytes(1, 1, 1));
    ok_or_throw(lik_selftest_leave_timeout(64, ws.data_ptr(), ws.numel(), cur_stream()), "selftest_leave_timeout");
}

void check_cuda(const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

void check_q(const at::Tensor& q) {
    check_cuda(q, "q");
    TORCH_CHECK(q.scalar_type() == torch::kHalf, "q must be fp16");
    TORCH_CHECK(q.dim() == 3, "q must be [batch, n_heads, head_dim]");
    TORCH_CHECK(q.size(2) == 128, "only head_dim=128 supported");
}

// Length of the buffer a [batch, heads, seq, inner...] tensor is a prefix of:
// the tensor is either contiguous or a view t = buffer[:, :, :n] of a
// contiguous [batch, heads, buf, inner...] buffer (the layout a preallocated
// cache hands out), so the rows of one (batch, head) start buf rows apart.
int64_t seq_buffer(const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.dim() >= 3, name, " must have [batch, heads, seq, ...] dimensions");
    const char* msg = " must be contiguous or a sequence prefix of a contiguous buffer";
    int64_t inner = 1;
    for (int64_t d = t.dim() - 1; d >= 3; --d) {
        TORCH_CHECK(t.size(d) == 1 || t.stride(d) == inner, name, msg);
        inner *= t.size(d);
    }
    TORCH_CHECK(t.size(2) <= 1 || t.stride(2) == inner, name, msg);
    int64_t buf = t.size(2);
    if (t.size(1) > 1) {
        TORCH_CHECK(t.stride(1) % inner == 0 && t.stride(1) / inner >= t.size(2), name, msg);
        buf = t.stride(1) / inner;
    } else if (t.size(0) > 1) {
        TORCH_CHECK(t.stride(0) % inner == 0 && t.stride(0) / inner >= t.size(2), name, msg);
        buf = t.stride(0) / inner;
    }
    TORCH_CHECK(t.size(0) <= 1 || t.size(1) <= 1 || t.stride(0) == t.size(1) * buf * inner, name, msg);
    return buf;
}

// The common buffer length of a call's per-position tensors (codes and
// per-token scales share one row index).
int64_t kv_buffer(std::initializer_list<std::pair<const at::Tensor*, const char*>> ts) {
    int64_t buf = -1;
    for (const auto& t : ts) {
        const int64_t b = seq_buffer(*t.first, t.second);
        TORCH_CHECK(buf < 0 || b == buf, t.second, " is a prefix of a buffer of another length than the K codes");
        buf = b;
    }
    return buf;
}

void check_kv4(const at::Tensor& t, const char* name, at::ScalarType dt, int64_t last, bool view_ok = false) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(view_ok || t.is_contiguous(), name, " must be contiguous");
    TORCH_CHECK(t.scalar_type() == dt, name, " has the wrong dtype");
    TORCH_CHECK(t.dim() == 4, name, " must be [batch, n_kv_heads, seqlen, ", last, "]");
    TORCH_CHECK(t.size(3) == last, name, " last dim must be ", last);
}

void check_same_device(const at::Tensor& a, const at::Tensor& b) {
    TORCH_CHECK(a.device() == b.device(), "all tensors must be on the same device");
}

int64_t live_len(int64_t seqlen, int64_t buf) {
    const int64_t s = seqlen > 0 ? seqlen : buf;
    TORCH_CHECK(s <= buf, "seqlen exceeds allocated cache length");
    return s;
}

void check_heads(const at::Tensor& q, const at::Tensor& k) {
    TORCH_CHECK(k.size(0) == q.size(0), "batch mismatch between q and the KV cache");
    TORCH_CHECK(k.size(1) > 0 && q.size(1) % k.size(1) == 0, "n_heads must be a multiple of n_kv_heads");
}

void check_tok_scale(const at::Tensor& s, const at::Tensor& codes, const char* name, bool view_ok = false) {
    TORCH_CHECK(s.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(view_ok || s.is_contiguous(), name, " must be contiguous");
    TORCH_CHECK(s.scalar_type() == torch::kHalf, name, " must be fp16");
    TORCH_CHECK(s.dim() == 3 && s.size(0) == codes.size(0) && s.size(1) == codes.size(1) &&
                    s.size(2) == codes.size(2),
                name, " must be [batch, n_kv_heads, seqlen]");
}

void check_group_scale(const at::Tensor& s, const at::Tensor& codes, const char* name, bool view_ok = false) {
    TORCH_CHECK(s.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(view_ok || s.is_contiguous(), name, " must be contiguous");
    TORCH_CHECK(s.scalar_type() == torch::kHalf, name, " must be fp16");
    TORCH_CHECK(s.dim() == 4 && s.size(0) == codes.size(0) && s.size(1) == codes.size(1) && s.size(3) == 128,
                name, " must be [batch, n_kv_heads, n_groups, head_dim]");
}

// ---------------------------------------------------------------- attention

torch::Tensor decode_attention(torch::Tensor q, torch::Tensor k, torch::Tensor v, double softmax_scale,
                               int64_t seqlen) {
    check_q(q);
    check_kv4(k, "k", torch::kHalf, 128, true);
    check_kv4(v, "v", torch::kHalf, 128, true);
    TORCH_CHECK(k.sizes() == v.sizes(), "k and v must have the same shape");
    check_same_device(q, k);
    check_same_device(q, v);
    check_heads(q, k);
    const c10::cuda::CUDAGuard guard(q.device());
    const int64_t buf = kv_buffer({{&k, "k"}, {&v, "v"}});
    const int64_t s = live_len(seqlen, k.size(2));
    auto out = torch::empty_like(q);
    const size_t wb = lik_decode_workspace_bytes(q.size(0), q.size(1), k.size(1));
    at::Tensor& ws = workspace(q, wb);
    ok_or_throw(lik_decode_attention_f16(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), q.size(0),
                                         q.size(1), k.size(1), q.size(2), s, buf,
                                         static_cast<float>(softmax_scale), ws.data_ptr(), ws.numel(),
                                         cur_stream()),
                "decode_attention");
    return out;
}

torch::Tensor decode_attention_v3(torch::Tensor q, torch::Tensor k, torch::Tensor v, double softmax_scale) {
    // The reference's single-warp v3 kernel has no separate implementation
    // here: the same split-sequence kernel serves every length.
    return decode_attention(q, k, v, softmax_scale, -1);
}

torch::Tensor decode_attention_int8(torch::Tensor q, torch::Tensor k_q, torch::Tensor k_scale, torch::Tensor v_q,
                                    torch::Tensor v_scale, double softmax_scale, int64_t seqlen) {
    check_q(q);
    check_kv4(k_q, "k_q", torch::kInt8, 128, true);
    check_kv4(v_q, "v_q", torch::kInt8, 128, true);
    TORCH_CHECK(k_q.sizes() == v_q.sizes(), "k_q and v_q must have the same shape");
    check_tok_scale(k_scale, k_q, "k_scale", true);
    check_tok_scale(v_scale, v_q, "v_scale", true);
    for (auto* t : {&k_q, &v_q, &k_scale, &v_scale}) check_same_device(q, *t);
    check_heads(q, k_q);
    const c10::cuda::CUDAGuard guard(q.device());
    const int64_t buf = kv_buffer({{&k_q, "k_q"}, {&v_q, "v_q"}, {&k_scale, "k_scale"}, {&v_scale, "v_scale"}});
    const int64_t s = live_len(seqlen, k_q.size(2));
    auto out = torch::empty_like(q);
    at::Tensor& ws = workspace(q, lik_decode_workspace_bytes(q.size(0), q.size(1), k_q.size(1)));
    ok_or_throw(lik_decode_attention_int8(q.data_ptr(), k_q.data_ptr<int8_t>(), k_scale.data_ptr(),
                                          v_q.data_ptr<int8_t>(), v_scale.data_ptr(), out.data_ptr(), q.size(0),
                                          q.size(1), k_q.size(1), q.size(2), s, buf,
                                          static_cast<float>(softmax_scale), ws.data_ptr(), ws.numel(),
                                          cur_stream()),
                "decode_attention_int8");
    return out;
}

torch::Tensor decode_attention_int4(torch::Tensor q, torch::Tensor k_q, torch::Tensor k_scale, torch::Tensor v_q,
                                    torch::Tensor v_scale, int64_t group_size, double softmax_scale,
                                    int64_t seqlen) {
    check_q(q);
    check_kv4(k_q, "k_q", torch::kInt8, 64, true);
    check_kv4(v_q, "v_q", torch::kInt8, 64, true);
    TORCH_CHECK(k_q.sizes() == v_q.sizes(), "k_q and v_q must have the same shape");
    check_group_scale(k_scale, k_q, "k_scale", true);
    check_tok_scale(v_scale, v_q, "v_scale", true);
    TORCH_CHECK(group_size > 0, "group_size must be positive");
    for (auto* t : {&k_q, &v_q, &k_scale, &v_scale}) check_same_device(q, *t);
    check_heads(q, k_q);
    const c10::cuda::CUDAGuard guard(q.device());
    const int64_t buf = kv_buffer({{&k_q, "k_q"}, {&v_q, "v_q"}, {&v_scale, "v_scale"}});
    const int64_t gbuf = seq_buffer(k_scale, "k_scale");
    const int64_t s = live_len(seqlen, k_q.size(2));
    auto out = torch::empty_like(q);
    at::Tensor& ws = workspace(q, lik_decode_workspace_bytes(q.size(0), q.size(1), k_q.size(1)));
    ok_or_throw(lik_decode_attention_int4(q.data_ptr(), k_q.data_ptr<int8_t>(), k_scale.data_ptr(),
                                          v_q.data_ptr<int8_t>(), v_scale.data_ptr(), out.data_ptr(), q.size(0),
                                          q.size(1), k_q.size(1), q.size(2), s, buf, group_size, gbuf,
                                          static_cast<float>(softmax_scale), ws.data_ptr(), ws.numel(),
                                          cur_stream()),
                "decode_attention_int4");
    return out;
}

torch::Tensor decode_attention_int4_asym(torch::Tensor q, torch::Tensor k_q, torch::Tensor k_scale,
                                         torch::Tensor k_zero, torch::Tensor v_q, torch::Tensor v_scale,
                                         torch::Tensor v_zero, int64_t group_size, double softmax_scale,
                                         int64_t seqlen) {
    check_q(q);
    check_kv4(k_q, "k_q", torch::kInt8, 64, true);
    check_kv4(v_q, "v_q", torch::kInt8, 64, true);
    TORCH_CHECK(k_q.sizes() == v_q.sizes(), "k_q and v_q must have the same shape");
    check_group_scale(k_scale, k_q, "k_scale", true);
    check_group_scale(k_zero, k_q, "k_zero", true);
    TORCH_CHECK(k_zero.sizes() == k_scale.sizes(), "k_zero must match k_scale");
    check_tok_scale(v_scale, v_q, "v_scale", true);
    check_tok_scale(v_zero, v_q, "v_zero", true);
    TORCH_CHECK(group_size > 0, "group_size must be positive");
    for (auto* t : {&k_q, &v_q, &k_scale, &v_scale, &k_zero, &v_zero}) check_same_device(q, *t);
    check_heads(q, k_q);
    const c10::cuda::CUDAGuard guard(q.device());
    const int64_t buf = kv_buffer({{&k_q, "k_q"}, {&v_q, "v_q"}, {&v_scale, "v_scale"}, {&v_zero, "v_zero"}});
    const int64_t gbuf = seq_buffer(k_scale, "k_scale");
    TORCH_CHECK(seq_buffer(k_zero, "k_zero") == gbuf, "k_zero and k_scale must share one buffer layout");
    const int64_t s = live_len(seqlen, k_q.size(2));
    auto out = torch::empty_like(q);
    at::Tensor& ws = workspace(q, lik_decode_workspace_bytes(q.size(0), q.size(1), k_q.size(1)));
    ok_or_throw(lik_decode_attention_int4_asym(
                    q.data_ptr(), k_q.data_ptr<int8_t>(), k_scale.data_ptr(), k_zero.data_ptr(),
                    v_q.data_ptr<int8_t>(), v_scale.data_ptr(), v_zero.data_ptr(), out.data_ptr(), q.size(0),
                    q.size(1), k_q.size(1), q.size(2), s, buf, group_size, gbuf,
                    static_cast<float>(softmax_scale), ws.data_ptr(), ws.numel(), cur_stream()),
                "decode_attention_int4_asym");
    return out;
}

// ---------------------------------------------------------------- quantize

void check_x(const at::Tensor& x) {
    check_cuda(x, "x");
    TORCH_CHECK(x.scalar_type() == torch::kHalf, "x must be fp16");
    TORCH_CHECK(x.dim() == 4, "x must be [batch, n_kv_heads, seqlen, head_dim]");
    TORCH_CHECK(x.size(3) == 128, "only head_dim=128 supported");
}

std::tuple<torch::Tensor, torch::Tensor> quantize_per_token(torch::Tensor x) {
    check_x(x);
    const c10::cuda::CUDAGuard guard(x.device());
    const auto B = x.size(0), H = x.size(1), S = x.size(2);
    auto q = torch::empty({B, H, S, 128}, x.options().dtype(torch::kInt8));
    auto s = torch::empty({B, H, S}, x.options().dtype(torch::kHalf));
    ok_or_throw(lik_quantize_per_token_int8(x.data_ptr(), q.data_ptr<int8_t>(), s.data_ptr(), B, H, S, 128, 0, S,
                                            cur_stream()),
                "quantize_per_token");
    return {q, s};
}

std::tuple<torch::Tensor, torch::Tensor> quantize_v_per_token_int4(torch::Tensor x) {
    check_x(x);
    const c10::cuda::CUDAGuard guard(x.device());
    const auto B = x.size(0), H = x.size(1), S = x.size(2);
    auto q = torch::empty({B, H, S, 64}, x.options().dtype(torch::kInt8));
    auto s = torch::empty({B, H, S}, x.options().dtype(torch::kHalf));
    ok_or_throw(lik_quantize_v_per_token_int4(x.data_ptr(), q.data_ptr<int8_t>(), s.data_ptr(), B, H, S, 128, 0,
                                              S, cur_stream()),
                "quantize_v_per_token_int4");
    return {q, s};
}

std::tuple<torch::Tensor, torch::Tensor> quantize_k_per_channel_groupwise_int4(torch::Tensor x,
                                                                                int64_t group_size) {
    check_x(x);
    TORCH_CHECK(group_size > 0, "group_size must be positive");
    const c10::cuda::CUDAGuard guard(x.device());
    const auto B = x.size(0), H = x.size(1), S = x.size(2);
    const int64_t ng = (S + group_size - 1) / group_size;
    auto q = torch::empty({B, H, S, 64}, x.options().dtype(torch::kInt8));
    auto s = torch::empty({B, H, ng, 128}, x.options().dtype(torch::kHalf));
    ok_or_throw(lik_quantize_k_per_channel_groupwise_int4(x.data_ptr(), q.data_ptr<int8_t>(), s.data_ptr(), B, H,
                                                          S, 128, group_size, 0, S, ng, cur_stream()),
                "quantize_k_per_channel_groupwise_int4");
    return {q, s};
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> quantize_v_per_token_int4_asym(torch::Tensor x) {
    check_x(x);
    const c10::cuda::CUDAGuard guard(x.device());
    const auto B = x.size(0), H = x.size(1), S = x.size(2);
    auto q = torch::empty({B, H, S, 64}, x.options().dtype(torch::kInt8));
    auto s = torch::empty({B, H, S}, x.options().dtype(torch::kHalf));
    auto z = torch::empty({B, H, S}, x.options().dtype(torch::kHalf));
    ok_or_throw(lik_quantize_v_per_token_int4_asym(x.data_ptr(), q.data_ptr<int8_t>(), s.data_ptr(), z.data_ptr(),
                                                   B, H, S, 128, 0, S, cur_stream()),
                "quantize_v_per_token_int4_asym");
    return {q, s, z};
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> quantize_k_per_channel_groupwise_int4_asym(
    torch::Tensor x, int64_t group_size) {
    check_x(x);
    TORCH_CHECK(group_size > 0, "group_size must be positive");
    const c10::cuda::CUDAGuard guard(x.device());
    const auto B = x.size(0), H = x.size(1), S = x.size(2);
    const int64_t ng = (S + group_size - 1) / group_size;
    auto q = torch::empty({B, H, S, 64}, x.options().dtype(torch::kInt8));
    auto s = torch::empty({B, H, ng, 128}, x.options().dtype(torch::kHalf));
    auto z = torch::empty({B, H, ng, 128}, x.options().dtype(torch::kHalf));
    ok_or_throw(lik_quantize_k_per_channel_groupwise_int4_asym(x.data_ptr(), q.data_ptr<int8_t>(), s.data_ptr(),
                                                               z.data_ptr(), B, H, S, 128, group_size, 0, S, ng,
                                                               cur_stream()),
                "quantize_k_per_channel_groupwise_int4_asym");
    return {q, s, z};
}

// ------------------------------------------------ append into a preallocated cache
//
// x [B, Hkv, n, 128] fp16 is quantized into rows [pos, pos + n) of a cache
// whose codes are [B, Hkv, buf_len, 128 or 64] and per-token scales
// [B, Hkv, buf_len] (per-group K scales [B, Hkv, n_groups_buf, 128]).

void check_cache(const at::Tensor& x, const at::Tensor& codes, int64_t last, int64_t pos) {
    check_x(x);
    check_kv4(codes, "codes", torch::kInt8, last);
    check_same_device(x, codes);
    TORCH_CHECK(codes.size(0) == x.size(0) && codes.size(1) == x.size(1), "cache batch/heads mismatch");
    TORCH_CHECK(pos >= 0 && pos + x.size(2) <= codes.size(2), "append overflows the cache");
}

void quantize_per_token_into(torch::Tensor x, torch::Tensor codes, torch::Tensor scale, int64_t pos) {
    check_cache(x, codes, 128, pos);
    check_tok_scale(scale, codes, "scale");
    const c10::cuda::CUDAGuard guard(x.device());
    ok_or_throw(lik_quantize_per_token_int8(x.data_ptr(), codes.data_ptr<int8_t>(), scale.data_ptr(), x.size(0),
                                            x.size(1), x.size(2), 128, pos, codes.size(2), cur_stream()),
                "quantize_per_token_into");
}

void quantize_v_per_token_int4_into(torch::Tensor x, torch::Tensor codes, torch::Tensor scale, int64_t pos,
                                    c10::optional<torch::Tensor> zero) {
    check_cache(x, codes, 64, pos);
    check_tok_scale(scale, codes, "scale");
    const c10::cuda::CUDAGuard guard(x.device());
    lik_status st;
    if (zero.has_value()) {
        check_tok_scale(*zero, codes, "zero");
        st = lik_quantize_v_per_token_int4_asym(x.data_ptr(), codes.data_ptr<int8_t>(), scale.data_ptr(),
                                                zero->data_ptr(), x.size(0), x.size(1), x.size(2), 128, pos,
                                                codes.size(2), cur_stream());
    } else {
        st = lik_quantize_v_per_token_int4(x.data_ptr(), codes.data_ptr<int8_t>(), scale.data_ptr(), x.size(0),
                                           x.size(1), x.size(2), 128, pos, codes.size(2), cur_stream());
    }
    ok_or_throw(st, "quantize_v_per_token_int4_into");
}

void quantize_k_per_channel_groupwise_int4_into(torch::Tensor x, torch::Tensor codes, torch::Tensor scale,
                                                int64_t group_size, int64_t pos,
                                                c10::optional<torch::Tensor> zero) {
    check_cache(x, codes, 64, pos);
    check_group_scale(scale, codes, "scale");
    TORCH_CHECK(group_size > 0, "group_size must be positive");
    const c10::cuda::CUDAGuard guard(x.device());
    lik_status st;
    if (zero.has_value()) {
        check_group_scale(*zero, codes, "zero");
        st = lik_quantize_k_per_channel_groupwise_int4_asym(x.data_ptr(), codes.data_ptr<int8_t>(),
                                                            scale.data_ptr(), zero->data_ptr(), x.size(0),
                                                            x.size(1), x.size(2), 128, group_size, pos,
                                                            codes.size(2), scale.size(2), cur_stream());
    } else {
        st = lik_quantize_k_per_channel_groupwise_int4(x.data_ptr(), codes.data_ptr<int8_t>(), scale.data_ptr(),
                                                       x.size(0), x.size(1), x.size(2), 128, group_size, pos,
                                                       codes.size(2), scale.size(2), cur_stream());
    }
    ok_or_throw(st, "quantize_k_per_channel_groupwise_int4_into");
}

// ---------------------------------------------------------------- paged

torch::Tensor paged_decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                     torch::Tensor block_tables, torch::Tensor context_lens, double softmax_scale,
                                     int64_t max_context_len, c10::optional<torch::Tensor> k_scale,
                                     c10::optional<torch::Tensor> v_scale, int64_t group_size,
                                     c10::optional<torch::Tensor> k_zero, c10::optional<torch::Tensor> v_zero) {
    check_q(q);
    check_cuda(k_cache, "k_cache");
    check_cuda(v_cache, "v_cache");
    TORCH_CHECK(k_cache.sizes() == v_cache.sizes(), "k_cache and v_cache must have the same shape");
    TORCH_CHECK(k_cache.dim() == 4, "caches must be [num_blocks, n_kv_heads, block_size, row]");
    check_cuda(block_tables, "block_tables");
    check_cuda(context_lens, "context_lens");
    TORCH_CHECK(block_tables.scalar_type() == torch::kInt32 && block_tables.dim() == 2 &&
                    block_tables.size(0) == q.size(0),
                "block_tables must be int32 [batch, max_blocks_per_seq]");
    TORCH_CHECK(context_lens.scalar_type() == torch::kInt32 && context_lens.dim() == 1 &&
                    context_lens.size(0) == q.size(0),
                "context_lens must be int32 [batch]");
    const int64_t hkv = k_cache.size(1);
    TORCH_CHECK(hkv > 0 && q.size(1) % hkv == 0, "n_heads must be a multiple of n_kv_heads");
    int fmt;
    if (k_cache.scalar_type() == torch::kHalf) {
        TORCH_CHECK(k_cache.size(3) == 128, "fp16 cache rows must be 128 wide");
        fmt = 0;
    } else {
        TORCH_CHECK(k_cache.scalar_type() == torch::kInt8, "caches must be fp16 or int8 codes");
        TORCH_CHECK(k_scale.has_value() && v_scale.has_value(), "quantized caches need k_scale and v_scale");
        if (k_cache.size(3) == 128) {
            fmt = 1;
        } else {
            TORCH_CHECK(k_cache.size(3) == 64, "packed INT4 rows must be 64 bytes");
            fmt = k_zero.has_value() ? 3 : 2;
        }
    }
    for (auto* t : {&k_cache, &v_cache, &block_tables, &context_lens}) check_same_device(q, *t);
    const c10::cuda::CUDAGuard guard(q.device());
    auto out = torch::empty_like(q);
    at::Tensor& ws = workspace(q, lik_decode_workspace_bytes(q.size(0), q.size(1), hkv));
    auto ptr = [](const c10::optional<torch::Tensor>& t) -> const void* {
        return t.has_value() ? t->data_ptr() : nullptr;
    };
    ok_or_throw(lik_decode_attention_paged(fmt, q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), ptr(k_scale),
                                           ptr(v_scale), ptr(k_zero), ptr(v_zero),
                                           block_tables.data_ptr<int32_t>(), context_lens.data_ptr<int32_t>(),
                                           out.data_ptr(), q.size(0), q.size(1), hkv, 128, k_cache.size(0),
                                           k_cache.size(2),
                                           block_tables.size(1), max_context_len, group_size,
                                           static_cast<float>(softmax_scale), ws.data_ptr(), ws.numel(),
                                           cur_stream()),
                "paged_decode_attention");
    return out;
}

// Append new tokens x [n_tokens, n_kv_heads, 128] fp16 (the new K or V) into
// a paged cache at slot_mapping (int64 [n_tokens]; negative = skip). The row
// format follows the cache: fp16 cache -> copy; int8 cache with 128-byte rows
// -> INT8 per token (scale); 64-byte rows -> INT4 per token (scale, and zero
// for the asymmetric format).
void paged_append(torch::Tensor x, torch::Tensor slot_mapping, torch::Tensor cache,
                  c10::optional<torch::Tensor> scale, c10::optional<torch::Tensor> zero) {
    check_cuda(x, "x");
    check_cuda(slot_mapping, "slot_mapping");
    check_cuda(cache, "cache");
    TORCH_CHECK(x.scalar_type() == torch::kHalf && x.dim() == 3 && x.size(2) == 128,
                "x must be fp16 [n_tokens, n_kv_heads, 128]");
    TORCH_CHECK(slot_mapping.scalar_type() == torch::kInt64 && slot_mapping.dim() == 1 &&
                    slot_mapping.size(0) == x.size(0),
                "slot_mapping must be int64 [n_tokens]");
    TORCH_CHECK(cache.dim() == 4 && cache.size(1) == x.size(1),
                "cache must be [num_blocks, n_kv_heads, block_size, row] with x's head count");
    int fmt;
    if (cache.scalar_type() == torch::kHalf) {
        TORCH_CHECK(cache.size(3) == 128, "fp16 cache rows must be 128 wide");
        fmt = 0;
    } else {
        TORCH_CHECK(cache.scalar_type() == torch::kInt8, "cache must be fp16 or int8 codes");
        TORCH_CHECK(scale.has_value(), "a quantized cache needs its per-token scale");
        if (cache.size(3) == 128) {
            fmt = 1;
        } else {
            TORCH_CHECK(cache.size(3) == 64, "packed INT4 rows must be 64 bytes");
            fmt = zero.has_value() ? 3 : 2;
        }
    }
    for (const auto* t : {&scale, &zero}) {
        if (!t->has_value()) continue;
        const auto& u = **t;
        check_cuda(u, "scale / zero");
        TORCH_CHECK(u.scalar_type() == torch::kHalf && u.dim() == 3 && u.size(0) == cache.size(0) &&
                        u.size(1) == cache.size(1) && u.size(2) == cache.size(2),
                    "scale / zero must be fp16 [num_blocks, n_kv_heads, block_size]");
        check_same_device(x, u);
    }
    check_same_device(x, slot_mapping);
    check_same_device(x, cache);
    const c10::cuda::CUDAGuard guard(x.device());
    ok_or_throw(lik_paged_append(fmt, x.data_ptr(), slot_mapping.data_ptr<int64_t>(), x.size(0), x.size(1), 128,
                                 cache.data_ptr(), scale.has_value() ? scale->data_ptr() : nullptr,
                                 zero.has_value() ? zero->data_ptr() : nullptr, cache.size(0), cache.size(2),
                                 cur_stream()),
                "paged_append");
}

// ---------------------------------------------------------------- dequantize

std::tuple<torch::Tensor, torch::Tensor> dequant_out(const torch::Tensor& codes, int64_t s) {
    auto o = codes.options().dtype(torch::kHalf);
    return {torch::empty({codes.size(0), codes.size(1), s, 128}, o),
            torch::empty({codes.size(0), codes.size(1), s, 128}, o)};
}

std::tuple<torch::Tensor, torch::Tensor> dequantize_int8(torch::Tensor k_q, torch::Tensor k_scale, torch::Tensor v_q,
                                                         torch::Tensor v_scale, int64_t seqlen) {
    check_kv4(k_q, "k_q", torch::kInt8, 128);
    check_kv4(v_q, "v_q", torch::kInt8, 128);
    TORCH_CHECK(k_q.sizes() == v_q.sizes(), "k_q and v_q must have the same shape");
    check_tok_scale(k_scale, k_q, "k_scale");
    check_tok_scale(v_scale, v_q, "v_scale");
    const c10::cuda::CUDAGuard guard(k_q.device());
    const int64_t s = live_len(seqlen, k_q.size(2));
    auto [ko, vo] = dequant_out(k_q, s);
    ok_or_throw(lik_dequantize_int8(k_q.data_ptr<int8_t>(), k_scale.data_ptr(), v_q.data_ptr<int8_t>(),
                                    v_scale.data_ptr(), ko.data_ptr(), vo.data_ptr(), k_q.size(0), k_q.size(1), s,
                                    k_q.size(2), 128, cur_stream()),
                "dequantize_int8");
    return {ko, vo};
}

std::tuple<torch::Tensor, torch::Tensor> dequantize_int4(torch::Tensor k_q, torch::Tensor k_scale, torch::Tensor v_q,
                                                         torch::Tensor v_scale, int64_t group_size, int64_t seqlen,
                                                         c10::optional<torch::Tensor> k_zero,
                                                         c10::optional<torch::Tensor> v_zero) {
    check_kv4(k_q, "k_q", torch::kInt8, 64);
    check_kv4(v_q, "v_q", torch::kInt8, 64);
    TORCH_CHECK(k_q.sizes() == v_q.sizes(), "k_q and v_q must have the same shape");
    check_group_scale(k_scale, k_q, "k_scale");
    check_tok_scale(v_scale, v_q, "v_scale");
    TORCH_CHECK(k_zero.has_value() == v_zero.has_value(), "give both zero points or neither");
    const c10::cuda::CUDAGuard guard(k_q.device());
    const int64_t s = live_len(seqlen, k_q.size(2));
    auto [ko, vo] = dequant_out(k_q, s);
    lik_status st;
    if (k_zero.has_value()) {
        check_group_scale(*k_zero, k_q, "k_zero");
        check_tok_scale(*v_zero, v_q, "v_zero");
        st = lik_dequantize_int4_asym(k_q.data_ptr<int8_t>(), k_scale.data_ptr(), k_zero->data_ptr(),
                                      v_q.data_ptr<int8_t>(), v_scale.data_ptr(), v_zero->data_ptr(), ko.data_ptr(),
                                      vo.data_ptr(), k_q.size(0), k_q.size(1), s, k_q.size(2), 128, group_size,
                                      k_scale.size(2), cur_stream());
    } else {
        st = lik_dequantize_int4(k_q.data_ptr<int8_t>(), k_scale.data_ptr(), v_q.data_ptr<int8_t>(),
                                 v_scale.data_ptr(), ko.data_ptr(), vo.data_ptr(), k_q.size(0), k_q.size(1), s,
                                 k_q.size(2), 128, group_size, k_scale.size(2), cur_stream());
    }
    ok_or_throw(st, "dequantize_int4");
    return {ko, vo};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    namespace py = pybind11;
    m.doc() = "B200 (sm_100a) GQA decode attention over fp16 / INT8 / INT4-KIVI KV caches";
    m.def("decode_attention", &decode_attention,
          "Decode attention over an fp16 KV cache (split-sequence, fused combine)", py::arg("q"), py::arg("k"),
          py::arg("v"), py::arg("softmax_scale"), py::arg("seqlen") = -1);
    m.def("decode_attention_v3", &decode_attention_v3, "Alias of decode_attention over the whole cache",
          py::arg("q"), py::arg("k"), py::arg("v"), py::arg("softmax_scale"));
    m.def("quantize_per_token", &quantize_per_token, "INT8 per-token symmetric KV quantization", py::arg("x"));
    m.def("decode_attention_int8", &decode_attention_int8, "Decode attention over an INT8 per-token KV cache",
          py::arg("q"), py::arg("k_q"), py::arg("k_scale"), py::arg("v_q"), py::arg("v_scale"),
          py::arg("softmax_scale"), py::arg("seqlen") = -1);
    m.def("quantize_k_per_channel_groupwise_int4", &quantize_k_per_channel_groupwise_int4,
          "INT4 per-channel groupwise quantization (KIVI K), packed", py::arg("x"), py::arg("group_size"));
    m.def("quantize_v_per_token_int4", &quantize_v_per_token_int4,
          "INT4 per-token quantization (KIVI V), packed", py::arg("x"));
    m.def("decode_attention_int4", &decode_attention_int4, "Decode attention over a KIVI INT4 KV cache",
          py::arg("q"), py::arg("k_q"), py::arg("k_scale"), py::arg("v_q"), py::arg("v_scale"),
          py::arg("group_size"), py::arg("softmax_scale"), py::arg("seqlen") = -1);
    m.def("quantize_k_per_channel_groupwise_int4_asym", &quantize_k_per_channel_groupwise_int4_asym,
          "Asymmetric INT4 per-channel groupwise quantization (scale + zero), packed", py::arg("x"),
          py::arg("group_size"));
    m.def("quantize_v_per_token_int4_asym", &quantize_v_per_token_int4_asym,
          "Asymmetric INT4 per-token quantization (scale + zero), packed", py::arg("x"));
    m.def("decode_attention_int4_asym", &decode_attention_int4_asym,
          "Decode attention over an asymmetric INT4 KIVI KV cache", py::arg("q"), py::arg("k_q"),
          py::arg("k_scale"), py::arg("k_zero"), py::arg("v_q"), py::arg("v_scale"), py::arg("v_zero"),
          py::arg("group_size"), py::arg("softmax_scale"), py::arg("seqlen") = -1);
    m.def("quantize_per_token_into", &quantize_per_token_into,
          "INT8 per-token quantize of new tokens into a preallocated cache at pos", py::arg("x"),
          py::arg("codes"), py::arg("scale"), py::arg("pos"));
    m.def("quantize_v_per_token_int4_into", &quantize_v_per_token_int4_into,
          "INT4 per-token quantize (zero given: asymmetric) into a preallocated cache at pos", py::arg("x"),
          py::arg("codes"), py::arg("scale"), py::arg("pos"), py::arg("zero") = py::none());
    m.def("quantize_k_per_channel_groupwise_int4_into", &quantize_k_per_channel_groupwise_int4_into,
          "INT4 per-channel groupwise quantize (zero given: asymmetric) into a preallocated cache at pos "
          "(a multiple of group_size)",
          py::arg("x"), py::arg("codes"), py::arg("scale"), py::arg("group_size"), py::arg("pos"),
          py::arg("zero") = py::none());
    m.def("check_device_errors", &check_device_errors,
          "Raise if a decode kernel on this device recorded a device-side error (bounded wait expired, "
          "out-of-range block-table entry); the affected workspaces are reset first");
    m.def("_selftest_leave_timeout", &selftest_leave_timeout,
          "Test hook: leave a bounded-wait timeout in the current stream's workspace");
    m.def("paged_decode_attention", &paged_decode_attention,
          "Decode attention over a paged KV cache (block tables, per-sequence lengths); the format follows the "
          "cache dtype (fp16, int8 codes, packed int4; zero points given: asymmetric INT4)",
          py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("block_tables"), py::arg("context_lens"),
          py::arg("softmax_scale"), py::arg("max_context_len"), py::arg("k_scale") = py::none(),
          py::arg("v_scale") = py::none(), py::arg("group_size") = 0, py::arg("k_zero") = py::none(),
          py::arg("v_zero") = py::none());
    m.def("paged_append", &paged_append,
          "Append new K or V tokens into a paged cache at slot_mapping (fp16 copy or per-token quantize)",
          py::arg("x"), py::arg("slot_mapping"), py::arg("cache"), py::arg("scale") = py::none(),
          py::arg("zero") = py::none());
    m.def("dequantize_int8", &dequantize_int8, "INT8 per-token KV -> fp16 K, V (first seqlen positions)",
          py::arg("k_q"), py::arg("k_scale"), py::arg("v_q"), py::arg("v_scale"), py::arg("seqlen") = -1);
    m.def("dequantize_int4", &dequantize_int4,
          "INT4 KIVI KV -> fp16 K, V (zero points given: asymmetric format)", py::arg("k_q"), py::arg("k_scale"),
          py::arg("v_q"), py::arg("v_scale"), py::arg("group_size"), py::arg("seqlen") = -1,
          py::arg("k_zero") = py::none(), py::arg("v_zero") = py::none());
}
