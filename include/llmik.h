/*
 * llmik.h - C ABI of the B200 (sm_100a) GQA decode / KV-quantization library
 * (libllmik_b200.so).
 *
 * Plain C: raw device pointers, 64-bit sizes, an opaque CUDA stream
 * (cudaStream_t passed as void*; NULL = legacy default stream) and a status
 * return. No torch types, no exceptions, no process abort: every entry point
 * validates its arguments and returns a lik_status; lik_last_error() gives a
 * human-readable detail for the calling thread's most recent failure.
 *
 * All launches are asynchronous on `stream`. Pointers must be device (or
 * managed) memory of the current device. Tensor layouts are row-major and
 * follow the reference extension (bindings/extension.cpp):
 *
 *   q, out          [batch, n_heads, head_dim]                     fp16
 *   k, v (fp16)     [batch, n_kv_heads, kv_buf_len, head_dim]      fp16
 *   k_q, v_q (int8) [batch, n_kv_heads, kv_buf_len, head_dim]      int8
 *   k_q, v_q (int4) [batch, n_kv_heads, kv_buf_len, head_dim / 2]  packed,
 *                   byte = (code[2i] & 0xF) | (code[2i+1] & 0xF) << 4
 *   per-token scale / zero      [batch, n_kv_heads, kv_buf_len]               fp16
 *   per-channel-group scale/zero [batch, n_kv_heads, n_groups_buf, head_dim]  fp16
 *
 * `seqlen` is the live KV length attended over (the first `seqlen` positions
 * of each [kv_buf_len, ...] slab); kv_buf_len >= seqlen is the allocated
 * length (row stride), as in bindings/extension.cpp:26-44. head_dim must be
 * 128 and n_heads a multiple of n_kv_heads.
 *
 * Attention entry points use a caller-owned WORKSPACE (split-sequence partial
 * results and per-unit completion counters). Size it with
 * lik_decode_workspace_bytes() and zero it once with lik_workspace_init();
 * every call leaves it zeroed again. Calls that may run concurrently (different
 * streams) need different workspaces.
 */
#ifndef LLMIK_H
#define LLMIK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LLMIK_ABI_VERSION 2

typedef enum lik_status {
    LIK_OK = 0,
    LIK_ERR_INVALID_ARGUMENT = 1,   /* null pointer, bad shape, seqlen > kv_buf_len, ... */
    LIK_ERR_UNSUPPORTED = 2,        /* head_dim != 128 and similar */
    LIK_ERR_MISALIGNED = 3,         /* a pointer lacks the 16-byte alignment required */
    LIK_ERR_WORKSPACE = 4,          /* workspace missing or too small */
    LIK_ERR_CUDA = 5,               /* a CUDA runtime call or launch failed */
    LIK_ERR_DEVICE_TIMEOUT = 6,     /* a bounded device-side wait gave up */
    LIK_ERR_DEVICE_BAD_BLOCK = 7    /* a paged block-table entry was outside [0, num_blocks) */
} lik_status;

/* ---- library information and errors ---------------------------------- */

int lik_abi_version(void);
const char* lik_status_string(lik_status status);
/* Detail of the calling thread's last failing call ("" if none). */
const char* lik_last_error(void);

/* ---- workspace -------------------------------------------------------- */

/* Upper bound of the workspace that the attention entry points need for this
 * head configuration on the current device (independent of seqlen). */
size_t lik_decode_workspace_bytes(int64_t batch, int64_t n_heads, int64_t n_kv_heads);

/* Zero a workspace (cudaMemsetAsync on `stream`). Needed once after
 * allocation. */
lik_status lik_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* Read (and clear) the device error word that kernels set when a bounded
 * device-side wait expires (*device_error = 1, LIK_ERR_DEVICE_TIMEOUT) or a
 * paged block-table entry is out of range (2, LIK_ERR_DEVICE_BAD_BLOCK).
 * Synchronizes `stream`. *device_error = 0 means no error. After an error the
 * whole workspace is zeroed again on `stream` (a kernel that gave up may have
 * left unit counters behind), so it can be reused as is. */
lik_status lik_workspace_check(void* workspace, size_t workspace_bytes, void* stream,
                               int* device_error);

/* Failure-detection self test of the recovery path (no reference
 * counterpart): a one-warp kernel runs the decode kernels' bounded wait
 * (`polls` polls) on a barrier nothing arrives at and, when it gives up,
 * leaves what a decode kernel that gave up leaves: the timeout code in the
 * error word and a non-zero unit counter. Target: `workspace` (a zeroed decode
 * workspace of `workspace_bytes`), or, when workspace is NULL, the fixed
 * scratch of lik_decode_attention_f16_noalloc on the current device. The
 * next lik_workspace_check / lik_decode_noalloc_check must report the error
 * and reset the scratch. Asynchronous on `stream`. */
lik_status lik_selftest_leave_timeout(int64_t polls, void* workspace, size_t workspace_bytes, void* stream);

/* Failure-detection self test (no reference counterpart): runs a one-warp
 * kernel that waits, with the decode kernels' bounded poll loop limited to
 * `polls` polls, on a shared-memory barrier nothing arrives at. The wait must
 * give up and report: returns LIK_ERR_DEVICE_TIMEOUT with *device_error = 1
 * (synchronizes `stream`); the CUDA context stays usable. */
lik_status lik_selftest_bounded_wait(int64_t polls, int* device_error, void* stream);

/* ---- decode attention (single query token per sequence) -------------- */

/* fp16 KV. Replaces launch_decode_attention_splitk
 * (kernels/attention/fused_attention_splitk.cu:233-250) and
 * launch_decode_attention (kernels/attention/fused_attention.cu:110-119),
 * declared in kernels/attention/fused_attention.cuh:17-41; op
 * bindings/extension.cpp:26-83. */
lik_status lik_decode_attention_f16(
    const void* q, const void* k, const void* v, void* out,
    int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
    int64_t seqlen, int64_t kv_buf_len, float softmax_scale,
    void* workspace, size_t workspace_bytes, void* stream);

/* fp16 KV decode that allocates nothing and takes no workspace: for callers
 * that cannot call cudaMalloc when they launch attention (a runtime whose
 * device memory is already carved into its own pool, or a binding that only
 * holds the raw pointers it was given). No counterpart in the reference.
 * Same arguments and results as lik_decode_attention_f16 minus the
 * workspace. Its scratch is a fixed 4 MiB array inside the library that every
 * GPU loading the library keeps until exit (zero when the library loads);
 * shapes whose lik_decode_workspace_bytes() exceeds 4 MiB are rejected with
 * LIK_ERR_WORKSPACE. The first call on each device looks up that array's
 * device address (a host-side query, no device work), so make that first call
 * before any stream capture. All calls on a device share the one array:
 * calls that can overlap on the GPU (other streams, other host threads) race
 * and give wrong results; serialize them. A bounded device-side wait that
 * expires inside this path leaves its code in the array's error word; read and
 * clear it with lik_decode_noalloc_check. */
lik_status lik_decode_attention_f16_noalloc(
    const void* q, const void* k, const void* v, void* out,
    int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
    int64_t seqlen, int64_t kv_buf_len, float softmax_scale, void* stream);

/* Error check of the allocation-free path (no counterpart in the reference):
 * reads the device error word of lik_decode_attention_f16_noalloc's fixed
 * scratch on the current device after the work queued on `stream`
 * (synchronizes `stream`), like lik_workspace_check does for a caller-owned
 * workspace: *device_error = 0 and LIK_OK when clean; otherwise the code
 * (1 = a bounded wait expired), LIK_ERR_DEVICE_TIMEOUT, and the whole scratch
 * is zeroed again on `stream` so that later calls start from a clean state. */
lik_status lik_decode_noalloc_check(void* stream, int* device_error);

/* INT8 per-token KV: K = k_q * k_scale[token], V = v_q * v_scale[token].
 * Replaces launch_decode_attention_int8
 * (kernels/attention/fused_attention_int8.cu:109-122, declared
 * fused_attention.cuh:54-60; op bindings/extension.cpp:152-194). Unlike the
 * reference it also takes a live length / buffer stride. */
lik_status lik_decode_attention_int8(
    const void* q, const int8_t* k_q, const void* k_scale,
    const int8_t* v_q, const void* v_scale, void* out,
    int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
    int64_t seqlen, int64_t kv_buf_len, float softmax_scale,
    void* workspace, size_t workspace_bytes, void* stream);

/* INT4 KIVI, symmetric (reference format): signed nibbles in [-7, 7];
 * K = code * k_scale[group(token), channel], V = code * v_scale[token].
 * Replaces launch_decode_attention_int4
 * (kernels/attention/fused_attention_int4.cu:120-135, declared
 * fused_attention.cuh:73-80; op bindings/extension.cpp:269-314).
 * n_groups_buf is k_scale's group extent (k_scale.size(2) in the op);
 * ceil(seqlen / group_size) <= n_groups_buf. */
lik_status lik_decode_attention_int4(
    const void* q, const int8_t* k_q, const void* k_scale,
    const int8_t* v_q, const void* v_scale, void* out,
    int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
    int64_t seqlen, int64_t kv_buf_len, int64_t group_size, int64_t n_groups_buf,
    float softmax_scale, void* workspace, size_t workspace_bytes, void* stream);

/* INT4 KIVI, asymmetric (scale + zero; no reference counterpart, the format of
 * the benchmark's INT4 configuration): unsigned nibbles 0..15;
 * K = code * k_scale[g, c] + k_zero[g, c], V = code * v_scale[t] + v_zero[t]. */
lik_status lik_decode_attention_int4_asym(
    const void* q, const int8_t* k_q, const void* k_scale, const void* k_zero,
    const int8_t* v_q, const void* v_scale, const void* v_zero, void* out,
    int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
    int64_t seqlen, int64_t kv_buf_len, int64_t group_size, int64_t n_groups_buf,
    float softmax_scale, void* workspace, size_t workspace_bytes, void* stream);

/* Paged KV (block tables; vLLM-style layout, no reference counterpart: the
 * reference has only contiguous caches). kv_format: 0 fp16, 1 INT8 per token,
 * 2 INT4 KIVI symmetric, 3 INT4 KIVI asymmetric. Layouts:
 *   k_cache, v_cache  [num_blocks, n_kv_heads, block_size, 128 | 64]
 *   per-token scale / zero  [num_blocks, n_kv_heads, block_size]
 *   K group scale / zero    [num_blocks, n_kv_heads, block_size / group_size, 128]
 *   block_tables int32 [batch, max_blocks_per_seq]; context_lens int32 [batch]
 * Sequence b attends over its first context_lens[b] positions (clamped to
 * [0, max_context_len]; each must be >= 1); position t lives at row t %
 * block_size of block block_tables[b][t / block_size]. block_size is a
 * multiple of 16 (and of group_size for INT4); scale/zero pointers are
 * 16-byte aligned. num_blocks is the number of blocks in the caches: a table
 * entry a sequence reaches that lies outside [0, num_blocks) is never read
 * through; its tile is masked and the workspace error word records
 * LIK_ERR_DEVICE_BAD_BLOCK (lik_workspace_check). Same workspace rules as the
 * contiguous entry points. */
lik_status lik_decode_attention_paged(
    int kv_format, const void* q, const void* k_cache, const void* v_cache,
    const void* k_scale, const void* v_scale, const void* k_zero, const void* v_zero,
    const int32_t* block_tables, const int32_t* context_lens, void* out,
    int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
    int64_t num_blocks, int64_t block_size, int64_t max_blocks_per_seq, int64_t max_context_len,
    int64_t group_size, float softmax_scale,
    void* workspace, size_t workspace_bytes, void* stream);

/* Append new tokens into a paged cache (the layout lik_decode_attention_paged
 * reads; no reference counterpart: the reference appends only to contiguous
 * caches, with torch.cat). x: the new K or the new V, [n_tokens, n_kv_heads,
 * 128] fp16, contiguous. slot_mapping: [n_tokens] int64; token i is written
 * to row slot % block_size of block slot / block_size; slots < 0 (padding) or
 * >= num_blocks * block_size are skipped. row_format: 0 fp16 (cache rows of
 * 128 halves, scale/zero unused), 1 INT8 per token (codes + scale), 2 INT4
 * per token symmetric (KIVI V: packed signed nibbles + scale), 3 INT4 per
 * token asymmetric (V of the asymmetric format: unsigned nibbles + scale +
 * zero). cache [num_blocks, n_kv_heads, block_size, 128 | 64]; scale, zero
 * [num_blocks, n_kv_heads, block_size] fp16. Codes and scales are those of the
 * contiguous quantizers (bit-exact with the oracle). The INT4 K format is
 * quantized per channel over groups of tokens and cannot be appended one
 * token at a time: use lik_quantize_k_per_channel_groupwise_int4[_asym] on a
 * block's rows once its group is complete. */
lik_status lik_paged_append(
    int row_format, const void* x, const int64_t* slot_mapping,
    int64_t n_tokens, int64_t n_kv_heads, int64_t head_dim,
    void* cache, void* scale, void* zero,
    int64_t num_blocks, int64_t block_size, void* stream);

/* ---- KV quantize / pack --------------------------------------------- */
/*
 * Source x: [batch, n_kv_heads, n_tokens, head_dim] fp16, contiguous.
 * Destination: a cache of allocated length dst_buf_len (>= dst_pos + n_tokens);
 * the n_tokens quantized rows land at positions [dst_pos, dst_pos + n_tokens)
 * of every (batch, kv_head) slab. With dst_pos = 0 and dst_buf_len = n_tokens
 * this is the reference op's contiguous output.
 *
 * Codes are bit-identical to reference/kv_cache_ref.py on x.float():
 * scale = max(absmax / qmax, 1e-8) and code = clamp(rint(x / scale)) with IEEE
 * division and round-half-to-even; the stored scale is fp16(scale).
 */

/* INT8 per token. Replaces launch_quantize_per_token
 * (kernels/kv_cache/kv_compress.cu:69-79, decl kv_compress.cuh:19-22; op
 * bindings/extension.cpp:120-146). */
lik_status lik_quantize_per_token_int8(
    const void* x, int8_t* codes, void* scale,
    int64_t batch, int64_t n_kv_heads, int64_t n_tokens, int64_t head_dim,
    int64_t dst_pos, int64_t dst_buf_len, void* stream);

/* INT4 per token, packed (KIVI V). Replaces launch_quantize_v_per_token_int4
 * (kernels/kv_cache/kv_compress.cu:219-228, decl kv_compress.cuh:44-48; op
 * bindings/extension.cpp:235-261). */
lik_status lik_quantize_v_per_token_int4(
    const void* x, int8_t* packed, void* scale,
    int64_t batch, int64_t n_kv_heads, int64_t n_tokens, int64_t head_dim,
    int64_t dst_pos, int64_t dst_buf_len, void* stream);

/* INT4 per channel over groups of group_size tokens, packed (KIVI K). The
 * short last group uses its real tokens (the reference zero-pads, which leaves
 * an absolute maximum unchanged). dst_pos must be a multiple of group_size;
 * scales land at groups [dst_pos / group_size, ...) of a scale buffer with
 * n_groups_buf groups. Replaces launch_quantize_k_per_channel_groupwise_int4
 * (kernels/kv_cache/kv_compress.cu:159-170, decl kv_compress.cuh:36-40; op
 * bindings/extension.cpp:200-229). */
lik_status lik_quantize_k_per_channel_groupwise_int4(
    const void* x, int8_t* packed, void* scale,
    int64_t batch, int64_t n_kv_heads, int64_t n_tokens, int64_t head_dim,
    int64_t group_size, int64_t dst_pos, int64_t dst_buf_len, int64_t n_groups_buf,
    void* stream);

/* Asymmetric INT4 per token (V side of the asymmetric KIVI format; no
 * reference counterpart): scale = fp16(max((max - min) / 15, 2^-24)),
 * zero = fp16(min), code = clamp(rint((x - zero) / scale), 0, 15) using the
 * stored fp16 scale and zero. */
lik_status lik_quantize_v_per_token_int4_asym(
    const void* x, int8_t* packed, void* scale, void* zero,
    int64_t batch, int64_t n_kv_heads, int64_t n_tokens, int64_t head_dim,
    int64_t dst_pos, int64_t dst_buf_len, void* stream);

/* Asymmetric INT4 per channel over token groups (K side; no reference
 * counterpart). Same group rules as the symmetric K entry point. */
lik_status lik_quantize_k_per_channel_groupwise_int4_asym(
    const void* x, int8_t* packed, void* scale, void* zero,
    int64_t batch, int64_t n_kv_heads, int64_t n_tokens, int64_t head_dim,
    int64_t group_size, int64_t dst_pos, int64_t dst_buf_len, int64_t n_groups_buf,
    void* stream);

/* ---- dequantize to fp16 (prefill / materialize) ---------------------- */
/*
 * Codes of the first `seqlen` positions of caches with allocated length
 * kv_buf_len -> contiguous fp16 K and V [batch, n_kv_heads, seqlen, head_dim],
 * each value fp16(code * scale [+ zero]) -- the rounding of the reference's
 * dequantize helpers. Replaces the PyTorch materialize path
 * Int4KIVICache._materialize_fp16 (integration/kv_int4_cache.py:226-245,
 * helpers :41-67) and the test-side dequantization of INT8 caches
 * (tests/test_kv_cache.py:282-283).
 */
lik_status lik_dequantize_int8(
    const int8_t* k_q, const void* k_scale, const int8_t* v_q, const void* v_scale,
    void* k_out, void* v_out, int64_t batch, int64_t n_kv_heads, int64_t seqlen,
    int64_t kv_buf_len, int64_t head_dim, void* stream);

lik_status lik_dequantize_int4(
    const int8_t* k_q, const void* k_scale, const int8_t* v_q, const void* v_scale,
    void* k_out, void* v_out, int64_t batch, int64_t n_kv_heads, int64_t seqlen,
    int64_t kv_buf_len, int64_t head_dim, int64_t group_size, int64_t n_groups_buf,
    void* stream);

/* Asymmetric INT4 KIVI variant (no reference counterpart). */
lik_status lik_dequantize_int4_asym(
    const int8_t* k_q, const void* k_scale, const void* k_zero,
    const int8_t* v_q, const void* v_scale, const void* v_zero,
    void* k_out, void* v_out, int64_t batch, int64_t n_kv_heads, int64_t seqlen,
    int64_t kv_buf_len, int64_t head_dim, int64_t group_size, int64_t n_groups_buf,
    void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* LLMIK_H */
