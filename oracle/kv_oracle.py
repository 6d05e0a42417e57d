"""CPU oracle for the GQA decode / KV-quantization hot path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker or the timed CPU baseline. The product path
(``llmik_cuda``) never calls into it and has no CPU fallback.

This is a numpy restatement of the reference's PyTorch oracles:

* ``reference/kv_cache_ref.py`` (symmetric per-token and per-channel-groupwise
  quantization, and the INT8 / KIVI presets),
* ``reference/attention_ref.py`` (fp32 eager GQA decode attention),
* the INT4 nibble packing of ``kernels/kv_cache/kv_compress.cuh:25-28`` and the
  unpack helper of ``tests/test_kv_cache.py:295-314``.

Pinning: ``tests/golden/make_golden.py`` imports the real reference modules and
writes their outputs to ``tests/golden/*.npz``; ``tests/test_oracle_golden.py``
checks every function here against those vectors (codes and scales bit-exact,
attention to fp32 round-off).

The asymmetric (scale + zero) INT4 KIVI format asked for by the benchmark
configuration has NO reference implementation (the reference only mentions it in
its design notes), so ``quantize_*_asym`` below are this project's own
definition: parity for them is UNPINNED by the reference.

Bit-exactness conventions (shared with the CUDA kernels):

* the input is fp16 data viewed as fp32 (``x.float()`` in the reference tests),
* ``scale = max(absmax / qmax, 1e-8)`` in fp32 with IEEE division,
* ``code = clamp(rint(x / scale), -qmax, qmax)`` with IEEE division and
  round-half-to-even (``torch.round``),
* the stored scale is ``fp16(scale)`` (round to nearest even).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
F16 = np.float16
HEAD_DIM = 128
LOG2E = 1.4426950408889634

# Smallest positive fp16 subnormal. The asymmetric scale is clamped to it so the
# stored fp16 scale is never zero (a zero scale would make dequant lossy and the
# division undefined).
ASYM_SCALE_FLOOR = F32(2.0 ** -24)


def _qmax(bits: int) -> int:
    """Symmetric code bound 2^(bits-1)-1 (reference/kv_cache_ref.py:32-43)."""
    assert bits in (4, 8), bits
    return (1 << (bits - 1)) - 1


def _as_f32(x) -> np.ndarray:
    x = np.asarray(x)
    return x.astype(F32, copy=False)


# ---------------------------------------------------------------------------
# Symmetric quantizers (reference-pinned)
# ---------------------------------------------------------------------------

def quantize_per_token(x, bits: int):
    """Symmetric per-token quantization (reference/kv_cache_ref.py:46-62).

    x: [..., seqlen, head_dim] (fp16 values; computed in fp32).
    Returns (codes int8 [..., seqlen, head_dim], scale fp32 [..., seqlen]).
    """
    x = _as_f32(x)
    qmax = _qmax(bits)
    absmax = np.abs(x).max(axis=-1, keepdims=True)
    scale = np.maximum(absmax / F32(qmax), F32(1e-8)).astype(F32)
    q = np.clip(np.rint(x / scale), -qmax, qmax).astype(np.int8)
    return q, scale[..., 0]


def dequantize_per_token(q, scale) -> np.ndarray:
    """reference/kv_cache_ref.py:65-70: codes * scale in fp32."""
    return q.astype(F32) * _as_f32(scale)[..., None]


def quantize_per_channel_groupwise(x, bits: int, group_size: int):
    """Symmetric per-(group, channel) quantization along seqlen
    (reference/kv_cache_ref.py:73-112). The short last group is zero padded,
    which cannot change an absolute maximum.

    x: [b, h, seqlen, d]. Returns (codes int8 [b,h,seqlen,d],
    scale fp32 [b,h,ceil(seqlen/gs),d]).
    """
    x = _as_f32(x)
    qmax = _qmax(bits)
    b, h, s, d = x.shape
    ng = (s + group_size - 1) // group_size
    pad = ng * group_size - s
    if pad:
        x = np.concatenate([x, np.zeros((b, h, pad, d), F32)], axis=2)
    xg = x.reshape(b, h, ng, group_size, d)
    absmax = np.abs(xg).max(axis=3)
    scale = np.maximum(absmax / F32(qmax), F32(1e-8)).astype(F32)
    q = np.clip(np.rint(xg / scale[:, :, :, None, :]), -qmax, qmax).astype(np.int8)
    return q.reshape(b, h, ng * group_size, d)[:, :, :s], scale


def dequantize_per_channel_groupwise(q, scale, group_size: int) -> np.ndarray:
    """reference/kv_cache_ref.py:115-129."""
    s = q.shape[2]
    idx = np.arange(s) // group_size
    return q.astype(F32) * _as_f32(scale)[:, :, idx, :]


def quantize_kv_int8_per_token(k, v):
    """INT8 preset (reference/kv_cache_ref.py:136-146)."""
    kq, ks = quantize_per_token(k, 8)
    vq, vs = quantize_per_token(v, 8)
    return kq, ks, vq, vs


def quantize_kv_kivi_int4(k, v, group_size: int = 32):
    """KIVI INT4 preset (reference/kv_cache_ref.py:159-169)."""
    kq, ks = quantize_per_channel_groupwise(k, 4, group_size)
    vq, vs = quantize_per_token(v, 4)
    return kq, ks, vq, vs


# ---------------------------------------------------------------------------
# Packing (kernels/kv_cache/kv_compress.cuh:25-28, tests/test_kv_cache.py:295-314)
# ---------------------------------------------------------------------------

def pack_int4(q) -> np.ndarray:
    """[..., d] int codes -> [..., d/2] int8; byte = (q_even & 0xF) | (q_odd & 0xF) << 4."""
    q = np.asarray(q).astype(np.int32)
    lo = q[..., 0::2] & 0xF
    hi = q[..., 1::2] & 0xF
    return (lo | (hi << 4)).astype(np.uint8).view(np.int8)


def unpack_int4_signed(packed) -> np.ndarray:
    """Inverse of pack_int4 for signed codes: nibbles sign-extended."""
    p = np.asarray(packed).view(np.uint8).astype(np.int32)
    lo = p & 0xF
    hi = p >> 4
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    out = np.stack([lo, hi], axis=-1).reshape(*p.shape[:-1], p.shape[-1] * 2)
    return out.astype(np.int8)


def unpack_int4_unsigned(packed) -> np.ndarray:
    """Inverse of pack_int4 for unsigned (asymmetric) codes 0..15."""
    p = np.asarray(packed).view(np.uint8).astype(np.int32)
    out = np.stack([p & 0xF, p >> 4], axis=-1).reshape(*p.shape[:-1], p.shape[-1] * 2)
    return out.astype(np.uint8)


# ---------------------------------------------------------------------------
# Asymmetric INT4 KIVI (this project's definition; parity UNPINNED)
# ---------------------------------------------------------------------------

def _asym_params(mn, mx):
    """scale_h = fp16(max((mx-mn)/15, 2^-24)), zero_h = fp16(mn); both returned
    as fp16 plus their exact fp32 values used for quantizing."""
    scale = np.maximum((mx - mn) / F32(15), ASYM_SCALE_FLOOR).astype(F32)
    scale_h = scale.astype(F16)
    zero_h = mn.astype(F16)
    return scale_h, zero_h, scale_h.astype(F32), zero_h.astype(F32)


def quantize_v_per_token_int4_asym(x):
    """Per-token asymmetric INT4 over the 128 channels of each token.

    code = clamp(rint((x - zero) / scale), 0, 15), computed in fp32 with the
    fp16-ROUNDED scale and zero (the values dequantization will use), so that
    x ~= code * scale + zero reconstructs with the stored parameters.
    Returns (codes uint8 [..., s, d], scale fp16 [..., s], zero fp16 [..., s]).
    """
    x = _as_f32(x)
    mn = x.min(axis=-1)
    mx = x.max(axis=-1)
    sh, zh, sf, zf = _asym_params(mn, mx)
    q = np.clip(np.rint((x - zf[..., None]) / sf[..., None]), 0, 15).astype(np.uint8)
    return q, sh, zh


def quantize_k_per_channel_groupwise_int4_asym(x, group_size: int):
    """Per-(group, channel) asymmetric INT4 along seqlen. The short last group
    takes min/max over its real tokens only (no zero padding, which would
    distort an asymmetric range).
    Returns (codes uint8 [b,h,s,d], scale fp16 [b,h,ng,d], zero fp16 [b,h,ng,d]).
    """
    x = _as_f32(x)
    b, h, s, d = x.shape
    ng = (s + group_size - 1) // group_size
    q = np.empty((b, h, s, d), np.uint8)
    sh = np.empty((b, h, ng, d), F16)
    zh = np.empty((b, h, ng, d), F16)
    for g in range(ng):
        t0, t1 = g * group_size, min((g + 1) * group_size, s)
        xg = x[:, :, t0:t1, :]
        s_h, z_h, sf, zf = _asym_params(xg.min(axis=2), xg.max(axis=2))
        sh[:, :, g] = s_h
        zh[:, :, g] = z_h
        q[:, :, t0:t1] = np.clip(np.rint((xg - zf[:, :, None]) / sf[:, :, None]), 0, 15)
    return q, sh, zh


def dequantize_asym_per_token(q, scale, zero) -> np.ndarray:
    return q.astype(F32) * _as_f32(scale)[..., None] + _as_f32(zero)[..., None]


def dequantize_asym_per_channel_groupwise(q, scale, zero, group_size: int) -> np.ndarray:
    idx = np.arange(q.shape[2]) // group_size
    return q.astype(F32) * _as_f32(scale)[:, :, idx, :] + _as_f32(zero)[:, :, idx, :]


# ---------------------------------------------------------------------------
# Attention (reference/attention_ref.py:43-80, 108-123)
# ---------------------------------------------------------------------------

def decode_attention(q, k, v, scale: float | None = None, seqlen: int | None = None):
    """Single-query GQA attention in fp32.

    q: [b, hq, d]; k, v: [b, hkv, s_buf, d] (attends to the first ``seqlen``
    positions; all of them when None). Returns fp32 [b, hq, d]; callers round
    to fp16 to match the reference's ``.to(q.dtype)``.

    The reference expands KV with ``repeat_interleave`` (query head i uses KV
    head i // (hq/hkv)); grouping q as [b, hkv, G, d] is the same mapping
    without the copy.
    """
    q = _as_f32(q)
    k = _as_f32(k)
    v = _as_f32(v)
    b, hq, d = q.shape
    hkv = k.shape[1]
    if seqlen is not None:
        k = k[:, :, :seqlen]
        v = v[:, :, :seqlen]
    if scale is None:
        scale = 1.0 / np.sqrt(d)
    g = hq // hkv
    qg = q.reshape(b, hkv, g, d)
    scores = np.matmul(qg, np.swapaxes(k, -1, -2)) * F32(scale)  # [b,hkv,g,s]
    scores = scores - scores.max(axis=-1, keepdims=True)
    p = np.exp(scores)
    p = p / p.sum(axis=-1, keepdims=True)
    out = np.matmul(p, v)  # [b,hkv,g,d]
    return out.reshape(b, hq, d).astype(F32)


def decode_attention_f16_out(q, k, v, scale=None, seqlen=None) -> np.ndarray:
    """decode_attention rounded to fp16, as the reference returns q.dtype."""
    return decode_attention(q, k, v, scale, seqlen).astype(F16)


# Dequantize-to-fp16 views used to check the fused-dequant kernels
# (tests/test_kv_cache.py:282-283, 400-402): the kernel and the oracle see
# identical fp16-rounded dequantized KV.

def dequant_int8_to_f16(kq, ks, vq, vs):
    k = dequantize_per_token(kq, ks).astype(F16)
    v = dequantize_per_token(vq, vs).astype(F16)
    return k, v


def dequant_kivi_sym_to_f16(kq_packed, ks, vq_packed, vs, group_size):
    kq = unpack_int4_signed(kq_packed)
    vq = unpack_int4_signed(vq_packed)
    k = dequantize_per_channel_groupwise(kq, ks, group_size).astype(F16)
    v = dequantize_per_token(vq, vs).astype(F16)
    return k, v


def dequant_kivi_asym_to_f16(kq_packed, ks, kz, vq_packed, vs, vz, group_size):
    kq = unpack_int4_unsigned(kq_packed)
    vq = unpack_int4_unsigned(vq_packed)
    k = dequantize_asym_per_channel_groupwise(kq, ks, kz, group_size).astype(F16)
    v = dequantize_asym_per_token(vq, vs, vz).astype(F16)
    return k, v


# Exactly dequantized views (fp32 code * scale [+ zero], no fp16 rounding):
# the reference's fp32 attention (reference/attention_ref.py:43-80) on the
# quantized values themselves. The reference's CUDA INT4 kernel folds the K
# group scale into q and never forms fp16 K
# (kernels/attention/fused_attention_int4.cu:74-83); kernels that fold scales
# the same way are checked against these.

def dequant_int8_exact(kq, ks, vq, vs):
    return dequantize_per_token(kq, ks), dequantize_per_token(vq, vs)


def dequant_kivi_sym_exact(kq_packed, ks, vq_packed, vs, group_size):
    kq = unpack_int4_signed(kq_packed)
    vq = unpack_int4_signed(vq_packed)
    return dequantize_per_channel_groupwise(kq, ks, group_size), dequantize_per_token(vq, vs)


def dequant_kivi_asym_exact(kq_packed, ks, kz, vq_packed, vs, vz, group_size):
    kq = unpack_int4_unsigned(kq_packed)
    vq = unpack_int4_unsigned(vq_packed)
    return (dequantize_asym_per_channel_groupwise(kq, ks, kz, group_size),
            dequantize_asym_per_token(vq, vs, vz))


# ---------------------------------------------------------------------------
# Seeded synthetic inputs (benchmark configurations)
# ---------------------------------------------------------------------------

OUTLIER_CHANNELS = (0, 37, 74, 111)   # 4 of 128 K channels scaled x10 (config 3)
