"""B200 (sm_100a) drop-in for the reference's ``llmik_cuda`` extension.

Exports the decode-path op surface of ``bindings/extension.cpp:476-494`` with
the same names, argument order, defaults and error behaviour (validation
failures raise ``RuntimeError``):

    decode_attention(q, k, v, softmax_scale, seqlen=-1)
    decode_attention_v3(q, k, v, softmax_scale)
    quantize_per_token(x) -> (q_int8, scale_fp16)
    decode_attention_int8(q, k_q, k_scale, v_q, v_scale, softmax_scale, seqlen=-1)
    quantize_k_per_channel_groupwise_int4(x, group_size) -> (packed, scale)
    quantize_v_per_token_int4(x) -> (packed, scale)
    decode_attention_int4(q, k_q, k_scale, v_q, v_scale, group_size, softmax_scale, seqlen=-1)

plus the asymmetric INT4 KIVI format (``*_asym``) and in-place append
quantizers (``*_into``) that write new tokens into a preallocated cache.

The ops run only on the CUDA library ``libllmik_b200.so`` built by
``build.py``; importing this package without the built extension raises
ImportError - there is no CPU fallback. The reference's out-of-scope ops
(``w4a16_*``, ``rmsnorm``, ``silu_mul``, ``rope``) are not provided.
"""
from __future__ import annotations

import os as _os

_here = _os.path.dirname(_os.path.abspath(__file__))

try:
    import torch as _torch  # noqa: F401  (loads libc10 / libtorch for _C)
    from . import _C
except ImportError as _e:  # pragma: no cover - exercised on unbuilt trees
    raise ImportError(
        "llmik_cuda: the CUDA extension is not built. Run "
        "`python llm-inference-kernels_b200/build.py` (needs nvcc for sm_100a). "
        f"Underlying error: {_e}"
    ) from _e

decode_attention = _C.decode_attention
decode_attention_v3 = _C.decode_attention_v3
quantize_per_token = _C.quantize_per_token
decode_attention_int8 = _C.decode_attention_int8
quantize_k_per_channel_groupwise_int4 = _C.quantize_k_per_channel_groupwise_int4
quantize_v_per_token_int4 = _C.quantize_v_per_token_int4
decode_attention_int4 = _C.decode_attention_int4

quantize_k_per_channel_groupwise_int4_asym = _C.quantize_k_per_channel_groupwise_int4_asym
quantize_v_per_token_int4_asym = _C.quantize_v_per_token_int4_asym
decode_attention_int4_asym = _C.decode_attention_int4_asym
quantize_per_token_into = _C.quantize_per_token_into
quantize_v_per_token_int4_into = _C.quantize_v_per_token_int4_into
quantize_k_per_channel_groupwise_int4_into = _C.quantize_k_per_channel_groupwise_int4_into
dequantize_int8 = _C.dequantize_int8
paged_decode_attention = _C.paged_decode_attention
dequantize_int4 = _C.dequantize_int4
paged_append = _C.paged_append
check_device_errors = _C.check_device_errors

LIBRARY_PATH = _os.path.join(_here, "libllmik_b200.so")

__all__ = [
    "decode_attention", "decode_attention_v3", "quantize_per_token", "decode_attention_int8",
    "quantize_k_per_channel_groupwise_int4", "quantize_v_per_token_int4", "decode_attention_int4",
    "quantize_k_per_channel_groupwise_int4_asym", "quantize_v_per_token_int4_asym",
    "decode_attention_int4_asym", "quantize_per_token_into", "quantize_v_per_token_int4_into",
    "quantize_k_per_channel_groupwise_int4_into", "dequantize_int8", "dequantize_int4", "paged_decode_attention", "paged_append",
    "check_device_errors", "LIBRARY_PATH",
]
