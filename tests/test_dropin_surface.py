"""Drop-in surface: every llmik_cuda op the reference's own callers use on the
decode path exists here.

REFERENCE_CALLS lists, per op, the reference files that call it
(``llmik_cuda.<op>(`` in integration/*.py, tests/*.py, benchmarks/*.py). When
``LLMIK_REFERENCE`` points at a reference checkout the list is re-derived from
it and must agree. The W4A16 GEMM and fused RMSNorm/SwiGLU/RoPE ops are
outside this path."""
import inspect
import os
import re
from pathlib import Path

import pytest

REFERENCE_CALLS = {
    "decode_attention": ["benchmarks/bench_attention.py", "benchmarks/bench_decode_step.py",
                         "benchmarks/bench_kv_cache.py", "integration/attention_patch.py",
                         "integration/prealloc_cache.py", "tests/test_attention.py"],
    "decode_attention_int4": ["benchmarks/bench_kv_cache.py", "integration/attention_patch.py",
                              "tests/test_kv_cache.py"],
    "decode_attention_int8": ["benchmarks/bench_kv_cache.py", "tests/test_kv_cache.py"],
    "quantize_k_per_channel_groupwise_int4": ["benchmarks/bench_kv_cache.py", "integration/attention_patch.py",
                                              "integration/kv_int4_cache.py", "tests/test_kv_cache.py"],
    "quantize_per_token": ["benchmarks/bench_kv_cache.py", "tests/test_kv_cache.py"],
    "quantize_v_per_token_int4": ["benchmarks/bench_kv_cache.py", "integration/attention_patch.py",
                                  "integration/kv_int4_cache.py", "tests/test_kv_cache.py"],
}
OUT_OF_SCOPE = {"w4a16_gemm", "w4a16_dequantize", "rmsnorm", "silu_mul", "rope"}


def test_every_reference_decode_op_exists():
    import llmik_cuda
    missing = sorted(n for n in REFERENCE_CALLS if not hasattr(llmik_cuda, n))
    assert not missing, missing


@pytest.mark.skipif(not os.environ.get("LLMIK_REFERENCE"), reason="LLMIK_REFERENCE not set")
def test_call_list_matches_a_reference_checkout():
    ref = Path(os.environ["LLMIK_REFERENCE"])
    calls = {}
    for sub in ("integration", "tests", "benchmarks"):
        for f in sorted((ref / sub).glob("*.py")):
            for m in re.finditer(r"\b(?:llmik_cuda|llmik)\.([a-z_0-9]+)\s*\(", f.read_text()):
                calls.setdefault(m.group(1), set()).add(f"{sub}/{f.name}")
    got = {k: sorted(v) for k, v in calls.items() if k not in OUT_OF_SCOPE}
    assert got == REFERENCE_CALLS


def test_reference_signatures_and_defaults():
    import llmik_cuda as L
    doc = L.decode_attention.__doc__
    assert "softmax_scale" in doc and "seqlen: typing.SupportsInt = -1" in doc
    assert "group_size" in L.decode_attention_int4.__doc__
    for name in ("decode_attention_v3", "quantize_per_token", "decode_attention_int8",
                 "quantize_k_per_channel_groupwise_int4", "quantize_v_per_token_int4"):
        assert callable(getattr(L, name))
