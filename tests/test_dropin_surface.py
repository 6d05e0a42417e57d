"""Drop-in surface: every llmik_cuda op the reference's own callers use on the
decode path exists here. Scans the reference checkout when it is present
(integration/*.py, tests/*.py, benchmarks/*.py); skipped elsewhere.
The W4A16 GEMM and fused RMSNorm/SwiGLU/RoPE ops are outside this path."""
import inspect
import os
import re
from pathlib import Path

import pytest

REF = Path(os.environ.get("LLMIK_REFERENCE", "/root/reference"))
OUT_OF_SCOPE = {"w4a16_gemm", "w4a16_dequantize", "rmsnorm", "silu_mul", "rope"}


def _called_ops():
    names = set()
    for sub in ("integration", "tests", "benchmarks"):
        for f in (REF / sub).glob("*.py"):
            for m in re.finditer(r"\b(?:llmik_cuda|llmik)\.([a-z_0-9]+)\s*\(", f.read_text()):
                names.add(m.group(1))
    return names


@pytest.mark.skipif(not (REF / "integration").is_dir(), reason="reference checkout not present")
def test_every_reference_decode_op_exists():
    import llmik_cuda
    called = _called_ops() - OUT_OF_SCOPE
    assert {"decode_attention", "decode_attention_int4", "quantize_per_token"} <= called
    missing = sorted(n for n in called if not hasattr(llmik_cuda, n))
    assert not missing, missing


def test_reference_signatures_and_defaults():
    import llmik_cuda as L
    doc = L.decode_attention.__doc__
    assert "softmax_scale" in doc and "seqlen: typing.SupportsInt = -1" in doc
    assert "group_size" in L.decode_attention_int4.__doc__
    for name in ("decode_attention_v3", "quantize_per_token", "decode_attention_int8",
                 "quantize_k_per_channel_groupwise_int4", "quantize_v_per_token_int4"):
        assert callable(getattr(L, name))
