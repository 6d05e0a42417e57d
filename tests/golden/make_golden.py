"""Generate the golden vectors that pin the CPU oracle to the reference.

Run where a reference checkout is available, naming its location::

    LLMIK_REFERENCE=<reference checkout> python tests/golden/make_golden.py

It imports the reference's own PyTorch oracles (``reference/kv_cache_ref.py``,
``reference/attention_ref.py``) and its test-side INT4 unpack helper
(``tests/test_kv_cache.py:295-314``, whose behaviour `_ref_unpack` below restates, since
that module is a pytest file), runs them on seeded inputs, and writes
``tests/golden/*.npz``. The GPU box never needs the reference: the tests only
read the committed ``.npz`` files.
"""
from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

if not os.environ.get("LLMIK_REFERENCE"):
    sys.exit("set LLMIK_REFERENCE to the reference checkout")
REF = Path(os.environ["LLMIK_REFERENCE"])
OUT = Path(__file__).resolve().parent

sys.path.insert(0, str(REF))
from reference import attention_ref, kv_cache_ref  # noqa: E402


def _ref_unpack(packed: torch.Tensor) -> torch.Tensor:
    """The reference test helper's unpack convention (sign-extend each nibble)."""
    *prefix, half_d = packed.shape
    p = packed.to(torch.int32) & 0xFF
    lo = ((p & 0x0F) << 4).to(torch.int8) >> 4
    hi = (p & 0xF0).to(torch.int8) >> 4
    return torch.stack([lo, hi], dim=-1).reshape(*prefix, 2 * half_d).to(torch.int8)


def _make_x(b, s, seed, outliers=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(b, 8, s, 128, generator=g)
    if outliers:                     # tests/test_kv_cache.py:51 pattern
        x[..., ::17] *= 3.5
    return x.to(torch.float16)


def _tie_rows():
    """Tokens whose values hit exact rounding ties and the all-zero case."""
    rows = torch.zeros(4, 128)
    # int8: absmax 127 -> scale exactly 1.0; x.5 values are ties.
    rows[0, 0] = 127.0
    rows[0, 1:9] = torch.tensor([2.5, -3.5, 0.5, -0.5, 1.5, 126.5, -126.5, 4.5])
    # int4: absmax 7 -> scale 1.0
    rows[1, 0] = -7.0
    rows[1, 1:7] = torch.tensor([2.5, -3.5, 0.5, -0.5, 1.5, 6.5])
    # all zeros -> scale clamps to 1e-8, codes 0
    # row 3: tiny values (scale below fp16 normal range)
    rows[3, :] = 1e-6 * torch.linspace(-1, 1, 128)
    return rows.to(torch.float16)


def quant_cases():
    out = {}
    x = _make_x(2, 100, seed=1)
    ties = _tie_rows()
    x[0, 0, :4] = ties
    out["x"] = x.numpy()
    for bits in (8, 4):
        q, s = kv_cache_ref.quantize_per_token(x.float(), bits)
        out[f"tok{bits}_q"] = q.numpy()
        out[f"tok{bits}_s32"] = s.numpy()
        out[f"tok{bits}_s16"] = s.to(torch.float16).numpy()
    for gs in (32, 128, 7):
        q, s = kv_cache_ref.quantize_per_channel_groupwise(x.float(), 4, gs)
        out[f"chan4_g{gs}_q"] = q.numpy()
        out[f"chan4_g{gs}_s32"] = s.numpy()
        out[f"chan4_g{gs}_s16"] = s.to(torch.float16).numpy()
    # presets
    k = _make_x(1, 64, seed=2)
    v = _make_x(1, 64, seed=3, outliers=False)
    out["preset_k"] = k.numpy()
    out["preset_v"] = v.numpy()
    kq, ks, vq, vs = kv_cache_ref.quantize_kv_int8_per_token(k.float(), v.float())
    out.update(int8_kq=kq.numpy(), int8_ks=ks.numpy(), int8_vq=vq.numpy(), int8_vs=vs.numpy())
    kq, ks, vq, vs = kv_cache_ref.quantize_kv_kivi_int4(k.float(), v.float(), group_size=32)
    out.update(kivi_kq=kq.numpy(), kivi_ks=ks.numpy(), kivi_vq=vq.numpy(), kivi_vs=vs.numpy())
    # unpack convention over every byte value
    allbytes = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.int8).reshape(1, 256)
    out["unpack_bytes"] = allbytes.numpy()
    out["unpack_codes"] = _ref_unpack(allbytes).numpy()
    np.savez_compressed(OUT / "quant_golden.npz", **out)


def attention_cases():
    out = {}
    # Config 0: B=1, 32 q heads, 8 kv heads, S=512, N(0,1) cast to fp16.
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 32, 1, 128, generator=g).to(torch.float16)
    k = torch.randn(1, 8, 512, 128, generator=g).to(torch.float16)
    v = torch.randn(1, 8, 512, 128, generator=g).to(torch.float16)
    scale = 1.0 / math.sqrt(128)
    ref16 = attention_ref.decode_attention(q, k, v, scale=scale)
    ref32 = attention_ref.decode_attention(q.float(), k.float(), v.float(), scale=scale)
    out.update(c0_q=q.squeeze(2).numpy(), c0_k=k.numpy(), c0_v=v.numpy(),
               c0_out16=ref16.squeeze(2).numpy(), c0_out32=ref32.squeeze(2).numpy(),
               scale=np.float32(scale))
    # INT8 and KIVI attention on dequantized KV (small, ragged length 77).
    k = _make_x(2, 77, seed=4)
    v = _make_x(2, 77, seed=5, outliers=False)
    qq = torch.randn(2, 32, 1, 128, generator=g).to(torch.float16)
    kq, ks, vq, vs = kv_cache_ref.quantize_kv_int8_per_token(k.float(), v.float())
    kd, vd = kv_cache_ref.dequantize_kv_int8_per_token(kq, ks.half(), vq, vs.half())
    out.update(i8_q=qq.squeeze(2).numpy(), i8_k=k.numpy(), i8_v=v.numpy(),
               i8_out32=attention_ref.decode_attention(qq.float(), kd.float(), vd.float(),
                                                       scale=scale).squeeze(2).numpy())
    kq, ks, vq, vs = kv_cache_ref.quantize_kv_kivi_int4(k.float(), v.float(), group_size=32)
    kd, vd = kv_cache_ref.dequantize_kv_kivi_int4(kq, ks.half(), vq, vs.half(), group_size=32)
    out["kivi_out32"] = attention_ref.decode_attention(
        qq.float(), kd.float(), vd.float(), scale=scale).squeeze(2).numpy()
    np.savez_compressed(OUT / "attention_golden.npz", **out)


if __name__ == "__main__":
    quant_cases()
    attention_cases()
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)
