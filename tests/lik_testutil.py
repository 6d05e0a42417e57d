"""Helpers shared by the test modules (seeded inputs, oracle comparisons)."""
from __future__ import annotations

import math
import re
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "llmik.h"

# Attention tolerance against the fp32 oracle on identical (dequantized) KV.
ATOL = 2e-3
RTOL = 1e-2


def header_functions() -> list[str]:
    """Every function declared in include/llmik.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(lik_[a-z0-9_]+)\s*\(", text)))


def assert_attn_close(out, ref, atol=ATOL, rtol=RTOL):
    out = np.asarray(out, np.float32)
    ref = np.asarray(ref, np.float32)
    err = np.abs(out - ref)
    bound = atol + rtol * np.abs(ref)
    bad = err > bound
    assert not bad.any(), (
        f"{bad.sum()} / {bad.size} outside atol={atol} rtol={rtol}; max abs err {err.max():.3e}")


def randn_f16(gen, *shape):
    import torch
    return torch.randn(*shape, generator=gen, dtype=torch.float32).to(torch.float16)


def scale_for(d=128):
    return 1.0 / math.sqrt(d)


# Which dequantized KV a decode kernel is compared against. The tensor-pipe
# kernels (INT8, and INT4 with K group sizes that are multiples of 16) fold
# the scales into q and the softmax weights, as the reference's own CUDA INT4
# kernel does, so they attend over the exact quantized values: they are
# checked against the oracle on exactly dequantized (fp32) KV. The CUDA-core
# INT4 kernel (other group sizes) dequantizes to fp16 first, exactly as the
# oracle's fp16 view does, and is checked against that view.

def tensor_pipe(fmt: str, group_size: int | None = None) -> bool:
    return fmt == "int8" or (group_size is not None and group_size % 16 == 0)


def attn_kv_int8(kq, ks, vq, vs):
    from oracle import kv_oracle as O
    return O.dequant_int8_exact(kq, ks, vq, vs)


def attn_kv_kivi_sym(kq, ks, vq, vs, gs):
    from oracle import kv_oracle as O
    if tensor_pipe("int4", gs):
        return O.dequant_kivi_sym_exact(kq, ks, vq, vs, gs)
    return O.dequant_kivi_sym_to_f16(kq, ks, vq, vs, gs)


def attn_kv_kivi_asym(kq, ks, kz, vq, vs, vz, gs):
    from oracle import kv_oracle as O
    if tensor_pipe("int4", gs):
        return O.dequant_kivi_asym_exact(kq, ks, kz, vq, vs, vz, gs)
    return O.dequant_kivi_asym_to_f16(kq, ks, kz, vq, vs, vz, gs)
