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
