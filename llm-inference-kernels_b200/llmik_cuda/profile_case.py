"""Small decode case for profiling (ncu) and quick timing.

    python -m llmik_cuda.profile_case {f16|int8|int4|int4_asym} [launches]

Config-1 shape (batch 8, 32 query / 8 KV heads, head_dim 128, seqlen 4096),
one copy of the inputs (~134 MB of fp16 KV, larger than L2), seeded N(0,1),
a few launches. Small enough for an `ncu --set full` capture to finish in
about a minute.
"""
from __future__ import annotations

import math
import sys

import torch

import llmik_cuda as L


def main(argv):
    fmt = argv[1] if len(argv) > 1 else "f16"
    n = int(argv[2]) if len(argv) > 2 else 3
    sc = 1.0 / math.sqrt(128)
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(8, 32, 128, device="cuda", generator=g).half()
    k = torch.randn(8, 8, 4096, 128, device="cuda", generator=g).half()
    v = torch.randn(8, 8, 4096, 128, device="cuda", generator=g).half()
    if fmt == "f16":
        def f():
            return L.decode_attention(q, k, v, sc)
    elif fmt == "int8":
        kq, ks = L.quantize_per_token(k)
        vq, vs = L.quantize_per_token(v)

        def f():
            return L.decode_attention_int8(q, kq, ks, vq, vs, sc)
    elif fmt == "int4":
        kq, ks = L.quantize_k_per_channel_groupwise_int4(k, 128)
        vq, vs = L.quantize_v_per_token_int4(v)

        def f():
            return L.decode_attention_int4(q, kq, ks, vq, vs, 128, sc)
    else:
        kq, ks, kz = L.quantize_k_per_channel_groupwise_int4_asym(k, 128)
        vq, vs, vz = L.quantize_v_per_token_int4_asym(v)

        def f():
            return L.decode_attention_int4_asym(q, kq, ks, kz, vq, vs, vz, 128, sc)
    for _ in range(n):
        f()
    torch.cuda.synchronize()
    print("ok", fmt)


if __name__ == "__main__":
    main(sys.argv)
