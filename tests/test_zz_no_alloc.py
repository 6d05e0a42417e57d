"""The allocation-free decode entry point (lik_decode_attention_f16_noalloc).

It exists for callers that cannot allocate device memory when they launch
attention (a pre-carved memory pool, or a binding holding only raw pointers):
its scratch is a fixed array inside the library. This file is named so pytest
collects it last. It checks, through the C ABI, that two calls in a row match
the regular entry point that takes a caller-owned workspace, and that a shape
needing more than the fixed 4 MiB of scratch is refused.
"""
import ctypes
import math

import pytest
import torch

from lik_testutil import assert_attn_close

pytestmark = pytest.mark.gpu
SCALE = 1.0 / math.sqrt(128)


def _inputs(b, hq, hkv, s, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, hq, 128, generator=g).half().cuda()
    k = torch.randn(b, hkv, s, 128, generator=g).half().cuda()
    v = torch.randn(b, hkv, s, 128, generator=g).half().cuda()
    return q, k, v


def test_noalloc_matches_workspace_entry_point_twice():
    from llmik_cuda import cabi
    lib = cabi.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for b, s, seed in ((8, 4096, 1), (3, 777, 2)):   # two calls in a row, different shapes
        q, k, v = _inputs(b, 32, 8, s, seed)
        ref = torch.empty_like(q)
        wb = lib.lik_decode_workspace_bytes(b, 32, 8)
        ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
        cabi.call("lik_workspace_init", ws.data_ptr(), wb, stream)
        cabi.call("lik_decode_attention_f16", q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(),
                  b, 32, 8, 128, s, s, SCALE, ws.data_ptr(), wb, stream)
        out = torch.empty_like(q)
        cabi.call("lik_decode_attention_f16_noalloc", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                  b, 32, 8, 128, s, s, SCALE, stream)
        torch.cuda.synchronize()
        assert_attn_close(out.cpu().numpy(), ref.float().cpu().numpy())


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from llmik_cuda import cabi
    lib = cabi.lib()
    d = ctypes.c_void_p(256)
    # 2^20 units of counters need far more than the fixed 4 MiB
    st = lib.lik_decode_attention_f16_noalloc(d, d, d, d, 1 << 15, 32, 8, 128, 16, 16, SCALE, None)
    assert st == 4
    assert b"4 MiB" in lib.lik_last_error()
