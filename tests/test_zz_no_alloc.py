"""The allocation-free decode entry point (lik_decode_attention_f16_noalloc).

It exists for callers that cannot allocate device memory when they launch
attention (a pre-carved memory pool, or a binding holding only raw pointers):
its scratch is a fixed array inside the library. This file is named so pytest
collects it last. It checks, through the C ABI, that two calls in a row match
both the regular entry point that takes a caller-owned workspace and the CPU
oracle, that a shape needing more than the fixed 4 MiB of scratch is refused,
and that a device-side timeout left in the fixed scratch is reported by
lik_decode_noalloc_check and cleared.
"""
import ctypes
import math

import pytest
import torch

from lik_testutil import assert_attn_close
from oracle import kv_oracle as O

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
        assert_attn_close(out.cpu().numpy(),
                          O.decode_attention(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), SCALE))


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from llmik_cuda import cabi
    lib = cabi.lib()
    d = ctypes.c_void_p(256)
    # 2^20 units of counters need far more than the fixed 4 MiB
    st = lib.lik_decode_attention_f16_noalloc(d, d, d, d, 1 << 15, 32, 8, 128, 16, 16, SCALE, None)
    assert st == 4
    assert b"4 MiB" in lib.lik_last_error()


def test_noalloc_check_reports_and_clears_a_timeout():
    """A bounded wait that expires inside the allocation-free path leaves its
    code (and possibly a stale unit counter) in the fixed scratch. Emulated by
    the self-test kernel, whose own bounded wait runs out (no GPU fault): the
    check reports it once, zeroes the scratch, and the next call is right."""
    from llmik_cuda import cabi
    lib = cabi.lib()
    stream = torch.cuda.current_stream().cuda_stream
    err = ctypes.c_int(-1)
    q, k, v = _inputs(2, 32, 8, 900, 3)
    out = torch.empty_like(q)
    cabi.call("lik_decode_attention_f16_noalloc", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
              2, 32, 8, 128, 900, 900, SCALE, stream)
    assert lib.lik_decode_noalloc_check(stream, ctypes.byref(err)) == 0 and err.value == 0
    cabi.call("lik_selftest_leave_timeout", 64, None, 0, stream)
    assert lib.lik_decode_noalloc_check(stream, ctypes.byref(err)) == 6 and err.value == 1
    assert lib.lik_decode_noalloc_check(stream, ctypes.byref(err)) == 0 and err.value == 0
    out.zero_()
    cabi.call("lik_decode_attention_f16_noalloc", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
              2, 32, 8, 128, 900, 900, SCALE, stream)
    torch.cuda.synchronize()
    assert_attn_close(out.cpu().numpy(), O.decode_attention(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(),
                                                            SCALE))
