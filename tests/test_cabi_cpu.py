"""C-ABI library checks that need no GPU: it loads, exports every function the
header declares, and rejects bad arguments before touching the device."""
import ctypes as C

import pytest

from lik_testutil import header_functions

cabi = pytest.importorskip("llmik_cuda.cabi")


def test_library_exports_every_header_function():
    names = header_functions()
    assert len(names) >= 15
    lib = cabi.lib()
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(cabi.SIGNATURES), "ctypes signatures out of sync with include/llmik.h"
    assert lib.lik_abi_version() == 2


def test_status_strings():
    lib = cabi.lib()
    assert lib.lik_status_string(0) == b"ok"
    assert lib.lik_status_string(6) == b"device-side wait timed out"
    assert lib.lik_status_string(7) == b"block-table entry out of range"


@pytest.mark.parametrize("head_dim,seqlen,buf,nh,nkv,status", [
    (64, 16, 16, 32, 8, 2),      # head_dim != 128 -> unsupported
    (128, 17, 16, 32, 8, 1),     # seqlen > kv_buf_len
    (128, 0, 16, 32, 8, 1),      # empty sequence
    (128, 16, 16, 30, 8, 1),     # n_heads % n_kv_heads != 0
])
def test_decode_rejects_bad_shapes_before_launch(head_dim, seqlen, buf, nh, nkv, status):
    lib = cabi.lib()
    dummy = C.c_void_p(16)
    st = lib.lik_decode_attention_f16(dummy, dummy, dummy, dummy, 1, nh, nkv, head_dim, seqlen, buf,
                                      0.1, dummy, 1 << 20, None)
    assert st == status
    assert lib.lik_last_error()


def test_quantize_rejects_bad_destination():
    lib = cabi.lib()
    d = C.c_void_p(16)
    # append window overflows the destination
    assert lib.lik_quantize_per_token_int8(d, d, d, 1, 8, 10, 128, 5, 12, None) == 1
    # K group append must start on a group boundary
    assert lib.lik_quantize_k_per_channel_groupwise_int4(d, d, d, 1, 8, 32, 128, 32, 16, 64, 4, None) == 1
    # misaligned source pointer
    assert lib.lik_quantize_per_token_int8(C.c_void_p(18), d, d, 1, 8, 4, 128, 0, 4, None) == 3


def test_zero_batch_is_a_noop():
    lib = cabi.lib()
    assert lib.lik_decode_attention_f16(None, None, None, None, 0, 32, 8, 128, 16, 16, 0.1, None, 0, None) == 0


def test_torch_glue_validates_like_the_reference():
    torch = pytest.importorskip("torch")
    import llmik_cuda
    q = torch.zeros(1, 32, 128, dtype=torch.half)
    k = torch.zeros(1, 8, 4, 128, dtype=torch.half)
    with pytest.raises(RuntimeError, match="CUDA"):
        llmik_cuda.decode_attention(q, k, k, 0.1)
    with pytest.raises(RuntimeError, match="CUDA"):
        llmik_cuda.quantize_per_token(k)
    # the reference's out-of-scope ops are deliberately absent
    assert not hasattr(llmik_cuda, "w4a16_gemm")
