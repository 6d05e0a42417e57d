"""GPU parity of the fused-dequant decode attention kernels against the fp32
oracle on identical (fp16-rounded dequantized) KV: |out - ref| <= 2e-3 +
1e-2 |ref| for every element."""
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from lik_testutil import assert_attn_close, attn_kv_int8, attn_kv_kivi_asym, attn_kv_kivi_sym
from oracle import kv_oracle as O

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"
SCALE = 1.0 / math.sqrt(128)


@pytest.fixture(scope="module")
def L():
    import llmik_cuda
    return llmik_cuda


def _inputs(b, hq, hkv, s, seed, buf=None, k_outliers=False):
    g = torch.Generator().manual_seed(seed)
    buf = buf or s
    q = torch.randn(b, hq, 128, generator=g).to(torch.float16)
    k = torch.randn(b, hkv, buf, 128, generator=g)
    if k_outliers:
        k[..., list(O.OUTLIER_CHANNELS)] *= 10.0
    v = torch.randn(b, hkv, buf, 128, generator=g)
    return q, k.to(torch.float16), v.to(torch.float16)


def test_config0_against_reference_golden(L):
    ag = np.load(G / "attention_golden.npz")
    q, k, v = (torch.from_numpy(ag[n]).cuda() for n in ("c0_q", "c0_k", "c0_v"))
    out = L.decode_attention(q, k, v, float(ag["scale"]))
    assert_attn_close(out.cpu().numpy(), ag["c0_out32"])
    out3 = L.decode_attention_v3(q, k, v, float(ag["scale"]))
    assert torch.equal(out, out3)


def test_int8_and_kivi_against_reference_golden(L):
    ag = np.load(G / "attention_golden.npz")
    q, k, v = (torch.from_numpy(ag[n]).cuda() for n in ("i8_q", "i8_k", "i8_v"))
    kq, ks = L.quantize_per_token(k)
    vq, vs = L.quantize_per_token(v)
    assert_attn_close(L.decode_attention_int8(q, kq, ks, vq, vs, SCALE).cpu().numpy(), ag["i8_out32"])
    kq, ks = L.quantize_k_per_channel_groupwise_int4(k, 32)
    vq, vs = L.quantize_v_per_token_int4(v)
    out = L.decode_attention_int4(q, kq, ks, vq, vs, 32, SCALE)
    assert_attn_close(out.cpu().numpy(), ag["kivi_out32"])


SHAPES = [
    # b, hq, hkv, s
    (1, 32, 8, 1), (1, 32, 8, 2), (2, 32, 8, 31), (1, 32, 8, 33), (1, 32, 8, 127), (3, 32, 8, 129),
    (1, 32, 8, 512), (8, 32, 8, 2048), (8, 32, 8, 4096), (2, 8, 8, 300), (2, 16, 8, 300),
    (2, 64, 8, 300), (1, 12, 4, 1000), (2, 6, 2, 77),
]


@pytest.mark.parametrize("b,hq,hkv,s", SHAPES)
def test_f16(L, b, hq, hkv, s):
    q, k, v = _inputs(b, hq, hkv, s, seed=s * 31 + hq)
    out = L.decode_attention(q.cuda(), k.cuda(), v.cuda(), SCALE)
    assert_attn_close(out.cpu().numpy(), O.decode_attention(q.numpy(), k.numpy(), v.numpy(), SCALE))


@pytest.mark.parametrize("b,hq,hkv,s", SHAPES)
def test_int8(L, b, hq, hkv, s):
    q, k, v = _inputs(b, hq, hkv, s, seed=s * 37 + hq)
    kq, ks = L.quantize_per_token(k.cuda())
    vq, vs = L.quantize_per_token(v.cuda())
    out = L.decode_attention_int8(q.cuda(), kq, ks, vq, vs, SCALE)
    kd, vd = attn_kv_int8(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(), vs.cpu().numpy())
    assert_attn_close(out.cpu().numpy(), O.decode_attention(q.numpy(), kd, vd, SCALE))


@pytest.mark.parametrize("gs", [32, 128, 7])
@pytest.mark.parametrize("b,hq,hkv,s", SHAPES)
def test_int4_kivi(L, b, hq, hkv, s, gs):
    q, k, v = _inputs(b, hq, hkv, s, seed=s * 41 + gs, k_outliers=True)
    kq, ks = L.quantize_k_per_channel_groupwise_int4(k.cuda(), gs)
    vq, vs = L.quantize_v_per_token_int4(v.cuda())
    out = L.decode_attention_int4(q.cuda(), kq, ks, vq, vs, gs, SCALE)
    kd, vd = attn_kv_kivi_sym(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(),
                                       vs.cpu().numpy(), gs)
    assert_attn_close(out.cpu().numpy(), O.decode_attention(q.numpy(), kd, vd, SCALE))


@pytest.mark.parametrize("gs", [32, 128, 5])
@pytest.mark.parametrize("b,hq,hkv,s", SHAPES)
def test_int4_asym(L, b, hq, hkv, s, gs):
    q, k, v = _inputs(b, hq, hkv, s, seed=s * 43 + gs, k_outliers=True)
    kq, ks, kz = L.quantize_k_per_channel_groupwise_int4_asym(k.cuda(), gs)
    vq, vs, vz = L.quantize_v_per_token_int4_asym(v.cuda())
    out = L.decode_attention_int4_asym(q.cuda(), kq, ks, kz, vq, vs, vz, gs, SCALE)
    kd, vd = attn_kv_kivi_asym(kq.cpu().numpy(), ks.cpu().numpy(), kz.cpu().numpy(),
                                        vq.cpu().numpy(), vs.cpu().numpy(), vz.cpu().numpy(), gs)
    assert_attn_close(out.cpu().numpy(), O.decode_attention(q.numpy(), kd, vd, SCALE))


@pytest.mark.parametrize("fmt", ["f16", "int4_asym"])
def test_config4_context_length(L, fmt):
    """Config 4's 32768-position context (3 sequences of a rank's shard; the
    full 64-sequence shape is checked row by row inside bench.py)."""
    b, hq, hkv, s, gs = 3, 32, 8, 32768, 128
    q, k, v = _inputs(b, hq, hkv, s, seed=4444, k_outliers=fmt != "f16")
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    if fmt == "f16":
        out = L.decode_attention(qc, kc, vc, SCALE)
        kd, vd = k.numpy(), v.numpy()
    else:
        kq, ks, kz = L.quantize_k_per_channel_groupwise_int4_asym(kc, gs)
        vq, vs, vz = L.quantize_v_per_token_int4_asym(vc)
        out = L.decode_attention_int4_asym(qc, kq, ks, kz, vq, vs, vz, gs, SCALE)
        kd, vd = attn_kv_kivi_asym(kq.cpu().numpy(), ks.cpu().numpy(), kz.cpu().numpy(),
                                   vq.cpu().numpy(), vs.cpu().numpy(), vz.cpu().numpy(), gs)
    assert_attn_close(out.cpu().numpy(), O.decode_attention(q.numpy(), kd, vd, SCALE))


@pytest.mark.parametrize("fmt", ["f16", "int8", "int4", "int4_asym"])
@pytest.mark.parametrize("s,buf", [(1, 64), (100, 256), (1000, 1003), (4095, 4096)])
def test_live_length_in_preallocated_cache(L, fmt, s, buf):
    """`seqlen` < allocated length reads the live prefix in place
    (integration/prealloc_cache.py); rows past seqlen hold garbage."""
    q, k, v = _inputs(2, 32, 8, s, seed=s + buf, buf=buf)
    k[:, :, s:] = 1e4     # would dominate the softmax if read
    v[:, :, s:] = float("nan")
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    gs = 32
    if fmt == "f16":
        out = L.decode_attention(qc, kc, vc, SCALE, s)
        kd, vd = k.numpy(), v.numpy()
    elif fmt == "int8":
        kq, ks = L.quantize_per_token(kc)
        vq, vs = L.quantize_per_token(vc)
        out = L.decode_attention_int8(qc, kq, ks, vq, vs, SCALE, s)
        kd, vd = attn_kv_int8(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(), vs.cpu().numpy())
    elif fmt == "int4":
        kq, ks = L.quantize_k_per_channel_groupwise_int4(kc, gs)
        vq, vs = L.quantize_v_per_token_int4(vc)
        out = L.decode_attention_int4(qc, kq, ks, vq, vs, gs, SCALE, s)
        kd, vd = attn_kv_kivi_sym(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(),
                                           vs.cpu().numpy(), gs)
    else:
        kq, ks, kz = L.quantize_k_per_channel_groupwise_int4_asym(kc, gs)
        vq, vs, vz = L.quantize_v_per_token_int4_asym(vc)
        out = L.decode_attention_int4_asym(qc, kq, ks, kz, vq, vs, vz, gs, SCALE, s)
        kd, vd = attn_kv_kivi_asym(kq.cpu().numpy(), ks.cpu().numpy(), kz.cpu().numpy(),
                                            vq.cpu().numpy(), vs.cpu().numpy(), vz.cpu().numpy(), gs)
    ref = O.decode_attention(q.numpy(), kd, vd, SCALE, seqlen=s)
    assert np.isfinite(out.cpu().numpy()).all()
    assert_attn_close(out.cpu().numpy(), ref)


def test_unaligned_token_scales_take_the_plain_load_path(L):
    """kv_buf_len % 8 != 0 makes per-token scale rows unaligned for bulk
    copies; the kernel falls back to plain loads."""
    q, k, v = _inputs(3, 32, 8, 203, seed=5)
    kq, ks = L.quantize_per_token(k.cuda())
    vq, vs = L.quantize_per_token(v.cuda())
    out = L.decode_attention_int8(q.cuda(), kq, ks, vq, vs, SCALE)
    kd, vd = attn_kv_int8(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(), vs.cpu().numpy())
    assert_attn_close(out.cpu().numpy(), O.decode_attention(q.numpy(), kd, vd, SCALE))


def test_repeated_calls_are_deterministic_and_workspace_self_cleans(L):
    q, k, v = _inputs(8, 32, 8, 4096, seed=1)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    outs = [L.decode_attention(qc, kc, vc, SCALE) for _ in range(5)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


@pytest.mark.parametrize("fmt", ["f16", "int8", "int4", "int4_asym"])
@pytest.mark.parametrize("b,s", [(128, 100), (64, 300), (40, 1)])
def test_many_short_units_per_cta(L, fmt, b, s):
    """Many short units: every CTA range holds several unit ends in
    consecutive tiles (whole units and partial ones), so finished segments are
    handed from the streaming warps to the finishing warp back to back. The
    result must match the oracle and be identical on a repeated call."""
    q, k, v = _inputs(b, 32, 8, s, seed=b * 7 + s, k_outliers=fmt.startswith("int4"))
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    if fmt == "f16":
        run = lambda: L.decode_attention(qc, kc, vc, SCALE)
        kd, vd = k.numpy(), v.numpy()
    elif fmt == "int8":
        kq, ks = L.quantize_per_token(kc)
        vq, vs = L.quantize_per_token(vc)
        run = lambda: L.decode_attention_int8(qc, kq, ks, vq, vs, SCALE)
        kd, vd = attn_kv_int8(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(), vs.cpu().numpy())
    elif fmt == "int4":
        kq, ks = L.quantize_k_per_channel_groupwise_int4(kc, 32)
        vq, vs = L.quantize_v_per_token_int4(vc)
        run = lambda: L.decode_attention_int4(qc, kq, ks, vq, vs, 32, SCALE)
        kd, vd = attn_kv_kivi_sym(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(),
                                           vs.cpu().numpy(), 32)
    else:
        kq, ks, kz = L.quantize_k_per_channel_groupwise_int4_asym(kc, 32)
        vq, vs, vz = L.quantize_v_per_token_int4_asym(vc)
        run = lambda: L.decode_attention_int4_asym(qc, kq, ks, kz, vq, vs, vz, 32, SCALE)
        kd, vd = attn_kv_kivi_asym(kq.cpu().numpy(), ks.cpu().numpy(), kz.cpu().numpy(),
                                            vq.cpu().numpy(), vs.cpu().numpy(), vz.cpu().numpy(), 32)
    out = run()
    assert_attn_close(out.cpu().numpy(), O.decode_attention(q.numpy(), kd, vd, SCALE))
    assert torch.equal(run(), out)


def test_64bit_offsets():
    """A cache whose byte offsets exceed 2^31 (K and V 2.4 GB each)."""
    import llmik_cuda as L
    b, hkv, s = 9, 8, 131072
    g = torch.Generator(device="cuda").manual_seed(0)
    k = torch.randn(b, hkv, s, 128, device="cuda", generator=g, dtype=torch.float16)
    v = torch.randn(b, hkv, s, 128, device="cuda", generator=g, dtype=torch.float16)
    q = torch.randn(b, 32, 128, device="cuda", generator=g, dtype=torch.float16)
    out = L.decode_attention(q, k, v, SCALE)
    last = slice(b - 1, b)
    ref = O.decode_attention(q[last].cpu().numpy(), k[last].cpu().numpy(), v[last].cpu().numpy(), SCALE)
    assert_attn_close(out[last].cpu().numpy(), ref)
    del k, v
    torch.cuda.empty_cache()


def test_properties_at_config1_size(L):
    """Size-independent checks at the benchmark shape (B=8, 32/8 heads, S=4096):
    constant V -> output equals it; linearity in V; KV position permutation
    invariance."""
    q, k, v = _inputs(8, 32, 8, 4096, seed=9)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    const = torch.full_like(vc, 0.25)
    out = L.decode_attention(qc, kc, const, SCALE).float()
    assert torch.allclose(out, torch.full_like(out, 0.25), atol=2e-3)
    v2 = torch.randn_like(vc.float()).half()
    a = L.decode_attention(qc, kc, vc, SCALE).float()
    b2 = L.decode_attention(qc, kc, v2, SCALE).float()
    ab = L.decode_attention(qc, kc, ((vc.float() + v2.float()) * 0.5).half(), SCALE).float()
    assert torch.allclose(ab, (a + b2) * 0.5, atol=2e-3, rtol=1e-2)
    perm = torch.randperm(4096, device="cuda")
    p = L.decode_attention(qc, kc[:, :, perm].contiguous(), vc[:, :, perm].contiguous(), SCALE).float()
    assert torch.allclose(p, a, atol=2e-3, rtol=1e-2)


def test_cabi_direct_decode_and_workspace_check(L):
    """Decode through the raw C ABI with a caller-owned workspace; the
    device error word stays clear."""
    from llmik_cuda import cabi
    lib = cabi.lib()
    q, k, v = _inputs(2, 32, 8, 777, seed=2)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    out = torch.empty_like(qc)
    wb = lib.lik_decode_workspace_bytes(2, 32, 8)
    ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    cabi.call("lik_workspace_init", ws.data_ptr(), wb, stream)
    for _ in range(3):
        cabi.call("lik_decode_attention_f16", qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(),
                  2, 32, 8, 128, 777, 777, SCALE, ws.data_ptr(), wb, stream)
    import ctypes
    err = ctypes.c_int(-1)
    cabi.call("lik_workspace_check", ws.data_ptr(), wb, stream, ctypes.byref(err))
    assert err.value == 0
    assert_attn_close(out.cpu().numpy(), O.decode_attention(q.numpy(), k.numpy(), v.numpy(), SCALE))
    # a too-small workspace is rejected, not overrun
    with pytest.raises(cabi.LikError, match="WORKSPACE"):
        cabi.call("lik_decode_attention_f16", qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(),
                  2, 32, 8, 128, 777, 777, SCALE, ws.data_ptr(), 300, stream)


def test_workspace_shared_across_shapes(L):
    """A shared workspace used first by a small call (whose partial results
    stay behind) and then by a call with more units must give correct results."""
    for b, s in ((1, 512), (2, 4096), (9, 2048), (1, 700), (12, 1500)):
        q, k, v = _inputs(b, 32, 8, s, seed=b * 1000 + s)
        out = L.decode_attention(q.cuda(), k.cuda(), v.cuda(), SCALE)
        assert_attn_close(out.cpu().numpy(), O.decode_attention(q.numpy(), k.numpy(), v.numpy(), SCALE))


def test_bounded_wait_expires_into_an_error_status(L):
    """A device wait that nothing will satisfy gives up after its poll limit,
    the host reads the error, and the context keeps working."""
    import ctypes
    from llmik_cuda import cabi
    lib = cabi.lib()
    err = ctypes.c_int(-1)
    st = lib.lik_selftest_bounded_wait(1000, ctypes.byref(err), torch.cuda.current_stream().cuda_stream)
    assert st == 6 and err.value == 1
    assert b"bounded" in lib.lik_last_error()
    q, k, v = _inputs(1, 32, 8, 64, seed=0)
    out = L.decode_attention(q.cuda(), k.cuda(), v.cuda(), SCALE)
    assert_attn_close(out.cpu().numpy(), O.decode_attention(q.numpy(), k.numpy(), v.numpy(), SCALE))
