"""GPU parity of the quantize/pack kernels: bit-exact against the oracle (and,
for the reference formats, against the reference-generated golden vectors)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import kv_oracle as O

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def L():
    import llmik_cuda
    return llmik_cuda


def _x(b, s, seed, outliers=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(b, 8, s, 128, generator=g)
    if outliers:
        x[..., ::17] *= 3.5
    return x.to(torch.float16)


def test_golden_vectors_on_gpu(L):
    """Codes and fp16 scales equal the reference oracle's output bit for bit."""
    qg = np.load(G / "quant_golden.npz")
    x = torch.from_numpy(qg["x"]).cuda()
    q, s = L.quantize_per_token(x)
    np.testing.assert_array_equal(q.cpu().numpy(), qg["tok8_q"])
    np.testing.assert_array_equal(s.cpu().numpy(), qg["tok8_s16"])
    q, s = L.quantize_v_per_token_int4(x)
    np.testing.assert_array_equal(O.unpack_int4_signed(q.cpu().numpy()), qg["tok4_q"])
    np.testing.assert_array_equal(s.cpu().numpy(), qg["tok4_s16"])
    for gs in (32, 128, 7):
        q, s = L.quantize_k_per_channel_groupwise_int4(x, gs)
        np.testing.assert_array_equal(O.unpack_int4_signed(q.cpu().numpy()), qg[f"chan4_g{gs}_q"])
        np.testing.assert_array_equal(s.cpu().numpy(), qg[f"chan4_g{gs}_s16"])


@pytest.mark.parametrize("b,s", [(1, 1), (1, 128), (2, 100), (4, 1024), (8, 4096)])
def test_per_token_int8_and_int4_bit_exact(L, b, s):
    x = _x(b, s, seed=s)
    xn = x.numpy()
    q, sc = L.quantize_per_token(x.cuda())
    rq, rs = O.quantize_per_token(xn, 8)
    np.testing.assert_array_equal(q.cpu().numpy(), rq)
    np.testing.assert_array_equal(sc.cpu().numpy(), rs.astype(np.float16))
    q, sc = L.quantize_v_per_token_int4(x.cuda())
    rq, rs = O.quantize_per_token(xn, 4)
    np.testing.assert_array_equal(q.cpu().numpy(), O.pack_int4(rq))
    np.testing.assert_array_equal(sc.cpu().numpy(), rs.astype(np.float16))


@pytest.mark.parametrize("b,s,gs", [(1, 128, 32), (4, 1024, 128), (2, 100, 32), (2, 100, 128),
                                    (1, 37, 1), (1, 300, 7), (8, 4096, 128), (1, 257, 256)])
def test_k_groupwise_int4_bit_exact(L, b, s, gs):
    x = _x(b, s, seed=s + gs)
    q, sc = L.quantize_k_per_channel_groupwise_int4(x.cuda(), gs)
    rq, rs = O.quantize_per_channel_groupwise(x.numpy(), 4, gs)
    np.testing.assert_array_equal(q.cpu().numpy(), O.pack_int4(rq))
    np.testing.assert_array_equal(sc.cpu().numpy(), rs.astype(np.float16))


@pytest.mark.parametrize("b,s,gs", [(1, 128, 128), (2, 100, 32), (8, 4096, 128), (1, 77, 7)])
def test_asym_int4_bit_exact(L, b, s, gs):
    x = _x(b, s, seed=7 * s + gs)
    q, sc, z = L.quantize_v_per_token_int4_asym(x.cuda())
    rq, rs, rz = O.quantize_v_per_token_int4_asym(x.numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), O.pack_int4(rq))
    np.testing.assert_array_equal(sc.cpu().numpy(), rs)
    np.testing.assert_array_equal(z.cpu().numpy(), rz)
    q, sc, z = L.quantize_k_per_channel_groupwise_int4_asym(x.cuda(), gs)
    rq, rs, rz = O.quantize_k_per_channel_groupwise_int4_asym(x.numpy(), gs)
    np.testing.assert_array_equal(q.cpu().numpy(), O.pack_int4(rq))
    np.testing.assert_array_equal(sc.cpu().numpy(), rs)
    np.testing.assert_array_equal(z.cpu().numpy(), rz)


def test_exact_ties_round_half_to_even(L):
    """Rows built so that x / scale lands exactly on half-integers (scale 1):
    the kernels' fast rounding must send these through the exact division and
    round half to even like the oracle."""
    halves = np.array([0.5, 1.5, 2.5, 3.5, -0.5, -1.5, -2.5, -6.5, 6.5, 5.5, -5.5, 4.5], np.float32)
    x = np.zeros((1, 8, 16, 128), np.float32)
    for t in range(16):
        row = np.resize(np.roll(halves, t), 128)
        x[0, :, t] = row
        x[0, :, t, 0] = 127.0 if t % 2 == 0 else 7.0   # per-token absmax: scale 1 for int8 / int4
    x16 = torch.from_numpy(x).half()
    xc = x16.cuda()
    q, sc = L.quantize_per_token(xc)
    rq, rs = O.quantize_per_token(x16.numpy(), 8)
    np.testing.assert_array_equal(q.cpu().numpy(), rq)
    np.testing.assert_array_equal(sc.cpu().numpy(), rs.astype(np.float16))
    q, sc = L.quantize_v_per_token_int4(xc)
    rq, rs = O.quantize_per_token(x16.numpy(), 4)
    np.testing.assert_array_equal(q.cpu().numpy(), O.pack_int4(rq))
    # asymmetric: min -7.5 and max 7.5 give scale 1 and zero -7.5, so
    # (x - zero) / scale is a half-integer wherever x is an integer
    xa = np.resize(np.arange(-7, 8, dtype=np.float32), (1, 8, 16, 128)).copy()
    xa[..., 0], xa[..., 1] = -7.5, 7.5
    xa16 = torch.from_numpy(xa).half()
    q, sc, z = L.quantize_v_per_token_int4_asym(xa16.cuda())
    rq, rs, rz = O.quantize_v_per_token_int4_asym(xa16.numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), O.pack_int4(rq))
    np.testing.assert_array_equal(sc.cpu().numpy(), rs)
    np.testing.assert_array_equal(z.cpu().numpy(), rz)
    # per-channel groups along tokens: every group holds -7.5 and 7.5 (asym:
    # scale 1, zero -7.5) or 7 (sym: scale 1), the other tokens sit on ties
    for gs in (16, 7):
        t = np.arange(16)
        col = np.resize(np.arange(-7, 8, dtype=np.float32), 16)
        col[t % gs == 0], col[t % gs == 1] = -7.5, 7.5
        xk = np.broadcast_to(col[None, None, :, None], (1, 8, 16, 128)).astype(np.float16)
        q, sc, z = L.quantize_k_per_channel_groupwise_int4_asym(torch.from_numpy(xk.copy()).cuda(), gs)
        rq, rs, rz = O.quantize_k_per_channel_groupwise_int4_asym(xk, gs)
        np.testing.assert_array_equal(q.cpu().numpy(), O.pack_int4(rq))
        np.testing.assert_array_equal(sc.cpu().numpy(), rs)
        col = np.resize(halves, 16)
        col[t % gs == 0] = 7.0
        xk = np.broadcast_to(col[None, None, :, None], (1, 8, 16, 128)).astype(np.float16)
        q, sc = L.quantize_k_per_channel_groupwise_int4(torch.from_numpy(xk.copy()).cuda(), gs)
        rq, rs = O.quantize_per_channel_groupwise(xk, 4, gs)
        np.testing.assert_array_equal(q.cpu().numpy(), O.pack_int4(rq))


def test_constant_and_zero_rows(L):
    x = torch.zeros(1, 8, 40, 128, dtype=torch.float16)
    x[0, 1] = 3.0          # constant rows: asym range 0 -> scale floor
    x[0, 2, :, 5] = -2.0
    xc = x.cuda()
    for fn, bits in ((L.quantize_per_token, 8), (L.quantize_v_per_token_int4, 4)):
        q, s = fn(xc)
        rq, rs = O.quantize_per_token(x.numpy(), bits)
        got = q.cpu().numpy() if bits == 8 else O.unpack_int4_signed(q.cpu().numpy())
        np.testing.assert_array_equal(got, rq)
        np.testing.assert_array_equal(s.cpu().numpy(), rs.astype(np.float16))
    q, s, z = L.quantize_v_per_token_int4_asym(xc)
    rq, rs, rz = O.quantize_v_per_token_int4_asym(x.numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), O.pack_int4(rq))
    np.testing.assert_array_equal(s.cpu().numpy(), rs)


def test_append_into_preallocated_cache_matches_one_shot(L):
    """Quantizing token chunks into a cache at increasing positions gives the
    same bytes as quantizing the whole sequence at once."""
    x = _x(2, 256, seed=3).cuda()
    buf = 320
    codes8 = torch.zeros(2, 8, buf, 128, dtype=torch.int8, device="cuda")
    sc8 = torch.zeros(2, 8, buf, dtype=torch.float16, device="cuda")
    codes4 = torch.zeros(2, 8, buf, 64, dtype=torch.int8, device="cuda")
    sc4 = torch.zeros(2, 8, buf, dtype=torch.float16, device="cuda")
    kq = torch.zeros(2, 8, buf, 64, dtype=torch.int8, device="cuda")
    ks = torch.zeros(2, 8, buf // 32, 128, dtype=torch.float16, device="cuda")
    kz = torch.zeros_like(ks)
    for pos in range(0, 256, 64):
        chunk = x[:, :, pos:pos + 64].contiguous()
        L.quantize_per_token_into(chunk, codes8, sc8, pos)
        L.quantize_v_per_token_int4_into(chunk, codes4, sc4, pos)
        L.quantize_k_per_channel_groupwise_int4_into(chunk, kq, ks, 32, pos, kz)
    q, s = L.quantize_per_token(x)
    assert torch.equal(codes8[:, :, :256], q) and torch.equal(sc8[:, :, :256], s)
    q, s = L.quantize_v_per_token_int4(x)
    assert torch.equal(codes4[:, :, :256], q) and torch.equal(sc4[:, :, :256], s)
    q, s, z = L.quantize_k_per_channel_groupwise_int4_asym(x, 32)
    assert torch.equal(kq[:, :, :256], q) and torch.equal(ks[:, :, :8], s) and torch.equal(kz[:, :, :8], z)
    assert (codes8[:, :, 256:] == 0).all()   # nothing written past the appended rows


def test_cabi_direct_quantize(L):
    """The same kernel through the raw C ABI (ctypes, device pointers)."""
    from llmik_cuda import cabi
    x = _x(1, 33, seed=11).cuda()
    q = torch.empty(1, 8, 33, 128, dtype=torch.int8, device="cuda")
    s = torch.empty(1, 8, 33, dtype=torch.float16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    cabi.call("lik_quantize_per_token_int8", x.data_ptr(), q.data_ptr(), s.data_ptr(), 1, 8, 33, 128, 0, 33,
              stream)
    torch.cuda.synchronize()
    rq, rs = O.quantize_per_token(x.cpu().numpy(), 8)
    np.testing.assert_array_equal(q.cpu().numpy(), rq)
    np.testing.assert_array_equal(s.cpu().numpy(), rs.astype(np.float16))
