"""The append-in-place quantized cache (llmik_cuda.cache) against a restatement
of the reference's cat-based INT4 KIVI cache (integration/kv_int4_cache.py)
driven by the same token stream: identical codes and scales, identical
attention outputs and identical materialized fp16 KV, with no torch.cat and no
reallocation of the cache."""
import math

import numpy as np
import pytest
import torch

from lik_testutil import assert_attn_close
from oracle import kv_oracle as O

pytestmark = pytest.mark.gpu
SCALE = 1.0 / math.sqrt(128)


@pytest.fixture(scope="module")
def L():
    import llmik_cuda
    return llmik_cuda


class CatKIVICache:
    """Function-level restatement of Int4KIVICache (integration/kv_int4_cache.py):
    fp16 residual grown with torch.cat (:115-122), full groups drained into
    packed storage grown with torch.cat (:125-147), residual quantized on the
    fly before attention (:174-206), fp16 materialize (:226-245)."""

    def __init__(self, L, gs, asym=False):
        self.L, self.gs, self.asym = L, gs, asym
        self.q = None      # list of storage tensors (k_q, k_s, v_q, v_s[, k_z, v_z])
        self.kr = self.vr = None

    def _qk(self, x):
        if self.asym:
            return self.L.quantize_k_per_channel_groupwise_int4_asym(x, self.gs)
        return self.L.quantize_k_per_channel_groupwise_int4(x, self.gs)

    def _qv(self, x):
        if self.asym:
            return self.L.quantize_v_per_token_int4_asym(x)
        return self.L.quantize_v_per_token_int4(x)

    def _store(self, kq, vq):
        parts = (kq[0], kq[1], vq[0], vq[1]) + ((kq[2], vq[2]) if self.asym else ())
        return parts

    def append(self, k, v):
        self.kr = k if self.kr is None else torch.cat([self.kr, k], dim=2)
        self.vr = v if self.vr is None else torch.cat([self.vr, v], dim=2)
        while self.kr.shape[2] >= self.gs:
            ck = self.kr[:, :, :self.gs].contiguous()
            cv = self.vr[:, :, :self.gs].contiguous()
            new = self._store(self._qk(ck), self._qv(cv))
            self.q = list(new) if self.q is None else [torch.cat([a, b], dim=2) for a, b in zip(self.q, new)]
            self.kr = self.kr[:, :, self.gs:]
            self.vr = self.vr[:, :, self.gs:]

    def quantized(self):
        if self.kr is None or self.kr.shape[2] == 0:
            return self.q
        new = self._store(self._qk(self.kr.contiguous()), self._qv(self.vr.contiguous()))
        if self.q is None:
            return list(new)
        return [torch.cat([a, b], dim=2) for a, b in zip(self.q, new)]

    def attend(self, q):
        t = self.quantized()
        if self.asym:
            return self.L.decode_attention_int4_asym(q, t[0], t[1], t[4], t[2], t[3], t[5], self.gs, SCALE)
        return self.L.decode_attention_int4(q, t[0], t[1], t[2], t[3], self.gs, SCALE)

    def materialize(self):
        ks, vs = [], []
        if self.q is not None:
            t = [x.cpu().numpy() for x in self.q]
            if self.asym:
                k, v = O.dequant_kivi_asym_to_f16(t[0], t[1], t[4], t[2], t[3], t[5], self.gs)
            else:
                k, v = O.dequant_kivi_sym_to_f16(t[0], t[1], t[2], t[3], self.gs)
            ks.append(torch.from_numpy(k))
            vs.append(torch.from_numpy(v))
        if self.kr is not None and self.kr.shape[2]:
            ks.append(self.kr.cpu())
            vs.append(self.vr.cpu())
        return torch.cat(ks, dim=2), torch.cat(vs, dim=2)


@pytest.mark.parametrize("fmt,gs", [("int4", 32), ("int4", 128), ("int4_asym", 128), ("int4", 7)])
def test_kivi_cache_matches_cat_based_reference(L, fmt, gs):
    from llmik_cuda.cache import QuantizedKVCache
    asym = fmt == "int4_asym"
    B, H, HQ = 2, 8, 32
    g = torch.Generator(device="cuda").manual_seed(gs)
    cache = QuantizedKVCache(B, H, max_len=600, fmt=fmt, group_size=gs)
    ref = CatKIVICache(L, gs, asym)
    buf_k = cache.layers[0].k
    # prefill of 300 positions, then 45 single-token decode steps
    chunks = [300] + [1] * 45
    for step, n in enumerate(chunks):
        k = torch.randn(B, H, n, 128, generator=g, device="cuda").half()
        v = torch.randn(B, H, n, 128, generator=g, device="cuda").half()
        cache.append(k, v)
        ref.append(k, v)
        q = torch.randn(B, HQ, 128, generator=g, device="cuda").half()
        out = cache.attend(q, SCALE)
        out_ref = ref.attend(q)
        assert torch.equal(out, out_ref), f"attention differs at step {step}"
        if step in (0, 7, 44):
            view = cache.quantized_view()
            t = ref.quantized()
            for a, b in zip(view, t):
                assert torch.equal(a, b)
            km, vm = cache.materialize_fp16()
            kr, vr = ref.materialize()
            assert torch.equal(km.cpu(), kr) and torch.equal(vm.cpu(), vr)
    assert cache.layers[0].k.data_ptr() == buf_k.data_ptr()   # never reallocated
    assert cache.seq_length() == 345


@pytest.mark.parametrize("fmt", ["int8", "fp16"])
def test_int8_and_fp16_cache_against_oracle(L, fmt):
    from llmik_cuda.cache import QuantizedKVCache
    B, H, HQ = 3, 8, 32
    g = torch.Generator().manual_seed(1)
    cache = QuantizedKVCache(B, H, max_len=400, fmt=fmt)
    ks, vs = [], []
    for n in (257, 1, 1, 30):
        k = torch.randn(B, H, n, 128, generator=g).half()
        v = torch.randn(B, H, n, 128, generator=g).half()
        ks.append(k)
        vs.append(v)
        cache.append(k.cuda(), v.cuda())
    q = torch.randn(B, HQ, 128, generator=g).half()
    out = cache.attend(q.cuda(), SCALE).float().cpu().numpy()
    k, v = torch.cat(ks, 2).numpy(), torch.cat(vs, 2).numpy()
    if fmt == "int8":
        kq, kscale, vq, vscale = O.quantize_kv_int8_per_token(k, v)
        k16, v16 = O.dequant_int8_to_f16(kq, kscale.astype(np.float16), vq, vscale.astype(np.float16))
        km, vm = cache.materialize_fp16()
        np.testing.assert_array_equal(km.cpu().numpy(), k16)
        np.testing.assert_array_equal(vm.cpu().numpy(), v16)
        k, v = O.dequant_int8_exact(kq, kscale.astype(np.float16), vq, vscale.astype(np.float16))
    assert_attn_close(out, O.decode_attention(q.numpy(), k, v, SCALE))


def test_dequantize_ops_bit_exact(L):
    g = torch.Generator().manual_seed(3)
    k = torch.randn(2, 8, 300, 128, generator=g).half()
    v = torch.randn(2, 8, 300, 128, generator=g).half()
    kc, vc = k.cuda(), v.cuda()
    kq, ks = L.quantize_per_token(kc)
    vq, vs = L.quantize_per_token(vc)
    km, vm = L.dequantize_int8(kq, ks, vq, vs, 250)
    rk, rv = O.dequant_int8_to_f16(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(), vs.cpu().numpy())
    np.testing.assert_array_equal(km.cpu().numpy(), rk[:, :, :250])
    np.testing.assert_array_equal(vm.cpu().numpy(), rv[:, :, :250])
    for gs in (32, 7):
        kq, ks = L.quantize_k_per_channel_groupwise_int4(kc, gs)
        vq, vs = L.quantize_v_per_token_int4(vc)
        km, vm = L.dequantize_int4(kq, ks, vq, vs, gs)
        rk, rv = O.dequant_kivi_sym_to_f16(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(), vs.cpu().numpy(), gs)
        np.testing.assert_array_equal(km.cpu().numpy(), rk)
        np.testing.assert_array_equal(vm.cpu().numpy(), rv)
        kq, ks, kz = L.quantize_k_per_channel_groupwise_int4_asym(kc, gs)
        vq, vs, vz = L.quantize_v_per_token_int4_asym(vc)
        km, vm = L.dequantize_int4(kq, ks, vq, vs, gs, -1, kz, vz)
        rk, rv = O.dequant_kivi_asym_to_f16(kq.cpu().numpy(), ks.cpu().numpy(), kz.cpu().numpy(),
                                            vq.cpu().numpy(), vs.cpu().numpy(), vz.cpu().numpy(), gs)
        np.testing.assert_array_equal(km.cpu().numpy(), rk)
        np.testing.assert_array_equal(vm.cpu().numpy(), rv)


def test_dequantize_int4_with_unaligned_group_scales(L):
    """K group scales / zeros that do not start on a 16-byte boundary (a view
    one element into a larger buffer) take the per-channel load path and give
    the same fp16 values."""
    g = torch.Generator().manual_seed(4)
    k = torch.randn(1, 8, 200, 128, generator=g).half().cuda()
    v = torch.randn(1, 8, 200, 128, generator=g).half().cuda()
    kq, ks, kz = L.quantize_k_per_channel_groupwise_int4_asym(k, 32)
    vq, vs, vz = L.quantize_v_per_token_int4_asym(v)

    def shifted(t):
        buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
        view = buf[1:].view(t.shape)
        view.copy_(t)
        assert view.data_ptr() % 16 != 0
        return view

    ref = L.dequantize_int4(kq, ks, vq, vs, 32, -1, kz, vz)
    got = L.dequantize_int4(kq, shifted(ks), vq, vs, 32, -1, shifted(kz), vz)
    assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])
