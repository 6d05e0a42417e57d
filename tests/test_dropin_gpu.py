"""The reference's decode call sequences, run on the GPU against llmik_cuda.

The reference's integration modules cannot be imported on the GPU box (they
live in the reference checkout and need its transformers version), so each
test restates the call sequence of one caller in test code and drives the new
library through it:

* the patched SDPA of ``integration/attention_patch.py:44-69`` (un-expand the
  repeat_kv heads, squeeze the query, ``decode_attention``, unsqueeze; prefill
  falls through to the stock SDPA);
* the INT4 decode forward of ``integration/attention_patch.py:233-243``:
  ``append_only(k, v, layer_idx)`` -> ``get_quantized_for_attention(layer_idx)``
  -> ``decode_attention_int4(q, k_packed, k_scale, v_packed, v_scale,
  group_size, scale)``, once on a cat-based restatement of ``Int4KIVICache``
  (integration/kv_int4_cache.py:101-206) and once on ``QuantizedKVCache``;
* the ``v6_decode`` hook of ``integration/prealloc_cache.py:91-99``: the cache's
  ``update`` returns the whole preallocated buffers at decode time and the hook
  attends over ``cache.cur_attn_len`` positions.
"""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from lik_testutil import assert_attn_close, attn_kv_int8, attn_kv_kivi_asym, attn_kv_kivi_sym
from oracle import kv_oracle as O
from test_cache_gpu import CatKIVICache

pytestmark = pytest.mark.gpu
D = 128
SCALE = 1.0 / math.sqrt(D)


@pytest.fixture(scope="module")
def L():
    import llmik_cuda
    return llmik_cuda


def repeat_kv(x, n_rep):
    """transformers' repeat_kv: each kv head repeated n_rep times in place."""
    b, h, s, d = x.shape
    return x[:, :, None].expand(b, h, n_rep, s, d).reshape(b, h * n_rep, s, d)


def make_decode_sdpa(L, n_kv_heads):
    """The patched SDPA's behaviour: q_len 1 goes to decode_attention over
    the un-expanded kv heads; anything else to the stock SDPA."""

    def patched(query, key, value, *args, **kwargs):
        if query.dim() != 4 or query.size(2) != 1:
            return F.scaled_dot_product_attention(query, key, value, *args, **kwargs)
        n_rep = query.size(1) // n_kv_heads
        k = key[:, ::n_rep].contiguous()
        v = value[:, ::n_rep].contiguous()
        out = L.decode_attention(query.squeeze(2).contiguous(), k, v, 1.0 / math.sqrt(query.size(-1)))
        return out.unsqueeze(2)

    return patched


@pytest.mark.parametrize("b,hq,hkv,s", [(2, 32, 8, 777), (1, 32, 32, 100), (3, 16, 2, 4096)])
def test_patched_sdpa_decode_and_prefill(L, b, hq, hkv, s):
    g = torch.Generator(device="cuda").manual_seed(s)
    q = torch.randn(b, hq, 1, D, generator=g, device="cuda").half()
    k = torch.randn(b, hkv, s, D, generator=g, device="cuda").half()
    v = torch.randn(b, hkv, s, D, generator=g, device="cuda").half()
    n_rep = hq // hkv
    sdpa = make_decode_sdpa(L, hkv)
    out = sdpa(q, repeat_kv(k, n_rep), repeat_kv(v, n_rep))
    assert out.shape == (b, hq, 1, D) and out.dtype == torch.float16
    ref = O.decode_attention(q.squeeze(2).cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), SCALE)
    assert_attn_close(out.squeeze(2).cpu().numpy(), ref)
    # the stock path the patch replaces, in fp32 on the expanded heads
    stock = F.scaled_dot_product_attention(q.float(), repeat_kv(k, n_rep).float(), repeat_kv(v, n_rep).float())
    assert_attn_close(out.float().cpu().numpy(), stock.cpu().numpy())
    # prefill (q_len > 1) is not touched
    qp = torch.randn(b, hq, 4, D, generator=g, device="cuda").half()
    kp, vp = repeat_kv(k[:, :, :4], n_rep), repeat_kv(v[:, :, :4], n_rep)
    assert torch.equal(sdpa(qp, kp, vp, is_causal=True), F.scaled_dot_product_attention(qp, kp, vp, is_causal=True))


def _int4_call(L, t, q, gs, asym):
    """decode_attention_int4(_asym) with the reference's positional arguments
    (no live length) on a get_quantized_for_attention tuple
    (k, k_scale, v, v_scale[, k_zero, v_zero])."""
    if asym:
        return L.decode_attention_int4_asym(q, t[0], t[1], t[4], t[2], t[3], t[5], gs, SCALE)
    return L.decode_attention_int4(q, t[0], t[1], t[2], t[3], gs, SCALE)


@pytest.mark.parametrize("fmt,gs", [("int4", 32), ("int4", 128), ("int4_asym", 128), ("int4", 7)])
def test_int4_decode_forward_sequence(L, fmt, gs):
    from llmik_cuda.cache import QuantizedKVCache
    asym = fmt == "int4_asym"
    B, HKV, HQ, layer = 2, 8, 32, 1
    g = torch.Generator(device="cuda").manual_seed(100 + gs)
    cache = QuantizedKVCache(B, HKV, max_len=512, fmt=fmt, group_size=gs, num_layers=2)
    ref = CatKIVICache(L, gs, asym)
    k = torch.randn(B, HKV, 130, D, generator=g, device="cuda").half()
    v = torch.randn(B, HKV, 130, D, generator=g, device="cuda").half()
    cache.append_only(k, v, layer)      # prefill
    ref.append(k, v)
    for step in range(40):
        k1 = torch.randn(B, HKV, 1, D, generator=g, device="cuda").half()
        v1 = torch.randn(B, HKV, 1, D, generator=g, device="cuda").half()
        q = torch.randn(B, HQ, 1, D, generator=g, device="cuda").half()
        cache.append_only(k1.contiguous(), v1.contiguous(), layer)
        ref.append(k1, v1)
        t = cache.get_quantized_for_attention(layer)
        tr = ref.quantized()
        assert cache.get_seq_length(layer) == 131 + step == t[0].shape[2]
        for a, b in zip(t, tr):
            assert torch.equal(a, b)
        q_flat = q.squeeze(2).contiguous()
        out = _int4_call(L, t, q_flat, gs, asym)
        # the cat-based cache's contiguous tensors give the same bits
        assert torch.equal(out, _int4_call(L, tr, q_flat, gs, asym))
        if step % 13 == 0:
            n = [x.cpu().numpy() for x in tr]
            if asym:
                kk, vv = attn_kv_kivi_asym(n[0], n[1], n[4], n[2], n[3], n[5], gs)
            else:
                kk, vv = attn_kv_kivi_sym(n[0], n[1], n[2], n[3], gs)
            assert_attn_close(out.cpu().numpy(), O.decode_attention(q_flat.cpu().numpy(), kk, vv, SCALE))
    # update() keeps the HF contract: fp16 K/V of every stored position
    kf, vf = cache.update(k1, v1, layer)
    assert kf.shape == (B, HKV, 171, D) and vf.dtype == torch.float16


def test_int8_quantized_views_feed_the_int8_op(L):
    from llmik_cuda.cache import QuantizedKVCache
    B, HKV, HQ = 3, 4, 16
    g = torch.Generator(device="cuda").manual_seed(8)
    cache = QuantizedKVCache(B, HKV, max_len=1000, fmt="int8")
    k = torch.randn(B, HKV, 333, D, generator=g, device="cuda").half()
    v = torch.randn(B, HKV, 333, D, generator=g, device="cuda").half()
    cache.append_only(k, v, 0)
    q = torch.randn(B, HQ, D, generator=g, device="cuda").half()
    kq, ks, vq, vs = cache.get_quantized_for_attention(0)
    assert not kq.is_contiguous()       # prefix views of the 1000-position buffers
    out = L.decode_attention_int8(q, kq, ks, vq, vs, SCALE)
    assert torch.equal(out, L.decode_attention_int8(q, kq.contiguous(), ks.contiguous(), vq.contiguous(),
                                                    vs.contiguous(), SCALE))
    kk, vv = attn_kv_int8(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(), vs.cpu().numpy())
    assert_attn_close(out.cpu().numpy(), O.decode_attention(q.cpu().numpy(), kk, vv, SCALE))


def test_views_of_other_layouts_are_rejected(L):
    q = torch.zeros(1, 8, D, dtype=torch.float16, device="cuda")
    k = torch.zeros(1, 2, 64, D, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="prefix of a contiguous buffer|contiguous"):
        L.decode_attention(q, k[:, :, ::2], k[:, :, ::2], SCALE)
    with pytest.raises(RuntimeError, match="contiguous"):
        L.decode_attention(q, k.transpose(1, 2).contiguous().transpose(1, 2), k, SCALE)
    kb = torch.zeros(1, 2, 128, D, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="another length"):
        L.decode_attention(q, k, kb[:, :, :64], SCALE)


def test_v6_decode_hook_over_the_live_length(L):
    """PreallocCache + v6_decode: decode-time update returns the whole
    buffers (NaN past the live prefix); the hook passes cur_attn_len."""
    from llmik_cuda.cache import QuantizedKVCache
    B, HKV, HQ, MAX = 2, 8, 32, 700
    g = torch.Generator(device="cuda").manual_seed(6)
    cache = QuantizedKVCache(B, HKV, max_len=MAX, fmt="fp16", num_layers=2)
    for lay in cache.layers:
        lay.k.fill_(float("nan"))
        lay.v.fill_(float("nan"))

    def hook(query, key, value):
        if query.size(2) > 1:
            n_rep = query.size(1) // key.size(1)
            return F.scaled_dot_product_attention(query, repeat_kv(key, n_rep), repeat_kv(value, n_rep))
        out = L.decode_attention(query.squeeze(2).contiguous(), key, value,
                                 1.0 / math.sqrt(query.size(-1)), cache.cur_attn_len)
        return out.unsqueeze(2)

    kp = torch.randn(B, HKV, 257, D, generator=g, device="cuda").half()
    vp = torch.randn(B, HKV, 257, D, generator=g, device="cuda").half()
    for lay in range(2):
        kr, vr = cache.update(kp, vp, lay)
        assert kr is kp and vr is vp                  # prefill returns its own K/V
    ks, vs = [kp], [vp]
    for step in range(20):
        k1 = torch.randn(B, HKV, 1, D, generator=g, device="cuda").half()
        v1 = torch.randn(B, HKV, 1, D, generator=g, device="cuda").half()
        ks.append(k1)
        vs.append(v1)
        for lay in range(2):
            key, value = cache.update(k1, v1, lay)
            assert key.shape[2] == MAX and cache.cur_attn_len == 258 + step
            q = torch.randn(B, HQ, 1, D, generator=g, device="cuda").half()
            out = hook(q, key, value)
            if step % 7 == 0:
                kk, vv = torch.cat(ks, 2).cpu().numpy(), torch.cat(vs, 2).cpu().numpy()
                ref = O.decode_attention(q.squeeze(2).cpu().numpy(), kk, vv, SCALE)
                assert np.isfinite(out.float().cpu().numpy()).all()
                assert_attn_close(out.squeeze(2).cpu().numpy(), ref)
