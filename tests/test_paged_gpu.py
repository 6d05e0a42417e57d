"""Paged KV decode (block tables, ragged per-sequence lengths) for every KV
format, against the fp32 oracle on each sequence's own live positions."""
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


def _pagify(x, lens, bs, perm, n_blocks):
    """[B, H, S, ...] contiguous -> [n_blocks, H, bs, ...] pages (unused rows garbage)."""
    B, H = x.shape[:2]
    rest = x.shape[3:]
    pages = torch.full((n_blocks, H, bs) + tuple(rest), 7, dtype=x.dtype, device=x.device)
    if x.dtype == torch.float16:
        pages.fill_(float("nan"))
    table = torch.zeros(B, max(-(-int(l) // bs) for l in lens), dtype=torch.int32)
    k = 0
    for b in range(B):
        for blk in range(-(-int(lens[b]) // bs)):
            page = perm[k]
            k += 1
            seg = x[b, :, blk * bs:(blk + 1) * bs]
            pages[page, :, :seg.shape[1]] = seg
            table[b, blk] = page
    return pages, table


def _groups_pagify(s, lens, bs, gs, table):
    """K group scales [B, H, ng, 128] -> [n_blocks, H, bs/gs, 128] following table."""
    n_blocks = int(table.max()) + 1
    out = torch.ones((n_blocks, s.shape[1], bs // gs, 128), dtype=s.dtype, device=s.device)
    for b in range(s.shape[0]):
        for blk in range(-(-int(lens[b]) // bs)):
            g = s[b, :, blk * bs // gs:(blk + 1) * bs // gs]
            out[int(table[b, blk]), :, :g.shape[1]] = g
    return out


@pytest.mark.parametrize("fmt", ["f16", "int8", "int4", "int4_asym"])
@pytest.mark.parametrize("bs,gs", [(16, 16), (64, 32), (256, 128)])
def test_paged_matches_oracle(L, fmt, bs, gs):
    g = torch.Generator().manual_seed(bs + gs)
    B, H, HQ = 5, 8, 32
    lens = [1, 97, 600, 257, 4 * bs]
    S = max(lens)
    n_blocks = sum(-(-l // bs) for l in lens) + 3
    perm = torch.randperm(n_blocks, generator=g).tolist()
    q = torch.randn(B, HQ, 128, generator=g).half()
    k = torch.randn(B, H, S, 128, generator=g).half()
    v = torch.randn(B, H, S, 128, generator=g).half()
    kc, vc = k.cuda(), v.cuda()
    ctx = torch.tensor(lens, dtype=torch.int32).cuda()
    kw = {}
    if fmt == "f16":
        kp, table = _pagify(kc, lens, bs, perm, n_blocks)
        vp, _ = _pagify(vc, lens, bs, perm, n_blocks)
        kd, vd = k.numpy(), v.numpy()
    elif fmt == "int8":
        kq, ks = L.quantize_per_token(kc)
        vq, vs = L.quantize_per_token(vc)
        kp, table = _pagify(kq, lens, bs, perm, n_blocks)
        vp, _ = _pagify(vq, lens, bs, perm, n_blocks)
        kw = dict(k_scale=_pagify(ks, lens, bs, perm, n_blocks)[0], v_scale=_pagify(vs, lens, bs, perm, n_blocks)[0])
        kd, vd = O.dequant_int8_to_f16(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(), vs.cpu().numpy())
    else:
        asym = fmt == "int4_asym"
        if asym:
            kq, ks, kz = L.quantize_k_per_channel_groupwise_int4_asym(kc, gs)
            vq, vs, vz = L.quantize_v_per_token_int4_asym(vc)
        else:
            kq, ks = L.quantize_k_per_channel_groupwise_int4(kc, gs)
            vq, vs = L.quantize_v_per_token_int4(vc)
        kp, table = _pagify(kq, lens, bs, perm, n_blocks)
        vp, _ = _pagify(vq, lens, bs, perm, n_blocks)
        kw = dict(k_scale=_groups_pagify(ks, lens, bs, gs, table), v_scale=_pagify(vs, lens, bs, perm, n_blocks)[0],
                  group_size=gs)
        if asym:
            kw.update(k_zero=_groups_pagify(kz, lens, bs, gs, table), v_zero=_pagify(vz, lens, bs, perm, n_blocks)[0])
            kd, vd = O.dequant_kivi_asym_to_f16(kq.cpu().numpy(), ks.cpu().numpy(), kz.cpu().numpy(),
                                                vq.cpu().numpy(), vs.cpu().numpy(), vz.cpu().numpy(), gs)
        else:
            kd, vd = O.dequant_kivi_sym_to_f16(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(),
                                               vs.cpu().numpy(), gs)
    out = L.paged_decode_attention(q.cuda(), kp, vp, table.cuda(), ctx, SCALE, S, **kw).float().cpu().numpy()
    assert np.isfinite(out).all()
    for b, l in enumerate(lens):
        ref = O.decode_attention(q[b:b + 1].numpy(), kd[b:b + 1], vd[b:b + 1], SCALE, seqlen=l)
        assert_attn_close(out[b:b + 1], ref)
