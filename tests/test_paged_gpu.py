"""Paged KV decode (block tables, ragged per-sequence lengths) for every KV
format, against the fp32 oracle on each sequence's own live positions."""
import math

import numpy as np
import pytest
import torch

from lik_testutil import assert_attn_close, attn_kv_int8, attn_kv_kivi_asym, attn_kv_kivi_sym
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
        kd, vd = attn_kv_int8(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(), vs.cpu().numpy())
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
            kd, vd = attn_kv_kivi_asym(kq.cpu().numpy(), ks.cpu().numpy(), kz.cpu().numpy(),
                                                vq.cpu().numpy(), vs.cpu().numpy(), vz.cpu().numpy(), gs)
        else:
            kd, vd = attn_kv_kivi_sym(kq.cpu().numpy(), ks.cpu().numpy(), vq.cpu().numpy(),
                                               vs.cpu().numpy(), gs)
    out = L.paged_decode_attention(q.cuda(), kp, vp, table.cuda(), ctx, SCALE, S, **kw).float().cpu().numpy()
    assert np.isfinite(out).all()
    for b, l in enumerate(lens):
        ref = O.decode_attention(q[b:b + 1].numpy(), kd[b:b + 1], vd[b:b + 1], SCALE, seqlen=l)
        assert_attn_close(out[b:b + 1], ref)


def _contig_rows(L, fmt, x):
    """Reference rows for x [n_tokens, H, 128]: the contiguous quantizers run on
    x viewed as one sequence [1, H, n_tokens, 128]; returns per-(token, head)
    codes / scale / zero laid out [n_tokens, H, ...]."""
    xc = x.permute(1, 0, 2).unsqueeze(0).contiguous()
    if fmt == "f16":
        return (x,)
    if fmt == "int8":
        q, s = L.quantize_per_token(xc)
        return q[0].permute(1, 0, 2), s[0].permute(1, 0)
    if fmt == "int4":
        q, s = L.quantize_v_per_token_int4(xc)
        return q[0].permute(1, 0, 2), s[0].permute(1, 0)
    q, s, z = L.quantize_v_per_token_int4_asym(xc)
    return q[0].permute(1, 0, 2), s[0].permute(1, 0), z[0].permute(1, 0)


@pytest.mark.parametrize("fmt", ["f16", "int8", "int4", "int4_asym"])
def test_paged_append_matches_contiguous_quantizers(L, fmt):
    """Tokens appended through a scrambled slot mapping (with padding slots)
    land in the right block rows with the contiguous quantizers' codes,
    scales and zeros; rows no slot names stay untouched."""
    g = torch.Generator().manual_seed(11)
    T, H, bs, nb = 45, 8, 16, 6
    x = torch.randn(T, H, 128, generator=g).half().cuda()
    x[3, 2, 5] = 40.0                              # an outlier row
    slots = torch.randperm(nb * bs, generator=g)[:T].clone()
    slots[[4, 17, 30]] = -1                        # padding tokens
    slots_d = slots.cuda()
    row = 128 if fmt in ("f16", "int8") else 64
    dt = torch.float16 if fmt == "f16" else torch.int8
    cache = torch.full((nb, H, bs, row), 3, dtype=dt, device="cuda")
    scale = torch.full((nb, H, bs), 9.0, dtype=torch.float16, device="cuda") if fmt != "f16" else None
    zero = torch.full((nb, H, bs), 9.0, dtype=torch.float16, device="cuda") if fmt == "int4_asym" else None
    before = cache.clone()
    L.paged_append(x, slots_d, cache, scale, zero)
    ref = _contig_rows(L, fmt, x)
    written = torch.zeros(nb, bs, dtype=torch.bool)
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        blk, off = divmod(s, bs)
        written[blk, off] = True
        assert torch.equal(cache[blk, :, off], ref[0][t])
        if scale is not None:
            assert torch.equal(scale[blk, :, off], ref[1][t])
        if zero is not None:
            assert torch.equal(zero[blk, :, off], ref[2][t])
    untouched = ~written.cuda()
    assert torch.equal(cache.permute(0, 2, 1, 3)[untouched], before.permute(0, 2, 1, 3)[untouched])


def test_paged_append_then_decode(L):
    """A paged INT8 cache filled by paged_append (prefill, then one decode
    token per sequence) attends like the oracle over the dequantized rows."""
    g = torch.Generator().manual_seed(12)
    B, H, HQ, bs = 3, 8, 32, 16
    lens = [40, 1, 77]
    n_blocks = sum(-(-(l + 1) // bs) for l in lens) + 2
    perm = torch.randperm(n_blocks, generator=g).tolist()
    maxb = max(-(-(l + 1) // bs) for l in lens)
    table = torch.zeros(B, maxb, dtype=torch.int32)
    k = 0
    for b, l in enumerate(lens):
        for blk in range(-(-(l + 1) // bs)):
            table[b, blk] = perm[k]
            k += 1
    kc = torch.zeros(n_blocks, H, bs, 128, dtype=torch.int8, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.ones(n_blocks, H, bs, dtype=torch.float16, device="cuda")
    vs = torch.ones_like(ks)
    seqs = [torch.randn(l + 1, H, 128, generator=g).half() for l in lens]   # prefill + 1 new token

    def slots_for(b, t0, t1):
        return torch.tensor([int(table[b, t // bs]) * bs + t % bs for t in range(t0, t1)], dtype=torch.int64)

    for phase in ("prefill", "decode"):
        for b, l in enumerate(lens):
            t0, t1 = (0, l) if phase == "prefill" else (l, l + 1)
            xk = seqs[b][t0:t1].cuda()
            sl = slots_for(b, t0, t1).cuda()
            L.paged_append(xk, sl, kc, ks)
            L.paged_append(xk.flip(2).contiguous(), sl, vc, vs)   # V = K reversed along channels
    q = torch.randn(B, HQ, 128, generator=g).half()
    ctx = torch.tensor([l + 1 for l in lens], dtype=torch.int32)
    out = L.paged_decode_attention(q.cuda(), kc, vc, table.cuda(), ctx.cuda(), SCALE, max(lens) + 1,
                                   k_scale=ks, v_scale=vs)
    for b, l in enumerate(lens):
        xb = seqs[b].permute(1, 0, 2).unsqueeze(0).numpy()           # [1, H, l+1, 128]
        kq, kscale = O.quantize_per_token(xb, 8)
        vq, vscale = O.quantize_per_token(np.ascontiguousarray(xb[..., ::-1]), 8)
        kd, vd = attn_kv_int8(kq, kscale.astype(np.float16), vq, vscale.astype(np.float16))
        ref = O.decode_attention(q[b:b + 1].numpy(), kd, vd, SCALE)
        assert_attn_close(out[b:b + 1].cpu().numpy(), ref)


@pytest.mark.parametrize("fmt", ["f16", "int4_asym"])
def test_out_of_range_block_entry_is_masked_and_reported(L, fmt):
    """A block-table entry outside [0, num_blocks) is never read through: the
    tile holding it is masked, the workspace error word records it and
    check_device_errors() raises (and resets the workspace); other sequences
    are unaffected and the next call is clean."""
    g = torch.Generator().manual_seed(3)
    B, H, HQ, bs, gs = 2, 8, 32, 64, 64
    lens = [300, 300]
    n_blocks = 10
    q = torch.randn(B, HQ, 128, generator=g).half()
    k = torch.randn(B, H, 320, 128, generator=g).half()
    v = torch.randn(B, H, 320, 128, generator=g).half()
    perm = list(range(n_blocks))
    ctx = torch.tensor(lens, dtype=torch.int32).cuda()
    kw = {}
    if fmt == "f16":
        kp, table = _pagify(k.cuda(), lens, bs, perm, n_blocks)
        vp, _ = _pagify(v.cuda(), lens, bs, perm, n_blocks)
        kd, vd = k.numpy(), v.numpy()
    else:
        kq, ks, kz = L.quantize_k_per_channel_groupwise_int4_asym(k.cuda(), gs)
        vq, vs, vz = L.quantize_v_per_token_int4_asym(v.cuda())
        kp, table = _pagify(kq, lens, bs, perm, n_blocks)
        vp, _ = _pagify(vq, lens, bs, perm, n_blocks)
        kw = dict(k_scale=_groups_pagify(ks, lens, bs, gs, table), v_scale=_pagify(vs, lens, bs, perm, n_blocks)[0],
                  group_size=gs, k_zero=_groups_pagify(kz, lens, bs, gs, table),
                  v_zero=_pagify(vz, lens, bs, perm, n_blocks)[0])
        kd, vd = attn_kv_kivi_asym(kq.cpu().numpy(), ks.cpu().numpy(), kz.cpu().numpy(),
                                            vq.cpu().numpy(), vs.cpu().numpy(), vz.cpu().numpy(), gs)
    L.check_device_errors()  # clean before
    bad = table.clone()
    bad[1, 1] = 1 << 20   # far past the cache
    bad[1, 3] = -5
    out = L.paged_decode_attention(q.cuda(), kp, vp, bad.cuda(), ctx, SCALE, max(lens), **kw).float().cpu().numpy()
    ref0 = O.decode_attention(q[:1].numpy(), kd[:1], vd[:1], SCALE, seqlen=lens[0])
    assert_attn_close(out[:1], ref0)
    with pytest.raises(RuntimeError, match="block-table"):
        L.check_device_errors()
    L.check_device_errors()  # reset: clean again
    out = L.paged_decode_attention(q.cuda(), kp, vp, table.cuda(), ctx, SCALE, max(lens), **kw).float().cpu().numpy()
    for b in range(B):
        assert_attn_close(out[b:b + 1], O.decode_attention(q[b:b + 1].numpy(), kd[b:b + 1], vd[b:b + 1], SCALE,
                                                           seqlen=lens[b]))
    L.check_device_errors()


def test_check_device_errors_reports_and_resets_a_timeout(L):
    """A kernel whose bounded wait ran out leaves the timeout code and a stale
    unit counter in the stream's workspace (emulated by a self-test kernel
    whose own wait runs out; no GPU fault). check_device_errors() raises once,
    resets the workspace, and decode results are right afterwards."""
    g = torch.Generator().manual_seed(4)
    q = torch.randn(2, 32, 128, generator=g).half().cuda()
    k = torch.randn(2, 8, 1000, 128, generator=g).half().cuda()
    v = torch.randn(2, 8, 1000, 128, generator=g).half().cuda()
    L.decode_attention(q, k, v, SCALE)
    L.check_device_errors()
    L._C._selftest_leave_timeout()
    with pytest.raises(RuntimeError, match="wait expired"):
        L.check_device_errors()
    L.check_device_errors()
    out = L.decode_attention(q, k, v, SCALE).float().cpu().numpy()
    assert_attn_close(out, O.decode_attention(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), SCALE))
