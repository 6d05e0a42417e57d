"""Preallocated, append-in-place quantized KV cache for decode.

Replaces the caller side of the reference's INT4 decode path,
``Int4KIVICache`` (integration/kv_int4_cache.py:70-245), which grows its packed
tensors with ``torch.cat`` on every drained group (:137-144) and re-concatenates
the whole cache with the re-quantized residual on every decode step
(:174-206). Here every layer owns fixed buffers of ``max_len`` positions; new
tokens are quantized straight into place by the CUDA append kernels and
attention reads the live prefix through the kernels' ``seqlen`` argument, so a
decode step costs two or three small kernel launches plus the attention
kernel, independent of the cache length.

Formats:

* ``"int4"``      - KIVI, reference symmetric format: K per channel over groups
  of ``group_size`` positions, V per token, signed nibbles;
* ``"int4_asym"`` - KIVI with scale + zero point (unsigned nibbles);
* ``"int8"``      - symmetric INT8 per token for K and V;
* ``"fp16"``      - unquantized (the reference's ``PreallocCache``,
  integration/prealloc_cache.py:42-78).

INT4 K needs ``group_size`` positions to form a group. Positions of the
current, incomplete group stay in an fp16 residual buffer (at most
``group_size - 1`` positions, as in the reference); before attention that
partial group is quantized into the group's slot of the packed buffer (the
reference quantizes the residual on the fly in the same way), and the slot is
rewritten when the group fills. V is quantized per token, so each V position
is final when it is appended. The codes and scales seen by the attention
kernel therefore equal those of the reference cache for the same token stream.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _C

HEAD_DIM = 128


class _Layer:
    __slots__ = ("k", "v", "ks", "vs", "kz", "vz", "kres", "vres", "n", "nres")


class QuantizedKVCache:
    """Per-layer preallocated KV cache with in-place quantized append.

    Args:
        batch, n_kv_heads: cache geometry; head_dim is 128.
        max_len: positions preallocated per layer.
        fmt: "int4", "int4_asym", "int8" or "fp16".
        group_size: K group length for the INT4 formats (the reference's
            KIVI default is 32; the benchmark configuration uses 128).
        num_layers: layers held by this cache object.
    """

    def __init__(self, batch: int, n_kv_heads: int, max_len: int, fmt: str = "int4",
                 group_size: int = 32, num_layers: int = 1, device: Optional[torch.device] = None):
        if fmt not in ("int4", "int4_asym", "int8", "fp16"):
            raise ValueError(f"unknown format {fmt!r}")
        if fmt.startswith("int4") and group_size <= 0:
            raise ValueError("group_size must be positive")
        self.batch, self.n_kv_heads, self.max_len = batch, n_kv_heads, max_len
        self.fmt, self.group_size = fmt, group_size
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.layers = [self._alloc() for _ in range(num_layers)]
        # positions the next attention call covers (set by every append), the
        # attribute the reference's PreallocCache hands its decode hook
        self.cur_attn_len = 0

    # ---- allocation ----------------------------------------------------
    def _alloc(self) -> _Layer:
        B, H, S, d = self.batch, self.n_kv_heads, self.max_len, self.device
        L = _Layer()
        L.kz = L.vz = L.kres = L.vres = None
        L.n = L.nres = 0
        if self.fmt == "fp16":
            L.k = torch.empty(B, H, S, HEAD_DIM, dtype=torch.float16, device=d)
            L.v = torch.empty_like(L.k)
            L.ks = L.vs = None
        elif self.fmt == "int8":
            L.k = torch.empty(B, H, S, HEAD_DIM, dtype=torch.int8, device=d)
            L.v = torch.empty_like(L.k)
            L.ks = torch.empty(B, H, S, dtype=torch.float16, device=d)
            L.vs = torch.empty_like(L.ks)
        else:
            gs = self.group_size
            ng = (S + gs - 1) // gs
            L.k = torch.empty(B, H, S, HEAD_DIM // 2, dtype=torch.int8, device=d)
            L.v = torch.empty_like(L.k)
            L.ks = torch.empty(B, H, ng, HEAD_DIM, dtype=torch.float16, device=d)
            L.vs = torch.empty(B, H, S, dtype=torch.float16, device=d)
            if self.fmt == "int4_asym":
                L.kz = torch.empty_like(L.ks)
                L.vz = torch.empty_like(L.vs)
            L.kres = torch.empty(B, H, gs, HEAD_DIM, dtype=torch.float16, device=d)
            L.vres = torch.empty_like(L.kres)  # fp16 V of the open group (returned by materialize_fp16)
        return L

    # ---- queries -------------------------------------------------------
    def seq_length(self, layer: int = 0) -> int:
        return self.layers[layer].n

    def stored_bytes(self, layer: int = 0) -> int:
        """Bytes of the live positions (codes, scales, zeros, fp16 residual)."""
        L, n = self.layers[layer], self.layers[layer].n
        per_pos = {"fp16": 2 * 2 * HEAD_DIM, "int8": 2 * (HEAD_DIM + 2)}.get(self.fmt)
        if per_pos is not None:
            return n * self.batch * self.n_kv_heads * per_pos
        bh = self.batch * self.n_kv_heads
        zeros = 2 if self.fmt == "int4_asym" else 1
        full_groups = (n - L.nres) // self.group_size
        b = bh * n * HEAD_DIM                      # packed K + V (2 x n x 64 bytes)
        b += bh * n * 2 * zeros                    # V scale (+ zero)
        b += bh * full_groups * HEAD_DIM * 2 * zeros   # K group scale (+ zero)
        b += bh * L.nres * HEAD_DIM * 2 * 2        # fp16 residual (K and V)
        return b

    # ---- append ----------------------------------------------------------
    def append(self, k: torch.Tensor, v: torch.Tensor, layer: int = 0) -> None:
        """Append k, v [batch, n_kv_heads, n_new, 128] fp16 at the end."""
        L = self.layers[layer]
        n_new = k.shape[2]
        if L.n + n_new > self.max_len:
            raise RuntimeError(f"cache overflow: {L.n} + {n_new} > max_len {self.max_len}")
        k = k.contiguous()
        v = v.contiguous()
        pos = L.n
        if self.fmt == "fp16":
            L.k[:, :, pos:pos + n_new].copy_(k)
            L.v[:, :, pos:pos + n_new].copy_(v)
        elif self.fmt == "int8":
            _C.quantize_per_token_into(k, L.k, L.ks, pos)
            _C.quantize_per_token_into(v, L.v, L.vs, pos)
        else:
            _C.quantize_v_per_token_int4_into(v, L.v, L.vs, pos, L.vz)
            self._append_k_int4(L, k, v)
        L.n += n_new
        self.cur_attn_len = L.n

    def _append_k_int4(self, L: _Layer, k: torch.Tensor, v: torch.Tensor) -> None:
        gs = self.group_size
        n_new = k.shape[2]
        done = 0
        if L.nres:                                  # complete the open group first
            take = min(gs - L.nres, n_new)
            L.kres[:, :, L.nres:L.nres + take].copy_(k[:, :, :take])
            L.vres[:, :, L.nres:L.nres + take].copy_(v[:, :, :take])
            L.nres += take
            done = take
            if L.nres == gs:
                self._quantize_group(L, L.kres, (L.n - (gs - take)) // gs * gs)
                L.nres = 0
        full = (n_new - done) // gs * gs            # whole groups straight from the input
        if full:
            start = L.n + done
            self._quantize_group(L, k[:, :, done:done + full].contiguous(), start)
            done += full
        rest = n_new - done
        if rest:
            L.kres[:, :, :rest].copy_(k[:, :, done:])
            L.vres[:, :, :rest].copy_(v[:, :, done:])
            L.nres = rest

    def _quantize_group(self, L: _Layer, x: torch.Tensor, pos: int) -> None:
        _C.quantize_k_per_channel_groupwise_int4_into(x, L.k, L.ks, self.group_size, pos, L.kz)

    def _flush_residual(self, L: _Layer) -> None:
        """Quantize the open partial group into its slot (as the reference
        does on the fly before each decode attention call)."""
        if self.fmt.startswith("int4") and L.nres:
            self._quantize_group(L, L.kres[:, :, :L.nres].contiguous(), L.n - L.nres)

    # ---- attention -------------------------------------------------------
    def attend(self, q: torch.Tensor, softmax_scale: float, layer: int = 0) -> torch.Tensor:
        """Single-query attention of q [batch, n_heads, 128] fp16 over the
        layer's live positions."""
        L = self.layers[layer]
        if L.n == 0:
            raise RuntimeError("attention over an empty cache")
        if self.fmt == "fp16":
            return _C.decode_attention(q, L.k, L.v, softmax_scale, L.n)
        if self.fmt == "int8":
            return _C.decode_attention_int8(q, L.k, L.ks, L.v, L.vs, softmax_scale, L.n)
        self._flush_residual(L)
        if self.fmt == "int4":
            return _C.decode_attention_int4(q, L.k, L.ks, L.v, L.vs, self.group_size, softmax_scale, L.n)
        return _C.decode_attention_int4_asym(q, L.k, L.ks, L.kz, L.v, L.vs, L.vz, self.group_size,
                                             softmax_scale, L.n)

    def quantized_view(self, layer: int = 0):
        """(codes and scales) covering the live positions, in the layout the
        decode ops take; the open group is quantized first."""
        L = self.layers[layer]
        self._flush_residual(L)
        n = L.n
        if self.fmt == "int8":
            return L.k[:, :, :n], L.ks[:, :, :n], L.v[:, :, :n], L.vs[:, :, :n]
        if self.fmt.startswith("int4"):
            ng = (n + self.group_size - 1) // self.group_size
            out = (L.k[:, :, :n], L.ks[:, :, :ng], L.v[:, :, :n], L.vs[:, :, :n])
            if self.fmt == "int4_asym":
                out = out + (L.kz[:, :, :ng], L.vz[:, :, :n])
            return out
        return L.k[:, :, :n], L.v[:, :, :n]

    def materialize_fp16(self, layer: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
        """fp16 K, V [batch, n_kv_heads, n, 128] of the live positions (the
        prefill path, Int4KIVICache._materialize_fp16): quantized positions
        are dequantized by the CUDA kernel, the open group is returned as the
        exact fp16 values it still holds, like the reference."""
        L = self.layers[layer]
        n = L.n
        if self.fmt == "fp16":
            return L.k[:, :, :n].clone(), L.v[:, :, :n].clone()
        if self.fmt == "int8":
            return _C.dequantize_int8(L.k, L.ks, L.v, L.vs, n)
        nq = n - L.nres
        k, v = _C.dequantize_int4(L.k, L.ks, L.v, L.vs, self.group_size, n, L.kz, L.vz)
        if L.nres:
            k[:, :, nq:] = L.kres[:, :, :L.nres]
            v[:, :, nq:] = L.vres[:, :, :L.nres]
        return k, v

    # ---- the reference caches' method names ------------------------------
    # Int4KIVICache (integration/kv_int4_cache.py:85-160,174-206) and
    # PreallocCache (integration/prealloc_cache.py:42-78) callers use these.
    def append_only(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int) -> None:
        """Int4KIVICache.append_only: store [batch, n_kv_heads, n_new, 128]
        fp16 K/V without producing fp16 K/V."""
        self.append(key_states, value_states, layer_idx)

    def get_quantized_for_attention(self, layer_idx: int):
        """Int4KIVICache.get_quantized_for_attention: the codes and scales of
        every stored position, ready for the decode op ("int4":
        (k_packed, k_scale, v_packed, v_scale); "int4_asym" adds (k_zero,
        v_zero); "int8": (k_q, k_scale, v_q, v_scale)). The tensors are
        sequence-prefix views of the preallocated buffers, which the decode
        ops accept as they are: nothing is concatenated or copied."""
        if self.fmt == "fp16":
            raise RuntimeError("an fp16 cache holds no quantized tensors")
        return self.quantized_view(layer_idx)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.seq_length(layer_idx)

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs=None) -> Tuple[torch.Tensor, torch.Tensor]:
        """The HF cache contract. fp16 cache: PreallocCache.update (prefill
        returns its own K/V; a one-token decode step returns the whole buffers,
        whose live prefix ``cur_attn_len`` the decode hook attends over).
        Quantized caches: Int4KIVICache.update (append, then fp16 K/V of all
        stored positions)."""
        self.append(key_states, value_states, layer_idx)
        if self.fmt == "fp16":
            if key_states.shape[2] > 1:
                return key_states, value_states
            L = self.layers[layer_idx]
            return L.k, L.v
        return self.materialize_fp16(layer_idx)
