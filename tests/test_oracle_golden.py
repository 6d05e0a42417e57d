"""Pin the numpy oracle to the reference's own PyTorch oracle outputs.

The fixtures in tests/golden/*.npz were produced by tests/golden/make_golden.py,
which imports reference/kv_cache_ref.py and reference/attention_ref.py. Codes and
scales must match bit for bit; attention to fp32 round-off.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import kv_oracle as O

G = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def qg():
    return np.load(G / "quant_golden.npz")


@pytest.fixture(scope="module")
def ag():
    return np.load(G / "attention_golden.npz")


@pytest.mark.parametrize("bits", [8, 4])
def test_per_token_bit_exact(qg, bits):
    q, s = O.quantize_per_token(qg["x"], bits)
    np.testing.assert_array_equal(q, qg[f"tok{bits}_q"])
    np.testing.assert_array_equal(s, qg[f"tok{bits}_s32"])
    np.testing.assert_array_equal(s.astype(np.float16), qg[f"tok{bits}_s16"])


@pytest.mark.parametrize("gs", [32, 128, 7])
def test_per_channel_groupwise_bit_exact(qg, gs):
    q, s = O.quantize_per_channel_groupwise(qg["x"], 4, gs)
    np.testing.assert_array_equal(q, qg[f"chan4_g{gs}_q"])
    np.testing.assert_array_equal(s, qg[f"chan4_g{gs}_s32"])
    np.testing.assert_array_equal(s.astype(np.float16), qg[f"chan4_g{gs}_s16"])


def test_presets_bit_exact(qg):
    k, v = qg["preset_k"], qg["preset_v"]
    for got, name in zip(O.quantize_kv_int8_per_token(k, v), ("int8_kq", "int8_ks", "int8_vq", "int8_vs")):
        np.testing.assert_array_equal(got, qg[name])
    for got, name in zip(O.quantize_kv_kivi_int4(k, v, 32), ("kivi_kq", "kivi_ks", "kivi_vq", "kivi_vs")):
        np.testing.assert_array_equal(got, qg[name])


def test_unpack_convention(qg):
    np.testing.assert_array_equal(O.unpack_int4_signed(qg["unpack_bytes"]), qg["unpack_codes"])
    # pack is the exact inverse on the signed range the quantizers emit
    codes = np.arange(-7, 8, dtype=np.int8)
    grid = np.stack(np.meshgrid(codes, codes), -1).reshape(-1, 2)
    np.testing.assert_array_equal(O.unpack_int4_signed(O.pack_int4(grid)), grid)


def test_ties_and_zero_rows(qg):
    q8 = qg["tok8_q"][0, 0, :4]
    assert list(q8[0, :9]) == [127, 2, -4, 0, 0, 2, 126, -126, 4]
    assert (q8[2] == 0).all()
    q4 = qg["tok4_q"][0, 0, 1]
    assert list(q4[:7]) == [-7, 2, -4, 0, 0, 2, 6]


def test_attention_config0(ag):
    out = O.decode_attention(ag["c0_q"], ag["c0_k"], ag["c0_v"], float(ag["scale"]))
    np.testing.assert_allclose(out, ag["c0_out32"], rtol=1e-5, atol=1e-6)
    d16 = np.abs(out.astype(np.float16).astype(np.float32) - ag["c0_out16"].astype(np.float32))
    assert d16.max() <= 2.0 ** -10  # at most one fp16 ulp at |x|<1 from fp32 order differences


def test_attention_on_dequantized_int8_and_kivi(ag):
    k, v, q = ag["i8_k"], ag["i8_v"], ag["i8_q"]
    kq, ks, vq, vs = O.quantize_kv_int8_per_token(k, v)
    kd, vd = O.dequant_int8_to_f16(kq, ks.astype(np.float16), vq, vs.astype(np.float16))
    out = O.decode_attention(q, kd, vd, float(ag["scale"]))
    np.testing.assert_allclose(out, ag["i8_out32"], rtol=1e-5, atol=1e-6)
    kq, ks, vq, vs = O.quantize_kv_kivi_int4(k, v, 32)
    kd, vd = O.dequant_kivi_sym_to_f16(O.pack_int4(kq), ks.astype(np.float16),
                                       O.pack_int4(vq), vs.astype(np.float16), 32)
    out = O.decode_attention(q, kd, vd, float(ag["scale"]))
    np.testing.assert_allclose(out, ag["kivi_out32"], rtol=1e-5, atol=1e-6)


def test_asym_roundtrip_bounds():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 8, 100, 128)).astype(np.float16)
    q, s, z = O.quantize_v_per_token_int4_asym(x)
    assert q.max() <= 15
    rec = O.dequantize_asym_per_token(q, s, z)
    err = np.abs(rec - x.astype(np.float32))
    assert (err <= s.astype(np.float32)[..., None] * 0.5 * 1.01 + 1e-3).all()
    for gs in (32, 128):
        q, s, z = O.quantize_k_per_channel_groupwise_int4_asym(x, gs)
        rec = O.dequantize_asym_per_channel_groupwise(q, s, z, gs)
        idx = np.arange(100) // gs
        bound = s.astype(np.float32)[:, :, idx, :] * 0.5 * 1.01 + 1e-3
        assert (np.abs(rec - x.astype(np.float32)) <= bound).all()
