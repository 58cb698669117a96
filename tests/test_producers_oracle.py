"""CPU checks of the producer restatements in the oracle (no GPU).

The reference's producers are Triton GPU kernels (triton_ops.py:52-345) that cannot
run in this container, so parity against them is unpinned.  These tests check that
the restatement computes the reference's formulas: its outputs are compared with
float64 evaluations of the same expressions, within the precision of the output
format (bf16, or e4m3 codes with 1x128 scales).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from inputs import activations, bits
from oracle import oracle as O

E4M3_REL = 4e-2   # relative Frobenius error of a 1x128 e4m3 round trip on these inputs
BF16_REL = 5e-3   # relative Frobenius error of bf16 rounding


def _f64(bf16_bits):
    return O.bf16_to_f32(bf16_bits).astype(np.float64)


def _param(b, t, h, seed, std=0.1):
    g = torch.Generator().manual_seed(seed)
    return bits((torch.randn(b, t, h, generator=g) * std).to(torch.bfloat16))


def _rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def _dequant(q, sfa, M, H):
    return O.dequant_act_f32(q, sfa[:, :M]).astype(np.float64).reshape(M, H)


def test_exp_cw_within_one_ulp():
    xs = np.concatenate([np.linspace(-87.0, 88.0, 4001), np.random.default_rng(0).normal(0, 4, 4000)])
    for x in xs.astype(np.float32):
        e, r = O.exp_cw(float(x)), math.exp(float(x))
        assert abs(e - r) <= np.spacing(np.float32(r)), (x, e, r)
    assert O.exp_cw(100.0) == math.inf and O.exp_cw(-120.0) == 0.0


def test_adanorm_restatement_follows_formula():
    B, S, H = 2, 16, 2048
    x = bits(activations(B * S, H, seed=1)).reshape(B, S, H)
    sc, sh = _param(B, 1, H, 2), _param(B, 1, H, 3)
    q, sfa = O.adanorm_quant(x, sc, sh)
    xf = _f64(x).reshape(B, S, H)
    y = xf / np.sqrt((xf * xf).mean(-1, keepdims=True) + 1e-5)
    z = y * (1.0 + _f64(sc)) + _f64(sh)
    assert _rel(_dequant(q, sfa, B * S, H), z.reshape(B * S, H)) < E4M3_REL


def test_rms_fma_restatement_follows_formula():
    B, S, H = 1, 24, 4096
    x = bits(activations(B * S, H, seed=4)).reshape(B, S, H)
    y = bits(activations(B * S, H, seed=5)).reshape(B, S, H)
    z = _param(B, S, H, 6, std=0.5)
    xn, out = O.rms_fma(x, y, z, quantize=False)
    o = _f64(x) + _f64(y) * _f64(z)
    assert _rel(_f64(xn), o) < BF16_REL
    ref = o / np.sqrt((o * o).mean(-1, keepdims=True))
    assert _rel(_f64(out).reshape(B, S, H), ref) < BF16_REL
    _, q, sfa = O.rms_fma(x, y, z, quantize=True)
    assert _rel(_dequant(q, sfa, B * S, H), ref.reshape(B * S, H)) < E4M3_REL


def test_gated_attention_restatement_follows_formula():
    M, H, heads = 40, 2048, 32
    x = bits(activations(M, H, seed=7))
    g = np.random.default_rng(8).normal(0, 3, (M, heads)).astype(np.float32)
    out = O.gated_attention(x, g, quantize=False)
    gate = 2.0 / (1.0 + np.exp(-g.astype(np.float64)))
    ref = _f64(x) * np.repeat(gate, H // heads, axis=1)
    assert _rel(_f64(out), ref) < BF16_REL
    q, sfa = O.gated_attention(x, g, quantize=True)
    assert _rel(_dequant(q, sfa, M, H), ref) < E4M3_REL


def test_gelu_quant_restatement_follows_formula():
    M, K = 32, 1024
    x = bits(activations(M, K, seed=9))
    q, sfa = O.gelu_quant(x)
    xf = _f64(x)
    ref = xf / (1.0 + np.exp(-1.702 * xf))
    assert _rel(_dequant(q, sfa, M, K), ref) < E4M3_REL


@pytest.mark.parametrize("H", [100, 8320, 0])
def test_producers_reject_bad_rows_without_device(H):
    from ltx_kernels import _lib
    L = _lib.load()
    rc = L.ltxfp8_adanorm_quantize(16, 1, 4, H, 16, 0, 0, 16, 0, 0, 16, 16, 4, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED_SHAPE
    rc = L.ltxfp8_rms_fma(16, 16, 1, 4, H, 16, 0, 0, 16, 16, 4, None, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED_SHAPE
    rc = L.ltxfp8_gated_attention(16, 16, _lib.DTYPE_BF16, 4, H, 1, 16, 16, 4, None, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED_SHAPE


def test_gated_attention_rejects_bad_heads_without_device():
    from ltx_kernels import _lib
    L = _lib.load()
    rc = L.ltxfp8_gated_attention(16, 16, _lib.DTYPE_BF16, 4, 2048, 3, 16, 16, 4, None, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED_SHAPE
    rc = L.ltxfp8_gated_attention(16, 16, _lib.DTYPE_BF16, 4, 2048, 512, 16, 16, 4, None, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED_SHAPE  # dim_head 4 is not a multiple of 8


def _rope_tables(rows, dim, seed):
    g = np.random.default_rng(seed)
    ang = g.uniform(-np.pi, np.pi, (rows, dim))
    return O.f32_to_bf16(np.cos(ang).astype(np.float32)), O.f32_to_bf16(np.sin(ang).astype(np.float32))


def test_rms_norm_rope_restatement_follows_formula():
    """x / rms(x) * w, then the interleaved rotation of ltx-core's rope.py (pairs (2i, 2i+1))."""
    rows, dim = 12, 4096
    x = bits(activations(rows, dim, seed=10))
    cos, sin = _rope_tables(rows, dim, 11)
    w = _param(1, 1, dim, 12, std=0.3)[0, 0] + 0  # weights around 1
    w = O.f32_to_bf16((1.0 + O.bf16_to_f32(w)).astype(np.float32))
    out = O.rms_norm_rope(x, cos, sin, w)
    xf = _f64(x)
    v = xf / np.sqrt((xf * xf).mean(-1, keepdims=True)) * _f64(w)
    c, s = _f64(cos), _f64(sin)
    rot = np.empty_like(v)
    rot[:, 0::2], rot[:, 1::2] = -v[:, 1::2], v[:, 0::2]
    assert _rel(_f64(out), v * c + rot * s) < BF16_REL
    q = O.rms_norm_rope(x, cos, sin, w, out_fp8=True)
    assert _rel(O.e4m3_to_f32(q).astype(np.float64), v * c + rot * s) < 0.06  # plain e4m3 cast, no scales


def test_rms_norm_split_rope_restatement_follows_formula():
    """(x / rms(x)) * w per head split into halves a, b: (a cos - b sin, b cos + a sin)."""
    B, S, H, heads = 2, 5, 2048, 16
    d = H // heads
    x = bits(activations(B * S, H, seed=13)).reshape(B, S, H)
    g = np.random.default_rng(14)
    ang = g.uniform(-np.pi, np.pi, (1, heads, S, d // 2))
    cos = O.f32_to_bf16(np.cos(ang).astype(np.float32))
    sin = O.f32_to_bf16(np.sin(ang).astype(np.float32))
    out = O.rms_norm_split_rope(x, cos, sin)
    xf = _f64(x)
    v = xf / np.sqrt((xf * xf).mean(-1, keepdims=True) + 1e-6)
    vh = v.reshape(B, S, heads, 2, d // 2)
    c = np.transpose(_f64(cos), (0, 2, 1, 3))[:, :, :, None, :]   # [1, S, heads, 1, d/2]
    s = np.transpose(_f64(sin), (0, 2, 1, 3))[:, :, :, None, :]
    a, b = vh[:, :, :, 0:1, :], vh[:, :, :, 1:2, :]
    ref = np.concatenate([a * c - b * s, b * c + a * s], axis=3).reshape(B, S, H)
    assert _rel(_f64(out), ref) < BF16_REL


def test_fp6_pack_roundtrip_and_layout():
    """Pack layout of fp6_pack.cu:8-41 on a hand-checked group, and the round trip of
    FP6-range codes (top two exponent bits zero)."""
    c = np.array([[0x9F, 0x01, 0x15, 0x80, 0x00, 0x1F, 0x8A, 0x11]], np.uint8)
    v = [0x3F, 0x01, 0x15, 0x20, 0x00, 0x1F, 0x2A, 0x11]           # s -> bit 5, bits 4..0 kept
    p0 = v[0] << 18 | v[1] << 12 | v[2] << 6 | v[3]
    p1 = v[4] << 18 | v[5] << 12 | v[6] << 6 | v[7]
    expect = [p0 >> 16, (p0 >> 8) & 0xFF, p0 & 0xFF, p1 >> 16, (p1 >> 8) & 0xFF, p1 & 0xFF]
    assert O.fp6_pack(c).tolist() == [expect]
    g = np.random.default_rng(0)
    codes = g.integers(0, 256, (16, 256), dtype=np.uint8) & 0x9F   # FP6-range codes
    assert np.array_equal(O.fp6_unpack(O.fp6_pack(codes), 256), codes)
    w = np.random.default_rng(1).normal(0, 0.02, (128, 256)).astype(np.float32)
    q, s = O.quant_weight_128x128(w, 0.1172)
    assert ((q & 0x60) == 0).all()                                 # the FP6 quantiser never sets them


def test_fp6_to_tc_layout():
    """The tensor core's 6-bit order on a hand-built group: codes 0..15 (6-bit values
    equal to the e4m3 codes below 32) land at bits 6i of a little-endian 96-bit word;
    a sign bit (e4m3 bit 7) lands at bit 6i + 5."""
    c = np.arange(128, dtype=np.uint8).reshape(1, 128) % 16
    c[0, 16] |= 0x80
    tc = O.fp6_to_tc(O.fp6_pack(c), 128)
    assert tc.shape == (1, 96)
    word = sum(i << (6 * i) for i in range(16))
    assert tc[0, :12].tolist() == list(word.to_bytes(12, "little"))
    assert tc[0, 12:24].tolist() == list((word | (1 << 5)).to_bytes(12, "little"))
