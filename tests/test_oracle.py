"""The CPU oracle against the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from ltx-kernels' torch functions)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O


@pytest.mark.parametrize("case", ["act_ragged", "act_4096", "act_edge"])
def test_activation_quant_matches_reference(golden, case):
    d = golden("act_quant.npz")
    x = d[f"{case}_x"]
    M = x.shape[0]
    q, s = O.quant_act_1x128(x)
    assert O.codes_equal(q, d[f"{case}_q"]).all()
    assert O.scales_equal(s[:, :M], d[f"{case}_s"]).all()


def test_activation_quant_codes_bitwise_except_nan_sign(golden):
    d = golden("act_quant.npz")
    q, _ = O.quant_act_1x128(d["act_4096_x"])
    assert np.array_equal(q, d["act_4096_q"])  # no NaN groups here: fully bitwise


@pytest.mark.parametrize("case", ["w_f32", "w_bf16"])
def test_weight_quant_matches_reference(golden, case):
    d = golden("weight_quant.npz")
    q, s = O.quant_weight_128x128(d[f"{case}_w"])
    assert O.codes_equal(q, d[f"{case}_q"]).all()
    assert O.scales_equal(s, d[f"{case}_s"]).all()


def test_reference_cpu_gemm_path(golden):
    """dequant(A) . dequant(W)^T + bias in fp32, as the reference's CPU path computes it."""
    g = golden("gemm_ref.npz")
    M, K = g["x"].shape
    N = g["w"].shape[0]
    aq, asc = O.quant_act_1x128(g["x"])
    wq, wsc = O.quant_weight_128x128(g["w"])
    d = O.gemm_dequant_f32(aq, asc, wq, wsc, g["bias"])
    assert np.array_equal(O.f32_to_bf16(d), g["d_bf16"])
    m = O.error_metrics(d, g["d_f32"])
    assert m["rel_fro"] < 1e-6


def test_promoted_order_close_to_reference(golden):
    """The SM89 kernel's per-128-K promotion order differs from one fp32 matmul only by rounding."""
    g = golden("gemm_ref.npz")
    M, K = g["x"].shape
    N = g["w"].shape[0]
    aq, asc = O.quant_act_1x128(g["x"])
    wq, wsc = O.quant_weight_128x128(g["w"])
    f, _ = O.gemm_promoted(aq, asc, asc.shape[1], wq, wsc, g["bias"], M, N, K)
    m = O.error_metrics(f, g["d_f32"])
    assert m["rel_fro"] < 1e-5 and m["max_abs_norm"] < 1e-5


def test_gelu_tanh_matches_torch(golden):
    """bf16 GELU-tanh: exact, except where 1 + tanh cancels (|error| < 1e-6 there)."""
    g = golden("gelu_ref.npz")
    y = O.gelu_tanh_bf16(g["x"])
    a, b = O.bf16_to_f32(y), O.bf16_to_f32(g["y"])
    exact = y == g["y"]
    assert exact.mean() > 0.99
    assert np.all(exact | (np.abs(a - b) <= 1e-6))


def test_e4m3_roundtrip_all_codes():
    codes = np.arange(256, dtype=np.uint8)
    f = O.e4m3_to_f32(codes)
    back = O.f32_to_e4m3(f)
    nan = (codes & 0x7F) == 0x7F
    assert np.array_equal(back[~nan], codes[~nan])
    assert np.all((back[nan] & 0x7F) == 0x7F)


def test_e4m3_rounding_edges():
    vals = np.array([448.0, 464.0, 464.01, 480.0, 1e9, np.inf, 2.0 ** -10, 1.5 * 2.0 ** -9, 2.0 ** -6 * 0.99,
                     -0.0, 0.0], np.float32)
    got = O.f32_to_e4m3(vals)
    # torch: 448 -> 0x7E; 464 ties to even 0x7E; above 464 -> NaN; 2^-10 ties to 0; 1.5*2^-9 ties to 0x02
    assert list(got[:8]) == [0x7E, 0x7E, 0x7F, 0x7F, 0x7F, 0x7F, 0x00, 0x02]
    assert got[8] == 0x08 and got[9] == 0x80 and got[10] == 0x00


def test_bf16_rounding_matches_numpy_reference():
    rng = np.random.default_rng(0)
    f = rng.standard_normal(10000).astype(np.float32) * 100
    h = O.f32_to_bf16(f)
    # round-to-nearest-even on the upper 16 bits
    u = f.view(np.uint32).astype(np.uint64)
    ref = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    assert np.array_equal(h, ref)
