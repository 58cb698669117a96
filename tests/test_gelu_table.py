"""The GELU table scheme of csrc/gelu.cuh, restated on the CPU against torch's CUDA
GELU-tanh of every bf16 value (tests/golden/torch_gpu_gelu_bf16.npz, recorded on a B200):
inputs with a biased exponent in [111, 131] are looked up, the rest have the closed forms
the kernel uses (x/2 with ties-to-even for tiny |x|, x for large positive x, -0 for large
negative x, +inf -> +inf, -inf and NaN -> the canonical NaN)."""
from __future__ import annotations

import numpy as np

LO, HI = 111, 131
WINDOW = (HI - LO + 1) * 128


def _closed_form(h: np.ndarray) -> np.ndarray:
    mag, neg = h & 0x7FFF, h >> 15
    half = np.where(mag >= 0x100, h - 0x80, (neg << 15) | ((mag >> 1) + (mag & (mag >> 1) & 1)))
    big = np.where(mag < 0x7F80, np.where(neg == 1, 0x8000, h), np.where(h == 0x7F80, 0x7F80, 0x7FFF))
    return np.where(mag < (LO << 7), half, big)


def test_gelu_closed_forms_outside_the_window(golden):
    g = golden("torch_gpu_gelu_bf16.npz")
    x, y = g["x"].astype(np.int64), g["y"].astype(np.int64)
    idx = (x & 0x7FFF) - (LO << 7)
    outside = (idx < 0) | (idx >= WINDOW)
    got = _closed_form(x)
    nan = lambda u: ((u & 0x7F80) == 0x7F80) & ((u & 0x7F) != 0)
    ok = (got == y) | (nan(got) & nan(y))
    assert ok[outside].all(), np.nonzero(outside & ~ok)[0][:10]
    # the window is needed: inside it the closed forms are wrong for many inputs
    assert (~ok[~outside]).sum() > 1000


def test_gelu_table_layout_addresses_every_window_entry_once():
    h = np.arange(65536, dtype=np.int64)
    idx = (h & 0x7FFF) - (LO << 7)
    inside = (idx >= 0) & (idx < WINDOW)
    entry = (idx[inside] << 1) | (h[inside] >> 15)  # entry (index, sign) at 2 * index + sign
    assert np.array_equal(np.sort(entry), np.arange(2 * WINDOW))
