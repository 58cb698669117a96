"""Seeded synthetic inputs with the value distributions of BASELINE.json's configs.

Activations: bf16 ~N(0,1) with a seeded 1% of channels scaled x20 (outliers).
Weights: ~N(0, 0.02).  Bias: ~N(0, 0.01) rounded to bf16, then fp32.
LoRA A, B: ~N(0, 0.01) bf16.  All generated on the CPU from torch.Generator seeds.
"""
from __future__ import annotations

import numpy as np
import torch


def activations(M: int, K: int, seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g, dtype=torch.float32)
    ch = torch.randperm(K, generator=g)[: max(1, K // 100)]
    x[:, ch] *= 20.0
    return x.to(torch.bfloat16)


def weights(N: int, K: int, seed: int = 1, std: float = 0.02) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(N, K, generator=g, dtype=torch.float32) * std


def bias(N: int, seed: int = 2) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16).float()


def lora(N: int, K: int, r: int, seed: int = 3):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(r, K, generator=g) * 0.01).to(torch.bfloat16)
    b = (torch.randn(N, r, generator=g) * 0.01).to(torch.bfloat16)
    return a, b


def bits(t: torch.Tensor) -> np.ndarray:
    """CPU tensor -> numpy bit patterns (bf16 -> uint16, e4m3 -> uint8)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def scales_mn(s: torch.Tensor, M: int) -> np.ndarray:
    """(M, KB) MN-major scale view -> numpy [KB, M] (element (m, kb) at [kb, m])."""
    return s.detach().t().cpu().contiguous().numpy()[:, :M]
