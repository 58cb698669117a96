"""Fused blockwise-FP8 layers beyond the reference's op set.

* ``fp8_linear`` -- one call for quantise (if bf16) + GEMM + epilogue
  (bias, GELU-tanh, 1x128 requantisation, runtime LoRA).
* ``BlockwiseFP8FeedForward`` -- the DiT FFN (ltx-core/src/ltx_core/model/
  transformer/feed_forward.py:6-15: Linear(d, 4d) -> GELU-tanh -> Linear(4d, d)):
  the up projection writes bf16 ``h``, one streaming pass applies torch's GELU and
  quantises it for the down projection (``ops.gelu_tanh_quantize_1x128``).  The GEMM
  epilogue can do the same in-kernel (``fused_epilogue=True``, no bf16 hidden state),
  with identical codes and scales, but the GEMM's epilogue warps are on its critical
  path, so the separate pass is faster at every measured size (3-16 %).
* ``BlockwiseFP8LoRALinear`` -- ``W x + alpha B (A x)`` at run time: the skinny
  ``A x`` GEMM runs first, ``B (A x)`` is folded into the FP8 GEMM as extra bf16
  K blocks.  The reference instead merges LoRA into the weights at load time
  (ltx_core/quantization/blockwise/_impl.py:277-301).
"""
from __future__ import annotations

from typing import Optional, Tuple, Union

import torch
import torch.nn as nn

from . import ops
from .functional import blockwise_quantize_triton, quant_mode_code
from .linear import BlockwiseFP8Linear

Activation = Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]


def _as_quantized(x: Activation) -> Tuple[torch.Tensor, torch.Tensor, tuple]:
    if isinstance(x, tuple):
        q, s = x
        lead = tuple(q.shape[:-1])
        return q.reshape(-1, q.shape[-1]), s, lead
    lead = tuple(x.shape[:-1])
    q, s = ops.quantize_1x128(x, quant_mode_code())
    return q, s, lead


def fp8_linear(x: Activation, weight: torch.Tensor, weight_scale: torch.Tensor, bias: Optional[torch.Tensor] = None,
               *, gelu: bool = False, requant: bool = False, write_d: bool = True,
               lora: Optional[Tuple[torch.Tensor, torch.Tensor, float]] = None, x_bf16: Optional[torch.Tensor] = None):
    """Blockwise FP8 linear with a fused epilogue.

    ``x`` is bf16 ``[..., K]`` or a pre-quantised ``(e4m3 [..., K], scales)`` pair.
    ``lora = (A [r, K] bf16, B [N, r] bf16, alpha)`` adds ``alpha * B (A x)``; it needs
    the bf16 input (``x`` itself, or ``x_bf16`` when ``x`` is pre-quantised).
    Returns bf16 ``[..., N]``, or with ``requant`` a tuple ``(bf16 or None, e4m3, scales)``.
    ``gelu=True`` is torch's GELU-tanh (the reference applies ``F.gelu(approximate="tanh")``
    to the bf16 output, gelu_approx.py:10); the input quantisation and the requantisation
    use the arithmetic of ``functional.set_quant_mode`` (default: the reference's GPU kernels).
    """
    ax = lb = None
    alpha = 1.0
    if lora is not None:
        la, lb, alpha = lora
        src = x if not isinstance(x, tuple) else x_bf16
        if src is None:
            raise RuntimeError("fp8_linear: runtime LoRA needs the bf16 activations")
        ax = ops.lora_a(src, la)
    q, s, lead = _as_quantized(x)
    res = ops.gemm(q, s, weight, weight_scale, bias, gelu=gelu, requant=requant, write_d=write_d,
                   lora_ax=ax, lora_b=lb, lora_alpha=alpha, requant_mode=quant_mode_code())
    N = weight.shape[0]
    if requant:
        d, qo, so = res
        return (None if d is None else d.view(*lead, N)), qo.view(*lead, N), so
    return res.view(*lead, N)


class BlockwiseFP8FeedForward(nn.Module):
    """FFN: up projection, torch's GELU-tanh + 1x128 requantisation of the hidden state,
    down projection.  ``fused_epilogue``: GELU and requant inside the up projection's
    GEMM epilogue instead of a separate streaming pass (same results)."""

    def __init__(self, dim: int, dim_out: int, mult: int = 4, bias: bool = True, device=None,
                 fused_epilogue: bool = False):
        super().__init__()
        inner = int(dim * mult)
        self.proj_in = BlockwiseFP8Linear(dim, inner, bias=bias, device=device)
        self.proj_out = BlockwiseFP8Linear(inner, dim_out, bias=bias, device=device)
        self.fused_epilogue = fused_epilogue

    @classmethod
    def from_linears(cls, up: BlockwiseFP8Linear, down: BlockwiseFP8Linear) -> "BlockwiseFP8FeedForward":
        ff = cls.__new__(cls)
        nn.Module.__init__(ff)
        ff.proj_in = up
        ff.proj_out = down
        ff.fused_epilogue = False
        return ff

    def forward(self, x: Activation) -> torch.Tensor:
        if self.fused_epilogue:
            _, hq, hs = fp8_linear(x, self.proj_in.weight, self.proj_in.weight_scale, self.proj_in.bias,
                                   gelu=True, requant=True, write_d=False)
        else:
            h = fp8_linear(x, self.proj_in.weight, self.proj_in.weight_scale, self.proj_in.bias)
            hq, hs = ops.gelu_tanh_quantize_1x128(h, quant_mode_code())
            hq = hq.view(*h.shape)
        return fp8_linear((hq, hs), self.proj_out.weight, self.proj_out.weight_scale, self.proj_out.bias)


class BlockwiseFP8LoRALinear(BlockwiseFP8Linear):
    """BlockwiseFP8Linear plus a runtime LoRA ``alpha * B (A x)`` (bf16 A ``[r, in]``, B ``[out, r]``)."""

    def __init__(self, in_features: int, out_features: int, rank: int, alpha: float = 1.0, bias: bool = True,
                 device=None, dtype=None):
        super().__init__(in_features, out_features, bias, device, dtype)
        self.rank = rank
        self.alpha = alpha
        self.lora_A = nn.Parameter(torch.zeros(rank, in_features, device=device, dtype=torch.bfloat16),
                                   requires_grad=False)
        self.lora_B = nn.Parameter(torch.zeros(out_features, rank, device=device, dtype=torch.bfloat16),
                                   requires_grad=False)

    def forward(self, x):
        if isinstance(x, tuple):
            raise RuntimeError("BlockwiseFP8LoRALinear needs the bf16 input for the LoRA term")
        return fp8_linear(x, self.weight, self.weight_scale, self.bias, lora=(self.lora_A, self.lora_B, self.alpha))
