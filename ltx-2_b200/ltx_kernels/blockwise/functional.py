"""Blockwise FP8 functional ops on sm_100a kernels.

Mirrors the names ltx-core imports from ltx-kernels/src/ltx_kernels/blockwise/
functional.py and triton_ops.py (ltx_core/quantization/blockwise/_impl.py:12-23):

* ``blockwise::quantize`` -- same op name and schema as the Triton op
  (triton_ops.py:128-151): bf16 ``[b, s, h]`` -> (e4m3 ``[b, s, h]``, fp32 scales
  ``(b*s, h/128)`` with strides ``(1, align4(b*s))``).
* ``blockwise::dequantize`` -- same as triton_ops.py:414-433.
* ``blockwise_quantize_weights`` / ``fp8_blockwise_quantize_weights_torch`` --
  128x128 weight quantisation (functional.py:128-135,149-150), bit-exact.

The activation quantiser's arithmetic is selectable (``set_quant_mode``):
``"torch"`` (default) is bit-exact with the reference's ``blockwise_quantize_torch``;
``"triton"`` reproduces the Triton kernel's division instruction.

Names that belong to other parts of the reference (FP6 packing, the fused
AdaLN / residual / gated-attention producers, RMSNorm+RoPE) are exported so the
import list resolves, and raise ``NotImplementedError`` when called.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .. import _lib as L
from . import ops

FP8_SCALE_MAX = 448.0
FP6_SCALE_MAX = 0.1172

_QUANT_MODE = L.QUANT_TORCH


def set_quant_mode(mode: str) -> None:
    """Select the activation quantiser's arithmetic: ``"torch"`` or ``"triton"``."""
    global _QUANT_MODE
    _QUANT_MODE = {"torch": L.QUANT_TORCH, "triton": L.QUANT_TRITON}[mode]


def get_quant_mode() -> str:
    return "triton" if _QUANT_MODE == L.QUANT_TRITON else "torch"


@torch.library.custom_op("blockwise::quantize", mutates_args=())
def _quant_blockwise(x: torch.Tensor, use_gelu: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    if use_gelu:
        raise NotImplementedError(
            "blockwise::quantize(use_gelu=True) applies x*sigmoid(1.702x) (triton_ops.py:98-100), which no "
            "ltx-core caller uses; the FFN's GELU-tanh is fused into the GEMM epilogue instead")
    b, s, h = x.shape
    q, sc = ops.quantize_1x128(x, _QUANT_MODE)
    return q.view(b, s, h), sc


@_quant_blockwise.register_fake
def _quant_blockwise_fake(x: torch.Tensor, use_gelu: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    b, s, h = x.shape
    q = torch.empty((b, s, h), dtype=torch.float8_e4m3fn, device=x.device)
    return q, ops.empty_act_scales(b * s, h // 128, x.device)


@torch.library.custom_op("blockwise::dequantize", mutates_args=())
def _dequant_blockwise(x: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    b, s, h = x.shape
    return ops.dequantize_1x128(x.reshape(b * s, h), scales).view(b, s, h)


@_dequant_blockwise.register_fake
def _dequant_blockwise_fake(x: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    return torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)


def blockwise_quantize_triton(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """The reference's name for ``blockwise::quantize(x, False)`` (triton_ops.py:153-154,440)."""
    return _quant_blockwise(x, False)


run_quant_blockwise_tma_aligned = blockwise_quantize_triton


def blockwise_dequantize_triton(x: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    return _dequant_blockwise(x, scales)


def blockwise_dequantize(x: Tuple[torch.Tensor, torch.Tensor]) -> torch.Tensor:
    """(e4m3 ``[b, s, h]``, scales) -> bf16 (functional.py:157-159)."""
    x_fp8, scales = x
    return blockwise_dequantize_triton(x_fp8, scales)


def blockwise_quantize_weights(w: torch.Tensor, block_size: int = 128,
                               scale_max: float = FP8_SCALE_MAX) -> Tuple[torch.Tensor, torch.Tensor]:
    """W ``[N, K]`` -> (e4m3 ``[N, K]``, fp32 ``[N/128, K/128]``), functional.py:128-135."""
    if block_size != 128 or scale_max != FP8_SCALE_MAX:
        raise NotImplementedError("only 128x128 blocks with the e4m3 range (448) are provided")
    return ops.quantize_weight_128x128(w)


def fp8_blockwise_quantize_weights_torch(x: torch.Tensor, block_size: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    return blockwise_quantize_weights(x, block_size, FP8_SCALE_MAX)


def blockwise_quantize_torch(x: torch.Tensor, block_size: int = 128,
                             scale_max: float = FP8_SCALE_MAX) -> Tuple[torch.Tensor, torch.Tensor]:
    """Same outputs as the reference's torch quantiser (functional.py:138-144): e4m3
    ``[b, n, h]`` and contiguous fp32 scales ``[h/128, b*n]``, computed by the CUDA
    kernel in its bit-exact torch mode."""
    if block_size != 128 or scale_max != FP8_SCALE_MAX:
        raise NotImplementedError("only 1x128 groups with the e4m3 range (448) are provided")
    b, n, h = x.shape
    q, s = ops.quantize_1x128(x, L.QUANT_TORCH)
    return q.view(b, n, h), s.t().contiguous()


def _not_provided(name: str):
    def fn(*args, **kwargs):
        raise NotImplementedError(f"{name} is outside the blockwise-FP8 linear path ltx-2_b200 provides")
    fn.__name__ = name
    return fn


fp6_blockwise_quantize_weights_torch = _not_provided("fp6_blockwise_quantize_weights_torch")
fp6_pack_tensor = _not_provided("fp6_pack_tensor")
fp6_unpack_tensor = _not_provided("fp6_unpack_tensor")
blockwise_quantize_adanorm_triton = _not_provided("blockwise_quantize_adanorm_triton")
blockwise_quantize_rms_fma_triton = _not_provided("blockwise_quantize_rms_fma_triton")
gated_attention_triton = _not_provided("gated_attention_triton")
rms_norm_rope = _not_provided("rms_norm_rope")
rms_norm_split_rope = _not_provided("rms_norm_split_rope")
