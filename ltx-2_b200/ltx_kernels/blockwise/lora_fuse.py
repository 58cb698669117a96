"""Load-time LoRA merge into blockwise-FP8 weights on the GPU.

The reference merges LoRAs when the checkpoint is loaded
(ltx-core/src/ltx_core/quantization/blockwise/_impl.py:263-301 with
ltx-core/src/ltx_core/loader/fuse_loras.py:99-150): the aggregated update
``delta = sum((B * strength) @ A)`` is added to the dequantised bf16 weight and the
sum is requantised in 128x128 blocks.  ``blockwise_fp8_fuse`` does the dequantise,
add and requantise steps in one kernel (``ltxfp8_lora_fuse_weight``) with the same
roundings as the three reference passes, so the merged codes and scales are
bit-identical to the reference's for the same delta.
"""
from __future__ import annotations

from typing import Iterable, Optional, Sequence, Tuple

import torch

from .. import _lib as L
from .ops import _DeviceGuard, _require_cuda, _stream


def aggregate_lora_products(products: Iterable[Tuple[torch.Tensor, torch.Tensor, float]],
                            dtype: torch.dtype = torch.bfloat16) -> Optional[torch.Tensor]:
    """``sum((B * strength) @ A)`` over ``(A [r, K], B [N, r], strength)`` items with the
    reference's rounding pattern (fuse_loras.py:99-116): the first product is
    ``matmul(B * strength, A).to(dtype)``, the next ones ``addmm_(B, A, alpha=strength)``.
    These are plain library GEMMs, as in the reference."""
    agg = None
    for a, b, strength in products:
        if agg is None:
            agg = torch.matmul(b * strength, a).to(dtype=dtype)
        else:
            agg.addmm_(b, a, alpha=strength)
    return agg


def blockwise_fp8_fuse(weight_fp8: torch.Tensor, weight_scale: torch.Tensor, deltas: torch.Tensor,
                       inplace: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """(e4m3 [N, K], fp32 [N/128, K/128]) + bf16 delta [N, K] -> merged (e4m3, scales).

    Equals ``fp8_blockwise_quantize_weights_torch(dequant(W) + deltas.to(bf16))`` of
    _impl.py:294-297.  With ``inplace`` the weight and scale tensors are overwritten."""
    _require_cuda("blockwise_fp8_fuse", weight_fp8, weight_scale, deltas)
    if weight_fp8.dtype != torch.float8_e4m3fn or weight_fp8.dim() != 2 or not weight_fp8.is_contiguous():
        raise RuntimeError("blockwise_fp8_fuse: weight must be a contiguous float8_e4m3fn [N, K] tensor")
    N, K = weight_fp8.shape
    if weight_scale.dtype != torch.float32 or tuple(weight_scale.shape) != (N // 128, K // 128) \
            or not weight_scale.is_contiguous():
        raise RuntimeError(f"blockwise_fp8_fuse: weight_scale must be contiguous fp32 [{N // 128}, {K // 128}]")
    if tuple(deltas.shape) != (N, K):
        raise RuntimeError(f"blockwise_fp8_fuse: deltas shape {tuple(deltas.shape)} != {(N, K)}")
    d = deltas.to(dtype=torch.bfloat16).contiguous()
    if inplace:
        q_out, s_out = weight_fp8, weight_scale
    else:
        q_out = torch.empty_like(weight_fp8)
        s_out = torch.empty_like(weight_scale)
    with _DeviceGuard(weight_fp8):
        L.check(L.load().ltxfp8_lora_fuse_weight(weight_fp8.data_ptr(), weight_scale.data_ptr(), d.data_ptr(), N, K,
                                                  q_out.data_ptr(), s_out.data_ptr(), _stream(weight_fp8)))
    return q_out, s_out


def blockwise_fp8_fuse_rule(key: str, weight: torch.Tensor, deltas: torch.Tensor, model_sd) -> dict:
    """Drop-in for ltx-core's ``_blockwise_fp8_fuse`` fuse function (_impl.py:277-301):
    returns the merged ``key`` and its ``.weight_scale`` companion.  Layers without a
    companion scale are bf16 and merge as ``deltas + weight`` (fuse_loras.py:61-68)."""
    scale_key = key.replace(".weight", ".weight_scale")
    sd = model_sd.sd
    if scale_key not in sd:
        deltas.add_(weight)
        return {key: deltas.to(dtype=weight.dtype)}
    dev = weight.device if weight.is_cuda else torch.device("cuda", torch.cuda.current_device())
    scale = sd[scale_key].to(device=dev)
    q, s = blockwise_fp8_fuse(weight.to(device=dev).contiguous(), scale.contiguous(), deltas.to(device=dev))
    return {key: q.to(device=weight.device), scale_key: s.to(device=weight.device)}


def merge_loras(weight_fp8: torch.Tensor, weight_scale: torch.Tensor,
                loras: Sequence[Tuple[torch.Tensor, torch.Tensor, float]]) -> Tuple[torch.Tensor, torch.Tensor]:
    """Aggregate ``(A, B, strength)`` LoRAs and merge them into one blockwise-FP8 weight."""
    deltas = aggregate_lora_products(loras, torch.bfloat16)
    if deltas is None:
        return weight_fp8, weight_scale
    return blockwise_fp8_fuse(weight_fp8, weight_scale, deltas)
