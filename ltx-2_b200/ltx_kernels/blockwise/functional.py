"""Blockwise FP8 functional ops on sm_100a kernels.

Mirrors the names ltx-core imports from ltx-kernels/src/ltx_kernels/blockwise/
functional.py and triton_ops.py (ltx_core/quantization/blockwise/_impl.py:12-23):

* ``blockwise::quantize`` -- same op name and schema as the Triton op
  (triton_ops.py:128-151): bf16 ``[b, s, h]`` -> (e4m3 ``[b, s, h]``, fp32 scales
  ``(b*s, h/128)`` with strides ``(1, align4(b*s))``).
* ``blockwise::dequantize`` -- same as triton_ops.py:414-433.
* ``blockwise_quantize_weights`` / ``fp8_blockwise_quantize_weights_torch`` --
  128x128 weight quantisation (functional.py:128-135,149-150), bit-exact.

The arithmetic of every quantising op here, and of the fused GEMM epilogue's
requantisation in ``fused.py``, is selectable (``set_quant_mode``):
``"triton"`` (default) is the reference's GPU path -- its Triton kernels as compiled
for the B200 (the same divisions, exp, bf16 steps and reduction order);
``"torch"`` uses IEEE-rounded arithmetic throughout and is bit-exact with the
reference's CPU function ``blockwise_quantize_torch`` and with the CPU oracle's
restatement of the producers.

* ``blockwise::adanorm``, ``blockwise::quant_rms_fma``, ``blockwise::rms_fma``,
  ``blockwise::gated_attention`` and ``blockwise::quantize(use_gelu=True)`` -- the
  fused producers of triton_ops.py:52-345 (csrc/producers.cuh).

* ``rms_norm_rope`` / ``rms_norm_split_rope`` (ops ``q8_kernels_ops::rms_norm_rope``,
  ``q8_kernels_ops::rms_norm_split_rope``) -- q/k RMSNorm + RoPE of the reference's
  ops_cpp extension (csrc/ops/rms_norm*_cuda.cu).
* FP6 weights: ``fp6_blockwise_quantize_weights_torch``, ``fp6_pack_tensor`` /
  ``fp6_unpack_tensor`` (ops ``q8_kernels_ops::fp6_pack`` / ``fp6_unpack``).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .. import _lib as L
from . import ops

FP8_SCALE_MAX = 448.0
FP6_SCALE_MAX = 0.1172

_QUANT_MODE = L.QUANT_TRITON


def set_quant_mode(mode: str) -> None:
    """Select the quantising ops' arithmetic (process-wide): ``"triton"`` (the
    reference's GPU kernels, the default) or ``"torch"`` (IEEE, the reference's CPU
    function)."""
    global _QUANT_MODE
    _QUANT_MODE = {"torch": L.QUANT_TORCH, "triton": L.QUANT_TRITON}[mode]


def get_quant_mode() -> str:
    return "triton" if _QUANT_MODE == L.QUANT_TRITON else "torch"


def quant_mode_code() -> int:
    """The current mode as the C ABI's LTXFP8_QUANT_* value."""
    return _QUANT_MODE


@torch.library.custom_op("blockwise::quantize", mutates_args=())
def _quant_blockwise(x: torch.Tensor, use_gelu: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    b, s, h = x.shape
    if use_gelu:
        # x * sigmoid(1.702 x) before the quantiser (triton_ops.py:98-100,119-120)
        q, sc = ops.gelu_quantize_1x128(x, _QUANT_MODE)
    else:
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


def blockwise_quantize_gelu_triton(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """``blockwise::quantize(x, True)``: quantise x * sigmoid(1.702 x) (triton_ops.py:156-157,441)."""
    return _quant_blockwise(x, True)


run_quant_blockwise_tma_aligned = blockwise_quantize_triton
run_quant_blockwise_gelu_tma_aligned = blockwise_quantize_gelu_triton


# ----------------------------------------------------------------------------- fused producers
# Same op names, schemas and outputs as the reference's Triton producers
# (triton_ops.py:158-345); arithmetic as documented in csrc/producers.cuh.
def _scales_like(num_rows: int, h: int, device) -> torch.Tensor:
    return ops.empty_act_scales(num_rows, h // 128, device)


@torch.library.custom_op("blockwise::adanorm", mutates_args=())
def _adanorm(x: torch.Tensor, w: Optional[torch.Tensor], norm_scale: torch.Tensor, norm_shift: torch.Tensor,
             out_dtype: torch.dtype, hd_scale: Optional[float]) -> Tuple[torch.Tensor, torch.Tensor]:
    """RMSNorm (eps 1e-5) -> bf16 -> x * (1 + norm_scale) + norm_shift -> 1x128 e4m3
    (triton_ops.py:158-186).  ``w`` and ``hd_scale`` are accepted and unused, as in the
    reference; the output is always e4m3."""
    b, s, h = x.shape
    q, sc = ops.adanorm_quantize(x, norm_scale, norm_shift, _QUANT_MODE)
    return q.view(b, s, h), sc


@_adanorm.register_fake
def _adanorm_fake(x, w, norm_scale, norm_shift, out_dtype, hd_scale):
    b, s, h = x.shape
    return (torch.empty((b, s, h), dtype=torch.float8_e4m3fn, device=x.device), _scales_like(b * s, h, x.device))


@torch.library.custom_op("blockwise::quant_rms_fma", mutates_args=("x",))
def _quant_rms_fma(x: torch.Tensor, y: torch.Tensor, z: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """x += y * z in place, RMS-normalise, 1x128 e4m3 (triton_ops.py:234-262)."""
    b, s, h = x.shape
    q, sc = ops.rms_fma(x, y, z, True, _QUANT_MODE)
    return q.view(b, s, h), sc


@_quant_rms_fma.register_fake
def _quant_rms_fma_fake(x, y, z):
    b, s, h = x.shape
    return (torch.empty((b, s, h), dtype=torch.float8_e4m3fn, device=x.device), _scales_like(b * s, h, x.device))


@torch.library.custom_op("blockwise::rms_fma", mutates_args=("x",))
def _rms_fma(x: torch.Tensor, y: torch.Tensor, z: torch.Tensor) -> torch.Tensor:
    """x += y * z in place, RMS-normalise, bf16 out (triton_ops.py:265-290)."""
    b, s, h = x.shape
    return ops.rms_fma(x, y, z, False, _QUANT_MODE).view(b, s, h)


@_rms_fma.register_fake
def _rms_fma_fake(x, y, z):
    return torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)


@torch.library.custom_op("blockwise::gated_attention", mutates_args=())
def _gated_attention(x: torch.Tensor, gate_logits: torch.Tensor, quantize: bool = True
                     ) -> Tuple[torch.Tensor, torch.Tensor]:
    """x * 2 sigmoid(gate_logits) per head, then 1x128 e4m3 (triton_ops.py:309-384).
    With quantize=False the bf16 output comes with None in place of the scales, as the
    reference's op returns (triton_ops.py:367-370, 384)."""
    b, t, h = x.shape
    if quantize:
        q, sc = ops.gated_attention(x, gate_logits, True, _QUANT_MODE)
        return q.view(b, t, h), sc
    out = ops.gated_attention(x, gate_logits, False, _QUANT_MODE)
    return out.view(b, t, h), None


@_gated_attention.register_fake
def _gated_attention_fake(x, gate_logits, quantize=True):
    b, t, h = x.shape
    if quantize:
        return (torch.empty((b, t, h), dtype=torch.float8_e4m3fn, device=x.device), _scales_like(b * t, h, x.device))
    return torch.empty((b, t, h), dtype=torch.bfloat16, device=x.device), None


def blockwise_quantize_adanorm_triton(x: torch.Tensor, w: Optional[torch.Tensor], norm_scale: torch.Tensor,
                                      norm_shift: torch.Tensor, out_dtype: torch.dtype = torch.float8_e4m3fn,
                                      hd_scale: Optional[float] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """triton_ops.py:438 (``run_quant_blockwise_norm_tma_aligned``)."""
    return _adanorm(x, w, norm_scale, norm_shift, out_dtype, hd_scale)


def blockwise_quantize_rms_fma_triton(x: torch.Tensor, y: torch.Tensor, z: torch.Tensor
                                      ) -> Tuple[torch.Tensor, torch.Tensor]:
    """triton_ops.py:442 (``run_quant_blockwise_rms_fma``); updates x in place."""
    return _quant_rms_fma(x, y, z)


def rms_fma_triton(x: torch.Tensor, y: torch.Tensor, z: torch.Tensor) -> torch.Tensor:
    """triton_ops.py:443 (``run_rms_fma``); updates x in place."""
    return _rms_fma(x, y, z)


def gated_attention_triton(x: torch.Tensor, gate_logits: torch.Tensor, quantize: bool = True):
    """triton_ops.py:444 (``run_gated_attention``): (e4m3, scales), or (bf16, None)."""
    return _gated_attention(x, gate_logits, quantize)


# ----------------------------------------------------------------------------- RMSNorm + RoPE
# Same op names and schemas as the reference's ops_cpp registrations
# (ltx-kernels/src/ltx_kernels/blockwise/functional.py:25-74).
@torch.library.custom_op("q8_kernels_ops::rms_norm_rope", mutates_args=())
def _rms_norm_rope_cuda(x: torch.Tensor, weights: Optional[torch.Tensor], cos_freqs: torch.Tensor,
                        sin_freqs: torch.Tensor, out_16bit: bool) -> torch.Tensor:
    return ops.rms_norm_rope(x, cos_freqs, sin_freqs, weights, out_fp8=not out_16bit)


@_rms_norm_rope_cuda.register_fake
def _rms_norm_rope_cuda_fake(x, weights, cos_freqs, sin_freqs, out_16bit):
    return torch.empty(x.shape, dtype=torch.bfloat16 if out_16bit else torch.float8_e4m3fn, device=x.device)


@torch.library.custom_op("q8_kernels_ops::rms_norm_split_rope", mutates_args=())
def _rms_norm_split_rope_cuda(x: torch.Tensor, sin_freqs: torch.Tensor, cos_freqs: torch.Tensor,
                              weights: torch.Tensor, out_fp8: bool) -> torch.Tensor:
    return ops.rms_norm_split_rope(x, cos_freqs, sin_freqs, weights, out_fp8=out_fp8)


@_rms_norm_split_rope_cuda.register_fake
def _rms_norm_split_rope_cuda_fake(x, sin_freqs, cos_freqs, weights, out_fp8):
    return torch.empty(x.shape, dtype=torch.float8_e4m3fn if out_fp8 else torch.bfloat16, device=x.device)


def rms_norm_rope(x: torch.Tensor, cos_freqs: torch.Tensor, sin_freqs: torch.Tensor,
                  weights: Optional[torch.Tensor] = None, out_fp8: bool = False) -> torch.Tensor:
    """RMSNorm (no epsilon) + interleaved RoPE (functional.py:93-102 of the reference)."""
    return torch.ops.q8_kernels_ops.rms_norm_rope(x, weights, cos_freqs, sin_freqs, not out_fp8)


def rms_norm_split_rope(x: torch.Tensor, cos_freqs: torch.Tensor, sin_freqs: torch.Tensor,
                        weights: Optional[torch.Tensor] = None, out_fp8: bool = False) -> torch.Tensor:
    """RMSNorm (eps 1e-6) + split RoPE (functional.py:105-125 of the reference)."""
    if weights is None:
        weights = torch.ones(x.shape[-1], dtype=x.dtype, device=x.device)
    return torch.ops.q8_kernels_ops.rms_norm_split_rope(x, sin_freqs, cos_freqs, weights, out_fp8)


run_quant_blockwise_norm_tma_aligned = blockwise_quantize_adanorm_triton
run_quant_blockwise_rms_fma = blockwise_quantize_rms_fma_triton
run_rms_fma = rms_fma_triton
run_gated_attention = gated_attention_triton


def blockwise_dequantize_triton(x: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    return _dequant_blockwise(x, scales)


def blockwise_dequantize(x: Tuple[torch.Tensor, torch.Tensor]) -> torch.Tensor:
    """(e4m3 ``[b, s, h]``, scales) -> bf16 (functional.py:157-159)."""
    x_fp8, scales = x
    return blockwise_dequantize_triton(x_fp8, scales)


def blockwise_quantize_weights(w: torch.Tensor, block_size: int = 128,
                               scale_max: float = FP8_SCALE_MAX) -> Tuple[torch.Tensor, torch.Tensor]:
    """W ``[N, K]`` -> (e4m3 ``[N, K]``, fp32 ``[N/128, K/128]``), functional.py:128-135."""
    if block_size != 128:
        raise NotImplementedError("only 128x128 blocks are provided")
    return ops.quantize_weight_128x128(w, scale_max)


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


def fp6_blockwise_quantize_weights_torch(x: torch.Tensor, block_size: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """128x128 weight quant into the FP6 range (scale_max 0.1172, functional.py:153-154)."""
    return blockwise_quantize_weights(x, block_size, FP6_SCALE_MAX)


@torch.library.custom_op("q8_kernels_ops::fp6_pack", mutates_args=())
def _fp6_pack(x: torch.Tensor) -> torch.Tensor:
    """e4m3 codes [m, n] -> 6-bit packed uint8 [m, n*3/4] (functional.py:163-178)."""
    return ops.fp6_pack(x)


@_fp6_pack.register_fake
def _fp6_pack_fake(x: torch.Tensor) -> torch.Tensor:
    m, n = x.shape
    return torch.empty(m, (n * 3) // 4, dtype=torch.uint8, device=x.device)


@torch.library.custom_op("q8_kernels_ops::fp6_unpack", mutates_args=())
def _fp6_unpack(x: torch.Tensor, original_n: int) -> torch.Tensor:
    """6-bit packed uint8 [m, n*3/4] -> e4m3 codes uint8 [m, n] (functional.py:181-197)."""
    return ops.fp6_unpack(x, original_n)


@_fp6_unpack.register_fake
def _fp6_unpack_fake(x: torch.Tensor, original_n: int) -> torch.Tensor:
    return torch.empty(x.shape[0], original_n, dtype=torch.uint8, device=x.device)


def fp6_pack_tensor(x: torch.Tensor) -> torch.Tensor:
    return torch.ops.q8_kernels_ops.fp6_pack(x)


def fp6_unpack_tensor(x: torch.Tensor, original_n: int) -> torch.Tensor:
    return torch.ops.q8_kernels_ops.fp6_unpack(x, original_n)


fp6_pack = fp6_pack_tensor
fp6_unpack = fp6_unpack_tensor
