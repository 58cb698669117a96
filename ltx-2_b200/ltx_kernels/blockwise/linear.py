"""Blockwise FP8 linear layer and the ``blockwise::fp8_gemm`` custom op, on sm_100a kernels.

Mirrors ltx-kernels/src/ltx_kernels/blockwise/linear.py of Lightricks/LTX-2:
same op name and schema (``blockwise::fp8_gemm(Tensor[] a, Tensor[] b, Tensor?
bias, bool use_fast_accum) -> Tensor``, linear.py:55-75), same module classes,
parameters and weight/scale layout (linear.py:111-209), so ltx-core's blockwise
policy (ltx_core/quantization/blockwise/_impl.py:12-24,97-115) can use it unchanged.

Differences, all deliberate:
* the GEMM is the tcgen05/TMEM kernel of ``ltxfp8_gemm``; ``use_fast_accum`` is
  accepted and ignored -- accumulation is always fp32 (the reference forces fp32
  on Blackwell anyway, linear.py:98-102);
* any K % 128 == 0 is accepted (the SM89 kernel only takes K in {2048, 4096,
  8192, 16384}, kernels/geforce/static_switch.h:12-34);
* the activation quantiser is the CUDA kernel of ``ltxfp8_quantize_1x128``.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.nn as nn

from . import ops
from .functional import blockwise_quantize_triton, blockwise_quantize_weights


@torch.library.custom_op("blockwise::fp8_gemm", mutates_args=())
def blockwise_fp8_gemm(
    a: List[torch.Tensor],
    b: List[torch.Tensor],
    bias: Optional[torch.Tensor],
    use_fast_accum: bool,
) -> torch.Tensor:
    return ops.gemm(a[0], a[1], b[0], b[1], bias)


@blockwise_fp8_gemm.register_fake
def blockwise_fp8_gemm_fake(
    a: List[torch.Tensor],
    b: List[torch.Tensor],
    bias: Optional[torch.Tensor],
    use_fast_accum: bool,
) -> torch.Tensor:
    return torch.empty(a[0].shape[0], b[0].shape[0], dtype=torch.bfloat16, device=b[0].device)


@torch.library.custom_op("blockwise::fp6_gemm", mutates_args=())
def blockwise_fp6_gemm(
    a: List[torch.Tensor],
    b: List[torch.Tensor],
    bias: Optional[torch.Tensor],
) -> torch.Tensor:
    """``blockwise::fp8_gemm`` with a 6-bit weight ``b = (w6_tc, sfb6)`` from
    ``ops.fp6_to_tc``: the tensor core reads the packed codes directly.  No
    reference counterpart (the reference unpacks to e4m3 first, linear.py:244-250)."""
    return ops.gemm(a[0], a[1], b[0], b[1], bias, w_fp6=True)


@blockwise_fp6_gemm.register_fake
def blockwise_fp6_gemm_fake(
    a: List[torch.Tensor],
    b: List[torch.Tensor],
    bias: Optional[torch.Tensor],
) -> torch.Tensor:
    return torch.empty(a[0].shape[0], b[0].shape[0], dtype=torch.bfloat16, device=b[0].device)


def is_16bit(x) -> bool:
    return x.dtype == torch.float16 or x.dtype == torch.bfloat16


class BlockwiseGemmLinearFunc(torch.autograd.Function):
    """Forward-only blockwise FP8 linear (linear.py:82-104): quantise a bf16 input
    (or take a pre-quantised ``(e4m3, scales)`` pair), GEMM, view to ``(b, n, out)``."""

    @staticmethod
    def forward(ctx, a, w, bias):
        if is_16bit(a[0]):
            a = blockwise_quantize_triton(a[0])
        b, n, h = a[0].shape
        out_h, _ = w[0].shape
        new_a = (a[0].view(-1, h), a[1])
        d = blockwise_fp8_gemm(list(new_a), list(w), bias, False)
        return d.view(b, n, out_h)


def blockwise_linear_func(a, b, bias=None):
    return BlockwiseGemmLinearFunc.apply(a, b, bias)


class BlockwiseLinear(nn.Module):
    """Base class of the blockwise quantised linear layers (linear.py:111-148)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        if bias:
            # fp32: the GEMM's bias operand is float* (api.cpp:52-56).
            self.bias = nn.Parameter(torch.empty(out_features, device=device, dtype=torch.float32),
                                     requires_grad=False)
        else:
            self.register_parameter("bias", None)

    @property
    def fp8weight(self):
        raise NotImplementedError("Subclasses must implement the weight property")

    def forward(self, x):
        if not isinstance(x, tuple):
            x = (x, None)
        return blockwise_linear_func(x, (self.fp8weight, self.weight_scale), self.bias)

    @classmethod
    def from_linear(cls, linear: nn.Linear, transform_weights=True):
        raise NotImplementedError("Subclasses must implement from_linear method")


class BlockwiseFP8Linear(BlockwiseLinear):
    """e4m3 weight ``[out, in]`` with fp32 128x128 block scales ``[out/128, in/128]``
    (linear.py:151-209)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None):
        super().__init__(in_features, out_features, bias, device, dtype)
        assert in_features % 128 == 0, f"in_features must be divisible by 128, got {in_features}"
        assert out_features % 128 == 0, f"out_features must be divisible by 128, got {out_features}"
        self.weight = nn.Parameter(torch.empty(out_features, in_features, device=device, dtype=torch.float8_e4m3fn),
                                   requires_grad=False)
        self.weight_scale = nn.Parameter(
            torch.ones(out_features // 128, in_features // 128, device=device, dtype=torch.float32),
            requires_grad=False)

    @property
    def fp8weight(self):
        return self.weight

    @classmethod
    def from_linear(cls, linear: nn.Linear, transform_weights=True):
        layer = cls(linear.in_features, linear.out_features, linear.bias is not None, device=linear.weight.device)
        if transform_weights:
            w_fp8, w_scales = blockwise_quantize_weights(linear.weight.data.cuda())
        else:
            w_fp8 = torch.empty(linear.out_features, linear.in_features, dtype=torch.float8_e4m3fn,
                                device=linear.weight.device)
            w_scales = torch.ones(w_fp8.shape[0] // 128, w_fp8.shape[1] // 128, device=w_fp8.device,
                                  dtype=torch.float32)
        layer.weight.data = w_fp8
        layer.weight_scale.data = w_scales
        if linear.bias is not None:
            layer.bias.data = linear.bias.data.to(torch.float32)
        return layer


class BlockwiseFP6Linear(BlockwiseLinear):
    """FP6-range weights stored 6-bit packed ``[out, in*3/4]`` uint8 with fp32 128x128
    block scales ``[out/128, in/128]`` (linear.py:212-284).

    The reference's forward unpacks the codes to an e4m3 weight and runs the FP8 GEMM
    (linear.py:244-250).  Here the forward rewrites the packed codes into the tensor
    core's 6-bit order (``ops.fp6_to_tc``, same size) and the GEMM streams them at 6
    bits per element as e2m3 operands, with identical results.  ``keep_tc_weight``
    (default False) keeps that copy between calls (0.75 byte per weight element more
    memory, no per-call rewrite); ``weight`` and ``weight_scale`` stay in the
    reference's layout either way.  ``fp8weight`` still gives the unpacked e4m3 codes."""

    keep_tc_weight: bool = False

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None):
        assert in_features % 8 == 0, f"in_features must be divisible by 8 for fp6_pack, got {in_features}"
        assert in_features % 128 == 0, f"in_features must be divisible by 128, got {in_features}"
        assert out_features % 128 == 0, f"out_features must be divisible by 128, got {out_features}"
        super().__init__(in_features, out_features, bias, device, dtype)
        self.weight = nn.Parameter(torch.empty(out_features, (in_features // 4) * 3, device=device, dtype=torch.uint8),
                                   requires_grad=False)
        self.weight_scale = nn.Parameter(
            torch.ones(out_features // 128, in_features // 128, device=device, dtype=torch.float32),
            requires_grad=False)

    @property
    def fp8weight(self):
        from .functional import fp6_unpack_tensor
        return fp6_unpack_tensor(self.weight, self.in_features).view(torch.float8_e4m3fn)

    def tc_weight(self):
        """``(w6_tc, sfb6)``: the weight in the tensor core's 6-bit order and its scales
        x 2^-6, cached while ``keep_tc_weight`` is set and the parameters are unchanged."""
        key = (self.weight.data_ptr(), self.weight._version, self.weight_scale.data_ptr(),
               self.weight_scale._version)
        cached = self.__dict__.get("_tc_cache")
        if self.keep_tc_weight and cached is not None and cached[0] == key:
            return cached[1]
        tc = ops.fp6_to_tc(self.weight, self.weight_scale)
        self.__dict__["_tc_cache"] = (key, tc) if self.keep_tc_weight else None
        return tc

    def forward(self, x):
        a = x if isinstance(x, tuple) else (x, None)
        if is_16bit(a[0]):
            a = blockwise_quantize_triton(a[0])
        b, n, h = a[0].shape
        d = blockwise_fp6_gemm([a[0].view(-1, h), a[1]], list(self.tc_weight()), self.bias)
        return d.view(b, n, self.out_features)

    @classmethod
    def from_linear(cls, linear: nn.Linear, transform_weights=True):
        from .functional import fp6_blockwise_quantize_weights_torch, fp6_pack_tensor
        layer = cls(linear.in_features, linear.out_features, linear.bias is not None, device=linear.weight.device)
        if transform_weights:
            w_fp6, w_scales = fp6_blockwise_quantize_weights_torch(linear.weight.data.cuda())
            layer.weight.data = fp6_pack_tensor(w_fp6.view(torch.uint8))
            layer.weight_scale.data = w_scales
        if linear.bias is not None:
            layer.bias.data = linear.bias.data.to(torch.float32)
        return layer
