"""FP6 weights: pack / unpack kernels, the FP6-range weight quantiser and the FP6 linear.

Packing is byte work and must be bit-exact with the oracle's restatement of
ltx-kernels/csrc/ops/fp6_pack.cu; the quantiser with scale_max 0.1172 is the pinned
128x128 weight quantiser with another range (functional.py:22,153-154).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from inputs import activations, bits, scales_mn, weights
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n", [(1, 8), (37, 1024), (512, 4096)])
def test_fp6_pack_unpack_bit_exact(cuda_device, m, n):
    import ltx_kernels.blockwise.functional as F
    g = np.random.default_rng(m + n)
    codes = g.integers(0, 256, (m, n), dtype=np.uint8)
    packed = F.fp6_pack_tensor(torch.from_numpy(codes).to(cuda_device))
    torch.cuda.synchronize()
    assert packed.shape == (m, n * 3 // 4)
    assert np.array_equal(packed.cpu().numpy(), O.fp6_pack(codes))
    un = F.fp6_unpack_tensor(packed, n)
    torch.cuda.synchronize()
    assert np.array_equal(un.cpu().numpy(), O.fp6_unpack(O.fp6_pack(codes), n))
    assert np.array_equal(un.cpu().numpy(), codes & 0x9F)  # the two top exponent bits come back zero


def test_fp6_weight_quant_and_linear(cuda_device):
    import torch.nn as nn
    import ltx_kernels.blockwise.functional as F
    from ltx_kernels.blockwise import BlockwiseFP6Linear, ops
    N, K, M = 512, 1024, 300
    w = weights(N, K, seed=21)
    q, s = F.fp6_blockwise_quantize_weights_torch(w.to(cuda_device))
    torch.cuda.synchronize()
    oq, os_ = O.quant_weight_128x128(w.numpy(), 0.1172)
    assert O.codes_equal(bits(q), oq).all() and O.scales_equal(s.cpu().numpy(), os_).all()
    assert ((bits(q) & 0x60) == 0).all()

    lin = nn.Linear(K, N, bias=True)
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(torch.randn(N, generator=torch.Generator().manual_seed(3)) * 0.01)
    layer = BlockwiseFP6Linear.from_linear(lin.to(cuda_device))
    assert layer.weight.dtype == torch.uint8 and layer.weight.shape == (N, K * 3 // 4)
    assert torch.equal(layer.fp8weight.view(torch.uint8), q.view(torch.uint8))
    x = activations(M, K, seed=22).to(cuda_device)
    y = layer(x.view(1, M, K))
    aq, asc = ops.quantize_1x128(x)
    torch.cuda.synchronize()
    ref = O.gemm_dequant_f32(bits(aq), scales_mn(asc, M), bits(q), s.cpu().numpy(), lin.bias.detach().float().cpu().numpy())
    m = O.error_metrics(O.bf16_to_f32(bits(y.view(M, N))), ref)
    assert m["rel_fro"] <= 1e-2 and m["bound_excess"] <= 0, m  # |d - ref| <= 2e-2 + 1 bf16 ulp


def _fp6_weight(N, K, seed, dev):
    """FP6-range codes and scales of a random weight, packed as the reference packs them."""
    from ltx_kernels.blockwise import ops
    w = weights(N, K, seed=seed).to(dev)
    q, s = ops.quantize_weight_128x128(w, scale_max=0.1172)
    return q, s, ops.fp6_pack(q.view(torch.uint8))


@pytest.mark.parametrize("N,K", [(128, 128), (256, 2048), (384, 4096)])
def test_fp6_to_tc_layout_and_scales(cuda_device, N, K):
    """Byte work, bit-exact: the kernel's reordering against the oracle's, and the
    scales x 2^-6 exactly."""
    from ltx_kernels.blockwise import ops
    q, s, w6 = _fp6_weight(N, K, 30 + N, cuda_device)
    tc, s6 = ops.fp6_to_tc(w6, s)
    torch.cuda.synchronize()
    assert tc.shape == w6.shape and tc.dtype == torch.uint8
    assert np.array_equal(tc.cpu().numpy(), O.fp6_to_tc(w6.cpu().numpy(), K))
    assert torch.equal(s6, s * 0.015625)


@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (64, 4096, 4096), (300, 384, 2048), (2048, 4096, 4096),
                                   (128, 4096, 16384)])
def test_fp6_weight_gemm_equals_unpacked_fp8_gemm(cuda_device, M, N, K):
    """The 6-bit weight path (TMA 16 x 6-bit loads, e2m3 B operand, scales x 2^-6) gives
    the same bf16 bits as the FP8 GEMM on the unpacked e4m3 codes, with and without
    split-K, with the GELU + requant epilogue and with a LoRA term; and it is within
    the GEMM bar of the oracle."""
    from ltx_kernels import _lib as L
    from ltx_kernels.blockwise import ops
    q, s, w6 = _fp6_weight(N, K, M + N + K, cuda_device)
    w8 = ops.fp6_unpack(w6, K).view(torch.float8_e4m3fn)
    assert torch.equal(w8.view(torch.uint8), q.view(torch.uint8))
    tc, s6 = ops.fp6_to_tc(w6, s)
    x = activations(M, K, seed=M + 7).to(cuda_device)
    aq, asc = ops.quantize_1x128(x)
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(5)) * 0.1).to(cuda_device)
    r = 16
    lax = (torch.randn(M, r, generator=torch.Generator().manual_seed(6)) * 0.1).to(torch.bfloat16).to(cuda_device)
    lb = (torch.randn(N, r, generator=torch.Generator().manual_seed(7)) * 0.1).to(torch.bfloat16).to(cuda_device)
    for kw in ({}, dict(split_k=False), dict(gelu=True, requant=True), dict(lora_ax=lax, lora_b=lb, lora_alpha=0.5)):
        ref = ops.gemm(aq, asc, w8, s, bias, **kw)
        out = ops.gemm(aq, asc, tc, s6, bias, w_fp6=True, **kw)
        torch.cuda.synchronize()
        if isinstance(ref, tuple):
            for a, b in zip(ref, out):
                assert torch.equal(a.view(torch.uint8) if a.dtype == torch.float8_e4m3fn else a,
                                   b.view(torch.uint8) if b.dtype == torch.float8_e4m3fn else b), kw
        else:
            assert torch.equal(ref, out), kw
    assert L.device_status() == 0
    if M * N * K <= 2048 * 4096 * 4096:
        y = ops.gemm(aq, asc, tc, s6, bias, w_fp6=True)
        torch.cuda.synchronize()
        oref = O.gemm_dequant_f32(bits(aq), scales_mn(asc, M), bits(q), s.cpu().numpy(), bias.cpu().numpy())
        m = O.error_metrics(O.bf16_to_f32(bits(y)), oref)
        assert m["bound_excess"] <= 0, m  # |d - ref| <= 2e-2 + 1 bf16 ulp


def test_fp6_linear_streams_6bit_weight(cuda_device):
    """BlockwiseFP6Linear's forward runs the 6-bit GEMM (no e4m3 copy of the weight) and
    equals the reference's unpack-then-FP8 forward bit for bit, with and without the
    cached tensor-core copy; the cache follows in-place weight updates."""
    import torch.nn as nn
    from ltx_kernels.blockwise import BlockwiseFP6Linear
    from ltx_kernels.blockwise.linear import blockwise_linear_func
    N, K, M = 512, 1024, 200
    lin = nn.Linear(K, N, bias=True)
    with torch.no_grad():
        lin.weight.copy_(weights(N, K, seed=40))
    layer = BlockwiseFP6Linear.from_linear(lin.to(cuda_device))
    x = activations(M, K, seed=41).to(cuda_device).view(1, M, K)
    ref = blockwise_linear_func((x, None), (layer.fp8weight, layer.weight_scale), layer.bias)
    y = layer(x)
    assert torch.equal(y, ref)
    layer.keep_tc_weight = True
    assert torch.equal(layer(x), ref) and torch.equal(layer(x), ref)
    cached = layer.tc_weight()
    assert layer.tc_weight()[0] is cached[0]
    with torch.no_grad():
        layer.weight_scale.mul_(2.0)
    assert layer.tc_weight()[0] is not cached[0]
    ref2 = blockwise_linear_func((x, None), (layer.fp8weight, layer.weight_scale), layer.bias)
    assert torch.equal(layer(x), ref2)
