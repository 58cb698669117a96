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
