"""Load-time LoRA merge (ltxfp8_lora_fuse_weight) against the reference's three passes.

The reference (ltx-core/src/ltx_core/quantization/blockwise/_impl.py:263-301) dequantises
the weight to bf16, adds the bf16 LoRA delta and requantises in 128x128 blocks.  The
oracle composes the same three steps (dequant, bf16 add, the pinned weight quantiser),
so codes and scales must match bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from inputs import activations, bits, lora as make_lora, scales_mn, weights
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _reference_merge(wq, wsc, delta):
    """dequant (scale per 128x128 block) -> bf16 + delta (fp32 add, bf16 round) -> 128x128 quant."""
    N, K = wq.shape
    scales_rows = np.repeat(wsc, 128, axis=0)                       # [N, K/128], one row per weight row
    w_bf16 = O.dequant_1x128(wq, scales_rows, scales_rows.shape[1], 1)
    merged = O.f32_to_bf16(O.bf16_to_f32(w_bf16) + O.bf16_to_f32(delta))
    return O.quant_weight_128x128(merged)


@pytest.mark.parametrize("N,K,r", [(256, 512, 32), (1024, 2048, 128), (128, 128, 16)])
def test_lora_fuse_bit_exact(cuda_device, N, K, r):
    from ltx_kernels.blockwise import lora_fuse, ops
    w = weights(N, K, seed=N + K)
    wq, wsc = ops.quantize_weight_128x128(w.to(cuda_device))
    a, b = make_lora(N, K, r, seed=K)
    delta = lora_fuse.aggregate_lora_products([(a.to(cuda_device), b.to(cuda_device), 0.8)])
    q2, s2 = lora_fuse.blockwise_fp8_fuse(wq, wsc, delta)
    torch.cuda.synchronize()
    oq, os_ = _reference_merge(bits(wq), wsc.cpu().numpy(), bits(delta))
    assert O.codes_equal(bits(q2), oq).all()
    assert O.scales_equal(s2.cpu().numpy(), os_).all()
    # in place gives the same
    wq_i, wsc_i = wq.clone(), wsc.clone()
    lora_fuse.blockwise_fp8_fuse(wq_i, wsc_i, delta, inplace=True)
    torch.cuda.synchronize()
    assert torch.equal(wq_i.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(wsc_i, s2)


def test_fuse_rule_and_merged_gemm(cuda_device):
    """The ltx-core fuse-rule drop-in; the merged weight's GEMM against the dequantised
    merged weight (the reference's load-time result), and the runtime-LoRA GEMM against
    the exact dequant(W) x + s B (A x).  Requantising W + delta snaps small deltas back
    onto W's e4m3 grid, so only the runtime route keeps the whole LoRA term."""
    from ltx_kernels.blockwise import lora_fuse, ops

    class _SD:
        def __init__(self, sd):
            self.sd = sd

    M, N, K, r, strength = 256, 512, 1024, 64, 0.7
    w = weights(N, K, seed=3)
    wq, wsc = ops.quantize_weight_128x128(w.to(cuda_device))
    a, b = make_lora(N, K, r, seed=4)
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    delta = lora_fuse.aggregate_lora_products([(ad, bd, strength)])
    sd = _SD({"blk.ff.weight": wq, "blk.ff.weight_scale": wsc,
              "blk.norm.weight": torch.ones(N, K, device=cuda_device, dtype=torch.bfloat16)})
    out = lora_fuse.blockwise_fp8_fuse_rule("blk.ff.weight", wq, delta.clone(), sd)
    assert set(out) == {"blk.ff.weight", "blk.ff.weight_scale"}
    q2, s2 = lora_fuse.blockwise_fp8_fuse(wq, wsc, delta)
    assert torch.equal(out["blk.ff.weight"].view(torch.uint8), q2.view(torch.uint8))
    plain = lora_fuse.blockwise_fp8_fuse_rule("blk.norm.weight", sd.sd["blk.norm.weight"], delta.clone(), sd)
    assert torch.equal(plain["blk.norm.weight"], (delta.float() + 1).to(torch.bfloat16))

    x = activations(M, K, seed=5)
    aq, asc = ops.quantize_1x128(x.to(cuda_device))
    d_merged = ops.gemm(aq, asc, q2, s2)
    ax = ops.lora_a(x.to(cuda_device), ad)
    d_runtime = ops.gemm(aq, asc, wq, wsc, lora_ax=ax, lora_b=bd, lora_alpha=strength)
    torch.cuda.synchronize()
    ref_merged = O.gemm_dequant_f32(bits(aq), scales_mn(asc, M), bits(q2), s2.cpu().numpy(), None)
    m = O.error_metrics(O.bf16_to_f32(bits(d_merged)), ref_merged)
    assert m["rel_fro"] <= 1e-2 and m["bound_excess"] <= 0, m  # |d - ref| <= 2e-2 + 1 bf16 ulp
    ref_exact = O.gemm_dequant_f32(bits(aq), scales_mn(asc, M), bits(wq), wsc.cpu().numpy(), None) \
        + O.lora_exact_f32(bits(x), bits(a), bits(b), strength)
    m = O.error_metrics(O.bf16_to_f32(bits(d_runtime)), ref_exact)
    assert m["rel_fro"] <= 1e-2 and m["bound_excess"] <= 0, m  # |d - ref| <= 2e-2 + 1 bf16 ulp
