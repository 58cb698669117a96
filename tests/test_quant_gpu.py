"""GPU parity of the quantisation kernels against the CPU oracle (bit-exact)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from inputs import activations, bits, scales_mn, weights
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _run_quant(x_bf16_cpu, dev, mode=0):
    from ltx_kernels.blockwise import ops
    q, s = ops.quantize_1x128(x_bf16_cpu.to(dev), mode)
    torch.cuda.synchronize()
    return bits(q), scales_mn(s, x_bf16_cpu.shape[0])


@pytest.mark.parametrize("M,K", [(1, 128), (3, 256), (37, 512), (200, 4096), (1000, 2048), (64, 16384)])
def test_quant_bit_exact_vs_oracle(cuda_device, M, K):
    x = activations(M, K, seed=M + K)
    q, s = _run_quant(x, cuda_device)
    oq, os_ = O.quant_act_1x128(bits(x))
    assert np.array_equal(q, oq)
    assert O.scales_equal(s, os_[:, :M]).all()


@pytest.mark.parametrize("case", ["act_ragged", "act_4096", "act_edge"])
def test_quant_matches_reference_fixtures(cuda_device, golden, case):
    """The kernel reproduces the reference's blockwise_quantize_torch outputs."""
    d = golden("act_quant.npz")
    x = torch.from_numpy(d[f"{case}_x"].view(np.int16).copy()).view(torch.bfloat16)
    q, s = _run_quant(x, cuda_device)
    assert O.codes_equal(q, d[f"{case}_q"]).all()
    assert O.scales_equal(s, d[f"{case}_s"]).all()


def test_quant_scale_layout_and_strided_input(cuda_device):
    """Scales come back as the reference's (M, K/128) view with strides (1, align4(M));
    a row-strided input view quantises like its contiguous copy."""
    from ltx_kernels.blockwise import ops
    x = activations(13, 1024, seed=5).to(cuda_device)
    big = torch.zeros(13, 1536, dtype=torch.bfloat16, device=cuda_device)
    big[:, :1024] = x
    q1, s1 = ops.quantize_1x128(x)
    q2, s2 = ops.quantize_1x128(big[:, :1024])
    assert s1.shape == (13, 8) and s1.stride() == (1, 16)
    assert torch.equal(q1.view(torch.uint8), q2.view(torch.uint8))
    assert torch.equal(s1, s2)


def test_quant_op_and_torch_variant(cuda_device):
    """blockwise::quantize runs the functional layer's arithmetic (default: triton, the
    reference's GPU kernel); blockwise_quantize_torch is always the torch arithmetic."""
    import ltx_kernels.blockwise.functional as F
    from ltx_kernels import _lib as L
    from ltx_kernels.blockwise import ops
    x = activations(2 * 17, 512, seed=9).view(2, 17, 512).to(cuda_device)
    q, s = torch.ops.blockwise.quantize(x, False)
    qt, st = ops.quantize_1x128(x, L.QUANT_TRITON)
    assert q.shape == (2, 17, 512) and s.shape == (34, 4)
    assert torch.equal(q.view(torch.uint8).view(34, 512), qt.view(torch.uint8)) and torch.equal(s, st)
    q2, s2 = F.blockwise_quantize_torch(x)
    q3, s3 = ops.quantize_1x128(x, L.QUANT_TORCH)
    assert torch.equal(q2.view(torch.uint8).view(34, 512), q3.view(torch.uint8))
    assert torch.equal(s2, s3.t())
    F.set_quant_mode("torch")
    try:
        q4, s4 = torch.ops.blockwise.quantize(x, False)
    finally:
        F.set_quant_mode("triton")
    assert torch.equal(q4.view(torch.uint8).view(34, 512), q3.view(torch.uint8)) and torch.equal(s4, s3)
    qg, sg = torch.ops.blockwise.quantize(x, True)  # GELU (sigmoid form) before the quantiser
    assert qg.shape == (2, 17, 512) and not torch.equal(qg.view(torch.uint8), q.view(torch.uint8))


def test_quant_triton_mode_close(cuda_device):
    """The Triton-division mode differs from the torch mode by at most 2 ulp in the
    scales and one code step; the bulk of groups agree exactly."""
    from ltx_kernels.blockwise import ops
    x = activations(512, 4096, seed=11).to(cuda_device)
    qa, sa = ops.quantize_1x128(x, 0)
    qb, sb = ops.quantize_1x128(x, 1)
    ua = sa.t().contiguous().view(torch.int32).long()
    ub = sb.t().contiguous().view(torch.int32).long()
    assert (ua - ub).abs().max().item() <= 4
    da = qa.view(torch.uint8).long()
    db = qb.view(torch.uint8).long()
    assert (da - db).abs().max().item() <= 1
    assert (da == db).float().mean().item() > 0.99


@pytest.mark.parametrize("N,K,dtype", [(128, 128, torch.float32), (384, 256, torch.bfloat16),
                                       (256, 512, torch.float16), (1024, 4096, torch.float32)])
def test_weight_quant_bit_exact(cuda_device, N, K, dtype):
    from ltx_kernels.blockwise import ops
    w = weights(N, K, seed=N).to(dtype)
    w[:128, :128] = 0  # an all-zero block
    q, s = ops.quantize_weight_128x128(w.to(cuda_device))
    torch.cuda.synchronize()
    wn = bits(w) if dtype == torch.bfloat16 else w.float().numpy()
    oq, os_ = O.quant_weight_128x128(wn)
    assert O.codes_equal(bits(q), oq).all()
    assert O.scales_equal(s.cpu().numpy(), os_).all()


def test_weight_quant_matches_reference_fixtures(cuda_device, golden):
    import ltx_kernels.blockwise.functional as F
    d = golden("weight_quant.npz")
    for name, dt in (("w_f32", torch.float32), ("w_bf16", torch.bfloat16)):
        wn = d[f"{name}_w"]
        w = torch.from_numpy(wn.view(np.int16).copy()).view(torch.bfloat16) if dt == torch.bfloat16 else torch.from_numpy(wn)
        q, s = F.fp8_blockwise_quantize_weights_torch(w.to(cuda_device))
        assert O.codes_equal(bits(q), d[f"{name}_q"]).all()
        assert O.scales_equal(s.cpu().numpy(), d[f"{name}_s"]).all()


@pytest.mark.parametrize("M,K", [(5, 256), (300, 1024)])
def test_dequant_bit_exact(cuda_device, M, K):
    from ltx_kernels.blockwise import ops
    x = activations(M, K, seed=21)
    q, s = ops.quantize_1x128(x.to(cuda_device))
    out = ops.dequantize_1x128(q, s)
    ref = O.dequant_1x128(bits(q), scales_mn(s, M).T.copy(), K // 128, 1)
    assert np.array_equal(bits(out), ref)


def test_dequant_weight_layout_via_fuse_helper(cuda_device):
    """The reference's fuse rule dequantises weights by repeating the block scales per row
    (_impl.py:264-274); the dequant op must accept that strided layout."""
    import ltx_kernels.blockwise.functional as F
    w = weights(256, 384, seed=4)
    q, s = F.fp8_blockwise_quantize_weights_torch(w.to(cuda_device))
    rows = s.repeat_interleave(128, dim=0)
    out = F.blockwise_dequantize((q.unsqueeze(0), rows)).view(256, 384)
    ref = O.dequant_1x128(bits(q), rows.cpu().numpy(), rows.shape[1], 1)
    assert np.array_equal(bits(out), ref)


@pytest.mark.parametrize("M,K", [(512, 128), (37, 640), (1000, 2048)])
def test_gelu_tanh_quant_equals_torch_gelu_then_quant(cuda_device, M, K):
    """The FFN's GELU + requant in one pass equals torch's CUDA F.gelu(approximate="tanh")
    followed by the 1x128 quantiser, codes and scales bit for bit, in both arithmetics;
    (512, 128) holds every bf16 bit pattern once."""
    import torch.nn.functional as F
    from ltx_kernels import _lib as L
    from ltx_kernels.blockwise import ops
    if (M, K) == (512, 128):
        x = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).reshape(M, K).to(cuda_device)
    else:
        x = (activations(M, K, seed=M + K) * 4.0).to(torch.bfloat16).to(cuda_device)
        x[0, :128] = 0.0
        x[min(1, M - 1), 128:256] = 1e-30
    y = F.gelu(x, approximate="tanh")
    for mode in (L.QUANT_TORCH, L.QUANT_TRITON):
        q, s = ops.gelu_tanh_quantize_1x128(x, mode)
        rq, rs = ops.quantize_1x128(y, mode)
        torch.cuda.synchronize()
        a, b = q.view(torch.uint8), rq.view(torch.uint8)
        same = (a == b) | (((a & 0x7F) == 0x7F) & ((b & 0x7F) == 0x7F))
        assert bool(same.all()), (mode, int((~same).sum()))
        sv, rv = s.view(torch.int32), rs.view(torch.int32)
        assert bool(((sv == rv) | (torch.isnan(s) & torch.isnan(rs))).all()), mode
