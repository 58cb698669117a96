"""GPU parity of the fused producers (csrc/producers.cuh) against the C oracle.

The kernels fix every rounding step (fp32 row sums in a stated order, IEEE sqrt and
division, a Cody-Waite exp), so codes, scales, the in-place residual update and the
bf16 outputs must match the oracle bit for bit.  The reference's Triton producers
(ltx-kernels/src/ltx_kernels/blockwise/triton_ops.py:52-345) cannot run here; how
the restatement follows them is tested on the CPU in test_oracle.py.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from inputs import activations, bits, scales_mn
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _param(b, t, h, seed, std=0.1):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(b, t, h, generator=g) * std).to(torch.bfloat16)


def _x(b, s, h, seed):
    return activations(b * s, h, seed=seed).view(b, s, h)


def _assert_quant_equal(q, s, oq, os_, M):
    assert O.codes_equal(bits(q).reshape(M, -1), oq).all()
    assert O.scales_equal(scales_mn(s, M), os_[:, :M]).all()


@pytest.mark.parametrize("B,S,H,per_token", [
    (2, 37, 4096, False),   # broadcast AdaLN parameters, the DiT video width
    (1, 100, 2048, True),   # per-token parameters, the audio width
    (3, 5, 1152, False),    # H % 256 == 128: the last load has one group
    (1, 9, 8192, True),     # widest row
    (4, 3, 128, False),     # one group per row
])
def test_adanorm_bit_exact(cuda_device, B, S, H, per_token):
    from ltx_kernels.blockwise import ops
    x = _x(B, S, H, seed=H + S)
    T = S if per_token else 1
    sc, sh = _param(B, T, H, seed=1), _param(B, T, H, seed=2)
    q, s = ops.adanorm_quantize(x.to(cuda_device), sc.to(cuda_device), sh.to(cuda_device))
    torch.cuda.synchronize()
    oq, os_ = O.adanorm_quant(bits(x), bits(sc), bits(sh))
    _assert_quant_equal(q, s, oq, os_, B * S)


@pytest.mark.parametrize("B,S,H,per_token", [(2, 33, 4096, False), (1, 64, 2048, True), (2, 7, 1152, True)])
def test_rms_fma_bit_exact(cuda_device, B, S, H, per_token):
    from ltx_kernels.blockwise import ops
    x, y = _x(B, S, H, seed=3), _x(B, S, H, seed=4)
    z = _param(B, S if per_token else 1, H, seed=5, std=0.5)
    xd = x.to(cuda_device)
    q, s = ops.rms_fma(xd, y.to(cuda_device), z.to(cuda_device), quantize=True)
    torch.cuda.synchronize()
    ox, oq, os_ = O.rms_fma(bits(x), bits(y), bits(z), quantize=True)
    assert np.array_equal(bits(xd).reshape(B * S, H), ox.reshape(B * S, H))  # residual updated in place
    _assert_quant_equal(q, s, oq, os_, B * S)
    # the bf16 variant on the original residual
    xd2 = x.to(cuda_device)
    out = ops.rms_fma(xd2, y.to(cuda_device), z.to(cuda_device), quantize=False)
    torch.cuda.synchronize()
    ox2, oout = O.rms_fma(bits(x), bits(y), bits(z), quantize=False)
    assert np.array_equal(bits(xd2).reshape(B * S, H), ox2.reshape(B * S, H))
    assert np.array_equal(bits(out), oout)


def test_rms_fma_zero_row(cuda_device):
    """A row that sums to zero has no epsilon to save it (triton_ops.py:222-224): the
    reference and this kernel both produce NaN codes there; other rows are unaffected."""
    from ltx_kernels.blockwise import ops
    B, S, H = 1, 4, 256
    x, y = _x(B, S, H, seed=6), _x(B, S, H, seed=7)
    x[0, 2] = 0
    y[0, 2] = 0
    z = _param(B, 1, H, seed=8)
    q, s = ops.rms_fma(x.to(cuda_device), y.to(cuda_device), z.to(cuda_device))
    torch.cuda.synchronize()
    _, oq, os_ = O.rms_fma(bits(x), bits(y), bits(z))
    _assert_quant_equal(q, s, oq, os_, B * S)
    assert ((bits(q).reshape(S, H)[2] & 0x7F) == 0x7F).all()


@pytest.mark.parametrize("M,H,heads,gate_dtype,quantize", [
    (77, 4096, 32, torch.bfloat16, True),
    (50, 2048, 32, torch.bfloat16, True),    # dim_head 64: a group spans two heads
    (31, 2048, 16, torch.float32, True),
    (64, 4096, 32, torch.bfloat16, False),
    (9, 1152, 9, torch.float32, False),
])
def test_gated_attention_bit_exact(cuda_device, M, H, heads, gate_dtype, quantize):
    from ltx_kernels.blockwise import ops
    x = activations(M, H, seed=M).view(1, M, H)
    g = torch.Generator().manual_seed(M + 1)
    logits = (torch.randn(1, M, heads, generator=g) * 3.0).to(gate_dtype)
    logits[0, 0, 0] = 60.0     # saturated gates
    logits[0, 1 % M, 0] = -60.0
    res = ops.gated_attention(x.to(cuda_device), logits.to(cuda_device), quantize=quantize)
    torch.cuda.synchronize()
    lg = logits[0].numpy() if gate_dtype == torch.float32 else bits(logits[0])
    if quantize:
        q, s = res
        oq, os_ = O.gated_attention(bits(x[0]), lg, True)
        _assert_quant_equal(q, s, oq, os_, M)
    else:
        assert np.array_equal(bits(res), O.gated_attention(bits(x[0]), lg, False))


@pytest.mark.parametrize("M,K", [(1, 128), (37, 1024), (300, 4096)])
def test_gelu_quant_bit_exact(cuda_device, M, K):
    from ltx_kernels.blockwise import ops
    x = activations(M, K, seed=K)
    q, s = ops.gelu_quantize_1x128(x.to(cuda_device))
    torch.cuda.synchronize()
    oq, os_ = O.gelu_quant(bits(x))
    _assert_quant_equal(q, s, oq, os_, M)


def test_producer_custom_ops(cuda_device):
    """The reference's op names and Python entry points return what the kernels do in the
    functional layer's arithmetic (default: the reference's GPU kernels, triton mode)."""
    import ltx_kernels.blockwise.functional as F
    from ltx_kernels import _lib as L
    from ltx_kernels.blockwise import ops
    assert F.get_quant_mode() == "triton" and F.quant_mode_code() == L.QUANT_TRITON
    mode = F.quant_mode_code()
    B, S, H = 2, 19, 2048
    x = _x(B, S, H, seed=9).to(cuda_device)
    sc, sh = _param(B, 1, H, seed=10).to(cuda_device), _param(B, 1, H, seed=11).to(cuda_device)
    q, s = F.blockwise_quantize_adanorm_triton(x, None, sc, sh, torch.float8_e4m3fn, 1.0)
    q2, s2 = ops.adanorm_quantize(x, sc, sh, mode)
    assert q.shape == (B, S, H) and s.shape == (B * S, H // 128) and s.stride() == (1, 40)
    assert torch.equal(q.view(torch.uint8).view(B * S, H), q2.view(torch.uint8))
    assert torch.equal(s, s2)

    y = _x(B, S, H, seed=12).to(cuda_device)
    xa, xb = x.clone(), x.clone()
    q, s = F.blockwise_quantize_rms_fma_triton(xa, y, sc)
    q2, s2 = ops.rms_fma(xb, y, sc, True, mode)
    assert torch.equal(xa, xb) and not torch.equal(xa, x)
    assert torch.equal(q.view(torch.uint8).view(B * S, H), q2.view(torch.uint8)) and torch.equal(s, s2)
    out = F.rms_fma_triton(x.clone(), y, sc)
    assert out.shape == (B, S, H) and out.dtype == torch.bfloat16

    logits = (torch.randn(B, S, 32, device=cuda_device)).to(torch.bfloat16)
    q, s = F.gated_attention_triton(x, logits)
    assert q.dtype == torch.float8_e4m3fn and q.shape == (B, S, H)
    out, none = F.gated_attention_triton(x, logits, quantize=False)
    assert none is None and out.dtype == torch.bfloat16 and out.shape == (B, S, H)

    q, s = torch.ops.blockwise.quantize(x, True)
    q2, s2 = ops.gelu_quantize_1x128(x, mode)
    assert torch.equal(q.view(torch.uint8).view(B * S, H), q2.view(torch.uint8)) and torch.equal(s, s2)


def test_producers_two_arithmetics_close(cuda_device):
    """The triton mode (the reference's kernels: bf16 row sums in Triton's order, checked
    against them by test_ref_fixtures_gpu.py) and the IEEE torch mode (fp32 sums, pinned
    by the oracle) quantise the same normalised values: their dequantised outputs agree
    to well within one e4m3 step, and most codes are identical."""
    from ltx_kernels import _lib as L
    from ltx_kernels.blockwise import ops
    B, S, H = 1, 256, 4096
    x = _x(B, S, H, seed=13).to(cuda_device)
    sc, sh = _param(B, 1, H, seed=14).to(cuda_device), _param(B, 1, H, seed=15).to(cuda_device)
    qa, sa = ops.adanorm_quantize(x, sc, sh, L.QUANT_TORCH)
    qb, sb = ops.adanorm_quantize(x, sc, sh, L.QUANT_TRITON)
    assert (qa.view(torch.uint8) == qb.view(torch.uint8)).float().mean().item() > 0.9
    da, db = ops.dequantize_1x128(qa, sa).float(), ops.dequantize_1x128(qb, sb).float()
    rel = ((da - db).norm() / da.norm()).item()
    assert rel < 2e-2, rel


def _rope_tables(shape, seed):
    g = torch.Generator().manual_seed(seed)
    ang = (torch.rand(shape, generator=g) * 2 - 1) * 3.14159
    return ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)


@pytest.mark.parametrize("rows,dim,affine,out_fp8", [(64, 4096, True, False), (37, 2048, False, False),
                                                     (20, 1000, True, False), (16, 4096, True, True)])
def test_rms_norm_rope_bit_exact(cuda_device, rows, dim, affine, out_fp8):
    import ltx_kernels.blockwise.functional as F
    x = activations(rows, dim, seed=dim + rows)
    cos, sin = _rope_tables((rows, dim), seed=rows)
    w = (torch.randn(dim, generator=torch.Generator().manual_seed(5)) * 0.2 + 1).to(torch.bfloat16) if affine else None
    out = F.rms_norm_rope(x.view(1, rows, dim).to(cuda_device), cos.view(1, rows, dim).to(cuda_device),
                          sin.view(1, rows, dim).to(cuda_device), None if w is None else w.to(cuda_device), out_fp8)
    torch.cuda.synchronize()
    ref = O.rms_norm_rope(bits(x), bits(cos), bits(sin), None if w is None else bits(w), out_fp8)
    if out_fp8:
        assert O.codes_equal(bits(out).reshape(rows, dim), ref).all()
    else:
        assert np.array_equal(bits(out).reshape(rows, dim), ref)


@pytest.mark.parametrize("B,S,H,heads,bcast,swapped,out_fp8", [
    (2, 33, 4096, 32, True, True, False),    # the DiT video q/k: d = 128, freq table shared over the batch
    (1, 20, 2048, 32, False, False, False),  # d = 64
    (2, 9, 4096, 16, False, True, False),    # d = 256
    (1, 17, 1152, 36, True, False, False),   # d = 32, H % 256 == 128
    (2, 8, 4096, 32, False, True, True),     # saturating e4m3 output
])
def test_rms_norm_split_rope_bit_exact(cuda_device, B, S, H, heads, bcast, swapped, out_fp8):
    import ltx_kernels.blockwise.functional as F
    d = H // heads
    x = activations(B * S, H, seed=H + S).view(B, S, H)
    fb = 1 if bcast else B
    cos, sin = _rope_tables((fb, heads, S, d // 2), seed=S)
    w = (torch.randn(H, generator=torch.Generator().manual_seed(6)) * 0.2 + 1).to(torch.bfloat16)
    cd, sd = cos.to(cuda_device), sin.to(cuda_device)
    if swapped:  # logical [b, n, s, d/2] over a physical [b, s, n, d/2] buffer, as apply_split_rotary_emb hands it
        cd = cd.transpose(1, 2).contiguous().transpose(1, 2)
        sd = sd.transpose(1, 2).contiguous().transpose(1, 2)
    out = F.rms_norm_split_rope(x.to(cuda_device), cd, sd, w.to(cuda_device), out_fp8)
    torch.cuda.synchronize()
    ref = O.rms_norm_split_rope(bits(x), bits(cos), bits(sin), bits(w), out_fp8)
    if out_fp8:
        assert O.codes_equal(bits(out), ref).all()
    else:
        assert np.array_equal(bits(out), ref)
