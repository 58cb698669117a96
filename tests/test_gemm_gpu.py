"""GPU parity of the tcgen05 blockwise GEMM and its fused epilogues against the oracle.

Tolerance (the parity bar): relative Frobenius error <= 1e-2 and, element by
element, |D - ref| <= 2e-2 + one bf16 ulp of |ref| against the reference's
dequantise-then-fp32-matmul result.  The ulp term is what a correctly rounded
bf16 output needs (one ulp is already 0.0625 at |D| in [8, 16)); it does not grow
with max|ref| the way a normalised bound would.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from inputs import activations, bias as make_bias, bits, lora as make_lora, scales_mn, weights
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_FRO = 1e-2
ABS_TOL = 2e-2


def _problem(M, N, K, dev, seed=0, with_bias=True):
    from ltx_kernels.blockwise import ops
    x = activations(M, K, seed=seed)
    w = weights(N, K, seed=seed + 1)
    b = make_bias(N, seed=seed + 2) if with_bias else None
    aq, asc = ops.quantize_1x128(x.to(dev))
    wq, wsc = ops.quantize_weight_128x128(w.to(dev))
    return x, aq, asc, wq, wsc, (None if b is None else b.to(dev))


def _oracle(aq, asc, wq, wsc, b, rows=None):
    M = aq.shape[0]
    return O.gemm_dequant_f32(bits(aq), scales_mn(asc, M), bits(wq), wsc.cpu().numpy(),
                              None if b is None else b.cpu().numpy(), rows=rows)


def _check(out_bf16, ref_f32):
    m = O.error_metrics(O.bf16_to_f32(bits(out_bf16)), ref_f32, abs_tol=ABS_TOL)
    assert np.isfinite(O.bf16_to_f32(bits(out_bf16))).all()
    assert m["rel_fro"] <= REL_FRO and m["bound_excess"] <= 0, m
    return m


@pytest.mark.parametrize("M,N,K", [
    (128, 256, 128),      # one tile, one K block
    (1, 128, 256),        # single row, half tile in N
    (37, 384, 512),       # ragged M, N % 256 == 128
    (200, 640, 384),      # K not a power of two
    (256, 512, 1024),
    (1000, 1024, 2048),   # several tiles per CTA row
])
def test_gemm_small_shapes(cuda_device, M, N, K):
    from ltx_kernels.blockwise import ops
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=M)
    d = ops.gemm(aq, asc, wq, wsc, b)
    torch.cuda.synchronize()
    m = _check(d, _oracle(aq, asc, wq, wsc, b))
    assert m["rel_fro"] < 3e-3


def test_gemm_matches_promoted_order_oracle(cuda_device):
    """Against the SM89 kernel's per-128-K promotion order (scalar C restatement)."""
    from ltx_kernels.blockwise import ops
    M, N, K = 64, 256, 512
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=3)
    d = ops.gemm(aq, asc, wq, wsc, b)
    sa = asc.t().contiguous().cpu().numpy()
    f, h = O.gemm_promoted(bits(aq), sa, sa.shape[1], bits(wq), wsc.cpu().numpy(), b.cpu().numpy(), M, N, K)
    _check(d, f)
    # differences are bf16 rounding flips only
    diff = np.abs(bits(d).astype(np.int32) - h.astype(np.int32))
    assert (diff <= 1).all() and (diff == 0).mean() > 0.98


def test_gemm_no_bias_and_reference_fixture(cuda_device, golden):
    """The reference's own CPU GEMM result (gemm_ref.npz) from its own quantised operands."""
    from ltx_kernels.blockwise import ops
    g = golden("gemm_ref.npz")
    M, K = g["x"].shape
    aq = torch.from_numpy(g["aq"]).view(torch.float8_e4m3fn).to(cuda_device)
    asc = torch.from_numpy(g["asc"]).to(cuda_device)          # contiguous [K/128, M]
    wq = torch.from_numpy(g["wq"]).view(torch.float8_e4m3fn).to(cuda_device)
    wsc = torch.from_numpy(g["wsc"]).to(cuda_device)
    bias = torch.from_numpy(g["bias"]).to(cuda_device)
    d = ops.gemm(aq, asc, wq, wsc, bias)
    _check(d, g["d_f32"])
    d0 = ops.gemm(aq, asc, wq, wsc, None)
    ref0 = g["d_f32"] - g["bias"][None, :]
    _check(d0, ref0)


def test_gemm_zero_rows_give_nan_like_reference(cuda_device):
    """All-zero token rows quantise to NaN codes with scale 0 (reference behaviour for
    padded rows); their GEMM output is NaN while other rows stay exact."""
    from ltx_kernels.blockwise import ops
    M, N, K = 8, 256, 256
    x = activations(M, K, seed=1)
    x[3] = 0
    w = weights(N, K)
    aq, asc = ops.quantize_1x128(x.to(cuda_device))
    wq, wsc = ops.quantize_weight_128x128(w.to(cuda_device))
    d = ops.gemm(aq, asc, wq, wsc, None).float().cpu()
    assert torch.isnan(d[3]).all()
    keep = [i for i in range(M) if i != 3]
    ref = _oracle(aq, asc, wq, wsc, None, rows=np.array(keep))
    m = O.error_metrics(d[keep].numpy(), ref)
    assert m["rel_fro"] <= REL_FRO


def test_gemm_custom_op_and_blockwise_cpp_shim(cuda_device):
    import blockwise_cpp
    from ltx_kernels.blockwise import ops
    M, N, K = 96, 512, 1024
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=8)
    d1 = torch.ops.blockwise.fp8_gemm([aq, asc], [wq, wsc], b, True)
    d2 = torch.empty(M, N, dtype=torch.bfloat16, device=cuda_device)
    blockwise_cpp.fp8_gemm_nt_sm89((aq, asc), (wq, wsc), d2, bias=b, use_fast_accum=True)
    d3 = ops.gemm(aq, asc, wq, wsc, b)
    assert torch.equal(d1, d3) and torch.equal(d2, d3)


def test_gemm_is_deterministic(cuda_device):
    from ltx_kernels.blockwise import ops
    x, aq, asc, wq, wsc, b = _problem(777, 1280, 1024, cuda_device, seed=4)
    d1 = ops.gemm(aq, asc, wq, wsc, b)
    d2 = ops.gemm(aq, asc, wq, wsc, b)
    assert torch.equal(d1, d2)


# --------------------------------------------------------------------------- fused epilogues
def test_gelu_epilogue(cuda_device):
    """GELU-tanh on bf16(acc + bias), rounded to bf16: compare with torch's own CUDA gelu
    applied to this kernel's plain bf16 output (the reference's unfused chain)."""
    from ltx_kernels.blockwise import ops
    M, N, K = 300, 768, 1024
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=6)
    d_plain = ops.gemm(aq, asc, wq, wsc, b)
    d_gelu = ops.gemm(aq, asc, wq, wsc, b, gelu=True)
    ref = torch.nn.functional.gelu(d_plain, approximate="tanh")
    a, r = d_gelu.float(), ref.float()
    exact = (a == r)
    assert exact.float().mean().item() > 0.99
    ulp = (bits(d_gelu).astype(np.int32) - bits(ref).astype(np.int32))
    close = (np.abs(ulp) <= 1) | (np.abs(a.cpu().numpy() - r.cpu().numpy()) <= 1e-6)
    assert close.all()


@pytest.mark.parametrize("gelu", [False, True])
def test_requant_epilogue_bit_exact(cuda_device, gelu):
    """Requantised codes/scales are bit-exact with the oracle's 1x128 quantisation of the
    kernel's own bf16 output (written alongside)."""
    from ltx_kernels.blockwise import ops
    M, N, K = 259, 1024, 512
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=7)
    d, q, s = ops.gemm(aq, asc, wq, wsc, b, gelu=gelu, requant=True, write_d=True)
    assert s.shape == (M, N // 128) and s.stride() == (1, 260)
    oq, os_ = O.quant_act_1x128(bits(d))
    assert O.codes_equal(bits(q), oq).all()
    assert O.scales_equal(scales_mn(s, M), os_[:, :M]).all()
    # skip_d: same codes without writing D
    _, q2, s2 = ops.gemm(aq, asc, wq, wsc, b, gelu=gelu, requant=True, write_d=False)
    assert torch.equal(q.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(s, s2)


def test_ffn_pair_matches_unfused_chain(cuda_device):
    """FFN: up (GELU + requant fused) -> down, vs the reference's chain
    GEMM -> bf16 -> F.gelu -> quantise -> GEMM, evaluated with the oracle."""
    from ltx_kernels.blockwise import ops
    M, D, H = 200, 512, 2048
    x = activations(M, D, seed=12)
    w1 = weights(H, D, seed=13)
    w2 = weights(D, H, seed=14)
    b1, b2 = make_bias(H, seed=15).to(cuda_device), make_bias(D, seed=16).to(cuda_device)
    aq, asc = ops.quantize_1x128(x.to(cuda_device))
    w1q, w1s = ops.quantize_weight_128x128(w1.to(cuda_device))
    w2q, w2s = ops.quantize_weight_128x128(w2.to(cuda_device))
    _, hq, hs = ops.gemm(aq, asc, w1q, w1s, b1, gelu=True, requant=True, write_d=False)
    out = ops.gemm(hq, hs, w2q, w2s, b2)
    # oracle chain
    h = O.f32_to_bf16(_oracle(aq, asc, w1q, w1s, b1))
    g = O.gelu_tanh_bf16(h)
    gq, gs = O.quant_act_1x128(g)
    ref = O.gemm_dequant_f32(gq, gs, bits(w2q), w2s.cpu().numpy(), b2.cpu().numpy())
    _check(out, ref)


@pytest.mark.parametrize("r", [16, 32, 128])
def test_lora_a_kernel(cuda_device, r):
    from ltx_kernels.blockwise import ops
    M, K = 300, 1024
    x = activations(M, K, seed=30)
    a, _ = make_lora(256, K, r)
    ax = ops.lora_a(x.to(cuda_device), a.to(cuda_device))
    ref = O.bf16_to_f32(bits(x)) @ O.bf16_to_f32(bits(a)).T
    m = O.error_metrics(O.bf16_to_f32(bits(ax)), ref)
    assert m["rel_fro"] < 4e-3, m


@pytest.mark.parametrize("r", [32, 128])
def test_gemm_with_runtime_lora(cuda_device, r):
    """dequant(W) x + alpha B (A x) + bias: exact LoRA math as the oracle."""
    from ltx_kernels.blockwise.fused import fp8_linear
    M, N, K = 333, 768, 1024
    x = activations(M, K, seed=40)
    w = weights(N, K, seed=41)
    b = make_bias(N, seed=42)
    la, lb = make_lora(N, K, r, seed=43)
    la = la * 8
    lb = lb * 8   # make the LoRA term visible above the base error
    from ltx_kernels.blockwise import ops
    wq, wsc = ops.quantize_weight_128x128(w.to(cuda_device))
    dev = cuda_device
    out = fp8_linear(x.to(dev), wq, wsc, b.to(dev), lora=(la.to(dev), lb.to(dev), 0.5))
    aq, asc = ops.quantize_1x128(x.to(dev))
    base = _oracle(aq, asc, wq, wsc, b.to(dev))
    ref = base + O.lora_exact_f32(bits(x), bits(la), bits(lb), 0.5)
    m = _check(out, ref)
    lora_only = O.lora_exact_f32(bits(x), bits(la), bits(lb), 0.5)
    # the LoRA term is not negligible, and without it the error would be large
    assert np.linalg.norm(lora_only) / np.linalg.norm(ref) > 0.05
    assert m["rel_fro"] < 5e-3


# --------------------------------------------------------------------------- both kernels on every shape class
@pytest.fixture
def gemm_variant():
    from ltx_kernels import _lib
    yield _lib.set_gemm_variant
    _lib.set_gemm_variant(_lib.GEMM_AUTO)


@pytest.mark.parametrize("variant", [1, 2], ids=["one_cta", "cta_pair"])
@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (100, 384, 256), (128, 256, 512), (129, 640, 384),
                                   (300, 1024, 1024), (513, 256, 2048)])
def test_gemm_kernel_variants(cuda_device, gemm_variant, variant, M, N, K):
    from ltx_kernels.blockwise import ops
    gemm_variant(variant)
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=M + N)
    d = ops.gemm(aq, asc, wq, wsc, b)
    torch.cuda.synchronize()
    m = _check(d, _oracle(aq, asc, wq, wsc, b))
    assert m["rel_fro"] < 3e-3


@pytest.mark.parametrize("variant", [1, 2], ids=["one_cta", "cta_pair"])
def test_fused_epilogues_variants(cuda_device, gemm_variant, variant):
    """GELU + requant and LoRA through each kernel; both kernels agree bit-for-bit."""
    from ltx_kernels.blockwise import ops
    M, N, K, r = 300, 768, 1024, 32
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=77)
    la, lb = make_lora(N, K, r, seed=78)
    ax = ops.lora_a(x.to(cuda_device), la.to(cuda_device))
    gemm_variant(variant)
    d, q, s = ops.gemm(aq, asc, wq, wsc, b, gelu=True, requant=True, write_d=True, split_k=False)
    oq, os_ = O.quant_act_1x128(bits(d))
    assert O.codes_equal(bits(q), oq).all()
    assert O.scales_equal(scales_mn(s, M), os_[:, :M]).all()
    dl = ops.gemm(aq, asc, wq, wsc, b, lora_ax=ax, lora_b=lb.to(cuda_device), lora_alpha=0.5, split_k=False)
    gemm_variant(1 if variant == 2 else 2)
    d2, q2, s2 = ops.gemm(aq, asc, wq, wsc, b, gelu=True, requant=True, write_d=True, split_k=False)
    dl2 = ops.gemm(aq, asc, wq, wsc, b, lora_ax=ax, lora_b=lb.to(cuda_device), lora_alpha=0.5, split_k=False)
    # Same promotion order in both kernels (no split-K): identical results.
    assert torch.equal(d, d2) and torch.equal(q.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(s, s2)
    assert torch.equal(dl, dl2)


def test_bounded_wait_failure_path(cuda_device):
    """A barrier nothing arrives on: the kernel's wait gives up after ~1 s, records a
    status the host reads, and the context stays usable for the next GEMM."""
    import time
    from ltx_kernels import _lib
    from ltx_kernels.blockwise import ops
    t0 = time.time()
    st = _lib.selftest_wait_timeout(1_000_000_000, torch.cuda.current_stream().cuda_stream)
    dt = time.time() - t0
    assert st == _lib.SELFTEST_STATUS
    assert 0.9 < dt < 30
    assert ops.device_status() == 0          # read-and-clear left the word clean
    x, aq, asc, wq, wsc, b = _problem(64, 256, 256, cuda_device, seed=90)
    d = ops.gemm(aq, asc, wq, wsc, b)
    _check(d, _oracle(aq, asc, wq, wsc, b))


def test_gemm_in_cuda_graph(cuda_device):
    """The C ABI neither allocates nor synchronises: a captured graph replays the
    quantiser and both GEMM epilogues with results identical to eager launches."""
    from ltx_kernels.blockwise import ops
    M, K, N = 256, 512, 384
    x = activations(M, K, seed=91).to(cuda_device)
    wq, wsc = ops.quantize_weight_128x128(weights(N, K, seed=92).to(cuda_device))
    b = make_bias(N).to(cuda_device)

    def run():
        aq, asc = ops.quantize_1x128(x)
        d = ops.gemm(aq, asc, wq, wsc, b)
        _, q, s = ops.gemm(aq, asc, wq, wsc, b, gelu=True, requant=True, write_d=False)
        return d, q, s

    eager = run()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        run()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = run()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out[0], eager[0])
    assert torch.equal(out[1].view(torch.uint8), eager[1].view(torch.uint8)) and torch.equal(out[2], eager[2])


# --------------------------------------------------------------------------- split-K for skinny M
@pytest.mark.parametrize("M,N,K", [(1, 128, 4096), (100, 256, 4096), (128, 2048, 2048), (256, 4096, 4096),
                                   (96, 384, 2560)])
def test_splitk_skinny_shapes(cuda_device, M, N, K):
    from ltx_kernels.blockwise import ops
    ws = ops.gemm_workspace_bytes(M, N, K, cuda_device)
    assert ws > 0  # these shapes have few output tiles: split-K engages
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=K + M)
    d = ops.gemm(aq, asc, wq, wsc, b)
    d1 = ops.gemm(aq, asc, wq, wsc, b, split_k=False)
    m = _check(d, _oracle(aq, asc, wq, wsc, b))
    assert m["rel_fro"] < 3e-3
    # split order differs from the single-unit promotion only by fp32 summation order
    diff = (d.float() - d1.float()).abs().max().item()
    assert diff <= 0.02 * d1.float().abs().max().item()
    assert torch.equal(d, ops.gemm(aq, asc, wq, wsc, b))  # deterministic


def test_splitk_fused_epilogues(cuda_device):
    """GELU + requant and LoRA through the split-K reduction."""
    from ltx_kernels.blockwise import ops
    M, N, K, r = 128, 1024, 2048, 32
    assert ops.gemm_workspace_bytes(M, N, K, cuda_device) > 0
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=123)
    d, q, s = ops.gemm(aq, asc, wq, wsc, b, gelu=True, requant=True, write_d=True)
    oq, os_ = O.quant_act_1x128(bits(d))
    assert O.codes_equal(bits(q), oq).all()
    assert O.scales_equal(scales_mn(s, M), os_[:, :M]).all()
    ref = O.bf16_to_f32(O.gelu_tanh_bf16(O.f32_to_bf16(_oracle(aq, asc, wq, wsc, b))))
    _check(d, ref)
    la, lb = make_lora(N, K, r, seed=124)
    ax = ops.lora_a(x.to(cuda_device), la.to(cuda_device))
    dl = ops.gemm(aq, asc, wq, wsc, b, lora_ax=ax, lora_b=lb.to(cuda_device), lora_alpha=0.5)
    ref = _oracle(aq, asc, wq, wsc, b) + O.lora_exact_f32(bits(x), bits(la), bits(lb), 0.5)
    _check(dl, ref)


@pytest.mark.parametrize("M,N,K", [(6144, 4096, 16384), (5000, 4096, 8192), (6144, 8192, 8192)])
def test_tail_wave_split(cuda_device, M, N, K):
    """A mostly empty last wave of long tiles is split along K (the 8-GPU DiT shard sizes):
    its M-tile rows run as a second, skinny split-K launch.  Same result as the unsplit
    kernel up to fp32 summation order, deterministic; bias, GELU + requant and LoRA rows
    addressed correctly on both sides of the split row."""
    from ltx_kernels.blockwise import ops
    plan = ops.gemm_plan(M, N, K, cuda_device)
    r0 = plan["split_row0"]
    assert 0 < r0 < M and r0 % 128 == 0 and plan["splits"] > 1 and plan["launches"] == 3, plan
    assert plan["workspace_bytes"] == ops.gemm_workspace_bytes(M, N, K, cuda_device) > 0
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=M + N)
    d = ops.gemm(aq, asc, wq, wsc, b)
    d1 = ops.gemm(aq, asc, wq, wsc, b, split_k=False)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([np.arange(0, M, max(1, M // 40)), [r0 - 1, r0, r0 + 1, M - 1]]))
    ri = torch.from_numpy(rows).to(cuda_device)
    ref = O.gemm_dequant_f32(bits(aq[ri]), scales_mn(asc, M)[:, rows], bits(wq), wsc.cpu().numpy(), b.cpu().numpy())
    m = O.error_metrics(O.bf16_to_f32(bits(d[ri])), ref, abs_tol=ABS_TOL)
    assert m["rel_fro"] <= REL_FRO and m["bound_excess"] <= 0, m
    m1 = O.error_metrics(O.bf16_to_f32(bits(d)), O.bf16_to_f32(bits(d1)), abs_tol=ABS_TOL)
    assert m1["bound_excess"] <= 0, m1
    assert torch.equal(d[:r0], d1[:r0])  # the unsplit rows run the same kernel over the same K order
    assert torch.equal(d, ops.gemm(aq, asc, wq, wsc, b))
    # fused GELU + requant through the split rows' reduction
    _, q, s = ops.gemm(aq, asc, wq, wsc, b, gelu=True, requant=True, write_d=True)
    dg = ops.gemm(aq, asc, wq, wsc, b, gelu=True)
    torch.cuda.synchronize()
    oq, os_ = O.quant_act_1x128(bits(dg[ri]))
    assert O.codes_equal(bits(q[ri]), oq).all()
    assert O.scales_equal(scales_mn(s, M)[:, rows], os_[:, : len(rows)]).all()
    # runtime LoRA: the split rows read their own LoRA rows
    la, lb = make_lora(N, K, 32, seed=M)
    ax = ops.lora_a(x.to(cuda_device), la.to(cuda_device))
    dl = ops.gemm(aq, asc, wq, wsc, b, lora_ax=ax, lora_b=lb.to(cuda_device), lora_alpha=0.5)
    dl1 = ops.gemm(aq, asc, wq, wsc, b, lora_ax=ax, lora_b=lb.to(cuda_device), lora_alpha=0.5, split_k=False)
    torch.cuda.synchronize()
    assert torch.equal(dl[:r0], dl1[:r0])
    diff = (dl.float() - dl1.float()).abs().max().item()
    assert diff <= 0.02 * dl1.float().abs().max().item()


@pytest.mark.parametrize("M,N,K", [(6000, 2304, 16384), (8000, 6144, 8192)])
def test_long_k_ragged_shapes(cuda_device, M, N, K):
    """Long K (8192, 16384) with ragged M and an odd number of 256-column tiles (2304 =
    9 x 256), several M groups of the rasterisation: bias and the fused GELU + requant
    against the oracle on a sample of rows, and deterministic."""
    from ltx_kernels.blockwise import ops
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=N + K)
    d = ops.gemm(aq, asc, wq, wsc, b, split_k=False)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([np.arange(0, M, max(1, M // 48)), [M - 129, M - 128, M - 1]]))
    ri = torch.from_numpy(rows).to(cuda_device)
    ref = O.gemm_dequant_f32(bits(aq[ri]), scales_mn(asc, M)[:, rows], bits(wq), wsc.cpu().numpy(), b.cpu().numpy())
    _check(d[ri], ref)
    assert torch.equal(d, ops.gemm(aq, asc, wq, wsc, b, split_k=False))
    _, q, s = ops.gemm(aq, asc, wq, wsc, b, gelu=True, requant=True, write_d=True, split_k=False)
    dg = ops.gemm(aq, asc, wq, wsc, b, gelu=True, split_k=False)
    torch.cuda.synchronize()
    oq, os_ = O.quant_act_1x128(bits(dg[ri]))
    assert O.codes_equal(bits(q[ri]), oq).all()
    assert O.scales_equal(scales_mn(s, M)[:, rows], os_[:, : len(rows)]).all()


# --------------------------------------------------------------------------- staged epilogue
@pytest.mark.parametrize("M,N,K", [(37, 384, 512), (130, 640, 256), (1, 128, 128), (300, 1152, 1024)])
@pytest.mark.parametrize("gelu,requant,write_d", [(False, False, True), (True, False, True), (False, True, True),
                                                  (False, True, False), (True, True, True), (True, True, False)])
def test_staged_epilogue_combinations(cuda_device, M, N, K, gelu, requant, write_d):
    """Every epilogue combination through the staging tile and the TMA stores, at ragged
    M (rows beyond M inside a tile) and N with an empty 128-column half tile: values
    against the oracle, codes bit-exact against quantising the bf16 result, and no row
    beyond M written (the output is a view into a larger buffer holding a sentinel)."""
    from ltx_kernels.blockwise import ops
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=M * 7 + N)
    ref = _oracle(aq, asc, wq, wsc, b)
    if gelu:
        ref = O.bf16_to_f32(O.gelu_tanh_bf16(O.f32_to_bf16(ref)))
    pad = 130
    big = torch.full((M + pad, N), -7.25, dtype=torch.bfloat16, device=cuda_device)
    res = ops.gemm(aq, asc, wq, wsc, b, out=big[:M], gelu=gelu, requant=requant, write_d=write_d, split_k=False)
    torch.cuda.synchronize()
    assert (big[M:] == -7.25).all()
    if requant:
        d, q, s = res
        # the bf16 values the codes quantise: this call's D, or the same GEMM with D written
        dd = d if write_d else ops.gemm(aq, asc, wq, wsc, b, gelu=gelu, split_k=False)
        oq, os_ = O.quant_act_1x128(bits(dd))
        assert O.codes_equal(bits(q), oq).all()
        assert O.scales_equal(scales_mn(s, M), os_[:, :M]).all()
        if not write_d:
            assert d is None and (big == -7.25).all()
            return
    else:
        d = res
    _check(d, ref)


def test_gemm_rejects_bad_out(cuda_device):
    from ltx_kernels.blockwise import ops
    M, N, K = 64, 256, 256
    x, aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed=77)
    for bad in (torch.empty(M, N - 128, dtype=torch.bfloat16, device=cuda_device),
                torch.empty(M, N, dtype=torch.float32, device=cuda_device),
                torch.empty(N, M, dtype=torch.bfloat16, device=cuda_device).t(),
                torch.empty(M, N, dtype=torch.bfloat16)):
        with pytest.raises(RuntimeError):
            ops.gemm(aq, asc, wq, wsc, b, out=bad)


def test_gemm_empty_token_batch(cuda_device):
    """No tokens: empty results with the right shapes and nothing launched (the C ABI
    takes M >= 1), through ops.gemm and the layer modules."""
    from ltx_kernels.blockwise import BlockwiseFP8FeedForward, BlockwiseFP8Linear, ops
    K, N = 256, 384
    x = torch.empty((0, K), dtype=torch.bfloat16, device=cuda_device)
    aq, asc = ops.quantize_1x128(x)
    wq, wsc = ops.quantize_weight_128x128(weights(N, K, seed=5).to(cuda_device))
    b = make_bias(N).to(cuda_device)
    d = ops.gemm(aq, asc, wq, wsc, b)
    assert tuple(d.shape) == (0, N) and d.dtype == torch.bfloat16
    d2, q, s = ops.gemm(aq, asc, wq, wsc, b, gelu=True, requant=True, write_d=True)
    assert tuple(d2.shape) == (0, N) and tuple(q.shape) == (0, N) and tuple(s.shape) == (0, N // 128)
    lin = BlockwiseFP8Linear(K, N, device=cuda_device)
    lin.weight.data, lin.weight_scale.data, lin.bias.data = wq, wsc, b
    assert tuple(lin(x.view(1, 0, K)).shape) == (1, 0, N)
    down = BlockwiseFP8Linear(N, K, device=cuda_device)
    down.weight.data, down.weight_scale.data = ops.quantize_weight_128x128(weights(K, N, seed=6).to(cuda_device))
    ff = BlockwiseFP8FeedForward.from_linears(lin, down)
    assert tuple(ff(x).shape) == (0, K)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
