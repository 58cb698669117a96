"""Token streaming from host memory (ltx_kernels.blockwise.host_stream): chunked,
copy-overlapped calls give the whole-batch result row for row."""
from __future__ import annotations

import pytest
import torch

from inputs import activations, bias as make_bias, lora as make_lora, weights

pytestmark = pytest.mark.gpu


def _linear(K, N, dev, seed, lora_rank=0):
    from ltx_kernels.blockwise import BlockwiseFP8Linear, BlockwiseFP8LoRALinear
    from ltx_kernels.blockwise import ops
    if lora_rank:
        m = BlockwiseFP8LoRALinear(K, N, lora_rank, alpha=0.5, device=dev)
        la, lb = make_lora(N, K, lora_rank, seed=seed + 7)
        m.lora_A.data, m.lora_B.data = la.to(dev), lb.to(dev)
    else:
        m = BlockwiseFP8Linear(K, N, device=dev)
    wq, ws = ops.quantize_weight_128x128(weights(N, K, seed=seed).to(dev))
    m.weight.data, m.weight_scale.data = wq, ws
    m.bias.data = make_bias(N, seed=seed + 1).to(dev)
    return m


@pytest.mark.parametrize("rows,chunk,pinned", [(3000, 1024, True), (1000, 4096, True), (777, 256, False)])
def test_ffn_streamed_equals_whole_batch(cuda_device, rows, chunk, pinned):
    from ltx_kernels.blockwise import BlockwiseFP8FeedForward, TokenStreamer, ops
    D, H = 512, 1024
    ff = BlockwiseFP8FeedForward.from_linears(_linear(D, H, cuda_device, 1), _linear(H, D, cuda_device, 2))
    x = activations(rows, D, seed=rows)
    st = TokenStreamer(ff, D, chunk, cuda_device)
    b = st.bounds(rows)
    sizes = [b[i + 1] - b[i] for i in range(len(b) - 1)]
    assert b[0] == 0 and b[-1] == rows and min(sizes) > 0 and max(sizes) <= chunk
    # the GEMM plans at the chunk and batch row counts agree here: results are bit-identical
    for m in set(sizes) | {rows}:
        assert ops.gemm_plan(m, H, D, cuda_device)["splits"] == 1
        assert ops.gemm_plan(m, D, H, cuda_device)["splits"] == 1
    with torch.inference_mode():
        ref = ff(x.to(cuda_device)[None])[0].cpu()
        xh = x.pin_memory() if pinned else x.clone()
        out = torch.empty(rows, D, dtype=torch.bfloat16)
        out = out.pin_memory() if pinned else out
        for _ in range(2):  # reused slots and events across calls
            out.fill_(0)
            st(xh, out)
            torch.cuda.current_stream().synchronize()
            assert torch.equal(out, ref)


def test_lora_linear_streamed(cuda_device):
    from ltx_kernels.blockwise import stream_tokens
    K, N, rows = 1024, 768, 1500
    lin = _linear(K, N, cuda_device, 5, lora_rank=32)
    x = activations(rows, K, seed=9)
    with torch.inference_mode():
        ref = lin(x.to(cuda_device)[None])[0].cpu()
        out = stream_tokens(lin, x.pin_memory(), torch.empty(rows, N, dtype=torch.bfloat16).pin_memory(),
                            chunk_tokens=512)
        torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_stream_ordering_against_caller_stream(cuda_device):
    """Work queued on the caller's stream before the call is visible to the layer, and
    events recorded after the call cover the last copy."""
    from ltx_kernels.blockwise import stream_tokens
    K, N, rows = 512, 512, 2048
    lin = _linear(K, N, cuda_device, 11)
    x = activations(rows, K, seed=3)
    xh = x.pin_memory()
    out = torch.empty(rows, N, dtype=torch.bfloat16).pin_memory()
    with torch.inference_mode():
        ref = lin(x.to(cuda_device)[None])[0].cpu()
        e1 = torch.cuda.Event()
        torch.cuda._sleep(2_000_000)  # caller-stream work ahead of the call
        stream_tokens(lin, xh, out, chunk_tokens=512)
        e1.record()
        e1.synchronize()
    assert torch.equal(out, ref)


def test_stream_rejects_bad_buffers(cuda_device):
    from ltx_kernels.blockwise import TokenStreamer
    st = TokenStreamer(lambda t: t, 256, 128, cuda_device)
    with pytest.raises(RuntimeError):
        st(torch.zeros(10, 256, dtype=torch.bfloat16, device=cuda_device), torch.zeros(10, 256, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError):
        st(torch.zeros(10, 128, dtype=torch.bfloat16), torch.zeros(10, 256, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError):
        st(torch.zeros(10, 256, dtype=torch.bfloat16), torch.zeros(9, 256, dtype=torch.bfloat16))


def test_stream_with_split_k_chunks(cuda_device):
    """Chunks small enough to take split-K with another split count than the whole batch:
    rows agree with the whole-batch result to fp32 summation order."""
    from ltx_kernels.blockwise import TokenStreamer, ops
    K, N, rows, chunk = 4096, 1024, 640, 128
    lin = _linear(K, N, cuda_device, 21)
    assert ops.gemm_plan(chunk, N, K, cuda_device)["splits"] != ops.gemm_plan(rows, N, K, cuda_device)["splits"]
    x = activations(rows, K, seed=21)
    with torch.inference_mode():
        ref = lin(x.to(cuda_device)[None])[0].float().cpu()
        out = torch.empty(rows, N, dtype=torch.bfloat16).pin_memory()
        TokenStreamer(lin, K, chunk, cuda_device)(x.pin_memory(), out)
        torch.cuda.synchronize()
    diff = (out.float() - ref).abs().max().item()
    assert diff <= 0.02 * ref.abs().max().item()


@pytest.mark.parametrize("rows", [300, 2048])
def test_ffn_module_paths_agree(cuda_device, rows):
    """BlockwiseFP8FeedForward: the default path (up projection to bf16, then one GELU +
    requant pass) and the fused-epilogue path give identical outputs, in both
    arithmetics; and both equal the reference's unfused chain written with torch's GELU."""
    import torch.nn.functional as Fn
    from ltx_kernels import _lib as L
    from ltx_kernels.blockwise import BlockwiseFP8FeedForward, ops
    import ltx_kernels.blockwise.functional as F
    D, H = 512, 2048
    up, down = _linear(D, H, cuda_device, 11), _linear(H, D, cuda_device, 12)
    ff = BlockwiseFP8FeedForward.from_linears(up, down)
    x = activations(rows, D, seed=rows + 5).to(cuda_device)
    before = F.get_quant_mode()
    try:
        for mode in ("triton", "torch"):
            F.set_quant_mode(mode)
            ff.fused_epilogue = False
            y_split = ff(x)
            ff.fused_epilogue = True
            y_fused = ff(x)
            code = L.QUANT_TRITON if mode == "triton" else L.QUANT_TORCH
            q, s = ops.quantize_1x128(x, code)
            h = Fn.gelu(ops.gemm(q, s, up.weight, up.weight_scale, up.bias), approximate="tanh")
            hq, hs = ops.quantize_1x128(h, code)
            y_chain = ops.gemm(hq, hs, down.weight, down.weight_scale, down.bias)
            torch.cuda.synchronize()
            assert torch.equal(y_split, y_fused), mode
            assert torch.equal(y_split.reshape(rows, D), y_chain), mode
    finally:
        F.set_quant_mode(before)
