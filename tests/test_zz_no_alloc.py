"""ltxfp8_gemm_static_scratch (no device allocation) against ltxfp8_gemm and the oracle.

Some hosts of this GEMM cannot hand it device memory per call: their device
memory is owned by an arena or a framework allocator they do not control, or
the GEMM runs from a plugin's enqueue/execute hook where allocating is not
allowed.  For them the entry point takes its split-K scratch from a fixed array
in the library's device globals instead of a caller workspace.

Calls through the C ABI on shapes that need split-K scratch must give exactly
the D of ltxfp8_gemm with a caller workspace (same plan, same kernels, same
fixed-order reduction, so bit-identical), on consecutive calls that reuse the
array with stale partials from the previous call, including a shape whose plan
splits only its last M-tile rows (three launches, partials of rows from
split_row0 upward).  One case per shape is also checked against the oracle's
dequantise-then-fp32-matmul result with the GEMM parity bar.  This file is
collected last so it runs both after the other GPU tests and alone.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from inputs import activations, bias as make_bias, bits, scales_mn, weights
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_FRO = 1e-2
ABS_TOL = 2e-2  # plus one bf16 ulp of |ref|, element by element


def _problem(M, N, K, dev, seed):
    from ltx_kernels.blockwise import ops
    aq, asc = ops.quantize_1x128(activations(M, K, seed=seed).to(dev))
    wq, wsc = ops.quantize_weight_128x128(weights(N, K, seed=seed + 1).to(dev))
    b = make_bias(N, seed=seed + 2).to(dev)
    return aq, asc, wq, wsc, b


def _static_scratch_gemm(aq, asc, wq, wsc, b, gelu):
    from ltx_kernels import _lib as L
    from ltx_kernels.blockwise import ops
    M, K = aq.shape
    N = wq.shape[0]
    d = torch.empty((M, N), dtype=torch.bfloat16, device=aq.device)
    ep = L.Epilogue()
    ep.gelu_tanh = 1 if gelu else 0
    rc = L.load().ltxfp8_gemm_static_scratch(aq.data_ptr(), asc.data_ptr(), ops.scale_layout(asc, M, K // 128),
                                             wq.data_ptr(), wsc.data_ptr(), b.data_ptr(), d.data_ptr(), M, N, K,
                                             ctypes.byref(ep), torch.cuda.current_stream().cuda_stream)
    L.check(rc)
    return d


def _oracle_rows(aq, asc, wq, wsc, b, gelu, rows):
    M = aq.shape[0]
    ri = torch.from_numpy(rows).to(aq.device)
    ref = O.gemm_dequant_f32(bits(aq[ri]), scales_mn(asc, M)[:, rows], bits(wq), wsc.cpu().numpy(),
                             b.cpu().numpy())
    if gelu:
        ref = O.bf16_to_f32(O.gelu_tanh_bf16(O.f32_to_bf16(ref)))
    return ref


def test_static_scratch_matches_workspace_gemm(cuda_device):
    from ltx_kernels.blockwise import ops
    cases = [
        # (M, N, K, gelu, seed)
        (128, 4096, 4096, False, 11),   # skinny: every tile split (2 launches)
        (200, 1024, 2048, True, 23),    # ragged M, GELU in the reduction
        (1280, 4096, 8192, False, 31),  # tail split: rows >= split_row0 split (3 launches)
        (128, 4096, 4096, False, 37),   # first shape again, new data, stale partials in the array
    ]
    for M, N, K, gelu, seed in cases:
        plan = ops.gemm_plan(M, N, K, cuda_device)
        assert plan["workspace_bytes"] > 0, plan
        if M == 1280:
            assert plan["split_row0"] > 0 and plan["launches"] == 3, plan
        aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed)
        ref = ops.gemm(aq, asc, wq, wsc, b, gelu=gelu)           # ltxfp8_gemm, caller workspace
        out = _static_scratch_gemm(aq, asc, wq, wsc, b, gelu)    # ltxfp8_gemm_static_scratch
        again = _static_scratch_gemm(aq, asc, wq, wsc, b, gelu)  # second call in a row, same array
        torch.cuda.synchronize()
        assert torch.equal(out, ref), (M, N, K)
        assert torch.equal(again, ref), (M, N, K)
        r0 = plan["split_row0"]
        rows = np.unique(np.array([0, 1, M // 2, max(r0 - 1, 0), min(r0, M - 1), M - 1]))
        m = O.error_metrics(O.bf16_to_f32(bits(out[torch.from_numpy(rows).to(cuda_device)])),
                            _oracle_rows(aq, asc, wq, wsc, b, gelu, rows), abs_tol=ABS_TOL)
        assert m["rel_fro"] <= REL_FRO and m["bound_excess"] <= 0, (M, N, K, m)
