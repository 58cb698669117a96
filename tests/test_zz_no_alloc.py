"""ltxfp8_gemm_static_scratch (no device allocation) against ltxfp8_gemm.

The entry point takes its split-K scratch from a fixed array in the library's
device globals instead of a caller workspace.  Calls through the C ABI on
skinny shapes (split-K engaged) must give the same D as ltxfp8_gemm with a
caller workspace, within the GEMM parity tolerance, on consecutive calls that
reuse the array with stale partials from the previous call.  This file is
collected last so it runs both after the other GPU tests and alone.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from inputs import activations, bias as make_bias, bits, weights
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_FRO = 1e-2
MAX_ABS_NORM = 2e-2


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


def _close(out, ref):
    m = O.error_metrics(O.bf16_to_f32(bits(out)), O.bf16_to_f32(bits(ref)))
    assert m["rel_fro"] <= REL_FRO and m["max_abs_norm"] <= MAX_ABS_NORM, m


def test_static_scratch_matches_workspace_gemm(cuda_device):
    from ltx_kernels.blockwise import ops
    cases = [
        # (M, N, K, gelu, seed): skinny outputs, so each needs split-K scratch
        (128, 4096, 4096, False, 11),
        (200, 1024, 2048, True, 23),   # ragged M, different partial layout
        (128, 4096, 4096, False, 37),  # first shape again, new data, stale partials in the array
    ]
    for M, N, K, gelu, seed in cases:
        assert ops.gemm_workspace_bytes(M, N, K, cuda_device) > 0
        aq, asc, wq, wsc, b = _problem(M, N, K, cuda_device, seed)
        ref = ops.gemm(aq, asc, wq, wsc, b, gelu=gelu)           # ltxfp8_gemm, caller workspace
        out = _static_scratch_gemm(aq, asc, wq, wsc, b, gelu)    # ltxfp8_gemm_static_scratch
        torch.cuda.synchronize()
        assert np.isfinite(O.bf16_to_f32(bits(out))).all()
        _close(out, ref)
