"""The C-ABI library without a GPU: it loads, exports every symbol include/ltxfp8.h
declares, and rejects invalid arguments before touching a device."""
from __future__ import annotations

import ctypes
import os
import re

import pytest
import torch

from conftest import REPO


def _declared_symbols():
    src = open(os.path.join(REPO, "include", "ltxfp8.h")).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(ltxfp8_\w+)\s*\(", src, re.M)))


def test_header_declares_the_boundary():
    syms = _declared_symbols()
    for s in ("ltxfp8_quantize_1x128", "ltxfp8_gemm", "ltxfp8_lora_a", "ltxfp8_dequantize_1x128",
              "ltxfp8_quantize_weight_128x128", "ltxfp8_device_status"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    from ltx_kernels import _lib
    L = _lib.load()
    for s in _declared_symbols():
        assert hasattr(L, s), s
        assert s in _lib.SIGNATURES, s
    assert L.ltxfp8_version() >> 16 == 1


@pytest.mark.parametrize("M,N,K", [(0, 256, 256), (64, 100, 256), (64, 256, 200), (64, 256, 0)])
def test_gemm_rejects_bad_shapes_without_device(M, N, K):
    from ltx_kernels import _lib
    L = _lib.load()
    rc = L.ltxfp8_gemm(16, 16, max(M, 1), 16, 16, None, 16, M, N, K, None, None)
    assert rc == _lib.ERR_UNSUPPORTED_SHAPE
    assert "gemm" in L.ltxfp8_last_error().decode()


def test_gemm_rejects_misaligned_operands_without_device():
    from ltx_kernels import _lib
    L = _lib.load()
    rc = L.ltxfp8_gemm(17, 16, 128, 16, 16, None, 16, 128, 256, 256, None, None)
    assert rc == _lib.ERR_MISALIGNED
    rc = L.ltxfp8_gemm(16, 16, 64, 16, 16, None, 16, 128, 256, 256, None, None)  # sfa_ld < M
    assert rc == _lib.ERR_INVALID_ARGUMENT


def test_gemm_rejects_bad_lora_rank_without_device():
    from ltx_kernels import _lib
    L = _lib.load()
    ep = _lib.Epilogue()
    ep.lora_ax = 16
    ep.lora_b = 16
    ep.lora_r = 24
    rc = L.ltxfp8_gemm(16, 16, 128, 16, 16, None, 16, 128, 256, 256, ctypes.byref(ep), None)
    assert rc == _lib.ERR_UNSUPPORTED_SHAPE


def test_quantize_rejects_bad_arguments_without_device():
    from ltx_kernels import _lib
    L = _lib.load()
    assert L.ltxfp8_quantize_1x128(16, 4, 100, 100, 16, 100, 16, 4, 0, None) == _lib.ERR_UNSUPPORTED_SHAPE
    assert L.ltxfp8_quantize_1x128(16, 4, 128, 128, 16, 128, 16, 4, 7, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.ltxfp8_quantize_1x128(16, 0, 128, 128, 16, 128, 16, 0, 0, None) == _lib.OK  # M == 0: no-op
    assert L.ltxfp8_lora_a(16, 16, 16, 8, 128, 8, None) == _lib.ERR_UNSUPPORTED_SHAPE


def test_ops_refuse_cpu_tensors():
    """No CPU fallback exists: the product path raises on host tensors."""
    from ltx_kernels.blockwise import ops
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.quantize_1x128(torch.zeros(4, 128, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.quantize_weight_128x128(torch.zeros(128, 128))


def test_custom_op_names_and_schemas():
    import ltx_kernels.blockwise  # noqa: F401  (registers the ops)
    assert "Tensor[] a, Tensor[] b, Tensor? bias, bool use_fast_accum" in str(torch.ops.blockwise.fp8_gemm.default._schema)
    assert "Tensor x, bool use_gelu" in str(torch.ops.blockwise.quantize.default._schema)
    assert "Tensor x, Tensor scales" in str(torch.ops.blockwise.dequantize.default._schema)


def test_fake_tensor_shapes():
    """The ops' fake (meta) implementations give the reference's output shapes and scale strides."""
    import ltx_kernels.blockwise  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(2, 5, 256, dtype=torch.bfloat16)
        q, s = torch.ops.blockwise.quantize(x, False)
        assert q.shape == (2, 5, 256) and q.dtype == torch.float8_e4m3fn
        assert s.shape == (10, 2) and s.stride() == (1, 12)
        a = torch.empty(10, 256, dtype=torch.float8_e4m3fn)
        w = torch.empty(384, 256, dtype=torch.float8_e4m3fn)
        d = torch.ops.blockwise.fp8_gemm([a, s], [w, torch.empty(3, 2)], None, False)
        assert d.shape == (10, 384) and d.dtype == torch.bfloat16


def test_fp6_entry_points_reject_bad_arguments_without_device():
    """The 6-bit weight path validates before touching a device: shapes, null pointers,
    the tensor-core copy's 32-byte alignment and the GEMM's shape rules."""
    from ltx_kernels import _lib
    L = _lib.load()
    assert L.ltxfp8_fp6_to_tc(16, 16, 100, 128, 32, 16, None) == _lib.ERR_UNSUPPORTED_SHAPE
    assert L.ltxfp8_fp6_to_tc(None, 16, 128, 128, 32, 16, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.ltxfp8_fp6_to_tc(16, 16, 128, 128, 48, 16, None) == _lib.ERR_MISALIGNED
    assert "fp6_to_tc" in L.ltxfp8_last_error().decode()
    assert L.ltxfp8_gemm_fp6w(16, 16, 128, 32, 16, None, 16, 128, 100, 256, None, None) == _lib.ERR_UNSUPPORTED_SHAPE
    assert L.ltxfp8_gemm_fp6w(16, 16, 128, 48, 16, None, 16, 128, 256, 256, None, None) == _lib.ERR_MISALIGNED


def test_fp6_linear_keeps_the_reference_parameters():
    """BlockwiseFP6Linear's state dict is the reference's (linear.py:212-243): the packed
    uint8 weight [out, in*3/4], fp32 block scales and bias; the tensor-core copy of the
    weight is never a parameter or buffer, and it is kept only on request."""
    import ltx_kernels.blockwise  # noqa: F401
    from ltx_kernels.blockwise import BlockwiseFP6Linear
    layer = BlockwiseFP6Linear(1024, 512, bias=True, device="cpu")
    sd = layer.state_dict()
    assert sorted(sd) == ["bias", "weight", "weight_scale"]
    assert sd["weight"].shape == (512, 768) and sd["weight"].dtype == torch.uint8
    assert sd["weight_scale"].shape == (4, 8) and sd["weight_scale"].dtype == torch.float32
    assert sd["bias"].dtype == torch.float32
    assert layer.keep_tc_weight is False
    assert "blockwise::fp6_gemm" in str(torch.ops.blockwise.fp6_gemm.default._schema)
