"""Drop-in for the reference's compiled ``blockwise_cpp`` module
(ltx-kernels/csrc/blockwise/api.cpp:67-82), backed by the sm_100a C-ABI.

``fp8_gemm_nt_sm89(a, b, d, bias=None, use_fast_accum=True)`` writes ``d`` in
place like the pybind function it replaces, so the reference's own
``linear.py`` (``from blockwise_cpp import fp8_gemm_nt_sm89``, linear.py:30)
runs on the tcgen05 kernel without edits.  ``use_fast_accum`` is ignored:
accumulation is always fp32.

This directory (``ltx-2_b200/dropin``) holds only this module, so putting it
first on ``sys.path`` replaces the compiled GEMM and nothing else: the name
``ltx_kernels`` keeps resolving to the reference's package.  The C-ABI binding
(``ltx_kernels/_lib.py``, ``ltx_kernels/blockwise/ops.py`` of this repository) is
therefore loaded from its files under the private package name ``_ltxb200``.
"""
from __future__ import annotations

import importlib
import os
import sys
import types
from typing import Optional, Sequence

import torch

_KERNELS = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "ltx_kernels")


def _load_ops():
    if "_ltxb200.blockwise.ops" not in sys.modules:
        for name, path in (("_ltxb200", _KERNELS), ("_ltxb200.blockwise", os.path.join(_KERNELS, "blockwise"))):
            if name not in sys.modules:
                pkg = types.ModuleType(name)
                pkg.__path__ = [path]  # package without running its __init__ (which imports by the public name)
                sys.modules[name] = pkg
    return importlib.import_module("_ltxb200.blockwise.ops")


ops = _load_ops()


def fp8_gemm_nt_sm89(a: Sequence[torch.Tensor], b: Sequence[torch.Tensor], d: torch.Tensor,
                     bias: Optional[torch.Tensor] = None, use_fast_accum: bool = True) -> None:
    if d.dtype != torch.bfloat16 or not d.is_contiguous() or tuple(d.shape) != (a[0].shape[0], b[0].shape[0]):
        raise RuntimeError("d must be a contiguous bf16 [M, N] tensor")
    ops.gemm(a[0], a[1], b[0], b[1], bias, out=d)


def fp8_gemm_nt_sm100(a: Sequence[torch.Tensor], b: Sequence[torch.Tensor], d: torch.Tensor,
                      bias: Optional[torch.Tensor] = None, use_fast_accum: bool = True) -> None:
    fp8_gemm_nt_sm89(a, b, d, bias=bias, use_fast_accum=use_fast_accum)


# Hopper entry point of the same module (api.cpp:70-75); on sm_100 it is the same kernel.
def fp8_gemm_nt_sm90(a, b, d, bias=None, c=None, num_sms=132) -> None:
    if c is not None:
        raise RuntimeError("the C-accumulate operand of fp8_gemm_nt_sm90 is not supported")
    fp8_gemm_nt_sm89(a, b, d, bias=bias)
