"""The reference's own code calling into this repository (CPU; needs the reference checkout).

Two clean interpreters, as a user would set them up:

* Option A -- ``ltx-2_b200/dropin`` first on ``sys.path``, then the reference's
  ``ltx-kernels/src`` and ``ltx-core/src``: the reference's ``ltx_kernels.blockwise.linear``
  and ``ltx_core.quantization.blockwise._impl`` import unchanged, and their
  ``from blockwise_cpp import fp8_gemm_nt_sm89`` (``linear.py:30``) resolves to this
  repository's module, while ``ltx_kernels`` stays the reference's package.
* Option B -- ``ltx-2_b200`` first on ``sys.path`` (``ltx_kernels`` is this repository's),
  then ``ltx-core/src``: ``_impl.py:12-24`` imports every name it needs from this package.

In both, the torch ops the reference code calls (``blockwise::*``, ``q8_kernels_ops::*``)
are probed: schema strings and fake (meta) outputs must be identical to what the
reference's own registrations give.  The compiled extensions the reference imports at
module load (``ops_cpp``, ``all2all_cpp``) are empty stubs, as in
``tests/golden/make_golden.py``; no kernel runs.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("LTX2_REFERENCE", "/root/reference")
REF_PKGS = os.path.join(REF, "packages")

pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF_PKGS, "ltx-core", "src")),
                                reason="reference checkout not present")

_PROBE = r'''
import json, sys, types
for name, attrs in (("ops_cpp", ("fp6_pack", "fp6_unpack", "rms_norm_rope", "rms_norm_split_rope")),
                    ("all2all_cpp", ("All2All",))):
    if name not in sys.modules:
        m = types.ModuleType(name)
        for a in attrs:
            setattr(m, a, None)
        sys.modules[name] = m
import torch
from ltx_core.quantization.blockwise import _impl
import ltx_kernels.blockwise.linear as L
import ltx_kernels.blockwise.functional as F
out = {"linear_file": L.__file__, "functional_file": F.__file__,
       "impl_fp8_linear": _impl.BlockwiseFP8Linear.__module__, "schemas": {}, "fake": {}}
try:
    import blockwise_cpp
    out["blockwise_cpp_file"] = blockwise_cpp.__file__
except ImportError as e:
    out["blockwise_cpp_file"] = "ImportError: " + str(e)
ops = ["blockwise::fp8_gemm", "blockwise::quantize", "blockwise::dequantize", "blockwise::adanorm",
       "blockwise::quant_rms_fma", "blockwise::rms_fma", "blockwise::gated_attention",
       "q8_kernels_ops::rms_norm_rope", "q8_kernels_ops::rms_norm_split_rope", "q8_kernels_ops::fp6_pack",
       "q8_kernels_ops::fp6_unpack"]
for op in ops:
    ns, name = op.split("::")
    out["schemas"][op] = str(getattr(getattr(torch.ops, ns), name).default._schema)

def desc(t):
    if t is None:
        return None
    if isinstance(t, (tuple, list)):
        return [desc(u) for u in t]
    return [list(t.shape), list(t.stride()), str(t.dtype)]

from torch._subclasses.fake_tensor import FakeTensorMode
E = lambda *s, dt=torch.bfloat16: torch.empty(*s, dtype=dt, device="meta")
with FakeTensorMode():
    B, S, H, NH = 2, 150, 512, 4
    a8, sfa = E(300, 512, dt=torch.float8_e4m3fn), E(4, 300, dt=torch.float32).t()
    w8, sfb = E(256, 512, dt=torch.float8_e4m3fn), E(2, 4, dt=torch.float32)
    x, y = E(B, S, H), E(B, S, H)
    cases = {
        "fp8_gemm": lambda: torch.ops.blockwise.fp8_gemm([a8, sfa], [w8, sfb], None, False),
        "fp8_gemm_bias": lambda: torch.ops.blockwise.fp8_gemm([a8, sfa], [w8, sfb], E(256, dt=torch.float32), False),
        "quantize": lambda: torch.ops.blockwise.quantize(x, False),
        "quantize_gelu": lambda: torch.ops.blockwise.quantize(x, True),
        "dequantize": lambda: torch.ops.blockwise.dequantize(E(B, S, H, dt=torch.float8_e4m3fn),
                                                             E(4, 300, dt=torch.float32).t()),
        "adanorm": lambda: torch.ops.blockwise.adanorm(x, None, E(B, 1, H), E(B, 1, H), torch.float8_e4m3fn, None),
        "quant_rms_fma": lambda: torch.ops.blockwise.quant_rms_fma(x, y, E(B, 1, H)),
        "rms_fma": lambda: torch.ops.blockwise.rms_fma(x, y, E(B, 1, H)),
        "gated_attention_q": lambda: torch.ops.blockwise.gated_attention(x, E(B, S, NH), True),
        "gated_attention_bf16": lambda: torch.ops.blockwise.gated_attention(x, E(B, S, NH), False),
        "rms_norm_rope": lambda: torch.ops.q8_kernels_ops.rms_norm_rope(x, None, E(B, S, H), E(B, S, H), True),
        "rms_norm_rope_fp8": lambda: torch.ops.q8_kernels_ops.rms_norm_rope(x, E(H), E(B, S, H), E(B, S, H), False),
        "rms_norm_split_rope": lambda: torch.ops.q8_kernels_ops.rms_norm_split_rope(
            x, E(B, NH, S, H // NH // 2), E(B, NH, S, H // NH // 2), E(H), False),
        "fp6_pack": lambda: torch.ops.q8_kernels_ops.fp6_pack(E(256, 512, dt=torch.uint8)),
        "fp6_unpack": lambda: torch.ops.q8_kernels_ops.fp6_unpack(E(256, 384, dt=torch.uint8), 512),
    }
    for k, f in cases.items():
        try:
            out["fake"][k] = desc(f())
        except Exception as e:  # a missing fake is reported, not hidden
            out["fake"][k] = "error: " + type(e).__name__ + ": " + str(e)[:200]
print("PROBE" + json.dumps(out))
'''


def _run(paths):
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join(paths)
    env["CUDA_VISIBLE_DEVICES"] = ""
    r = subprocess.run([sys.executable, "-c", _PROBE], env=env, capture_output=True, text=True, timeout=600,
                       cwd="/")
    assert r.returncode == 0, r.stderr[-3000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("PROBE")][-1]
    return json.loads(line[len("PROBE"):])


@pytest.fixture(scope="module")
def reference_alone():
    """The reference's own registrations (no repository code on the path)."""
    return _run([os.path.join(REF_PKGS, "ltx-kernels", "src"), os.path.join(REF_PKGS, "ltx-core", "src")])


def test_option_a_reference_code_on_our_gemm_module(reference_alone):
    got = _run([os.path.join(REPO, "ltx-2_b200", "dropin"), os.path.join(REF_PKGS, "ltx-kernels", "src"),
                os.path.join(REF_PKGS, "ltx-core", "src")])
    assert got["linear_file"].startswith(REF_PKGS)                    # the reference's linear.py ...
    assert got["blockwise_cpp_file"].startswith(os.path.join(REPO, "ltx-2_b200", "dropin"))  # ... on our GEMM
    assert got["impl_fp8_linear"] == "ltx_kernels.blockwise.linear"
    assert got["schemas"] == reference_alone["schemas"]
    assert got["fake"] == reference_alone["fake"]


def test_option_b_ltx_core_on_our_package(reference_alone):
    got = _run([os.path.join(REPO, "ltx-2_b200"), os.path.join(REF_PKGS, "ltx-core", "src")])
    assert got["linear_file"].startswith(os.path.join(REPO, "ltx-2_b200"))
    assert got["functional_file"].startswith(os.path.join(REPO, "ltx-2_b200"))
    assert got["schemas"] == reference_alone["schemas"]
    for k, v in reference_alone["fake"].items():
        assert not str(v).startswith("error"), (k, v)
        assert got["fake"][k] == v, (k, got["fake"][k], v)
