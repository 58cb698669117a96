"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference's own pure-torch functions from Lightricks/LTX-2's
``ltx-kernels`` package on seeded inputs and stores inputs and outputs as
compressed ``.npz`` files next to this script:

* ``blockwise_quantize_torch``   (ltx-kernels/src/ltx_kernels/blockwise/functional.py:138-144)
* ``blockwise_quantize_weights`` (functional.py:128-135)
* the reference's CPU GEMM path: dequantise both operands, fp32 ``torch.matmul``,
  add the fp32 bias, cast to bf16 (functional.py:138-144 + the SM89 contract of
  csrc/blockwise/kernels/geforce/gemm.cu:203-253)
* ``torch.nn.functional.gelu(approximate="tanh")`` on bf16 (ltx-core/.../gelu_approx.py:10)

The reference package imports two compiled extensions (``ops_cpp``, ``all2all_cpp``)
at module load; they are replaced by empty stub modules because none of the
functions above touches them.

Usage (needs the reference checkout, so it runs in the build container only):
    python tests/golden/make_golden.py /path/to/LTX-2
The fixtures are committed; the tests never read the reference at run time.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(ref_root: str):
    for name, attrs in (("ops_cpp", ("fp6_pack", "fp6_unpack", "rms_norm_rope", "rms_norm_split_rope")),
                        ("all2all_cpp", ("All2All",))):
        mod = types.ModuleType(name)
        for a in attrs:
            setattr(mod, a, None)
        sys.modules[name] = mod
    sys.path.insert(0, os.path.join(ref_root, "packages", "ltx-kernels", "src"))
    from ltx_kernels.blockwise import functional  # noqa: PLC0415
    return functional


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float8_e4m3fn:
        return t.contiguous().view(torch.uint8).numpy().copy()
    return t.contiguous().numpy().copy()


def synth_activations(M: int, K: int, seed: int) -> torch.Tensor:
    """bf16 ~N(0,1), a seeded 1% of channels scaled x20 (the BASELINE.json recipe)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g, dtype=torch.float32)
    n_out = max(1, K // 100)
    ch = torch.randperm(K, generator=g)[:n_out]
    x[:, ch] *= 20.0
    return x.to(torch.bfloat16)


def edge_activations(K: int) -> torch.Tensor:
    """Rows exercising the quantiser's edge cases."""
    g = torch.Generator().manual_seed(7)
    x = torch.randn(10, K, generator=g, dtype=torch.float32)
    x[0] = 0.0                                   # all-zero groups -> NaN codes, scale 0
    x[1, 5] = float("inf")                       # +inf in group 0 -> scale 0 ... NaN codes
    x[2, 130] = float("-inf")                    # -inf in group 1
    x[3] = torch.randn(K, generator=g) * 1e-30   # tiny values (bf16 normals near 1e-30)
    x[4] = torch.randn(K, generator=g) * 1e30    # huge values
    x[5] = torch.tensor([(-1.0) ** i * 2.0 ** ((i % 17) - 8) for i in range(K)])  # exact powers of two
    x[6, 3] = float("nan")                       # NaN propagates through the abs-max
    x[7, :128] = -0.0                            # negative zeros
    x[8, :] = 448.0                              # saturating-scale boundary: s == 1
    x[9, ::2] = 1.0
    x[9, 1::2] = 3.0                             # constant group magnitudes
    return x.to(torch.bfloat16)


def main(ref_root: str) -> None:
    functional = _import_reference(ref_root)
    torch.manual_seed(0)

    # --- activation quantisation --------------------------------------------------
    acts = {
        "act_ragged": synth_activations(37, 512, seed=0),
        "act_4096": synth_activations(96, 4096, seed=1),
        "act_edge": edge_activations(256),
    }
    out = {}
    for name, x in acts.items():
        M, K = x.shape
        q, s = functional.blockwise_quantize_torch(x.view(1, M, K))
        out[f"{name}_x"] = _bits(x)
        out[f"{name}_q"] = _bits(q.view(M, K))
        out[f"{name}_s"] = _bits(s)          # [K/128, M] contiguous (transpose of the MN-major view)
    np.savez_compressed(os.path.join(HERE, "act_quant.npz"), **out)

    # --- weight quantisation --------------------------------------------------------
    g = torch.Generator().manual_seed(3)
    w32 = torch.randn(256, 384, generator=g) * 0.02
    w32[0:128, 128:256] = 0.0                    # an all-zero block -> NaN codes, scale 0
    wbf = (torch.randn(384, 256, generator=g) * 0.02).to(torch.bfloat16)
    out = {}
    for name, w in (("w_f32", w32), ("w_bf16", wbf)):
        q, s = functional.blockwise_quantize_weights(w)
        out[f"{name}_w"] = _bits(w)
        out[f"{name}_q"] = _bits(q)
        out[f"{name}_s"] = _bits(s)
    np.savez_compressed(os.path.join(HERE, "weight_quant.npz"), **out)

    # --- the reference's CPU GEMM path ------------------------------------------------
    M, K, N = 80, 512, 384
    x = synth_activations(M, K, seed=5)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16).float()
    aq, asc = functional.blockwise_quantize_torch(x.view(1, M, K))
    wq, wsc = functional.blockwise_quantize_weights(w)
    a_deq = aq.view(M, K).float() * asc.t().repeat_interleave(128, dim=1)
    w_deq = wq.float() * wsc.repeat_interleave(128, dim=0).repeat_interleave(128, dim=1)
    d32 = torch.matmul(a_deq, w_deq.t()) + bias
    np.savez_compressed(os.path.join(HERE, "gemm_ref.npz"),
                        x=_bits(x), w=_bits(w), bias=_bits(bias), aq=_bits(aq.view(M, K)), asc=_bits(asc),
                        wq=_bits(wq), wsc=_bits(wsc), d_f32=_bits(d32), d_bf16=_bits(d32.to(torch.bfloat16)))

    # --- GELU-tanh on bf16 (torch CPU) ------------------------------------------------------
    xs = torch.linspace(-8, 8, 4001).to(torch.bfloat16)
    xs = torch.cat([xs, (torch.randn(4000, generator=g) * 3).to(torch.bfloat16)])
    y = torch.nn.functional.gelu(xs, approximate="tanh")
    np.savez_compressed(os.path.join(HERE, "gelu_ref.npz"), x=_bits(xs), y=_bits(y))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LTX2_REFERENCE_ROOT", ""))
