"""Record the reference's own GPU kernels on seeded inputs as golden fixtures (run on a B200).

The reference runs its activation quantiser and its fused producers as Triton kernels
(``ltx-kernels/src/ltx_kernels/blockwise/triton_ops.py:52-151,194-384``), its q/k
RMSNorm + RoPE as CUDA kernels of ``ops_cpp`` (``csrc/ops/rms_norm_rope_cuda.cu``,
``rms_norm_split_rope_cuda.cu``), and its FFN GELU as torch's CUDA
``F.gelu(approximate="tanh")`` (``ltx-core/.../gelu_approx.py:10``).  Their last-bit
behaviour depends on GPU instructions (approximate division and exponential, bf16
arithmetic, the order of Triton's reductions), so it is recorded here from the kernels
themselves, built from the reference's sources by ``oracle/build_ref.py`` and loaded by
``oracle/refpath.py``.  Inputs come from CPU ``torch.Generator`` seeds.

Files written (inputs and outputs as bit patterns: bf16 -> uint16, e4m3 -> uint8):
* ``ref_gpu_quant.npz``      -- ``blockwise::quantize`` (use_gelu False / True)
* ``ref_gpu_producers.npz``  -- ``blockwise::adanorm`` (broadcast and per-token modulation),
  ``quant_rms_fma``, ``rms_fma``, ``gated_attention`` (quantised and bf16), H = 4096 and 2048
* ``ref_gpu_rope.npz``       -- ``rms_norm_rope`` (with / without weights, bf16 / e4m3) and
  ``rms_norm_split_rope`` (bf16 / e4m3)
* ``torch_gpu_gelu_bf16.npz`` -- torch's CUDA GELU-tanh of every bf16 bit pattern

Usage (GPU box, with oracle/_ref built):  python tests/golden/make_ref_gpu_golden.py [OUT_DIR]
The fixtures are committed under tests/golden/; tests never run this script.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import refpath  # noqa: E402


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy().copy()
    return t.numpy().copy()


def acts(B, S, H, seed, edge=True):
    """bf16 ~N(0,1) with 1 % outlier channels x20; a few edge rows when `edge`."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, S, H, generator=g)
    x[..., torch.randperm(H, generator=g)[: max(1, H // 100)]] *= 20.0
    if edge:
        x[0, 0] = 0.0                                   # an all-zero row
        x[0, 1] *= 1e-3                                 # small values
        x[0, 2] *= 300.0                                # large values
        x[-1, -1, : H // 2] = 0.0                       # half-zero row (zero groups)
    return x.to(torch.bfloat16)


def small(shape, std, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)


def main(out_dir: str) -> None:
    os.makedirs(out_dir, exist_ok=True)
    dev = torch.device("cuda", 0)
    T = refpath.triton_ops()
    R = refpath.ops()
    meta = {"torch": torch.__version__, "gpu": torch.cuda.get_device_name(0)}
    try:
        import triton
        meta["triton"] = triton.__version__
    except ImportError:
        pass

    # ---- activation quantiser (triton_ops.py:102-151)
    q = {}
    for K, B, S, seed in ((4096, 2, 19, 1), (2048, 1, 23, 2)):
        x = acts(B, S, K, seed)
        for gelu in (False, True):
            c, s = T._quant_blockwise_tma_aligned_func(x.to(dev), gelu)
            tag = f"k{K}_{'gelu' if gelu else 'plain'}"
            q[f"{tag}_x"] = bits(x)
            q[f"{tag}_codes"] = bits(c)
            q[f"{tag}_scales"] = bits(s.t().contiguous())  # [K/128, align4(M)] as stored
    np.savez_compressed(os.path.join(out_dir, "ref_gpu_quant.npz"), **q, **{f"meta_{k}": v for k, v in meta.items()})

    # ---- producers (triton_ops.py:52-96, 194-307, 309-384)
    p = {}
    for H, B, S, heads, seed in ((4096, 2, 19, 32, 10), (2048, 2, 11, 16, 20)):
        tag = f"h{H}"
        x, y = acts(B, S, H, seed), acts(B, S, H, seed + 1, edge=False)
        sc_b, sh_b = small((B, 1, H), 0.1, seed + 2), small((B, 1, H), 0.1, seed + 3)
        sc_t, sh_t = small((B, S, H), 0.1, seed + 4), small((B, S, H), 0.1, seed + 5)
        z_b, z_t = small((B, 1, H), 0.1, seed + 6), small((B, S, H), 0.1, seed + 7)
        lg = small((B, S, heads), 3.0, seed + 8)
        for name, t in (("x", x), ("y", y), ("scale_b", sc_b), ("shift_b", sh_b), ("scale_t", sc_t),
                        ("shift_t", sh_t), ("z_b", z_b), ("z_t", z_t), ("logits", lg)):
            p[f"{tag}_{name}"] = bits(t)
        xd, yd = x.to(dev), y.to(dev)
        for mod, (sc, sh) in (("b", (sc_b, sh_b)), ("t", (sc_t, sh_t))):
            c, s = T.run_quant_blockwise_norm_tma_aligned(xd, None, sc.to(dev), sh.to(dev), torch.float8_e4m3fn, None)
            p[f"{tag}_adanorm_{mod}_codes"], p[f"{tag}_adanorm_{mod}_scales"] = bits(c), bits(s.t().contiguous())
        for zm, z in (("b", z_b), ("t", z_t)):
            xx = xd.clone()
            c, s = T.run_quant_blockwise_rms_fma(xx, yd, z.to(dev))
            p[f"{tag}_qrmsfma_{zm}_codes"], p[f"{tag}_qrmsfma_{zm}_scales"] = bits(c), bits(s.t().contiguous())
            p[f"{tag}_qrmsfma_{zm}_xout"] = bits(xx)
            xx = xd.clone()
            o = T.run_rms_fma(xx, yd, z.to(dev))
            p[f"{tag}_rmsfma_{zm}_out"], p[f"{tag}_rmsfma_{zm}_xout"] = bits(o), bits(xx)
        c, s = T.run_gated_attention(xd, lg.to(dev), True)
        p[f"{tag}_gated_codes"], p[f"{tag}_gated_scales"] = bits(c), bits(s.t().contiguous())
        o, _ = T.run_gated_attention(xd, lg.to(dev), False)
        p[f"{tag}_gated_out"] = bits(o)
    np.savez_compressed(os.path.join(out_dir, "ref_gpu_producers.npz"), **p)

    # ---- q/k RMSNorm + RoPE (ops_cpp)
    r = {}
    B, S, H, heads = 2, 13, 4096, 32
    x = acts(B, S, H, 30)
    w = (1 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(31))).to(torch.bfloat16)
    ang = torch.rand(B, S, H, generator=torch.Generator().manual_seed(32)) * 6.0
    cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    angs = torch.rand(B, heads, S, H // heads // 2, generator=torch.Generator().manual_seed(33)) * 6.0
    cs, sn = angs.cos().to(torch.bfloat16), angs.sin().to(torch.bfloat16)
    for name, t in (("x", x), ("w", w), ("cos", cos), ("sin", sin), ("split_cos", cs), ("split_sin", sn)):
        r[name] = bits(t)
    xd = x.to(dev)
    for affine in (False, True):
        for fp8 in (False, True):
            o = R.rms_norm_rope(xd, w.to(dev) if affine else None, cos.to(dev), sin.to(dev), not fp8)
            r[f"rope_w{int(affine)}_fp8{int(fp8)}"] = bits(o)
    for fp8 in (False, True):
        o = R.rms_norm_split_rope(xd, sn.to(dev), cs.to(dev), w.to(dev), fp8)
        r[f"split_rope_fp8{int(fp8)}"] = bits(o)
    np.savez_compressed(os.path.join(out_dir, "ref_gpu_rope.npz"), **r)

    # ---- torch's CUDA GELU-tanh over every bf16 value
    allb = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    ge = torch.nn.functional.gelu(allb.to(dev), approximate="tanh")
    np.savez_compressed(os.path.join(out_dir, "torch_gpu_gelu_bf16.npz"), x=bits(allb), y=bits(ge))
    torch.cuda.synchronize()
    print("wrote", sorted(os.listdir(out_dir)))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
