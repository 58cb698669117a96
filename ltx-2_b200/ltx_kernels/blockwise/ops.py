"""Tensor-level wrappers of the sm_100a C-ABI (include/ltxfp8.h).

These functions take and return torch tensors, allocate outputs with torch's
caching allocator, and launch on the current CUDA stream.  They never
synchronise and never fall back to another implementation: non-CUDA inputs,
unsupported shapes and a missing library raise.

Layout conventions are those of Lightricks/LTX-2's ltx-kernels blockwise path:
activation scales are MN-major -- element (m, kb) at ``sfa[kb * ld + m]`` --
exposed as an ``(M, K/128)`` view with strides ``(1, align4(M))``
(ltx-kernels/src/ltx_kernels/blockwise/triton_ops.py:134-135).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .. import _lib as L


def align4(n: int) -> int:
    """get_tma_aligned_size(n, 4) (triton_ops.py:9-11)."""
    return (n + 3) // 4 * 4


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(name: str, *ts: Optional[torch.Tensor]) -> None:
    """CUDA tensors, all on one device (a kernel handed another GPU's pointer would read
    memory its device may not map)."""
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{name}: ltx-2_b200 kernels need CUDA (sm_100) tensors, got {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{name}: all tensors must be on one device, got {dev} and {t.device}")


class _DeviceGuard:
    """Switch to the tensor's device only when it differs from the current one."""

    def __init__(self, t: torch.Tensor):
        self.idx = t.device.index
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if self.idx is not None and self.idx != cur:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def scale_layout(s: torch.Tensor, M: int, KB: int) -> int:
    """Leading dimension of an activation-scale tensor holding (m, kb) at [kb * ld + m].

    Accepts the reference's two layouts: the ``(M, KB)`` MN-major view returned
    by blockwise::quantize (stride (1, ld)), and the contiguous ``(KB, M)``
    tensor returned by blockwise_quantize_torch (functional.py:144)."""
    if s.dtype != torch.float32:
        raise RuntimeError(f"activation scales must be float32, got {s.dtype}")
    if tuple(s.shape) == (M, KB) and (s.stride(0) == 1 or M == 1) and (KB == 1 or s.stride(1) >= M):
        return s.stride(1) if KB > 1 else max(M, 1)
    if tuple(s.shape) == (KB, M) and (s.stride(1) == 1 or M == 1) and (KB == 1 or s.stride(0) >= M):
        return s.stride(0) if KB > 1 else max(M, 1)
    raise RuntimeError(
        f"activation scales of shape {tuple(s.shape)} strides {s.stride()} are not an MN-major "
        f"({M}, {KB}) view or a contiguous ({KB}, {M}) tensor")


def empty_act_scales(M: int, KB: int, device) -> torch.Tensor:
    """An (M, KB) fp32 view with strides (1, align4(M)), as blockwise::quantize returns."""
    ld = align4(M)
    return torch.empty_strided((M, KB), (1, ld), dtype=torch.float32, device=device)


# ----------------------------------------------------------------------------- quantisers
def quantize_1x128(x: torch.Tensor, mode: int = L.QUANT_TORCH) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [..., K] -> (e4m3 [M, K], fp32 scales (M, K/128) MN-major view)."""
    _require_cuda("quantize_1x128", x)
    if x.dtype != torch.bfloat16:
        raise RuntimeError(f"quantize_1x128 expects bf16 input, got {x.dtype}")
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    q = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device)
    s = empty_act_scales(M, K // 128 if K % 128 == 0 else 0, x.device)
    with _DeviceGuard(x):
        L.check(L.load().ltxfp8_quantize_1x128(x2.data_ptr(), M, K, x2.stride(0), q.data_ptr(), K, s.data_ptr(),
                                                align4(M), mode, _stream(x)))
    return q, s


def quantize_weight_128x128(w: torch.Tensor, scale_max: float = 448.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """W [N, K] (fp32/bf16/fp16) -> (e4m3 [N, K], fp32 scales [N/128, K/128]); s = (1/amax)*scale_max."""
    _require_cuda("quantize_weight_128x128", w)
    dt = {torch.float32: L.DTYPE_F32, torch.bfloat16: L.DTYPE_BF16, torch.float16: L.DTYPE_F16}.get(w.dtype)
    if dt is None:
        raise RuntimeError(f"quantize_weight_128x128: unsupported dtype {w.dtype}")
    if w.dim() != 2:
        raise RuntimeError("quantize_weight_128x128 expects a 2-D weight")
    w = w.contiguous()
    N, K = w.shape
    q = torch.empty((N, K), dtype=torch.float8_e4m3fn, device=w.device)
    s = torch.empty((N // 128, K // 128), dtype=torch.float32, device=w.device)
    with _DeviceGuard(w):
        if scale_max == 448.0:
            L.check(L.load().ltxfp8_quantize_weight_128x128(w.data_ptr(), dt, N, K, q.data_ptr(), s.data_ptr(),
                                                             _stream(w)))
        else:
            L.check(L.load().ltxfp8_quantize_weight_128x128_scaled(w.data_ptr(), dt, N, K, float(scale_max),
                                                                    q.data_ptr(), s.data_ptr(), _stream(w)))
    return q, s


def fp6_pack(x: torch.Tensor) -> torch.Tensor:
    """e4m3 codes (uint8 or float8_e4m3fn) [m, n], n % 8 == 0 -> packed uint8 [m, n*3/4]."""
    _require_cuda("fp6_pack", x)
    if x.dim() != 2 or x.element_size() != 1:
        raise RuntimeError("fp6_pack: expected a 2-D one-byte tensor")
    x = x.contiguous().view(torch.uint8)
    m, n = x.shape
    out = torch.empty((m, n * 3 // 4), dtype=torch.uint8, device=x.device)
    with _DeviceGuard(x):
        L.check(L.load().ltxfp8_fp6_pack(x.data_ptr(), m, n, out.data_ptr(), _stream(x)))
    return out


def fp6_unpack(x: torch.Tensor, original_n: int) -> torch.Tensor:
    """Packed uint8 [m, n*3/4] -> e4m3 codes uint8 [m, n] (dropped exponent bits zero)."""
    _require_cuda("fp6_unpack", x)
    if x.dim() != 2 or x.dtype != torch.uint8:
        raise RuntimeError("fp6_unpack: expected a 2-D uint8 tensor")
    m, npk = x.shape
    if npk != original_n * 3 // 4:
        raise RuntimeError(f"fp6_unpack: packed size mismatch: expected {original_n * 3 // 4}, got {npk}")
    x = x.contiguous()
    out = torch.empty((m, original_n), dtype=torch.uint8, device=x.device)
    with _DeviceGuard(x):
        L.check(L.load().ltxfp8_fp6_unpack(x.data_ptr(), m, original_n, out.data_ptr(), _stream(x)))
    return out


def fp6_to_tc(w6: torch.Tensor, sfb: torch.Tensor, out: Optional[torch.Tensor] = None,
              out_scales: Optional[torch.Tensor] = None):
    """Packed FP6 weight uint8 [N, K*3/4] (:func:`fp6_pack`'s layout) and its fp32
    scales [N/128, K/128] -> ``(w6_tc, sfb6)`` for ``gemm(..., w_fp6=True)``: the codes
    in the tensor core's 6-bit order and the scales x 2^-6."""
    _require_cuda("fp6_to_tc", w6, sfb)
    if w6.dim() != 2 or w6.dtype != torch.uint8 or w6.shape[1] % 3:
        raise RuntimeError("fp6_to_tc: expected a packed uint8 [N, K*3/4] weight")
    N, K = w6.shape[0], w6.shape[1] // 3 * 4
    if N % 128 or K % 128:
        raise RuntimeError(f"fp6_to_tc: N and K must be multiples of 128 (N={N} K={K})")
    if sfb.dtype != torch.float32 or tuple(sfb.shape) != (N // 128, K // 128):
        raise RuntimeError(f"fp6_to_tc: scales must be fp32 [{N // 128}, {K // 128}]")
    w6 = w6.contiguous()
    sfb = sfb.contiguous()
    if out is None:
        out = torch.empty_like(w6)
    if out_scales is None:
        out_scales = torch.empty_like(sfb)
    if out.shape != w6.shape or out.dtype != torch.uint8 or not out.is_contiguous() or out.data_ptr() % 32:
        raise RuntimeError("fp6_to_tc: out must be a contiguous, 32-byte aligned uint8 tensor of the weight's shape")
    if out_scales.shape != sfb.shape or out_scales.dtype != torch.float32 or not out_scales.is_contiguous():
        raise RuntimeError("fp6_to_tc: out_scales must be contiguous fp32 of the scales' shape")
    with _DeviceGuard(w6):
        L.check(L.load().ltxfp8_fp6_to_tc(w6.data_ptr(), sfb.data_ptr(), N, K, out.data_ptr(),
                                          out_scales.data_ptr(), _stream(w6)))
    return out, out_scales


def dequantize_1x128(q: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """e4m3 [M, K] + scales (M, K/128) with any strides -> bf16 [M, K]."""
    _require_cuda("dequantize_1x128", q, scales)
    K = q.shape[-1]
    q2 = q.reshape(-1, K).contiguous()
    M = q2.shape[0]
    if scales.dim() != 2 or scales.shape[0] != M:
        raise RuntimeError(f"dequantize_1x128: scales shape {tuple(scales.shape)} does not match {M} rows")
    out = torch.empty((M, K), dtype=torch.bfloat16, device=q.device)
    with _DeviceGuard(q):
        L.check(L.load().ltxfp8_dequantize_1x128(q2.data_ptr(), scales.data_ptr(), scales.stride(0),
                                                  scales.stride(1), M, K, out.data_ptr(), _stream(q)))
    return out


# ----------------------------------------------------------------------------- fused producers
def _rows3(x: torch.Tensor, name: str) -> Tuple[int, int, int]:
    if x.dim() != 3:
        raise RuntimeError(f"{name}: expected a [b, s, h] tensor, got shape {tuple(x.shape)}")
    if x.dtype != torch.bfloat16:
        raise RuntimeError(f"{name}: expected bf16, got {x.dtype}")
    if not x.is_contiguous():
        raise RuntimeError(f"{name}: x must be contiguous")
    return x.shape[0], x.shape[1], x.shape[2]


def _param3(p: torch.Tensor, b: int, s: int, h: int, name: str) -> Tuple[int, int]:
    """(batch stride, token stride) of a [b, 1 or s, h] bf16 parameter; token stride 0
    when it broadcasts over the sequence (triton_ops.py:161,213)."""
    if p.dtype != torch.bfloat16:
        raise RuntimeError(f"{name}: expected bf16, got {p.dtype}")
    if p.dim() != 3 or p.shape[0] != b or p.shape[1] not in (1, s) or p.shape[2] != h or p.stride(2) != 1:
        raise RuntimeError(f"{name}: expected a [{b}, 1 or {s}, {h}] tensor with unit inner stride, "
                           f"got shape {tuple(p.shape)} strides {p.stride()}")
    return p.stride(0), (0 if p.shape[1] == 1 else p.stride(1))


def adanorm_quantize(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                     mode: int = L.QUANT_TORCH) -> Tuple[torch.Tensor, torch.Tensor]:
    """RMSNorm + AdaLN modulation + 1x128 quant: bf16 [b, s, h] -> (e4m3 [b*s, h], scales)."""
    _require_cuda("adanorm_quantize", x, scale, shift)
    b, s, h = _rows3(x, "adanorm_quantize")
    # The reference decides broadcasting from norm_scale alone (triton_ops.py:161).
    sc_bs, sc_ss = _param3(scale, b, s, h, "adanorm_quantize: scale")
    sh_bs, sh_ss = _param3(shift, b, s, h, "adanorm_quantize: shift")
    if sc_ss == 0:
        sh_ss = 0
    M = b * s
    q = torch.empty((M, h), dtype=torch.float8_e4m3fn, device=x.device)
    sfa = empty_act_scales(M, h // 128 if h % 128 == 0 else 0, x.device)
    with _DeviceGuard(x):
        L.check(L.load().ltxfp8_adanorm_quantize(x.data_ptr(), b, s, h, scale.data_ptr(), sc_bs, sc_ss,
                                                  shift.data_ptr(), sh_bs, sh_ss, q.data_ptr(), sfa.data_ptr(),
                                                  align4(M), mode, _stream(x)))
    return q, sfa


def rms_fma(x: torch.Tensor, y: torch.Tensor, z: torch.Tensor, quantize: bool = True,
            mode: int = L.QUANT_TORCH):
    """x <- x + y * z (in place), then RMS-normalise; returns (e4m3 [b*s, h], scales) or bf16 [b*s, h]."""
    _require_cuda("rms_fma", x, y, z)
    b, s, h = _rows3(x, "rms_fma")
    if y.shape != x.shape or y.dtype != torch.bfloat16 or not y.is_contiguous():
        raise RuntimeError("rms_fma: y must be a contiguous bf16 tensor shaped like x")
    z_bs, z_ss = _param3(z, b, s, h, "rms_fma: z")
    M = b * s
    q = sfa = out = None
    if quantize:
        q = torch.empty((M, h), dtype=torch.float8_e4m3fn, device=x.device)
        sfa = empty_act_scales(M, h // 128 if h % 128 == 0 else 0, x.device)
    else:
        out = torch.empty((M, h), dtype=torch.bfloat16, device=x.device)
    with _DeviceGuard(x):
        L.check(L.load().ltxfp8_rms_fma(x.data_ptr(), y.data_ptr(), b, s, h, z.data_ptr(), z_bs, z_ss,
                                         None if q is None else q.data_ptr(),
                                         None if sfa is None else sfa.data_ptr(), align4(M),
                                         None if out is None else out.data_ptr(), mode, _stream(x)))
    return (q, sfa) if quantize else out


def gated_attention(x: torch.Tensor, gate_logits: torch.Tensor, quantize: bool = True,
                    mode: int = L.QUANT_TORCH):
    """x bf16 [b, t, h] * 2 sigmoid(gate_logits [b, t, heads]) per head; quantised or bf16 [b*t, h]."""
    _require_cuda("gated_attention", x, gate_logits)
    b, t, h = _rows3(x, "gated_attention")
    heads = gate_logits.shape[-1]
    if gate_logits.shape[:-1] != x.shape[:-1]:
        raise RuntimeError(f"gated_attention: gate_logits shape {tuple(gate_logits.shape)} does not match x")
    gdt = {torch.bfloat16: L.DTYPE_BF16, torch.float32: L.DTYPE_F32}.get(gate_logits.dtype)
    if gdt is None:
        raise RuntimeError(f"gated_attention: gate logits must be bf16 or fp32, got {gate_logits.dtype}")
    g = gate_logits.contiguous()
    M = b * t
    q = sfa = out = None
    if quantize:
        q = torch.empty((M, h), dtype=torch.float8_e4m3fn, device=x.device)
        sfa = empty_act_scales(M, h // 128 if h % 128 == 0 else 0, x.device)
    else:
        out = torch.empty((M, h), dtype=torch.bfloat16, device=x.device)
    with _DeviceGuard(x):
        L.check(L.load().ltxfp8_gated_attention(x.data_ptr(), g.data_ptr(), gdt, M, h, heads,
                                                 None if q is None else q.data_ptr(),
                                                 None if sfa is None else sfa.data_ptr(), align4(M),
                                                 None if out is None else out.data_ptr(), mode, _stream(x)))
    return (q, sfa) if quantize else out


def gelu_quantize_1x128(x: torch.Tensor, mode: int = L.QUANT_TORCH) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [..., K] -> 1x128 quant of x * sigmoid(1.702 x): (e4m3 [M, K], scales)."""
    _require_cuda("gelu_quantize_1x128", x)
    if x.dtype != torch.bfloat16:
        raise RuntimeError(f"gelu_quantize_1x128 expects bf16 input, got {x.dtype}")
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    q = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device)
    s = empty_act_scales(M, K // 128 if K % 128 == 0 else 0, x.device)
    with _DeviceGuard(x):
        L.check(L.load().ltxfp8_gelu_quantize_1x128(x2.data_ptr(), M, K, x2.stride(0), q.data_ptr(), K,
                                                     s.data_ptr(), align4(M), mode, _stream(x)))
    return q, s


def gelu_tanh_quantize_1x128(x: torch.Tensor, mode: int = L.QUANT_TORCH) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [..., K] -> 1x128 quant of torch's ``F.gelu(x, approximate="tanh")`` (bf16):
    (e4m3 [M, K], scales).  The reference FFN's GELU followed by the down projection's
    input quantisation (gelu_approx.py:10, linear.py:91-93), in one pass over x."""
    _require_cuda("gelu_tanh_quantize_1x128", x)
    if x.dtype != torch.bfloat16:
        raise RuntimeError(f"gelu_tanh_quantize_1x128 expects bf16 input, got {x.dtype}")
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    q = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device)
    s = empty_act_scales(M, K // 128 if K % 128 == 0 else 0, x.device)
    with _DeviceGuard(x):
        L.check(L.load().ltxfp8_gelu_tanh_quantize_1x128(x2.data_ptr(), M, K, x2.stride(0), q.data_ptr(), K,
                                                          s.data_ptr(), align4(M), mode, _stream(x)))
    return q, s


def rms_norm_rope(x: torch.Tensor, cos_freqs: torch.Tensor, sin_freqs: torch.Tensor,
                  weights: Optional[torch.Tensor] = None, out_fp8: bool = False) -> torch.Tensor:
    """RMSNorm + interleaved RoPE over the last dim of bf16 x; cos/sin reshape to (rows, dim)."""
    _require_cuda("rms_norm_rope", x, cos_freqs, sin_freqs, weights)
    for name, t in (("x", x), ("cos_freqs", cos_freqs), ("sin_freqs", sin_freqs)):
        if t.dtype != torch.bfloat16:
            raise RuntimeError(f"rms_norm_rope: {name} must be bf16, got {t.dtype}")
    dim = x.shape[-1]
    x2 = x.reshape(-1, dim).contiguous()
    rows = x2.shape[0]
    c2 = cos_freqs.reshape(-1, dim).contiguous()
    s2 = sin_freqs.reshape(-1, dim).contiguous()
    if c2.shape[0] != rows or s2.shape[0] != rows:
        raise RuntimeError(f"rms_norm_rope: cos/sin have {c2.shape[0]}/{s2.shape[0]} rows of {dim}, x has {rows}")
    w = None
    if weights is not None:
        if weights.dtype != torch.bfloat16 or weights.numel() != dim:
            raise RuntimeError("rms_norm_rope: weights must be bf16 [dim]")
        w = weights.contiguous()
    out = torch.empty(x.shape, dtype=torch.float8_e4m3fn if out_fp8 else torch.bfloat16, device=x.device)
    with _DeviceGuard(x):
        L.check(L.load().ltxfp8_rms_norm_rope(x2.data_ptr(), rows, dim, c2.data_ptr(), s2.data_ptr(), dim,
                                               None if w is None else w.data_ptr(), out.data_ptr(), int(out_fp8),
                                               _stream(x)))
    return out


def rms_norm_split_rope(x: torch.Tensor, cos_freqs: torch.Tensor, sin_freqs: torch.Tensor,
                        weights: Optional[torch.Tensor] = None, out_fp8: bool = False) -> torch.Tensor:
    """RMSNorm + split RoPE: x bf16 [b, s, h]; cos/sin [b or 1, heads, s, d/2] (any outer
    strides, unit inner stride -- e.g. the swapaxes view of apply_split_rotary_emb)."""
    _require_cuda("rms_norm_split_rope", x, cos_freqs, sin_freqs, weights)
    b, s, h = _rows3(x, "rms_norm_split_rope")
    if cos_freqs.shape != sin_freqs.shape or cos_freqs.dim() != 4:
        raise RuntimeError("rms_norm_split_rope: cos_freqs and sin_freqs must both be [b, heads, s, d/2]")
    fb, heads, fs, half = cos_freqs.shape
    if fb not in (1, b) or fs != s or heads * half * 2 != h:
        raise RuntimeError(f"rms_norm_split_rope: freq shape {tuple(cos_freqs.shape)} does not match x {tuple(x.shape)}")
    strides = []
    for t in (cos_freqs, sin_freqs):
        if t.dtype != torch.bfloat16 or t.stride(3) != 1:
            raise RuntimeError("rms_norm_split_rope: freqs must be bf16 with a unit inner stride")
        strides.append((0 if fb == 1 else t.stride(0), t.stride(1), t.stride(2)))
    w = None
    if weights is not None:
        if weights.dtype != torch.bfloat16 or weights.numel() != h:
            raise RuntimeError("rms_norm_split_rope: weights must be bf16 [h]")
        w = weights.contiguous()
    out = torch.empty(x.shape, dtype=torch.float8_e4m3fn if out_fp8 else torch.bfloat16, device=x.device)
    (cb, cn, cs), (sb, sn, ss) = strides
    with _DeviceGuard(x):
        L.check(L.load().ltxfp8_rms_norm_split_rope(x.data_ptr(), b, s, h, heads, cos_freqs.data_ptr(), cb, cn, cs,
                                                     sin_freqs.data_ptr(), sb, sn, ss,
                                                     None if w is None else w.data_ptr(), out.data_ptr(),
                                                     int(out_fp8), _stream(x)))
    return out


# ----------------------------------------------------------------------------- GEMM
def gemm(a_q: torch.Tensor, sfa: torch.Tensor, w_q: torch.Tensor, sfb: torch.Tensor,
         bias: Optional[torch.Tensor] = None, *, out: Optional[torch.Tensor] = None,
         gelu=False, requant: bool = False, write_d: bool = True,
         lora_ax: Optional[torch.Tensor] = None, lora_b: Optional[torch.Tensor] = None,
         lora_alpha: float = 1.0, split_k: bool = True, requant_mode: int = L.QUANT_TORCH,
         w_fp6: bool = False):
    """Blockwise FP8 GEMM with fused epilogue.

    ``gelu``: False, True (torch's GELU-tanh formula, bf16 results identical to
    ``F.gelu(approximate="tanh")``) or ``"fast"`` (the same function through
    approximate instructions, within one bf16 ulp).  Returns D (bf16 [M, N]) when
    ``requant`` is False, else ``(D or None, q, scales)`` where ``q``/``scales`` are the
    1x128 quantisation of the (GELU'd) bf16 output in the layout blockwise::quantize
    produces, with ``requant_mode``'s arithmetic (QUANT_TORCH or QUANT_TRITON).
    Skinny shapes get a split-K workspace from the caching allocator unless
    ``split_k`` is False.  ``w_fp6``: ``w_q``/``sfb`` are a 6-bit weight from
    :func:`fp6_to_tc` (uint8 [N, K*3/4]), read by the tensor core as e2m3."""
    _require_cuda("gemm", a_q, sfa, w_q, sfb, bias, lora_ax, lora_b)
    if a_q.dim() != 2 or w_q.dim() != 2:
        raise RuntimeError("gemm expects 2-D operands")
    M, K = a_q.shape
    N, K2 = w_q.shape
    if w_fp6:
        if w_q.dtype != torch.uint8 or K2 * 4 != K * 3:
            raise RuntimeError(f"gemm: a 6-bit weight must be uint8 [N, {K * 3 // 4}] from fp6_to_tc")
        if w_q.data_ptr() % 32:
            raise RuntimeError("gemm: a 6-bit weight must be 32-byte aligned")
    elif K != K2:
        raise RuntimeError(f"gemm: K mismatch ({K} vs {K2})")
    if a_q.dtype != torch.float8_e4m3fn or (not w_fp6 and w_q.dtype != torch.float8_e4m3fn):
        raise RuntimeError("gemm: operands must be float8_e4m3fn")
    if not a_q.is_contiguous() or not w_q.is_contiguous():
        raise RuntimeError("gemm: operands must be contiguous (K-major)")
    KB = K // 128
    ld = scale_layout(sfa, M, KB)
    if sfb.dtype != torch.float32 or tuple(sfb.shape) != (N // 128, KB) or not sfb.is_contiguous():
        raise RuntimeError(f"gemm: weight scales must be contiguous fp32 [{N // 128}, {KB}]")
    if bias is not None:
        if bias.dtype != torch.float32 or bias.numel() != N:
            raise RuntimeError("gemm: bias must be fp32 [N] (the SM89 contract takes float*)")
        bias = bias.contiguous()
    if out is not None and (out.dtype != torch.bfloat16 or tuple(out.shape) != (M, N) or not out.is_contiguous()
                            or out.device != a_q.device):
        raise RuntimeError(f"gemm: out must be a contiguous bf16 [{M}, {N}] tensor on {a_q.device}")
    if requant and not write_d:
        d = None
    else:
        d = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=a_q.device)
    if M == 0:  # no tokens: empty results, nothing to launch (the C ABI takes M >= 1)
        if requant:
            return d, torch.empty((0, N), dtype=torch.float8_e4m3fn, device=a_q.device), \
                empty_act_scales(0, N // 128, a_q.device)
        return d
    ep = L.Epilogue()
    if gelu == "fast":
        ep.gelu_tanh = L.GELU_TANH_FAST
    elif gelu is True or gelu == "tanh":
        ep.gelu_tanh = L.GELU_TANH
    elif gelu is False or gelu is None:
        ep.gelu_tanh = L.GELU_NONE
    else:
        raise RuntimeError(f"gemm: gelu must be False, True or 'fast', got {gelu!r}")
    ep.requant_mode = requant_mode
    q = s = None
    if requant:
        q = torch.empty((M, N), dtype=torch.float8_e4m3fn, device=a_q.device)
        s = empty_act_scales(M, N // 128, a_q.device)
        ep.requant_q = q.data_ptr()
        ep.requant_scales = s.data_ptr()
        ep.requant_ld = align4(M)
        ep.skip_d = 0 if write_d else 1
    if lora_ax is not None:
        if lora_b is None:
            raise RuntimeError("gemm: lora_b is required with lora_ax")
        r = lora_ax.shape[1]
        if lora_ax.dtype != torch.bfloat16 or lora_b.dtype != torch.bfloat16 or tuple(lora_ax.shape) != (M, r) \
                or tuple(lora_b.shape) != (N, r):
            raise RuntimeError("gemm: LoRA operands must be bf16 ax [M, r] and B [N, r]")
        lora_ax = lora_ax.contiguous()
        lora_b = lora_b.contiguous()
        ep.lora_ax = lora_ax.data_ptr()
        ep.lora_b = lora_b.data_ptr()
        ep.lora_r = r
        ep.lora_alpha = float(lora_alpha)
    with _DeviceGuard(a_q):
        ws_bytes = gemm_workspace_bytes(M, N, K, a_q.device) if split_k else 0
        ws = None
        if ws_bytes:
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=a_q.device)
            ep.workspace = ws.data_ptr()
            ep.workspace_bytes = ws_bytes
        fn = L.load().ltxfp8_gemm_fp6w if w_fp6 else L.load().ltxfp8_gemm
        L.check(fn(a_q.data_ptr(), sfa.data_ptr(), ld, w_q.data_ptr(), sfb.data_ptr(),
                   None if bias is None else bias.data_ptr(),
                   None if d is None else d.data_ptr(), M, N, K, ep, _stream(a_q)))
    if requant:
        return d, q, s
    return d


_WS_CACHE: dict = {}


def gemm_workspace_bytes(M: int, N: int, K: int, device) -> int:
    """Split-K scratch the GEMM would use at this shape (0 when it needs none)."""
    key = (torch.cuda.current_device() if device is None else device.index, M, N, K)
    v = _WS_CACHE.get(key)
    if v is None:
        import ctypes
        n = ctypes.c_size_t(0)
        L.check(L.load().ltxfp8_gemm_workspace_bytes(M, N, K, ctypes.byref(n)))
        v = _WS_CACHE[key] = n.value
    return v


_PLAN_CACHE: dict = {}


def gemm_plan(M: int, N: int, K: int, device) -> dict:
    """How ``gemm`` (with split-K allowed) launches this shape: workspace bytes, kernel
    launches per call, K splits and the first split row (``M``: no split)."""
    key = (torch.cuda.current_device() if device is None else device.index, M, N, K)
    v = _PLAN_CACHE.get(key)
    if v is None:
        import ctypes
        info = L.GemmPlanInfo()
        L.check(L.load().ltxfp8_gemm_plan(M, N, K, ctypes.byref(info)))
        v = _PLAN_CACHE[key] = {"workspace_bytes": info.workspace_bytes, "launches": info.launches,
                                "splits": info.splits, "split_row0": info.split_row0}
    return dict(v)


def lora_a(x: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
    """x bf16 [..., K] . A bf16 [r, K]^T -> bf16 [M, r]."""
    _require_cuda("lora_a", x, a)
    if x.dtype != torch.bfloat16 or a.dtype != torch.bfloat16:
        raise RuntimeError("lora_a expects bf16 operands")
    K = x.shape[-1]
    x2 = x.reshape(-1, K).contiguous()
    a = a.contiguous()
    r = a.shape[0]
    if a.shape[1] != K:
        raise RuntimeError("lora_a: K mismatch")
    M = x2.shape[0]
    ax = torch.empty((M, r), dtype=torch.bfloat16, device=x.device)
    with _DeviceGuard(x):
        L.check(L.load().ltxfp8_lora_a(x2.data_ptr(), a.data_ptr(), ax.data_ptr(), M, K, r, _stream(x)))
    return ax


def device_status(clear: bool = True) -> int:
    """The kernels' bounded-wait status word for the current device (0 = healthy)."""
    return L.device_status(torch.cuda.current_stream().cuda_stream, clear)
