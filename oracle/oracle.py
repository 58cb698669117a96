"""CPU oracle for the blockwise-FP8 linear path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module; the product path (``ltx-2_b200/``) never does.

Two layers:

* ``liboracle`` -- ``ltxfp8_oracle.c`` compiled with gcc: the bit-exact
  restatements of the reference's quantisers, dequantiser and the SM89 GEMM's
  per-128-K promotion order.  Each C function cites the reference lines it
  follows.
* numpy helpers -- the reference's CPU GEMM path (dequantise both operands, fp32
  matmul, add fp32 bias, cast to bf16), as described for the CPU baseline of
  ``blockwise_quantize_torch`` + ``blockwise_quantize_weights``
  (ltx-kernels/src/ltx_kernels/blockwise/functional.py:128-144), plus the exact
  LoRA math ``dequant(W) x + alpha * B (A x)`` for the runtime-LoRA extension.

bf16 tensors are carried as ``np.uint16`` bit patterns, e4m3 codes as ``np.uint8``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "ltxfp8_oracle.c")
_BUILD = os.path.join(_HERE, "_build")
_LIB_PATH = os.path.join(_BUILD, "liboracle.so")

FP8_SCALE_MAX = 448.0


def build(force: bool = False) -> str:
    """Compile the C oracle with gcc (IEEE single precision, no FMA contraction)."""
    os.makedirs(_BUILD, exist_ok=True)
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(_SRC):
        cmd = ["gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off", "-fno-fast-math",
               "-o", _LIB_PATH, _SRC, "-lm"]
        subprocess.check_call(cmd)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, i64, f32, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
        L.orc_quant_act_1x128.argtypes = [vp, i64, i64, i64, vp, i64, vp, i64, f32]
        L.orc_quant_weight_128x128.argtypes = [vp, i32, i64, i64, vp, vp, f32]
        L.orc_dequant_1x128.argtypes = [vp, vp, i64, i64, i64, i64, vp]
        L.orc_gemm_promoted.argtypes = [vp, vp, i64, vp, vp, vp, i64, i64, i64, vp, vp]
        L.orc_gelu_tanh_bf16_array.argtypes = [vp, i64, vp]
        L.orc_e4m3_to_f32_array.argtypes = [vp, i64, vp]
        L.orc_f32_to_e4m3_array.argtypes = [vp, i64, vp]
        L.orc_f32_to_bf16_array.argtypes = [vp, i64, vp]
        L.orc_adanorm_quant.argtypes = [vp, i64, i64, i64, vp, i64, i64, vp, i64, i64, vp, vp, i64]
        L.orc_rms_fma.argtypes = [vp, vp, i64, i64, i64, vp, i64, i64, vp, vp, i64, vp]
        L.orc_gated_attention.argtypes = [vp, vp, i32, i64, i64, i64, vp, vp, i64, vp]
        L.orc_gelu_quant.argtypes = [vp, i64, i64, vp, vp, i64]
        L.orc_rms_norm_rope.argtypes = [vp, i64, i64, vp, vp, i64, vp, vp, i32]
        L.orc_rms_norm_split_rope.argtypes = [vp, i64, i64, i64, i64, vp, i64, i64, i64, vp, i64, i64, i64, vp, vp,
                                              i32]
        L.orc_exp_cw.argtypes = [f32]
        L.orc_exp_cw.restype = f32
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def align4(n: int) -> int:
    """get_tma_aligned_size(n, 4) of triton_ops.py:9-11."""
    return (n + 3) // 4 * 4


# ----------------------------------------------------------------------------- conversions
def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    f = np.ascontiguousarray(f, dtype=np.float32)
    out = np.empty(f.shape, np.uint16)
    lib().orc_f32_to_bf16_array(_p(f), f.size, _p(out))
    return out


_E4M3_LUT = None


def e4m3_to_f32(c: np.ndarray) -> np.ndarray:
    global _E4M3_LUT
    if _E4M3_LUT is None:
        codes = np.arange(256, dtype=np.uint8)
        _E4M3_LUT = np.empty(256, np.float32)
        lib().orc_e4m3_to_f32_array(_p(codes), 256, _p(_E4M3_LUT))
    return _E4M3_LUT[np.asarray(c, dtype=np.uint8)]


def f32_to_e4m3(f: np.ndarray) -> np.ndarray:
    f = np.ascontiguousarray(f, dtype=np.float32)
    out = np.empty(f.shape, np.uint8)
    lib().orc_f32_to_e4m3_array(_p(f), f.size, _p(out))
    return out


# ----------------------------------------------------------------------------- quantisers
def quant_act_1x128(x_bf16: np.ndarray, sfa_ld: int | None = None):
    """Activation quant, 1x128 groups (functional.py:138-144, triton_ops.py:102-151).

    Returns (codes uint8 [M,K], scale buffer float32 [K/128, sfa_ld]); the scale of
    (m, kb) sits at buffer[kb, m], i.e. the MN-major layout of triton_ops.py:134-135.
    Entries m >= M of the buffer are left NaN (the reference leaves them unset).
    """
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    M, K = x.shape
    assert K % 128 == 0
    ld = align4(M) if sfa_ld is None else sfa_ld
    q = np.empty((M, K), np.uint8)
    sfa = np.full((K // 128, ld), np.nan, np.float32)
    lib().orc_quant_act_1x128(_p(x), M, K, K, _p(q), K, _p(sfa), ld, FP8_SCALE_MAX)
    return q, sfa


def quant_weight_128x128(w: np.ndarray, scale_max: float = FP8_SCALE_MAX):
    """Weight quant, 128x128 blocks (functional.py:128-135).  w: float32 or bf16 bits."""
    if w.dtype == np.uint16:
        dt = 1
    else:
        w = w.astype(np.float32)
        dt = 0
    w = np.ascontiguousarray(w)
    N, K = w.shape
    assert N % 128 == 0 and K % 128 == 0
    q = np.empty((N, K), np.uint8)
    s = np.empty((N // 128, K // 128), np.float32)
    lib().orc_quant_weight_128x128(_p(w), dt, N, K, _p(q), _p(s), scale_max)
    return q, s


def dequant_1x128(q: np.ndarray, scales: np.ndarray, row_stride: int, col_stride: int) -> np.ndarray:
    """bf16 dequant with strided scales (triton_ops.py:387-433)."""
    q = np.ascontiguousarray(q, dtype=np.uint8)
    M, K = q.shape
    sc = np.ascontiguousarray(scales, dtype=np.float32)
    out = np.empty((M, K), np.uint16)
    lib().orc_dequant_1x128(_p(q), _p(sc), row_stride, col_stride, M, K, _p(out))
    return out


def gelu_tanh_bf16(x_bf16: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    y = np.empty_like(x)
    lib().orc_gelu_tanh_bf16_array(_p(x), x.size, _p(y))
    return y


# ----------------------------------------------------------------------------- fused producers
# Restatements of the reference's Triton producers (triton_ops.py:52-345) with the
# arithmetic the CUDA kernels fix (fp32 row sums in lane/butterfly order, IEEE
# sqrt + division, Cody-Waite exp).  Parity against the reference is unpinned:
# its Triton kernels cannot run here.  All inputs are bf16 bit patterns (uint16).
def _u16(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint16)


def _param_strides(p: np.ndarray, S: int):
    """(buffer, bstride, sstride) of a [B, 1 or S, H] parameter (sstride 0 broadcasts)."""
    B, T, H = p.shape
    return _u16(p), T * H, (0 if T == 1 else H)


def adanorm_quant(x: np.ndarray, scale: np.ndarray, shift: np.ndarray, sfa_ld: int | None = None):
    """x [B, S, H], scale/shift [B, 1 or S, H] -> (codes [B*S, H], scales [H/128, ld])."""
    x = _u16(x)
    B, S, H = x.shape
    M = B * S
    ld = align4(M) if sfa_ld is None else sfa_ld
    sc, sc_bs, sc_ss = _param_strides(scale, S)
    sh, sh_bs, sh_ss = _param_strides(shift, S)
    q = np.empty((M, H), np.uint8)
    sfa = np.full((H // 128, ld), np.nan, np.float32)
    lib().orc_adanorm_quant(_p(x), B, S, H, _p(sc), sc_bs, sc_ss, _p(sh), sh_bs, sh_ss, _p(q), _p(sfa), ld)
    return q, sfa


def rms_fma(x: np.ndarray, y: np.ndarray, z: np.ndarray, quantize: bool = True, sfa_ld: int | None = None):
    """x, y [B, S, H], z [B, 1 or S, H] -> (updated x, codes, scales) or (updated x, bf16 out)."""
    x = _u16(x).copy()
    y = _u16(y)
    B, S, H = x.shape
    M = B * S
    zb, z_bs, z_ss = _param_strides(z, S)
    if quantize:
        ld = align4(M) if sfa_ld is None else sfa_ld
        q = np.empty((M, H), np.uint8)
        sfa = np.full((H // 128, ld), np.nan, np.float32)
        lib().orc_rms_fma(_p(x), _p(y), B, S, H, _p(zb), z_bs, z_ss, _p(q), _p(sfa), ld, None)
        return x, q, sfa
    out = np.empty((M, H), np.uint16)
    lib().orc_rms_fma(_p(x), _p(y), B, S, H, _p(zb), z_bs, z_ss, None, None, 0, _p(out))
    return x, out


def gated_attention(x: np.ndarray, logits: np.ndarray, quantize: bool = True, sfa_ld: int | None = None):
    """x [M, H] bf16 bits; logits [M, heads] bf16 bits (uint16) or float32."""
    x = _u16(x)
    M, H = x.shape
    heads = logits.shape[-1]
    f32 = logits.dtype == np.float32
    lg = np.ascontiguousarray(logits, dtype=np.float32 if f32 else np.uint16)
    if quantize:
        ld = align4(M) if sfa_ld is None else sfa_ld
        q = np.empty((M, H), np.uint8)
        sfa = np.full((H // 128, ld), np.nan, np.float32)
        lib().orc_gated_attention(_p(x), _p(lg), int(f32), M, H, heads, _p(q), _p(sfa), ld, None)
        return q, sfa
    out = np.empty((M, H), np.uint16)
    lib().orc_gated_attention(_p(x), _p(lg), int(f32), M, H, heads, None, None, 0, _p(out))
    return out


def gelu_quant(x: np.ndarray, sfa_ld: int | None = None):
    """x [M, K] bf16 bits -> 1x128 quant of x * sigmoid(1.702 x)."""
    x = _u16(x)
    M, K = x.shape
    ld = align4(M) if sfa_ld is None else sfa_ld
    q = np.empty((M, K), np.uint8)
    sfa = np.full((K // 128, ld), np.nan, np.float32)
    lib().orc_gelu_quant(_p(x), M, K, _p(q), _p(sfa), ld)
    return q, sfa


def rms_norm_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, w: np.ndarray | None = None,
                  out_fp8: bool = False) -> np.ndarray:
    """Interleaved RoPE after RMSNorm; x, cos, sin [rows, dim] bf16 bits, w [dim] or None.
    Returns bf16 bits, or e4m3 codes (torch conversion) when out_fp8."""
    x, cos, sin = _u16(x), _u16(cos), _u16(sin)
    rows, dim = x.shape
    out = np.empty((rows, dim), np.uint8 if out_fp8 else np.uint16)
    lib().orc_rms_norm_rope(_p(x), rows, dim, _p(cos), _p(sin), dim, None if w is None else _p(_u16(w)), _p(out),
                            1 if out_fp8 else 0)
    return out


def rms_norm_split_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, w: np.ndarray | None = None,
                        out_fp8: bool = False) -> np.ndarray:
    """Split RoPE after RMSNorm; x [B, S, H], cos/sin [B or 1, heads, S, d/2] bf16 bits
    (contiguous; batch 1 broadcasts).  Returns bf16 bits or saturating e4m3 codes."""
    x, cos, sin = _u16(x), _u16(cos), _u16(sin)
    B, S, H = x.shape
    fb, heads, fs, half = cos.shape
    sb = 0 if fb == 1 else heads * fs * half
    out = np.empty((B, S, H), np.uint8 if out_fp8 else np.uint16)
    lib().orc_rms_norm_split_rope(_p(x), B, S, H, heads, _p(cos), sb, fs * half, half, _p(sin), sb, fs * half, half,
                                  None if w is None else _p(_u16(w)), _p(out), 2 if out_fp8 else 0)
    return out


def fp6_pack(codes: np.ndarray) -> np.ndarray:
    """e4m3 codes [m, n] -> [m, n*3/4]: keep bit 7 and bits 4..0 of each code, four 6-bit
    values per 3 bytes, most significant first (ltx-kernels/csrc/ops/fp6_pack.cu:8-41)."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    m, n = c.shape
    v = (((c & 0x80) >> 2) | (c & 0x1F)).astype(np.uint32).reshape(m, n // 4, 4)
    p = (v[..., 0] << 18) | (v[..., 1] << 12) | (v[..., 2] << 6) | v[..., 3]
    out = np.stack([(p >> 16) & 0xFF, (p >> 8) & 0xFF, p & 0xFF], axis=-1).astype(np.uint8)
    return out.reshape(m, n * 3 // 4)


def fp6_unpack(packed: np.ndarray, n: int) -> np.ndarray:
    """Inverse of fp6_pack with the two dropped exponent bits zero (fp6_pack.cu:87-103)."""
    b = np.ascontiguousarray(packed, dtype=np.uint8).reshape(packed.shape[0], n // 4, 3).astype(np.uint32)
    p = (b[..., 0] << 16) | (b[..., 1] << 8) | b[..., 2]
    v = np.stack([(p >> 18) & 0x3F, (p >> 12) & 0x3F, (p >> 6) & 0x3F, p & 0x3F], axis=-1)
    return (((v & 0x20) << 2) | (v & 0x1F)).astype(np.uint8).reshape(packed.shape[0], n)


def fp6_to_tc(packed: np.ndarray, n: int) -> np.ndarray:
    """fp6_pack's layout -> the 6-bit operand layout of the tensor core (not a reference
    function: the layout the TMA's 16 x 6-bit type and kind::f8f6f4's e2m3 operand
    read): every 16 codes of a row in 12 bytes, code i at bits 6i..6i+5 of their
    little-endian 96-bit word."""
    m = packed.shape[0]
    b = np.ascontiguousarray(packed, dtype=np.uint8).reshape(m, n // 4, 3).astype(np.uint32)
    p = (b[..., 0] << 16) | (b[..., 1] << 8) | b[..., 2]
    v = np.stack([(p >> 18) & 0x3F, (p >> 12) & 0x3F, (p >> 6) & 0x3F, p & 0x3F], axis=-1)
    v = v.reshape(m, n // 16, 16).astype(np.uint64)
    bits = np.zeros((m, n // 16, 96), dtype=np.uint8)
    for i in range(16):
        for j in range(6):
            bits[..., 6 * i + j] = ((v[..., i] >> np.uint64(j)) & np.uint64(1)).astype(np.uint8)
    out = np.packbits(bits.reshape(m, n // 16, 12, 8), axis=-1, bitorder="little")
    return out.reshape(m, n * 3 // 4)


def exp_cw(x: float) -> float:
    return float(lib().orc_exp_cw(x))


# ----------------------------------------------------------------------------- GEMM oracles
def gemm_promoted(A, sfa, sfa_ld, W, sfb, bias, M, N, K):
    """The SM89 kernel's promotion order in scalar C (gemm.cu:150-222).  Small sizes only.

    Returns (fp32 result before the bf16 cast, bf16 result)."""
    A = np.ascontiguousarray(A, np.uint8)
    W = np.ascontiguousarray(W, np.uint8)
    sfa = np.ascontiguousarray(sfa, np.float32)
    sfb = np.ascontiguousarray(sfb, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    f = np.empty((M, N), np.float32)
    h = np.empty((M, N), np.uint16)
    lib().orc_gemm_promoted(_p(A), _p(sfa), sfa_ld, _p(W), _p(sfb), _p(b), M, N, K, _p(f), _p(h))
    return f, h


def dequant_act_f32(q: np.ndarray, sfa: np.ndarray, rows: np.ndarray | None = None) -> np.ndarray:
    """fp32 dequant of activation codes with an MN-major scale buffer [K/128, ld]."""
    M, K = q.shape
    idx = np.arange(M) if rows is None else rows
    s = sfa[:, idx].T                                   # [len(idx), K/128]
    return e4m3_to_f32(q[idx]) * np.repeat(s, 128, axis=1)


def dequant_weight_f32(wq: np.ndarray, sfb: np.ndarray) -> np.ndarray:
    s = np.repeat(np.repeat(sfb, 128, axis=0), 128, axis=1)
    return e4m3_to_f32(wq) * s


def gemm_dequant_f32(aq, sfa, wq, sfb, bias=None, rows=None, w_deq=None) -> np.ndarray:
    """The reference's CPU path: dequantise, fp32 matmul, add fp32 bias (fp32 result).

    ``rows`` restricts the check to a subset of output rows (for full-size shapes).
    ``w_deq`` may pass a precomputed dequantised weight."""
    a = dequant_act_f32(aq, sfa, rows)
    w = dequant_weight_f32(wq, sfb) if w_deq is None else w_deq
    d = a @ w.T
    if bias is not None:
        d = d + bias.astype(np.float32)[None, :]
    return d.astype(np.float32)


def lora_exact_f32(x_bf16_rows: np.ndarray, lora_a_bf16: np.ndarray, lora_b_bf16: np.ndarray,
                   alpha: float) -> np.ndarray:
    """alpha * B (A x) in fp32 from bf16 operands (the runtime-LoRA term)."""
    x = bf16_to_f32(x_bf16_rows)
    a = bf16_to_f32(lora_a_bf16)
    b = bf16_to_f32(lora_b_bf16)
    return (alpha * ((x @ a.T) @ b.T)).astype(np.float32)


# ----------------------------------------------------------------------------- metrics
def bf16_ulp(a: np.ndarray) -> np.ndarray:
    """Spacing of bf16 values at |a| (8 significant bits): 2^(floor(log2|a|) - 7), 0 at 0."""
    a = np.abs(np.asarray(a, np.float64))
    _, e = np.frexp(a)  # a = m 2^e, m in [0.5, 1)
    ulp = np.ldexp(1.0, np.maximum(e - 8, -133))
    return np.where(a == 0, 0.0, ulp)


def error_metrics(out: np.ndarray, ref: np.ndarray, abs_tol: float = 2e-2) -> dict:
    """Error of a bf16 result against an fp32/fp64 reference.

    * ``rel_fro``       -- ||out - ref||_F / ||ref||_F.
    * ``max_abs``       -- max |out - ref| (raw).
    * ``max_abs_norm``  -- max |out - ref| / max |ref| (informative).
    * ``bound_excess``  -- max over elements of |out - ref| - (abs_tol + ulp_bf16(|ref|)):
      <= 0 means every element is within ``abs_tol`` absolute plus one bf16 ulp of the
      reference, which a correctly rounded bf16 result always meets (its rounding
      error is at most half an ulp), however large the element.
    * ``frac_over_abs`` -- fraction of elements with |out - ref| > abs_tol.
    """
    o = out.astype(np.float64)
    r = ref.astype(np.float64)
    diff = np.abs(o - r)
    fro = float(np.linalg.norm(o - r) / max(np.linalg.norm(r), 1e-30))
    mx = float(np.max(diff)) if diff.size else 0.0
    scale = float(np.max(np.abs(r))) if r.size else 1.0
    excess = float(np.max(diff - (abs_tol + bf16_ulp(r)))) if diff.size else -abs_tol
    over = float(np.mean(diff > abs_tol)) if diff.size else 0.0
    return {"rel_fro": fro, "max_abs": mx, "max_abs_norm": mx / max(scale, 1e-30), "bound_excess": excess,
            "frac_over_abs": over}


def codes_equal(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Bitwise equality of e4m3 codes where both NaN encodings (0x7F, 0xFF) count as equal.

    A 0 * inf product yields the host FPU's default NaN (negative on x86, positive on
    the GPU); the sign of that NaN carries no information."""
    a = np.asarray(a, np.uint8)
    b = np.asarray(b, np.uint8)
    nan_a = (a & 0x7F) == 0x7F
    nan_b = (b & 0x7F) == 0x7F
    return (a == b) | (nan_a & nan_b)


def scales_equal(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Bitwise fp32 equality, NaN == NaN."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))
