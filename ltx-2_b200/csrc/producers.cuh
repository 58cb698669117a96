// Fused producers of the GEMM's A operand: per-token normalisation / gating
// followed by the 1x128 e4m3 quantisation (HBM-bound streaming kernels).
//
//   adanorm_quant_kernel    RMSNorm (eps 1e-5) -> bf16 -> x * (1 + scale) + shift -> quant
//                           (ltx-kernels/src/ltx_kernels/blockwise/triton_ops.py:52-96,158-186)
//   rms_fma_kernel          x <- x + y * z (in place), o = x * rsqrt(mean(x^2)) -> quant or bf16
//                           (triton_ops.py:188-290)
//   gated_attention_kernel  o = x * 2 sigmoid(gate_logit[token, head]) -> quant or bf16
//                           (triton_ops.py:293-345)
//   gelu_quant_kernel       o = x * sigmoid(1.702 x) -> quant  (triton_ops.py:98-126, USE_GELU)
//
// Layout: one warp per token row (H <= 32 * 8 * kChunks bf16).  Lane l owns the
// 16-byte chunks c = 32 i + l; a 1x128 group is 16 consecutive chunks, so load i
// of lanes 0-15 is group 2i and of lanes 16-31 group 2i+1, and a group's abs-max
// is a 16-lane shuffle reduction.
//
// Two arithmetics (the template mode):
//  * kQuantTriton -- the reference's kernels as Triton 3.6 compiles them for sm_100:
//    bf16 operations where the Triton source keeps bf16 (its promotion rules), the
//    bf16 row sum of squares in the order of Triton's reduction tree with the
//    multiply-add fusion the compiler chose for each kernel, fused bf16 multiply-adds
//    where it fuses them, and the instructions it emits (ex2.approx for exp, div.full
//    for fp32 division, libdevice's rsqrtf).  Checked against the reference's kernels
//    on the B200 (GPU fixtures in tests/golden/ref_gpu_producers.npz): bit-exact except
//    where the fp32 1/sqrt reaches a quantised output unrounded (the quantised
//    residual-FMA path) and a few rows whose bf16 row sum the compiled kernel rounds
//    differently (rates stated in the tests).
//  * kQuantTorch -- every step an IEEE-rounded operation (fp32 row sums in a fixed
//    lane order, 1/sqrt as sqrt + division, e^x from fused multiply-adds), which the
//    CPU oracle reproduces bit for bit.
#pragma once

#include "quant.cuh"

namespace ltxfp8 {

constexpr int kProdWarps = 8;  // rows per 256-thread block

// e^x from IEEE operations only: Cody-Waite argument reduction x = k ln2 + r
// (ln2 split into a 15-bit head and a tail so k * head is exact), the Taylor
// series of e^r to degree 7 in Horner form (|r| <= ln2/2, truncation < 2^-27
// relative), and an exact two-step scaling by 2^k.  Deterministic on any IEEE
// fp32 machine with a fused multiply-add; accurate to about 1 ulp.
__device__ __forceinline__ float exp_cw(float x) {
  if (x != x) return x;
  if (x > 88.8f) return __int_as_float(0x7f800000);
  if (x < -104.0f) return 0.0f;
  const float k = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = fmaf(-k, 0.693145751953125f, x);
  r = fmaf(-k, 1.42860682030941723212e-6f, r);
  float p = 1.98412698412698413e-4f;         // 1/7!
  p = fmaf(p, r, 1.38888888888888889e-3f);  // 1/6!
  p = fmaf(p, r, 8.33333333333333333e-3f);  // 1/5!
  p = fmaf(p, r, 4.16666666666666667e-2f);  // 1/4!
  p = fmaf(p, r, 1.66666666666666667e-1f);  // 1/3!
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ki = static_cast<int>(k);
  const int k1 = ki / 2, k2 = ki - k1;
  p = __fmul_rn(p, __int_as_float((k1 + 127) << 23));
  return __fmul_rn(p, __int_as_float((k2 + 127) << 23));
}

// 1 / (1 + e^-x) with an IEEE division.
__device__ __forceinline__ float sigmoid_cw(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cw(-x))); }

__device__ __forceinline__ float warp_sum_butterfly(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// bf16x2 lanes of a 16-byte chunk.  bf16 sums and products computed in fp32 and
// rounded once equal the correctly rounded bf16 operations: a product of two
// bf16 values is exact in fp32, and a sum whose fp32 rounding is inexact has its
// addends more than 16 binades apart, which keeps it off every bf16 midpoint.
// So the packed __hadd2 / __hmul2_rn below compute bf16(a + b) and bf16(a * b)
// (the _rn multiply keeps the compiler from contracting a product and a following
// sum into one fused rounding).
__device__ __forceinline__ __nv_bfloat162 bf2(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }
__device__ __forceinline__ uint32_t u32(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ float2 f2(__nv_bfloat162 v) { return __bfloat1622float2(v); }
__device__ __forceinline__ uint32_t word(const uint4& v, int k) { return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w; }

// 1/sqrt as an IEEE square root followed by an IEEE division.
__device__ __forceinline__ float rsqrt_ieee(float x) { return __fdiv_rn(1.0f, __fsqrt_rn(x)); }

__device__ __forceinline__ float bf16_rn(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// tl.exp on fp32 as Triton compiles it: 2^(x log2 e) with the product rounded first
// and the approximate ex2 instruction.  tl.rsqrt is libdevice's rsqrtf, which Triton
// links and CUDA's rsqrtf also is (the closest match measured against the reference's
// kernels; see the producer fixtures' tests).
__device__ __forceinline__ float exp_triton(float x) {
  float r;
  asm("ex2.approx.f32 %0, %1;" : "=f"(r) : "f"(__fmul_rn(x, 1.44269504088896341f)));
  return r;
}
// tl.sigmoid(x) = 1 / (1 + exp(-x)) in fp32, the division being div.full.
__device__ __forceinline__ float sigmoid_triton(float x) { return div_full(1.0f, __fadd_rn(1.0f, exp_triton(-x))); }

// Row sum of squares the way the reference's Triton kernels reduce a bf16 row of
// H = 1024 r elements (triton_ops.py:82-83, 220-221; Triton keeps tl.sum of a bf16
// tensor in bf16).  The compiled kernel lays the row out as 4 warps x 32 lanes x 8
// contiguous values per repetition: element r*1024 + t*8 + e is register j = 8r + e
// of thread t.  Each thread sums its registers in order, every step rounded to bf16:
// the first as bf16(x*x), later ones fused (acc = fma(x, x, acc), one rounding) or as
// acc + bf16(x*x), following the fusion the compiler chose in that kernel (every
// step in the AdaLN kernel, the even ones in the residual-FMA kernel).  The 32 lanes
// of each warp then combine by an xor butterfly (16, 8, 4, 2, 1) and the four warps
// as (w0 + w2) + (w1 + w3).  Lane l here plays threads w*32 + l, w = 0..3: its load i
// (chunk 32 i + l) is repetition i/4 of thread (i%4)*32 + l.
enum SumsqFusion : int { kFuseAll = 0, kFuseEven = 1 };

template <int kFusion>
__device__ __forceinline__ void triton_sumsq_chunk(__nv_bfloat16 (&acc)[4], int i, const uint4& v) {
  const int w = i & 3, r = i >> 2;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t u = word(v, k);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_bfloat16 x = __ushort_as_bfloat16(static_cast<unsigned short>(h ? (u >> 16) : (u & 0xFFFFu)));
      const int j = r * 8 + 2 * k + h;
      if (j == 0)
        acc[w] = __hmul_rn(x, x);
      else if (kFusion == kFuseAll || (j & 1) == 0)
        acc[w] = __hfma(x, x, acc[w]);
      else
        acc[w] = __hadd_rn(acc[w], __hmul_rn(x, x));
    }
  }
}

__device__ __forceinline__ float triton_sumsq_finish(__nv_bfloat16 (&acc)[4]) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int w = 0; w < 4; ++w) acc[w] = __hadd_rn(acc[w], __shfl_xor_sync(0xffffffffu, acc[w], off));
  return __bfloat162float(__hadd_rn(__hadd_rn(acc[0], acc[2]), __hadd_rn(acc[1], acc[3])));
}

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ uint4 pack_bf16x8(const float (&f)[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

// 1x128 quantisation of the 8 values this lane holds of one group (the group's
// other 120 values are in the 15 lanes sharing this half-warp): codes to q8
// (8 bytes), the group's stored scale 1/s to *sfa by the half-warp's first lane.
template <int kMode>
__device__ __forceinline__ void quant_group8(const float (&f)[8], bool valid, uint8_t* q8, float* sfa_elem,
                                             int l16) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = (kMode == kQuantTriton) ? fmaxf(amax, fabsf(f[i])) : fmax_nan(amax, fabsf(f[i]));
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, amax, off, 16);
    amax = (kMode == kQuantTriton) ? fmaxf(amax, o) : fmax_nan(amax, o);
  }
  float s, inv;
  group_scale<kMode>(amax, s, inv);
  const bool in_range = (kMode == kQuantTriton) || isfinite(s);
  uint32_t w[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float v0 = __fmul_rn(f[4 * i], s), v1 = __fmul_rn(f[4 * i + 1], s);
    const float v2 = __fmul_rn(f[4 * i + 2], s), v3 = __fmul_rn(f[4 * i + 3], s);
    const uint16_t lo = in_range ? f32x2_to_e4m3x2_inrange(v0, v1) : f32x2_to_e4m3x2(v0, v1);
    const uint16_t hi = in_range ? f32x2_to_e4m3x2_inrange(v2, v3) : f32x2_to_e4m3x2(v2, v3);
    w[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  }
  if (valid) {
    *reinterpret_cast<uint2*>(q8) = make_uint2(w[0], w[1]);
    if (l16 == 0) *sfa_elem = inv;
  }
}


struct ProducerOut {
  uint8_t* q;      // e4m3 [M, H] or null
  float* sfa;      // sfa[kb * sfa_ld + m]
  int64_t sfa_ld;
  __nv_bfloat16* out;  // bf16 [M, H] (unquantised output) or null
};

// sum += bf16(v*v) over the 8 values of a chunk, in element order.
__device__ __forceinline__ float sumsq_chunk(float acc, const uint4& v) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __nv_bfloat162 x = bf2(word(v, k));
    const float2 sq = f2(__hmul2_rn(x, x));
    acc = __fadd_rn(acc, sq.x);
    acc = __fadd_rn(acc, sq.y);
  }
  return acc;
}

// The norm producers make two passes over a row: the first reduces the row's sum
// of squares, the second re-reads the row (an L2 hit: the warp read or wrote it
// microseconds earlier) to normalise and quantise.  Nothing of the row stays in
// registers between the passes, which keeps the register count low and lets many
// rows per SM be in flight.

// x bf16 [B*S, H]; scale/shift element (b, s, h) at p[b * bstride + s * sstride + h].
template <int kChunks, int kMode>
__global__ void __launch_bounds__(kProdWarps * 32, 8) adanorm_quant_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t M, int64_t S, int H, const __nv_bfloat16* __restrict__ scale,
    int64_t scale_bs, int64_t scale_ss, const __nv_bfloat16* __restrict__ shift, int64_t shift_bs, int64_t shift_ss,
    ProducerOut o) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, l16 = lane & 15;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kProdWarps + warp;
  if (row >= M) return;
  const int nchunks = H / 8;
  const __nv_bfloat16* xr = x + row * H;
  // mean of the bf16 squares, + eps, 1/sqrt (triton_ops.py:82-85)
  float r;
  if constexpr (kMode == kQuantTriton) {
    __nv_bfloat16 acc[4] = {};
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int c = i * 32 + lane;
      if (c < nchunks) triton_sumsq_chunk<kFuseAll>(acc, i, ldg16(xr + c * 8));
    }
    r = rsqrtf(__fadd_rn(div_full(triton_sumsq_finish(acc), static_cast<float>(H)), 1e-5f));
  } else {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int c = i * 32 + lane;
      if (c < nchunks) acc = sumsq_chunk(acc, ldg16(xr + c * 8));
    }
    r = rsqrt_ieee(__fadd_rn(__fdiv_rn(warp_sum_butterfly(acc), static_cast<float>(H)), 1e-5f));
  }
  const int64_t b = row / S, s = row - b * S;
  const __nv_bfloat16* scr = scale + b * scale_bs + s * scale_ss;
  const __nv_bfloat16* shr = shift + b * shift_bs + s * shift_ss;
  const __nv_bfloat162 one = __float2bfloat162_rn(1.0f);
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = i * 32 + lane;
    const bool valid = c < nchunks;
    if (i * 32 >= nchunks) break;  // warp-uniform: no group of this load exists
    uint4 xv = make_uint4(0, 0, 0, 0), sc = xv, sh = xv;
    if (valid) {
      xv = ldg16(xr + c * 8);
      sc = ldg16(scr + c * 8);
      sh = ldg16(shr + c * 8);
    }
    float f[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 xf = f2(bf2(word(xv, k)));
      // (x * x_norm).to(bf16), then x * (1.0 + norm_scales) + norm_shift in bf16: the
      // reference's compiled kernel fuses the last multiply-add (one rounding)
      const __nv_bfloat162 y = __float22bfloat162_rn(make_float2(__fmul_rn(xf.x, r), __fmul_rn(xf.y, r)));
      const __nv_bfloat162 t = __hadd2(one, bf2(word(sc, k)));
      const float2 z = kMode == kQuantTriton ? f2(__hfma2(y, t, bf2(word(sh, k))))
                                             : f2(__hadd2(__hmul2_rn(y, t), bf2(word(sh, k))));
      f[2 * k] = z.x;
      f[2 * k + 1] = z.y;
    }
    quant_group8<kMode>(f, valid, o.q + row * H + c * 8, o.sfa + static_cast<int64_t>(c / 16) * o.sfa_ld + row, l16);
  }
}

// x, y bf16 [B*S, H]; z (b, s, h) at z[b * bstride + s * sstride + h].
// x <- bf16(x + bf16(y z)); o = x * rsqrt(mean(bf16(x^2))) in fp32; quantised
// (o.q) or rounded to bf16 (o.out).  The second pass reads back the updated x
// (this thread's own stores, through the coherent path).
template <int kChunks, int kMode, bool kQuant>
__global__ void __launch_bounds__(kProdWarps * 32, 8) rms_fma_kernel(__nv_bfloat16* __restrict__ x,
                                                                   const __nv_bfloat16* __restrict__ y, int64_t M,
                                                                   int64_t S, int H,
                                                                   const __nv_bfloat16* __restrict__ z, int64_t z_bs,
                                                                   int64_t z_ss, ProducerOut o) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, l16 = lane & 15;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kProdWarps + warp;
  if (row >= M) return;
  const int nchunks = H / 8;
  __nv_bfloat16* xr = x + row * H;
  const __nv_bfloat16* yr = y + row * H;
  const int64_t b = row / S, s = row - b * S;
  const __nv_bfloat16* zr = z + b * z_bs + s * z_ss;
  float acc = 0.0f;
  __nv_bfloat16 tacc[4] = {};
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = i * 32 + lane;
    if (c < nchunks) {
      const uint4 xv = *reinterpret_cast<const uint4*>(xr + c * 8);
      const uint4 yv = ldg16(yr + c * 8), zv = ldg16(zr + c * 8);
      uint4 ov;
      if constexpr (kMode == kQuantTriton) {
        // x + y * z in bf16, fused by the reference's compiled kernel (one rounding)
        ov = make_uint4(u32(__hfma2(bf2(yv.x), bf2(zv.x), bf2(xv.x))), u32(__hfma2(bf2(yv.y), bf2(zv.y), bf2(xv.y))),
                        u32(__hfma2(bf2(yv.z), bf2(zv.z), bf2(xv.z))), u32(__hfma2(bf2(yv.w), bf2(zv.w), bf2(xv.w))));
        triton_sumsq_chunk<kFuseEven>(tacc, i, ov);
      } else {
        // bf16(x + bf16(y * z))
        ov = make_uint4(u32(__hadd2(bf2(xv.x), __hmul2_rn(bf2(yv.x), bf2(zv.x)))),
                        u32(__hadd2(bf2(xv.y), __hmul2_rn(bf2(yv.y), bf2(zv.y)))),
                        u32(__hadd2(bf2(xv.z), __hmul2_rn(bf2(yv.z), bf2(zv.z)))),
                        u32(__hadd2(bf2(xv.w), __hmul2_rn(bf2(yv.w), bf2(zv.w)))));
        acc = sumsq_chunk(acc, ov);
      }
      *reinterpret_cast<uint4*>(xr + c * 8) = ov;  // residual stream updated in place
    }
  }
  // no epsilon (triton_ops.py:222-224)
  const float r = kMode == kQuantTriton
                      ? rsqrtf(div_full(triton_sumsq_finish(tacc), static_cast<float>(H)))
                      : rsqrt_ieee(__fdiv_rn(warp_sum_butterfly(acc), static_cast<float>(H)));
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = i * 32 + lane;
    const bool valid = c < nchunks;
    if (i * 32 >= nchunks) break;
    float f[8];
    bf16x8_to_f32(valid ? *reinterpret_cast<const uint4*>(xr + c * 8) : make_uint4(0, 0, 0, 0), f);
#pragma unroll
    for (int k = 0; k < 8; ++k) f[k] = __fmul_rn(f[k], r);
    if constexpr (kQuant) {
      quant_group8<kMode>(f, valid, o.q + row * H + c * 8, o.sfa + static_cast<int64_t>(c / 16) * o.sfa_ld + row,
                          l16);
    } else {
      if (valid) *reinterpret_cast<uint4*>(o.out + row * H + c * 8) = pack_bf16x8(f);
    }
  }
}

// x bf16 [M, H] viewed as [heads, H/heads]; gate_logits [M, heads] (bf16 or fp32);
// o = x * 2 sigmoid(logit) in fp32, quantised or rounded to bf16.
template <int kChunks, int kMode, bool kQuant, bool kGateF32>
__global__ void __launch_bounds__(kProdWarps * 32, 8) gated_attention_kernel(const __nv_bfloat16* __restrict__ x,
                                                                        const void* __restrict__ gate_logits,
                                                                        int64_t M, int H, int heads, ProducerOut o) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, l16 = lane & 15;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kProdWarps + warp;
  if (row >= M) return;
  const int nchunks = H / 8;
  const int dim_head = H / heads;
  const __nv_bfloat16* xr = x + row * H;
  // 2 sigmoid(logit) of heads `lane` and `lane + 32` (heads <= 64), broadcast below.
  float gate_lo = 0.0f, gate_hi = 0.0f;
#pragma unroll
  for (int part = 0; part < 2; ++part) {
    const int h = lane + 32 * part;
    if (h < heads) {
      float g;
      if constexpr (kGateF32) {
        g = __ldg(static_cast<const float*>(gate_logits) + row * heads + h);
      } else {
        g = __bfloat162float(static_cast<const __nv_bfloat16*>(gate_logits)[row * heads + h]);
      }
      const float gate = __fmul_rn(2.0f, kMode == kQuantTriton ? sigmoid_triton(g) : sigmoid_cw(g));
      if (part == 0) gate_lo = gate; else gate_hi = gate;
    }
  }
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = i * 32 + lane;
    const bool valid = c < nchunks;
    if (i * 32 >= nchunks) break;
    float f[8];
    bf16x8_to_f32(valid ? ldg16(xr + c * 8) : make_uint4(0, 0, 0, 0), f);
    // dim_head % 8 == 0: a chunk lies within one head
    const int head = valid ? (c * 8) / dim_head : 0;
    const float glo = __shfl_sync(0xffffffffu, gate_lo, head & 31);
    const float ghi = __shfl_sync(0xffffffffu, gate_hi, head & 31);
    const float gate = head < 32 ? glo : ghi;
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = __fmul_rn(f[j], gate);
    if constexpr (kQuant) {
      quant_group8<kMode>(f, valid, o.q + row * H + c * 8, o.sfa + static_cast<int64_t>(c / 16) * o.sfa_ld + row,
                          l16);
    } else {
      if (valid) *reinterpret_cast<uint4*>(o.out + row * H + c * 8) = pack_bf16x8(f);
    }
  }
}

// x bf16 [M, K] (row stride x_ld) -> gelu(x) = x sigmoid(1.702 x) in fp32 -> quant.
// Half-warp per 1x128 group as in quant_act_1x128_kernel.
template <int kMode>
__global__ void __launch_bounds__(256) gelu_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_ld, int64_t M,
                                                         int64_t KB, uint8_t* __restrict__ q, int64_t q_ld,
                                                         float* __restrict__ sfa, int64_t sfa_ld) {
  const int t = threadIdx.x;
  const int l16 = t & 15;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kQuantRowsPerBlock + (t >> 4);
  const int64_t kb0 = static_cast<int64_t>(blockIdx.y) * kQuantGroupsPerThread;
  const bool row_ok = row < M;
  uint4 v[kQuantGroupsPerThread];
#pragma unroll
  for (int u = 0; u < kQuantGroupsPerThread; ++u) {
    const int64_t kb = kb0 + u;
    v[u] = (row_ok && kb < KB) ? ldg16(x + row * x_ld + kb * 128 + l16 * 8) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int u = 0; u < kQuantGroupsPerThread; ++u) {
    const int64_t kb = kb0 + u;
    float f[8];
    bf16x8_to_f32(v[u], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float a = __fmul_rn(1.702f, f[j]);
      f[j] = __fmul_rn(f[j], kMode == kQuantTriton ? sigmoid_triton(a) : sigmoid_cw(a));
    }
    const bool valid = row_ok && kb < KB;
    quant_group8<kMode>(f, valid, q + row * q_ld + kb * 128 + l16 * 8, sfa + kb * sfa_ld + row, l16);
  }
}

// ---------------------------------------------------------------------------
// RMSNorm + RoPE for the attention q/k (ltx-kernels/csrc/ops/rms_norm_rope_cuda.cu,
// rms_norm_split_rope_cuda.cu).  Row sums of x^2 in fp32 with fused multiply-adds in
// the lanes' chunk order, then the xor butterfly; 1/sqrt as IEEE sqrt + division.

enum RopeOut : int {
  kRopeBf16 = 0,       // bf16, round to nearest even
  kRopeE4m3Torch = 1,  // e4m3 with torch's conversion (overflow -> NaN): c10::Float8_e4m3fn(float)
  kRopeE4m3Sat = 2,    // e4m3, saturating: __nv_fp8_e4m3(float)
};

template <int kOut>
__device__ __forceinline__ void rope_store8(void* out, int64_t elem, const float (&v)[8]) {
  if constexpr (kOut == kRopeBf16) {
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + elem) = pack_bf16x8(v);
  } else {
    uint32_t w[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint16_t lo = kOut == kRopeE4m3Torch ? f32x2_to_e4m3x2(v[4 * i], v[4 * i + 1])
                                                 : f32x2_to_e4m3x2_inrange(v[4 * i], v[4 * i + 1]);
      const uint16_t hi = kOut == kRopeE4m3Torch ? f32x2_to_e4m3x2(v[4 * i + 2], v[4 * i + 3])
                                                 : f32x2_to_e4m3x2_inrange(v[4 * i + 2], v[4 * i + 3]);
      w[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
    *reinterpret_cast<uint2*>(static_cast<uint8_t*>(out) + elem) = make_uint2(w[0], w[1]);
  }
}

// fp32 sum of x^2 over this lane's chunks of a bf16 row (fused multiply-adds in element order).
template <int kChunks>
__device__ __forceinline__ float lane_sumsq_f32(const __nv_bfloat16* xr, int lane, int nchunks) {
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = i * 32 + lane;
    if (c < nchunks) {
      float f[8];
      bf16x8_to_f32(ldg16(xr + c * 8), f);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc = fmaf(f[k], f[k], acc);
    }
  }
  return acc;
}

// Interleaved RoPE: x bf16 [rows, dim]; cos/sin bf16 with row r at p + r * f_rs;
// w bf16 [dim] or null.  v = x * (rsqrt(sum(x^2) * (1/dim)) [* w]) (no epsilon,
// rms_norm_rope_cuda.cu:125-150); pairs (2i, 2i+1):
//   out[2i]   = v[2i] cos[2i] - v[2i+1] sin[2i]      (:160-170)
//   out[2i+1] = v[2i+1] cos[2i+1] + v[2i] sin[2i+1]
template <int kChunks, bool kAffine, int kOut>
__global__ void __launch_bounds__(kProdWarps * 32, 4) rms_norm_rope_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t rows, int dim, const __nv_bfloat16* __restrict__ cosf,
    const __nv_bfloat16* __restrict__ sinf, int64_t f_rs, const __nv_bfloat16* __restrict__ w, void* __restrict__ out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kProdWarps + warp;
  if (row >= rows) return;
  const int nchunks = dim / 8;
  const __nv_bfloat16* xr = x + row * dim;
  const float ss = warp_sum_butterfly(lane_sumsq_f32<kChunks>(xr, lane, nchunks));
  const float n = rsqrt_ieee(__fmul_rn(ss, __frcp_rn(static_cast<float>(dim))));
  const __nv_bfloat16* cr = cosf + row * f_rs;
  const __nv_bfloat16* sr = sinf + row * f_rs;
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = i * 32 + lane;
    if (c < nchunks) {
      float v[8], cs[8], sn[8], o[8];
      bf16x8_to_f32(ldg16(xr + c * 8), v);
      bf16x8_to_f32(ldg16(cr + c * 8), cs);
      bf16x8_to_f32(ldg16(sr + c * 8), sn);
      if constexpr (kAffine) {
        float wv[8];
        bf16x8_to_f32(ldg16(w + c * 8), wv);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = __fmul_rn(v[k], __fmul_rn(n, wv[k]));
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = __fmul_rn(v[k], n);
      }
#pragma unroll
      for (int k = 0; k < 8; k += 2) {
        o[k] = fmaf(v[k], cs[k], -__fmul_rn(v[k + 1], sn[k]));
        o[k + 1] = fmaf(v[k + 1], cs[k + 1], __fmul_rn(v[k], sn[k + 1]));
      }
      rope_store8<kOut>(out, row * dim + c * 8, o);
    }
  }
}

// Split RoPE: x bf16 [B, S, H] as heads of d = H / heads values, each head as two
// halves (first, second) of d/2; cos/sin [B or 1, heads, S, d/2] by strides
// (sb, sn, ss), inner stride 1.  v = (x * rsqrt(sum(x^2) / H + 1e-6)) [* w]
// (rms_norm_split_rope_cuda.cu:73-105), then
//   first[j]  = cos[j] first[j] - sin[j] second[j]
//   second[j] = cos[j] second[j] + sin[j] first[j]     (:107-140)
// d/16 (the chunk distance between the halves) is a power of two <= 16, so the
// partner chunk sits in lane ^ (d/16) of the same load.
template <int kChunks, bool kAffine, int kOut>
__global__ void __launch_bounds__(kProdWarps * 32, 4) rms_norm_split_rope_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t B, int64_t S, int H, int heads,
    const __nv_bfloat16* __restrict__ cosf, int64_t c_sb, int64_t c_sn, int64_t c_ss,
    const __nv_bfloat16* __restrict__ sinf, int64_t s_sb, int64_t s_sn, int64_t s_ss,
    const __nv_bfloat16* __restrict__ w, void* __restrict__ out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kProdWarps + warp;
  if (row >= B * S) return;
  const int nchunks = H / 8;
  const int d = H / heads, half = d / 2, partner = d / 16;
  const __nv_bfloat16* xr = x + row * H;
  const float ss = warp_sum_butterfly(lane_sumsq_f32<kChunks>(xr, lane, nchunks));
  const float r = rsqrt_ieee(__fadd_rn(__fdiv_rn(ss, static_cast<float>(H)), 1e-6f));
  const int64_t bi = row / S, si = row - bi * S;
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    if (i * 32 >= nchunks) break;  // warp-uniform
    const int c = i * 32 + lane;
    const bool valid = c < nchunks;
    float v[8];
    bf16x8_to_f32(valid ? ldg16(xr + c * 8) : make_uint4(0, 0, 0, 0), v);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = __fmul_rn(v[k], r);
    if constexpr (kAffine) {
      float wv[8];
      bf16x8_to_f32(valid ? ldg16(w + c * 8) : make_uint4(0, 0, 0, 0), wv);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = __fmul_rn(v[k], wv[k]);
    }
    float other[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) other[k] = __shfl_xor_sync(0xffffffffu, v[k], partner);
    if (valid) {
      const int e = c * 8, hd = e / d, p = e - hd * d;
      const bool first = p < half;
      const int j = first ? p : p - half;
      float cs[8], sn[8], o[8];
      bf16x8_to_f32(ldg16(cosf + bi * c_sb + hd * c_sn + si * c_ss + j), cs);
      bf16x8_to_f32(ldg16(sinf + bi * s_sb + hd * s_sn + si * s_ss + j), sn);
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = fmaf(first ? -sn[k] : sn[k], other[k], __fmul_rn(cs[k], v[k]));
      rope_store8<kOut>(out, row * H + e, o);
    }
  }
}

}  // namespace ltxfp8
