// Quantisation kernels: per-token 1x128 activation quant, 128x128 weight quant,
// and the 1x128 dequantiser.  All three are HBM-bound streaming kernels.
#pragma once

#include "gelu.cuh"
#include "ptx.cuh"

namespace ltxfp8 {

// Activation-quant modes.
enum QuantMode : int {
  kQuantTorch = 0,   // s = (1/amax)*448 with IEEE roundings, NaN-propagating amax (functional.py:138-144)
  kQuantTriton = 1,  // s = 448/amax and 1/s via div.full.f32, NaN-ignoring amax (triton_ops.py:13-22)
};

constexpr int kQuantRowsPerBlock = 16;   // 16 lanes per 128-group, 16 groups per 256-thread block
constexpr int kQuantGroupsPerThread = 4; // groups in flight per thread (4 x 16 B loads)


// Scale pair for one group from its abs-max.
template <int kMode>
__device__ __forceinline__ void group_scale(float amax, float& s, float& inv) {
  if constexpr (kMode == kQuantTriton) {
    s = div_full(448.0f, amax);
    inv = div_full(1.0f, s);
  } else {
    s = __fmul_rn(__frcp_rn(amax), 448.0f);
    inv = __frcp_rn(s);
  }
}

// x: bf16 [M, K] (row stride x_ld elements) -> q: e4m3 [M, K] (row stride q_ld),
// sfa[kb * sfa_ld + m] = 1 / s.  Block = 16 rows x kQuantGroupsPerThread groups;
// each half-warp owns one row-group of 128 values (8 per lane, one 16 B load).
// Replaces _block_quant_kernel (ltx-kernels/src/ltx_kernels/blockwise/triton_ops.py:102-126).
template <int kMode>
__global__ void __launch_bounds__(256) quant_act_1x128_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_ld,
                                                              int64_t M, int64_t KB, uint8_t* __restrict__ q,
                                                              int64_t q_ld, float* __restrict__ sfa,
                                                              int64_t sfa_ld) {
  const int t = threadIdx.x;
  const int l16 = t & 15;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kQuantRowsPerBlock + (t >> 4);
  const int64_t kb0 = static_cast<int64_t>(blockIdx.y) * kQuantGroupsPerThread;
  const bool row_ok = row < M;

  uint4 v[kQuantGroupsPerThread];
#pragma unroll
  for (int u = 0; u < kQuantGroupsPerThread; ++u) {
    const int64_t kb = kb0 + u;
    if (row_ok && kb < KB) {
      v[u] = __ldg(reinterpret_cast<const uint4*>(x + row * x_ld + kb * 128 + l16 * 8));
    } else {
      v[u] = make_uint4(0, 0, 0, 0);
    }
  }

#pragma unroll
  for (int u = 0; u < kQuantGroupsPerThread; ++u) {
    const int64_t kb = kb0 + u;
    float f[8];
    bf16x8_to_f32(v[u], f);
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
    // A finite scale keeps every |x * s| <= 448, where the saturating hardware
    // conversion equals torch's; only non-finite scales need torch's overflow-to-NaN
    // patch.  The Triton kernel converts with the saturating instruction throughout.
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
    if (row_ok && kb < KB) {
      *reinterpret_cast<uint2*>(q + row * q_ld + kb * 128 + l16 * 8) = make_uint2(w[0], w[1]);
      if (l16 == 0) sfa[kb * sfa_ld + row] = inv;
    }
  }
}

// torch's GELU-tanh, then the 1x128 quantiser: the reference FFN's unfused chain
// h = F.gelu(linear1(x), approximate="tanh") (bf16) followed by blockwise::quantize
// (ltx-core/src/ltx_core/model/transformer/gelu_approx.py:10, ltx-kernels/.../linear.py:91-93),
// from the up projection's bf16 output.  Codes and scales equal quant_act_1x128_kernel
// applied to torch's bf16 GELU output.  A persistent grid: every CTA fills the 10.5 KB
// GELU table once, then walks units of 16 rows x kQuantGroupsPerThread groups, groups
// fastest (consecutive CTAs read consecutive bytes of the same rows).
constexpr int kGeluQuantGroups = 4;  // 1x128 groups per thread and unit

template <int kMode>
__global__ void __launch_bounds__(256) gelu_tanh_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_ld,
                                                              int64_t M, int64_t KB, uint8_t* __restrict__ q,
                                                              int64_t q_ld, float* __restrict__ sfa,
                                                              int64_t sfa_ld) {
  __shared__ __align__(16) uint16_t tab[2 * kGeluTabWindow];
  gelu_table_fill(tab, static_cast<int>(threadIdx.x), 256);
  __syncthreads();
  const int t = threadIdx.x;
  const int l16 = t & 15;
  const int64_t row_blocks = (M + kQuantRowsPerBlock - 1) / kQuantRowsPerBlock;
  const int64_t kb_blocks = (KB + kGeluQuantGroups - 1) / kGeluQuantGroups;
  const int64_t units = row_blocks * kb_blocks;
  for (int64_t unit = blockIdx.x; unit < units; unit += gridDim.x) {
    const int64_t rb = unit / kb_blocks, kbb = unit - rb * kb_blocks;
    const int64_t row = rb * kQuantRowsPerBlock + (t >> 4);
    const int64_t kb0 = kbb * kGeluQuantGroups;
    const bool row_ok = row < M;
    uint4 v[kGeluQuantGroups];
#pragma unroll
    for (int u = 0; u < kGeluQuantGroups; ++u) {
      const int64_t kb = kb0 + u;
      v[u] = (row_ok && kb < KB) ? __ldg(reinterpret_cast<const uint4*>(x + row * x_ld + kb * 128 + l16 * 8))
                                 : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kGeluQuantGroups; ++u) {
      const int64_t kb = kb0 + u;
      const uint4 g = gelu_bf16x8(v[u], smem_u32(tab));
      float f[8];
      bf16x8_to_f32(g, f);
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
      if (row_ok && kb < KB) {
        *reinterpret_cast<uint2*>(q + row * q_ld + kb * 128 + l16 * 8) = make_uint2(w[0], w[1]);
        if (l16 == 0) sfa[kb * sfa_ld + row] = inv;
      }
    }
  }
}

// Second half of the 128x128 block quantiser: each of the 256 threads holds 64
// consecutive values f of one row of the block.  Block abs-max (NaN-propagating,
// as torch's abs().max()), s = (1/amax)*scale_max, codes e4m3(f*s) with torch's
// conversion to `qrow` (this thread's 64 bytes), scale 1/s to *scale by thread 0.
__device__ __forceinline__ void quant_block_128x128_store(const float (&f)[64], float* red, uint8_t* qrow,
                                                          float* scale, float scale_max = 448.0f) {
  const int t = threadIdx.x;
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 64; ++i) amax = fmax_nan(amax, fabsf(f[i]));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmax_nan(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if ((t & 31) == 0) red[t >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmax_nan(amax, red[i]);
  const float s = __fmul_rn(__frcp_rn(amax), scale_max);
  uint32_t words[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint16_t lo = f32x2_to_e4m3x2(__fmul_rn(f[4 * i], s), __fmul_rn(f[4 * i + 1], s));
    const uint16_t hi = f32x2_to_e4m3x2(__fmul_rn(f[4 * i + 2], s), __fmul_rn(f[4 * i + 3], s));
    words[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  }
  uint4* dst = reinterpret_cast<uint4*>(qrow);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_uint4(words[4 * i], words[4 * i + 1], words[4 * i + 2], words[4 * i + 3]);
  if (t == 0) *scale = __frcp_rn(s);
}

// Weight quant over 128x128 blocks: one block of 256 threads per (kb, nb); each
// thread owns 64 consecutive values of one row.  s = (1/amax)*448, scale = 1/s
// (ltx-kernels/src/ltx_kernels/blockwise/functional.py:128-135).
// in_dtype: 0 = fp32, 1 = bf16, 2 = fp16.
__global__ void __launch_bounds__(256) quant_weight_128x128_kernel(const void* __restrict__ w, int in_dtype, int64_t K,
                                                                   int64_t KB, uint8_t* __restrict__ q,
                                                                   float* __restrict__ sfb, float scale_max) {
  __shared__ float red[8];
  const int t = threadIdx.x;
  const int64_t kb = blockIdx.x, nb = blockIdx.y;
  const int64_t r = nb * 128 + (t >> 1);
  const int64_t c0 = kb * 128 + (t & 1) * 64;
  float f[64];
  if (in_dtype == 0) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(w) + r * K + c0);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 a = __ldg(p + i);
      f[4 * i] = a.x; f[4 * i + 1] = a.y; f[4 * i + 2] = a.z; f[4 * i + 3] = a.w;
    }
  } else if (in_dtype == 1) {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(w) + r * K + c0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float g[8];
      bf16x8_to_f32(__ldg(p + i), g);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[8 * i + j] = g[j];
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __half*>(w) + r * K + c0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 a = __ldg(p + i);
      const uint32_t ww[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half2 h = *reinterpret_cast<const __half2*>(&ww[j]);
        const float2 g = __half22float2(h);
        f[8 * i + 2 * j] = g.x;
        f[8 * i + 2 * j + 1] = g.y;
      }
    }
  }
  quant_block_128x128_store(f, red, q + r * K + c0, sfb + nb * KB + kb, scale_max);
}

// Dequant: out[m, k] = bf16(float(q[m, k]) * scales[m * rs + (k / 128) * cs]).
// Each thread converts 16 codes (one 16 B load, two 16 B stores).
// Replaces _blockwise_dequantize_kernel (ltx-kernels/src/ltx_kernels/blockwise/triton_ops.py:387-411).
__global__ void __launch_bounds__(256) dequant_1x128_kernel(const uint8_t* __restrict__ q, const float* __restrict__ sc,
                                                            int64_t rs, int64_t cs, int64_t M, int64_t K,
                                                            __nv_bfloat16* __restrict__ out) {
  const int64_t chunks_per_row = K / 16;
  const int64_t total = M * chunks_per_row;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = c / chunks_per_row;
    const int64_t k0 = (c - m * chunks_per_row) * 16;
    const float s = __ldg(sc + m * rs + (k0 / 128) * cs);
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(q + m * K + k0));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_fp8x2_storage_t lo = static_cast<__nv_fp8x2_storage_t>(w[i] & 0xFFFFu);
      const __nv_fp8x2_storage_t hi = static_cast<__nv_fp8x2_storage_t>(w[i] >> 16);
      const float2 a = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(lo, __NV_E4M3)));
      const float2 b = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(hi, __NV_E4M3)));
      o[2 * i] = pack_bf16x2(__fmul_rn(a.x, s), __fmul_rn(a.y, s));
      o[2 * i + 1] = pack_bf16x2(__fmul_rn(b.x, s), __fmul_rn(b.y, s));
    }
    uint4* dst = reinterpret_cast<uint4*>(out + m * K + k0);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// Load-time LoRA merge into a blockwise-FP8 weight, one 256-thread block per
// 128x128 block (thread: 64 consecutive values of one row):
//   w  = bf16(float(code) * scale)        the 2-D dequantisation (_impl.py:263-274)
//   w' = bf16(w + delta)                   merged = bf16_weight + deltas (_impl.py:296)
//   (q', scale') = 128x128 quant of w'     fp8_blockwise_quantize_weights_torch (_impl.py:297)
// q/sfb may alias q_out/sfb_out (each block reads its inputs before writing).
__global__ void __launch_bounds__(256) lora_fuse_weight_kernel(const uint8_t* q, const float* sfb,
                                                               const __nv_bfloat16* __restrict__ delta, int64_t K,
                                                               int64_t KB, uint8_t* q_out, float* sfb_out) {
  __shared__ float red[8];
  const int t = threadIdx.x;
  const int64_t kb = blockIdx.x, nb = blockIdx.y;
  const int64_t r = nb * 128 + (t >> 1);
  const int64_t c0 = kb * 128 + (t & 1) * 64;
  const float s = sfb[nb * KB + kb];
  float f[64];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 v = *reinterpret_cast<const uint4*>(q + r * K + c0 + 16 * i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 a = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(
          static_cast<__nv_fp8x2_storage_t>(w[j] & 0xFFFFu), __NV_E4M3)));
      const float2 b = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(
          static_cast<__nv_fp8x2_storage_t>(w[j] >> 16), __NV_E4M3)));
      f[16 * i + 4 * j] = a.x;
      f[16 * i + 4 * j + 1] = a.y;
      f[16 * i + 4 * j + 2] = b.x;
      f[16 * i + 4 * j + 3] = b.y;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float dl[8];
    bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(delta + r * K + c0 + 8 * i)), dl);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[8 * i + j] = bf16_round(__fadd_rn(bf16_round(__fmul_rn(f[8 * i + j], s)), dl[j]));
  }
  __syncthreads();  // every thread of the block has read its codes and the block scale
  quant_block_128x128_store(f, red, q_out + r * K + c0, sfb_out + nb * KB + kb);
}

// FP6 packing (ltx-kernels/csrc/ops/fp6_pack.cu:8-41,90-112): an e4m3 code whose
// two top exponent bits are zero keeps its sign (bit 7) and bits 4..0 as a 6-bit
// value; four values v0..v3 fill 3 bytes most-significant first
// (v0 << 18 | v1 << 12 | v2 << 6 | v3, high byte first).  Unpacking restores the
// two dropped bits as zero.  One thread per 8 codes <-> 6 packed bytes.
__global__ void __launch_bounds__(256) fp6_pack_kernel(const uint8_t* __restrict__ x, int64_t groups,
                                                       uint8_t* __restrict__ out) {
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(x + g * 8));
    uint32_t p[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t w = h == 0 ? v.x : v.y;
      uint32_t acc = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t b = (w >> (8 * i)) & 0xFFu;
        acc = (acc << 6) | ((b & 0x80u) >> 2) | (b & 0x1Fu);
      }
      p[h] = acc;  // 24 bits, v0 in the top six
    }
    const uint8_t bytes[6] = {static_cast<uint8_t>(p[0] >> 16), static_cast<uint8_t>(p[0] >> 8),
                              static_cast<uint8_t>(p[0]), static_cast<uint8_t>(p[1] >> 16),
                              static_cast<uint8_t>(p[1] >> 8), static_cast<uint8_t>(p[1])};
    uint16_t* o = reinterpret_cast<uint16_t*>(out + g * 6);
#pragma unroll
    for (int i = 0; i < 3; ++i) o[i] = static_cast<uint16_t>(bytes[2 * i] | (bytes[2 * i + 1] << 8));
  }
}

__global__ void __launch_bounds__(256) fp6_unpack_kernel(const uint8_t* __restrict__ x, int64_t groups,
                                                         uint8_t* __restrict__ out) {
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint16_t* in = reinterpret_cast<const uint16_t*>(x + g * 6);
    uint8_t bytes[6];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const uint16_t u = __ldg(in + i);
      bytes[2 * i] = static_cast<uint8_t>(u & 0xFFu);
      bytes[2 * i + 1] = static_cast<uint8_t>(u >> 8);
    }
    uint32_t w[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t p = (static_cast<uint32_t>(bytes[3 * h]) << 16) | (static_cast<uint32_t>(bytes[3 * h + 1]) << 8) |
                         bytes[3 * h + 2];
      uint32_t word = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t v6 = (p >> (18 - 6 * i)) & 0x3Fu;
        word |= (((v6 & 0x20u) << 2) | (v6 & 0x1Fu)) << (8 * i);
      }
      w[h] = word;
    }
    *reinterpret_cast<uint2*>(out + g * 8) = make_uint2(w[0], w[1]);
  }
}

// Packed FP6 weight -> the tensor core's 6-bit order, and its scales -> x 2^-6.
// A 6-bit code (s, e1, e0, m2, m1, m0) of the packing above is, read as e2m3
// (bias 1), 2^6 times the e4m3 value it stands for (bias 7, top exponent bits 0;
// subnormals alike), so codes read as e2m3 with scales x 2^-6 give the same
// products.  The layout: every 16 codes of a row fill 12 bytes, code i at bits
// 6i .. 6i+5 of their little-endian 96-bit word (the packing above fills 3 bytes
// per 4 codes most-significant first).  One thread per 16 codes.
__global__ void __launch_bounds__(256) fp6_to_tc_kernel(const uint8_t* __restrict__ x, int64_t chunks,
                                                        uint8_t* __restrict__ out, const float* __restrict__ sfb,
                                                        int64_t n_scales, float* __restrict__ sfb_out) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int64_t c = tid; c < chunks; c += stride) {
    const uint32_t* in = reinterpret_cast<const uint32_t*>(x + c * 12);
    const uint32_t i0 = __ldg(in), i1 = __ldg(in + 1), i2 = __ldg(in + 2);
    uint8_t b[12];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      b[k] = static_cast<uint8_t>(i0 >> (8 * k));
      b[4 + k] = static_cast<uint8_t>(i1 >> (8 * k));
      b[8 + k] = static_cast<uint8_t>(i2 >> (8 * k));
    }
    uint64_t lo = 0, hi = 0;  // bits 0-63 and 64-95 of the output word
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint32_t p = (static_cast<uint32_t>(b[3 * g]) << 16) | (static_cast<uint32_t>(b[3 * g + 1]) << 8) | b[3 * g + 2];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint64_t v6 = (p >> (18 - 6 * i)) & 0x3Fu;
        const int bit = 6 * (4 * g + i);
        if (bit + 6 <= 64) {
          lo |= v6 << bit;
        } else if (bit >= 64) {
          hi |= v6 << (bit - 64);
        } else {
          lo |= v6 << bit;
          hi |= v6 >> (64 - bit);
        }
      }
    }
    uint32_t* o = reinterpret_cast<uint32_t*>(out + c * 12);
    o[0] = static_cast<uint32_t>(lo);
    o[1] = static_cast<uint32_t>(lo >> 32);
    o[2] = static_cast<uint32_t>(hi);
  }
  for (int64_t i = tid; i < n_scales; i += stride) sfb_out[i] = sfb[i] * 0.015625f;
}

}  // namespace ltxfp8
