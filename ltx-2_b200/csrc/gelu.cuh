// torch's GELU-tanh on bf16 values through a small shared-memory table (sm_100a).
#pragma once

#include "ptx.cuh"

namespace ltxfp8 {

// torch's GELU-tanh of a bf16 input, rounded to bf16: the bf16 result of
// F.gelu(x, approximate="tanh") on a bf16 tensor (GELU's input in the GEMM epilogue is
// the bf16 value bf16(acc + bias)).  Only inputs with a biased exponent in
// [kGeluTabExpLo, kGeluTabExpHi] (|x| in [2^-16, 32)) are looked up: a table of those
// 21 x 128 x 2 results (10.5 KB), entry (mantissa-and-exponent index i, sign s) at
// 2 i + s, filled in shared memory by every CTA at start with one gelu_tanh_torch per
// entry.  Outside the window torch's result has a closed form in bf16, checked on all
// 65536 inputs:
//   |x| < 2^-16      tanhf(u) = u and 1 + u rounds to 1, so the result is bf16(0.5 x):
//                    the exponent minus one, or a halved subnormal rounded to even;
//   x >= 32          tanhf(u) = 1: the result is x;
//   x <= -32         1 + tanhf(u) = 0: the result is -0.0;
//   +inf -> +inf, -inf and NaN -> the canonical NaN.
constexpr uint32_t kGeluTabExpLo = 111, kGeluTabExpHi = 131;
constexpr uint32_t kGeluTabWindow = (kGeluTabExpHi - kGeluTabExpLo + 1) * 128;  // entries per sign
constexpr uint32_t kGeluTabBytes = 2 * kGeluTabWindow * 2;                      // 10.5 KB

__device__ __forceinline__ void gelu_table_fill(uint16_t* tab, int tid, int nthreads) {
  for (int i = tid; i < static_cast<int>(2 * kGeluTabWindow); i += nthreads) {
    const uint32_t neg = static_cast<uint32_t>(i) & 1u, idx = static_cast<uint32_t>(i) >> 1;
    const uint32_t h = (neg << 15) | ((kGeluTabExpLo << 7) + idx);
    tab[i] = __bfloat16_as_ushort(__float2bfloat16_rn(gelu_tanh_torch(__uint_as_float(h << 16))));
  }
}

__device__ __forceinline__ uint32_t gelu_lds_u16(uint32_t addr) {
  uint16_t t;
  asm("ld.shared.u16 %0, [%1];" : "=h"(t) : "r"(addr));
  return t;
}

// Any input: the table entry is read at a clamped index and the closed forms are
// selected around it (no branches).
__device__ __forceinline__ uint32_t gelu_bf16_lookup(uint32_t tab_smem, uint32_t h) {
  const uint32_t mag = h & 0x7FFFu, neg = h >> 15;
  const uint32_t idx = mag - (kGeluTabExpLo << 7);
  const bool in = idx < kGeluTabWindow;
  const uint32_t t = gelu_lds_u16(tab_smem + (in ? (idx << 2) | (neg << 1) : 0u));
  const uint32_t half = mag >= 0x100u ? h - 0x80u                                        // exponent - 1
                                      : (neg << 15) | ((mag >> 1) + (mag & (mag >> 1) & 1u));  // halved subnormal
  const uint32_t big = mag < 0x7F80u ? (neg ? 0x8000u : h) : (h == 0x7F80u ? 0x7F80u : 0x7FFFu);
  return in ? t : (mag < (kGeluTabExpLo << 7) ? half : big);
}

// torch's GELU of 8 packed bf16 values.  Warp-collective (all 32 lanes): when every
// lane's 8 inputs lie in the table's window, as activations almost always do, each
// result is one shared-memory load at a computed offset; otherwise the general form.
__device__ __forceinline__ uint4 gelu_bf16x8(const uint4& v, uint32_t tab_smem) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t off[8];
  bool out = false;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const uint32_t h = (w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
    const uint32_t idx = (h & 0x7FFFu) - (kGeluTabExpLo << 7);
    out |= idx >= kGeluTabWindow;
    off[e] = (idx << 2) | ((h >> 14) & 2u);
  }
  uint32_t r[4];
  if (!__any_sync(0xffffffffu, out)) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      r[i] = gelu_lds_u16(tab_smem + off[2 * i]) | (gelu_lds_u16(tab_smem + off[2 * i + 1]) << 16);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      r[i] = gelu_bf16_lookup(tab_smem, w[i] & 0xFFFFu) | (gelu_bf16_lookup(tab_smem, w[i] >> 16) << 16);
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// GELU of 8 packed bf16 values, in place: torch's formula through the table, or the
// fast form x / (1 + 2^a) (within one bf16 ulp), chosen per launch (warp-uniform).
__device__ __forceinline__ void gelu_bf16x8_inplace(uint32_t (&w4)[4], bool fast, const uint16_t* tab) {
  if (fast) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 y = gelu_tanh_f32x2(make_float2(__uint_as_float(w4[i] << 16), __uint_as_float(w4[i] & 0xFFFF0000u)));
      w4[i] = pack_bf16x2(y.x, y.y);
    }
  } else {
    const uint4 r = gelu_bf16x8(make_uint4(w4[0], w4[1], w4[2], w4[3]), smem_u32(tab));
    w4[0] = r.x;
    w4[1] = r.y;
    w4[2] = r.z;
    w4[3] = r.w;
  }
}

}  // namespace ltxfp8
