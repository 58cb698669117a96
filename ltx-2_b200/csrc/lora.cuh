// Skinny LoRA-A GEMM for sm_100a: Ax[M, r] = bf16( x[M, K] . A[r, K]^T ), bf16
// operands, fp32 accumulation in TMEM.  HBM-bound (reads x once).
//
// The reference has no runtime LoRA (it merges LoRA deltas into the weights at
// load time, ltx-core/src/ltx_core/quantization/blockwise/_impl.py:277-301);
// this kernel provides the x A^T half of a runtime alpha * B (A x) term whose
// B half is folded into the FP8 GEMM as extra bf16 K blocks.
//
// One CTA per 128 rows, two CTAs per SM (96 KB of ring each, so 24576 rows run
// in one wave): warp 0 streams 64-wide K chunks of x (16 KB) and A (r x 128 B)
// through a TMA ring, warp 1 issues tcgen05.mma.kind::f16 (M128, N = r, K16)
// accumulating over all of K in TMEM, warps 4-7 drain the r accumulator columns
// to bf16.
#pragma once

#include "ptx.cuh"

namespace ltxfp8 {

constexpr int kLoraThreads = 256;
constexpr uint32_t kLoraXBytes = 128 * 128;  // 128 rows x 64 bf16
constexpr uint32_t kLoraSmemBudget = 96 * 1024;  // two CTAs per SM: one wave for 24576 rows

enum LoraStatus : unsigned int {
  kStLoraProducer = 0x4C010001u,
  kStLoraMma = 0x4C010002u,
  kStLoraEpi = 0x4C010003u,
  kStLoraDrain = 0x4C010004u,
};

struct LoraParams {
  int M, K, r;
  int num_chunks;     // K / 64
  int stages;
  uint32_t stage_bytes;  // kLoraXBytes + r * 128
  uint32_t tmem_cols;    // power of two >= max(32, r)
  __nv_bfloat16* ax;     // [M, r]
};

__global__ void __launch_bounds__(kLoraThreads, 2)
    lora_a_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmA,
                  const LoraParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.stages * p.stage_bytes);
  uint64_t* empty = full + p.stages;
  uint64_t* done = empty + p.stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x) / 32, 0);
  const int lane = static_cast<int>(lane_id());
  const int m0 = blockIdx.x * 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmA);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    bool ok = true;
    int c = 0;
    for (; c < p.num_chunks; ++c) {
      const uint32_t s = c % p.stages, ph = (c / p.stages) & 1u;
      if (!mbar_wait(&empty[s], ph ^ 1u, kStLoraProducer)) {
        ok = false;
        break;
      }
      uint8_t* sx = smem + s * p.stage_bytes;
      mbar_arrive_expect_tx(&full[s], p.stage_bytes);
      tma_load_2d(&tmX, &full[s], sx, c * 64, m0);
      tma_load_2d(&tmA, &full[s], sx + kLoraXBytes, c * 64, 0);
    }
    if (!ok) {
      const int first = c > p.stages ? c - p.stages : 0;
      for (int i = first; i < c; ++i) mbar_wait(&full[i % p.stages], (i / p.stages) & 1u, kStLoraDrain);
    }
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = make_idesc(1u, 128u, static_cast<uint32_t>(p.r));
    bool ok = true;
    for (int c = 0; c < p.num_chunks; ++c) {
      const uint32_t s = c % p.stages, ph = (c / p.stages) & 1u;
      if (!mbar_wait(&full[s], ph, kStLoraMma)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t x_addr = smem_u32(smem + s * p.stage_bytes);
      const uint64_t xdesc = sw128_kmajor_desc(x_addr);
      const uint64_t adesc = sw128_kmajor_desc(x_addr + kLoraXBytes);
#pragma unroll
      for (int j = 0; j < 4; ++j) mma_f16(tmem_base, xdesc + 2u * j, adesc + 2u * j, idesc, (c > 0 || j > 0) ? 1u : 0u);
      tc_commit(&empty[s]);
    }
    (void)ok;
    tc_commit(done);  // fires when every MMA above has completed
  } else if (warp >= 4) {
    const int sp = warp & 3;
    const int row = m0 + sp * 32 + lane;
    const bool waited = mbar_wait(done, 0u, kStLoraEpi);
    if (__all_sync(0xffffffffu, waited)) {
      tc_fence_after_sync();
      for (int c0 = 0; c0 < p.r; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(sp * 32) << 16) + c0, v);
        tmem_wait_ld();
        if (row < p.M) {
          // r % 16 == 0; a 32-column slice may run past r by 16 columns.
          const int ncols = min(32, p.r - c0);
          uint4* dst = reinterpret_cast<uint4*>(p.ax + static_cast<int64_t>(row) * p.r + c0);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (i * 8 < ncols) {
              dst[i] = make_uint4(pack_bf16x2(__uint_as_float(v[8 * i]), __uint_as_float(v[8 * i + 1])),
                                  pack_bf16x2(__uint_as_float(v[8 * i + 2]), __uint_as_float(v[8 * i + 3])),
                                  pack_bf16x2(__uint_as_float(v[8 * i + 4]), __uint_as_float(v[8 * i + 5])),
                                  pack_bf16x2(__uint_as_float(v[8 * i + 6]), __uint_as_float(v[8 * i + 7])));
            }
          }
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    // In the failure path the MMA thread may have stopped early; `done` was
    // still committed after its last MMA, so wait for it before freeing TMEM.
    mbar_wait(done, 0u, kStLoraDrain);
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

}  // namespace ltxfp8
