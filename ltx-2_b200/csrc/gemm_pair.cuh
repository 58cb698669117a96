// Blockwise-scaled FP8 GEMM over CTA pairs (tcgen05.mma.cta_group::2), sm_100a.
//
// Same math and operand contract as fp8_blockwise_gemm_kernel (gemm.cuh):
//   D[m, n] = bf16( sum_kb sfa[m, kb] * sfb[n/128, kb] * (A[m, kb] . W[n, kb]) + bias[n] )
// (the reference's fp8_gemm_nt_sm89, ltx-kernels/csrc/blockwise/api.cpp:42-65 and
// kernels/geforce/gemm.cu:26-275), with the fused GELU / requant / LoRA epilogues.
//
// Layout of the work:
//   * A cluster of two CTAs (on two SMs) owns a 256 x 256 output tile.  CTA r
//     loads rows [128r, 128r+128) of the tile's A block and rows [128r, 128r+128)
//     of its W block (an N half); the pair MMA (M256 N256 K32) reads both CTAs'
//     shared memory, and CTA r's TMEM receives output rows [128r, 128r+128) for
//     all 256 columns.  Per SM and K block this moves 32 KB through shared
//     memory instead of 48 KB for a one-CTA 128 x 256 tile.  Loads are plain
//     (no multicast); only their completion is counted on the leader's barrier.
//   * warp 0  TMA producer (both CTAs); warp 1  TMEM allocation (both CTAs) and
//     MMA issue (leader CTA only); warps 4-11  per-128-K promotion of the TMEM
//     partials into fp32 registers (one row, 128 columns per thread), then
//     y = bf16(acc + bias) (GELU-tanh applied when fused) and its 1x128 group
//     abs-max into a 64 KB shared staging tile; warps 2-3  drain the staging
//     tile with TMA stores (bf16 D and/or the requantised e4m3 codes) while the
//     promotion warps already work on the next tile.  Epilogue and staging layout
//     are those of the one-CTA kernel, per CTA over its 128 rows.
#pragma once

#include "gemm.cuh"

namespace ltxfp8 {
namespace pair {

constexpr int kTileM = 256;            // per CTA pair
constexpr int kTileN = 256;
constexpr int kRowsPerCta = 128;
constexpr int kBK = 128;
constexpr int kStages = 4;
constexpr uint32_t kABytes = kRowsPerCta * kBK;     // 16 KB: this CTA's A rows
constexpr uint32_t kBBytes = kRowsPerCta * kBK;     // 16 KB: this CTA's W rows (N half)
constexpr uint32_t kStageBytes = kABytes + kBBytes; // 32 KB
constexpr uint32_t kStageTx = 2 * kStageBytes;      // both CTAs' bytes land on the leader's barrier
constexpr uint32_t kStagingBytes = kRowsPerCta * kTileN * 2;  // bf16 [128, 256]
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;
constexpr int kScaleRing = 4;  // K blocks of scales in flight per promotion thread
// Per promotion thread: kScaleRing slots of (sfa, sfb), slot-major so that a
// warp's 32 lanes read 32 consecutive words.
constexpr uint32_t kScaleRingBytes = 256 * kScaleRing * 2 * 4;
constexpr uint32_t kStagingAmaxBytes = 2 * kRowsPerCta * 4;  // abs-max per (128-column half, row)
constexpr uint32_t kBarrierBytes = 256;
constexpr uint32_t kSmemBytes =
    kStages * kStageBytes + kStagingBytes + kStagingAmaxBytes + kScaleRingBytes + 1024 + kBarrierBytes + kGeluTabBytes;

constexpr uint32_t kRegsCtrl = 40;   // warps 0-3: producer, MMA, store warps
constexpr uint32_t kRegsEpi = 232;   // warps 4-11: promotion
constexpr uint32_t kLaunchRegs = 168;
static_assert(128 * kRegsCtrl + 256 * kRegsEpi <= kThreads * kLaunchRegs, "register split exceeds launch");

enum PairStatus : unsigned int {
  kStPProducerEmpty = 0x47020001u,
  kStPMmaTmemEmpty = 0x47020002u,
  kStPMmaFull = 0x47020003u,
  kStPEpiTmemFull = 0x47020004u,
  kStPStagingEmpty = 0x47020005u,
  kStPStagingFull = 0x47020006u,
  kStPDrain = 0x47020007u,
};

struct Params {
  GemmParams g;  // m_tiles / n_tiles / total_tiles count 256 x 256 pair tiles here
};


// acc += scale * partial for one K block, 128 columns read in two TMEM round
// trips of 64; the TMEM buffer is released on the leader's barrier after the
// second one, before the last 32 packed FMAs.
__device__ __forceinline__ bool promote_pair(uint64_t* tfull, uint32_t tempty_leader, uint32_t tmem_base, int sp,
                                             int half, uint32_t it, float scale, int lane, float2 (&acc)[64]) {
  const uint32_t buf = it & 1u, bph = (it >> 1) & 1u;
  if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], bph, kStPEpiTmemFull))) return false;
  tc_fence_after_sync();
  const uint32_t taddr = tmem_base + (static_cast<uint32_t>(sp * 32) << 16) + buf * kTileN + half * 128;
  const float2 s2 = make_float2(scale, scale);
  uint32_t r0[32], r1[32];
  tmem_ld_32x32b_x32(taddr + 0, r0);
  tmem_ld_32x32b_x32(taddr + 32, r1);
  tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    acc[j] = __ffma2_rn(s2, make_float2(__uint_as_float(r0[2 * j]), __uint_as_float(r0[2 * j + 1])), acc[j]);
    acc[16 + j] = __ffma2_rn(s2, make_float2(__uint_as_float(r1[2 * j]), __uint_as_float(r1[2 * j + 1])), acc[16 + j]);
  }
  tmem_ld_32x32b_x32(taddr + 64, r0);
  tmem_ld_32x32b_x32(taddr + 96, r1);
  tmem_wait_ld();
  tc_fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive_cluster(tempty_leader + buf * 8u);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    acc[32 + j] = __ffma2_rn(s2, make_float2(__uint_as_float(r0[2 * j]), __uint_as_float(r0[2 * j + 1])), acc[32 + j]);
    acc[48 + j] = __ffma2_rn(s2, make_float2(__uint_as_float(r1[2 * j]), __uint_as_float(r1[2 * j + 1])), acc[48 + j]);
  }
  return true;
}


template <bool kGelu, bool kRequant>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_blockwise_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                   const __grid_constant__ CUtensorMap tmLX, const __grid_constant__ CUtensorMap tmLB,
                                   const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmQ,
                                   const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* staging = smem + kStages * kStageBytes;
  float* stg_amax = reinterpret_cast<float*>(staging + kStagingBytes);  // [2 halves][128 rows]
  uint8_t* scale_ring = staging + kStagingBytes + kStagingAmaxBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(scale_ring + kScaleRingBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;  // [2]
  uint64_t* tempty = tfull + 2;       // [2]   (used in the leader CTA)
  uint64_t* stg_full = tempty + 2;    // [1]
  uint64_t* stg_empty = stg_full + 1; // [1]
  uint64_t* drain = stg_empty + 1;    // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  uint16_t* gelu_tab = reinterpret_cast<uint16_t*>(scale_ring + kScaleRingBytes + kBarrierBytes);

  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x) / 32, 0);
  const int lane = static_cast<int>(lane_id());
  const uint32_t rank = cluster_ctarank();
  if (kGelu && !(p.flags & kGemmGeluFast)) gelu_table_fill(gelu_tab, static_cast<int>(threadIdx.x), kThreads);
  const bool leader = rank == 0;
  const int cluster_id = static_cast<int>(blockIdx.x) >> 1;
  const int num_clusters = static_cast<int>(gridDim.x) >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 16);  // 8 promotion warps in each CTA of the pair
    }
    mbar_init(stg_full, 8);
    mbar_init(stg_empty, 2);
    mbar_init(drain, 1);
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (p.num_lora > 0) {
      tma_prefetch_desc(&tmLX);
      tma_prefetch_desc(&tmLB);
    }
    if (p.flags & kGemmWriteD) tma_prefetch_desc(&tmD);
    if (kRequant) tma_prefetch_desc(&tmQ);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync();  // barrier inits and TMEM allocation visible across the pair
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int num_blocks = p.num_kb + p.num_lora;
  const uint32_t full_leader = mapa_shared(smem_u32(full), 0);
  const uint32_t tempty_leader = mapa_shared(smem_u32(tempty), 0);

  if (warp < 4) {
    setmaxnreg_dec<kRegsCtrl>();
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ TMA producer (both CTAs)
      uint32_t it = 0;
      bool ok = true;
      for (int tile = cluster_id; tile < p.total_tiles && ok; tile += num_clusters) {
        int mt, nt;
        gemm_tile_coords(tile, p, mt, nt);
        const int m0 = mt * kTileM + static_cast<int>(rank) * kRowsPerCta;
        const int n0 = nt * kTileN + static_cast<int>(rank) * kRowsPerCta;
        for (int kb = 0; kb < num_blocks; ++kb, ++it) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, kStPProducerEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * kStageBytes;
          uint8_t* sb = sa + kABytes;
          if (leader) mbar_arrive_expect_tx(&full[s], kStageTx);
          const uint32_t bar = full_leader + s * 8u;
          if (kb < p.num_kb) {
            tma_load_2d_pair(&tmA, bar, sa, kb * kBK, m0);
            tma_load_2d_pair(&tmB, bar, sb, kb * kBK, n0);
          } else {
            const int c = (kb - p.num_kb) * kLoraChunk;
            tma_load_2d_pair(&tmLX, bar, sa, c, m0);
            tma_load_2d_pair(&tmLB, bar, sb, c, n0);
          }
        }
      }
      if (!ok && leader) {
        // Both CTAs' loads complete on the leader's barriers: let the ones in flight land.
        const uint32_t first = it > static_cast<uint32_t>(kStages) ? it - kStages : 0u;
        for (uint32_t i = first; i < it; ++i) mbar_wait(&full[i % kStages], (i / kStages) & 1u, kStPDrain);
      }
    } else if (warp == 1) {
      // ------------------------------------------------------------ MMA issue (leader CTA)
      if (leader && lane == 0) {
        constexpr uint32_t kIdescF8 = make_idesc(0u, kTileM, kTileN);
        constexpr uint32_t kIdescBF16 = make_idesc(1u, kTileM, kTileN);
        uint32_t it = 0;
        bool ok = true;
        for (int tile = cluster_id; tile < p.total_tiles && ok; tile += num_clusters) {
          for (int kb = 0; kb < num_blocks; ++kb, ++it) {
            const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
            const uint32_t buf = it & 1u, bph = (it >> 1) & 1u;
            if (!mbar_wait(&tempty[buf], bph ^ 1u, kStPMmaTmemEmpty)) {
              ok = false;
              break;
            }
            tc_fence_after_sync();
            if (!mbar_wait(&full[s], ph, kStPMmaFull)) {
              ok = false;
              break;
            }
            tc_fence_after_sync();
            const uint32_t a_addr = smem_u32(smem + s * kStageBytes);
            const uint64_t adesc = sw128_kmajor_desc(a_addr);
            const uint64_t bdesc = sw128_kmajor_desc(a_addr + kABytes);
            const uint32_t d_tmem = tmem_base + buf * kTileN;
            if (kb < p.num_kb) {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                mma_f8f6f4_pair(d_tmem, adesc + 2u * j, bdesc + 2u * j, kIdescF8, j > 0 ? 1u : 0u);
            } else {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                mma_f16_pair(d_tmem, adesc + 2u * j, bdesc + 2u * j, kIdescBF16, j > 0 ? 1u : 0u);
            }
            tc_commit_pair_mc(&empty[s], 0x3);
            tc_commit_pair_mc(&tfull[buf], 0x3);
          }
        }
        // `drain` flips in both CTAs once every pair MMA issued above has completed.
        tc_commit_pair_mc(drain, 0x3);
      }
    } else if (warp >= 2) {
      // ------------------------------------------------------------ staging -> global (warps 2, 3)
      // (Only whole warps 2 and 3 enter: lanes 1-31 of warp 0 must not, their
      // lane 0 is the producer and never joins these warp-wide votes.)  As in the
      // one-CTA kernel: warp pw owns the 32-row slices pw*32 and 64 + pw*32 of this
      // CTA's 128 rows; lane 0 issues the TMA stores.
      const int pw = warp - 2;  // 0 or 1
      const bool write_d = (p.flags & kGemmWriteD) != 0;
      uint32_t tcount = 0;
      for (int tile = cluster_id; tile < p.total_tiles; tile += num_clusters, ++tcount) {
        int mt, nt;
        gemm_tile_coords(tile, p, mt, nt);
        const int m0 = mt * kTileM + static_cast<int>(rank) * kRowsPerCta;
        const int n0 = nt * kTileN;
        if (!__all_sync(0xffffffffu, mbar_wait(stg_full, tcount & 1u, kStPStagingFull))) break;
        if constexpr (kRequant) {
#pragma unroll 1
          for (int j = 0; j < 4; ++j) {
            const int g = j & 1;
            const int rb = (j >> 1) * 64 + pw * 32;
            const int r = rb + lane;
            const int col0 = n0 + g * 128;
            if (col0 >= p.N) continue;  // warp-uniform: N % 128 == 0
            const bool slice_ok = m0 + rb < p.M;
            if (write_d) {
              if (lane == 0 && slice_ok) {
                tma_store_2d(&tmD, staging + (2 * g) * kStagingBlockBytes + rb * 128, col0, m0 + rb);
                tma_store_2d(&tmD, staging + (2 * g + 1) * kStagingBlockBytes + rb * 128, col0 + 64, m0 + rb);
                tma_store_commit();
                tma_store_wait_read();  // the codes below overwrite the slice
              }
              __syncwarp();
            }
            float s, s_inv;
            requant_scale(stg_amax[g * kRowsPerCta + r], (p.flags & kGemmRequantTriton) != 0, s, s_inv);
            const bool in_range = isfinite(s) || (p.flags & kGemmRequantTriton) != 0;
            uint8_t* qrow = staging + (2 * g) * kStagingBlockBytes + r * 128;
#pragma unroll 1
            for (int k = 0; k < 8; ++k) {  // 16 codes from bf16 chunks 2k, 2k+1
              uint32_t w4[4];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint4 v = *reinterpret_cast<const uint4*>(staging + gemm_staging_off(r, g * 16 + 2 * k + h));
                float f[8];
                bf16x8_to_f32(v, f);
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                  const float v0 = __fmul_rn(f[4 * i], s), v1 = __fmul_rn(f[4 * i + 1], s);
                  const float v2 = __fmul_rn(f[4 * i + 2], s), v3 = __fmul_rn(f[4 * i + 3], s);
                  const uint16_t lo = in_range ? f32x2_to_e4m3x2_inrange(v0, v1) : f32x2_to_e4m3x2(v0, v1);
                  const uint16_t hi = in_range ? f32x2_to_e4m3x2_inrange(v2, v3) : f32x2_to_e4m3x2(v2, v3);
                  w4[2 * h + i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
                }
              }
              // Code chunk k replaces bf16 chunk k of the block, already read (k <= 2k).
              *reinterpret_cast<uint4*>(qrow + ((k ^ (r & 7)) * 16)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
            if (m0 + r < p.M) p.s_out[static_cast<int64_t>(col0 / 128) * p.s_out_ld + m0 + r] = s_inv;
            __syncwarp();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && slice_ok) {
              tma_store_2d(&tmQ, staging + (2 * g) * kStagingBlockBytes + rb * 128, col0, m0 + rb);
              tma_store_commit();
            }
          }
        } else {
          // bf16 D (GELU already applied by the promotion warps), stored as staged.
          if (lane == 0) {
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
              const int rb = h * 64 + pw * 32;
              if (m0 + rb >= p.M) continue;
#pragma unroll 1
              for (int b4 = 0; b4 < 4; ++b4)
                if (n0 + b4 * 64 < p.N)
                  tma_store_2d(&tmD, staging + b4 * kStagingBlockBytes + rb * 128, n0 + b4 * 64, m0 + rb);
            }
            tma_store_commit();
          }
        }
        // The staging tile may be overwritten once the stores have read it.
        if (lane == 0) tma_store_wait_read();
        __syncwarp();
        if (lane == 0) mbar_arrive(stg_empty);
      }
      if (lane == 0) tma_store_wait_all();
      __syncwarp();
    }
  } else {
    setmaxnreg_inc<kRegsEpi>();
    // -------------------------------------------------------------- promotion (warps 4-11)
    const int sp = warp & 3;
    const int half = (warp - 4) >> 2;
    const int r_local = sp * 32 + lane;  // row within this CTA's 128
    const uint32_t ring_base = smem_u32(scale_ring) + static_cast<uint32_t>((warp - 4) * 32 + lane) * 4u;
    uint32_t it = 0, tcount = 0;
    bool ok = true;
    for (int tile = cluster_id; tile < p.total_tiles && ok; tile += num_clusters, ++tcount) {
      int mt, nt;
      gemm_tile_coords(tile, p, mt, nt);
      const int row = mt * kTileM + static_cast<int>(rank) * kRowsPerCta + r_local;
      const bool row_ok = row < p.M;
      const int col0 = nt * kTileN + half * 128;
      const bool col_ok = col0 < p.N;
      const int nb = col0 / 128;
      const float* sfa_row = p.sfa + row;
      const float* sfb_blk = p.sfb + static_cast<int64_t>(nb) * p.num_kb;

      float2 acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = make_float2(0.f, 0.f);

      // The scales of K block kb are copied (cp.async, 4 B each) kScaleRing
      // blocks ahead into this thread's ring slots; one commit group per block
      // keeps the group count uniform even where nothing is copied.
      auto prefetch = [&](int kb) {
        if (kb < p.num_kb) {
          const uint32_t slot = ring_base + static_cast<uint32_t>(kb % kScaleRing) * (2u * 256u * 4u);
          if (row_ok) cp_async_4(slot, sfa_row + static_cast<int64_t>(kb) * p.sfa_ld);
          if (col_ok) cp_async_4(slot + 256u * 4u, sfb_blk + kb);
        }
        cp_async_commit();
      };
#pragma unroll
      for (int j = 0; j < kScaleRing; ++j) prefetch(j);
      for (int kb = 0; kb < num_blocks; ++kb) {
        cp_async_wait<kScaleRing - 1>();
        float scale = p.lora_alpha;
        if (kb < p.num_kb) {
          const uint32_t slot = ring_base + static_cast<uint32_t>(kb % kScaleRing) * (2u * 256u * 4u);
          scale = lds_f32(slot) * lds_f32(slot + 256u * 4u);
        }
        prefetch(kb + kScaleRing);
        ok = promote_pair(tfull, tempty_leader, tmem_base, sp, half, it, scale, lane, acc);
        ++it;
        if (!ok) break;
      }
      cp_async_wait<0>();
      if (!ok) break;

      // y = bf16(acc + bias) (+ GELU) into the staging tile once the store warps
      // have drained it, and the group's abs-max for the requantisation.
      if (!__all_sync(0xffffffffu, mbar_wait(stg_empty, (tcount & 1u) ^ 1u, kStPStagingEmpty))) {
        ok = false;
        break;
      }
      const bool has_bias = (p.flags & kGemmBias) != 0 && col_ok;
      const bool gelu_fast = (p.flags & kGemmGeluFast) != 0;
      const float4* bias4 = reinterpret_cast<const float4*>(p.bias + col0);
      float gmax = 0.0f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {  // 16 chunks of 8 columns
        float4 b0 = make_float4(0.f, 0.f, 0.f, 0.f), b1 = b0;
        if (has_bias) {
          b0 = __ldg(bias4 + 2 * c);
          b1 = __ldg(bias4 + 2 * c + 1);
        }
        const float2 a0 = acc[4 * c], a1 = acc[4 * c + 1], a2 = acc[4 * c + 2], a3 = acc[4 * c + 3];
        uint32_t w4[4] = {pack_bf16x2(a0.x + b0.x, a0.y + b0.y), pack_bf16x2(a1.x + b0.z, a1.y + b0.w),
                          pack_bf16x2(a2.x + b1.x, a2.y + b1.y), pack_bf16x2(a3.x + b1.z, a3.y + b1.w)};
        if constexpr (kGelu) {
          gelu_bf16x8_inplace(w4, gelu_fast, gelu_tab);
        }
        if constexpr (kRequant) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            gmax = fmax_nan(gmax, fmax_nan(fabsf(__uint_as_float(w4[i] << 16)),
                                           fabsf(__uint_as_float(w4[i] & 0xFFFF0000u))));
        }
        *reinterpret_cast<uint4*>(staging + gemm_staging_off(r_local, half * 16 + c)) =
            make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
      if constexpr (kRequant) stg_amax[half * kRowsPerCta + r_local] = gmax;
      fence_proxy_async_smem();  // the store warps hand these bytes straight to TMA
      __syncwarp();
      if (lane == 0) mbar_arrive(stg_full);
    }
  }

  // ---------------------------------------------------------------- teardown
  if (warp == 1) mbar_wait(drain, 0u, kStPDrain);  // all pair MMAs into this CTA's TMEM are done
  tc_fence_before_sync();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace pair
}  // namespace ltxfp8
