// Blockwise-scaled FP8 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   D[m, n] = bf16( sum_kb sfa[m, kb] * sfb[n/128, kb] * (A[m, kb] . W[n, kb]) + bias[n] )
//
// A e4m3 [M, K] and W e4m3 [N, K] are K-contiguous ("NT"); sfa is MN-major
// (element (m, kb) at sfa[kb * sfa_ld + m]); sfb is [N/128, K/128] row-major.
// This is the contract of the reference's fp8_gemm_nt_sm89
// (ltx-kernels/csrc/blockwise/api.cpp:42-65, kernels/geforce/gemm.cu:26-275).
//
// Design (one CTA per SM, persistent over 128 x 256 output tiles):
//   warp 0      TMA producer: one 128-wide K block of A (16 KB) and W (32 KB)
//               per pipeline stage, 3 stages, 128 B swizzle.
//   warp 1      MMA issuer: 4 x tcgen05.mma.kind::f8f6f4 (M128 N256 K32) per K
//               block into one of two 256-column TMEM buffers, then
//               tcgen05.commit to release the smem stage and hand the TMEM
//               buffer to the epilogue.
//   warps 4-11  promotion + epilogue: each thread owns one row and 128 columns.
//               Per K block it reads the raw partial sums from TMEM and folds
//               them into fp32 registers with the block's scale
//               sfa[m,kb] * sfb[nb,kb] (the same promotion the reference does
//               after every 128-K block, gemm.cu:185-199).  The two TMEM buffers
//               let the tensor core run one K block ahead of the promotion.
//               After the last block: y = bf16(acc + bias), optionally
//               GELU-tanh (rounded to bf16), into a 64 KB shared staging tile,
//               plus the abs-max of the thread's 1x128 group when the output is
//               requantised, then straight on to the next tile.
//   warps 2-3   drain the staging tile with TMA stores: the bf16 tile, and/or
//               its 1x128 requantisation to e4m3 for the next layer (codes
//               written over the consumed bf16, then stored by TMA), so that
//               work overlaps the next tile's K loop.
//   LoRA        alpha * (x A^T) B^T is folded in as extra K blocks of bf16 MMAs
//               (kind::f16) over [x A^T | B], promoted with scale alpha.
#pragma once

#include "gelu.cuh"
#include "ptx.cuh"

namespace ltxfp8 {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 128;
constexpr int kStages = 3;
constexpr uint32_t kABytes = kBM * kBK;               // 16 KB
constexpr uint32_t kBBytes = kBN * kBK;               // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;   // 48 KB
// W as packed 6-bit codes (kGemmWeightFp6): the TMA reads 96 B of each 128-code
// row and writes them to shared memory as 16-code groups of 12 B with 4 B gaps
// (the MMA's layout for 6-bit operands), so the B tile keeps its 128 B rows and
// swizzle and only its transaction byte count changes.
constexpr uint32_t kBBytesFp6 = kBBytes / 4 * 3;      // 24 KB
constexpr uint32_t kStagingBytes = kBM * kBN * 2;     // 64 KB: bf16 [128, 256] epilogue tile
constexpr int kGemmThreads = 384;
constexpr uint32_t kTmemCols = 512;                   // 2 x 256 fp32 accumulator columns
constexpr int kLoraChunk = 64;                        // bf16 K elements per LoRA block (128 B rows)
constexpr uint32_t kStagingAmaxBytes = 2 * kBM * 4;  // abs-max per (128-column half, row)
constexpr uint32_t kGemmBarrierBytes = 256;
constexpr uint32_t kGemmSmemBytes = kStages * kStageBytes + kStagingBytes + kStagingAmaxBytes + 1024 /*align*/ +
                                    kGemmBarrierBytes + kGeluTabBytes;

// Register split between the producer/MMA warpgroup and the two epilogue
// warpgroups; the launch must provide kGemmThreads * kGemmLaunchRegs.
constexpr uint32_t kRegsCtrl = 40;
constexpr uint32_t kRegsEpi = 232;
constexpr uint32_t kGemmLaunchRegs = 168;
static_assert(128 * kRegsCtrl + 256 * kRegsEpi <= kGemmThreads * kGemmLaunchRegs, "register split exceeds launch");

enum GemmFlags : int {
  kGemmBias = 1,            // add fp32 bias[n]
  kGemmWriteD = 2,          // write the bf16 result (the GELU output when GELU is on)
  kGemmLora = 4,            // extra bf16 K blocks with scale lora_alpha
  kGemmGeluFast = 8,        // GELU as x / (1 + 2^a) with approximate instructions (else torch's formula)
  kGemmRequantTriton = 16,  // requantisation scales as the Triton quantiser computes them (div.full)
  kGemmWeightFp6 = 32,      // W is e2m3 codes packed 6 bits each in the tensor core's order
                            // (ltxfp8_fp6_to_tc), its scales already multiplied by 2^-6
};

// Scale pair of a requantised 1x128 group from its abs-max: the Triton quantiser's
// divisions (triton_ops.py:19-21) or torch's reciprocal-multiply (functional.py:142-144).
__device__ __forceinline__ void requant_scale(float amax, bool triton, float& s, float& inv) {
  if (triton) {
    s = div_full(448.0f, amax);
    inv = div_full(1.0f, s);
  } else {
    s = __fmul_rn(__frcp_rn(amax), 448.0f);
    inv = __frcp_rn(s);
  }
}

// Device status codes recorded when a bounded wait gives up.
enum GemmStatus : unsigned int {
  kStProducerEmpty = 0x47010001u,
  kStMmaTmemEmpty = 0x47010002u,
  kStMmaFull = 0x47010003u,
  kStEpiTmemFull = 0x47010004u,
  kStDrain = 0x47010005u,
  kStStagingFull = 0x47010006u,
  kStStagingEmpty = 0x47010007u,
};

struct GemmParams {
  int M, N, K;
  int num_kb;         // K / 128
  int num_lora;       // LoRA K blocks (ceil(r / 64)), 0 without LoRA
  int m_tiles, n_tiles, group_m, total_tiles;
  const float* sfa;
  int64_t sfa_ld;
  const float* sfb;   // [N/128, num_kb]
  const float* bias;  // [N] fp32, may be null
  __nv_bfloat16* d;   // [M, N]
  uint8_t* q_out;     // [M, N] e4m3 (requant)
  float* s_out;       // requant scales at s_out[nb * s_out_ld + m]
  int64_t s_out_ld;
  float lora_alpha;
  int flags;
  // Split-K for skinny M: each output tile's K blocks are divided among k_splits
  // work units; unit u = tile * k_splits + split writes its fp32 partial (no
  // bias) to the 128 x 256 workspace block ws[u * 128 * 256], and
  // splitk_reduce_kernel sums a tile's partials in split order.  k_splits = 1:
  // no split.
  int k_splits;
  int kb_per_split;
  float* ws;
};

// Grouped rasterisation: consecutive tile indices walk group_m M-tiles down a
// column of N-tiles, so the CTAs resident at one time share A and W tiles in L2.
__device__ __forceinline__ void gemm_tile_coords(int tile, const GemmParams& p, int& mt, int& nt) {
  const int per_group = p.group_m * p.n_tiles;
  const int g = tile / per_group;
  const int first_m = g * p.group_m;
  const int gm = min(p.group_m, p.m_tiles - first_m);
  const int r = tile - g * per_group;
  mt = first_m + r % gm;
  nt = r / gm;
}

// One work unit: an output tile and a contiguous range of its K blocks (the
// whole range unless split-K is on); LoRA blocks ride with the last split.
struct GemmUnit {
  int mt, nt, split, kb_begin, n_fp8, n_blocks;
};

__device__ __forceinline__ GemmUnit gemm_unit(int u, const GemmParams& p) {
  GemmUnit w;
  const int tile = u / p.k_splits;
  w.split = u - tile * p.k_splits;
  gemm_tile_coords(tile, p, w.mt, w.nt);
  w.kb_begin = w.split * p.kb_per_split;
  w.n_fp8 = min(p.kb_per_split, p.num_kb - w.kb_begin);
  w.n_blocks = w.n_fp8 + (w.split == p.k_splits - 1 ? p.num_lora : 0);
  return w;
}

constexpr int kScalePrefetch = 4;

// Epilogue staging tile, bf16 [128, 256], as four 16 KB column blocks of 64
// columns (block b: columns 64b .. 64b+63), each laid out as TMA's 128 B swizzle
// expects for a [rows, 64] bf16 box: row r at r * 128, its 16 B chunk c (8
// columns) at position c ^ (r & 7).  32 lanes touching one chunk of 32
// consecutive rows then spread over all banks, and any 32-row slice of a block is
// itself a valid TMA box.  `chunk` counts 8-column chunks across the tile (0..31).
constexpr uint32_t kStagingBlockBytes = kBM * 128;  // 16 KB
__device__ __forceinline__ uint32_t gemm_staging_off(int r, int chunk) {
  return static_cast<uint32_t>(chunk >> 3) * kStagingBlockBytes + static_cast<uint32_t>(r) * 128u +
         static_cast<uint32_t>(((chunk & 7) ^ (r & 7)) * 16);
}

// The staged tile's second pass: GELU (in place) and the 1x128 group abs-max of one
// 8-column chunk (`chunk`, counted across the tile) of this thread's row.  The pass
// over a tile runs one chunk per K block of the next tile, while the tensor core
// works, instead of between the tiles where the MMA would wait for the TMEM buffers.
template <bool kGelu, bool kRequant>
__device__ __forceinline__ void staged_post_chunk(uint8_t* staging, int r_local, int chunk, bool gelu_fast,
                                                  const uint16_t* gelu_tab, float& gmax) {
  uint4* ptr = reinterpret_cast<uint4*>(staging + gemm_staging_off(r_local, chunk));
  const uint4 v = *ptr;
  uint32_t w4[4] = {v.x, v.y, v.z, v.w};
  if constexpr (kGelu) {
    gelu_bf16x8_inplace(w4, gelu_fast, gelu_tab);
    *ptr = make_uint4(w4[0], w4[1], w4[2], w4[3]);
  }
  if constexpr (kRequant) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      gmax = fmax_nan(gmax, fmax_nan(fabsf(__uint_as_float(w4[i] << 16)), fabsf(__uint_as_float(w4[i] & 0xFFFF0000u))));
  }
}

// Fold one K block's raw partial sums (TMEM buffer `it & 1`) into the fp32
// accumulators of this thread's row: acc += scale * partial, 128 columns as 64
// packed f32x2 FMAs.  Releases the TMEM buffer as soon as it has been read.
__device__ __forceinline__ bool promote_kblock(uint64_t* tfull, uint64_t* tempty, uint32_t tmem_base, int sp,
                                               int half, uint32_t it, float scale, int lane, float2 (&acc)[64]) {
  const uint32_t buf = it & 1u, bph = (it >> 1) & 1u;
  // Warp-uniform outcome: the TMEM loads below are .sync.aligned.
  if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], bph, kStEpiTmemFull))) return false;
  tc_fence_after_sync();
  const uint32_t taddr = tmem_base + (static_cast<uint32_t>(sp * 32) << 16) + buf * kBN + half * 128;
  const float2 s2 = make_float2(scale, scale);
  // Columns 64-127 are loaded while columns 0-63 are folded in, so the buffer is
  // released one TMEM round trip after the first (1.4 % on the plain full-size GEMMs).
  uint32_t r0[32], r1[32], r2[32], r3[32];
  tmem_ld_32x32b_x32(taddr + 0, r0);
  tmem_ld_32x32b_x32(taddr + 32, r1);
  tmem_wait_ld();
  tmem_ld_32x32b_x32(taddr + 64, r2);
#pragma unroll
  for (int j = 0; j < 16; ++j)
    acc[j] = __ffma2_rn(s2, make_float2(__uint_as_float(r0[2 * j]), __uint_as_float(r0[2 * j + 1])), acc[j]);
  tmem_ld_32x32b_x32(taddr + 96, r3);
#pragma unroll
  for (int j = 0; j < 16; ++j)
    acc[16 + j] = __ffma2_rn(s2, make_float2(__uint_as_float(r1[2 * j]), __uint_as_float(r1[2 * j + 1])), acc[16 + j]);
  tmem_wait_ld();
  tc_fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive(&tempty[buf]);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    acc[32 + j] = __ffma2_rn(s2, make_float2(__uint_as_float(r2[2 * j]), __uint_as_float(r2[2 * j + 1])), acc[32 + j]);
    acc[48 + j] = __ffma2_rn(s2, make_float2(__uint_as_float(r3[2 * j]), __uint_as_float(r3[2 * j + 1])), acc[48 + j]);
  }
  return true;
}

template <bool kGelu, bool kRequant>
__global__ void __launch_bounds__(kGemmThreads, 1)
    fp8_blockwise_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                              const __grid_constant__ CUtensorMap tmLX, const __grid_constant__ CUtensorMap tmLB,
                              const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmQ,
                              const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* staging = smem + kStages * kStageBytes;
  float* stg_amax = reinterpret_cast<float*>(staging + kStagingBytes);  // [2 halves][128 rows]
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + kStagingBytes + kStagingAmaxBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;   // [2]
  uint64_t* tempty = tfull + 2;        // [2]
  uint64_t* stg_full = tempty + 2;     // [1] promotion warps -> store warps
  uint64_t* stg_empty = stg_full + 1;  // [1] store warps -> promotion warps
  uint64_t* drain = stg_empty + 1;     // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  uint16_t* gelu_tab = reinterpret_cast<uint16_t*>(staging + kStagingBytes + kStagingAmaxBytes + kGemmBarrierBytes);

  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x) / 32, 0);
  const int lane = static_cast<int>(lane_id());

  if (kGelu && !(p.flags & kGemmGeluFast)) gelu_table_fill(gelu_tab, static_cast<int>(threadIdx.x), kGemmThreads);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // one arrival per epilogue warp
    }
    mbar_init(stg_full, 8);      // one arrival per promotion warp
    mbar_init(stg_empty, 2);     // one arrival per store warp
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
    if (p.k_splits == 1) {
      if (p.flags & kGemmWriteD) tma_prefetch_desc(&tmD);
      if (kRequant) tma_prefetch_desc(&tmQ);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 4) {
    setmaxnreg_dec<kRegsCtrl>();
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ TMA producer
      uint32_t it = 0;
      bool ok = true;
      const int total_units = p.total_tiles * p.k_splits;
      const uint32_t tx_fp8 = (p.flags & kGemmWeightFp6) ? kABytes + kBBytesFp6 : kStageBytes;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        const GemmUnit w = gemm_unit(u, p);
        const int m0 = w.mt * kBM, n0 = w.nt * kBN;
        for (int kb = 0; kb < w.n_blocks; ++kb, ++it) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, kStProducerEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * kStageBytes;
          uint8_t* sb = sa + kABytes;
          mbar_arrive_expect_tx(&full[s], kb < w.n_fp8 ? tx_fp8 : kStageBytes);
          if (kb < w.n_fp8) {
            tma_load_2d(&tmA, &full[s], sa, (w.kb_begin + kb) * kBK, m0);
            tma_load_2d(&tmB, &full[s], sb, (w.kb_begin + kb) * kBK, n0);
          } else {
            const int c = (kb - w.n_fp8) * kLoraChunk;
            tma_load_2d(&tmLX, &full[s], sa, c, m0);
            tma_load_2d(&tmLB, &full[s], sb, c, n0);
          }
        }
      }
      if (!ok) {
        // Let the loads already in flight land before the CTA exits.
        const uint32_t first = it > static_cast<uint32_t>(kStages) ? it - kStages : 0u;
        for (uint32_t i = first; i < it; ++i) mbar_wait(&full[i % kStages], (i / kStages) & 1u, kStDrain);
      }
    } else if (warp == 1 && lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t kIdescF8 = make_idesc(0u, kBM, kBN);
      constexpr uint32_t kIdescBF16 = make_idesc(1u, kBM, kBN);
      const uint32_t idesc_f8 = (p.flags & kGemmWeightFp6) ? with_b_format(kIdescF8, kFmtE2M3) : kIdescF8;
      uint32_t it = 0;
      bool ok = true;
      const int total_units = p.total_tiles * p.k_splits;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        const GemmUnit w = gemm_unit(u, p);
        for (int kb = 0; kb < w.n_blocks; ++kb, ++it) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
          const uint32_t buf = it & 1u, bph = (it >> 1) & 1u;
          if (!mbar_wait(&tempty[buf], bph ^ 1u, kStMmaTmemEmpty)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          if (!mbar_wait(&full[s], ph, kStMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t a_addr = smem_u32(smem + s * kStageBytes);
          const uint64_t adesc = sw128_kmajor_desc(a_addr);
          const uint64_t bdesc = sw128_kmajor_desc(a_addr + kABytes);
          const uint32_t d_tmem = tmem_base + buf * kBN;
          if (kb < w.n_fp8) {
#pragma unroll
            for (int j = 0; j < 4; ++j)  // 4 x K32 (32 B of each 128 B row)
              mma_f8f6f4(d_tmem, adesc + 2u * j, bdesc + 2u * j, idesc_f8, j > 0 ? 1u : 0u);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)  // 4 x K16 bf16 (32 B of each 128 B row)
              mma_f16(d_tmem, adesc + 2u * j, bdesc + 2u * j, kIdescBF16, j > 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
          tc_commit(&tfull[buf]);
        }
      }
      // Every MMA this thread issued has completed once `drain` flips.
      tc_commit(drain);
      mbar_wait(drain, 0u, kStDrain);
    } else if (warp >= 2 && p.k_splits == 1) {
      // ------------------------------------------------------------ staging -> global (warps 2, 3)
      // (Whole warps 2 and 3 only: lanes 1-31 of warps 0 and 1 must not enter,
      // their lane 0 never joins the warp-wide votes below.)  Warp pw owns the
      // 32-row slices pw*32 and 64 + pw*32 of the tile: its passes and stores need
      // no synchronisation with the other store warp.  Lane 0 issues the TMA stores.
      const int pw = warp - 2;
      const bool write_d = (p.flags & kGemmWriteD) != 0;
      uint32_t tcount = 0;
      for (int u = blockIdx.x; u < p.total_tiles; u += gridDim.x, ++tcount) {
        int mt, nt;
        gemm_tile_coords(u, p, mt, nt);
        const int m0 = mt * kBM, n0 = nt * kBN;
        if (!__all_sync(0xffffffffu, mbar_wait(stg_full, tcount & 1u, kStStagingFull))) break;
        if constexpr (kRequant) {
          // 1x128 requantisation of the staged bf16 values (the reference
          // quantises the bf16 GEMM / GELU output).  One lane per group: step j
          // covers 32 consecutive rows of one 128-column half.  If D is wanted the
          // bf16 slice goes out first; the codes are then written over the slice's
          // first column block and go out as one TMA box.
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
            requant_scale(stg_amax[g * kBM + r], (p.flags & kGemmRequantTriton) != 0, s, s_inv);
            // a finite scale keeps every product within 448 (plain hardware conversion); the
            // Triton quantiser always converts with saturation
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
          // bf16 D (GELU already applied by the promotion warps): the tile goes out
          // as staged (the promotion warps fenced it for the async proxy).
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
    // -------------------------------------------------------------- promotion + epilogue
    const int sp = warp & 3;          // TMEM sub-partition: rows 32*sp .. 32*sp+31
    const int half = (warp - 4) >> 2; // which 128-column half of the 256-wide tile
    uint32_t it = 0;
    uint32_t tcount = 0;              // staged tiles so far (staging barrier phases)
    bool ok = true;
    const int total_units = p.total_tiles * p.k_splits;
    // Second pass over the staged tile (GELU / requant abs-max), deferred: post_c is
    // the next chunk of it to process, 16 when none is pending.
    constexpr bool kPost = kGelu || kRequant;
    const bool gelu_fast = (p.flags & kGemmGeluFast) != 0;
    const int r_local = sp * 32 + lane;
    int post_c = 16;
    float gmax = 0.0f;  // abs-max of this thread's 1x128 group of the staged tile
    auto post_step = [&]() {
      staged_post_chunk<kGelu, kRequant>(staging, r_local, half * 16 + post_c, gelu_fast, gelu_tab, gmax);
      if (++post_c == 16) {
        if constexpr (kRequant) stg_amax[half * kBM + r_local] = gmax;
        fence_proxy_async_smem();  // the store warps hand these bytes straight to TMA
        __syncwarp();
        if (lane == 0) mbar_arrive(stg_full);
      }
    };
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      const GemmUnit w = gemm_unit(u, p);
      const int row = w.mt * kBM + sp * 32 + lane;
      const bool row_ok = row < p.M;
      const int col0 = w.nt * kBN + half * 128;
      const bool col_ok = col0 < p.N;  // N % 128 == 0: a 128-column slab is all in or all out
      const int nb = col0 / 128;
      const float* sfa_row = p.sfa + row + static_cast<int64_t>(w.kb_begin) * p.sfa_ld;
      const float* sfb_blk = p.sfb + static_cast<int64_t>(nb) * p.num_kb + w.kb_begin;

      float2 acc[64];  // column pairs (2j, 2j+1) of this thread's row
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = make_float2(0.f, 0.f);

      // Scales of K block kb are loaded kScalePrefetch blocks before their use.
      // The loop body is unrolled kScalePrefetch times so every prefetch lives
      // in its own register until consumed (no register rotation that would
      // stall on a load still in flight).
      float sa[kScalePrefetch], sb[kScalePrefetch];
#pragma unroll
      for (int j = 0; j < kScalePrefetch; ++j) {
        sa[j] = (row_ok && j < w.n_fp8) ? __ldg(sfa_row + static_cast<int64_t>(j) * p.sfa_ld) : 0.f;
        sb[j] = (col_ok && j < w.n_fp8) ? __ldg(sfb_blk + j) : 0.f;
      }
      for (int kb0 = 0; kb0 < w.n_blocks && ok; kb0 += kScalePrefetch) {
#pragma unroll
        for (int j = 0; j < kScalePrefetch; ++j) {
          const int kb = kb0 + j;
          if (kb < w.n_blocks && ok) {
            const float scale = kb < w.n_fp8 ? sa[j] * sb[j] : p.lora_alpha;
            const int kn = kb + kScalePrefetch;
            sa[j] = (row_ok && kn < w.n_fp8) ? __ldg(sfa_row + static_cast<int64_t>(kn) * p.sfa_ld) : 0.f;
            sb[j] = (col_ok && kn < w.n_fp8) ? __ldg(sfb_blk + kn) : 0.f;
            ok = promote_kblock(tfull, tempty, tmem_base, sp, half, it, scale, lane, acc);
            ++it;
            if constexpr (kPost) {
              if (post_c < 16 && ok) post_step();
            }
          }
        }
      }
      if (!ok) break;
      if (p.k_splits > 1) {
        // Split-K unit: the raw fp32 partial (no bias) for the reduction kernel,
        // block u of the workspace, row-major 128 x 256.  A split launch runs one
        // unit per CTA (units <= SMs), so the pipeline stages are idle here: each
        // warp transposes its 32 rows x 128 columns through its own 16 KB of them
        // and stores whole 512 B rows (lane = row would touch 32 lines per store).
        if (!col_ok) continue;  // warp-uniform
        uint8_t* tr = smem + static_cast<uint32_t>(warp - 4) * (32u * 512u);
#pragma unroll
        for (int c = 0; c < 32; ++c)
          *reinterpret_cast<float4*>(tr + lane * 512 + ((c ^ (lane & 7)) * 16)) =
              make_float4(acc[2 * c].x, acc[2 * c].y, acc[2 * c + 1].x, acc[2 * c + 1].y);
        __syncwarp();
        float* wsu = p.ws + (static_cast<int64_t>(u) * kBM + sp * 32) * kBN + half * 128;
#pragma unroll 4
        for (int i = 0; i < 32; ++i) {
          if (w.mt * kBM + sp * 32 + i >= p.M) break;  // warp-uniform
          reinterpret_cast<float4*>(wsu + static_cast<int64_t>(i) * kBN)[lane] =
              *reinterpret_cast<const float4*>(tr + i * 512 + ((lane ^ (i & 7)) * 16));
        }
        __syncwarp();
        continue;
      }
      // bf16(acc + bias) into the staging tile once the store warps have drained
      // the previous one.  Every promotion warp arrives once per tile, in range or not.
      if constexpr (kPost) {
        while (post_c < 16) post_step();  // the previous tile's pass, if the K loop was too short
      }
      if (!__all_sync(0xffffffffu, mbar_wait(stg_empty, (tcount & 1u) ^ 1u, kStStagingEmpty))) {
        ok = false;
        break;
      }
      const bool has_bias = (p.flags & kGemmBias) != 0 && col_ok;
      const float4* bias4 = reinterpret_cast<const float4*>(p.bias + col0);
#pragma unroll
      for (int c = 0; c < 16; ++c) {  // 16 chunks of 8 columns
        float4 b0 = make_float4(0.f, 0.f, 0.f, 0.f), b1 = b0;
        if (has_bias) {
          b0 = __ldg(bias4 + 2 * c);
          b1 = __ldg(bias4 + 2 * c + 1);
        }
        const float2 a0 = acc[4 * c], a1 = acc[4 * c + 1], a2 = acc[4 * c + 2], a3 = acc[4 * c + 3];
        // The reference applies GELU to the bf16 tensor bf16(acc + bias) and rounds
        // the result to bf16: the second pass reads these values back.
        *reinterpret_cast<uint4*>(staging + gemm_staging_off(r_local, half * 16 + c)) =
            make_uint4(pack_bf16x2(a0.x + b0.x, a0.y + b0.y), pack_bf16x2(a1.x + b0.z, a1.y + b0.w),
                       pack_bf16x2(a2.x + b1.x, a2.y + b1.y), pack_bf16x2(a3.x + b1.z, a3.y + b1.w));
      }
      if constexpr (kPost) {
        post_c = 0;
        gmax = 0.0f;
      } else {
        fence_proxy_async_smem();  // the store warps hand these bytes straight to TMA
        __syncwarp();
        if (lane == 0) mbar_arrive(stg_full);
      }
      ++tcount;
    }
    if constexpr (kPost) {
      if (ok)
        while (post_c < 16) post_step();  // the last tile's pass
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Split-K reduction: out = epilogue( sum_split partial + bias ), summing each
// tile's unit partials in split order (deterministic).  One half-warp per (tile
// row, 128-column group): 16 lanes x 8 columns, so the 1x128 requantisation needs
// no cross-row reduction.  Epilogue semantics are those of the GEMM kernel.
template <bool kGelu, bool kRequant>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const GemmParams p) {
  const int64_t total = static_cast<int64_t>(p.total_tiles) * kBM * 2;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * 16 + (threadIdx.x >> 4);
  const int l16 = threadIdx.x & 15;
  const int st = static_cast<int>(gid / (kBM * 2));
  const int r = static_cast<int>((gid >> 1) % kBM), g = static_cast<int>(gid & 1);
  int mt = 0, nt = 0;
  if (gid < total) gemm_tile_coords(st, p, mt, nt);
  const int row = mt * kBM + r;
  const int col = nt * kBN + g * 128 + l16 * 8;
  const int grp = col / 128;
  // Whole half-warps are in or out (N % 128 == 0), so the requant shuffles stay uniform.
  const bool active = gid < total && row < p.M && col < p.N;
  float f[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = 0.f;
  if (active) {
    const int64_t split_stride = static_cast<int64_t>(kBM) * kBN;
    const float* src = p.ws + (static_cast<int64_t>(st) * p.k_splits * kBM + r) * kBN + g * 128 + l16 * 8;
    for (int sp = 0; sp < p.k_splits; ++sp) {
      const float4 a = *reinterpret_cast<const float4*>(src + sp * split_stride);
      const float4 b = *reinterpret_cast<const float4*>(src + sp * split_stride + 4);
      f[0] += a.x; f[1] += a.y; f[2] += a.z; f[3] += a.w;
      f[4] += b.x; f[5] += b.y; f[6] += b.z; f[7] += b.w;
    }
    if (p.flags & kGemmBias) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(p.bias + col));
      const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + col + 4));
      f[0] += a.x; f[1] += a.y; f[2] += a.z; f[3] += a.w;
      f[4] += b.x; f[5] += b.y; f[6] += b.z; f[7] += b.w;
    }
  }
  if constexpr (kGelu || kRequant) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float y = bf16_round(f[i]);
      if constexpr (kGelu) y = bf16_round((p.flags & kGemmGeluFast) ? gelu_tanh_f32(y) : gelu_tanh_torch(y));
      f[i] = y;
    }
  }
  const int64_t off = static_cast<int64_t>(row) * p.N + col;
  if (active && (p.flags & kGemmWriteD)) {
    *reinterpret_cast<uint4*>(p.d + off) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                                      pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
  }
  if constexpr (kRequant) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmax_nan(amax, fabsf(f[i]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmax_nan(amax, __shfl_xor_sync(0xffffffffu, amax, o, 16));
    float s, s_inv;
    requant_scale(amax, (p.flags & kGemmRequantTriton) != 0, s, s_inv);
    const bool in_range = isfinite(s) || (p.flags & kGemmRequantTriton) != 0;
    uint32_t w[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float v0 = __fmul_rn(f[4 * j], s), v1 = __fmul_rn(f[4 * j + 1], s);
      const float v2 = __fmul_rn(f[4 * j + 2], s), v3 = __fmul_rn(f[4 * j + 3], s);
      const uint16_t lo = in_range ? f32x2_to_e4m3x2_inrange(v0, v1) : f32x2_to_e4m3x2(v0, v1);
      const uint16_t hi = in_range ? f32x2_to_e4m3x2_inrange(v2, v3) : f32x2_to_e4m3x2(v2, v3);
      w[j] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
    if (active) {
      *reinterpret_cast<uint2*>(p.q_out + off) = make_uint2(w[0], w[1]);
      if (l16 == 0) p.s_out[static_cast<int64_t>(grp) * p.s_out_ld + row] = s_inv;
    }
  }
}

}  // namespace ltxfp8
