// C-ABI entry points of the sm_100a blockwise-FP8 linear layer (include/ltxfp8.h).
//
// Host side: argument validation (the reference's TORCH_CHECK / Python asserts
// become negative return codes), TMA tensor-map encoding, launch configuration.
// Nothing here allocates device memory or synchronises a stream, except
// ltxfp8_device_status which exists to read the device status word.
#include "ltxfp8.h"

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>

#include "gemm.cuh"
#include "gemm_pair.cuh"
#include "lora.cuh"
#include "producers.cuh"
#include "ptx.cuh"
#include "quant.cuh"

using namespace ltxfp8;

// Split-K scratch of ltxfp8_gemm_static_scratch: a fixed 32 MiB array in the
// module's global memory, so that entry point needs no allocation.  Every GPU
// that loads this library's kernels holds it until the process exits.  32 MiB
// covers the split-K plan of every shape on a 148-SM device: each split unit
// keeps a 128 x 256 fp32 block (128 KiB) and the split units of a launch fit in
// one wave (at most sms = 148 units, 18.5 MiB).
constexpr size_t kStaticScratchBytes = LTXFP8_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) float g_gemm_static_scratch[kStaticScratchBytes / sizeof(float)];

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(LTXFP8_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// 2-D tensor map over a row-major [outer, inner] array, 128 B swizzle.
int make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(LTXFP8_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LTXFP8_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return LTXFP8_OK;
}

struct DeviceInfo {
  bool init = false;
  int sms = 0;
  int major = 0, minor = 0;
  bool gemm_ready[4] = {false, false, false, false};
  bool pair_ready[4] = {false, false, false, false};
  int pair_clusters = 0;  // co-resident 2-CTA clusters of the pair kernel
  bool lora_ready = false;
  float* static_scratch = nullptr;  // device address of g_gemm_static_scratch (ltxfp8_gemm_static_scratch)
};

// 0 = choose by shape, 1 = one-CTA kernel, 2 = CTA-pair kernel.
std::atomic<int> g_gemm_variant{0};

std::mutex g_dev_mu;
DeviceInfo g_dev[64];

int device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(LTXFP8_ERR_DEVICE, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.init) {
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
    d.init = true;
  }
  if (d.major != 10 || d.minor != 0)
    return fail(LTXFP8_ERR_DEVICE, "this library is built for sm_100a (B200); device %d is sm_%d%d", dev, d.major,
                d.minor);
  *out = &d;
  return LTXFP8_OK;
}

template <bool kGelu, bool kRequant>
int gemm_prepare(DeviceInfo* d) {
  const int idx = (kGelu ? 1 : 0) | (kRequant ? 2 : 0);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (d->gemm_ready[idx]) return LTXFP8_OK;
  auto kern = fp8_blockwise_gemm_kernel<kGelu, kRequant>;
  cudaFuncAttributes attr;
  cudaError_t e = cudaFuncGetAttributes(&attr, kern);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes(gemm)");
  // The warpgroups re-split their registers with setmaxnreg; that only works if
  // the launch reserves the full per-thread budget the split assumes.
  if (attr.numRegs < static_cast<int>(kGemmLaunchRegs))
    return fail(LTXFP8_ERR_CUDA, "gemm kernel compiled with %d registers/thread, register split needs %u",
                attr.numRegs, kGemmLaunchRegs);
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmemBytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm smem)");
  d->gemm_ready[idx] = true;
  return LTXFP8_OK;
}

template <bool kGelu, bool kRequant>
int gemm_launch(DeviceInfo* d, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& lx,
                const CUtensorMap& lb, const CUtensorMap& md, const CUtensorMap& mq, const GemmParams& p,
                cudaStream_t stream) {
  int rc = gemm_prepare<kGelu, kRequant>(d);
  if (rc) return rc;
  const int units = p.total_tiles * p.k_splits;
  // Split-K units write their partials through the pipeline stages' shared
  // memory, which is only idle if every CTA runs exactly one unit.
  if (p.k_splits > 1 && units > d->sms)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "gemm: split-K launch of %d units exceeds the %d SMs", units, d->sms);
  const int grid = units < d->sms ? units : d->sms;
  fp8_blockwise_gemm_kernel<kGelu, kRequant><<<grid, kGemmThreads, kGemmSmemBytes, stream>>>(a, b, lx, lb, md, mq, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  return LTXFP8_OK;
}


// Split-K plan for a skinny launch of the one-CTA kernel (at most sms/2 tiles of
// 128 x 256): every tile's K blocks are divided into S units of at least two
// blocks, at most 16, all units in one wave (tiles x S <= sms).  A cost model in
// units of one K block of one tile (~0.5 us) picks S and skips splits that do not
// pay: the split wave costs ceil(kb / S), plus ~6 for the reduction launch, plus
// ~0.1 per unit for the fp32 partials written and read back (128 KiB each); the
// unsplit wave costs kb.
struct SplitPlan {
  int splits, kb_per_split;
};

SplitPlan splitk_plan(int sms, int64_t total_tiles, int64_t num_kb) {
  SplitPlan pl{1, static_cast<int>(num_kb)};
  if (num_kb < 4 || total_tiles * 2 > sms) return pl;
  int64_t max_s = sms / total_tiles;
  if (max_s > num_kb / 2) max_s = num_kb / 2;
  if (max_s > 16) max_s = 16;
  double best = static_cast<double>(num_kb);
  int64_t best_s = 1;
  for (int64_t sp = 2; sp <= max_s; ++sp) {
    const int64_t kbps = (num_kb + sp - 1) / sp;
    const double cost = static_cast<double>(kbps) + 6.0 + 0.105 * static_cast<double>(total_tiles * sp);
    if (cost < best) {
      best = cost;
      best_s = sp;
    }
  }
  if (best_s < 2) return pl;
  const int64_t kbps = (num_kb + best_s - 1) / best_s;
  pl.kb_per_split = static_cast<int>(kbps);
  pl.splits = static_cast<int>((num_kb + kbps - 1) / kbps);
  return pl;
}

// How one ltxfp8_gemm call is launched: output rows [0, split_row0) as one
// unsplit GEMM, rows [split_row0, M) as a split-K GEMM (plus its reduction).
//  * skinny outputs (at most sms/2 tiles): split_row0 = 0, every tile split;
//  * outputs whose last wave of tiles would leave more than half the SMs idle,
//    for K >= 8192: the last M-tile rows that cover that wave become their own
//    skinny split-K launch, the rest fills whole waves.  (A sparse last wave runs
//    at a higher clock under the power cap, so short tiles do not gain: measured
//    +11 % at K = 16384, +3 % at K = 8192, -4 % at K = 4096 when the same split
//    ran inside one launch.)
//  * otherwise split_row0 = M: one unsplit launch.
constexpr int64_t kTailSplitMinKb = 64;

struct GemmPlan {
  int64_t split_row0;
  int64_t split_tiles;  // output tiles of the split rows
  SplitPlan split;      // split.splits == 1: no split launch
};

GemmPlan gemm_plan(int sms, int64_t M, int64_t N, int64_t K) {
  const int64_t m_tiles = (M + kBM - 1) / kBM, n_tiles = (N + kBN - 1) / kBN;
  const int64_t tiles = m_tiles * n_tiles, num_kb = K / kBK;
  GemmPlan g{M, 0, SplitPlan{1, static_cast<int>(num_kb)}};
  if (tiles * 2 <= sms) {
    const SplitPlan sp = splitk_plan(sms, tiles, num_kb);
    if (sp.splits > 1) g = GemmPlan{0, tiles, sp};
    return g;
  }
  const int64_t rem = tiles % sms;
  if (num_kb < kTailSplitMinKb || rem == 0 || rem * 2 > sms) return g;
  const int64_t tail_m_tiles = (rem + n_tiles - 1) / n_tiles;
  const int64_t tail_tiles = tail_m_tiles * n_tiles;
  if (tail_m_tiles >= m_tiles || tail_tiles * 2 > sms) return g;
  const SplitPlan sp = splitk_plan(sms, tail_tiles, num_kb);
  if (sp.splits > 1) g = GemmPlan{(m_tiles - tail_m_tiles) * kBM, tail_tiles, sp};
  return g;
}

size_t splitk_bytes(const GemmPlan& g) {
  if (g.split.splits < 2) return 0;
  return static_cast<size_t>(g.split_tiles) * static_cast<size_t>(g.split.splits) * kBM * kBN * 4u;
}

// Kernel launches of one call: the unsplit GEMM, the split GEMM, its reduction.
int gemm_plan_launches(const GemmPlan& g) {
  if (g.split.splits < 2) return 1;
  return (g.split_row0 > 0 ? 1 : 0) + 2;
}

template <bool kGelu, bool kRequant>
int splitk_reduce_launch(const DeviceInfo* d, const GemmParams& p, cudaStream_t stream) {
  const int64_t groups = static_cast<int64_t>(p.total_tiles) * kBM * 2;
  const unsigned blocks = static_cast<unsigned>((groups + 15) / 16);
  splitk_reduce_kernel<kGelu, kRequant><<<blocks, 256, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "split-K reduce launch");
  (void)d;
  return LTXFP8_OK;
}

template <bool kGelu, bool kRequant>
int gemm_launch_full(DeviceInfo* d, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& lx,
                     const CUtensorMap& lb, const CUtensorMap& md, const CUtensorMap& mq, const GemmParams& p,
                     cudaStream_t stream) {
  int rc = gemm_launch<kGelu, kRequant>(d, a, b, lx, lb, md, mq, p, stream);
  if (rc || p.k_splits == 1) return rc;
  return splitk_reduce_launch<kGelu, kRequant>(d, p, stream);
}

template <bool kGelu, bool kRequant>
int gemm_pair_launch(DeviceInfo* d, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& lx,
                     const CUtensorMap& lb, const CUtensorMap& md, const CUtensorMap& mq, const GemmParams& p,
                     cudaStream_t stream) {
  auto kern = pair::fp8_blockwise_gemm_pair_kernel<kGelu, kRequant>;
  const int idx = (kGelu ? 1 : 0) | (kRequant ? 2 : 0);
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(pair::kThreads);
  cfg.dynamicSmemBytes = pair::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!d->pair_ready[idx]) {
      cudaFuncAttributes fa;
      cudaError_t e = cudaFuncGetAttributes(&fa, kern);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes(gemm pair)");
      if (fa.numRegs < static_cast<int>(pair::kLaunchRegs))
        return fail(LTXFP8_ERR_CUDA, "pair gemm kernel compiled with %d registers/thread, register split needs %u",
                    fa.numRegs, pair::kLaunchRegs);
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pair::kSmemBytes);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm pair smem)");
      // A persistent grid must fit in one wave: launch exactly as many clusters as can be resident.
      cfg.gridDim = dim3(2 * (d->sms / 2));
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters(gemm pair)");
      if (n < 1) return fail(LTXFP8_ERR_CUDA, "no 2-CTA cluster of the pair gemm fits on this device");
      d->pair_clusters = n;
      d->pair_ready[idx] = true;
    }
  }
  const int clusters = p.total_tiles < d->pair_clusters ? p.total_tiles : d->pair_clusters;
  cfg.gridDim = dim3(2 * clusters);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, b, lx, lb, md, mq, p);
  if (e != cudaSuccess) return cuda_fail(e, "gemm pair launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm pair launch");
  return LTXFP8_OK;
}

// Self-test of the failure path: one warp waits on an mbarrier nothing will
// arrive on, with a short limit; the bounded wait records kStSelftest and the
// kernel returns normally.
constexpr unsigned int kStSelftest = 0x5E1F0001u;

__global__ void selftest_wait_kernel(unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbarrier_init();
  }
  __syncwarp();
  (void)mbar_wait(&bar, 0u, kStSelftest, limit_ns);
}

// Producers: per-row chunk count (16 B per lane per load) for a row of H bf16.
int producer_chunks(int64_t H) {
  const int64_t n = (H / 8 + 31) / 32;
  return n <= 4 ? 4 : n <= 8 ? 8 : n <= 16 ? 16 : n <= 32 ? 32 : 0;
}

int producer_check(const char* name, int64_t M, int64_t H, int flags) {
  if (M < 0 || H <= 0 || H % 128 != 0 || H > 8192)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "%s: need H %% 128 == 0, 0 < H <= 8192, M >= 0 (M=%lld H=%lld)", name,
                (long long)M, (long long)H);
  if (M > (static_cast<int64_t>(1) << 31) * kProdWarps)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "%s: too many rows", name);
  if (flags != LTXFP8_QUANT_TORCH && flags != LTXFP8_QUANT_TRITON)
    return fail(LTXFP8_ERR_INVALID_ARGUMENT, "%s: unknown quant mode %d", name, flags);
  return LTXFP8_OK;
}

int producer_out(const char* name, int64_t M, void* q, float* sfa, int64_t sfa_ld, void* out, bool allow_bf16,
                 ProducerOut* o) {
  o->q = static_cast<uint8_t*>(q);
  o->sfa = sfa;
  o->sfa_ld = sfa_ld;
  o->out = static_cast<__nv_bfloat16*>(out);
  if (q) {
    if (!sfa) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "%s: sfa is null", name);
    if (sfa_ld < M) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "%s: sfa_ld < M", name);
    if (!aligned(q, 16) || !aligned(sfa, 4)) return fail(LTXFP8_ERR_MISALIGNED, "%s: q must be 16-byte aligned", name);
  } else {
    if (!allow_bf16) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "%s: q is null", name);
    if (!out) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "%s: need q or out", name);
    if (!aligned(out, 16)) return fail(LTXFP8_ERR_MISALIGNED, "%s: out must be 16-byte aligned", name);
  }
  return LTXFP8_OK;
}

template <int kChunks, int kMode>
cudaError_t adanorm_launch(const DeviceInfo* d, cudaStream_t s, const __nv_bfloat16* x, int64_t M, int64_t S, int H,
                           const __nv_bfloat16* sc, int64_t sc_bs, int64_t sc_ss, const __nv_bfloat16* sh,
                           int64_t sh_bs, int64_t sh_ss, ProducerOut o) {
  (void)d;
  dim3 grid(static_cast<unsigned>((M + kProdWarps - 1) / kProdWarps));
  adanorm_quant_kernel<kChunks, kMode><<<grid, kProdWarps * 32, 0, s>>>(x, M, S, H, sc, sc_bs, sc_ss, sh, sh_bs,
                                                                        sh_ss, o);
  return cudaGetLastError();
}

template <int kChunks, int kMode>
cudaError_t rms_fma_launch(const DeviceInfo* d, cudaStream_t s, __nv_bfloat16* x, const __nv_bfloat16* y, int64_t M,
                           int64_t S, int H, const __nv_bfloat16* z, int64_t z_bs, int64_t z_ss, ProducerOut o) {
  (void)d;
  dim3 grid(static_cast<unsigned>((M + kProdWarps - 1) / kProdWarps));
  if (o.q)
    rms_fma_kernel<kChunks, kMode, true><<<grid, kProdWarps * 32, 0, s>>>(x, y, M, S, H, z, z_bs, z_ss, o);
  else
    rms_fma_kernel<kChunks, kMode, false><<<grid, kProdWarps * 32, 0, s>>>(x, y, M, S, H, z, z_bs, z_ss, o);
  return cudaGetLastError();
}

template <int kChunks, int kMode>
cudaError_t gated_launch(const DeviceInfo* d, cudaStream_t s, const __nv_bfloat16* x, const void* g, bool g_f32,
                         int64_t M, int H, int heads, ProducerOut o) {
  (void)d;
  dim3 grid(static_cast<unsigned>((M + kProdWarps - 1) / kProdWarps));
  if (o.q) {
    if (g_f32) gated_attention_kernel<kChunks, kMode, true, true><<<grid, kProdWarps * 32, 0, s>>>(x, g, M, H, heads, o);
    else gated_attention_kernel<kChunks, kMode, true, false><<<grid, kProdWarps * 32, 0, s>>>(x, g, M, H, heads, o);
  } else {
    if (g_f32) gated_attention_kernel<kChunks, kMode, false, true><<<grid, kProdWarps * 32, 0, s>>>(x, g, M, H, heads, o);
    else gated_attention_kernel<kChunks, kMode, false, false><<<grid, kProdWarps * 32, 0, s>>>(x, g, M, H, heads, o);
  }
  return cudaGetLastError();
}

// err = fn<kChunks, kMode>(args...) for the row length's chunk count and the mode.
#define LTXFP8_PRODUCER_DISPATCH(err, fn, chunks, mode, ...)                                        \
  do {                                                                                             \
    const bool tri_ = (mode) == LTXFP8_QUANT_TRITON;                                               \
    switch (chunks) {                                                                              \
      case 4: err = tri_ ? fn<4, kQuantTriton>(__VA_ARGS__) : fn<4, kQuantTorch>(__VA_ARGS__); break;     \
      case 8: err = tri_ ? fn<8, kQuantTriton>(__VA_ARGS__) : fn<8, kQuantTorch>(__VA_ARGS__); break;     \
      case 16: err = tri_ ? fn<16, kQuantTriton>(__VA_ARGS__) : fn<16, kQuantTorch>(__VA_ARGS__); break;  \
      default: err = tri_ ? fn<32, kQuantTriton>(__VA_ARGS__) : fn<32, kQuantTorch>(__VA_ARGS__); break;  \
    }                                                                                              \
  } while (0)

}  // namespace

extern "C" {

int ltxfp8_version(void) { return (1 << 16) | 0; }

const char* ltxfp8_last_error(void) { return t_last_error.c_str(); }

int ltxfp8_quantize_1x128(const void* x, int64_t M, int64_t K, int64_t x_ld, void* q, int64_t q_ld, float* sfa,
                          int64_t sfa_ld, int flags, void* stream) {
  if (M < 0 || K <= 0 || K % 128 != 0) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "quantize: need K %% 128 == 0, K > 0, M >= 0 (M=%lld K=%lld)", (long long)M, (long long)K);
  if (flags != LTXFP8_QUANT_TORCH && flags != LTXFP8_QUANT_TRITON) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "quantize: unknown mode %d", flags);
  if (M == 0) return LTXFP8_OK;
  if (!x || !q || !sfa) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "quantize: null pointer");
  if (x_ld < K || q_ld < K || sfa_ld < M) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "quantize: leading dimension too small");
  if (!aligned(x, 16) || x_ld % 8 != 0) return fail(LTXFP8_ERR_MISALIGNED, "quantize: x must be 16-byte aligned with x_ld %% 8 == 0");
  if (!aligned(q, 8) || q_ld % 8 != 0) return fail(LTXFP8_ERR_MISALIGNED, "quantize: q must be 8-byte aligned with q_ld %% 8 == 0");
  if (!aligned(sfa, 4)) return fail(LTXFP8_ERR_MISALIGNED, "quantize: sfa must be 4-byte aligned");
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  const int64_t KB = K / 128;
  dim3 grid(static_cast<unsigned>((M + kQuantRowsPerBlock - 1) / kQuantRowsPerBlock),
            static_cast<unsigned>((KB + kQuantGroupsPerThread - 1) / kQuantGroupsPerThread));
  if (grid.y > 65535u) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "quantize: K too large");
  auto s = static_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* qb = static_cast<uint8_t*>(q);
  if (flags == LTXFP8_QUANT_TRITON)
    quant_act_1x128_kernel<kQuantTriton><<<grid, 256, 0, s>>>(xb, x_ld, M, KB, qb, q_ld, sfa, sfa_ld);
  else
    quant_act_1x128_kernel<kQuantTorch><<<grid, 256, 0, s>>>(xb, x_ld, M, KB, qb, q_ld, sfa, sfa_ld);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
  return LTXFP8_OK;
}

int ltxfp8_quantize_weight_128x128(const void* w, int dtype, int64_t N, int64_t K, void* q, float* sfb,
                                   void* stream) {
  if (N <= 0 || K <= 0 || N % 128 != 0 || K % 128 != 0)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "quantize_weight: N and K must be positive multiples of 128 (N=%lld K=%lld)", (long long)N, (long long)K);
  if (dtype < LTXFP8_DTYPE_F32 || dtype > LTXFP8_DTYPE_F16) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "quantize_weight: unknown dtype %d", dtype);
  if (!w || !q || !sfb) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "quantize_weight: null pointer");
  if (!aligned(w, 16) || !aligned(q, 16) || !aligned(sfb, 4)) return fail(LTXFP8_ERR_MISALIGNED, "quantize_weight: w and q must be 16-byte aligned");
  if (N / 128 > 65535) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "quantize_weight: N too large");
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  dim3 grid(static_cast<unsigned>(K / 128), static_cast<unsigned>(N / 128));
  quant_weight_128x128_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(w, dtype, K, K / 128,
                                                                                    static_cast<uint8_t*>(q), sfb,
                                                                                    448.0f);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "quantize_weight launch");
  return LTXFP8_OK;
}

int ltxfp8_quantize_weight_128x128_scaled(const void* w, int dtype, int64_t N, int64_t K, float scale_max, void* q,
                                          float* sfb, void* stream) {
  if (!(scale_max > 0.0f) || !(scale_max <= 448.0f))
    return fail(LTXFP8_ERR_INVALID_ARGUMENT, "quantize_weight_scaled: scale_max must be in (0, 448]");
  if (N <= 0 || K <= 0 || N % 128 != 0 || K % 128 != 0)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "quantize_weight_scaled: N and K must be positive multiples of 128 (N=%lld K=%lld)", (long long)N, (long long)K);
  if (dtype < LTXFP8_DTYPE_F32 || dtype > LTXFP8_DTYPE_F16) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "quantize_weight_scaled: unknown dtype %d", dtype);
  if (!w || !q || !sfb) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "quantize_weight_scaled: null pointer");
  if (!aligned(w, 16) || !aligned(q, 16) || !aligned(sfb, 4)) return fail(LTXFP8_ERR_MISALIGNED, "quantize_weight_scaled: w and q must be 16-byte aligned");
  if (N / 128 > 65535) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "quantize_weight_scaled: N too large");
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  dim3 grid(static_cast<unsigned>(K / 128), static_cast<unsigned>(N / 128));
  quant_weight_128x128_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(w, dtype, K, K / 128,
                                                                                    static_cast<uint8_t*>(q), sfb,
                                                                                    scale_max);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "quantize_weight_scaled launch");
  return LTXFP8_OK;
}

static int fp6_launch(bool pack, const void* x, int64_t m, int64_t n, void* out, void* stream) {
  const char* name = pack ? "fp6_pack" : "fp6_unpack";
  if (m < 0 || n <= 0 || n % 8 != 0)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "%s: need n %% 8 == 0, n > 0 (n=%lld)", name, (long long)n);
  if (m == 0) return LTXFP8_OK;
  if (!x || !out) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned(pack ? x : out, 8) || !aligned(pack ? out : x, 2))
    return fail(LTXFP8_ERR_MISALIGNED, "%s: the unpacked buffer must be 8-byte and the packed one 2-byte aligned", name);
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  const int64_t groups = m * (n / 8);
  int64_t blocks = (groups + 255) / 256;
  const int64_t cap = static_cast<int64_t>(d->sms) * 8;
  if (blocks > cap) blocks = cap;
  auto s = static_cast<cudaStream_t>(stream);
  if (pack)
    fp6_pack_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(static_cast<const uint8_t*>(x), groups,
                                                                   static_cast<uint8_t*>(out));
  else
    fp6_unpack_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(static_cast<const uint8_t*>(x), groups,
                                                                     static_cast<uint8_t*>(out));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, name);
  return LTXFP8_OK;
}

int ltxfp8_fp6_pack(const void* x, int64_t m, int64_t n, void* out, void* stream) {
  return fp6_launch(true, x, m, n, out, stream);
}

int ltxfp8_fp6_unpack(const void* x, int64_t m, int64_t n, void* out, void* stream) {
  return fp6_launch(false, x, m, n, out, stream);
}

int ltxfp8_fp6_to_tc(const void* w6, const float* sfb, int64_t N, int64_t K, void* w6_tc, float* sfb_tc,
                     void* stream) {
  if (N <= 0 || K <= 0 || N % 128 != 0 || K % 128 != 0)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "fp6_to_tc: N and K must be positive multiples of 128");
  if (!w6 || !sfb || !w6_tc || !sfb_tc) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "fp6_to_tc: null pointer");
  if (!aligned(w6, 4) || !aligned(w6_tc, 32) || !aligned(sfb, 4) || !aligned(sfb_tc, 4))
    return fail(LTXFP8_ERR_MISALIGNED, "fp6_to_tc: packed weight 4-byte, output 32-byte aligned");
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  const int64_t chunks = N * K / 16;
  int64_t blocks = (chunks + 255) / 256;
  const int64_t cap = static_cast<int64_t>(d->sms) * 8;
  if (blocks > cap) blocks = cap;
  fp6_to_tc_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(w6), chunks, static_cast<uint8_t*>(w6_tc), sfb, (N / 128) * (K / 128), sfb_tc);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fp6_to_tc launch");
  return LTXFP8_OK;
}

int ltxfp8_dequantize_1x128(const void* q, const float* scales, int64_t row_stride, int64_t col_stride, int64_t M,
                            int64_t K, void* out, void* stream) {
  if (M < 0 || K <= 0 || K % 128 != 0) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "dequantize: K must be a positive multiple of 128");
  if (M == 0) return LTXFP8_OK;
  if (!q || !scales || !out) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "dequantize: null pointer");
  if (!aligned(q, 16) || !aligned(out, 16) || !aligned(scales, 4)) return fail(LTXFP8_ERR_MISALIGNED, "dequantize: q and out must be 16-byte aligned");
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  const int64_t chunks = M * (K / 16);
  int64_t blocks = (chunks + 255) / 256;
  const int64_t cap = static_cast<int64_t>(d->sms) * 8;
  if (blocks > cap) blocks = cap;
  dequant_1x128_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(q), scales, row_stride, col_stride, M, K, static_cast<__nv_bfloat16*>(out));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "dequantize launch");
  return LTXFP8_OK;
}

int ltxfp8_lora_fuse_weight(const void* q, const float* sfb, const void* delta, int64_t N, int64_t K, void* q_out,
                            float* sfb_out, void* stream) {
  if (N <= 0 || K <= 0 || N % 128 != 0 || K % 128 != 0)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "lora_fuse_weight: N and K must be positive multiples of 128 (N=%lld K=%lld)",
                (long long)N, (long long)K);
  if (!q || !sfb || !delta || !q_out || !sfb_out) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "lora_fuse_weight: null pointer");
  if (!aligned(q, 16) || !aligned(delta, 16) || !aligned(q_out, 16) || !aligned(sfb, 4) || !aligned(sfb_out, 4))
    return fail(LTXFP8_ERR_MISALIGNED, "lora_fuse_weight: q, delta, q_out must be 16-byte aligned");
  if (N / 128 > 65535) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "lora_fuse_weight: N too large");
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  dim3 grid(static_cast<unsigned>(K / 128), static_cast<unsigned>(N / 128));
  lora_fuse_weight_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(q), sfb, static_cast<const __nv_bfloat16*>(delta), K, K / 128,
      static_cast<uint8_t*>(q_out), sfb_out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "lora_fuse_weight launch");
  return LTXFP8_OK;
}

int ltxfp8_adanorm_quantize(const void* x, int64_t B, int64_t S, int64_t H, const void* scale,
                            int64_t scale_bstride, int64_t scale_sstride, const void* shift, int64_t shift_bstride,
                            int64_t shift_sstride, void* q, float* sfa, int64_t sfa_ld, int flags, void* stream) {
  if (B < 0 || S < 0) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "adanorm: negative B or S");
  const int64_t M = B * S;
  int rc = producer_check("adanorm", M, H, flags);
  if (rc) return rc;
  if (M == 0) return LTXFP8_OK;
  if (!x || !scale || !shift) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "adanorm: null pointer");
  if (!aligned(x, 16) || !aligned(scale, 16) || !aligned(shift, 16) || scale_bstride % 8 || scale_sstride % 8 ||
      shift_bstride % 8 || shift_sstride % 8)
    return fail(LTXFP8_ERR_MISALIGNED, "adanorm: x, scale, shift must be 16-byte aligned with strides %% 8 == 0");
  ProducerOut o;
  rc = producer_out("adanorm", M, q, sfa, sfa_ld, nullptr, false, &o);
  if (rc) return rc;
  DeviceInfo* d;
  rc = device_info(&d);
  if (rc) return rc;
  cudaError_t e = cudaSuccess;
  LTXFP8_PRODUCER_DISPATCH(e, adanorm_launch, producer_chunks(H), flags, d, static_cast<cudaStream_t>(stream),
                           static_cast<const __nv_bfloat16*>(x), M, S, static_cast<int>(H),
                           static_cast<const __nv_bfloat16*>(scale), scale_bstride, scale_sstride,
                           static_cast<const __nv_bfloat16*>(shift), shift_bstride, shift_sstride, o);
  if (e != cudaSuccess) return cuda_fail(e, "adanorm launch");
  return LTXFP8_OK;
}

int ltxfp8_rms_fma(void* x, const void* y, int64_t B, int64_t S, int64_t H, const void* z, int64_t z_bstride,
                   int64_t z_sstride, void* q, float* sfa, int64_t sfa_ld, void* out, int flags, void* stream) {
  if (B < 0 || S < 0) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "rms_fma: negative B or S");
  const int64_t M = B * S;
  int rc = producer_check("rms_fma", M, H, flags);
  if (rc) return rc;
  if (M == 0) return LTXFP8_OK;
  if (!x || !y || !z) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "rms_fma: null pointer");
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(z, 16) || z_bstride % 8 || z_sstride % 8)
    return fail(LTXFP8_ERR_MISALIGNED, "rms_fma: x, y, z must be 16-byte aligned with strides %% 8 == 0");
  ProducerOut o;
  rc = producer_out("rms_fma", M, q, sfa, sfa_ld, out, true, &o);
  if (rc) return rc;
  DeviceInfo* d;
  rc = device_info(&d);
  if (rc) return rc;
  cudaError_t e = cudaSuccess;
  LTXFP8_PRODUCER_DISPATCH(e, rms_fma_launch, producer_chunks(H), flags, d, static_cast<cudaStream_t>(stream),
                           static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(y), M, S,
                           static_cast<int>(H), static_cast<const __nv_bfloat16*>(z), z_bstride, z_sstride, o);
  if (e != cudaSuccess) return cuda_fail(e, "rms_fma launch");
  return LTXFP8_OK;
}

int ltxfp8_gated_attention(const void* x, const void* gate_logits, int gate_dtype, int64_t M, int64_t H,
                           int64_t heads, void* q, float* sfa, int64_t sfa_ld, void* out, int flags, void* stream) {
  int rc = producer_check("gated_attention", M, H, flags);
  if (rc) return rc;
  if (heads <= 0 || heads > 64 || H % heads != 0 || (H / heads) % 8 != 0)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE,
                "gated_attention: need 1 <= heads <= 64 and H / heads a multiple of 8 (H=%lld heads=%lld)",
                (long long)H, (long long)heads);
  if (gate_dtype != LTXFP8_DTYPE_BF16 && gate_dtype != LTXFP8_DTYPE_F32)
    return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gated_attention: gate logits must be bf16 or fp32");
  if (M == 0) return LTXFP8_OK;
  if (!x || !gate_logits) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gated_attention: null pointer");
  if (!aligned(x, 16) || !aligned(gate_logits, gate_dtype == LTXFP8_DTYPE_F32 ? 4 : 2))
    return fail(LTXFP8_ERR_MISALIGNED, "gated_attention: x must be 16-byte aligned");
  ProducerOut o;
  rc = producer_out("gated_attention", M, q, sfa, sfa_ld, out, true, &o);
  if (rc) return rc;
  DeviceInfo* d;
  rc = device_info(&d);
  if (rc) return rc;
  cudaError_t e = cudaSuccess;
  LTXFP8_PRODUCER_DISPATCH(e, gated_launch, producer_chunks(H), flags, d, static_cast<cudaStream_t>(stream),
                           static_cast<const __nv_bfloat16*>(x), gate_logits, gate_dtype == LTXFP8_DTYPE_F32, M,
                           static_cast<int>(H), static_cast<int>(heads), o);
  if (e != cudaSuccess) return cuda_fail(e, "gated_attention launch");
  return LTXFP8_OK;
}

int ltxfp8_rms_norm_rope(const void* x, int64_t rows, int64_t dim, const void* cos_freqs, const void* sin_freqs,
                         int64_t freq_row_stride, const void* weights, void* out, int out_fp8, void* stream) {
  if (rows < 0 || dim <= 0 || dim % 8 != 0 || dim > 8192)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "rms_norm_rope: need dim %% 8 == 0, 0 < dim <= 8192 (dim=%lld)",
                (long long)dim);
  if (rows == 0) return LTXFP8_OK;
  if (rows > (static_cast<int64_t>(1) << 31) * kProdWarps) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "rms_norm_rope: too many rows");
  if (!x || !cos_freqs || !sin_freqs || !out) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "rms_norm_rope: null pointer");
  if (!aligned(x, 16) || !aligned(cos_freqs, 16) || !aligned(sin_freqs, 16) || !aligned(out, 16) ||
      (weights && !aligned(weights, 16)) || freq_row_stride % 8 != 0)
    return fail(LTXFP8_ERR_MISALIGNED, "rms_norm_rope: operands must be 16-byte aligned, freq_row_stride %% 8 == 0");
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  const int ch = producer_chunks(dim);
  dim3 grid(static_cast<unsigned>((rows + kProdWarps - 1) / kProdWarps));
  auto s = static_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* cb = static_cast<const __nv_bfloat16*>(cos_freqs);
  const auto* sb = static_cast<const __nv_bfloat16*>(sin_freqs);
  const auto* wb = static_cast<const __nv_bfloat16*>(weights);
  const int di = static_cast<int>(dim);
#define LTXFP8_ROPE_LAUNCH(C, A, O) \
  rms_norm_rope_kernel<C, A, O><<<grid, kProdWarps * 32, 0, s>>>(xb, rows, di, cb, sb, freq_row_stride, wb, out)
#define LTXFP8_ROPE_OUT(C, A) \
  do { if (out_fp8) LTXFP8_ROPE_LAUNCH(C, A, kRopeE4m3Torch); else LTXFP8_ROPE_LAUNCH(C, A, kRopeBf16); } while (0)
#define LTXFP8_ROPE_AFF(C) do { if (wb) LTXFP8_ROPE_OUT(C, true); else LTXFP8_ROPE_OUT(C, false); } while (0)
  switch (ch) {
    case 4: LTXFP8_ROPE_AFF(4); break;
    case 8: LTXFP8_ROPE_AFF(8); break;
    case 16: LTXFP8_ROPE_AFF(16); break;
    default: LTXFP8_ROPE_AFF(32); break;
  }
#undef LTXFP8_ROPE_AFF
#undef LTXFP8_ROPE_OUT
#undef LTXFP8_ROPE_LAUNCH
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "rms_norm_rope launch");
  return LTXFP8_OK;
}

int ltxfp8_rms_norm_split_rope(const void* x, int64_t B, int64_t S, int64_t H, int64_t heads, const void* cos_freqs,
                               int64_t cos_bstride, int64_t cos_hstride, int64_t cos_sstride, const void* sin_freqs,
                               int64_t sin_bstride, int64_t sin_hstride, int64_t sin_sstride, const void* weights,
                               void* out, int out_fp8, void* stream) {
  if (B < 0 || S < 0) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "rms_norm_split_rope: negative B or S");
  const int64_t M = B * S;
  int rc = producer_check("rms_norm_split_rope", M, H, LTXFP8_QUANT_TORCH);
  if (rc) return rc;
  const int64_t dh = heads > 0 ? H / heads : 0;
  if (heads <= 0 || H % heads != 0 || !(dh == 16 || dh == 32 || dh == 64 || dh == 128 || dh == 256))
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "rms_norm_split_rope: head size H / heads must be 16, 32, 64, 128 or 256 "
                "(H=%lld heads=%lld)", (long long)H, (long long)heads);
  if (M == 0) return LTXFP8_OK;
  if (!x || !cos_freqs || !sin_freqs || !out) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "rms_norm_split_rope: null pointer");
  if (!aligned(x, 16) || !aligned(cos_freqs, 16) || !aligned(sin_freqs, 16) || !aligned(out, 16) ||
      (weights && !aligned(weights, 16)) || cos_bstride % 8 || cos_hstride % 8 || cos_sstride % 8 || sin_bstride % 8 ||
      sin_hstride % 8 || sin_sstride % 8)
    return fail(LTXFP8_ERR_MISALIGNED, "rms_norm_split_rope: operands must be 16-byte aligned, strides %% 8 == 0");
  DeviceInfo* d;
  rc = device_info(&d);
  if (rc) return rc;
  const int ch = producer_chunks(H);
  dim3 grid(static_cast<unsigned>((M + kProdWarps - 1) / kProdWarps));
  auto s = static_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* cb = static_cast<const __nv_bfloat16*>(cos_freqs);
  const auto* sb = static_cast<const __nv_bfloat16*>(sin_freqs);
  const auto* wb = static_cast<const __nv_bfloat16*>(weights);
  const int hi = static_cast<int>(H), ni = static_cast<int>(heads);
#define LTXFP8_SROPE_LAUNCH(C, A, O)                                                                        \
  rms_norm_split_rope_kernel<C, A, O><<<grid, kProdWarps * 32, 0, s>>>(xb, B, S, hi, ni, cb, cos_bstride,   \
                                                                       cos_hstride, cos_sstride, sb,        \
                                                                       sin_bstride, sin_hstride, sin_sstride, wb, out)
#define LTXFP8_SROPE_OUT(C, A) \
  do { if (out_fp8) LTXFP8_SROPE_LAUNCH(C, A, kRopeE4m3Sat); else LTXFP8_SROPE_LAUNCH(C, A, kRopeBf16); } while (0)
#define LTXFP8_SROPE_AFF(C) do { if (wb) LTXFP8_SROPE_OUT(C, true); else LTXFP8_SROPE_OUT(C, false); } while (0)
  switch (ch) {
    case 4: LTXFP8_SROPE_AFF(4); break;
    case 8: LTXFP8_SROPE_AFF(8); break;
    case 16: LTXFP8_SROPE_AFF(16); break;
    default: LTXFP8_SROPE_AFF(32); break;
  }
#undef LTXFP8_SROPE_AFF
#undef LTXFP8_SROPE_OUT
#undef LTXFP8_SROPE_LAUNCH
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "rms_norm_split_rope launch");
  return LTXFP8_OK;
}

int ltxfp8_gelu_quantize_1x128(const void* x, int64_t M, int64_t K, int64_t x_ld, void* q, int64_t q_ld, float* sfa,
                               int64_t sfa_ld, int flags, void* stream) {
  if (M < 0 || K <= 0 || K % 128 != 0) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "gelu_quantize: need K %% 128 == 0, K > 0, M >= 0 (M=%lld K=%lld)", (long long)M, (long long)K);
  if (flags != LTXFP8_QUANT_TORCH && flags != LTXFP8_QUANT_TRITON) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gelu_quantize: unknown mode %d", flags);
  if (M == 0) return LTXFP8_OK;
  if (!x || !q || !sfa) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gelu_quantize: null pointer");
  if (x_ld < K || q_ld < K || sfa_ld < M) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gelu_quantize: leading dimension too small");
  if (!aligned(x, 16) || x_ld % 8 != 0) return fail(LTXFP8_ERR_MISALIGNED, "gelu_quantize: x must be 16-byte aligned with x_ld %% 8 == 0");
  if (!aligned(q, 8) || q_ld % 8 != 0) return fail(LTXFP8_ERR_MISALIGNED, "gelu_quantize: q must be 8-byte aligned with q_ld %% 8 == 0");
  if (!aligned(sfa, 4)) return fail(LTXFP8_ERR_MISALIGNED, "gelu_quantize: sfa must be 4-byte aligned");
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  const int64_t KB = K / 128;
  dim3 grid(static_cast<unsigned>((M + kQuantRowsPerBlock - 1) / kQuantRowsPerBlock),
            static_cast<unsigned>((KB + kQuantGroupsPerThread - 1) / kQuantGroupsPerThread));
  if (grid.y > 65535u) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "gelu_quantize: K too large");
  auto s = static_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* qb = static_cast<uint8_t*>(q);
  if (flags == LTXFP8_QUANT_TRITON)
    gelu_quant_kernel<kQuantTriton><<<grid, 256, 0, s>>>(xb, x_ld, M, KB, qb, q_ld, sfa, sfa_ld);
  else
    gelu_quant_kernel<kQuantTorch><<<grid, 256, 0, s>>>(xb, x_ld, M, KB, qb, q_ld, sfa, sfa_ld);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gelu_quantize launch");
  return LTXFP8_OK;
}

int ltxfp8_gelu_tanh_quantize_1x128(const void* x, int64_t M, int64_t K, int64_t x_ld, void* q, int64_t q_ld,
                                    float* sfa, int64_t sfa_ld, int flags, void* stream) {
  if (M < 0 || K <= 0 || K % 128 != 0) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "gelu_tanh_quantize: need K %% 128 == 0, K > 0, M >= 0 (M=%lld K=%lld)", (long long)M, (long long)K);
  if (flags != LTXFP8_QUANT_TORCH && flags != LTXFP8_QUANT_TRITON) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gelu_tanh_quantize: unknown mode %d", flags);
  if (M == 0) return LTXFP8_OK;
  if (!x || !q || !sfa) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gelu_tanh_quantize: null pointer");
  if (x_ld < K || q_ld < K || sfa_ld < M) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gelu_tanh_quantize: leading dimension too small");
  if (!aligned(x, 16) || x_ld % 8 != 0) return fail(LTXFP8_ERR_MISALIGNED, "gelu_tanh_quantize: x must be 16-byte aligned with x_ld %% 8 == 0");
  if (!aligned(q, 8) || q_ld % 8 != 0) return fail(LTXFP8_ERR_MISALIGNED, "gelu_tanh_quantize: q must be 8-byte aligned with q_ld %% 8 == 0");
  if (!aligned(sfa, 4)) return fail(LTXFP8_ERR_MISALIGNED, "gelu_tanh_quantize: sfa must be 4-byte aligned");
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  const int64_t KB = K / 128;
  const int64_t units = ((M + kQuantRowsPerBlock - 1) / kQuantRowsPerBlock) *
                        ((KB + kGeluQuantGroups - 1) / kGeluQuantGroups);
  // Persistent grid, one wave: each CTA fills its GELU table once.
  static std::atomic<int> per_sm{0};
  if (per_sm.load() == 0) {
    int n = 0;
    cudaError_t oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gelu_tanh_quant_kernel<kQuantTriton>, 256, 0);
    if (oe != cudaSuccess) return cuda_fail(oe, "gelu_tanh_quantize occupancy");
    per_sm.store(n > 0 ? n : 1);
  }
  const int64_t cap = static_cast<int64_t>(d->sms) * per_sm.load();
  const unsigned grid = static_cast<unsigned>(units < cap ? units : cap);
  auto s = static_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* qb = static_cast<uint8_t*>(q);
  if (flags == LTXFP8_QUANT_TRITON)
    gelu_tanh_quant_kernel<kQuantTriton><<<grid, 256, 0, s>>>(xb, x_ld, M, KB, qb, q_ld, sfa, sfa_ld);
  else
    gelu_tanh_quant_kernel<kQuantTorch><<<grid, 256, 0, s>>>(xb, x_ld, M, KB, qb, q_ld, sfa, sfa_ld);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gelu_tanh_quantize launch");
  return LTXFP8_OK;
}

// One launch (plus its split-K reduction) of the GEMM over output rows
// [row0, row0 + rows): the operands and outputs of those rows are addressed by
// offsetting A, sfa, D, the requant outputs and the LoRA rows; N, K, W, sfb and
// the bias are shared.  split != nullptr: split-K with that plan, partials in
// the caller's workspace.
static int gemm_rows(DeviceInfo* d, const void* A, const float* sfa, int64_t sfa_ld, const void* W, const float* sfb,
                     const float* bias, void* D, int64_t M, int64_t N, int64_t K, const ltxfp8_epilogue& e,
                     int64_t row0, int64_t rows, const SplitPlan* split, bool use_pair, cudaStream_t stream,
                     bool w_fp6 = false) {
  const bool write_d = !e.skip_d;
  const bool lora = e.lora_ax != nullptr;
  const int tile_m = use_pair ? pair::kTileM : kBM;
  const int tile_n = use_pair ? pair::kTileN : kBN;
  const uint32_t w_rows_per_load = use_pair ? pair::kRowsPerCta : kBN;  // W rows each CTA loads
  const auto* a_rows = static_cast<const uint8_t*>(A) + row0 * K;

  CUtensorMap ma, mb, mlx, mlb;
  int rc = make_map_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, a_rows, K, rows, K, kBK, kBM);
  if (rc) return rc;
  if (w_fp6)  // 6-bit codes: K elements in K * 3 / 4 bytes per row
    rc = make_map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_16U6_ALIGN16B, W, K, N, K / 4 * 3, kBK, w_rows_per_load);
  else
    rc = make_map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, W, K, N, K, kBK, w_rows_per_load);
  if (rc) return rc;
  if (lora) {
    const auto* lx_rows = static_cast<const __nv_bfloat16*>(e.lora_ax) + row0 * e.lora_r;
    rc = make_map_2d(&mlx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lx_rows, e.lora_r, rows, e.lora_r * 2, kLoraChunk, kBM);
    if (rc) return rc;
    rc = make_map_2d(&mlb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, e.lora_b, e.lora_r, N, e.lora_r * 2, kLoraChunk,
                     w_rows_per_load);
    if (rc) return rc;
  } else {
    mlx = ma;  // unused
    mlb = mb;
  }

  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.M = static_cast<int>(rows);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.num_kb = static_cast<int>(K / kBK);
  p.num_lora = lora ? static_cast<int>((e.lora_r + kLoraChunk - 1) / kLoraChunk) : 0;
  p.m_tiles = static_cast<int>((rows + tile_m - 1) / tile_m);
  p.n_tiles = static_cast<int>((N + tile_n - 1) / tile_n);
  // Rasterisation for L2 reuse: group enough M tiles that one group's A slab is
  // ~24 MB and sweep the N tiles within the group, so the CTAs resident at one
  // time share A and W tiles through L2.  (Walking N fastest to keep a whole
  // <= 67 MB weight resident measured worse: the weight does not stay in L2.)
  int64_t gm = (24ll << 20) / (static_cast<int64_t>(tile_m) * K);
  if (gm < 1) gm = 1;
  if (gm > p.m_tiles) gm = p.m_tiles;
  p.group_m = static_cast<int>(gm);
  p.total_tiles = p.m_tiles * p.n_tiles;
  p.sfa = sfa + row0;
  p.sfa_ld = sfa_ld;
  p.sfb = sfb;
  p.bias = bias;
  p.d = write_d ? static_cast<__nv_bfloat16*>(D) + row0 * N : nullptr;
  p.q_out = e.requant_q ? static_cast<uint8_t*>(e.requant_q) + row0 * N : nullptr;
  p.s_out = e.requant_scales ? e.requant_scales + row0 : nullptr;
  p.s_out_ld = e.requant_ld;
  p.lora_alpha = e.lora_alpha;
  p.flags = (bias ? kGemmBias : 0) | (write_d ? kGemmWriteD : 0) | (lora ? kGemmLora : 0) |
            (e.gelu_tanh == LTXFP8_GELU_TANH_FAST ? kGemmGeluFast : 0) |
            (e.requant_mode == LTXFP8_QUANT_TRITON ? kGemmRequantTriton : 0) | (w_fp6 ? kGemmWeightFp6 : 0);
  p.k_splits = 1;
  p.kb_per_split = p.num_kb;
  p.ws = nullptr;
  if (split) {
    p.k_splits = split->splits;
    p.kb_per_split = split->kb_per_split;
    p.ws = static_cast<float*>(e.workspace);
  }

  const bool gelu = e.gelu_tanh != 0, requant = e.requant_q != nullptr;
  // Output maps for the staged epilogue's TMA stores (both kernels): bf16 D in
  // [32, 64] boxes, e4m3 codes in [32, 128] boxes, 128 B swizzle (the staging
  // tile's layout).
  CUtensorMap md = ma, mq = ma;
  if (!split) {
    if (write_d) {
      rc = make_map_2d(&md, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.d, N, rows, N * 2, 64, 32);
      if (rc) return rc;
    }
    if (e.requant_q) {
      rc = make_map_2d(&mq, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.q_out, N, rows, N, 128, 32);
      if (rc) return rc;
    }
  }
  if (use_pair) {
    if (gelu && requant) return gemm_pair_launch<true, true>(d, ma, mb, mlx, mlb, md, mq, p, stream);
    if (gelu) return gemm_pair_launch<true, false>(d, ma, mb, mlx, mlb, md, mq, p, stream);
    if (requant) return gemm_pair_launch<false, true>(d, ma, mb, mlx, mlb, md, mq, p, stream);
    return gemm_pair_launch<false, false>(d, ma, mb, mlx, mlb, md, mq, p, stream);
  }
  if (gelu && requant) return gemm_launch_full<true, true>(d, ma, mb, mlx, mlb, md, mq, p, stream);
  if (gelu) return gemm_launch_full<true, false>(d, ma, mb, mlx, mlb, md, mq, p, stream);
  if (requant) return gemm_launch_full<false, true>(d, ma, mb, mlx, mlb, md, mq, p, stream);
  return gemm_launch_full<false, false>(d, ma, mb, mlx, mlb, md, mq, p, stream);
}

static int gemm_entry(const void* A, const float* sfa, int64_t sfa_ld, const void* W, const float* sfb,
                      const float* bias, void* D, int64_t M, int64_t N, int64_t K, const ltxfp8_epilogue* ep,
                      void* stream, bool w_fp6) {
  ltxfp8_epilogue none;
  memset(&none, 0, sizeof(none));
  const ltxfp8_epilogue& e = ep ? *ep : none;
  if (M < 1 || N < 128 || K < 128 || N % 128 != 0 || K % 128 != 0)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "gemm: need M >= 1 and N, K positive multiples of 128 (M=%lld N=%lld K=%lld)",
                (long long)M, (long long)N, (long long)K);
  if (M > 0x7FFFFFFF || N > 0x7FFFFFFF || K > 0x7FFFFFFF) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "gemm: dimension exceeds int32");
  if (!A || !sfa || !W || !sfb) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm: null operand");
  if (sfa_ld < M) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm: sfa_ld (%lld) < M (%lld)", (long long)sfa_ld, (long long)M);
  const bool write_d = !e.skip_d;
  if (write_d && !D) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm: D is null");
  if (!write_d && !e.requant_q) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm: skip_d needs requant_q");
  if (!aligned(A, 16) || !aligned(W, 16)) return fail(LTXFP8_ERR_MISALIGNED, "gemm: A and W must be 16-byte aligned");
  if (w_fp6 && !aligned(W, 32)) return fail(LTXFP8_ERR_MISALIGNED, "gemm_fp6w: W must be 32-byte aligned");
  if (write_d && !aligned(D, 16)) return fail(LTXFP8_ERR_MISALIGNED, "gemm: D must be 16-byte aligned");
  if (!aligned(sfa, 4) || !aligned(sfb, 4)) return fail(LTXFP8_ERR_MISALIGNED, "gemm: scales must be 4-byte aligned");
  if (bias && !aligned(bias, 16)) return fail(LTXFP8_ERR_MISALIGNED, "gemm: bias must be 16-byte aligned");
  if (e.gelu_tanh < LTXFP8_GELU_NONE || e.gelu_tanh > LTXFP8_GELU_TANH_FAST)
    return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm: unknown gelu_tanh mode %d", e.gelu_tanh);
  if (e.requant_mode != LTXFP8_QUANT_TORCH && e.requant_mode != LTXFP8_QUANT_TRITON)
    return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm: unknown requant_mode %d", e.requant_mode);
  if (e.requant_q) {
    if (!e.requant_scales) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm: requant_scales is null");
    if (e.requant_ld < M) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm: requant_ld < M");
    if (!aligned(e.requant_q, 16) || !aligned(e.requant_scales, 4)) return fail(LTXFP8_ERR_MISALIGNED, "gemm: requant outputs misaligned");
  }
  const bool lora = e.lora_ax != nullptr;
  if (lora) {
    if (!e.lora_b) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm: lora_b is null");
    if (e.lora_r < 16 || e.lora_r > 256 || e.lora_r % 16 != 0) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "gemm: lora_r must be a multiple of 16 in [16, 256]");
    if (!aligned(e.lora_ax, 16) || !aligned(e.lora_b, 16)) return fail(LTXFP8_ERR_MISALIGNED, "gemm: LoRA operands must be 16-byte aligned");
  }
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;

  // Default: the one-CTA kernel.  The CTA-pair kernel (256-row tiles over two
  // SMs) is selected explicitly; it halves the W bytes each SM streams but is
  // not yet faster on the FFN shapes.
  // 6-bit weights run on the one-CTA kernel only.
  auto s = static_cast<cudaStream_t>(stream);
  const bool use_pair = !w_fp6 && g_gemm_variant.load() == 2;
  if (use_pair) return gemm_rows(d, A, sfa, sfa_ld, W, sfb, bias, D, M, N, K, e, 0, M, nullptr, true, s);
  const GemmPlan g = gemm_plan(d->sms, M, N, K);
  const size_t need = splitk_bytes(g);
  if (need == 0 || !e.workspace || need > e.workspace_bytes)
    return gemm_rows(d, A, sfa, sfa_ld, W, sfb, bias, D, M, N, K, e, 0, M, nullptr, false, s, w_fp6);
  if (!aligned(e.workspace, 16)) return fail(LTXFP8_ERR_MISALIGNED, "gemm: workspace must be 16-byte aligned");
  if (g.split_row0 > 0) {
    rc = gemm_rows(d, A, sfa, sfa_ld, W, sfb, bias, D, M, N, K, e, 0, g.split_row0, nullptr, false, s, w_fp6);
    if (rc) return rc;
  }
  return gemm_rows(d, A, sfa, sfa_ld, W, sfb, bias, D, M, N, K, e, g.split_row0, M - g.split_row0, &g.split, false, s,
                   w_fp6);
}

int ltxfp8_gemm(const void* A, const float* sfa, int64_t sfa_ld, const void* W, const float* sfb,
                const float* bias, void* D, int64_t M, int64_t N, int64_t K, const ltxfp8_epilogue* ep,
                void* stream) {
  return gemm_entry(A, sfa, sfa_ld, W, sfb, bias, D, M, N, K, ep, stream, false);
}

int ltxfp8_gemm_fp6w(const void* A, const float* sfa, int64_t sfa_ld, const void* W6, const float* sfb6,
                     const float* bias, void* D, int64_t M, int64_t N, int64_t K, const ltxfp8_epilogue* ep,
                     void* stream) {
  return gemm_entry(A, sfa, sfa_ld, W6, sfb6, bias, D, M, N, K, ep, stream, true);
}

int ltxfp8_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, size_t* bytes) {
  if (!bytes) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm_workspace_bytes: null pointer");
  *bytes = 0;
  if (M < 1 || N < 128 || K < 128 || N % 128 != 0 || K % 128 != 0) return LTXFP8_OK;
  if (g_gemm_variant.load() == 2) return LTXFP8_OK;
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  *bytes = splitk_bytes(gemm_plan(d->sms, M, N, K));
  return LTXFP8_OK;
}

int ltxfp8_gemm_plan_for_sms(int64_t M, int64_t N, int64_t K, int sms, ltxfp8_gemm_plan_info* info) {
  if (!info) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm_plan: null pointer");
  memset(info, 0, sizeof(*info));
  if (M < 1 || N < 128 || K < 128 || N % 128 != 0 || K % 128 != 0)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "gemm_plan: need M >= 1 and N, K positive multiples of 128");
  if (sms < 1) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm_plan: sms must be positive");
  info->launches = 1;
  info->splits = 1;
  info->split_row0 = M;
  const GemmPlan g = gemm_plan(sms, M, N, K);
  if (g.split.splits < 2) return LTXFP8_OK;
  info->workspace_bytes = splitk_bytes(g);
  info->launches = gemm_plan_launches(g);
  info->splits = g.split.splits;
  info->split_row0 = g.split_row0;
  return LTXFP8_OK;
}

int ltxfp8_gemm_plan(int64_t M, int64_t N, int64_t K, ltxfp8_gemm_plan_info* info) {
  if (!info) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm_plan: null pointer");
  memset(info, 0, sizeof(*info));
  if (M < 1 || N < 128 || K < 128 || N % 128 != 0 || K % 128 != 0)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "gemm_plan: need M >= 1 and N, K positive multiples of 128");
  info->launches = 1;
  info->splits = 1;
  info->split_row0 = M;
  if (g_gemm_variant.load() == 2) return LTXFP8_OK;
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  return ltxfp8_gemm_plan_for_sms(M, N, K, d->sms, info);
}

int ltxfp8_gemm_static_scratch(const void* A, const float* sfa, int64_t sfa_ld, const void* W, const float* sfb,
                               const float* bias, void* D, int64_t M, int64_t N, int64_t K,
                               const ltxfp8_epilogue* ep, void* stream) {
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  {
    // Once per device, with that device current: the device address of the array.
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!d->static_scratch) {
      void* ptr = nullptr;
      cudaError_t err = cudaGetSymbolAddress(&ptr, g_gemm_static_scratch);
      if (err != cudaSuccess) return cuda_fail(err, "gemm_static_scratch: cudaGetSymbolAddress");
      d->static_scratch = static_cast<float*>(ptr);
    }
  }
  size_t need = 0;
  rc = ltxfp8_gemm_workspace_bytes(M, N, K, &need);
  if (rc) return rc;
  if (need > kStaticScratchBytes)
    return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE,
                "gemm_static_scratch: M=%lld N=%lld K=%lld needs %zu bytes of split-K scratch, the static array holds %zu",
                (long long)M, (long long)N, (long long)K, need, kStaticScratchBytes);
  ltxfp8_epilogue e;
  if (ep) {
    e = *ep;
  } else {
    memset(&e, 0, sizeof(e));
  }
  // Each split writes every partial the reduction reads before the reduction
  // runs, so nothing in the array has to start at zero.
  e.workspace = need ? d->static_scratch : nullptr;
  e.workspace_bytes = need ? kStaticScratchBytes : 0;
  return ltxfp8_gemm(A, sfa, sfa_ld, W, sfb, bias, D, M, N, K, &e, stream);
}

int ltxfp8_gemm_set_variant(int variant) {
  if (variant < 0 || variant > 2) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "gemm_set_variant: unknown variant %d", variant);
  g_gemm_variant.store(variant);
  return LTXFP8_OK;
}

int ltxfp8_lora_a(const void* x, const void* lora_a, void* ax, int64_t M, int64_t K, int64_t r, void* stream) {
  if (M < 0 || K <= 0 || K % 64 != 0) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "lora_a: K must be a positive multiple of 64");
  if (r < 16 || r > 256 || r % 16 != 0) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "lora_a: r must be a multiple of 16 in [16, 256]");
  if (M == 0) return LTXFP8_OK;
  if (M > 0x7FFFFFFF || K > 0x7FFFFFFF) return fail(LTXFP8_ERR_UNSUPPORTED_SHAPE, "lora_a: dimension exceeds int32");
  if (!x || !lora_a || !ax) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "lora_a: null pointer");
  if (!aligned(x, 16) || !aligned(lora_a, 16) || !aligned(ax, 16)) return fail(LTXFP8_ERR_MISALIGNED, "lora_a: operands must be 16-byte aligned");
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  CUtensorMap mx, ma;
  rc = make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, K, M, K * 2, 64, 128);
  if (rc) return rc;
  rc = make_map_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lora_a, K, r, K * 2, 64, static_cast<uint32_t>(r));
  if (rc) return rc;
  LoraParams p;
  p.M = static_cast<int>(M);
  p.K = static_cast<int>(K);
  p.r = static_cast<int>(r);
  p.num_chunks = static_cast<int>(K / 64);
  p.stage_bytes = kLoraXBytes + static_cast<uint32_t>(r) * 128u;
  p.stages = static_cast<int>(kLoraSmemBudget / p.stage_bytes);
  if (p.stages > 8) p.stages = 8;
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(r)) cols <<= 1;
  p.tmem_cols = cols;
  p.ax = static_cast<__nv_bfloat16*>(ax);
  const uint32_t smem = p.stages * p.stage_bytes + 1024 + 256;
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!d->lora_ready) {
      cudaError_t e = cudaFuncSetAttribute(lora_a_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kLoraSmemBudget + 1024 + 256);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(lora_a smem)");
      d->lora_ready = true;
    }
  }
  const unsigned grid = static_cast<unsigned>((M + 127) / 128);
  lora_a_kernel<<<grid, kLoraThreads, smem, static_cast<cudaStream_t>(stream)>>>(mx, ma, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "lora_a launch");
  return LTXFP8_OK;
}

int ltxfp8_selftest_wait_timeout(unsigned long long limit_ns, unsigned int* status, void* stream) {
  if (!status) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "selftest: null pointer");
  if (limit_ns == 0 || limit_ns > 10000000000ull)
    return fail(LTXFP8_ERR_INVALID_ARGUMENT, "selftest: limit must be in (0, 10 s]");
  DeviceInfo* d;
  int rc = device_info(&d);
  if (rc) return rc;
  unsigned int prior = 0;
  rc = ltxfp8_device_status(&prior, 1, stream);  // start from a clear word
  if (rc) return rc;
  auto s = static_cast<cudaStream_t>(stream);
  selftest_wait_kernel<<<1, 32, 0, s>>>(limit_ns);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "selftest");
  return ltxfp8_device_status(status, 1, stream);
}

int ltxfp8_device_status(unsigned int* status, int clear, void* stream) {
  if (!status) return fail(LTXFP8_ERR_INVALID_ARGUMENT, "device_status: null pointer");
  auto s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyFromSymbolAsync(status, g_device_status, sizeof(unsigned int), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "device_status read");
  if (clear) {
    static const unsigned int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_device_status, &zero, sizeof(unsigned int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "device_status clear");
  }
  return LTXFP8_OK;
}

}  // extern "C"
