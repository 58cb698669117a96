/*
 * ltxfp8 -- C ABI of the B200 (sm_100a) blockwise-FP8 linear layer.
 *
 * Plain pointers and sizes only.  Every device pointer is a CUDA device
 * address on the current device; `stream` is a cudaStream_t (NULL = legacy
 * default stream).  No entry point allocates device memory or synchronises the
 * stream, so every call can be enqueued inside CUDA-graph capture.  Each call
 * returns LTXFP8_OK (0) or a negative error code; ltxfp8_last_error() gives a
 * human-readable message for the calling thread.
 *
 * Layouts (those of Lightricks/LTX-2's ltx-kernels blockwise path):
 *   activations  bf16 [M, K] row-major (K contiguous)
 *   act codes    e4m3fn [M, K] row-major
 *   act scales   fp32, MN-major: scale of (row m, K-block kb) at sfa[kb * sfa_ld + m],
 *                sfa_ld >= M (the reference uses align4(M))
 *   weights      e4m3fn [N, K] row-major; scales fp32 [N/128, K/128] row-major
 *   bias         fp32 [N] or NULL
 *   output       bf16 [M, N] row-major
 */
#ifndef LTXFP8_H
#define LTXFP8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LTXFP8_OK 0
#define LTXFP8_ERR_INVALID_ARGUMENT (-1)
#define LTXFP8_ERR_UNSUPPORTED_SHAPE (-2)
#define LTXFP8_ERR_MISALIGNED (-3)
#define LTXFP8_ERR_CUDA (-4)
#define LTXFP8_ERR_DEVICE (-5)       /* wrong architecture or no device */
#define LTXFP8_ERR_DEVICE_STATUS (-6) /* a kernel recorded a bounded-wait timeout */

/* Activation-quantisation modes (flags of ltxfp8_quantize_1x128). */
#define LTXFP8_QUANT_TORCH 0  /* s = (1/amax)*448, IEEE roundings: bit-exact with blockwise_quantize_torch */
#define LTXFP8_QUANT_TRITON 1 /* s = 448/amax, 1/s via div.full.f32: the arithmetic of the Triton kernel */

/* Input dtypes for ltxfp8_quantize_weight_128x128. */
#define LTXFP8_DTYPE_F32 0
#define LTXFP8_DTYPE_BF16 1
#define LTXFP8_DTYPE_F16 2

/* Library version, (major << 16) | minor. */
int ltxfp8_version(void);

/* Message for the last error returned on the calling thread ("" if none). */
const char* ltxfp8_last_error(void);

/*
 * Per-token 1x128 activation quantisation.
 *   x      bf16 [M, K], row stride x_ld elements (x_ld >= K, x_ld % 8 == 0)
 *   q      e4m3 [M, K], row stride q_ld bytes (q_ld % 8 == 0)
 *   sfa    fp32, element (m, kb) at sfa[kb * sfa_ld + m], sfa_ld >= M
 *   K % 128 == 0.  flags: LTXFP8_QUANT_TORCH or LTXFP8_QUANT_TRITON.
 * Replaces the Triton op blockwise::quantize with use_gelu=False
 * (ltx-kernels/src/ltx_kernels/blockwise/triton_ops.py:128-151, kernel :102-126)
 * and blockwise_quantize_torch (functional.py:138-144).
 */
int ltxfp8_quantize_1x128(const void* x, int64_t M, int64_t K, int64_t x_ld, void* q, int64_t q_ld, float* sfa,
                          int64_t sfa_ld, int flags, void* stream);

/*
 * 128x128 block weight quantisation: w [N, K] (dtype LTXFP8_DTYPE_*) ->
 * q e4m3 [N, K] and sfb fp32 [N/128, K/128].  N % 128 == 0, K % 128 == 0.
 * Replaces blockwise_quantize_weights
 * (ltx-kernels/src/ltx_kernels/blockwise/functional.py:128-135).
 */
int ltxfp8_quantize_weight_128x128(const void* w, int dtype, int64_t N, int64_t K, void* q, float* sfb,
                                   void* stream);

/*
 * As ltxfp8_quantize_weight_128x128 with s = (1/amax) * scale_max, 0 < scale_max <= 448:
 * scale_max 0.1172 gives the FP6-range weights of fp6_blockwise_quantize_weights_torch
 * (ltx-kernels/src/ltx_kernels/blockwise/functional.py:22,153-154), whose codes keep the
 * two top exponent bits zero.
 */
int ltxfp8_quantize_weight_128x128_scaled(const void* w, int dtype, int64_t N, int64_t K, float scale_max, void* q,
                                          float* sfb, void* stream);

/*
 * FP6 packing of e4m3 codes [m, n] (n % 8 == 0) into [m, n * 3 / 4] bytes: each code
 * keeps bit 7 and bits 4..0 (the two top exponent bits are dropped), four 6-bit values
 * fill 3 bytes most-significant first; ltxfp8_fp6_unpack restores them with the
 * dropped bits zero.  Packed buffers 2-byte, unpacked 8-byte aligned.
 * Replace ops_cpp.fp6_pack / fp6_unpack (ltx-kernels/csrc/ops/fp6_pack.cu:8-211,
 * fp6_bitpack.cpp:18-73).
 */
int ltxfp8_fp6_pack(const void* x, int64_t m, int64_t n, void* out, void* stream);
int ltxfp8_fp6_unpack(const void* x, int64_t m, int64_t n, void* out, void* stream);

/*
 * A packed FP6 weight w6 [N, K * 3 / 4] (ltxfp8_fp6_pack's layout) and its scales
 * sfb [N/128, K/128] -> the operands of ltxfp8_gemm_fp6w: the same 6-bit codes in the
 * tensor core's order (every 16 codes of a row in 12 bytes, code i at bits 6i..6i+5
 * of their little-endian 96-bit word; w6_tc 32-byte aligned, same size as w6) and the
 * scales x 2^-6 (a code read as e2m3 is 2^6 times the e4m3 value it stands for).
 * N, K multiples of 128.
 */
int ltxfp8_fp6_to_tc(const void* w6, const float* sfb, int64_t N, int64_t K, void* w6_tc, float* sfb_tc,
                     void* stream);

/*
 * 1x128 dequantisation: out[m, k] = bf16(e4m3(q[m, k]) * scales[m * row_stride + (k/128) * col_stride]).
 * K % 128 == 0.  Replaces blockwise::dequantize
 * (ltx-kernels/src/ltx_kernels/blockwise/triton_ops.py:387-433).
 */
int ltxfp8_dequantize_1x128(const void* q, const float* scales, int64_t row_stride, int64_t col_stride, int64_t M,
                            int64_t K, void* out, void* stream);

/*
 * Load-time LoRA merge into a blockwise-FP8 weight:
 *   (q_out, sfb_out) = 128x128 quant of bf16(bf16(e4m3(q) * sfb) + delta)
 * q e4m3 [N, K], sfb fp32 [N/128, K/128], delta bf16 [N, K] (the aggregated LoRA
 * update sum (B * strength) @ A); N, K multiples of 128.  q_out / sfb_out may be q /
 * sfb (in place).  Replaces _blockwise_fp8_fuse
 * (ltx-core/src/ltx_core/quantization/blockwise/_impl.py:263-301), which dequantises,
 * adds and requantises in three torch/Triton passes.
 */
int ltxfp8_lora_fuse_weight(const void* q, const float* sfb, const void* delta, int64_t N, int64_t K, void* q_out,
                            float* sfb_out, void* stream);

/*
 * Fused producers of the GEMM's A operand.  Rows are tokens of a [B, S, H]
 * bf16 tensor with contiguous rows (row stride H), M = B * S, H % 128 == 0,
 * H <= 8192.  Per-batch/per-token parameter tensors are addressed as
 * p[b * bstride + s * sstride + h] (sstride 0 broadcasts over the S tokens).
 * Quantised outputs use the layout of ltxfp8_quantize_1x128 with q_ld = H;
 * flags selects the quantiser arithmetic (LTXFP8_QUANT_*).  Row sums of squares
 * are accumulated in fp32 in a fixed order and 1/sqrt is an IEEE sqrt and
 * division (the reference sums the bf16 squares in bf16 and uses the fast rsqrt).
 */

/*
 * AdaLN producer: y = bf16(x * rsqrt(mean(bf16(x^2)) + 1e-5));
 * z = bf16(bf16(y * bf16(1 + scale)) + shift); (q, sfa) = 1x128 quant of z.
 * scale, shift bf16.  Replaces blockwise::adanorm / blockwise_quantize_adanorm_triton
 * (ltx-kernels/src/ltx_kernels/blockwise/triton_ops.py:52-96,158-186).
 */
int ltxfp8_adanorm_quantize(const void* x, int64_t B, int64_t S, int64_t H, const void* scale,
                            int64_t scale_bstride, int64_t scale_sstride, const void* shift, int64_t shift_bstride,
                            int64_t shift_sstride, void* q, float* sfa, int64_t sfa_ld, int flags, void* stream);

/*
 * Residual update + RMS norm: x <- bf16(x + bf16(y * z)) in place;
 * o = x * rsqrt(mean(bf16(x^2))) in fp32 (no epsilon).  With q != NULL,
 * (q, sfa) = 1x128 quant of o (blockwise::quant_rms_fma); otherwise out = bf16(o)
 * (blockwise::rms_fma).  y bf16 [M, H], z bf16.
 * Replaces _quant_rms_sum_mult_kernel and its two ops (triton_ops.py:188-290).
 */
int ltxfp8_rms_fma(void* x, const void* y, int64_t B, int64_t S, int64_t H, const void* z, int64_t z_bstride,
                   int64_t z_sstride, void* q, float* sfa, int64_t sfa_ld, void* out, int flags, void* stream);

/*
 * Gated attention output: o = x * 2 sigmoid(gate_logits[m, h / (H / heads)]) in fp32,
 * x bf16 [M, H], gate_logits [M, heads] of gate_dtype (LTXFP8_DTYPE_BF16 or _F32),
 * heads <= 64, (H / heads) % 8 == 0.  With q != NULL the 1x128 quant of o, otherwise out = bf16(o).
 * Replaces blockwise::gated_attention / gated_attention_triton (triton_ops.py:293-345).
 */
int ltxfp8_gated_attention(const void* x, const void* gate_logits, int gate_dtype, int64_t M, int64_t H,
                           int64_t heads, void* q, float* sfa, int64_t sfa_ld, void* out, int flags, void* stream);

/*
 * GELU (sigmoid form) + quant: o = x * sigmoid(1.702 x) in fp32, then the 1x128
 * quant of o; arguments as ltxfp8_quantize_1x128.  Replaces blockwise::quantize
 * with use_gelu=True (triton_ops.py:98-100,102-151).
 */
int ltxfp8_gelu_quantize_1x128(const void* x, int64_t M, int64_t K, int64_t x_ld, void* q, int64_t q_ld, float* sfa,
                               int64_t sfa_ld, int flags, void* stream);

/*
 * torch's GELU-tanh + quant: y = bf16 result of F.gelu(x, approximate="tanh") on the
 * bf16 input, then the 1x128 quant of y; arguments as ltxfp8_quantize_1x128.
 * Replaces the reference FFN's unfused chain after the up projection: F.gelu
 * (ltx-core/src/ltx_core/model/transformer/gelu_approx.py:10) on the bf16 GEMM output,
 * then blockwise::quantize in the down projection (ltx-kernels/.../linear.py:91-93).
 * Codes and scales equal ltxfp8_quantize_1x128 applied to torch's GELU output.
 */
int ltxfp8_gelu_tanh_quantize_1x128(const void* x, int64_t M, int64_t K, int64_t x_ld, void* q, int64_t q_ld,
                                    float* sfa, int64_t sfa_ld, int flags, void* stream);

/*
 * RMSNorm + interleaved RoPE for attention q/k: per row of x bf16 [rows, dim]
 * (dim % 8 == 0, dim <= 8192), v = x * (rsqrt(sum(x^2) * (1/dim)) * w) (no epsilon;
 * weights bf16 [dim] or NULL for none), then for each pair (2i, 2i+1)
 * out[2i] = v[2i] cos[2i] - v[2i+1] sin[2i], out[2i+1] = v[2i+1] cos[2i+1] + v[2i] sin[2i+1],
 * with cos/sin bf16 rows at p + row * freq_row_stride.  out: bf16 [rows, dim], or
 * e4m3 (torch's conversion, overflow to NaN) when out_fp8.  Sums of squares in
 * fp32 with fused multiply-adds in a fixed order; 1/sqrt is an IEEE sqrt and division.
 * Replaces ops_cpp.rms_norm_rope (ltx-kernels/csrc/ops/rms_norm_rope.cpp:62-114,
 * rms_norm_rope_cuda.cu:56-175), which is built with --use_fast_math.
 */
int ltxfp8_rms_norm_rope(const void* x, int64_t rows, int64_t dim, const void* cos_freqs, const void* sin_freqs,
                         int64_t freq_row_stride, const void* weights, void* out, int out_fp8, void* stream);

/*
 * RMSNorm + split RoPE: x bf16 [B, S, H] seen as `heads` heads of d = H / heads
 * values, each split into halves a = [0, d/2) and b = [d/2, d);
 * v = (x * rsqrt(sum(x^2) / H + 1e-6)) * w (weights bf16 [H] or NULL), then
 * out_a = cos v_a - sin v_b, out_b = cos v_b + sin v_a, with cos/sin element
 * (b, head, s, j) at p[b * bstride + head * hstride + s * sstride + j]
 * (bstride 0 broadcasts one table over the batch).  d in {16, 32, 64, 128, 256},
 * H % 128 == 0, H <= 8192.  out: bf16, or saturating e4m3 when out_fp8.
 * Replaces ops_cpp.rms_norm_split_rope (ltx-kernels/csrc/ops/rms_norm_split_rope.cpp:28-111,
 * rms_norm_split_rope_cuda.cu:42-150).
 */
int ltxfp8_rms_norm_split_rope(const void* x, int64_t B, int64_t S, int64_t H, int64_t heads, const void* cos_freqs,
                               int64_t cos_bstride, int64_t cos_hstride, int64_t cos_sstride, const void* sin_freqs,
                               int64_t sin_bstride, int64_t sin_hstride, int64_t sin_sstride, const void* weights,
                               void* out, int out_fp8, void* stream);

/* Epilogue options of ltxfp8_gemm (all zero = plain bias + bf16 store). */
/* ltxfp8_epilogue.gelu_tanh */
#define LTXFP8_GELU_NONE 0
#define LTXFP8_GELU_TANH 1      /* torch's CUDA GELU-tanh, 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) in fp32
                                   with CUDA's tanhf, as F.gelu(approximate="tanh") computes it (gelu_approx.py:10) */
#define LTXFP8_GELU_TANH_FAST 2 /* the same function as x / (1 + 2^a) with approximate exp2 and reciprocal:
                                   no cancellation, within one bf16 ulp of LTXFP8_GELU_TANH */

typedef struct ltxfp8_epilogue {
  int gelu_tanh;          /* LTXFP8_GELU_*: apply GELU to bf16(acc + bias), rounding the result to bf16 */
  void* requant_q;        /* non-NULL: write the 1x128 e4m3 quantisation of the bf16 result, [M, N] */
  float* requant_scales;  /* its scales, element (m, nb) at requant_scales[nb * requant_ld + m] */
  int64_t requant_ld;     /* >= M */
  int skip_d;             /* non-zero: do not write D (only valid with requant_q) */
  const void* lora_ax;    /* non-NULL: bf16 [M, lora_r], the LoRA down projection x A^T */
  const void* lora_b;     /* bf16 [N, lora_r], the LoRA up projection */
  int64_t lora_r;         /* rank, multiple of 16, <= 256 */
  float lora_alpha;       /* scale of the LoRA term */
  void* workspace;        /* optional fp32 scratch for split-K on skinny M (see ltxfp8_gemm_workspace_bytes) */
  size_t workspace_bytes; /* its size; split-K is used only when it is large enough */
  int requant_mode;       /* arithmetic of the requantisation's scales: LTXFP8_QUANT_TORCH (0) or
                             LTXFP8_QUANT_TRITON, as for ltxfp8_quantize_1x128 */
} ltxfp8_epilogue;

/*
 * Blockwise-scaled FP8 GEMM (NT) with fused epilogue:
 *   D = bf16( sum_kb sfa[m,kb] sfb[n/128,kb] (A W^T)_kb + alpha B (x A^T)^T + bias )
 *   optionally followed by GELU-tanh and 1x128 requantisation.
 * M >= 1, N % 128 == 0, K % 128 == 0 (any K, not only 2048/4096/8192/16384).
 * ep may be NULL.
 * Replaces blockwise_cpp.fp8_gemm_nt_sm89 (ltx-kernels/csrc/blockwise/api.cpp:42-65,
 * sm89_fp8_gemm_1d2d.hpp:17-37, kernels/geforce/gemm.cu:256-275) and the
 * unfused F.gelu + requant of the FFN (ltx-core/.../gelu_approx.py:10,
 * ltx-kernels/.../linear.py:91-93).
 */
int ltxfp8_gemm(const void* A, const float* sfa, int64_t sfa_ld, const void* W, const float* sfb,
                const float* bias, void* D, int64_t M, int64_t N, int64_t K, const ltxfp8_epilogue* ep,
                void* stream);

/*
 * ltxfp8_gemm with a 6-bit weight: W6 and sfb6 from ltxfp8_fp6_to_tc.  The weight
 * streams from memory at 6 bits per element straight into the tensor core
 * (kind::f8f6f4 with an e2m3 B operand), with no unpacked copy; the result is the
 * same as ltxfp8_gemm on ltxfp8_fp6_unpack's e4m3 codes with the original scales.
 * W6 32-byte aligned; every epilogue option is available.
 * Replaces BlockwiseFP6Linear's fp8weight unpack followed by the FP8 GEMM
 * (ltx-kernels/src/ltx_kernels/blockwise/linear.py:212-250, csrc/ops/fp6_pack.cu:112-211).
 */
int ltxfp8_gemm_fp6w(const void* A, const float* sfa, int64_t sfa_ld, const void* W6, const float* sfb6,
                     const float* bias, void* D, int64_t M, int64_t N, int64_t K, const ltxfp8_epilogue* ep,
                     void* stream);

/*
 * Scratch bytes ltxfp8_gemm would use for split-K at this shape on the current
 * device (0 when it splits nothing).  Skinny GEMMs (few 128 x 256 output tiles)
 * divide each tile's K blocks among several CTAs, write fp32 partials to the
 * workspace and reduce them in a fixed order (deterministic); for K >= 8192 a
 * mostly empty last wave of output tiles is split the same way (its rows as a
 * second, skinny launch).  No reference counterpart (the SM89 kernel has no
 * split-K).
 */
int ltxfp8_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, size_t* bytes);

/* How ltxfp8_gemm launches a shape on the current device when given the workspace. */
typedef struct ltxfp8_gemm_plan_info {
  size_t workspace_bytes; /* = ltxfp8_gemm_workspace_bytes */
  int launches;           /* kernel launches of one call (GEMMs and the split-K reduction) */
  int splits;             /* K splits of the split rows; 1: no split */
  int64_t split_row0;     /* rows [0, split_row0) unsplit, [split_row0, M) split; M: no split */
} ltxfp8_gemm_plan_info;

/* Fills *info for an M x N x K GEMM on the current device (no reference counterpart). */
int ltxfp8_gemm_plan(int64_t M, int64_t N, int64_t K, ltxfp8_gemm_plan_info* info);

/* The same plan for a GPU with `sms` streaming multiprocessors; a host computation
   only (no CUDA call), for planning and tests without a device. */
int ltxfp8_gemm_plan_for_sms(int64_t M, int64_t N, int64_t K, int sms, ltxfp8_gemm_plan_info* info);

/* Size of the static split-K array of ltxfp8_gemm_static_scratch. */
#define LTXFP8_STATIC_SCRATCH_BYTES (32ull << 20)

/*
 * ltxfp8_gemm for callers that cannot allocate device memory per call: a host
 * whose memory is all owned by its own arena or a framework's allocator, or a
 * plugin whose launch hook (an enqueue or execute callback) must not allocate.
 * Same arguments, results and errors as ltxfp8_gemm; ep->workspace and
 * ep->workspace_bytes are ignored.  The split-K scratch of skinny shapes comes
 * from one fixed 32 MiB array in the library's device globals instead of the
 * caller: every GPU that loads the library's kernels holds those 32 MiB until
 * the process exits.  A shape whose split-K plan needs more than 32 MiB returns
 * LTXFP8_ERR_UNSUPPORTED_SHAPE (none does on a 148-SM B200).
 * The first call on each device looks up the array's device address, with
 * that device current; make that first call before any stream capture.
 * All calls on a device share the array and it keeps the last call's partials
 * (nothing in it needs to start at zero): calls that can overlap on the GPU
 * (other streams, other host threads) race on it, so issue them on one stream.
 * No reference counterpart.
 */
int ltxfp8_gemm_static_scratch(const void* A, const float* sfa, int64_t sfa_ld, const void* W, const float* sfb,
                               const float* bias, void* D, int64_t M, int64_t N, int64_t K,
                               const ltxfp8_epilogue* ep, void* stream);

/*
 * Select the GEMM kernel: 0 = default (the one-CTA kernel), 1 = the one-CTA
 * kernel (128 x 256 tiles per SM), 2 = the CTA-pair kernel (256 x 256 tiles
 * over two SMs of a cluster, tcgen05 cta_group::2).  Process-wide; meant for tests and tuning.  No reference
 * counterpart (the reference has one kernel per architecture, linear.py:25-45).
 */
int ltxfp8_gemm_set_variant(int variant);

/*
 * LoRA down projection: ax bf16 [M, r] = x bf16 [M, K] . lora_a bf16 [r, K]^T (fp32 accumulation).
 * K % 64 == 0, r % 16 == 0, 16 <= r <= 256.  No reference counterpart: the
 * reference merges LoRA into the weights at load time
 * (ltx-core/src/ltx_core/quantization/blockwise/_impl.py:277-301); this is the
 * runtime form of that term.
 */
int ltxfp8_lora_a(const void* x, const void* lora_a, void* ax, int64_t M, int64_t K, int64_t r, void* stream);

/*
 * Read (and optionally clear) the device status word that kernels set when a
 * bounded wait gives up.  Synchronises the given stream.  *status = 0 means
 * no kernel has failed since the last clear.
 */
int ltxfp8_device_status(unsigned int* status, int clear, void* stream);

/*
 * Failure-path self-test: launches one warp that waits, with a limit of
 * `limit_ns`, on a barrier nothing arrives on; the bounded wait gives up,
 * records 0x5E1F0001 in the device status word and the kernel returns.
 * Synchronises `stream`; *status receives the word (then cleared).  Shows that
 * a stuck pipeline ends with an error the host can read, not a hung GPU.
 * No reference counterpart (the reference's IPC barrier traps on timeout,
 * ltx-kernels/csrc/include/cuda/utils.cuh:264-295).
 */
int ltxfp8_selftest_wait_timeout(unsigned long long limit_ns, unsigned int* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LTXFP8_H */
