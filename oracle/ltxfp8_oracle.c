/*
 * CPU oracle for the blockwise-FP8 linear path.  TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic of Lightricks/LTX-2's
 * `ltx-kernels` blockwise path so that the CUDA kernels can be checked
 * against it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it; the product path never does.
 *
 * Every function cites the reference lines it follows (paths are relative
 * to the reference repository's packages/ directory).
 *
 * Conventions
 *   bf16 values travel as uint16_t bit patterns, e4m3fn codes as uint8_t.
 *   fp32 -> e4m3fn follows torch's c10 conversion (round to nearest even on
 *   the e4m3 grid, no saturation: magnitudes above 464 become NaN, 0x7F|sign),
 *   which is what `tensor.to(torch.float8_e4m3fn)` does in
 *   ltx-kernels/src/ltx_kernels/blockwise/functional.py:133,143.
 *   The scale is formed the way torch evaluates `scale_max / amax` for a Python
 *   scalar numerator: Tensor.__rtruediv__ is `self.reciprocal() * other`, so
 *   s = RN(RN(1 / amax) * scale_max) -- two IEEE roundings, not one division --
 *   and the stored scale `1 / s` is RN(1 / s) (functional.py:131,134,142,144).
 *
 * Parity pin: the quantisers are checked bit-for-bit against fixtures made by
 * the reference's own torch functions (tests/golden/make_golden.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#if defined(__FLT_EVAL_METHOD__) && __FLT_EVAL_METHOD__ != 0
#error "oracle needs IEEE single-precision evaluation (FLT_EVAL_METHOD 0)"
#endif

static inline float f32_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t bits_from_f32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float orc_bf16_to_f32(uint16_t h) { return f32_from_bits((uint32_t)h << 16); }

/* fp32 -> bf16, round to nearest even; NaN stays a quiet NaN of the same sign. */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t u = bits_from_f32(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

/* e4m3fn code -> fp32 (exact).  0x7F / 0xFF are NaN; there is no infinity. */
float orc_e4m3_to_f32(uint8_t c) {
    uint32_t s = (c >> 7) & 1u, e = (c >> 3) & 0xfu, m = c & 7u;
    float v;
    if (e == 15u && m == 7u) return s ? -NAN : NAN;
    if (e == 0u) v = ldexpf((float)m, -9);                 /* subnormal: m * 2^-9 */
    else v = ldexpf(1.0f + (float)m / 8.0f, (int)e - 7);   /* normal */
    return s ? -v : v;
}

/* fp32 -> e4m3fn code with c10 semantics (round to nearest even, overflow to NaN). */
uint8_t orc_f32_to_e4m3(float f) {
    uint32_t u = bits_from_f32(f);
    uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint8_t)(sign | 0x7fu);   /* NaN */
    float x = f32_from_bits(a);
    /* 464 is the midpoint between 448 (max finite) and 480 (the NaN pattern);
       ties go to the even code 0x7E, anything above rounds onto the NaN pattern. */
    if (x > 464.0f) return (uint8_t)(sign | 0x7fu);
    if (x >= 0.015625f) {                                  /* normal range, >= 2^-6 */
        int e; float fr = frexpf(x, &e);                    /* x = fr * 2^e, fr in [0.5,1) */
        /* mantissa in units of 2^(e-1-3): x / 2^(e-4) in [8,16) */
        float scaled = ldexpf(fr, 4);                       /* in [8,16) exactly */
        float r = nearbyintf(scaled);                       /* RNE (default rounding mode) */
        int ee = e - 1 + 7;                                 /* biased exponent */
        int mm = (int)r - 8;
        if (mm == 8) { mm = 0; ee += 1; }
        if (ee > 15) return (uint8_t)(sign | 0x7fu);
        return (uint8_t)(sign | (uint8_t)(ee << 3) | (uint8_t)mm);
    }
    /* subnormal range: multiples of 2^-9 */
    float r = nearbyintf(ldexpf(x, 9));
    int mm = (int)r;
    if (mm >= 8) return (uint8_t)(sign | (1u << 3));       /* rounds up to 2^-6 */
    return (uint8_t)(sign | (uint8_t)mm);
}

/* abs-max with NaN propagation, as torch's `abs().max()` reduction does. */
static inline float amax_nan(float a, float b) {
    if (isnan(a) || isnan(b)) return NAN;
    return a > b ? a : b;
}

/*
 * Activation quantisation, 1x128 groups per token.
 * Follows blockwise_quantize_torch (ltx-kernels/src/ltx_kernels/blockwise/functional.py:138-144)
 * and the Triton _quantize/_block_quant_kernel (triton_ops.py:13-22,102-126):
 *   s = (1 / amax(|x|)) * 448 (torch's reciprocal-then-multiply, see the header);
 *   q = e4m3(float(x) * s); stored scale = 1 / s.
 * x: bf16 [M, K] with row stride x_ld; q: [M, K] row stride q_ld;
 * sfa: MN-major, element (m, kb) at sfa[kb * sfa_ld + m] (triton_ops.py:134-135,147-148).
 * scale_max is 448 for FP8 (functional.py:21).
 */
void orc_quant_act_1x128(const uint16_t* x, int64_t M, int64_t K, int64_t x_ld,
                         uint8_t* q, int64_t q_ld, float* sfa, int64_t sfa_ld,
                         float scale_max) {
    int64_t KB = K / 128;
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t kb = 0; kb < KB; ++kb) {
            const uint16_t* g = x + m * x_ld + kb * 128;
            float amax = 0.0f;
            for (int i = 0; i < 128; ++i) amax = amax_nan(amax, fabsf(orc_bf16_to_f32(g[i])));
            volatile float r = 1.0f / amax;
            volatile float s = r * scale_max;
            for (int i = 0; i < 128; ++i) {
                volatile float v = orc_bf16_to_f32(g[i]) * s;
                q[m * q_ld + kb * 128 + i] = orc_f32_to_e4m3(v);
            }
            volatile float inv = 1.0f / s;
            sfa[kb * sfa_ld + m] = inv;
        }
    }
}

/*
 * Weight quantisation, 128x128 blocks.
 * Follows blockwise_quantize_weights (functional.py:128-135):
 *   s = (1 / amax) * 448 over the 128x128 block; q = e4m3(float(w) * s); scale = 1 / s,
 *   scales stored row-major [N/128, K/128].
 * w_dtype: 0 = fp32, 1 = bf16 (bit patterns).
 */
void orc_quant_weight_128x128(const void* w, int w_dtype, int64_t N, int64_t K,
                              uint8_t* q, float* sfb, float scale_max) {
    int64_t NB = N / 128, KB = K / 128;
    const float* wf = (const float*)w;
    const uint16_t* wh = (const uint16_t*)w;
#define WVAL(r, c) (w_dtype == 0 ? wf[(r) * K + (c)] : orc_bf16_to_f32(wh[(r) * K + (c)]))
    for (int64_t nb = 0; nb < NB; ++nb) {
        for (int64_t kb = 0; kb < KB; ++kb) {
            float amax = 0.0f;
            for (int64_t r = nb * 128; r < nb * 128 + 128; ++r)
                for (int64_t c = kb * 128; c < kb * 128 + 128; ++c)
                    amax = amax_nan(amax, fabsf(WVAL(r, c)));
            volatile float rcp = 1.0f / amax;
            volatile float s = rcp * scale_max;
            for (int64_t r = nb * 128; r < nb * 128 + 128; ++r)
                for (int64_t c = kb * 128; c < kb * 128 + 128; ++c) {
                    volatile float v = WVAL(r, c) * s;
                    q[r * K + c] = orc_f32_to_e4m3(v);
                }
            volatile float inv = 1.0f / s;
            sfb[nb * KB + kb] = inv;
        }
    }
#undef WVAL
}

/*
 * Dequantisation to bf16: out = bf16(float(q) * scale[m, k/128]).
 * Follows _blockwise_dequantize_kernel (triton_ops.py:387-411): the scale of
 * (row, block) is read at scales[row * row_stride + block * col_stride].
 */
void orc_dequant_1x128(const uint8_t* q, const float* scales, int64_t row_stride,
                       int64_t col_stride, int64_t M, int64_t K, uint16_t* out) {
    for (int64_t m = 0; m < M; ++m)
        for (int64_t k = 0; k < K; ++k) {
            float s = scales[m * row_stride + (k / 128) * col_stride];
            volatile float v = orc_e4m3_to_f32(q[m * K + k]) * s;
            out[m * K + k] = orc_f32_to_bf16(v);
        }
}

/*
 * Blockwise GEMM in the reference kernel's promotion order
 * (ltx-kernels/csrc/blockwise/kernels/geforce/gemm.cu:150-222):
 *   for each 128-wide K block: p = sum_k e4m3(A[m,k]) * e4m3(W[n,k])  (fp32)
 *                              D += (sfa[m,kb] * sfb[n/128,kb]) * p
 *   D += bias[n];  out = bf16(D)
 * A [M,K] codes, W [N,K] codes, sfa at sfa[kb*sfa_ld + m], sfb [N/128, K/128].
 * bias may be NULL.  Writes fp32 D (before the bf16 cast) to out_f32 if given
 * and the bf16 result to out_bf16 if given.
 */
void orc_gemm_promoted(const uint8_t* A, const float* sfa, int64_t sfa_ld,
                       const uint8_t* W, const float* sfb, const float* bias,
                       int64_t M, int64_t N, int64_t K,
                       float* out_f32, uint16_t* out_bf16) {
    int64_t KB = K / 128;
    float lut[256];
    for (int i = 0; i < 256; ++i) lut[i] = orc_e4m3_to_f32((uint8_t)i);
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t n = 0; n < N; ++n) {
            float d = 0.0f;
            for (int64_t kb = 0; kb < KB; ++kb) {
                float p = 0.0f;
                const uint8_t* a = A + m * K + kb * 128;
                const uint8_t* w = W + n * K + kb * 128;
                for (int i = 0; i < 128; ++i) p = fmaf(lut[a[i]], lut[w[i]], p);
                float s = sfa[kb * sfa_ld + m] * sfb[(n / 128) * KB + kb];
                d = fmaf(s, p, d);
            }
            if (bias) d += bias[n];
            if (out_f32) out_f32[m * N + n] = d;
            if (out_bf16) out_bf16[m * N + n] = orc_f32_to_bf16(d);
        }
    }
}

/*
 * GELU, tanh approximation, on bf16 values, result rounded to bf16.
 * The reference applies torch.nn.functional.gelu(x, approximate="tanh") to the
 * GEMM's bf16 output (ltx-core/src/ltx_core/model/transformer/gelu_approx.py:10):
 *   0.5 * x * (1 + tanh(sqrt(2/pi) * (x + 0.044715 x^3))) in fp32, cast to bf16.
 */
uint16_t orc_gelu_tanh_bf16(uint16_t xh) {
    float x = orc_bf16_to_f32(xh);
    const float kBeta = 0.7978845608028654f;   /* sqrt(2/pi) */
    const float kKappa = 0.044715f;
    float x3 = x * x * x;
    float inner = kBeta * fmaf(kKappa, x3, x);
    float y = 0.5f * x * (1.0f + tanhf(inner));
    return orc_f32_to_bf16(y);
}

void orc_gelu_tanh_bf16_array(const uint16_t* x, int64_t n, uint16_t* y) {
    for (int64_t i = 0; i < n; ++i) y[i] = orc_gelu_tanh_bf16(x[i]);
}

void orc_e4m3_to_f32_array(const uint8_t* c, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = orc_e4m3_to_f32(c[i]);
}

void orc_f32_to_e4m3_array(const float* f, int64_t n, uint8_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = orc_f32_to_e4m3(f[i]);
}

void orc_f32_to_bf16_array(const float* f, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = orc_f32_to_bf16(f[i]);
}

/* ------------------------------------------------------------------------
 * Fused producers (ltx-kernels/src/ltx_kernels/blockwise/triton_ops.py:52-96,
 * 98-126, 188-290, 293-345).  Parity unpinned: the reference runs these as
 * Triton GPU kernels, which cannot execute in this container, and its tests
 * hold no fixtures for them.  The restatement keeps the reference's dtype
 * semantics (Triton promotion rules: bf16 op bf16 -> bf16, bf16 op fp32 -> fp32,
 * a Python float scalar takes the tensor's dtype) and fixes the arithmetic the
 * reference leaves to the compiler:
 *   - row sums of bf16(x^2) accumulate in fp32 in the CUDA kernels' order:
 *     per lane l of 32, its 16-byte chunks c = 32 i + l (8 values each) in order,
 *     then an xor butterfly over the lanes with offsets 16, 8, 4, 2, 1
 *     (the reference reduces in bf16 in Triton's layout order);
 *   - 1/sqrt(v) = RN(1 / RN(sqrt(v))) (the reference: rsqrt approximation);
 *   - e^x by Cody-Waite reduction and the degree-7 Taylor series (exp_cw below),
 *     1/(1+e) by IEEE division (the reference: fast exp and division);
 *   - quantisation in the torch arithmetic of orc_quant_act_1x128 on fp32 inputs.
 * -------------------------------------------------------------------- */

static float rn_bf16(float v) { return orc_bf16_to_f32(orc_f32_to_bf16(v)); }

/* e^x: x = k ln2 + r with ln2 = 0.693145751953125 (15 significant bits, so k*head
   is exact) + 1.42860682030941723212e-6; e^r by Taylor to degree 7 (Horner, fma);
   scale by 2^k in two exact halves. */
static float exp_cw(float x) {
    if (x != x) return x;
    if (x > 88.8f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    volatile float t = x * 1.44269504088896341f;
    float k = rintf(t);
    float r = fmaf(-k, 0.693145751953125f, x);
    r = fmaf(-k, 1.42860682030941723212e-6f, r);
    float p = 1.98412698412698413e-4f;
    p = fmaf(p, r, 1.38888888888888889e-3f);
    p = fmaf(p, r, 8.33333333333333333e-3f);
    p = fmaf(p, r, 4.16666666666666667e-2f);
    p = fmaf(p, r, 1.66666666666666667e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ki = (int)k;
    int k1 = ki / 2, k2 = ki - k1;
    volatile float a = p * f32_from_bits((uint32_t)(k1 + 127) << 23);
    volatile float b = a * f32_from_bits((uint32_t)(k2 + 127) << 23);
    return b;
}

float orc_exp_cw(float x) { return exp_cw(x); }

static float sigmoid_cw(float x) {
    volatile float e = exp_cw(-x);
    volatile float d = 1.0f + e;
    volatile float s = 1.0f / d;
    return s;
}

static float rsqrt_ieee(float v) {
    volatile float sq = sqrtf(v);
    volatile float r = 1.0f / sq;
    return r;
}

/* Sum of bf16(x^2) over a row of H bf16 values in the kernels' lane/butterfly order. */
static float row_sumsq_bf16(const float* x, int64_t H) {
    float part[32];
    int64_t nchunks = H / 8;
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int64_t c = l; c < nchunks; c += 32)
            for (int j = 0; j < 8; ++j) {
                volatile float sq = x[c * 8 + j] * x[c * 8 + j];
                volatile float s = acc + rn_bf16(sq);
                acc = s;
            }
        part[l] = acc;
    }
    for (int off = 16; off > 0; off >>= 1) {
        float nxt[32];
        for (int l = 0; l < 32; ++l) {
            volatile float s = part[l] + part[l ^ off];
            nxt[l] = s;
        }
        memcpy(part, nxt, sizeof(part));
    }
    return part[0];
}

/* Torch-arithmetic 1x128 quantisation of one row of fp32 values. */
static void quant_row_f32(const float* v, int64_t H, int64_t m, uint8_t* q, float* sfa, int64_t sfa_ld) {
    for (int64_t kb = 0; kb < H / 128; ++kb) {
        const float* g = v + kb * 128;
        float amax = 0.0f;
        for (int i = 0; i < 128; ++i) amax = amax_nan(amax, fabsf(g[i]));
        volatile float r = 1.0f / amax;
        volatile float s = r * 448.0f;
        for (int i = 0; i < 128; ++i) {
            volatile float t = g[i] * s;
            q[m * H + kb * 128 + i] = orc_f32_to_e4m3(t);
        }
        volatile float inv = 1.0f / s;
        sfa[kb * sfa_ld + m] = inv;
    }
}

/*
 * AdaLN producer, _block_quant_norm_kernel (triton_ops.py:52-96):
 *   x_norm = sum(bf16(x*x)) / H; r = rsqrt(x_norm + 1e-5)        (:82-84)
 *   y = bf16(x * r)                                               (:85, bf16 * fp32 -> fp32)
 *   z = bf16(bf16(y * bf16(1 + scale)) + shift)                   (:86, bf16 arithmetic)
 *   (q, sfa) = quant(z)                                           (:88-92)
 * scale/shift of (b, s) at p[b * bs + s * ss] (ss = 0 broadcasts, :74-80).
 */
void orc_adanorm_quant(const uint16_t* x, int64_t B, int64_t S, int64_t H,
                       const uint16_t* scale, int64_t sc_bs, int64_t sc_ss,
                       const uint16_t* shift, int64_t sh_bs, int64_t sh_ss,
                       uint8_t* q, float* sfa, int64_t sfa_ld) {
    float* row = (float*)malloc(sizeof(float) * (size_t)H);
    for (int64_t b = 0; b < B; ++b)
        for (int64_t s = 0; s < S; ++s) {
            int64_t m = b * S + s;
            for (int64_t h = 0; h < H; ++h) row[h] = orc_bf16_to_f32(x[m * H + h]);
            float ss = row_sumsq_bf16(row, H);
            volatile float mean = ss / (float)H;
            volatile float me = mean + 1e-5f;
            float r = rsqrt_ieee(me);
            const uint16_t* sc = scale + b * sc_bs + s * sc_ss;
            const uint16_t* sh = shift + b * sh_bs + s * sh_ss;
            for (int64_t h = 0; h < H; ++h) {
                volatile float xy = row[h] * r;
                float y = rn_bf16(xy);
                volatile float tt = 1.0f + orc_bf16_to_f32(sc[h]);
                float t = rn_bf16(tt);
                volatile float u = y * t;
                volatile float z = rn_bf16(u) + orc_bf16_to_f32(sh[h]);
                row[h] = rn_bf16(z);
            }
            quant_row_f32(row, H, m, q, sfa, sfa_ld);
        }
    free(row);
}

/*
 * Residual FMA + RMS, _quant_rms_sum_mult_kernel (triton_ops.py:188-232):
 *   o = bf16(x + bf16(y * z)); x <- o                              (:209-211, bf16 arithmetic)
 *   r = rsqrt(sum(bf16(o*o)) / H)                                  (:213-215, no epsilon)
 *   v = o * r (fp32)                                               (:216)
 *   QUANTIZE: (q, sfa) = quant(v) (:218-223); else out = bf16(v)   (:225-226)
 * x is updated in place; q == NULL selects the bf16 output.
 */
void orc_rms_fma(uint16_t* x, const uint16_t* y, int64_t B, int64_t S, int64_t H,
                 const uint16_t* z, int64_t z_bs, int64_t z_ss,
                 uint8_t* q, float* sfa, int64_t sfa_ld, uint16_t* out) {
    float* row = (float*)malloc(sizeof(float) * (size_t)H);
    for (int64_t b = 0; b < B; ++b)
        for (int64_t s = 0; s < S; ++s) {
            int64_t m = b * S + s;
            const uint16_t* zr = z + b * z_bs + s * z_ss;
            for (int64_t h = 0; h < H; ++h) {
                volatile float yz = orc_bf16_to_f32(y[m * H + h]) * orc_bf16_to_f32(zr[h]);
                volatile float o = orc_bf16_to_f32(x[m * H + h]) + rn_bf16(yz);
                uint16_t ob = orc_f32_to_bf16(o);
                x[m * H + h] = ob;
                row[h] = orc_bf16_to_f32(ob);
            }
            float ss = row_sumsq_bf16(row, H);
            volatile float mean = ss / (float)H;
            float r = rsqrt_ieee(mean);
            for (int64_t h = 0; h < H; ++h) {
                volatile float v = row[h] * r;
                row[h] = v;
            }
            if (q) quant_row_f32(row, H, m, q, sfa, sfa_ld);
            else for (int64_t h = 0; h < H; ++h) out[m * H + h] = orc_f32_to_bf16(row[h]);
        }
    free(row);
}

/*
 * Gated attention, _gated_attention_kernel (triton_ops.py:271-306):
 *   gate = 2 * sigmoid(float(logit[m, head]))   (:287-289)
 *   v = float(x) * gate                          (:293-297)
 *   QUANTIZE: quant(v) (:299-304); else out = bf16(v) (:305-306)
 * logits: bf16 bit patterns (gate_f32 = 0) or fp32 (gate_f32 = 1), [M, heads].
 */
void orc_gated_attention(const uint16_t* x, const void* logits, int gate_f32, int64_t M, int64_t H,
                         int64_t heads, uint8_t* q, float* sfa, int64_t sfa_ld, uint16_t* out) {
    float* row = (float*)malloc(sizeof(float) * (size_t)H);
    int64_t dh = H / heads;
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t h = 0; h < H; ++h) {
            int64_t hd = h / dh;
            float g = gate_f32 ? ((const float*)logits)[m * heads + hd]
                               : orc_bf16_to_f32(((const uint16_t*)logits)[m * heads + hd]);
            volatile float gate = 2.0f * sigmoid_cw(g);
            volatile float v = orc_bf16_to_f32(x[m * H + h]) * gate;
            row[h] = v;
        }
        if (q) quant_row_f32(row, H, m, q, sfa, sfa_ld);
        else for (int64_t h = 0; h < H; ++h) out[m * H + h] = orc_f32_to_bf16(row[h]);
    }
    free(row);
}

/*
 * GELU (sigmoid form) + quant, _block_quant_kernel with USE_GELU (triton_ops.py:98-126):
 *   v = x * sigmoid(1.702 * x) in fp32 (:98-100,119-120); (q, sfa) = quant(v).
 */
void orc_gelu_quant(const uint16_t* x, int64_t M, int64_t K, uint8_t* q, float* sfa, int64_t sfa_ld) {
    float* row = (float*)malloc(sizeof(float) * (size_t)K);
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t k = 0; k < K; ++k) {
            float xv = orc_bf16_to_f32(x[m * K + k]);
            volatile float t = 1.702f * xv;
            volatile float v = xv * sigmoid_cw(t);
            row[k] = v;
        }
        quant_row_f32(row, K, m, q, sfa, sfa_ld);
    }
    free(row);
}

/* ------------------------------------------------------------------------
 * RMSNorm + RoPE for attention q/k (ltx-kernels/csrc/ops/rms_norm_rope_cuda.cu,
 * rms_norm_split_rope_cuda.cu).  Parity unpinned: the reference builds these with
 * torch headers and a fast-math flag and they cannot run here.  Restated with the
 * arithmetic the CUDA kernels fix: sum of x^2 by fused multiply-adds in the lanes'
 * chunk order then the xor butterfly, 1/sqrt as IEEE sqrt then division.
 * -------------------------------------------------------------------- */

static float row_sumsq_fma(const float* x, int64_t H) {
    float part[32];
    int64_t nchunks = H / 8;
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int64_t c = l; c < nchunks; c += 32)
            for (int j = 0; j < 8; ++j) acc = fmaf(x[c * 8 + j], x[c * 8 + j], acc);
        part[l] = acc;
    }
    for (int off = 16; off > 0; off >>= 1) {
        float nxt[32];
        for (int l = 0; l < 32; ++l) {
            volatile float s = part[l] + part[l ^ off];
            nxt[l] = s;
        }
        memcpy(part, nxt, sizeof(part));
    }
    return part[0];
}

/* e4m3 with the saturating conversion of __nv_fp8_e4m3(float): finite overflow and
   infinities become +-448, NaN stays NaN. */
static uint8_t f32_to_e4m3_sat(float f) {
    if (f != f) return orc_f32_to_e4m3(f);
    if (fabsf(f) > 448.0f) return (uint8_t)((bits_from_f32(f) >> 24 & 0x80u) | 0x7Eu);
    return orc_f32_to_e4m3(f);
}

static void store_rope(void* out, int64_t idx, float v, int mode) {
    if (mode == 0) ((uint16_t*)out)[idx] = orc_f32_to_bf16(v);
    else if (mode == 1) ((uint8_t*)out)[idx] = orc_f32_to_e4m3(v);
    else ((uint8_t*)out)[idx] = f32_to_e4m3_sat(v);
}

/*
 * Interleaved RoPE (rms_norm_rope_cuda.cu:125-170):
 *   n = rsqrt(sum(x^2) * (1/dim)); v = x * (n * w) (or x * n);
 *   out[2i] = v[2i] cos[2i] - v[2i+1] sin[2i]; out[2i+1] = v[2i+1] cos[2i+1] + v[2i] sin[2i+1]
 *   (as fmaf(v0, c, -(v1 s)) and fmaf(v1, c, v0 s)).
 * cos/sin row r at p + r * f_rs; w may be NULL; out_mode 0 bf16, 1 e4m3 (torch conversion).
 */
void orc_rms_norm_rope(const uint16_t* x, int64_t rows, int64_t dim, const uint16_t* cosf, const uint16_t* sinf,
                       int64_t f_rs, const uint16_t* w, void* out, int out_mode) {
    float* v = (float*)malloc(sizeof(float) * (size_t)dim);
    volatile float inv_dim = 1.0f / (float)dim;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t h = 0; h < dim; ++h) v[h] = orc_bf16_to_f32(x[r * dim + h]);
        float ss = row_sumsq_fma(v, dim);
        volatile float m = ss * inv_dim;
        float n = rsqrt_ieee(m);
        for (int64_t h = 0; h < dim; ++h) {
            volatile float sc = w ? n * orc_bf16_to_f32(w[h]) : n;
            volatile float t = v[h] * sc;
            v[h] = t;
        }
        const uint16_t* cr = cosf + r * f_rs;
        const uint16_t* sr = sinf + r * f_rs;
        for (int64_t h = 0; h < dim; h += 2) {
            volatile float a = v[h + 1] * orc_bf16_to_f32(sr[h]);
            float o0 = fmaf(v[h], orc_bf16_to_f32(cr[h]), -a);
            volatile float b = v[h] * orc_bf16_to_f32(sr[h + 1]);
            float o1 = fmaf(v[h + 1], orc_bf16_to_f32(cr[h + 1]), b);
            store_rope(out, r * dim + h, o0, out_mode);
            store_rope(out, r * dim + h + 1, o1, out_mode);
        }
    }
    free(v);
}

/*
 * Split RoPE (rms_norm_split_rope_cuda.cu:73-140): heads of d = H / heads, halves
 * a = [0, d/2), b = [d/2, d); r = rsqrt(sum(x^2) / H + 1e-6); v = (x * r) * w;
 *   out_a[j] = fmaf(-sin[j], v_b[j], cos[j] v_a[j]); out_b[j] = fmaf(sin[j], v_a[j], cos[j] v_b[j])
 * cos/sin element (b, head, s, j) at p[b * sb + head * sn + s * ss + j]; w may be NULL;
 * out_mode 0 bf16, 2 saturating e4m3.
 */
void orc_rms_norm_split_rope(const uint16_t* x, int64_t B, int64_t S, int64_t H, int64_t heads,
                             const uint16_t* cosf, int64_t c_sb, int64_t c_sn, int64_t c_ss,
                             const uint16_t* sinf, int64_t s_sb, int64_t s_sn, int64_t s_ss,
                             const uint16_t* w, void* out, int out_mode) {
    float* v = (float*)malloc(sizeof(float) * (size_t)H);
    int64_t d = H / heads, half = d / 2;
    for (int64_t b = 0; b < B; ++b)
        for (int64_t s = 0; s < S; ++s) {
            int64_t r = b * S + s;
            for (int64_t h = 0; h < H; ++h) v[h] = orc_bf16_to_f32(x[r * H + h]);
            float ss = row_sumsq_fma(v, H);
            volatile float mean = ss / (float)H;
            volatile float me = mean + 1e-6f;
            float rr = rsqrt_ieee(me);
            for (int64_t h = 0; h < H; ++h) {
                volatile float t = v[h] * rr;
                if (w) { volatile float u = t * orc_bf16_to_f32(w[h]); v[h] = u; }
                else v[h] = t;
            }
            for (int64_t e = 0; e < H; ++e) {
                int64_t hd = e / d, p = e % d;
                int first = p < half;
                int64_t j = first ? p : p - half;
                float cs = orc_bf16_to_f32(cosf[b * c_sb + hd * c_sn + s * c_ss + j]);
                float sn = orc_bf16_to_f32(sinf[b * s_sb + hd * s_sn + s * s_ss + j]);
                float other = v[first ? e + half : e - half];
                volatile float cv = cs * v[e];
                float o = fmaf(first ? -sn : sn, other, cv);
                store_rope(out, r * H + e, o, out_mode);
            }
        }
    free(v);
}
