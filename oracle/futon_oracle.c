/*
 * futon_oracle.c — CPU restatement of futon's encoder forward pass.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path, never part
 * of it. See futon_oracle.h for the reference files restated and the parity
 * pin. Compile with -ffp-contract=off (no fused multiply-adds): Go does not
 * fuse on amd64 (mathf32.go:14-16), and every float32 expression below is
 * evaluated in the same order and precision as the Go source it cites.
 */
#include "futon_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

#define SET_ERR(...) do { if (err && errlen) snprintf(err, errlen, __VA_ARGS__); } while (0)

/* ------------------------------------------------------------------------ */
/* float32 transcendentals — native/mathf32.go:22-120                        */
/* ------------------------------------------------------------------------ */

static const float kExpOverflow = 88.72283f;    /* mathf32.go:27 */
static const float kExpUnderflow = -87.33654f;  /* mathf32.go:28 */
static const float kExpClampLo = -104.0f;       /* mathf32.go:31 */
static const float kLog2e = 1.4426950408889634f;
static const float kLn2Hi = 0.693145751953125f;
static const float kLn2Lo = 1.428606820309417e-06f;
static const float kRoundMagic = 12582912.0f;

static inline float f32_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* expF32, mathf32.go:44-72: range reduction x = k ln2 + r, Cephes single-
 * precision minimax polynomial, scale by 2^k. */
float fo_exp(float x) {
    if (x < kExpUnderflow) return 0.0f;
    float kf = (x * kLog2e + kRoundMagic) - kRoundMagic;
    int32_t k = (int32_t)kf;
    float r = x - kf * kLn2Hi;
    r -= kf * kLn2Lo;
    float p = 1.9875691500e-4f;
    p = p * r + 1.3981999507e-3f;
    p = p * r + 8.3334519073e-3f;
    p = p * r + 4.1665795894e-2f;
    p = p * r + 1.6666665459e-1f;
    p = p * r + 5.0000001201e-1f;
    p = (p * r + 1.0f) * r + 1.0f;
    int32_t e = k + 127;
    if (e <= 0) return 0.0f;
    if (e >= 255) return p * f32_from_bits((uint32_t)(e - 1) << 23) * 2.0f;
    return p * f32_from_bits((uint32_t)e << 23);
}

/* erfcPos, mathf32.go:77-94: Numerical Recipes erfcc Chebyshev fit. */
static float erfc_pos(float a) {
    float t = 1.0f / (1.0f + 0.5f * a);
    float p = 0.17087277f;
    p = p * t - 0.82215223f;
    p = p * t + 1.48851587f;
    p = p * t - 1.13520398f;
    p = p * t + 0.27886807f;
    p = p * t - 0.18628806f;
    p = p * t + 0.09678418f;
    p = p * t + 0.37409196f;
    p = p * t + 1.00002368f;
    p = p * t - 1.26551223f;
    float e = p - a * a;
    if (e < kExpClampLo) e = kExpClampLo;
    return t * fo_exp(e);
}

/* geluF32, mathf32.go:100-111: exact-erf GELU through erfc. */
float fo_gelu(float x) {
    const float inv_sqrt2 = 0.7071067811865476f;
    float a = x * inv_sqrt2;
    if (a < 0) a = -a;
    float c = erfc_pos(a);
    if (x < 0) return 0.5f * x * c;
    return 0.5f * x * (2.0f - c);
}

/* sigmoidF32, mathf32.go:115-124. */
float fo_sigmoid(float x) {
    float e = -x;
    if (e < kExpClampLo) e = kExpClampLo;
    if (e > kExpOverflow) return 0.0f;
    return 1.0f / (1.0f + fo_exp(e));
}

/* ------------------------------------------------------------------------ */
/* GEMMs — the Kernel.MatMulT contract (kernel.go:26-36): dst = a·bᵀ + bias  */
/* ------------------------------------------------------------------------ */

/* matMulTRows, kernel.go:223-283. Per output element: s += (((a0 b0 + a1 b1)
 * + a2 b2) + a3 b3) for each 4-chunk of k, then the scalar tail, then +bias.
 * The 4-row micro-kernel and the remainder rows share that per-element
 * order, so one loop restates both. */
void fo_matmul_t(float *dst, const float *a, const float *b, int m, int n, int k,
                 const float *bias) {
    for (int i = 0; i < m; i++) {
        const float *ai = a + (size_t)i * k;
        float *di = dst + (size_t)i * n;
        for (int j = 0; j < n; j++) {
            const float *bj = b + (size_t)j * k;
            float s = 0.0f;
            int p = 0;
            for (; p + 4 <= k; p += 4) {
                float t = ai[p] * bj[p] + ai[p + 1] * bj[p + 1];
                t = t + ai[p + 2] * bj[p + 2];
                t = t + ai[p + 3] * bj[p + 3];
                s += t;
            }
            for (; p < k; p++) s += ai[p] * bj[p];
            if (bias) s += bias[j];
            di[j] = s;
        }
    }
}

int fo_has_avx2(void) {
#if defined(__x86_64__)
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
#else
    return 0;
#endif
}

#if defined(__x86_64__)
/* REDUCE1, kernel_avx2_amd64.s:20-25: fold high 128 onto low, two hadds. */
__attribute__((target("avx2,fma"))) static inline float reduce8(__m256 v) {
    __m128 lo = _mm256_castps256_ps128(v);
    __m128 hi = _mm256_extractf128_ps(v, 1);
    lo = _mm_add_ps(lo, hi);
    lo = _mm_hadd_ps(lo, lo);
    lo = _mm_hadd_ps(lo, lo);
    return _mm_cvtss_f32(lo);
}

/* dot4x2f32 panel (kernel_avx2_amd64.s:77-93) and its Go wrapper
 * (kernel_avx2_amd64.go:47-90): 4 rows × 2 cols, one 8-lane FMA chain per
 * (row, col) over k8 = k &^ 7, fixed reduction, scalar tail, then bias. */
__attribute__((target("avx2,fma"))) static void matmul_avx2_impl(
    float *dst, const float *a, const float *b, int m, int n, int k, const float *bias) {
    int k8 = k & ~7;
    for (int i = 0; i < m; i += 4) {
        int last = m - 1;
        const float *ar[4];
        for (int r = 0; r < 4; r++) ar[r] = a + (size_t)(i + r < last ? i + r : last) * k;
        int rows = m - i < 4 ? m - i : 4;
        for (int j = 0; j < n; j += 2) {
            int j1 = j + 1 < n ? j + 1 : j;
            const float *b0 = b + (size_t)j * k, *b1 = b + (size_t)j1 * k;
            float out[8] = {0};
            if (k8 > 0) {
                __m256 acc[8];
                for (int q = 0; q < 8; q++) acc[q] = _mm256_setzero_ps();
                for (int p = 0; p < k8; p += 8) {
                    __m256 y8 = _mm256_loadu_ps(b0 + p), y9 = _mm256_loadu_ps(b1 + p);
                    for (int r = 0; r < 4; r++) {
                        __m256 av = _mm256_loadu_ps(ar[r] + p);
                        acc[2 * r] = _mm256_fmadd_ps(y8, av, acc[2 * r]);
                        acc[2 * r + 1] = _mm256_fmadd_ps(y9, av, acc[2 * r + 1]);
                    }
                }
                for (int q = 0; q < 8; q++) out[q] = reduce8(acc[q]);
            }
            for (int r = 0; r < rows; r++) {
                const float *arow = a + (size_t)(i + r) * k;
                float s0 = out[2 * r], s1 = out[2 * r + 1];
                for (int p = k8; p < k; p++) {
                    s0 += arow[p] * b0[p];
                    s1 += arow[p] * b1[p];
                }
                if (bias) { s0 += bias[j]; s1 += bias[j1]; }
                dst[(size_t)(i + r) * n + j] = s0;
                if (j1 != j) dst[(size_t)(i + r) * n + j1] = s1;
            }
        }
    }
}
#endif

void fo_matmul_t_avx2(float *dst, const float *a, const float *b, int m, int n, int k,
                      const float *bias) {
#if defined(__x86_64__)
    if (fo_has_avx2()) { matmul_avx2_impl(dst, a, b, m, n, k, bias); return; }
#endif
    fo_matmul_t(dst, a, b, m, n, k, bias);
}

/* ------------------------------------------------------------------------ */
/* Q8 — native/quant.go                                                      */
/* ------------------------------------------------------------------------ */

/* quantizeRowQ8, quant.go:42-70: symmetric absmax, scale = amax/127 (f32),
 * codes round(v * (127/amax)) in float64 with half away from zero, clamped
 * to ±127. An all-zero row gets scale 0 and zero codes. */
float fo_quantize_row_q8(int8_t *dst, const float *src, int n) {
    float amax = 0.0f;
    for (int i = 0; i < n; i++) {
        float v = src[i];
        if (v < 0) v = -v;
        if (v > amax) amax = v;
    }
    if (amax == 0.0f) {
        memset(dst, 0, (size_t)n);
        return 0.0f;
    }
    float scale = amax / 127.0f;
    double inv = 127.0 / (double)amax;
    for (int i = 0; i < n; i++) {
        double q = round((double)src[i] * inv);
        if (q > 127) q = 127;
        else if (q < -127) q = -127;
        dst[i] = (int8_t)q;
    }
    return scale;
}

#if defined(__x86_64__)
/* The exact int32 dot of two int8 rows with AVX2: products widened to int16
 * pairs summed into int32 lanes (|q| <= 127, so a pair is at most 32,258
 * and no lane can overflow for k < 2^17). Integer addition is associative,
 * so the sum is the scalar loop's sum bit for bit, in any order. */
__attribute__((target("avx2"))) static int32_t dot_q8_avx2(const int8_t *a, const int8_t *b, int k) {
    __m256i acc = _mm256_setzero_si256();
    int p = 0;
    for (; p + 16 <= k; p += 16) {
        __m256i va = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)(a + p)));
        __m256i vb = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)(b + p)));
        acc = _mm256_add_epi32(acc, _mm256_madd_epi16(va, vb));
    }
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(acc), _mm256_extracti128_si256(acc, 1));
    s = _mm_hadd_epi32(s, s);
    s = _mm_hadd_epi32(s, s);
    int32_t sum = _mm_cvtsi128_si32(s);
    for (; p < k; p++) sum += (int32_t)a[p] * (int32_t)b[p];
    return sum;
}
#endif

/* matMulTQ8 inner loop, quant.go:114-136, over already-quantised operands:
 * exact int32 dot, then float32(sum) * (sA * sB) + bias. The reference's
 * loop is scalar (quant_amd64.go:5-8); fo_matmul_t_q8_prequant_scalar
 * restates it, and fo_matmul_t_q8_prequant computes the same exact integer
 * sums with AVX2 where the host has it (the CPU suite checks the two agree
 * bit for bit), which makes full-length (2048-token) Q8 forwards practical
 * as a parity check. */
void fo_matmul_t_q8_prequant_scalar(float *dst, const int8_t *qa, const float *a_scale,
                                    const int8_t *qb, const float *b_scale, int m, int n, int k,
                                    const float *bias) {
    for (int i = 0; i < m; i++) {
        const int8_t *ai = qa + (size_t)i * k;
        float sA = a_scale[i];
        for (int j = 0; j < n; j++) {
            const int8_t *bj = qb + (size_t)j * k;
            int32_t sum = 0;
            for (int p = 0; p < k; p++) sum += (int32_t)ai[p] * (int32_t)bj[p];
            float s = (float)sum * (sA * b_scale[j]);
            if (bias) s += bias[j];
            dst[(size_t)i * n + j] = s;
        }
    }
}

void fo_matmul_t_q8_prequant(float *dst, const int8_t *qa, const float *a_scale,
                             const int8_t *qb, const float *b_scale, int m, int n, int k,
                             const float *bias) {
#if defined(__x86_64__)
    if (fo_has_avx2()) {
        for (int i = 0; i < m; i++) {
            const int8_t *ai = qa + (size_t)i * k;
            float sA = a_scale[i];
            for (int j = 0; j < n; j++) {
                int32_t sum = dot_q8_avx2(ai, qb + (size_t)j * k, k);
                float s = (float)sum * (sA * b_scale[j]);
                if (bias) s += bias[j];
                dst[(size_t)i * n + j] = s;
            }
        }
        return;
    }
#endif
    fo_matmul_t_q8_prequant_scalar(dst, qa, a_scale, qb, b_scale, m, n, k, bias);
}

/* matMulTQ8, quant.go:99-137: dynamic per-row activation quantisation, then
 * the exact integer GEMM. */
void fo_matmul_t_q8(float *dst, const float *a, const int8_t *qb, const float *scales,
                    int m, int n, int k, const float *bias) {
    int8_t *qa = (int8_t *)malloc((size_t)m * k + 1);
    float *sa = (float *)malloc(sizeof(float) * (size_t)(m > 0 ? m : 1));
    for (int i = 0; i < m; i++) sa[i] = fo_quantize_row_q8(qa + (size_t)i * k, a + (size_t)i * k, k);
    fo_matmul_t_q8_prequant(dst, qa, sa, qb, scales, m, n, k, bias);
    free(qa);
    free(sa);
}

/* ------------------------------------------------------------------------ */
/* Row ops — native/model.go                                                  */
/* ------------------------------------------------------------------------ */

/* layerNormRows, model.go:743-769: fp64 mean and variance, f32 apply. */
void fo_layernorm_rows(float *x, int rows, int h, const float *w, const float *b, float eps) {
    for (int r = 0; r < rows; r++) {
        float *row = x + (size_t)r * h;
        double mean = 0;
        for (int i = 0; i < h; i++) mean += (double)row[i];
        mean /= (double)h;
        double var = 0;
        for (int i = 0; i < h; i++) {
            double d = (double)row[i] - mean;
            var += d * d;
        }
        var /= (double)h;
        float inv = (float)(1.0 / sqrt(var + (double)eps));
        float mf = (float)mean;
        if (w) {
            for (int i = 0; i < h; i++) row[i] = (row[i] - mf) * inv * w[i] + b[i];
        } else {
            for (int i = 0; i < h; i++) row[i] = (row[i] - mf) * inv;
        }
    }
}

/* softmaxScaled, model.go:717-739. */
void fo_softmax_scaled(float *row, int n, float scale) {
    float maxv = row[0];
    for (int i = 1; i < n; i++) if (row[i] > maxv) maxv = row[i];
    maxv *= scale;
    double sum = 0;
    for (int i = 0; i < n; i++) {
        float d = row[i] * scale - maxv;
        if (d < kExpClampLo) d = kExpClampLo;
        float e = fo_exp(d);
        row[i] = e;
        sum += (double)e;
    }
    float inv = (float)(1.0 / sum);
    for (int i = 0; i < n; i++) row[i] *= inv;
}

/* precomputeRoPE, model.go:306-318: angles in float64, stored as f32. */
void fo_rope_tables(int max_seq, int head_dim, double theta, float *cos_out, float *sin_out) {
    int half = head_dim / 2;
    for (int t = 0; t < max_seq; t++) {
        for (int i = 0; i < half; i++) {
            double freq = 1.0 / pow(theta, (double)(2 * i) / (double)head_dim);
            double angle = (double)t * freq;
            cos_out[(size_t)t * half + i] = (float)cos(angle);
            sin_out[(size_t)t * half + i] = (float)sin(angle);
        }
    }
}

/* rotateHalf, model.go:705-712 (NeoX, non-interleaved). */
static void rotate_half(float *x, const float *c, const float *s, int half) {
    for (int i = 0; i < half; i++) {
        float x1 = x[i], x2 = x[i + half];
        x[i] = x1 * c[i] - x2 * s[i];
        x[i + half] = x2 * c[i] + x1 * s[i];
    }
}

/* ------------------------------------------------------------------------ */
/* Model                                                                     */
/* ------------------------------------------------------------------------ */

enum { Q_QKV = 0, Q_OUT, Q_FC1, Q_GATE, Q_FC2, Q_COUNT };

struct fo_model {
    fo_cfg cfg;
    int head_dim;
    int gemm_mode;
    const float *g[FO_GLOBAL_COUNT];
    const float **layer; /* num_layers * FO_L_COUNT */
    int q8;
    int8_t **q8_data;    /* num_layers * Q_COUNT */
    float **q8_scale;
    float *rope_cos, *rope_sin;
};

int fo_effective_max_seq_len(const fo_model *m) {
    const fo_cfg *c = &m->cfg;
    if (c->max_trained > 0 && c->max_trained < c->max_seq_len) return c->max_trained;
    return c->max_seq_len;
}

fo_model *fo_create(const fo_cfg *cfg, const float *const *tensors, int q8, int gemm_mode,
                    char *err, size_t errlen) {
    if (cfg->hidden <= 0 || cfg->num_heads <= 0 || cfg->hidden % cfg->num_heads != 0 ||
        cfg->num_layers <= 0 || cfg->inter <= 0 || cfg->vocab <= 0) {
        SET_ERR("oracle: invalid architecture");
        return NULL;
    }
    fo_model *m = (fo_model *)calloc(1, sizeof(*m));
    m->cfg = *cfg;
    m->head_dim = cfg->hidden / cfg->num_heads;
    m->gemm_mode = gemm_mode;
    for (int i = 0; i < FO_GLOBAL_COUNT; i++) m->g[i] = tensors[i];
    size_t nl = (size_t)cfg->num_layers * FO_L_COUNT;
    m->layer = (const float **)calloc(nl, sizeof(float *));
    for (size_t i = 0; i < nl; i++) m->layer[i] = tensors[FO_GLOBAL_COUNT + i];

    if (!m->g[FO_WORD] || !m->g[FO_EMB_NORM_W] || !m->g[FO_EMB_NORM_B] ||
        (!cfg->rope && !m->g[FO_POS]) || (cfg->type_vocab > 0 && !m->g[FO_TYPE])) {
        SET_ERR("oracle: missing embedding tensor");
        fo_destroy(m);
        return NULL;
    }
    for (int li = 0; li < cfg->num_layers; li++) {
        const float **L = m->layer + (size_t)li * FO_L_COUNT;
        if (!L[FO_L_QKV_W] || !L[FO_L_OUT_W] || !L[FO_L_NORM1_W] || !L[FO_L_NORM1_B] ||
            !L[FO_L_FC1_W] || !L[FO_L_FC2_W] || !L[FO_L_NORM2_W] || !L[FO_L_NORM2_B] ||
            (cfg->swiglu && !L[FO_L_GATE_W])) {
            SET_ERR("oracle: layer %d missing a required tensor", li);
            fo_destroy(m);
            return NULL;
        }
    }

    /* Requantise the layer GEMM weights (model.go:265-289). */
    m->q8 = q8 ? 1 : 0;
    if (m->q8) {
        int h = cfg->hidden, inter = cfg->inter;
        m->q8_data = (int8_t **)calloc((size_t)cfg->num_layers * Q_COUNT, sizeof(int8_t *));
        m->q8_scale = (float **)calloc((size_t)cfg->num_layers * Q_COUNT, sizeof(float *));
        for (int li = 0; li < cfg->num_layers; li++) {
            const float **L = m->layer + (size_t)li * FO_L_COUNT;
            const float *w[Q_COUNT] = {L[FO_L_QKV_W], L[FO_L_OUT_W], L[FO_L_FC1_W],
                                       L[FO_L_GATE_W], L[FO_L_FC2_W]};
            int nn[Q_COUNT] = {3 * h, h, inter, inter, h};
            int kk[Q_COUNT] = {h, h, h, h, inter};
            for (int s = 0; s < Q_COUNT; s++) {
                if (!w[s]) continue;
                int8_t *d = (int8_t *)malloc((size_t)nn[s] * kk[s]);
                float *sc = (float *)malloc(sizeof(float) * (size_t)nn[s]);
                for (int j = 0; j < nn[s]; j++)
                    sc[j] = fo_quantize_row_q8(d + (size_t)j * kk[s], w[s] + (size_t)j * kk[s], kk[s]);
                m->q8_data[li * Q_COUNT + s] = d;
                m->q8_scale[li * Q_COUNT + s] = sc;
            }
        }
    }
    if (cfg->rope) {
        int ms = fo_effective_max_seq_len(m);
        int half = m->head_dim / 2;
        m->rope_cos = (float *)malloc(sizeof(float) * (size_t)ms * (half > 0 ? half : 1));
        m->rope_sin = (float *)malloc(sizeof(float) * (size_t)ms * (half > 0 ? half : 1));
        fo_rope_tables(ms, m->head_dim, cfg->rope_theta, m->rope_cos, m->rope_sin);
    }
    return m;
}

void fo_destroy(fo_model *m) {
    if (!m) return;
    if (m->q8_data) {
        for (int i = 0; i < m->cfg.num_layers * Q_COUNT; i++) {
            free(m->q8_data[i]);
            free(m->q8_scale[i]);
        }
        free(m->q8_data);
        free(m->q8_scale);
    }
    free(m->rope_cos);
    free(m->rope_sin);
    free((void *)m->layer);
    free(m);
}

const int8_t *fo_q8_data(const fo_model *m, int li, int slot) {
    if (!m->q8 || li < 0 || li >= m->cfg.num_layers || slot < 0 || slot >= Q_COUNT) return NULL;
    return m->q8_data[li * Q_COUNT + slot];
}
const float *fo_q8_scale(const fo_model *m, int li, int slot) {
    if (!m->q8 || li < 0 || li >= m->cfg.num_layers || slot < 0 || slot >= Q_COUNT) return NULL;
    return m->q8_scale[li * Q_COUNT + slot];
}

/* mmT, model.go:74-88: dispatch to the Q8 or float GEMM. */
static void mmt(const fo_model *m, float *dst, const float *a, int li, int slot,
                const float *w, int rows, int n, int k, const float *bias) {
    if (m->q8) {
        fo_matmul_t_q8(dst, a, m->q8_data[li * Q_COUNT + slot], m->q8_scale[li * Q_COUNT + slot],
                       rows, n, k, bias);
        return;
    }
    if (m->gemm_mode == FO_GEMM_AVX2) fo_matmul_t_avx2(dst, a, w, rows, n, k, bias);
    else fo_matmul_t(dst, a, w, rows, n, k, bias);
}

typedef struct {
    float *x, *pooled, *qkv, *q, *k, *vT, *scores, *head_out, *attn_cat, *attn_out, *ffn_h,
        *ffn_gate, *ffn_out;
} scratch_t;

static int pad_seq(int seq) { return (seq + 7) & ~7; } /* model.go:532 */

/* attendHead, model.go:646-701, for one head of one sequence: qkv holds the
 * sequence's [seq, 3h] rows; the first `rows` queries (seq, or 1 for the
 * CLS-pruned last layer, model.go:403-410) attend over all seq keys (padded
 * to a multiple of 8 with zeros, model.go:532); head_out receives [rows, hd].
 * rope_cos/rope_sin ([positions, hd/2]) are NULL for absolute-position packs.
 * q [seq, hd], k [kp, hd], vT [hd, kp] and scores [rows, kp] are scratch. */
static void attend_head_core(int gemm_mode, const float *qkv, int seq, int rows, int h, int hd,
                             int head, const float *rope_cos, const float *rope_sin, float *q,
                             float *k, float *vT, float *scores, float *head_out) {
    int half = hd / 2;
    float scale = (float)(1.0 / sqrt((double)hd));
    int kp = pad_seq(seq);
    memset(k + (size_t)seq * hd, 0, sizeof(float) * (size_t)(kp - seq) * hd);
    for (int d = 0; d < hd; d++)
        memset(vT + (size_t)d * kp + seq, 0, sizeof(float) * (size_t)(kp - seq));
    int qo = head * hd, ko = h + head * hd, vo = 2 * h + head * hd;
    for (int t = 0; t < seq; t++) {
        const float *row = qkv + (size_t)t * 3 * h;
        if (t < rows) memcpy(q + (size_t)t * hd, row + qo, sizeof(float) * hd);
        memcpy(k + (size_t)t * hd, row + ko, sizeof(float) * hd);
        for (int d = 0; d < hd; d++) vT[(size_t)d * kp + t] = row[vo + d];
    }
    if (rope_cos) {
        for (int t = 0; t < seq; t++) {
            const float *c = rope_cos + (size_t)t * half, *sn = rope_sin + (size_t)t * half;
            if (t < rows) rotate_half(q + (size_t)t * hd, c, sn, half);
            rotate_half(k + (size_t)t * hd, c, sn, half);
        }
    }
    if (gemm_mode == FO_GEMM_AVX2) fo_matmul_t_avx2(scores, q, k, rows, kp, hd, NULL);
    else fo_matmul_t(scores, q, k, rows, kp, hd, NULL);
    for (int t = 0; t < rows; t++) {
        float *row = scores + (size_t)t * kp;
        fo_softmax_scaled(row, seq, scale);
        memset(row + seq, 0, sizeof(float) * (size_t)(kp - seq));
    }
    if (gemm_mode == FO_GEMM_AVX2) fo_matmul_t_avx2(head_out, scores, vT, rows, hd, kp, NULL);
    else fo_matmul_t(head_out, scores, vT, rows, hd, kp, NULL);
}

static void attend_head(const fo_model *m, scratch_t *s, int head, int seq, int rows) {
    int h = m->cfg.hidden, hd = m->head_dim;
    attend_head_core(m->gemm_mode, s->qkv, seq, rows, h, hd, head,
                     m->cfg.rope ? m->rope_cos : NULL, m->cfg.rope ? m->rope_sin : NULL, s->q,
                     s->k, s->vT, s->scores, s->head_out);
    for (int t = 0; t < rows; t++)
        memcpy(s->attn_cat + (size_t)t * h + head * hd, s->head_out + (size_t)t * hd,
               sizeof(float) * hd);
}

int fo_attend_head(const float *qkv, int seq, int rows, int h, int hd, int head,
                   const float *rope_cos, const float *rope_sin, int gemm_mode, float *out) {
    if (seq <= 0 || rows <= 0 || rows > seq || hd <= 0 || h % hd || head < 0 || head >= h / hd)
        return -1;
    int kp = pad_seq(seq);
    size_t n = (size_t)seq * hd + (size_t)kp * hd + (size_t)hd * kp + (size_t)rows * kp;
    float *buf = (float *)calloc(n, sizeof(float));
    if (!buf) return -1;
    float *q = buf, *k = q + (size_t)seq * hd, *vT = k + (size_t)kp * hd, *sc = vT + (size_t)hd * kp;
    attend_head_core(gemm_mode, qkv, seq, rows, h, hd, head, rope_cos, rope_sin, q, k, vT, sc, out);
    free(buf);
    return 0;
}

static void add_into(float *dst, const float *src, size_t n) {
    for (size_t i = 0; i < n; i++) dst[i] += src[i];
}

/* layerForward, model.go:550-635. */
static void layer_forward(const fo_model *m, int li, scratch_t *s, int seq, int rows) {
    const fo_cfg *c = &m->cfg;
    int h = c->hidden, inter = c->inter;
    const float **L = m->layer + (size_t)li * FO_L_COUNT;
    float eps = (float)c->eps;
    mmt(m, s->qkv, s->x, li, Q_QKV, L[FO_L_QKV_W], seq, 3 * h, h, L[FO_L_QKV_B]);
    for (int head = 0; head < c->num_heads; head++) attend_head(m, s, head, seq, rows);
    mmt(m, s->attn_out, s->attn_cat, li, Q_OUT, L[FO_L_OUT_W], rows, h, h, L[FO_L_OUT_B]);
    add_into(s->attn_out, s->x, (size_t)rows * h);
    memcpy(s->x, s->attn_out, sizeof(float) * (size_t)rows * h);
    fo_layernorm_rows(s->x, rows, h, L[FO_L_NORM1_W], L[FO_L_NORM1_B], eps);
    size_t ne = (size_t)rows * inter;
    if (!c->swiglu) {
        mmt(m, s->ffn_h, s->x, li, Q_FC1, L[FO_L_FC1_W], rows, inter, h, L[FO_L_FC1_B]);
        for (size_t i = 0; i < ne; i++) s->ffn_h[i] = fo_gelu(s->ffn_h[i]);
    } else {
        mmt(m, s->ffn_h, s->x, li, Q_FC1, L[FO_L_FC1_W], rows, inter, h, L[FO_L_FC1_B]);
        mmt(m, s->ffn_gate, s->x, li, Q_GATE, L[FO_L_GATE_W], rows, inter, h, L[FO_L_GATE_B]);
        for (size_t i = 0; i < ne; i++) {
            float g = s->ffn_gate[i];
            s->ffn_h[i] *= g * fo_sigmoid(g);
        }
    }
    mmt(m, s->ffn_out, s->ffn_h, li, Q_FC2, L[FO_L_FC2_W], rows, h, inter, L[FO_L_FC2_B]);
    add_into(s->ffn_out, s->x, (size_t)rows * h);
    memcpy(s->x, s->ffn_out, sizeof(float) * (size_t)rows * h);
    fo_layernorm_rows(s->x, rows, h, L[FO_L_NORM2_W], L[FO_L_NORM2_B], eps);
}

/* EncodeTokensKernel, model.go:346-457. */
int fo_encode(const fo_model *m, const int32_t *ids, int n, int out_dim, float *out, char *err,
              size_t errlen) {
    const fo_cfg *c = &m->cfg;
    if (n <= 0) { SET_ERR("native: empty token sequence"); return -1; }
    int emax = fo_effective_max_seq_len(m);
    if (n > emax) {
        SET_ERR("native: sequence length %d exceeds effective max_seq_len %d", n, emax);
        return -1;
    }
    if (out_dim < 0 || out_dim > c->hidden) {
        SET_ERR("native: requested dim %d outside [1,%d]", out_dim, c->hidden);
        return -1;
    }
    if (out_dim != 0 && out_dim != c->hidden && !c->matryoshka) {
        SET_ERR("native: pack does not support matryoshka truncation to %d", out_dim);
        return -1;
    }
    for (int t = 0; t < n; t++) {
        if (ids[t] < 0 || ids[t] >= c->vocab) {
            SET_ERR("native: token id %d outside vocab of %d", ids[t], c->vocab);
            return -1;
        }
    }
    int seq = n, h = c->hidden, inter = c->inter, hd = m->head_dim, kp = pad_seq(seq);
    scratch_t s;
    size_t tot = 0;
    size_t sz[13] = {(size_t)seq * h, (size_t)h, (size_t)seq * 3 * h, (size_t)seq * hd,
                     (size_t)kp * hd, (size_t)hd * kp, (size_t)seq * kp, (size_t)seq * hd,
                     (size_t)seq * h, (size_t)seq * h, (size_t)seq * inter,
                     (size_t)seq * inter, (size_t)seq * h};
    for (int i = 0; i < 13; i++) tot += sz[i];
    float *buf = (float *)calloc(tot, sizeof(float));
    if (!buf) { SET_ERR("oracle: out of memory"); return -1; }
    float **slots[13] = {&s.x, &s.pooled, &s.qkv, &s.q, &s.k, &s.vT, &s.scores, &s.head_out,
                         &s.attn_cat, &s.attn_out, &s.ffn_h, &s.ffn_gate, &s.ffn_out};
    size_t off = 0;
    for (int i = 0; i < 13; i++) { *slots[i] = buf + off; off += sz[i]; }

    /* Embeddings (model.go:384-396). */
    for (int t = 0; t < seq; t++) {
        float *row = s.x + (size_t)t * h;
        memcpy(row, m->g[FO_WORD] + (size_t)ids[t] * h, sizeof(float) * h);
        if (c->type_vocab > 0) add_into(row, m->g[FO_TYPE], (size_t)h);
        if (!c->rope) add_into(row, m->g[FO_POS] + (size_t)t * h, (size_t)h);
    }
    fo_layernorm_rows(s.x, seq, h, m->g[FO_EMB_NORM_W], m->g[FO_EMB_NORM_B], (float)c->eps);

    for (int li = 0; li < c->num_layers; li++) {
        int rows = (li == c->num_layers - 1 && !c->pool_mean) ? 1 : seq;
        layer_forward(m, li, &s, seq, rows);
    }

    /* Pooling (model.go:416-430). */
    memset(s.pooled, 0, sizeof(float) * h);
    if (!c->pool_mean) {
        memcpy(s.pooled, s.x, sizeof(float) * h);
    } else {
        for (int t = 0; t < seq; t++) add_into(s.pooled, s.x + (size_t)t * h, (size_t)h);
        float inv = 1.0f / (float)seq;
        for (int i = 0; i < h; i++) s.pooled[i] *= inv;
    }
    int d = h;
    /* Matryoshka (model.go:433-439). */
    if (out_dim != 0 && out_dim != h) {
        if (c->matryoshka_ln) fo_layernorm_rows(s.pooled, 1, h, NULL, NULL, 1e-5f);
        d = out_dim;
    }
    /* L2 (model.go:441-453). */
    if (c->normalize) {
        double ss = 0;
        for (int i = 0; i < d; i++) ss += (double)s.pooled[i] * (double)s.pooled[i];
        if (ss > 0) {
            float inv = (float)(1.0 / sqrt(ss));
            for (int i = 0; i < d; i++) s.pooled[i] *= inv;
        }
    }
    memcpy(out, s.pooled, sizeof(float) * d);
    free(buf);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Batch: bounded worker pool, longest first (provider.go:152-202)           */
/* ------------------------------------------------------------------------ */

typedef struct {
    const fo_model *m;
    const int32_t *ids, *cu;
    const int *order;
    int nseq, out_dim, dim;
    float *out;
    int next;
    int failed;
    pthread_mutex_t mu;
    char *err;
    size_t errlen;
} batch_t;

static void *batch_worker(void *arg) {
    batch_t *b = (batch_t *)arg;
    char local[256];
    for (;;) {
        pthread_mutex_lock(&b->mu);
        int idx = b->next < b->nseq && !b->failed ? b->order[b->next++] : -1;
        pthread_mutex_unlock(&b->mu);
        if (idx < 0) break;
        int lo = b->cu[idx], n = b->cu[idx + 1] - lo;
        if (fo_encode(b->m, b->ids + lo, n, b->out_dim, b->out + (size_t)idx * b->dim, local,
                      sizeof local) != 0) {
            pthread_mutex_lock(&b->mu);
            if (!b->failed) {
                b->failed = 1;
                if (b->err && b->errlen) snprintf(b->err, b->errlen, "native: batch item %d: %s", idx, local);
            }
            pthread_mutex_unlock(&b->mu);
        }
    }
    return NULL;
}

static const int32_t *g_sort_cu;
static int cmp_len_desc(const void *pa, const void *pb) {
    int a = *(const int *)pa, b = *(const int *)pb;
    int la = g_sort_cu[a + 1] - g_sort_cu[a], lb = g_sort_cu[b + 1] - g_sort_cu[b];
    if (la != lb) return lb - la;
    return a - b; /* stable */
}

int fo_encode_batch(const fo_model *m, const int32_t *ids, const int32_t *cu_seqlens, int nseq,
                    int out_dim, float *out, int threads, char *err, size_t errlen) {
    if (nseq <= 0) return 0;
    if (threads < 1) threads = 1;
    if (threads > nseq) threads = nseq;
    int *order = (int *)malloc(sizeof(int) * (size_t)nseq);
    for (int i = 0; i < nseq; i++) order[i] = i;
    static pthread_mutex_t sort_mu = PTHREAD_MUTEX_INITIALIZER;
    pthread_mutex_lock(&sort_mu);
    g_sort_cu = cu_seqlens;
    qsort(order, (size_t)nseq, sizeof(int), cmp_len_desc);
    pthread_mutex_unlock(&sort_mu);
    batch_t b;
    memset(&b, 0, sizeof b);
    b.m = m; b.ids = ids; b.cu = cu_seqlens; b.order = order; b.nseq = nseq;
    b.out_dim = out_dim;
    b.dim = (out_dim == 0) ? m->cfg.hidden : out_dim;
    b.out = out; b.err = err; b.errlen = errlen;
    pthread_mutex_init(&b.mu, NULL);
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    for (int t = 0; t < threads; t++) pthread_create(&th[t], NULL, batch_worker, &b);
    for (int t = 0; t < threads; t++) pthread_join(th[t], NULL);
    pthread_mutex_destroy(&b.mu);
    free(th);
    free(order);
    return b.failed ? -1 : 0;
}
