/* CPU oracle: fp32 restatement of the reference's DiT / PatchEncoder math.
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Paths in citations are relative
 * to the MaurerAnton/dots.tts.cpp source tree. */
#include "oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* --------------------------------------------------------------------------
 * primitives
 * ------------------------------------------------------------------------ */

/* LayerNorm without affine, eps 1e-5 (include/dit_manual.h:16-21). */
static void ln_noaffine(float *out, const float *x, int n) {
    float mean = 0.0f;
    for (int i = 0; i < n; i++) mean += x[i];
    mean /= (float)n;
    float var = 0.0f;
    for (int i = 0; i < n; i++) { float d = x[i] - mean; var += d * d; }
    float inv = 1.0f / sqrtf(var / (float)n + 1e-5f);
    for (int i = 0; i < n; i++) out[i] = (x[i] - mean) * inv;
}

/* y = W x + b for one row, accumulated in input order (include/dit_manual.h:30-61). */
static void linear1(float *y, const float *x, const float *w, const float *b, int in, int out) {
    for (int o = 0; o < out; o++) {
        const float *wr = w + (size_t)o * in;
        float s = 0.0f;
        for (int i = 0; i < in; i++) s += wr[i] * x[i];
        y[o] = b ? b[o] + s : s;
    }
}

void orc_linear_rows(float *y, const float *x, int rows, const float *w, const float *b, int in, int out) {
    #pragma omp parallel for schedule(static)
    for (int o = 0; o < out; o++) {
        const float *wr = w + (size_t)o * in;
        for (int r = 0; r < rows; r++) {
            const float *xr = x + (size_t)r * in;
            float s = 0.0f;
            for (int i = 0; i < in; i++) s += wr[i] * xr[i];
            y[(size_t)r * out + o] = b ? b[o] + s : s;
        }
    }
}

static float silu(float x) { return x / (1.0f + expf(-x)); }

/* GELU, tanh approximation (include/dit_manual.h:186-192). */
static float gelu_tanh(float x) {
    const float c1 = 0.7978845608028654f, c2 = 0.044715f;
    float x3 = x * x * x;
    return 0.5f * x * (1.0f + tanhf(c1 * (x + c2 * x3)));
}

/* --------------------------------------------------------------------------
 * conditioning
 * ------------------------------------------------------------------------ */

/* Sinusoid [cos(t f_i) | sin(t f_i)], f_i = exp(-ln(1e4) i / 128)
 * (src/e2e_pipeline_v4.cpp:58-60, src/modules/backbone/dit_forward.cpp:23-25). */
void orc_sinusoid(float t, float *se) {
    const int half = 128;
    for (int i = 0; i < half; i++) {
        float f = expf(-logf(10000.0f) * (float)i / (float)half);
        se[i] = cosf(t * f);
        se[half + i] = sinf(t * f);
    }
}

/* compute_cond with speaker_scale (src/e2e_pipeline_v4.cpp:57-71). */
void orc_compute_cond(const orc_dit *m, float t, const float *spk, float spk_scale, float *cond) {
    float se[256], h1[ORC_D];
    orc_sinusoid(t, se);
    linear1(h1, se, m->t_w1, m->t_b1, 256, ORC_D);
    for (int o = 0; o < ORC_D; o++) h1[o] = h1[o] / (1.0f + expf(-h1[o]));
    linear1(cond, h1, m->t_w2, m->t_b2, ORC_D, ORC_D);
    if (spk) {
        float tt[ORC_D];
        linear1(tt, spk, m->spk_w1, m->spk_b1, ORC_SPK, ORC_D);
        float mean = 0.0f;
        for (int i = 0; i < ORC_D; i++) mean += tt[i];
        mean /= ORC_D;
        float var = 0.0f;
        for (int i = 0; i < ORC_D; i++) { float d = tt[i] - mean; var += d * d; }
        var = var / ORC_D + 1e-5f;
        float istd = 1.0f / sqrtf(var);
        for (int i = 0; i < ORC_D; i++) {
            float x = (tt[i] - mean) * istd;
            if (m->spk_ln_w) x *= m->spk_ln_w[i];
            if (m->spk_ln_b) x += m->spk_ln_b[i];
            cond[i] += x * spk_scale;
        }
    }
}

/* --------------------------------------------------------------------------
 * attention (include/dit_manual.h:88-146)
 * Q,K,V without bias; per-head RMS qk-norm eps 1e-6 with a [64] gain; RoPE
 * half-split on pos (or 0..L-1), theta advanced multiplicatively; scores
 * scaled by 1/sqrt(64); masked entries -inf; softmax; P.V; O projection.
 * ------------------------------------------------------------------------ */
static void rms_head(float *v, const float *g) {
    float ss = 0.0f;
    for (int d = 0; d < ORC_HD; d++) ss += v[d] * v[d];
    float inv = 1.0f / sqrtf(ss / ORC_HD + 1e-6f);
    for (int d = 0; d < ORC_HD; d++) { float y = v[d] * inv; if (g) y *= g[d]; v[d] = y; }
}

/* DiT RoPE pairing: ORC_ROPE_HALF (manual_attention, include/dit_manual.h:111-128)
 * or ORC_ROPE_ADJACENT (ggml_rope mode 0 as called by the hybrid DiT path,
 * src/modules/backbone/dit_attention.cpp:53-54). */
static int g_dit_rope = ORC_ROPE_HALF;
void orc_set_dit_rope(int mode) { g_dit_rope = mode; }

static void rope_adjacent(float *v, int p);

static void rope_half(float *q, float *k, float pos) {
    const int half = ORC_HD / 2;
    float theta = 1.0f;
    float ts = powf(10000.0f, -2.0f / (float)ORC_HD);
    for (int d = 0; d < half; d++) {
        float cs = cosf(pos * theta), sn = sinf(pos * theta);
        float q0 = q[d], q1 = q[d + half], k0 = k[d], k1 = k[d + half];
        q[d] = q0 * cs - q1 * sn; q[d + half] = q1 * cs + q0 * sn;
        k[d] = k0 * cs - k1 * sn; k[d + half] = k1 * cs + k0 * sn;
        theta *= ts;
    }
}

void orc_attention(float *out, const float *x, int L,
                   const float *wq, const float *wk, const float *wv, const float *wo,
                   const float *bo, const float *qn, const float *kn,
                   const uint8_t *mask, const float *pos) {
    size_t n = (size_t)L * ORC_D;
    float *q = (float *)malloc(n * sizeof(float));
    float *k = (float *)malloc(n * sizeof(float));
    float *v = (float *)malloc(n * sizeof(float));
    float *ctx = (float *)malloc(n * sizeof(float));
    orc_linear_rows(q, x, L, wq, NULL, ORC_D, ORC_D);
    orc_linear_rows(k, x, L, wk, NULL, ORC_D, ORC_D);
    orc_linear_rows(v, x, L, wv, NULL, ORC_D, ORC_D);
    /* per (token, head): norm + rope (the reference copies heads out, normalises
     * then rotates; per-token order is identical) */
    #pragma omp parallel for schedule(static)
    for (int t = 0; t < L; t++) {
        for (int h = 0; h < ORC_H; h++) {
            float *qh = q + (size_t)t * ORC_D + h * ORC_HD;
            float *kh = k + (size_t)t * ORC_D + h * ORC_HD;
            rms_head(qh, qn);
            rms_head(kh, kn);
            if (g_dit_rope == ORC_ROPE_ADJACENT) {
                rope_adjacent(qh, pos ? (int)pos[t] : t);
                rope_adjacent(kh, pos ? (int)pos[t] : t);
            } else {
                rope_half(qh, kh, pos ? pos[t] : (float)t);
            }
        }
    }
    const float scale = 1.0f / sqrtf((float)ORC_HD);
    #pragma omp parallel
    {
        float *s = (float *)malloc((size_t)L * sizeof(float));
        #pragma omp for collapse(2) schedule(static)
        for (int h = 0; h < ORC_H; h++) {
            for (int i = 0; i < L; i++) {
                const float *qi = q + (size_t)i * ORC_D + h * ORC_HD;
                for (int j = 0; j < L; j++) {
                    const float *kj = k + (size_t)j * ORC_D + h * ORC_HD;
                    float acc = 0.0f;
                    for (int d = 0; d < ORC_HD; d++) acc += qi[d] * kj[d];
                    s[j] = acc * scale;
                    if (mask && !mask[(size_t)i * L + j]) s[j] = -INFINITY;
                }
                /* manual_softmax (include/dit_manual.h:83-86) */
                float mx = s[0];
                for (int j = 1; j < L; j++) if (s[j] > mx) mx = s[j];
                float sum = 0.0f;
                for (int j = 0; j < L; j++) { s[j] = expf(s[j] - mx); sum += s[j]; }
                for (int j = 0; j < L; j++) s[j] /= sum;
                float *ci = ctx + (size_t)i * ORC_D + h * ORC_HD;
                for (int d = 0; d < ORC_HD; d++) {
                    float acc = 0.0f;
                    for (int j = 0; j < L; j++) acc += s[j] * v[(size_t)j * ORC_D + h * ORC_HD + d];
                    ci[d] = acc;
                }
            }
        }
        free(s);
    }
    orc_linear_rows(out, ctx, L, wo, bo, ORC_D, ORC_D);
    free(q); free(k); free(v); free(ctx);
}

/* --------------------------------------------------------------------------
 * DiT block (include/dit_manual.h:148-199)
 * ada = W_ada SiLU(c) + b -> shift_msa, scale_msa, gate_msa, shift_mlp,
 * scale_mlp, gate_mlp; h = x + g_msa * Attn(LN(x)(1+s)+sh);
 * out = h + g_mlp * FFN(LN(h)(1+s')+sh'), FFN = W2 GELU_tanh(W1 u + b1) + b2.
 * ffn_mode ORC_FFN_AS_WRITTEN reproduces the shipped code, whose FFN projects
 * token 0 only and leaves rows 1.. of the GELU input at whatever the
 * thread_local scratch held (zero on the first call of a fresh thread); this
 * restatement uses zeros for those rows.
 * ------------------------------------------------------------------------ */
static void dit_adaln(float *ada, const float *cond, const float *w, const float *b, int nout) {
    float cs[ORC_D];
    for (int i = 0; i < ORC_D; i++) cs[i] = cond[i] / (1.0f + expf(-cond[i]));
    #pragma omp parallel for schedule(static)
    for (int o = 0; o < nout; o++) {
        float s = b ? b[o] : 0.0f;
        const float *wr = w + (size_t)o * ORC_D;
        for (int i = 0; i < ORC_D; i++) s += wr[i] * cs[i];
        ada[o] = s;
    }
}

static void dit_block_fwd_fp8(float *out, const float *x, const float *cond, const orc_dit_block *b,
                              int L, const uint8_t *mask, const float *pos);
static int g_dit_fp8;

void orc_dit_block_fwd(float *out, const float *x, const float *cond, const orc_dit_block *b,
                       int L, const uint8_t *mask, const float *pos, int ffn_mode) {
    if (g_dit_fp8 && ffn_mode == ORC_FFN_PER_TOKEN) { dit_block_fwd_fp8(out, x, cond, b, L, mask, pos); return; }
    const int D = ORC_D;
    float *ada = (float *)malloc(6 * D * sizeof(float));
    dit_adaln(ada, cond, b->ada_w, b->ada_b, 6 * D);
    const float *sm = ada, *scm = ada + D, *gm = ada + 2 * D;
    const float *sml = ada + 3 * D, *scl = ada + 4 * D, *gml = ada + 5 * D;
    size_t n = (size_t)L * D;
    float *mod = (float *)malloc(n * sizeof(float));
    float *ao = (float *)malloc(n * sizeof(float));
    float *h = (float *)malloc(n * sizeof(float));
    for (int t = 0; t < L; t++) {
        float *mr = mod + (size_t)t * D;
        ln_noaffine(mr, x + (size_t)t * D, D);
        for (int i = 0; i < D; i++) mr[i] = mr[i] * (1.0f + scm[i]) + sm[i];
    }
    orc_attention(ao, mod, L, b->wq, b->wk, b->wv, b->wo, b->bo, b->qn, b->kn, mask, pos);
    for (size_t i = 0; i < n; i++) h[i] = x[i] + gm[i % D] * ao[i];
    for (int t = 0; t < L; t++) {
        float *mr = mod + (size_t)t * D;
        ln_noaffine(mr, h + (size_t)t * D, D);
        for (int i = 0; i < D; i++) mr[i] = mr[i] * (1.0f + scl[i]) + sml[i];
    }
    float *f1 = (float *)calloc((size_t)L * ORC_F, sizeof(float));
    float *f2 = (float *)calloc(n, sizeof(float));
    int rows = (ffn_mode == ORC_FFN_AS_WRITTEN) ? 1 : L;
    orc_linear_rows(f1, mod, rows, b->w1, b->b1, D, ORC_F);
    for (size_t i = 0; i < (size_t)L * ORC_F; i++) f1[i] = gelu_tanh(f1[i]);
    orc_linear_rows(f2, f1, rows, b->w2, b->b2, ORC_F, D);
    for (size_t i = 0; i < n; i++) out[i] = h[i] + gml[i % D] * f2[i];
    free(ada); free(mod); free(ao); free(h); free(f1); free(f2);
}

/* --------------------------------------------------------------------------
 * FP8 (e4m3) arithmetic of the engine's FP8 weight path, restated on the CPU.
 * This path has no counterpart in the reference (whose DiT is fp32): it is the
 * exact quantisation recipe of the engine's DTTS_DTYPE_FP8 mode, so the engine
 * can be checked against it at the bf16 tolerance, and against the fp32 block
 * at the FP8 tolerance.
 *   e4m3: 1 sign, 4 exponent (bias 7), 3 mantissa bits; largest finite 448;
 *   subnormals m * 2^-9; round to nearest even, saturating at +-448.
 *   weights: per output channel, s_w = amax / 448, q = e4m3(w * (448 / amax)).
 *   LN outputs (QKV and FFN1 inputs): per row, s = amax / 448.
 *   attention output (O input): per row s_o = B / 448 with
 *     B = 1.02 * max_{j in sequence} unorm_j * max_d |Wv_d|,  unorm = 1.08 |u|,
 *     a bound on |softmax . V| (a convex mix of V rows).
 *   GELU output (FFN2 input): per row s_g = 1.02 * max(unorm2 * max_j |W1_j|
 *     + max_j |b1_j|, 0.17) / 448, a bound on |gelu(W1 u + b1)|.
 * ------------------------------------------------------------------------ */
uint8_t orc_e4m3_encode(float x) {
    const uint8_t sign = signbit(x) ? 0x80 : 0;
    if (isnan(x)) return 0x7F;
    const float a = fabsf(x);
    if (a >= 448.0f) return sign | 0x7E;
    if (a < 0.015625f) return sign | (uint8_t)rintf(a * 512.0f);   /* subnormal; 8 -> 2^-6 */
    int e;
    frexpf(a, &e);
    int E = e - 1;                                   /* a in [2^E, 2^(E+1)) */
    float q = rintf(ldexpf(a, 3 - E));               /* 1.mmm scaled to [8, 16] */
    if (q >= 16.0f) { q = 8.0f; E += 1; }
    if (E > 8 || (E == 8 && q > 14.0f)) return sign | 0x7E;
    return sign | (uint8_t)(((E + 7) << 3) | ((int)q - 8));
}

float orc_e4m3_decode(uint8_t b) {
    const int E = (b >> 3) & 15, m = b & 7;
    if (E == 15 && m == 7) return NAN;
    const float v = E == 0 ? ldexpf((float)m, -9) : ldexpf((float)(8 + m), E - 10);
    return (b & 0x80) ? -v : v;
}

static float fq(float x, float inv, float s) { return orc_e4m3_decode(orc_e4m3_encode(x * inv)) * s; }

static float row_amax(const float *x, int n) {
    float m = 0.0f;
    for (int i = 0; i < n; i++) m = fmaxf(m, fabsf(x[i]));
    return m;
}

static float row_norm(const float *x, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += x[i] * x[i];
    return sqrtf(s);
}

/* per-row quantise-dequantise with the row's own absmax */
static void fq_row_amax(float *x, int n) {
    const float amax = row_amax(x, n);
    if (amax == 0.0f) return;
    const float inv = 448.0f / amax, s = amax / 448.0f;
    for (int i = 0; i < n; i++) x[i] = fq(x[i], inv, s);
}

/* fake-quantised copy of one [rows][cols] weight, per output row; also the
 * largest dequantised row norm */
typedef struct { const float *src; size_t n; float probe; float *w; float max_norm; } fq_weight;
#define FQ_CACHE 160
static fq_weight g_fq[FQ_CACHE];
static int g_fq_n = 0;
static int g_dit_fp8 = 0;

void orc_set_dit_fp8(int on) {
    for (int i = 0; i < g_fq_n; i++) free(g_fq[i].w);
    g_fq_n = 0;
    g_dit_fp8 = on;
}

static const fq_weight *fq_weight_get(const float *w, int rows, int cols) {
    const size_t n = (size_t)rows * cols;
    const float probe = w[0] + w[n / 2] + w[n - 1];
    for (int i = 0; i < g_fq_n; i++)
        if (g_fq[i].src == w && g_fq[i].n == n && g_fq[i].probe == probe) return &g_fq[i];
    fq_weight *e = &g_fq[g_fq_n++];
    e->src = w; e->n = n; e->probe = probe;
    e->w = (float *)malloc(n * sizeof(float));
    float mn = 0.0f;
    #pragma omp parallel for schedule(static) reduction(max:mn)
    for (int r = 0; r < rows; r++) {
        const float *src = w + (size_t)r * cols;
        float *dst = e->w + (size_t)r * cols;
        const float amax = row_amax(src, cols);
        if (amax == 0.0f) {
            memset(dst, 0, (size_t)cols * sizeof(float));
        } else {
            const float inv = 448.0f / amax, sc = amax / 448.0f;
            for (int c = 0; c < cols; c++) dst[c] = fq(src[c], inv, sc);
        }
        mn = fmaxf(mn, row_norm(dst, cols));
    }
    e->max_norm = mn;
    return e;
}

/* DiT block with the engine's FP8 arithmetic (FFN on every token). */
static void dit_block_fwd_fp8(float *out, const float *x, const float *cond, const orc_dit_block *b,
                              int L, const uint8_t *mask, const float *pos) {
    const int D = ORC_D;
    float *ada = (float *)malloc(6 * D * sizeof(float));
    dit_adaln(ada, cond, b->ada_w, b->ada_b, 6 * D);
    const float *sm = ada, *scm = ada + D, *gm = ada + 2 * D;
    const float *sml = ada + 3 * D, *scl = ada + 4 * D, *gml = ada + 5 * D;
    if (g_fq_n + 6 > FQ_CACHE) orc_set_dit_fp8(g_dit_fp8);   /* cache full: start over */
    const fq_weight *wq = fq_weight_get(b->wq, D, D), *wk = fq_weight_get(b->wk, D, D);
    const fq_weight *wv = fq_weight_get(b->wv, D, D), *wo = fq_weight_get(b->wo, D, D);
    const fq_weight *w1 = fq_weight_get(b->w1, ORC_F, D), *w2 = fq_weight_get(b->w2, D, ORC_F);
    float b1max = 0.0f;
    for (int j = 0; j < ORC_F; j++) b1max = fmaxf(b1max, fabsf(b->b1 ? b->b1[j] : 0.0f));
    size_t n = (size_t)L * D;
    float *mod = (float *)malloc(n * sizeof(float));
    float *h = (float *)malloc(n * sizeof(float));
    float *q = (float *)malloc(n * sizeof(float));
    float *k = (float *)malloc(n * sizeof(float));
    float *v = (float *)malloc(n * sizeof(float));
    float *ctx = (float *)malloc(n * sizeof(float));
    float *ao = (float *)malloc(n * sizeof(float));
    float *unorm = (float *)malloc((size_t)L * sizeof(float));
    for (int t = 0; t < L; t++) {
        float *mr = mod + (size_t)t * D;
        ln_noaffine(mr, x + (size_t)t * D, D);
        for (int i = 0; i < D; i++) mr[i] = mr[i] * (1.0f + scm[i]) + sm[i];
        unorm[t] = 1.08f * row_norm(mr, D);
        fq_row_amax(mr, D);
    }
    orc_linear_rows(q, mod, L, wq->w, NULL, D, D);
    orc_linear_rows(k, mod, L, wk->w, NULL, D, D);
    orc_linear_rows(v, mod, L, wv->w, NULL, D, D);
    for (int t = 0; t < L; t++)
        for (int hh = 0; hh < ORC_H; hh++) {
            float *qh = q + (size_t)t * D + hh * ORC_HD, *kh = k + (size_t)t * D + hh * ORC_HD;
            rms_head(qh, b->qn);
            rms_head(kh, b->kn);
            if (g_dit_rope == ORC_ROPE_ADJACENT) {
                rope_adjacent(qh, pos ? (int)pos[t] : t);
                rope_adjacent(kh, pos ? (int)pos[t] : t);
            } else {
                rope_half(qh, kh, pos ? pos[t] : (float)t);
            }
        }
    const float scale = 1.0f / sqrtf((float)ORC_HD);
    #pragma omp parallel
    {
        float *sc = (float *)malloc((size_t)L * sizeof(float));
        #pragma omp for collapse(2) schedule(static)
        for (int hh = 0; hh < ORC_H; hh++)
            for (int i = 0; i < L; i++) {
                const float *qi = q + (size_t)i * D + hh * ORC_HD;
                for (int j = 0; j < L; j++) {
                    const float *kj = k + (size_t)j * D + hh * ORC_HD;
                    float acc = 0.0f;
                    for (int d = 0; d < ORC_HD; d++) acc += qi[d] * kj[d];
                    sc[j] = acc * scale;
                    if (mask && !mask[(size_t)i * L + j]) sc[j] = -INFINITY;
                }
                float mx = sc[0];
                for (int j = 1; j < L; j++) if (sc[j] > mx) mx = sc[j];
                float sum = 0.0f;
                for (int j = 0; j < L; j++) { sc[j] = expf(sc[j] - mx); sum += sc[j]; }
                for (int j = 0; j < L; j++) sc[j] /= sum;
                float *ci = ctx + (size_t)i * D + hh * ORC_HD;
                for (int d = 0; d < ORC_HD; d++) {
                    float acc = 0.0f;
                    for (int j = 0; j < L; j++) acc += sc[j] * v[(size_t)j * D + hh * ORC_HD + d];
                    ci[d] = acc;
                }
            }
        free(sc);
    }
    /* attention output: one scale per sequence from the bound on |V| */
    float umax = 0.0f;
    for (int t = 0; t < L; t++) umax = fmaxf(umax, unorm[t]);
    const float bo_ = 1.02f * umax * wv->max_norm;
    if (bo_ > 0.0f) {
        const float inv = 448.0f / bo_, s = bo_ / 448.0f;
        for (size_t i = 0; i < n; i++) ctx[i] = fq(ctx[i], inv, s);
    }
    orc_linear_rows(ao, ctx, L, wo->w, b->bo, D, D);
    for (size_t i = 0; i < n; i++) h[i] = x[i] + gm[i % D] * ao[i];
    float *sg = (float *)malloc((size_t)L * sizeof(float));
    for (int t = 0; t < L; t++) {
        float *mr = mod + (size_t)t * D;
        ln_noaffine(mr, h + (size_t)t * D, D);
        for (int i = 0; i < D; i++) mr[i] = mr[i] * (1.0f + scl[i]) + sml[i];
        sg[t] = 1.02f * fmaxf(1.08f * row_norm(mr, D) * w1->max_norm + b1max, 0.17f);
        fq_row_amax(mr, D);
    }
    float *f1 = (float *)malloc((size_t)L * ORC_F * sizeof(float));
    float *f2 = (float *)malloc(n * sizeof(float));
    orc_linear_rows(f1, mod, L, w1->w, b->b1, D, ORC_F);
    for (int t = 0; t < L; t++) {
        const float inv = 448.0f / sg[t], s = sg[t] / 448.0f;
        float *fr = f1 + (size_t)t * ORC_F;
        for (int j = 0; j < ORC_F; j++) fr[j] = fq(gelu_tanh(fr[j]), inv, s);
    }
    orc_linear_rows(f2, f1, L, w2->w, b->b2, ORC_F, D);
    for (size_t i = 0; i < n; i++) out[i] = h[i] + gml[i % D] * f2[i];
    free(ada); free(mod); free(h); free(q); free(k); free(v); free(ctx); free(ao); free(unorm);
    free(sg); free(f1); free(f2);
}

/* --------------------------------------------------------------------------
 * Velocity forward: input_layer -> blocks -> output adaLN + LN + out_proj
 * (src/e2e_pipeline_v4.cpp:441-478).  Writes the last n_out tokens of
 * out_all [L][128] (n_out = L gives every row).
 * ------------------------------------------------------------------------ */
void orc_dit_velocity(const orc_dit *m, const float *x_in, int L, const float *cond,
                      const uint8_t *mask, const float *pos, int ffn_mode,
                      int n_out, float *out) {
    const int D = ORC_D;
    size_t n = (size_t)L * D;
    float *h = (float *)malloc(n * sizeof(float));
    float *bo = (float *)malloc(n * sizeof(float));
    orc_linear_rows(h, x_in, L, m->in_w, m->in_b, D, D);
    for (int i = 0; i < m->n_layers; i++) {
        orc_dit_block_fwd(bo, h, cond, &m->blocks[i], L, mask, pos, ffn_mode);
        float *tmp = h; h = bo; bo = tmp;
    }
    float mod_raw[2 * ORC_D];
    dit_adaln(mod_raw, cond, m->oada_w, m->oada_b, 2 * D);
    const float *shift = mod_raw, *scale = mod_raw + D;
    int t0 = L - n_out;
    for (int t = t0; t < L; t++) {
        float ln[ORC_D];
        ln_noaffine(ln, h + (size_t)t * D, D);
        for (int j = 0; j < D; j++) ln[j] = ln[j] * (1.0f + scale[j]) + shift[j];
        linear1(out + (size_t)(t - t0) * ORC_LAT, ln, m->out_w, m->out_b, D, ORC_LAT);
    }
    free(h); free(bo);
}

/* --------------------------------------------------------------------------
 * EOS head of the v4 pipeline (src/e2e_pipeline_v4.cpp:598-619):
 * s = W1 h + b1 (input order), a = s / (1 + e^-s) and, as the shipped code
 * does, a = s * a when as_written (:608-609); logits = W2 a + b2;
 * p = softmax(logits)[1].
 * ------------------------------------------------------------------------ */
float orc_eos_prob(const float *w1, const float *b1, const float *w2, const float *b2, const float *h,
                   int as_written) {
    float a[ORC_LLM];
    for (int o = 0; o < ORC_LLM; o++) {
        float s = b1 ? b1[o] : 0.0f;
        for (int i = 0; i < ORC_LLM; i++) s += w1[(size_t)o * ORC_LLM + i] * h[i];
        a[o] = s / (1.0f + expf(-s));
        if (as_written) a[o] = s * a[o];
    }
    float lg[2];
    for (int o = 0; o < 2; o++) {
        float s = b2 ? b2[o] : 0.0f;
        for (int i = 0; i < ORC_LLM; i++) s += w2[(size_t)o * ORC_LLM + i] * a[i];
        lg[o] = s;
    }
    const float mx = fmaxf(lg[0], lg[1]);
    const float sum = expf(lg[0] - mx) + expf(lg[1] - mx);
    return expf(lg[1] - mx) / sum;
}

/* --------------------------------------------------------------------------
 * FM mask / position ids (src/e2e_pipeline_v4.cpp:120-155).
 * ------------------------------------------------------------------------ */
void orc_build_fm_mask(uint8_t *mask, int total_len, int fm_len, int patch, int hidden_patch) {
    int latent_start = total_len - patch;
    int block_start = fm_len > hidden_patch ? fm_len - hidden_patch : 0;
    memset(mask, 0, (size_t)total_len * total_len);
    for (int i = 0; i < block_start; i++)
        for (int j = 0; j <= i; j++) mask[(size_t)i * total_len + j] = 1;
    for (int i = block_start; i < fm_len; i++) {
        for (int j = 0; j < fm_len; j++) mask[(size_t)i * total_len + j] = 1;
        for (int j = latent_start; j < total_len; j++) mask[(size_t)i * total_len + j] = 1;
    }
    for (int i = latent_start; i < total_len; i++) {
        for (int j = 0; j < fm_len; j++) mask[(size_t)i * total_len + j] = 1;
        for (int j = latent_start; j < total_len; j++) mask[(size_t)i * total_len + j] = 1;
    }
    for (int i = fm_len; i < latent_start; i++) mask[(size_t)i * total_len + i] = 1;
}

void orc_build_fm_pos(float *pos, int total_len, int fm_len, int patch) {
    int latent_start = total_len - patch;
    for (int i = 0; i < fm_len; i++) pos[i] = (float)i;
    for (int i = latent_start; i < total_len; i++) pos[i] = (float)(fm_len + i - latent_start);
    for (int i = fm_len; i < latent_start; i++) pos[i] = 0.0f;
}

/* --------------------------------------------------------------------------
 * Euler + CFG solve for one latent patch per utterance
 * (src/e2e_pipeline_v4.cpp:395-526).  layout 0: v4 mask + pos ids;
 * layout 1: no mask, positions 0..L-1.  cfg_form 0: v = vc + s (vc - vu)
 * (v4, :509-512); cfg_form 1: v = vu + s (vc - vu) (src/e2e_pipeline.cpp:444).
 * ------------------------------------------------------------------------ */
void orc_euler_solve(const orc_dit *m, int n_utt, int fm_len, int patch,
                     const float *fm_cond, const float *fm_uncond,
                     const float *z0, const float *spk, float spk_scale,
                     int nfe, float cfg_scale, int cfg_form, int layout, int ffn_mode,
                     float *z_out) {
    const int D = ORC_D;
    int total = fm_len + patch;
    int pf = patch * ORC_LAT;
    uint8_t *mask = NULL;
    float *pos = NULL;
    if (layout == 0) {
        mask = (uint8_t *)malloc((size_t)total * total);
        pos = (float *)malloc((size_t)total * sizeof(float));
        orc_build_fm_mask(mask, total, fm_len, patch, 1);
        orc_build_fm_pos(pos, total, fm_len, patch);
    }
    float *xc = (float *)malloc((size_t)total * D * sizeof(float));
    float *xu = (float *)malloc((size_t)total * D * sizeof(float));
    float *vc = (float *)malloc((size_t)pf * sizeof(float));
    float *vu = (float *)malloc((size_t)pf * sizeof(float));
    const float dt = 1.0f / (float)nfe;
    for (int u = 0; u < n_utt; u++) {
        float *z = z_out + (size_t)u * pf;
        memcpy(z, z0 + (size_t)u * pf, (size_t)pf * sizeof(float));
        memcpy(xc, fm_cond + (size_t)u * fm_len * D, (size_t)fm_len * D * sizeof(float));
        memcpy(xu, fm_uncond + (size_t)u * fm_len * D, (size_t)fm_len * D * sizeof(float));
        for (int step = 0; step < nfe; step++) {
            float t = (float)step * dt;
            for (int p = 0; p < patch; p++) {
                float *dst = xc + (size_t)(total - patch + p) * D;
                linear1(dst, z + p * ORC_LAT, m->coord_w, m->coord_b, ORC_LAT, D);
                memcpy(xu + (size_t)(total - patch + p) * D, dst, D * sizeof(float));
            }
            float cond[ORC_D];
            orc_compute_cond(m, t, spk ? spk + (size_t)u * ORC_SPK : NULL, spk_scale, cond);
            orc_dit_velocity(m, xc, total, cond, mask, pos, ffn_mode, patch, vc);
            orc_dit_velocity(m, xu, total, cond, mask, pos, ffn_mode, patch, vu);
            for (int i = 0; i < pf; i++) {
                float v = (cfg_form == 0) ? vc[i] + cfg_scale * (vc[i] - vu[i])
                                          : vu[i] + cfg_scale * (vc[i] - vu[i]);
                z[i] += v * dt;
            }
        }
    }
    free(mask); free(pos); free(xc); free(xu); free(vc); free(vu);
}

/* --------------------------------------------------------------------------
 * PatchEncoder (src/modules/backbone/patchenc.cpp:146-239)
 * ------------------------------------------------------------------------ */

/* ggml_rms_norm (sum of squares in double, scale = 1/sqrtf(mean + eps)) then
 * optional elementwise weight (patchenc.cpp:172-173,210-211). */
static void rms_norm_w(float *out, const float *x, const float *w, int n, float eps) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    float mean = (float)(ss / n);
    float scale = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < n; i++) { float y = x[i] * scale; if (w) y *= w[i]; out[i] = y; }
}

/* ggml_rope mode 0 (adjacent pairs) with freq_base 1e4, freq_scale 1:
 * theta starts at p and is multiplied by 1e4^(-2/64) per pair. */
static void rope_adjacent(float *v, int p) {
    float theta_scale = powf(10000.0f, -2.0f / (float)ORC_HD);
    float theta = (float)p;
    for (int i = 0; i < ORC_HD; i += 2) {
        float c = cosf(theta), s = sinf(theta);
        float x0 = v[i], x1 = v[i + 1];
        v[i] = x0 * c - x1 * s;
        v[i + 1] = x0 * s + x1 * c;
        theta *= theta_scale;
    }
}

/* causal Conv1d(128->128, k=2, s=2) with taps at frames 2o-1 and 2o
 * (patchenc.cpp:19-39): frames [seq][128] -> out [seq/2][128]. */
void orc_pe_conv(float *out, const float *frames, int seq, const float *w, const float *b) {
    const int C = ORC_LAT, T = seq / 2;
    for (int o = 0; o < T; o++)
        for (int oc = 0; oc < C; oc++) {
            float s = b ? b[oc] : 0.0f;
            for (int ic = 0; ic < C; ic++) {
                int wb = (oc * C + ic) * 2;
                int i0 = 2 * o - 1;
                if (i0 >= 0 && i0 < seq) s += frames[(size_t)i0 * C + ic] * w[wb + 0];
                int i1 = 2 * o;
                if (i1 >= 0 && i1 < seq) s += frames[(size_t)i1 * C + ic] * w[wb + 1];
            }
            out[(size_t)o * C + oc] = s;
        }
}

/* causal per-head softmax(QK^T/8)V over 16 heads of 64 (patchenc.cpp:59-101):
 * q, k, v, ctx [T][1024]. */
void orc_pe_causal_attention(float *ctx, const float *q, const float *k, const float *v, int T) {
    const int D = ORC_D;
    const float scale = 1.0f / sqrtf((float)ORC_HD);
    #pragma omp parallel
    {
        float *s = (float *)malloc((size_t)T * sizeof(float));
        #pragma omp for collapse(2) schedule(static)
        for (int hh = 0; hh < ORC_H; hh++)
            for (int ti = 0; ti < T; ti++) {
                for (int tj = 0; tj < T; tj++) {
                    float acc = 0.0f;
                    for (int d = 0; d < ORC_HD; d++)
                        acc += q[(size_t)ti * D + hh * ORC_HD + d] * k[(size_t)tj * D + hh * ORC_HD + d];
                    s[tj] = acc * scale;
                }
                for (int tj = ti + 1; tj < T; tj++) s[tj] = -INFINITY;
                float mx = s[0];
                for (int tj = 1; tj < T; tj++) if (s[tj] > mx) mx = s[tj];
                float sum = 0.0f;
                for (int tj = 0; tj < T; tj++) { s[tj] = expf(s[tj] - mx); sum += s[tj]; }
                for (int tj = 0; tj < T; tj++) s[tj] /= sum;
                for (int d = 0; d < ORC_HD; d++) {
                    float acc = 0.0f;
                    for (int tj = 0; tj < T; tj++) acc += s[tj] * v[(size_t)tj * D + hh * ORC_HD + d];
                    ctx[(size_t)ti * D + hh * ORC_HD + d] = acc;
                }
            }
        free(s);
    }
}

void orc_pe_forward(const orc_pe *m, const float *frames, int n_patches, int pair_mode,
                    float *out, float *h_last) {
    const int D = ORC_D, C = ORC_LAT;
    int seq = n_patches * 4;
    int T = seq / 2;
    float *xc = (float *)malloc((size_t)T * C * sizeof(float));
    orc_pe_conv(xc, frames, seq, m->conv_w, m->conv_b);
    size_t n = (size_t)T * D;
    float *h = (float *)malloc(n * sizeof(float));
    orc_linear_rows(h, xc, T, m->in_w, m->in_b, C, D);
    float *xn = (float *)malloc(n * sizeof(float));
    float *q = (float *)malloc(n * sizeof(float));
    float *k = (float *)malloc(n * sizeof(float));
    float *v = (float *)malloc(n * sizeof(float));
    float *ctx = (float *)malloc(n * sizeof(float));
    float *ao = (float *)malloc(n * sizeof(float));
    float *f1 = (float *)malloc((size_t)T * ORC_F * sizeof(float));
    float *f2 = (float *)malloc(n * sizeof(float));
    for (int li = 0; li < m->n_layers; li++) {
        const orc_pe_layer *l = &m->layers[li];
        for (int t = 0; t < T; t++) rms_norm_w(xn + (size_t)t * D, h + (size_t)t * D, l->attn_norm_w, D, 1e-6f);
        orc_linear_rows(q, xn, T, l->wq, NULL, D, D);
        orc_linear_rows(k, xn, T, l->wk, NULL, D, D);
        orc_linear_rows(v, xn, T, l->wv, NULL, D, D);
        /* no qk-norm (patchenc.cpp:283-284); rope on q and k, positions 0..T-1 */
        for (int t = 0; t < T; t++)
            for (int hh = 0; hh < ORC_H; hh++) {
                rope_adjacent(q + (size_t)t * D + hh * ORC_HD, t);
                rope_adjacent(k + (size_t)t * D + hh * ORC_HD, t);
            }
        orc_pe_causal_attention(ctx, q, k, v, T);
        orc_linear_rows(ao, ctx, T, l->wo, l->bo, D, D);
        for (size_t i = 0; i < n; i++) h[i] += ao[i];
        for (int t = 0; t < T; t++) rms_norm_w(xn + (size_t)t * D, h + (size_t)t * D, l->ffn_norm_w, D, 1e-6f);
        orc_linear_rows(f1, xn, T, l->w1, l->b1, D, ORC_F);
        for (size_t i = 0; i < (size_t)T * ORC_F; i++) f1[i] = silu(f1[i]);
        orc_linear_rows(f2, f1, T, l->w2, l->b2, ORC_F, D);
        for (size_t i = 0; i < n; i++) h[i] += f2[i];
    }
    if (h_last) memcpy(h_last, h, n * sizeof(float));
    /* output pairs -> out_proj(2048 -> 1536) (patchenc.cpp:225-238) */
    float *cat = (float *)malloc((size_t)n_patches * 2 * D * sizeof(float));
    for (int qi = 0; qi < n_patches; qi++)
        for (int s = 0; s < 2; s++) {
            int tok;
            if (pair_mode == ORC_PAIR_ADJACENT) {
                tok = 2 * qi + s;
            } else {
                /* reshape [D,2,n] -> permute(0,2,1,3) -> [D,n,2] -> [2D,n]:
                 * flat index f = i + D*p + D*n*j, output row qi covers
                 * f in [2D qi, 2D qi + 2D), i.e. g = 2 qi + s -> p = g % n, j = g / n */
                int g = 2 * qi + s;
                tok = 2 * (g % n_patches) + g / n_patches;
            }
            memcpy(cat + (size_t)qi * 2 * D + s * D, h + (size_t)tok * D, D * sizeof(float));
        }
    orc_linear_rows(out, cat, n_patches, m->out_w, m->out_b, 2 * D, ORC_LLM);
    free(cat); free(xc); free(h); free(xn); free(q); free(k); free(v); free(ctx); free(ao); free(f1); free(f2);
}
