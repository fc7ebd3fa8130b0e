/* CPU oracle: BigVGAN v2 decoder (the vocoder behind the latents).
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  A plain fp32 restatement of
 * src/modules/vocoder/bigvgan_cpp.cpp and src/modules/vocoder/lstm.cpp of
 * MaurerAnton/dots.tts.cpp, time-major ([time][channels]) like the reference,
 * with its loops reordered for speed (weights transposed so inner products
 * run over contiguous channels) and OpenMP over independent outputs.  The
 * arithmetic per output is the reference's; only the summation order differs.
 * Pinned against the reference's own bigvgan_decode compiled into oracle/_ref. */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

const int orc_voc_up_in[ORC_VOC_STAGES] = {1536, 768, 384, 192, 96, 48};
const int orc_voc_up_out[ORC_VOC_STAGES] = {768, 384, 192, 96, 48, 24};
const int orc_voc_up_stride[ORC_VOC_STAGES] = {10, 6, 4, 2, 2, 2};
const int orc_voc_up_kernel[ORC_VOC_STAGES] = {20, 12, 8, 4, 4, 4};
const int orc_voc_rb_kernel[3] = {3, 7, 11};
const int orc_voc_rb_dil[3] = {1, 3, 5};

#define VOC_AA_TAPS 12

static float *vbuf(size_t n) {
    float *p = (float *)malloc(n * sizeof(float));
    if (!p) abort();
    return p;
}

/* w [oc][ic][K] -> wt [oc][K][ic] */
static float *transpose_okc(const float *w, int oc, int ic, int K) {
    float *wt = vbuf((size_t)oc * ic * K);
    for (int o = 0; o < oc; o++)
        for (int c = 0; c < ic; c++)
            for (int k = 0; k < K; k++) wt[((size_t)o * K + k) * ic + c] = w[((size_t)o * ic + c) * K + k];
    return wt;
}

/* Conv1d, stride 1: out[t][o] = b[o] + sum_k sum_c in[t + k*dil - pad_left][c] w[o][c][k],
 * zero outside [0, len).  Causal (bigvgan_cpp.cpp:147-171): pad_left = dil (K - 1).
 * Non-causal conv_pre (:389-405): pad_left = 2. */
static void conv1d(float *out, const float *in, int ic, int len, const float *w, const float *b, int oc, int K,
                   int dil, int pad_left) {
    float *wt = transpose_okc(w, oc, ic, K);
    #pragma omp parallel for schedule(static)
    for (int t = 0; t < len; t++) {
        for (int o = 0; o < oc; o++) {
            float s = b ? b[o] : 0.f;
            for (int k = 0; k < K; k++) {
                const int ts = t + k * dil - pad_left;
                if (ts < 0 || ts >= len) continue;
                const float *x = in + (size_t)ts * ic, *ww = wt + ((size_t)o * K + k) * ic;
                float a = 0.f;
                for (int c = 0; c < ic; c++) a += x[c] * ww[c];
                s += a;
            }
            out[(size_t)t * oc + o] = s;
        }
    }
    free(wt);
}

/* Causal ConvTranspose1d with K = 2 stride (bigvgan_cpp.cpp:176-205): the full
 * output (len-1) stride + K is trimmed to len * stride.  Output sample
 * q stride + r gathers in[q] w[.][.][r] and in[q-1] w[.][.][r + stride]. */
static void convT1d_causal(float *out, const float *in, int ic, int len, const float *w, const float *b, int oc,
                           int stride, int K) {
    /* wt[r][o][j][c]: tap j = 0 (in[q], k = r) and j = 1 (in[q-1], k = r + stride) */
    float *wt = vbuf((size_t)stride * oc * 2 * ic);
    for (int r = 0; r < stride; r++)
        for (int o = 0; o < oc; o++)
            for (int j = 0; j < 2; j++)
                for (int c = 0; c < ic; c++) {
                    const int k = r + j * stride;
                    wt[(((size_t)r * oc + o) * 2 + j) * ic + c] = k < K ? w[((size_t)c * oc + o) * K + k] : 0.f;
                }
    const int olen = len * stride;
    #pragma omp parallel for schedule(static)
    for (int ot = 0; ot < olen; ot++) {
        const int q = ot / stride, r = ot % stride;
        for (int o = 0; o < oc; o++) {
            float s = 0.f;
            for (int j = 0; j < 2; j++) {
                const int i = q - j;
                if (i < 0) continue;
                const float *x = in + (size_t)i * ic, *ww = wt + (((size_t)r * oc + o) * 2 + j) * ic;
                float a = 0.f;
                for (int c = 0; c < ic; c++) a += x[c] * ww[c];
                s += a;
            }
            out[(size_t)ot * oc + o] = s + (b ? b[o] : 0.f);
        }
    }
    free(wt);
}

/* Activation1d (bigvgan_cpp.cpp:33-124), per channel c of x [len][ch]:
 *   up:   u[j] = 2 sum_{k = j mod 2, k+2, ..., k <= min(j, 11)} f_up[k] x[(j - k) / 2],  j < 2 len
 *         (ConvTranspose1d stride 2, no padding, trimmed to 2 len: :41-62)
 *   snake: a = e^clamp(alpha, +-20), b = e^clamp(beta, +-20);
 *         s = u + sin^2(a u) / (b + 1e-9); a non-finite u gives 0, a non-finite s gives u (:103-117)
 *   down: out[t] = sum_k f_down[k] s[max(0, 2t + k - 11)]  (replicate left pad of 11, stride 2: :66-92) */
void orc_voc_activation(float *x, int len, int ch, const float *alpha, const float *beta, const float *filt_up,
                        const float *filt_down, int fch) {
    float *s = vbuf((size_t)2 * len * ch);
    #pragma omp parallel for schedule(static)
    for (int c = 0; c < ch; c++) {
        const float *fu = filt_up + (fch == 1 ? 0 : (size_t)c * VOC_AA_TAPS);
        const float *fd = filt_down + (fch == 1 ? 0 : (size_t)c * VOC_AA_TAPS);
        float a = alpha ? alpha[c] : 1.0f, b = beta ? beta[c] : 1.0f;
        a = expf(a > 20.0f ? 20.0f : (a < -20.0f ? -20.0f : a));
        b = expf(b > 20.0f ? 20.0f : (b < -20.0f ? -20.0f : b));
        for (int j = 0; j < 2 * len; j++) {
            float u = 0.f;
            for (int k = j & 1; k < VOC_AA_TAPS && k <= j; k += 2) u += x[(size_t)((j - k) / 2) * ch + c] * fu[k] * 2.0f;
            float v;
            if (isnan(u) || isinf(u)) {
                v = 0.f;
            } else {
                const float sn = sinf(a * u);
                v = u + (1.0f / (b + 1e-9f)) * sn * sn;
                if (isnan(v) || isinf(v)) v = u;
            }
            s[(size_t)j * ch + c] = v;
        }
        for (int t = 0; t < len; t++) {
            float o = 0.f;
            for (int k = 0; k < VOC_AA_TAPS; k++) {
                int j = 2 * t + k - (VOC_AA_TAPS - 1);
                if (j < 0) j = 0;
                o += s[(size_t)j * ch + c] * fd[k];
            }
            x[(size_t)t * ch + c] = o;
        }
    }
    free(s);
}

/* lstm.cpp:9-104: 4 layers, hidden 512, gates i, f, g, o; the output of the
 * last layer plus the layer-0 input (skip). */
static void lstm4_skip(const orc_voc *m, const float *x, int T, float *out) {
    const int H = 512;
    float *h = vbuf(4 * H), *c = vbuf(4 * H), *in = vbuf(H), *g = vbuf(4 * H);
    memset(h, 0, 4 * H * sizeof(float));
    memset(c, 0, 4 * H * sizeof(float));
    for (int t = 0; t < T; t++) {
        memcpy(in, x + (size_t)t * H, H * sizeof(float));
        for (int l = 0; l < 4; l++) {
            const float *wi = m->lstm_w_ih[l], *wh = m->lstm_w_hh[l];
            float *hl = h + l * H, *cl = c + l * H;
            #pragma omp parallel for schedule(static)
            for (int i = 0; i < 4 * H; i++) {
                float a = m->lstm_b_ih[l][i] + m->lstm_b_hh[l][i];
                const float *ri = wi + (size_t)i * H, *rh = wh + (size_t)i * H;
                for (int j = 0; j < H; j++) a += in[j] * ri[j] + hl[j] * rh[j];
                g[i] = a;
            }
            for (int j = 0; j < H; j++) {
                const float ig = 1.0f / (1.0f + expf(-g[j])), fg = 1.0f / (1.0f + expf(-g[H + j]));
                const float gg = tanhf(g[2 * H + j]), og = 1.0f / (1.0f + expf(-g[3 * H + j]));
                cl[j] = fg * cl[j] + ig * gg;
                hl[j] = og * tanhf(cl[j]);
            }
            memcpy(in, hl, H * sizeof(float));
        }
        for (int j = 0; j < H; j++) out[(size_t)t * H + j] = x[(size_t)t * H + j] + in[j];
    }
    free(h); free(c); free(in); free(g);
}

static void linear_rows(float *y, const float *x, int T, const float *w, const float *b, int in, int out) {
    #pragma omp parallel for schedule(static)
    for (int t = 0; t < T; t++)
        for (int o = 0; o < out; o++) {
            float s = b ? b[o] : 0.f;
            const float *xr = x + (size_t)t * in, *wr = w + (size_t)o * in;
            for (int i = 0; i < in; i++) s += xr[i] * wr[i];
            y[(size_t)t * out + o] = s;
        }
}

/* post_proj (1x1 conv) -> Linear 128->512 -> LSTM (skip) -> Linear 512->128
 * (bigvgan_cpp.cpp:344-377) */
void orc_voc_bottleneck(const orc_voc *m, const float *latent, int T, float *out128) {
    float *p = vbuf((size_t)T * 128), *z = vbuf((size_t)T * 512), *l = vbuf((size_t)T * 512);
    linear_rows(p, latent, T, m->post_proj_w, m->post_proj_b, 128, 128);
    linear_rows(z, p, T, m->mi_w1, m->mi_b1, 128, 512);
    lstm4_skip(m, z, T, l);
    linear_rows(out128, l, T, m->mi_w2, m->mi_b2, 512, 128);
    free(p); free(z); free(l);
}

void orc_voc_decode(const orc_voc *m, const float *aa_filter, const float *latent, int n_frames, float *audio) {
    const int T0 = n_frames;
    float *bott = vbuf((size_t)T0 * 128);
    orc_voc_bottleneck(m, latent, T0, bott);
    float *x = vbuf((size_t)T0 * 1536);
    conv1d(x, bott, 128, T0, m->conv_pre_w, m->conv_pre_b, 1536, 5, 1, 2);   /* :384-405 */
    free(bott);
    int ch = 1536, len = T0;
    for (int s = 0; s < ORC_VOC_STAGES; s++) {                                 /* :412-496 */
        const int oc = orc_voc_up_out[s], st = orc_voc_up_stride[s];
        const int olen = len * st;
        float *up = vbuf((size_t)olen * oc);
        convT1d_causal(up, x, ch, len, m->ups_w[s], m->ups_b[s], oc, st, orc_voc_up_kernel[s]);
        free(x);
        ch = oc; len = olen;
        const size_t n = (size_t)len * ch;
        float *acc = vbuf(n), *r = vbuf(n), *a = vbuf(n), *y = vbuf(n);
        memset(acc, 0, n * sizeof(float));
        for (int j = 0; j < 3; j++) {
            const int rb = s * 3 + j, K = orc_voc_rb_kernel[j];
            memcpy(r, up, n * sizeof(float));
            for (int p = 0; p < 3; p++) {
                const int dil = orc_voc_rb_dil[p];
                /* r += c2(a2(c1(a1(r))))  (:441-481) */
                memcpy(a, r, n * sizeof(float));
                orc_voc_activation(a, len, ch, m->alpha[rb][2 * p], m->beta[rb][2 * p], aa_filter, aa_filter, 1);
                conv1d(y, a, ch, len, m->c1_w[rb][p], m->c1_b[rb][p], ch, K, dil, dil * (K - 1));
                orc_voc_activation(y, len, ch, m->alpha[rb][2 * p + 1], m->beta[rb][2 * p + 1], aa_filter, aa_filter, 1);
                conv1d(a, y, ch, len, m->c2_w[rb][p], m->c2_b[rb][p], ch, K, 1, K - 1);
                for (size_t i = 0; i < n; i++) r[i] += a[i];
            }
            for (size_t i = 0; i < n; i++) acc[i] += r[i];
        }
        for (size_t i = 0; i < n; i++) acc[i] /= 3.0f;
        free(up); free(r); free(a); free(y);
        x = acc;
    }
    /* activation_post with its per-channel filters, conv_post (causal K=7, no
     * bias), tanh x 1.92 (:499-525) */
    orc_voc_activation(x, len, ch, m->post_alpha, m->post_beta, m->post_filt_up, m->post_filt_down, ch);
    float *o = vbuf((size_t)len);
    conv1d(o, x, ch, len, m->conv_post_w, NULL, 1, 7, 1, 6);
    for (int i = 0; i < len; i++) audio[i] = tanhf(o[i]) * 1.92f;
    free(o); free(x);
}
