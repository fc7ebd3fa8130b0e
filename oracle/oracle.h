/* CPU oracle for the DiT flow-matching head and the PatchEncoder.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py load this library, and only as
 * the checker or the CPU baseline; the CUDA engine never calls it.
 *
 * It restates, in plain fp32 C, the reference's CPU arithmetic for this path
 * (MaurerAnton/dots.tts.cpp; file:line citations are on each function in
 * oracle.c).  The DiT half is pinned against the reference's own
 * include/dit_manual.h compiled into oracle/_ref (see oracle/Makefile); the
 * PatchEncoder half restates src/modules/backbone/patchenc.cpp, whose ggml
 * operators (rms_norm, rope mode 0, silu) are not vendored in the reference,
 * so their exact numerics are restated from ggml's published definitions.
 *
 * Layouts: every matrix is row-major [out][in] (PyTorch Linear), activations
 * are row-major [tokens][features], all fp32. */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_D      1024   /* DIT_HIDDEN_SIZE / PATCHENC_HIDDEN            */
#define ORC_H      16     /* heads                                         */
#define ORC_HD     64     /* head dim                                      */
#define ORC_F      4096   /* FFN size                                      */
#define ORC_LAT    128    /* VAE latent dim                                */
#define ORC_LLM    1536   /* LLM hidden (hidden_proj input, PE output)     */
#define ORC_SPK    512    /* speaker x-vector dim                          */

/* One DiT block (include/dit.h:47-72 field meanings). */
typedef struct {
    const float *wq, *wk, *wv, *wo;  /* [1024][1024] */
    const float *bo;                 /* [1024] or NULL */
    const float *qn, *kn;            /* [64] per-head RMS gains, or NULL */
    const float *w1, *b1;            /* [4096][1024], [4096] */
    const float *w2, *b2;            /* [1024][4096], [1024] */
    const float *ada_w, *ada_b;      /* [6144][1024], [6144] */
} orc_dit_block;

/* Whole DiT (include/dit.h:74-126). */
typedef struct {
    int n_layers;
    const orc_dit_block *blocks;
    const float *t_w1, *t_b1;        /* [1024][256], [1024] */
    const float *t_w2, *t_b2;        /* [1024][1024], [1024] */
    const float *spk_w1, *spk_b1;    /* [1024][512], [1024] */
    const float *spk_ln_w, *spk_ln_b;/* [1024] */
    const float *oada_w, *oada_b;    /* [2048][1024], [2048] */
    const float *out_w, *out_b;      /* [128][1024], [128] */
    const float *in_w, *in_b;        /* [1024][1024], [1024] */
    const float *hid_w, *hid_b;      /* [1024][1536], [1024] */
    const float *lat_w, *lat_b;      /* [1024][128], [1024] */
    const float *coord_w, *coord_b;  /* [1024][128], [1024] */
} orc_dit;

typedef struct {
    const float *attn_norm_w;        /* [1024] or NULL */
    const float *wq, *wk, *wv, *wo;  /* [1024][1024] */
    const float *bo;                 /* [1024] or NULL */
    const float *ffn_norm_w;         /* [1024] or NULL */
    const float *w1, *b1;            /* [4096][1024], [4096] */
    const float *w2, *b2;            /* [1024][4096], [1024] */
} orc_pe_layer;

typedef struct {
    int n_layers;
    const orc_pe_layer *layers;
    const float *conv_w, *conv_b;    /* [128][128][2], [128] */
    const float *in_w, *in_b;        /* [1024][128], [1024] */
    const float *out_w, *out_b;      /* [1536][2048], [1536] */
} orc_pe;

/* rope pairing */
#define ORC_ROPE_HALF      0   /* (d, d+32): dit_manual.h:111-128            */
#define ORC_ROPE_ADJACENT  1   /* (2i, 2i+1): ggml_rope mode 0, patchenc.cpp:115-116 */

/* FFN variants of the DiT block */
#define ORC_FFN_PER_TOKEN  0   /* every token (what the model means)          */
#define ORC_FFN_AS_WRITTEN 1   /* token 0 only, rows 1.. read a zeroed scratch, dit_manual.h:173-196 */

/* PatchEncoder output pairing */
#define ORC_PAIR_ADJACENT  0   /* output p = out_proj([h_2p | h_2p+1])        */
#define ORC_PAIR_AS_WRITTEN 1  /* ggml permute as written, patchenc.cpp:230-232 */

/* FP8 (e4m3) quantisation recipe of the engine's FP8 weight path (no
 * counterpart in the reference, whose DiT is fp32): orc_set_dit_fp8(1) makes
 * every DiT block (FFN per token) use it; (0) restores fp32.  Both calls drop
 * the cache of fake-quantised weights. */
void    orc_set_dit_fp8(int on);
uint8_t orc_e4m3_encode(float x);
float   orc_e4m3_decode(uint8_t b);

int  orc_num_threads(void);
void orc_set_dit_rope(int mode);
void orc_set_threads(int n);

void orc_sinusoid(float t, float *se256);
void orc_compute_cond(const orc_dit *m, float t, const float *spk, float spk_scale, float *cond);
void orc_linear_rows(float *y, const float *x, int rows, const float *w, const float *b, int in, int out);

void orc_attention(float *out, const float *x, int L,
                   const float *wq, const float *wk, const float *wv, const float *wo,
                   const float *bo, const float *qn, const float *kn,
                   const uint8_t *mask, const float *pos);

void orc_dit_block_fwd(float *out, const float *x, const float *cond, const orc_dit_block *b,
                       int L, const uint8_t *mask, const float *pos, int ffn_mode);

void orc_dit_velocity(const orc_dit *m, const float *x_in, int L, const float *cond,
                      const uint8_t *mask, const float *pos, int ffn_mode,
                      int n_out, float *out);

float orc_eos_prob(const float *w1, const float *b1, const float *w2, const float *b2, const float *h,
                   int as_written);

void orc_build_fm_mask(uint8_t *mask, int total_len, int fm_len, int patch, int hidden_patch);
void orc_build_fm_pos(float *pos, int total_len, int fm_len, int patch);

void orc_euler_solve(const orc_dit *m, int n_utt, int fm_len, int patch,
                     const float *fm_cond, const float *fm_uncond,
                     const float *z0, const float *spk, float spk_scale,
                     int nfe, float cfg_scale, int cfg_form, int layout, int ffn_mode,
                     float *z_out);

void orc_pe_forward(const orc_pe *m, const float *frames, int n_patches, int pair_mode,
                    float *out, float *h_last);
/* The two PatchEncoder pieces the reference writes as plain C (patchenc.cpp:19-39,
 * :59-101), for comparison with the reference's own: frames [seq][128] -> out
 * [seq/2][128]; q, k, v, ctx [T][1024]. */
void orc_pe_conv(float *out, const float *frames, int seq, const float *w, const float *b);
void orc_pe_causal_attention(float *ctx, const float *q, const float *k, const float *v, int T);


/* ---------------------------------------------------------------- vocoder
 * BigVGAN v2 decoder as the reference runs it (src/modules/vocoder/
 * bigvgan_cpp.cpp:325-542, include/bigvgan_cpp.h): post_proj, dec_mi_layer
 * (Linear 128->512, 4-layer LSTM with skip, Linear 512->128), conv_pre, six
 * causal upsampling stages of three AMP blocks each, activation_post,
 * conv_post, tanh x 1.92.  Tensor names in the comments are the checkpoint's. */
#define ORC_VOC_STAGES 6
#define ORC_VOC_RB     18
typedef struct {
    const float *post_proj_w, *post_proj_b;          /* post_proj.weight [128][128][1], .bias [128]      */
    const float *mi_w1, *mi_b1;                      /* dec_mi_layer.0.weight [512][128], .bias [512]    */
    const float *mi_w2, *mi_b2;                      /* dec_mi_layer.2.weight [128][512], .bias [128]    */
    const float *lstm_w_ih[4], *lstm_w_hh[4];        /* dec_mi_layer.1.lstm.weight_{ih,hh}_l{l} [2048][512] */
    const float *lstm_b_ih[4], *lstm_b_hh[4];        /* .bias_{ih,hh}_l{l} [2048]                        */
    const float *conv_pre_w, *conv_pre_b;            /* decoder.conv_pre [1536][128][5], [1536]          */
    const float *ups_w[ORC_VOC_STAGES];              /* decoder.ups.{s}.0.weight [in][out][2 stride]     */
    const float *ups_b[ORC_VOC_STAGES];              /* decoder.ups.{s}.0.bias [out]                     */
    const float *c1_w[ORC_VOC_RB][3], *c1_b[ORC_VOC_RB][3];   /* decoder.resblocks.{r}.convs1.{j} [ch][ch][k] */
    const float *c2_w[ORC_VOC_RB][3], *c2_b[ORC_VOC_RB][3];   /* decoder.resblocks.{r}.convs2.{j}             */
    const float *alpha[ORC_VOC_RB][6], *beta[ORC_VOC_RB][6];  /* decoder.resblocks.{r}.activations.{a}.act.{alpha,beta} [ch] */
    const float *post_alpha, *post_beta;             /* decoder.activation_post.act.{alpha,beta} [24]    */
    const float *post_filt_up, *post_filt_down;      /* ...upsample.filter, ...downsample.lowpass.filter [24][1][12] */
    const float *conv_post_w;                        /* decoder.conv_post.weight [1][24][7], no bias     */
} orc_voc;

/* Stage geometry (bigvgan_cpp.cpp:207-210) and AMP constants (:407, :418). */
extern const int orc_voc_up_in[ORC_VOC_STAGES], orc_voc_up_out[ORC_VOC_STAGES];
extern const int orc_voc_up_stride[ORC_VOC_STAGES], orc_voc_up_kernel[ORC_VOC_STAGES];
extern const int orc_voc_rb_kernel[3], orc_voc_rb_dil[3];

/* aa_filter: the 12-tap low-pass filter the AMP activations use
 * (bigvgan_cpp.cpp:27-31). audio [n_frames * 1920]. */
void orc_voc_decode(const orc_voc *m, const float *aa_filter, const float *latent, int n_frames, float *audio);
/* The pieces, for focused tests: Activation1d (up x2, SnakeBeta with log-scale
 * alpha/beta, down x2; :33-124) in place on x [len][ch]; filt [fch][12] with
 * fch = 1 (shared) or ch; and the dec_mi_layer bottleneck (:344-377). */
void orc_voc_activation(float *x, int len, int ch, const float *alpha, const float *beta,
                        const float *filt_up, const float *filt_down, int fch);
void orc_voc_bottleneck(const orc_voc *m, const float *latent, int n_frames, float *out128);

#ifdef __cplusplus
}
#endif
