/* dtts.h - C ABI of the B200 (sm_100a) engine for the dots.tts DiT flow-matching
 * head and PatchEncoder.
 *
 * Plain pointers and sizes only.  Every function returns an int status
 * (DTTS_OK = 0, negative DTTS_ERR_* on failure); dtts_last_error() gives a
 * one-line reason for the calling thread's last failure.  The engine never
 * falls back to the CPU: without a usable sm_100 device, create calls fail
 * with DTTS_ERR_NO_DEVICE.
 *
 * Memory conventions (all fp32 unless noted, row-major, weights PyTorch
 * [out][in] as in the reference's safetensors checkpoint):
 *   DTTS_MEM_HOST    pointers are host memory; the call is synchronous and
 *                    copies in and out itself.
 *   DTTS_MEM_DEVICE  pointers are device memory on the engine's device; the
 *                    call only enqueues work on the engine's stream
 *                    (dtts_*_set_stream), dtts_*_sync() waits and reports
 *                    device-side errors.
 * One engine serves one device; calls on one engine must be serialised by
 * the caller (the reference is single-threaded host code).  Independent
 * engines (one per GPU, one host thread each) run concurrently.
 *
 * Reference interfaces replaced (paths in MaurerAnton/dots.tts.cpp):
 *   dtts_dit_create*          load_dit_weights        src/utils/dit_loader.cpp:15
 *                                                     (+ dit_model, include/dit.h:74-126)
 *   dtts_dit_velocity         manual_dit_block x18 + output layer
 *                                                     include/dit_manual.h:148,
 *                                                     src/e2e_pipeline_v4.cpp:438-478
 *                             dit_forward_raw         include/dit.h:152
 *   dtts_dit_euler_solve      Euler + CFG loop        src/e2e_pipeline_v4.cpp:402-533
 *   dtts_attn_*               manual_attention        include/dit_manual.h:88
 *   dtts_pe_create*           load_patchenc_weights   src/utils/patchenc_loader.cpp:14
 *   dtts_pe_forward           patchenc_forward        include/patchenc.h:70
 *   dtts_pe_stream_reset      patchenc_stream_init    include/patchenc.h:80 (declared only)
 *   dtts_pe_decode            patchenc_decode_step    include/patchenc.h:85 (declared only)
 *   dtts_st_*                 SafeTensorsFile         include/safetensors.h:23
 */
#ifndef DTTS_H
#define DTTS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DTTS_OK                0
#define DTTS_ERR_ARG          -1   /* bad argument or shape                          */
#define DTTS_ERR_CUDA         -2   /* CUDA runtime / launch error                     */
#define DTTS_ERR_OOM          -3   /* device allocation failed                        */
#define DTTS_ERR_TIMEOUT      -4   /* a kernel wait or a host wait hit its limit       */
#define DTTS_ERR_NONFINITE    -5   /* the velocity contained NaN/Inf                   */
#define DTTS_ERR_UNSUPPORTED  -6   /* valid request this build does not implement      */
#define DTTS_ERR_IO           -7   /* file missing / malformed / tensor absent          */
#define DTTS_ERR_NO_DEVICE    -8   /* no sm_100 device with that ordinal                */

#define DTTS_DTYPE_BF16  0   /* bf16 weights and activations, fp32 accumulate/residual */
#define DTTS_DTYPE_FP8   1   /* DiT only: the four block projections in e4m3 x e4m3 ->
                                 fp32 (tcgen05 kind::f8f6f4); weights with one fp32 scale per
                                 output channel, activations with one scale per token row
                                 (LayerNorm outputs: row absmax; attention and GELU outputs:
                                 a per-row bound, see dtts_fp8_quantize_rows); adaLN,
                                 input/output layers, attention core and residual as bf16 */
#define DTTS_DTYPE_F32   2   /* fp32 everywhere (attention sublayer only)              */

#define DTTS_MEM_HOST    0
#define DTTS_MEM_DEVICE  1

#define DTTS_CFG_V4      0   /* v = v_c + s (v_c - v_u)  src/e2e_pipeline_v4.cpp:511 */
#define DTTS_CFG_V3      1   /* v = v_u + s (v_c - v_u)  src/e2e_pipeline.cpp:444    */

#define DTTS_LAYOUT_FM_MASK  0 /* v4 FM mask + position ids, src/e2e_pipeline_v4.cpp:120-155 */
#define DTTS_LAYOUT_FULL     1 /* no mask, positions 0..L-1                                  */

#define DTTS_ROPE_HALF       0 /* pairs (d, d+32): manual_attention, include/dit_manual.h:111-128  */
#define DTTS_ROPE_ADJACENT   1 /* pairs (2i, 2i+1): ggml_rope mode 0, src/modules/backbone/dit_attention.cpp:53-54 */

#define DTTS_PAIR_ADJACENT   0 /* PE output p = out_proj([h_2p | h_2p+1])                       */
#define DTTS_PAIR_AS_WRITTEN 1 /* patchenc.cpp:230-232 reshape/permute as written (n_patches > 1) */

/* ------------------------------------------------------------------ weights */
typedef struct dtts_dit_block_weights {
    const float *wq, *wk, *wv, *wo;   /* [1024][1024]                          */
    const float *bo;                  /* [1024] or NULL                        */
    const float *qn, *kn;             /* [64] per-head RMS gains or NULL       */
    const float *w1, *b1;             /* [4096][1024], [4096]                  */
    const float *w2, *b2;             /* [1024][4096], [1024]                  */
    const float *ada_w, *ada_b;       /* [6144][1024], [6144]                  */
} dtts_dit_block_weights;

typedef struct dtts_dit_weights {
    int n_layers;                     /* 18 for the real model                 */
    const dtts_dit_block_weights *blocks;
    const float *t_w1, *t_b1;         /* time MLP [1024][256], [1024]          */
    const float *t_w2, *t_b2;         /* [1024][1024], [1024]                  */
    const float *spk_w1, *spk_b1;     /* xvec_proj.0 [1024][512], [1024]       */
    const float *spk_ln_w, *spk_ln_b; /* xvec_proj.1 LayerNorm [1024]          */
    const float *oada_w, *oada_b;     /* output adaLN [2048][1024], [2048]     */
    const float *out_w, *out_b;       /* output linear [128][1024], [128]      */
    const float *in_w, *in_b;         /* input_layer [1024][1024], [1024]      */
    const float *hid_w, *hid_b;       /* hidden_proj [1024][1536], [1024]      */
    const float *lat_w, *lat_b;       /* latent_proj [1024][128], [1024]       */
    const float *coord_w, *coord_b;   /* coordinate_proj [1024][128], [1024]   */
    const float *eos_w1, *eos_b1;     /* eos_proj.0 [1536][1536], [1536] or NULL */
    const float *eos_w2, *eos_b2;     /* eos_proj.2 [2][1536], [2]             */
} dtts_dit_weights;

typedef struct dtts_attn_weights {
    const float *wq, *wk, *wv, *wo;   /* [1024][1024] */
    const float *bo;                  /* [1024] or NULL */
    const float *qn, *kn;             /* [64] or NULL */
} dtts_attn_weights;

typedef struct dtts_pe_layer_weights {
    const float *attn_norm_w;         /* [1024] or NULL */
    const float *wq, *wk, *wv, *wo;   /* [1024][1024]   */
    const float *bo;                  /* [1024] or NULL */
    const float *ffn_norm_w;          /* [1024] or NULL */
    const float *w1, *b1;             /* [4096][1024], [4096] */
    const float *w2, *b2;             /* [1024][4096], [1024] */
} dtts_pe_layer_weights;

typedef struct dtts_pe_weights {
    int n_layers;                     /* 24 for the real model */
    const dtts_pe_layer_weights *layers;
    const float *conv_w, *conv_b;     /* ds_proj [128][128][2], [128] */
    const float *in_w, *in_b;         /* in_proj [1024][128], [1024]  */
    const float *out_w, *out_b;       /* out_proj [1536][2048], [1536] */
} dtts_pe_weights;

typedef struct dtts_dit dtts_dit;
typedef struct dtts_attn dtts_attn;
typedef struct dtts_pe dtts_pe;

/* ------------------------------------------------------------------ general */
const char *dtts_version(void);
const char *dtts_status_string(int status);
const char *dtts_last_error(void);
int dtts_device_count(int *n);       /* number of sm_100 devices visible */

/* ------------------------------------------------------------------ DiT */
int dtts_dit_create(const dtts_dit_weights *w, int dtype, int device, dtts_dit **out);
/* Loads the velocity head from a safetensors checkpoint using the reference's
 * tensor names (src/utils/dit_loader.cpp:47-115); F32, F16 and BF16 tensors. */
int dtts_dit_create_from_safetensors(const char *path, int n_layers, int dtype, int device, dtts_dit **out);
int dtts_dit_destroy(dtts_dit *e);
int dtts_dit_set_stream(dtts_dit *e, void *cuda_stream);  /* NULL: the engine's own stream */
int dtts_dit_sync(dtts_dit *e);

/* One velocity forward for `rows` independent sequences of L tokens:
 *   x_in  [rows][L][1024]  DiT input sequence (before input_layer)
 *   cond  [rows][1024]     raw conditioning c (SiLU is applied inside)
 *   mask  [L][L] uint8 (1 = attend) or NULL (bidirectional)
 *   pos   [L] position ids or NULL (0..L-1)
 *   out   [rows][n_out][128] output-layer rows L-n_out .. L-1 (n_out = L: all)
 * == manual_dit_block over all layers + output layer, with the FFN applied to
 * every token. */
int dtts_dit_velocity(dtts_dit *e, const float *x_in, const float *cond, const uint8_t *mask, const float *pos,
                      int rows, int L, int n_out, float *out, int mem);

/* The block stack alone on `rows` sequences of L tokens: h_out = block_{n-1}(...
 * block_0(h_in)), each block = manual_dit_block (include/dit_manual.h:148) with
 * the FFN applied to every token.  h_in, h_out [rows][L][1024], cond
 * [rows][1024] raw c.  A model created with only block weights serves this
 * call (the drop-in manual_dit_block uses one such engine per block). */
int dtts_dit_blocks(dtts_dit *e, const float *h_in, const float *cond, const uint8_t *mask, const float *pos,
                    int rows, int L, float *h_out, int mem);
/* RoPE pairing of the DiT (default DTTS_ROPE_HALF, the live manual_dit_block
 * path; DTTS_ROPE_ADJACENT reproduces the ggml DiT path behind dit_forward_raw). */
int dtts_dit_set_rope(dtts_dit *e, int mode);
/* c = compute_cond(t, spk) on the device (src/e2e_pipeline_v4.cpp:57-71):
 * time MLP of the sinusoid of t, plus speaker_scale * LN(xvec_proj(spk)) when
 * spk != NULL.  Host pointers (spk [512], cond [1024]); synchronous. */
int dtts_dit_cond(dtts_dit *e, float t, const float *spk, float spk_scale, float *cond);

typedef struct dtts_solve_args {
    int n_utt;                 /* utterances; 2*n_utt CFG rows run per step        */
    int fm_len;                /* history tokens; L = fm_len + patch                */
    int patch;                 /* noise frames (4 in the model)                     */
    const float *fm_cond;      /* [n_utt][fm_len][1024]  fm_buffer                  */
    const float *fm_uncond;    /* [n_utt][fm_len][1024]  fm_cfg_buffer              */
    const float *z0;           /* [n_utt][patch][128]    initial noise              */
    const float *spk;          /* [n_utt][512] x-vectors or NULL                    */
    float spk_scale;           /* speaker_scale (1.5 in v4)                         */
    int nfe;                   /* Euler steps, t_k = k / nfe                        */
    float cfg_scale;
    int cfg_form;              /* DTTS_CFG_V4 / DTTS_CFG_V3                         */
    int layout;                /* DTTS_LAYOUT_FM_MASK / DTTS_LAYOUT_FULL            */
    float *z_out;              /* [n_utt][patch][128]                               */
    int mem;                   /* DTTS_MEM_HOST / DTTS_MEM_DEVICE                   */
    int use_graph;             /* capture the whole solve in one CUDA graph         */
} dtts_solve_args;
int dtts_dit_euler_solve(dtts_dit *e, const dtts_solve_args *a);

/* ------------------------------------------------------------------ FM history on the device
 * The autoregressive loop's flow-matching buffers (src/e2e_pipeline_v4.cpp:324-340, 551-588),
 * resident on the engine's device for n_utt utterances: the conditional rows and the CFG rows
 * (null hidden state), each up to `capacity` rows per utterance.  Projections are fp32 GEMMs
 * with the model's hidden_proj / latent_proj; the EOS head uses eos_proj.  Host buffers make
 * the calls synchronous; device buffers enqueue them on the engine stream. */
typedef struct dtts_fm dtts_fm;
#define DTTS_EOS_SILU        0   /* eos_proj.0 -> SiLU -> eos_proj.2 (the model's definition)           */
#define DTTS_EOS_AS_WRITTEN  1   /* s * SiLU(s) between the two layers, as src/e2e_pipeline_v4.cpp:608-609 computes */
int dtts_fm_create(dtts_dit *e, int n_utt, int capacity, dtts_fm **out);
int dtts_fm_destroy(dtts_fm *f);
/* Restarts every utterance with one row: hidden_proj(hidden0[u]) (conditional) and
 * hidden_proj(0) (CFG).  hidden0 [n_utt][1536]  (src/e2e_pipeline_v4.cpp:329-340) */
int dtts_fm_start(dtts_fm *f, const float *hidden0, int mem);
/* Appends latent_proj(z[u][p]) for p < patch (<= 16) to both row sets; z are the solver's raw
 * latents [n_utt][patch][128]  (src/e2e_pipeline_v4.cpp:551-556) */
int dtts_fm_append_latents(dtts_fm *f, const float *z, int patch, int mem);
/* Appends hidden_proj(h[u]) to the conditional rows and hidden_proj(0) to the CFG rows
 * (:576-586).  If eos_prob is not NULL it also receives, per utterance, the EOS head's
 * probability softmax(eos_proj.2(act(eos_proj.0(h))))[1] (:598-619); eos_act is
 * DTTS_EOS_SILU or DTTS_EOS_AS_WRITTEN.  h [n_utt][1536], eos_prob [n_utt]. */
int dtts_fm_append_hidden(dtts_fm *f, const float *h, float *eos_prob, int eos_act, int mem);
int dtts_fm_length(dtts_fm *f, int *rows);
/* Copies the current rows to the host: cond, uncond [n_utt][length][1024]. */
int dtts_fm_read(dtts_fm *f, float *cond, float *uncond);
/* The Euler + CFG solve on the current history: a->n_utt, fm_len, fm_cond and fm_uncond are
 * taken from f; a->z0, spk, z_out (and a->mem, which describes them) as in dtts_dit_euler_solve. */
int dtts_fm_solve(dtts_fm *f, const dtts_solve_args *a);

/* Host only (no device needed): the attention mask and position ids a solve builds for
 * `total` rows of which the first fm_len are history and the last `patch` are noise
 * (build_fm_attn_mask / build_fm_pos_ids, src/e2e_pipeline_v4.cpp:120-155; the solve uses
 * total = fm_len + patch and hidden_patch = 1).  mask [total][total] uint8 (1 = attend) and
 * pos [total], either may be NULL. */
int dtts_fm_layout(int total, int fm_len, int patch, int hidden_patch, uint8_t *mask, float *pos);

/* Launch kinds of dtts_dit_solve_timeline. */
#define DTTS_TL_GEMM_QKV       0   /* QKV projection + qk-norm + RoPE epilogue  */
#define DTTS_TL_GEMM_O         1   /* attention output projection, gated residual */
#define DTTS_TL_GEMM_FFN1      2   /* FFN up projection + GELU                   */
#define DTTS_TL_GEMM_FFN2      3   /* FFN down projection, gated residual        */
#define DTTS_TL_ATTENTION      4   /* softmax(QK^T/8)V core                      */
#define DTTS_TL_LN_MODULATE    5   /* LayerNorm + shift/scale (both per block)   */
#define DTTS_TL_GEMM_ADALN     6   /* adaLN of every step, once per solve        */
#define DTTS_TL_GEMM_INPUT     7   /* input_layer                                */
#define DTTS_TL_OUT_HEAD       8   /* output adaLN-LN + out_proj                 */
#define DTTS_TL_CFG_EULER      9   /* CFG combine + Euler update + coord_proj    */
#define DTTS_TL_CONDITIONING  10   /* history rows, time MLP, speaker, c rows    */
#define DTTS_TL_KINDS         11
/* Device time of every launch of one solve, in place: the solve of `a` (device
 * buffers) is captured into a CUDA graph with a timing event before and after
 * each launch and replayed `reps` times.  us_total[k] = summed device time (us)
 * of kind-k launches in one solve (mean over reps), counts[k] = kind-k launches
 * per solve.  Runs one ordinary solve first; a->z_out receives its result. */
int dtts_dit_solve_timeline(dtts_dit *e, const dtts_solve_args *a, int reps, float *us_total, int *counts);

/* Kernel-level timing of one launch type at the shapes of the last solve or
 * velocity call, on the engine stream with CUDA events (after 3 warm-up
 * launches).  kind: 0 QKV GEMM, 1 O GEMM, 2 FFN1 GEMM, 3 FFN2 GEMM,
 * 4 attention, 5 LayerNorm+modulate, 6 adaLN GEMM, 7 input_layer GEMM.
 * Reports the mean device time of one launch and its algorithmic FLOPs and
 * bytes (operands read once, results written once). */
int dtts_dit_profile_kernel(dtts_dit *e, int kind, int iters, float *us_per_launch, double *flops, double *bytes);
/* Tile configuration of one GEMM of the block stack ("qkv", "o", "ffn1",
 * "ffn2", "adaln", "input"): tile width bn (128/192/256, dividing N),
 * epi_warps (4/8) epilogue warps, ksplit (1/2/4/8, residual GEMMs only).
 * Results are identical up to fp32 summation order; with ksplit > 1 the
 * partial sums reach the residual in run-dependent order, so repeated runs
 * may differ in the last bits.  Defaults (ksplit 1) are tuned for B200. */
int dtts_dit_tune(dtts_dit *e, const char *gemm, int bn, int epi_warps, int ksplit);
/* on = 1: the LayerNorm + adaLN modulation that follows each gated residual
 * (dit_manual.h:158-168) runs in the epilogue of the residual GEMM itself, LN2
 * in the O projection and the next block's LN1 in FFN2.  on = 0 (the default,
 * unless DTTS_FUSE_LN=1 is set when the engine is created): standalone
 * LayerNorm kernels, which are faster on B200.  Both give identical results.
 * The fused form needs the residual GEMMs at ksplit 1 with a tile width of 128
 * or 256 (dtts_dit_tune) and falls back to the standalone kernels otherwise.
 * It is a cooperative launch whose CTAs wait on one another's arrivals
 * (bounded, DTTS_ERR_TIMEOUT on expiry). */
int dtts_dit_set_fused_ln(dtts_dit *e, int on);
/* Kernel launches enqueued by the last solve / velocity call (all engine kernels). */
int dtts_dit_last_launch_count(dtts_dit *e, int *n);

/* ------------------------------------------------------------------ attention sublayer */
int dtts_attn_create(const dtts_attn_weights *w, int dtype, int device, dtts_attn **out);
int dtts_attn_destroy(dtts_attn *a);
/* out = manual_attention(x): x, out [rows][L][1024]; mask [L][L] or NULL; pos [L] or NULL */
int dtts_attn_forward(dtts_attn *a, const float *x, int rows, int L, const uint8_t *mask, const float *pos,
                      float *out);
/* mean device time (us) of the attention core kernel (post-QKV, pre-O) of the last forward */
int dtts_attn_profile_core(dtts_attn *a, int iters, float *us_per_launch);

/* fp32 attention sublayer that performs no device allocation (no counterpart
 * in the reference).  For callers that may not allocate GPU memory while they
 * run -- a host that gives the library a fixed memory budget, a plugin whose
 * runtime forbids allocation during execution, a real-time audio thread where
 * an allocation could block -- every argument is a device pointer the caller
 * owns (x, out [rows][L][1024]; weights as in dtts_attn_weights; mask [L][L]
 * and pos [L] or NULL) and the intermediates live in one fixed array compiled
 * into the library: 4.06 MiB on a device from the first call there (from
 * library load when CUDA_MODULE_LOADING=EAGER) until the process exits.
 * Limits: rows * L <= DTTS_NOALLOC_MAX_TOKENS and L <= 256; larger shapes
 * return DTTS_ERR_ARG.  Work is enqueued on `cuda_stream` (NULL: the default
 * stream) on the current device; the call returns without waiting.  The first
 * call on a device (and the first after a device reset) looks up the array's
 * address and sets a kernel attribute, so make that first call before any
 * stream capture.  All calls on a device share the array: calls whose work
 * overlaps on the GPU race and must be serialised by the caller.  Nothing in
 * the array needs to start at zero. */
#define DTTS_NOALLOC_MAX_TOKENS 256
int dtts_attn_forward_f32_noalloc(const float *x, const float *wq, const float *wk, const float *wv, const float *wo,
                                  const float *bo, const float *qn, const float *kn, const uint8_t *mask,
                                  const float *pos, int rows, int L, float *out, void *cuda_stream);

/* ------------------------------------------------------------------ PatchEncoder */
/* max_batch sequences, each with a KV cache of max_tokens tokens (2 per patch). */
int dtts_pe_create(const dtts_pe_weights *w, int dtype, int device, int max_batch, int max_tokens, dtts_pe **out);
int dtts_pe_create_from_safetensors(const char *path, int n_layers, int dtype, int device, int max_batch,
                                    int max_tokens, dtts_pe **out);
int dtts_pe_destroy(dtts_pe *p);
int dtts_pe_set_stream(dtts_pe *p, void *cuda_stream);
int dtts_pe_sync(dtts_pe *p);
/* Stateless full forward (patchenc_forward): frames [B][n_frames][128],
 * n_frames a multiple of 4; out [B][n_frames/4][1536]. Resets the streams. */
int dtts_pe_forward(dtts_pe *p, const float *frames, int B, int n_frames, int pair_mode, float *out, int mem);
/* Starts B empty streams (no history, zero conv tail). */
int dtts_pe_stream_reset(dtts_pe *p, int B);
/* Appends n_frames (multiple of 4) to each of the B streams: one patch = one
 * decode step; a prefill is the same call with many patches.  out
 * [B][n_frames/4][1536].  Causal, so equal to the stateless forward over the
 * whole prefix (adjacent pairing). */
int dtts_pe_decode(dtts_pe *p, const float *frames, int B, int n_frames, float *out, int mem);
int dtts_pe_stream_length(dtts_pe *p, int *tokens);

/* ------------------------------------------------------------------ LLM decoder step
 * The autoregressive loop's Qwen2.5-1.5B step (src/llm_manual.cpp): a batch of B sequences
 * advancing together.  bf16 weights and K/V cache, fp32 residual and attention arithmetic.
 * Embedding lookup stays with the caller: the calls take embeddings. */
typedef struct dtts_llm dtts_llm;
typedef struct dtts_llm_layer_weights {
    const float *an, *fn;             /* input_layernorm, post_attention_layernorm [1536] */
    const float *qw, *qb;             /* q_proj [1536][1536], [1536]                     */
    const float *kw, *kb, *vw, *vb;   /* k_proj, v_proj [256][1536], [256]               */
    const float *ow, *ob;             /* o_proj [1536][1536], bias or NULL               */
    const float *gw, *uw;             /* gate_proj, up_proj [8960][1536]                 */
    const float *dw;                  /* down_proj [1536][8960]                          */
} dtts_llm_layer_weights;
typedef struct dtts_llm_weights {
    int n_layers;                     /* 28 for Qwen2.5-1.5B */
    const dtts_llm_layer_weights *layers;
    const float *final_norm;          /* model.norm [1536] */
} dtts_llm_weights;
/* Replaces load_llm_weights (src/llm_manual.cpp:13): weights uploaded once; K/V cache for
 * max_batch sequences of max_seq tokens. */
int dtts_llm_create(const dtts_llm_weights *w, int device, int max_batch, int max_seq, dtts_llm **out);
int dtts_llm_destroy(dtts_llm *e);
int dtts_llm_set_stream(dtts_llm *e, void *cuda_stream);
/* llm_kv_cache_init (src/llm_manual.cpp:237) for B prompts at once: emb [B][n_tok][1536] ->
 * hidden [B][n_tok][1536] after the final norm; restarts the caches. */
int dtts_llm_prefill(dtts_llm *e, const float *emb, int B, int n_tok, float *hidden, int mem);
/* llm_kv_cache_step (src/llm_manual.cpp:342): one embedding per sequence, emb [B][1536] ->
 * hidden [B][1536]; B must match the prefill. */
int dtts_llm_step(dtts_llm *e, const float *emb, int B, float *hidden, int mem);
int dtts_llm_length(dtts_llm *e, int *tokens);

/* ------------------------------------------------------------------ vocoder
 * BigVGAN v2 decoder (src/modules/vocoder/bigvgan_cpp.cpp, include/bigvgan_cpp.h): the
 * latents of an utterance [n_frames][128] to audio [n_frames * 1920] at 24 kHz.  Convolutions
 * run as tcgen05 GEMMs over taps on bf16 time-major activations (fp32 accumulate, fp32
 * residual stream); the LSTM bottleneck and the activations are fp32.  Tensor names below
 * are the checkpoint's (bigvgan_load, bigvgan_cpp.cpp:203-290). */
typedef struct dtts_voc dtts_voc;
typedef struct dtts_voc_weights {
    const float *post_proj_w, *post_proj_b;   /* post_proj.weight [128][128][1], .bias [128]          */
    const float *mi_w1, *mi_b1;               /* dec_mi_layer.0.weight [512][128], .bias [512]        */
    const float *mi_w2, *mi_b2;               /* dec_mi_layer.2.weight [128][512], .bias [128]        */
    const float *lstm_w_ih[4], *lstm_w_hh[4]; /* dec_mi_layer.1.lstm.weight_{ih,hh}_l{0..3} [2048][512] */
    const float *lstm_b_ih[4], *lstm_b_hh[4]; /* dec_mi_layer.1.lstm.bias_{ih,hh}_l{0..3} [2048]      */
    const float *conv_pre_w, *conv_pre_b;     /* decoder.conv_pre [1536][128][5], [1536]              */
    const float *ups_w[6], *ups_b[6];         /* decoder.ups.{s}.0 [in][out][2 stride], [out]          */
    const float *c1_w[18][3], *c1_b[18][3];   /* decoder.resblocks.{r}.convs1.{j} [ch][ch][k], [ch]    */
    const float *c2_w[18][3], *c2_b[18][3];   /* decoder.resblocks.{r}.convs2.{j}                      */
    const float *alpha[18][6], *beta[18][6];  /* decoder.resblocks.{r}.activations.{a}.act.alpha/.beta */
    const float *post_alpha, *post_beta;      /* decoder.activation_post.act.alpha/.beta [24]          */
    const float *post_filt_up;                /* decoder.activation_post.upsample.filter [24][1][12]   */
    const float *post_filt_down;              /* ...downsample.lowpass.filter [24][1][12]              */
    const float *conv_post_w;                 /* decoder.conv_post.weight [1][24][7] (no bias)         */
} dtts_voc_weights;
/* Replaces bigvgan_load (bigvgan_cpp.cpp:203): weights uploaded once; work buffers for
 * utterances of up to max_frames latent frames. */
int dtts_voc_create(const dtts_voc_weights *w, int device, int max_frames, dtts_voc **out);
int dtts_voc_destroy(dtts_voc *v);
int dtts_voc_set_stream(dtts_voc *v, void *cuda_stream);
/* bigvgan_decode (bigvgan_cpp.cpp:325): latent [n_frames][128] -> audio [n_frames * 1920]. */
int dtts_voc_decode(dtts_voc *v, const float *latent, int n_frames, float *audio, int mem);
/* The 12-tap low-pass filter of the AMP activations (BigVGAN's kaiser_sinc_filter1d with
 * cutoff 0.25, half width 0.3), as the engine computes it. */
int dtts_voc_aa_filter(float *taps12);
/* One Activation1d (up x2, SnakeBeta, down x2) on x [len][ch] fp32 (host), out fp32;
 * filt_up / filt_down hold 12 taps shared by all channels (fch = 1) or [ch][12] (fch = ch);
 * alpha / beta are the log-scale parameters [ch]. */
int dtts_selftest_voc_activation(const float *x, int len, int ch, const float *alpha, const float *beta,
                                 const float *filt_up, const float *filt_down, int fch, float *out);

/* ------------------------------------------------------------------ self-test
 * Failure detection without a fault: one kernel thread waits on an mbarrier that
 * nothing completes, through the bounded wait of every engine kernel (2 s of
 * %globaltimer); it must give up, leave its code in *code (1: producer wait) and
 * return DTTS_ERR_TIMEOUT with the context still usable. */
int dtts_selftest_wait_limit(int device, int *code);
/* A time convolution through the tcgen05 GEMM over taps, as the vocoder runs it:
 * out[t][o] = bias[o] + sum_k sum_c x[t + k dil - pad_left][c] w[o][c][k] (zero outside
 * [0, T)); x [T][C], w [N][C][K], inputs rounded to bf16; C % 64 == 0, bn | N. */
int dtts_selftest_conv(const float *x, int T, int C, const float *w, const float *bias, int N, int K, int dil,
                       int pad_left, int bn, float *out, int device);
/* ------------------------------------------------------------------ kernel self-tests
 * One engine kernel in isolation on host data (no reference counterpart):
 * inputs are rounded to bf16 on the host exactly as the engine stores them. */
/* C[M][N] = A[M][K] B[N][K]^T (+ bias) with the tcgen05 GEMM; bn = 64, 128, 192 or 256 */
int dtts_selftest_gemm(const float *A, const float *B, const float *bias, float *C, int M, int N, int K, int bn,
                       int device);
/* C[M][N] = a_scale[m] b_scale[n] sum_k A[m][k] B[n][k] (+ bias) with e4m3 bytes A
 * [M][K], B [N][K] through the kind::f8f6f4 GEMM; bn = 128 or 256, K % 128 == 0 */
int dtts_selftest_gemm_e4m3(const uint8_t *A, const float *a_scale, const uint8_t *B, const float *b_scale,
                            const float *bias, float *C, int M, int N, int K, int bn, int device);
/* attention core: q [rows][Tq][1024], k/v [rows][kv_len][1024], out like q */
int dtts_selftest_attention(const float *q, const float *k, const float *v, float *out, int rows, int Tq,
                            int kv_len, const uint8_t *mask, int causal, int q_pos0, int use_f32, int device);

/* e4m3 conversion (round to nearest even, saturating at +-448) of n floats on
 * the device, the conversion every FP8 kernel uses for its activations. */
int dtts_selftest_e4m3(const float *x, uint8_t *out, int n, int device);

/* Host only: the FP8 engine's weight quantisation (no counterpart in the
 * reference, whose DiT is fp32).  w [rows][cols] row-major, one scale per row
 * (output channel): scale[r] = max_c |w[r][c]| / 448 and q[r][c] =
 * e4m3(w[r][c] * 448 / max_c |w[r][c]|); an all-zero row gets scale 0.
 * Dequantised weight = e4m3 value * scale. */
int dtts_fp8_quantize_rows(const float *w, int rows, int cols, uint8_t *q, float *scale);

/* ------------------------------------------------------------------ safetensors (host only) */
typedef struct dtts_st dtts_st;
int dtts_st_open(const char *path, dtts_st **out);
int dtts_st_close(dtts_st *f);
int dtts_st_count(dtts_st *f, int *n);
/* shape of tensor `name` (ndim <= 8); returns DTTS_ERR_IO if absent */
int dtts_st_shape(dtts_st *f, const char *name, int *ndim, int64_t *shape);
/* reads tensor `name` converted to fp32 into dst (n elements exactly) */
int dtts_st_read_f32(dtts_st *f, const char *name, float *dst, size_t n);

#ifdef __cplusplus
}
#endif
#endif /* DTTS_H */
