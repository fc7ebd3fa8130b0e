// dit_manual.h - drop-in replacement for the reference's header of the same name
// (MaurerAnton/dots.tts.cpp include/dit_manual.h).
//
// Put this repository's include/ directory ahead of the reference's on the
// include path and compile dots.tts.cpp_b200/dropin/dtts_dropin.cpp into the
// program (link libdtts.so): every function keeps its name, signature and
// argument meaning, and the two heavy ones run on the B200 engine:
//
//   manual_attention   include/dit_manual.h:88   -> dtts_attn (fp32 sublayer)
//   manual_dit_block   include/dit_manual.h:148  -> dtts_dit_blocks (bf16 block,
//                                                   FFN applied to every token)
//
// The small host helpers (LayerNorm, RMSNorm, linear, RoPE, softmax) stay on
// the host with the reference's arithmetic, for callers that use them around
// the DiT (e.g. src/e2e_pipeline_v4.cpp:443,465,472).
//
// Weights are read through the dit_block's ggml_tensor views and uploaded on
// the first call for a given weight set; they must not change afterwards
// (call dtts_dropin_release() first).  Device errors abort with a message:
// the reference's signatures have no error return.
#pragma once

#include "dit.h"
#include "dots_tts.h"

void manual_layernorm(float *out, const float *x, int n);
void manual_rms_norm(float *out, const float *x, const float *weight, int n);
void manual_linear(float *out, const float *x, const float *w, const float *bias, int in_feat, int out_feat);
void manual_rope_theta(float *q, float *k, int seq_len, int head_dim, float rope_theta);
void manual_rope(float *q, float *k, int seq_len, int head_dim);
void manual_softmax(float *x, int n);

void manual_attention(float *out, const float *x, const float *qw, const float *kw, const float *vw, const float *ow,
                      const float *qb, const float *kb, const float *vb, const float *ob, const float *qnw,
                      const float *knw, int n_tokens, int hidden, int n_heads, int head_dim,
                      const bool *attn_mask = nullptr, const float *pos_ids = nullptr);

void manual_dit_block(const float *x_in, const float *cond, const dit_block &block, float *out, int n_tokens,
                      const bool *attn_mask = nullptr, const float *pos_ids = nullptr);

// Device used by the drop-in engines (default 0; set before the first call).
void dtts_dropin_set_device(int device);
// Destroys every engine the drop-in layer created (weights are re-uploaded on next use).
void dtts_dropin_release();
