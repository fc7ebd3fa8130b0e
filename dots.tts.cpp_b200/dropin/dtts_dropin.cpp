// Drop-in definitions of the reference's DiT / PatchEncoder entry points on top
// of the B200 engine (libdtts.so, include/dtts.h).
//
// Compile this file into a program built against the reference's headers
// (MaurerAnton/dots.tts.cpp include/: dit.h, patchenc.h, dots_tts.h,
// dots_tts_util.h and its ggml.h), with this repository's include/ first on
// the include path so that "dit_manual.h" is the replacement header, and link
// libdtts.so.  It replaces:
//   manual_attention, manual_dit_block, manual_* helpers   include/dit_manual.h
//   dit_forward_raw                                         include/dit.h:152 (src/modules/backbone/dit_forward.cpp)
//   patchenc_forward                                        include/patchenc.h:70 (src/modules/backbone/patchenc.cpp)
//   patchenc_stream_init / _free / patchenc_decode_step     include/patchenc.h:80-90 (declared, never defined there)
//
// One engine is created per weight set (keyed by the model / block / weight
// address) on the first call and reused; weights are uploaded once.
#include "dit.h"
#include "patchenc.h"
#include "dots_tts_util.h"
#include "dit_manual.h"
#include "dtts.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

namespace {

int g_device = 0;
std::mutex g_mu;
std::map<const void *, dtts_dit *> g_dit;     // dit_model* / dit_block* -> engine
std::map<const void *, dtts_attn *> g_attn;   // q weight data -> fp32 attention sublayer

[[noreturn]] void die(const char *what, int st) {
    fprintf(stderr, "dtts drop-in: %s failed: %s (%s)\n", what, dtts_status_string(st), dtts_last_error());
    abort();
}

void check(int st, const char *what) {
    if (st != DTTS_OK) die(what, st);
}

const float *td(ggml_tensor *t) { return t ? tensor_data(t) : nullptr; }

dtts_dit_block_weights block_weights(const dit_block &b) {
    dtts_dit_block_weights w;
    std::memset(&w, 0, sizeof(w));
    w.wq = td(b.attn_q_weight); w.wk = td(b.attn_k_weight); w.wv = td(b.attn_v_weight); w.wo = td(b.attn_o_weight);
    w.bo = td(b.attn_o_bias); w.qn = td(b.q_norm_w); w.kn = td(b.k_norm_w);
    w.w1 = td(b.ffn_w1); w.b1 = td(b.ffn_b1); w.w2 = td(b.ffn_w2); w.b2 = td(b.ffn_b2);
    w.ada_w = td(b.adaln_linear_w); w.ada_b = td(b.adaln_linear_b);
    return w;
}

dtts_dit *model_engine(dit_model &m) {
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_dit.find(&m);
    if (it != g_dit.end()) return it->second;
    std::vector<dtts_dit_block_weights> blocks;
    for (int i = 0; i < m.n_layers; i++) blocks.push_back(block_weights(m.layers[i]));
    dtts_dit_weights w;
    std::memset(&w, 0, sizeof(w));
    w.n_layers = m.n_layers;
    w.blocks = blocks.data();
    w.t_w1 = td(m.t_embed_w1); w.t_b1 = td(m.t_embed_b1); w.t_w2 = td(m.t_embed_w2); w.t_b2 = td(m.t_embed_b2);
    w.spk_w1 = td(m.spk_proj_w1); w.spk_b1 = td(m.spk_proj_b1); w.spk_ln_w = td(m.spk_ln_w); w.spk_ln_b = td(m.spk_ln_b);
    w.oada_w = td(m.out_adaln_w); w.oada_b = td(m.out_adaln_b); w.out_w = td(m.out_proj_w); w.out_b = td(m.out_proj_b);
    w.in_w = td(m.input_layer_w); w.in_b = td(m.input_layer_b);
    w.hid_w = td(m.hidden_proj_w); w.hid_b = td(m.hidden_proj_b);
    w.lat_w = td(m.latent_proj_w); w.lat_b = td(m.latent_proj_b);
    w.coord_w = td(m.coord_proj_w); w.coord_b = td(m.coord_proj_b);
    w.eos_w1 = td(m.eos_proj_w1); w.eos_b1 = td(m.eos_proj_b1);
    w.eos_w2 = td(m.eos_proj_w2); w.eos_b2 = td(m.eos_proj_b2);
    dtts_dit *e = nullptr;
    check(dtts_dit_create(&w, DTTS_DTYPE_BF16, g_device, &e), "dtts_dit_create");
    g_dit[&m] = e;
    return e;
}

dtts_dit *block_engine(const dit_block &b) {
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_dit.find(&b);
    if (it != g_dit.end()) return it->second;
    dtts_dit_block_weights bw = block_weights(b);
    dtts_dit_weights w;
    std::memset(&w, 0, sizeof(w));
    w.n_layers = 1;
    w.blocks = &bw;
    dtts_dit *e = nullptr;
    check(dtts_dit_create(&w, DTTS_DTYPE_BF16, g_device, &e), "dtts_dit_create (block)");
    g_dit[&b] = e;
    return e;
}

std::vector<uint8_t> mask_bytes(const bool *m, int n) {
    std::vector<uint8_t> out;
    if (m) {
        out.resize((size_t)n * n);
        for (size_t i = 0; i < out.size(); i++) out[i] = m[i] ? 1 : 0;
    }
    return out;
}

}  // namespace

// ------------------------------------------------------------------ host helpers
// Same arithmetic as the reference's inline helpers (include/dit_manual.h:16-86).
void manual_layernorm(float *out, const float *x, int n) {
    float mean = 0;
    for (int i = 0; i < n; i++) mean += x[i];
    mean /= n;
    float var = 0;
    for (int i = 0; i < n; i++) { const float d = x[i] - mean; var += d * d; }
    const float inv_std = 1.0f / sqrtf(var / n + 1e-5f);
    for (int i = 0; i < n; i++) out[i] = (x[i] - mean) * inv_std;
}

void manual_rms_norm(float *out, const float *x, const float *weight, int n) {
    float ss = 0;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    const float inv = 1.0f / sqrtf(ss / n + 1e-6f);
    for (int i = 0; i < n; i++) { float v = x[i] * inv; if (weight) v *= weight[i]; out[i] = v; }
}

void manual_linear(float *out, const float *x, const float *w, const float *bias, int in_feat, int out_feat) {
    for (int o = 0; o < out_feat; o++) {
        const float *wr = w + (size_t)o * in_feat;
        float s = bias ? bias[o] : 0.0f;
        for (int i = 0; i < in_feat; i++) s += wr[i] * x[i];
        out[o] = s;
    }
}

void manual_rope_theta(float *q, float *k, int seq_len, int head_dim, float rope_theta) {
    const int half = head_dim / 2;
    const float ts = powf(rope_theta, -2.0f / (float)head_dim);
    for (int s = 0; s < seq_len; s++) {
        float theta = 1.0f;
        for (int d = 0; d < half; d++) {
            const float cs = cosf((float)s * theta), sn = sinf((float)s * theta);
            const int i1 = s * head_dim + d, i2 = i1 + half;
            const float q0 = q[i1], q1 = q[i2], k0 = k[i1], k1 = k[i2];
            q[i1] = q0 * cs - q1 * sn; q[i2] = q1 * cs + q0 * sn;
            k[i1] = k0 * cs - k1 * sn; k[i2] = k1 * cs + k0 * sn;
            theta *= ts;
        }
    }
}

void manual_rope(float *q, float *k, int seq_len, int head_dim) { manual_rope_theta(q, k, seq_len, head_dim, 10000.0f); }

void manual_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) mx = x[i] > mx ? x[i] : mx;
    float sum = 0;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

// ------------------------------------------------------------------ device-backed DiT math
void manual_attention(float *out, const float *x, const float *qw, const float *kw, const float *vw, const float *ow,
                      const float *qb, const float *kb, const float *vb, const float *ob, const float *qnw,
                      const float *knw, int n_tokens, int hidden, int n_heads, int head_dim, const bool *attn_mask,
                      const float *pos_ids) {
    if (hidden != 1024 || n_heads != 16 || head_dim != 64) die("manual_attention (only 1024 = 16 x 64 supported)", DTTS_ERR_UNSUPPORTED);
    if (qb || kb || vb) die("manual_attention (q/k/v biases are not supported)", DTTS_ERR_UNSUPPORTED);
    dtts_attn *a = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        auto it = g_attn.find(qw);
        if (it == g_attn.end()) {
            dtts_attn_weights w = {qw, kw, vw, ow, ob, qnw, knw};
            check(dtts_attn_create(&w, DTTS_DTYPE_F32, g_device, &a), "dtts_attn_create");
            g_attn[qw] = a;
        } else {
            a = it->second;
        }
    }
    std::vector<uint8_t> m = mask_bytes(attn_mask, n_tokens);
    check(dtts_attn_forward(a, x, 1, n_tokens, attn_mask ? m.data() : nullptr, pos_ids, out), "dtts_attn_forward");
}

void manual_dit_block(const float *x_in, const float *cond, const dit_block &block, float *out, int n_tokens,
                      const bool *attn_mask, const float *pos_ids) {
    dtts_dit *e = block_engine(block);
    std::vector<uint8_t> m = mask_bytes(attn_mask, n_tokens);
    check(dtts_dit_blocks(e, x_in, cond, attn_mask ? m.data() : nullptr, pos_ids, 1, n_tokens, out, DTTS_MEM_HOST),
          "dtts_dit_blocks");
}

// dit_forward_raw follows the reference's ggml DiT (src/modules/backbone/dit_forward.cpp:113-156):
// no mask, positions 0..L-1, ggml_rope mode 0 (adjacent pairs, dit_attention.cpp:53-54), and
// compute_cond adding the speaker term without a scale (dit_forward.cpp:31-35).
void dit_forward_raw(dit_model &model, const float *x, int seq_len, float t_val, const float *speaker_emb,
                     float *out) {
    dtts_dit *e = model_engine(model);
    check(dtts_dit_set_rope(e, DTTS_ROPE_ADJACENT), "dtts_dit_set_rope");
    float cond[1024];
    check(dtts_dit_cond(e, t_val, speaker_emb, 1.0f, cond), "dtts_dit_cond");
    check(dtts_dit_velocity(e, x, cond, nullptr, nullptr, 1, seq_len, seq_len, out, DTTS_MEM_HOST), "dtts_dit_velocity");
}

// ------------------------------------------------------------------ PatchEncoder
namespace {
dtts_pe_weights pe_weights(patch_encoder &enc, std::vector<dtts_pe_layer_weights> &layers) {
    layers.clear();
    for (int i = 0; i < enc.n_layers; i++) {
        patchenc_layer &l = enc.layers[i];
        dtts_pe_layer_weights w;
        std::memset(&w, 0, sizeof(w));
        w.attn_norm_w = td(l.attn_norm_w);
        w.wq = td(l.attn_q_weight); w.wk = td(l.attn_k_weight); w.wv = td(l.attn_v_weight); w.wo = td(l.attn_o_weight);
        w.bo = td(l.attn_o_bias); w.ffn_norm_w = td(l.ffn_norm_w);
        w.w1 = td(l.ffn_w1); w.b1 = td(l.ffn_b1); w.w2 = td(l.ffn_w2); w.b2 = td(l.ffn_b2);
        layers.push_back(w);
    }
    dtts_pe_weights w;
    std::memset(&w, 0, sizeof(w));
    w.n_layers = enc.n_layers;
    w.layers = layers.data();
    w.conv_w = td(enc.conv_weight); w.conv_b = td(enc.conv_bias);
    w.in_w = td(enc.in_proj_w); w.in_b = td(enc.in_proj_b);
    w.out_w = td(enc.out_proj_w); w.out_b = td(enc.out_proj_b);
    return w;
}

constexpr int kStreamTokens = 1024;   // KV cache per stream: 512 patches

struct pe_slot {
    dtts_pe *pe;
    int tokens;                           // token capacity the engine was created with
};
std::map<const void *, pe_slot> g_pe;     // patch_encoder* -> stateless engine

dtts_pe *pe_engine(patch_encoder &enc, int tokens) {
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_pe.find(&enc);
    if (it != g_pe.end()) {
        if (it->second.tokens >= tokens) return it->second.pe;
        dtts_pe_destroy(it->second.pe);
        g_pe.erase(it);
    }
    const int cap = tokens > kStreamTokens ? tokens : kStreamTokens;
    std::vector<dtts_pe_layer_weights> layers;
    dtts_pe_weights w = pe_weights(enc, layers);
    dtts_pe *p = nullptr;
    check(dtts_pe_create(&w, DTTS_DTYPE_BF16, g_device, 1, cap, &p), "dtts_pe_create");
    g_pe[&enc] = pe_slot{p, cap};
    return p;
}
}  // namespace

struct patchenc_stream_state {
    dtts_pe *pe;
};

// Output pairs follow the reference's reshape/permute exactly (patchenc.cpp:230-232).
// Unlike the reference, x is not overwritten and ctx is not reset.
ggml_tensor *patchenc_forward(patch_encoder &enc, ggml_context *ctx, ggml_tensor *x, int n_patches) {
    dtts_pe *p = pe_engine(enc, 2 * n_patches);
    std::vector<float> out((size_t)n_patches * 1536);
    check(dtts_pe_forward(p, tensor_data(x), 1, 4 * n_patches, DTTS_PAIR_AS_WRITTEN, out.data(), DTTS_MEM_HOST),
          "dtts_pe_forward");
    ggml_tensor *r = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, 1536, n_patches);
    std::memcpy(tensor_data(r), out.data(), out.size() * sizeof(float));
    return r;
}

patchenc_stream_state *patchenc_stream_init(patch_encoder &enc) {
    std::vector<dtts_pe_layer_weights> layers;
    dtts_pe_weights w = pe_weights(enc, layers);
    patchenc_stream_state *st = new patchenc_stream_state();
    check(dtts_pe_create(&w, DTTS_DTYPE_BF16, g_device, 1, kStreamTokens, &st->pe), "dtts_pe_create (stream)");
    check(dtts_pe_stream_reset(st->pe, 1), "dtts_pe_stream_reset");
    return st;
}

void patchenc_stream_free(patchenc_stream_state *st) {
    if (!st) return;
    dtts_pe_destroy(st->pe);
    delete st;
}

void patchenc_decode_step(patch_encoder &enc, patchenc_stream_state *st, ggml_context *ctx, float *patch,
                          float *llm_emb_out) {
    (void)enc;
    (void)ctx;
    check(dtts_pe_decode(st->pe, patch, 1, 4, llm_emb_out, DTTS_MEM_HOST), "dtts_pe_decode");
}

// ------------------------------------------------------------------ housekeeping
void dtts_dropin_set_device(int device) { g_device = device; }

void dtts_dropin_release() {
    std::lock_guard<std::mutex> lock(g_mu);
    for (auto &kv : g_dit) dtts_dit_destroy(kv.second);
    for (auto &kv : g_attn) dtts_attn_destroy(kv.second);
    for (auto &kv : g_pe) dtts_pe_destroy(kv.second.pe);
    g_dit.clear();
    g_attn.clear();
    g_pe.clear();
}
