// Thin extern "C" driver around the reference's own header-only DiT math
// (include/dit_manual.h of MaurerAnton/dots.tts.cpp), compiled in place from
// the reference tree by oracle/Makefile into oracle/_ref/libdtts_ref.so.
//
// TEST INFRASTRUCTURE ONLY: used by tests/ to pin the C oracle (oracle.c)
// and by bench.py's reference arm as the reference's CPU path.
//
// Everything below only marshals plain arrays into the reference's structs
// (dit_block, ggml_tensor views) and calls:
//   manual_attention   include/dit_manual.h:88-146
//   manual_dit_block   include/dit_manual.h:148-199 (as shipped)
// plus a per-token-FFN block built from the same primitives, and the
// velocity forward wired like src/e2e_pipeline_v4.cpp:441-478.
#include "ref_views.h"
#include <vector>
#include <cstdint>
#include <cstdlib>
#include <omp.h>

// Block flow of manual_dit_block with the FFN applied to every token.  The
// single change from include/dit_manual.h:171-197 is the per-token loop
// around the two FFN projections; all arithmetic goes through the
// reference's own manual_layernorm / manual_attention / manual_linear.
void dit_block_per_token_ffn(const float *x_in, const float *cond, const dit_block &block,
                             float *out, int n_tokens, const bool *attn_mask, const float *pos_ids) {
    const int hidden = DIT_HIDDEN_SIZE;
    std::vector<float> cs(1024), ada(6 * hidden);
    for (int i = 0; i < 1024; i++) cs[i] = cond[i] / (1.0f + expf(-cond[i]));
    {
        float *aw = tensor_data(block.adaln_linear_w);
        float *ab = block.adaln_linear_b ? tensor_data(block.adaln_linear_b) : nullptr;
        for (int o = 0; o < 6 * hidden; o++) {
            float s = ab ? ab[o] : 0.0f;
            for (int i = 0; i < hidden; i++) s += aw[o * hidden + i] * cs[i];
            ada[o] = s;
        }
    }
    const float *sm = ada.data(), *scm = sm + hidden, *gm = sm + 2 * hidden;
    const float *sml = sm + 3 * hidden, *scl = sm + 4 * hidden, *gml = sm + 5 * hidden;
    std::vector<float> normed((size_t)n_tokens * hidden), mod((size_t)n_tokens * hidden),
        ao((size_t)n_tokens * hidden), h((size_t)n_tokens * hidden);
    for (int t = 0; t < n_tokens; t++) {
        manual_layernorm(&normed[(size_t)t * hidden], x_in + (size_t)t * hidden, hidden);
        for (int i = 0; i < hidden; i++) mod[(size_t)t * hidden + i] = normed[(size_t)t * hidden + i] * (1.0f + scm[i]) + sm[i];
    }
    manual_attention(ao.data(), mod.data(), tensor_data(block.attn_q_weight), tensor_data(block.attn_k_weight),
                     tensor_data(block.attn_v_weight), tensor_data(block.attn_o_weight),
                     nullptr, nullptr, nullptr, block.attn_o_bias ? tensor_data(block.attn_o_bias) : nullptr,
                     block.q_norm_w ? tensor_data(block.q_norm_w) : nullptr,
                     block.k_norm_w ? tensor_data(block.k_norm_w) : nullptr,
                     n_tokens, hidden, DIT_NUM_HEADS, DIT_HEAD_SIZE, attn_mask, pos_ids);
    for (size_t i = 0; i < h.size(); i++) h[i] = x_in[i] + gm[i % hidden] * ao[i];
    for (int t = 0; t < n_tokens; t++) {
        manual_layernorm(&normed[(size_t)t * hidden], &h[(size_t)t * hidden], hidden);
        for (int i = 0; i < hidden; i++) mod[(size_t)t * hidden + i] = normed[(size_t)t * hidden + i] * (1.0f + scl[i]) + sml[i];
    }
    std::vector<float> ft(DIT_FFN_SIZE), fo(hidden);
    const float c1 = 0.7978845608028654f, c2 = 0.044715f;
    for (int t = 0; t < n_tokens; t++) {
        manual_linear(ft.data(), &mod[(size_t)t * hidden], tensor_data(block.ffn_w1),
                      block.ffn_b1 ? tensor_data(block.ffn_b1) : nullptr, hidden, DIT_FFN_SIZE);
        for (int i = 0; i < DIT_FFN_SIZE; i++) { float x = ft[i]; float x3 = x * x * x; ft[i] = 0.5f * x * (1.0f + tanhf(c1 * (x + c2 * x3))); }
        manual_linear(fo.data(), ft.data(), tensor_data(block.ffn_w2),
                      block.ffn_b2 ? tensor_data(block.ffn_b2) : nullptr, DIT_FFN_SIZE, hidden);
        for (int i = 0; i < hidden; i++) out[(size_t)t * hidden + i] = h[(size_t)t * hidden + i] + gml[i] * fo[i];
    }
}

extern "C" {

int ref_num_threads(void) { return omp_get_max_threads(); }
void ref_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }

void ref_manual_attention(float *out, const float *x, int n_tokens,
                          const float *wq, const float *wk, const float *wv, const float *wo,
                          const float *bo, const float *qn, const float *kn,
                          const uint8_t *mask, const float *pos) {
    BoolMask bm(mask, n_tokens);
    manual_attention(out, x, wq, wk, wv, wo, nullptr, nullptr, nullptr, bo, qn, kn,
                     n_tokens, DIT_HIDDEN_SIZE, DIT_NUM_HEADS, DIT_HEAD_SIZE, bm.p, pos);
}

// ffn_mode: ORC_FFN_PER_TOKEN or ORC_FFN_AS_WRITTEN (manual_dit_block verbatim).
void ref_dit_block(float *out, const float *x, const float *cond, const orc_dit_block *b,
                   int n_tokens, const uint8_t *mask, const float *pos, int ffn_mode) {
    BlockViews bv(b);
    BoolMask bm(mask, n_tokens);
    if (ffn_mode == ORC_FFN_AS_WRITTEN)
        manual_dit_block(x, cond, bv.blk, out, n_tokens, bm.p, pos);
    else
        dit_block_per_token_ffn(x, cond, bv.blk, out, n_tokens, bm.p, pos);
}

// Velocity forward wired like src/e2e_pipeline_v4.cpp:441-478; writes the
// last n_out rows of out_all [L][128].
void ref_dit_velocity(const orc_dit *m, const float *x_in, int L, const float *cond,
                      const uint8_t *mask, const float *pos, int ffn_mode, int n_out, float *out) {
    const int D = DIT_HIDDEN_SIZE;
    BoolMask bm(mask, L);
    std::vector<float> h((size_t)L * D), bo((size_t)L * D);
    for (int ti = 0; ti < L; ti++)
        manual_linear(&h[(size_t)ti * D], x_in + (size_t)ti * D, m->in_w, m->in_b, D, D);
    float *hp = h.data(), *bp = bo.data();
    for (int i = 0; i < m->n_layers; i++) {
        BlockViews bv(&m->blocks[i]);
        if (ffn_mode == ORC_FFN_AS_WRITTEN) manual_dit_block(hp, cond, bv.blk, bp, L, bm.p, pos);
        else dit_block_per_token_ffn(hp, cond, bv.blk, bp, L, bm.p, pos);
        float *tmp = hp; hp = bp; bp = tmp;
    }
    float cs2[1024];
    for (int i = 0; i < D; i++) cs2[i] = cond[i] / (1.0f + expf(-cond[i]));
    std::vector<float> mod_raw(2 * D);
    for (int o = 0; o < 2 * D; o++) {
        float s = m->oada_b ? m->oada_b[o] : 0.0f;
        for (int i = 0; i < D; i++) s += m->oada_w[(size_t)o * D + i] * cs2[i];
        mod_raw[o] = s;
    }
    const float *shift = mod_raw.data(), *scale = shift + D;
    std::vector<float> ln(D), row(VAE_LATENT_DIM);
    for (int ti = L - n_out; ti < L; ti++) {
        manual_layernorm(ln.data(), hp + (size_t)ti * D, D);
        for (int j = 0; j < D; j++) ln[j] = ln[j] * (1.0f + scale[j]) + shift[j];
        manual_linear(out + (size_t)(ti - (L - n_out)) * VAE_LATENT_DIM, ln.data(), m->out_w, m->out_b, D, VAE_LATENT_DIM);
    }
}

}  // extern "C"
