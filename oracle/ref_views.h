// Views of the oracle's plain weight arrays as the reference's structs
// (dit_block over ggml_tensor, bool masks), shared by ref_driver.cpp and
// ref_pipeline.cpp.  TEST INFRASTRUCTURE ONLY.
#pragma once
#include "dit_manual.h"
#include "oracle.h"
#include <cstdint>

// A contiguous fp32 ggml_tensor header over a caller-owned array: ne0 x ne1
// (ggml order: ne0 fastest, i.e. [ne1][ne0] row-major).  The DiT math reads
// only the data pointer; the PatchEncoder's operators also read the shape.
struct TensorView {
    ggml_tensor t;
    explicit TensorView(const float *p, int64_t ne0 = 0, int64_t ne1 = 1) {
        t.type = GGML_TYPE_F32;
        t.ne[0] = ne0; t.ne[1] = ne1; t.ne[2] = t.ne[3] = 1;
        t.nb[0] = sizeof(float);
        for (int i = 1; i < 4; i++) t.nb[i] = t.nb[i - 1] * (size_t)t.ne[i - 1];
        t.data = const_cast<float *>(p);
        t.view_offs = 0;
    }
};

struct BlockViews {
    TensorView q, k, v, o, ob, qn, kn, w1, b1, w2, b2, aw, ab;
    dit_block blk;
    explicit BlockViews(const orc_dit_block *b)
        : q(b->wq), k(b->wk), v(b->wv), o(b->wo), ob(b->bo), qn(b->qn), kn(b->kn),
          w1(b->w1), b1(b->b1), w2(b->w2), b2(b->b2), aw(b->ada_w), ab(b->ada_b) {
        blk.attn_q_weight = &q.t; blk.attn_k_weight = &k.t; blk.attn_v_weight = &v.t;
        blk.attn_o_weight = &o.t; blk.attn_o_bias = b->bo ? &ob.t : nullptr;
        blk.q_norm_w = b->qn ? &qn.t : nullptr; blk.k_norm_w = b->kn ? &kn.t : nullptr;
        blk.ffn_w1 = &w1.t; blk.ffn_b1 = b->b1 ? &b1.t : nullptr;
        blk.ffn_w2 = &w2.t; blk.ffn_b2 = b->b2 ? &b2.t : nullptr;
        blk.adaln_linear_w = &aw.t; blk.adaln_linear_b = b->ada_b ? &ab.t : nullptr;
        blk.attn_norm_w = nullptr; blk.ffn_norm_w = nullptr;
    }
};

// The reference takes a plain bool array for the mask.
struct BoolMask {
    bool *p = nullptr;
    BoolMask(const uint8_t *mask, int L) {
        if (mask) { p = new bool[(size_t)L * L]; for (size_t i = 0; i < (size_t)L * L; i++) p[i] = mask[i] != 0; }
    }
    ~BoolMask() { delete[] p; }
};

// manual_dit_block (include/dit_manual.h:148-199) with the FFN applied to
// every token; defined in ref_driver.cpp.
void dit_block_per_token_ffn(const float *x_in, const float *cond, const dit_block &block,
                             float *out, int n_tokens, const bool *attn_mask, const float *pos_ids);
