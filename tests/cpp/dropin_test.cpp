// Drives the drop-in definitions (dots.tts.cpp_b200/dropin/dtts_dropin.cpp)
// exactly as a reference program would: ggml_tensor views over host weights,
// the reference's structs (dit_model, dit_block, patch_encoder) and its
// function names.  tests/test_gpu_dropin.py writes the weights and inputs,
// runs this program and checks every output against the oracle.
//
//   dropin_test WEIGHTS.safetensors IN.bin OUT.bin L_ATT L_RAW N_PATCHES
//
// IN.bin  (float32, in order): x [L_ATT][1024], mask [L_ATT][L_ATT] (0/1),
//         pos [L_ATT], cond [1024], x_raw [L_RAW][1024], t, spk [512],
//         frames [4*N_PATCHES][128]
// OUT.bin (float32, in order): attention with mask+pos [L_ATT][1024],
//         attention with the default arguments [L_ATT][1024],
//         block 1 (block 0 (x)) with mask+pos [L_ATT][1024], block 0 (x)
//         again (engine reuse) [L_ATT][1024], dit_forward_raw [L_RAW][128],
//         patchenc_forward [N][1536], patchenc_decode_step per patch [N][1536],
//         host helpers: layernorm(x0) [1024], rms_norm(x0, q_norm gain) [64],
//         linear(x0, out_proj) [128], softmax(pos) [L_ATT], rope q,k [L_ATT][64] x 2
#include "dit.h"
#include "dit_manual.h"
#include "dots_tts_util.h"
#include "dtts.h"
#include "patchenc.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <string>
#include <vector>

struct ggml_context {
    std::deque<ggml_tensor> tensors;
    std::deque<std::vector<float>> data;
};

ggml_tensor *ggml_new_tensor_2d(ggml_context *ctx, ggml_type type, int64_t ne0, int64_t ne1) {
    ctx->data.emplace_back((size_t)(ne0 * ne1), 0.0f);
    ggml_tensor t{};
    t.type = type;
    t.ne[0] = ne0; t.ne[1] = ne1; t.ne[2] = 1; t.ne[3] = 1;
    t.data = ctx->data.back().data();
    ctx->tensors.push_back(t);
    return &ctx->tensors.back();
}

namespace {

struct Weights {
    dtts_st *f = nullptr;
    ggml_context ctx;
    ggml_tensor *get(const std::string &name) {
        int ndim = 0;
        int64_t shape[8];
        if (dtts_st_shape(f, name.c_str(), &ndim, shape) != DTTS_OK) {
            fprintf(stderr, "missing tensor %s\n", name.c_str());
            exit(2);
        }
        int64_t n = 1;
        for (int i = 0; i < ndim; i++) n *= shape[i];
        ggml_tensor *t = ggml_new_tensor_2d(&ctx, GGML_TYPE_F32, n, 1);
        if (dtts_st_read_f32(f, name.c_str(), tensor_data(t), (size_t)n) != DTTS_OK) {
            fprintf(stderr, "cannot read %s\n", name.c_str());
            exit(2);
        }
        return t;
    }
};

std::vector<float> take(const std::vector<float> &in, size_t &off, size_t n) {
    if (off + n > in.size()) {
        fprintf(stderr, "input file too short\n");
        exit(2);
    }
    std::vector<float> v(in.begin() + off, in.begin() + off + n);
    off += n;
    return v;
}

}  // namespace

int main(int argc, char **argv) {
    if (argc != 7) {
        fprintf(stderr, "usage: %s WEIGHTS IN OUT L_ATT L_RAW N_PATCHES\n", argv[0]);
        return 2;
    }
    const int La = atoi(argv[4]), Lr = atoi(argv[5]), NP = atoi(argv[6]);
    Weights W;
    if (dtts_st_open(argv[1], &W.f) != DTTS_OK) {
        fprintf(stderr, "cannot open %s: %s\n", argv[1], dtts_last_error());
        return 2;
    }

    // ---- the reference's structs over ggml_tensor views
    dit_model dit;
    dit.n_layers = 2;
    dit.layers.resize(2);
    for (int i = 0; i < 2; i++) {
        const std::string p = "velocity_field_predictor.blocks." + std::to_string(i) + ".";
        dit_block &b = dit.layers[i];
        std::memset(&b, 0, sizeof(b));
        b.attn_q_weight = W.get(p + "attn.q_proj.weight");
        b.attn_k_weight = W.get(p + "attn.k_proj.weight");
        b.attn_v_weight = W.get(p + "attn.v_proj.weight");
        b.attn_o_weight = W.get(p + "attn.o_proj.weight");
        b.attn_o_bias = W.get(p + "attn.o_proj.bias");
        b.q_norm_w = W.get(p + "attn.q_norm.weight");
        b.k_norm_w = W.get(p + "attn.k_norm.weight");
        b.ffn_w1 = W.get(p + "ffn.fc1.weight");
        b.ffn_b1 = W.get(p + "ffn.fc1.bias");
        b.ffn_w2 = W.get(p + "ffn.fc2.weight");
        b.ffn_b2 = W.get(p + "ffn.fc2.bias");
        b.adaln_linear_w = W.get(p + "adaLN_modulation.1.weight");
        b.adaln_linear_b = W.get(p + "adaLN_modulation.1.bias");
    }
    const std::string v = "velocity_field_predictor.";
    dit.t_embed_w1 = W.get(v + "time_embedder.mlp.0.weight");
    dit.t_embed_b1 = W.get(v + "time_embedder.mlp.0.bias");
    dit.t_embed_w2 = W.get(v + "time_embedder.mlp.2.weight");
    dit.t_embed_b2 = W.get(v + "time_embedder.mlp.2.bias");
    dit.spk_proj_w1 = W.get("xvec_proj.0.weight");
    dit.spk_proj_b1 = W.get("xvec_proj.0.bias");
    dit.spk_ln_w = W.get("xvec_proj.1.weight");
    dit.spk_ln_b = W.get("xvec_proj.1.bias");
    dit.out_adaln_w = W.get(v + "output_layer.adaLN_modulation.1.weight");
    dit.out_adaln_b = W.get(v + "output_layer.adaLN_modulation.1.bias");
    dit.out_proj_w = W.get(v + "output_layer.linear.weight");
    dit.out_proj_b = W.get(v + "output_layer.linear.bias");
    dit.input_layer_w = W.get(v + "input_layer.weight");
    dit.input_layer_b = W.get(v + "input_layer.bias");
    dit.hidden_proj_w = nullptr;
    dit.latent_proj_w = nullptr;
    dit.coord_proj_w = nullptr;
    dit.hidden_proj_b = dit.latent_proj_b = dit.coord_proj_b = nullptr;
    dit.eos_proj_w1 = dit.eos_proj_b1 = dit.eos_proj_w2 = dit.eos_proj_b2 = nullptr;

    patch_encoder enc;
    enc.n_layers = 2;
    enc.layers.resize(2);
    for (int i = 0; i < 2; i++) {
        const std::string p = "patch_encoder.encoder.layers." + std::to_string(i) + ".";
        patchenc_layer &l = enc.layers[i];
        std::memset(&l, 0, sizeof(l));
        l.attn_q_weight = W.get(p + "attn.q_proj.weight");
        l.attn_k_weight = W.get(p + "attn.k_proj.weight");
        l.attn_v_weight = W.get(p + "attn.v_proj.weight");
        l.attn_o_weight = W.get(p + "attn.o_proj.weight");
        l.attn_o_bias = W.get(p + "attn.o_proj.bias");
        l.attn_norm_w = W.get(p + "attn_norm.weight");
        l.ffn_norm_w = W.get(p + "ffn_norm.weight");
        l.ffn_w1 = W.get(p + "ffn.fc1.weight");
        l.ffn_b1 = W.get(p + "ffn.fc1.bias");
        l.ffn_w2 = W.get(p + "ffn.fc2.weight");
        l.ffn_b2 = W.get(p + "ffn.fc2.bias");
    }
    enc.conv_weight = W.get("patch_encoder.ds_proj.weight");
    enc.conv_bias = W.get("patch_encoder.ds_proj.bias");
    enc.in_proj_w = W.get("patch_encoder.in_proj.weight");
    enc.in_proj_b = W.get("patch_encoder.in_proj.bias");
    enc.out_proj_w = W.get("patch_encoder.out_proj.weight");
    enc.out_proj_b = W.get("patch_encoder.out_proj.bias");
    enc.final_norm_w = nullptr;
    dtts_st_close(W.f);

    // ---- inputs
    std::vector<float> in;
    {
        FILE *fp = fopen(argv[2], "rb");
        if (!fp) { fprintf(stderr, "cannot open %s\n", argv[2]); return 2; }
        fseek(fp, 0, SEEK_END);
        const long sz = ftell(fp);
        fseek(fp, 0, SEEK_SET);
        in.resize((size_t)sz / sizeof(float));
        if (fread(in.data(), sizeof(float), in.size(), fp) != in.size()) { fclose(fp); return 2; }
        fclose(fp);
    }
    size_t off = 0;
    const std::vector<float> x = take(in, off, (size_t)La * 1024);
    const std::vector<float> maskf = take(in, off, (size_t)La * La);
    const std::vector<float> pos = take(in, off, (size_t)La);
    const std::vector<float> cond = take(in, off, 1024);
    const std::vector<float> x_raw = take(in, off, (size_t)Lr * 1024);
    const float t_val = take(in, off, 1)[0];
    const std::vector<float> spk = take(in, off, 512);
    std::vector<float> frames = take(in, off, (size_t)4 * NP * 128);
    std::unique_ptr<bool[]> mask(new bool[(size_t)La * La]);
    for (size_t i = 0; i < (size_t)La * La; i++) mask[i] = maskf[i] != 0.0f;

    std::vector<float> out;
    auto emit = [&](const float *p, size_t n) { out.insert(out.end(), p, p + n); };
    std::vector<float> buf((size_t)La * 1024), buf2((size_t)La * 1024);

    // ---- manual_attention (block 0 weights), with and without mask/positions
    const dit_block &b0 = dit.layers[0];
    const dit_block &b1 = dit.layers[1];
    manual_attention(buf.data(), x.data(), tensor_data(b0.attn_q_weight), tensor_data(b0.attn_k_weight),
                     tensor_data(b0.attn_v_weight), tensor_data(b0.attn_o_weight), nullptr, nullptr, nullptr,
                     tensor_data(b0.attn_o_bias), tensor_data(b0.q_norm_w), tensor_data(b0.k_norm_w), La, 1024, 16, 64,
                     mask.get(), pos.data());
    emit(buf.data(), buf.size());
    manual_attention(buf.data(), x.data(), tensor_data(b0.attn_q_weight), tensor_data(b0.attn_k_weight),
                     tensor_data(b0.attn_v_weight), tensor_data(b0.attn_o_weight), nullptr, nullptr, nullptr,
                     tensor_data(b0.attn_o_bias), tensor_data(b0.q_norm_w), tensor_data(b0.k_norm_w), La, 1024, 16, 64);
    emit(buf.data(), buf.size());

    // ---- manual_dit_block: block 1 (block 0 (x)), then block 0 again
    manual_dit_block(x.data(), cond.data(), b0, buf.data(), La, mask.get(), pos.data());
    manual_dit_block(buf.data(), cond.data(), b1, buf2.data(), La, mask.get(), pos.data());
    emit(buf2.data(), buf2.size());
    manual_dit_block(x.data(), cond.data(), b0, buf.data(), La, mask.get(), pos.data());
    emit(buf.data(), buf.size());

    // ---- dit_forward_raw
    std::vector<float> raw((size_t)Lr * 128);
    dit_forward_raw(dit, x_raw.data(), Lr, t_val, spk.data(), raw.data());
    emit(raw.data(), raw.size());

    // ---- patchenc_forward, then the stream one patch at a time
    ggml_context ctx;
    ggml_tensor *xt = ggml_new_tensor_2d(&ctx, GGML_TYPE_F32, 128, 4 * NP);
    std::memcpy(tensor_data(xt), frames.data(), frames.size() * sizeof(float));
    ggml_tensor *pe = patchenc_forward(enc, &ctx, xt, NP);
    if (pe->ne[0] != 1536 || pe->ne[1] != NP) { fprintf(stderr, "patchenc_forward shape\n"); return 3; }
    emit(tensor_data(pe), (size_t)NP * 1536);
    patchenc_stream_state *st = patchenc_stream_init(enc);
    std::vector<float> emb(1536);
    for (int p = 0; p < NP; p++) {
        patchenc_decode_step(enc, st, &ctx, frames.data() + (size_t)p * 4 * 128, emb.data());
        emit(emb.data(), emb.size());
    }
    patchenc_stream_free(st);

    // ---- host helpers
    std::vector<float> h(1024);
    manual_layernorm(h.data(), x.data(), 1024);
    emit(h.data(), 1024);
    manual_rms_norm(h.data(), x.data(), tensor_data(b0.q_norm_w), 64);
    emit(h.data(), 64);
    manual_linear(h.data(), x.data(), tensor_data(dit.out_proj_w), tensor_data(dit.out_proj_b), 1024, 128);
    emit(h.data(), 128);
    std::vector<float> sm(pos);
    manual_softmax(sm.data(), La);
    emit(sm.data(), sm.size());
    std::vector<float> q(x.begin(), x.begin() + (size_t)La * 64), k(x.begin() + (size_t)La * 64, x.begin() + (size_t)La * 128);
    manual_rope(q.data(), k.data(), La, 64);
    emit(q.data(), q.size());
    emit(k.data(), k.size());

    dtts_dropin_release();

    FILE *fo = fopen(argv[3], "wb");
    if (!fo) { fprintf(stderr, "cannot write %s\n", argv[3]); return 2; }
    fwrite(out.data(), sizeof(float), out.size(), fo);
    fclose(fo);
    printf("dropin_test: wrote %zu floats\n", out.size());
    return 0;
}
