// Drop-in definitions of the reference's BigVGAN vocoder entry points on top of
// the B200 engine (libdtts.so, include/dtts.h).
//
// Compile this file into a program built against the reference's headers
// (MaurerAnton/dots.tts.cpp include/: bigvgan_cpp.h, safetensors.h) in place of
// src/modules/vocoder/bigvgan_cpp.cpp and lstm.cpp, and link libdtts.so.  It
// replaces:
//   bigvgan_load    include/bigvgan_cpp.h:42 (bigvgan_cpp.cpp:209): the checkpoint's tensors into
//                   the BigVGANDecoder struct, read with this library's safetensors reader
//   bigvgan_decode  include/bigvgan_cpp.h:43 (bigvgan_cpp.cpp:325): one dtts_voc engine per
//                   decoder struct, created on the first call from the struct's tensors
//   bigvgan_free    include/bigvgan_cpp.h:45 (bigvgan_cpp.cpp:320): releases the engine and the buffers
// Weights are uploaded on the first decode and must not change afterwards.
#include "bigvgan_cpp.h"
#include "dtts.h"

#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <string>

namespace {

std::mutex g_mu;
struct Engine { dtts_voc *voc; int max_frames; };
std::map<const BigVGANDecoder *, Engine> g_voc;

const float *ptr(const BigVGANTensor &t) { return t.data.empty() ? nullptr : t.data.data(); }

bool read_tensor(dtts_st *f, const std::string &name, BigVGANTensor &t) {
    t.data.clear();
    t.n0 = t.n1 = t.n2 = 1;
    int nd = 0;
    int64_t sh[8] = {0};
    if (dtts_st_shape(f, name.c_str(), &nd, sh) != DTTS_OK || nd < 1 || nd > 3) return false;
    size_t n = 1;
    for (int i = 0; i < nd; i++) n *= (size_t)sh[i];
    t.n0 = (int)sh[0];
    t.n1 = nd > 1 ? (int)sh[1] : 1;
    t.n2 = nd > 2 ? (int)sh[2] : 1;
    t.data.resize(n);
    if (dtts_st_read_f32(f, name.c_str(), t.data.data(), n) != DTTS_OK) { t.data.clear(); return false; }
    return true;
}

dtts_voc_weights weights_of(const BigVGANDecoder &d) {
    dtts_voc_weights w = {};
    w.post_proj_w = ptr(d.post_proj_w); w.post_proj_b = ptr(d.post_proj_b);
    w.mi_w1 = ptr(d.mi_w1); w.mi_b1 = ptr(d.mi_b1); w.mi_w2 = ptr(d.mi_w2); w.mi_b2 = ptr(d.mi_b2);
    for (int l = 0; l < 4; l++) {
        w.lstm_w_ih[l] = ptr(d.mi_lstm_w_ih[l]); w.lstm_w_hh[l] = ptr(d.mi_lstm_w_hh[l]);
        w.lstm_b_ih[l] = ptr(d.mi_lstm_b_ih[l]); w.lstm_b_hh[l] = ptr(d.mi_lstm_b_hh[l]);
    }
    w.conv_pre_w = ptr(d.conv_pre_w); w.conv_pre_b = ptr(d.conv_pre_b);
    for (int s = 0; s < 6; s++) { w.ups_w[s] = ptr(d.ups_w[s]); w.ups_b[s] = ptr(d.ups_b[s]); }
    for (int r = 0; r < 18; r++) {
        for (int j = 0; j < 3; j++) {
            w.c1_w[r][j] = ptr(d.rb_conv1_w[r][j]); w.c1_b[r][j] = ptr(d.rb_conv1_b[r][j]);
            w.c2_w[r][j] = ptr(d.rb_conv2_w[r][j]); w.c2_b[r][j] = ptr(d.rb_conv2_b[r][j]);
        }
        for (int a = 0; a < 6; a++) { w.alpha[r][a] = ptr(d.rb_alpha[r][a]); w.beta[r][a] = ptr(d.rb_beta[r][a]); }
    }
    w.post_alpha = ptr(d.act_post_alpha); w.post_beta = ptr(d.act_post_beta);
    w.post_filt_up = ptr(d.act_post_filter_up); w.post_filt_down = ptr(d.act_post_filter_down);
    w.conv_post_w = ptr(d.conv_post_w);
    return w;
}

}  // namespace

bool bigvgan_load(const char *sf_path, BigVGANDecoder &dec) {
    dtts_st *f = nullptr;
    if (dtts_st_open(sf_path, &f) != DTTS_OK) {
        fprintf(stderr, "bigvgan_load: %s\n", dtts_last_error());
        return false;
    }
    static const int up_in[6] = {1536, 768, 384, 192, 96, 48}, up_out[6] = {768, 384, 192, 96, 48, 24};
    static const int up_s[6] = {10, 6, 4, 2, 2, 2}, up_k[6] = {20, 12, 8, 4, 4, 4};
    int loaded = 0;
    auto rd = [&](const std::string &n, BigVGANTensor &t) { loaded += read_tensor(f, n, t) ? 1 : 0; };
    rd("decoder.conv_pre.weight", dec.conv_pre_w);
    rd("decoder.conv_pre.bias", dec.conv_pre_b);
    for (int s = 0; s < 6; s++) {
        rd("decoder.ups." + std::to_string(s) + ".0.weight", dec.ups_w[s]);
        rd("decoder.ups." + std::to_string(s) + ".0.bias", dec.ups_b[s]);
        dec.ups_in[s] = up_in[s]; dec.ups_out[s] = up_out[s]; dec.ups_stride[s] = up_s[s]; dec.ups_kernel[s] = up_k[s];
    }
    for (int r = 0; r < 18; r++) {
        const std::string p = "decoder.resblocks." + std::to_string(r) + ".";
        for (int j = 0; j < 3; j++) {
            const std::string js = std::to_string(j);
            rd(p + "convs1." + js + ".weight", dec.rb_conv1_w[r][j]);
            rd(p + "convs1." + js + ".bias", dec.rb_conv1_b[r][j]);
            rd(p + "convs2." + js + ".weight", dec.rb_conv2_w[r][j]);
            rd(p + "convs2." + js + ".bias", dec.rb_conv2_b[r][j]);
        }
        for (int a = 0; a < 6; a++) {
            rd(p + "activations." + std::to_string(a) + ".act.alpha", dec.rb_alpha[r][a]);
            rd(p + "activations." + std::to_string(a) + ".act.beta", dec.rb_beta[r][a]);
        }
    }
    rd("decoder.conv_post.weight", dec.conv_post_w);
    rd("decoder.activation_post.act.alpha", dec.act_post_alpha);
    rd("decoder.activation_post.act.beta", dec.act_post_beta);
    rd("decoder.activation_post.upsample.filter", dec.act_post_filter_up);
    rd("decoder.activation_post.downsample.lowpass.filter", dec.act_post_filter_down);
    rd("post_proj.weight", dec.post_proj_w);
    rd("post_proj.bias", dec.post_proj_b);
    rd("dec_mi_layer.0.weight", dec.mi_w1);
    rd("dec_mi_layer.0.bias", dec.mi_b1);
    rd("dec_mi_layer.2.weight", dec.mi_w2);
    rd("dec_mi_layer.2.bias", dec.mi_b2);
    for (int l = 0; l < 4; l++) {
        const std::string ls = std::to_string(l);
        rd("dec_mi_layer.1.lstm.weight_ih_l" + ls, dec.mi_lstm_w_ih[l]);
        rd("dec_mi_layer.1.lstm.weight_hh_l" + ls, dec.mi_lstm_w_hh[l]);
        rd("dec_mi_layer.1.lstm.bias_ih_l" + ls, dec.mi_lstm_b_ih[l]);
        rd("dec_mi_layer.1.lstm.bias_hh_l" + ls, dec.mi_lstm_b_hh[l]);
    }
    dtts_st_close(f);
    return loaded > 10;   // the reference's acceptance rule (bigvgan_cpp.cpp:317)
}

bool bigvgan_decode(BigVGANDecoder &dec, const float *latent, int n_frames, float *audio_out, int *n_samples) {
    if (!latent || !audio_out || n_frames < 1) return false;
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_voc.find(&dec);
    if (it != g_voc.end() && it->second.max_frames < n_frames) {
        dtts_voc_destroy(it->second.voc);
        g_voc.erase(it);
        it = g_voc.end();
    }
    if (it == g_voc.end()) {
        const int cap = n_frames > 256 ? n_frames : 256;
        const dtts_voc_weights w = weights_of(dec);
        dtts_voc *v = nullptr;
        const int st = dtts_voc_create(&w, 0, cap, &v);
        if (st != DTTS_OK) {
            fprintf(stderr, "bigvgan_decode: dtts_voc_create: %s (%s)\n", dtts_status_string(st), dtts_last_error());
            return false;
        }
        it = g_voc.emplace(&dec, Engine{v, cap}).first;
    }
    const int st = dtts_voc_decode(it->second.voc, latent, n_frames, audio_out, DTTS_MEM_HOST);
    if (st != DTTS_OK) {
        fprintf(stderr, "bigvgan_decode: %s (%s)\n", dtts_status_string(st), dtts_last_error());
        return false;
    }
    if (n_samples) *n_samples = n_frames * 1920;
    return true;
}

void bigvgan_free(BigVGANDecoder &dec) {
    {
        std::lock_guard<std::mutex> lock(g_mu);
        auto it = g_voc.find(&dec);
        if (it != g_voc.end()) {
            dtts_voc_destroy(it->second.voc);
            g_voc.erase(it);
        }
    }
    dec.buf1.clear(); dec.buf2.clear(); dec.buf3.clear();
}
