// Thin extern "C" driver around the reference's own BigVGAN decoder
// (src/modules/vocoder/bigvgan_cpp.cpp and lstm.cpp of MaurerAnton/dots.tts.cpp),
// compiled in place from the reference tree by oracle/Makefile into
// oracle/_ref/libdtts_ref.so.
//
// TEST INFRASTRUCTURE ONLY: tests/ use it to pin the C restatement
// (voc_oracle.c) and as the CPU timing baseline of the vocoder.  It copies
// plain arrays into the reference's BigVGANDecoder (include/bigvgan_cpp.h) and
// calls bigvgan_decode (bigvgan_cpp.cpp:325).  The decoder prints progress
// lines and writes three small debug dumps under /tmp (bigvgan_cpp.cpp:447,
// :455, :489), as it does in the reference.
#include "bigvgan_cpp.h"
#include "safetensors.h"
#include <cstring>

// bigvgan_load references these; the driver never opens a file.
bool SafeTensorsFile::open(const char *) { return false; }
void SafeTensorsFile::close() {}

namespace {
void put(BigVGANTensor &t, const float *p, size_t n, int n0, int n1 = 1, int n2 = 1) {
    t.n0 = n0; t.n1 = n1; t.n2 = n2;
    if (p) t.data.assign(p, p + n); else t.data.clear();
}
}  // namespace

extern "C" {

// The same weight struct as oracle.h's orc_voc (field for field).
typedef struct {
    const float *post_proj_w, *post_proj_b, *mi_w1, *mi_b1, *mi_w2, *mi_b2;
    const float *lstm_w_ih[4], *lstm_w_hh[4], *lstm_b_ih[4], *lstm_b_hh[4];
    const float *conv_pre_w, *conv_pre_b;
    const float *ups_w[6], *ups_b[6];
    const float *c1_w[18][3], *c1_b[18][3], *c2_w[18][3], *c2_b[18][3];
    const float *alpha[18][6], *beta[18][6];
    const float *post_alpha, *post_beta, *post_filt_up, *post_filt_down;
    const float *conv_post_w;
} ref_voc;

// audio [n_frames * 1920]; returns the sample count bigvgan_decode reports.
int ref_voc_decode(const ref_voc *w, const float *latent, int n_frames, float *audio) {
    static const int up_in[6] = {1536, 768, 384, 192, 96, 48}, up_out[6] = {768, 384, 192, 96, 48, 24};
    static const int up_s[6] = {10, 6, 4, 2, 2, 2}, up_k[6] = {20, 12, 8, 4, 4, 4}, rb_k[3] = {3, 7, 11};
    BigVGANDecoder d;
    put(d.conv_pre_w, w->conv_pre_w, (size_t)1536 * 128 * 5, 1536, 128, 5);
    put(d.conv_pre_b, w->conv_pre_b, 1536, 1536);
    for (int s = 0; s < 6; s++) {
        put(d.ups_w[s], w->ups_w[s], (size_t)up_in[s] * up_out[s] * up_k[s], up_in[s], up_out[s], up_k[s]);
        put(d.ups_b[s], w->ups_b[s], up_out[s], up_out[s]);
        d.ups_in[s] = up_in[s]; d.ups_out[s] = up_out[s]; d.ups_stride[s] = up_s[s]; d.ups_kernel[s] = up_k[s];
    }
    for (int rb = 0; rb < 18; rb++) {
        const int ch = up_out[rb / 3], K = rb_k[rb % 3];
        for (int j = 0; j < 3; j++) {
            put(d.rb_conv1_w[rb][j], w->c1_w[rb][j], (size_t)ch * ch * K, ch, ch, K);
            put(d.rb_conv1_b[rb][j], w->c1_b[rb][j], ch, ch);
            put(d.rb_conv2_w[rb][j], w->c2_w[rb][j], (size_t)ch * ch * K, ch, ch, K);
            put(d.rb_conv2_b[rb][j], w->c2_b[rb][j], ch, ch);
        }
        for (int a = 0; a < 6; a++) {
            put(d.rb_alpha[rb][a], w->alpha[rb][a], ch, ch);
            put(d.rb_beta[rb][a], w->beta[rb][a], ch, ch);
        }
    }
    put(d.conv_post_w, w->conv_post_w, 24 * 7, 1, 24, 7);
    put(d.act_post_alpha, w->post_alpha, 24, 24);
    put(d.act_post_beta, w->post_beta, 24, 24);
    put(d.act_post_filter_up, w->post_filt_up, 24 * 12, 24, 1, 12);
    put(d.act_post_filter_down, w->post_filt_down, 24 * 12, 24, 1, 12);
    put(d.post_proj_w, w->post_proj_w, 128 * 128, 128, 128, 1);
    put(d.post_proj_b, w->post_proj_b, 128, 128);
    put(d.mi_w1, w->mi_w1, 512 * 128, 512, 128);
    put(d.mi_b1, w->mi_b1, 512, 512);
    put(d.mi_w2, w->mi_w2, 128 * 512, 128, 512);
    put(d.mi_b2, w->mi_b2, 128, 128);
    for (int l = 0; l < 4; l++) {
        put(d.mi_lstm_w_ih[l], w->lstm_w_ih[l], 2048 * 512, 2048, 512);
        put(d.mi_lstm_w_hh[l], w->lstm_w_hh[l], 2048 * 512, 2048, 512);
        put(d.mi_lstm_b_ih[l], w->lstm_b_ih[l], 2048, 2048);
        put(d.mi_lstm_b_hh[l], w->lstm_b_hh[l], 2048, 2048);
    }
    int n_samples = 0;
    bigvgan_decode(d, latent, n_frames, audio, &n_samples);
    bigvgan_free(d);
    return n_samples;
}

}  // extern "C"
