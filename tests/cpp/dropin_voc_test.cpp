// Drives the vocoder drop-in (dots.tts.cpp_b200/dropin/dtts_dropin_voc.cpp) the
// way the reference's pipelines do (src/e2e_pipeline_v4.cpp:650-653): a
// BigVGANDecoder filled by bigvgan_load from a safetensors checkpoint, then
// bigvgan_decode on the latents, then bigvgan_free.
//   dropin_voc_test WEIGHTS LATENTS(f32 [n][128]) OUT(f32 audio) N_FRAMES
#include "bigvgan_cpp.h"

#include <cstdio>
#include <cstdlib>
#include <vector>

int main(int argc, char **argv) {
    if (argc != 5) {
        fprintf(stderr, "usage: %s WEIGHTS LATENTS OUT N_FRAMES\n", argv[0]);
        return 2;
    }
    const int n = atoi(argv[4]);
    BigVGANDecoder dec;
    if (!bigvgan_load(argv[1], dec)) { fprintf(stderr, "bigvgan_load failed\n"); return 3; }
    std::vector<float> lat((size_t)n * 128), audio((size_t)n * 1920);
    FILE *fp = fopen(argv[2], "rb");
    if (!fp || fread(lat.data(), 4, lat.size(), fp) != lat.size()) { fprintf(stderr, "cannot read latents\n"); return 2; }
    fclose(fp);
    int ns = 0;
    if (!bigvgan_decode(dec, lat.data(), n, audio.data(), &ns) || ns != n * 1920) {
        fprintf(stderr, "bigvgan_decode failed (%d samples)\n", ns);
        return 4;
    }
    // a second call on the same decoder reuses its engine
    std::vector<float> again(audio.size());
    if (!bigvgan_decode(dec, lat.data(), n, again.data(), &ns)) return 4;
    for (size_t i = 0; i < audio.size(); i++)
        if (audio[i] != again[i]) { fprintf(stderr, "second decode differs at %zu\n", i); return 5; }
    bigvgan_free(dec);
    FILE *fo = fopen(argv[3], "wb");
    if (!fo || fwrite(audio.data(), 4, audio.size(), fo) != audio.size()) { fprintf(stderr, "cannot write\n"); return 2; }
    fclose(fo);
    return 0;
}
