// Thin extern "C" driver around the reference's own Qwen2 LLM step
// (src/llm_manual.cpp of MaurerAnton/dots.tts.cpp), compiled in place from the
// reference tree by oracle/Makefile into oracle/_ref/libdtts_ref.so.
//
// TEST INFRASTRUCTURE ONLY: tests/ use it as the checker of the device LLM
// step.  It marshals plain arrays into the reference's LLMWeights and calls
//   llm_kv_cache_init   src/llm_manual.cpp:237 (prompt, fills the KV cache)
//   llm_kv_cache_step   src/llm_manual.cpp:342 (one embedding per call)
// The prompt's embeddings stand in for the embedding table: row t of
// prompt_emb is token t.
#include "llm_manual.h"
#include "safetensors.h"
#include <cstring>
#include <vector>

// llm_manual.cpp's loader references these two members; the driver never
// loads a file, so they only satisfy the linker.
const st_tensor_info *SafeTensorsFile::find(const char *) const { return nullptr; }
bool SafeTensorsFile::load_raw(const st_tensor_info &, float *, size_t) { return false; }

extern "C" {

typedef struct {
    const float *an, *fn, *qw, *qb, *kw, *kb, *vw, *vb, *ow, *ob, *gw, *uw, *dw;
} ref_llm_layer;

// prompt_hidden [n_tok][1536] (final-normed hidden of every prompt token),
// step_hidden [n_steps][1536] (one per step_emb row).
void ref_llm_run(int n_layers, const ref_llm_layer *layers, const float *final_norm, const float *prompt_emb,
                 int n_tok, const float *step_emb, int n_steps, float *prompt_hidden, float *step_hidden) {
    std::vector<LLMWeights::Layer> L(n_layers);
    for (int i = 0; i < n_layers; i++) {
        const ref_llm_layer &s = layers[i];
        LLMWeights::Layer &d = L[i];
        d.an = const_cast<float *>(s.an); d.fn = const_cast<float *>(s.fn);
        d.qw = const_cast<float *>(s.qw); d.qb = const_cast<float *>(s.qb);
        d.kw = const_cast<float *>(s.kw); d.kb = const_cast<float *>(s.kb);
        d.vw = const_cast<float *>(s.vw); d.vb = const_cast<float *>(s.vb);
        d.ow = const_cast<float *>(s.ow); d.ob = const_cast<float *>(s.ob);
        d.gw = const_cast<float *>(s.gw); d.uw = const_cast<float *>(s.uw);
        d.dw = const_cast<float *>(s.dw);
    }
    LLMWeights w;
    w.embed_w = const_cast<float *>(prompt_emb);
    w.layers = L.data();
    w.final_norm = const_cast<float *>(final_norm);
    w.n_layers = n_layers;
    std::vector<int> ids(n_tok);
    for (int t = 0; t < n_tok; t++) ids[t] = t;
    LLMKVCache cache;
    std::memset(&cache, 0, sizeof(cache));
    llm_kv_cache_init(w, ids.data(), n_tok, prompt_hidden, cache);
    for (int s = 0; s < n_steps; s++) llm_kv_cache_step(w, step_emb + (size_t)s * 1536, cache, step_hidden + (size_t)s * 1536);
    llm_kv_cache_free(cache);
}

}  // extern "C"
