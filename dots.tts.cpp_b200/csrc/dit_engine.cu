// DiT flow-matching velocity head on sm_100a, behind the C ABI in dtts.h.
//
// Per velocity forward over `rows` sequences of L tokens (M = rows * L):
//   adaLN GEMM    a = SiLU(c) W_ada^T + b for every block and the output layer
//                 at once (one GEMM, N = 6144 * n_layers + 2048)
//   input GEMM    h = x_in W_in^T + b_in                       (fp32 residual)
//   per block     LN+modulate -> QKV GEMM (+qk-norm, RoPE epilogue) ->
//                 attention -> O GEMM (+gated residual epilogue) ->
//                 LN+modulate -> FFN1 GEMM (+GELU-tanh) -> FFN2 GEMM (+gated residual)
//   output head   LN+modulate + out_proj on the last P tokens of each row
// The Euler solve wraps it: per step the time MLP, the CFG combine, the Euler
// update and the coordinate projection of z into the noise tokens, all on the
// device, and the whole solve is captured once into a CUDA graph.
#include "kernels.cuh"

#include <cstdlib>
#include "runtime.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

using namespace dtts;

namespace {

constexpr int kAdaPerLayer = 6 * kD;
constexpr int kFmMaxPatch = 16;   // latent frames per dtts_fm_append_latents call

// launch kinds of the solve timeline (DTTS_TL_* in include/dtts.h); 0..4 are
// the block-op codes of enqueue_block_op
constexpr int TL_LN = DTTS_TL_LN_MODULATE, TL_GEMM_ADALN = DTTS_TL_GEMM_ADALN, TL_GEMM_INPUT = DTTS_TL_GEMM_INPUT,
              TL_OUT_HEAD = DTTS_TL_OUT_HEAD, TL_EULER = DTTS_TL_CFG_EULER, TL_COND = DTTS_TL_CONDITIONING;
static_assert(DTTS_TL_GEMM_QKV == 0 && DTTS_TL_GEMM_O == 1 && DTTS_TL_GEMM_FFN1 == 2 && DTTS_TL_GEMM_FFN2 == 3 &&
                  DTTS_TL_ATTENTION == 4,
              "timeline kinds 0..4 are the block-op codes");

// Tile configuration of one GEMM: tile width BN, epilogue warps, K splits.
struct GemmTune {
    int bn, nw, ks;
};

// ---------------------------------------------------------------- host tables
// RoPE (cos, sin) per token for the half-split rotation of
// include/dit_manual.h:111-128: theta_d = (1e4^(-2/64))^d advanced by repeated
// multiplication, angle = pos * theta_d, evaluated with the host's cosf/sinf
// exactly as the reference does.
void rope_half_table(const float *pos, int L, std::vector<float2> &tab) {
    tab.resize((size_t)L * 32);
    const float ts = powf(10000.0f, -2.0f / 64.0f);
    for (int t = 0; t < L; t++) {
        const float p = pos ? pos[t] : (float)t;
        float theta = 1.0f;
        for (int d = 0; d < 32; d++) {
            tab[(size_t)t * 32 + d] = make_float2(cosf(p * theta), sinf(p * theta));
            theta *= ts;
        }
    }
}

// (cos, sin) per token for ggml_rope mode 0 (adjacent pairs), the pairing of
// the reference's ggml DiT path (src/modules/backbone/dit_attention.cpp:53-54):
// theta starts at the position and is multiplied by 1e4^(-2/64) per pair.
void rope_adjacent_table(const float *pos, int L, std::vector<float2> &tab) {
    tab.resize((size_t)L * 32);
    const float ts = powf(10000.0f, -2.0f / 64.0f);
    for (int t = 0; t < L; t++) {
        float theta = pos ? (float)(int)pos[t] : (float)t;
        for (int d = 0; d < 32; d++) {
            tab[(size_t)t * 32 + d] = make_float2(cosf(theta), sinf(theta));
            theta *= ts;
        }
    }
}

// Sinusoidal time embedding [cos(t f_i) | sin(t f_i)], f_i = exp(-ln(1e4) i / 128)
// (src/e2e_pipeline_v4.cpp:58-60).
void sinusoid(float t, float *se) {
    for (int i = 0; i < 128; i++) {
        const float f = expf(-logf(10000.0f) * (float)i / 128.0f);
        se[i] = cosf(t * f);
        se[128 + i] = sinf(t * f);
    }
}

// Attention mask of the FM sequence (src/e2e_pipeline_v4.cpp:120-146): causal
// history, the last history block and the latent queries see all history and
// all latents, padding positions only themselves.
void fm_mask(uint8_t *mask, int total, int fm_len, int patch, int hidden_patch) {
    const int latent_start = total - patch;
    const int block_start = fm_len > hidden_patch ? fm_len - hidden_patch : 0;
    std::memset(mask, 0, (size_t)total * total);
    for (int i = 0; i < block_start; i++)
        for (int j = 0; j <= i; j++) mask[(size_t)i * total + j] = 1;
    for (int i = block_start; i < fm_len; i++) {
        for (int j = 0; j < fm_len; j++) mask[(size_t)i * total + j] = 1;
        for (int j = latent_start; j < total; j++) mask[(size_t)i * total + j] = 1;
    }
    for (int i = latent_start; i < total; i++) {
        for (int j = 0; j < fm_len; j++) mask[(size_t)i * total + j] = 1;
        for (int j = latent_start; j < total; j++) mask[(size_t)i * total + j] = 1;
    }
    for (int i = fm_len; i < latent_start; i++) mask[(size_t)i * total + i] = 1;
}

// Position ids (src/e2e_pipeline_v4.cpp:149-155).
void fm_pos(float *pos, int total, int fm_len, int patch) {
    const int latent_start = total - patch;
    for (int i = 0; i < fm_len; i++) pos[i] = (float)i;
    for (int i = latent_start; i < total; i++) pos[i] = (float)(fm_len + i - latent_start);
    for (int i = fm_len; i < latent_start; i++) pos[i] = 0.0f;
}

int upload_f32(DeviceArena &a, const float *h, size_t n, float **out, cudaStream_t s) {
    *out = nullptr;
    if (!h) return DTTS_OK;
    void *d = a.alloc(n * sizeof(float));
    if (!d) { set_error("cudaMalloc of %zu bytes failed", n * sizeof(float)); return DTTS_ERR_OOM; }
    DTTS_CUDA(cudaMemcpyAsync(d, h, n * sizeof(float), cudaMemcpyHostToDevice, s));
    *out = static_cast<float *>(d);
    return DTTS_OK;
}

// Uploads h [rows][cols] as its transpose [cols][rows]; `keep` holds the host
// copy until the stream has been synchronised.
int upload_f32_transposed(DeviceArena &a, const float *h, size_t rows, size_t cols, float **out, cudaStream_t s,
                          std::vector<float> &keep) {
    *out = nullptr;
    if (!h) return DTTS_OK;
    keep.resize(rows * cols);
    for (size_t r = 0; r < rows; r++)
        for (size_t c = 0; c < cols; c++) keep[c * rows + r] = h[r * cols + c];
    return upload_f32(a, keep.data(), keep.size(), out, s);
}

// Uploads the row-concatenation of `parts` (each rows_i x cols fp32) as bf16.
int upload_bf16_concat(DeviceArena &a, const std::vector<std::pair<const float *, size_t>> &parts, size_t cols,
                       bf16 **out, cudaStream_t s) {
    size_t rows = 0;
    for (auto &p : parts) rows += p.second;
    std::vector<uint16_t> tmp(rows * cols);
    size_t r0 = 0;
    for (auto &p : parts) {
        if (p.first) f32_to_bf16_host(p.first, tmp.data() + r0 * cols, p.second * cols);
        else std::memset(tmp.data() + r0 * cols, 0, p.second * cols * 2);
        r0 += p.second;
    }
    void *d = a.alloc(tmp.size() * 2);
    if (!d) { set_error("cudaMalloc of %zu bytes failed", tmp.size() * 2); return DTTS_ERR_OOM; }
    DTTS_CUDA(cudaMemcpyAsync(d, tmp.data(), tmp.size() * 2, cudaMemcpyHostToDevice, s));
    DTTS_CUDA(cudaStreamSynchronize(s));  // tmp goes out of scope
    *out = static_cast<bf16 *>(d);
    return DTTS_OK;
}

GemmOp make_op(const CUtensorMap &ta, const CUtensorMap &tb, int M, int N, int K, int epi, int *err,
               const GemmTune &t) {
    GemmOp op;
    std::memset(&op, 0, sizeof(op));
    op.ta = ta;
    op.tb = tb;
    op.M = M; op.N = N; op.K = K;
    op.bn = t.bn;
    op.nw = t.nw;
    op.epi = epi;
    op.ep.err = err;
    op.ep.tok_per_row = 1;
    op.ep.ksplit = t.ks;
    return op;
}

}  // namespace

struct dtts_dit {
    int device = 0, dtype = DTTS_DTYPE_BF16, num_sms = 148;
    cudaStream_t own_stream = nullptr, stream = nullptr;
    DeviceArena wts, ws;
    int n_layers = 0, n_ada = 0;

    struct Layer {
        bf16 *wqkv = nullptr, *wo = nullptr, *w1 = nullptr, *w2 = nullptr;
        float *bo = nullptr, *b1 = nullptr, *b2 = nullptr, *qn = nullptr, *kn = nullptr;
        CUtensorMap tqkv, to, t1, t2;
        // FP8 path: e4m3 weights with one scale per output channel, and the
        // bounds that size the attention-output and GELU-output scales
        uint8_t *qkv8 = nullptr, *o8 = nullptr, *w18 = nullptr, *w28 = nullptr;
        float *sqkv = nullptr, *so = nullptr, *s1 = nullptr, *s2 = nullptr;
        float vbound = 0.f;    // largest |row| of the dequantised Wv
        float w1n = 0.f;       // largest |row| of the dequantised W1
        float b1max = 0.f;     // largest |b1|
    };
    std::vector<Layer> layers;
    bf16 *w_ada = nullptr, *w_in = nullptr;
    float *b_ada = nullptr, *b_in = nullptr;
    CUtensorMap t_ada, t_in;
    // tile configurations (tunable, see dtts_dit_tune)
    // defaults from a sweep on B200 at 128 CFG rows x L = 64 (8192 tokens); no
    // K split by default, so every result is bit-reproducible (split partials
    // reach the residual in run-dependent order).  The O projection's short
    // mainloop (K = 1024) leaves its epilogue exposed: 8 epilogue warps there
    // (31.0 against 32.9 us in place); FFN2 (K = 4096) is faster with 4.
    GemmTune tu_qkv{256, 8, 1}, tu_o{256, 8, 1}, tu_ffn1{256, 4, 1}, tu_ffn2{256, 4, 1}, tu_ada{256, 8, 1},
        tu_in{256, 4, 1};
    float *t_w1 = nullptr, *t_b1 = nullptr, *t_w2 = nullptr, *t_b2 = nullptr;
    float *spk_w1 = nullptr, *spk_b1 = nullptr, *spk_lw = nullptr, *spk_lb = nullptr;
    // output and coordinate projections stored transposed: out_wt [1024][128], coord_wt [128][1024]
    float *out_wt = nullptr, *out_b = nullptr, *coord_wt = nullptr, *coord_b = nullptr;
    // FM history projections and the EOS head (fp32, dtts_fm_*)
    float *hid_w = nullptr, *hid_b = nullptr, *lat_w = nullptr, *lat_b = nullptr;
    float *eos_w1 = nullptr, *eos_b1 = nullptr, *eos_w2 = nullptr, *eos_b2 = nullptr;
    int *d_err = nullptr;
    bool has_in = false, has_out = false;
    int rope_mode = ROPE_HALF;   // DTTS_ROPE_HALF / DTTS_ROPE_ADJACENT
    void rope_table(const float *pos, int L, std::vector<float2> &tab) const {
        if (rope_mode == ROPE_ADJACENT) rope_adjacent_table(pos, L, tab);
        else rope_half_table(pos, L, tab);
    }

    // workspace
    int cap_tok = 0, cap_rows = 0, cap_L = 0, cap_nfe = 0;
    bf16 *x_in = nullptr, *act = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr,
         *ffn = nullptr, *a_cond = nullptr;
    float *h = nullptr, *ada = nullptr, *vel = nullptr, *temb = nullptr, *h1 = nullptr, *spk_c = nullptr,
          *z = nullptr, *in_a = nullptr, *in_b = nullptr, *cond_f32 = nullptr, *se_tab = nullptr,
          *spk_in = nullptr;
    float2 *rope = nullptr;
    uint8_t *mask = nullptr;
    uint32_t *mask_bits = nullptr;   // [L][ceil(L/32)]
    CUtensorMap t_x_in, t_act, t_att, t_ffn, t_acond, t_h;
    // FP8 path workspace: e4m3 operands and their per-row scales
    uint8_t *act8 = nullptr, *att8 = nullptr, *ffn8 = nullptr;
    float *s_act = nullptr, *s_att = nullptr, *s_ffn = nullptr, *inv_ffn = nullptr, *unorm = nullptr;
    CUtensorMap t_act8, t_att8, t_ffn8;
    // Optionally (DTTS_FUSE_LN=1 or dtts_dit_set_fused_ln) the LayerNorm +
    // modulation after each residual GEMM runs in that GEMM's epilogue
    // (EPI_RESID_GATED_LN): LN2 in the O projection, the next block's LN1 in
    // FFN2.  Needs ksplit 1 and a tile width of 128 or 256.  Both forms give the
    // same bits; the standalone kernels are the default because they are faster
    // on B200 (the GEMM's 4-8 epilogue warps per SM normalise rows at a fraction
    // of the rate of the LayerNorm kernel's 24).
    bool fuse_ln = false;
    bool discard_qkv = true;   // DTTS_L2_DISCARD=0: keep the dead q / k / v lines (see AttnArgs)
    unsigned *ln_cnt = nullptr;   // one arrival counter per 128-token block, zero at rest
    bool ln_fused(const GemmTune &t) const { return fuse_ln && t.ks == 1 && t.bn % 128 == 0; }
    bool fp8() const { return dtype == DTTS_DTYPE_FP8; }

    // shapes of the last forward (for profiling) and launch accounting
    int last_rows = 0, last_L = 0, last_P = 0;
    bool last_mask = false;
    int launches = 0;

    // solve graph
    cudaGraphExec_t gexec = nullptr;
    std::string gkey;

    // launch timeline (dtts_dit_solve_timeline): one timing event before and
    // one after every launch of a captured solve; tl_kind[i] is the kind of
    // launch i, timed by events 2i and 2i+1
    bool tl_on = false;
    std::vector<cudaEvent_t> tl_ev;
    std::vector<int> tl_kind;
    int tl_begin(int kind) {
        const size_t i = tl_kind.size();
        if (2 * i + 1 >= tl_ev.size()) return -1;   // pool exhausted: launch not timed
        cudaEventRecordWithFlags(tl_ev[2 * i], stream, cudaEventRecordExternal);
        tl_kind.push_back(kind);
        return (int)i;
    }
    void tl_end(int i) { cudaEventRecordWithFlags(tl_ev[2 * (size_t)i + 1], stream, cudaEventRecordExternal); }
    struct TlScope {
        dtts_dit *e;
        int idx;
        TlScope(dtts_dit *e_, int kind) : e(e_), idx(e_->tl_on ? e_->tl_begin(kind) : -1) {}
        ~TlScope() { if (idx >= 0) e->tl_end(idx); }
    };

    // the fp32 residual stream h is kept in L2 across the kernels of a forward
    // (DTTS_L2_PERSIST=0 turns it off)
    L2Window l2w;
    bool l2_held = false;

    ~dtts_dit() {
        if (gexec) cudaGraphExecDestroy(gexec);
        if (l2_held) l2_persist_release(device);
        ws.free_all();
        wts.free_all();
        if (own_stream) cudaStreamDestroy(own_stream);
        for (cudaEvent_t ev : tl_ev) cudaEventDestroy(ev);
    }

    int ensure_workspace(int rows, int L, int nfe);
    int build_weight_maps();
    // Every kernel of a forward is launched with programmatic stream
    // serialization (DTTS_PDL=0 turns it off): a GEMM requests its first weight
    // tiles and every kernel sets up while the kernel before it finishes.
    int gemm(GemmOp op) {
        launches++;
        op.pdl = 1;
        DTTS_CUDA(launch_gemm(op, num_sms, stream));
        return DTTS_OK;
    }
    // modulation source of the current forward: row r of sequence tokens uses
    // ada_cur + (r / rows_per_ada) * n_ada
    const float *ada_cur = nullptr;
    int rows_per_ada = 1;
    int last_ada_rows = 0;
    int enqueue_forward(int rows, int L, int P);
    int enqueue_block_op(int kind, int l, int rows, int L);
    int enqueue_solve(const dtts_solve_args *a);
    int finish(bool host_wait);
};

int dtts_dit::ensure_workspace(int rows, int L, int nfe) {
    const long long tok = (long long)rows * L;
    if (tok <= cap_tok && rows <= cap_rows && L <= cap_L && nfe <= cap_nfe) return DTTS_OK;
    if (gexec) { cudaGraphExecDestroy(gexec); gexec = nullptr; gkey.clear(); }
    DTTS_CUDA(cudaStreamSynchronize(stream));
    ws.free_all();
    cap_tok = (int)std::max<long long>(tok, cap_tok);
    cap_rows = std::max(rows, cap_rows);
    cap_L = std::max(L, cap_L);
    cap_nfe = std::max(std::max(nfe, cap_nfe), 1);
    const size_t T = (size_t)cap_tok, R = (size_t)std::max(cap_rows, 1);
    auto A = [&](size_t bytes) { return ws.alloc(bytes); };
    x_in = (bf16 *)A(T * kD * 2);
    act = (bf16 *)A(T * kD * 2);
    q = (bf16 *)A(T * kD * 2);
    k = (bf16 *)A(T * kD * 2);
    v = (bf16 *)A(T * kD * 2);
    att = (bf16 *)A(T * kD * 2);
    ffn = (bf16 *)A(T * kF * 2);
    h = (float *)A(T * kD * 4);
    in_a = (float *)A(T * kD * 4);
    in_b = (float *)A(T * kD * 4);
    a_cond = (bf16 *)A(R * (size_t)cap_nfe * kD * 2);
    ada = (float *)A(R * (size_t)cap_nfe * n_ada * 4);
    vel = (float *)A(T * kLat * 4);
    z = (float *)A(T * kLat * 4);
    ln_cnt = (unsigned *)A((T / 128 + 1) * sizeof(unsigned));
    cond_f32 = (float *)A(R * kD * 4);
    spk_c = (float *)A(R * kD * 4);
    spk_in = (float *)A(R * kSpk * 4);
    temb = (float *)A((size_t)cap_nfe * kD * 4);
    h1 = (float *)A((size_t)cap_nfe * kD * 4);
    se_tab = (float *)A((size_t)cap_nfe * 256 * 4);
    rope = (float2 *)A((size_t)cap_L * 32 * sizeof(float2));
    mask = (uint8_t *)A((size_t)cap_L * cap_L);
    mask_bits = (uint32_t *)A((size_t)cap_L * ((cap_L + 31) / 32) * 4);
    if (fp8()) {
        act8 = (uint8_t *)A(T * kD);
        att8 = (uint8_t *)A(T * kD);
        ffn8 = (uint8_t *)A(T * kF);
        s_act = (float *)A(T * 4);
        s_att = (float *)A(T * 4);
        s_ffn = (float *)A(T * 4);
        inv_ffn = (float *)A(T * 4);
        unorm = (float *)A(T * 4);
    }
    for (void *p : ws.ptrs)
        if (!p) { set_error("workspace allocation failed (%lld tokens)", tok); cap_tok = cap_rows = cap_L = 0; ws.free_all(); return DTTS_ERR_OOM; }
    DTTS_CUDA(cudaMemsetAsync(ln_cnt, 0, (T / 128 + 1) * sizeof(unsigned), stream));
    bool ok = make_tmap_bf16(&t_x_in, x_in, T, kD, 128) && make_tmap_bf16(&t_act, act, T, kD, 128) &&
              make_tmap_bf16(&t_att, att, T, kD, 128) && make_tmap_bf16(&t_ffn, ffn, T, kF, 128) &&
              make_tmap_bf16(&t_acond, a_cond, R * (size_t)cap_nfe, kD, 128) && make_tmap_f32_resid(&t_h, h, T, kD);
    DTTS_CHECK(ok, DTTS_ERR_CUDA, "cuTensorMapEncodeTiled failed for a workspace buffer");
    if (fp8()) {
        ok = make_tmap_e4m3(&t_act8, act8, T, kD, 128) && make_tmap_e4m3(&t_att8, att8, T, kD, 128) &&
             make_tmap_e4m3(&t_ffn8, ffn8, T, kF, 128);
        DTTS_CHECK(ok, DTTS_ERR_CUDA, "cuTensorMapEncodeTiled failed for an e4m3 workspace buffer");
    }
    // L2 residency of h: a set-aside of h's size (capped by the device) and a
    // window over h whose hit ratio is the fraction of it the set-aside holds.
    // Only while h takes at most 40% of L2: a larger set-aside starves the
    // q/k/v and FFN activations that each kernel hands to the next (at 128 MB
    // of h, 256 utterances x 64 tokens, every block kernel ran 1.3-3x slower).
    l2w = L2Window{};
    static const bool l2_on = [] {
        const char *e = std::getenv("DTTS_L2_PERSIST");
        return !(e && e[0] == '0');
    }();
    int l2_size = 0;
    cudaDeviceGetAttribute(&l2_size, cudaDevAttrL2CacheSize, device);
    cudaGetLastError();
    const bool l2_fits = (double)T * kD * 4 <= 0.4 * (double)l2_size;
    if (l2_held && !l2_fits) { l2_persist_release(device); l2_held = false; }
    if (l2_on && l2_fits) {
        const size_t hb = T * kD * 4;
        int max_win = 0;
        cudaDeviceGetAttribute(&max_win, cudaDevAttrMaxAccessPolicyWindowSize, device);
        cudaGetLastError();
        if (max_win > 0) {
            const size_t granted = l2_persist_acquire(device, hb);
            if (granted > 0) {
                if (l2_held) l2_persist_release(device);   // one reference per engine
                l2_held = true;
                const size_t win = std::min(hb, (size_t)max_win);
                l2w.base = h;
                l2w.bytes = win;
                l2w.hit_ratio = granted >= win ? 1.0f : (float)granted / (float)win;
            }
        }
    }
    return DTTS_OK;
}

// Weight tensor maps: the TMA box height of B is the GEMM's tile width.
int dtts_dit::build_weight_maps() {
    for (int l = 0; l < n_layers; l++) {
        Layer &L = layers[l];
        bool ok;
        if (fp8())
            ok = make_tmap_e4m3(&L.tqkv, L.qkv8, 3 * kD, kD, tu_qkv.bn) &&
                 make_tmap_e4m3(&L.to, L.o8, kD, kD, tu_o.bn) && make_tmap_e4m3(&L.t1, L.w18, kF, kD, tu_ffn1.bn) &&
                 make_tmap_e4m3(&L.t2, L.w28, kD, kF, tu_ffn2.bn);
        else
            ok = make_tmap_bf16(&L.tqkv, L.wqkv, 3 * kD, kD, tu_qkv.bn) &&
                 make_tmap_bf16(&L.to, L.wo, kD, kD, tu_o.bn) && make_tmap_bf16(&L.t1, L.w1, kF, kD, tu_ffn1.bn) &&
                 make_tmap_bf16(&L.t2, L.w2, kD, kF, tu_ffn2.bn);
        DTTS_CHECK(ok, DTTS_ERR_CUDA, "cuTensorMapEncodeTiled failed for block %d", l);
    }
    bool ok = make_tmap_bf16(&t_ada, w_ada, n_ada, kD, tu_ada.bn) && make_tmap_bf16(&t_in, w_in, kD, kD, tu_in.bn);
    DTTS_CHECK(ok, DTTS_ERR_CUDA, "cuTensorMapEncodeTiled failed (adaLN / input_layer)");
    return DTTS_OK;
}

// One launch of a per-block operation (used by the forward and by profiling).
// kind: 0 QKV, 1 O, 2 FFN1, 3 FFN2, 4 attention, 5 LN1, 6 LN2
int dtts_dit::enqueue_block_op(int kind, int l, int rows, int L) {
    const int M = rows * L;
    const Layer &Ly = layers[l];
    const float *ada_l = ada_cur + (long long)l * kAdaPerLayer;
    const int tpr = L * rows_per_ada;   // tokens sharing one modulation row
    // LN2 runs inside the O projection and LN1 of blocks after the first inside
    // the previous block's FFN2 when those are fused
    if ((kind == 6 && ln_fused(tu_o)) || (kind == 5 && l > 0 && ln_fused(tu_ffn2))) return DTTS_OK;
    TlScope tl_scope(this, kind == 6 ? TL_LN : kind);
    switch (kind) {
        case 5:
        case 6: {
            const long long off = kind == 5 ? 0 : 3 * kD;
            launches++;
            if (fp8()) {
                if (kind == 5)
                    launch_ln_modulate_f8(h, act8, M, ada_l + off, ada_l + off + kD, n_ada, tpr, s_act, unorm, nullptr,
                                          nullptr, 0.f, 0.f, stream, true);
                else
                    launch_ln_modulate_f8(h, act8, M, ada_l + off, ada_l + off + kD, n_ada, tpr, s_act, nullptr, s_ffn,
                                          inv_ffn, Ly.w1n, Ly.b1max, stream, true);
                return DTTS_OK;
            }
            launch_ln_modulate(h, act, M, ada_l + off, ada_l + off + kD, n_ada, tpr, stream, true);
            return DTTS_OK;
        }
        case 0: {
            GemmOp op = make_op(fp8() ? t_act8 : t_act, Ly.tqkv, M, 3 * kD, kD, EPI_QKV, d_err, tu_qkv);
            if (fp8()) { op.f8 = 1; op.ep.row_scale = s_act; op.ep.col_scale = Ly.sqkv; }
            op.ep.q = q; op.ep.k = k; op.ep.v = v;
            op.ep.ldq = kD; op.ep.ldkv = kD;
            op.ep.tok_per_row = L; op.ep.kv_cap = L; op.ep.kv_start = 0;
            op.ep.qk_norm = 1; op.ep.qn = Ly.qn; op.ep.kn = Ly.kn;
            op.ep.rope = rope; op.ep.rope_mode = rope_mode;
            return gemm(op);
        }
        case 4: {
            AttnArgs a{};
            a.q = q; a.ldq = kD; a.k = k; a.v = v; a.ldkv = kD; a.o = att; a.ldo = kD;
            a.rows = rows; a.Tq = L; a.kv_len = L; a.kv_cap = L; a.q_pos0 = 0; a.causal = 0;
            a.mask = last_mask ? mask : nullptr;
            a.mask_bits = last_mask ? mask_bits : nullptr;
            a.scale = 1.0f / sqrtf(64.0f);
            a.err = d_err;
            a.discard_qkv = discard_qkv;   // q, k, v are rewritten by the next block's QKV GEMM
            if (fp8()) { a.o8 = att8; a.o_scale = s_att; a.unorm = unorm; a.vbound = Ly.vbound; }
            launches++;
            launch_attention_bf16(a, stream, true);
            return DTTS_OK;
        }
        case 1: {
            GemmOp op = make_op(fp8() ? t_att8 : t_att, Ly.to, M, kD, kD, EPI_RESID_GATED, d_err, tu_o);
            if (fp8()) { op.f8 = 1; op.ep.row_scale = s_att; op.ep.col_scale = Ly.so; }
            op.tr = t_h;
            op.ep.bias = Ly.bo; op.ep.resid = h; op.ep.ldr = kD;
            op.ep.gate = ada_l + 2 * kD; op.ep.gate_ld = n_ada; op.ep.tok_per_row = tpr;
            if (ln_fused(tu_o)) {   // + LN2 of this block
                op.epi = EPI_RESID_GATED_LN;
                op.ep.ln_count = ln_cnt;
                op.ep.ln = ln_params(ada_l + 3 * kD, ada_l + 4 * kD, n_ada, tpr, fp8() ? (void *)act8 : (void *)act);
                if (fp8()) {
                    op.ep.ln.row_scale = s_act; op.ep.ln.g_scale = s_ffn; op.ep.ln.g_inv = inv_ffn;
                    op.ep.ln.w1n = Ly.w1n; op.ep.ln.b1max = Ly.b1max;
                }
            }
            return gemm(op);
        }
        case 2: {
            if (fp8()) {
                GemmOp op = make_op(t_act8, Ly.t1, M, kF, kD, EPI_GELU_F8, d_err, tu_ffn1);
                op.f8 = 1; op.ep.row_scale = s_act; op.ep.col_scale = Ly.s1; op.ep.out_inv = inv_ffn;
                op.ep.bias = Ly.b1; op.ep.out = ffn8; op.ep.ldo = kF;
                return gemm(op);
            }
            GemmOp op = make_op(t_act, Ly.t1, M, kF, kD, EPI_GELU_BF16, d_err, tu_ffn1);
            op.ep.bias = Ly.b1; op.ep.out = ffn; op.ep.ldo = kF;
            return gemm(op);
        }
        case 3: {
            GemmOp op = make_op(fp8() ? t_ffn8 : t_ffn, Ly.t2, M, kD, kF, EPI_RESID_GATED, d_err, tu_ffn2);
            if (fp8()) { op.f8 = 1; op.ep.row_scale = s_ffn; op.ep.col_scale = Ly.s2; }
            op.tr = t_h;
            op.ep.bias = Ly.b2; op.ep.resid = h; op.ep.ldr = kD;
            op.ep.gate = ada_l + 5 * kD; op.ep.gate_ld = n_ada; op.ep.tok_per_row = tpr;
            // bf16: the 8 KB-per-token A (67 MB at 8192 tokens) is then read once from
            // DRAM, not once per N pass (FFN2 73 against 77 us in place); the e4m3 A
            // fits in L2 either way
            op.ep.mb_major = fp8() ? 0 : 1;
            if (l + 1 < n_layers && ln_fused(tu_ffn2)) {   // + LN1 of the next block
                const float *ada_n = ada_l + kAdaPerLayer;
                op.epi = EPI_RESID_GATED_LN;
                op.ep.ln_count = ln_cnt;
                op.ep.ln = ln_params(ada_n, ada_n + kD, n_ada, tpr, fp8() ? (void *)act8 : (void *)act);
                if (fp8()) { op.ep.ln.row_scale = s_act; op.ep.ln.unorm = unorm; }
            }
            return gemm(op);
        }
    }
    set_error("unknown block op %d", kind);
    return DTTS_ERR_ARG;
}

// Expects x_in (bf16), the modulation rows at ada_cur, rope and mask filled.
int dtts_dit::enqueue_forward(int rows, int L, int P) {
    const int M = rows * L;
    last_rows = rows; last_L = L; last_P = P;
    L2WindowScope l2_scope(l2w);
    {   // input layer
        TlScope tl_scope(this, TL_GEMM_INPUT);
        GemmOp op = make_op(t_x_in, t_in, M, kD, kD, EPI_F32, d_err, tu_in);
        op.ep.bias = b_in; op.ep.out = h; op.ep.ldo = kD;
        int st = gemm(op);
        if (st) return st;
    }
    static const int order[7] = {5, 0, 4, 1, 6, 2, 3};
    for (int l = 0; l < n_layers; l++)
        for (int i = 0; i < 7; i++) {
            int st = enqueue_block_op(order[i], l, rows, L);
            if (st) return st;
        }
    const long long oo = (long long)n_layers * kAdaPerLayer;
    launches++;
    TlScope tl_scope(this, TL_OUT_HEAD);
    launch_out_head(h, rows, L, P, ada_cur + oo, ada_cur + oo + kD, n_ada, rows_per_ada, out_wt, out_b, vel, d_err,
                    stream);
    DTTS_CUDA(cudaGetLastError());
    return DTTS_OK;
}

int dtts_dit::enqueue_solve(const dtts_solve_args *a) {
    const int rows = 2 * a->n_utt, L = a->fm_len + a->patch;
    launches += 2;
    {
        TlScope tl_scope(this, TL_COND);
        launch_history_rows(in_a, a->n_utt, a->fm_len, x_in, L, 2, 0, stream);
    }
    {
        TlScope tl_scope(this, TL_COND);
        launch_history_rows(in_b, a->n_utt, a->fm_len, x_in, L, 2, 1, stream);
    }
    if (a->spk) {
        launches++;
        TlScope tl_scope(this, TL_COND);
        launch_speaker_cond(spk_in, a->n_utt, spk_w1, spk_b1, spk_lw, spk_lb, a->spk_scale, spk_c, stream);
    }
    const float dt = 1.0f / (float)a->nfe;
    // Conditioning of every step up front: c depends only on t_k and the
    // speaker, so one adaLN GEMM covers all steps and utterances (cond and
    // uncond rows of an utterance share c).
    launches += 3;
    {
        TlScope tl_scope(this, TL_COND);
        launch_time_mlp(se_tab, a->nfe, t_w1, t_b1, t_w2, t_b2, h1, temb, stream);
    }
    {
        TlScope tl_scope(this, TL_COND);
        launch_cond_rows(temb, a->nfe, a->spk ? spk_c : nullptr, a->n_utt, a_cond, stream);
    }
    {
        TlScope tl_scope(this, TL_GEMM_ADALN);
        GemmOp op = make_op(t_acond, t_ada, a->nfe * a->n_utt, n_ada, kD, EPI_F32, d_err, tu_ada);
        op.ep.bias = b_ada; op.ep.out = ada; op.ep.ldo = n_ada;
        int st = gemm(op);
        if (st) return st;
        last_ada_rows = a->nfe * a->n_utt;
    }
    launches++;
    {
        TlScope tl_scope(this, TL_EULER);
        launch_cfg_euler(vel, z, a->n_utt, a->patch, a->cfg_scale, a->cfg_form, dt, 0, coord_wt, coord_b, x_in, L,
                         stream);
    }
    rows_per_ada = 2;
    for (int step = 0; step < a->nfe; step++) {
        ada_cur = ada + (size_t)step * a->n_utt * n_ada;
        int st = enqueue_forward(rows, L, a->patch);
        if (st) return st;
        launches++;
        TlScope tl_scope(this, TL_EULER);
        launch_cfg_euler(vel, z, a->n_utt, a->patch, a->cfg_scale, a->cfg_form, dt, 1, coord_wt, coord_b, x_in, L,
                         stream);
    }
    DTTS_CUDA(cudaGetLastError());
    return DTTS_OK;
}

int dtts_dit::finish(bool host_wait) {
    if (!host_wait) return DTTS_OK;
    int st = stream_wait(stream, 300.0);
    if (st) return st;
    int err = 0;
    DTTS_CUDA(cudaMemcpy(&err, d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (err) {
        cudaMemset(d_err, 0, sizeof(int));
        // a fused LayerNorm wait that gave up leaves its block counters raised
        if (ln_cnt) cudaMemset(ln_cnt, 0, ((size_t)cap_tok / 128 + 1) * sizeof(unsigned));
        if (err == DEVERR_NONFINITE) { set_error("non-finite velocity"); return DTTS_ERR_NONFINITE; }
        set_error("device wait limit reached (code %d)", err);
        return DTTS_ERR_TIMEOUT;
    }
    return DTTS_OK;
}

// FP8 weights of one block: e4m3 with one scale per output channel (the rows
// of the PyTorch [out][in] matrices), plus the bounds the FP8 forward needs:
// the largest dequantised row norm of Wv and of W1, and max |b1|.
int upload_block_e4m3(DeviceArena &a, const dtts_dit_block_weights &b, dtts_dit::Layer &L, cudaStream_t s) {
    struct Part { const float *w; size_t rows, cols; };
    auto upload = [&](std::initializer_list<Part> parts, uint8_t **dq, float **dsc, float *max_norm_last) -> int {
        size_t rows = 0, cols = parts.begin()->cols;
        for (const Part &p : parts) rows += p.rows;
        std::vector<uint8_t> q(rows * cols);
        std::vector<float> sc(rows), nrm(rows);
        size_t r0 = 0;
        for (const Part &p : parts) {
            e4m3_quantize_rows(p.w, p.rows, p.cols, q.data() + r0 * cols, sc.data() + r0, nrm.data() + r0);
            r0 += p.rows;
        }
        if (max_norm_last) {   // bound over the rows of the last part
            const Part &p = *(parts.end() - 1);
            float m = 0.f;
            for (size_t r = rows - p.rows; r < rows; r++) m = std::max(m, nrm[r]);
            *max_norm_last = m;
        }
        void *d = a.alloc(q.size()), *ds = a.alloc(sc.size() * 4);
        if (!d || !ds) { set_error("cudaMalloc of e4m3 weights failed"); return DTTS_ERR_OOM; }
        DTTS_CUDA(cudaMemcpyAsync(d, q.data(), q.size(), cudaMemcpyHostToDevice, s));
        DTTS_CUDA(cudaMemcpyAsync(ds, sc.data(), sc.size() * 4, cudaMemcpyHostToDevice, s));
        DTTS_CUDA(cudaStreamSynchronize(s));   // host copies go out of scope
        *dq = static_cast<uint8_t *>(d);
        *dsc = static_cast<float *>(ds);
        return DTTS_OK;
    };
    int st;
    if ((st = upload({{b.wq, kD, kD}, {b.wk, kD, kD}, {b.wv, kD, kD}}, &L.qkv8, &L.sqkv, &L.vbound))) return st;
    if ((st = upload({{b.wo, kD, kD}}, &L.o8, &L.so, nullptr))) return st;
    if ((st = upload({{b.w1, kF, kD}}, &L.w18, &L.s1, &L.w1n))) return st;
    if ((st = upload({{b.w2, kD, kF}}, &L.w28, &L.s2, nullptr))) return st;
    L.b1max = 0.f;
    if (b.b1)
        for (int j = 0; j < kF; j++) L.b1max = std::max(L.b1max, std::fabs(b.b1[j]));
    return DTTS_OK;
}

// =========================================================================
// C ABI
// =========================================================================
extern "C" {

int dtts_dit_create(const dtts_dit_weights *w, int dtype, int device, dtts_dit **out) {
    DTTS_CHECK(w && out, DTTS_ERR_ARG, "null argument");
    *out = nullptr;
    DTTS_CHECK(w->n_layers >= 1 && w->n_layers <= 64 && w->blocks, DTTS_ERR_ARG, "n_layers %d invalid", w->n_layers);
    DTTS_CHECK(dtype == DTTS_DTYPE_BF16 || dtype == DTTS_DTYPE_FP8, DTTS_ERR_UNSUPPORTED,
               "DiT dtype %d not supported (bf16 or fp8)", dtype);
    // Global weights are checked by the calls that need them: a model with
    // only blocks serves dtts_dit_blocks (manual_dit_block).
    for (int l = 0; l < w->n_layers; l++) {
        const dtts_dit_block_weights &b = w->blocks[l];
        DTTS_CHECK(b.wq && b.wk && b.wv && b.wo && b.w1 && b.w2 && b.ada_w, DTTS_ERR_ARG,
                   "missing a required weight in block %d", l);
    }
    int nsm = 0;
    int st = check_device(device, &nsm);
    if (st) return st;
    DeviceGuard g(device);
    std::unique_ptr<dtts_dit> e(new dtts_dit());
    e->device = device; e->dtype = dtype; e->num_sms = nsm; e->n_layers = w->n_layers;
    {
        const char *fl = std::getenv("DTTS_FUSE_LN");
        e->fuse_ln = fl && fl[0] == '1';
        const char *dl = std::getenv("DTTS_L2_DISCARD");
        e->discard_qkv = !(dl && dl[0] == '0');
    }
    if (dtype == DTTS_DTYPE_FP8) {
        // e4m3 mainloops take half the time, so the epilogue decides: eight
        // epilogue warps for the FFN1 tiles too (sweep at 8192 tokens)
        e->tu_ffn1 = {256, 8, 1};
    }
    DTTS_CUDA(cudaStreamCreateWithFlags(&e->own_stream, cudaStreamNonBlocking));
    e->stream = e->own_stream;
    DTTS_CUDA(gemm_prepare_attributes());
    DTTS_CUDA(attention_short_prepare());
    cudaStream_t s = e->stream;
    e->d_err = (int *)e->wts.alloc(sizeof(int));
    DTTS_CHECK(e->d_err, DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemsetAsync(e->d_err, 0, sizeof(int), s));

    e->layers.resize(w->n_layers);
    for (int l = 0; l < w->n_layers; l++) {
        const dtts_dit_block_weights &b = w->blocks[l];
        dtts_dit::Layer &L = e->layers[l];
        if (dtype == DTTS_DTYPE_FP8) {
            if ((st = upload_block_e4m3(e->wts, b, L, s))) return st;
        } else {
            if ((st = upload_bf16_concat(e->wts, {{b.wq, kD}, {b.wk, kD}, {b.wv, kD}}, kD, &L.wqkv, s))) return st;
            if ((st = upload_bf16_concat(e->wts, {{b.wo, kD}}, kD, &L.wo, s))) return st;
            if ((st = upload_bf16_concat(e->wts, {{b.w1, kF}}, kD, &L.w1, s))) return st;
            if ((st = upload_bf16_concat(e->wts, {{b.w2, kD}}, kF, &L.w2, s))) return st;
        }
        if ((st = upload_f32(e->wts, b.bo, kD, &L.bo, s))) return st;
        if ((st = upload_f32(e->wts, b.b1, kF, &L.b1, s))) return st;
        if ((st = upload_f32(e->wts, b.b2, kD, &L.b2, s))) return st;
        if ((st = upload_f32(e->wts, b.qn, kHD, &L.qn, s))) return st;
        if ((st = upload_f32(e->wts, b.kn, kHD, &L.kn, s))) return st;
    }
    // adaLN of all blocks followed by the output adaLN: one [n_ada][1024] matrix
    e->n_ada = w->n_layers * kAdaPerLayer + 2 * kD;
    {
        std::vector<std::pair<const float *, size_t>> parts;
        std::vector<float> bias((size_t)e->n_ada, 0.f);
        for (int l = 0; l < w->n_layers; l++) {
            parts.push_back({w->blocks[l].ada_w, (size_t)kAdaPerLayer});
            if (w->blocks[l].ada_b)
                std::memcpy(&bias[(size_t)l * kAdaPerLayer], w->blocks[l].ada_b, kAdaPerLayer * 4);
        }
        parts.push_back({w->oada_w, (size_t)2 * kD});
        if (w->oada_b) std::memcpy(&bias[(size_t)w->n_layers * kAdaPerLayer], w->oada_b, 2 * kD * 4);
        if ((st = upload_bf16_concat(e->wts, parts, kD, &e->w_ada, s))) return st;
        if ((st = upload_f32(e->wts, bias.data(), bias.size(), &e->b_ada, s))) return st;
        DTTS_CUDA(cudaStreamSynchronize(s));
    }
    if ((st = upload_bf16_concat(e->wts, {{w->in_w, kD}}, kD, &e->w_in, s))) return st;   // zeros if absent
    e->has_in = w->in_w != nullptr;
    e->has_out = w->out_w != nullptr && w->oada_w != nullptr;
    if ((st = upload_f32(e->wts, w->in_b, kD, &e->b_in, s))) return st;
    if ((st = upload_f32(e->wts, w->t_w1, (size_t)kD * 256, &e->t_w1, s))) return st;
    if ((st = upload_f32(e->wts, w->t_b1, kD, &e->t_b1, s))) return st;
    if ((st = upload_f32(e->wts, w->t_w2, (size_t)kD * kD, &e->t_w2, s))) return st;
    if ((st = upload_f32(e->wts, w->t_b2, kD, &e->t_b2, s))) return st;
    if ((st = upload_f32(e->wts, w->spk_w1, (size_t)kD * kSpk, &e->spk_w1, s))) return st;
    if ((st = upload_f32(e->wts, w->spk_b1, kD, &e->spk_b1, s))) return st;
    if ((st = upload_f32(e->wts, w->spk_ln_w, kD, &e->spk_lw, s))) return st;
    if ((st = upload_f32(e->wts, w->spk_ln_b, kD, &e->spk_lb, s))) return st;
    std::vector<float> out_wt_host, coord_wt_host;
    if ((st = upload_f32_transposed(e->wts, w->out_w, kLat, kD, &e->out_wt, s, out_wt_host))) return st;
    if ((st = upload_f32(e->wts, w->out_b, kLat, &e->out_b, s))) return st;
    if ((st = upload_f32_transposed(e->wts, w->coord_w, kD, kLat, &e->coord_wt, s, coord_wt_host))) return st;
    if ((st = upload_f32(e->wts, w->coord_b, kD, &e->coord_b, s))) return st;
    if ((st = upload_f32(e->wts, w->hid_w, (size_t)kD * kLLM, &e->hid_w, s))) return st;
    if ((st = upload_f32(e->wts, w->hid_b, kD, &e->hid_b, s))) return st;
    if ((st = upload_f32(e->wts, w->lat_w, (size_t)kD * kLat, &e->lat_w, s))) return st;
    if ((st = upload_f32(e->wts, w->lat_b, kD, &e->lat_b, s))) return st;
    if ((st = upload_f32(e->wts, w->eos_w1, (size_t)kLLM * kLLM, &e->eos_w1, s))) return st;
    if ((st = upload_f32(e->wts, w->eos_b1, kLLM, &e->eos_b1, s))) return st;
    if ((st = upload_f32(e->wts, w->eos_w2, (size_t)2 * kLLM, &e->eos_w2, s))) return st;
    if ((st = upload_f32(e->wts, w->eos_b2, 2, &e->eos_b2, s))) return st;
    DTTS_CUDA(cudaStreamSynchronize(s));
    if ((st = e->build_weight_maps())) return st;
    *out = e.release();
    return DTTS_OK;
}

int dtts_dit_destroy(dtts_dit *e) {
    if (!e) return DTTS_OK;
    DeviceGuard g(e->device);
    cudaStreamSynchronize(e->stream);
    delete e;
    return DTTS_OK;
}

int dtts_dit_set_stream(dtts_dit *e, void *stream) {
    DTTS_CHECK(e, DTTS_ERR_ARG, "null engine");
    e->stream = stream ? static_cast<cudaStream_t>(stream) : e->own_stream;
    return DTTS_OK;
}

int dtts_dit_sync(dtts_dit *e) {
    DTTS_CHECK(e, DTTS_ERR_ARG, "null engine");
    DeviceGuard g(e->device);
    return e->finish(true);
}

int dtts_dit_velocity(dtts_dit *e, const float *x_in, const float *cond, const uint8_t *mask, const float *pos,
                      int rows, int L, int n_out, float *out, int mem) {
    DTTS_CHECK(e && x_in && cond && out, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(rows >= 1 && L >= 1 && L <= 4096 && n_out >= 1 && n_out <= L, DTTS_ERR_ARG,
               "bad shape rows=%d L=%d n_out=%d", rows, L, n_out);
    DTTS_CHECK(mem == DTTS_MEM_HOST || mem == DTTS_MEM_DEVICE, DTTS_ERR_ARG, "bad mem kind %d", mem);
    DTTS_CHECK(e->has_in && e->has_out, DTTS_ERR_ARG, "model lacks input_layer / output layer weights");
    DeviceGuard g(e->device);
    int st = e->ensure_workspace(rows, L, 1);
    if (st) return st;
    // this call overwrites the RoPE / mask tables a captured solve reads
    if (e->gexec) { DTTS_CUDA(cudaStreamSynchronize(e->stream)); cudaGraphExecDestroy(e->gexec); e->gexec = nullptr; }
    e->gkey.clear();
    e->launches = 0;
    const cudaMemcpyKind in_kind = mem == DTTS_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    cudaStream_t s = e->stream;
    const size_t ntok = (size_t)rows * L;
    DTTS_CUDA(cudaMemcpyAsync(e->in_a, x_in, ntok * kD * 4, in_kind, s));
    DTTS_CUDA(cudaMemcpyAsync(e->cond_f32, cond, (size_t)rows * kD * 4, in_kind, s));
    std::vector<float2> rt;
    std::vector<float> hpos;
    if (pos) {
        hpos.resize(L);
        DTTS_CUDA(cudaMemcpy(hpos.data(), pos, L * 4, mem == DTTS_MEM_HOST ? cudaMemcpyHostToHost : cudaMemcpyDeviceToHost));
    }
    e->rope_table(pos ? hpos.data() : nullptr, L, rt);
    DTTS_CUDA(cudaMemcpyAsync(e->rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice, s));
    e->last_mask = mask != nullptr;
    std::vector<uint32_t> bits;
    if (mask) {
        std::vector<uint8_t> hm((size_t)L * L);
        DTTS_CUDA(cudaMemcpy(hm.data(), mask, hm.size(), mem == DTTS_MEM_HOST ? cudaMemcpyHostToHost : cudaMemcpyDeviceToHost));
        bits.resize((size_t)L * ((L + 31) / 32));
        pack_mask_bits(hm.data(), L, L, bits.data());
        DTTS_CUDA(cudaMemcpyAsync(e->mask, hm.data(), hm.size(), cudaMemcpyHostToDevice, s));
        DTTS_CUDA(cudaMemcpyAsync(e->mask_bits, bits.data(), bits.size() * 4, cudaMemcpyHostToDevice, s));
        DTTS_CUDA(cudaStreamSynchronize(s));   // host copies go out of scope
    }
    e->launches += 2;
    launch_f32_to_bf16(e->in_a, e->x_in, (long long)ntok * kD, s);
    launch_silu_bf16(e->cond_f32, e->a_cond, (long long)rows * kD, s);
    {
        GemmOp op = make_op(e->t_acond, e->t_ada, rows, e->n_ada, kD, EPI_F32, e->d_err, e->tu_ada);
        op.ep.bias = e->b_ada; op.ep.out = e->ada; op.ep.ldo = e->n_ada;
        if ((st = e->gemm(op))) return st;
    }
    e->last_ada_rows = rows;
    e->ada_cur = e->ada;
    e->rows_per_ada = 1;
    if ((st = e->enqueue_forward(rows, L, n_out))) return st;
    const cudaMemcpyKind out_kind = mem == DTTS_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
    DTTS_CUDA(cudaMemcpyAsync(out, e->vel, (size_t)rows * n_out * kLat * 4, out_kind, s));
    return e->finish(mem == DTTS_MEM_HOST);
}

}  // extern "C"

// The solve; fm_stride > 0: fm_cond / fm_uncond are device buffers holding
// each utterance's rows fm_stride rows apart (the FM history of dtts_fm),
// whatever a->mem says about the other buffers.
static int euler_solve_impl(dtts_dit *e, const dtts_solve_args *a, long long fm_stride) {
    DTTS_CHECK(e && a, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(a->fm_cond && a->fm_uncond && a->z0 && a->z_out, DTTS_ERR_ARG, "null buffer in solve args");
    DTTS_CHECK(a->n_utt >= 1 && a->fm_len >= 0 && a->patch >= 1 && a->nfe >= 1 && a->nfe <= 1000, DTTS_ERR_ARG,
               "bad solve shape n_utt=%d fm_len=%d patch=%d nfe=%d", a->n_utt, a->fm_len, a->patch, a->nfe);
    DTTS_CHECK(a->fm_len + a->patch <= 4096, DTTS_ERR_ARG, "sequence too long");
    DTTS_CHECK(a->cfg_form == DTTS_CFG_V4 || a->cfg_form == DTTS_CFG_V3, DTTS_ERR_ARG, "bad cfg_form");
    DTTS_CHECK(a->layout == DTTS_LAYOUT_FM_MASK || a->layout == DTTS_LAYOUT_FULL, DTTS_ERR_ARG, "bad layout");
    DTTS_CHECK(a->mem == DTTS_MEM_HOST || a->mem == DTTS_MEM_DEVICE, DTTS_ERR_ARG, "bad mem kind");
    DTTS_CHECK(!a->spk || (e->spk_w1 && e->spk_lw), DTTS_ERR_ARG, "speaker vectors given but xvec_proj weights absent");
    DTTS_CHECK(e->has_in && e->has_out && e->coord_wt && e->t_w1 && e->t_w2, DTTS_ERR_ARG,
               "model lacks input/output/coordinate/time-embedding weights needed by the solve");
    DeviceGuard g(e->device);
    const int rows = 2 * a->n_utt, L = a->fm_len + a->patch;
    int st = e->ensure_workspace(rows, L, a->nfe);
    if (st) return st;
    cudaStream_t s = e->stream;
    const cudaMemcpyKind in_kind = a->mem == DTTS_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    const size_t hist = (size_t)a->n_utt * a->fm_len * kD * 4;
    if (hist && fm_stride > 0) {
        const size_t w = (size_t)a->fm_len * kD * 4, sp = (size_t)fm_stride * kD * 4;
        DTTS_CUDA(cudaMemcpy2DAsync(e->in_a, w, a->fm_cond, sp, w, a->n_utt, cudaMemcpyDeviceToDevice, s));
        DTTS_CUDA(cudaMemcpy2DAsync(e->in_b, w, a->fm_uncond, sp, w, a->n_utt, cudaMemcpyDeviceToDevice, s));
    } else if (hist) {
        DTTS_CUDA(cudaMemcpyAsync(e->in_a, a->fm_cond, hist, in_kind, s));
        DTTS_CUDA(cudaMemcpyAsync(e->in_b, a->fm_uncond, hist, in_kind, s));
    }
    DTTS_CUDA(cudaMemcpyAsync(e->z, a->z0, (size_t)a->n_utt * a->patch * kLat * 4, in_kind, s));
    if (a->spk) DTTS_CUDA(cudaMemcpyAsync(e->spk_in, a->spk, (size_t)a->n_utt * kSpk * 4, in_kind, s));

    char keybuf[256];
    snprintf(keybuf, sizeof(keybuf), "%d/%d/%d/%d/%a/%d/%d/%d/%a/%p", a->n_utt, a->fm_len, a->patch, a->nfe,
             a->cfg_scale, a->cfg_form, a->layout, a->spk != nullptr, a->spk_scale, (void *)s);
    const std::string key(keybuf);
    const bool tables_current = (key == e->gkey);
    if (!tables_current) {
        // constant tables for this shape: mask, RoPE, sinusoids
        std::vector<float> pos(L);
        std::vector<uint8_t> m;
        if (a->layout == DTTS_LAYOUT_FM_MASK) {
            m.resize((size_t)L * L);
            fm_mask(m.data(), L, a->fm_len, a->patch, 1);
            fm_pos(pos.data(), L, a->fm_len, a->patch);
        } else {
            for (int i = 0; i < L; i++) pos[i] = (float)i;
        }
        std::vector<float2> rt;
        e->rope_table(pos.data(), L, rt);
        std::vector<float> se((size_t)a->nfe * 256);
        const float dt = 1.0f / (float)a->nfe;
        for (int k = 0; k < a->nfe; k++) sinusoid((float)k * dt, &se[(size_t)k * 256]);
        DTTS_CUDA(cudaMemcpyAsync(e->rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice, s));
        DTTS_CUDA(cudaMemcpyAsync(e->se_tab, se.data(), se.size() * 4, cudaMemcpyHostToDevice, s));
        std::vector<uint32_t> bits;
        if (!m.empty()) {
            bits.resize((size_t)L * ((L + 31) / 32));
            pack_mask_bits(m.data(), L, L, bits.data());
            DTTS_CUDA(cudaMemcpyAsync(e->mask, m.data(), m.size(), cudaMemcpyHostToDevice, s));
            DTTS_CUDA(cudaMemcpyAsync(e->mask_bits, bits.data(), bits.size() * 4, cudaMemcpyHostToDevice, s));
        }
        DTTS_CUDA(cudaStreamSynchronize(s));  // host tables go out of scope
        if (e->gexec) { cudaGraphExecDestroy(e->gexec); e->gexec = nullptr; }
        e->gkey = key;
    }
    e->last_mask = a->layout == DTTS_LAYOUT_FM_MASK;
    if (a->use_graph) {
        if (!e->gexec) {
            e->launches = 0;
            cudaGraph_t graph = nullptr;
            DTTS_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
            st = e->enqueue_solve(a);
            cudaError_t ce = cudaStreamEndCapture(s, &graph);
            if (st) { if (graph) cudaGraphDestroy(graph); return st; }
            DTTS_CUDA(ce);
            ce = cudaGraphInstantiate(&e->gexec, graph, 0);
            cudaGraphDestroy(graph);
            DTTS_CUDA(ce);
        }
        DTTS_CUDA(cudaGraphLaunch(e->gexec, s));
    } else {
        e->launches = 0;
        if ((st = e->enqueue_solve(a))) return st;
    }
    const cudaMemcpyKind out_kind = a->mem == DTTS_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
    DTTS_CUDA(cudaMemcpyAsync(a->z_out, e->z, (size_t)a->n_utt * a->patch * kLat * 4, out_kind, s));
    return e->finish(a->mem == DTTS_MEM_HOST);
}

extern "C" {

int dtts_dit_euler_solve(dtts_dit *e, const dtts_solve_args *a) { return euler_solve_impl(e, a, 0); }

int dtts_dit_blocks(dtts_dit *e, const float *h_in, const float *cond, const uint8_t *mask, const float *pos, int rows,
                    int L, float *h_out, int mem) {
    DTTS_CHECK(e && h_in && cond && h_out, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(rows >= 1 && L >= 1 && L <= 4096, DTTS_ERR_ARG, "bad shape rows=%d L=%d", rows, L);
    DTTS_CHECK(mem == DTTS_MEM_HOST || mem == DTTS_MEM_DEVICE, DTTS_ERR_ARG, "bad mem kind %d", mem);
    DeviceGuard g(e->device);
    int st = e->ensure_workspace(rows, L, 1);
    if (st) return st;
    if (e->gexec) { DTTS_CUDA(cudaStreamSynchronize(e->stream)); cudaGraphExecDestroy(e->gexec); e->gexec = nullptr; }
    e->gkey.clear();
    e->launches = 0;
    const cudaMemcpyKind in_kind = mem == DTTS_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    cudaStream_t s = e->stream;
    const size_t ntok = (size_t)rows * L;
    DTTS_CUDA(cudaMemcpyAsync(e->h, h_in, ntok * kD * 4, in_kind, s));
    DTTS_CUDA(cudaMemcpyAsync(e->cond_f32, cond, (size_t)rows * kD * 4, in_kind, s));
    std::vector<float> hpos;
    std::vector<float2> rt;
    if (pos) {
        hpos.resize(L);
        DTTS_CUDA(cudaMemcpy(hpos.data(), pos, L * 4, mem == DTTS_MEM_HOST ? cudaMemcpyHostToHost : cudaMemcpyDeviceToHost));
    }
    e->rope_table(pos ? hpos.data() : nullptr, L, rt);
    DTTS_CUDA(cudaMemcpyAsync(e->rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice, s));
    e->last_mask = mask != nullptr;
    std::vector<uint8_t> hm;
    std::vector<uint32_t> bits;
    if (mask) {
        hm.resize((size_t)L * L);
        DTTS_CUDA(cudaMemcpy(hm.data(), mask, hm.size(), mem == DTTS_MEM_HOST ? cudaMemcpyHostToHost : cudaMemcpyDeviceToHost));
        bits.resize((size_t)L * ((L + 31) / 32));
        pack_mask_bits(hm.data(), L, L, bits.data());
        DTTS_CUDA(cudaMemcpyAsync(e->mask, hm.data(), hm.size(), cudaMemcpyHostToDevice, s));
        DTTS_CUDA(cudaMemcpyAsync(e->mask_bits, bits.data(), bits.size() * 4, cudaMemcpyHostToDevice, s));
    }
    e->launches++;
    launch_silu_bf16(e->cond_f32, e->a_cond, (long long)rows * kD, s);
    {
        GemmOp op = make_op(e->t_acond, e->t_ada, rows, e->n_ada, kD, EPI_F32, e->d_err, e->tu_ada);
        op.ep.bias = e->b_ada; op.ep.out = e->ada; op.ep.ldo = e->n_ada;
        if ((st = e->gemm(op))) return st;
    }
    e->last_ada_rows = rows;
    e->ada_cur = e->ada;
    e->rows_per_ada = 1;
    e->last_rows = rows; e->last_L = L; e->last_P = 0;
    static const int order[7] = {5, 0, 4, 1, 6, 2, 3};
    for (int l = 0; l < e->n_layers; l++)
        for (int i = 0; i < 7; i++)
            if ((st = e->enqueue_block_op(order[i], l, rows, L))) return st;
    const cudaMemcpyKind out_kind = mem == DTTS_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
    DTTS_CUDA(cudaMemcpyAsync(h_out, e->h, ntok * kD * 4, out_kind, s));
    return e->finish(mem == DTTS_MEM_HOST);
}

int dtts_dit_set_rope(dtts_dit *e, int mode) {
    DTTS_CHECK(e, DTTS_ERR_ARG, "null engine");
    DTTS_CHECK(mode == DTTS_ROPE_HALF || mode == DTTS_ROPE_ADJACENT, DTTS_ERR_ARG, "bad rope mode %d", mode);
    if (e->gexec) { DeviceGuard g(e->device); DTTS_CUDA(cudaStreamSynchronize(e->stream)); cudaGraphExecDestroy(e->gexec); e->gexec = nullptr; }
    e->gkey.clear();
    e->rope_mode = mode;
    return DTTS_OK;
}

int dtts_dit_cond(dtts_dit *e, float t, const float *spk, float spk_scale, float *cond) {
    DTTS_CHECK(e && cond, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(e->t_w1 && e->t_w2, DTTS_ERR_ARG, "model lacks time-embedding weights");
    DTTS_CHECK(!spk || (e->spk_w1 && e->spk_lw), DTTS_ERR_ARG, "speaker vector given but xvec_proj weights absent");
    DeviceGuard g(e->device);
    int st = e->ensure_workspace(1, 1, 1);
    if (st) return st;
    cudaStream_t s = e->stream;
    float se[256];
    sinusoid(t, se);
    DTTS_CUDA(cudaMemcpyAsync(e->se_tab, se, sizeof(se), cudaMemcpyHostToDevice, s));
    launch_time_mlp(e->se_tab, 1, e->t_w1, e->t_b1, e->t_w2, e->t_b2, e->h1, e->temb, s);
    if (spk) {
        DTTS_CUDA(cudaMemcpyAsync(e->spk_in, spk, kSpk * 4, cudaMemcpyHostToDevice, s));
        launch_speaker_cond(e->spk_in, 1, e->spk_w1, e->spk_b1, e->spk_lw, e->spk_lb, spk_scale, e->spk_c, s);
        launch_add_f32(e->temb, e->spk_c, e->cond_f32, kD, s);
        DTTS_CUDA(cudaMemcpyAsync(cond, e->cond_f32, kD * 4, cudaMemcpyDeviceToHost, s));
    } else {
        DTTS_CUDA(cudaMemcpyAsync(cond, e->temb, kD * 4, cudaMemcpyDeviceToHost, s));
    }
    DTTS_CUDA(cudaGetLastError());
    return e->finish(true);
}

int dtts_dit_tune(dtts_dit *e, const char *gemm, int bn, int epi_warps, int ksplit) {
    DTTS_CHECK(e && gemm, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(bn == 128 || bn == 192 || bn == 256, DTTS_ERR_ARG, "bn must be 128, 192 or 256");
    DTTS_CHECK(epi_warps == 4 || epi_warps == 8, DTTS_ERR_ARG, "epi_warps must be 4 or 8");
    DTTS_CHECK(ksplit == 1 || ksplit == 2 || ksplit == 4 || ksplit == 8, DTTS_ERR_ARG, "ksplit must be 1, 2, 4 or 8");
    const std::string g(gemm);
    GemmTune t{bn, epi_warps, ksplit};
    GemmTune *dst = g == "qkv" ? &e->tu_qkv : g == "o" ? &e->tu_o : g == "ffn1" ? &e->tu_ffn1 : g == "ffn2" ? &e->tu_ffn2
                  : g == "adaln" ? &e->tu_ada : g == "input" ? &e->tu_in : nullptr;
    DTTS_CHECK(dst, DTTS_ERR_ARG, "unknown GEMM '%s' (qkv, o, ffn1, ffn2, adaln, input)", gemm);
    const int n = g == "qkv" ? 3 * kD : g == "ffn1" ? kF : g == "adaln" ? e->n_ada : kD;
    DTTS_CHECK(n % bn == 0, DTTS_ERR_ARG, "N = %d is not a multiple of bn %d", n, bn);
    const bool resid = g == "o" || g == "ffn2";
    DTTS_CHECK(ksplit == 1 || resid, DTTS_ERR_ARG, "ksplit > 1 only for the residual GEMMs (o, ffn2)");
    DeviceGuard gd(e->device);
    DTTS_CUDA(cudaStreamSynchronize(e->stream));
    *dst = t;
    if (e->gexec) { cudaGraphExecDestroy(e->gexec); e->gexec = nullptr; }
    e->gkey.clear();
    return e->build_weight_maps();
}

int dtts_dit_set_fused_ln(dtts_dit *e, int on) {
    DTTS_CHECK(e, DTTS_ERR_ARG, "null argument");
    DeviceGuard gd(e->device);
    DTTS_CUDA(cudaStreamSynchronize(e->stream));
    e->fuse_ln = on != 0;
    if (e->gexec) { cudaGraphExecDestroy(e->gexec); e->gexec = nullptr; }
    e->gkey.clear();
    return DTTS_OK;
}

int dtts_dit_last_launch_count(dtts_dit *e, int *n) {
    DTTS_CHECK(e && n, DTTS_ERR_ARG, "null argument");
    *n = e->launches;
    return DTTS_OK;
}

int dtts_dit_solve_timeline(dtts_dit *e, const dtts_solve_args *a, int reps, float *us_total, int *counts) {
    DTTS_CHECK(e && a && us_total && counts, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(a->mem == DTTS_MEM_DEVICE, DTTS_ERR_ARG, "the timeline takes device buffers");
    DTTS_CHECK(reps >= 1 && reps <= 100, DTTS_ERR_ARG, "reps %d out of range", reps);
    // one ordinary solve: validates the arguments, sizes the workspace and
    // uploads this shape's tables
    int st = dtts_dit_euler_solve(e, a);
    if (st) return st;
    DeviceGuard g(e->device);
    cudaStream_t s = e->stream;
    const int saved_launches = e->launches;
    const size_t need = 2 * (size_t)(saved_launches + 16);
    while (e->tl_ev.size() < need) {
        cudaEvent_t ev;
        DTTS_CUDA(cudaEventCreate(&ev));
        e->tl_ev.push_back(ev);
    }
    e->tl_kind.clear();
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    DTTS_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    e->tl_on = true;
    cudaError_t ce = cudaMemcpyAsync(e->z, a->z0, (size_t)a->n_utt * a->patch * kLat * 4, cudaMemcpyDeviceToDevice, s);
    st = ce == cudaSuccess ? e->enqueue_solve(a) : DTTS_ERR_CUDA;
    e->tl_on = false;
    cudaError_t ce2 = cudaStreamEndCapture(s, &graph);
    e->launches = saved_launches;
    if (st || ce != cudaSuccess || ce2 != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        if (st) return st;
        DTTS_CUDA(ce != cudaSuccess ? ce : ce2);
    }
    ce = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    DTTS_CUDA(ce);
    for (int k = 0; k < DTTS_TL_KINDS; k++) { us_total[k] = 0.f; counts[k] = 0; }
    for (size_t i = 0; i < e->tl_kind.size(); i++) counts[e->tl_kind[i]]++;
    std::vector<double> acc(DTTS_TL_KINDS, 0.0);
    for (int r = 0; r < reps && !st; r++) {
        ce = cudaGraphLaunch(exec, s);
        if (ce != cudaSuccess) { st = DTTS_ERR_CUDA; set_error("timeline graph launch: %s", cudaGetErrorString(ce)); break; }
        if ((st = stream_wait(s, 120.0))) break;
        for (size_t i = 0; i < e->tl_kind.size(); i++) {
            float ms = 0.f;
            ce = cudaEventElapsedTime(&ms, e->tl_ev[2 * i], e->tl_ev[2 * i + 1]);
            if (ce != cudaSuccess) { st = DTTS_ERR_CUDA; set_error("timeline event: %s", cudaGetErrorString(ce)); break; }
            acc[e->tl_kind[i]] += ms;
        }
    }
    cudaGraphExecDestroy(exec);
    if (st) return st;
    for (int k = 0; k < DTTS_TL_KINDS; k++) us_total[k] = (float)(acc[k] * 1000.0 / reps);
    return e->finish(true);
}

int dtts_dit_profile_kernel(dtts_dit *e, int kind, int iters, float *us, double *flops, double *bytes) {
    DTTS_CHECK(e && us, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(e->last_rows > 0, DTTS_ERR_ARG, "run a solve or velocity call first");
    DTTS_CHECK(kind >= 0 && kind <= 7 && iters >= 1, DTTS_ERR_ARG, "bad kind/iters");
    DeviceGuard g(e->device);
    const int rows = e->last_rows, L = e->last_L;
    const double M = (double)rows * L;
    auto one = [&]() -> int {
        switch (kind) {
            case 0: return e->enqueue_block_op(0, 0, rows, L);
            case 1: return e->enqueue_block_op(1, 0, rows, L);
            case 2: return e->enqueue_block_op(2, 0, rows, L);
            case 3: return e->enqueue_block_op(3, 0, rows, L);
            case 4: return e->enqueue_block_op(4, 0, rows, L);
            case 5: return e->enqueue_block_op(5, 0, rows, L);
            case 6: {
                GemmOp op = make_op(e->t_acond, e->t_ada, e->last_ada_rows, e->n_ada, kD, EPI_F32, e->d_err, e->tu_ada);
                op.ep.bias = e->b_ada; op.ep.out = e->ada; op.ep.ldo = e->n_ada;
                return e->gemm(op);
            }
            case 7: {
                GemmOp op = make_op(e->t_x_in, e->t_in, (int)M, kD, kD, EPI_F32, e->d_err, e->tu_in);
                op.ep.bias = e->b_in; op.ep.out = e->h; op.ep.ldo = kD;
                return e->gemm(op);
            }
        }
        return DTTS_ERR_ARG;
    };
    cudaStream_t s = e->stream;
    int st;
    for (int i = 0; i < 3; i++)
        if ((st = one())) return st;
    cudaEvent_t e0, e1;
    DTTS_CUDA(cudaEventCreate(&e0));
    DTTS_CUDA(cudaEventCreate(&e1));
    DTTS_CUDA(cudaEventRecord(e0, s));
    for (int i = 0; i < iters; i++)
        if ((st = one())) return st;
    DTTS_CUDA(cudaEventRecord(e1, s));
    if ((st = stream_wait(s, 120.0))) return st;
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *us = ms * 1000.0f / iters;
    double f = 0, b = 0;
    const double W = 2.0;  // bytes per bf16
    switch (kind) {
        case 0: f = 2 * M * 3 * kD * kD; b = W * (M * kD + 3.0 * kD * kD + 3 * M * kD); break;
        case 1: f = 2 * M * kD * kD; b = W * (M * kD + 1.0 * kD * kD) + 8 * M * kD; break;
        case 2: f = 2 * M * kF * kD; b = W * (M * kD + 1.0 * kF * kD + M * kF); break;
        case 3: f = 2 * M * kD * kF; b = W * (M * kF + 1.0 * kF * kD) + 8 * M * kD; break;
        case 4: f = 4.0 * rows * kH * (double)L * L * kHD; b = W * 4 * M * kD; break;
        case 5: f = 0; b = M * kD * 4 + M * kD * 2; break;
        case 6: {
            const double ar = e->last_ada_rows;
            f = 2.0 * ar * e->n_ada * kD; b = W * ((double)e->n_ada * kD + ar * kD) + 4.0 * ar * e->n_ada;
            break;
        }
        case 7: f = 2 * M * kD * kD; b = W * (M * kD + 1.0 * kD * kD) + 4 * M * kD; break;
    }
    if (flops) *flops = f;
    if (bytes) *bytes = b;
    return e->finish(true);
}

// ---------------------------------------------------------------- FM history
struct dtts_fm {
    dtts_dit *e = nullptr;
    int n_utt = 0, cap = 0, len = 0;
    DeviceArena mem;
    float *cond = nullptr, *uncond = nullptr;   // [n_utt][cap][1024]
    float *tmp = nullptr;                       // [n_utt * kFmMaxPatch][1024] projected rows
    float *hin = nullptr;                       // [n_utt][1536]
    float *zin = nullptr;                       // [n_utt][kFmMaxPatch][128]
    float *h1 = nullptr, *logits = nullptr, *prob = nullptr;   // EOS head
    float *null_row = nullptr;                  // hidden_proj(0) = its bias
    ~dtts_fm() { mem.free_all(); }
};

int dtts_fm_create(dtts_dit *e, int n_utt, int capacity, dtts_fm **out) {
    DTTS_CHECK(e && out, DTTS_ERR_ARG, "null argument");
    *out = nullptr;
    DTTS_CHECK(n_utt >= 1 && capacity >= 1 && capacity <= 4096, DTTS_ERR_ARG, "bad FM history shape %d x %d", n_utt,
               capacity);
    DTTS_CHECK(e->hid_w && e->lat_w, DTTS_ERR_ARG, "the model lacks hidden_proj / latent_proj weights");
    DeviceGuard g(e->device);
    std::unique_ptr<dtts_fm> f(new dtts_fm());
    f->e = e; f->n_utt = n_utt; f->cap = capacity;
    const size_t rows = (size_t)n_utt * capacity;
    auto A = [&](size_t bytes) { return (float *)f->mem.alloc(bytes); };
    f->cond = A(rows * kD * 4);
    f->uncond = A(rows * kD * 4);
    f->tmp = A((size_t)n_utt * kFmMaxPatch * kD * 4);
    f->hin = A((size_t)n_utt * kLLM * 4);
    f->zin = A((size_t)n_utt * kFmMaxPatch * kLat * 4);
    f->h1 = A((size_t)n_utt * kLLM * 4);
    f->logits = A((size_t)n_utt * 2 * 4);
    f->prob = A((size_t)n_utt * 4);
    f->null_row = A((size_t)kD * 4);
    DTTS_CHECK(f->cond && f->uncond && f->tmp && f->hin && f->zin && f->h1 && f->logits && f->prob && f->null_row,
               DTTS_ERR_OOM, "FM history allocation failed");
    // hidden_proj of a zero vector is its bias (src/e2e_pipeline_v4.cpp:338-339)
    if (e->hid_b)
        DTTS_CUDA(cudaMemcpyAsync(f->null_row, e->hid_b, (size_t)kD * 4, cudaMemcpyDeviceToDevice, e->stream));
    else
        DTTS_CUDA(cudaMemsetAsync(f->null_row, 0, (size_t)kD * 4, e->stream));
    DTTS_CUDA(cudaStreamSynchronize(e->stream));
    *out = f.release();
    return DTTS_OK;
}

int dtts_fm_destroy(dtts_fm *f) {
    if (!f) return DTTS_OK;
    DeviceGuard g(f->e->device);
    cudaStreamSynchronize(f->e->stream);
    delete f;
    return DTTS_OK;
}

static int fm_copy_in(dtts_fm *f, float *dst, const float *src, size_t bytes, int mem) {
    DTTS_CHECK(mem == DTTS_MEM_HOST || mem == DTTS_MEM_DEVICE, DTTS_ERR_ARG, "bad mem kind");
    DTTS_CUDA(cudaMemcpyAsync(dst, src, bytes, mem == DTTS_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice,
                              f->e->stream));
    return DTTS_OK;
}

int dtts_fm_start(dtts_fm *f, const float *hidden0, int mem) {
    DTTS_CHECK(f && hidden0, DTTS_ERR_ARG, "null argument");
    dtts_dit *e = f->e;
    DeviceGuard g(e->device);
    int st = fm_copy_in(f, f->hin, hidden0, (size_t)f->n_utt * kLLM * 4, mem);
    if (st) return st;
    launch_gemm_f32(f->hin, e->hid_w, e->hid_b, f->tmp, f->n_utt, kD, kLLM, e->stream);
    launch_fm_place_rows(f->tmp, f->cond, f->n_utt, 1, f->cap, 0, 0, e->stream);
    launch_fm_place_rows(f->null_row, f->uncond, f->n_utt, 1, f->cap, 0, 1, e->stream);
    DTTS_CUDA(cudaGetLastError());
    f->len = 1;
    return e->finish(mem == DTTS_MEM_HOST);
}

int dtts_fm_append_latents(dtts_fm *f, const float *z, int patch, int mem) {
    DTTS_CHECK(f && z, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(f->len >= 1, DTTS_ERR_ARG, "call dtts_fm_start first");
    DTTS_CHECK(patch >= 1 && patch <= kFmMaxPatch, DTTS_ERR_ARG, "patch %d out of [1, %d]", patch, kFmMaxPatch);
    DTTS_CHECK(f->len + patch <= f->cap, DTTS_ERR_ARG, "FM history full (%d + %d > %d rows)", f->len, patch, f->cap);
    dtts_dit *e = f->e;
    DeviceGuard g(e->device);
    int st = fm_copy_in(f, f->zin, z, (size_t)f->n_utt * patch * kLat * 4, mem);
    if (st) return st;
    launch_gemm_f32(f->zin, e->lat_w, e->lat_b, f->tmp, f->n_utt * patch, kD, kLat, e->stream);
    launch_fm_place_rows(f->tmp, f->cond, f->n_utt, patch, f->cap, f->len, 0, e->stream);
    launch_fm_place_rows(f->tmp, f->uncond, f->n_utt, patch, f->cap, f->len, 0, e->stream);
    DTTS_CUDA(cudaGetLastError());
    f->len += patch;
    return e->finish(mem == DTTS_MEM_HOST);
}

int dtts_fm_append_hidden(dtts_fm *f, const float *h, float *eos_prob, int eos_act, int mem) {
    DTTS_CHECK(f && h, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(f->len >= 1, DTTS_ERR_ARG, "call dtts_fm_start first");
    DTTS_CHECK(f->len + 1 <= f->cap, DTTS_ERR_ARG, "FM history full (%d rows)", f->cap);
    DTTS_CHECK(eos_act == DTTS_EOS_SILU || eos_act == DTTS_EOS_AS_WRITTEN, DTTS_ERR_ARG, "bad eos_act %d", eos_act);
    dtts_dit *e = f->e;
    DTTS_CHECK(!eos_prob || (e->eos_w1 && e->eos_w2), DTTS_ERR_ARG, "the model lacks eos_proj weights");
    DeviceGuard g(e->device);
    int st = fm_copy_in(f, f->hin, h, (size_t)f->n_utt * kLLM * 4, mem);
    if (st) return st;
    launch_gemm_f32(f->hin, e->hid_w, e->hid_b, f->tmp, f->n_utt, kD, kLLM, e->stream);
    launch_fm_place_rows(f->tmp, f->cond, f->n_utt, 1, f->cap, f->len, 0, e->stream);
    launch_fm_place_rows(f->null_row, f->uncond, f->n_utt, 1, f->cap, f->len, 1, e->stream);
    if (eos_prob) {
        launch_gemm_f32(f->hin, e->eos_w1, e->eos_b1, f->h1, f->n_utt, kLLM, kLLM, e->stream);
        launch_eos_act(f->h1, f->n_utt, eos_act == DTTS_EOS_AS_WRITTEN, e->stream);
        launch_gemm_f32(f->h1, e->eos_w2, e->eos_b2, f->logits, f->n_utt, 2, kLLM, e->stream);
        launch_eos_prob(f->logits, f->n_utt, f->prob, e->stream);
        DTTS_CUDA(cudaMemcpyAsync(eos_prob, f->prob, (size_t)f->n_utt * 4,
                                  mem == DTTS_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, e->stream));
    }
    DTTS_CUDA(cudaGetLastError());
    f->len += 1;
    return e->finish(mem == DTTS_MEM_HOST);
}

int dtts_fm_length(dtts_fm *f, int *rows) {
    DTTS_CHECK(f && rows, DTTS_ERR_ARG, "null argument");
    *rows = f->len;
    return DTTS_OK;
}

int dtts_fm_read(dtts_fm *f, float *cond, float *uncond) {
    DTTS_CHECK(f && cond && uncond, DTTS_ERR_ARG, "null argument");
    dtts_dit *e = f->e;
    DeviceGuard g(e->device);
    const size_t w = (size_t)f->len * kD * 4, sp = (size_t)f->cap * kD * 4;
    DTTS_CUDA(cudaMemcpy2DAsync(cond, w, f->cond, sp, w, f->n_utt, cudaMemcpyDeviceToHost, e->stream));
    DTTS_CUDA(cudaMemcpy2DAsync(uncond, w, f->uncond, sp, w, f->n_utt, cudaMemcpyDeviceToHost, e->stream));
    return e->finish(true);
}

int dtts_fm_solve(dtts_fm *f, const dtts_solve_args *a) {
    DTTS_CHECK(f && a, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(f->len >= 1, DTTS_ERR_ARG, "empty FM history");
    dtts_solve_args b = *a;
    b.n_utt = f->n_utt;
    b.fm_len = f->len;
    b.fm_cond = f->cond;
    b.fm_uncond = f->uncond;
    return euler_solve_impl(f->e, &b, f->cap);
}

int dtts_fm_layout(int total, int fm_len, int patch, int hidden_patch, uint8_t *mask, float *pos) {
    DTTS_CHECK(mask || pos, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(total >= 1 && patch >= 0 && fm_len >= 0 && fm_len + patch <= total && hidden_patch >= 0,
               DTTS_ERR_ARG, "bad layout total=%d fm_len=%d patch=%d hidden_patch=%d", total, fm_len, patch,
               hidden_patch);
    if (mask) fm_mask(mask, total, fm_len, patch, hidden_patch);
    if (pos) fm_pos(pos, total, fm_len, patch);
    return DTTS_OK;
}

}  // extern "C"
