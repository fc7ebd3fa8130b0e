// The DiT self-attention sublayer on its own (include/dit_manual.h:88-146):
// Q/K/V projections, per-head RMS qk-norm, half-split RoPE, softmax attention,
// O projection.  DTTS_DTYPE_F32 runs every step in fp32 (SIMT GEMMs and fp32
// attention, for the fp32 parity bar); DTTS_DTYPE_BF16 runs the same tcgen05
// GEMMs and bf16 attention kernel as the full DiT.
#include "kernels.cuh"
#include "runtime.h"

#include <cmath>
#include <cstring>
#include <memory>
#include <vector>

using namespace dtts;

struct dtts_attn {
    int device = 0, dtype = DTTS_DTYPE_F32, num_sms = 148;
    cudaStream_t stream = nullptr;
    DeviceArena wts, ws;
    float *wq = nullptr, *wk = nullptr, *wv = nullptr, *wo = nullptr, *bo = nullptr, *qn = nullptr, *kn = nullptr;
    bf16 *wqkv16 = nullptr, *wo16 = nullptr;
    CUtensorMap t_wqkv, t_wo;
    int *d_err = nullptr;
    // workspace
    int cap_tok = 0, cap_L = 0;
    float *x = nullptr, *qf = nullptr, *kf = nullptr, *vf = nullptr, *ctx = nullptr, *out = nullptr;
    bf16 *x16 = nullptr, *q16 = nullptr, *k16 = nullptr, *v16 = nullptr, *ctx16 = nullptr;
    float2 *rope = nullptr;
    uint8_t *mask = nullptr;
    uint32_t *mask_bits = nullptr;
    CUtensorMap t_x16, t_ctx16;
    // last shapes
    int last_rows = 0, last_L = 0;
    bool last_mask = false;

    ~dtts_attn() {
        ws.free_all();
        wts.free_all();
        if (stream) cudaStreamDestroy(stream);
    }

    int ensure(int rows, int L) {
        const long long tok = (long long)rows * L;
        if (tok <= cap_tok && L <= cap_L) return DTTS_OK;
        DTTS_CUDA(cudaStreamSynchronize(stream));
        ws.free_all();
        cap_tok = (int)std::max<long long>(tok, cap_tok);
        cap_L = std::max(L, cap_L);
        const size_t T = cap_tok;
        x = (float *)ws.alloc(T * kD * 4);
        out = (float *)ws.alloc(T * kD * 4);
        rope = (float2 *)ws.alloc((size_t)cap_L * 32 * sizeof(float2));
        mask = (uint8_t *)ws.alloc((size_t)cap_L * cap_L);
        mask_bits = (uint32_t *)ws.alloc((size_t)cap_L * ((cap_L + 31) / 32) * 4);
        if (dtype == DTTS_DTYPE_F32) {
            qf = (float *)ws.alloc(T * kD * 4);
            kf = (float *)ws.alloc(T * kD * 4);
            vf = (float *)ws.alloc(T * kD * 4);
            ctx = (float *)ws.alloc(T * kD * 4);
        } else {
            x16 = (bf16 *)ws.alloc(T * kD * 2);
            q16 = (bf16 *)ws.alloc(T * kD * 2);
            k16 = (bf16 *)ws.alloc(T * kD * 2);
            v16 = (bf16 *)ws.alloc(T * kD * 2);
            ctx16 = (bf16 *)ws.alloc(T * kD * 2);
        }
        for (void *p : ws.ptrs)
            if (!p) { ws.free_all(); cap_tok = cap_L = 0; set_error("workspace allocation failed"); return DTTS_ERR_OOM; }
        if (dtype != DTTS_DTYPE_F32) {
            bool ok = make_tmap_bf16(&t_x16, x16, T, kD, 128) && make_tmap_bf16(&t_ctx16, ctx16, T, kD, 128);
            DTTS_CHECK(ok, DTTS_ERR_CUDA, "tensor map (attention workspace)");
        }
        return DTTS_OK;
    }

    void enqueue_core(int rows, int L) {
        AttnArgs a{};
        a.rows = rows; a.Tq = L; a.kv_len = L; a.kv_cap = L; a.q_pos0 = 0; a.causal = 0;
        a.mask = last_mask ? mask : nullptr;
        a.mask_bits = last_mask ? mask_bits : nullptr;
        a.scale = 1.0f / sqrtf(64.0f);
        a.ldq = a.ldkv = a.ldo = kD;
        if (dtype == DTTS_DTYPE_F32) {
            a.q = qf; a.k = kf; a.v = vf; a.o = ctx;
            launch_attention_f32(a, stream);
        } else {
            a.q = q16; a.k = k16; a.v = v16; a.o = ctx16;
            launch_attention_bf16(a, stream);
        }
    }
};

namespace {
void rope_half(const float *pos, int L, std::vector<float2> &tab) {
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

int up_f32(DeviceArena &a, const float *h, size_t n, float **out) {
    *out = nullptr;
    if (!h) return DTTS_OK;
    void *d = a.alloc(n * 4);
    DTTS_CHECK(d, DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemcpy(d, h, n * 4, cudaMemcpyHostToDevice));
    *out = (float *)d;
    return DTTS_OK;
}

int up_bf16(DeviceArena &a, const std::vector<const float *> &parts, size_t rows_each, size_t cols, bf16 **out) {
    std::vector<uint16_t> tmp(parts.size() * rows_each * cols);
    for (size_t i = 0; i < parts.size(); i++) f32_to_bf16_host(parts[i], tmp.data() + i * rows_each * cols, rows_each * cols);
    void *d = a.alloc(tmp.size() * 2);
    DTTS_CHECK(d, DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemcpy(d, tmp.data(), tmp.size() * 2, cudaMemcpyHostToDevice));
    *out = (bf16 *)d;
    return DTTS_OK;
}
}  // namespace

extern "C" {

int dtts_attn_create(const dtts_attn_weights *w, int dtype, int device, dtts_attn **out) {
    DTTS_CHECK(w && out, DTTS_ERR_ARG, "null argument");
    *out = nullptr;
    DTTS_CHECK(w->wq && w->wk && w->wv && w->wo, DTTS_ERR_ARG, "missing projection weight");
    DTTS_CHECK(dtype == DTTS_DTYPE_F32 || dtype == DTTS_DTYPE_BF16, DTTS_ERR_UNSUPPORTED, "dtype %d", dtype);
    int nsm = 0, st = check_device(device, &nsm);
    if (st) return st;
    DeviceGuard g(device);
    std::unique_ptr<dtts_attn> a(new dtts_attn());
    a->device = device; a->dtype = dtype; a->num_sms = nsm;
    DTTS_CUDA(cudaStreamCreateWithFlags(&a->stream, cudaStreamNonBlocking));
    a->d_err = (int *)a->wts.alloc(4);
    DTTS_CHECK(a->d_err, DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemset(a->d_err, 0, 4));
    if ((st = up_f32(a->wts, w->bo, kD, &a->bo))) return st;
    if ((st = up_f32(a->wts, w->qn, kHD, &a->qn))) return st;
    if ((st = up_f32(a->wts, w->kn, kHD, &a->kn))) return st;
    if (dtype == DTTS_DTYPE_F32) {
        DTTS_CUDA(attention_f32_prepare());
        if ((st = up_f32(a->wts, w->wq, (size_t)kD * kD, &a->wq))) return st;
        if ((st = up_f32(a->wts, w->wk, (size_t)kD * kD, &a->wk))) return st;
        if ((st = up_f32(a->wts, w->wv, (size_t)kD * kD, &a->wv))) return st;
        if ((st = up_f32(a->wts, w->wo, (size_t)kD * kD, &a->wo))) return st;
    } else {
        DTTS_CUDA(gemm_prepare_attributes());
        DTTS_CUDA(attention_short_prepare());
        if ((st = up_bf16(a->wts, {w->wq, w->wk, w->wv}, kD, kD, &a->wqkv16))) return st;
        if ((st = up_bf16(a->wts, {w->wo}, kD, kD, &a->wo16))) return st;
        bool ok = make_tmap_bf16(&a->t_wqkv, a->wqkv16, 3 * kD, kD, 256) && make_tmap_bf16(&a->t_wo, a->wo16, kD, kD, 256);
        DTTS_CHECK(ok, DTTS_ERR_CUDA, "tensor map (attention weights)");
    }
    *out = a.release();
    return DTTS_OK;
}

int dtts_attn_destroy(dtts_attn *a) {
    if (!a) return DTTS_OK;
    DeviceGuard g(a->device);
    cudaStreamSynchronize(a->stream);
    delete a;
    return DTTS_OK;
}

int dtts_attn_forward(dtts_attn *a, const float *x, int rows, int L, const uint8_t *mask, const float *pos,
                      float *out) {
    DTTS_CHECK(a && x && out, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(rows >= 1 && L >= 1, DTTS_ERR_ARG, "bad shape rows=%d L=%d", rows, L);
    DTTS_CHECK(a->dtype != DTTS_DTYPE_F32 || L <= 400, DTTS_ERR_ARG, "fp32 attention supports L <= 400");
    DeviceGuard g(a->device);
    int st = a->ensure(rows, L);
    if (st) return st;
    cudaStream_t s = a->stream;
    const int M = rows * L;
    std::vector<float2> rt;
    rope_half(pos, L, rt);
    DTTS_CUDA(cudaMemcpyAsync(a->rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice, s));
    a->last_mask = mask != nullptr;
    std::vector<uint32_t> bits;
    if (mask) {
        bits.resize((size_t)L * ((L + 31) / 32));
        pack_mask_bits(mask, L, L, bits.data());
        DTTS_CUDA(cudaMemcpyAsync(a->mask, mask, (size_t)L * L, cudaMemcpyHostToDevice, s));
        DTTS_CUDA(cudaMemcpyAsync(a->mask_bits, bits.data(), bits.size() * 4, cudaMemcpyHostToDevice, s));
    }
    DTTS_CUDA(cudaMemcpyAsync(a->x, x, (size_t)M * kD * 4, cudaMemcpyHostToDevice, s));
    if (a->dtype == DTTS_DTYPE_F32) {
        launch_gemm_f32(a->x, a->wq, nullptr, a->qf, M, kD, kD, s);
        launch_gemm_f32(a->x, a->wk, nullptr, a->kf, M, kD, kD, s);
        launch_gemm_f32(a->x, a->wv, nullptr, a->vf, M, kD, kD, s);
        launch_qk_norm_rope_f32(a->qf, a->kf, M, L, 1, a->qn, a->kn, a->rope, ROPE_HALF, 0, s);
        a->enqueue_core(rows, L);
        launch_gemm_f32(a->ctx, a->wo, a->bo, a->out, M, kD, kD, s);
    } else {
        launch_f32_to_bf16(a->x, a->x16, (long long)M * kD, s);
        GemmOp op;
        std::memset(&op, 0, sizeof(op));
        op.ta = a->t_x16; op.tb = a->t_wqkv; op.M = M; op.N = 3 * kD; op.K = kD; op.bn = 256; op.epi = EPI_QKV;
        op.ep.err = a->d_err; op.ep.q = a->q16; op.ep.k = a->k16; op.ep.v = a->v16; op.ep.ldq = kD; op.ep.ldkv = kD;
        op.ep.tok_per_row = L; op.ep.kv_cap = L; op.ep.kv_start = 0; op.ep.qk_norm = 1;
        op.ep.qn = a->qn; op.ep.kn = a->kn; op.ep.rope = a->rope; op.ep.rope_mode = ROPE_HALF;
        DTTS_CUDA(launch_gemm(op, a->num_sms, s));
        a->enqueue_core(rows, L);
        GemmOp oo;
        std::memset(&oo, 0, sizeof(oo));
        oo.ta = a->t_ctx16; oo.tb = a->t_wo; oo.M = M; oo.N = kD; oo.K = kD; oo.bn = 256; oo.epi = EPI_F32;
        oo.ep.err = a->d_err; oo.ep.bias = a->bo; oo.ep.out = a->out; oo.ep.ldo = kD; oo.ep.tok_per_row = 1;
        DTTS_CUDA(launch_gemm(oo, a->num_sms, s));
    }
    DTTS_CUDA(cudaGetLastError());
    DTTS_CUDA(cudaMemcpyAsync(out, a->out, (size_t)M * kD * 4, cudaMemcpyDeviceToHost, s));
    if ((st = stream_wait(s, 120.0))) return st;
    int err = 0;
    DTTS_CUDA(cudaMemcpy(&err, a->d_err, 4, cudaMemcpyDeviceToHost));
    if (err) { cudaMemset(a->d_err, 0, 4); set_error("device wait limit reached (code %d)", err); return DTTS_ERR_TIMEOUT; }
    a->last_rows = rows;
    a->last_L = L;
    return DTTS_OK;
}

int dtts_attn_profile_core(dtts_attn *a, int iters, float *us) {
    DTTS_CHECK(a && us && iters >= 1, DTTS_ERR_ARG, "bad argument");
    DTTS_CHECK(a->last_rows > 0, DTTS_ERR_ARG, "run dtts_attn_forward first");
    DeviceGuard g(a->device);
    for (int i = 0; i < 3; i++) a->enqueue_core(a->last_rows, a->last_L);
    cudaEvent_t e0, e1;
    DTTS_CUDA(cudaEventCreate(&e0));
    DTTS_CUDA(cudaEventCreate(&e1));
    DTTS_CUDA(cudaEventRecord(e0, a->stream));
    for (int i = 0; i < iters; i++) a->enqueue_core(a->last_rows, a->last_L);
    DTTS_CUDA(cudaEventRecord(e1, a->stream));
    int st = stream_wait(a->stream, 120.0);
    if (st) return st;
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *us = ms * 1000.0f / iters;
    return DTTS_OK;
}

}  // extern "C"
