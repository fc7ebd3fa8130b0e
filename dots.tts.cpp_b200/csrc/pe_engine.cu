// PatchEncoder (src/modules/backbone/patchenc.cpp:146-239) on sm_100a, with
// the streaming decode the reference declares but never defines
// (include/patchenc.h:78-90): a per-sequence KV cache of post-RoPE keys and
// values for every layer plus the last input frame (the causal conv tail).
//
// One call appends n_frames (a multiple of 4) to B streams:
//   conv (k=2, s=2, taps 2t-1, 2t of [tail | frames]) -> in_proj GEMM ->
//   24 x [RMSNorm*w -> QKV GEMM (RoPE epilogue, K/V written into the cache) ->
//         causal attention over cache + new tokens -> O GEMM (+residual) ->
//         RMSNorm*w -> FFN1 GEMM (+SiLU) -> FFN2 GEMM (+residual)] ->
//   token pairs -> out_proj GEMM.
// Attention and conv are causal, so any split of a sequence into calls gives
// the stateless forward over the whole prefix.
#include "kernels.cuh"
#include "runtime.h"

#include <cmath>
#include <cstring>
#include <memory>
#include <vector>

using namespace dtts;

namespace {
constexpr int kBN = 256;
// Calls of at most kSmallTok tokens (decode steps) use 128-wide tiles and split
// every layer GEMM along K so that about 128 CTAs stream the weights: QKV and
// FFN1 reduce-add into zeroed fp32 rows (finished by pe_qkv_finish_kernel and
// pe_silu_kernel, which zero them again behind themselves), O and FFN2 into the
// residual.  Partial sums arrive in run-dependent order.  These calls read the
// cache position from device memory and replay one CUDA graph per shape.
constexpr int kBNs = 128;
constexpr long long kSmallTok = 256;
constexpr int kKsQKV = 8, kKsO = 16, kKsF1 = 4, kKsF2 = 16;

// Split-K QKV finish for token m = b * T + t at cache position p = start + t:
// RoPE on adjacent pairs of q and k (the EPI_QKV epilogue's rotation), q to
// bf16 rows, k and v into the caches, then the fp32 row is zeroed for the next
// reduce-add.  One block of 256 threads per token.
__global__ void __launch_bounds__(256) pe_qkv_finish_kernel(float *__restrict__ qkv, int T, int start,
                                                            const int *__restrict__ start_dev,
                                                            const float2 *__restrict__ rope, bf16 *__restrict__ q,
                                                            bf16 *__restrict__ kc, bf16 *__restrict__ vc, int cap) {
    pdl_wait();
    pdl_trigger();
    if (start_dev) start = *start_dev;
    const int m = blockIdx.x, b = m / T, t = m % T, p = start + t;
    float2 *row = reinterpret_cast<float2 *>(qkv + (long long)m * 3 * kD);
    const long long crow = ((long long)b * cap + p) * kD;
    for (int i = threadIdx.x; i < kD / 2; i += blockDim.x) {
        const float2 cs = rope[(long long)p * 32 + (i & 31)];
        const float2 xq = row[i], xk = row[kD / 2 + i], xv = row[kD + i];
        row[i] = row[kD / 2 + i] = row[kD + i] = make_float2(0.f, 0.f);
        reinterpret_cast<uint32_t *>(q + (long long)m * kD)[i] =
            pack_bf16x2(xq.x * cs.x - xq.y * cs.y, xq.x * cs.y + xq.y * cs.x);
        reinterpret_cast<uint32_t *>(kc + crow)[i] = pack_bf16x2(xk.x * cs.x - xk.y * cs.y, xk.x * cs.y + xk.y * cs.x);
        reinterpret_cast<uint32_t *>(vc + crow)[i] = pack_bf16x2(xv.x, xv.y);
    }
}

// ffn = bf16(silu(x)) over n4 groups of four, x zeroed behind the read
__global__ void pe_silu_kernel(float *__restrict__ x, bf16 *__restrict__ ffn, long long n4) {
    pdl_wait();
    pdl_trigger();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    float4 v = reinterpret_cast<float4 *>(x)[i];
    reinterpret_cast<float4 *>(x)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    v.x = silu_f(v.x); v.y = silu_f(v.y); v.z = silu_f(v.z); v.w = silu_f(v.w);
    reinterpret_cast<uint2 *>(ffn)[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
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

GemmOp op0(const CUtensorMap &ta, const CUtensorMap &tb, int M, int N, int K, int epi, int *err) {
    GemmOp op;
    std::memset(&op, 0, sizeof(op));
    op.ta = ta; op.tb = tb; op.M = M; op.N = N; op.K = K; op.bn = kBN; op.epi = epi;
    op.ep.err = err; op.ep.tok_per_row = 1;
    return op;
}
}  // namespace

struct dtts_pe {
    int device = 0, dtype = DTTS_DTYPE_BF16, num_sms = 148;
    cudaStream_t own_stream = nullptr, stream = nullptr;
    DeviceArena wts, cache, ws;
    int n_layers = 0, max_batch = 0, max_tokens = 0;
    struct Layer {
        bf16 *wqkv = nullptr, *wo = nullptr, *w1 = nullptr, *w2 = nullptr;
        float *bo = nullptr, *b1 = nullptr, *b2 = nullptr, *an = nullptr, *fn = nullptr;
        CUtensorMap tqkv, to, t1, t2;
        CUtensorMap tqkv_s, to_s, t1_s, t2_s;   // 128-row boxes for kBNs tiles
    };
    std::vector<Layer> layers;
    float *conv_w = nullptr, *conv_b = nullptr, *in_b = nullptr, *out_b = nullptr;
    bf16 *in_w = nullptr, *out_w = nullptr;
    CUtensorMap t_inw, t_outw, t_inw_s, t_outw_s;
    bf16 *kc = nullptr, *vc = nullptr;   // [n_layers][max_batch][max_tokens][1024]
    float *tail[2] = {nullptr, nullptr}; // [max_batch][128]: tail[0] read, tail[1] written then copied back
    int *d_len = nullptr;                // cache length on the device (graph-captured steps)
    float2 *rope = nullptr;              // [max_tokens][32], adjacent-pair rotation
    int *d_err = nullptr;
    int cur_B = 0, cur_len = 0;
    // workspace
    long long cap_tok = 0;
    float *frames = nullptr, *h = nullptr, *outf = nullptr;
    bf16 *conv = nullptr, *act = nullptr, *q = nullptr, *att = nullptr, *ffn = nullptr, *pairs = nullptr;
    CUtensorMap t_conv, t_act, t_att, t_ffn, t_pairs, t_h;
    // split-K targets of the small path ([kSmallTok][3 * 1024] and
    // [kSmallTok][4096] fp32), all zero between calls
    float *qkv32 = nullptr, *ffn32 = nullptr;
    CUtensorMap t_qkv32, t_ffn32;
    int launches = 0;
    // decode graphs, keyed by (B, n_frames); dropped when the workspace moves
    struct Graph { int B, n_frames; cudaGraphExec_t exec; };
    std::vector<Graph> graphs;
    void drop_graphs() {
        for (Graph &g : graphs) cudaGraphExecDestroy(g.exec);
        graphs.clear();
    }

    ~dtts_pe() {
        drop_graphs();
        ws.free_all();
        cache.free_all();
        wts.free_all();
        if (own_stream) cudaStreamDestroy(own_stream);
    }

    int ensure(long long tok) {
        if (tok <= cap_tok) return DTTS_OK;
        DTTS_CUDA(cudaStreamSynchronize(stream));
        drop_graphs();
        ws.free_all();
        cap_tok = std::max<long long>(tok, 64);
        const size_t T = (size_t)cap_tok;
        frames = (float *)ws.alloc(T * 2 * kLat * 4);
        conv = (bf16 *)ws.alloc(T * kLat * 2);
        h = (float *)ws.alloc(T * kD * 4);
        act = (bf16 *)ws.alloc(T * kD * 2);
        q = (bf16 *)ws.alloc(T * kD * 2);
        att = (bf16 *)ws.alloc(T * kD * 2);
        ffn = (bf16 *)ws.alloc(T * kF * 2);
        pairs = (bf16 *)ws.alloc(T * kD * 2);   // [T/2][2048]
        outf = (float *)ws.alloc((T / 2 + 1) * kLLM * 4);
        qkv32 = (float *)ws.alloc((size_t)kSmallTok * 3 * kD * 4);
        ffn32 = (float *)ws.alloc((size_t)kSmallTok * kF * 4);
        for (void *p : ws.ptrs)
            if (!p) { ws.free_all(); cap_tok = 0; set_error("workspace allocation failed"); return DTTS_ERR_OOM; }
        bool ok = make_tmap_bf16(&t_conv, conv, T, kLat, 128) && make_tmap_bf16(&t_act, act, T, kD, 128) &&
                  make_tmap_bf16(&t_att, att, T, kD, 128) && make_tmap_bf16(&t_ffn, ffn, T, kF, 128) &&
                  make_tmap_bf16(&t_pairs, pairs, T / 2 > 0 ? T / 2 : 1, 2 * kD, 128) &&
                  make_tmap_f32_resid(&t_h, h, T, kD) && make_tmap_f32_resid(&t_qkv32, qkv32, kSmallTok, 3 * kD) &&
                  make_tmap_f32_resid(&t_ffn32, ffn32, kSmallTok, kF);
        DTTS_CHECK(ok, DTTS_ERR_CUDA, "tensor map (PatchEncoder workspace)");
        DTTS_CUDA(cudaMemsetAsync(qkv32, 0, (size_t)kSmallTok * 3 * kD * 4, stream));
        DTTS_CUDA(cudaMemsetAsync(ffn32, 0, (size_t)kSmallTok * kF * 4, stream));
        return DTTS_OK;
    }

    // every GEMM of a call follows another kernel: programmatic launch
    int gemm(GemmOp op) {
        launches++;
        op.pdl = 1;
        DTTS_CUDA(launch_gemm(op, num_sms, stream));
        return DTTS_OK;
    }

    // frames already in `this->frames` ([B][n_frames][128]); output in outf.
    // dev_pos: positions come from d_len (graph capture) instead of cur_len.
    int enqueue_append(int B, int n_frames, int pair_mode, bool dev_pos) {
        const int T = n_frames / 2, M = B * T, n_out = n_frames / 4;
        const bool small = (long long)M <= kSmallTok;
        const int bn = small ? kBNs : kBN;
        launches++;
        launch_pe_conv(frames, B, n_frames, tail[0], conv_w, conv_b, conv, tail[1], stream);
        // every kernel after the conv starts programmatically behind the one before it
        int st;
        {
            GemmOp op = op0(t_conv, small ? t_inw_s : t_inw, M, kD, kLat, EPI_F32, d_err);
            op.bn = bn;
            op.ep.bias = in_b; op.ep.out = h; op.ep.ldo = kD;
            if ((st = gemm(op))) return st;
        }
        const size_t layer_stride = (size_t)max_batch * max_tokens * kD;
        for (int l = 0; l < n_layers; l++) {
            const Layer &Ly = layers[l];
            launches++;
            launch_rms_norm(h, act, M, Ly.an, stream, true);
            if (small) {
                GemmOp op = op0(t_act, Ly.tqkv_s, M, 3 * kD, kD, EPI_RESID, d_err);
                op.bn = bn; op.tr = t_qkv32;
                op.ep.resid = qkv32; op.ep.ldr = 3 * kD; op.ep.ksplit = kKsQKV;
                if ((st = gemm(op))) return st;
                launches++;
                launch_k(pdl_enabled(), pe_qkv_finish_kernel, dim3(M), dim3(256), 0, stream, qkv32, T, cur_len,
                         (const int *)(dev_pos ? d_len : nullptr), (const float2 *)rope, q, kc + l * layer_stride,
                         vc + l * layer_stride, max_tokens);
            } else {
                GemmOp op = op0(t_act, Ly.tqkv, M, 3 * kD, kD, EPI_QKV, d_err);
                op.bn = bn;
                op.ep.q = q; op.ep.ldq = kD;
                op.ep.k = kc + l * layer_stride; op.ep.v = vc + l * layer_stride; op.ep.ldkv = kD;
                op.ep.tok_per_row = T; op.ep.kv_cap = max_tokens; op.ep.kv_start = cur_len;
                op.ep.kv_start_dev = dev_pos ? d_len : nullptr;
                op.ep.qk_norm = 0; op.ep.rope = rope; op.ep.rope_mode = ROPE_ADJACENT;
                if ((st = gemm(op))) return st;
            }
            {
                AttnArgs a{};
                a.q = q; a.ldq = kD; a.k = kc + l * layer_stride; a.v = vc + l * layer_stride; a.ldkv = kD;
                a.o = att; a.ldo = kD; a.rows = B; a.Tq = T; a.kv_len = cur_len + T; a.kv_cap = max_tokens;
                a.q_pos0 = cur_len; a.causal = 1; a.mask = nullptr; a.scale = 1.0f / sqrtf(64.0f);
                a.kv_base_dev = dev_pos ? d_len : nullptr;
                a.err = d_err;
                launches++;
                launch_attention_bf16(a, stream, true);
            }
            {
                GemmOp op = op0(t_att, small ? Ly.to_s : Ly.to, M, kD, kD, EPI_RESID, d_err);
                op.bn = bn;
                op.ep.ksplit = small ? kKsO : 1;
                op.tr = t_h;
                op.ep.bias = Ly.bo; op.ep.resid = h; op.ep.ldr = kD;
                if ((st = gemm(op))) return st;
            }
            launches++;
            launch_rms_norm(h, act, M, Ly.fn, stream, true);
            if (small) {
                GemmOp op = op0(t_act, Ly.t1_s, M, kF, kD, EPI_RESID, d_err);
                op.bn = bn; op.tr = t_ffn32;
                op.ep.bias = Ly.b1; op.ep.resid = ffn32; op.ep.ldr = kF; op.ep.ksplit = kKsF1;
                if ((st = gemm(op))) return st;
                launches++;
                const long long n4 = (long long)M * kF / 4;
                launch_k(pdl_enabled(), pe_silu_kernel, dim3((unsigned)((n4 + 255) / 256)), dim3(256), 0, stream,
                         ffn32, ffn, n4);
            } else {
                GemmOp op = op0(t_act, Ly.t1, M, kF, kD, EPI_SILU_BF16, d_err);
                op.ep.bias = Ly.b1; op.ep.out = ffn; op.ep.ldo = kF;
                if ((st = gemm(op))) return st;
            }
            {
                GemmOp op = op0(t_ffn, small ? Ly.t2_s : Ly.t2, M, kD, kF, EPI_RESID, d_err);
                op.bn = bn;
                op.ep.ksplit = small ? kKsF2 : 1;
                // prefill: the 8 KB-per-token activations are read once from DRAM,
                // not once per N pass (M-block-major tiles)
                op.ep.mb_major = small ? 0 : 1;
                op.tr = t_h;
                op.ep.bias = Ly.b2; op.ep.resid = h; op.ep.ldr = kD;
                if ((st = gemm(op))) return st;
            }
        }
        launches++;
        launch_pe_pairs(h, B, T, pair_mode, pairs, stream, true);
        {
            GemmOp op = op0(t_pairs, small ? t_outw_s : t_outw, B * n_out, kLLM, 2 * kD, EPI_F32, d_err);
            op.bn = bn;
            op.ep.bias = out_b; op.ep.out = outf; op.ep.ldo = kLLM;
            if ((st = gemm(op))) return st;
        }
        launches++;
        launch_advance_len(d_len, T, stream, true);
        DTTS_CUDA(cudaMemcpyAsync(tail[0], tail[1], (size_t)B * kLat * 4, cudaMemcpyDeviceToDevice, stream));
        DTTS_CUDA(cudaGetLastError());
        return DTTS_OK;
    }

    int finish(bool host_wait) {
        if (!host_wait) return DTTS_OK;
        int st = stream_wait(stream, 300.0);
        if (st) return st;
        int err = 0;
        DTTS_CUDA(cudaMemcpy(&err, d_err, 4, cudaMemcpyDeviceToHost));
        if (err) {
            // an abandoned call may leave partial sums in the split-K targets
            cudaMemset(d_err, 0, 4);
            if (qkv32) cudaMemset(qkv32, 0, (size_t)kSmallTok * 3 * kD * 4);
            if (ffn32) cudaMemset(ffn32, 0, (size_t)kSmallTok * kF * 4);
            set_error("device wait limit reached (code %d)", err);
            return DTTS_ERR_TIMEOUT;
        }
        return DTTS_OK;
    }

    int append(const float *frames_in, int B, int n_frames, int pair_mode, float *out, int mem) {
        DTTS_CHECK(frames_in && out, DTTS_ERR_ARG, "null argument");
        DTTS_CHECK(n_frames >= 4 && n_frames % 4 == 0, DTTS_ERR_ARG, "n_frames %d must be a positive multiple of 4", n_frames);
        DTTS_CHECK(B == cur_B && B >= 1, DTTS_ERR_ARG, "batch %d does not match the %d open streams", B, cur_B);
        DTTS_CHECK(cur_len + n_frames / 2 <= max_tokens, DTTS_ERR_ARG, "KV cache full (%d + %d > %d tokens)", cur_len,
                   n_frames / 2, max_tokens);
        DTTS_CHECK(mem == DTTS_MEM_HOST || mem == DTTS_MEM_DEVICE, DTTS_ERR_ARG, "bad mem kind");
        DeviceGuard g(device);
        const long long tok = (long long)B * (n_frames / 2);
        int st = ensure(tok);
        if (st) return st;
        const cudaMemcpyKind ik = mem == DTTS_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
        DTTS_CUDA(cudaMemcpyAsync(frames, frames_in, (size_t)B * n_frames * kLat * 4, ik, stream));
        if (tok <= kSmallTok && pair_mode == DTTS_PAIR_ADJACENT) {
            // decode step: one graph per (B, n_frames), positions from d_len
            cudaGraphExec_t exec = nullptr;
            for (Graph &g : graphs)
                if (g.B == B && g.n_frames == n_frames) exec = g.exec;
            if (!exec) {
                launches = 0;
                cudaGraph_t graph = nullptr;
                DTTS_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
                st = enqueue_append(B, n_frames, pair_mode, true);
                cudaError_t ce = cudaStreamEndCapture(stream, &graph);
                if (st) { if (graph) cudaGraphDestroy(graph); return st; }
                DTTS_CUDA(ce);
                ce = cudaGraphInstantiate(&exec, graph, 0);
                cudaGraphDestroy(graph);
                DTTS_CUDA(ce);
                graphs.push_back({B, n_frames, exec});
            }
            DTTS_CUDA(cudaGraphLaunch(exec, stream));
        } else {
            launches = 0;
            if ((st = enqueue_append(B, n_frames, pair_mode, false))) return st;
        }
        const cudaMemcpyKind ok = mem == DTTS_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
        DTTS_CUDA(cudaMemcpyAsync(out, outf, (size_t)B * (n_frames / 4) * kLLM * 4, ok, stream));
        cur_len += n_frames / 2;
        return finish(mem == DTTS_MEM_HOST);
    }
};

extern "C" {

int dtts_pe_create(const dtts_pe_weights *w, int dtype, int device, int max_batch, int max_tokens, dtts_pe **out) {
    DTTS_CHECK(w && out, DTTS_ERR_ARG, "null argument");
    *out = nullptr;
    DTTS_CHECK(w->n_layers >= 1 && w->n_layers <= 64 && w->layers, DTTS_ERR_ARG, "n_layers %d invalid", w->n_layers);
    DTTS_CHECK(max_batch >= 1 && max_tokens >= 2 && max_tokens <= 65536, DTTS_ERR_ARG, "bad capacity %d x %d",
               max_batch, max_tokens);
    DTTS_CHECK(dtype == DTTS_DTYPE_BF16, DTTS_ERR_UNSUPPORTED, "PatchEncoder dtype %d not supported", dtype);
    DTTS_CHECK(w->conv_w && w->in_w && w->out_w, DTTS_ERR_ARG, "missing a required PatchEncoder weight");
    for (int l = 0; l < w->n_layers; l++) {
        const dtts_pe_layer_weights &L = w->layers[l];
        DTTS_CHECK(L.wq && L.wk && L.wv && L.wo && L.w1 && L.w2, DTTS_ERR_ARG, "missing weight in layer %d", l);
    }
    int nsm = 0, st = check_device(device, &nsm);
    if (st) return st;
    DeviceGuard g(device);
    std::unique_ptr<dtts_pe> p(new dtts_pe());
    p->device = device; p->dtype = dtype; p->num_sms = nsm; p->n_layers = w->n_layers;
    p->max_batch = max_batch; p->max_tokens = max_tokens;
    DTTS_CUDA(cudaStreamCreateWithFlags(&p->own_stream, cudaStreamNonBlocking));
    p->stream = p->own_stream;
    DTTS_CUDA(gemm_prepare_attributes());
    DTTS_CUDA(attention_short_prepare());
    p->d_err = (int *)p->wts.alloc(4);
    DTTS_CHECK(p->d_err, DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemset(p->d_err, 0, 4));
    p->layers.resize(w->n_layers);
    for (int l = 0; l < w->n_layers; l++) {
        const dtts_pe_layer_weights &s = w->layers[l];
        dtts_pe::Layer &L = p->layers[l];
        if ((st = up_bf16(p->wts, {s.wq, s.wk, s.wv}, kD, kD, &L.wqkv))) return st;
        if ((st = up_bf16(p->wts, {s.wo}, kD, kD, &L.wo))) return st;
        if ((st = up_bf16(p->wts, {s.w1}, kF, kD, &L.w1))) return st;
        if ((st = up_bf16(p->wts, {s.w2}, kD, kF, &L.w2))) return st;
        if ((st = up_f32(p->wts, s.bo, kD, &L.bo))) return st;
        if ((st = up_f32(p->wts, s.b1, kF, &L.b1))) return st;
        if ((st = up_f32(p->wts, s.b2, kD, &L.b2))) return st;
        if ((st = up_f32(p->wts, s.attn_norm_w, kD, &L.an))) return st;
        if ((st = up_f32(p->wts, s.ffn_norm_w, kD, &L.fn))) return st;
        bool ok = make_tmap_bf16(&L.tqkv, L.wqkv, 3 * kD, kD, kBN) && make_tmap_bf16(&L.to, L.wo, kD, kD, kBN) &&
                  make_tmap_bf16(&L.t1, L.w1, kF, kD, kBN) && make_tmap_bf16(&L.t2, L.w2, kD, kF, kBN) &&
                  make_tmap_bf16(&L.tqkv_s, L.wqkv, 3 * kD, kD, kBNs) && make_tmap_bf16(&L.to_s, L.wo, kD, kD, kBNs) &&
                  make_tmap_bf16(&L.t1_s, L.w1, kF, kD, kBNs) && make_tmap_bf16(&L.t2_s, L.w2, kD, kF, kBNs);
        DTTS_CHECK(ok, DTTS_ERR_CUDA, "tensor map (PatchEncoder layer %d)", l);
    }
    {
        // ds conv weight [oc][ic][2] -> [ic][2][oc], read coalesced by pe_conv_kernel
        std::vector<float> wt((size_t)kLat * kLat * 2);
        for (int o = 0; o < kLat; o++)
            for (int i = 0; i < kLat; i++)
                for (int k = 0; k < 2; k++) wt[((size_t)i * 2 + k) * kLat + o] = w->conv_w[((size_t)o * kLat + i) * 2 + k];
        if ((st = up_f32(p->wts, wt.data(), wt.size(), &p->conv_w))) return st;
    }
    if ((st = up_f32(p->wts, w->conv_b, kLat, &p->conv_b))) return st;
    if ((st = up_bf16(p->wts, {w->in_w}, kD, kLat, &p->in_w))) return st;
    if ((st = up_f32(p->wts, w->in_b, kD, &p->in_b))) return st;
    if ((st = up_bf16(p->wts, {w->out_w}, kLLM, 2 * kD, &p->out_w))) return st;
    if ((st = up_f32(p->wts, w->out_b, kLLM, &p->out_b))) return st;
    bool ok = make_tmap_bf16(&p->t_inw, p->in_w, kD, kLat, kBN) && make_tmap_bf16(&p->t_outw, p->out_w, kLLM, 2 * kD, kBN) &&
              make_tmap_bf16(&p->t_inw_s, p->in_w, kD, kLat, kBNs) &&
              make_tmap_bf16(&p->t_outw_s, p->out_w, kLLM, 2 * kD, kBNs);
    DTTS_CHECK(ok, DTTS_ERR_CUDA, "tensor map (PatchEncoder projections)");
    // KV cache and conv tails
    const size_t cache_elems = (size_t)w->n_layers * max_batch * max_tokens * kD;
    p->kc = (bf16 *)p->cache.alloc(cache_elems * 2);
    p->vc = (bf16 *)p->cache.alloc(cache_elems * 2);
    p->tail[0] = (float *)p->cache.alloc((size_t)max_batch * kLat * 4);
    p->tail[1] = (float *)p->cache.alloc((size_t)max_batch * kLat * 4);
    p->rope = (float2 *)p->cache.alloc((size_t)max_tokens * 32 * sizeof(float2));
    p->d_len = (int *)p->cache.alloc(sizeof(int));
    DTTS_CHECK(p->kc && p->vc && p->tail[0] && p->tail[1] && p->rope && p->d_len, DTTS_ERR_OOM,
               "KV cache allocation failed (%zu MB)", cache_elems * 4 >> 20);
    // ggml_rope mode 0: theta starts at the position and is multiplied by
    // 1e4^(-2/64) for each successive adjacent pair.
    std::vector<float2> rt((size_t)max_tokens * 32);
    const float theta_scale = powf(10000.0f, -2.0f / 64.0f);
    for (int pos = 0; pos < max_tokens; pos++) {
        float theta = (float)pos;
        for (int i = 0; i < 32; i++) {
            rt[(size_t)pos * 32 + i] = make_float2(cosf(theta), sinf(theta));
            theta *= theta_scale;
        }
    }
    DTTS_CUDA(cudaMemcpy(p->rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice));
    *out = p.release();
    return DTTS_OK;
}

int dtts_pe_destroy(dtts_pe *p) {
    if (!p) return DTTS_OK;
    DeviceGuard g(p->device);
    cudaStreamSynchronize(p->stream);
    delete p;
    return DTTS_OK;
}

int dtts_pe_set_stream(dtts_pe *p, void *stream) {
    DTTS_CHECK(p, DTTS_ERR_ARG, "null engine");
    p->stream = stream ? static_cast<cudaStream_t>(stream) : p->own_stream;
    return DTTS_OK;
}

int dtts_pe_sync(dtts_pe *p) {
    DTTS_CHECK(p, DTTS_ERR_ARG, "null engine");
    DeviceGuard g(p->device);
    return p->finish(true);
}

int dtts_pe_stream_reset(dtts_pe *p, int B) {
    DTTS_CHECK(p, DTTS_ERR_ARG, "null engine");
    DTTS_CHECK(B >= 1 && B <= p->max_batch, DTTS_ERR_ARG, "batch %d out of [1, %d]", B, p->max_batch);
    DeviceGuard g(p->device);
    p->cur_B = B;
    p->cur_len = 0;
    // empty streams: zero conv tail (tap 2t-1 of the first token reads nothing)
    // and cache length 0, in stream order with the calls that follow
    DTTS_CUDA(cudaMemsetAsync(p->tail[0], 0, (size_t)p->max_batch * kLat * 4, p->stream));
    DTTS_CUDA(cudaMemsetAsync(p->d_len, 0, sizeof(int), p->stream));
    return DTTS_OK;
}

int dtts_pe_forward(dtts_pe *p, const float *frames, int B, int n_frames, int pair_mode, float *out, int mem) {
    DTTS_CHECK(p, DTTS_ERR_ARG, "null engine");
    DTTS_CHECK(pair_mode == DTTS_PAIR_ADJACENT || pair_mode == DTTS_PAIR_AS_WRITTEN, DTTS_ERR_ARG, "bad pair_mode");
    int st = dtts_pe_stream_reset(p, B);
    if (st) return st;
    return p->append(frames, B, n_frames, pair_mode, out, mem);
}

int dtts_pe_decode(dtts_pe *p, const float *frames, int B, int n_frames, float *out, int mem) {
    DTTS_CHECK(p, DTTS_ERR_ARG, "null engine");
    return p->append(frames, B, n_frames, DTTS_PAIR_ADJACENT, out, mem);
}

int dtts_pe_stream_length(dtts_pe *p, int *tokens) {
    DTTS_CHECK(p && tokens, DTTS_ERR_ARG, "null argument");
    *tokens = p->cur_len;
    return DTTS_OK;
}

}  // extern "C"
