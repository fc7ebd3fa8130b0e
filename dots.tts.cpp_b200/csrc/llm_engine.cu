// The LLM decoder step of the autoregressive loop (Qwen2.5-1.5B as run by
// src/llm_manual.cpp): llm_kv_cache_init (:237) over a prompt and
// llm_kv_cache_step (:342), one new embedding per sequence, on sm_100a for a
// batch of sequences advancing together.
//
// Per layer: RMSNorm (eps 1e-6, gain) -> q|k|v projection with biases
// (tcgen05 GEMM, fp32 out) -> RoPE (half-split pairs, theta 1e6, angle
// pos * theta_d with theta_d advanced by repeated multiplication) on q and k,
// k and v appended to a bf16 cache -> grouped-query attention (12 query heads
// over 2 key/value heads of 128, causal) -> o_proj (+bias) into the fp32
// residual -> RMSNorm -> gate|up projection -> SiLU(gate) * up -> down_proj
// into the residual; then the final RMSNorm.
#include "kernels.cuh"
#include "runtime.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <vector>

using namespace dtts;

namespace {

constexpr int kLH = 1536, kLF = 8960, kLNH = 12, kLNKV = 2, kLHD = 128, kLKV = kLNKV * kLHD;
constexpr int kLQKV = kLH + 2 * kLKV;   // 2048 columns: q | k | v

// ---------------------------------------------------------------- kernels
// RMSNorm of 1536-wide rows, one warp per row (manual_rms_norm,
// include/dit_manual.h:23-27): out = x / sqrt(mean(x^2) + 1e-6) * w.
template <bool OUT_BF16>
__global__ void __launch_bounds__(256) llm_rms_norm_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                           void *__restrict__ out, int M) {
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= M) return;
    const float4 *xr = reinterpret_cast<const float4 *>(x + (long long)row * kLH);
    float4 v[12];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 12; j++) {
        v[j] = xr[lane + 32 * j];
        ss += (v[j].x * v[j].x + v[j].y * v[j].y) + (v[j].z * v[j].z + v[j].w * v[j].w);
    }
    const float inv = 1.0f / sqrtf(warp_sum(ss) / (float)kLH + 1e-6f);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
#pragma unroll
    for (int j = 0; j < 12; j++) {
        const int c4 = lane + 32 * j;
        const float4 g = w ? __ldg(w4 + c4) : make_float4(1.f, 1.f, 1.f, 1.f);
        const float4 o = make_float4(v[j].x * inv * g.x, v[j].y * inv * g.y, v[j].z * inv * g.z, v[j].w * inv * g.w);
        if constexpr (OUT_BF16)
            reinterpret_cast<uint2 *>(out)[(long long)row * (kLH / 4) + c4] = make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
        else
            reinterpret_cast<float4 *>(out)[(long long)row * (kLH / 4) + c4] = o;
    }
}

// RoPE on q (12 heads) and k (2 heads) of token m = b * T + t at position
// pos0 + t, q to qout (fp32), k and v appended to the caches
// [b][kv head][cap][128] (bf16).  One block of 256 threads per token; work
// item i < 14 * 64 rotates pair (d, d + 64), d = i % 64, of q/k head i / 64,
// and the 256 v values follow.  pos_dev, if set, holds pos0 on the device
// (graph-captured steps); zero: each qkv value is cleared by the thread that
// read it (the next split-K reduce-add target).
__global__ void __launch_bounds__(256) llm_rope_cache_kernel(float *__restrict__ qkv, int T, int pos0,
                                                              const int *__restrict__ pos_dev,
                                                              const float2 *__restrict__ rope, float *__restrict__ qout,
                                                              bf16 *__restrict__ kc, bf16 *__restrict__ vc, int cap,
                                                              int zero) {
    pdl_wait();
    pdl_trigger();
    if (pos_dev) pos0 = *pos_dev;
    const int m = blockIdx.x, b = m / T, t = m % T, p = pos0 + t;
    float *row = qkv + (long long)m * kLQKV;
    constexpr int kRot = (kLNH + kLNKV) * 64;
    for (int i = threadIdx.x; i < kRot + kLKV; i += blockDim.x) {
        if (i < kRot) {
            const int hh = i >> 6, d = i & 63;
            const int c = hh * kLHD + d;   // q heads, then k heads (columns 1536..1791)
            const float2 cs = rope[(long long)p * 64 + d];
            const float x0 = row[c], x1 = row[c + 64];
            if (zero) row[c] = row[c + 64] = 0.f;
            const float y0 = x0 * cs.x - x1 * cs.y, y1 = x1 * cs.x + x0 * cs.y;
            if (hh < kLNH) {
                qout[(long long)m * kLH + c] = y0;
                qout[(long long)m * kLH + c + 64] = y1;
            } else {
                bf16 *dst = kc + (((long long)b * kLNKV + (hh - kLNH)) * cap + p) * kLHD;
                dst[d] = __float2bfloat16_rn(y0);
                dst[d + 64] = __float2bfloat16_rn(y1);
            }
        } else {
            const int j = i - kRot, hv = j >> 7, d = j & 127;
            const float x = row[kLH + kLKV + j];
            if (zero) row[kLH + kLKV + j] = 0.f;
            vc[(((long long)b * kLNKV + hv) * cap + p) * kLHD + d] = __float2bfloat16_rn(x);
        }
    }
}

// Grouped-query causal attention, one warp per (token m, query head): the
// lanes form two groups of 16 (g = lane / 16); lane c of group g owns dims
// 8c .. 8c+7 of key 2u + g, so each 16-byte load instruction reads two whole
// 256-byte K (or V) rows and a score needs a 4-step shuffle within the group.
// Keys 0 .. pos0 + t of the token's sequence, 16 per round; online softmax in
// fp32 (scores pre-scaled by log2(e) / sqrt(128), exp2); the two groups' P.V
// are merged at the end; the output row goes to ao (bf16, the o_proj input).
__global__ void __launch_bounds__(256, 2) llm_attn_kernel(const float *__restrict__ q, const bf16 *__restrict__ kc,
                                                       const bf16 *__restrict__ vc, int T, int pos0,
                                                       const int *__restrict__ pos_dev, int cap, int M,
                                                       bf16 *__restrict__ ao) {
    pdl_wait();
    pdl_trigger();
    if (pos_dev) pos0 = *pos_dev;
    const int wid = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (wid >= M * kLNH) return;
    const int m = wid / kLNH, h = wid % kLNH, b = m / T, t = m % T;
    const int kvh = h * kLNKV / kLNH;
    const int g = lane >> 4, c = lane & 15;
    const int n_keys = pos0 + t + 1;
    const float sc = 1.4426950408889634f / sqrtf((float)kLHD);
    float qv[8];
    {
        const float4 *q4 = reinterpret_cast<const float4 *>(q + (long long)m * kLH + h * kLHD + 8 * c);
        const float4 a = q4[0], bq = q4[1];
        qv[0] = a.x * sc; qv[1] = a.y * sc; qv[2] = a.z * sc; qv[3] = a.w * sc;
        qv[4] = bq.x * sc; qv[5] = bq.y * sc; qv[6] = bq.z * sc; qv[7] = bq.w * sc;
    }
    const bf16 *kb = kc + ((long long)b * kLNKV + kvh) * cap * kLHD + 8 * c;
    const bf16 *vb = vc + ((long long)b * kLNKV + kvh) * cap * kLHD + 8 * c;
    constexpr int U = 8;   // key pairs per round
    float mx = -INFINITY, l = 0.f, acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = 0.f;
    for (int j0 = 0; j0 < n_keys; j0 += 2 * U) {
        uint4 kr[U], vr[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = min(j0 + 2 * u + g, n_keys - 1);   // past the end: a valid row, masked below
            kr[u] = *reinterpret_cast<const uint4 *>(kb + (long long)j * kLHD);
            vr[u] = *reinterpret_cast<const uint4 *>(vb + (long long)j * kLHD);
        }
        float sv[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const uint32_t w[4] = {kr[u].x, kr[u].y, kr[u].z, kr[u].w};
            float d = 0.f;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                // bf16 pair -> two floats by bit placement (exact)
                d = fmaf(qv[2 * i], __uint_as_float(w[i] << 16), d);
                d = fmaf(qv[2 * i + 1], __uint_as_float(w[i] & 0xFFFF0000u), d);
            }
            sv[u] = d;
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1)
#pragma unroll
            for (int u = 0; u < U; u++) sv[u] += __shfl_xor_sync(0xffffffffu, sv[u], o);
        float bm = mx;
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (j0 + 2 * u + g >= n_keys) sv[u] = -INFINITY;
            bm = fmaxf(bm, sv[u]);
        }
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 16));
        const float corr = exp2f(mx - bm);
        l *= corr;
#pragma unroll
        for (int i = 0; i < 8; i++) acc[i] *= corr;
#pragma unroll
        for (int u = 0; u < U; u++) {
            const float p = exp2f(sv[u] - bm);
            l += p;
            const uint32_t w[4] = {vr[u].x, vr[u].y, vr[u].z, vr[u].w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                acc[2 * i] = fmaf(p, __uint_as_float(w[i] << 16), acc[2 * i]);
                acc[2 * i + 1] = fmaf(p, __uint_as_float(w[i] & 0xFFFF0000u), acc[2 * i + 1]);
            }
        }
        mx = bm;
    }
    // merge the two key groups (lanes c and c + 16)
    l += __shfl_xor_sync(0xffffffffu, l, 16);
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 16);
    if (g == 0) {
        const float inv = 1.0f / l;
        reinterpret_cast<uint4 *>(ao + (long long)m * kLH + h * kLHD)[c] =
            make_uint4(pack_bf16x2(acc[0] * inv, acc[1] * inv), pack_bf16x2(acc[2] * inv, acc[3] * inv),
                       pack_bf16x2(acc[4] * inv, acc[5] * inv), pack_bf16x2(acc[6] * inv, acc[7] * inv));
    }
}

// out[m][j] = gate / (1 + e^-gate) * up with gu[m] = gate[8960] | up[8960]
// (src/llm_manual.cpp:333-334, :468), four columns per thread; zero: gu is
// cleared behind the read.
__global__ void llm_swiglu_kernel(float *__restrict__ gu, bf16 *__restrict__ out, long long n4, int zero) {
    pdl_wait();
    pdl_trigger();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const long long m = i / (kLF / 4), j4 = i % (kLF / 4);
    float4 *g4 = reinterpret_cast<float4 *>(gu + m * 2 * kLF) + j4;
    float4 *u4 = reinterpret_cast<float4 *>(gu + m * 2 * kLF + kLF) + j4;
    const float4 g = *g4, u = *u4;
    if (zero) *g4 = *u4 = make_float4(0.f, 0.f, 0.f, 0.f);
    reinterpret_cast<uint2 *>(out)[i] =
        make_uint2(pack_bf16x2(g.x / (1.0f + expf(-g.x)) * u.x, g.y / (1.0f + expf(-g.y)) * u.y),
                   pack_bf16x2(g.z / (1.0f + expf(-g.z)) * u.z, g.w / (1.0f + expf(-g.w)) * u.w));
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

// row-concatenation of parts (rows_i x cols fp32) uploaded as bf16
int up_bf16(DeviceArena &a, const std::vector<std::pair<const float *, size_t>> &parts, size_t cols, bf16 **out) {
    size_t rows = 0;
    for (auto &p : parts) rows += p.second;
    std::vector<uint16_t> tmp(rows * cols);
    size_t r0 = 0;
    for (auto &p : parts) {
        f32_to_bf16_host(p.first, tmp.data() + r0 * cols, p.second * cols);
        r0 += p.second;
    }
    void *d = a.alloc(tmp.size() * 2);
    DTTS_CHECK(d, DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemcpy(d, tmp.data(), tmp.size() * 2, cudaMemcpyHostToDevice));
    *out = (bf16 *)d;
    return DTTS_OK;
}

}  // namespace

struct dtts_llm {
    int device = 0, num_sms = 148, n_layers = 0, max_batch = 0, max_seq = 0;
    cudaStream_t own_stream = nullptr, stream = nullptr;
    DeviceArena wts, cache, ws;
    struct Layer {
        bf16 *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wd = nullptr;
        float *bqkv = nullptr, *bo = nullptr, *an = nullptr, *fn = nullptr;
        CUtensorMap tqkv, to, tgu, td;             // 256-row boxes
        CUtensorMap tqkv_s, to_s, tgu_s, td_s;     // 128-row boxes (small batches)
    };
    std::vector<Layer> layers;
    float *final_norm = nullptr;
    bf16 *kc = nullptr, *vc = nullptr;   // [n_layers][max_batch][2][max_seq][128]
    float2 *rope = nullptr;              // [max_seq][64]
    int *d_len = nullptr;                // cache length on the device (graph-captured steps)
    int *d_err = nullptr;
    // step graphs, one per batch size; dropped when the workspace moves
    struct Graph { int B; cudaGraphExec_t exec; };
    std::vector<Graph> graphs;
    void drop_graphs() {
        for (Graph &g : graphs) cudaGraphExecDestroy(g.exec);
        graphs.clear();
    }
    int cur_B = 0, cur_len = 0;
    long long cap_tok = 0;
    float *h = nullptr, *qkv = nullptr, *q = nullptr, *gu = nullptr;
    bf16 *act = nullptr, *ao = nullptr, *ffn = nullptr;
    CUtensorMap t_act, t_ao, t_ffn, t_h, t_qkv_r, t_gu_r;   // *_r: fp32 reduce-add targets

    ~dtts_llm() {
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
        h = (float *)ws.alloc(T * kLH * 4);
        qkv = (float *)ws.alloc(T * kLQKV * 4);
        q = (float *)ws.alloc(T * kLH * 4);
        gu = (float *)ws.alloc(T * 2 * kLF * 4);
        act = (bf16 *)ws.alloc(T * kLH * 2);
        ao = (bf16 *)ws.alloc(T * kLH * 2);
        ffn = (bf16 *)ws.alloc(T * kLF * 2);
        DTTS_CHECK(h && qkv && q && gu && act && ao && ffn, DTTS_ERR_OOM, "LLM workspace allocation failed");
        bool ok = make_tmap_bf16(&t_act, act, T, kLH, 128) && make_tmap_bf16(&t_ao, ao, T, kLH, 128) &&
                  make_tmap_bf16(&t_ffn, ffn, T, kLF, 128) && make_tmap_f32_resid(&t_h, h, T, kLH) &&
                  make_tmap_f32_resid(&t_qkv_r, qkv, T, kLQKV) && make_tmap_f32_resid(&t_gu_r, gu, T, 2 * kLF);
        DTTS_CHECK(ok, DTTS_ERR_CUDA, "tensor map (LLM workspace)");
        return DTTS_OK;
    }

    GemmOp op(const CUtensorMap &ta, const CUtensorMap &tb, int M, int N, int K, int epi, int bn) {
        GemmOp o;
        std::memset(&o, 0, sizeof(o));
        o.ta = ta; o.tb = tb; o.M = M; o.N = N; o.K = K; o.bn = bn; o.nw = 4; o.epi = epi;
        o.ep.err = d_err; o.ep.tok_per_row = 1; o.ep.ksplit = 1;
        o.pdl = 1;   // every GEMM follows another kernel
        return o;
    }

    // emb already in h ([B * T][1536]); runs every layer and the final norm into
    // `out`, then advances d_len; dev_pos: positions from d_len, not pos0
    int enqueue(int B, int T, int pos0, bool dev_pos, float *out) {
        const int *pd = dev_pos ? d_len : nullptr;
        const int M = B * T;
        const bool small = M <= 256;
        const int bn = small ? 128 : 256;
        const size_t layer_stride = (size_t)max_batch * kLNKV * max_seq * kLHD;
        // few rows: the QKV and gate|up GEMMs split K so that about 128 CTAs
        // stream the weights, partial sums reduce-added into fp32 rows that are
        // zeroed here once and then by their readers behind each read
        if (small) {
            DTTS_CUDA(cudaMemsetAsync(qkv, 0, (size_t)M * kLQKV * 4, stream));
            DTTS_CUDA(cudaMemsetAsync(gu, 0, (size_t)M * 2 * kLF * 4, stream));
        }
        // every kernel but the first starts programmatically behind the one before it
        const bool pdl = pdl_enabled();
        for (int l = 0; l < n_layers; l++) {
            const Layer &L = layers[l];
            launch_k(pdl && l > 0, llm_rms_norm_kernel<true>, dim3((M + 7) / 8), dim3(256), 0, stream,
                     (const float *)h, (const float *)L.an, (void *)act, M);
            if (small) {
                GemmOp o = op(t_act, L.tqkv_s, M, kLQKV, kLH, EPI_RESID, bn);
                o.tr = t_qkv_r; o.ep.bias = L.bqkv; o.ep.resid = qkv; o.ep.ldr = kLQKV; o.ep.ksplit = 8;
                DTTS_CUDA(launch_gemm(o, num_sms, stream));
            } else {
                GemmOp o = op(t_act, L.tqkv, M, kLQKV, kLH, EPI_F32, bn);
                o.ep.bias = L.bqkv; o.ep.out = qkv; o.ep.ldo = kLQKV;
                DTTS_CUDA(launch_gemm(o, num_sms, stream));
            }
            launch_k(pdl, llm_rope_cache_kernel, dim3(M), dim3(256), 0, stream, qkv, T, pos0, pd, (const float2 *)rope,
                     q, kc + l * layer_stride, vc + l * layer_stride, max_seq, small ? 1 : 0);
            launch_k(pdl, llm_attn_kernel, dim3((M * kLNH + 7) / 8), dim3(256), 0, stream, (const float *)q,
                     (const bf16 *)(kc + l * layer_stride), (const bf16 *)(vc + l * layer_stride), T, pos0, pd,
                     max_seq, M, ao);
            {
                GemmOp o = op(t_ao, small ? L.to_s : L.to, M, kLH, kLH, EPI_RESID, bn);
                o.tr = t_h; o.ep.bias = L.bo; o.ep.resid = h; o.ep.ldr = kLH;
                o.ep.ksplit = small ? 8 : 1;
                DTTS_CUDA(launch_gemm(o, num_sms, stream));
            }
            launch_k(pdl, llm_rms_norm_kernel<true>, dim3((M + 7) / 8), dim3(256), 0, stream, (const float *)h,
                     (const float *)L.fn, (void *)act, M);
            if (small) {
                GemmOp o = op(t_act, L.tgu_s, M, 2 * kLF, kLH, EPI_RESID, bn);
                o.tr = t_gu_r; o.ep.resid = gu; o.ep.ldr = 2 * kLF; o.ep.ksplit = 2;
                DTTS_CUDA(launch_gemm(o, num_sms, stream));
            } else {
                GemmOp o = op(t_act, L.tgu, M, 2 * kLF, kLH, EPI_F32, bn);
                o.ep.out = gu; o.ep.ldo = 2 * kLF;
                DTTS_CUDA(launch_gemm(o, num_sms, stream));
            }
            const long long nf4 = (long long)M * kLF / 4;
            launch_k(pdl, llm_swiglu_kernel, dim3((unsigned)((nf4 + 255) / 256)), dim3(256), 0, stream, gu, ffn, nf4,
                     small ? 1 : 0);
            {
                GemmOp o = op(t_ffn, small ? L.td_s : L.td, M, kLH, kLF, EPI_RESID, bn);
                o.tr = t_h; o.ep.resid = h; o.ep.ldr = kLH;
                o.ep.ksplit = small ? 10 : 1;
                // prefill: the 17.5 KB-per-token activations are read once from DRAM,
                // not once per N pass (M-block-major tiles)
                o.ep.mb_major = small ? 0 : 1;
                DTTS_CUDA(launch_gemm(o, num_sms, stream));
            }
        }
        launch_k(pdl, llm_rms_norm_kernel<false>, dim3((M + 7) / 8), dim3(256), 0, stream, (const float *)h,
                 (const float *)final_norm, (void *)out, M);
        launch_advance_len(d_len, T, stream, true);
        DTTS_CUDA(cudaGetLastError());
        return DTTS_OK;
    }

    int run(const float *emb, int B, int T, float *hidden, int mem) {
        DTTS_CHECK(emb && hidden, DTTS_ERR_ARG, "null argument");
        DTTS_CHECK(mem == DTTS_MEM_HOST || mem == DTTS_MEM_DEVICE, DTTS_ERR_ARG, "bad mem kind");
        DTTS_CHECK(cur_len + T <= max_seq, DTTS_ERR_ARG, "KV cache full (%d + %d > %d tokens)", cur_len, T, max_seq);
        DeviceGuard g(device);
        const long long M = (long long)B * T;
        int st = ensure(M + 1);
        if (st) return st;
        // the final norm writes into qkv's space (fp32, at least M x 1536), then out
        float *outd = qkv;
        DTTS_CUDA(cudaMemcpyAsync(h, emb, (size_t)M * kLH * 4,
                                  mem == DTTS_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, stream));
        if (T == 1) {
            // decode step: one graph per batch size, positions from d_len
            cudaGraphExec_t exec = nullptr;
            for (Graph &g : graphs)
                if (g.B == B) exec = g.exec;
            if (!exec) {
                cudaGraph_t graph = nullptr;
                DTTS_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
                st = enqueue(B, 1, 0, true, outd);
                cudaError_t ce = cudaStreamEndCapture(stream, &graph);
                if (st) { if (graph) cudaGraphDestroy(graph); return st; }
                DTTS_CUDA(ce);
                ce = cudaGraphInstantiate(&exec, graph, 0);
                cudaGraphDestroy(graph);
                DTTS_CUDA(ce);
                graphs.push_back({B, exec});
            }
            DTTS_CUDA(cudaGraphLaunch(exec, stream));
        } else if ((st = enqueue(B, T, cur_len, false, outd))) {
            return st;
        }
        DTTS_CUDA(cudaMemcpyAsync(hidden, outd, (size_t)M * kLH * 4,
                                  mem == DTTS_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, stream));
        cur_len += T;
        if (mem != DTTS_MEM_HOST) return DTTS_OK;
        if ((st = stream_wait(stream, 300.0))) return st;
        int err = 0;
        DTTS_CUDA(cudaMemcpy(&err, d_err, 4, cudaMemcpyDeviceToHost));
        if (err) { cudaMemset(d_err, 0, 4); set_error("device wait limit reached (code %d)", err); return DTTS_ERR_TIMEOUT; }
        return DTTS_OK;
    }
};

extern "C" {

int dtts_llm_create(const dtts_llm_weights *w, int device, int max_batch, int max_seq, dtts_llm **out) {
    DTTS_CHECK(w && out, DTTS_ERR_ARG, "null argument");
    *out = nullptr;
    DTTS_CHECK(w->n_layers >= 1 && w->n_layers <= 64 && w->layers && w->final_norm, DTTS_ERR_ARG,
               "n_layers %d invalid or final norm missing", w->n_layers);
    DTTS_CHECK(max_batch >= 1 && max_seq >= 1 && max_seq <= 32768, DTTS_ERR_ARG, "bad capacity %d x %d", max_batch,
               max_seq);
    for (int l = 0; l < w->n_layers; l++) {
        const dtts_llm_layer_weights &L = w->layers[l];
        DTTS_CHECK(L.qw && L.kw && L.vw && L.ow && L.gw && L.uw && L.dw, DTTS_ERR_ARG, "missing weight in layer %d", l);
    }
    int nsm = 0, st = check_device(device, &nsm);
    if (st) return st;
    DeviceGuard g(device);
    std::unique_ptr<dtts_llm> e(new dtts_llm());
    e->device = device; e->num_sms = nsm; e->n_layers = w->n_layers; e->max_batch = max_batch; e->max_seq = max_seq;
    DTTS_CUDA(cudaStreamCreateWithFlags(&e->own_stream, cudaStreamNonBlocking));
    e->stream = e->own_stream;
    DTTS_CUDA(gemm_prepare_attributes());
    e->d_err = (int *)e->wts.alloc(4);
    DTTS_CHECK(e->d_err, DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemset(e->d_err, 0, 4));
    e->layers.resize(w->n_layers);
    std::vector<float> bqkv(kLQKV);
    for (int l = 0; l < w->n_layers; l++) {
        const dtts_llm_layer_weights &s = w->layers[l];
        dtts_llm::Layer &L = e->layers[l];
        if ((st = up_bf16(e->wts, {{s.qw, kLH}, {s.kw, kLKV}, {s.vw, kLKV}}, kLH, &L.wqkv))) return st;
        if ((st = up_bf16(e->wts, {{s.ow, kLH}}, kLH, &L.wo))) return st;
        if ((st = up_bf16(e->wts, {{s.gw, kLF}, {s.uw, kLF}}, kLH, &L.wgu))) return st;
        if ((st = up_bf16(e->wts, {{s.dw, kLH}}, kLF, &L.wd))) return st;
        std::fill(bqkv.begin(), bqkv.end(), 0.f);
        if (s.qb) std::memcpy(bqkv.data(), s.qb, kLH * 4);
        if (s.kb) std::memcpy(bqkv.data() + kLH, s.kb, kLKV * 4);
        if (s.vb) std::memcpy(bqkv.data() + kLH + kLKV, s.vb, kLKV * 4);
        if ((st = up_f32(e->wts, bqkv.data(), kLQKV, &L.bqkv))) return st;
        if ((st = up_f32(e->wts, s.ob, kLH, &L.bo))) return st;
        if ((st = up_f32(e->wts, s.an, kLH, &L.an))) return st;
        if ((st = up_f32(e->wts, s.fn, kLH, &L.fn))) return st;
        bool ok = make_tmap_bf16(&L.tqkv, L.wqkv, kLQKV, kLH, 256) && make_tmap_bf16(&L.to, L.wo, kLH, kLH, 256) &&
                  make_tmap_bf16(&L.tgu, L.wgu, 2 * kLF, kLH, 256) && make_tmap_bf16(&L.td, L.wd, kLH, kLF, 256) &&
                  make_tmap_bf16(&L.tqkv_s, L.wqkv, kLQKV, kLH, 128) && make_tmap_bf16(&L.to_s, L.wo, kLH, kLH, 128) &&
                  make_tmap_bf16(&L.tgu_s, L.wgu, 2 * kLF, kLH, 128) && make_tmap_bf16(&L.td_s, L.wd, kLH, kLF, 128);
        DTTS_CHECK(ok, DTTS_ERR_CUDA, "tensor map (LLM layer %d)", l);
    }
    if ((st = up_f32(e->wts, w->final_norm, kLH, &e->final_norm))) return st;
    const size_t cache_elems = (size_t)w->n_layers * max_batch * kLNKV * max_seq * kLHD;
    e->kc = (bf16 *)e->cache.alloc(cache_elems * 2);
    e->vc = (bf16 *)e->cache.alloc(cache_elems * 2);
    e->rope = (float2 *)e->cache.alloc((size_t)max_seq * 64 * sizeof(float2));
    e->d_len = (int *)e->cache.alloc(sizeof(int));
    DTTS_CHECK(e->kc && e->vc && e->rope && e->d_len, DTTS_ERR_OOM, "LLM KV cache allocation failed (%zu MB)", cache_elems * 4 >> 20);
    // (cos, sin)(pos * theta_d), theta_d = (1e6^(-2/128))^d by repeated
    // multiplication, as src/llm_manual.cpp:398-403 and :449-451 compute them
    std::vector<float2> rt((size_t)max_seq * 64);
    const float ts = powf(1000000.0f, -2.0f / (float)kLHD);
    for (int p = 0; p < max_seq; p++) {
        float theta = 1.0f;
        for (int d = 0; d < 64; d++) {
            rt[(size_t)p * 64 + d] = make_float2(cosf((float)p * theta), sinf((float)p * theta));
            theta *= ts;
        }
    }
    DTTS_CUDA(cudaMemcpy(e->rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice));
    *out = e.release();
    return DTTS_OK;
}

int dtts_llm_destroy(dtts_llm *e) {
    if (!e) return DTTS_OK;
    DeviceGuard g(e->device);
    cudaStreamSynchronize(e->stream);
    delete e;
    return DTTS_OK;
}

int dtts_llm_set_stream(dtts_llm *e, void *stream) {
    DTTS_CHECK(e, DTTS_ERR_ARG, "null engine");
    e->stream = stream ? static_cast<cudaStream_t>(stream) : e->own_stream;
    return DTTS_OK;
}

int dtts_llm_prefill(dtts_llm *e, const float *emb, int B, int n_tok, float *hidden, int mem) {
    DTTS_CHECK(e, DTTS_ERR_ARG, "null engine");
    DTTS_CHECK(B >= 1 && B <= e->max_batch && n_tok >= 1, DTTS_ERR_ARG, "bad prefill shape %d x %d", B, n_tok);
    DeviceGuard g(e->device);
    e->cur_B = B;
    e->cur_len = 0;
    DTTS_CUDA(cudaMemsetAsync(e->d_len, 0, sizeof(int), e->stream));
    return e->run(emb, B, n_tok, hidden, mem);
}

int dtts_llm_step(dtts_llm *e, const float *emb, int B, float *hidden, int mem) {
    DTTS_CHECK(e, DTTS_ERR_ARG, "null engine");
    DTTS_CHECK(B == e->cur_B && e->cur_len > 0, DTTS_ERR_ARG, "step needs a prefill of the same %d sequences", B);
    return e->run(emb, B, 1, hidden, mem);
}

int dtts_llm_length(dtts_llm *e, int *tokens) {
    DTTS_CHECK(e && tokens, DTTS_ERR_ARG, "null argument");
    *tokens = e->cur_len;
    return DTTS_OK;
}

}  // extern "C"
