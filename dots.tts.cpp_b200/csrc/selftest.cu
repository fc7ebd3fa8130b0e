// Self-test entry points: run one engine kernel in isolation on host data so
// tests can check it against a CPU reference (bf16 rounding is applied to the
// inputs on the host, exactly as the engine stores them).
#include "kernels.cuh"
#include "runtime.h"

#include <cstring>
#include <vector>

using namespace dtts;

namespace {
struct Scratch {
    DeviceArena a;
    ~Scratch() { a.free_all(); }
};

// One thread waits on an mbarrier that nothing arrives at, through the same
// bounded wait every GEMM wait uses: after the limit it records the code in
// the error word, raises the abort flag and returns.
__global__ void wait_limit_selftest_kernel(int *err) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) (void)mbar_wait(&bar, 0, &abort_flag, err, DEVERR_TIMEOUT_PRODUCER);
    __syncthreads();
}
}  // namespace

extern "C" {

// C[M][N] = A[M][K] B[N][K]^T (+ bias[N]) through the tcgen05 GEMM kernel with
// the fp32-output epilogue; bn = 64, 128, 192 or 256.
int dtts_selftest_gemm(const float *A, const float *B, const float *bias, float *C, int M, int N, int K, int bn,
                       int device) {
    DTTS_CHECK(A && B && C, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(M >= 1 && K >= 64 && K % 64 == 0 && (bn == 64 || bn == 128 || bn == 192 || bn == 256) && N % bn == 0,
               DTTS_ERR_ARG, "bad GEMM shape M=%d N=%d K=%d bn=%d", M, N, K, bn);
    int nsm = 0, st = check_device(device, &nsm);
    if (st) return st;
    DeviceGuard g(device);
    DTTS_CUDA(gemm_prepare_attributes());
    Scratch s;
    std::vector<uint16_t> ha((size_t)M * K), hb((size_t)N * K);
    f32_to_bf16_host(A, ha.data(), ha.size());
    f32_to_bf16_host(B, hb.data(), hb.size());
    void *da = s.a.alloc(ha.size() * 2), *db = s.a.alloc(hb.size() * 2), *dc = s.a.alloc((size_t)M * N * 4);
    void *dbias = bias ? s.a.alloc((size_t)N * 4) : nullptr;
    int *derr = (int *)s.a.alloc(4);
    DTTS_CHECK(da && db && dc && derr && (!bias || dbias), DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemcpy(da, ha.data(), ha.size() * 2, cudaMemcpyHostToDevice));
    DTTS_CUDA(cudaMemcpy(db, hb.data(), hb.size() * 2, cudaMemcpyHostToDevice));
    if (bias) DTTS_CUDA(cudaMemcpy(dbias, bias, (size_t)N * 4, cudaMemcpyHostToDevice));
    DTTS_CUDA(cudaMemset(dc, 0xff, (size_t)M * N * 4));
    DTTS_CUDA(cudaMemset(derr, 0, 4));
    GemmOp op;
    std::memset(&op, 0, sizeof(op));
    bool ok = make_tmap_bf16(&op.ta, da, M, K, 128) && make_tmap_bf16(&op.tb, db, N, K, bn);
    DTTS_CHECK(ok, DTTS_ERR_CUDA, "tensor map encode failed");
    op.M = M; op.N = N; op.K = K; op.bn = bn; op.epi = EPI_F32;
    op.ep.out = dc; op.ep.ldo = N; op.ep.bias = (const float *)dbias; op.ep.err = derr; op.ep.tok_per_row = 1;
    DTTS_CUDA(launch_gemm(op, nsm, 0));
    if ((st = stream_wait(0, 60.0))) return st;
    int err = 0;
    DTTS_CUDA(cudaMemcpy(&err, derr, 4, cudaMemcpyDeviceToHost));
    DTTS_CHECK(err == 0, DTTS_ERR_TIMEOUT, "GEMM kernel wait limit reached (code %d)", err);
    DTTS_CUDA(cudaMemcpy(C, dc, (size_t)M * N * 4, cudaMemcpyDeviceToHost));
    return DTTS_OK;
}

// C[M][N] = a_scale[m] b_scale[n] (A[M][K] B[N][K]^T) (+ bias[N]) with e4m3
// A and B (bytes) through the kind::f8f6f4 GEMM; bn = 128 or 256, K % 128 == 0.
int dtts_selftest_gemm_e4m3(const uint8_t *A, const float *a_scale, const uint8_t *B, const float *b_scale,
                            const float *bias, float *C, int M, int N, int K, int bn, int device) {
    DTTS_CHECK(A && a_scale && B && b_scale && C, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(M >= 1 && K >= 128 && K % 128 == 0 && (bn == 128 || bn == 256) && N % bn == 0, DTTS_ERR_ARG,
               "bad GEMM shape M=%d N=%d K=%d bn=%d", M, N, K, bn);
    int nsm = 0, st = check_device(device, &nsm);
    if (st) return st;
    DeviceGuard g(device);
    DTTS_CUDA(gemm_prepare_attributes());
    Scratch s;
    void *da = s.a.alloc((size_t)M * K), *db = s.a.alloc((size_t)N * K), *dc = s.a.alloc((size_t)M * N * 4);
    float *dsa = (float *)s.a.alloc((size_t)M * 4), *dsb = (float *)s.a.alloc((size_t)N * 4);
    void *dbias = bias ? s.a.alloc((size_t)N * 4) : nullptr;
    int *derr = (int *)s.a.alloc(4);
    DTTS_CHECK(da && db && dc && dsa && dsb && derr && (!bias || dbias), DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemcpy(da, A, (size_t)M * K, cudaMemcpyHostToDevice));
    DTTS_CUDA(cudaMemcpy(db, B, (size_t)N * K, cudaMemcpyHostToDevice));
    DTTS_CUDA(cudaMemcpy(dsa, a_scale, (size_t)M * 4, cudaMemcpyHostToDevice));
    DTTS_CUDA(cudaMemcpy(dsb, b_scale, (size_t)N * 4, cudaMemcpyHostToDevice));
    if (bias) DTTS_CUDA(cudaMemcpy(dbias, bias, (size_t)N * 4, cudaMemcpyHostToDevice));
    DTTS_CUDA(cudaMemset(dc, 0xff, (size_t)M * N * 4));
    DTTS_CUDA(cudaMemset(derr, 0, 4));
    GemmOp op;
    std::memset(&op, 0, sizeof(op));
    bool ok = make_tmap_e4m3(&op.ta, da, M, K, 128) && make_tmap_e4m3(&op.tb, db, N, K, bn);
    DTTS_CHECK(ok, DTTS_ERR_CUDA, "tensor map encode failed");
    op.M = M; op.N = N; op.K = K; op.bn = bn; op.epi = EPI_F32; op.f8 = 1;
    op.ep.out = dc; op.ep.ldo = N; op.ep.bias = (const float *)dbias; op.ep.err = derr; op.ep.tok_per_row = 1;
    op.ep.row_scale = dsa; op.ep.col_scale = dsb;
    DTTS_CUDA(launch_gemm(op, nsm, 0));
    if ((st = stream_wait(0, 60.0))) return st;
    int err = 0;
    DTTS_CUDA(cudaMemcpy(&err, derr, 4, cudaMemcpyDeviceToHost));
    DTTS_CHECK(err == 0, DTTS_ERR_TIMEOUT, "GEMM kernel wait limit reached (code %d)", err);
    DTTS_CUDA(cudaMemcpy(C, dc, (size_t)M * N * 4, cudaMemcpyDeviceToHost));
    return DTTS_OK;
}

// Attention core alone: q [rows][Tq][1024], k/v [rows][kv_len][1024] (fp32,
// rounded to bf16 on upload), out [rows][Tq][1024] fp32.  mask [Tq][kv_len] or
// NULL; causal with the first query at absolute position q_pos0.
int dtts_selftest_attention(const float *q, const float *k, const float *v, float *out, int rows, int Tq,
                            int kv_len, const uint8_t *mask, int causal, int q_pos0, int use_f32, int device) {
    DTTS_CHECK(q && k && v && out, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(rows >= 1 && Tq >= 1 && kv_len >= 1, DTTS_ERR_ARG, "bad attention shape");
    int nsm = 0, st = check_device(device, &nsm);
    if (st) return st;
    DeviceGuard g(device);
    Scratch s;
    const size_t nq = (size_t)rows * Tq * kD, nk = (size_t)rows * kv_len * kD;
    const size_t esz = use_f32 ? 4 : 2;
    void *dq = s.a.alloc(nq * esz), *dk = s.a.alloc(nk * esz), *dv = s.a.alloc(nk * esz), *dout = s.a.alloc(nq * esz);
    void *dm = mask ? s.a.alloc((size_t)Tq * kv_len) : nullptr;
    const int mw = (kv_len + 31) / 32;
    void *dbits = mask ? s.a.alloc((size_t)Tq * mw * 4) : nullptr;
    DTTS_CHECK(dq && dk && dv && dout && (!mask || (dm && dbits)), DTTS_ERR_OOM, "cudaMalloc failed");
    if (use_f32) {
        DTTS_CUDA(attention_f32_prepare());
        DTTS_CUDA(cudaMemcpy(dq, q, nq * 4, cudaMemcpyHostToDevice));
        DTTS_CUDA(cudaMemcpy(dk, k, nk * 4, cudaMemcpyHostToDevice));
        DTTS_CUDA(cudaMemcpy(dv, v, nk * 4, cudaMemcpyHostToDevice));
    } else {
        DTTS_CUDA(attention_short_prepare());
        std::vector<uint16_t> t(std::max(nq, nk));
        f32_to_bf16_host(q, t.data(), nq);
        DTTS_CUDA(cudaMemcpy(dq, t.data(), nq * 2, cudaMemcpyHostToDevice));
        f32_to_bf16_host(k, t.data(), nk);
        DTTS_CUDA(cudaMemcpy(dk, t.data(), nk * 2, cudaMemcpyHostToDevice));
        f32_to_bf16_host(v, t.data(), nk);
        DTTS_CUDA(cudaMemcpy(dv, t.data(), nk * 2, cudaMemcpyHostToDevice));
    }
    if (mask) {
        DTTS_CUDA(cudaMemcpy(dm, mask, (size_t)Tq * kv_len, cudaMemcpyHostToDevice));
        std::vector<uint32_t> bits((size_t)Tq * mw);
        pack_mask_bits(mask, Tq, kv_len, bits.data());
        DTTS_CUDA(cudaMemcpy(dbits, bits.data(), bits.size() * 4, cudaMemcpyHostToDevice));
    }
    AttnArgs a{};
    a.q = dq; a.k = dk; a.v = dv; a.o = dout; a.ldq = a.ldkv = a.ldo = kD;
    a.rows = rows; a.Tq = Tq; a.kv_len = kv_len; a.kv_cap = kv_len; a.q_pos0 = q_pos0; a.causal = causal;
    a.mask = (const uint8_t *)dm; a.mask_bits = (const uint32_t *)dbits; a.scale = 0.125f;
    if (use_f32) DTTS_CUDA(launch_attention_f32(a, 0));
    else launch_attention_bf16(a, 0);
    DTTS_CUDA(cudaGetLastError());
    if ((st = stream_wait(0, 60.0))) return st;
    if (use_f32) {
        DTTS_CUDA(cudaMemcpy(out, dout, nq * 4, cudaMemcpyDeviceToHost));
    } else {
        std::vector<uint16_t> t(nq);
        DTTS_CUDA(cudaMemcpy(t.data(), dout, nq * 2, cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < nq; i++) { uint32_t u = (uint32_t)t[i] << 16; std::memcpy(&out[i], &u, 4); }
    }
    return DTTS_OK;
}

// Time convolution through the GEMM over taps (EpiParams::tap_*):
// out[t][o] = bias[o] + sum_k sum_c x[t + k dil - pad_left][c] w[o][c][k], rows
// outside [0, T) zero; x [T][C] and w [N][C][K] rounded to bf16 as the engine
// stores them; C % 64 == 0.
int dtts_selftest_conv(const float *x, int T, int C, const float *w, const float *bias, int N, int K, int dil,
                       int pad_left, int bn, float *out, int device) {
    DTTS_CHECK(x && w && out, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(T >= 1 && C >= 64 && C % 64 == 0 && K >= 1 && K <= 32 && dil >= 1 && pad_left >= 0 &&
                   (bn == 64 || bn == 128 || bn == 192 || bn == 256) && N % bn == 0,
               DTTS_ERR_ARG, "bad conv shape T=%d C=%d N=%d K=%d bn=%d", T, C, N, K, bn);
    int nsm = 0, st = check_device(device, &nsm);
    if (st) return st;
    DeviceGuard g(device);
    DTTS_CUDA(gemm_prepare_attributes());
    Scratch s;
    std::vector<float> bop((size_t)N * K * C);
    for (int o = 0; o < N; o++)
        for (int c = 0; c < C; c++)
            for (int k = 0; k < K; k++) bop[((size_t)o * K + k) * C + c] = w[((size_t)o * C + c) * K + k];
    std::vector<uint16_t> ha((size_t)T * C), hb(bop.size());
    f32_to_bf16_host(x, ha.data(), ha.size());
    f32_to_bf16_host(bop.data(), hb.data(), hb.size());
    void *da = s.a.alloc(ha.size() * 2), *db = s.a.alloc(hb.size() * 2), *dc = s.a.alloc((size_t)T * N * 4);
    void *dbias = bias ? s.a.alloc((size_t)N * 4) : nullptr;
    int *derr = (int *)s.a.alloc(4);
    DTTS_CHECK(da && db && dc && derr && (!bias || dbias), DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemcpy(da, ha.data(), ha.size() * 2, cudaMemcpyHostToDevice));
    DTTS_CUDA(cudaMemcpy(db, hb.data(), hb.size() * 2, cudaMemcpyHostToDevice));
    if (bias) DTTS_CUDA(cudaMemcpy(dbias, bias, (size_t)N * 4, cudaMemcpyHostToDevice));
    DTTS_CUDA(cudaMemset(derr, 0, 4));
    GemmOp op;
    std::memset(&op, 0, sizeof(op));
    bool ok = make_tmap_bf16(&op.ta, da, T, C, 128) && make_tmap_bf16(&op.tb, db, N, (size_t)K * C, bn);
    DTTS_CHECK(ok, DTTS_ERR_CUDA, "tensor map encode failed");
    op.M = T; op.N = N; op.K = K * C; op.bn = bn; op.nw = 4; op.epi = EPI_F32;
    op.ep.out = dc; op.ep.ldo = N; op.ep.bias = (const float *)dbias; op.ep.err = derr; op.ep.tok_per_row = 1;
    op.ep.tap_kb = C / 64; op.ep.tap_base = -pad_left; op.ep.tap_step = dil;
    DTTS_CUDA(launch_gemm(op, nsm, 0));
    if ((st = stream_wait(0, 60.0))) return st;
    int err = 0;
    DTTS_CUDA(cudaMemcpy(&err, derr, 4, cudaMemcpyDeviceToHost));
    DTTS_CHECK(err == 0, DTTS_ERR_TIMEOUT, "GEMM kernel wait limit reached (code %d)", err);
    DTTS_CUDA(cudaMemcpy(out, dc, (size_t)T * N * 4, cudaMemcpyDeviceToHost));
    return DTTS_OK;
}

int dtts_selftest_wait_limit(int device, int *code) {
    DTTS_CHECK(code, DTTS_ERR_ARG, "null argument");
    *code = 0;
    int nsm = 0, st = check_device(device, &nsm);
    if (st) return st;
    DeviceGuard g(device);
    Scratch s;
    int *derr = (int *)s.a.alloc(4);
    DTTS_CHECK(derr, DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemset(derr, 0, 4));
    wait_limit_selftest_kernel<<<1, 32>>>(derr);
    DTTS_CUDA(cudaGetLastError());
    if ((st = stream_wait(0, 30.0))) return st;
    DTTS_CUDA(cudaMemcpy(code, derr, 4, cudaMemcpyDeviceToHost));
    if (*code) {
        set_error("device wait limit reached (code %d)", *code);
        return DTTS_ERR_TIMEOUT;
    }
    return DTTS_OK;
}

int dtts_selftest_e4m3(const float *x, uint8_t *out, int n, int device) {
    DTTS_CHECK(x && out && n >= 1, DTTS_ERR_ARG, "bad e4m3 self-test arguments");
    int nsm = 0, st = check_device(device, &nsm);
    if (st) return st;
    DeviceGuard g(device);
    Scratch s;
    float *dx = (float *)s.a.alloc((size_t)n * 4);
    uint8_t *dy = (uint8_t *)s.a.alloc((size_t)n);
    DTTS_CHECK(dx && dy, DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemcpy(dx, x, (size_t)n * 4, cudaMemcpyHostToDevice));
    launch_e4m3_selftest(dx, dy, n, 0);
    DTTS_CUDA(cudaGetLastError());
    DTTS_CUDA(cudaDeviceSynchronize());
    DTTS_CUDA(cudaMemcpy(out, dy, (size_t)n, cudaMemcpyDeviceToHost));
    return DTTS_OK;
}

}  // extern "C"
