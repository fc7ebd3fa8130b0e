// BigVGAN v2 decoder (src/modules/vocoder/bigvgan_cpp.cpp:325-542 and
// lstm.cpp of the reference) on sm_100a.
//
// Layout: every activation is time-major [time][channels], channels padded to
// a multiple of 64 (at least 64) with zeros that stay zero: padded weights
// and biases are zero and SnakeBeta(0) = 0.
//   bottleneck   post_proj, Linear 128->512, 4 x LSTM(512) with skip,
//                Linear 512->128: fp32 SIMT GEMMs + one cooperative kernel
//                running the four LSTM layers as a dataflow wavefront (per-step
//                counters, T + 3 dependent steps)
//   conv_pre     K = 5, centred: tcgen05 GEMM over taps (bf16 out)
//   6 stages     causal ConvTranspose1d (K = 2 stride) as `stride` GEMMs, one
//                per output phase r: out[q s + r] = W_r . [x[q] | x[q-1]],
//                written with row stride s; then three AMP blocks, each
//                r += c2(act(c1(act(r)))) x 3 with dilations 1, 3, 5:
//                act = Activation1d (fp32 in, bf16 out), c1 a GEMM over taps
//                (fp32 out + bias), c2 a GEMM over taps reduce-added into the
//                fp32 residual r (+ bias); the stage output is the mean of
//                the three blocks
//   post         Activation1d with per-channel filters, conv_post (K = 7,
//                causal, no bias), tanh x 1.92
// The convolution GEMMs read A = activations through a 2-D tensor map whose
// rows outside [0, T) are TMA zero fill, shifted per tap (EpiParams::tap_*),
// so causal padding costs nothing.
#include "kernels.cuh"
#include "runtime.h"

#include <cmath>
#include <cstring>
#include <memory>
#include <vector>

using namespace dtts;

namespace {
constexpr int kStages = 6, kRb = 18, kTaps = 12;
constexpr int kUpIn[kStages] = {1536, 768, 384, 192, 96, 48};
constexpr int kUpOut[kStages] = {768, 384, 192, 96, 48, 24};
constexpr int kUpStride[kStages] = {10, 6, 4, 2, 2, 2};
constexpr int kRbK[3] = {3, 7, 11};
constexpr int kRbDil[3] = {1, 3, 5};
constexpr int kHop = 1920;
constexpr int kLstmH = 512, kLstmCtas = 64, kLstmUnits = kLstmH / kLstmCtas;   // CTAs per layer, 8 units each
constexpr size_t kLstmSmem = (32 * kLstmH + 2 * kLstmH + 32) * sizeof(float);

inline int cpad(int c) { return c <= 64 ? 64 : (c + 63) / 64 * 64; }

// ------------------------------------------------------------------ filter
// BigVGAN's kaiser_sinc_filter1d (the alias-free activation's low-pass
// filter): Kaiser window with beta from the attenuation
// A = 2.285 (K/2 - 1) pi (4 half_width) + 7.95, sinc sampled at half-integer
// times for even K, taps normalised to sum 1.  The reference hard-codes the
// K = 12, cutoff 0.25, half width 0.3 result (bigvgan_cpp.cpp:27-31).
constexpr double kPi = 3.14159265358979323846;

double bessel_i0(double x) {
    double term = 1.0, sum = 1.0;
    for (int k = 1; k < 200; k++) {
        term *= (x / (2.0 * k)) * (x / (2.0 * k));
        sum += term;
        if (term < 1e-17 * sum) break;
    }
    return sum;
}

void kaiser_sinc(float *f, double cutoff, double half_width, int K) {
    const int half = K / 2;
    const double A = 2.285 * (half - 1) * kPi * (4.0 * half_width) + 7.95;
    const double beta = A > 50.0 ? 0.1102 * (A - 8.7) : A >= 21.0 ? 0.5842 * pow(A - 21.0, 0.4) + 0.07886 * (A - 21.0) : 0.0;
    std::vector<double> v(K);
    double sum = 0.0;
    for (int n = 0; n < K; n++) {
        const double r = 2.0 * n / (K - 1) - 1.0;
        const double win = bessel_i0(beta * sqrt(std::max(0.0, 1.0 - r * r))) / bessel_i0(beta);
        const double t = (K % 2 == 0) ? (n - half + 0.5) : (n - half);
        const double x = 2.0 * cutoff * t;
        const double sinc = x == 0.0 ? 1.0 : sin(kPi * x) / (kPi * x);
        v[n] = 2.0 * cutoff * win * sinc;
        sum += v[n];
    }
    for (int n = 0; n < K; n++) f[n] = (float)(v[n] / sum);
}

// ------------------------------------------------------------------ kernels
// Activation1d (bigvgan_cpp.cpp:33-124).  A warp takes 32 channels (one per
// lane) and 16 consecutive output times t_w .. t_w + 15, entirely in
// registers:
//   x[i]  = x at t_w - 11 + i, i < 27 (zero before t = 0)
//   s[i]  = SnakeBeta(u) at j = 2 t_w - 11 + i, i < 43, where
//           u[j] = 2 sum_q f_up[2q + (j mod 2)] x[floor(j / 2) - q], q < 6
//           (ConvTranspose1d x2 trimmed to 2T; x before 0 contributes 0);
//           s at j < 0 is s at j = 0 (the replicate pad of the down filter)
//   out[t_w + o] = sum_k f_down[k] s[2o + k]           (conv1d, stride 2)
// SnakeBeta: u + sin^2(a u) inv_b with a = e^clamp(alpha), inv_b =
// 1 / (e^clamp(beta) + 1e-9); a non-finite u gives 0, a non-finite result u.
// sin is the hardware approximation (__sinf: absolute error about 1e-6 for
// |a u| < 10).  Lanes of channels >= ch write zeros.
constexpr int kActTW = 16, kActWarps = 8;
struct ActArgs {
    const float *x; int ldx;
    void *y; int ldy; int y_bf16;
    int T, ch;
    const float *a, *inv_b;          // [ch]: e^clamp(alpha), 1 / (e^clamp(beta) + 1e-9)
    const float *fu, *fd; int fch;   // [fch][12]
};

__device__ __forceinline__ float snake(float u, float a, float ib) {
    if (!isfinite(u)) return 0.f;
    const float sn = __sinf(a * u);
    const float v = fmaf(ib * sn, sn, u);
    return isfinite(v) ? v : u;
}

__global__ void __launch_bounds__(kActWarps * 32) voc_act_kernel(const ActArgs p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x * 32 + lane;
    const int tw = (blockIdx.y * kActWarps + warp) * kActTW;
    if (tw >= p.T) return;
    const bool live = c < p.ch;
    const int n_out = min(kActTW, p.T - tw);
    float o[kActTW];
    if (__any_sync(0xffffffffu, live)) {
        float fu[kTaps], fd[kTaps];
        const float *fup = p.fu + (p.fch == 1 ? 0 : (long long)(live ? c : 0) * kTaps);
        const float *fdp = p.fd + (p.fch == 1 ? 0 : (long long)(live ? c : 0) * kTaps);
#pragma unroll
        for (int k = 0; k < kTaps; k++) { fu[k] = __ldg(fup + k); fd[k] = __ldg(fdp + k); }
        const float a = live ? __ldg(p.a + c) : 1.f, ib = live ? __ldg(p.inv_b + c) : 1.f;
        float x[kActTW + 11];
#pragma unroll
        for (int i = 0; i < kActTW + 11; i++) {
            const int t = tw - 11 + i;
            x[i] = (live && t >= 0 && t < p.T) ? __ldg(p.x + (long long)t * p.ldx + c) : 0.f;
        }
        float s[2 * kActTW + 11];
#pragma unroll
        for (int i = 0; i < 2 * kActTW + 11; i++) {
            // j = 2 t_w - 11 + i is odd for even i: taps 1, 3, .., 11 on x[i/2 + 5 - q];
            // even for odd i: taps 0, 2, .., 10 on x[(i - 1)/2 + 6 - q]
            float u = 0.f;
#pragma unroll
            for (int q = 0; q < 6; q++) {
                if (i % 2 == 0) u = fmaf(x[i / 2 + 5 - q], fu[2 * q + 1], u);
                else u = fmaf(x[(i - 1) / 2 + 6 - q], fu[2 * q], u);
            }
            s[i] = snake(2.0f * u, a, ib);
        }
        if (tw == 0) {
#pragma unroll
            for (int i = 0; i < 11; i++) s[i] = s[11];   // j < 0: replicate s[0]
        }
#pragma unroll
        for (int q = 0; q < kActTW; q++) {
            float v = 0.f;
#pragma unroll
            for (int k = 0; k < kTaps; k++) v = fmaf(s[2 * q + k], fd[k], v);
            o[q] = live ? v : 0.f;
        }
    } else {
#pragma unroll
        for (int q = 0; q < kActTW; q++) o[q] = 0.f;
    }
    if (c >= p.ldy) return;
#pragma unroll
    for (int q = 0; q < kActTW; q++) {
        if (q >= n_out) break;
        const long long off = (long long)(tw + q) * p.ldy + c;
        if (p.y_bf16) reinterpret_cast<bf16 *>(p.y)[off] = __float2bfloat16_rn(o[q]);
        else reinterpret_cast<float *>(p.y)[off] = o[q];
    }
}

void launch_act(const ActArgs &p, int cp, cudaStream_t s) {
    dim3 grid((cp + 31) / 32, (p.T + kActTW * kActWarps - 1) / (kActTW * kActWarps));
    voc_act_kernel<<<grid, kActWarps * 32, 0, s>>>(p);
}

// x = (r0 + r1 + r2) / 3 (bigvgan_cpp.cpp:485-494), as bf16 and optionally fp32
__global__ void voc_mean3_kernel(const float4 *__restrict__ r0, const float4 *__restrict__ r1,
                                 const float4 *__restrict__ r2, uint2 *__restrict__ xb, float4 *__restrict__ xf,
                                 long long n4) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const float4 a = r0[i], b = r1[i], c = r2[i];
    const float4 m = make_float4((a.x + b.x + c.x) / 3.0f, (a.y + b.y + c.y) / 3.0f, (a.z + b.z + c.z) / 3.0f,
                                 (a.w + b.w + c.w) / 3.0f);
    if (xb) xb[i] = make_uint2(pack_bf16x2(m.x, m.y), pack_bf16x2(m.z, m.w));
    if (xf) xf[i] = m;
}

// conv_post (Conv1d(24, 1, 7), causal, no bias) and tanh x 1.92
// (bigvgan_cpp.cpp:509-521): a block stages rows t0-6 .. t0+255 of the first
// 24 channels in shared memory, then one thread per output sample.
constexpr int kPostT = 256;
__global__ void __launch_bounds__(kPostT) voc_post_kernel(const float *__restrict__ x, int ldx, int T,
                                                          const float *__restrict__ w, float *__restrict__ audio) {
    __shared__ float xs[kPostT + 6][24];
    __shared__ float ws[24 * 7];
    const int t0 = blockIdx.x * kPostT;
    for (int i = threadIdx.x; i < (kPostT + 6) * 24; i += kPostT) {
        const int r = i / 24, c = i % 24, t = t0 - 6 + r;
        xs[r][c] = (t >= 0 && t < T) ? x[(long long)t * ldx + c] : 0.f;
    }
    if (threadIdx.x < 24 * 7) ws[threadIdx.x] = w[threadIdx.x];
    __syncthreads();
    const int t = t0 + threadIdx.x;
    if (t >= T) return;
    float s = 0.f;
    for (int k = 0; k < 7; k++)
        for (int c = 0; c < 24; c++) s += xs[threadIdx.x + k][c] * ws[c * 7 + k];
    audio[t] = tanhf(s) * 1.92f;
}

// The 4-layer LSTM (lstm.cpp:12-104) as a dataflow wavefront: CTA b serves
// layer l = b / 64 and hidden units 8 (b mod 64) .. +7; it keeps their 32 W_hh
// rows (gates i, f, g, o) in shared memory, and layers 1..3 read their 32 W_ih
// rows from global memory (L2-resident) each step.  Layer 0's input
// projection (x W_ih^T + b_ih + b_hh for every t) is precomputed in gin0.
// Step t of layer l waits until all 64 CTAs of layer l have published h^l[t-1]
// and all 64 of layer l-1 have published h^(l-1)[t] (counters cnt[l][t],
// incremented after each CTA's write; bounded wait, error code on expiry), so
// the layers advance together without a global barrier: T + 3 dependent steps
// instead of 4 T.  Launched cooperatively (all CTAs resident).

struct LstmArgs {
    const float *gin0;                 // [T][2048] layer-0 input projection + biases
    const float *w_ih[4], *w_hh[4];    // [2048][512]
    const float *b_g[4];               // [2048] b_ih + b_hh
    float *h;                          // [4][T][512]
    int T;
    unsigned *cnt;                     // [4][T] CTAs that published h^l[t], zero at launch
    int *err;
};

__global__ void __launch_bounds__(256) voc_lstm_kernel(const LstmArgs p) {
    extern __shared__ float sm[];
    float *w = sm;                        // [32][512] W_hh rows of this CTA
    float *hs = sm + 32 * kLstmH;         // h^l[t-1]
    float *xs = hs + kLstmH;              // h^(l-1)[t]
    float *gs = xs + kLstmH;              // [32] gate pre-activations
    __shared__ int abort_flag;
    const int l = blockIdx.x / kLstmCtas, q0 = (blockIdx.x % kLstmCtas) * kLstmUnits;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float *whh = p.w_hh[l], *wih = p.w_ih[l];
    for (int i = tid; i < 32 * kLstmH; i += 256) {
        const int r = i / kLstmH, k = i % kLstmH;   // r = gate * 8 + unit
        w[i] = whh[(long long)((r >> 3) * kLstmH + q0 + (r & 7)) * kLstmH + k];
    }
    if (tid == 0) abort_flag = 0;
    float cst = 0.f;
    float *hl = p.h + (long long)l * p.T * kLstmH;
    const float *hprev_layer = l ? p.h + (long long)(l - 1) * p.T * kLstmH : nullptr;
    for (int t = 0; t < p.T; t++) {
        if (tid == 0) {
            const unsigned *need0 = t ? p.cnt + (long long)l * p.T + (t - 1) : nullptr;
            const unsigned *need1 = l ? p.cnt + (long long)(l - 1) * p.T + t : nullptr;
            const unsigned long long t0 = globaltimer_ns();
            while ((need0 && ld_acquire_u32(need0) < (unsigned)kLstmCtas) ||
                   (need1 && ld_acquire_u32(need1) < (unsigned)kLstmCtas)) {
                if (globaltimer_ns() - t0 > kWaitLimitNs) {
                    atomicExch(p.err, DEVERR_TIMEOUT_BARRIER);
                    abort_flag = 1;
                    break;
                }
            }
        }
        __syncthreads();
        if (abort_flag) return;
        for (int k = tid; k < kLstmH; k += 256) {
            hs[k] = t ? __ldcg(hl + (long long)(t - 1) * kLstmH + k) : 0.f;
            if (l) xs[k] = __ldcg(hprev_layer + (long long)t * kLstmH + k);
        }
        __syncthreads();
        // warp w: rows 4w .. 4w+3, their W_ih loads all issued together
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        int grow[4];
#pragma unroll
        for (int qq = 0; qq < 4; qq++) {
            const int r = warp * 4 + qq;
            grow[qq] = (r >> 3) * kLstmH + q0 + (r & 7);
        }
        if (l) {
#pragma unroll
            for (int k = lane; k < kLstmH; k += 32) {
                const float xv = xs[k];
#pragma unroll
                for (int qq = 0; qq < 4; qq++) acc[qq] += __ldg(wih + (long long)grow[qq] * kLstmH + k) * xv;
            }
        }
#pragma unroll
        for (int k = lane; k < kLstmH; k += 32) {
            const float hv = hs[k];
#pragma unroll
            for (int qq = 0; qq < 4; qq++) acc[qq] += w[(warp * 4 + qq) * kLstmH + k] * hv;
        }
#pragma unroll
        for (int qq = 0; qq < 4; qq++) {
            const float v = warp_sum(acc[qq]);
            if (lane == 0)
                gs[warp * 4 + qq] = v + (l ? __ldg(p.b_g[l] + grow[qq]) : p.gin0[(long long)t * 4 * kLstmH + grow[qq]]);
        }
        __syncthreads();
        if (tid < kLstmUnits) {
            const float gi = gs[tid], gf = gs[8 + tid], gg = gs[16 + tid], go = gs[24 + tid];
            const float iv = 1.0f / (1.0f + expf(-gi)), fv = 1.0f / (1.0f + expf(-gf));
            const float gv = tanhf(gg), ov = 1.0f / (1.0f + expf(-go));
            cst = fv * cst + iv * gv;
            hl[(long long)t * kLstmH + q0 + tid] = ov * tanhf(cst);
        }
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            atomicAdd(p.cnt + (long long)l * p.T + t, 1u);   // this CTA's units of h^l[t] are out
        }
    }
}

// ------------------------------------------------------------------ host helpers
int up_f32(DeviceArena &a, const float *h, size_t n, float **out) {
    *out = nullptr;
    void *d = a.alloc(n * 4);
    DTTS_CHECK(d, DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemcpy(d, h, n * 4, cudaMemcpyHostToDevice));
    *out = (float *)d;
    return DTTS_OK;
}

// zero-padded copy of a [n] vector to [np]
int up_f32_pad(DeviceArena &a, const float *h, size_t n, size_t np, float **out) {
    std::vector<float> v(np, 0.f);
    if (h) std::memcpy(v.data(), h, n * 4);
    return up_f32(a, v.data(), np, out);
}

int up_bf16(DeviceArena &a, const std::vector<float> &v, bf16 **out) {
    std::vector<uint16_t> tmp(v.size());
    f32_to_bf16_host(v.data(), tmp.data(), v.size());
    void *d = a.alloc(tmp.size() * 2);
    DTTS_CHECK(d, DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemcpy(d, tmp.data(), tmp.size() * 2, cudaMemcpyHostToDevice));
    *out = (bf16 *)d;
    return DTTS_OK;
}

// Activation constants: a = e^clamp(alpha, +-20), inv_b = 1 / (e^clamp(beta, +-20) + 1e-9),
// in float as the reference evaluates them (bigvgan_cpp.cpp:103-110); padded channels 1, 1.
void snake_consts(const float *alpha, const float *beta, int ch, int cp, std::vector<float> &a, std::vector<float> &ib) {
    a.assign(cp, 1.f);
    ib.assign(cp, 1.f);
    for (int c = 0; c < ch; c++) {
        float al = alpha ? alpha[c] : 1.0f, be = beta ? beta[c] : 1.0f;
        // no alpha/beta tensor: the reference uses 1 and still exponentiates (log scale)
        al = expf(al > 20.0f ? 20.0f : (al < -20.0f ? -20.0f : al));
        be = expf(be > 20.0f ? 20.0f : (be < -20.0f ? -20.0f : be));
        a[c] = al;
        ib[c] = 1.0f / (be + 1e-9f);
    }
}

GemmOp conv_op(const CUtensorMap &ta, const CUtensorMap &tb, int M, int N, int K, int epi, int bn, int *err) {
    GemmOp op;
    std::memset(&op, 0, sizeof(op));
    op.ta = ta; op.tb = tb; op.M = M; op.N = N; op.K = K; op.bn = bn; op.nw = 4; op.epi = epi;
    op.ep.err = err; op.ep.tok_per_row = 1; op.ep.ksplit = 1;
    return op;
}
}  // namespace

struct dtts_voc {
    int device = 0, num_sms = 148, max_frames = 0;
    cudaStream_t own_stream = nullptr, stream = nullptr;
    // the three AMP blocks of a stage are independent until their mean: blocks
    // 1 and 2 run on side streams, forked from and joined back into `stream`
    cudaStream_t side[2] = {nullptr, nullptr};
    cudaEvent_t ev_fork = nullptr, ev_join[2] = {nullptr, nullptr};
    DeviceArena wts, ws;
    int *d_err = nullptr;
    unsigned *d_cnt = nullptr;   // [4][max_frames] LSTM step counters
    // bottleneck (fp32)
    float *pp_w = nullptr, *pp_b = nullptr, *mi_w1 = nullptr, *mi_b1 = nullptr, *mi_w2 = nullptr, *mi_b2 = nullptr;
    float *w_ih[4] = {}, *w_hh[4] = {}, *b_g[4] = {};
    // convolutions (bf16 B operands [N][taps * cp_in]) and biases (fp32, padded)
    bf16 *w_pre = nullptr; float *b_pre = nullptr; CUtensorMap t_pre;
    bf16 *w_up[kStages] = {}; float *b_up[kStages] = {};
    CUtensorMap t_up[kStages][2];                         // all phases stacked along N; boxes of 64 / 128 rows
    bf16 *w_c1[kRb][3] = {}, *w_c2[kRb][3] = {};
    float *b_c1[kRb][3] = {}, *b_c2[kRb][3] = {};
    CUtensorMap t_c1[kRb][3][3], t_c2[kRb][3][3];          // boxes of 64 / 128 / 192 rows (tile widths)
    float *act_a[kRb][6] = {}, *act_ib[kRb][6] = {};
    float *aa = nullptr;                                  // [12] AMP filter
    float *post_a = nullptr, *post_ib = nullptr, *post_fu = nullptr, *post_fd = nullptr, *post_w = nullptr;
    // workspace
    float *lat = nullptr, *pp = nullptr, *z = nullptr, *gin = nullptr, *hl = nullptr, *sk = nullptr, *bott = nullptr;
    float *audio = nullptr;
    bf16 *bott16 = nullptr, *x0 = nullptr;                // conv_pre in / out
    float *r[3] = {}, *y[3] = {}, *xf = nullptr;          // stage buffers (one residual + scratch per block), fp32
    bf16 *a16[3] = {}, *xin = nullptr;                    // GEMM A operands
    size_t stage_elems = 0;
    int maps_T0 = -1;                                     // n_frames the activation maps were encoded for
    CUtensorMap t_bott, t_x0, t_xin[kStages], t_a[kStages][3], t_r[kStages][3];

    ~dtts_voc() {
        ws.free_all();
        wts.free_all();
        for (int i = 0; i < 2; i++) {
            if (side[i]) cudaStreamDestroy(side[i]);
            if (ev_join[i]) cudaEventDestroy(ev_join[i]);
        }
        if (ev_fork) cudaEventDestroy(ev_fork);
        if (own_stream) cudaStreamDestroy(own_stream);
    }

    // the widest tile (192 or 128) that still gives every SM a tile (the three
    // AMP blocks run concurrently); else 64
    int bn_for(long long M, int N) const {
        const long long mt = (M + 127) / 128;
        if (N % 192 == 0 && N % 128 != 0 && mt * (N / 192) * 3 >= num_sms) return 192;
        if (N % 128 == 0 && mt * (N / 128) * 3 >= num_sms) return 128;
        return 64;
    }

    int alloc_ws() {
        const size_t F = (size_t)max_frames;
        size_t mx = 0;
        for (int s = 0; s < kStages; s++) {
            size_t T = F;
            for (int q = 0; q <= s; q++) T *= kUpStride[q];
            mx = std::max(mx, T * (size_t)cpad(kUpOut[s]));
        }
        stage_elems = mx;
        lat = (float *)ws.alloc(F * 128 * 4);
        pp = (float *)ws.alloc(F * 128 * 4);
        z = (float *)ws.alloc(F * kLstmH * 4);
        gin = (float *)ws.alloc(F * 4 * kLstmH * 4);
        hl = (float *)ws.alloc(4 * F * kLstmH * 4);
        sk = (float *)ws.alloc(F * kLstmH * 4);
        bott = (float *)ws.alloc(F * 128 * 4);
        bott16 = (bf16 *)ws.alloc(F * 128 * 2);
        x0 = (bf16 *)ws.alloc(F * 1536 * 2);
        for (int j = 0; j < 3; j++) r[j] = (float *)ws.alloc(mx * 4);
        for (int j = 0; j < 3; j++) {
            y[j] = (float *)ws.alloc(mx * 4);
            a16[j] = (bf16 *)ws.alloc(mx * 2);
        }
        xf = (float *)ws.alloc(mx * 4);
        xin = (bf16 *)ws.alloc(mx * 2);
        audio = (float *)ws.alloc(F * kHop * 4);
        for (void *p : ws.ptrs)
            DTTS_CHECK(p, DTTS_ERR_OOM, "vocoder workspace allocation failed (%d frames)", max_frames);
        return DTTS_OK;
    }

    // tensor maps over the activations for an utterance of T0 frames (rows = exact lengths,
    // so rows past the end read as zero)
    int encode_maps(int T0) {
        if (T0 == maps_T0) return DTTS_OK;
        bool ok = make_tmap_bf16(&t_bott, bott16, T0, 128, 128) && make_tmap_bf16(&t_x0, x0, T0, 1536, 128);
        long long Tin = T0;
        for (int s = 0; s < kStages && ok; s++) {
            const int cin = s == 0 ? 1536 : cpad(kUpOut[s - 1]), cp = cpad(kUpOut[s]);
            const long long T = Tin * kUpStride[s];
            if (s > 0) ok = ok && make_tmap_bf16(&t_xin[s], xin, Tin, cin, 128);
            for (int j = 0; j < 3 && ok; j++)
                ok = make_tmap_bf16(&t_a[s][j], a16[j], T, cp, 128) && make_tmap_f32_resid(&t_r[s][j], r[j], T, cp);
            Tin = T;
        }
        DTTS_CHECK(ok, DTTS_ERR_CUDA, "tensor map (vocoder activations, %d frames)", T0);
        maps_T0 = T0;
        return DTTS_OK;
    }

    int gemm(const GemmOp &op, cudaStream_t s) {
        DTTS_CUDA(launch_gemm(op, num_sms, s));
        return DTTS_OK;
    }

    // AMP block j of stage s: r[j] += c2(act(c1(act(r[j])))) for dilations 1, 3, 5 (:427-483)
    int amp_block(int s, int j, long long T, cudaStream_t strm) {
        const int cp = cpad(kUpOut[s]), ch = kUpOut[s], rb = s * 3 + j, K = kRbK[j];
        const int bn = bn_for(T, cp), bi = bn == 192 ? 2 : bn == 128 ? 1 : 0;
        int st;
        for (int p = 0; p < 3; p++) {
            ActArgs aa1{r[j], cp, a16[j], cp, 1, (int)T, ch, act_a[rb][2 * p], act_ib[rb][2 * p], aa, aa, 1};
            launch_act(aa1, cp, strm);
            {
                GemmOp op = conv_op(t_a[s][j], t_c1[rb][p][bi], (int)T, cp, K * cp, EPI_F32, bn, d_err);
                op.ep.bias = b_c1[rb][p]; op.ep.out = y[j]; op.ep.ldo = cp;
                op.ep.tap_kb = cp / 64; op.ep.tap_base = -kRbDil[p] * (K - 1); op.ep.tap_step = kRbDil[p];
                if ((st = gemm(op, strm))) return st;
            }
            ActArgs aa2{y[j], cp, a16[j], cp, 1, (int)T, ch, act_a[rb][2 * p + 1], act_ib[rb][2 * p + 1], aa, aa, 1};
            launch_act(aa2, cp, strm);
            {
                GemmOp op = conv_op(t_a[s][j], t_c2[rb][p][bi], (int)T, cp, K * cp, EPI_RESID, bn, d_err);
                op.tr = t_r[s][j];
                op.ep.bias = b_c2[rb][p]; op.ep.resid = r[j]; op.ep.ldr = cp;
                op.ep.tap_kb = cp / 64; op.ep.tap_base = -(K - 1); op.ep.tap_step = 1;
                if ((st = gemm(op, strm))) return st;
            }
        }
        return DTTS_OK;
    }

    int lstm(int T) {
        DTTS_CUDA(cudaMemsetAsync(d_cnt, 0, (size_t)4 * T * sizeof(unsigned), stream));
        LstmArgs a{};
        a.gin0 = gin;
        for (int l = 0; l < 4; l++) { a.w_ih[l] = w_ih[l]; a.w_hh[l] = w_hh[l]; a.b_g[l] = b_g[l]; }
        a.h = hl; a.T = T; a.cnt = d_cnt; a.err = d_err;
        void *args[] = {(void *)&a};
        DTTS_CUDA(cudaLaunchCooperativeKernel((const void *)voc_lstm_kernel, dim3(4 * kLstmCtas), dim3(256), args,
                                              kLstmSmem, stream));
        return DTTS_OK;
    }

    // the whole decode on `stream`, latents already in `lat`, audio to `audio`
    int enqueue(int T0) {
        int st;
        // ---- bottleneck (bigvgan_cpp.cpp:344-377)
        launch_gemm_f32(lat, pp_w, pp_b, pp, T0, 128, 128, stream);
        launch_gemm_f32(pp, mi_w1, mi_b1, z, T0, kLstmH, 128, stream);
        launch_gemm_f32(z, w_ih[0], b_g[0], gin, T0, 4 * kLstmH, kLstmH, stream);
        if ((st = lstm(T0))) return st;
        // skip: z + h of the last layer
        launch_add_f32(z, hl + (size_t)3 * T0 * kLstmH, sk, (long long)T0 * kLstmH, stream);
        launch_gemm_f32(sk, mi_w2, mi_b2, bott, T0, 128, kLstmH, stream);
        launch_f32_to_bf16(bott, bott16, (long long)T0 * 128, stream);
        // ---- conv_pre: centred K = 5 (taps at t - 2 .. t + 2), bf16 out (:384-405)
        {
            GemmOp op = conv_op(t_bott, t_pre, T0, 1536, 5 * 128, EPI_BF16, 128, d_err);
            op.ep.bias = b_pre; op.ep.out = x0; op.ep.ldo = 1536;
            op.ep.tap_kb = 2; op.ep.tap_base = -2; op.ep.tap_step = 1;
            if ((st = gemm(op, stream))) return st;
        }
        long long Tin = T0;
        for (int s = 0; s < kStages; s++) {
            const int cin = s == 0 ? 1536 : cpad(kUpOut[s - 1]), cp = cpad(kUpOut[s]);
            const int str = kUpStride[s];
            const long long T = Tin * str;
            // ---- causal ConvTranspose1d as one GEMM: the output phases stacked along N
            // (row q of [T_in][stride * cp] is rows q stride .. q stride + stride-1 of
            // [T][cp]), each phase's K = [x[q] | x[q-1]] (:176-205, :415-420)
            {
                const int N = str * cp, bn = bn_for(Tin, N);
                GemmOp op = conv_op(s == 0 ? t_x0 : t_xin[s], t_up[s][bn == 128], (int)Tin, N, 2 * cin, EPI_F32, bn, d_err);
                op.ep.bias = b_up[s]; op.ep.out = r[0]; op.ep.ldo = N;
                op.ep.tap_kb = cin / 64; op.ep.tap_base = 0; op.ep.tap_step = -1;
                if ((st = gemm(op, stream))) return st;
            }
            const size_t n = (size_t)T * cp;
            DTTS_CUDA(cudaMemcpyAsync(r[1], r[0], n * 4, cudaMemcpyDeviceToDevice, stream));
            DTTS_CUDA(cudaMemcpyAsync(r[2], r[0], n * 4, cudaMemcpyDeviceToDevice, stream));
            // ---- three AMP blocks, concurrently (:427-483)
            DTTS_CUDA(cudaEventRecord(ev_fork, stream));
            for (int i = 0; i < 2; i++) DTTS_CUDA(cudaStreamWaitEvent(side[i], ev_fork, 0));
            for (int j = 0; j < 3; j++)
                if ((st = amp_block(s, j, T, j == 0 ? stream : side[j - 1]))) return st;
            for (int i = 0; i < 2; i++) {
                DTTS_CUDA(cudaEventRecord(ev_join[i], side[i]));
                DTTS_CUDA(cudaStreamWaitEvent(stream, ev_join[i], 0));
            }
            const long long n4 = (long long)(n / 4);
            const bool last = s == kStages - 1;
            voc_mean3_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, stream>>>(
                (const float4 *)r[0], (const float4 *)r[1], (const float4 *)r[2], last ? nullptr : (uint2 *)xin,
                last ? (float4 *)xf : nullptr, n4);
            Tin = T;
        }
        // ---- activation_post, conv_post, tanh (:499-521)
        const int cp = cpad(24);
        ActArgs ap{xf, cp, y[0], cp, 0, (int)Tin, 24, post_a, post_ib, post_fu, post_fd, 24};
        launch_act(ap, cp, stream);
        voc_post_kernel<<<(unsigned)((Tin + kPostT - 1) / kPostT), kPostT, 0, stream>>>(y[0], cp, (int)Tin, post_w, audio);
        DTTS_CUDA(cudaGetLastError());
        return DTTS_OK;
    }

    int decode(const float *latent, int n_frames, float *audio_out, int mem) {
        DTTS_CHECK(latent && audio_out, DTTS_ERR_ARG, "null argument");
        DTTS_CHECK(n_frames >= 1 && n_frames <= max_frames, DTTS_ERR_ARG, "n_frames %d out of [1, %d]", n_frames,
                   max_frames);
        DTTS_CHECK(mem == DTTS_MEM_HOST || mem == DTTS_MEM_DEVICE, DTTS_ERR_ARG, "bad mem kind");
        DeviceGuard g(device);
        int st = encode_maps(n_frames);
        if (st) return st;
        const cudaMemcpyKind ik = mem == DTTS_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
        DTTS_CUDA(cudaMemcpyAsync(lat, latent, (size_t)n_frames * 128 * 4, ik, stream));
        if ((st = enqueue(n_frames))) return st;
        const cudaMemcpyKind ok = mem == DTTS_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
        DTTS_CUDA(cudaMemcpyAsync(audio_out, audio, (size_t)n_frames * kHop * 4, ok, stream));
        if (mem != DTTS_MEM_HOST) return DTTS_OK;
        if ((st = stream_wait(stream, 300.0))) return st;
        int err = 0;
        DTTS_CUDA(cudaMemcpy(&err, d_err, 4, cudaMemcpyDeviceToHost));
        if (err) { cudaMemset(d_err, 0, 4); set_error("device wait limit reached (code %d)", err); return DTTS_ERR_TIMEOUT; }
        return DTTS_OK;
    }
};

namespace {
// B operand of a convolution over taps: B[o][tap * cpi + c] = W[o][c][tap] (W [oc][ic][K])
std::vector<float> conv_b_operand(const float *W, int oc, int ic, int K, int cpo, int cpi) {
    std::vector<float> v((size_t)cpo * K * cpi, 0.f);
    for (int o = 0; o < oc; o++)
        for (int c = 0; c < ic; c++)
            for (int k = 0; k < K; k++) v[((size_t)o * K + k) * cpi + c] = W[((size_t)o * ic + c) * K + k];
    return v;
}
}  // namespace

extern "C" {

int dtts_voc_aa_filter(float *taps12) {
    DTTS_CHECK(taps12, DTTS_ERR_ARG, "null argument");
    kaiser_sinc(taps12, 0.25, 0.3, kTaps);
    return DTTS_OK;
}

int dtts_voc_create(const dtts_voc_weights *w, int device, int max_frames, dtts_voc **out) {
    DTTS_CHECK(w && out, DTTS_ERR_ARG, "null argument");
    *out = nullptr;
    DTTS_CHECK(max_frames >= 1 && max_frames <= 100000, DTTS_ERR_ARG, "max_frames %d out of [1, 100000]", max_frames);
    DTTS_CHECK(w->post_proj_w && w->mi_w1 && w->mi_w2 && w->conv_pre_w && w->conv_post_w && w->post_filt_up &&
                   w->post_filt_down,
               DTTS_ERR_ARG, "missing a required vocoder weight");
    for (int l = 0; l < 4; l++)
        DTTS_CHECK(w->lstm_w_ih[l] && w->lstm_w_hh[l], DTTS_ERR_ARG, "missing LSTM layer %d weights", l);
    for (int s = 0; s < kStages; s++) DTTS_CHECK(w->ups_w[s], DTTS_ERR_ARG, "missing decoder.ups.%d", s);
    for (int rb = 0; rb < kRb; rb++)
        for (int j = 0; j < 3; j++)
            DTTS_CHECK(w->c1_w[rb][j] && w->c2_w[rb][j], DTTS_ERR_ARG, "missing resblock %d conv %d", rb, j);
    int nsm = 0, st = check_device(device, &nsm);
    if (st) return st;
    DeviceGuard g(device);
    std::unique_ptr<dtts_voc> v(new dtts_voc());
    v->device = device; v->num_sms = nsm; v->max_frames = max_frames;
    DTTS_CUDA(cudaStreamCreateWithFlags(&v->own_stream, cudaStreamNonBlocking));
    v->stream = v->own_stream;
    for (int i = 0; i < 2; i++) {
        DTTS_CUDA(cudaStreamCreateWithFlags(&v->side[i], cudaStreamNonBlocking));
        DTTS_CUDA(cudaEventCreateWithFlags(&v->ev_join[i], cudaEventDisableTiming));
    }
    DTTS_CUDA(cudaEventCreateWithFlags(&v->ev_fork, cudaEventDisableTiming));
    DTTS_CUDA(gemm_prepare_attributes());
    DTTS_CUDA(cudaFuncSetAttribute((const void *)voc_lstm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kLstmSmem));
    DeviceArena &A = v->wts;
    v->d_err = (int *)A.alloc(4);
    v->d_cnt = (unsigned *)A.alloc((size_t)4 * max_frames * sizeof(unsigned));
    DTTS_CHECK(v->d_err && v->d_cnt, DTTS_ERR_OOM, "cudaMalloc failed");
    DTTS_CUDA(cudaMemset(v->d_err, 0, 4));
    // bottleneck
    std::vector<float> zero(4 * kLstmH, 0.f);
    if ((st = up_f32(A, w->post_proj_w, 128 * 128, &v->pp_w))) return st;
    if ((st = up_f32_pad(A, w->post_proj_b, 128, 128, &v->pp_b))) return st;
    if ((st = up_f32(A, w->mi_w1, (size_t)kLstmH * 128, &v->mi_w1))) return st;
    if ((st = up_f32_pad(A, w->mi_b1, kLstmH, kLstmH, &v->mi_b1))) return st;
    if ((st = up_f32(A, w->mi_w2, (size_t)128 * kLstmH, &v->mi_w2))) return st;
    if ((st = up_f32_pad(A, w->mi_b2, 128, 128, &v->mi_b2))) return st;
    for (int l = 0; l < 4; l++) {
        if ((st = up_f32(A, w->lstm_w_ih[l], (size_t)4 * kLstmH * kLstmH, &v->w_ih[l]))) return st;
        if ((st = up_f32(A, w->lstm_w_hh[l], (size_t)4 * kLstmH * kLstmH, &v->w_hh[l]))) return st;
        // b_ih + b_hh, summed in float as lstm.cpp:26 starts each gate
        std::vector<float> bg(4 * kLstmH);
        for (int i = 0; i < 4 * kLstmH; i++)
            bg[i] = (w->lstm_b_ih[l] ? w->lstm_b_ih[l][i] : 0.f) + (w->lstm_b_hh[l] ? w->lstm_b_hh[l][i] : 0.f);
        if ((st = up_f32(A, bg.data(), bg.size(), &v->b_g[l]))) return st;
    }
    // conv_pre
    if ((st = up_bf16(A, conv_b_operand(w->conv_pre_w, 1536, 128, 5, 1536, 128), &v->w_pre))) return st;
    if ((st = up_f32_pad(A, w->conv_pre_b, 1536, 1536, &v->b_pre))) return st;
    bool ok = make_tmap_bf16(&v->t_pre, v->w_pre, 1536, 5 * 128, 128);
    // upsampling: phase r, B_r[o][j * cpi + c] = W[c][o][r + j stride] (W [ic][oc][2 stride])
    for (int s = 0; s < kStages && ok; s++) {
        const int ic = kUpIn[s], oc = kUpOut[s], cpi = s == 0 ? 1536 : cpad(ic), cpo = cpad(oc), str = kUpStride[s];
        const int K = 2 * str;
        std::vector<float> bop((size_t)str * cpo * 2 * cpi, 0.f);
        for (int ph = 0; ph < str; ph++)
            for (int o = 0; o < oc; o++)
                for (int j = 0; j < 2; j++)
                    for (int c = 0; c < ic; c++)
                        bop[(((size_t)ph * cpo + o) * 2 + j) * cpi + c] = w->ups_w[s][((size_t)c * oc + o) * K + ph + j * str];
        if ((st = up_bf16(A, bop, &v->w_up[s]))) return st;
        // bias per output column of the stacked phases: b[o] at column ph * cpo + o
        std::vector<float> bias((size_t)str * cpo, 0.f);
        for (int ph = 0; ph < str; ph++)
            for (int o = 0; o < oc; o++) bias[(size_t)ph * cpo + o] = w->ups_b[s] ? w->ups_b[s][o] : 0.f;
        if ((st = up_f32(A, bias.data(), bias.size(), &v->b_up[s]))) return st;
        ok = make_tmap_bf16(&v->t_up[s][0], v->w_up[s], (size_t)str * cpo, 2 * cpi, 64) &&
             make_tmap_bf16(&v->t_up[s][1], v->w_up[s], (size_t)str * cpo, 2 * cpi, 128);
    }
    // AMP blocks
    for (int rb = 0; rb < kRb && ok; rb++) {
        const int ch = kUpOut[rb / 3], cp = cpad(ch), K = kRbK[rb % 3];
        for (int j = 0; j < 3 && ok; j++) {
            if ((st = up_bf16(A, conv_b_operand(w->c1_w[rb][j], ch, ch, K, cp, cp), &v->w_c1[rb][j]))) return st;
            if ((st = up_bf16(A, conv_b_operand(w->c2_w[rb][j], ch, ch, K, cp, cp), &v->w_c2[rb][j]))) return st;
            if ((st = up_f32_pad(A, w->c1_b[rb][j], ch, cp, &v->b_c1[rb][j]))) return st;
            if ((st = up_f32_pad(A, w->c2_b[rb][j], ch, cp, &v->b_c2[rb][j]))) return st;
            for (int bi = 0; bi < 3 && ok; bi++) {
                const unsigned wide = bi == 2 ? 192 : 128;   // a tile width is usable when it divides cp
                const unsigned box = (bi && cp % wide == 0) ? wide : 64;
                ok = make_tmap_bf16(&v->t_c1[rb][j][bi], v->w_c1[rb][j], cp, (size_t)K * cp, box) &&
                     make_tmap_bf16(&v->t_c2[rb][j][bi], v->w_c2[rb][j], cp, (size_t)K * cp, box);
            }
        }
        for (int a = 0; a < 6; a++) {
            std::vector<float> av, ib;
            snake_consts(w->alpha[rb][a], w->beta[rb][a], ch, cp, av, ib);
            if ((st = up_f32(A, av.data(), cp, &v->act_a[rb][a]))) return st;
            if ((st = up_f32(A, ib.data(), cp, &v->act_ib[rb][a]))) return st;
        }
    }
    DTTS_CHECK(ok, DTTS_ERR_CUDA, "tensor map (vocoder weights)");
    // filters, activation_post, conv_post
    float aa[kTaps];
    kaiser_sinc(aa, 0.25, 0.3, kTaps);
    if ((st = up_f32(A, aa, kTaps, &v->aa))) return st;
    {
        std::vector<float> av, ib;
        snake_consts(w->post_alpha, w->post_beta, 24, 24, av, ib);
        if ((st = up_f32(A, av.data(), 24, &v->post_a))) return st;
        if ((st = up_f32(A, ib.data(), 24, &v->post_ib))) return st;
    }
    if ((st = up_f32(A, w->post_filt_up, 24 * kTaps, &v->post_fu))) return st;
    if ((st = up_f32(A, w->post_filt_down, 24 * kTaps, &v->post_fd))) return st;
    if ((st = up_f32(A, w->conv_post_w, 24 * 7, &v->post_w))) return st;
    if ((st = v->alloc_ws())) return st;
    *out = v.release();
    return DTTS_OK;
}

int dtts_voc_destroy(dtts_voc *v) {
    if (!v) return DTTS_OK;
    DeviceGuard g(v->device);
    // a decode that failed between fork and join can leave work on the side streams
    cudaStreamSynchronize(v->stream);
    for (int i = 0; i < 2; i++)
        if (v->side[i]) cudaStreamSynchronize(v->side[i]);
    delete v;
    return DTTS_OK;
}

int dtts_voc_set_stream(dtts_voc *v, void *stream) {
    DTTS_CHECK(v, DTTS_ERR_ARG, "null engine");
    v->stream = stream ? static_cast<cudaStream_t>(stream) : v->own_stream;
    return DTTS_OK;
}

int dtts_voc_decode(dtts_voc *v, const float *latent, int n_frames, float *audio, int mem) {
    DTTS_CHECK(v, DTTS_ERR_ARG, "null engine");
    return v->decode(latent, n_frames, audio, mem);
}

int dtts_selftest_voc_activation(const float *x, int len, int ch, const float *alpha, const float *beta,
                                 const float *filt_up, const float *filt_down, int fch, float *out) {
    DTTS_CHECK(x && out && filt_up && filt_down, DTTS_ERR_ARG, "null argument");
    DTTS_CHECK(len >= 1 && ch >= 1 && ch <= 4096 && (fch == 1 || fch == ch), DTTS_ERR_ARG, "bad shape");
    int nsm = 0, st = check_device(0, &nsm);
    if (st) return st;
    DeviceGuard g(0);
    std::vector<float> av, ib;
    snake_consts(alpha, beta, ch, ch, av, ib);
    DeviceArena A;
    float *dx = nullptr, *dy = nullptr, *da = nullptr, *dib = nullptr, *dfu = nullptr, *dfd = nullptr;
    st = up_f32(A, x, (size_t)len * ch, &dx);
    if (!st) st = up_f32(A, av.data(), ch, &da);
    if (!st) st = up_f32(A, ib.data(), ch, &dib);
    if (!st) st = up_f32(A, filt_up, (size_t)fch * kTaps, &dfu);
    if (!st) st = up_f32(A, filt_down, (size_t)fch * kTaps, &dfd);
    if (!st) {
        dy = (float *)A.alloc((size_t)len * ch * 4);
        if (!dy) { set_error("cudaMalloc failed"); st = DTTS_ERR_OOM; }
    }
    if (!st) {
        ActArgs p{dx, ch, dy, ch, 0, len, ch, da, dib, dfu, dfd, fch};
        launch_act(p, ch, 0);
        cudaError_t e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaMemcpy(out, dy, (size_t)len * ch * 4, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) { set_error("voc activation selftest: %s", cudaGetErrorString(e)); st = DTTS_ERR_CUDA; }
    }
    A.free_all();
    return st;
}

}  // extern "C"
