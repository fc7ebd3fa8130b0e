// fp32 DiT attention sublayer that performs no device allocation.
//
// Some callers cannot allocate GPU memory while they run: a host application
// that hands the library a fixed memory budget up front, a plugin inside an
// inference runtime that forbids allocation in its execute callback, or a
// real-time audio thread where a cudaMalloc could block or fail.  For them,
// dtts_attn_forward_f32_noalloc takes every input, weight and output as device
// pointers the caller already owns, and keeps its intermediates (Q, K, V,
// attention context, RoPE table) in one file-scope __device__ array compiled
// into the library.  Limits: rows * L <= DTTS_NOALLOC_MAX_TOKENS (256) and
// L <= 256.  The array occupies 4.06 MiB on a device from the first call
// there (from library load when CUDA_MODULE_LOADING=EAGER) until the process
// exits.
#include "kernels.cuh"
#include "runtime.h"

#include <cuda.h>
#include <mutex>

using namespace dtts;

namespace {

constexpr int kMaxTok = 256;                       // DTTS_NOALLOC_MAX_TOKENS
constexpr int kMaxL = 256;
constexpr size_t kActFloats = (size_t)kMaxTok * kD;   // one [tokens][1024] fp32 activation
constexpr size_t kRopeFloats = (size_t)kMaxL * 32 * 2;
constexpr size_t kScratchFloats = 4 * kActFloats + kRopeFloats;

// Q, K, V, context, then the RoPE table.  Shared by every call on this GPU.
static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

// Host-side device address of g_noalloc_scratch, looked up once per device
// and context: the context it was looked up in is kept beside it, so a device
// reset (which destroys the primary context, its module and the kernel
// attribute set below) leads to a fresh set-up instead of a stale address.
constexpr int kMaxDevices = 64;
float *g_scratch_addr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};
std::mutex g_setup_mutex;

typedef CUresult (*CtxGetCurrentFn)(CUcontext *);

CtxGetCurrentFn ctx_get_current_fn() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    });
    return fn;
}

// RoPE (cos, sin) table of the half-split rotation: theta_d = (1e4^(-2/64))^d
// by repeated multiplication, angle = pos[t] * theta_d (t when pos is null).
__global__ void noalloc_rope_table_kernel(const float *__restrict__ pos, int L, float2 *__restrict__ tab) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= L) return;
    const float p = pos ? pos[t] : (float)t;
    const float ts = powf(10000.0f, -2.0f / 64.0f);
    float theta = 1.0f;
    for (int d = 0; d < 32; d++) {
        float s, c;
        sincosf(p * theta, &s, &c);
        tab[t * 32 + d] = make_float2(c, s);
        theta *= ts;
    }
}

// Once per device (and again after the device's context was replaced), with
// that device current: find where the array lives and opt the fp32 attention
// kernel into its shared-memory size.
int setup_device(int dev, float **out) {
    CtxGetCurrentFn get_ctx = ctx_get_current_fn();
    DTTS_CHECK(get_ctx, DTTS_ERR_CUDA, "cuCtxGetCurrent is not available from the driver");
    // NULL when the runtime has not yet made a context current on this thread
    CUcontext ctx = nullptr;
    if (get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (ctx && g_scratch_addr[dev] && g_scratch_ctx[dev] == ctx) { *out = g_scratch_addr[dev]; return DTTS_OK; }
    // the lookup makes the device's primary context current when it is not yet
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    DTTS_CHECK(get_ctx(&ctx) == CUDA_SUCCESS && ctx, DTTS_ERR_CUDA, "no current CUDA context on device %d", dev);
    DTTS_CUDA(attention_f32_prepare());
    g_scratch_addr[dev] = static_cast<float *>(p);
    g_scratch_ctx[dev] = ctx;
    *out = g_scratch_addr[dev];
    return DTTS_OK;
}

}  // namespace

extern "C" int dtts_attn_forward_f32_noalloc(const float *x, const float *wq, const float *wk, const float *wv,
                                             const float *wo, const float *bo, const float *qn, const float *kn,
                                             const uint8_t *mask, const float *pos, int rows, int L, float *out,
                                             void *stream) {
    DTTS_CHECK(x && wq && wk && wv && wo && out, DTTS_ERR_ARG, "null input, weight or output pointer");
    DTTS_CHECK(rows >= 1 && L >= 1, DTTS_ERR_ARG, "bad shape rows=%d L=%d", rows, L);
    DTTS_CHECK(L <= kMaxL, DTTS_ERR_ARG, "L = %d exceeds the no-allocation limit of %d tokens per row", L, kMaxL);
    DTTS_CHECK((long long)rows * L <= kMaxTok, DTTS_ERR_ARG,
               "rows * L = %lld exceeds the no-allocation scratch limit of %d tokens", (long long)rows * L, kMaxTok);
    int dev = -1;
    DTTS_CUDA(cudaGetDevice(&dev));
    DTTS_CHECK(dev >= 0 && dev < kMaxDevices, DTTS_ERR_NO_DEVICE, "device %d out of range", dev);
    float *base = nullptr;
    int st = setup_device(dev, &base);
    if (st) return st;
    float *q = base, *k = base + kActFloats, *v = base + 2 * kActFloats, *ctx = base + 3 * kActFloats;
    float2 *rope = reinterpret_cast<float2 *>(base + 4 * kActFloats);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int M = rows * L;
    // Every scratch element read below is written earlier in this call, so
    // nothing needs clearing between calls.
    noalloc_rope_table_kernel<<<(L + 63) / 64, 64, 0, s>>>(pos, L, rope);
    launch_gemm_f32(x, wq, nullptr, q, M, kD, kD, s);
    launch_gemm_f32(x, wk, nullptr, k, M, kD, kD, s);
    launch_gemm_f32(x, wv, nullptr, v, M, kD, kD, s);
    launch_qk_norm_rope_f32(q, k, M, L, 1, qn, kn, rope, ROPE_HALF, 0, s);
    AttnArgs a{};
    a.q = q; a.k = k; a.v = v; a.o = ctx; a.ldq = a.ldkv = a.ldo = kD;
    a.rows = rows; a.Tq = L; a.kv_len = L; a.kv_cap = L; a.q_pos0 = 0; a.causal = 0;
    a.mask = mask; a.scale = 1.0f / sqrtf(64.0f);
    DTTS_CUDA(launch_attention_f32(a, s));
    launch_gemm_f32(ctx, wo, bo, out, M, kD, kD, s);
    DTTS_CUDA(cudaGetLastError());
    return DTTS_OK;
}
