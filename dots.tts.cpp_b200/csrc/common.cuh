// Shared device helpers for the sm_100a kernels: mbarriers, TMA, tcgen05
// (UMMA + TMEM), bounded waits, bf16 packing.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#define DTTS_DEV __device__ __forceinline__

namespace dtts {

typedef __nv_bfloat16 bf16;

// model widths: hidden, heads, head dim, FFN, latent, LLM hidden, speaker
constexpr int kD = 1024, kH = 16, kHD = 64, kF = 4096, kLat = 128, kLLM = 1536, kSpk = 512;

// Error codes that kernels write into the engine's device error word.
enum DeviceError : int {
    DEVERR_NONE = 0,
    DEVERR_TIMEOUT_PRODUCER = 1,
    DEVERR_TIMEOUT_MMA = 2,
    DEVERR_TIMEOUT_EPILOGUE = 3,
    DEVERR_NONFINITE = 4,
    DEVERR_TIMEOUT_BARRIER = 5,   // a grid barrier between CTAs of one kernel
};

// Every spin on an mbarrier gives up after this long (globaltimer ns).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

DTTS_DEV uint32_t smem_u32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while the kernel before it in the stream still
// runs.  Every kernel here calls pdl_wait() in all threads before its first
// access to memory that an earlier kernel writes or reads (only constant
// weights may be fetched before it), so memory effects keep the stream
// order; after an ordinary launch pdl_wait() returns at once.  pdl_trigger()
// lets the next kernel's CTAs be scheduled once every CTA of this grid has
// issued it.
DTTS_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
DTTS_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// L2 access-policy window that launch_k attaches to every launch made by the
// calling thread while it is set (bytes > 0): accesses inside [base, base +
// bytes) are marked persisting with probability hit_ratio, so a buffer that
// every kernel of a forward reads and writes (the DiT's fp32 residual stream)
// stays in L2 between kernels instead of being evicted by the streams of
// weights and activations around it.  Launches captured into a CUDA graph keep
// the window as a kernel-node attribute.
struct L2Window {
    void *base = nullptr;
    size_t bytes = 0;
    float hit_ratio = 0.f;
};
inline L2Window &l2_window() {
    static thread_local L2Window w;
    return w;
}
// Sets the calling thread's window for the scope and restores the previous one.
struct L2WindowScope {
    L2Window prev;
    explicit L2WindowScope(const L2Window &w) : prev(l2_window()) { l2_window() = w; }
    ~L2WindowScope() { l2_window() = prev; }
};

// k<<<grid, block, smem, s>>>(args...) with the calling thread's L2 window, if
// any.  flags: kLaunchPdl (the value of `true`), programmatic stream
// serialization (the kernel must follow the pdl_wait rule); kLaunchCoop, a
// cooperative launch (every CTA resident at once, so its CTAs may wait on one
// another).
constexpr unsigned kLaunchPdl = 1u, kLaunchCoop = 2u;
template <typename... P, typename... A>
inline cudaError_t launch_k(unsigned flags, void (*k)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            A &&...args) {
    cudaLaunchAttribute attr[3];
    int n = 0;
    if (flags & kLaunchCoop) {
        attr[n].id = cudaLaunchAttributeCooperative;
        attr[n].val.cooperative = 1;
        n++;
    }
    if (flags & kLaunchPdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        n++;
    }
    const L2Window &w = l2_window();
    if (w.bytes > 0) {
        attr[n].id = cudaLaunchAttributeAccessPolicyWindow;
        attr[n].val.accessPolicyWindow.base_ptr = w.base;
        attr[n].val.accessPolicyWindow.num_bytes = w.bytes;
        attr[n].val.accessPolicyWindow.hitRatio = w.hit_ratio;
        attr[n].val.accessPolicyWindow.hitProp = cudaAccessPropertyPersisting;
        attr[n].val.accessPolicyWindow.missProp = cudaAccessPropertyStreaming;
        n++;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, k, static_cast<A &&>(args)...);
}

DTTS_DEV unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
DTTS_DEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
DTTS_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
DTTS_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
DTTS_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
DTTS_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Gives up after
// kWaitLimitNs (or as soon as another role of the CTA has given up), records
// `code` in the device error word, raises the CTA's abort flag and returns
// false.  A correct kernel never reaches the limit.
DTTS_DEV bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    unsigned long long t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            if (err) atomicCAS(err, 0, code);
            *abort_flag = 1;
            return false;
        }
    }
}

// --------------------------------------------------------------------- TMA
// 2-D tiled load of box (x = inner/K coordinate, y = row) into shared memory,
// completing on `bar`.  x is always a multiple of 64 bf16 (128 bytes).
DTTS_DEV void tma_load_2d(void *smem_dst, const CUtensorMap *tm, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
            "r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
// 1-D bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// from global into this CTA's shared memory, completing on `bar`.
DTTS_DEV void bulk_load_1d(void *smem_dst, const void *gsrc, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(smem_dst)),
                 "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
DTTS_DEV void tma_prefetch_desc(const CUtensorMap *tm) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

// Bulk tensor reduce-add (fp32) of a shared-memory box into global memory,
// tracked by the issuing thread's bulk async-group.
DTTS_DEV void tma_reduce_add_2d(const CUtensorMap *tm, const void *smem_src, int x, int y) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(tm)),
                 "r"(smem_u32(smem_src)), "r"(x), "r"(y)
                 : "memory");
}
DTTS_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// at most N of this thread's bulk groups may still be reading shared memory
template <int N>
DTTS_DEV void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }
// at most N of this thread's bulk groups may still be in flight
template <int N>
DTTS_DEV void bulk_wait() { asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory"); }
// orders this thread's generic-proxy shared-memory writes before later async-proxy (TMA) reads
DTTS_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// orders this thread's completed async-proxy (bulk) global writes before its later generic-proxy accesses
DTTS_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
// Invalidates the 128-byte L2 line at p (128-byte aligned) without writing it
// back: for data no kernel will read again before it is overwritten.
DTTS_DEV void l2_discard_line(const void *p) { asm volatile("discard.global.L2 [%0], 128;" ::"l"(p) : "memory"); }
// acquire load of a counter that other CTAs raise (bounded inter-CTA waits)
DTTS_DEV unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ----------------------------------------------------------------- tcgen05
DTTS_DEV void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
}
DTTS_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
DTTS_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
DTTS_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DTTS_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Arrives on `bar` once every tcgen05 op issued so far by this thread is done.
DTTS_DEV void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// D(tmem) (+)= A(smem) * B(smem)^T, bf16 inputs, fp32 accumulate.
DTTS_DEV void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart.
// Fields (sm100 UMMA descriptor): start address >> 4 [0,14), leading byte
// offset >> 4 [16,30) (unused for swizzled K-major, 1), stride byte offset >> 4
// [32,46) = 1024 >> 4, version [46,48) = 1, layout [61,64) = 2 (SWIZZLE_128B).
DTTS_DEV uint64_t sdesc_k128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor, kind::f16 with bf16 A/B, fp32 D, both K-major.
// Fields: D format [4,6) = 1 (f32), A format [7,10) = 1 (bf16), B format
// [10,13) = 1, N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// Instruction descriptor for tcgen05.mma kind::f8f6f4 with both operands
// e4m3 (format code 0 in bits 7-9 and 10-12), fp32 accumulate, K-major A and B.
__host__ __device__ constexpr uint32_t idesc_e4m3(int M, int N) {
    return (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, e4m3 x e4m3 -> fp32, M=128, K=32 per call.
DTTS_DEV void tc_mma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Four floats to four e4m3 bytes (round to nearest even, saturating at +-448),
// a in the lowest byte.
DTTS_DEV uint32_t pack_e4m3x4(float a, float b, float c, float d) {
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
    return lo | (hi << 16);
}

// 32 lanes x 32 consecutive fp32 columns from TMEM.  The wait is fused into
// the same asm so no use of the registers can be scheduled before it.
DTTS_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Two 32-column TMEM loads (lo at taddr_lo, hi at taddr_hi) behind a single
// wait: the second load is in flight while the first completes, so a
// 64-column chunk pays one TMEM round trip instead of two.
DTTS_DEV void tmem_ld32x2(uint32_t taddr_lo, uint32_t taddr_hi, float (&lo)[32], float (&hi)[32]) {
    uint32_t a[32], b[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]),
          "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]), "=r"(a[14]), "=r"(a[15]),
          "=r"(a[16]), "=r"(a[17]), "=r"(a[18]), "=r"(a[19]), "=r"(a[20]), "=r"(a[21]), "=r"(a[22]), "=r"(a[23]),
          "=r"(a[24]), "=r"(a[25]), "=r"(a[26]), "=r"(a[27]), "=r"(a[28]), "=r"(a[29]), "=r"(a[30]), "=r"(a[31]),
          "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7]),
          "=r"(b[8]), "=r"(b[9]), "=r"(b[10]), "=r"(b[11]), "=r"(b[12]), "=r"(b[13]), "=r"(b[14]), "=r"(b[15]),
          "=r"(b[16]), "=r"(b[17]), "=r"(b[18]), "=r"(b[19]), "=r"(b[20]), "=r"(b[21]), "=r"(b[22]), "=r"(b[23]),
          "=r"(b[24]), "=r"(b[25]), "=r"(b[26]), "=r"(b[27]), "=r"(b[28]), "=r"(b[29]), "=r"(b[30]), "=r"(b[31])
        : "r"(taddr_lo), "r"(taddr_hi)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) { lo[i] = __uint_as_float(a[i]); hi[i] = __uint_as_float(b[i]); }
}

// ------------------------------------------------------------------ misc
DTTS_DEV uint32_t pack_bf16x2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}
DTTS_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
DTTS_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// 2^x by the hardware approximation (MUFU ex2, subnormal results flushed to
// zero), for softmax numerators whose argument is <= 0.
DTTS_DEV float ex2_hw(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// tanh by the hardware approximation (MUFU), used in the bf16 GELU epilogue.
DTTS_DEV float tanh_hw(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

}  // namespace dtts
