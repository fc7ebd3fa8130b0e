// tcgen05 / TMEM / TMA GEMM for sm_100a with fused epilogues.
//
//   C[M, N] = A[M, K] * B[N, K]^T     A, B bf16 K-major (PyTorch Linear: B is
//                                      the [out, in] weight), fp32 accumulate
//
// One persistent CTA per SM, 6 warps:
//   warp 0      TMA producer: A tile 128x64 and B tile BNx64 per stage,
//               128-byte swizzle, mbarrier complete_tx
//   warp 1      TMEM allocator + MMA issuer (one thread): 4 x
//               tcgen05.mma.cta_group::1.kind::f16 (128 x BN x 16) per stage,
//               tcgen05.commit frees the stage
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, fused op, store
// Two TMEM accumulators (2 x BN fp32 columns) let the epilogue of tile i run
// while the MMAs of tile i+1 accumulate.  Every mbarrier wait is bounded
// (common.cuh); on expiry the CTA drains and returns with an error code.
//
// Shape rules (checked on the host): N % BN == 0, K % 64 == 0, M >= 1; rows
// past M are zero-filled by TMA and never stored.
#pragma once
#include "common.cuh"

namespace dtts {

enum EpiKind : int {
    EPI_BF16 = 0,     // out_bf16 = acc + bias
    EPI_GELU_BF16,    // out_bf16 = gelu_tanh(acc + bias)          (DiT FFN1)
    EPI_SILU_BF16,    // out_bf16 = silu(acc + bias)               (PE FFN1)
    EPI_F32,          // out_f32  = acc + bias                     (adaLN, projections)
    EPI_RESID,        // resid   += acc + bias                     (PE residual)
    EPI_RESID_GATED,  // resid   += gate[row] * (acc + bias)       (DiT gated residual)
    EPI_QKV,          // q/k/v split, optional per-head RMS norm, RoPE, bf16 stores
};

enum RopeMode : int { ROPE_HALF = 0, ROPE_ADJACENT = 1 };

struct EpiParams {
    const float *bias;        // [N] or nullptr
    void *out;                // EPI_BF16/GELU/SILU: bf16; EPI_F32: f32
    long long ldo;
    float *resid;             // EPI_RESID*: fp32 [M][ldr]
    long long ldr;
    const float *gate;        // EPI_RESID_GATED: gate[(m / tok_per_row) * gate_ld + n]
    long long gate_ld;
    int tok_per_row;          // tokens per sequence row (L); maps token m -> (row, t)
    // EPI_QKV: columns [0,1024) -> q, [1024,2048) -> k, [2048,3072) -> v
    bf16 *q, *k, *v;
    long long ldq, ldkv;      // q[m*ldq + c]; k/v[((m/T)*kv_cap + kv_start + m%T) * ldkv + c]
    int kv_cap, kv_start;
    int qk_norm;              // per-head RMS norm (eps 1e-6) of q and k before RoPE
    const float *qn, *kn;     // its gains [64], or nullptr for none
    const float2 *rope;       // [positions][32] (cos, sin); row index = kv_start + m%T
    int rope_mode;
    int *err;                 // device error word
};

template <int BN>
struct GemmCfg {
    static constexpr int BM = 128, BK = 64;
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 8 ? 8 : (200 * 1024) / STAGE_BYTES;
    static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 1024;  // +1024 alignment slack
    static constexpr uint32_t IDESC = idesc_bf16(BM, BN);
    static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN");
    static_assert(2 * BN <= 512, "two accumulators must fit in TMEM");
};

DTTS_DEV float gelu_tanh_fast(float x) {
    const float c1 = 0.7978845608028654f, c2 = 0.044715f;
    return 0.5f * x * (1.0f + tanh_hw(c1 * (x + c2 * x * x * x)));
}
DTTS_DEV float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// Stores 32 consecutive bf16 values (64 bytes, 16-byte aligned).
DTTS_DEV void store_bf16x32(bf16 *dst, const float (&v)[32]) {
    uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint4 u;
        u.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
        u.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
        u.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
        u.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
        d[i] = u;
    }
}

DTTS_DEV void add_bias32(float (&v)[32], const float *bias, int n0) {
    if (!bias) return;
    const float4 *b4 = reinterpret_cast<const float4 *>(bias + n0);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float4 b = __ldg(b4 + i);
        v[4 * i + 0] += b.x; v[4 * i + 1] += b.y; v[4 * i + 2] += b.z; v[4 * i + 3] += b.w;
    }
}

// One 32-column chunk for the non-QKV epilogues.  m < M is guaranteed.
template <int EPI>
DTTS_DEV void epilogue_chunk(const EpiParams &ep, int m, int n0, float (&v)[32]) {
    add_bias32(v, ep.bias, n0);
    if constexpr (EPI == EPI_BF16 || EPI == EPI_GELU_BF16 || EPI == EPI_SILU_BF16) {
        if constexpr (EPI == EPI_GELU_BF16) {
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = gelu_tanh_fast(v[i]);
        }
        if constexpr (EPI == EPI_SILU_BF16) {
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = silu_f(v[i]);
        }
        store_bf16x32(reinterpret_cast<bf16 *>(ep.out) + (long long)m * ep.ldo + n0, v);
    } else if constexpr (EPI == EPI_F32) {
        float4 *d = reinterpret_cast<float4 *>(reinterpret_cast<float *>(ep.out) + (long long)m * ep.ldo + n0);
#pragma unroll
        for (int i = 0; i < 8; i++) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else if constexpr (EPI == EPI_RESID || EPI == EPI_RESID_GATED) {
        float4 *r = reinterpret_cast<float4 *>(ep.resid + (long long)m * ep.ldr + n0);
        const float4 *g4 = nullptr;
        if constexpr (EPI == EPI_RESID_GATED)
            g4 = reinterpret_cast<const float4 *>(ep.gate + (long long)(m / ep.tok_per_row) * ep.gate_ld + n0);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float4 x = r[i];
            if constexpr (EPI == EPI_RESID_GATED) {
                float4 g = __ldg(g4 + i);
                x.x += g.x * v[4 * i + 0]; x.y += g.y * v[4 * i + 1];
                x.z += g.z * v[4 * i + 2]; x.w += g.w * v[4 * i + 3];
            } else {
                x.x += v[4 * i + 0]; x.y += v[4 * i + 1]; x.z += v[4 * i + 2]; x.w += v[4 * i + 3];
            }
            r[i] = x;
        }
    }
}

// One 64-column head for EPI_QKV: lo = columns [0,32), hi = [32,64).
DTTS_DEV void epilogue_head(const EpiParams &ep, int m, int n0, float (&lo)[32], float (&hi)[32]) {
    const int sect = n0 >> 10;          // 0 q, 1 k, 2 v
    const int c = n0 & 1023;
    const int t = m % ep.tok_per_row;
    const int r = m / ep.tok_per_row;
    if (sect < 2) {
        if (ep.qk_norm) {
            const float *g = sect == 0 ? ep.qn : ep.kn;
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < 32; i++) ss += lo[i] * lo[i] + hi[i] * hi[i];
            const float inv = 1.0f / sqrtf(ss / 64.0f + 1e-6f);
#pragma unroll
            for (int i = 0; i < 32; i++) {
                lo[i] *= inv;
                hi[i] *= inv;
            }
            if (g) {
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    lo[i] *= __ldg(g + i);
                    hi[i] *= __ldg(g + 32 + i);
                }
            }
        }
        const float2 *cs = ep.rope + (long long)(ep.kv_start + t) * 32;
        if (ep.rope_mode == ROPE_HALF) {
            // pairs (d, d + 32), frequency index d
#pragma unroll
            for (int d = 0; d < 32; d++) {
                float2 e = __ldg(cs + d);
                float x1 = lo[d], x2 = hi[d];
                lo[d] = x1 * e.x - x2 * e.y;
                hi[d] = x2 * e.x + x1 * e.y;
            }
        } else {
            // adjacent pairs (2i, 2i + 1), frequency index i
#pragma unroll
            for (int i = 0; i < 16; i++) {
                float2 e = __ldg(cs + i);
                float x0 = lo[2 * i], x1 = lo[2 * i + 1];
                lo[2 * i] = x0 * e.x - x1 * e.y;
                lo[2 * i + 1] = x0 * e.y + x1 * e.x;
            }
#pragma unroll
            for (int i = 0; i < 16; i++) {
                float2 e = __ldg(cs + 16 + i);
                float x0 = hi[2 * i], x1 = hi[2 * i + 1];
                hi[2 * i] = x0 * e.x - x1 * e.y;
                hi[2 * i + 1] = x0 * e.y + x1 * e.x;
            }
        }
    }
    bf16 *dst;
    if (sect == 0) {
        dst = ep.q + (long long)m * ep.ldq + c;
    } else {
        long long row = (long long)r * ep.kv_cap + ep.kv_start + t;
        dst = (sect == 1 ? ep.k : ep.v) + row * ep.ldkv + c;
    }
    store_bf16x32(dst, lo);
    store_bf16x32(dst + 32, hi);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                   int K, EpiParams ep) {
    using Cfg = GemmCfg<BN>;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * Cfg::A_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * Cfg::STAGE_BYTES);
    uint64_t *full = bars;
    uint64_t *empty = bars + STAGES;
    uint64_t *tfull = bars + 2 * STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *fin_bar = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin_bar + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_m = (M + Cfg::BM - 1) / Cfg::BM;
    const int num_n = N / BN;
    const int num_tiles = num_m * num_n;
    const int kblocks = K / Cfg::BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int a = 0; a < 2; a++) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], 128); }
        mbar_init(fin_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmA); tma_prefetch_desc(&tmB); }
    if (warp == 1) { tmem_alloc(tmem_slot, Cfg::TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            int stage = 0;
            uint32_t phase = 0;
            int last_par[STAGES];  // parity of the last load issued per stage, -1: none
#pragma unroll
            for (int s = 0; s < STAGES; s++) last_par[s] = -1;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                const int mb = tile % num_m, nb = tile / num_m;
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, ep.err, DEVERR_TIMEOUT_PRODUCER)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
                    tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full[stage], kb * Cfg::BK, mb * Cfg::BM);
                    tma_load_2d(sB + stage * Cfg::B_BYTES, &tmB, &full[stage], kb * Cfg::BK, nb * BN);
                    last_par[stage] = static_cast<int>(phase);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {
                // Drain: wait (bounded) for every load still in flight so no TMA
                // write lands in shared memory after the CTA has exited.  A stage
                // is re-armed only after its previous phase was consumed, so the
                // last issued parity is the one to wait for.
                for (int s = 0; s < STAGES; s++) {
                    if (last_par[s] < 0) continue;
                    const unsigned long long t0 = globaltimer_ns();
                    while (!mbar_try_wait(&full[s], static_cast<uint32_t>(last_par[s])))
                        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            int stage = 0;
            uint32_t phase = 0;
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, it++) {
                const int acc = it & 1;
                const uint32_t acc_phase = (it >> 1) & 1;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, ep.err, DEVERR_TIMEOUT_MMA)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, ep.err, DEVERR_TIMEOUT_MMA)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * Cfg::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
                    for (int k = 0; k < Cfg::BK / 16; k++) {
                        tc_mma_bf16(d_tmem, sdesc_k128(a0 + k * 32), sdesc_k128(b0 + k * 32), Cfg::IDESC,
                                    (kb | k) != 0 ? 1u : 0u);
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                tc_commit(&tfull[acc]);
            }
            // Every MMA this thread issued must be finished before TMEM is freed
            // (normally already implied by the epilogue having drained).
            tc_commit(fin_bar);
            const unsigned long long t0 = globaltimer_ns();
            while (!mbar_try_wait(fin_bar, 0))
                if (globaltimer_ns() - t0 > kWaitLimitNs) break;
        }
    } else {
        // ---------------- epilogue (warps 2..5 -> TMEM lane quadrant warp % 4)
        const int quad = warp & 3;
        int it = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, it++) {
            const int acc = it & 1;
            const uint32_t acc_phase = (it >> 1) & 1;
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, ep.err, DEVERR_TIMEOUT_EPILOGUE)) break;
            tc_fence_after();
            const int mb = tile % num_m, nb = tile / num_m;
            const int m = mb * Cfg::BM + quad * 32 + lane;
            const uint32_t tbase = tmem_base + acc * BN + (static_cast<uint32_t>(quad * 32) << 16);
            if constexpr (EPI == EPI_QKV) {
#pragma unroll 1
                for (int h = 0; h < BN / 64; h++) {
                    float lo[32], hi[32];
                    tmem_ld32(tbase + h * 64, lo);
                    tmem_ld32(tbase + h * 64 + 32, hi);
                    if (m < M) epilogue_head(ep, m, nb * BN + h * 64, lo, hi);
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < BN / 32; c++) {
                    float v[32];
                    tmem_ld32(tbase + c * 32, v);
                    if (m < M) epilogue_chunk<EPI>(ep, m, nb * BN + c * 32, v);
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

}  // namespace dtts
