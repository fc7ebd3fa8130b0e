// tcgen05 / TMEM / TMA GEMM for sm_100a with fused epilogues.
//
//   C[M, N] = A[M, K] * B[N, K]^T     A, B bf16 K-major (PyTorch Linear: B is
//                                      the [out, in] weight), fp32 accumulate
//   F8 = 1: A, B e4m3 (kind::f8f6f4), C = row_scale[m] * col_scale[n] * acc,
//           so A carries one scale per row and B one per output channel
//
// One persistent CTA per SM:
//   warp 0      TMA producer: A tile 128x64 and B tile BNx64 per stage (bf16;
//               128x128 and BNx128 for e4m3, the same 128-byte rows),
//               128-byte swizzle, mbarrier complete_tx
//   warp 1      TMEM allocator + MMA issuer (one thread): 4 x
//               tcgen05.mma.cta_group::1.kind::f16 (128 x BN x 16) per stage,
//               tcgen05.commit frees the stage
//   warps 2..   NW epilogue warps: tcgen05.ld 32 lanes x 32 columns, fused op,
//               then each warp stages its 32 rows x 128 bytes in shared memory
//               (16-byte chunks XOR-swizzled by row) and writes them back with
//               8 lanes per row, 4 full 128-byte row segments per instruction.
// Two TMEM accumulators (2 x BN fp32 columns) let the epilogue of one tile run
// while the MMAs of the next accumulate.  Work units are (tile, K split).  The
// residual epilogues never read the residual: each warp stages gate * (acc +
// bias) and adds it into the fp32 residual with a TMA bulk reduce-add
// (cp.reduce.async.bulk.tensor ... .add), double-buffered, so K splits simply
// add their partials.  Every
// mbarrier wait is bounded (common.cuh); on expiry the CTA drains and returns
// with an error code in the device error word.
//
// EPI_RESID_GATED_LN also applies the next LayerNorm + modulation to the
// residual rows it completes.  When an epilogue warp's reduce-adds for a tile
// have landed it arrives on the tile's 128-row block counter; arrivals wait on
// nothing.  After its last tile the CTA's mainloop buffers are free: each
// epilogue warp then waits (bounded) until its blocks show every arrival,
// copies its share of their rows into those buffers with bulk copies, and
// normalises them (ln_rows.cuh).  The launch is cooperative, so every CTA whose
// arrivals are awaited is resident.
//
// Shape rules (checked on the host): N % BN == 0, K % (BK * ksplit) == 0,
// ksplit > 1 only for EPI_RESID / EPI_RESID_GATED; rows past M are
// zero-filled by TMA and never stored.  EPI_RESID_GATED_LN: N = kD, ksplit 1,
// BN 128 or 256.
#pragma once
#include "common.cuh"
#include "ln_rows.cuh"

namespace dtts {

enum EpiKind : int {
    EPI_BF16 = 0,     // out_bf16 = acc + bias
    EPI_GELU_BF16,    // out_bf16 = gelu_tanh(acc + bias)          (DiT FFN1)
    EPI_SILU_BF16,    // out_bf16 = silu(acc + bias)               (PE FFN1)
    EPI_F32,          // out_f32  = acc + bias                     (adaLN, projections)
    EPI_RESID,        // resid   += acc + bias                     (PE residual)
    EPI_RESID_GATED,  // resid   += gate[row] * (acc + bias)       (DiT gated residual)
    EPI_QKV,          // q/k/v split, optional per-head RMS norm, RoPE, bf16 stores
    EPI_GELU_F8,      // out_e4m3 = e4m3(gelu_tanh(acc + bias) * out_inv[row])  (DiT FFN1, FP8 path)
    // EPI_QKV with adjacent-pair RoPE.  Callers ask for EPI_QKV and set
    // ep.rope_mode; launch_gemm picks this instance for ROPE_ADJACENT, so each
    // kernel compiles one rotation (with both in one body, the 8-warp bf16
    // kernel spilled at its 168-register cap).
    EPI_QKV_ADJ,
    // EPI_RESID_GATED, then y = LN(resid) * (1 + scale) + shift of the rows
    // the launch completes (ep.ln; bf16 rows, e4m3 rows when F8)
    EPI_RESID_GATED_LN,
};

enum RopeMode : int { ROPE_HALF = 0, ROPE_ADJACENT = 1 };

struct EpiParams {
    const float *bias;        // [N] or nullptr
    // EPI_RESID*: the residual is also described by the third tensor map of the
    // kernel (fp32, box 32 x 32, 128-byte swizzle) for the bulk reduce-add
    void *out;                // EPI_BF16/GELU/SILU: bf16; EPI_F32: f32
    long long ldo;
    float *resid;             // EPI_RESID*: fp32 [M][ldr]
    long long ldr;
    const float *gate;        // EPI_RESID_GATED: gate[(m / tok_per_row) * gate_ld + n]
    long long gate_ld;
    int tok_per_row;          // tokens per gate row / per sequence; maps token m -> (row, t)
    // EPI_QKV: columns [0,1024) -> q, [1024,2048) -> k, [2048,3072) -> v
    bf16 *q, *k, *v;
    long long ldq, ldkv;      // q[m*ldq + c]; k/v[((m/T)*kv_cap + kv_start + m%T) * ldkv + c]
    int kv_cap, kv_start;
    const int *kv_start_dev;  // if set, kv_start is read from device memory (graph-captured decode)
    int qk_norm;              // per-head RMS norm (eps 1e-6) of q and k before RoPE
    const float *qn, *kn;     // its gains [64], or nullptr for none
    const float2 *rope;       // [positions][32] (cos, sin); row index = kv_start + m%T
    int rope_mode;
    int ksplit;               // K splits (>= 1)
    int *err;                 // device error word
    // e4m3 operands (F8 = 1): acc * row_scale[m] * col_scale[n] before the bias
    const float *row_scale;   // [M]
    const float *col_scale;   // [N]
    const float *out_inv;     // EPI_GELU_F8: per-row factor applied before the e4m3 conversion
    // Convolution as a GEMM over taps (tap_kb > 0): K is taps x channels, tap-major,
    // tap_kb k-blocks per tap.  K-block kb of tap j = kb / tap_kb reads A at
    // column (kb mod tap_kb) * BK and row m + tap_base + j * tap_step; rows
    // outside [0, M) read as zero (TMA fill), which is the zero padding of a
    // causal (or centred) time convolution over A = [time][channels].
    int tap_kb, tap_base, tap_step;
    // EPI_RESID_GATED_LN: the LayerNorm's modulation rows and output, and one
    // arrival counter per 128-row block (zero between launches; the last warp
    // to leave a block's wait puts it back to zero)
    LnParams ln;
    unsigned *ln_count;
    // 1: tiles M block by M block (the N tiles of a block on neighbouring
    // CTAs, sharing its A rows through L2), for a GEMM whose A does not stay in
    // L2 across N passes; 0: N block by N block (neighbours share a weight tile)
    int mb_major;
};

__host__ __device__ constexpr bool is_gated(int epi) { return epi == EPI_RESID_GATED || epi == EPI_RESID_GATED_LN; }
__host__ __device__ constexpr bool is_resid(int epi) { return epi == EPI_RESID || is_gated(epi); }
__host__ __device__ constexpr bool is_qkv(int epi) { return epi == EPI_QKV || epi == EPI_QKV_ADJ; }

constexpr int kRopeSmemRows = 64;   // sequences up to this length read RoPE from shared memory
// Shared-memory RoPE row stride in float2: 32 pairs + 2 of padding (272 bytes).
// Each lane reads its own token's row, so with 256-byte rows the 8 lanes of a
// 16-byte load phase would all hit the same four banks; 272 bytes spreads them.
constexpr int kRopeRowF2 = 34;

template <int BN, int NW, int EPI, int F8 = 0>
struct GemmCfg {
    static constexpr int BM = 128;
    static constexpr int BK = F8 ? 128 : 64;   // elements per stage: 128 bytes of K either way
    static constexpr int A_BYTES = BM * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGE_BUFS = is_resid(EPI) ? 2 : 1;  // staging buffers per epilogue warp
    static constexpr int STAGE_STAGING = NW * STAGE_BUFS * 32 * 128;  // 32 rows x 128 bytes each
    static constexpr int SMEM_MAX = 227 * 1024;
    static constexpr int BAR_BYTES = 256;
    // EPI_QKV: the q/k RMS gains (128 floats) and up to kRopeSmemRows rows of
    // the RoPE table staged in shared memory once per CTA
    static constexpr int CONST_BYTES = is_qkv(EPI) ? 512 + kRopeSmemRows * kRopeRowF2 * 8 : 0;
    static constexpr int STAGES_FIT = (SMEM_MAX - STAGE_STAGING - CONST_BYTES - BAR_BYTES - 1024) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
    static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGE_STAGING + CONST_BYTES + BAR_BYTES + 1024;  // +1024 alignment slack
    static constexpr int THREADS = 64 + NW * 32;
    static constexpr uint32_t IDESC = F8 ? idesc_e4m3(BM, BN) : idesc_bf16(BM, BN);
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN");
    static_assert(2 * BN <= 512, "two accumulators must fit in TMEM");
    static_assert(NW == 4 || NW == 8, "epilogue warps");
    static_assert(STAGES >= 3, "pipeline depth");
    static_assert(EPI != EPI_GELU_F8 || (F8 && BN % 128 == 0), "e4m3 output tiles are whole 128-byte rows");
};

DTTS_DEV float gelu_tanh_fast(float x) {
    const float c1 = 0.7978845608028654f, c2 = 0.044715f;
    return 0.5f * x * (1.0f + tanh_hw(c1 * (x + c2 * x * x * x)));
}
// x / (1 + e^-x) with the fast divide (2 ulp); for x < -88 the denominator is
// +inf and the result 0.
DTTS_DEV float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// ---- per-warp staging buffer: 32 rows x 128 bytes, 16-byte chunks swizzled by row
DTTS_DEV uint32_t stage_off(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

DTTS_DEV void stage_put(uint8_t *wbuf, int lane, const float (&v)[32]) {
#pragma unroll
    for (int c = 0; c < 8; c++)
        *reinterpret_cast<float4 *>(wbuf + stage_off(lane, c)) = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}
DTTS_DEV void stage_put_bf16(uint8_t *wbuf, int lane, const float (&lo)[32], const float (&hi)[32]) {
#pragma unroll
    for (int c = 0; c < 4; c++) {
        uint4 u;
        u.x = pack_bf16x2(lo[8 * c + 0], lo[8 * c + 1]); u.y = pack_bf16x2(lo[8 * c + 2], lo[8 * c + 3]);
        u.z = pack_bf16x2(lo[8 * c + 4], lo[8 * c + 5]); u.w = pack_bf16x2(lo[8 * c + 6], lo[8 * c + 7]);
        *reinterpret_cast<uint4 *>(wbuf + stage_off(lane, c)) = u;
        u.x = pack_bf16x2(hi[8 * c + 0], hi[8 * c + 1]); u.y = pack_bf16x2(hi[8 * c + 2], hi[8 * c + 3]);
        u.z = pack_bf16x2(hi[8 * c + 4], hi[8 * c + 5]); u.w = pack_bf16x2(hi[8 * c + 6], hi[8 * c + 7]);
        *reinterpret_cast<uint4 *>(wbuf + stage_off(lane, 4 + c)) = u;
    }
}

// Per-column constants of one 32-column chunk (e4m3 column scale, bias),
// loaded into registers BEFORE the chunk's TMEM read so that their latency
// overlaps it instead of following it.
struct Col32 {
    float4 s[8], b[8];
};
template <bool SCALE>
DTTS_DEV void col32_load(Col32 &c, const float *cs, const float *bias, int n0) {
    if constexpr (SCALE) {
        const float4 *s4 = reinterpret_cast<const float4 *>(cs + n0);
#pragma unroll
        for (int i = 0; i < 8; i++) c.s[i] = __ldg(s4 + i);
    }
    if (bias) {
        const float4 *b4 = reinterpret_cast<const float4 *>(bias + n0);
#pragma unroll
        for (int i = 0; i < 8; i++) c.b[i] = __ldg(b4 + i);
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) c.b[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}
// v = v * rs * scale + bias (SCALE) or v + bias
template <bool SCALE>
DTTS_DEV void col32_apply(float (&v)[32], const Col32 &c, float rs) {
#pragma unroll
    for (int i = 0; i < 8; i++) {
        if constexpr (SCALE) {
            v[4 * i + 0] = fmaf(v[4 * i + 0], rs * c.s[i].x, c.b[i].x);
            v[4 * i + 1] = fmaf(v[4 * i + 1], rs * c.s[i].y, c.b[i].y);
            v[4 * i + 2] = fmaf(v[4 * i + 2], rs * c.s[i].z, c.b[i].z);
            v[4 * i + 3] = fmaf(v[4 * i + 3], rs * c.s[i].w, c.b[i].w);
        } else {
            v[4 * i + 0] += c.b[i].x; v[4 * i + 1] += c.b[i].y; v[4 * i + 2] += c.b[i].z; v[4 * i + 3] += c.b[i].w;
        }
    }
}

DTTS_DEV void load_bias32(float (&v)[32], const float *bias, int n0) {
    if (!bias) return;
    const float4 *b4 = reinterpret_cast<const float4 *>(bias + n0);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float4 b = __ldg(b4 + i);
        v[4 * i + 0] += b.x; v[4 * i + 1] += b.y; v[4 * i + 2] += b.z; v[4 * i + 3] += b.w;
    }
}

// Per-thread head transform for EPI_QKV: lo = head columns [0,32), hi = [32,64).
// sgain: the q gains then the k gains (shared memory, ones where absent);
// srope: RoPE rows kv_start.. in shared memory (kRopeRowF2 float2 apart), or
// nullptr to read ep.rope (32 float2 apart).
// The RoPE rows are read with generic loads: they may be shared or global.
template <int MODE>
DTTS_DEV void qkv_head_transform(const EpiParams &ep, int m, int sect, float (&lo)[32], float (&hi)[32],
                                 const float *sgain, const float4 *srope, int kv_start) {
    if (sect == 2) return;  // v: plain
    const int t = m % ep.tok_per_row;
    if (ep.qk_norm) {
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
            s0 = fmaf(lo[i], lo[i], s0); s1 = fmaf(hi[i], hi[i], s1);
            s2 = fmaf(lo[i + 1], lo[i + 1], s2); s3 = fmaf(hi[i + 1], hi[i + 1], s3);
        }
        const float inv = 1.0f / sqrtf(((s0 + s1) + (s2 + s3)) / 64.0f + 1e-6f);
        const float4 *g4 = reinterpret_cast<const float4 *>(sgain + sect * 64);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 a = g4[i], b = g4[8 + i];
            lo[4 * i + 0] *= inv * a.x; lo[4 * i + 1] *= inv * a.y; lo[4 * i + 2] *= inv * a.z; lo[4 * i + 3] *= inv * a.w;
            hi[4 * i + 0] *= inv * b.x; hi[4 * i + 1] *= inv * b.y; hi[4 * i + 2] *= inv * b.z; hi[4 * i + 3] *= inv * b.w;
        }
    }
    const float4 *cs = srope ? srope + t * (kRopeRowF2 / 2)
                             : reinterpret_cast<const float4 *>(ep.rope + (long long)(kv_start + t) * 32);
    if constexpr (MODE == ROPE_HALF) {
        // pairs (d, d + 32), frequency index d
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const float4 e = cs[i];  // (cos_2i, sin_2i, cos_2i+1, sin_2i+1)
            float x1 = lo[2 * i], x2 = hi[2 * i];
            lo[2 * i] = x1 * e.x - x2 * e.y;
            hi[2 * i] = x2 * e.x + x1 * e.y;
            x1 = lo[2 * i + 1]; x2 = hi[2 * i + 1];
            lo[2 * i + 1] = x1 * e.z - x2 * e.w;
            hi[2 * i + 1] = x2 * e.z + x1 * e.w;
        }
    } else {
        // adjacent pairs (2i, 2i + 1), frequency index i
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 e = cs[i];  // frequencies 2i, 2i+1
            float x0 = lo[4 * i], x1 = lo[4 * i + 1];
            lo[4 * i] = x0 * e.x - x1 * e.y;
            lo[4 * i + 1] = x0 * e.y + x1 * e.x;
            x0 = lo[4 * i + 2]; x1 = lo[4 * i + 3];
            lo[4 * i + 2] = x0 * e.z - x1 * e.w;
            lo[4 * i + 3] = x0 * e.w + x1 * e.z;
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 e = cs[8 + i];  // frequencies 16 + 2i, 16 + 2i + 1
            float x0 = hi[4 * i], x1 = hi[4 * i + 1];
            hi[4 * i] = x0 * e.x - x1 * e.y;
            hi[4 * i + 1] = x0 * e.y + x1 * e.x;
            x0 = hi[4 * i + 2]; x1 = hi[4 * i + 3];
            hi[4 * i + 2] = x0 * e.z - x1 * e.w;
            hi[4 * i + 3] = x0 * e.w + x1 * e.z;
        }
    }
}

// Tile index -> (M block, N block): N-block-major (consecutive CTAs share the
// weight tile) or, with ep.mb_major and always for EPI_RESID_GATED_LN (whose
// blocks then complete in order), M-block-major.
template <int EPI>
DTTS_DEV void tile_coords(int tile, int num_m, int num_n, int mb_major, int &mb, int &nb) {
    if (EPI == EPI_RESID_GATED_LN || mb_major) { mb = tile / num_n; nb = tile - mb * num_n; }
    else { nb = tile / num_m; mb = tile - nb * num_m; }
}

template <int BN, int EPI, int NW, int F8 = 0>
__global__ void __launch_bounds__(GemmCfg<BN, NW, EPI, F8>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmR, int M, int N, int K, EpiParams ep) {
    using Cfg = GemmCfg<BN, NW, EPI, F8>;
    constexpr int STAGES = Cfg::STAGES;
    constexpr int EPI_THREADS = NW * 32;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * Cfg::A_BYTES;
    uint8_t *sStage = smem + STAGES * Cfg::STAGE_BYTES;
    uint8_t *sConst = sStage + Cfg::STAGE_STAGING;   // EPI_QKV: gains, RoPE rows
    uint64_t *bars = reinterpret_cast<uint64_t *>(sConst + Cfg::CONST_BYTES);
    uint64_t *full = bars;
    uint64_t *empty = bars + STAGES;
    uint64_t *tfull = bars + 2 * STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *fin_bar = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin_bar + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    uint64_t *ln_bar = fin_bar + 2;   // EPI_RESID_GATED_LN: one per epilogue warp
    static_assert((2 * STAGES + 6 + (EPI == EPI_RESID_GATED_LN ? NW : 0)) * 8 <= Cfg::BAR_BYTES, "barrier area");

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_m = (M + Cfg::BM - 1) / Cfg::BM;
    const int num_n = N / BN;
    const int num_tiles = num_m * num_n;
    const int ksplit = ep.ksplit > 0 ? ep.ksplit : 1;
    const int num_units = num_tiles * ksplit;
    const int kblocks = K / Cfg::BK / ksplit;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int a = 0; a < 2; a++) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], EPI_THREADS); }
        mbar_init(fin_bar, 1);
        if constexpr (EPI == EPI_RESID_GATED_LN)
            for (int w = 0; w < NW; w++) mbar_init(&ln_bar[w], 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmA); tma_prefetch_desc(&tmB); }
    if (warp == 1) { tmem_alloc(tmem_slot, Cfg::TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const bool producer = warp == 0 && lane == 0;
    if (!producer) { pdl_wait(); pdl_trigger(); }

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            int stage = 0;
            uint32_t phase = 0;
            int last_par[STAGES];  // parity of the last load issued per stage, -1: none
#pragma unroll
            for (int s = 0; s < STAGES; s++) last_par[s] = -1;
            // The first unit's weight (B) tiles do not depend on earlier
            // kernels: they are requested before the wait on the previous
            // kernel, into stages 0 .. npre-1, whose A tiles follow after it.
            int npre = 0;
            if (blockIdx.x < num_units) {
                const int tile = blockIdx.x % num_tiles, split = blockIdx.x / num_tiles;
                int mb, nb;
                tile_coords<EPI>(tile, num_m, num_n, ep.mb_major, mb, nb);
                const int kb0 = split * kblocks;
                npre = kblocks < STAGES ? kblocks : STAGES;
                for (int kb = 0; kb < npre; kb++) {
                    mbar_arrive_expect_tx(&full[kb], Cfg::STAGE_BYTES);   // B now, A after the wait
                    tma_load_2d(sB + kb * Cfg::B_BYTES, &tmB, &full[kb], (kb0 + kb) * Cfg::BK, nb * BN);
                    last_par[kb] = 0;
                }
            }
            pdl_wait();
            pdl_trigger();
            bool ok = true;
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
                const int tile = u % num_tiles, split = u / num_tiles;
                int mb, nb;
                tile_coords<EPI>(tile, num_m, num_n, ep.mb_major, mb, nb);
                const int kb0 = split * kblocks;
                for (int kb = 0; kb < kblocks; kb++) {
                    const bool pre = u == (int)blockIdx.x && kb < npre;   // stage == kb, phase 0, B in flight
                    if (!pre) {
                        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, ep.err, DEVERR_TIMEOUT_PRODUCER)) { ok = false; break; }
                        mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
                    }
                    int ax = (kb0 + kb) * Cfg::BK, ay = mb * Cfg::BM;
                    if (ep.tap_kb > 0) {
                        const int tap = (kb0 + kb) / ep.tap_kb;
                        ax = (kb0 + kb - tap * ep.tap_kb) * Cfg::BK;
                        ay += ep.tap_base + tap * ep.tap_step;
                    }
                    tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full[stage], ax, ay);
                    if (!pre)
                        tma_load_2d(sB + stage * Cfg::B_BYTES, &tmB, &full[stage], (kb0 + kb) * Cfg::BK, nb * BN);
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
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, it++) {
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
                    // four MMAs of 32 bytes of K (16 bf16 or 32 e4m3 elements)
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        if constexpr (F8)
                            tc_mma_f8(d_tmem, sdesc_k128(a0 + k * 32), sdesc_k128(b0 + k * 32), Cfg::IDESC,
                                      (kb | k) != 0 ? 1u : 0u);
                        else
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
        // ---------------- epilogue: warps 2.. ; TMEM lane quadrant = warp % 4,
        // with 8 warps the two warps of a quadrant take alternate column chunks
        const int ew = warp - 2;
        const int quad = warp & 3;
        float *sgain = nullptr;
        const float4 *srope = nullptr;
        const int kv_start = ep.kv_start_dev ? *ep.kv_start_dev : ep.kv_start;
        const bool kv_dense = ep.kv_cap == ep.tok_per_row && kv_start == 0;
        if constexpr (is_qkv(EPI)) {
            sgain = reinterpret_cast<float *>(sConst);
            float2 *rp = reinterpret_cast<float2 *>(sConst + 512);
            const int et = threadIdx.x - 64;
            for (int i = et; i < 128; i += EPI_THREADS) {
                const float *g = i < 64 ? ep.qn : ep.kn;
                sgain[i] = g ? __ldg(g + (i & 63)) : 1.0f;
            }
            const bool rope_smem = ep.rope != nullptr && ep.tok_per_row <= kRopeSmemRows;
            if (rope_smem)
                for (int i = et; i < ep.tok_per_row * 32; i += EPI_THREADS)
                    rp[(i >> 5) * kRopeRowF2 + (i & 31)] = __ldg(ep.rope + (long long)kv_start * 32 + i);
            asm volatile("bar.sync 1, %0;\n" ::"r"(EPI_THREADS) : "memory");
            if (rope_smem) srope = reinterpret_cast<const float4 *>(rp);
        }
        const int half = (NW == 8) ? (ew >> 2) : 0;
        constexpr int CSTEP = (NW == 8) ? 2 : 1;
        uint8_t *wbuf = sStage + ew * Cfg::STAGE_BUFS * 32 * 128;
        int cc = 0;                   // chunks issued by this warp (staging buffer parity)
        const int rsub = lane >> 3;   // row within a group of 4 (write-back phase)
        const int chunk = lane & 7;   // 16-byte chunk of the 128-byte row segment
        int it = 0;
        for (int u = blockIdx.x; u < num_units; u += gridDim.x, it++) {
            const int acc = it & 1;
            const uint32_t acc_phase = (it >> 1) & 1;
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, ep.err, DEVERR_TIMEOUT_EPILOGUE)) break;
            tc_fence_after();
            const int tile = u % num_tiles, split = u / num_tiles;
            int mb, nb;
            tile_coords<EPI>(tile, num_m, num_n, ep.mb_major, mb, nb);
            const int m_base = mb * Cfg::BM + quad * 32;
            const uint32_t tbase = tmem_base + acc * BN + (static_cast<uint32_t>(quad * 32) << 16);
            float rs = 0.f;   // e4m3 row scale of this thread's row
            if constexpr (F8)
                if (m_base + lane < M) rs = __ldg(ep.row_scale + m_base + lane);
            if constexpr (is_qkv(EPI) || EPI == EPI_BF16 || EPI == EPI_GELU_BF16 || EPI == EPI_SILU_BF16) {
                // 64 columns (one head / 128 bytes of bf16) per chunk
#pragma unroll 1
                for (int c = half; c < BN / 64; c += CSTEP) {
                    const int n0 = nb * BN + c * 64;
                    // the DiT QKV projection has no bias: bf16 QKV needs no column constants
                    constexpr bool kCols = F8 || !is_qkv(EPI);
                    Col32 cl, ch;
                    if constexpr (kCols) {
                        col32_load<F8 != 0>(cl, ep.col_scale, is_qkv(EPI) ? nullptr : ep.bias, n0);
                        col32_load<F8 != 0>(ch, ep.col_scale, is_qkv(EPI) ? nullptr : ep.bias, n0 + 32);
                    }
                    float lo[32], hi[32];
                    tmem_ld32x2(tbase + c * 64, tbase + c * 64 + 32, lo, hi);
                    if constexpr (kCols) {
                        col32_apply<F8 != 0>(lo, cl, rs);
                        col32_apply<F8 != 0>(hi, ch, rs);
                    }
                    const int m_self = m_base + lane;
                    if constexpr (is_qkv(EPI)) {
                        constexpr int kMode = EPI == EPI_QKV_ADJ ? ROPE_ADJACENT : ROPE_HALF;
                        if (m_self < M) qkv_head_transform<kMode>(ep, m_self, n0 >> 10, lo, hi, sgain, srope, kv_start);
                    } else {
                        if constexpr (EPI == EPI_GELU_BF16) {
#pragma unroll
                            for (int i = 0; i < 32; i++) { lo[i] = gelu_tanh_fast(lo[i]); hi[i] = gelu_tanh_fast(hi[i]); }
                        }
                        if constexpr (EPI == EPI_SILU_BF16) {
#pragma unroll
                            for (int i = 0; i < 32; i++) { lo[i] = silu_f(lo[i]); hi[i] = silu_f(hi[i]); }
                        }
                    }
                    __syncwarp();
                    stage_put_bf16(wbuf, lane, lo, hi);
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int r = rsub + 4 * i;
                        const int m = m_base + r;
                        const uint4 val = *reinterpret_cast<const uint4 *>(wbuf + stage_off(r, chunk));
                        if (m >= M) continue;
                        bf16 *dst;
                        if constexpr (is_qkv(EPI)) {
                            const int sect = n0 >> 10, col = (n0 & 1023) + chunk * 8;
                            if (sect == 0) {
                                dst = ep.q + (long long)m * ep.ldq + col;
                            } else {
                                // token m of sequence m / T sits at row m of a dense cache (the DiT)
                                const long long row = kv_dense ? (long long)m
                                                               : (long long)(m / ep.tok_per_row) * ep.kv_cap +
                                                                     kv_start + (m % ep.tok_per_row);
                                dst = (sect == 1 ? ep.k : ep.v) + row * ep.ldkv + col;
                            }
                        } else {
                            dst = reinterpret_cast<bf16 *>(ep.out) + (long long)m * ep.ldo + n0 + chunk * 8;
                        }
                        *reinterpret_cast<uint4 *>(dst) = val;
                    }
                }
            } else if constexpr (EPI == EPI_GELU_F8) {
                // e4m3 results: 128 columns (one 128-byte row segment) per pass,
                // built from four 32-column TMEM loads
                const float oinv = (m_base + lane < M) ? __ldg(ep.out_inv + m_base + lane) : 0.f;
#pragma unroll 1
                for (int sg = half; sg < BN / 128; sg += CSTEP) {
                    const int n_seg = nb * BN + sg * 128;
                    __syncwarp();
#pragma unroll 1
                    for (int sub = 0; sub < 4; sub++) {
                        const int n0 = n_seg + sub * 32;
                        Col32 cv;
                        col32_load<true>(cv, ep.col_scale, ep.bias, n0);
                        float v[32];
                        tmem_ld32(tbase + sg * 128 + sub * 32, v);
                        col32_apply<true>(v, cv, rs);
                        uint4 w0, w1;
                        w0.x = pack_e4m3x4(gelu_tanh_fast(v[0]) * oinv, gelu_tanh_fast(v[1]) * oinv,
                                           gelu_tanh_fast(v[2]) * oinv, gelu_tanh_fast(v[3]) * oinv);
                        w0.y = pack_e4m3x4(gelu_tanh_fast(v[4]) * oinv, gelu_tanh_fast(v[5]) * oinv,
                                           gelu_tanh_fast(v[6]) * oinv, gelu_tanh_fast(v[7]) * oinv);
                        w0.z = pack_e4m3x4(gelu_tanh_fast(v[8]) * oinv, gelu_tanh_fast(v[9]) * oinv,
                                           gelu_tanh_fast(v[10]) * oinv, gelu_tanh_fast(v[11]) * oinv);
                        w0.w = pack_e4m3x4(gelu_tanh_fast(v[12]) * oinv, gelu_tanh_fast(v[13]) * oinv,
                                           gelu_tanh_fast(v[14]) * oinv, gelu_tanh_fast(v[15]) * oinv);
                        w1.x = pack_e4m3x4(gelu_tanh_fast(v[16]) * oinv, gelu_tanh_fast(v[17]) * oinv,
                                           gelu_tanh_fast(v[18]) * oinv, gelu_tanh_fast(v[19]) * oinv);
                        w1.y = pack_e4m3x4(gelu_tanh_fast(v[20]) * oinv, gelu_tanh_fast(v[21]) * oinv,
                                           gelu_tanh_fast(v[22]) * oinv, gelu_tanh_fast(v[23]) * oinv);
                        w1.z = pack_e4m3x4(gelu_tanh_fast(v[24]) * oinv, gelu_tanh_fast(v[25]) * oinv,
                                           gelu_tanh_fast(v[26]) * oinv, gelu_tanh_fast(v[27]) * oinv);
                        w1.w = pack_e4m3x4(gelu_tanh_fast(v[28]) * oinv, gelu_tanh_fast(v[29]) * oinv,
                                           gelu_tanh_fast(v[30]) * oinv, gelu_tanh_fast(v[31]) * oinv);
                        *reinterpret_cast<uint4 *>(wbuf + stage_off(lane, 2 * sub)) = w0;
                        *reinterpret_cast<uint4 *>(wbuf + stage_off(lane, 2 * sub + 1)) = w1;
                    }
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int r = rsub + 4 * i;
                        const int m = m_base + r;
                        const uint4 val = *reinterpret_cast<const uint4 *>(wbuf + stage_off(r, chunk));
                        if (m >= M) continue;
                        *reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(ep.out) + (long long)m * ep.ldo + n_seg +
                                                   chunk * 16) = val;
                    }
                }
            } else if constexpr (EPI == EPI_F32) {
                // fp32 results: 32 columns (128 bytes) per chunk
#pragma unroll 1
                for (int c = half; c < BN / 32; c += CSTEP) {
                    const int n0 = nb * BN + c * 32;
                    Col32 cv;
                    col32_load<F8 != 0>(cv, ep.col_scale, ep.bias, n0);
                    float v[32];
                    tmem_ld32(tbase + c * 32, v);
                    col32_apply<F8 != 0>(v, cv, rs);
                    __syncwarp();
                    stage_put(wbuf, lane, v);
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int r = rsub + 4 * i;
                        const int m = m_base + r;
                        const float4 val = *reinterpret_cast<const float4 *>(wbuf + stage_off(r, chunk));
                        if (m >= M) continue;
                        *reinterpret_cast<float4 *>(reinterpret_cast<float *>(ep.out) + (long long)m * ep.ldo + n0 +
                                                    chunk * 4) = val;
                    }
                }
            } else {
                // residual: stage gate * (acc + bias) and bulk-reduce it into the
                // fp32 residual (32 rows x 32 columns per warp per chunk)
                const int m_self = m_base + lane;
                const float4 *g4 = nullptr;
                if constexpr (is_gated(EPI))
                    if (m_self < M) g4 = reinterpret_cast<const float4 *>(ep.gate + (long long)(m_self / ep.tok_per_row) * ep.gate_ld);
#pragma unroll 1
                for (int c = half; c < BN / 32; c += CSTEP, cc++) {
                    const int n0 = nb * BN + c * 32;
                    Col32 cv;
                    col32_load<F8 != 0>(cv, ep.col_scale, split == 0 ? ep.bias : nullptr, n0);
                    float4 gq[8];
                    if constexpr (is_gated(EPI)) {
#pragma unroll
                        for (int i = 0; i < 8; i++) gq[i] = g4 ? __ldg(g4 + (n0 >> 2) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                    float v[32];
                    tmem_ld32(tbase + c * 32, v);
                    col32_apply<F8 != 0>(v, cv, rs);
                    if (m_self >= M) {
#pragma unroll
                        for (int i = 0; i < 32; i++) v[i] = 0.f;
                    } else if constexpr (is_gated(EPI)) {
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            v[4 * i + 0] *= gq[i].x; v[4 * i + 1] *= gq[i].y; v[4 * i + 2] *= gq[i].z; v[4 * i + 3] *= gq[i].w;
                        }
                    }
                    uint8_t *buf = wbuf + (cc & 1) * 32 * 128;
                    if (lane == 0) bulk_wait_read<1>();   // the reduce that last read this buffer is done
                    __syncwarp();
                    stage_put(buf, lane, v);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0 && m_base < M) {
                        tma_reduce_add_2d(&tmR, buf, n0, m_base);
                        bulk_commit();
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
            if constexpr (EPI == EPI_RESID_GATED_LN) {
                // Once this warp's reduce-adds have landed, publish them and
                // arrive on the M block's counter (one arrival per warp of each
                // of the block's tiles).  Nothing here waits on another CTA.
                if (lane == 0) {
                    bulk_wait<0>();
                    fence_proxy_async_global();
                    __threadfence();
                    atomicAdd(ep.ln_count + mb, 1u);
                }
                __syncwarp();
            }
        }
        if constexpr (EPI == EPI_RESID_GATED_LN) {
            // LayerNorm of this CTA's share of each block it worked on: rows
            // [nb * per, (nb + 1) * per) of the block, rows_w of them per warp.
            // Every MMA of the CTA has completed (its last accumulator was
            // full), so the mainloop's stage buffers are free: each warp copies
            // its rows there with bulk copies (which need no L1, unlike loads
            // through the SM's small L1) after the block's counter shows every
            // arrival.  The warp's staging buffers hold the modulation row.
            constexpr int num_n_c = kD / BN;
            constexpr int per = Cfg::BM / num_n_c;
            constexpr int rows_w = (per + NW - 1) / NW;
            static_assert(NW * rows_w * kD * 4 <= STAGES * Cfg::STAGE_BYTES, "LayerNorm rows fit in the stage buffers");
            static_assert(Cfg::STAGE_BUFS * 32 * 128 >= 2 * kD * 4, "a warp's staging holds one modulation row");
            float *rows_s = reinterpret_cast<float *>(smem) + (size_t)ew * rows_w * kD;
            float *mod_s = reinterpret_cast<float *>(wbuf);   // [2][kD]: shift, scale
            ModRow st{-1, mod_s, mod_s + kD};
            const unsigned need = static_cast<unsigned>(num_n * NW);
            uint32_t lphase = 0;
            bool pending = false;   // lane 0: copies of phase lphase issued and not yet waited for
            bool ok = !*abort_flag;
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
                int mb, nb;
                tile_coords<EPI>(u % num_tiles, num_m, num_n, ep.mb_major, mb, nb);
                const int r_lo = mb * Cfg::BM + nb * per + ew * rows_w;
                const int r_hi = min(min(r_lo + rows_w, mb * Cfg::BM + (nb + 1) * per), M);
                const int nrows = r_hi - r_lo;   // may be <= 0 for a ragged last block
                unsigned *cnt = ep.ln_count + mb;
                int wok = 1;
                if (lane == 0) {
                    const unsigned long long t0 = globaltimer_ns();
                    while (ld_acquire_u32(cnt) < need)
                        if (globaltimer_ns() - t0 > kWaitLimitNs || *reinterpret_cast<volatile int *>(ep.err)) {
                            wok = 0;
                            atomicCAS(ep.err, 0, DEVERR_TIMEOUT_BARRIER);
                            break;
                        }
                    if (wok) {
                        if (nrows > 0) {
                            fence_proxy_async_global();
                            mbar_arrive_expect_tx(&ln_bar[ew], static_cast<uint32_t>(nrows) * kD * 4);
                            for (int i = 0; i < nrows; i++)
                                bulk_load_1d(rows_s + i * kD, ep.resid + (long long)(r_lo + i) * kD, kD * 4, &ln_bar[ew]);
                            pending = true;
                        }
                        // the last of the block's warps to leave re-arms the counter
                        if (atomicAdd(cnt, 1u) == 2u * need - 1u) atomicExch(cnt, 0u);
                    }
                }
                wok = __shfl_sync(0xffffffffu, wok, 0);
                if (!wok) { ok = false; break; }
                if (nrows <= 0) continue;
                const long long mr = r_lo / ep.ln.tok_per_row;
                if (mr != st.mr) {
                    ln_stage_mod(ep.ln, mr, mod_s, mod_s + kD, lane);
                    __syncwarp();
                    st.mr = mr;
                }
                if (!mbar_wait(&ln_bar[ew], lphase, abort_flag, ep.err, DEVERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
                pending = false;
                lphase ^= 1u;
                ln_rows_smem<rows_w, F8 != 0>(rows_s, nrows, r_lo, ep.ln, st, lane);
                // these rows' shared-memory reads before the next bulk copies overwrite them
                fence_proxy_async_smem();
                __syncwarp();
            }
            if (pending && lane == 0) {
                // copies may still be in flight into shared memory: wait for them
                // (bounded) before the CTA exits
                const unsigned long long t0 = globaltimer_ns();
                while (!mbar_try_wait(&ln_bar[ew], lphase))
                    if (globaltimer_ns() - t0 > kWaitLimitNs) break;
            }
        }
        if constexpr (is_resid(EPI)) {
            if (lane == 0) bulk_wait<0>();   // every reduce of this warp has landed
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
