// DiT attention at L = 64 on the 5th-generation tensor cores (tcgen05).
//
// A work unit is (sequence pair, head): the 128 query rows of two consecutive
// sequences (rows 64 p .. 64 p + 127 of the [rows * 64][1024] q / k / v
// buffers) and one head's 64 columns.  Per unit, one CTA of 4 warps:
//   TMA    Q, K, V tiles 128 rows x 64 columns (128-byte swizzle)
//   MMA 1  S = Q K^T into TMEM (128 x 128 fp32); only the two 64 x 64 blocks
//          on the diagonal (each sequence against its own keys) are read
//   all    thread i holds query row i: its 64 scores from TMEM, scaled by
//          log2(e)/8, masked (-inf), max, exp2, sum; P (bf16) written K-major
//          into shared memory with zeros off the diagonal block
//   MMA 2  O = P V (K = 128 keys; V read MN-major as loaded) into TMEM columns 0..63
//   all    O / l to bf16 (or to e4m3 with the sequence's scale bound, the FP8
//          engine), row i of the head's 64 output columns, while the next
//          unit's Q, K, V load
// Numerics are those of attn_short_kernel: fp32 scores and softmax, P rounded
// to bf16 for P V, fp32 accumulation.  Every mbarrier wait is bounded.
#include "kernels.cuh"

#include <cstdlib>

namespace dtts {

namespace {
constexpr int kTcThreads = 128;
constexpr int kTile = 128 * 128;             // bytes of one 128-row x 64-column bf16 tile
// shared memory: Q | K (later P, two 64-key chunks) | V | barriers
constexpr int kSmQ = 0, kSmK = kTile, kSmV = 2 * kTile, kSmBar = 3 * kTile;
constexpr int kTcSmem = kSmBar + 64 + 1024;  // + alignment slack
// O = P V reads B = V in its loaded layout, N (head dims) contiguous: the
// descriptor's transpose-B bit (16) marks B as MN-major
constexpr uint32_t kIdescS = idesc_bf16(128, 128), kIdescO = idesc_bf16(128, 64) | (1u << 16);

// byte offset of 16-byte unit u of row r in a K-major tile with 128-byte swizzle
DTTS_DEV uint32_t sw128(int r, int u) { return (uint32_t)(r * 128 + ((u ^ (r & 7)) << 4)); }

__global__ void __launch_bounds__(kTcThreads, 4)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, bf16 *__restrict__ out, long long ldo, int rows,
                   const uint32_t *__restrict__ mask_bits, float scale_log2, int *err, uint8_t *__restrict__ o8,
                   float *__restrict__ o_scale, const float *__restrict__ unorm, float vbound, const bf16 *dq,
                   const bf16 *dk, const bf16 *dv) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + kSmBar);
    uint64_t *mma = full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int n_pairs = (rows + 1) / 2, units = n_pairs * kH;

    if (tid == 0) {
        mbar_init(full, 1);
        mbar_init(mma, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tq); tma_prefetch_desc(&tk); tma_prefetch_desc(&tv);
    }
    if (warp == 0) { tmem_alloc(tmem_slot, 128); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;

    // this thread's query row within the pair, its sequence (0 / 1) and its mask words
    const int i = tid, s = i >> 6, qi = i & 63;
    uint32_t m0 = ~0u, m1 = ~0u;
    if (mask_bits) { m0 = mask_bits[qi * 2]; m1 = mask_bits[qi * 2 + 1]; }
    const uint32_t trow = tbase + (static_cast<uint32_t>(warp * 32) << 16);   // this warp's TMEM lanes

    // Q, K, V of unit v into the tiles, completing on `full`
    auto issue = [&](int v) {
        const int pv = v / kH, hv = v % kH;
        mbar_arrive_expect_tx(full, 3 * kTile);
        tma_load_2d(sm + kSmQ, &tq, full, hv * kHD, pv * 128);
        tma_load_2d(sm + kSmK, &tk, full, hv * kHD, pv * 128);
        tma_load_2d(sm + kSmV, &tv, full, hv * kHD, pv * 128);
    };
    bool pending = false;   // a load of phase `ph` has been issued and not yet waited for
    if (tid == 0 && (int)blockIdx.x < units) { issue(blockIdx.x); pending = true; }
    uint32_t ph = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ph ^= 1u) {
        const int pr = u / kH, h = u % kH;
        // every wait is followed by a CTA-wide vote, so that all threads leave the loop together
        if (__syncthreads_or(!mbar_wait(full, ph, abort_flag, err, DEVERR_TIMEOUT_PRODUCER))) break;
        pending = false;
        if (dq && pr * 128 + tid < rows * 64) {
            // this unit is the only reader of its rows' head slices (one 128-byte
            // line each): drop them from L2 without a write-back
            const long long off = (long long)(pr * 128 + tid) * kD + h * kHD;
            l2_discard_line(dq + off);
            l2_discard_line(dk + off);
            l2_discard_line(dv + off);
        }
        // ---- MMA 1: S = Q K^T (K = 64 head dims: four 16-element steps of 32 bytes)
        if (tid == 0) {
            tc_fence_after();
            const uint32_t qa = smem_u32(sm + kSmQ), ka = smem_u32(sm + kSmK);
#pragma unroll
            for (int k = 0; k < 4; k++)
                tc_mma_bf16(tbase, sdesc_k128(qa + k * 32), sdesc_k128(ka + k * 32), kIdescS, k ? 1u : 0u);
            tc_commit(mma);
        }
        // the mma barrier completes twice per unit: parity 0 after MMA 1, parity 1 after MMA 2
        if (__syncthreads_or(!mbar_wait(mma, 0, abort_flag, err, DEVERR_TIMEOUT_MMA))) break;
        tc_fence_after();
        // ---- softmax of query row i over its own sequence's 64 keys
        float sv[64];
        {
            float a[32], b[32];
            tmem_ld32(trow + s * 64, a);
            tmem_ld32(trow + s * 64 + 32, b);
#pragma unroll
            for (int k = 0; k < 32; k++) { sv[k] = a[k]; sv[32 + k] = b[k]; }
        }
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < 64; k++) {
            const bool ok = ((k < 32 ? m0 >> k : m1 >> (k - 32)) & 1u) != 0;
            sv[k] = ok ? sv[k] * scale_log2 : -INFINITY;
            mx = fmaxf(mx, sv[k]);
        }
        const float mu = mx == -INFINITY ? 0.f : mx;
        float l = 0.f;
#pragma unroll
        for (int k = 0; k < 64; k++) { sv[k] = exp2f(sv[k] - mu); l += sv[k]; }
        // P row i over 128 keys, in the Q and K tiles (dead after MMA 1): key chunk c
        // (keys 64 c .. 64 c + 63) at kSmQ + c * 16 KB; this sequence's chunk s holds
        // the 64 probabilities, chunk 1 - s zeros
        {
            uint8_t *pc = sm + kSmQ + s * kTile, *pz = sm + kSmQ + (1 - s) * kTile;
#pragma unroll
            for (int uu = 0; uu < 8; uu++) {
                uint4 w;
                w.x = pack_bf16x2(sv[8 * uu + 0], sv[8 * uu + 1]);
                w.y = pack_bf16x2(sv[8 * uu + 2], sv[8 * uu + 3]);
                w.z = pack_bf16x2(sv[8 * uu + 4], sv[8 * uu + 5]);
                w.w = pack_bf16x2(sv[8 * uu + 6], sv[8 * uu + 7]);
                *reinterpret_cast<uint4 *>(pc + sw128(i, uu)) = w;
                *reinterpret_cast<uint4 *>(pz + sw128(i, uu)) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        // ---- MMA 2: O = P V over 128 keys (eight 16-key steps); O into TMEM columns 0..63
        if (tid == 0) {
            tc_fence_after();
            const uint32_t pa = smem_u32(sm + kSmQ), va = smem_u32(sm + kSmV);
#pragma unroll
            for (int k = 0; k < 8; k++) {
                // A = P, K-major: key chunk k / 4, 32 bytes per 16 keys; B = V as loaded
                // ([keys][dims], dims contiguous: MN-major), 16 keys = two 1024-byte row groups
                const uint32_t c = k >> 2, o = (k & 3) * 32;
                tc_mma_bf16(tbase, sdesc_k128(pa + c * kTile + o), sdesc_k128(va + k * 2048), kIdescO, k ? 1u : 0u);
            }
            tc_commit(mma);
        }
        if (__syncthreads_or(!mbar_wait(mma, 1, abort_flag, err, DEVERR_TIMEOUT_MMA))) break;
        tc_fence_after();
        // the tiles and P are free (MMA 2 is done): the next unit's tiles load during
        // this unit's output stores
        if (tid == 0 && u + (int)gridDim.x < units) { issue(u + gridDim.x); pending = true; }
        // ---- O / l -> bf16 (or e4m3 with the sequence's bound), row i of the head's 64 columns
        {
            float a[32], b[32];
            tmem_ld32(trow, a);
            tmem_ld32(trow + 32, b);
            const float inv = l > 0.f ? 1.0f / l : 0.f;
            const int r = 2 * pr + s;
            if (o8) {
                // |softmax . V| <= 1.02 max_j unorm_j max_d |Wv_d| over the sequence (AttnArgs)
                float m = 0.f;
                if (r < rows) {
                    const int lane = tid & 31;
                    m = fmaxf(__ldg(unorm + (long long)r * 64 + lane), __ldg(unorm + (long long)r * 64 + 32 + lane));
                }
                const float bnd = 1.02f * warp_max(m) * vbound;
                const float f = inv * (bnd > 0.f ? 448.0f / bnd : 0.f);
                if (r < rows) {
                    uint8_t *og = o8 + (long long)(pr * 128 + i) * ldo + h * kHD;
#pragma unroll
                    for (int uu = 0; uu < 2; uu++) {
                        uint4 w;
                        w.x = pack_e4m3x4(a[16 * uu + 0] * f, a[16 * uu + 1] * f, a[16 * uu + 2] * f, a[16 * uu + 3] * f);
                        w.y = pack_e4m3x4(a[16 * uu + 4] * f, a[16 * uu + 5] * f, a[16 * uu + 6] * f, a[16 * uu + 7] * f);
                        w.z = pack_e4m3x4(a[16 * uu + 8] * f, a[16 * uu + 9] * f, a[16 * uu + 10] * f, a[16 * uu + 11] * f);
                        w.w = pack_e4m3x4(a[16 * uu + 12] * f, a[16 * uu + 13] * f, a[16 * uu + 14] * f, a[16 * uu + 15] * f);
                        reinterpret_cast<uint4 *>(og)[uu] = w;
                        w.x = pack_e4m3x4(b[16 * uu + 0] * f, b[16 * uu + 1] * f, b[16 * uu + 2] * f, b[16 * uu + 3] * f);
                        w.y = pack_e4m3x4(b[16 * uu + 4] * f, b[16 * uu + 5] * f, b[16 * uu + 6] * f, b[16 * uu + 7] * f);
                        w.z = pack_e4m3x4(b[16 * uu + 8] * f, b[16 * uu + 9] * f, b[16 * uu + 10] * f, b[16 * uu + 11] * f);
                        w.w = pack_e4m3x4(b[16 * uu + 12] * f, b[16 * uu + 13] * f, b[16 * uu + 14] * f, b[16 * uu + 15] * f);
                        reinterpret_cast<uint4 *>(og)[2 + uu] = w;
                    }
                    if (h == 0) o_scale[(long long)r * 64 + qi] = bnd / 448.0f;
                }
            } else if (r < rows) {
                bf16 *og = out + (long long)(pr * 128 + i) * ldo + h * kHD;
#pragma unroll
                for (int uu = 0; uu < 4; uu++) {
                    uint4 w;
                    w.x = pack_bf16x2(a[8 * uu + 0] * inv, a[8 * uu + 1] * inv);
                    w.y = pack_bf16x2(a[8 * uu + 2] * inv, a[8 * uu + 3] * inv);
                    w.z = pack_bf16x2(a[8 * uu + 4] * inv, a[8 * uu + 5] * inv);
                    w.w = pack_bf16x2(a[8 * uu + 6] * inv, a[8 * uu + 7] * inv);
                    reinterpret_cast<uint4 *>(og)[uu] = w;
                    w.x = pack_bf16x2(b[8 * uu + 0] * inv, b[8 * uu + 1] * inv);
                    w.y = pack_bf16x2(b[8 * uu + 2] * inv, b[8 * uu + 3] * inv);
                    w.z = pack_bf16x2(b[8 * uu + 4] * inv, b[8 * uu + 5] * inv);
                    w.w = pack_bf16x2(b[8 * uu + 6] * inv, b[8 * uu + 7] * inv);
                    reinterpret_cast<uint4 *>(og)[4 + uu] = w;
                }
            }
        }
        tc_fence_before();
        __syncthreads();   // TMEM, P and the tiles are free for the next unit
    }
    // after an abort, wait (bounded) for a load still in flight so that no TMA write
    // lands in shared memory after the CTA has exited
    if (tid == 0 && pending) {
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(full, ph))
            if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tbase, 128);
    }
}

// Bidirectional (optionally masked) attention for 64 < L <= 256 on tcgen05: a
// unit is (sequence r, head h, 128-query tile qt), the whole key range in one
// tile of NK = 128 or 256 keys.  Per unit, one CTA of 8 warps:
//   TMA    Q (128 rows), K and V (NK rows from the sequence's first token;
//          rows past L belong to the next sequence or are the zero fill)
//   MMA 1  S = Q K^T into TMEM columns 0..NK-1
//   all    query row i is owned by two threads, warps w and w + 4 (the TMEM
//          lanes of a warp are fixed by w mod 4), each over half of the keys:
//          pass 1 reads its half of S from TMEM for the row maximum, the two
//          halves meet in shared memory, pass 2 reads S again for exp2 and
//          the sum and writes P (bf16) K-major over the Q and K tiles (dead
//          after MMA 1); keys past L and masked keys get P = 0, V rows past L
//          are zeroed
//   MMA 2  O = P V (K = NK keys, V read MN-major as loaded) into TMEM
//          columns 0..63 (S is dead by then)
//   all    each thread of a row stores 32 of its 64 output columns, O / l in
//          bf16 (or e4m3 with the sequence's bound), while the next unit's
//          tiles load
// No running rescale is needed: the whole row is in TMEM.  Numerics are those
// of the L = 64 kernel (fp32 scores and softmax, P rounded to bf16).
constexpr int kLongThreads = 256;

template <int NK>
struct LongCfg {
    static constexpr int kSQ = 0;
    static constexpr int kSK = kTile;                                         // NK rows of 128 bytes
    static constexpr int kPBytes = NK * 256;                                  // 128 rows x NK keys bf16
    static constexpr int kSV = (kTile + NK * 128 > kPBytes) ? kTile + NK * 128 : kPBytes;
    static constexpr int kSRed = kSV + NK * 128;                              // row max / sum halves, FP8 bound
    static constexpr int kSBar = kSRed + (2 * 128 + 2 * 128 + 8) * 4;
    static constexpr int kSmem = kSBar + 64 + 1024;
    static constexpr uint32_t kIdescS = idesc_bf16(128, NK);
    static constexpr int kHalfChunks = NK / 64;                               // 32-key chunks per thread
};

template <int NK>
__global__ void __launch_bounds__(kLongThreads, 2)
    attn_tc_long_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, bf16 *__restrict__ out, long long ldo, int rows, int L,
                        const uint32_t *__restrict__ mask_bits, float scale_log2, int *err, uint8_t *__restrict__ o8,
                        float *__restrict__ o_scale, const float *__restrict__ unorm, float vbound) {
    using Cfg = LongCfg<NK>;
    constexpr int HC = Cfg::kHalfChunks;
    pdl_wait();
    pdl_trigger();
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = sm + Cfg::kSQ, *sK = sm + Cfg::kSK, *sV = sm + Cfg::kSV, *sP = sm;
    float *red_mx = reinterpret_cast<float *>(sm + Cfg::kSRed);   // [2][128] partial row maxima
    float *red_l = red_mx + 256;                                  // [2][128] partial row sums
    float *red_b = red_l + 256;                                   // [8] per-warp maxima of the FP8 bound
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + Cfg::kSBar);
    uint64_t *mma = full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int sub = warp & 3, hf = warp >> 2;     // TMEM lane quarter, key half
    const int i = sub * 32 + lane;                // query row within the tile
    const int n_qt = (L + 127) / 128, units = rows * kH * n_qt;
    const int W = (L + 31) / 32;                  // mask words per query row

    if (tid == 0) {
        mbar_init(full, 1);
        mbar_init(mma, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tq); tma_prefetch_desc(&tk); tma_prefetch_desc(&tv);
    }
    if (warp == 0) { tmem_alloc(tmem_slot, NK); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;
    const uint32_t trow = tbase + (static_cast<uint32_t>(sub * 32) << 16);   // this warp's TMEM lanes

    auto issue = [&](int v) {
        const int qv = v % n_qt, hv = (v / n_qt) % kH, rv = v / (n_qt * kH);
        mbar_arrive_expect_tx(full, kTile + 2 * NK * 128);
        tma_load_2d(sQ, &tq, full, hv * kHD, rv * L + qv * 128);
        tma_load_2d(sK, &tk, full, hv * kHD, rv * L);
        tma_load_2d(sV, &tv, full, hv * kHD, rv * L);
    };
    bool pending = false;
    if (tid == 0 && (int)blockIdx.x < units) { issue(blockIdx.x); pending = true; }
    uint32_t ph = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ph ^= 1u) {
        const int qt = u % n_qt, h = (u / n_qt) % kH, r = u / (n_qt * kH);
        const int q = qt * 128 + i;   // this thread's query within the sequence
        // validity words of this thread's 32-key chunks: mask bits and keys < L
        uint32_t vw[HC];
#pragma unroll
        for (int c = 0; c < HC; c++) {
            const int cc = hf * HC + c, left = L - 32 * cc;
            uint32_t w = left <= 0 ? 0u : (left >= 32 ? ~0u : ((1u << left) - 1u));
            if (mask_bits && q < L && left > 0) w &= __ldg(mask_bits + (long long)q * W + cc);
            vw[c] = w;
        }
        float bmax = 0.f;
        if (o8) {
            if (tid < L) bmax = __ldg(unorm + (long long)r * L + tid);
            bmax = warp_max(bmax);
        }
        if (__syncthreads_or(!mbar_wait(full, ph, abort_flag, err, DEVERR_TIMEOUT_PRODUCER))) break;
        pending = false;
        // ---- MMA 1: S = Q K^T (K = 64 head dims: four 16-element steps of 32 bytes)
        if (tid == 0) {
            tc_fence_after();
            const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK);
#pragma unroll
            for (int k = 0; k < 4; k++)
                tc_mma_bf16(tbase, sdesc_k128(qa + k * 32), sdesc_k128(ka + k * 32), Cfg::kIdescS, k ? 1u : 0u);
            tc_commit(mma);
        }
        // V rows past the sequence: zeroed (their P is 0, and 0 x NaN would not be)
        if (tid >= L && tid < NK) {
#pragma unroll
            for (int uu = 0; uu < 8; uu++) *reinterpret_cast<uint4 *>(sV + tid * 128 + uu * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        if (o8 && lane == 0) red_b[warp] = bmax;
        if (__syncthreads_or(!mbar_wait(mma, 0, abort_flag, err, DEVERR_TIMEOUT_MMA))) break;
        tc_fence_after();
        // ---- pass 1: maximum of this thread's half of the row (four independent chains).
        // A chunk pair no row of the warp may see is not read at all (the TMEM load is
        // warp-collective); fully visible chunks skip the per-key tests.
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
        for (int c = 0; c < HC; c += 2) {
            const uint32_t wa = c == 0 ? vw[0] : vw[HC - 2], wb = c == 0 ? vw[1] : vw[HC - 1];
            if (!__any_sync(0xffffffffu, (wa | wb) != 0u)) continue;
            float a[32], b[32];
            const uint32_t col = (uint32_t)(hf * HC + c) * 32;
            tmem_ld32x2(trow + col, trow + col + 32, a, b);
            if ((wa & wb) == 0xffffffffu) {
#pragma unroll
                for (int k = 0; k < 32; k++) {
                    m4[k & 3] = fmaxf(m4[k & 3], a[k]);
                    m4[k & 3] = fmaxf(m4[k & 3], b[k]);
                }
            } else {
#pragma unroll
                for (int k = 0; k < 32; k++) {
                    m4[k & 3] = fmaxf(m4[k & 3], ((wa >> k) & 1u) ? a[k] : -INFINITY);
                    m4[k & 3] = fmaxf(m4[k & 3], ((wb >> k) & 1u) ? b[k] : -INFINITY);
                }
            }
        }
        red_mx[hf * 128 + i] = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        __syncthreads();   // both halves of every row
        const float mx = fmaxf(red_mx[i], red_mx[128 + i]);
        // scores are scaled after the maximum: max(s) * c = max(s * c) for c > 0
        const float mu = mx == -INFINITY ? 0.f : mx * scale_log2;
        // ---- pass 2: P = exp2(s c - max) (bf16, K-major over the dead Q | K tiles), row sum
        float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
        for (int c = 0; c < HC; c += 2) {
            const int cc = hf * HC + c;
            const uint32_t wa = c == 0 ? vw[0] : vw[HC - 2], wb = c == 0 ? vw[1] : vw[HC - 1];
            float a[32], b[32];
            if (__any_sync(0xffffffffu, (wa | wb) != 0u)) {
                tmem_ld32x2(trow + (uint32_t)cc * 32, trow + (uint32_t)cc * 32 + 32, a, b);
                if ((wa & wb) == 0xffffffffu) {
#pragma unroll
                    for (int k = 0; k < 32; k++) {
                        a[k] = ex2_hw(fmaf(a[k], scale_log2, -mu));
                        b[k] = ex2_hw(fmaf(b[k], scale_log2, -mu));
                        l4[k & 3] += a[k] + b[k];
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < 32; k++) {
                        a[k] = ((wa >> k) & 1u) ? ex2_hw(fmaf(a[k], scale_log2, -mu)) : 0.f;
                        b[k] = ((wb >> k) & 1u) ? ex2_hw(fmaf(b[k], scale_log2, -mu)) : 0.f;
                        l4[k & 3] += a[k] + b[k];
                    }
                }
            } else {
#pragma unroll
                for (int k = 0; k < 32; k++) a[k] = b[k] = 0.f;
            }
            // keys 32 cc .. 32 cc + 63 are 16-byte units 0..7 of row i in 64-key chunk cc / 2
            uint8_t *pc = sP + (cc >> 1) * kTile;
#pragma unroll
            for (int uu = 0; uu < 4; uu++) {
                *reinterpret_cast<uint4 *>(pc + sw128(i, uu)) =
                    make_uint4(pack_bf16x2(a[8 * uu], a[8 * uu + 1]), pack_bf16x2(a[8 * uu + 2], a[8 * uu + 3]),
                               pack_bf16x2(a[8 * uu + 4], a[8 * uu + 5]), pack_bf16x2(a[8 * uu + 6], a[8 * uu + 7]));
                *reinterpret_cast<uint4 *>(pc + sw128(i, 4 + uu)) =
                    make_uint4(pack_bf16x2(b[8 * uu], b[8 * uu + 1]), pack_bf16x2(b[8 * uu + 2], b[8 * uu + 3]),
                               pack_bf16x2(b[8 * uu + 4], b[8 * uu + 5]), pack_bf16x2(b[8 * uu + 6], b[8 * uu + 7]));
            }
        }
        red_l[hf * 128 + i] = (l4[0] + l4[1]) + (l4[2] + l4[3]);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        // ---- MMA 2: O = P V over NK keys (NK / 16 steps); O into TMEM columns 0..63
        if (tid == 0) {
            tc_fence_after();
            const uint32_t pa = smem_u32(sP), va = smem_u32(sV);
#pragma unroll
            for (int k = 0; k < NK / 16; k++) {
                const uint32_t c = k >> 2, o = (k & 3) * 32;
                tc_mma_bf16(tbase, sdesc_k128(pa + c * kTile + o), sdesc_k128(va + k * 2048), kIdescO, k ? 1u : 0u);
            }
            tc_commit(mma);
        }
        if (__syncthreads_or(!mbar_wait(mma, 1, abort_flag, err, DEVERR_TIMEOUT_MMA))) break;
        tc_fence_after();
        // P and the tiles are free: the next unit's tiles load during this unit's stores
        if (tid == 0 && u + (int)gridDim.x < units) { issue(u + gridDim.x); pending = true; }
        {
            float a[32];
            tmem_ld32(trow + hf * 32, a);   // output columns 32 hf .. 32 hf + 31
            const float l = red_l[i] + red_l[128 + i];
            const float inv = l > 0.f ? 1.0f / l : 0.f;
            const long long row = (long long)r * L + q;
            if (o8) {
                // |softmax . V| <= 1.02 max_j unorm_j max_d |Wv_d| over the sequence (AttnArgs)
                float bm = red_b[0];
#pragma unroll
                for (int w2 = 1; w2 < 8; w2++) bm = fmaxf(bm, red_b[w2]);
                const float bnd = 1.02f * bm * vbound;
                const float f = inv * (bnd > 0.f ? 448.0f / bnd : 0.f);
                if (q < L) {
                    uint4 *og = reinterpret_cast<uint4 *>(o8 + row * ldo + h * kHD + hf * 32);
#pragma unroll
                    for (int uu = 0; uu < 2; uu++)
                        og[uu] = make_uint4(
                            pack_e4m3x4(a[16 * uu + 0] * f, a[16 * uu + 1] * f, a[16 * uu + 2] * f, a[16 * uu + 3] * f),
                            pack_e4m3x4(a[16 * uu + 4] * f, a[16 * uu + 5] * f, a[16 * uu + 6] * f, a[16 * uu + 7] * f),
                            pack_e4m3x4(a[16 * uu + 8] * f, a[16 * uu + 9] * f, a[16 * uu + 10] * f, a[16 * uu + 11] * f),
                            pack_e4m3x4(a[16 * uu + 12] * f, a[16 * uu + 13] * f, a[16 * uu + 14] * f, a[16 * uu + 15] * f));
                    if (h == 0 && hf == 0) o_scale[row] = bnd / 448.0f;
                }
            } else if (q < L) {
                uint4 *og = reinterpret_cast<uint4 *>(out + row * ldo + h * kHD + hf * 32);
#pragma unroll
                for (int uu = 0; uu < 4; uu++)
                    og[uu] = make_uint4(pack_bf16x2(a[8 * uu] * inv, a[8 * uu + 1] * inv),
                                        pack_bf16x2(a[8 * uu + 2] * inv, a[8 * uu + 3] * inv),
                                        pack_bf16x2(a[8 * uu + 4] * inv, a[8 * uu + 5] * inv),
                                        pack_bf16x2(a[8 * uu + 6] * inv, a[8 * uu + 7] * inv));
            }
        }
        tc_fence_before();
        __syncthreads();   // TMEM, P, the tiles and the row halves are free for the next unit
    }
    if (tid == 0 && pending) {
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(full, ph))
            if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tbase, NK);
    }
}

// Causal attention over a KV cache on tcgen05 (the PatchEncoder prefill, Tq >
// 64 tokens per sequence): a unit is (sequence r, head h, 128-query tile qt).
// Q rows r Tq + 128 qt .. (rows past the sequence belong to the next one and
// are never stored); keys come from the cache rows r cap + 128 kb .. in blocks
// of 128, as many as the tile's last query can see.  Per key block: S = Q K^T
// (TMEM columns 0..127), online softmax in fp32 by the thread that owns the
// query row (running max m, sum l, output O in registers rescaled by
// exp2(m_old - m_new)), P (bf16) K-major in shared memory, cache rows past the
// valid keys zeroed in V (they may hold anything), PV = P V (TMEM columns
// 128..191, V read MN-major) added into O.  O / l to bf16 at the end.
constexpr int kCaSmem = 5 * kTile + 64 + 1024;   // Q | K | V | P (two 64-key chunks) | barriers
constexpr uint32_t kIdescPV = idesc_bf16(128, 64) | (1u << 16);

__global__ void __launch_bounds__(kTcThreads, 2)
    attn_tc_causal_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv, bf16 *__restrict__ out, long long ldo, int B,
                          int Tq, int cap, int q_pos0, int kv_len, float scale_log2, int *err) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = sm, *sK = sm + kTile, *sV = sm + 2 * kTile, *sP = sm + 3 * kTile;
    uint64_t *qbar = reinterpret_cast<uint64_t *>(sm + 5 * kTile);
    uint64_t *kvbar = qbar + 1;
    uint64_t *mma = qbar + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(qbar + 3);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int n_qt = (Tq + 127) / 128, units = B * kH * n_qt;
    if (tid == 0) {
        mbar_init(qbar, 1);
        mbar_init(kvbar, 1);
        mbar_init(mma, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tq); tma_prefetch_desc(&tk); tma_prefetch_desc(&tv);
    }
    if (warp == 0) { tmem_alloc(tmem_slot, 256); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;
    const uint32_t trow = tbase + (static_cast<uint32_t>(warp * 32) << 16);
    const int i = tid;
    uint32_t qph = 0, kvph = 0;
    int q_out = -1, kv_out = -1;   // parity of a load issued and not yet seen complete, or -1
    bool failed = false;
    for (int u = blockIdx.x; u < units && !failed; u += gridDim.x) {
        const int qt = u % n_qt, h = (u / n_qt) % kH, r = u / (n_qt * kH);
        const int q_row0 = qt * 128;                        // first query of the tile (within the sequence)
        const int q_abs = q_pos0 + q_row0 + i;               // this thread's query position
        const int last_q = min(Tq - 1, q_row0 + 127);
        const int n_keys = min(kv_len, q_pos0 + last_q + 1);
        const int n_kb = (n_keys + 127) / 128;
        if (tid == 0) {
            mbar_arrive_expect_tx(qbar, kTile);
            tma_load_2d(sQ, &tq, qbar, h * kHD, r * Tq + q_row0);
        }
        q_out = (int)qph;
        float o[64];
#pragma unroll
        for (int d = 0; d < 64; d++) o[d] = 0.f;
        float m = -INFINITY, l = 0.f;
        for (int kb = 0; kb < n_kb; kb++) {
            if (tid == 0) {
                mbar_arrive_expect_tx(kvbar, 2 * kTile);
                tma_load_2d(sK, &tk, kvbar, h * kHD, r * cap + kb * 128);
                tma_load_2d(sV, &tv, kvbar, h * kHD, r * cap + kb * 128);
            }
            kv_out = (int)kvph;
            bool ok = true;
            if (kb == 0) {
                ok = mbar_wait(qbar, qph, abort_flag, err, DEVERR_TIMEOUT_PRODUCER);
                if (ok) { q_out = -1; qph ^= 1u; }
            }
            if (ok) {
                ok = mbar_wait(kvbar, kvph, abort_flag, err, DEVERR_TIMEOUT_PRODUCER);
                if (ok) { kv_out = -1; kvph ^= 1u; }
            }
            if (__syncthreads_or(!ok)) { failed = true; break; }
            if (tid == 0) {
                tc_fence_after();
                const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK);
#pragma unroll
                for (int k = 0; k < 4; k++)
                    tc_mma_bf16(tbase, sdesc_k128(qa + k * 32), sdesc_k128(ka + k * 32), kIdescS, k ? 1u : 0u);
                tc_commit(mma);
            }
            // cache rows past the valid keys may hold anything: zero them in V
            // (their P is 0, and 0 x NaN would not be)
            const int valid = n_keys - kb * 128;
            if (i >= valid) {
#pragma unroll
                for (int uu = 0; uu < 8; uu++) *reinterpret_cast<uint4 *>(sV + i * 128 + uu * 16) = make_uint4(0u, 0u, 0u, 0u);
            }
            if (__syncthreads_or(!mbar_wait(mma, 0, abort_flag, err, DEVERR_TIMEOUT_MMA))) { failed = true; break; }
            tc_fence_after();
            float sv[128];
#pragma unroll
            for (int c = 0; c < 4; c++) {
                float t32[32];
                tmem_ld32(trow + c * 32, t32);
#pragma unroll
                for (int k = 0; k < 32; k++) sv[32 * c + k] = t32[k];
            }
            float mx = m;
#pragma unroll
            for (int k = 0; k < 128; k++) {
                const int j = kb * 128 + k;
                sv[k] = (j < n_keys && j <= q_abs) ? sv[k] * scale_log2 : -INFINITY;
                mx = fmaxf(mx, sv[k]);
            }
            const float mu = mx == -INFINITY ? 0.f : mx;
            const float corr = exp2f(m - mu);   // m = -inf on the first block: 0
            l *= corr;
#pragma unroll
            for (int k = 0; k < 128; k++) { sv[k] = exp2f(sv[k] - mu); l += sv[k]; }
            m = mx;
#pragma unroll
            for (int c = 0; c < 2; c++)
#pragma unroll
                for (int uu = 0; uu < 8; uu++) {
                    const float *pv = sv + 64 * c + 8 * uu;
                    *reinterpret_cast<uint4 *>(sP + c * kTile + sw128(i, uu)) =
                        make_uint4(pack_bf16x2(pv[0], pv[1]), pack_bf16x2(pv[2], pv[3]), pack_bf16x2(pv[4], pv[5]),
                                   pack_bf16x2(pv[6], pv[7]));
                }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                const uint32_t pa = smem_u32(sP), va = smem_u32(sV);
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const uint32_t c = k >> 2, off = (k & 3) * 32;
                    tc_mma_bf16(tbase + 128, sdesc_k128(pa + c * kTile + off), sdesc_k128(va + k * 2048), kIdescPV,
                                k ? 1u : 0u);
                }
                tc_commit(mma);
            }
            if (__syncthreads_or(!mbar_wait(mma, 1, abort_flag, err, DEVERR_TIMEOUT_MMA))) { failed = true; break; }
            tc_fence_after();
            {
                float a[32], b2[32];
                tmem_ld32(trow + 128, a);
                tmem_ld32(trow + 160, b2);
#pragma unroll
                for (int d = 0; d < 32; d++) { o[d] = o[d] * corr + a[d]; o[32 + d] = o[32 + d] * corr + b2[d]; }
            }
            tc_fence_before();
            __syncthreads();   // K, V, P and TMEM are free for the next key block
        }
        if (failed) break;
        if (q_row0 + i < Tq) {
            const float inv = l > 0.f ? 1.0f / l : 0.f;
            uint4 *og = reinterpret_cast<uint4 *>(out + (long long)(r * Tq + q_row0 + i) * ldo + h * kHD);
#pragma unroll
            for (int uu = 0; uu < 8; uu++)
                og[uu] = make_uint4(pack_bf16x2(o[8 * uu] * inv, o[8 * uu + 1] * inv),
                                    pack_bf16x2(o[8 * uu + 2] * inv, o[8 * uu + 3] * inv),
                                    pack_bf16x2(o[8 * uu + 4] * inv, o[8 * uu + 5] * inv),
                                    pack_bf16x2(o[8 * uu + 6] * inv, o[8 * uu + 7] * inv));
        }
    }
    // after an abort, wait (bounded) for loads still in flight so that no TMA write
    // lands in shared memory after the CTA has exited
    if (tid == 0) {
        const unsigned long long t0 = globaltimer_ns();
        if (q_out >= 0)
            while (!mbar_try_wait(qbar, (uint32_t)q_out) && globaltimer_ns() - t0 < kWaitLimitNs) {}
        if (kv_out >= 0)
            while (!mbar_try_wait(kvbar, (uint32_t)kv_out) && globaltimer_ns() - t0 < kWaitLimitNs) {}
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tbase, 256);
    }
}
}  // namespace

cudaError_t attention_tc_prepare() {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(attn_tc_long_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             LongCfg<128>::kSmem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(attn_tc_long_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             LongCfg<256>::kSmem);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(attn_tc_causal_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kCaSmem);
}

bool attention_tc_eligible(const AttnArgs &a) {
    static const bool on = [] {
        const char *e = std::getenv("DTTS_ATTN_TC");
        return !(e && e[0] == '0');
    }();
    return on && a.Tq == 64 && a.kv_len == 64 && a.kv_cap == 64 && !a.causal && !a.kv_base_dev &&
           (!a.mask || a.mask_bits) && (!a.o8 || (a.o_scale && a.unorm)) && a.ldq == kD && a.ldkv == kD &&
           a.rows >= 1;
}

cudaError_t launch_attention_tc(const AttnArgs &a, int *err, cudaStream_t s, bool pdl) {
    if (!attention_tc_eligible(a)) return cudaErrorNotSupported;
    const unsigned long long R = (unsigned long long)a.rows * 64;
    CUtensorMap tq, tk, tv;
    if (!make_tmap_bf16(&tq, a.q, R, kD, 128) || !make_tmap_bf16(&tk, a.k, R, kD, 128) ||
        !make_tmap_bf16(&tv, a.v, R, kD, 128))
        return cudaErrorInvalidValue;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const int units = (a.rows + 1) / 2 * kH;
    const int grid = units < 4 * nsm ? units : 4 * nsm;   // 4 resident CTAs per SM (49 KB, 128 TMEM columns)
    const float sl = a.scale * 1.4426950408889634f;
    const bf16 *dq = a.discard_qkv ? reinterpret_cast<const bf16 *>(a.q) : nullptr;
    const bf16 *dk = a.discard_qkv ? reinterpret_cast<const bf16 *>(a.k) : nullptr;
    const bf16 *dv = a.discard_qkv ? reinterpret_cast<const bf16 *>(a.v) : nullptr;
    return launch_k(pdl && pdl_enabled(), attn_tc_kernel, dim3(grid), dim3(kTcThreads), (size_t)kTcSmem, s, tq, tk,
                    tv, reinterpret_cast<bf16 *>(a.o), (long long)a.ldo, a.rows, a.mask_bits, sl, err, a.o8, a.o_scale,
                    a.unorm, a.vbound, dq, dk, dv);
}

bool attention_tc_long_eligible(const AttnArgs &a) {
    static const bool on = [] {
        const char *e = std::getenv("DTTS_ATTN_TC");
        return !(e && e[0] == '0');
    }();
    return on && !a.causal && a.Tq > 64 && a.Tq <= 256 && a.kv_len == a.Tq && a.kv_cap == a.Tq && !a.kv_base_dev &&
           (!a.mask || a.mask_bits) && (!a.o8 || (a.o_scale && a.unorm)) && a.ldq == kD && a.ldkv == kD &&
           a.rows >= 1;
}

cudaError_t launch_attention_tc_long(const AttnArgs &a, int *err, cudaStream_t s, bool pdl) {
    if (!attention_tc_long_eligible(a)) return cudaErrorNotSupported;
    const int L = a.Tq, nk = L <= 128 ? 128 : 256;
    const unsigned long long R = (unsigned long long)a.rows * L;
    CUtensorMap tq, tk, tv;
    if (!make_tmap_bf16(&tq, a.q, R, kD, 128) || !make_tmap_bf16(&tk, a.k, R, kD, nk) ||
        !make_tmap_bf16(&tv, a.v, R, kD, nk))
        return cudaErrorInvalidValue;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const int units = a.rows * kH * ((L + 127) / 128);
    const float sl = a.scale * 1.4426950408889634f;
    if (nk == 128) {
        const int grid = units < 2 * nsm ? units : 2 * nsm;   // 2 resident CTAs per SM
        return launch_k(pdl && pdl_enabled(), attn_tc_long_kernel<128>, dim3(grid), dim3(kLongThreads),
                        (size_t)LongCfg<128>::kSmem, s, tq, tk, tv, reinterpret_cast<bf16 *>(a.o), (long long)a.ldo,
                        a.rows, L, a.mask_bits, sl, err, a.o8, a.o_scale, a.unorm, a.vbound);
    }
    const int grid = units < 2 * nsm ? units : 2 * nsm;   // 2 resident CTAs per SM (97 KB, 256 TMEM columns)
    return launch_k(pdl && pdl_enabled(), attn_tc_long_kernel<256>, dim3(grid), dim3(kLongThreads),
                    (size_t)LongCfg<256>::kSmem, s, tq, tk, tv, reinterpret_cast<bf16 *>(a.o), (long long)a.ldo,
                    a.rows, L, a.mask_bits, sl, err, a.o8, a.o_scale, a.unorm, a.vbound);
}

bool attention_tc_causal_eligible(const AttnArgs &a) {
    static const bool on = [] {
        const char *e = std::getenv("DTTS_ATTN_TC");
        return !(e && e[0] == '0');
    }();
    return on && a.causal && a.Tq > 64 && !a.kv_base_dev && !a.mask && !a.mask_bits && !a.o8 && a.ldq == kD &&
           a.ldkv == kD && a.rows >= 1 && a.q_pos0 >= 0 && a.kv_len >= a.q_pos0 + a.Tq && a.kv_len <= a.kv_cap;
}

cudaError_t launch_attention_tc_causal(const AttnArgs &a, int *err, cudaStream_t s, bool pdl) {
    if (!attention_tc_causal_eligible(a)) return cudaErrorNotSupported;
    CUtensorMap tq, tk, tv;
    const unsigned long long RQ = (unsigned long long)a.rows * a.Tq, RK = (unsigned long long)a.rows * a.kv_cap;
    if (!make_tmap_bf16(&tq, a.q, RQ, kD, 128) || !make_tmap_bf16(&tk, a.k, RK, kD, 128) ||
        !make_tmap_bf16(&tv, a.v, RK, kD, 128))
        return cudaErrorInvalidValue;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const int units = a.rows * kH * ((a.Tq + 127) / 128);
    const int grid = units < 2 * nsm ? units : 2 * nsm;   // 2 resident CTAs per SM (81 KB, 256 TMEM columns)
    return launch_k(pdl && pdl_enabled(), attn_tc_causal_kernel, dim3(grid), dim3(kTcThreads), (size_t)kCaSmem, s, tq,
                    tk, tv, reinterpret_cast<bf16 *>(a.o), (long long)a.ldo, a.rows, a.Tq, a.kv_cap, a.q_pos0, a.kv_len,
                    a.scale * 1.4426950408889634f, err);
}

}  // namespace dtts
