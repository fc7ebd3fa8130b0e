// Non-GEMM kernels: norms, attention (bf16 mma.sync and fp32), fp32 SIMT
// projections, conditioning, DiT output head, PatchEncoder conv/pairing.
#include "kernels.cuh"
#include <math.h>
#include <algorithm>

namespace dtts {

// =========================================================================
// norms: one warp per token row of 1024 fp32 values (8 x float4 per lane);
// the row arithmetic is ln_rows.cuh's, shared with the fused GEMM epilogue
// =========================================================================
__global__ void __launch_bounds__(256, 3) ln_modulate_kernel(const float *__restrict__ x, int M, LnParams p) {
    pdl_wait();
    pdl_trigger();
    const int row[1] = {static_cast<int>(blockIdx.x * 8 + (threadIdx.x >> 5))};
    if (row[0] >= M) return;
    const bool live[1] = {true};
    ln_rows_bf16<1>(x, p, row, live, threadIdx.x & 31);
}

LnParams ln_params(const float *shift, const float *scale, long long ada_ld, int tok_per_row, void *out) {
    LnParams p{};
    p.shift = shift; p.scale = scale; p.ada_ld = ada_ld; p.tok_per_row = tok_per_row; p.out = out;
    return p;
}

void launch_ln_modulate(const float *x, bf16 *y, int M, const float *shift, const float *scale, long long ada_ld,
                        int tok_per_row, cudaStream_t s, bool pdl) {
    launch_k(pdl && pdl_enabled(), ln_modulate_kernel, dim3((M + 7) / 8), dim3(256), 0, s, x, M,
             ln_params(shift, scale, ada_ld, tok_per_row, y));
}

// The same LayerNorm + modulation with an e4m3 output row (ln_rows_f8).
__global__ void __launch_bounds__(256, 3) ln_modulate_f8_kernel(const float *__restrict__ x, int M, LnParams p) {
    pdl_wait();
    pdl_trigger();
    const int row[1] = {static_cast<int>(blockIdx.x * 8 + (threadIdx.x >> 5))};
    if (row[0] >= M) return;
    const bool live[1] = {true};
    ln_rows_f8<1>(x, p, row, live, threadIdx.x & 31);
}

void launch_ln_modulate_f8(const float *x, uint8_t *y, int M, const float *shift, const float *scale,
                           long long ada_ld, int tok_per_row, float *row_scale, float *unorm, float *g_scale,
                           float *g_inv, float w1n, float b1max, cudaStream_t s, bool pdl) {
    LnParams p = ln_params(shift, scale, ada_ld, tok_per_row, y);
    p.row_scale = row_scale; p.unorm = unorm; p.g_scale = g_scale; p.g_inv = g_inv; p.w1n = w1n; p.b1max = b1max;
    launch_k(pdl && pdl_enabled(), ln_modulate_f8_kernel, dim3((M + 7) / 8), dim3(256), 0, s, x, M, p);
}

// e4m3 conversion of n values (device self-test of the rounding).
__global__ void e4m3_selftest_kernel(const float *__restrict__ x, uint8_t *__restrict__ y, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (4 * i + 3 < n) {
        const uint32_t p = pack_e4m3x4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
        y[4 * i] = p & 0xff; y[4 * i + 1] = (p >> 8) & 0xff; y[4 * i + 2] = (p >> 16) & 0xff; y[4 * i + 3] = p >> 24;
    } else {
        for (int k = 4 * i; k < n; k++) y[k] = pack_e4m3x4(x[k], 0.f, 0.f, 0.f) & 0xff;
    }
}

void launch_e4m3_selftest(const float *x, uint8_t *y, int n, cudaStream_t s) {
    const int quads = (n + 3) / 4;
    e4m3_selftest_kernel<<<(quads + 127) / 128, 128, 0, s>>>(x, y, n);
}

__global__ void __launch_bounds__(256) rms_norm_kernel(const float *__restrict__ x, bf16 *__restrict__ y, int M,
                                                       const float *__restrict__ w) {
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const float4 *xr = reinterpret_cast<const float4 *>(x + (long long)row * kD);
    float4 v[8];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        v[j] = xr[lane + 32 * j];
        s += (v[j].x * v[j].x + v[j].y * v[j].y) + (v[j].z * v[j].z + v[j].w * v[j].w);
    }
    const float inv = 1.0f / sqrtf(warp_sum(s) * (1.0f / kD) + 1e-6f);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    uint2 *yr = reinterpret_cast<uint2 *>(y + (long long)row * kD);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int c4 = lane + 32 * j;
        float4 g = w ? __ldg(w4 + c4) : make_float4(1.f, 1.f, 1.f, 1.f);
        yr[c4] = make_uint2(pack_bf16x2(v[j].x * inv * g.x, v[j].y * inv * g.y),
                            pack_bf16x2(v[j].z * inv * g.z, v[j].w * inv * g.w));
    }
}

void launch_rms_norm(const float *x, bf16 *y, int M, const float *w, cudaStream_t s, bool pdl) {
    launch_k(pdl && pdl_enabled(), rms_norm_kernel, dim3((M + 7) / 8), dim3(256), 0, s, x, y, M, w);
}

// =========================================================================
// bf16 attention, mma.sync m16n8k16, one CTA per (64-query tile, head, row).
// Q/K/V tiles of 64 x 64 bf16 staged in shared memory with a 16-byte-chunk XOR
// swizzle; scores and the online softmax in fp32; P rounded to bf16 for P.V.
// =========================================================================
DTTS_DEV uint32_t swz(int row, int chunk) { return row * 64 + ((chunk ^ (row & 7)) << 3); }

DTTS_DEV void cp_async16(void *smem, const void *gmem, bool valid) {
    const uint32_t sz = valid ? 16u : 0u;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(sz)
                 : "memory");
}
DTTS_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

DTTS_DEV void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
DTTS_DEV void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
DTTS_DEV void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Loads a 64 x 64 bf16 tile (rows >= valid_rows are zero-filled).
DTTS_DEV void load_tile64(bf16 *sm, const bf16 *g, long long ld, int valid_rows) {
    for (int idx = threadIdx.x; idx < 64 * 8; idx += 128) {
        const int row = idx >> 3, ch = idx & 7;
        const bool ok = row < valid_rows;
        const bf16 *src = ok ? g + (long long)row * ld + ch * 8 : g;
        cp_async16(sm + swz(row, ch), src, ok);
    }
}

// Bound on |softmax . V| of sequence r for the e4m3 output (see AttnArgs).
DTTS_DEV float attn_seq_bound(const AttnArgs &a, int r) {
    float m = 0.f;
    for (int j = threadIdx.x & 31; j < a.kv_len; j += 32) m = fmaxf(m, __ldg(a.unorm + (long long)r * a.kv_cap + j));
    return 1.02f * warp_max(m) * a.vbound;
}

// Stores this thread's part of a 64-column head output (query rows qi0, qi1;
// columns nt*8 + 2t, +1): bf16 into a.o, or e4m3 into a.o8 when it is set.
DTTS_DEV void attn_store(const AttnArgs &a, int r, int h, int qi0, int qi1, int t, const float (&o)[8][4],
                         float inv0, float inv1) {
    if (a.o8) {
        const float bnd = attn_seq_bound(a, r);
        const float qs = bnd > 0.f ? 448.0f / bnd : 0.f;
        const float f0 = inv0 * qs, f1 = inv1 * qs;
        uint8_t *og = a.o8 + (long long)r * a.Tq * a.ldo + h * kHD;
        // lanes t and t^1 swap halves so that each writes 4 consecutive bytes:
        // even t row qi0, columns 2t..2t+3; odd t row qi1, columns 2t-2..2t+1
        const bool even = (t & 1) == 0;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            const uint32_t p0 = __nv_cvt_float2_to_fp8x2(make_float2(o[nt][0] * f0, o[nt][1] * f0), __NV_SATFINITE, __NV_E4M3);
            const uint32_t p1 = __nv_cvt_float2_to_fp8x2(make_float2(o[nt][2] * f1, o[nt][3] * f1), __NV_SATFINITE, __NV_E4M3);
            const uint32_t other = __shfl_xor_sync(0xffffffffu, even ? p1 : p0, 1);
            const int qi = even ? qi0 : qi1;
            const int d = nt * 8 + 2 * (t & ~1);
            const uint32_t word = even ? (p0 | (other << 16)) : (other | (p1 << 16));
            if (qi < a.Tq) *reinterpret_cast<uint32_t *>(og + (long long)qi * a.ldo + d) = word;
        }
        if (h == 0 && t == 0) {
            if (qi0 < a.Tq) a.o_scale[(long long)r * a.Tq + qi0] = bnd / 448.0f;
            if (qi1 < a.Tq) a.o_scale[(long long)r * a.Tq + qi1] = bnd / 448.0f;
        }
        return;
    }
    bf16 *og = reinterpret_cast<bf16 *>(a.o) + (long long)r * a.Tq * a.ldo + h * kHD;
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
        const int d = nt * 8 + 2 * t;
        if (qi0 < a.Tq)
            *reinterpret_cast<uint32_t *>(og + (long long)qi0 * a.ldo + d) = pack_bf16x2(o[nt][0] * inv0, o[nt][1] * inv0);
        if (qi1 < a.Tq)
            *reinterpret_cast<uint32_t *>(og + (long long)qi1 * a.ldo + d) = pack_bf16x2(o[nt][2] * inv1, o[nt][3] * inv1);
    }
}

__global__ void advance_len_kernel(int *len, int add) {
    pdl_wait();
    pdl_trigger();
    *len += add;
}

void launch_advance_len(int *len, int add, cudaStream_t s, bool pdl) {
    launch_k(pdl && pdl_enabled(), advance_len_kernel, dim3(1), dim3(1), 0, s, len, add);
}

__global__ void __launch_bounds__(128) attn_bf16_kernel(AttnArgs a) {
    pdl_wait();
    pdl_trigger();
    if (a.kv_base_dev) {   // graph-captured decode: positions from device memory
        a.q_pos0 = *a.kv_base_dev;
        a.kv_len = a.q_pos0 + a.Tq;
    }
    __shared__ __align__(128) bf16 Qs[64 * 64];
    __shared__ __align__(128) bf16 Ks[64 * 64];
    __shared__ __align__(128) bf16 Vs[64 * 64];
    const int qt = blockIdx.x, h = blockIdx.y, r = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int q0 = qt * 64;
    const bf16 *qg = reinterpret_cast<const bf16 *>(a.q) + ((long long)r * a.Tq + q0) * a.ldq + h * kHD;
    const bf16 *kg = reinterpret_cast<const bf16 *>(a.k) + (long long)r * a.kv_cap * a.ldkv + h * kHD;
    const bf16 *vg = reinterpret_cast<const bf16 *>(a.v) + (long long)r * a.kv_cap * a.ldkv + h * kHD;

    load_tile64(Qs, qg, a.ldq, a.Tq - q0);
    asm volatile("cp.async.commit_group;\n" ::: "memory");

    // row indices of this thread's two query rows (within the tile)
    const int wr0 = warp * 16 + g, wr1 = wr0 + 8;
    const int qi0 = q0 + wr0, qi1 = q0 + wr1;

    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    uint32_t qf[4][4];

    // keys beyond the causal limit of the last query of this tile are never needed
    int kv_end = a.kv_len;
    if (a.causal) kv_end = min(kv_end, a.q_pos0 + min(q0 + 64, a.Tq));
    const int nkb = (kv_end + 63) / 64;

    for (int kb = 0; kb < nkb; kb++) {
        const int k0 = kb * 64;
        __syncthreads();  // previous K/V tile fully consumed
        load_tile64(Ks, kg + (long long)k0 * a.ldkv, a.ldkv, a.kv_len - k0);
        load_tile64(Vs, vg + (long long)k0 * a.ldkv, a.ldkv, a.kv_len - k0);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        cp_async_wait_all();
        __syncthreads();
        if (kb == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                const int row = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
                const int ch = 2 * kk + (lane >> 4);
                ldsm_x4(qf[kk], Qs + swz(row, ch));
            }
        }
        // S = Q K^T for 16 rows x 64 keys
        float sc[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
#pragma unroll
            for (int np = 0; np < 4; np++) {
                uint32_t b[4];
                const int key = np * 16 + (lane & 7) + 8 * (lane >> 4);
                const int ch = 2 * kk + ((lane >> 3) & 1);
                ldsm_x4(b, Ks + swz(key, ch));
                mma_bf16_16816(sc[2 * np], qf[kk], b[0], b[1]);
                mma_bf16_16816(sc[2 * np + 1], qf[kk], b[2], b[3]);
            }
        }
        // scale + mask
        uint32_t mb[2][2] = {{~0u, ~0u}, {~0u, ~0u}};   // [row g / g+8][key word within the block]
        if (a.mask_bits) {
            const int mw = (a.kv_len + 31) >> 5, w0 = k0 >> 5;
            if (qi0 < a.Tq) { mb[0][0] = a.mask_bits[(long long)qi0 * mw + w0]; if (w0 + 1 < mw) mb[0][1] = a.mask_bits[(long long)qi0 * mw + w0 + 1]; }
            if (qi1 < a.Tq) { mb[1][0] = a.mask_bits[(long long)qi1 * mw + w0]; if (w0 + 1 < mw) mb[1][1] = a.mask_bits[(long long)qi1 * mw + w0 + 1]; }
        }
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int kl = nt * 8 + 2 * t + (c & 1);
                const int key = k0 + kl;
                const int qi = (c < 2) ? qi0 : qi1;
                float s = sc[nt][c] * a.scale;
                bool ok = key < a.kv_len;
                if (a.causal) ok = ok && (key <= a.q_pos0 + qi);
                ok = ok && ((mb[c >> 1][kl >> 5] >> (kl & 31)) & 1u);
                s = ok ? s : -INFINITY;
                sc[nt][c] = s;
                if (c < 2) mx0 = fmaxf(mx0, s); else mx1 = fmaxf(mx1, s);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
        const float u0 = (n0 == -INFINITY) ? 0.f : n0, u1 = (n1 == -INFINITY) ? 0.f : n1;
        const float corr0 = expf(m0 - u0), corr1 = expf(m1 - u1);
        m0 = n0; m1 = n1;
        float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            sc[nt][0] = expf(sc[nt][0] - u0); sc[nt][1] = expf(sc[nt][1] - u0);
            sc[nt][2] = expf(sc[nt][2] - u1); sc[nt][3] = expf(sc[nt][3] - u1);
            rs0 += sc[nt][0] + sc[nt][1];
            rs1 += sc[nt][2] + sc[nt][3];
        }
        rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
        rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
        rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
        rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
        l0 = l0 * corr0 + rs0;
        l1 = l1 * corr1 + rs1;
#pragma unroll
        for (int i = 0; i < 8; i++) { o[i][0] *= corr0; o[i][1] *= corr0; o[i][2] *= corr1; o[i][3] *= corr1; }
        // O += P V
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            uint32_t pa[4];
            pa[0] = pack_bf16x2(sc[2 * kk][0], sc[2 * kk][1]);
            pa[1] = pack_bf16x2(sc[2 * kk][2], sc[2 * kk][3]);
            pa[2] = pack_bf16x2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
            pa[3] = pack_bf16x2(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
            for (int dp = 0; dp < 4; dp++) {
                uint32_t b[4];
                const int key = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
                const int ch = 2 * dp + (lane >> 4);
                ldsm_x4_t(b, Vs + swz(key, ch));
                mma_bf16_16816(o[2 * dp], pa, b[0], b[1]);
                mma_bf16_16816(o[2 * dp + 1], pa, b[2], b[3]);
            }
        }
    }
    const float inv0 = l0 > 0.f ? 1.0f / l0 : 0.f;
    const float inv1 = l1 > 0.f ? 1.0f / l1 : 0.f;
    attn_store(a, r, h, qi0, qi1, t, o, inv0, inv1);
}

// Short-sequence attention (Tq <= 64 and kv_len <= 64, the DiT at L <= 64):
// every CTA walks `per_cta` consecutive (row, head) pairs, prefetching the next
// pair's Q, K and V tiles with cp.async while it computes the current one; one
// key block, so the softmax is exact in one pass (exp2 of pre-scaled scores).
__global__ void __launch_bounds__(128, 5) attn_short_kernel(AttnArgs a, int n_pairs, int per_cta) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(128) uint8_t attn_smem[];
    bf16 *sm = reinterpret_cast<bf16 *>(attn_smem);   // [2 buffers][Q, K, V][64 * 64]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int p0 = blockIdx.x * per_cta;
    const int pend = min(p0 + per_cta, n_pairs);
    const float kLog2e = 1.4426950408889634f;
    const float sc = a.scale * kLog2e;
    auto issue = [&](int p, int buf) {
        const int r = p / kH, h = p % kH;
        bf16 *base = sm + buf * 3 * 64 * 64;
        load_tile64(base, reinterpret_cast<const bf16 *>(a.q) + (long long)r * a.Tq * a.ldq + h * kHD, a.ldq, a.Tq);
        load_tile64(base + 64 * 64, reinterpret_cast<const bf16 *>(a.k) + (long long)r * a.kv_cap * a.ldkv + h * kHD,
                    a.ldkv, a.kv_len);
        load_tile64(base + 2 * 64 * 64, reinterpret_cast<const bf16 *>(a.v) + (long long)r * a.kv_cap * a.ldkv + h * kHD,
                    a.ldkv, a.kv_len);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    };
    if (p0 < pend) issue(p0, 0);
    const int qi0 = warp * 16 + g, qi1 = qi0 + 8;
    // Which of this thread's 32 score slots (nt, c) may attend is the same for
    // every (row, head): key range, causality and the mask, folded into one word
    // (bit 4 nt + c) before the pair loop.
    uint32_t okbits = 0;
    {
        uint32_t mb[2][2] = {{~0u, ~0u}, {~0u, ~0u}};
        if (a.mask_bits) {
            const int mw = (a.kv_len + 31) >> 5;
            if (qi0 < a.Tq) { mb[0][0] = a.mask_bits[qi0 * mw]; if (mw > 1) mb[0][1] = a.mask_bits[qi0 * mw + 1]; }
            if (qi1 < a.Tq) { mb[1][0] = a.mask_bits[qi1 * mw]; if (mw > 1) mb[1][1] = a.mask_bits[qi1 * mw + 1]; }
        }
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int key = nt * 8 + 2 * t + (c & 1);
                const int qi = (c < 2) ? qi0 : qi1;
                bool ok = key < a.kv_len;
                if (a.causal) ok = ok && (key <= a.q_pos0 + qi);
                ok = ok && ((mb[c >> 1][key >> 5] >> (key & 31)) & 1u);
                okbits |= (ok ? 1u : 0u) << (4 * nt + c);
            }
    }
    for (int p = p0, it = 0; p < pend; p++, it++) {
        const int buf = it & 1;
        if (p + 1 < pend) {
            issue(p + 1, buf ^ 1);
            asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        }
        __syncthreads();
        const bf16 *Qs = sm + buf * 3 * 64 * 64, *Ks = Qs + 64 * 64, *Vs = Qs + 2 * 64 * 64;
        uint32_t qf[4][4];
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            const int row = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
            ldsm_x4(qf[kk], Qs + swz(row, 2 * kk + (lane >> 4)));
        }
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
#pragma unroll
            for (int np = 0; np < 4; np++) {
                uint32_t b[4];
                ldsm_x4(b, Ks + swz(np * 16 + (lane & 7) + 8 * (lane >> 4), 2 * kk + ((lane >> 3) & 1)));
                mma_bf16_16816(s[2 * np], qf[kk], b[0], b[1]);
                mma_bf16_16816(s[2 * np + 1], qf[kk], b[2], b[3]);
            }
        }
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const float v = ((okbits >> (4 * nt + c)) & 1u) ? s[nt][c] * sc : -INFINITY;
                s[nt][c] = v;
                if (c < 2) mx0 = fmaxf(mx0, v); else mx1 = fmaxf(mx1, v);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float u0 = mx0 == -INFINITY ? 0.f : mx0, u1 = mx1 == -INFINITY ? 0.f : mx1;
        float l0 = 0.f, l1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            s[nt][0] = exp2f(s[nt][0] - u0); s[nt][1] = exp2f(s[nt][1] - u0);
            s[nt][2] = exp2f(s[nt][2] - u1); s[nt][3] = exp2f(s[nt][3] - u1);
            l0 += s[nt][0] + s[nt][1];
            l1 += s[nt][2] + s[nt][3];
        }
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        float o[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            uint32_t pa[4];
            pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
            pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
            pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int dp = 0; dp < 4; dp++) {
                uint32_t b[4];
                ldsm_x4_t(b, Vs + swz(kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), 2 * dp + (lane >> 4)));
                mma_bf16_16816(o[2 * dp], pa, b[0], b[1]);
                mma_bf16_16816(o[2 * dp + 1], pa, b[2], b[3]);
            }
        }
        const float inv0 = l0 > 0.f ? 1.0f / l0 : 0.f, inv1 = l1 > 0.f ? 1.0f / l1 : 0.f;
        attn_store(a, p / kH, p % kH, qi0, qi1, t, o, inv0, inv1);
        __syncthreads();   // buffer `buf` is refilled two pairs from now
    }
}

constexpr int kShortSmem = 2 * 3 * 64 * 64 * 2;

void pack_mask_bits(const uint8_t *mask, int Tq, int kv_len, uint32_t *bits) {
    const int mw = (kv_len + 31) / 32;
    for (int i = 0; i < Tq; i++)
        for (int w = 0; w < mw; w++) {
            uint32_t v = 0;
            for (int b = 0; b < 32; b++) {
                const int j = 32 * w + b;
                if (j < kv_len && mask[(long long)i * kv_len + j]) v |= 1u << b;
            }
            bits[(long long)i * mw + w] = v;
        }
}

cudaError_t attention_short_prepare() {
    cudaError_t e = cudaFuncSetAttribute(attn_short_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kShortSmem);
    return e != cudaSuccess ? e : attention_tc_prepare();
}

// Decode attention (a few queries per sequence against a long cache, causal,
// no mask): one CTA of 4 warps per (row, query, head).  A warp reads 16 keys
// per round as four groups of four: lane l takes dims 8(l%8)..8(l%8)+7 of key
// 4u + l/8, so each 16-byte load instruction reads four whole 128-byte K (or V)
// rows and a score needs a 3-step shuffle reduction over 8 lanes.  Each group
// of 8 lanes accumulates its own keys' P.V over its 8 dims; the groups, then
// the warps (online-softmax states through shared memory), are merged at the
// end.  Scores are pre-scaled by log2(e) and exponentiated with exp2.
constexpr int kDecWarps = 4, kDecKeys = 16;

__global__ void __launch_bounds__(kDecWarps * 32, 8) attn_decode_kernel(const AttnArgs a) {
    pdl_wait();
    pdl_trigger();
    const int q_pos0 = a.kv_base_dev ? *a.kv_base_dev : a.q_pos0;
    const int kv_len = a.kv_base_dev ? q_pos0 + a.Tq : a.kv_len;
    const int h = blockIdx.x % kH, qi = (blockIdx.x / kH) % a.Tq, r = blockIdx.x / (kH * a.Tq);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 3, c = lane & 7;
    const int n_keys = a.causal ? min(kv_len, q_pos0 + qi + 1) : kv_len;
    const float sc = a.scale * 1.4426950408889634f;
    const bf16 *qg = reinterpret_cast<const bf16 *>(a.q) + ((long long)r * a.Tq + qi) * a.ldq + h * kHD + 8 * c;
    float qv[8];
    {
        const uint4 raw = *reinterpret_cast<const uint4 *>(qg);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            // bf16 pair -> two floats by bit placement (exact)
            qv[2 * i] = __uint_as_float(w[i] << 16) * sc; qv[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u) * sc;
        }
    }
    const long long rbase = (long long)r * a.kv_cap * a.ldkv + h * kHD + 8 * c;
    const bf16 *kg = reinterpret_cast<const bf16 *>(a.k) + rbase;
    const bf16 *vg = reinterpret_cast<const bf16 *>(a.v) + rbase;
    float mx = -INFINITY, l = 0.f, acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = 0.f;
    for (int j0 = warp * kDecKeys; j0 < n_keys; j0 += kDecWarps * kDecKeys) {
        uint4 kr[4], vr[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int j = min(j0 + 4 * u + g, n_keys - 1);   // past the end: a valid row, masked below
            kr[u] = *reinterpret_cast<const uint4 *>(kg + (long long)j * a.ldkv);
            vr[u] = *reinterpret_cast<const uint4 *>(vg + (long long)j * a.ldkv);
        }
        float s[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint32_t w[4] = {kr[u].x, kr[u].y, kr[u].z, kr[u].w};
            float d = 0.f;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                d = fmaf(qv[2 * i], __uint_as_float(w[i] << 16), d);
                d = fmaf(qv[2 * i + 1], __uint_as_float(w[i] & 0xFFFF0000u), d);
            }
            s[u] = d;
        }
#pragma unroll
        for (int o = 4; o > 0; o >>= 1)
#pragma unroll
            for (int u = 0; u < 4; u++) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o);
        float bm = mx;
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (j0 + 4 * u + g >= n_keys) s[u] = -INFINITY;
            bm = fmaxf(bm, s[u]);
        }
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 8));
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 16));
        const float corr = exp2f(mx - bm);
        l *= corr;
#pragma unroll
        for (int i = 0; i < 8; i++) acc[i] *= corr;
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const float p = exp2f(s[u] - bm);
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
    // merge the four key groups (lanes c, c + 8, c + 16, c + 24)
#pragma unroll
    for (int o = 8; o < 32; o <<= 1) {
        l += __shfl_xor_sync(0xffffffffu, l, o);
#pragma unroll
        for (int i = 0; i < 8; i++) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
    }
    __shared__ float sm_m[kDecWarps], sm_l[kDecWarps];
    __shared__ float4 sm_o[kDecWarps][16];
    if (lane == 0) { sm_m[warp] = mx; sm_l[warp] = l; }
    if (g == 0) {
        sm_o[warp][2 * c] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        sm_o[warp][2 * c + 1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    __syncthreads();
    if (warp == 0 && lane < 16) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDecWarps; w++) M = fmaxf(M, sm_m[w]);
        float L = 0.f;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kDecWarps; w++) {
            if (sm_m[w] == -INFINITY) continue;   // a warp that saw no key
            const float f = exp2f(sm_m[w] - M);
            const float4 o = sm_o[w][lane];
            L += sm_l[w] * f;
            x.x += o.x * f; x.y += o.y * f; x.z += o.z * f; x.w += o.w * f;
        }
        const float inv = L > 0.f ? 1.0f / L : 0.f;
        bf16 *og = reinterpret_cast<bf16 *>(a.o) + ((long long)r * a.Tq + qi) * a.ldo + h * kHD;
        reinterpret_cast<uint2 *>(og)[lane] = make_uint2(pack_bf16x2(x.x * inv, x.y * inv), pack_bf16x2(x.z * inv, x.w * inv));
    }
}

void launch_attention_bf16(const AttnArgs &a, cudaStream_t s, bool pdl) {
    pdl = pdl && pdl_enabled();
    if (a.Tq <= 8 && !a.mask && !a.mask_bits && !a.o8 && (a.kv_base_dev || a.kv_len > 64)) {
        launch_k(pdl, attn_decode_kernel, dim3(a.rows * a.Tq * kH), dim3(kDecWarps * 32), 0, s, a);
        return;
    }
    if (attention_tc_eligible(a)) {
        launch_attention_tc(a, a.err, s, pdl);
        return;
    }
    if (a.Tq <= 64 && a.kv_len <= 64 && !a.kv_base_dev) {
        const int n_pairs = a.rows * kH;
        int dev = 0, nsm = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        // one wave of resident CTAs (48 KB of shared memory each: 4 per SM on
        // B200), each with a few pairs to pipeline
        static int occ_cache[64] = {0};
        int occ = dev < 64 ? occ_cache[dev] : 0;
        if (occ <= 0) {
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, attn_short_kernel, 128, kShortSmem) != cudaSuccess ||
                occ < 1)
                occ = 1;
            if (dev < 64) occ_cache[dev] = occ;
        }
        const int target = nsm * occ;
        const int per_cta = std::max(1, (n_pairs + target - 1) / target);
        const int grid = (n_pairs + per_cta - 1) / per_cta;
        launch_k(pdl, attn_short_kernel, dim3(grid), dim3(128), (size_t)kShortSmem, s, a, n_pairs, per_cta);
        return;
    }
    if (attention_tc_long_eligible(a)) {
        launch_attention_tc_long(a, a.err, s, pdl);
        return;
    }
    if (attention_tc_causal_eligible(a)) {
        launch_attention_tc_causal(a, a.err, s, pdl);
        return;
    }
    launch_k(pdl, attn_bf16_kernel, dim3((a.Tq + 63) / 64, kH, a.rows), dim3(128), 0, s, a);
}

// =========================================================================
// fp32 attention (SIMT), one CTA per (head, row); K and V of the row/head in
// shared memory; each thread owns one query at a time.  Softmax as
// include/dit_manual.h:83-86 (max, exp, sum), then P.V.
// =========================================================================
__global__ void __launch_bounds__(128) attn_f32_kernel(AttnArgs a) {
    extern __shared__ float kvs[];
    float *Ks = kvs;
    float *Vs = kvs + (long long)a.kv_len * kHD;
    const int h = blockIdx.x, r = blockIdx.y;
    const float *kg = reinterpret_cast<const float *>(a.k) + (long long)r * a.kv_cap * a.ldkv + h * kHD;
    const float *vg = reinterpret_cast<const float *>(a.v) + (long long)r * a.kv_cap * a.ldkv + h * kHD;
    for (int idx = threadIdx.x; idx < a.kv_len * kHD; idx += blockDim.x) {
        const int j = idx / kHD, d = idx % kHD;
        Ks[idx] = kg[(long long)j * a.ldkv + d];
        Vs[idx] = vg[(long long)j * a.ldkv + d];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < a.Tq; i += blockDim.x) {
        const float *qg = reinterpret_cast<const float *>(a.q) + ((long long)r * a.Tq + i) * a.ldq + h * kHD;
        float q[kHD];
#pragma unroll
        for (int d = 0; d < kHD; d++) q[d] = qg[d];
        float mx = -INFINITY;
        for (int j = 0; j < a.kv_len; j++) {
            bool ok = true;
            if (a.causal) ok = j <= a.q_pos0 + i;
            if (a.mask) ok = ok && a.mask[(long long)i * a.kv_len + j] != 0;
            if (!ok) continue;
            float s = 0.f;
#pragma unroll
            for (int d = 0; d < kHD; d++) s += q[d] * Ks[j * kHD + d];
            mx = fmaxf(mx, s * a.scale);
        }
        float acc[kHD];
#pragma unroll
        for (int d = 0; d < kHD; d++) acc[d] = 0.f;
        float sum = 0.f;
        for (int j = 0; j < a.kv_len; j++) {
            bool ok = true;
            if (a.causal) ok = j <= a.q_pos0 + i;
            if (a.mask) ok = ok && a.mask[(long long)i * a.kv_len + j] != 0;
            if (!ok) continue;
            float s = 0.f;
#pragma unroll
            for (int d = 0; d < kHD; d++) s += q[d] * Ks[j * kHD + d];
            const float p = expf(s * a.scale - mx);
            sum += p;
#pragma unroll
            for (int d = 0; d < kHD; d++) acc[d] += p * Vs[j * kHD + d];
        }
        const float inv = sum > 0.f ? 1.0f / sum : 0.f;
        float *og = reinterpret_cast<float *>(a.o) + ((long long)r * a.Tq + i) * a.ldo + h * kHD;
#pragma unroll
        for (int d = 0; d < kHD; d++) og[d] = acc[d] * inv;
    }
}

cudaError_t attention_f32_prepare() {
    return cudaFuncSetAttribute(attn_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

cudaError_t launch_attention_f32(const AttnArgs &a, cudaStream_t s) {
    const size_t smem = (size_t)a.kv_len * kHD * 2 * sizeof(float);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    attn_f32_kernel<<<dim3(kH, a.rows), 128, smem, s>>>(a);
    return cudaGetLastError();
}

// =========================================================================
// fp32 SIMT GEMM: 64x64 tile, BK 16, 256 threads, 4x4 outputs per thread.
// Each output accumulates over k in increasing order; bias added last.
// =========================================================================
__global__ void __launch_bounds__(256) gemm_f32_kernel(const float *__restrict__ A, const float *__restrict__ B,
                                                       const float *__restrict__ bias, float *__restrict__ C, int M,
                                                       int N, int K) {
    __shared__ float As[16][64 + 4];
    __shared__ float Bs[16][64 + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int idx = threadIdx.x; idx < 64 * 16; idx += 256) {
            const int rr = idx >> 4, kk = idx & 15;
            const int gm = m0 + rr, gn = n0 + rr, gk = k0 + kk;
            As[kk][rr] = (gm < M && gk < K) ? A[(long long)gm * K + gk] : 0.f;
            Bs[kk][rr] = (gn < N && gk < K) ? B[(long long)gn * K + gk] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; kk++) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) { av[i] = As[kk][ty * 4 + i]; bv[i] = Bs[kk][tx * 4 + i]; }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] += av[i] * bv[j];
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int gm = m0 + ty * 4 + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int gn = n0 + tx * 4 + j;
            if (gn < N) C[(long long)gm * N + gn] = acc[i][j] + (bias ? bias[gn] : 0.f);
        }
    }
}

void launch_gemm_f32(const float *A, const float *B, const float *bias, float *C, int M, int N, int K,
                     cudaStream_t s) {
    dim3 grid((N + 63) / 64, (M + 63) / 64);
    gemm_f32_kernel<<<grid, 256, 0, s>>>(A, B, bias, C, M, N, K);
}

__global__ void qk_norm_rope_f32_kernel(float *q, float *k, int M, int tok_per_row, int qk_norm,
                                        const float *qn, const float *kn, const float2 *rope, int rope_mode,
                                        int pos_start) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // (token, head)
    if (idx >= (long long)M * kH) return;
    const int m = (int)(idx / kH), h = (int)(idx % kH);
    const int t = m % tok_per_row;
    const float2 *cs = rope + (long long)(pos_start + t) * 32;
    for (int which = 0; which < 2; which++) {
        float *p = (which == 0 ? q : k) + (long long)m * kD + h * kHD;
        const float *g = which == 0 ? qn : kn;
        float v[kHD];
#pragma unroll
        for (int d = 0; d < kHD; d++) v[d] = p[d];
        if (qk_norm) {
            float ss = 0.f;
#pragma unroll
            for (int d = 0; d < kHD; d++) ss += v[d] * v[d];
            const float inv = 1.0f / sqrtf(ss / kHD + 1e-6f);
#pragma unroll
            for (int d = 0; d < kHD; d++) { float y = v[d] * inv; if (g) y *= g[d]; v[d] = y; }
        }
        if (rope_mode == ROPE_HALF) {
#pragma unroll
            for (int d = 0; d < 32; d++) {
                const float2 e = cs[d];
                const float x1 = v[d], x2 = v[d + 32];
                v[d] = x1 * e.x - x2 * e.y;
                v[d + 32] = x2 * e.x + x1 * e.y;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const float2 e = cs[i];
                const float x0 = v[2 * i], x1 = v[2 * i + 1];
                v[2 * i] = x0 * e.x - x1 * e.y;
                v[2 * i + 1] = x0 * e.y + x1 * e.x;
            }
        }
#pragma unroll
        for (int d = 0; d < kHD; d++) p[d] = v[d];
    }
}

void launch_qk_norm_rope_f32(float *q, float *k, int M, int tok_per_row, int qk_norm, const float *qn,
                             const float *kn, const float2 *rope, int rope_mode, int pos_start, cudaStream_t s) {
    const long long n = (long long)M * kH;
    qk_norm_rope_f32_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(q, k, M, tok_per_row, qk_norm, qn, kn, rope,
                                                                         rope_mode, pos_start);
}

// =========================================================================
// conversions
// =========================================================================
__global__ void f32_to_bf16_kernel(const float *__restrict__ x, bf16 *__restrict__ y, long long n) {
    const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i + 3 < n) {
        const float4 v = *reinterpret_cast<const float4 *>(x + i);
        *reinterpret_cast<uint2 *>(y + i) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
    } else {
        for (long long j = i; j < n; j++) y[j] = __float2bfloat16_rn(x[j]);
    }
}
void launch_f32_to_bf16(const float *x, bf16 *y, long long n, cudaStream_t s) {
    const long long threads = (n + 3) / 4;
    f32_to_bf16_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, y, n);
}

__global__ void silu_bf16_kernel(const float *__restrict__ x, bf16 *__restrict__ y, long long n) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) { const float c = x[i]; y[i] = __float2bfloat16_rn(c / (1.0f + expf(-c))); }
}
void launch_silu_bf16(const float *x, bf16 *y, long long n, cudaStream_t s) {
    silu_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, y, n);
}

__global__ void add_f32_kernel(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ c,
                               long long n) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) c[i] = a[i] + b[i];
}
void launch_add_f32(const float *a, const float *b, float *c, long long n, cudaStream_t s) {
    add_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(a, b, c, n);
}

__global__ void history_rows_kernel(const float *__restrict__ src, int n_seq, int src_len, bf16 *__restrict__ dst,
                                    int L, int row_stride, int row_off) {
    const long long i4 = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // float4 index
    const long long total4 = (long long)n_seq * src_len * (kD / 4);
    if (i4 >= total4) return;
    const long long tok = i4 / (kD / 4);
    const int c4 = (int)(i4 % (kD / 4));
    const int u = (int)(tok / src_len), t = (int)(tok % src_len);
    const float4 v = reinterpret_cast<const float4 *>(src)[i4];
    const long long drow = ((long long)u * row_stride + row_off) * L + t;
    reinterpret_cast<uint2 *>(dst + drow * kD)[c4] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
}
void launch_history_rows(const float *src, int n_seq, int src_len, bf16 *dst, int L, int row_stride, int row_off,
                         cudaStream_t s) {
    const long long total4 = (long long)n_seq * src_len * (kD / 4);
    if (total4 == 0) return;
    history_rows_kernel<<<(unsigned)((total4 + 255) / 256), 256, 0, s>>>(src, n_seq, src_len, dst, L, row_stride,
                                                                          row_off);
}

// =========================================================================
// conditioning
// =========================================================================
// y[k][o] = act(W[o] . x[k] + b[o]) for nx input vectors; one warp per output
// row o (the row is read once, coalesced, for all nx inputs).
template <int IN, bool SILU>
__global__ void __launch_bounds__(256) warp_gemv_kernel(const float *__restrict__ x, int nx,
                                                        const float *__restrict__ w, const float *__restrict__ b,
                                                        float *__restrict__ y, int out) {
    constexpr int PER = IN / 32;
    const int o = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (o >= out) return;
    float wr[PER];
    const float *wrow = w + (long long)o * IN;
#pragma unroll
    for (int j = 0; j < PER; j++) wr[j] = wrow[lane + 32 * j];
    for (int k = 0; k < nx; k++) {
        const float *xk = x + (long long)k * IN;
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < PER; j++) s += wr[j] * xk[lane + 32 * j];
        s = warp_sum(s);
        if (lane == 0) {
            float v = s + (b ? b[o] : 0.f);
            if (SILU) v = v / (1.0f + expf(-v));
            y[(long long)k * out + o] = v;
        }
    }
}

void launch_time_mlp(const float *se, int n, const float *w1, const float *b1, const float *w2, const float *b2,
                     float *h1_scratch, float *temb, cudaStream_t s) {
    warp_gemv_kernel<256, true><<<kD / 8, 256, 0, s>>>(se, n, w1, b1, h1_scratch, kD);
    warp_gemv_kernel<kD, false><<<kD / 8, 256, 0, s>>>(h1_scratch, n, w2, b2, temb, kD);
}

// LayerNorm (affine, eps 1e-5) of y[u] in place, times scale: one block per row.
__global__ void __launch_bounds__(1024) speaker_ln_kernel(float *__restrict__ y, const float *__restrict__ lw,
                                                          const float *__restrict__ lb, float scale) {
    __shared__ float red[32];
    const int u = blockIdx.x, o = threadIdx.x;
    const float v0 = y[(long long)u * kD + o];
    float v = warp_sum(v0);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float mean = 0.f;
    for (int i = 0; i < 32; i++) mean += red[i];
    mean /= kD;
    __syncthreads();
    const float d = v0 - mean;
    v = warp_sum(d * d);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float var = 0.f;
    for (int i = 0; i < 32; i++) var += red[i];
    const float istd = 1.0f / sqrtf(var / kD + 1e-5f);
    float xo = d * istd;
    if (lw) xo *= lw[o];
    if (lb) xo += lb[o];
    y[(long long)u * kD + o] = xo * scale;
}

void launch_speaker_cond(const float *spk, int n_utt, const float *w, const float *b, const float *ln_w,
                         const float *ln_b, float scale, float *spk_c, cudaStream_t s) {
    warp_gemv_kernel<kSpk, false><<<kD / 8, 256, 0, s>>>(spk, n_utt, w, b, spk_c, kD);
    speaker_ln_kernel<<<n_utt, kD, 0, s>>>(spk_c, ln_w, ln_b, scale);
}

// a[k*n + u][c] = bf16(SiLU(temb[k][c] + spk_c[u][c]))
__global__ void cond_rows_kernel(const float *__restrict__ temb, int n_t, const float *__restrict__ spk_c, int n,
                                 bf16 *__restrict__ a) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n_t * n * kD) return;
    const long long row = i / kD;
    const int c = (int)(i % kD);
    const int k = (int)(row / n), u = (int)(row % n);
    float v = temb[(long long)k * kD + c];
    if (spk_c) v += spk_c[(long long)u * kD + c];
    a[i] = __float2bfloat16_rn(v / (1.0f + expf(-v)));
}

void launch_cond_rows(const float *temb, int n_t, const float *spk_c, int n, bf16 *a_cond, cudaStream_t s) {
    const long long tot = (long long)n_t * n * kD;
    cond_rows_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(temb, n_t, spk_c, n, a_cond);
}

// =========================================================================
// DiT output head: 8 tokens per block.  Each warp normalises and modulates one
// token row into shared memory; then thread (kg, c4) accumulates outputs
// 4c4..4c4+3 of the 8 tokens over k in [128 kg, 128 kg + 128), reading
// W_out^T [1024][128] as coalesced float4 rows, and the 8 K-group partials are
// summed through shared memory.
// =========================================================================
constexpr int kOutTok = 8;

__global__ void __launch_bounds__(256) out_head_kernel(const float *__restrict__ h, int rows, int L, int P,
                                                       const float *__restrict__ shift,
                                                       const float *__restrict__ scale, long long ada_ld,
                                                       int rows_per_ada, const float *__restrict__ wt,
                                                       const float *__restrict__ b, float *__restrict__ vel,
                                                       int *err) {
    __shared__ __align__(16) float u[kOutTok][kD];   // modulated rows; later the K-group partials
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tok0 = blockIdx.x * kOutTok;
    const int ntok = rows * P;
    {
        const int tk = tok0 + warp;
        if (tk < ntok) {
            const int r = tk / P, p = tk % P;
            const float4 *x = reinterpret_cast<const float4 *>(h + ((long long)r * L + (L - P + p)) * kD);
            float4 v[8];
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < 8; j++) { v[j] = x[lane + 32 * j]; sum += (v[j].x + v[j].y) + (v[j].z + v[j].w); }
            const float mean = warp_sum(sum) * (1.0f / kD);
            float q = 0.f;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float a0 = v[j].x - mean, a1 = v[j].y - mean, a2 = v[j].z - mean, a3 = v[j].w - mean;
                q += (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
            }
            const float inv = 1.0f / sqrtf(warp_sum(q) * (1.0f / kD) + 1e-5f);
            const long long ar = (long long)(r / rows_per_ada) * ada_ld;
            const float4 *sh = reinterpret_cast<const float4 *>(shift + ar);
            const float4 *sc = reinterpret_cast<const float4 *>(scale + ar);
            float4 *ur = reinterpret_cast<float4 *>(u[warp]);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int c4 = lane + 32 * j;
                const float4 a = __ldg(sh + c4), g = __ldg(sc + c4);
                ur[c4] = make_float4((v[j].x - mean) * inv * (1.0f + g.x) + a.x,
                                     (v[j].y - mean) * inv * (1.0f + g.y) + a.y,
                                     (v[j].z - mean) * inv * (1.0f + g.z) + a.z,
                                     (v[j].w - mean) * inv * (1.0f + g.w) + a.w);
            }
        } else {
            float4 *ur = reinterpret_cast<float4 *>(u[warp]);
#pragma unroll
            for (int j = 0; j < 8; j++) ur[lane + 32 * j] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    __syncthreads();
    const int c4 = lane, kg = warp;
    float4 acc[kOutTok];
#pragma unroll
    for (int t = 0; t < kOutTok; t++) acc[t] = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 *w4 = reinterpret_cast<const float4 *>(wt) + c4;
#pragma unroll 16
    for (int kk = 0; kk < kD / 8; kk++) {
        const int k = kg * (kD / 8) + kk;
        const float4 w = __ldg(w4 + (long long)k * (kLat / 4));
#pragma unroll
        for (int t = 0; t < kOutTok; t++) {
            const float xv = u[t][k];
            acc[t].x += w.x * xv; acc[t].y += w.y * xv; acc[t].z += w.z * xv; acc[t].w += w.w * xv;
        }
    }
    __syncthreads();   // every thread is done with u: reuse it for the partials [kg][t][c4]
    float4 *part = reinterpret_cast<float4 *>(&u[0][0]);
#pragma unroll
    for (int t = 0; t < kOutTok; t++) part[(kg * kOutTok + t) * 32 + c4] = acc[t];
    __syncthreads();
    {
        const int t = warp;
        float4 y = part[t * 32 + c4];
#pragma unroll
        for (int g = 1; g < 8; g++) {
            const float4 o = part[(g * kOutTok + t) * 32 + c4];
            y.x += o.x; y.y += o.y; y.z += o.z; y.w += o.w;
        }
        if (b) {
            const float4 bb = __ldg(reinterpret_cast<const float4 *>(b) + c4);
            y.x += bb.x; y.y += bb.y; y.z += bb.z; y.w += bb.w;
        }
        const int tok = tok0 + t;
        if (tok < ntok) {
            if (err && !(isfinite(y.x) && isfinite(y.y) && isfinite(y.z) && isfinite(y.w)))
                atomicCAS(err, 0, DEVERR_NONFINITE);
            reinterpret_cast<float4 *>(vel + (long long)tok * kLat)[c4] = y;
        }
    }
}

void launch_out_head(const float *h, int rows, int L, int P, const float *shift, const float *scale,
                     long long ada_ld, int rows_per_ada, const float *w_out_t, const float *b_out, float *vel, int *err,
                     cudaStream_t s) {
    const int ntok = rows * P;
    out_head_kernel<<<(ntok + kOutTok - 1) / kOutTok, 256, 0, s>>>(h, rows, L, P, shift, scale, ada_ld, rows_per_ada,
                                                                   w_out_t, b_out, vel, err);
}

// CFG combine + Euler update + coordinate projection, kEulerRows z rows
// (utterance, frame) per block.  The block updates its own rows of z in place
// (each row belongs to one block), then thread t computes outputs 4t..4t+3 of
// every row from coordinate_proj^T [128][1024] read as coalesced float4 rows.
constexpr int kEulerRows = 4;

__global__ void __launch_bounds__(256) cfg_euler_kernel(const float *__restrict__ vel, float *__restrict__ z, int nrows,
                                                        int P, float cfg_scale, int cfg_form, float dt, int update,
                                                        const float *__restrict__ wct, const float *__restrict__ bc,
                                                        bf16 *__restrict__ x_in, int L) {
    __shared__ float zs[kEulerRows][kLat];
    const int r0 = blockIdx.x * kEulerRows;
    for (int i = threadIdx.x; i < kEulerRows * kLat; i += blockDim.x) {
        const int rr = i / kLat, c = i % kLat, r = r0 + rr;
        float zv = 0.f;
        if (r < nrows) {
            const int u = r / P, p = r % P;
            float *zp = z + (long long)r * kLat;
            zv = zp[c];
            if (update) {
                const float vc = vel[((long long)(2 * u) * P + p) * kLat + c];
                const float vu = vel[((long long)(2 * u + 1) * P + p) * kLat + c];
                const float v = cfg_form == 0 ? vc + cfg_scale * (vc - vu) : vu + cfg_scale * (vc - vu);
                zv += v * dt;
                zp[c] = zv;
            }
        }
        zs[rr][c] = zv;
    }
    __syncthreads();
    const int o4 = threadIdx.x;   // outputs 4 o4 .. 4 o4 + 3
    float4 acc[kEulerRows];
#pragma unroll
    for (int rr = 0; rr < kEulerRows; rr++) acc[rr] = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 *w4 = reinterpret_cast<const float4 *>(wct) + o4;
#pragma unroll 16
    for (int k = 0; k < kLat; k++) {
        const float4 w = __ldg(w4 + (long long)k * (kD / 4));
#pragma unroll
        for (int rr = 0; rr < kEulerRows; rr++) {
            const float xv = zs[rr][k];
            acc[rr].x += w.x * xv; acc[rr].y += w.y * xv; acc[rr].z += w.z * xv; acc[rr].w += w.w * xv;
        }
    }
    const float4 bb = bc ? __ldg(reinterpret_cast<const float4 *>(bc) + o4) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int rr = 0; rr < kEulerRows; rr++) {
        const int r = r0 + rr;
        if (r >= nrows) break;
        const int u = r / P, p = r % P;
        const long long tok = L - P + p;
        __nv_bfloat162 lo = __floats2bfloat162_rn(acc[rr].x + bb.x, acc[rr].y + bb.y);
        __nv_bfloat162 hi = __floats2bfloat162_rn(acc[rr].z + bb.z, acc[rr].w + bb.w);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t *>(&lo);
        pk.y = *reinterpret_cast<uint32_t *>(&hi);
        *reinterpret_cast<uint2 *>(x_in + ((long long)(2 * u) * L + tok) * kD + 4 * o4) = pk;
        *reinterpret_cast<uint2 *>(x_in + ((long long)(2 * u + 1) * L + tok) * kD + 4 * o4) = pk;
    }
}

void launch_cfg_euler(const float *vel, float *z, int n_utt, int P, float cfg_scale, int cfg_form, float dt,
                      int update, const float *w_coord_t, const float *b_coord, bf16 *x_in, int L, cudaStream_t s) {
    const int nrows = n_utt * P;
    cfg_euler_kernel<<<(nrows + kEulerRows - 1) / kEulerRows, kD / 4, 0, s>>>(
        vel, z, nrows, P, cfg_scale, cfg_form, dt, update, w_coord_t, b_coord, x_in, L);
}

// =========================================================================
// FM history on the device
// =========================================================================
// Row (u, p) of src ([n_utt * P][1024], or one row broadcast to every (u, p)
// when broadcast != 0) to row u * cap + start + p of dst.
__global__ void fm_place_rows_kernel(const float *__restrict__ src, float *__restrict__ dst, int P, int cap, int start,
                                     int broadcast) {
    const int r = blockIdx.x, u = r / P, p = r % P;
    const float4 *s4 = reinterpret_cast<const float4 *>(src + (broadcast ? 0 : (long long)r * kD));
    float4 *d4 = reinterpret_cast<float4 *>(dst + ((long long)u * cap + start + p) * kD);
    for (int i = threadIdx.x; i < kD / 4; i += blockDim.x) d4[i] = s4[i];
}

void launch_fm_place_rows(const float *src, float *dst, int n_utt, int P, int cap, int start, int broadcast,
                          cudaStream_t s) {
    fm_place_rows_kernel<<<n_utt * P, 256, 0, s>>>(src, dst, P, cap, start, broadcast);
}

// EOS head activation in place: SiLU(s) = s sigmoid(s) (eos_proj.1), or the
// shipped code's s * (s / (1 + exp(-s))) (src/e2e_pipeline_v4.cpp:608-609).
__global__ void eos_act_kernel(float *__restrict__ x, long long n, int as_written) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = x[i];
    const float silu = v / (1.0f + expf(-v));
    x[i] = as_written ? v * silu : silu;
}

// p = softmax(logits[u][0..1])[1], as src/e2e_pipeline_v4.cpp:617-619.
__global__ void eos_prob_kernel(const float *__restrict__ logits, int n, float *__restrict__ prob) {
    const int u = blockIdx.x * blockDim.x + threadIdx.x;
    if (u >= n) return;
    const float a = logits[2 * u], b = logits[2 * u + 1];
    const float mx = fmaxf(a, b);
    const float sum = expf(a - mx) + expf(b - mx);
    prob[u] = expf(b - mx) / sum;
}

void launch_eos_act(float *h1, int n, int as_written, cudaStream_t s) {
    const long long tot = (long long)n * kLLM;
    eos_act_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(h1, tot, as_written);
}

void launch_eos_prob(const float *logits, int n, float *prob, cudaStream_t s) {
    eos_prob_kernel<<<(n + 127) / 128, 128, 0, s>>>(logits, n, prob);
}

// =========================================================================
// PatchEncoder
// =========================================================================
// Causal stride-2 conv (k = 2, taps 2t-1 and 2t, tap 2t-1 of the first token
// from `tail`): TOK tokens per block (16 for a prefill, 1 for a decode step),
// their input frames staged in shared memory; thread c computes output
// channel c of all of them from the transposed weight wt[ic][k][c] (coalesced
// across threads, 16 input channels of weights loaded ahead).  new_tail: the
// last frame.
template <int TOK>
__global__ void __launch_bounds__(128) pe_conv_kernel(const float *__restrict__ frames, int n_frames, int B,
                                                      const float *__restrict__ tail, const float *__restrict__ wt,
                                                      const float *__restrict__ bias, bf16 *__restrict__ out,
                                                      float *__restrict__ new_tail) {
    pdl_wait();
    pdl_trigger();
    __shared__ float f[TOK][2][kLat];
    const int T = n_frames / 2;
    const long long n_tok = (long long)B * T, tok0 = (long long)blockIdx.x * TOK;
    const int c = threadIdx.x;
    for (int i = 0; i < TOK; i++) {
        const long long g = tok0 + i;
        float v0 = 0.f, v1 = 0.f;
        if (g < n_tok) {
            const int b = (int)(g / T), t = (int)(g % T);
            const float *fb = frames + (long long)b * n_frames * kLat;
            v0 = t > 0 ? fb[(long long)(2 * t - 1) * kLat + c] : (tail ? tail[(long long)b * kLat + c] : 0.f);
            v1 = fb[(long long)(2 * t) * kLat + c];
            if (new_tail && t == T - 1) new_tail[(long long)b * kLat + c] = fb[(long long)(n_frames - 1) * kLat + c];
        }
        f[i][0][c] = v0;
        f[i][1][c] = v1;
    }
    __syncthreads();
    float s[TOK];
    const float b0 = bias ? bias[c] : 0.f;
#pragma unroll
    for (int i = 0; i < TOK; i++) s[i] = b0;
    for (int ic0 = 0; ic0 < kLat; ic0 += 16) {
        float w[16][2];
#pragma unroll
        for (int u = 0; u < 16; u++) {
            w[u][0] = __ldg(wt + ((ic0 + u) * 2 + 0) * kLat + c);
            w[u][1] = __ldg(wt + ((ic0 + u) * 2 + 1) * kLat + c);
        }
#pragma unroll
        for (int u = 0; u < 16; u++)
#pragma unroll
            for (int i = 0; i < TOK; i++) {
                s[i] += f[i][0][ic0 + u] * w[u][0];
                s[i] += f[i][1][ic0 + u] * w[u][1];
            }
    }
#pragma unroll
    for (int i = 0; i < TOK; i++)
        if (tok0 + i < n_tok) out[(tok0 + i) * kLat + c] = __float2bfloat16_rn(s[i]);
}

void launch_pe_conv(const float *frames, int B, int n_frames, const float *tail, const float *wt, const float *bias,
                    bf16 *out, float *new_tail, cudaStream_t s) {
    const long long n_tok = (long long)B * (n_frames / 2);
    if (n_tok >= 4096)
        pe_conv_kernel<16><<<(unsigned)((n_tok + 15) / 16), kLat, 0, s>>>(frames, n_frames, B, tail, wt, bias, out,
                                                                          new_tail);
    else
        pe_conv_kernel<1><<<(unsigned)n_tok, kLat, 0, s>>>(frames, n_frames, B, tail, wt, bias, out, new_tail);
}

__global__ void pe_pairs_kernel(const float *__restrict__ h, int T, int pair_mode, bf16 *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int n = T / 2;
    const int bq = blockIdx.x;             // b * n + q
    const int b = bq / n, q = bq % n;
    for (int c = threadIdx.x; c < 2 * kD; c += blockDim.x) {
        const int s = c / kD, i = c % kD;
        int tok;
        if (pair_mode == 0) {
            tok = 2 * q + s;
        } else {
            const int g = 2 * q + s;
            tok = 2 * (g % n) + g / n;
        }
        out[(long long)bq * 2 * kD + c] = __float2bfloat16_rn(h[((long long)b * T + tok) * kD + i]);
    }
}

void launch_pe_pairs(const float *h, int B, int T, int pair_mode, bf16 *out, cudaStream_t s, bool pdl) {
    launch_k(pdl && pdl_enabled(), pe_pairs_kernel, dim3(B * (T / 2)), dim3(256), 0, s, h, T, pair_mode, out);
}

}  // namespace dtts
