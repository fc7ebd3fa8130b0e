// LayerNorm (no affine, eps 1e-5) + adaLN modulation of token rows of kD fp32
// values, the DiT block's norm (dit_manual.h:16-21 and :158-168 of the
// reference):
//
//   y = LN(x) * (1 + scale[r]) + shift[r],   r = token / tok_per_row
//
// One warp per row; lane l holds the float4s at columns 4 (l + 32 j), j < 8.
// The standalone LayerNorm kernels (kernels.cu) and the residual GEMM's fused
// LayerNorm epilogue (gemm_tc.cuh, EPI_RESID_GATED_LN) both run these
// routines, so the two paths give the same bits: the standalone kernels read
// the rows from global memory, R rows loaded before any is reduced so that
// their L2 round trips overlap; the fused epilogue brings them into shared
// memory with bulk copies and also keeps a copy of the modulation row there
// (ModRow), since the GEMM's shared-memory carve-out leaves little L1.
#pragma once
#include "common.cuh"

namespace dtts {

struct LnParams {
    const float *shift, *scale;   // modulation rows [rows][ada_ld]
    long long ada_ld;
    int tok_per_row;              // tokens sharing one modulation row
    void *out;                    // [M][kD]: bf16, or e4m3 for ln_rows_f8
    // e4m3 output only: row_scale[token] = absmax / 448; unorm (optional)
    // receives 1.08 |u|; g_scale / g_inv (optional) the bound B on the row's
    // |gelu(W1 u + b1)|, B = 1.02 max(1.08 |u| w1n + b1max, 0.17), as B / 448
    // and 448 / B
    float *row_scale, *unorm, *g_scale, *g_inv;
    float w1n, b1max;
};

// A modulation row (shift, scale) staged in shared memory: rows whose
// token / tok_per_row == mr read it there.  mr = -1: none staged.
struct ModRow {
    long long mr;
    const float *shift, *scale;
};

// Copies modulation row mr into this warp's shared buffers (2 x kD floats).
DTTS_DEV void ln_stage_mod(const LnParams &p, long long mr, float *shift_s, float *scale_s, int lane) {
    const float4 *sh = reinterpret_cast<const float4 *>(p.shift + mr * p.ada_ld);
    const float4 *sc = reinterpret_cast<const float4 *>(p.scale + mr * p.ada_ld);
    float4 *ds = reinterpret_cast<float4 *>(shift_s), *dc = reinterpret_cast<float4 *>(scale_s);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        ds[lane + 32 * j] = __ldg(sh + lane + 32 * j);
        dc[lane + 32 * j] = __ldg(sc + lane + 32 * j);
    }
}

template <int R>
DTTS_DEV void ln_load_rows(const float *x, const int (&row)[R], const bool (&live)[R], float4 (&v)[R][8],
                           int lane) {
#pragma unroll
    for (int r = 0; r < R; r++)
        if (live[r]) {
            const float4 *xr = reinterpret_cast<const float4 *>(x + (long long)row[r] * kD);
#pragma unroll
            for (int j = 0; j < 8; j++) v[r][j] = __ldcg(xr + lane + 32 * j);
        }
}

// mean and 1 / sqrt(variance + 1e-5) of one row (two passes over registers)
DTTS_DEV void ln_stats(const float4 (&v)[8], float &mean, float &inv) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    mean = warp_sum(s) * (1.0f / kD);
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float e0 = v[j].x - mean, e1 = v[j].y - mean, e2 = v[j].z - mean, e3 = v[j].w - mean;
        q += (e0 * e0 + e1 * e1) + (e2 * e2 + e3 * e3);
    }
    inv = 1.0f / sqrtf(warp_sum(q) * (1.0f / kD) + 1e-5f);
}

// LayerNorm + modulation of one row held in v (lane layout above), bf16 out.
DTTS_DEV void ln_row_out_bf16(const float4 (&v)[8], const LnParams &p, int row, int lane) {
    float mean, inv;
    ln_stats(v, mean, inv);
    const long long mr = row / p.tok_per_row;
    const float4 *sh = reinterpret_cast<const float4 *>(p.shift + mr * p.ada_ld);
    const float4 *sc = reinterpret_cast<const float4 *>(p.scale + mr * p.ada_ld);
    uint2 *yr = reinterpret_cast<uint2 *>(reinterpret_cast<bf16 *>(p.out) + (long long)row * kD);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float4 a = __ldg(sh + lane + 32 * j), b = __ldg(sc + lane + 32 * j);
        const float4 &w = v[j];
        const float o0 = (w.x - mean) * inv * (1.0f + b.x) + a.x;
        const float o1 = (w.y - mean) * inv * (1.0f + b.y) + a.y;
        const float o2 = (w.z - mean) * inv * (1.0f + b.z) + a.z;
        const float o3 = (w.w - mean) * inv * (1.0f + b.w) + a.w;
        yr[lane + 32 * j] = make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
    }
}

// The same with an e4m3 output row, scaled by 448 / absmax before the
// conversion (v is overwritten).
DTTS_DEV void ln_row_out_f8(float4 (&v)[8], const LnParams &p, int row, int lane) {
    float mean, inv;
    ln_stats(v, mean, inv);
    const long long mr = row / p.tok_per_row;
    const float4 *sh = reinterpret_cast<const float4 *>(p.shift + mr * p.ada_ld);
    const float4 *sc = reinterpret_cast<const float4 *>(p.scale + mr * p.ada_ld);
    float amax = 0.f, ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float4 a = __ldg(sh + lane + 32 * j), b = __ldg(sc + lane + 32 * j);
        float4 &w = v[j];
        w.x = (w.x - mean) * inv * (1.0f + b.x) + a.x;
        w.y = (w.y - mean) * inv * (1.0f + b.y) + a.y;
        w.z = (w.z - mean) * inv * (1.0f + b.z) + a.z;
        w.w = (w.w - mean) * inv * (1.0f + b.w) + a.w;
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(w.x), fabsf(w.y)), fmaxf(fabsf(w.z), fabsf(w.w))));
        ss += (w.x * w.x + w.y * w.y) + (w.z * w.z + w.w * w.w);
    }
    amax = warp_max(amax);
    const float qinv = amax > 0.f ? 448.0f / amax : 0.f;
    uint32_t *yr = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(p.out) + (long long)row * kD);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float4 &w = v[j];
        yr[lane + 32 * j] = pack_e4m3x4(w.x * qinv, w.y * qinv, w.z * qinv, w.w * qinv);
    }
    const float nrm = sqrtf(warp_sum(ss));
    if (lane == 0) {
        p.row_scale[row] = amax / 448.0f;
        if (p.unorm) p.unorm[row] = 1.08f * nrm;
        if (p.g_scale) {
            const float bnd = 1.02f * fmaxf(1.08f * nrm * p.w1n + p.b1max, 0.17f);
            p.g_scale[row] = bnd / 448.0f;
            p.g_inv[row] = 448.0f / bnd;
        }
    }
}

// RW rows held in shared memory (rows_s[i * kD ..], i < n), rows row0 ..
// row0 + n - 1: the arithmetic of ln_row_out_*, value for value, but the rows'
// reductions are interleaved (one warp runs RW independent shuffle trees at
// once), which is what hides their latency when few warps do the work.
// st holds the modulation row of row0; rows of another modulation row read
// theirs from global memory one row at a time.  For e4m3 the modulated values
// are written back into rows_s between the two output passes.
template <int N>
DTTS_DEV void warp_sum_n(float (&v)[N]) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < N; i++) v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
}
template <int N>
DTTS_DEV void warp_max_n(float (&v)[N]) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = fmaxf(v[i], __shfl_xor_sync(0xffffffffu, v[i], o));
}

template <int RW, bool F8>
DTTS_DEV void ln_rows_smem(float *rows_s, int n, int row0, const LnParams &p, const ModRow &st, int lane) {
    // The loops over the 8 float4 columns of a lane stay rolled (this code runs
    // once per tile, cold in the instruction cache); the rows are unrolled
    // inside them, so the RW rows' dependency chains run side by side.
    const float4 *rs = reinterpret_cast<const float4 *>(rows_s) + lane;
    float mean[RW], inv[RW], t[RW];
#pragma unroll
    for (int r = 0; r < RW; r++) t[r] = 0.f;
#pragma unroll 1
    for (int j = 0; j < 8; j++)
#pragma unroll
        for (int r = 0; r < RW; r++) {
            const float4 w = rs[r * (kD / 4) + 32 * j];
            t[r] += (w.x + w.y) + (w.z + w.w);
        }
    warp_sum_n<RW>(t);
#pragma unroll
    for (int r = 0; r < RW; r++) { mean[r] = t[r] * (1.0f / kD); t[r] = 0.f; }
#pragma unroll 1
    for (int j = 0; j < 8; j++)
#pragma unroll
        for (int r = 0; r < RW; r++) {
            const float4 w = rs[r * (kD / 4) + 32 * j];
            const float e0 = w.x - mean[r], e1 = w.y - mean[r], e2 = w.z - mean[r], e3 = w.w - mean[r];
            t[r] += (e0 * e0 + e1 * e1) + (e2 * e2 + e3 * e3);
        }
    warp_sum_n<RW>(t);
#pragma unroll
    for (int r = 0; r < RW; r++) inv[r] = 1.0f / sqrtf(t[r] * (1.0f / kD) + 1e-5f);
    const bool shared_mod = st.mr == (long long)row0 / p.tok_per_row && st.mr == (long long)(row0 + n - 1) / p.tok_per_row;
    float amax[RW], ss[RW];
#pragma unroll
    for (int r = 0; r < RW; r++) { amax[r] = 0.f; ss[r] = 0.f; }
#pragma unroll 1
    for (int j = 0; j < 8; j++) {
        float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f), b4 = a4;
        if (shared_mod) {
            a4 = reinterpret_cast<const float4 *>(st.shift)[lane + 32 * j];
            b4 = reinterpret_cast<const float4 *>(st.scale)[lane + 32 * j];
        }
#pragma unroll
        for (int r = 0; r < RW; r++) {
            if (r >= n) continue;
            float4 a = a4, b = b4;
            if (!shared_mod) {
                const long long mr = (long long)(row0 + r) / p.tok_per_row;
                a = __ldg(reinterpret_cast<const float4 *>(p.shift + mr * p.ada_ld) + lane + 32 * j);
                b = __ldg(reinterpret_cast<const float4 *>(p.scale + mr * p.ada_ld) + lane + 32 * j);
            }
            float4 *wp = reinterpret_cast<float4 *>(rows_s) + lane + r * (kD / 4) + 32 * j;
            const float4 w = *wp;
            const float m = mean[r], iv = inv[r];
            const float o0 = (w.x - m) * iv * (1.0f + b.x) + a.x;
            const float o1 = (w.y - m) * iv * (1.0f + b.y) + a.y;
            const float o2 = (w.z - m) * iv * (1.0f + b.z) + a.z;
            const float o3 = (w.w - m) * iv * (1.0f + b.w) + a.w;
            if constexpr (F8) {
                *wp = make_float4(o0, o1, o2, o3);
                amax[r] = fmaxf(amax[r], fmaxf(fmaxf(fabsf(o0), fabsf(o1)), fmaxf(fabsf(o2), fabsf(o3))));
                ss[r] += (o0 * o0 + o1 * o1) + (o2 * o2 + o3 * o3);
            } else {
                uint2 *yr = reinterpret_cast<uint2 *>(reinterpret_cast<bf16 *>(p.out) + (long long)(row0 + r) * kD);
                yr[lane + 32 * j] = make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
            }
        }
    }
    if constexpr (F8) {
        warp_max_n<RW>(amax);
        warp_sum_n<RW>(ss);
        float qinv[RW];
#pragma unroll
        for (int r = 0; r < RW; r++) qinv[r] = amax[r] > 0.f ? 448.0f / amax[r] : 0.f;
#pragma unroll 1
        for (int j = 0; j < 8; j++)
#pragma unroll
            for (int r = 0; r < RW; r++) {
                if (r >= n) continue;
                const float4 w = rs[r * (kD / 4) + 32 * j];
                uint32_t *yr = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(p.out) + (long long)(row0 + r) * kD);
                yr[lane + 32 * j] = pack_e4m3x4(w.x * qinv[r], w.y * qinv[r], w.z * qinv[r], w.w * qinv[r]);
            }
        if (lane == 0)
#pragma unroll 1
            for (int r = 0; r < n; r++) {
                float am = 0.f, sq = 0.f;
#pragma unroll
                for (int i = 0; i < RW; i++)
                    if (i == r) { am = amax[i]; sq = ss[i]; }
                const int row = row0 + r;
                const float nrm = sqrtf(sq);
                p.row_scale[row] = am / 448.0f;
                if (p.unorm) p.unorm[row] = 1.08f * nrm;
                if (p.g_scale) {
                    const float bnd = 1.02f * fmaxf(1.08f * nrm * p.w1n + p.b1max, 0.17f);
                    p.g_scale[row] = bnd / 448.0f;
                    p.g_inv[row] = 448.0f / bnd;
                }
            }
    }
}

// R rows read from global memory (through L2), live[] uniform across the warp.
template <int R>
DTTS_DEV void ln_rows_bf16(const float *x, const LnParams &p, const int (&row)[R], const bool (&live)[R], int lane) {
    float4 v[R][8];
    ln_load_rows<R>(x, row, live, v, lane);
#pragma unroll
    for (int r = 0; r < R; r++)
        if (live[r]) ln_row_out_bf16(v[r], p, row[r], lane);
}

template <int R>
DTTS_DEV void ln_rows_f8(const float *x, const LnParams &p, const int (&row)[R], const bool (&live)[R], int lane) {
    float4 v[R][8];
    ln_load_rows<R>(x, row, live, v, lane);
#pragma unroll
    for (int r = 0; r < R; r++)
        if (live[r]) ln_row_out_f8(v[r], p, row[r], lane);
}

}  // namespace dtts
