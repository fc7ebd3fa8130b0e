// Launchers for the non-GEMM kernels of the DiT / PatchEncoder engines.
#pragma once
#include "common.cuh"
#include "gemm_tc.cuh"

namespace dtts {

// ------------------------------------------------------------ GEMM (tcgen05)
struct GemmOp {
    CUtensorMap ta, tb;
    CUtensorMap tr;   // residual (EPI_RESID*), from make_tmap_f32_resid
    int M, N, K;
    int bn;       // 128, 192 or 256 (64 with 4 epilogue warps)
    int nw;       // epilogue warps: 4 or 8
    int epi;      // EpiKind
    int f8;       // 1: A and B are e4m3 (tensor maps from make_tmap_e4m3)
    int pdl;      // 1: programmatic launch after the previous kernel (its weight tiles load early)
    EpiParams ep;
};
// Programmatic dependent launches on (the default) unless DTTS_PDL=0.
bool pdl_enabled();
// A K-major bf16 matrix [rows][cols] seen by TMA as 64-column x box_rows boxes
// with 128-byte swizzle.
bool make_tmap_bf16(CUtensorMap *m, const void *base, unsigned long long rows, unsigned long long cols,
                    unsigned int box_rows);
// A K-major e4m3 matrix [rows][cols] (one byte per element) seen by TMA as
// 128-column x box_rows boxes with 128-byte swizzle.
bool make_tmap_e4m3(CUtensorMap *m, const void *base, unsigned long long rows, unsigned long long cols,
                    unsigned int box_rows);
// The fp32 residual [rows][cols] as the target of the epilogue's bulk reduce-add.
bool make_tmap_f32_resid(CUtensorMap *m, const void *base, unsigned long long rows, unsigned long long cols);
cudaError_t launch_gemm(const GemmOp &op, int num_sms, cudaStream_t s);
cudaError_t gemm_prepare_attributes();

// ------------------------------------------------------------ norms
// y = bf16( LN(x) * (1 + scale[row]) + shift[row] ), LN without affine, eps 1e-5.
LnParams ln_params(const float *shift, const float *scale, long long ada_ld, int tok_per_row, void *out);
void launch_ln_modulate(const float *x, bf16 *y, int M, const float *shift, const float *scale,
                        long long ada_ld, int tok_per_row, cudaStream_t s, bool pdl = false);
// y = bf16( x / sqrt(mean(x^2) + 1e-6) * w )
void launch_rms_norm(const float *x, bf16 *y, int M, const float *w, cudaStream_t s, bool pdl = false);

// ------------------------------------------------------------ attention
struct AttnArgs {
    const void *q; long long ldq;          // row (r, i) = r*Tq + i
    const void *k; const void *v; long long ldkv;  // row (r, j) = r*kv_cap + j
    void *o; long long ldo;                // row (r, i) = r*Tq + i
    int rows, Tq, kv_len, kv_cap;
    int q_pos0;          // absolute position of query 0 (causal masking)
    int causal;
    const uint8_t *mask; // [Tq][kv_len] (1 = attend) or nullptr (fp32 kernel)
    const uint32_t *mask_bits;  // the same mask bit-packed, [Tq][ceil(kv_len/32)] words,
                                // bit k of word w = key 32w + k (bf16 kernels); nullptr: none
    float scale;
    // e4m3 output (DiT FP8 path), used instead of `o` when o8 is set:
    // o8[(r*Tq + i) * ldo + c] = e4m3(out * 448 / B_r) with the bound
    // B_r = 1.02 * max_{j < kv_len} unorm[r*kv_cap + j] * vbound on |out|
    // (softmax . V is a convex mix of V rows, |V_j,d| <= |u_j| |Wv_d|), and the
    // head-0 pass writes o_scale[r*Tq + i] = B_r / 448
    uint8_t *o8;
    float *o_scale;
    const float *unorm;
    float vbound;
    // if set (tiled kernel only): the cache length before this call is read
    // from device memory, q_pos0 = *kv_base_dev and kv_len = *kv_base_dev + Tq
    const int *kv_base_dev;
    // the q / k / v rows are dead after this call (the DiT forward's own
    // workspace): the tcgen05 L = 64 kernel drops their L2 lines once it has
    // loaded them, so they are never written back to DRAM
    int discard_qkv;
    int *err;            // device error word for bounded-wait expiry (tensor-core kernel), or nullptr
};
// Tq <= 64 and kv_len <= 64 take the pipelined short-sequence kernel (call
// attention_short_prepare() once per device first); longer ones the tiled kernel.
void launch_attention_bf16(const AttnArgs &a, cudaStream_t s, bool pdl = false);
// L = 64 on the tensor cores (attn_tc.cu): two sequences x one head per 128-row
// tile; used by launch_attention_bf16 when eligible (Tq = kv_len = kv_cap = 64,
// not causal, bf16 out, dense [rows * 64][1024] q/k/v; DTTS_ATTN_TC=0 turns it off).
bool attention_tc_eligible(const AttnArgs &a);
cudaError_t launch_attention_tc(const AttnArgs &a, int *err, cudaStream_t s, bool pdl);
// Bidirectional (optionally masked) attention for 64 < L <= 256 on the tensor
// cores (attn_tc.cu): 128-query tiles against the whole key range in TMEM; used by
// launch_attention_bf16 when eligible (Tq = kv_len = kv_cap, not causal, dense
// [rows * L][1024] q/k/v, bf16 or e4m3 out).
bool attention_tc_long_eligible(const AttnArgs &a);
cudaError_t launch_attention_tc_long(const AttnArgs &a, int *err, cudaStream_t s, bool pdl);
// Causal attention of a prefill (Tq > 64) over the KV cache on the tensor cores:
// 128-query tiles, 128-key blocks with an online softmax (attn_tc.cu).
bool attention_tc_causal_eligible(const AttnArgs &a);
cudaError_t launch_attention_tc_causal(const AttnArgs &a, int *err, cudaStream_t s, bool pdl);
cudaError_t attention_tc_prepare();
// *len += add on the device (KV length of a graph-captured decode step)
void launch_advance_len(int *len, int add, cudaStream_t s, bool pdl = false);
cudaError_t attention_short_prepare();
// Host helper: bit-packs a [Tq][kv_len] uint8 mask into [Tq][ceil(kv_len/32)] words.
void pack_mask_bits(const uint8_t *mask, int Tq, int kv_len, uint32_t *bits);
cudaError_t launch_attention_f32(const AttnArgs &a, cudaStream_t s);  // kv_len <= 400
cudaError_t attention_f32_prepare();  // per device, before the first fp32 launch

// ------------------------------------------------------------ fp32 SIMT path
// C[M][N] = A[M][K] * B[N][K]^T + bias (fp32 everywhere).
void launch_gemm_f32(const float *A, const float *B, const float *bias, float *C, int M, int N, int K,
                     cudaStream_t s);
// In-place per-head RMS norm (optional) + RoPE on q and k, fp32 [M][1024].
void launch_qk_norm_rope_f32(float *q, float *k, int M, int tok_per_row, int qk_norm, const float *qn,
                             const float *kn, const float2 *rope, int rope_mode, int pos_start,
                             cudaStream_t s);

// ------------------------------------------------------------ conversions
void launch_f32_to_bf16(const float *x, bf16 *y, long long n, cudaStream_t s);
// SiLU(x) -> bf16 (the A operand of the adaLN GEMM)
void launch_silu_bf16(const float *x, bf16 *y, long long n, cudaStream_t s);
// c = a + b (fp32, n elements)
void launch_add_f32(const float *a, const float *b, float *c, long long n, cudaStream_t s);
// Copy rows of a [n_seq][src_len][1024] fp32 tensor into tokens 0..src_len-1 of
// sequence rows (row_stride*u + row_off) of a [rows][L][1024] bf16 buffer.
void launch_history_rows(const float *src, int n_seq, int src_len, bf16 *dst, int L, int row_stride, int row_off,
                         cudaStream_t s);

// ------------------------------------------------------------ conditioning
// temb[k] = W2 SiLU(W1 se[k] + b1) + b2 for n sinusoids se[k] (256 entries,
// computed on the host); h1_scratch holds n x 1024.
void launch_time_mlp(const float *se, int n, const float *w1, const float *b1, const float *w2, const float *b2,
                     float *h1_scratch, float *temb, cudaStream_t s);
// spk_c[u] = scale * LN_affine(Wx spk[u] + bx), eps 1e-5
void launch_speaker_cond(const float *spk, int n_utt, const float *w, const float *b, const float *ln_w,
                         const float *ln_b, float scale, float *spk_c, cudaStream_t s);
// a_cond[k*n + u] = bf16(SiLU(temb[k] + spk_c[u])) for k < n_t, u < n  (spk_c may be null)
void launch_cond_rows(const float *temb, int n_t, const float *spk_c, int n, bf16 *a_cond, cudaStream_t s);

// LayerNorm + modulation to e4m3 rows (DiT FP8 path), see ln_rows.cuh.
void launch_ln_modulate_f8(const float *x, uint8_t *y, int M, const float *shift, const float *scale,
                           long long ada_ld, int tok_per_row, float *row_scale, float *unorm, float *g_scale,
                           float *g_inv, float w1n, float b1max, cudaStream_t s, bool pdl = false);
void launch_e4m3_selftest(const float *x, uint8_t *y, int n, cudaStream_t s);

// ------------------------------------------------------------ FM history
void launch_fm_place_rows(const float *src, float *dst, int n_utt, int P, int cap, int start, int broadcast,
                          cudaStream_t s);
void launch_eos_act(float *h1, int n, int as_written, cudaStream_t s);   // h1 [n][1536] in place
void launch_eos_prob(const float *logits, int n, float *prob, cudaStream_t s);

// ------------------------------------------------------------ DiT output head
// vel[r][p] = W_out (LN(h[r, L-P+p]) (1 + scale) + shift) + b_out, with the
// modulation of row r at shift/scale + (r / rows_per_ada) * ada_ld; w_out_t is
// W_out transposed, [1024][128]
void launch_out_head(const float *h, int rows, int L, int P, const float *shift, const float *scale,
                     long long ada_ld, int rows_per_ada, const float *w_out_t, const float *b_out, float *vel, int *err,
                     cudaStream_t s);
// CFG combine + Euler update + coord_proj of the new z into the noise tokens of
// both rows of each utterance (update = 0: only the coord_proj of z); w_coord_t
// is coordinate_proj's weight transposed, [128][1024]
void launch_cfg_euler(const float *vel, float *z, int n_utt, int P, float cfg_scale, int cfg_form, float dt,
                      int update, const float *w_coord_t, const float *b_coord, bf16 *x_in, int L,
                      cudaStream_t s);

// ------------------------------------------------------------ PatchEncoder
// causal Conv1d(128->128, k=2, s=2); tokens t of sequence b use frames 2t-1, 2t
// of the concatenation [tail[b] | frames[b]]; writes bf16 [B*T][128] and, if
// new_tail != nullptr, stores the last frame of each sequence there.  wt is the
// conv weight transposed to [in 128][tap 2][out 128].
void launch_pe_conv(const float *frames, int B, int n_frames, const float *tail, const float *wt, const float *bias,
                    bf16 *out, float *new_tail, cudaStream_t s);
// out[b*n + p] = bf16([h[b, tok0] | h[b, tok1]]) with the pairing rule
void launch_pe_pairs(const float *h, int B, int T, int pair_mode, bf16 *out, cudaStream_t s, bool pdl = false);

}  // namespace dtts
