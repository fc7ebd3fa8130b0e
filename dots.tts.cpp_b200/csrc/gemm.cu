// Host side of the tcgen05 GEMM: tensor-map encoding and launch dispatch.
#include "kernels.cuh"

#include <cstdlib>
#include <mutex>

namespace dtts {

bool pdl_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("DTTS_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

template <int BN, int EPI, int NW, int F8 = 0>
cudaError_t launch_one(const GemmOp &op, int num_sms, cudaStream_t s) {
    using Cfg = GemmCfg<BN, NW, EPI, F8>;
    const int units = ((op.M + Cfg::BM - 1) / Cfg::BM) * (op.N / BN) * (op.ep.ksplit > 0 ? op.ep.ksplit : 1);
    const int grid = units < num_sms ? units : num_sms;
    unsigned flags = op.pdl && pdl_enabled() ? kLaunchPdl : 0u;
    // the CTAs of the fused LayerNorm wait on one another's arrivals, so they
    // must all be resident: a cooperative launch (without the programmatic overlap)
    if constexpr (EPI == EPI_RESID_GATED_LN) flags = kLaunchCoop;
    return launch_k(flags, gemm_tc_kernel<BN, EPI, NW, F8>, dim3(grid), dim3(Cfg::THREADS),
                    (size_t)Cfg::SMEM_BYTES, s, op.ta, op.tb, op.tr, op.M, op.N, op.K, op.ep);
}

// e4m3 operands: the three epilogues of the DiT block's FP8 path, and fp32 output
template <int BN, int NW>
cudaError_t dispatch_epi_f8(const GemmOp &op, int num_sms, cudaStream_t s) {
    switch (op.epi) {
        case EPI_QKV:
            return op.ep.rope_mode == ROPE_ADJACENT ? launch_one<BN, EPI_QKV_ADJ, NW, 1>(op, num_sms, s)
                                                    : launch_one<BN, EPI_QKV, NW, 1>(op, num_sms, s);
        case EPI_RESID_GATED: return launch_one<BN, EPI_RESID_GATED, NW, 1>(op, num_sms, s);
        case EPI_RESID_GATED_LN:
            if constexpr (BN % 128 == 0) return launch_one<BN, EPI_RESID_GATED_LN, NW, 1>(op, num_sms, s);
            return cudaErrorInvalidValue;
        case EPI_F32: return launch_one<BN, EPI_F32, NW, 1>(op, num_sms, s);
        case EPI_GELU_F8:
            if constexpr (BN % 128 == 0) return launch_one<BN, EPI_GELU_F8, NW, 1>(op, num_sms, s);
            return cudaErrorInvalidValue;
        default: return cudaErrorInvalidValue;
    }
}

template <int BN, int NW>
cudaError_t dispatch_epi(const GemmOp &op, int num_sms, cudaStream_t s) {
    switch (op.epi) {
        case EPI_BF16: return launch_one<BN, EPI_BF16, NW>(op, num_sms, s);
        case EPI_GELU_BF16: return launch_one<BN, EPI_GELU_BF16, NW>(op, num_sms, s);
        case EPI_SILU_BF16: return launch_one<BN, EPI_SILU_BF16, NW>(op, num_sms, s);
        case EPI_F32: return launch_one<BN, EPI_F32, NW>(op, num_sms, s);
        case EPI_RESID: return launch_one<BN, EPI_RESID, NW>(op, num_sms, s);
        case EPI_RESID_GATED: return launch_one<BN, EPI_RESID_GATED, NW>(op, num_sms, s);
        case EPI_RESID_GATED_LN:
            if constexpr (BN % 128 == 0) return launch_one<BN, EPI_RESID_GATED_LN, NW>(op, num_sms, s);
            return cudaErrorInvalidValue;
        case EPI_QKV:
            return op.ep.rope_mode == ROPE_ADJACENT ? launch_one<BN, EPI_QKV_ADJ, NW>(op, num_sms, s)
                                                    : launch_one<BN, EPI_QKV, NW>(op, num_sms, s);
        default: return cudaErrorInvalidValue;
    }
}

template <int BN, int NW, int EPI, int F8 = 0>
cudaError_t prepare_one() {
    return cudaFuncSetAttribute((const void *)gemm_tc_kernel<BN, EPI, NW, F8>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN, NW, EPI, F8>::SMEM_BYTES);
}

template <int BN, int NW>
cudaError_t prepare_bn_f8() {
    cudaError_t e;
    if ((e = prepare_one<BN, NW, EPI_QKV, 1>()) != cudaSuccess) return e;
    if ((e = prepare_one<BN, NW, EPI_QKV_ADJ, 1>()) != cudaSuccess) return e;
    if ((e = prepare_one<BN, NW, EPI_F32, 1>()) != cudaSuccess) return e;
    if constexpr (BN % 128 == 0) {
        if ((e = prepare_one<BN, NW, EPI_GELU_F8, 1>()) != cudaSuccess) return e;
        if ((e = prepare_one<BN, NW, EPI_RESID_GATED_LN, 1>()) != cudaSuccess) return e;
    }
    return prepare_one<BN, NW, EPI_RESID_GATED, 1>();
}

template <int BN, int NW>
cudaError_t prepare_bn() {
    cudaError_t e;
    if ((e = prepare_one<BN, NW, EPI_BF16>()) != cudaSuccess) return e;
    if ((e = prepare_one<BN, NW, EPI_GELU_BF16>()) != cudaSuccess) return e;
    if ((e = prepare_one<BN, NW, EPI_SILU_BF16>()) != cudaSuccess) return e;
    if ((e = prepare_one<BN, NW, EPI_F32>()) != cudaSuccess) return e;
    if ((e = prepare_one<BN, NW, EPI_RESID>()) != cudaSuccess) return e;
    if ((e = prepare_one<BN, NW, EPI_RESID_GATED>()) != cudaSuccess) return e;
    if constexpr (BN % 128 == 0)
        if ((e = prepare_one<BN, NW, EPI_RESID_GATED_LN>()) != cudaSuccess) return e;
    if ((e = prepare_one<BN, NW, EPI_QKV>()) != cudaSuccess) return e;
    return prepare_one<BN, NW, EPI_QKV_ADJ>();
}

}  // namespace

// Opts every GEMM instantiation into its dynamic shared-memory size on the
// current device (attributes are per device; called when an engine is created).
cudaError_t gemm_prepare_attributes() {
    cudaError_t e;
    if ((e = prepare_bn<64, 4>()) != cudaSuccess) return e;
    if ((e = prepare_bn<128, 4>()) != cudaSuccess) return e;
    if ((e = prepare_bn<192, 4>()) != cudaSuccess) return e;
    if ((e = prepare_bn<256, 4>()) != cudaSuccess) return e;
    if ((e = prepare_bn<128, 8>()) != cudaSuccess) return e;
    if ((e = prepare_bn<192, 8>()) != cudaSuccess) return e;
    if ((e = prepare_bn<256, 8>()) != cudaSuccess) return e;
    if ((e = prepare_bn_f8<128, 4>()) != cudaSuccess) return e;
    if ((e = prepare_bn_f8<192, 4>()) != cudaSuccess) return e;
    if ((e = prepare_bn_f8<256, 4>()) != cudaSuccess) return e;
    if ((e = prepare_bn_f8<128, 8>()) != cudaSuccess) return e;
    if ((e = prepare_bn_f8<192, 8>()) != cudaSuccess) return e;
    return prepare_bn_f8<256, 8>();
}

bool make_tmap_e4m3(CUtensorMap *m, const void *base, unsigned long long rows, unsigned long long cols,
                    unsigned int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || !base || rows == 0 || cols % 128 != 0 || box_rows == 0 || box_rows > 256) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols};      // bytes between rows
    cuuint32_t box[2] = {128, box_rows}; // 128 e4m3 = 128 bytes: one swizzle atom row
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tmap_f32_resid(CUtensorMap *m, const void *base, unsigned long long rows, unsigned long long cols) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || !base || rows == 0 || cols % 32 != 0) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 4};
    cuuint32_t box[2] = {32, 32};        // 32 fp32 = 128 bytes per row, 32 rows: one warp's staging tile
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tmap_bf16(CUtensorMap *m, const void *base, unsigned long long rows, unsigned long long cols,
                    unsigned int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || !base || rows == 0 || cols % 64 != 0 || box_rows == 0 || box_rows > 256) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};  // bytes between rows
    cuuint32_t box[2] = {64, box_rows};  // 64 bf16 = 128 bytes: one swizzle atom row
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

cudaError_t launch_gemm(const GemmOp &op, int num_sms, cudaStream_t s) {
    const int ks = op.ep.ksplit > 0 ? op.ep.ksplit : 1;
    const int bk = op.f8 ? 128 : 64;
    if (op.M < 1 || op.K < bk * ks || op.K % (bk * ks) != 0 || op.N % op.bn != 0) return cudaErrorInvalidValue;
    if (ks > 1 && !is_resid(op.epi)) return cudaErrorInvalidValue;
    if (op.epi == EPI_RESID_GATED_LN) {
        // whole kD-wide rows, one arrival per warp of each tile, rows split evenly
        const int num_n = op.N / op.bn;
        if (op.N != kD || op.ep.ldr != kD || ks != 1 || op.bn % 128 != 0 || 128 % num_n != 0 || num_n > num_sms ||
            !op.ep.ln_count || !op.ep.err || !op.ep.ln.out || !op.ep.ln.shift || !op.ep.ln.scale || op.ep.ln.tok_per_row < 1 ||
            (op.f8 && !op.ep.ln.row_scale))
            return cudaErrorInvalidValue;
    }
    const int nw = op.nw == 8 ? 8 : 4;
    if (op.f8) {
        if (!op.ep.row_scale || !op.ep.col_scale) return cudaErrorInvalidValue;
        if (op.epi == EPI_GELU_F8 && (!op.ep.out_inv || op.bn % 128 != 0)) return cudaErrorInvalidValue;
        switch (op.bn * 16 + nw) {
            case 128 * 16 + 4: return dispatch_epi_f8<128, 4>(op, num_sms, s);
            case 192 * 16 + 4: return dispatch_epi_f8<192, 4>(op, num_sms, s);
            case 256 * 16 + 4: return dispatch_epi_f8<256, 4>(op, num_sms, s);
            case 128 * 16 + 8: return dispatch_epi_f8<128, 8>(op, num_sms, s);
            case 192 * 16 + 8: return dispatch_epi_f8<192, 8>(op, num_sms, s);
            case 256 * 16 + 8: return dispatch_epi_f8<256, 8>(op, num_sms, s);
            default: return cudaErrorInvalidValue;
        }
    }
    if (op.epi == EPI_GELU_F8) return cudaErrorInvalidValue;
    switch (op.bn * 16 + nw) {
        case 64 * 16 + 4: return dispatch_epi<64, 4>(op, num_sms, s);
        case 128 * 16 + 4: return dispatch_epi<128, 4>(op, num_sms, s);
        case 192 * 16 + 4: return dispatch_epi<192, 4>(op, num_sms, s);
        case 256 * 16 + 4: return dispatch_epi<256, 4>(op, num_sms, s);
        case 128 * 16 + 8: return dispatch_epi<128, 8>(op, num_sms, s);
        case 192 * 16 + 8: return dispatch_epi<192, 8>(op, num_sms, s);
        case 256 * 16 + 8: return dispatch_epi<256, 8>(op, num_sms, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace dtts
