// Host side of the tcgen05 GEMM: tensor-map encoding and launch dispatch.
#include "kernels.cuh"
#include <mutex>

namespace dtts {

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

template <int BN, int EPI>
cudaError_t launch_one(const GemmOp &op, int num_sms, cudaStream_t s) {
    using Cfg = GemmCfg<BN>;
    const int tiles = ((op.M + Cfg::BM - 1) / Cfg::BM) * (op.N / BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    gemm_tc_kernel<BN, EPI><<<grid, 192, Cfg::SMEM_BYTES, s>>>(op.ta, op.tb, op.M, op.N, op.K, op.ep);
    return cudaGetLastError();
}

template <int BN>
cudaError_t dispatch_epi(const GemmOp &op, int num_sms, cudaStream_t s) {
    switch (op.epi) {
        case EPI_BF16: return launch_one<BN, EPI_BF16>(op, num_sms, s);
        case EPI_GELU_BF16: return launch_one<BN, EPI_GELU_BF16>(op, num_sms, s);
        case EPI_SILU_BF16: return launch_one<BN, EPI_SILU_BF16>(op, num_sms, s);
        case EPI_F32: return launch_one<BN, EPI_F32>(op, num_sms, s);
        case EPI_RESID: return launch_one<BN, EPI_RESID>(op, num_sms, s);
        case EPI_RESID_GATED: return launch_one<BN, EPI_RESID_GATED>(op, num_sms, s);
        case EPI_QKV: return launch_one<BN, EPI_QKV>(op, num_sms, s);
        default: return cudaErrorInvalidValue;
    }
}

template <int BN>
cudaError_t prepare_bn() {
    using Cfg = GemmCfg<BN>;
    const void *fns[] = {
        (const void *)gemm_tc_kernel<BN, EPI_BF16>,        (const void *)gemm_tc_kernel<BN, EPI_GELU_BF16>,
        (const void *)gemm_tc_kernel<BN, EPI_SILU_BF16>,   (const void *)gemm_tc_kernel<BN, EPI_F32>,
        (const void *)gemm_tc_kernel<BN, EPI_RESID>,       (const void *)gemm_tc_kernel<BN, EPI_RESID_GATED>,
        (const void *)gemm_tc_kernel<BN, EPI_QKV>,
    };
    for (const void *f : fns) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace

// Opts every GEMM instantiation into its dynamic shared-memory size on the
// current device (attributes are per device; called when an engine is created).
cudaError_t gemm_prepare_attributes() {
    cudaError_t e = prepare_bn<128>();
    if (e != cudaSuccess) return e;
    return prepare_bn<256>();
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
    if (op.M < 1 || op.K % 64 != 0 || op.K < 64 || op.N % op.bn != 0) return cudaErrorInvalidValue;
    if (op.epi == EPI_QKV && op.N % 64 != 0) return cudaErrorInvalidValue;
    switch (op.bn) {
        case 128: return dispatch_epi<128>(op, num_sms, s);
        case 256: return dispatch_epi<256>(op, num_sms, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace dtts
