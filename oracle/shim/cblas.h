/* Stand-in for OpenBLAS's cblas.h, declaring only cblas_sgemm, which the
 * reference's manual_linear (include/dit_manual.h:30-61) calls with
 * RowMajor/NoTrans/Trans and M = 1.  The definition lives in cblas_shim.c:
 * a plain fp32 GEMM whose output columns are split across OpenMP threads,
 * standing in for a multi-threaded BLAS.  Test infrastructure only. */
#pragma once
#ifdef __cplusplus
extern "C" {
#endif
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                 int M, int N, int K, float alpha, const float *A, int lda,
                 const float *B, int ldb, float beta, float *C, int ldc);
#ifdef __cplusplus
}
#endif
