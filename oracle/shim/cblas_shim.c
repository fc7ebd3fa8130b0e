/* fp32 sgemm for the reference build (see cblas.h in this folder).
 * C = alpha * op(A) * op(B) + beta * C, row-major only.  Every output element
 * is one dot product accumulated in k order, so results do not depend on the
 * thread count. */
#include "cblas.h"
#include <stdlib.h>

void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                 int M, int N, int K, float alpha, const float *A, int lda,
                 const float *B, int ldb, float beta, float *C, int ldc) {
    if (order != CblasRowMajor) abort();
    long long work = (long long)M * N * K;
    #pragma omp parallel for collapse(2) schedule(static) if (work > 65536)
    for (int m = 0; m < M; m++) {
        for (int n = 0; n < N; n++) {
            float s = 0.0f;
            for (int k = 0; k < K; k++) {
                float a = (ta == CblasNoTrans) ? A[(long long)m * lda + k] : A[(long long)k * lda + m];
                float b = (tb == CblasNoTrans) ? B[(long long)k * ldb + n] : B[(long long)n * ldb + k];
                s += a * b;
            }
            float c = (beta == 0.0f) ? 0.0f : beta * C[(long long)m * ldc + n];
            C[(long long)m * ldc + n] = alpha * s + c;
        }
    }
}
