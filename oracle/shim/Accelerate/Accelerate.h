/* Stand-in for Apple's <Accelerate/Accelerate.h> when the speech-mac
 * reference is compiled on Linux for the oracle/_ref build.
 *
 * TEST INFRASTRUCTURE ONLY. The reference calls exactly one BLAS routine,
 * cblas_sgemm (src/phonon_transformer.c:305,352,390,513,557), with 32-bit int
 * sizes. This header forwards it to the ILP64 OpenBLAS 0.3.30 that ships
 * inside numpy (symbol scipy_cblas_sgemm64_, 64-bit integer arguments). The
 * enum values are the standard CBLAS ones. */
#ifndef ORACLE_ACCELERATE_SHIM_H
#define ORACLE_ACCELERATE_SHIM_H

#include <stdint.h>

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

void scipy_cblas_sgemm64_(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE transa,
                          enum CBLAS_TRANSPOSE transb, int64_t m, int64_t n, int64_t k, float alpha,
                          const float *a, int64_t lda, const float *b, int64_t ldb, float beta,
                          float *c, int64_t ldc);

static inline void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE transa,
                               enum CBLAS_TRANSPOSE transb, int m, int n, int k, float alpha,
                               const float *a, int lda, const float *b, int ldb, float beta,
                               float *c, int ldc) {
    scipy_cblas_sgemm64_(order, transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc);
}

#endif
