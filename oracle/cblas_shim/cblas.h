/*
 * Minimal CBLAS header used only to build the reference CPU library
 * (native/cpu/zilla_cpu.c, native/cpu/training_ops.c) with -DUSE_OPENBLAS.
 *
 * No system OpenBLAS is installed; numpy bundles OpenBLAS 0.3.30 as
 * libscipy_openblas64_*.so, whose CBLAS entry points carry a "scipy_"
 * prefix and a "64_" suffix and take 64-bit integer dimensions (ILP64).
 * This header declares the enum values of the CBLAS standard and maps
 * cblas_sgemm onto that symbol.  Test infrastructure only.
 */
#ifndef ZILLA_ORACLE_CBLAS_SHIM_H
#define ZILLA_ORACLE_CBLAS_SHIM_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

void scipy_cblas_sgemm64_(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta,
                          enum CBLAS_TRANSPOSE tb, int64_t m, int64_t n, int64_t k,
                          float alpha, const float *a, int64_t lda,
                          const float *b, int64_t ldb, float beta,
                          float *c, int64_t ldc);

static inline void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta,
                               enum CBLAS_TRANSPOSE tb, int m, int n, int k,
                               float alpha, const float *a, int lda,
                               const float *b, int ldb, float beta,
                               float *c, int ldc)
{
    scipy_cblas_sgemm64_(order, ta, tb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc);
}

#ifdef __cplusplus
}
#endif

#endif
