/*
 * Minimal <cblas.h> for compiling the reference kernel headers as a test
 * oracle.  TEST INFRASTRUCTURE ONLY: nothing in the shipped library includes
 * this file.
 *
 * The reference calls exactly one BLAS routine, cblas_sgemm, row-major only
 * (include/jules/Kernel/FlashAttention.h:74,92,184;
 *  include/jules/Kernel/FusedKernels.h:230,348,637).  The enum values are the
 * standard CBLAS ones so the call can be forwarded unchanged to an ILP64
 * OpenBLAS (numpy's bundled scipy_openblas64).
 */
#ifndef JULES_ORACLE_CBLAS_SHIM_H
#define JULES_ORACLE_CBLAS_SHIM_H

#ifdef __cplusplus
extern "C" {
#endif

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta,
                 enum CBLAS_TRANSPOSE tb, int M, int N, int K, float alpha,
                 const float* A, int lda, const float* B, int ldb, float beta,
                 float* C, int ldc);

/* Route cblas_sgemm to an ILP64 cblas_sgemm (e.g. scipy_cblas_sgemm64_).
 * NULL restores the built-in loop. */
void oracle_set_sgemm64(void* fn);

#ifdef __cplusplus
}
#endif

#endif
