/*
 * cblas_sgemm for the reference oracle build.  TEST INFRASTRUCTURE ONLY.
 *
 * Two back ends:
 *  - forwarding to an ILP64 OpenBLAS cblas_sgemm (numpy ships one as
 *    scipy_cblas_sgemm64_), installed at run time by oracle_set_sgemm64();
 *    this is what the CPU baseline times, standing in for the MKL the
 *    reference author used (benchmarks/bench_comparison.py:21,125);
 *  - a plain loop with double accumulation (the default), used when no
 *    OpenBLAS is available.
 * Only row-major is needed: every reference call site passes CblasRowMajor.
 */
#include "cblas.h"

#include <stddef.h>
#include <stdint.h>

typedef void (*sgemm64_fn)(int order, int ta, int tb, int64_t M, int64_t N,
                           int64_t K, float alpha, const float* A, int64_t lda,
                           const float* B, int64_t ldb, float beta, float* C,
                           int64_t ldc);

static sgemm64_fn g_sgemm64 = NULL;

void oracle_set_sgemm64(void* fn) { g_sgemm64 = (sgemm64_fn)fn; }

void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta,
                 enum CBLAS_TRANSPOSE tb, int M, int N, int K, float alpha,
                 const float* A, int lda, const float* B, int ldb, float beta,
                 float* C, int ldc) {
  if (g_sgemm64) {
    g_sgemm64((int)order, (int)ta, (int)tb, M, N, K, alpha, A, lda, B, ldb,
              beta, C, ldc);
    return;
  }
  /* Row-major loop: C[i,j] = alpha * sum_k op(A)[i,k] op(B)[k,j] + beta C. */
  for (int i = 0; i < M; i++) {
    for (int j = 0; j < N; j++) {
      double acc = 0.0;
      for (int k = 0; k < K; k++) {
        float a = (ta == CblasNoTrans) ? A[(size_t)i * lda + k]
                                       : A[(size_t)k * lda + i];
        float b = (tb == CblasNoTrans) ? B[(size_t)k * ldb + j]
                                       : B[(size_t)j * ldb + k];
        acc += (double)a * (double)b;
      }
      float prev = (beta == 0.0f) ? 0.0f : beta * C[(size_t)i * ldc + j];
      C[(size_t)i * ldc + j] = (float)(alpha * acc) + prev;
    }
  }
  (void)order;
}
