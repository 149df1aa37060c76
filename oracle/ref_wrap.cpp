// extern "C" wrappers around the reference's own CPU kernels, compiled
// straight from the reference sources (include/jules/Kernel/*.h) by
// oracle/Makefile into oracle/_ref/.  TEST INFRASTRUCTURE ONLY: this is the
// checker and the timed CPU baseline, never the product path.
//
// The reference headers define non-inline functions, so this must stay the
// only translation unit that includes them (ODR, FusedKernels.h:203).
#include "jules/Kernel/FlashAttention.h"  // pulls FusedKernels.h, TilePlanner.h, ExecutionArena.h
#include "jules/Kernel/InterleavedAutodiff.h"

#include <cstdlib>
#ifdef _OPENMP
#include <omp.h>
#endif

using namespace jules::kernel;

namespace {

ExecutionArena& arena() {
  // flashAttention never allocates from the arena; fusedMLPForward's small
  // branch (FusedKernels.h:669-700) does, sized M*N1 floats.
  static ExecutionArena a(64UL * 1024 * 1024);
  return a;
}

TilePlanner& planner() {
  // Autotune is disabled: TilePlanner::autoTune (TilePlanner.h:158-236) times
  // ~40 candidates x 11 full GEMMs, which is minutes at the config sizes.
  // The analytical choice (TilePlanner.h:97-136) is what remains.
  static TilePlanner p = [] {
    TilePlanner t;
    t.setAutoTune(false);
    return t;
  }();
  return p;
}

}  // namespace

extern "C" {

// OpenMP threads for the reference kernels (launchers such as torchrun set
// OMP_NUM_THREADS=1).
void ref_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#endif
}

int ref_has_avx512(void) {
#if defined(__AVX512F__)
  return 1;
#else
  return 0;
#endif
}

void ref_cache_info(size_t* out4) {
  const CacheInfo& c = planner().cacheInfo();
  out4[0] = c.l1d_bytes;
  out4[1] = c.l2_bytes;
  out4[2] = c.l3_bytes;
  out4[3] = (size_t)c.num_cores;
}

// FlashAttention.h:130-309
void ref_flash_attention(float* out, const float* Q, const float* K,
                         const float* V, int B, int H, int S, int D) {
  flashAttention(out, Q, K, V, B, H, S, D, arena(), planner());
}

// FlashAttention.h:52-100
void ref_standard_attention(float* out, const float* Q, const float* K,
                            const float* V, int B, int H, int S, int D) {
  standardAttention(out, Q, K, V, B, H, S, D, arena());
}

// FlashAttention.h:114-124
void ref_attention(float* out, const float* Q, const float* K, const float* V,
                   int B, int H, int S, int D) {
  attention(out, Q, K, V, B, H, S, D, arena(), planner());
}

// FusedKernels.h:1085-1115
int ref_should_use_flash(int S, int D, size_t l3) {
  return shouldUseFlashAttention(S, D, l3) ? 1 : 0;
}

// TilePlanner.h:97-136
void ref_tile_config(int M, int N, int K, int* out3) {
  TileConfig c = planner().computeAnalytical(M, N, K);
  out3[0] = c.tile_m;
  out3[1] = c.tile_n;
  out3[2] = c.tile_k;
}

// FusedKernels.h:378-458.  act follows ActivationType (FusedKernels.h:61-67).
void ref_tiled_matmul_act(const float* A, const float* B, float* C, int M,
                          int N, int K, int tm, int tn, int tk, int act) {
  TileConfig cfg{tm, tn, tk};
  tiledMatmulWithActivation(A, B, C, M, N, K, cfg, (ActivationType)act);
}

// FusedKernels.h:203-259 (argument order M, K, N as in the reference)
void ref_fused_matmul_relu(const float* X, const float* W, float* out, int M,
                           int K, int N) {
  fusedMatmulRelu(X, W, out, M, K, N);
}

// FusedKernels.h:265-372 (argument order M, K, N)
void ref_fused_matmul_bias_relu(const float* X, const float* W,
                                const float* bias, float* out, int M, int K,
                                int N) {
  fusedMatmulBiasRelu(X, W, bias, out, M, K, N);
}

// FusedKernels.h:532-600
void ref_fused_layernorm(float* out, const float* in, const float* gamma,
                         const float* beta, int M, int N, float eps) {
  fusedLayerNorm(out, in, gamma, beta, M, N, eps);
}

// FusedKernels.h:606-627
void ref_fused_gelu(float* out, const float* in, int N) {
  fusedGelu(out, in, N);
}

// FusedKernels.h:464-526
void ref_fused_softmax(float* out, const float* in, int M, int N) {
  fusedSoftmax(out, in, M, N);
}

// InterleavedAutodiff.h:55-160: 2-layer ReLU MLP forward, softmax
// cross-entropy, backward; returns the mean loss.
float ref_interleaved_mlp(const float* X, const float* W1, const float* b1, const float* W2,
                          const float* b2, const int32_t* targets, float* output, float* dW1,
                          float* db1, float* dW2, float* db2, float* dX, int M, int K1, int N1,
                          int N2) {
  return interleavedMLPForwardBackward(X, W1, b1, W2, b2, targets, output, dW1, db1, dW2, db2, dX,
                                       M, K1, N1, N2, arena(), planner())
      .loss;
}

// FusedKernels.h:867-1073.  Only the build without AVX-512 (the scalar
// branch) computes the documented product; see orc_matmul_int8.
void ref_matmul_int8(const int8_t* A, const int8_t* B, float* C, int M, int N, int K,
                     float scale_a, float scale_b, const float* bias) {
  matmulInt8(A, B, C, M, N, K, scale_a, scale_b, bias, nullptr);
}

// FusedKernels.h:766-854
float ref_fused_cross_entropy(const float* logits, const int32_t* targets, float* grad, int M,
                              int N) {
  return fusedCrossEntropyLoss(logits, targets, grad, M, N);
}

// FusedKernels.h:633-644
void ref_blas_matmul(const float* A, const float* B, float* C, int M, int N,
                     int K, float alpha, float beta, int transA, int transB) {
  blasMatmul(A, B, C, M, N, K, alpha, beta, transA != 0, transB != 0);
}

// FusedKernels.h:650-760
void ref_fused_mlp_forward(float* out, const float* X, const float* W1,
                           const float* b1, const float* W2, const float* b2,
                           int M, int K1, int N1, int N2) {
  MLPParams p{W1, b1, W2, b2, M, K1, N1, N2};
  fusedMLPForward(out, X, p, arena(), planner());
}

}  // extern "C"
