//===- FusedKernels.h - fused kernels on B200 (sm_100a) ----------*- C++ -*-===//
//
// Drop-in replacement for the reference's kernel layer
// (AVmakeralt/jules include/jules/Kernel/FusedKernels.h).  Same namespace,
// names, argument order (note (M,K,N) vs (M,N,K)) and defaults; the
// functions are declared here and defined once in the jules_b200 library,
// so any number of translation units may include this header.
//
// float* arguments are HOST pointers, as in the reference: each call stages
// its operands to the current GPU, runs fp32-accurate CUDA kernels (the
// GEMMs of tiledMatmulWithActivation, the plain blasMatmul and
// fusedMLPForward on tensor cores as 3xTF32 when M and N are at least 256)
// and copies the result back before returning.  The device-pointer C ABI in
// jules_kernels.h is the fast path (bf16 tensor cores, no copies).
//
//===----------------------------------------------------------------------===//
#ifndef JULES_KERNEL_FUSED_KERNELS_H
#define JULES_KERNEL_FUSED_KERNELS_H

#include <cstddef>
#include <cstdint>

#include "jules/Kernel/ExecutionArena.h"
#include "jules/Kernel/TilePlanner.h"

namespace jules {
namespace kernel {

// FusedKernels.h:61-67
enum class ActivationType {
  None,
  Relu,
  Sigmoid,
  Tanh,
  Gelu,
};

// C = act(A.B); A [M,K], B [K,N].  FusedKernels.h:69-72, 378-458.
void tiledMatmulWithActivation(const float* A, const float* B, float* C, int M, int N, int K,
                               const TileConfig& cfg, ActivationType act = ActivationType::None);

// ReLU(X.W); argument order (M,K,N).  FusedKernels.h:203-259.
void fusedMatmulRelu(const float* X, const float* W, float* output, int M, int K, int N);

// ReLU(X.W + bias); argument order (M,K,N).  FusedKernels.h:265-372.
void fusedMatmulBiasRelu(const float* X, const float* W, const float* bias, float* output, int M,
                         int K, int N);

// GELU(X.W + bias); argument order (M,K,N).  The GELU counterpart the
// reference lacks (its routing pass has no GELU name, KernelRoutingPass.cpp:88-94).
void fusedMatmulBiasGelu(const float* X, const float* W, const float* bias, float* output, int M,
                         int K, int N);

// FusedKernels.h:532-600
void fusedLayerNorm(float* output, const float* input, const float* gamma, const float* beta,
                    int M, int N, float epsilon = 1e-5f);

// FusedKernels.h:606-627
void fusedGelu(float* output, const float* input, int N);

// Row softmax over [M, N].  FusedKernels.h:464-526.
void fusedSoftmax(float* output, const float* input, int M, int N);

// Softmax + cross-entropy: writes grad = (softmax - onehot(targets)) / M and
// returns the mean of -log(p[target] + 1e-10).  FusedKernels.h:766-854.
// A target outside [0, N) throws std::runtime_error (undefined in the
// reference).
float fusedCrossEntropyLoss(const float* logits, const int32_t* targets, float* grad, int M, int N);

class ExecutionArena;

// int8 GEMM with int32 accumulation: C = float(A . B) * scale_A * scale_B
// (+ bias per column).  FusedKernels.h:867-1073 (the arena held the int32
// accumulator there; here it is unused and may be null).
void matmulInt8(const int8_t* A, const int8_t* B, float* C, int M, int N, int K, float scale_A,
                float scale_B, const float* bias = nullptr, ExecutionArena* arena = nullptr);

// Row-major SGEMM, C = alpha op(A) op(B) + beta C.  FusedKernels.h:633-644.
void blasMatmul(const float* A, const float* B, float* C, int M, int N, int K, float alpha = 1.0f,
                float beta = 0.0f, bool transA = false, bool transB = false);

// FusedKernels.h:650-657
struct MLPParams {
  const float* W1;
  const float* b1;
  const float* W2;
  const float* b2;
  int batch_size;
  int in_features;
  int hidden_features;
  int out_features;
};

// X.W1 + b1 -> ReLU -> .W2 + b2.  FusedKernels.h:659-760.
void fusedMLPForward(float* output, const float* X, const MLPParams& params, ExecutionArena& arena,
                     TilePlanner& planner);

// FusedKernels.h:1085-1115 (same decision rule).
bool shouldUseFlashAttention(int seq_len, int head_dim, size_t l3_bytes);

}  // namespace kernel
}  // namespace jules

#endif
