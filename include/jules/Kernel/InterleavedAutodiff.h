// jules_b200 replacement of the reference's jules::kernel interleaved MLP
// forward + backward (AVmakeralt/jules include/jules/Kernel/InterleavedAutodiff.h).
// Same namespace, types and signature; declared here, defined once in
// libjules_b200.so.  Host float* buffers are staged to the current GPU and
// the step runs there in fp32 (jules_mlp_fwd_bwd in jules_kernels.h).
#pragma once

#include <cstdint>

#include "jules/Kernel/ExecutionArena.h"
#include "jules/Kernel/FusedKernels.h"
#include "jules/Kernel/TilePlanner.h"

namespace jules {
namespace kernel {

// InterleavedAutodiff.h:42-48
struct MLPGradients {
  float* dW1;
  float* db1;
  float* dW2;
  float* db2;
  float* dX;
};

// InterleavedAutodiff.h:50-53
struct InterleavedMLPResult {
  float loss;
  MLPGradients grads;
};

// 2-layer ReLU MLP, softmax cross-entropy loss, gradients.
// InterleavedAutodiff.h:55-160.  dX may be null.  Failures throw
// std::runtime_error.
InterleavedMLPResult interleavedMLPForwardBackward(const float* X, const float* W1,
                                                   const float* b1, const float* W2,
                                                   const float* b2, const int32_t* targets,
                                                   float* output, float* dW1, float* db1,
                                                   float* dW2, float* db2, float* dX, int M,
                                                   int K1, int N1, int N2, ExecutionArena& arena,
                                                   TilePlanner& planner);

}  // namespace kernel
}  // namespace jules
