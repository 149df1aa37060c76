// Elementwise and reduction steps of the 2-layer MLP training step
// (jules_mlp_fwd_bwd; the reference's interleavedMLPForwardBackward,
// InterleavedAutodiff.h:55-160).  The matmuls run on jules_sgemm and the loss
// on the fused softmax + cross-entropy kernel; these kernels are the glue.
#pragma once

#include <cstdint>

namespace jb {
namespace train {

// x[i, j] = max(x[i, j] + b[j], 0)
__global__ void bias_relu_kernel(float* __restrict__ x, const float* __restrict__ b, int64_t M,
                                 int64_t N) {
  const int64_t n = M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    x[i] = fmaxf(x[i] + b[i % N], 0.0f);
}

// x[i, j] += b[j]
__global__ void bias_add_kernel(float* __restrict__ x, const float* __restrict__ b, int64_t M,
                                int64_t N) {
  const int64_t n = M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    x[i] += b[i % N];
}

// g[i] = a[i] > 0 ? g[i] : 0   (ReLU derivative; a = relu(h) > 0 exactly when h > 0)
__global__ void relu_grad_kernel(float* __restrict__ g, const float* __restrict__ a, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    if (!(a[i] > 0.0f)) g[i] = 0.0f;
}

// out[j] = sum_i x[i, j], in a fixed order: 32 columns per block, 8 row
// lanes striding over the rows, then the 8 partial sums added in lane order.
__global__ void __launch_bounds__(256) colsum_kernel(const float* __restrict__ x,
                                                     float* __restrict__ out, int64_t M,
                                                     int64_t N) {
  __shared__ float part[8][33];
  const int c = threadIdx.x & 31, r = threadIdx.x >> 5;
  const int64_t col = (int64_t)blockIdx.x * 32 + c;
  float s = 0.0f;
  if (col < N)
    for (int64_t i = r; i < M; i += 8) s += x[i * N + col];
  part[r][c] = s;
  __syncthreads();
  if (r == 0 && col < N) {
    float t = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += part[k][c];
    out[col] = t;
  }
}

}  // namespace train
}  // namespace jb
