// Row-wise softmax and fused softmax + cross-entropy (HBM-bound CUDA-core
// kernels).
//
// Softmax follows the reference's fusedSoftmax (FusedKernels.h:464-526): per
// row the max, e = exp(x - max) with its sum, then e * (1 / sum).  The loss
// follows fusedCrossEntropyLoss (FusedKernels.h:766-854): the same softmax p,
// row loss -log(p[target] + 1e-10), gradient (p - onehot(target)) / M, and the
// mean of the row losses.  Arithmetic is fp32 whatever the storage type.
//
// Rows of up to kWarpRowMax elements are held in one warp's registers (one
// read, one write).  Longer rows take one CTA each: an online pass keeps a
// running (max, sum) per thread and merges them, a second pass (served mostly
// by L2, the row was just read) writes the output.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

#include "simt.cuh"
#include "sm100.cuh"

namespace jb {
namespace rows {

constexpr int kWarpRowMax = 1024;  // 32 lanes x 32 registers
constexpr int kCtaThreads = 256;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Merge two (max, sum-of-exp relative to max) pairs.
__device__ __forceinline__ void ms_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;  // both empty
  s = s * expf(m - mn) + s2 * expf(m2 - mn);
  m = mn;
}

// Row loss of the fused cross-entropy, added into *loss already divided by M.
// An out-of-range target records kDevErrBadShape and contributes nothing
// (the reference leaves it undefined).
__device__ __forceinline__ bool target_ok(int t, int N) {
  if (t >= 0 && t < N) return true;
  record_error(kDevErrBadShape, 90);
  return false;
}

// One warp per row, N <= kWarpRowMax.  XENT: out is the gradient (may be
// null), targets/loss are used.
template <typename TIn, typename TOut, bool XENT>
__global__ void __launch_bounds__(256) softmax_warp_kernel(const TIn* __restrict__ in,
                                                           TOut* __restrict__ out,
                                                           const int32_t* __restrict__ targets,
                                                           float* __restrict__ loss, int64_t M,
                                                           int N, float inv_M) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  float loss_acc = 0.0f;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M;
       row += warps) {
    const TIn* x = in + row * N;
    float v[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const int c = lane + 32 * k;
      v[k] = c < N ? to_f32(x[c]) : -INFINITY;
    }
    float m = v[0];
#pragma unroll
    for (int k = 1; k < 32; ++k) m = fmaxf(m, v[k]);
    m = warp_max(m);
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      v[k] = (lane + 32 * k < N) ? expf(v[k] - m) : 0.0f;
      s += v[k];
    }
    s = warp_sum(s);
    const float inv = 1.0f / s;
    if (!XENT) {
      TOut* y = out + row * N;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const int c = lane + 32 * k;
        if (c < N) y[c] = from_f32<TOut>(v[k] * inv);
      }
    } else {
      const int t = targets[row];
      const bool tv = target_ok(t, N);
      if (out) {
        TOut* y = out + row * N;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const int c = lane + 32 * k;
          if (c < N) y[c] = from_f32<TOut>((v[k] * inv - (c == t ? 1.0f : 0.0f)) * inv_M);
        }
      }
      if (lane == 0 && tv) {
        const float p = expf(to_f32(x[t]) - m) * inv;
        loss_acc += -logf(p + 1e-10f) * inv_M;
      }
    }
  }
  if (XENT && lane == 0 && loss_acc != 0.0f) atomicAdd(loss, loss_acc);
}

// One CTA (256 threads) per row, any N.
template <typename TIn, typename TOut, bool XENT>
__global__ void __launch_bounds__(kCtaThreads) softmax_cta_kernel(const TIn* __restrict__ in,
                                                                  TOut* __restrict__ out,
                                                                  const int32_t* __restrict__ targets,
                                                                  float* __restrict__ loss,
                                                                  int64_t M, int N, float inv_M) {
  __shared__ float red_m[kCtaThreads / 32], red_s[kCtaThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float loss_acc = 0.0f;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const TIn* x = in + row * N;
    // Pass 1: running (max, sum of exp relative to max) per thread.
    float m = -INFINITY, s = 0.0f;
    for (int c = threadIdx.x; c < N; c += kCtaThreads) {
      const float xv = to_f32(x[c]);
      if (xv > m) {
        s = (m == -INFINITY ? 0.0f : s * expf(m - xv)) + 1.0f;
        m = xv;
      } else {
        s += expf(xv - m);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      ms_merge(m, s, m2, s2);
    }
    __syncthreads();  // red_* reuse across rows
    if (lane == 0) {
      red_m[warp] = m;
      red_s[warp] = s;
    }
    __syncthreads();
    m = red_m[0];
    s = red_s[0];
#pragma unroll
    for (int w = 1; w < kCtaThreads / 32; ++w) ms_merge(m, s, red_m[w], red_s[w]);
    const float inv = 1.0f / s;
    // Pass 2: write.
    int t = 0;
    bool tv = false;
    if (XENT) {
      t = targets[row];
      tv = t >= 0 && t < N;
      if (threadIdx.x == 0 && !target_ok(t, N)) tv = false;
    }
    if (!XENT || out) {
      TOut* y = out + row * N;
      for (int c = threadIdx.x; c < N; c += kCtaThreads) {
        const float p = expf(to_f32(x[c]) - m) * inv;
        y[c] = from_f32<TOut>(XENT ? (p - (c == t ? 1.0f : 0.0f)) * inv_M : p);
      }
    }
    if (XENT && threadIdx.x == 0 && tv) {
      const float p = expf(to_f32(x[t]) - m) * inv;
      loss_acc += -logf(p + 1e-10f) * inv_M;
    }
  }
  if (XENT && threadIdx.x == 0 && loss_acc != 0.0f) atomicAdd(loss, loss_acc);
}

}  // namespace rows
}  // namespace jb
