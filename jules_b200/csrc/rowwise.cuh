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
// read, one write).  Longer rows take one CTA each: with 16-byte aligned rows
// of up to 32K fp32 / 64K bf16 elements the row stays in the CTA's registers
// (softmax_reg_kernel: one vectorised read, one write); otherwise an online
// pass keeps a running (max, sum) per thread and merges them, and a second
// pass (served mostly by L2, the row was just read) writes the output.
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

// 16-byte vectors: 4 floats or 8 bf16.
template <typename T>
struct Vec16;
template <>
struct Vec16<float> {
  static constexpr int kN = 4;
  // load: read-only global memory (ld.global.nc); load_generic: any state
  // space (the staged rows in shared memory).
  __device__ __forceinline__ static void load(const float* p, float (&f)[4]) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
  }
  __device__ __forceinline__ static void load_generic(const float* p, float (&f)[4]) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
  }
  __device__ __forceinline__ static void store(float* p, const float (&f)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int kN = 8;
  __device__ __forceinline__ static void unpack(const uint4 v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ __forceinline__ static void load(const __nv_bfloat16* p, float (&f)[8]) {
    unpack(__ldg(reinterpret_cast<const uint4*>(p)), f);
  }
  __device__ __forceinline__ static void load_generic(const __nv_bfloat16* p, float (&f)[8]) {
    unpack(*reinterpret_cast<const uint4*>(p), f);
  }
  __device__ __forceinline__ static void store(__nv_bfloat16* p, const float (&f)[8]) {
    uint4 v;
    v.x = pack_bf16x2(f[0], f[1]);
    v.y = pack_bf16x2(f[2], f[3]);
    v.z = pack_bf16x2(f[4], f[5]);
    v.w = pack_bf16x2(f[6], f[7]);
    *reinterpret_cast<uint4*>(p) = v;
  }
};

// Block-wide max / sum over THREADS threads (smem scratch of THREADS/32).
template <int THREADS>
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int w = 1; w < THREADS / 32; ++w) t = fmaxf(t, red[w]);
  return t;
}
template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int w = 1; w < THREADS / 32; ++w) t += red[w];
  return t;
}

// One CTA per row with the row held in registers: NV 16-byte vectors per
// thread, so rows of up to THREADS * NV * Vec16<T>::kN elements take one
// vectorised read and one vectorised write.  Needs N to be a multiple of the
// vector width and 16-byte aligned rows; input and output share the type.
template <int THREADS, int NV, typename T, bool XENT>
__global__ void __launch_bounds__(THREADS) softmax_reg_kernel(const T* __restrict__ in,
                                                              T* __restrict__ out,
                                                              const int32_t* __restrict__ targets,
                                                              float* __restrict__ loss, int64_t M,
                                                              int N, float inv_M) {
  constexpr int E = Vec16<T>::kN;
  __shared__ float red[THREADS / 32];
  float loss_acc = 0.0f;
  const int nvec = N / E;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const T* x = in + row * N;
    float f[NV][E];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = threadIdx.x + k * THREADS;
      if (vi < nvec) {
        Vec16<T>::load(x + (size_t)vi * E, f[k]);
#pragma unroll
        for (int e = 0; e < E; ++e) m = fmaxf(m, f[k][e]);
      }
    }
    m = block_max<THREADS>(m, red);
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = threadIdx.x + k * THREADS;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        f[k][e] = (vi < nvec) ? __expf(f[k][e] - m) : 0.0f;
        sum += f[k][e];
      }
    }
    sum = block_sum<THREADS>(sum, red);
    const float inv = 1.0f / sum;
    int t = -1;
    bool tv = false;
    if (XENT) {
      t = targets[row];
      tv = t >= 0 && t < N;
      if (threadIdx.x == 0 && !target_ok(t, N)) tv = false;
    }
    if (!XENT || out) {
      T* y = out + row * N;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int vi = threadIdx.x + k * THREADS;
        if (vi < nvec) {
          float o[E];
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const float p = f[k][e] * inv;
            o[e] = XENT ? (p - (vi * E + e == t ? 1.0f : 0.0f)) * inv_M : p;
          }
          Vec16<T>::store(y + (size_t)vi * E, o);
        }
      }
    }
    if (XENT && threadIdx.x == 0 && tv) {
      const float p = __expf(to_f32(x[t]) - m) * inv;
      loss_acc += -logf(p + 1e-10f) * inv_M;
    }
  }
  if (XENT && threadIdx.x == 0 && loss_acc != 0.0f) atomicAdd(loss, loss_acc);
}

// As softmax_reg_kernel, for rows of 32 KB and more (one 1024-thread CTA per
// SM): the CTA is persistent over rows and the next row is copied into
// shared memory by one bulk copy (cp.async.bulk, completing on an mbarrier)
// as soon as the current row has moved from shared memory into registers,
// so the read of row r+1 overlaps the reductions and the output writes of
// row r.  Needs 16-byte aligned rows (N * sizeof(T) a multiple of 16).
constexpr int kStageChunk = 32768;  // bytes per bulk copy instruction

template <int THREADS, int NV, typename T, bool XENT>
__global__ void __launch_bounds__(THREADS) softmax_stage_kernel(const T* __restrict__ in,
                                                                T* __restrict__ out,
                                                                const int32_t* __restrict__ targets,
                                                                float* __restrict__ loss,
                                                                int64_t M, int N, float inv_M) {
  constexpr int E = Vec16<T>::kN;
  extern __shared__ __align__(16) uint8_t stage_raw[];
  T* row_buf = reinterpret_cast<T*>(stage_raw);
  __shared__ float red[THREADS / 32];
  __shared__ uint64_t full;
  __shared__ int abort_flag;
  const uint32_t row_bytes = (uint32_t)N * sizeof(T);
  const int nvec = N / E;
  auto issue = [&](int64_t row) {  // thread 0: bring `row` into row_buf
    mbar_arrive_expect_tx(&full, row_bytes);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(in + row * N);
    for (uint32_t o = 0; o < row_bytes; o += kStageChunk)
      bulk_load(stage_raw + o, src + o, min((uint32_t)kStageChunk, row_bytes - o), &full);
  };
  if (threadIdx.x == 0) {
    mbar_init(&full, 1);
    abort_flag = 0;
    fence_mbar_init();
    if (blockIdx.x < M) issue(blockIdx.x);
  }
  __syncthreads();
  float loss_acc = 0.0f;
  uint32_t phase = 0;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const bool ok = mbar_wait(&full, phase, 91, &abort_flag);
    if (__syncthreads_or(!ok)) break;  // uniform exit, no thread left at a barrier
    phase ^= 1u;
    float f[NV][E];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = threadIdx.x + k * THREADS;
      if (vi < nvec) {
        Vec16<T>::load_generic(row_buf + (size_t)vi * E, f[k]);
#pragma unroll
        for (int e = 0; e < E; ++e) m = fmaxf(m, f[k][e]);
      }
    }
    __syncthreads();  // row_buf fully read: the next row may land in it
    if (threadIdx.x == 0 && row + gridDim.x < M) issue(row + gridDim.x);
    m = block_max<THREADS>(m, red);
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = threadIdx.x + k * THREADS;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        f[k][e] = (vi < nvec) ? __expf(f[k][e] - m) : 0.0f;
        sum += f[k][e];
      }
    }
    sum = block_sum<THREADS>(sum, red);
    const float inv = 1.0f / sum;
    int t = -1;
    bool tv = false;
    if (XENT) {
      t = targets[row];
      tv = t >= 0 && t < N;
      if (threadIdx.x == 0 && !target_ok(t, N)) tv = false;
    }
    if (!XENT || out) {
      T* y = out + row * N;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int vi = threadIdx.x + k * THREADS;
        if (vi < nvec) {
          float o[E];
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const float p = f[k][e] * inv;
            o[e] = XENT ? (p - (vi * E + e == t ? 1.0f : 0.0f)) * inv_M : p;
          }
          Vec16<T>::store(y + (size_t)vi * E, o);
        }
      }
    }
    if (XENT && threadIdx.x == 0 && tv) {
      const float p = __expf(to_f32(in[row * N + t]) - m) * inv;
      loss_acc += -logf(p + 1e-10f) * inv_M;
    }
  }
  if (XENT && threadIdx.x == 0 && loss_acc != 0.0f) atomicAdd(loss, loss_acc);
}

}  // namespace rows
}  // namespace jb
