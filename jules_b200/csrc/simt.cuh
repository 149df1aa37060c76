// CUDA-core kernels: the fp32-exact paths behind the reference's float*
// API, and the general-shape paths (any M/N/K, any alignment, head_dim other
// than 128) that the tensor-core kernels do not take.
//
// All are GPU kernels; none falls back to the host.
#pragma once

#include "gemm_tc.cuh"  // act_fast, act_exact
#include "sm100.cuh"

namespace jb {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }


// ---------------------------------------------------------------------------
// GEMM: C = act(A.W + bias) (+ residual).  128x128 block tile, 8x8 per
// thread, K step 8, smem staged.  fp32 accumulation in k order.
// ---------------------------------------------------------------------------
namespace simt {

constexpr int GBM = 128, GBN = 128, GBK = 8;

template <typename TIn, typename TOut>
__global__ void __launch_bounds__(256)
    gemm_kernel(const TIn* __restrict__ A, const TIn* __restrict__ W,
                const float* __restrict__ bias, const TIn* __restrict__ residual,
                TOut* __restrict__ C, int M, int N, int K, int act, int exact) {
  __shared__ float As[GBK][GBM + 4];
  __shared__ float Ws[GBK][GBN + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * GBM, n0 = blockIdx.x * GBN;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  for (int k0 = 0; k0 < K; k0 += GBK) {
    // A tile: 128 rows x 8 k -> 1024 elements, 4 per thread.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256;
      const int r = e / GBK, kk = e % GBK;
      const int gm = m0 + r, gk = k0 + kk;
      As[kk][r] = (gm < M && gk < K) ? to_f32(A[(size_t)gm * K + gk]) : 0.0f;
    }
    // W tile: 8 k x 128 cols.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256;
      const int kk = e / GBN, c = e % GBN;
      const int gk = k0 + kk, gn = n0 + c;
      Ws[kk][c] = (gk < K && gn < N) ? to_f32(W[(size_t)gk * N + gn]) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < GBK; ++kk) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = As[kk][ty * 8 + i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = Ws[kk][tx * 8 + j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + ty * 8 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + tx * 8 + j;
      if (gn >= N) continue;
      float v = acc[i][j];
      if (bias) v += bias[gn];
      v = exact ? act_exact(v, act) : act_fast(v, act);
      if (residual) v += to_f32(residual[(size_t)gm * N + gn]);
      C[(size_t)gm * N + gn] = from_f32<TOut>(v);
    }
  }
}

// ---------------------------------------------------------------------------
// Row-major SGEMM with transposes, C = alpha op(A) op(B) + beta C (the
// cblas_sgemm contract the reference calls, FusedKernels.h:633-644).
// Same 128x128x8 tiling as gemm_kernel.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    sgemm_kernel(int ta, int tb, int M, int N, int K, float alpha, const float* __restrict__ A,
                 int lda, const float* __restrict__ Bm, int ldb, float beta,
                 float* __restrict__ C, int ldc) {
  __shared__ float As[GBK][GBM + 4];
  __shared__ float Ws[GBK][GBN + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * GBM, n0 = blockIdx.x * GBN;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  for (int k0 = 0; k0 < K; k0 += GBK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256;
      const int r = e / GBK, kk = e % GBK;
      const int gm = m0 + r, gk = k0 + kk;
      As[kk][r] = (gm < M && gk < K) ? (ta ? A[(size_t)gk * lda + gm] : A[(size_t)gm * lda + gk]) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256;
      const int kk = e / GBN, c = e % GBN;
      const int gk = k0 + kk, gn = n0 + c;
      Ws[kk][c] = (gk < K && gn < N) ? (tb ? Bm[(size_t)gn * ldb + gk] : Bm[(size_t)gk * ldb + gn]) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < GBK; ++kk) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = As[kk][ty * 8 + i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = Ws[kk][tx * 8 + j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + ty * 8 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + tx * 8 + j;
      if (gn >= N) continue;
      float* c = C + (size_t)gm * ldc + gn;
      *c = alpha * acc[i][j] + (beta == 0.0f ? 0.0f : beta * *c);
    }
  }
}

// ---------------------------------------------------------------------------
// Attention forward (any head_dim <= 256), online softmax in fp32.
// Block = 4 warps over BQ=16 query rows of one (b, h); key tiles of 32
// (lane <-> key for scores, lane <-> head-dim slice for P.V).
// Causal: key j > query i excluded; tiles past the block's last row skipped.
// Grouped-query: kv head = h / (Hq / Hkv).  lse = max + log(sum).
// ---------------------------------------------------------------------------
constexpr int ABQ = 16, ABK = 32;

template <typename TIn, typename TOut, int DPL>
__global__ void __launch_bounds__(128)
    attn_kernel(const TIn* __restrict__ Q, const TIn* __restrict__ Kp,
                const TIn* __restrict__ Vp, TOut* __restrict__ O, float* __restrict__ lse,
                int Hq, int Hkv, int S, int D, float scale, int causal) {
  constexpr int DMAX = DPL * 32;
  extern __shared__ float sm[];
  float* Qs = sm;                     // [ABQ][DMAX]
  float* Ks = Qs + ABQ * DMAX;        // [ABK][DMAX+1]
  float* Vs = Ks + ABK * (DMAX + 1);  // [ABK][DMAX]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int b = bh / Hq, h = bh % Hq;
  const int hk = h / (Hq / Hkv);
  const int q0 = blockIdx.x * ABQ;
  const TIn* qb = Q + (size_t)bh * S * D;
  const TIn* kb = Kp + ((size_t)b * Hkv + hk) * S * D;
  const TIn* vb = Vp + ((size_t)b * Hkv + hk) * S * D;

  for (int e = threadIdx.x; e < ABQ * DMAX; e += blockDim.x) {
    const int r = e / DMAX, d = e % DMAX;
    Qs[e] = (q0 + r < S && d < D) ? to_f32(qb[(size_t)(q0 + r) * D + d]) : 0.0f;
  }

  float m[4], l[4], acc[4][DPL];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[r][i] = 0.0f;
  }

  const int kv_end = causal ? min(S, q0 + ABQ) : S;
  for (int k0 = 0; k0 < kv_end; k0 += ABK) {
    __syncthreads();
    for (int e = threadIdx.x; e < ABK * DMAX; e += blockDim.x) {
      const int j = e / DMAX, d = e % DMAX;
      const bool in = (k0 + j < S) && d < D;
      Ks[j * (DMAX + 1) + d] = in ? to_f32(kb[(size_t)(k0 + j) * D + d]) : 0.0f;
      Vs[j * DMAX + d] = in ? to_f32(vb[(size_t)(k0 + j) * D + d]) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int qr = warp * 4 + r;
      const int qi = q0 + qr;
      if (qi >= S) continue;  // warp-uniform
      const int kj = k0 + lane;
      float sdot = 0.0f;
      const float* qrow = Qs + qr * DMAX;
      const float* krow = Ks + lane * (DMAX + 1);
      for (int d = 0; d < D; ++d) sdot = fmaf(qrow[d], krow[d], sdot);
      float sc = scale * sdot;
      const bool valid = (kj < S) && !(causal && kj > qi);
      if (!valid) sc = -INFINITY;
      float tmax = sc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float mnew = fmaxf(m[r], tmax);
      if (mnew == -INFINITY) continue;  // nothing visible yet (warp-uniform)
      const float p = valid ? expf(sc - mnew) : 0.0f;
      const float alpha = (m[r] == -INFINITY) ? 0.0f : expf(m[r] - mnew);
      float psum = p;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
      l[r] = l[r] * alpha + psum;
      m[r] = mnew;
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[r][i] *= alpha;
      for (int j = 0; j < ABK; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        const float* vrow = Vs + j * DMAX;
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[r][i] = fmaf(pj, vrow[lane + 32 * i], acc[r][i]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int qi = q0 + warp * 4 + r;
    if (qi >= S) continue;
    const float inv = 1.0f / l[r];
    TOut* orow = O + ((size_t)bh * S + qi) * D;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int d = lane + 32 * i;
      if (d < D) orow[d] = from_f32<TOut>(acc[r][i] * inv);
    }
    if (lse && lane == 0) lse[(size_t)bh * S + qi] = m[r] + logf(l[r]);
  }
}

// ---------------------------------------------------------------------------
// Register-tiled attention forward for head dims 32, 64 and 128 (the fp32
// path, C1's [1,8,512,64]): 32 query rows of one (b, h) per CTA, key tiles
// of 64, two groups of 128 threads taking alternate key tiles (each with its
// own shared-memory tiles and named barrier), merged at the end.  Within a
// group, 8 x 16 threads: thread (ty, tx) computes the scores of query rows
// 4ty..4ty+3 against keys 4tx..4tx+3 of the tile (Q and K staged transposed
// in shared memory, 16 FMAs per two float4 loads) and accumulates output
// dims tx*DPT.. of its four rows from P (staged key-major) and V.  Online softmax per row as attn_kernel (expf, running
// max and sum reduced over the 16 threads of a half warp); causal and
// padding masks; grouped-query heads.
// ---------------------------------------------------------------------------
constexpr int TRT = 4;               // query rows per thread
constexpr int TBQ = 8 * TRT, TBK = 64;  // query rows per CTA, keys per tile

// Four consecutive elements as fp32 (16-byte fp32 / 8-byte bf16 load).
__device__ __forceinline__ float4 load4_f32(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
__device__ __forceinline__ float4 load4_f32(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ float4 load4_f32(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

constexpr int kTileThreads = 256;

template <int D>
constexpr size_t attn_tile_smem_floats() {
  return D * TBQ + 2 * (D * (TBK + 4) + TBK * D + TBK * TBQ);
}

template <typename TIn, typename TOut, int D>
__global__ void __launch_bounds__(kTileThreads, 1)
    attn_tile_kernel(const TIn* __restrict__ Q, const TIn* __restrict__ Kp,
                     const TIn* __restrict__ Vp, TOut* __restrict__ O, float* __restrict__ lse,
                     int Hq, int Hkv, int S, float scale, int causal) {
  static_assert(D == 32 || D == 64 || D == 128, "head dim");
  constexpr int RT = TRT;
  constexpr int DPT = D / 16;     // output dims per thread
  constexpr int KT = TBK + 4;     // Kt row stride (16-byte multiple, fewer bank conflicts)
  extern __shared__ float sm[];
  const int grp = threadIdx.x >> 7;  // key-tile group: tiles grp, grp + 2, ...
  const int gt = threadIdx.x & 127;  // thread within the group
  float* Qt = sm;                                    // [D][TBQ], shared by both groups
  float* Kt = Qt + D * TBQ + grp * (D * KT + TBK * D + TBK * TBQ);  // [D][KT]
  float* Vs = Kt + D * KT;                           // [TBK][D]
  float* Pt = Vs + TBK * D;                          // [TBK][TBQ]
  // group-local barrier (ids 1, 2), 128 threads
  auto group_sync = [&]() { asm volatile("bar.sync %0, 128;" ::"r"(grp + 1) : "memory"); };

  const int tx = gt & 15, ty = gt >> 4;
  const int bh = blockIdx.y;
  const int b = bh / Hq, h = bh % Hq;
  const int hk = h / (Hq / Hkv);
  const int q0 = blockIdx.x * TBQ;
  const TIn* qb = Q + (size_t)bh * S * D;
  const TIn* kb = Kp + ((size_t)b * Hkv + hk) * S * D;
  const TIn* vb = Vp + ((size_t)b * Hkv + hk) * S * D;

  for (int e = threadIdx.x; e < TBQ * D; e += kTileThreads) {
    const int r = e / D, d = e % D;
    Qt[d * TBQ + r] = (q0 + r < S) ? to_f32(qb[(size_t)(q0 + r) * D + d]) : 0.0f;
  }
  __syncthreads();
  float m[RT], l[RT], acc[RT][DPT];
#pragma unroll
  for (int r = 0; r < RT; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int i = 0; i < DPT; ++i) acc[r][i] = 0.0f;
  }

  const int qi0 = q0 + RT * ty;  // this thread's first query row
  const int kv_end = causal ? min(S, q0 + TBQ) : S;
  // K / V tiles move through registers, 4 elements per load: the next
  // tile's loads are issued before the current tile's arithmetic (head dims
  // up to 64; at 128 the 32 registers per tensor would spill).
  constexpr int NV4 = TBK * D / 4 / 128;
  constexpr bool kPrefetch = D <= 64;
  float4 kr[NV4], vr[NV4];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int u = 0; u < NV4; ++u) {
      const int idx = gt + 128 * u;
      const int j = idx / (D / 4), d4 = idx % (D / 4);
      const bool in = k0 + j < S;
      kr[u] = in ? load4_f32(kb + (size_t)(k0 + j) * D + 4 * d4) : make_float4(0.f, 0.f, 0.f, 0.f);
      vr[u] = in ? load4_f32(vb + (size_t)(k0 + j) * D + 4 * d4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto stash = [&]() {
#pragma unroll
    for (int u = 0; u < NV4; ++u) {
      const int idx = gt + 128 * u;
      const int j = idx / (D / 4), d4 = idx % (D / 4);
      Kt[(4 * d4 + 0) * KT + j] = kr[u].x;
      Kt[(4 * d4 + 1) * KT + j] = kr[u].y;
      Kt[(4 * d4 + 2) * KT + j] = kr[u].z;
      Kt[(4 * d4 + 3) * KT + j] = kr[u].w;
      *reinterpret_cast<float4*>(Vs + j * D + 4 * d4) = vr[u];
    }
  };
  const int k_first = grp * TBK;
  if (kPrefetch && k_first < kv_end) fetch(k_first);
  for (int k0 = k_first; k0 < kv_end; k0 += 2 * TBK) {
    group_sync();  // previous tile's Kt / Vs / Pt fully consumed
    if (!kPrefetch) fetch(k0);
    stash();
    group_sync();
    if (kPrefetch && k0 + 2 * TBK < kv_end) fetch(k0 + 2 * TBK);  // in flight during this tile
    float sc[RT][4] = {};
#pragma unroll 8
    for (int d = 0; d < D; ++d) {
      const float4 q = *reinterpret_cast<const float4*>(Qt + d * TBQ + RT * ty);
      const float4 k = *reinterpret_cast<const float4*>(Kt + d * KT + 4 * tx);
      const float qv[RT] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        sc[r][0] = fmaf(qv[r], k.x, sc[r][0]);
        sc[r][1] = fmaf(qv[r], k.y, sc[r][1]);
        sc[r][2] = fmaf(qv[r], k.z, sc[r][2]);
        sc[r][3] = fmaf(qv[r], k.w, sc[r][3]);
      }
    }
    float p[RT][4];
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      const int qi = qi0 + r;
      float tmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int kj = k0 + 4 * tx + c;
        const bool valid = kj < S && !(causal && kj > qi);
        sc[r][c] = valid ? scale * sc[r][c] : -INFINITY;
        tmax = fmaxf(tmax, sc[r][c]);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float mnew = fmaxf(m[r], tmax);
      float psum = 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        p[r][c] = (sc[r][c] == -INFINITY) ? 0.0f : expf(sc[r][c] - mnew);
        psum += p[r][c];
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
      const float alpha = (m[r] == -INFINITY) ? 0.0f : expf(m[r] - mnew);
      l[r] = l[r] * alpha + psum;
      m[r] = mnew;
#pragma unroll
      for (int i = 0; i < DPT; ++i) acc[r][i] *= alpha;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<float4*>(Pt + (4 * tx + c) * TBQ + RT * ty) =
          make_float4(p[0][c], p[1][c], p[2][c], p[3][c]);
    group_sync();
#pragma unroll 4
    for (int j = 0; j < TBK; ++j) {
      const float4 pq = *reinterpret_cast<const float4*>(Pt + j * TBQ + RT * ty);
      const float pv[RT] = {pq.x, pq.y, pq.z, pq.w};
      const float* vrow = Vs + j * D + tx * DPT;
#pragma unroll
      for (int i = 0; i < DPT; i += 2) {
        const float2 v = *reinterpret_cast<const float2*>(vrow + i);
#pragma unroll
        for (int r = 0; r < RT; ++r) {
          acc[r][i] = fmaf(pv[r], v.x, acc[r][i]);
          acc[r][i + 1] = fmaf(pv[r], v.y, acc[r][i + 1]);
        }
      }
    }
  }
  // Merge: group 1 hands (m, l, acc) of each of its rows to the group-0
  // thread with the same (ty, tx) through its own (now free) tile memory.
  __syncthreads();
  float* xch = sm + D * TBQ + (D * KT + TBK * D + TBK * TBQ);  // group 1's tiles
  constexpr int XS = 2 * RT + RT * DPT;  // floats per thread: m, l at 2r, 2r+1; acc after
  if (grp == 1) {
    float* x = xch + gt * XS;
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      x[2 * r] = m[r];
      x[2 * r + 1] = l[r];
#pragma unroll
      for (int i = 0; i < DPT; ++i) x[2 * RT + r * DPT + i] = acc[r][i];
    }
  }
  __syncthreads();
  if (grp == 1) return;
  {
    const float* x = xch + gt * XS;
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      const float m1 = x[2 * r], l1 = x[2 * r + 1];
      const float mn = fmaxf(m[r], m1);
      if (mn == -INFINITY) continue;  // row with no visible key (padding)
      const float a0 = (m[r] == -INFINITY) ? 0.0f : expf(m[r] - mn);
      const float a1 = (m1 == -INFINITY) ? 0.0f : expf(m1 - mn);
      l[r] = l[r] * a0 + l1 * a1;
      m[r] = mn;
#pragma unroll
      for (int i = 0; i < DPT; ++i) acc[r][i] = acc[r][i] * a0 + x[2 * RT + r * DPT + i] * a1;
    }
  }
#pragma unroll
  for (int r = 0; r < RT; ++r) {
    const int qi = qi0 + r;
    if (qi >= S) continue;
    const float inv = 1.0f / l[r];
    TOut* orow = O + ((size_t)bh * S + qi) * D + tx * DPT;
#pragma unroll
    for (int i = 0; i < DPT; ++i) orow[i] = from_f32<TOut>(acc[r][i] * inv);
    if (lse && tx == 0) lse[(size_t)bh * S + qi] = m[r] + logf(l[r]);
  }
}

// ---------------------------------------------------------------------------
// LayerNorm over rows (include/jules/Kernel/FusedKernels.h:532-600): mean,
// biased variance (second pass over (x-mean)^2), inv_std = 1/sqrt(var+eps),
// y = (x-mean)*inv_std*gamma + beta.  One 256-thread block per row; fp32
// statistics.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float block_sum_256(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += red[w];
  return t;
}

template <typename TIn, typename TOut>
__global__ void __launch_bounds__(256)
    layernorm_kernel(const TIn* __restrict__ in, const float* __restrict__ gamma,
                     const float* __restrict__ beta, TOut* __restrict__ out,
                     float* __restrict__ mean_out, float* __restrict__ rstd_out, int64_t M,
                     int64_t N, float eps) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  if (row >= M) return;
  const TIn* x = in + row * N;
  float s = 0.0f;
  for (int64_t j = threadIdx.x; j < N; j += 256) s += to_f32(x[j]);
  const float mean = block_sum_256(s, red) / (float)N;
  float v = 0.0f;
  for (int64_t j = threadIdx.x; j < N; j += 256) {
    const float d = to_f32(x[j]) - mean;
    v = fmaf(d, d, v);
  }
  const float var = block_sum_256(v, red) / (float)N;
  const float inv_std = 1.0f / sqrtf(var + eps);
  TOut* y = out + row * N;
  // gamma == beta == NULL: no affine transform (the routed fusedLayerNorm form)
  for (int64_t j = threadIdx.x; j < N; j += 256)
    y[j] = from_f32<TOut>((to_f32(x[j]) - mean) * inv_std * (gamma ? gamma[j] : 1.0f) +
                          (beta ? beta[j] : 0.0f));
  if (threadIdx.x == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = inv_std;
  }
}

// Weights of the LayerNorm folded into the following GEMM (prepared once per
// weights): W'[k][n] = bf16(gamma[k] * W[k][n]), colsum[n] = sum over k of
// W'[k][n] as the tensor core sees it (the bf16 values, k in order), and
// c[n] = b[n] + sum over k of beta[k] * W[k][n].  One thread per column,
// walking k (consecutive threads read consecutive columns).
__global__ void __launch_bounds__(256)
    ln_fold_weights_kernel(const __nv_bfloat16* __restrict__ W, const float* __restrict__ gamma,
                           const float* __restrict__ beta, const float* __restrict__ b,
                           __nv_bfloat16* __restrict__ Wf, float* __restrict__ colsum,
                           float* __restrict__ cvec, int d, int n_cols) {
  const int n = blockIdx.x * 256 + threadIdx.x;
  if (n >= n_cols) return;
  float cs = 0.0f, cb = b ? b[n] : 0.0f;
  for (int k = 0; k < d; ++k) {
    const float w = __bfloat162float(W[(size_t)k * n_cols + n]);
    const __nv_bfloat16 wf = __float2bfloat16_rn(gamma[k] * w);
    Wf[(size_t)k * n_cols + n] = wf;
    cs += __bfloat162float(wf);
    cb = fmaf(beta[k], w, cb);
  }
  colsum[n] = cs;
  cvec[n] = cb;
}

// bf16 LayerNorm, one warp per row, for N % 8 == 0 and N <= 256 * NV: the
// row stays in registers as bf16 (NV 16-byte vectors per lane, all loads in
// flight at once), mean and biased variance by warp shuffles over two passes
// of the registers (the reference's two-pass statistics), one HBM read, no
// block barriers; 8 rows per 256-thread block.  Writes any of: the
// normalised row (out, with gamma/beta or without both), mean_out /
// rstd_out, and stats_out = (mean, rstd) per row (the row statistics the
// LayerNorm folded into a GEMM epilogue needs).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int NV>
__global__ void __launch_bounds__(256, NV <= 16 ? 2 : 1)
    layernorm_bf16_warp_kernel(const __nv_bfloat16* __restrict__ in,
                               const float* __restrict__ gamma, const float* __restrict__ beta,
                               __nv_bfloat16* __restrict__ out, float* __restrict__ mean_out,
                               float* __restrict__ rstd_out, float2* __restrict__ stats_out,
                               int64_t M, int N, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= M) return;
  const int nv = N >> 3;
  const uint4* x = reinterpret_cast<const uint4*>(in + row * N);
  uint4 xv[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    xv[i] = c < nv ? x[c] : make_uint4(0u, 0u, 0u, 0u);
  }
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&xv[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(p[j]);
      s += f.x + f.y;
    }
  }
  const float mean = warp_sum(s) / (float)N;
  float v = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (lane + 32 * i < nv) {
      const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&xv[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(p[j]);
        const float d0 = f.x - mean, d1 = f.y - mean;
        v = fmaf(d0, d0, v);
        v = fmaf(d1, d1, v);
      }
    }
  }
  const float var = warp_sum(v) / (float)N;
  const float inv_std = 1.0f / sqrtf(var + eps);
  if (lane == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = inv_std;
    if (stats_out) stats_out[row] = make_float2(mean, inv_std);
  }
  if (!out) return;
  uint4* y = reinterpret_cast<uint4*>(out + row * N);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    if (c < nv) {
      float g[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f}, bb[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (gamma) {
        const float4 g0 = reinterpret_cast<const float4*>(gamma)[2 * c];
        const float4 g1 = reinterpret_cast<const float4*>(gamma)[2 * c + 1];
        const float4 b0 = reinterpret_cast<const float4*>(beta)[2 * c];
        const float4 b1 = reinterpret_cast<const float4*>(beta)[2 * c + 1];
        g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w; g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
        bb[0] = b0.x; bb[1] = b0.y; bb[2] = b0.z; bb[3] = b0.w; bb[4] = b1.x; bb[5] = b1.y; bb[6] = b1.z; bb[7] = b1.w;
      }
      const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&xv[i]);
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(p[j]);
        o[j] = pack_bf16x2((f.x - mean) * inv_std * g[2 * j] + bb[2 * j],
                           (f.y - mean) * inv_std * g[2 * j + 1] + bb[2 * j + 1]);
      }
      y[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Vectorised bf16 LayerNorm for N % 8 == 0 and N <= 8 * 256 * LNV: the row
// stays in registers between the three passes (one HBM read).
template <int LNV>
__global__ void __launch_bounds__(256)
    layernorm_bf16_vec_kernel(const __nv_bfloat16* __restrict__ in,
                              const float* __restrict__ gamma, const float* __restrict__ beta,
                              __nv_bfloat16* __restrict__ out, float* __restrict__ mean_out,
                              float* __restrict__ rstd_out, int64_t M, int N, float eps) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  if (row >= M) return;
  const uint4* x = reinterpret_cast<const uint4*>(in + row * N);
  const int nv = N / 8;
  float xv[LNV][8];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < LNV; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c < nv) {
      const uint4 u = x[c];
      const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(p[j]);
        xv[i][2 * j] = f.x;
        xv[i][2 * j + 1] = f.y;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) s += xv[i][j];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) xv[i][j] = 0.0f;
    }
  }
  const float mean = block_sum_256(s, red) / (float)N;
  float v = 0.0f;
#pragma unroll
  for (int i = 0; i < LNV; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c < nv) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = xv[i][j] - mean;
        v = fmaf(d, d, v);
      }
    }
  }
  const float var = block_sum_256(v, red) / (float)N;
  const float inv_std = 1.0f / sqrtf(var + eps);
  uint4* y = reinterpret_cast<uint4*>(out + row * N);
#pragma unroll
  for (int i = 0; i < LNV; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c < nv) {
      const float4 g0 = reinterpret_cast<const float4*>(gamma)[2 * c];
      const float4 g1 = reinterpret_cast<const float4*>(gamma)[2 * c + 1];
      const float4 b0 = reinterpret_cast<const float4*>(beta)[2 * c];
      const float4 b1 = reinterpret_cast<const float4*>(beta)[2 * c + 1];
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (xv[i][j] - mean) * inv_std * g[j] + bb[j];
      uint4 u;
      u.x = pack_bf16x2(o[0], o[1]);
      u.y = pack_bf16x2(o[2], o[3]);
      u.z = pack_bf16x2(o[4], o[5]);
      u.w = pack_bf16x2(o[6], o[7]);
      y[c] = u;
    }
  }
  if (threadIdx.x == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = inv_std;
  }
}

// GELU-tanh elementwise (FusedKernels.h:606-627).
template <typename T>
__global__ void gelu_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = from_f32<T>(act_exact(to_f32(in[i]), 4));
}

// ---------------------------------------------------------------------------
// 3xTF32 operand split for the fp32 GEMM on tensor cores.  Each fp32 x is
// hi + lo + r with hi = tf32(x), lo = tf32(x - hi) (x - hi is exact in fp32)
// and |r| <= 2^-22 |x|.  K is cut into chunks of Kc (the last one shorter);
// chunk c of length L becomes 3L columns of the tf32 operands:
//   A  [M,K] -> A3  [M,3K]: per chunk [lo | hi | hi]
//   W  [K,N] -> W3T [N,3K]: per chunk [hi | lo | hi] of W's columns (W
//               transposed: the tf32 MMAs take B K-major)
// so that one chunk's product is loA hiW + hiA loW + hiA hiW, dropping only
// loA loW (<= 2^-22 |a w|).  The small terms come first, while the
// accumulator is still small: the MMAs' fp32 accumulation truncates toward
// zero, so each step costs up to an ulp of the running sum.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = to_tf32(x);
  lo = to_tf32(x - hi);
}

// Column k of the K columns -> offsets of its three copies in a 3K row.
__device__ __forceinline__ void chunk_cols(int k, int K, int Kc, int& o_first, int& L) {
  const int c = k / Kc;
  const int base = c * Kc;
  L = min(Kc, K - base);
  o_first = 3 * base + (k - base);  // first copy; the others at +L and +2L
}

// A [rows, K] -> A3 [rows, 3K].  Four columns per thread (K, Kc multiples of
// 4: a group never straddles a chunk; 16-byte aligned rows).
__global__ void split3_a_kernel(const float4* __restrict__ A, float* __restrict__ A3, int64_t rows,
                                int K, int Kc) {
  const int k4 = K / 4;
  const int64_t n = rows * k4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / k4;
    const int k = (int)(i - r * k4) * 4;
    const float4 x = A[i];
    float4 hi, lo;
    split_tf32(x.x, hi.x, lo.x);
    split_tf32(x.y, hi.y, lo.y);
    split_tf32(x.z, hi.z, lo.z);
    split_tf32(x.w, hi.w, lo.w);
    int o, L;
    chunk_cols(k, K, Kc, o, L);
    float* row = A3 + r * 3 * (int64_t)K;
    *reinterpret_cast<float4*>(row + o) = lo;
    *reinterpret_cast<float4*>(row + o + L) = hi;
    *reinterpret_cast<float4*>(row + o + 2 * L) = hi;
  }
}

// W [K,N] -> W3T [N,3K].  Block (32, 8) per 64 x 64 tile (16 loads in
// flight per thread): reads along N, 16-byte writes along K (both
// coalesced).
// Grid (ceil(N/64), ceil(K/64)).
constexpr int kSplitTile = 64;
__global__ void __launch_bounds__(256)
    split3_wt_kernel(const float* __restrict__ W, float* __restrict__ W3T, int K, int N, int Kc) {
  constexpr int T = kSplitTile;
  __shared__ float hi_s[T][T + 1], lo_s[T][T + 1];
  const int k0 = blockIdx.y * T, n0 = blockIdx.x * T;
#pragma unroll
  for (int i = threadIdx.y; i < T; i += 8) {
#pragma unroll
    for (int h = 0; h < T; h += 32) {
      const int k = k0 + i, n = n0 + h + threadIdx.x;
      float hv = 0.0f, lv = 0.0f;
      if (k < K && n < N) split_tf32(W[(size_t)k * N + n], hv, lv);
      hi_s[i][h + threadIdx.x] = hv;
      lo_s[i][h + threadIdx.x] = lv;
    }
  }
  __syncthreads();
  // Stores: 16 bytes (4 consecutive k of one n) per thread and copy; a warp
  // covers two rows of 64 k.  K and Kc are multiples of 4, so a group of 4
  // never straddles a chunk and every store is 16-byte aligned.
  const int tid = threadIdx.y * 32 + threadIdx.x;
#pragma unroll
  for (int it = tid; it < T * (T / 4); it += 256) {
    const int nl = it / (T / 4), kg = (it % (T / 4)) * 4;
    const int n = n0 + nl, k = k0 + kg;
    if (n < N && k < K) {
      int o, L;
      chunk_cols(k, K, Kc, o, L);
      float* row = W3T + (size_t)n * 3 * K;
      const float4 hv = make_float4(hi_s[kg][nl], hi_s[kg + 1][nl], hi_s[kg + 2][nl], hi_s[kg + 3][nl]);
      const float4 lv = make_float4(lo_s[kg][nl], lo_s[kg + 1][nl], lo_s[kg + 2][nl], lo_s[kg + 3][nl]);
      *reinterpret_cast<float4*>(row + o) = hv;
      *reinterpret_cast<float4*>(row + o + L) = lv;
      *reinterpret_cast<float4*>(row + o + 2 * L) = hv;
    }
  }
}

}  // namespace simt
}  // namespace jb
