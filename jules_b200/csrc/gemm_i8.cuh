// int8 GEMM with int32 accumulation on tcgen05 (kind::i8), fp32 epilogue:
//   C[i,j] = float(sum_k A[i,k] * B[k,j]) * (scale_a * scale_b) (+ bias[j])
// A [M,K] and B [K,N] row-major int8, C [M,N] fp32.  This is the contract of
// the reference's matmulInt8 (FusedKernels.h:867-1073): int32 accumulation
// (its scalar branch :1046-1057), then the scale and the bias per column
// (:1060-1065).
//
// Structure as the bf16 1-CTA GEMM (gemm_tc.cuh): persistent CTAs over
// 128x256 output tiles in grouped order, warp 0 TMA, warp 1 MMA issuer,
// warps 2-5 epilogue from one of two TMEM accumulators (2 x 256 s32 columns)
// while the other accumulates.  A k-block is 128 bytes of K (one 128-byte
// swizzle row): A as K-major, B read as MN-major (its rows are K), 4 MMA
// K-steps of 32 int8 each.
#pragma once

#include <cuda_fp8.h>

#include <type_traits>

#include "gemm_tc.cuh"
#include "simt.cuh"

namespace jb {
namespace gemm8 {

constexpr int BM = 128;
constexpr int BK = 128;  // int8 elements = bytes per k-block
constexpr int kThreads = 192;

// Instruction descriptor, kind::i8: s32 D (bits 4-5 = 2), s8 A and B (bits
// 7-9 and 10-12 = 1), B MN-major (bit 16), N >> 3 at 17, M >> 4 at 24.
__host__ __device__ constexpr uint32_t idesc_s8_s32(int M, int N, bool b_mn) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_i8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <int BN, int STAGES>
struct Smem8 {
  static constexpr int kABytes = BM * BK;
  static constexpr int kBBytes = BK * BN;
  alignas(1024) uint8_t a[STAGES][kABytes];
  alignas(1024) uint8_t b[STAGES][kBBytes];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint32_t tmem_base;
  int abort_flag;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_s8_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB, const float* __restrict__ bias,
                      float* __restrict__ C, int M, int N, int K, float scale) {
  static_assert(BN % 128 == 0 && BN <= 256, "BN must be 128 or 256");
  using S = Smem8<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  S& s = *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_k = (K + BK - 1) / BK;
  constexpr uint32_t kTmemCols = 2 * BN <= 256 ? 256 : 512;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], 128);
    }
    s.abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mi, ni;
        gemm::tile_coords(t, num_m, num_n, mi, ni);
        const int m0 = mi * BM;
        const int n0 = ni * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, 80, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&s.full[stage], S::kABytes + S::kBBytes);
          tma_load_2d(s.a[stage], &tmA, &s.full[stage], kb * BK, m0);
#pragma unroll
          for (int j = 0; j < BN / 128; ++j)
            tma_load_2d(s.b[stage] + j * (BK * 128), &tmB, &s.full[stage], n0 + j * 128, kb * BK);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8_s32(BM, BN, true);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&s.tempty[acc], acc_phase ^ 1u, 81, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, 82, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(s.a[stage]);
          const uint32_t b_base = smem_u32(s.b[stage]);
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            // K-major A: 32 int8 = 32 bytes further along the swizzle row.
            const uint64_t ad = sdesc_sw128(a_base + kk * 32, 16, 1024);
            // MN-major B: 32 K-rows of 128 bytes further; 128-column chunks
            // BK * 128 bytes apart.
            const uint64_t bd = sdesc_sw128(b_base + kk * 32 * 128, BK * 128, 1024);
            umma_i8_ss(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&s.empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        umma_commit(&s.tfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int mi, ni;
      gemm::tile_coords(t, num_m, num_n, mi, ni);
      const int m0 = mi * BM;
      const int n0 = ni * BN;
      if (!mbar_wait(&s.tfull[acc], acc_phase, 83, abort_flag)) break;
      tc_fence_after();
      const int row = m0 + row_in_tile;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(t_row + c * 32, r);
        tmem_ld_wait(r);
        const int col0 = n0 + c * 32;
        if (row < M && col0 < N) {
          float* crow = C + (size_t)row * N;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int col = col0 + g * 8;
            if (col < N) {  // N is a multiple of 16 on this path
              float v[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) v[j] = (float)(int32_t)r[g * 8 + j] * scale;
              if (bias) {
                const float4 b0 = *reinterpret_cast<const float4*>(bias + col);
                const float4 b1 = *reinterpret_cast<const float4*>(bias + col + 4);
                v[0] += b0.x; v[1] += b0.y; v[2] += b0.z; v[3] += b0.w;
                v[4] += b1.x; v[5] += b1.y; v[6] += b1.z; v[7] += b1.w;
              }
              gemm::store8(crow + col, v);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&s.tempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

// Instruction descriptor, kind::f8f6f4 with 8-bit floats: f32 D (bits 4-5 =
// 1), A and B formats at 7-9 and 10-12 (0 = E4M3, 1 = E5M2), B MN-major (bit
// 16), N >> 3 at 17, M >> 4 at 24.
constexpr int kFmtE4M3 = 0;
constexpr int kFmtE5M2 = 1;
__host__ __device__ constexpr uint32_t idesc_f8_f32(int M, int N, int a_fmt, int b_fmt, bool b_mn) {
  return (1u << 4) | ((uint32_t)a_fmt << 7) | ((uint32_t)b_fmt << 10) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

#define JB_MMA2_B8(kind, ai, bi, pr) \
  "tcgen05.mma.cta_group::2.kind::" kind " [%0], %" #ai ", %" #bi ", %10, " pr ";\n\t"
#define JB_MMA2_B8x4(kind)                                                   \
  "{\n\t.reg .pred p, q;\n\t"                                                \
  "setp.ne.b32 p, %9, 0;\n\t"                                                \
  "setp.eq.b32 q, %9, %9;\n\t" JB_MMA2_B8(kind, 1, 5, "p")                   \
      JB_MMA2_B8(kind, 2, 6, "q") JB_MMA2_B8(kind, 3, 7, "q") JB_MMA2_B8(kind, 4, 8, "q") "}"

// Four K=32 steps of the pair MMA on 8-bit operands: int8 (kind::i8, s32
// accumulators) or fp8 (kind::f8f6f4, f32 accumulators).
template <bool F8>
__device__ __forceinline__ void umma4_pair_b8(uint32_t d_tmem, const uint64_t (&a)[4],
                                              const uint64_t (&b)[4], uint32_t acc_first,
                                              uint32_t idesc) {
  if constexpr (F8) {
    asm volatile(JB_MMA2_B8x4("f8f6f4")::"r"(d_tmem), "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]),
                 "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "r"(acc_first), "r"(idesc)
                 : "memory");
  } else {
    asm volatile(JB_MMA2_B8x4("i8")::"r"(d_tmem), "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]),
                 "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "r"(acc_first), "r"(idesc)
                 : "memory");
  }
}

template <int STAGES>
struct Smem8p {
  static constexpr int kABytes = 128 * BK;  // this CTA's 128 rows of A
  static constexpr int kBBytes = BK * 128;  // this CTA's 128 columns of B
  alignas(1024) uint8_t a[STAGES][kABytes];
  alignas(1024) uint8_t b[STAGES][kBBytes];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint32_t tmem_base;
  int abort_flag;
};

// CTA-pair GEMM on 8-bit operands (cta_group::2, cluster of 2): 256 x 256
// output tiles, each CTA stages its 128 rows of A and its 128 columns of B,
// the leader issues M=256, N=256 MMAs for both, and each CTA's epilogue
// handles its own 128 rows (TMEM holds a CTA's rows x all 256 columns).  Same
// barrier protocol as gemm_bf16_tc2_kernel (gemm_tc.cuh).  Epilogue:
// v = acc * scale (+ bias[col]), activation, (+ residual), stored as TOut;
// acc is the s32 (F8 = false) or f32 (F8 = true) accumulator.
template <int STAGES, bool F8, typename TOut>
__device__ __forceinline__ void pair8_body(const CUtensorMap* tmA, const CUtensorMap* tmB,
                                           const float* __restrict__ bias,
                                           const __nv_bfloat16* __restrict__ residual,
                                           TOut* __restrict__ C, int M, int N, int K, float scale,
                                           uint32_t idesc, int act, int site) {
  constexpr int TM = 256, TN = 256;
  constexpr uint32_t kTmemCols = 2 * TN;
  using S = Smem8p<STAGES>;
  extern __shared__ uint8_t smem_raw[];
  S& s = *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair_id = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int num_m = (M + TM - 1) / TM;
  const int num_n = (N + TN - 1) / TN;
  const int num_tiles = num_m * num_n;
  const int num_k = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], 2 * 128);
    }
    s.abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(tmA);
    prefetch_tmap(tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(&s.tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair_id; t < num_tiles && ok; t += num_pairs) {
        int mi, ni;
        gemm::tile_coords(t, num_m, num_n, mi, ni);
        const int m0 = mi * TM + (int)rank * 128;
        const int n0 = ni * TN + (int)rank * 128;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, site, abort_flag)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&s.full[stage], 2 * (S::kABytes + S::kBBytes));
          tma_load_2d_pair(s.a[stage], tmA, &s.full[stage], kb * BK, m0);
          tma_load_2d_pair(s.b[stage], tmB, &s.full[stage], n0, kb * BK);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA) ----------------
    if (leader && lane == 0) {
      const uint32_t empty0 = smem_u32(&s.empty[0]);
      const uint32_t tfull0 = smem_u32(&s.tfull[0]);
      const uint32_t empty0_peer = mapa_shared(empty0, 1);
      const uint32_t tfull0_peer = mapa_shared(tfull0, 1);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair_id; t < num_tiles && ok; t += num_pairs) {
        if (!mbar_wait(&s.tempty[acc], acc_phase ^ 1u, site + 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * TN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, site + 2, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t a0 = sdesc_sw128(smem_u32(s.a[stage]), 16, 1024);
          const uint64_t b0 = sdesc_sw128(smem_u32(s.b[stage]), BK * 128, 1024);
          uint64_t ad[4], bd[4];
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            ad[kk] = a0 + kk * 2;    // +32 bytes (32 8-bit elements of K) inside the swizzle row
            bd[kk] = b0 + kk * 256;  // +32 K rows of 128 bytes
          }
          umma4_pair_b8<F8>(d_tmem, ad, bd, kb > 0 ? 1u : 0u, idesc);
          umma_commit_pair(empty0 + stage * 8);
          umma_commit_pair(empty0_peer + stage * 8);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair(tfull0 + acc * 8);
        umma_commit_pair(tfull0_peer + acc * 8);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5, both CTAs) ----------------
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t tempty0_leader = mapa_shared(smem_u32(&s.tempty[0]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair_id; t < num_tiles; t += num_pairs) {
      int mi, ni;
      gemm::tile_coords(t, num_m, num_n, mi, ni);
      const int m0 = mi * TM + (int)rank * 128;
      const int n0 = ni * TN;
      if (!mbar_wait(&s.tfull[acc], acc_phase, site + 3, abort_flag)) break;
      tc_fence_after();
      const int row = m0 + row_in_tile;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * TN;
#pragma unroll 1
      for (int c = 0; c < TN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(t_row + c * 32, r);
        tmem_ld_wait(r);
        const int col0 = n0 + c * 32;
        if (row < M && col0 < N) {
          TOut* crow = C + (size_t)row * N;
          const __nv_bfloat16* rrow = residual ? residual + (size_t)row * N : nullptr;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int col = col0 + g * 8;
            if (col < N) {  // N is a multiple of 16 on this path
              float v[8];
#pragma unroll
              for (int j = 0; j < 8; ++j)
                v[j] = (F8 ? __uint_as_float(r[g * 8 + j]) : (float)(int32_t)r[g * 8 + j]) * scale;
              gemm::epilogue8(v, bias, rrow, crow, col, act);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(tempty0_leader + acc * 8);
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, kTmemCols);
}

// int8: C = float(A . B) * scale (+ bias), fp32 out.
template <int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_s8_tc2_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB, const float* __restrict__ bias,
                       float* __restrict__ C, int M, int N, int K, float scale) {
  pair8_body<STAGES, false, float>(&tmA, &tmB, bias, nullptr, C, M, N, K, scale,
                                   idesc_s8_s32(256, 256, true), kActNone, 84);
}

// fp8 (E4M3 / E5M2 operands, the formats in idesc):
// C = act((A . B) * scale + bias) (+ residual), f32 accumulation, TOut out.
template <int STAGES, typename TOut>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_f8_tc2_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB, const float* __restrict__ bias,
                       const __nv_bfloat16* __restrict__ residual, TOut* __restrict__ C, int M,
                       int N, int K, float scale, uint32_t idesc, int act) {
  pair8_body<STAGES, true, TOut>(&tmA, &tmB, bias, residual, C, M, N, K, scale, idesc, act, 100);
}

// CUDA-core fallback for shapes the tensor-core path does not take (K or N
// not a multiple of 16, unaligned pointers): 16x16 output tiles, K in
// chunks of 64 staged through shared memory, exact int32 accumulation.
__global__ void __launch_bounds__(256) gemm_s8_simt_kernel(const int8_t* __restrict__ A,
                                                           const int8_t* __restrict__ B,
                                                           const float* __restrict__ bias,
                                                           float* __restrict__ C, int M, int N,
                                                           int K, float scale) {
  __shared__ int8_t sa[16][64];
  __shared__ int8_t sb[64][16];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int row = blockIdx.y * 16 + ty, col = blockIdx.x * 16 + tx;
  int32_t acc = 0;
  for (int k0 = 0; k0 < K; k0 += 64) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int r = i >> 6, kk = i & 63;
      const int gr = blockIdx.y * 16 + r, gk = k0 + kk;
      sa[r][kk] = (gr < M && gk < K) ? A[(size_t)gr * K + gk] : (int8_t)0;
      const int br = i >> 4, bc = i & 15;
      const int gbk = k0 + br, gbc = blockIdx.x * 16 + bc;
      sb[br][bc] = (gbk < K && gbc < N) ? B[(size_t)gbk * N + gbc] : (int8_t)0;
    }
    __syncthreads();
#pragma unroll 16
    for (int kk = 0; kk < 64; ++kk) acc += (int32_t)sa[ty][kk] * (int32_t)sb[kk][tx];
    __syncthreads();
  }
  if (row < M && col < N) {
    float v = (float)acc * scale;
    if (bias) v += bias[col];
    C[(size_t)row * N + col] = v;
  }
}

// One 8-bit float (format kFmtE4M3 / kFmtE5M2) to fp32 (exact).
__device__ __forceinline__ float f8_to_f32(uint8_t x, int fmt) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)x, fmt == kFmtE5M2 ? __NV_E5M2 : __NV_E4M3);
  return __half2float(__half(h));
}

// CUDA-core fp8 GEMM for shapes the tensor-core path does not take: 16x16
// output tiles, K in chunks of 64 decoded to fp32 in shared memory, fp32
// accumulation, the same epilogue as the tensor-core path.
template <typename TOut>
__global__ void __launch_bounds__(256) gemm_f8_simt_kernel(
    const uint8_t* __restrict__ A, const uint8_t* __restrict__ B, const float* __restrict__ bias,
    const __nv_bfloat16* __restrict__ residual, TOut* __restrict__ C, int M, int N, int K,
    float scale, int a_fmt, int b_fmt, int act) {
  __shared__ float sa[16][65];
  __shared__ float sb[64][17];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int row = blockIdx.y * 16 + ty, col = blockIdx.x * 16 + tx;
  float acc = 0.0f;
  for (int k0 = 0; k0 < K; k0 += 64) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int r = i >> 6, kk = i & 63;
      const int gr = blockIdx.y * 16 + r, gk = k0 + kk;
      sa[r][kk] = (gr < M && gk < K) ? f8_to_f32(A[(size_t)gr * K + gk], a_fmt) : 0.0f;
      const int br = i >> 4, bc = i & 15;
      const int gbk = k0 + br, gbc = blockIdx.x * 16 + bc;
      sb[br][bc] = (gbk < K && gbc < N) ? f8_to_f32(B[(size_t)gbk * N + gbc], b_fmt) : 0.0f;
    }
    __syncthreads();
#pragma unroll 16
    for (int kk = 0; kk < 64; ++kk) acc = fmaf(sa[ty][kk], sb[kk][tx], acc);
    __syncthreads();
  }
  if (row < M && col < N) {
    float v = acc * scale;
    if (bias) v += bias[col];
    v = act_fast(v, act);
    if (residual) v += __bfloat162float(residual[(size_t)row * N + col]);
    C[(size_t)row * N + col] = from_f32<TOut>(v);
  }
}

// ---------------------------------------------------------------------------
// Element type conversion (the reference's jules.cast as the mixed-precision
// pass inserts it around a matmul): fp32 / bf16 / E4M3 / E5M2 in any
// direction.  To bf16: round to nearest even.  To fp8: round to nearest
// even with saturation to the largest finite value (E4M3 +-448, E5M2
// +-57344); NaN stays NaN.  Codes: 0 fp32, 1 bf16, 2 E4M3, 3 E5M2.
__device__ __forceinline__ float load_as_f32(const void* p, int64_t i, int code) {
  switch (code) {
    case 0: return static_cast<const float*>(p)[i];
    case 1: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    case 2: return f8_to_f32(static_cast<const uint8_t*>(p)[i], kFmtE4M3);
    default: return f8_to_f32(static_cast<const uint8_t*>(p)[i], kFmtE5M2);
  }
}

__device__ __forceinline__ void store_from_f32(void* p, int64_t i, int code, float v) {
  switch (code) {
    case 0: static_cast<float*>(p)[i] = v; break;
    case 1: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    case 2:
      static_cast<uint8_t*>(p)[i] = (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
      break;
    default:
      static_cast<uint8_t*>(p)[i] = (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E5M2);
      break;
  }
}

// Scalar grid-stride form (any alignment).
__global__ void cast_kernel(const void* __restrict__ src, void* __restrict__ dst, int64_t n,
                            int src_code, int dst_code) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    store_from_f32(dst, i, dst_code, load_as_f32(src, i, src_code));
}

// Vector form for fp32 / bf16 -> fp8 with 16-byte aligned buffers and n a
// multiple of 8: 8 elements per thread per step (32 or 16 bytes read, 8
// written), the HBM-bound direction of the cast.
template <typename TIn>
__global__ void cast_to_f8_vec_kernel(const TIn* __restrict__ src, uint8_t* __restrict__ dst,
                                      int64_t n8, int fmt) {
  const __nv_fp8_interpretation_t f = fmt == kFmtE5M2 ? __NV_E5M2 : __NV_E4M3;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v[8];
    if constexpr (std::is_same<TIn, float>::value) {
      const float4 a = reinterpret_cast<const float4*>(src)[2 * i];
      const float4 b = reinterpret_cast<const float4*>(src)[2 * i + 1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
      const uint4 u = reinterpret_cast<const uint4*>(src)[i];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 t = __bfloat1622float2(h[j]);
        v[2 * j] = t.x;
        v[2 * j + 1] = t.y;
      }
    }
    uint2 o;
    uint16_t* op = reinterpret_cast<uint16_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      op[j] = (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(v[2 * j], v[2 * j + 1]), __NV_SATFINITE, f);
    reinterpret_cast<uint2*>(dst)[i] = o;
  }
}

}  // namespace gemm8
}  // namespace jb
