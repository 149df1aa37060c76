// Fused GEMM + bias + activation (+ residual) on tcgen05 tensor cores.
//
//   C[M,N] = act(A[M,K] . W[K,N] + bias[N]) (+ residual[M,N])
//
// A is row-major (K contiguous: the K-major UMMA operand); W is row-major
// [K,N] (N contiguous: the MN-major UMMA operand), exactly the layouts of the
// reference's tiledMatmulWithActivation / fusedMatmulBiasRelu
// (include/jules/Kernel/FusedKernels.h:265-458), so no transposed weight copy
// is needed.  bf16 operands, fp32 accumulation in TMEM, fp32 epilogue, one
// round-to-nearest-even cast to bf16 on store (the mixed-precision rules of
// lib/Passes/MixedPrecisionPass.cpp:350-459,490,632).
//
// Structure (one CTA per SM, persistent over 128 x BN output tiles):
//   warp 0      TMA producer: A box 64x128, W boxes 64x64, 128B swizzle,
//               STAGES-deep smem ring guarded by full/empty mbarriers.
//   warp 1      allocates TMEM (2 x BN fp32 columns) and issues
//               tcgen05.mma (M=128, N=BN, K=16) from one thread; commits free
//               smem stages and signal finished accumulators.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time, bias + activation
//               + residual in fp32, bf16 pack, 16-byte stores.  The two
//               accumulator buffers let the epilogue of tile i overlap the
//               mainloop of tile i+1.
#pragma once

#include "sm100.cuh"

namespace jb {

enum Act : int { kActNone = 0, kActRelu = 1, kActSigmoid = 2, kActTanh = 3, kActGelu = 4 };

// Fast activation for bf16-output epilogues (hardware tanh, ~2^-11 rel).
__device__ __forceinline__ float act_fast(float v, int act) {
  switch (act) {
    case kActRelu: return fmaxf(v, 0.0f);
    case kActSigmoid: return 0.5f + 0.5f * tanh_approx(0.5f * v);
    case kActTanh: return tanh_approx(v);
    case kActGelu: {
      const float u = 0.7978845608f * (v + 0.044715f * v * v * v);
      return 0.5f * v * (1.0f + tanh_approx(u));
    }
    default: return v;
  }
}

// Accurate activations (fp32 outputs): the scalar forms of
// include/jules/Kernel/FusedKernels.h:425-428, 616.
__device__ __forceinline__ float act_exact(float v, int act) {
  switch (act) {
    case 1: return fmaxf(v, 0.0f);
    case 2: return 1.0f / (1.0f + expf(-v));
    case 3: return tanhf(v);
    case 4: return 0.5f * v * (1.0f + tanhf(0.7978845608f * (v + 0.044715f * v * v * v)));
    default: return v;
  }
}

namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle row of bf16
constexpr int kThreads = 192;   // 1-CTA kernel: TMA, MMA, 4 epilogue warps
constexpr int kThreads2 = 320;  // pair kernel: TMA, MMA, 8 epilogue warps

// Tile order shared by both GEMM kernels: groups of kGroupM tile rows; inside
// a group m runs fastest and n advances once per group height, so the tiles
// resident at one time (one per SM or SM pair) cover a compact block of A row
// panels and W column panels that stays in L2 instead of sweeping all of one
// operand per tile row.
constexpr int kGroupM = 16;
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mi, int& ni) {
  const int per_group = kGroupM * num_n;
  const int g = t / per_group;
  const int idx = t - g * per_group;
  const int gm = min(kGroupM, num_m - g * kGroupM);
  mi = g * kGroupM + idx % gm;
  ni = idx / gm;
}

template <int BN, int STAGES>
struct Smem {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BK * BN * 2;
  alignas(1024) uint8_t a[STAGES][kABytes];
  alignas(1024) uint8_t b[STAGES][kBBytes];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint32_t tmem_base;
  int abort_flag;
};

// Stores 8 consecutive fp32 results as bf16 (one 16-byte store) or as fp32
// (two 16-byte stores).
__device__ __forceinline__ void store8(__nv_bfloat16* dst, const float (&v)[8]) {
  uint4 o;
  o.x = pack_bf16x2(v[0], v[1]);
  o.y = pack_bf16x2(v[2], v[3]);
  o.z = pack_bf16x2(v[4], v[5]);
  o.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(dst) = o;
}
__device__ __forceinline__ void store8(__half* dst, const float (&v)[8]) {
  uint4 o;
  o.x = pack_f16x2(v[0], v[1]);
  o.y = pack_f16x2(v[2], v[3]);
  o.z = pack_f16x2(v[4], v[5]);
  o.w = pack_f16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(dst) = o;
}
__device__ __forceinline__ void store8(float* dst, const float (&v)[8]) {
  reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// LayerNorm folded into the GEMM.  With W' = diag(gamma) W,
//   LN(x) . W = rstd * (x . W' - mean * colsum(W')) + beta . W,
// so a GEMM of the raw rows x against W' gives LN(x) . W from the row
// statistics (mean, rstd) and the column sums of W'; beta . W (+ the GEMM's
// own bias) arrives as the bias.  Applied to 8 accumulators of one row.
__device__ __forceinline__ void ln_fold8(float (&v)[8], float2 rs, const float* colsum) {
  const float4 c0 = *reinterpret_cast<const float4*>(colsum);
  const float4 c1 = *reinterpret_cast<const float4*>(colsum + 4);
  const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = rs.y * fmaf(-rs.x, cs[j], v[j]);
}

// TIn: the operands' type, __nv_bfloat16 or __half (the residual has it
// too).  TOut: TIn (one RNE cast at the store) or float.
template <int BN, int STAGES, typename TIn, typename TOut>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmW, const float* __restrict__ bias,
                        const TIn* __restrict__ residual, TOut* __restrict__ C,
                        int M, int N, int K, int act, const float2* __restrict__ ln_stats,
                        const float* __restrict__ ln_colsum) {
  static_assert(BN % 64 == 0 && BN <= 256, "BN must be a multiple of 64, at most 256");
  using S = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  S& s = *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_k = (K + BK - 1) / BK;
  constexpr uint32_t kTmemCols = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));

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
    prefetch_tmap(&tmW);
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
        tile_coords(t, num_m, num_n, mi, ni);
        const int m0 = mi * BM;
        const int n0 = ni * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&s.full[stage], S::kABytes + S::kBBytes);
          tma_load_2d(s.a[stage], &tmA, &s.full[stage], kb * BK, m0);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(s.b[stage] + j * (BK * 64 * 2), &tmW, &s.full[stage], n0 + j * 64, kb * BK);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16kind<TIn>(BM, BN, false, true);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&s.tempty[acc], acc_phase ^ 1u, 2, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, 3, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(s.a[stage]);
          const uint32_t b_base = smem_u32(s.b[stage]);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // K-major A: advance 16 elements = 32 bytes inside the swizzle row.
            const uint64_t ad = sdesc_sw128(a_base + kk * 32, 16, 1024);
            // MN-major W: advance 16 K-rows = 2048 bytes; 64-col chunks 8 KB apart.
            const uint64_t bd = sdesc_sw128(b_base + kk * 2048, BK * 64 * 2, 1024);
            umma_f16_ss(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
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
      tile_coords(t, num_m, num_n, mi, ni);
      const int m0 = mi * BM;
      const int n0 = ni * BN;
      if (!mbar_wait(&s.tfull[acc], acc_phase, 4, abort_flag)) break;
      tc_fence_after();
      const int row = m0 + row_in_tile;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      const float2 rs = ln_stats && row < M ? ln_stats[row] : make_float2(0.0f, 1.0f);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(t_row + c * 32, r);
        tmem_ld_wait(r);
        const int col0 = n0 + c * 32;
        if (row < M && col0 < N) {
          TOut* crow = C + (size_t)row * N;
          const TIn* rrow = residual ? residual + (size_t)row * N : nullptr;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int col = col0 + g * 8;
            if (col < N) {  // N is a multiple of 8 on this path
              float v[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(r[g * 8 + j]);
              if (ln_stats) ln_fold8(v, rs, ln_colsum + col);
              if (bias) {
                const float4 b0 = *reinterpret_cast<const float4*>(bias + col);
                const float4 b1 = *reinterpret_cast<const float4*>(bias + col + 4);
                v[0] += b0.x; v[1] += b0.y; v[2] += b0.z; v[3] += b0.w;
                v[4] += b1.x; v[5] += b1.y; v[6] += b1.z; v[7] += b1.w;
              }
#pragma unroll
              for (int j = 0; j < 8; ++j) v[j] = act_fast(v[j], act);
              if (rrow) {
                const uint4 rv = *reinterpret_cast<const uint4*>(rrow + col);
                const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float2 f = unpack2<TIn>(rw[j]);
                  v[2 * j] += f.x;
                  v[2 * j + 1] += f.y;
                }
              }
              store8(crow + col, v);
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

// ---------------------------------------------------------------------------
// CTA-pair version.  A cluster of two CTAs computes a 256 x 256 output tile
// with cta_group::2 MMAs (M=256, N=256, K=16): each CTA stages its own 128
// rows of A and its own 128 columns of W per k-block, the pair's tensor cores
// exchange the W halves, and each CTA's TMEM receives its 128 rows x 256
// columns of D.  Per SM and k-block this moves 32 KB into shared memory
// instead of 48 KB for the same MMA work, which is what the single-CTA kernel
// is bound by.
//   warp 0 (both CTAs)  TMA: own A rows and W columns; the bytes complete on
//                       the leader CTA's full barrier.
//   warp 1 (leader)     MMA issue; commits free the stage in both CTAs and
//                       mark the accumulator ready in both CTAs.
//   warps 2-9 (both)    epilogue of the CTA's 128 rows, two warps per TMEM
//                       lane quarter; they release the accumulator on the
//                       leader's barrier (512 arrivals).
//
// Tail split.  With T tiles on P resident pairs, the last round holds only
// r = T mod P tiles (all T when T < P).  When 2r <= P, those r tiles are run
// as 2r half-width units of 256 x 128 (M=256, N=128 MMAs over the full K), so
// the last round takes about half as long.  The halves are independent
// output tiles: nothing is combined, no scratch memory, no counters.
// ---------------------------------------------------------------------------
template <int STAGES, int TN>
struct Smem2 {
  static constexpr int kABytes = 128 * BK * 2;     // this CTA's 128 rows of A
  static constexpr int kBBytes = BK * (TN / 2) * 2;  // this CTA's TN/2 columns of W
  alignas(1024) uint8_t a[STAGES][kABytes];
  alignas(1024) uint8_t b[STAGES][kBBytes];
  // Epilogue staging: 4 KB per epilogue warp (32 rows of 128 bytes, their
  // 16-byte chunks XOR-swizzled by row & 7).
  alignas(128) float epi[8][32][32];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint32_t tmem_base;
  int abort_flag;
};

// Where the pair kernel's epilogue writes C: the local C (c[0]) and, for the
// sharded GEMM with the gather fused in, the same rows of every other rank's
// C mapped into this process (c[1..n-1]).  Local row r of the tile grid is
// row row_off + r of every C; A and the residual use local rows.  mc, when
// set, is C's NVLink multicast address (all ranks' C behind one address):
// each 16-byte chunk is then stored once and the switch writes it into every
// rank's C, instead of n stores over n links.
constexpr int kMaxOutDest = kMaxPeers;
template <typename TOut>
struct OutDest {
  TOut* c[kMaxOutDest];
  TOut* mc;
  int n;
  int row_off;
};

// Work unit u of the tail-split schedule: whole tiles first, then the two
// column halves of each tail tile.  n_off is the unit's first column inside
// its tile, cols its width (TN or TN/2).
struct PairUnit {
  int tile, n_off, cols;
};
template <int TN>
__device__ __forceinline__ PairUnit pair_unit(int u, int whole_units) {
  PairUnit r;
  if (u < whole_units) {
    r.tile = u;
    r.n_off = 0;
    r.cols = TN;
  } else {
    const int v = u - whole_units;
    r.tile = whole_units + (v >> 1);
    r.n_off = (v & 1) * (TN / 2);
    r.cols = TN / 2;
  }
  return r;
}

// Per-thread epilogue math for 8 consecutive columns of one row: bias,
// activation, residual, store (the 8-bit pair kernels).
template <typename TOut>
__device__ __forceinline__ void epilogue8(float (&v)[8], const float* bias,
                                          const __nv_bfloat16* rrow, TOut* crow, int col,
                                          int act) {
  if (bias) {
    const float4 b0 = *reinterpret_cast<const float4*>(bias + col);
    const float4 b1 = *reinterpret_cast<const float4*>(bias + col + 4);
    v[0] += b0.x; v[1] += b0.y; v[2] += b0.z; v[3] += b0.w;
    v[4] += b1.x; v[5] += b1.y; v[6] += b1.z; v[7] += b1.w;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = act_fast(v[j], act);
  if (rrow) {
    const uint4 rv = *reinterpret_cast<const uint4*>(rrow + col);
    const __nv_bfloat162* rp = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(rp[j]);
      v[2 * j] += f.x;
      v[2 * j + 1] += f.y;
    }
  }
  store8(crow + col, v);
}

// whole_units: tiles run at full width; num_units: whole_units + 2 x the
// number of tail tiles run as halves (== whole_units when nothing is split).
template <int STAGES, int TN, typename TIn, typename TOut>
__global__ void __launch_bounds__(kThreads2, 1)
    gemm_bf16_tc2_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmW, const float* __restrict__ bias,
                         const TIn* __restrict__ residual, const OutDest<TOut> out,
                         int M, int N, int K, int act, int whole_units, int num_units,
                         const float2* __restrict__ ln_stats, const float* __restrict__ ln_colsum) {
  static_assert(TN == 256, "pair tile N is 256 (its halves are 128)");
  constexpr int TM = 256;
  constexpr uint32_t kTmemCols = 2 * TN;  // two accumulators
  using S = Smem2<STAGES, TN>;
  // Operand bytes: 2 (bf16 / f16, kind::f16) or 4 (fp32 read as tf32,
  // kind::tf32).  A k-block is one 128-byte swizzle row of K (BKe elements);
  // a W box is one 128-byte row of N (also BKe elements); the stage sizes in
  // bytes are the same for both.
  constexpr int kE = (int)sizeof(TIn);
  constexpr int BKe = 128 / kE;
  static_assert(S::kABytes == 128 * BKe * kE && S::kBBytes == BKe * (TN / 2) * kE, "stage layout");
  // B operand: 16-bit W is read MN-major straight from [K,N]; the tf32 MMAs
  // take B K-major, so fp32 W comes transposed ([N,K], rows of K like A) in
  // boxes of 64 N rows.
  constexpr bool kBKMajor = kE == 4;
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
  const int num_k = (K + BKe - 1) / BKe;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], 2 * 256);
    }
    s.abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
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
      for (int u = pair_id; u < num_units && ok; u += num_pairs) {
        const PairUnit pu = pair_unit<TN>(u, whole_units);
        int mi, ni;
        tile_coords(pu.tile, num_m, num_n, mi, ni);
        const int cta_cols = pu.cols / 2;  // this CTA's share of the unit's W columns
        const int m0 = mi * TM + (int)rank * 128;
        const int n0 = ni * TN + pu.n_off + (int)rank * cta_cols;
        const uint32_t tx = 2u * (uint32_t)(S::kABytes + BKe * cta_cols * kE);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, 41, abort_flag)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&s.full[stage], tx);
          tma_load_2d_pair(s.a[stage], &tmA, &s.full[stage], kb * BKe, m0);
          if constexpr (kBKMajor) {
            for (int j = 0; j < cta_cols / 64; ++j)
              tma_load_2d_pair(s.b[stage] + j * (64 * 128), &tmW, &s.full[stage], kb * BKe, n0 + j * 64);
          } else {
            for (int j = 0; j < cta_cols / BKe; ++j)
              tma_load_2d_pair(s.b[stage] + j * (BKe * 128), &tmW, &s.full[stage], n0 + j * BKe, kb * BKe);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA) ----------------
    if (leader && lane == 0) {
      constexpr uint32_t idesc_full = idesc_f16kind<TIn>(TM, TN, false, !kBKMajor);
      constexpr uint32_t idesc_half = idesc_f16kind<TIn>(TM, TN / 2, false, !kBKMajor);
      const uint32_t empty0 = smem_u32(&s.empty[0]);
      const uint32_t tfull0 = smem_u32(&s.tfull[0]);
      const uint32_t empty0_peer = mapa_shared(empty0, 1);
      const uint32_t tfull0_peer = mapa_shared(tfull0, 1);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = pair_id; u < num_units && ok; u += num_pairs) {
        const PairUnit pu = pair_unit<TN>(u, whole_units);
        const uint32_t idesc = pu.cols == TN ? idesc_full : idesc_half;
        if (!mbar_wait(&s.tempty[acc], acc_phase ^ 1u, 42, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * TN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, 43, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t a0 = sdesc_sw128(smem_u32(s.a[stage]), 16, 1024);
          const uint64_t b0 = kBKMajor ? sdesc_sw128(smem_u32(s.b[stage]), 16, 1024)
                                       : sdesc_sw128(smem_u32(s.b[stage]), BKe * 128, 1024);
          uint64_t ad[4], bd[4];
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            ad[kk] = a0 + kk * 2;  // +32 bytes (one MMA's K) inside the swizzle row
            // K-major B like A; MN-major B: +16 K rows of 128 bytes
            bd[kk] = kBKMajor ? b0 + kk * 2 : b0 + kk * 128;
          }
          if constexpr (kE == 4)
            umma4_pair_ss_tf32(d_tmem, ad, bd, kb > 0 ? 1u : 0u, idesc);
          else
            umma4_pair_ss(d_tmem, ad, bd, kb > 0 ? 1u : 0u, idesc);
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
    // ---------------- epilogue (warps 2..9, both CTAs) ----------------
    // Each warp owns 32 rows (its TMEM lane quarter).  tcgen05.ld gives lane t
    // row t; bias, activation and residual are applied in that layout, the
    // results go through shared memory (4 KB per warp, 16-byte chunks
    // XOR-swizzled by row) and are read back so that 8 lanes cover 128
    // contiguous bytes of one row: every store writes 16 bytes, every
    // 8 lanes a whole 128-byte line, local or across NVLink.
    //   16-bit C: blocks of 64 columns (32 rows x 128 B); fp32 C: 32 columns.
    // Eight epilogue warps: two per TMEM lane quarter (warp & 3), each taking
    // half of the unit's columns (chalf).
    constexpr int kBlk = sizeof(TOut) == 2 ? 64 : 32;  // columns per staged block
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int chalf = ew >> 2;
    uint4* stage = reinterpret_cast<uint4*>(s.epi[ew]);  // [32 rows][8 chunks of 16 B]
    const int g = lane & 7;      // chunk (8 bf16 / 4 fp32 columns) this lane stores
    const int rsub = lane >> 3;  // first row this lane stores
    const uint32_t tempty0_leader = mapa_shared(smem_u32(&s.tempty[0]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = pair_id; u < num_units; u += num_pairs) {
      const PairUnit pu = pair_unit<TN>(u, whole_units);
      int mi, ni;
      tile_coords(pu.tile, num_m, num_n, mi, ni);
      const int m0 = mi * TM + (int)rank * 128 + quarter * 32;  // first row of this warp
      const int n0 = ni * TN + pu.n_off;
      if (!mbar_wait(&s.tfull[acc], acc_phase, 44, abort_flag)) break;
      tc_fence_after();
      const uint32_t t_warp = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * TN;
      const int my_row = m0 + lane;  // row of this lane in the TMEM layout
      const TIn* rrow = residual ? residual + (size_t)(my_row < M ? my_row : 0) * N : nullptr;
      const float2 rs = ln_stats && my_row < M ? ln_stats[my_row] : make_float2(0.0f, 1.0f);
#pragma unroll 1
      for (int cb = chalf * (pu.cols / 2); cb < (chalf + 1) * (pu.cols / 2); cb += kBlk) {
#pragma unroll
        for (int h = 0; h < kBlk / 32; ++h) {
          const int c0 = n0 + cb + h * 32;  // first column of these 32
          uint32_t r[32];
          tmem_ld32(t_warp + cb + h * 32, r);
          tmem_ld_wait(r);
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          if (c0 < N) {  // N is a multiple of 8: a 32-column group is all in or starts past N
            if constexpr (kE == 4) {
              // fp32 operands (3xTF32 by K chunks): `residual` is the fp32
              // sum of the earlier chunks (C itself, read here before this
              // warp's stores write it), added before bias and activation
              if (rrow) {
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                  if (c0 + j < N) {
                    const float4 p = *reinterpret_cast<const float4*>(rrow + c0 + j);
                    v[j] += p.x; v[j + 1] += p.y; v[j + 2] += p.z; v[j + 3] += p.w;
                  }
                }
              }
            }
            if (ln_stats) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                if (c0 + j < N) {
                  float w8[8];
#pragma unroll
                  for (int q = 0; q < 8; ++q) w8[q] = v[j + q];
                  ln_fold8(w8, rs, ln_colsum + c0 + j);
#pragma unroll
                  for (int q = 0; q < 8; ++q) v[j + q] = w8[q];
                }
              }
            }
            if (bias) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                if (c0 + j < N) {
                  const float4 bv = *reinterpret_cast<const float4*>(bias + c0 + j);
                  v[j] += bv.x; v[j + 1] += bv.y; v[j + 2] += bv.z; v[j + 3] += bv.w;
                }
              }
            }
            if constexpr (kE == 4) {  // fp32 operands (3xTF32): fp32-accurate activations
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = act_exact(v[j], act);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = act_fast(v[j], act);
            }
            if constexpr (kE == 2) {  // residual: 16-bit operands only
              if (rrow) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) {
                  if (c0 + j < N) {
                    const uint4 rv = *reinterpret_cast<const uint4*>(rrow + c0 + j);
                    const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                      const float2 f = unpack2<TIn>(rw[q]);
                      v[j + 2 * q] += f.x;
                      v[j + 2 * q + 1] += f.y;
                    }
                  }
                }
              }
            }
          }
          // this lane's row, chunks h*4 .. h*4+3 (bf16) or 0 .. 7 (fp32)
          if constexpr (sizeof(TOut) == 2) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              stage[lane * 8 + ((h * 4 + q) ^ (lane & 7))] =
                  make_uint4(pack2<TOut>(v[8 * q], v[8 * q + 1]), pack2<TOut>(v[8 * q + 2], v[8 * q + 3]),
                             pack2<TOut>(v[8 * q + 4], v[8 * q + 5]), pack2<TOut>(v[8 * q + 6], v[8 * q + 7]));
          } else {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              stage[lane * 8 + (q ^ (lane & 7))] =
                  make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                             __float_as_uint(v[4 * q + 2]), __float_as_uint(v[4 * q + 3]));
          }
        }
        __syncwarp();
        const int col = n0 + cb + g * (16 / (int)sizeof(TOut));
        if (col < N) {
#pragma unroll 4
          for (int i = 0; i < 8; ++i) {
            const int rr = rsub + 4 * i;
            const int row = m0 + rr;
            if (row >= M) break;  // rows only grow with i
            const uint4 val = stage[rr * 8 + (g ^ (rr & 7))];
            const size_t off = (size_t)(out.row_off + row) * N + col;
            if (out.mc) {
              multimem_st16(out.mc + off, val);
            } else {
#pragma unroll
              for (int p = 0; p < kMaxOutDest; ++p)
                if (p < out.n) *reinterpret_cast<uint4*>(out.c[p] + off) = val;
            }
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      mbar_arrive_cluster(tempty0_leader + acc * 8);
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
    // Peer stores must be visible system-wide before this rank signals the
    // others that its rows are in place (dist_signal_wait_kernel).
    if (out.mc) fence_proxy_alias();
    if (out.n > 1) __threadfence_system();
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, kTmemCols);
}

}  // namespace gemm
}  // namespace jb
