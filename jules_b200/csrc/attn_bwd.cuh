// Flash-attention backward on tcgen05 tensor cores (bf16, head_dim 128).
//
// Gradients of O = softmax(scale * Q K^T [causal mask]) V for dO given,
// from the forward's logsumexp (no second softmax pass):
//   P_ij  = exp(scale * q_i . k_j - lse_i)
//   dV_j  = sum_i P_ij dO_i             dP_ij = dO_i . v_j
//   dS_ij = P_ij (dP_ij - D_i),         D_i   = dO_i . O_i
//   dQ_i  = scale * sum_j dS_ij k_j     dK_j  = scale * sum_i dS_ij q_i
// Grouped-query heads: dK and dV of a kv head sum over the Hq/Hkv query
// heads that read it.  (The reference has no backward for attention; this is
// the gradient of the forward in attn_tc.cuh, whose recurrence follows the
// reference's flashAttention, include/jules/Kernel/FlashAttention.h:130-309.)
//
// Three kernels, no atomics (the gradients are deterministic):
//  * bwd_prep_kernel: per query row, -lse * log2(e) and -D = -dO . O into a
//    workspace padded to whole 128-row tiles (padding rows get -inf, so
//    their P is 0, and 0).
//  * bwd_dkdv_kernel: one CTA per (kv head, 128-key tile j), K_j and V_j
//    resident; for each (query head of the group, query tile i):
//      S^T = K_j Q_i^T and dP^T = V_j dO_i^T into TMEM (rows = keys),
//      softmax warps: P^T, dS^T as bf16 back into TMEM over S^T / dP^T,
//      dV += P^T dO_i and dK += dS^T Q_i with the A operand in TMEM.
//  * bwd_dq_kernel: one CTA per (query head, 128-query tile i), Q_i and dO_i
//    resident in TMEM; for each key tile j: S = Q_i K_j^T, dP = dO_i V_j^T,
//    dS into TMEM, dQ += dS K_j.
// (dQ kernel: Q_i and dO_i are copied into TMEM [384, 512) by the softmax
// warps, so S and dP read only K and V from shared memory.)
// Warp roles (10 warps): 0-7 softmax/epilogue (thread = TMEM lane = tile row;
// warps w and w+4 share a lane quarter and split its 128 columns), 8 TMA
// producer, 9 MMA issuer and TMEM owner.
// Ping-pong: each 128-row tile of the streamed operand is processed as two
// 64-row halves h = 0, 1 with their own S and dP in TMEM, so softmax group h
// (warps 4h..4h+3, thread = TMEM lane = tile row) works on half h while the
// tensor core runs the other half's gradient MMAs and next-tile S / dP.
// TMEM (512 columns): half h's S at [128h, +64) and dP at [128h + 64, +64);
// accumulators at [256, 384) and (dK/dV kernel) [384, 512).  The softmax
// writes its packed bf16 results into columns it has already read: P (dK/dV
// kernel) or dS (dQ kernel) over S, dS of the dK/dV kernel over dP.  The
// next S of a half overwrites them only after the MMAs reading them: one
// thread issues all MMAs and the tensor core runs them in issue order.
#pragma once

#include "attn_tc.cuh"
#include "simt.cuh"
#include "sm100.cuh"

namespace jb {
namespace attn_bwd {

constexpr int HD = 128;
constexpr int BT = 128;                 // rows per query / key tile
constexpr int BH2 = 64;                 // half tile: the unit of the softmax ping-pong
constexpr int kThreads = 320;
constexpr int kSoftmaxThreads = 256;    // warps 0-7: two per TMEM lane quarter
constexpr int kWarpProducer = 8;
constexpr int kWarpMma = 9;
constexpr int kChunk = 128 * 64 * 2;    // one 64-dim (128 B) swizzled box of 128 rows
constexpr int QS = 2;                   // Q / dO ring depth (dK/dV kernel)
constexpr int KS = 2;                   // K / V ring depth (dQ kernel)
constexpr float kLog2e = 1.4426950408889634f;

__host__ __device__ constexpr int padded_len(int S) { return (S + BT - 1) / BT * BT; }

// ---------------------------------------------------------------------------
// nlse2[bh, q] = -lse * log2(e), ndelta[bh, q] = -sum_d dO * O (fp32,
// negated for the fused multiply-adds of the kernels below); rows q in
// [S, Sp) are padding (nlse2 = -inf: their P is 0).  One warp per row, 4
// dims per lane.
__global__ void __launch_bounds__(256) bwd_prep_kernel(const __nv_bfloat16* __restrict__ O,
                                                       const __nv_bfloat16* __restrict__ dO,
                                                       const float* __restrict__ lse,
                                                       float* __restrict__ lse2,
                                                       float* __restrict__ delta, int BH, int S,
                                                       int Sp) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)BH * Sp;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int bh = (int)(row / Sp), q = (int)(row - (int64_t)bh * Sp);
    float d = 0.0f;
    if (q < S) {
      const size_t off = ((size_t)bh * S + q) * HD + lane * 4;
      const uint2 a = *reinterpret_cast<const uint2*>(O + off);
      const uint2 b = *reinterpret_cast<const uint2*>(dO + off);
      const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float2 x = __bfloat1622float2(a2[k]), y = __bfloat1622float2(b2[k]);
        d = fmaf(x.x, y.x, d);
        d = fmaf(x.y, y.y, d);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    }
    if (lane == 0) {
      lse2[row] = q < S ? -lse[(size_t)bh * S + q] * kLog2e : -INFINITY;
      delta[row] = -d;
    }
  }
}

__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 32 columns of S and dP (fp32) -> 16 columns of packed bf16 P and dS, two
// columns per f32x2 instruction:
//   x = s * scale*log2(e) + nlse2,  p = 2^x,  ds = p * (dp + ndelta).
// nl2 / nd2: the pair's -lse*log2(e) and -D (per column pair in the dK/dV
// kernel, the row's own value twice in the dQ kernel).  Masked scores arrive
// as -inf (p = 0).
template <bool WANT_P, typename PairF>
__device__ __forceinline__ void p_ds_chunk(const uint32_t (&s)[32], const uint32_t (&dp)[32],
                                           uint64_t scale2, PairF pair_at, uint32_t (&pk_p)[16],
                                           uint32_t (&pk_ds)[16]) {
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    uint64_t nl2, nd2;
    pair_at(2 * e, nl2, nd2);
    const uint64_t x2 = attn::fma2(attn::pk2(__uint_as_float(s[2 * e]), __uint_as_float(s[2 * e + 1])),
                                   scale2, nl2);
    float x0, x1;
    attn::upk2(x2, x0, x1);
    const uint64_t p2 = attn::pk2(ex2_approx(x0), ex2_approx(x1));
    const uint64_t g2 = attn::add2(attn::pk2(__uint_as_float(dp[2 * e]), __uint_as_float(dp[2 * e + 1])), nd2);
    const uint64_t ds2 = mul2(p2, g2);
    float a0, a1;
    if (WANT_P) {
      attn::upk2(p2, a0, a1);
      pk_p[e] = pack_bf16x2(a0, a1);
    }
    attn::upk2(ds2, a0, a1);
    pk_ds[e] = pack_bf16x2(a0, a1);
  }
}

// D (+)= sum over 4 K-steps of A[tmem] * B[smem].
__device__ __forceinline__ void umma4_ts(uint32_t d_tmem, const uint32_t (&a)[4],
                                         const uint64_t (&b)[4], uint32_t acc_first,
                                         uint32_t idesc) {
  umma_f16_ts(d_tmem, a[0], b[0], idesc, acc_first);
  umma_f16_ts(d_tmem, a[1], b[1], idesc, 1u);
  umma_f16_ts(d_tmem, a[2], b[2], idesc, 1u);
  umma_f16_ts(d_tmem, a[3], b[3], idesc, 1u);
}

// Causal / padding masks of one 32-column chunk: columns c >= lim, or
// c < lo, get -inf scores.  (One limit per row: a per-column predicate
// measured ~5x slower on the masked tiles.)
__device__ __forceinline__ void mask_from(uint32_t (&s)[32], int lim) {
#pragma unroll
  for (int c = 0; c < 32; ++c)
    if (c >= lim) s[c] = __float_as_uint(-INFINITY);
}
__device__ __forceinline__ void mask_below(uint32_t (&s)[32], int lo) {
#pragma unroll
  for (int c = 0; c < 32; ++c)
    if (c < lo) s[c] = __float_as_uint(-INFINITY);
}

// Stores 64 columns [c_begin, c_begin + 64) of a fp32 accumulator row
// (TMEM) as bf16 times mul.
__device__ __forceinline__ void store_row_bf16(uint32_t trow, __nv_bfloat16* dst, float mul,
                                               bool ok, int c_begin) {
#pragma unroll 1
  for (int c = c_begin; c < c_begin + 64; c += 32) {
    uint32_t o[32];
    tmem_ld32(trow + c, o);
    tmem_ld_wait(o);
    if (ok) {
      uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint4 v;
        v.x = pack_bf16x2(__uint_as_float(o[8 * g + 0]) * mul, __uint_as_float(o[8 * g + 1]) * mul);
        v.y = pack_bf16x2(__uint_as_float(o[8 * g + 2]) * mul, __uint_as_float(o[8 * g + 3]) * mul);
        v.z = pack_bf16x2(__uint_as_float(o[8 * g + 4]) * mul, __uint_as_float(o[8 * g + 5]) * mul);
        v.w = pack_bf16x2(__uint_as_float(o[8 * g + 6]) * mul, __uint_as_float(o[8 * g + 7]) * mul);
        d4[g] = v;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// dK / dV
// ---------------------------------------------------------------------------
struct SmemKV {
  alignas(1024) uint8_t k[2][kChunk];
  alignas(1024) uint8_t v[2][kChunk];
  alignas(1024) uint8_t q[QS][2][kChunk];
  alignas(1024) uint8_t dO[QS][2][kChunk];
  alignas(16) float lse2[QS][BT];
  alignas(16) float delta[QS][BT];
  uint64_t kv_full;
  uint64_t q_full[QS], q_empty[QS];
  uint64_t s_full[2], p_full[2], acc_full;
  uint32_t tmem_base;
  int abort_flag;
};

// Work order shared by both kernels: items (head, tile) come in groups of
// G consecutive heads; inside a group the tiles run longest-causal-first and,
// for each tile, the G heads back to back.  The ~148 CTAs resident at a time
// then stream the operands of a few heads (2 MB per head at S = 4096), which
// stay in L2, instead of one head each.  longest_first: tile 0 (key tiles,
// the dK/dV kernel) or tile n_t - 1 (query tiles, the dQ kernel) first.
__device__ __forceinline__ void decode_bwd_item(int w, int n_t, int heads, int G, bool causal,
                                                bool low_first, int& tile, int& head) {
  const int per_group = G * n_t;
  const int g = w / per_group;
  const int idx = w - g * per_group;
  const int gh = min(G, heads - g * G);
  const int r = idx / gh;
  head = g * G + (idx - r * gh);
  tile = (!causal || low_first) ? r : n_t - 1 - r;
}

// Query tiles of one work item: (query head h of the group, tile i), i from
// the diagonal (causal) or 0, heads outer.
__device__ __forceinline__ void kv_item_tile(int it, int i0, int n_qt, int& hh, int& i) {
  const int per_head = n_qt - i0;
  hh = it / per_head;
  i = i0 + (it - hh * per_head);
}

__global__ void __launch_bounds__(kThreads, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                    const float* __restrict__ lse2, const float* __restrict__ delta,
                    __nv_bfloat16* __restrict__ dK, __nv_bfloat16* __restrict__ dV, int B, int Hq,
                    int Hkv, int S, float scale, int causal) {
  extern __shared__ uint8_t smem_raw[];
  SmemKV& s = *reinterpret_cast<SmemKV*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                         ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int Sp = padded_len(S);
  const int n_t = Sp / BT;
  const int BHkv = B * Hkv;
  const int group = Hq / Hkv;
  // Work item: key tile j (0 = the longest under the causal mask) x kv head.
  int j, zkv;
  decode_bwd_item(blockIdx.x, n_t, BHkv, 8, causal != 0, true, j, zkv);
  const int b = zkv / Hkv, g = zkv - b * Hkv;
  const int i0 = causal ? j : 0;
  const int n_it = group * (n_t - i0);
  const float scale_log2 = scale * kLog2e;

  if (threadIdx.x == 0) {
    mbar_init(&s.kv_full, 1);
    for (int k = 0; k < QS; ++k) {
      mbar_init(&s.q_full[k], 1);
      mbar_init(&s.q_empty[k], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s.s_full[x], 1);
      mbar_init(&s.p_full[x], kSoftmaxThreads / 2);
    }
    mbar_init(&s.acc_full, 1);
    s.abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmdO);
  }
  if (warp == kWarpMma) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;

  if (warp == kWarpProducer) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&s.kv_full, 4 * kChunk);
      tma_load_3d(s.k[0], &tmK, &s.kv_full, 0, j * BT, zkv);
      tma_load_3d(s.k[1], &tmK, &s.kv_full, 64, j * BT, zkv);
      tma_load_3d(s.v[0], &tmV, &s.kv_full, 0, j * BT, zkv);
      tma_load_3d(s.v[1], &tmV, &s.kv_full, 64, j * BT, zkv);
      for (int it = 0; it < n_it; ++it) {
        int hh, i;
        kv_item_tile(it, i0, n_t, hh, i);
        const int bhq = b * Hq + g * group + hh;
        const int st = it % QS;
        const uint32_t ph = (uint32_t)(it / QS) & 1u;
        if (!mbar_wait(&s.q_empty[st], ph ^ 1u, 110, abort_flag)) break;
        mbar_arrive_expect_tx(&s.q_full[st], 4 * kChunk + 2 * BT * 4);
        tma_load_3d(s.q[st][0], &tmQ, &s.q_full[st], 0, i * BT, bhq);
        tma_load_3d(s.q[st][1], &tmQ, &s.q_full[st], 64, i * BT, bhq);
        tma_load_3d(s.dO[st][0], &tmdO, &s.q_full[st], 0, i * BT, bhq);
        tma_load_3d(s.dO[st][1], &tmdO, &s.q_full[st], 64, i * BT, bhq);
        const size_t off = (size_t)bhq * Sp + (size_t)i * BT;
        bulk_load(s.lse2[st], lse2 + off, BT * 4, &s.q_full[st]);
        bulk_load(s.delta[st], delta + off, BT * 4, &s.q_full[st]);
      }
    }
  } else if (warp == kWarpMma) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(BT, BH2, false, false);
      constexpr uint32_t idG = idesc_bf16_f32(BT, HD, false, true);
      constexpr uint64_t kChunkStep = kChunk >> 4;
      constexpr uint64_t kStageStep = (2 * kChunk) >> 4;
      constexpr uint64_t kHalfRows = (BH2 * 128) >> 4;  // 64 rows of 128 bytes
      // K-major descriptors (+2 per 32 bytes of K) and MN-major ones for
      // Q / dO as the B operand of dK / dV (+128 per 16 rows of 128 bytes).
      const uint64_t dk = sdesc_sw128(smem_u32(s.k[0]), 16, 1024);
      const uint64_t dv = sdesc_sw128(smem_u32(s.v[0]), 16, 1024);
      const uint64_t dq_k = sdesc_sw128(smem_u32(s.q[0][0]), 16, 1024);
      const uint64_t ddo_k = sdesc_sw128(smem_u32(s.dO[0][0]), 16, 1024);
      const uint64_t dq_mn = sdesc_sw128(smem_u32(s.q[0][0]), kChunk, 1024);
      const uint64_t ddo_mn = sdesc_sw128(smem_u32(s.dO[0][0]), kChunk, 1024);
      // S^T_x = K Q_x^T and dP^T_x = V dO_x^T for query half x of stage st.
      auto issue_s = [&](int x, int st) {
        uint64_t a[8], b[8];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t o = (kk >> 2) * kChunkStep + (kk & 3) * 2;
          a[kk] = dk + o;
          b[kk] = dq_k + st * kStageStep + x * kHalfRows + o;
        }
        umma8_ss(tbase + 128 * x, a, b, 0u, idS);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t o = (kk >> 2) * kChunkStep + (kk & 3) * 2;
          a[kk] = dv + o;
          b[kk] = ddo_k + st * kStageStep + x * kHalfRows + o;
        }
        umma8_ss(tbase + 128 * x + 64, a, b, 0u, idS);
        umma_commit(&s.s_full[x]);
      };
      // dV += P^T_x dO_x, dK += dS^T_x Q_x (A in TMEM, K = the half's 64 queries).
      auto issue_g = [&](int x, int st, uint32_t acc) {
        uint32_t ta[4];
        uint64_t b[4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          ta[kk] = tbase + 128 * x + kk * 8;
          b[kk] = ddo_mn + st * kStageStep + x * kHalfRows + kk * 128;
        }
        umma4_ts(tbase + 256, ta, b, acc, idG);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          ta[kk] = tbase + 128 * x + 64 + kk * 8;
          b[kk] = dq_mn + st * kStageStep + x * kHalfRows + kk * 128;
        }
        umma4_ts(tbase + 384, ta, b, acc, idG);
      };
      bool ok = mbar_wait(&s.kv_full, 0, 111, abort_flag) &&
                mbar_wait(&s.q_full[0], 0, 112, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
      }
      // Ping-pong: while softmax group x works on half x of query tile it,
      // the tensor core runs the other half's gradient and next-tile MMAs.
      for (int it = 0; it < n_it && ok; ++it) {
        const int st = it % QS;
        const bool more = it + 1 < n_it;
        const int st1 = (it + 1) % QS;
        const uint32_t ph1 = (uint32_t)((it + 1) / QS) & 1u;
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (!mbar_wait(&s.p_full[x], (uint32_t)it & 1u, 113, abort_flag)) { ok = false; break; }
          tc_fence_after();
          issue_g(x, st, (it > 0 || x > 0) ? 1u : 0u);
          if (x == 1) umma_commit(&s.q_empty[st]);
          if (more) {
            if (x == 0) {
              if (!mbar_wait(&s.q_full[st1], ph1, 117, abort_flag)) { ok = false; break; }
              tc_fence_after();
            }
            issue_s(x, st1);
          }
        }
      }
      umma_commit(&s.acc_full);
    }
  } else {
    // ---------------- softmax / epilogue: thread = key row ----------------
    // Group half (warps 4*half .. 4*half+3) owns query half `half` of every
    // tile: S^T at TMEM columns [128 half, +64), dP^T at [128 half + 64, +64).
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tbase + 128 * half + lane_off, tP = tS + 64;
    const uint64_t scale2 = attn::pk2(scale_log2, scale_log2);
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      int hh, i;
      kv_item_tile(it, i0, n_t, hh, i);
      const int st = it % QS;
      const uint32_t ph = (uint32_t)(it / QS) & 1u;
      // lse2 / delta arrived with q_full (async proxy): observe it directly.
      if (!mbar_wait(&s.q_full[st], ph, 114, abort_flag)) { ok = false; break; }
      if (!mbar_wait(&s.s_full[half], (uint32_t)it & 1u, 115, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const bool diag = causal && i == j;  // query q < key r is masked
      const uint64_t* nl = reinterpret_cast<const uint64_t*>(s.lse2[st] + BH2 * half);
      const uint64_t* nd = reinterpret_cast<const uint64_t*>(s.delta[st] + BH2 * half);
      const int qh = BH2 * half;  // first query of this half within the tile
#pragma unroll 1
      for (int c0 = 0; c0 < BH2; c0 += 32) {
        uint32_t sv[32], dv[32];
        tmem_ld32(tS + c0, sv);
        tmem_ld32(tP + c0, dv);
        tmem_ld_wait(sv);
        tmem_ld_wait(dv);
        if (diag) mask_below(sv, r - qh - c0);  // queries before key r are masked
        uint32_t pk_p[16], pk_ds[16];
        p_ds_chunk<true>(sv, dv, scale2,
                         [&](int c, uint64_t& l, uint64_t& d) {
                           l = nl[(c0 + c) >> 1];
                           d = nd[(c0 + c) >> 1];
                         },
                         pk_p, pk_ds);
        // packed into this half's own, already-read columns
        tmem_st16(tS + c0 / 2, pk_p);
        tmem_st16(tP + c0 / 2, pk_ds);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&s.p_full[half]);
    }
    if (ok && mbar_wait(&s.acc_full, 0, 116, abort_flag)) {
      tc_fence_after();
      const int key = j * BT + r;
      const bool row_ok = key < S;
      const size_t off = ((size_t)zkv * S + (row_ok ? key : 0)) * HD;
      store_row_bf16(tbase + 256 + lane_off, dV + off, 1.0f, row_ok, half * 64);
      store_row_bf16(tbase + 384 + lane_off, dK + off, scale, row_ok, half * 64);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kWarpMma) tmem_dealloc(tbase, 512);
}

// ---------------------------------------------------------------------------
// dQ
// ---------------------------------------------------------------------------
// Q_i and dO_i live in TMEM (columns [384, 448) and [448, 512), packed
// bf16 in the A-operand layout), written once per CTA by the softmax warps,
// so S and dP are TS MMAs that read only K and V from shared memory.
struct SmemQ {
  alignas(1024) uint8_t k[KS][2][kChunk];
  alignas(1024) uint8_t v[KS][2][kChunk];
  uint64_t q_full;  // Q and dO in TMEM
  uint64_t kv_full[KS], kv_empty[KS];
  uint64_t s_full[2], p_full[2], acc_full;
  uint32_t tmem_base;
  int abort_flag;
};

__global__ void __launch_bounds__(kThreads, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                  const float* __restrict__ lse2, const float* __restrict__ delta,
                  const __nv_bfloat16* __restrict__ Qg, const __nv_bfloat16* __restrict__ dOg,
                  __nv_bfloat16* __restrict__ dQ, int B, int Hq, int Hkv, int S, float scale,
                  int causal) {
  extern __shared__ uint8_t smem_raw[];
  SmemQ& s = *reinterpret_cast<SmemQ*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int Sp = padded_len(S);
  const int n_t = Sp / BT;
  const int BHq = B * Hq;
  const int group = Hq / Hkv;
  // Work item: query tile i (the longest under the causal mask first) x head;
  // groups of at least 8 heads, whole grouped-query sets.
  int i, bhq;
  decode_bwd_item(blockIdx.x, n_t, BHq, group >= 8 ? group : 8, causal != 0, false, i, bhq);
  const int zkv = (bhq / Hq) * Hkv + (bhq % Hq) / group;
  const int n_kv = causal ? i + 1 : n_t;
  const float scale_log2 = scale * kLog2e;

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, kSoftmaxThreads);
    for (int k = 0; k < KS; ++k) {
      mbar_init(&s.kv_full[k], 1);
      mbar_init(&s.kv_empty[k], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s.s_full[x], 1);
      mbar_init(&s.p_full[x], kSoftmaxThreads / 2);
    }
    mbar_init(&s.acc_full, 1);
    s.abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == kWarpMma) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;

  if (warp == kWarpProducer) {
    if (lane == 0) {
      for (int jj = 0; jj < n_kv; ++jj) {
        const int st = jj % KS;
        const uint32_t ph = (uint32_t)(jj / KS) & 1u;
        if (!mbar_wait(&s.kv_empty[st], ph ^ 1u, 120, abort_flag)) break;
        mbar_arrive_expect_tx(&s.kv_full[st], 4 * kChunk);
        tma_load_3d(s.k[st][0], &tmK, &s.kv_full[st], 0, jj * BT, zkv);
        tma_load_3d(s.k[st][1], &tmK, &s.kv_full[st], 64, jj * BT, zkv);
        tma_load_3d(s.v[st][0], &tmV, &s.kv_full[st], 0, jj * BT, zkv);
        tma_load_3d(s.v[st][1], &tmV, &s.kv_full[st], 64, jj * BT, zkv);
      }
    }
  } else if (warp == kWarpMma) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(BT, BH2, false, false);
      constexpr uint32_t idG = idesc_bf16_f32(BT, HD, false, true);
      constexpr uint64_t kChunkStep = kChunk >> 4;
      constexpr uint64_t kStageStep = (2 * kChunk) >> 4;
      constexpr uint64_t kHalfRows = (BH2 * 128) >> 4;  // 64 rows of 128 bytes
      const uint64_t dk_k = sdesc_sw128(smem_u32(s.k[0][0]), 16, 1024);
      const uint64_t dv_k = sdesc_sw128(smem_u32(s.v[0][0]), 16, 1024);
      const uint64_t dk_mn = sdesc_sw128(smem_u32(s.k[0][0]), kChunk, 1024);
      // S_x = Q K_x^T and dP_x = dO V_x^T for key half x of stage st; Q and
      // dO (A) from TMEM, 8 columns per K-step of 16 dims.
      auto issue_s = [&](int x, int st) {
        uint32_t a[8];
        uint64_t b[8];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t o = (kk >> 2) * kChunkStep + (kk & 3) * 2;
          a[kk] = tbase + 384 + kk * 8;
          b[kk] = dk_k + st * kStageStep + x * kHalfRows + o;
        }
        umma8_ts(tbase + 128 * x, a, b, 0u, idS);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t o = (kk >> 2) * kChunkStep + (kk & 3) * 2;
          a[kk] = tbase + 448 + kk * 8;
          b[kk] = dv_k + st * kStageStep + x * kHalfRows + o;
        }
        umma8_ts(tbase + 128 * x + 64, a, b, 0u, idS);
        umma_commit(&s.s_full[x]);
      };
      // dQ += dS_x K_x (A in TMEM, K = the half's 64 keys).
      auto issue_g = [&](int x, int st, uint32_t acc) {
        uint32_t ta[4];
        uint64_t b[4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          ta[kk] = tbase + 128 * x + kk * 8;
          b[kk] = dk_mn + st * kStageStep + x * kHalfRows + kk * 128;
        }
        umma4_ts(tbase + 256, ta, b, acc, idG);
      };
      bool ok = mbar_wait(&s.q_full, 0, 121, abort_flag) &&
                mbar_wait(&s.kv_full[0], 0, 122, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
      }
      for (int jj = 0; jj < n_kv && ok; ++jj) {
        const int st = jj % KS;
        const bool more = jj + 1 < n_kv;
        const int st1 = (jj + 1) % KS;
        const uint32_t ph1 = (uint32_t)((jj + 1) / KS) & 1u;
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (!mbar_wait(&s.p_full[x], (uint32_t)jj & 1u, 123, abort_flag)) { ok = false; break; }
          tc_fence_after();
          issue_g(x, st, (jj > 0 || x > 0) ? 1u : 0u);
          if (x == 1) umma_commit(&s.kv_empty[st]);
          if (more) {
            if (x == 0) {
              if (!mbar_wait(&s.kv_full[st1], ph1, 126, abort_flag)) { ok = false; break; }
              tc_fence_after();
            }
            issue_s(x, st1);
          }
        }
      }
      umma_commit(&s.acc_full);
    }
  } else {
    // ---------------- softmax / epilogue: thread = query row ----------------
    // Group half owns key half `half` of every key tile: S at TMEM columns
    // [128 half, +64), dP at [128 half + 64, +64).
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tbase + 128 * half + lane_off, tP = tS + 64;
    {
      // this thread's row of Q_i and dO_i, dims [64 half, +64), into TMEM
      const int q = i * BT + r;
      const bool row_ok = q < S;
      const size_t off = ((size_t)bhq * S + (row_ok ? q : 0)) * HD + half * 64;
      const uint4* qs = reinterpret_cast<const uint4*>(Qg + off);
      const uint4* ds = reinterpret_cast<const uint4*>(dOg + off);
      uint32_t qa[32], da[32];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint4 a = row_ok ? qs[u] : make_uint4(0u, 0u, 0u, 0u);
        const uint4 d = row_ok ? ds[u] : make_uint4(0u, 0u, 0u, 0u);
        qa[4 * u] = a.x; qa[4 * u + 1] = a.y; qa[4 * u + 2] = a.z; qa[4 * u + 3] = a.w;
        da[4 * u] = d.x; da[4 * u + 1] = d.y; da[4 * u + 2] = d.z; da[4 * u + 3] = d.w;
      }
      tmem_st32(tbase + 384 + 32 * half + lane_off, qa);
      tmem_st32(tbase + 448 + 32 * half + lane_off, da);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&s.q_full);
    }
    const size_t srow = (size_t)bhq * Sp + (size_t)i * BT + r;
    const float nl = lse2[srow], nd = delta[srow];
    const uint64_t nl2 = attn::pk2(nl, nl), nd2 = attn::pk2(nd, nd);
    const uint64_t scale2 = attn::pk2(scale_log2, scale_log2);
    bool ok = true;
    for (int jj = 0; jj < n_kv; ++jj) {
      if (!mbar_wait(&s.s_full[half], (uint32_t)jj & 1u, 124, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const int kh = BH2 * half;             // first key of this half within the tile
      const bool diag = causal && jj == i;   // key k > query r is masked
      const int kpad = S - jj * BT - kh;     // keys c >= kpad of this half are padding
      const bool masked = (diag && kh + BH2 - 1 > r) || kpad < BH2;
#pragma unroll 1
      for (int c0 = 0; c0 < BH2; c0 += 32) {
        uint32_t sv[32], dv[32];
        tmem_ld32(tS + c0, sv);
        tmem_ld32(tP + c0, dv);
        tmem_ld_wait(sv);
        tmem_ld_wait(dv);
        if (masked) {
          // keys c >= lim of this chunk are masked (padding, or beyond the row on the diagonal)
          int lim = kpad - c0;
          if (diag && r - kh - c0 + 1 < lim) lim = r - kh - c0 + 1;
          mask_from(sv, lim);
        }
        uint32_t pk_p[16], pk_ds[16];
        p_ds_chunk<false>(sv, dv, scale2,
                          [&](int, uint64_t& l, uint64_t& d) {
                            l = nl2;
                            d = nd2;
                          },
                          pk_p, pk_ds);
        tmem_st16(tS + c0 / 2, pk_ds);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&s.p_full[half]);
    }
    if (ok && mbar_wait(&s.acc_full, 0, 125, abort_flag)) {
      tc_fence_after();
      const int q = i * BT + r;
      const bool row_ok = q < S;
      store_row_bf16(tbase + 256 + lane_off, dQ + ((size_t)bhq * S + (row_ok ? q : 0)) * HD,
                     scale, row_ok, half * 64);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kWarpMma) tmem_dealloc(tbase, 512);
}

// ---------------------------------------------------------------------------
// CUDA-core path (fp32 inputs, head dims other than 128, unaligned buffers):
// one warp per query row (dQ) or key row (dK, dV), head dim spread over the
// lanes (up to kSimtDPL per lane), exact exp, fp32 throughout.
// ---------------------------------------------------------------------------
constexpr int kSimtDPL = 8;  // head dim <= 256

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ void load_row(const T* p, int D, int lane, float (&x)[kSimtDPL]) {
#pragma unroll
  for (int k = 0; k < kSimtDPL; ++k) {
    const int d = lane + 32 * k;
    x[k] = d < D ? to_f32<T>(p[d]) : 0.0f;
  }
}

__device__ __forceinline__ float dot_row(const float (&a)[kSimtDPL], const float (&b)[kSimtDPL]) {
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < kSimtDPL; ++k) s = fmaf(a[k], b[k], s);
  return warp_sum(s);
}

// delta[bh, q] = sum_d dO * O
template <typename T>
__global__ void __launch_bounds__(256) bwd_simt_delta_kernel(const T* __restrict__ O,
                                                             const T* __restrict__ dO,
                                                             float* __restrict__ delta,
                                                             int64_t rows, int D) {
  const int lane = threadIdx.x & 31;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    float o[kSimtDPL], g[kSimtDPL];
    load_row(O + row * D, D, lane, o);
    load_row(dO + row * D, D, lane, g);
    const float d = dot_row(o, g);
    if (lane == 0) delta[row] = d;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) bwd_simt_dq_kernel(
    const T* __restrict__ Q, const T* __restrict__ K, const T* __restrict__ V,
    const T* __restrict__ dO, const float* __restrict__ lse, const float* __restrict__ delta,
    T* __restrict__ dQ, int B, int Hq, int Hkv, int S, int D, float scale, int causal) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)B * Hq * S;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t bh = row / S;
    const int q = (int)(row - bh * S);
    const int64_t zkv = (bh / Hq) * Hkv + (bh % Hq) / (Hq / Hkv);
    float qv[kSimtDPL], gv[kSimtDPL], acc[kSimtDPL] = {};
    load_row(Q + row * D, D, lane, qv);
    load_row(dO + row * D, D, lane, gv);
    const float l = lse[row], dl = delta[row];
    const int n_k = causal ? q + 1 : S;
    for (int k = 0; k < n_k; ++k) {
      float kv[kSimtDPL], vv[kSimtDPL];
      load_row(K + (zkv * S + k) * D, D, lane, kv);
      load_row(V + (zkv * S + k) * D, D, lane, vv);
      const float p = expf(scale * dot_row(qv, kv) - l);
      const float ds = p * (dot_row(gv, vv) - dl);
#pragma unroll
      for (int c = 0; c < kSimtDPL; ++c) acc[c] = fmaf(ds, kv[c], acc[c]);
    }
#pragma unroll
    for (int c = 0; c < kSimtDPL; ++c) {
      const int d = lane + 32 * c;
      if (d < D) dQ[row * D + d] = from_f32<T>(acc[c] * scale);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) bwd_simt_dkdv_kernel(
    const T* __restrict__ Q, const T* __restrict__ K, const T* __restrict__ V,
    const T* __restrict__ dO, const float* __restrict__ lse, const float* __restrict__ delta,
    T* __restrict__ dK, T* __restrict__ dV, int B, int Hq, int Hkv, int S, int D, float scale,
    int causal) {
  const int lane = threadIdx.x & 31;
  const int group = Hq / Hkv;
  const int64_t rows = (int64_t)B * Hkv * S;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t zkv = row / S;
    const int k = (int)(row - zkv * S);
    const int64_t b = zkv / Hkv, g = zkv % Hkv;
    float kv[kSimtDPL], vv[kSimtDPL], ak[kSimtDPL] = {}, av[kSimtDPL] = {};
    load_row(K + row * D, D, lane, kv);
    load_row(V + row * D, D, lane, vv);
    for (int hh = 0; hh < group; ++hh) {
      const int64_t bh = b * Hq + g * group + hh;
      for (int q = causal ? k : 0; q < S; ++q) {
        float qv[kSimtDPL], gv[kSimtDPL];
        load_row(Q + (bh * S + q) * D, D, lane, qv);
        load_row(dO + (bh * S + q) * D, D, lane, gv);
        const float p = expf(scale * dot_row(qv, kv) - lse[bh * S + q]);
        const float ds = p * (dot_row(gv, vv) - delta[bh * S + q]);
#pragma unroll
        for (int c = 0; c < kSimtDPL; ++c) {
          av[c] = fmaf(p, gv[c], av[c]);
          ak[c] = fmaf(ds, qv[c], ak[c]);
        }
      }
    }
#pragma unroll
    for (int c = 0; c < kSimtDPL; ++c) {
      const int d = lane + 32 * c;
      if (d < D) {
        dK[row * D + d] = from_f32<T>(ak[c] * scale);
        dV[row * D + d] = from_f32<T>(av[c]);
      }
    }
  }
}

}  // namespace attn_bwd
}  // namespace jb
