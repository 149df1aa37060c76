// Flash-attention forward on tcgen05 tensor cores (bf16, head_dim 128).
//
// Computes, per (batch, query head) and query row i,
//   O_i = sum_j softmax_j(scale * q_i . k_j) v_j,   lse_i = log sum_j exp(...)
// with an optional causal mask (key j > query i excluded) and grouped-query
// heads (kv head = h / (Hq/Hkv)).  The online-softmax recurrence is that of
// the reference's flashAttention (include/jules/Kernel/FlashAttention.h:
// 176-254: running max, rescale of the accumulator by exp(old-new), running
// sum, final division, :287-305), moved to base 2 and with the rescale of O
// skipped while the running max grows by less than 2^8 (the final division
// uses the same stale max for O and the sum, so the result is unchanged).
//
// CTA = one 128-row query tile at a time (persistent over (tile, b, h) work
// items, longest causal tiles first), 6 warps:
//   warp 0     TMA producer: Q tile once per item; K and V tiles (128 keys x
//              128 dims, two 64-dim 128B-swizzled boxes each) in 2-deep rings.
//   warp 1     TMEM owner and MMA issuer: S_j = Q K_j^T into one of two TMEM
//              S buffers, then O += P_{j-1} V_{j-1}; the S MMA of tile j+1 is
//              issued before the PV MMA of tile j so the tensor core works
//              while the softmax warps process S_j.
//   warps 2-5  softmax, one query row per thread (TMEM lane = row): reads
//              S_j, masks, row max, exp2, row sum, writes P_j as bf16 into a
//              128B-swizzled smem tile (the K-major A operand of PV),
//              rescales O in TMEM when needed, and finally normalises O and
//              writes O and lse.
// TMEM columns: S0 [0,128), S1 [128,256), O [256,384) (512 allocated).
#pragma once

#include "sm100.cuh"

namespace jb {
namespace attn {

constexpr int HD = 128;   // head dim handled here
constexpr int BQ = 128;   // query rows per tile (MMA M)
constexpr int BKV = 128;  // keys per tile (MMA N of S, K of PV)
constexpr int KVS = 2;    // K and V ring depth
constexpr int kThreads = 192;
constexpr int kChunk = 128 * 64 * 2;  // one 64-dim (128 B) swizzled box of 128 rows
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct Smem {
  alignas(1024) uint8_t q[2][kChunk];
  alignas(1024) uint8_t k[KVS][2][kChunk];
  alignas(1024) uint8_t v[KVS][2][kChunk];
  alignas(1024) uint8_t p[2][kChunk];
  uint64_t q_full, q_empty;
  uint64_t k_full[KVS], k_empty[KVS];
  uint64_t v_full[KVS], v_empty[KVS];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full, p_empty;
  uint64_t o_full, o_empty;
  uint32_t tmem_base;
  int abort_flag;
};

// Work item w -> (q tile, b*Hq + h); longest causal tiles first.
__device__ __forceinline__ void decode_item(int w, int n_qt, int BH, int causal, int& qt,
                                            int& bh) {
  const int r = w / BH;
  bh = w % BH;
  qt = causal ? (n_qt - 1 - r) : r;
}

#define JB_W128(r)                                                                     \
  JB_W8(r, 0), JB_W8(r, 8), JB_W8(r, 16), JB_W8(r, 24), JB_W8(r, 32), JB_W8(r, 40),    \
      JB_W8(r, 48), JB_W8(r, 56), JB_W8(r, 64), JB_W8(r, 72), JB_W8(r, 80),            \
      JB_W8(r, 88), JB_W8(r, 96), JB_W8(r, 104), JB_W8(r, 112), JB_W8(r, 120)

__device__ __forceinline__ void tmem_ld_wait128(uint32_t (&r)[128]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : JB_W128(r) : : "memory");
}

__device__ __forceinline__ void tmem_ld32_at(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : JB_R8(r, 0), JB_R8(r, 8), JB_R8(r, 16), JB_R8(r, 24)
      : "r"(taddr));
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O,
                       float* __restrict__ lse, int B, int Hq, int Hkv, int S, float scale_log2,
                       int causal) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int BH = B * Hq;
  const int n_qt = (S + BQ - 1) / BQ;
  const int n_kv_full = (S + BKV - 1) / BKV;
  const int total = n_qt * BH;
  const int group = Hq / Hkv;

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    mbar_init(&s.q_empty, 1);
    for (int i = 0; i < KVS; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_empty[i], 128);
    }
    mbar_init(&s.p_full, 128);
    mbar_init(&s.p_empty, 1);
    mbar_init(&s.o_full, 1);
    mbar_init(&s.o_empty, 128);
    s.abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      uint32_t kvi = 0, wi = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x, ++wi) {
        int qt, bh;
        decode_item(w, n_qt, BH, causal, qt, bh);
        const int b = bh / Hq, h = bh % Hq;
        const int zkv = b * Hkv + h / group;
        const int n_kv = causal ? (qt + 1 < n_kv_full ? qt + 1 : n_kv_full) : n_kv_full;
        if (!mbar_wait(&s.q_empty, (wi & 1u) ^ 1u, 10, abort_flag)) break;
        mbar_arrive_expect_tx(&s.q_full, 2 * kChunk);
        tma_load_3d(s.q[0], &tmQ, &s.q_full, 0, qt * BQ, bh);
        tma_load_3d(s.q[1], &tmQ, &s.q_full, 64, qt * BQ, bh);
        for (int j = 0; j < n_kv; ++j, ++kvi) {
          const uint32_t st = kvi % KVS, ph = (kvi / KVS) & 1u;
          if (!mbar_wait(&s.k_empty[st], ph ^ 1u, 11, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&s.k_full[st], 2 * kChunk);
          tma_load_3d(s.k[st][0], &tmK, &s.k_full[st], 0, j * BKV, zkv);
          tma_load_3d(s.k[st][1], &tmK, &s.k_full[st], 64, j * BKV, zkv);
          if (!mbar_wait(&s.v_empty[st], ph ^ 1u, 12, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&s.v_full[st], 2 * kChunk);
          tma_load_3d(s.v[st][0], &tmV, &s.v_full[st], 0, j * BKV, zkv);
          tma_load_3d(s.v[st][1], &tmV, &s.v_full[st], 64, j * BKV, zkv);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(BQ, BKV, false, false);
      constexpr uint32_t idPV = idesc_bf16_f32(BQ, HD, false, true);
      const uint32_t tO = tbase + 256;
      uint32_t kvi = 0, sc = 0, pc = 0, wi = 0;
      bool ok = true;
      const uint32_t q0a = smem_u32(s.q[0]), q1a = smem_u32(s.q[1]);
      const uint32_t p0a = smem_u32(s.p[0]), p1a = smem_u32(s.p[1]);
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x, ++wi) {
        int qt, bh;
        decode_item(w, n_qt, BH, causal, qt, bh);
        const int n_kv = causal ? (qt + 1 < n_kv_full ? qt + 1 : n_kv_full) : n_kv_full;
        if (!mbar_wait(&s.q_full, wi & 1u, 20, abort_flag)) break;
        tc_fence_after();
        const uint32_t kv0 = kvi;
        auto issue_pv = [&](int jj) -> bool {
          const uint32_t st = (kv0 + jj) % KVS, ph = ((kv0 + jj) / KVS) & 1u;
          if (!mbar_wait(&s.p_full, pc & 1u, 21, abort_flag)) return false;
          if (jj == 0 && !mbar_wait(&s.o_empty, (wi & 1u) ^ 1u, 22, abort_flag)) return false;
          if (!mbar_wait(&s.v_full[st], ph, 23, abort_flag)) return false;
          tc_fence_after();
          const uint32_t va = smem_u32(s.v[st][0]);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk) {
            const uint64_t ad = sdesc_sw128((kk < 4 ? p0a : p1a) + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(va + kk * 2048, kChunk, 1024);
            umma_f16_ss(tO, ad, bd, idPV, (jj > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&s.v_empty[st]);
          umma_commit(&s.p_empty);
          ++pc;
          return true;
        };
        for (int j = 0; j < n_kv && ok; ++j) {
          const uint32_t st = (kv0 + j) % KVS, ph = ((kv0 + j) / KVS) & 1u;
          const uint32_t sb = sc & 1u, sph = (sc >> 1) & 1u;
          if (!mbar_wait(&s.k_full[st], ph, 24, abort_flag)) { ok = false; break; }
          if (!mbar_wait(&s.s_empty[sb], sph ^ 1u, 25, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k0a = smem_u32(s.k[st][0]), k1a = smem_u32(s.k[st][1]);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint64_t ad = sdesc_sw128((kk < 4 ? q0a : q1a) + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128((kk < 4 ? k0a : k1a) + (kk & 3) * 32, 16, 1024);
            umma_f16_ss(tbase + sb * BKV, ad, bd, idS, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s.k_empty[st]);
          umma_commit(&s.s_full[sb]);
          ++sc;
          if (j == n_kv - 1) umma_commit(&s.q_empty);
          if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
        }
        if (!ok) break;
        if (!issue_pv(n_kv - 1)) break;
        umma_commit(&s.o_full);
        kvi = kv0 + n_kv;
      }
    }
  } else {
    // ------------------------------ softmax ------------------------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row within the query tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tO = tbase + 256 + lane_off;
    uint32_t sc = 0, pw = 0, wi = 0;
    // swizzled row base inside a P chunk
    const uint32_t prow = (uint32_t)r * 128u;
    const uint32_t pswz = (uint32_t)(r & 7);
    for (int w = blockIdx.x; w < total; w += gridDim.x, ++wi) {
      int qt, bh;
      decode_item(w, n_qt, BH, causal, qt, bh);
      const int n_kv = causal ? (qt + 1 < n_kv_full ? qt + 1 : n_kv_full) : n_kv_full;
      const int q = qt * BQ + r;
      float m_run = -INFINITY, l_run = 0.0f;
      bool ok = true;
      for (int j = 0; j < n_kv; ++j) {
        const uint32_t sb = sc & 1u, sph = (sc >> 1) & 1u;
        if (!mbar_wait(&s.s_full[sb], sph, 30, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[128];
        const uint32_t ts = tbase + lane_off + sb * BKV;
        tmem_ld32_at(ts + 0, sr + 0);
        tmem_ld32_at(ts + 32, sr + 32);
        tmem_ld32_at(ts + 64, sr + 64);
        tmem_ld32_at(ts + 96, sr + 96);
        tmem_ld_wait128(sr);
        tc_fence_before();
        mbar_arrive(&s.s_empty[sb]);
        ++sc;

        float x[128];
#pragma unroll
        for (int c = 0; c < 128; ++c) x[c] = __uint_as_float(sr[c]) * scale_log2;
        if (j == n_kv - 1) {  // only the last tile can hold masked keys
          const int kbase = j * BKV;
          int lim = S - kbase;                         // keys >= S are padding
          if (causal && q - kbase + 1 < lim) lim = q - kbase + 1;  // keys > q
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c >= lim) x[c] = -INFINITY;
        }
        float mt = x[0];
#pragma unroll
        for (int c = 1; c < 128; ++c) mt = fmaxf(mt, x[c]);
        // Lazy rescale: keep the old max unless the new one exceeds it by
        // more than the threshold.
        const bool need = mt > m_run + kRescaleThreshold;
        const float m_new = need ? mt : m_run;
        const float alpha = need ? ex2_approx(m_run - m_new) : 1.0f;
        const float neg_m = (m_new == -INFINITY) ? 0.0f : -m_new;
        float rowsum = 0.0f;
        uint32_t pk[64];
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float e0 = ex2_approx(x[2 * c] + neg_m);
          const float e1 = ex2_approx(x[2 * c + 1] + neg_m);
          rowsum += e0 + e1;
          pk[c] = pack_bf16x2(e0, e1);
        }
        l_run = l_run * alpha + rowsum;
        m_run = m_new;

        // P buffer is free once the previous PV MMA has completed.
        if (pw > 0 && !mbar_wait(&s.p_empty, (pw - 1) & 1u, 31, abort_flag)) { ok = false; break; }
        tc_fence_after();
        if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            uint32_t o[32];
            tmem_ld32(tO + c, o);
            tmem_ld_wait(o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + c, o);
          }
          tmem_st_wait();
        }
        // P row -> two 128B-swizzled chunks (keys 0-63, 64-127).
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          uint8_t* base = s.p[ch] + prow;
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            uint4 v;
            v.x = pk[ch * 32 + g * 4 + 0];
            v.y = pk[ch * 32 + g * 4 + 1];
            v.z = pk[ch * 32 + g * 4 + 2];
            v.w = pk[ch * 32 + g * 4 + 3];
            *reinterpret_cast<uint4*>(base + (((uint32_t)g ^ pswz) << 4)) = v;
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&s.p_full);
        ++pw;
      }
      if (!ok) break;
      // ----- epilogue: O / l -> bf16, lse -----
      if (!mbar_wait(&s.o_full, wi & 1u, 32, abort_flag)) break;
      tc_fence_after();
      const float inv_l = 1.0f / l_run;
      const bool row_ok = q < S;
      __nv_bfloat16* orow = O + ((size_t)bh * S + (row_ok ? q : 0)) * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        uint32_t o[32];
        tmem_ld32(tO + c, o);
        tmem_ld_wait(o);
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(o[8 * g + 0]) * inv_l, __uint_as_float(o[8 * g + 1]) * inv_l);
            v.y = pack_bf16x2(__uint_as_float(o[8 * g + 2]) * inv_l, __uint_as_float(o[8 * g + 3]) * inv_l);
            v.z = pack_bf16x2(__uint_as_float(o[8 * g + 4]) * inv_l, __uint_as_float(o[8 * g + 5]) * inv_l);
            v.w = pack_bf16x2(__uint_as_float(o[8 * g + 6]) * inv_l, __uint_as_float(o[8 * g + 7]) * inv_l);
            dst[g] = v;
          }
        }
      }
      if (lse && row_ok) lse[(size_t)bh * S + q] = (m_run + log2f(l_run)) * 0.69314718055994531f;
      tc_fence_before();
      mbar_arrive(&s.o_empty);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

}  // namespace attn
}  // namespace jb
