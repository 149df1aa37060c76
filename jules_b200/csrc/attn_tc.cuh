// Flash-attention forward on tcgen05 tensor cores (bf16 or fp16, head_dim
// 128 or 64: template parameters TEl and HDIM).
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
// Work item = two 128-row query tiles (256 rows) of one (b, h); persistent
// CTAs take items longest-causal-first.  Under the causal mask tile 0 runs
// one key step fewer than tile 1 (the last key tile is past all its rows).
// 12 warps (3 warpgroups):
//   warp 8     TMA producer: both Q tiles once per item; K and V tiles
//              (128 keys x 128 dims as two 64-dim 128B-swizzled boxes) in
//              2-deep rings shared by the two query tiles.
//   warp 9     TMEM owner and MMA issuer.  Per key tile j the order is
//              PV(0,j-1), S(0,j), PV(1,j-1), S(1,j): while softmax group 0
//              works on S(0,j) the tensor core runs S(1,j) and PV(1,j-1), and
//              the other way round (ping-pong).  Warps 10-11 only hold the
//              warpgroup's registers low.
//   warps 0-3  softmax group 0 (query tile 0), one row per thread (TMEM lane
//   warps 4-7  = row); group 1 (query tile 1).  Each reads S from TMEM, masks,
//              takes the row max and the exponentials (MUFU ex2), writes P as bf16
//              back over S in TMEM, rescales O when needed, and at the end
//              normalises O and writes O and lse.
// PV runs with P as the TMEM A operand (no shared-memory round trip).
// TMEM columns: S/P tile 0 [0,128), S/P tile 1 [128,256), O tile 0 [256,384),
// O tile 1 [384,512).  S(t,j+1) reuses the columns of P(t,j): the tensor core
// executes one thread's MMAs in issue order, and the softmax only writes P(t,j+1)
// after the commit of S(t,j+1), which follows PV(t,j).
#pragma once

#include "sm100.cuh"

namespace jb {
namespace attn {

constexpr int HD = 128;   // largest head dim handled here (64 is the other)
constexpr int BQ = 128;   // query rows per tile (MMA M)
constexpr int NQT = 2;    // query tiles per work item
constexpr int BKV = 128;  // keys per tile (MMA N of S, K of PV)
constexpr int KVS = 2;    // K and V ring depth
constexpr int kThreads = 384;  // 3 warpgroups
// Register split (setmaxnreg): launched at 168 per thread (65536 / 384, in
// steps of 8); the producer/MMA warpgroup drops to kRegsCtl and the two
// softmax warpgroups rise to kRegsSoftmax.  Per SM sub-partition (one warp of
// each warpgroup): 2*200 + 104 = 504 <= 512; per block 8*32*200 + 4*32*104 =
// 64512 = 384*168.  (Both regions compile without spills at this split.)
constexpr int kRegsLaunch = 168;
constexpr int kRegsSoftmax = 200;
constexpr int kRegsCtl = 104;
static_assert(2 * kRegsSoftmax + kRegsCtl <= 512, "sub-partition register file");
static_assert(8 * kRegsSoftmax + 4 * kRegsCtl <= 12 * kRegsLaunch, "block register budget");
constexpr int kWarpProducer = 8;
constexpr int kWarpMma = 9;
constexpr int kChunk = 128 * 64 * 2;  // one 64-dim (128 B) swizzled box of 128 rows
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// Where the epilogue writes O and lse: the local buffers (index 0) and, for
// the sharded call with the gather fused in, the same (b, h) rows of every
// other rank's buffers mapped into this process.  lse entries are null when
// no logsumexp is wanted.
struct AttnOut {
  __nv_bfloat16* o[kMaxPeers];
  float* lse[kMaxPeers];
  // NVLink multicast addresses of O and lse (all ranks' buffers behind one
  // address, the switch replicating each store), or null: then o[] / lse[]
  // are stored one by one.
  __nv_bfloat16* o_mc;
  float* lse_mc;
  int n;
};

// With the gather fused in (kGather), the dynamic shared memory continues
// after Smem with the epilogue staging: 2 KB per softmax warp, 32 rows x 64
// bytes (32 bf16 columns of O), 16-byte chunks XOR-swizzled by (row >> 1) & 3.
constexpr int kEpiBytes = 8 * 32 * 64;

struct Smem {
  alignas(1024) uint8_t q[NQT][2][kChunk];
  alignas(1024) uint8_t k[KVS][2][kChunk];
  alignas(1024) uint8_t v[KVS][2][kChunk];
  uint64_t q_full, q_empty;
  uint64_t k_full[KVS], k_empty[KVS];
  uint64_t v_full[KVS], v_empty[KVS];
  uint64_t s_full[NQT], p_full[NQT], o_full[NQT], o_empty[NQT];
  uint32_t tmem_base;
  int abort_flag;
};

// Work item w -> (query-tile pair, b*Hq + h).  Items come in groups of G
// consecutive (b, h) (whole grouped-query sets, at least 8 heads); inside a
// group the pairs run longest-causal-first and, for each pair, the heads of
// the group run back to back.  The ~148 items resident at one time therefore
// read the K/V of a few heads, which stay in L2, and the end of the grid
// holds the shortest items.
__device__ __forceinline__ int head_group(int group) {
  return group >= 8 ? group : group * (8 / group);
}
__device__ __forceinline__ void decode_item(int w, int n_pairs, int BH, int G, int causal,
                                            int& pair, int& bh) {
  const int per_group = G * n_pairs;
  const int g = w / per_group;
  const int idx = w - g * per_group;
  const int gh = min(G, BH - g * G);
  const int r = idx / gh;
  bh = g * G + idx % gh;
  pair = causal ? (n_pairs - 1 - r) : r;
}

// Key tiles query tile t of a pair needs (causal: up to its last row); the
// item's count is tile 1's.  Under the causal mask tile 0 needs one fewer:
// the pair's last key tile lies entirely after tile 0's rows.
__device__ __forceinline__ int kv_tiles_t(int pair, int t, int n_kv_full, int causal) {
  if (!causal) return n_kv_full;
  const int n = 2 * pair + t + 1;
  return n < n_kv_full ? n : n_kv_full;
}
__device__ __forceinline__ int kv_tiles(int pair, int n_kv_full, int causal) {
  if (!causal) return n_kv_full;
  const int n = 2 * pair + 2;
  return n < n_kv_full ? n : n_kv_full;
}

// Packed fp32 pairs (sm_100 f32x2 instructions: one issue slot, two lanes).
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
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

template <int HDIM, typename TEl, bool kGather>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const AttnOut out, int B,
                       int Hq, int Hkv, int S, float scale_log2, int causal) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int BH = B * Hq;
  const int n_pairs = (S + NQT * BQ - 1) / (NQT * BQ);
  const int n_kv_full = (S + BKV - 1) / BKV;
  const int total = n_pairs * BH;
  const int group = Hq / Hkv;
  const int hgroup = head_group(group);

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    mbar_init(&s.q_empty, 1);
    for (int i = 0; i < KVS; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
    }
    for (int t = 0; t < NQT; ++t) {
      mbar_init(&s.s_full[t], 1);
      mbar_init(&s.p_full[t], 128);
      mbar_init(&s.o_full[t], 1);
      mbar_init(&s.o_empty[t], 128);
    }
    s.abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
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

  if (warp >= 8) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsCtl));
  if (warp == kWarpProducer) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      uint32_t kvi = 0, wi = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x, ++wi) {
        int pair, bh;
        decode_item(w, n_pairs, BH, hgroup, causal, pair, bh);
        const int b = bh / Hq, h = bh % Hq;
        const int zkv = b * Hkv + h / group;
        const int n_kv = kv_tiles(pair, n_kv_full, causal);
        const int q0 = pair * NQT * BQ;
        if (!mbar_wait(&s.q_empty, (wi & 1u) ^ 1u, 10, abort_flag)) break;
        constexpr int kBoxes = HDIM / 64;  // 64-dim boxes per row
        mbar_arrive_expect_tx(&s.q_full, NQT * kBoxes * kChunk);
#pragma unroll
        for (int t = 0; t < NQT; ++t) {
          tma_load_3d(s.q[t][0], &tmQ, &s.q_full, 0, q0 + t * BQ, bh);
          if (kBoxes == 2) tma_load_3d(s.q[t][1], &tmQ, &s.q_full, 64, q0 + t * BQ, bh);
        }
        for (int j = 0; j < n_kv; ++j, ++kvi) {
          const uint32_t st = kvi % KVS, ph = (kvi / KVS) & 1u;
          if (!mbar_wait(&s.k_empty[st], ph ^ 1u, 11, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&s.k_full[st], kBoxes * kChunk);
          tma_load_3d(s.k[st][0], &tmK, &s.k_full[st], 0, j * BKV, zkv);
          if (kBoxes == 2) tma_load_3d(s.k[st][1], &tmK, &s.k_full[st], 64, j * BKV, zkv);
          if (!mbar_wait(&s.v_empty[st], ph ^ 1u, 12, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&s.v_full[st], kBoxes * kChunk);
          tma_load_3d(s.v[st][0], &tmV, &s.v_full[st], 0, j * BKV, zkv);
          if (kBoxes == 2) tma_load_3d(s.v[st][1], &tmV, &s.v_full[st], 64, j * BKV, zkv);
        }
      }
    }
  } else if (warp == kWarpMma) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16kind<TEl>(BQ, BKV, false, false);
      constexpr uint32_t idPV = idesc_f16kind<TEl>(BQ, HDIM, false, true);
      uint32_t kvi = 0, wi = 0;
      uint32_t pvc_t[NQT] = {0, 0};  // completed key steps per tile (barrier phases)
      bool ok = true;
      // Descriptors for every operand slot, built once.  A K step moves the
      // start-address field (bytes >> 4): +2 per 32 bytes inside a 128-byte
      // swizzle row (K-major), +128 per 16 rows of 128 bytes (MN-major V).
      // Q/K: two 64-dim chunks kChunk bytes apart, so chunk 1 = chunk 0 +
      // kChunk >> 4 in the same field.
      const uint64_t dq0 = sdesc_sw128(smem_u32(s.q[0][0]), 16, 1024);
      const uint64_t dk0 = sdesc_sw128(smem_u32(s.k[0][0]), 16, 1024);
      const uint64_t dv0 = sdesc_sw128(smem_u32(s.v[0][0]), kChunk, 1024);
      constexpr uint64_t kChunkStep = kChunk >> 4;           // next 64-dim chunk
      constexpr uint64_t kStageStep = (2 * kChunk) >> 4;     // next Q tile / ring slot
      auto issue_s = [&](int t, uint32_t st) {
        const uint64_t qa = dq0 + t * kStageStep, kb = dk0 + st * kStageStep;
        if constexpr (HDIM == 128) {
          uint64_t a[8], b[8];
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            a[kk] = qa + (kk >> 2) * kChunkStep + (kk & 3) * 2;
            b[kk] = kb + (kk >> 2) * kChunkStep + (kk & 3) * 2;
          }
          umma8_ss(tbase + t * BKV, a, b, 0u, idS);
        } else {  // one 64-dim chunk: 4 K-steps
          uint64_t a[4], b[4];
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            a[kk] = qa + kk * 2;
            b[kk] = kb + kk * 2;
          }
          umma4_ss(tbase + t * BKV, a, b, 0u, idS);
        }
        umma_commit(&s.s_full[t]);
      };
      auto issue_pv = [&](int t, uint32_t st, bool accumulate) {
        uint32_t pa[8];
        uint64_t b[8];
        const uint64_t vb = dv0 + st * kStageStep;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          pa[kk] = tbase + t * BKV + kk * 8;
          b[kk] = vb + kk * 128;
        }
        umma8_ts(tbase + 256 + t * HDIM, pa, b, accumulate ? 1u : 0u, idPV);
      };
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x, ++wi) {
        int pair, bh;
        decode_item(w, n_pairs, BH, hgroup, causal, pair, bh);
        const int n_kv = kv_tiles(pair, n_kv_full, causal);
        const int nk[NQT] = {kv_tiles_t(pair, 0, n_kv_full, causal), n_kv};
        if (!mbar_wait(&s.q_full, wi & 1u, 20, abort_flag)) break;
        const uint32_t kv0 = kvi;
        {
          const uint32_t st = kv0 % KVS, ph = (kv0 / KVS) & 1u;
          if (!mbar_wait(&s.k_full[st], ph, 21, abort_flag)) break;
          tc_fence_after();
          issue_s(0, st);
          issue_s(1, st);
          umma_commit(&s.k_empty[st]);
          if (n_kv == 1) umma_commit(&s.q_empty);
        }
        for (int j = 0; j < n_kv && ok; ++j) {
          const uint32_t st = (kv0 + j) % KVS, ph = ((kv0 + j) / KVS) & 1u;
          const uint32_t st1 = (kv0 + j + 1) % KVS, ph1 = ((kv0 + j + 1) / KVS) & 1u;
#pragma unroll
          for (int t = 0; t < NQT; ++t) {
            if (j >= nk[t]) continue;  // tile 0's steps end one early under the causal mask
            const uint32_t g = pvc_t[t] + j;
            const bool more = j + 1 < nk[t];
            // the first tile of this step waits for V; the first to issue the
            // next step's S waits for K
            const bool first = t == 0 || j >= nk[0];
            const bool kfirst = t == 0 || j + 1 >= nk[0];
            bool kready = false;
            {
              // Poll every barrier this group needs at once; the slow path
              // (rare) waits on them one by one.
              const uint32_t r0 = mbar_try_wait(&s.p_full[t], g & 1u) ? 1u : 0u;
              const uint32_t r1 = (j != 0) ? 1u : (mbar_try_wait(&s.o_empty[t], (wi & 1u) ^ 1u) ? 1u : 0u);
              const uint32_t r2 = !first ? 1u : (mbar_try_wait(&s.v_full[st], ph) ? 1u : 0u);
              const uint32_t r3 = (kfirst && more) ? (mbar_try_wait(&s.k_full[st1], ph1) ? 1u : 0u) : 0u;
              kready = r3 != 0u;
              if ((r0 & r1 & r2) == 0u) {
                if (!mbar_wait(&s.p_full[t], g & 1u, 22, abort_flag)) { ok = false; break; }
                if (j == 0 && !mbar_wait(&s.o_empty[t], (wi & 1u) ^ 1u, 23, abort_flag)) { ok = false; break; }
                if (first && !mbar_wait(&s.v_full[st], ph, 24, abort_flag)) { ok = false; break; }
              }
            }
            tc_fence_after();
            issue_pv(t, st, j > 0);
            if (t == NQT - 1) umma_commit(&s.v_empty[st]);
            if (!more) umma_commit(&s.o_full[t]);
            if (more) {
              if (kfirst && !kready) {
                if (!mbar_wait(&s.k_full[st1], ph1, 25, abort_flag)) { ok = false; break; }
                tc_fence_after();
              }
              issue_s(t, st1);
              if (t == NQT - 1) {
                umma_commit(&s.k_empty[st1]);
                if (j + 1 == n_kv - 1) umma_commit(&s.q_empty);
              }
            }
          }
        }
        if (!ok) break;
        pvc_t[0] += nk[0];
        pvc_t[1] += nk[1];
        kvi = kv0 + n_kv;
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    // ------------------------------ softmax groups ------------------------------
    const int t = warp >> 2;          // query tile of this group (warpgroup 0 or 1)
    const int quarter = warp & 3;     // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tbase + t * BKV + lane_off;
    const uint32_t tO = tbase + 256 + t * HDIM + lane_off;
    uint32_t pvc = 0, wi = 0;
    for (int w = blockIdx.x; w < total; w += gridDim.x, ++wi) {
      int pair, bh;
      decode_item(w, n_pairs, BH, hgroup, causal, pair, bh);
      const int n_kv = kv_tiles_t(pair, t, n_kv_full, causal);  // this tile's key steps
      const int qt0 = pair * NQT * BQ + t * BQ;  // first row of this tile
      const int q = qt0 + r;
      float m_run = -INFINITY, l_run = 0.0f;
      bool ok = true;
      for (int j = 0; j < n_kv; ++j) {
        const uint32_t g = pvc + j;
        if (!mbar_wait(&s.s_full[t], g & 1u, 30, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld32_at(tS + 0, sr + 0);
        tmem_ld32_at(tS + 32, sr + 32);
        tmem_ld32_at(tS + 64, sr + 64);
        tmem_ld32_at(tS + 96, sr + 96);
        tmem_ld_wait128(sr);
        const int kbase = j * BKV;
        if (kbase + BKV > S || (causal && kbase + BKV - 1 > qt0)) {
          int lim = S - kbase;                                      // keys >= S are padding
          if (causal && q - kbase + 1 < lim) lim = q - kbase + 1;   // keys > q
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c >= lim) sr[c] = __float_as_uint(-INFINITY);
        }
        // Row max of the raw scores (scale > 0 commutes with max).
        // Four independent chains; chain k takes columns 8m + 2k and 8m + 2k + 1
        // (m = 0..15).
        float mx[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mx[k] = fmaxf(__uint_as_float(sr[2 * k]), __uint_as_float(sr[2 * k + 1]));
#pragma unroll
        for (int m = 1; m < 16; ++m) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mx[k] = max3(mx[k], __uint_as_float(sr[8 * m + 2 * k]),
                         __uint_as_float(sr[8 * m + 2 * k + 1]));
        }
        const float mt = max3(mx[0], mx[1], fmaxf(mx[2], mx[3])) * scale_log2;
        // Lazy rescale: keep the old max unless the new one exceeds it by
        // more than the threshold.
        const bool need = mt > m_run + kRescaleThreshold;
        const float m_new = need ? mt : m_run;
        const float alpha = need ? ex2_approx(m_run - m_new) : 1.0f;
        const float neg_m = (m_new == -INFINITY) ? 0.0f : -m_new;
        const uint64_t scale2 = pk2(scale_log2, scale_log2);
        const uint64_t negm2 = pk2(neg_m, neg_m);
        uint64_t sum2[2] = {pk2(0.0f, 0.0f), pk2(0.0f, 0.0f)};
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t pk[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int e = half * 64 + 2 * c;
            // x = s * scale*log2(e) - m, two lanes per instruction
            const uint64_t x2 =
                fma2(pk2(__uint_as_float(sr[e]), __uint_as_float(sr[e + 1])), scale2, negm2);
            float x0, x1;
            upk2(x2, x0, x1);
            const float e0 = ex2_approx(x0), e1 = ex2_approx(x1);
            sum2[c & 1] = add2(sum2[c & 1], pk2(e0, e1));
            pk[c] = pack2<TEl>(e0, e1);
          }
          // P (pairs of the operand type) over the first 64 columns of this tile's S.
          tmem_st32(tS + half * 32, pk);
        }
        float sa, sb, sc2, sd;
        upk2(sum2[0], sa, sb);
        upk2(sum2[1], sc2, sd);
        const float rowsum = (sa + sb) + (sc2 + sd);
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // PV(t, j-1) has completed: its commit precedes S(t, j)'s.
#pragma unroll 1
          for (int c = 0; c < HDIM; c += 32) {
            uint32_t o[32];
            tmem_ld32(tO + c, o);
            tmem_ld_wait(o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + c, o);
          }
        }
        tmem_st_wait();
        l_run = l_run * alpha + rowsum;
        m_run = m_new;
        tc_fence_before();
        mbar_arrive(&s.p_full[t]);
      }
      if (!ok) break;
      // ----- epilogue: O / l -> bf16, lse -----
      if (!mbar_wait(&s.o_full[t], wi & 1u, 32, abort_flag)) break;
      tc_fence_after();
      // O / l as bf16.  Local output only: each lane stores its own row.
      // With the gather fused in, 32 columns at a time go through shared
      // memory so that 4 lanes write 64 contiguous bytes of one row (8 rows
      // per store instruction) into every rank's O over NVLink.
      const float inv_l = 1.0f / l_run;
      const bool row_ok = q < S;
      const int row0 = qt0 + quarter * 32;  // first row of this warp
      if constexpr (!kGather) {
        __nv_bfloat16* orow = out.o[0] + ((size_t)bh * S + (row_ok ? q : 0)) * HDIM;
#pragma unroll 1
        for (int c = 0; c < HDIM; c += 32) {
          uint32_t o[32];
          tmem_ld32(tO + c, o);
          tmem_ld_wait(o);
          if (row_ok) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
            for (int g8 = 0; g8 < 4; ++g8) {
              uint4 v;
              v.x = pack2<TEl>(__uint_as_float(o[8 * g8 + 0]) * inv_l, __uint_as_float(o[8 * g8 + 1]) * inv_l);
              v.y = pack2<TEl>(__uint_as_float(o[8 * g8 + 2]) * inv_l, __uint_as_float(o[8 * g8 + 3]) * inv_l);
              v.z = pack2<TEl>(__uint_as_float(o[8 * g8 + 4]) * inv_l, __uint_as_float(o[8 * g8 + 5]) * inv_l);
              v.w = pack2<TEl>(__uint_as_float(o[8 * g8 + 6]) * inv_l, __uint_as_float(o[8 * g8 + 7]) * inv_l);
              dst[g8] = v;
            }
          }
        }
      } else {
      uint4* stg = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(&s) +
                                            ((sizeof(Smem) + 127) & ~size_t(127))) + warp * 32 * 4;
#pragma unroll 1
      for (int c = 0; c < HDIM; c += 32) {
        uint32_t o[32];
        tmem_ld32(tO + c, o);
        tmem_ld_wait(o);
#pragma unroll
        for (int g8 = 0; g8 < 4; ++g8) {
          uint4 v;
          v.x = pack2<TEl>(__uint_as_float(o[8 * g8 + 0]) * inv_l, __uint_as_float(o[8 * g8 + 1]) * inv_l);
          v.y = pack2<TEl>(__uint_as_float(o[8 * g8 + 2]) * inv_l, __uint_as_float(o[8 * g8 + 3]) * inv_l);
          v.z = pack2<TEl>(__uint_as_float(o[8 * g8 + 4]) * inv_l, __uint_as_float(o[8 * g8 + 5]) * inv_l);
          v.w = pack2<TEl>(__uint_as_float(o[8 * g8 + 6]) * inv_l, __uint_as_float(o[8 * g8 + 7]) * inv_l);
          stg[lane * 4 + (g8 ^ ((lane >> 1) & 3))] = v;
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rr = (lane >> 2) + 8 * i;
          if (row0 + rr < S) {
            const uint4 v = stg[rr * 4 + ((lane & 3) ^ ((rr >> 1) & 3))];
            const size_t off = ((size_t)bh * S + row0 + rr) * HDIM + c + (lane & 3) * 8;
            if (out.o_mc) {
              multimem_st16(out.o_mc + off, v);
            } else {
#pragma unroll
              for (int p = 0; p < kMaxPeers; ++p)
                if (p < out.n) *reinterpret_cast<uint4*>(out.o[p] + off) = v;
            }
          }
        }
        __syncwarp();
      }
      }
      if (out.lse[0] && row_ok) {
        const float l = (m_run + log2f(l_run)) * 0.69314718055994531f;
        if (kGather && out.lse_mc) {
          multimem_st_f32(out.lse_mc + (size_t)bh * S + q, l);
        } else {
#pragma unroll
          for (int p = 0; p < kMaxPeers; ++p)
            if (p < out.n) out.lse[p][(size_t)bh * S + q] = l;
        }
      }
      tc_fence_before();
      mbar_arrive(&s.o_empty[t]);
      pvc += n_kv;
    }
  }

  // Peer stores must be visible system-wide before this rank signals the
  // others that its units are in place (dist_signal_wait_kernel).
  if (kGather && out.o_mc) fence_proxy_alias();
  if (kGather) __threadfence_system();
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kWarpMma) tmem_dealloc(tbase, 512);
}

}  // namespace attn
}  // namespace jb
