// sm_100a building blocks: mbarriers, TMA tile loads, tcgen05 (TMEM alloc,
// UMMA issue/commit, TMEM loads/stores) and descriptor encoders.
//
// Written from the PTX ISA (tcgen05 / cp.async.bulk.tensor / mbarrier
// sections).  Every wait is bounded: on timeout it records an error word in
// device memory and returns false, so a stuck pipeline ends the kernel
// instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

namespace jb {

// ---------------------------------------------------------------------------
// Device error word.  Kernels OR bits in; the host reads and clears it with
// jules_device_error().  Bit layout: low byte = kind, next bytes = site id.
// ---------------------------------------------------------------------------
enum : uint32_t {
  kDevErrTimeout = 1u,   // bounded mbarrier wait expired
  kDevErrBadShape = 2u,  // kernel received a shape it cannot handle
};

__device__ unsigned int g_dev_error;

__device__ __forceinline__ void record_error(uint32_t kind, uint32_t site) {
  atomicOr(&g_dev_error, kind | (site << 8));
}

// Most output buffers a kernel epilogue writes the same tile to: the local
// one and, for the multi-GPU entry points with the gather fused in, every
// other rank's (mapped into this process) - at most 8 GPUs of one node.
constexpr int kMaxPeers = 8;

// Wall-clock limit for any single mbarrier wait (ns).  Generous: a healthy
// pipeline stage completes in microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity has completed.  Returns false
// (and records kDevErrTimeout | site) if that takes longer than limit_ns,
// or soon after *abort is set by another warp.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, uint32_t site,
                                              volatile int* abort_flag, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (abort_flag && *abort_flag) return false;
      if (globaltimer() - t0 > limit_ns) {
        record_error(kDevErrTimeout, site);
        if (abort_flag) *abort_flag = 1;
        return false;
      }
    }
  }
}

// The pipelines' wait: bounded by kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t site,
                                          volatile int* abort_flag) {
  return mbar_wait_for(bar, parity, site, abort_flag, kWaitLimitNs);
}

// ---------------------------------------------------------------------------
// TMA (tiled, no cluster features).  Coordinates are element indices,
// innermost first.  The innermost coordinate times the element size must be
// a multiple of 16 bytes; callers only pass multiples of 128 bytes.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Untiled bulk copy global -> shared, completing on an mbarrier (no cluster
// features).  Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (cluster of 2) for cta_group::2 MMAs.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Arrive on an mbarrier given by its shared::cluster address (own or peer).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// Tile load of one CTA of a pair; the transaction bytes complete on the
// barrier at the same offset in the even (leader) CTA of the pair: address
// bit 24 selects the CTA of the pair.
constexpr uint32_t kPairLeaderMask = 0xFEFFFFFFu;
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar) & kPairLeaderMask), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory
// ---------------------------------------------------------------------------
// Whole-warp instruction.  Writes the allocated TMEM address to *dst.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem], bf16/fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem].
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Back-to-back K=16 steps from one thread.  A single asm block sets the
// accumulate predicates once (first step: acc_first, then 1) so the issuing
// thread spends no dependent arithmetic between MMAs; descriptors are passed
// precomputed.
#define JB_L8(a) "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7])
#define JB_U8(a) "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7])
#define JB_MMA_SS(ai, bi, pr) \
  "tcgen05.mma.cta_group::1.kind::f16 [%0], %" #ai ", %" #bi ", %18, " pr ";\n\t"

// D (+)= sum over 8 K-steps of A[smem] * B[smem].
__device__ __forceinline__ void umma8_ss(uint32_t d_tmem, const uint64_t (&a)[8],
                                         const uint64_t (&b)[8], uint32_t acc_first,
                                         uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %17, 0;\n\t"
      "setp.eq.b32 q, %17, %17;\n\t"
      JB_MMA_SS(1, 9, "p") JB_MMA_SS(2, 10, "q") JB_MMA_SS(3, 11, "q") JB_MMA_SS(4, 12, "q")
      JB_MMA_SS(5, 13, "q") JB_MMA_SS(6, 14, "q") JB_MMA_SS(7, 15, "q") JB_MMA_SS(8, 16, "q")
      "}" ::"r"(d_tmem), JB_L8(a), JB_L8(b), "r"(acc_first), "r"(idesc)
      : "memory");
}

#define JB_MMA_SS4(ai, bi, pr) \
  "tcgen05.mma.cta_group::1.kind::f16 [%0], %" #ai ", %" #bi ", %10, " pr ";\n\t"
// D (+)= sum over 4 K-steps of A[smem] * B[smem].
__device__ __forceinline__ void umma4_ss(uint32_t d_tmem, const uint64_t (&a)[4],
                                         const uint64_t (&b)[4], uint32_t acc_first,
                                         uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %9, 0;\n\t"
      "setp.eq.b32 q, %9, %9;\n\t"
      JB_MMA_SS4(1, 5, "p") JB_MMA_SS4(2, 6, "q") JB_MMA_SS4(3, 7, "q") JB_MMA_SS4(4, 8, "q")
      "}" ::"r"(d_tmem), "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]),
      "l"(b[2]), "l"(b[3]), "r"(acc_first), "r"(idesc)
      : "memory");
}

#define JB_MMA_TS(ai, bi, pr) \
  "tcgen05.mma.cta_group::1.kind::f16 [%0], [%" #ai "], %" #bi ", %18, " pr ";\n\t"

// D (+)= sum over 8 K-steps of A[tmem] * B[smem].
__device__ __forceinline__ void umma8_ts(uint32_t d_tmem, const uint32_t (&a)[8],
                                         const uint64_t (&b)[8], uint32_t acc_first,
                                         uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %17, 0;\n\t"
      "setp.eq.b32 q, %17, %17;\n\t"
      JB_MMA_TS(1, 9, "p") JB_MMA_TS(2, 10, "q") JB_MMA_TS(3, 11, "q") JB_MMA_TS(4, 12, "q")
      JB_MMA_TS(5, 13, "q") JB_MMA_TS(6, 14, "q") JB_MMA_TS(7, 15, "q") JB_MMA_TS(8, 16, "q")
      "}" ::"r"(d_tmem), JB_U8(a), JB_L8(b), "r"(acc_first), "r"(idesc)
      : "memory");
}

// Pair versions (issued by the leader CTA of a cluster of 2).
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

#define JB_MMA2_SS(ai, bi, pr) \
  "tcgen05.mma.cta_group::2.kind::f16 [%0], %" #ai ", %" #bi ", %10, " pr ";\n\t"
#define JB_MMA2_SS_TF32(ai, bi, pr) \
  "tcgen05.mma.cta_group::2.kind::tf32 [%0], %" #ai ", %" #bi ", %10, " pr ";\n\t"
// Four K=8 steps of the pair MMA on tf32 operands: D (+)= A[smem] * B[smem].
__device__ __forceinline__ void umma4_pair_ss_tf32(uint32_t d_tmem, const uint64_t (&a)[4],
                                                   const uint64_t (&b)[4], uint32_t acc_first,
                                                   uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %9, 0;\n\t"
      "setp.eq.b32 q, %9, %9;\n\t"
      JB_MMA2_SS_TF32(1, 5, "p") JB_MMA2_SS_TF32(2, 6, "q") JB_MMA2_SS_TF32(3, 7, "q")
      JB_MMA2_SS_TF32(4, 8, "q")
      "}" ::"r"(d_tmem), "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]),
      "l"(b[2]), "l"(b[3]), "r"(acc_first), "r"(idesc)
      : "memory");
}
// Four K=16 steps of the pair MMA: D (+)= A[smem] * B[smem].
__device__ __forceinline__ void umma4_pair_ss(uint32_t d_tmem, const uint64_t (&a)[4],
                                              const uint64_t (&b)[4], uint32_t acc_first,
                                              uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %9, 0;\n\t"
      "setp.eq.b32 q, %9, %9;\n\t"
      JB_MMA2_SS(1, 5, "p") JB_MMA2_SS(2, 6, "q") JB_MMA2_SS(3, 7, "q") JB_MMA2_SS(4, 8, "q")
      "}" ::"r"(d_tmem), "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]),
      "l"(b[2]), "l"(b[3]), "r"(acc_first), "r"(idesc)
      : "memory");
}

// Arrive on the barrier at a shared::cluster address (own CTA or its pair
// peer) when the pair MMAs issued so far by this thread have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_addr) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          cluster_addr)
      : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this
// thread have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Instruction descriptor, kind::f16 with bf16 A/B and fp32 D.
//  bits 4-5 D format (1 = f32), 7-9 A format (1 = bf16), 10-12 B format,
//  15 A major (1 = MN), 16 B major, 17-22 N>>3, 24-28 M>>4.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor for A and B of one type (the two operands always
// share it): kind::f16 with format 0 for f16, 1 for bf16; kind::tf32 (fp32
// operands read as tf32) with format 2.
template <typename T>
__host__ __device__ constexpr uint32_t idesc_f16kind(int M, int N, bool a_mn, bool b_mn) {
  return std::is_same<T, __half>::value
             ? (idesc_bf16_f32(M, N, a_mn, b_mn) & ~((7u << 7) | (7u << 10)))
         : std::is_same<T, float>::value
             ? ((idesc_bf16_f32(M, N, a_mn, b_mn) & ~((7u << 7) | (7u << 10))) | (2u << 7) | (2u << 10))
             : idesc_bf16_f32(M, N, a_mn, b_mn);
}

// fp32 -> tf32 (round to nearest, ties away from zero): the low 13 mantissa
// bits of the result are zero.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand.
//  bits 0-13 start>>4, 16-29 leading byte offset>>4, 32-45 stride byte
//  offset>>4, 46-47 version (1 on sm_100), 61-63 layout (2 = 128B swizzle).
// K-major: rows of 128 B, 8-row groups SBO apart (LBO unused, 16).
// MN-major: 64-element MN chunks LBO apart, 8-row K groups SBO apart.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// ---------------------------------------------------------------------------
// TMEM <-> registers.  32x32b shape: thread t of the warp reads TMEM lane
// (32*(warp%4) + t); .xN reads N consecutive 32-bit columns.
// The wait takes the destination registers as in/out operands so no use of
// them can be scheduled before it.
// ---------------------------------------------------------------------------
#define JB_R8(r, o) "=r"(r[o + 0]), "=r"(r[o + 1]), "=r"(r[o + 2]), "=r"(r[o + 3]), \
                    "=r"(r[o + 4]), "=r"(r[o + 5]), "=r"(r[o + 6]), "=r"(r[o + 7])
#define JB_W8(r, o) "+r"(r[o + 0]), "+r"(r[o + 1]), "+r"(r[o + 2]), "+r"(r[o + 3]), \
                    "+r"(r[o + 4]), "+r"(r[o + 5]), "+r"(r[o + 6]), "+r"(r[o + 7])
#define JB_I8(r, o) "r"(r[o + 0]), "r"(r[o + 1]), "r"(r[o + 2]), "r"(r[o + 3]), \
                    "r"(r[o + 4]), "r"(r[o + 5]), "r"(r[o + 6]), "r"(r[o + 7])

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : JB_R8(r, 0), JB_R8(r, 8), JB_R8(r, 16), JB_R8(r, 24)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : JB_W8(r, 0), JB_W8(r, 8), JB_W8(r, 16), JB_W8(r, 24)
               :
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : JB_R8(r, 0), JB_R8(r, 8)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : JB_W8(r, 0), JB_W8(r, 8) : : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      JB_I8(r, 0), JB_I8(r, 8), JB_I8(r, 16), JB_I8(r, 24)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      JB_I8(r, 0), JB_I8(r, 8)
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Small numeric helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Two floats as one 32-bit pair of the 16-bit element type T (round to
// nearest even), and back.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) { return pack_bf16x2(lo, hi); }
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) { return pack_f16x2(lo, hi); }

template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t v);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t v) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t v) {
  return __half22float2(*reinterpret_cast<const __half2*>(&v));
}

// NVLink multicast stores (NVLS): one store to a multicast address is
// replicated by the NVSwitch into the same offset of every member GPU's
// buffer, this GPU's included.  16 bytes (four 32-bit words, bit patterns
// of any 16-bit or 32-bit type) or one fp32 word.
__device__ __forceinline__ void multimem_st16(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void multimem_st_f32(float* mc, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc), "f"(v) : "memory");
}
// Orders this thread's accesses through the multicast alias of a buffer
// before its later accesses through other aliases (the signal that follows
// the stores goes through unicast addresses).
__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

}  // namespace jb
