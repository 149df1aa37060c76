//===- FlashAttention.h - flash attention on B200 (sm_100a) ------*- C++ -*-===//
//
// Drop-in replacement for the reference's attention entry points
// (AVmakeralt/jules include/jules/Kernel/FlashAttention.h:42-134).  Same
// signatures; float* are HOST pointers [batch, heads, seq, head_dim]; the
// call stages to the GPU, runs the fp32 kernel and copies O back.
//
// flashAttentionBf16 is the device-pointer extension the configs need:
// bf16 in/out, causal mask, grouped-query heads and a logsumexp output.
//
//===----------------------------------------------------------------------===//
#ifndef JULES_KERNEL_FLASH_ATTENTION_H
#define JULES_KERNEL_FLASH_ATTENTION_H

#include "jules/Kernel/ExecutionArena.h"
#include "jules/Kernel/FusedKernels.h"
#include "jules/Kernel/TilePlanner.h"

namespace jules {
namespace kernel {

void flashAttention(float* output, const float* Q, const float* K, const float* V, int batch,
                    int heads, int seq, int head_dim, ExecutionArena& arena, TilePlanner& planner);

void standardAttention(float* output, const float* Q, const float* K, const float* V, int batch,
                       int heads, int seq, int head_dim, ExecutionArena& arena);

void attention(float* output, const float* Q, const float* K, const float* V, int batch, int heads,
               int seq, int head_dim, ExecutionArena& arena, TilePlanner& planner);

// Device pointers, bf16 (stored as uint16_t bit patterns).  Q/O [B,Hq,S,D],
// K/V [B,Hkv,S,D], lse [B,Hq,S] (nullable).  Returns a JULES_* status.
int flashAttentionBf16(uint16_t* output, float* lse, const uint16_t* Q, const uint16_t* K,
                       const uint16_t* V, int batch, int q_heads, int kv_heads, int seq,
                       int head_dim, bool causal, void* stream = nullptr);

}  // namespace kernel
}  // namespace jules

#endif
