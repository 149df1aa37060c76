//===- ExecutionArena.h - device workspace arena (B200) --------*- C++ -*-===//
//
// Same names and members as the reference's ExecutionArena / CacheInfo
// (AVmakeralt/jules include/jules/Kernel/ExecutionArena.h:41-199), but the
// arena is a block of GPU memory: allocate<T>() returns DEVICE pointers
// (64-byte aligned bump allocation, reset() frees everything) and overflow
// throws std::bad_alloc instead of calling abort() (:140-143).
// CacheInfo describes the GPU: l1d_bytes = shared memory per SM, l2_bytes and
// l3_bytes = L2 size (the GPU has no L3), line_bytes = 128, num_cores = SMs.
//
//===----------------------------------------------------------------------===//
#ifndef JULES_KERNEL_EXECUTION_ARENA_H
#define JULES_KERNEL_EXECUTION_ARENA_H

#include <cstddef>
#include <cstdint>
#include <new>

namespace jules {
namespace kernel {

struct CacheInfo {
  size_t l1d_bytes;
  size_t l2_bytes;
  size_t l3_bytes;
  size_t line_bytes;
  int num_cores;
  static CacheInfo detect();
};

class ExecutionArena {
 public:
  static constexpr size_t DEFAULT_MAX_SIZE = 256UL * 1024 * 1024;
  explicit ExecutionArena(size_t maxSize = DEFAULT_MAX_SIZE);
  ~ExecutionArena();
  ExecutionArena(const ExecutionArena&) = delete;
  ExecutionArena& operator=(const ExecutionArena&) = delete;

  template <typename T>
  T* allocate(size_t count) {
    return static_cast<T*>(allocateBytes(count * sizeof(T)));
  }
  void* allocateBytes(size_t bytes);
  void reset() { offset_ = 0; }
  void resetAndZero();
  // Host-side prefetch hints have no GPU meaning; kept for source
  // compatibility and ignored.
  void prefetch(const void*, size_t, int = 1) const {}
  template <typename T>
  void prefetchTensor(const T*, size_t, int = 1) const {}

  size_t usedBytes() const { return offset_; }
  size_t highWaterMark() const { return highWaterMark_; }
  size_t capacity() const { return maxSize_; }
  char* rawBuffer() { return buffer_; }
  const char* rawBuffer() const { return buffer_; }

 private:
  char* buffer_;
  size_t maxSize_;
  size_t offset_;
  size_t highWaterMark_;
};

}  // namespace kernel
}  // namespace jules

#endif
