// Host staging memory: a bump arena over one aligned, huge-page-advised
// mapping.
//
// Allocation is a pointer bump (alignment 256 B, the granularity the copy
// engines like); `reset()` releases everything at once.  The mapping is
// first touched by the calling thread, so with the launcher's NUMA pinning
// (the thread runs on the GPU's node) its pages land next to that GPU.  The
// Python side page-locks the whole mapping once (cudaHostRegister), turning
// every slot carved from it into a DMA-able pinned buffer without one
// cudaHostAlloc per buffer.
//
// Reference: MemoryPool (include/core/memory_pool.hpp:12-53, mmap arena with a
// 64-byte bump pointer and reset) and MemoryManager::allocate
// (include/core/memory_manager.hpp:287-329, mmap + MAP_HUGETLB + mbind).
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>

namespace lkrt {

class HostArena {
 public:
  explicit HostArena(size_t capacity);
  ~HostArena();
  HostArena(const HostArena&) = delete;
  HostArena& operator=(const HostArena&) = delete;

  // nullptr when the arena is exhausted
  void* allocate(size_t bytes, size_t align = 256);
  void reset();

  void* base() const { return base_; }
  size_t capacity() const { return cap_; }
  size_t used() const { return used_; }
  size_t peak() const { return peak_; }
  size_t allocations() const { return count_; }

 private:
  void* base_ = nullptr;
  size_t cap_ = 0;
  size_t used_ = 0;
  size_t peak_ = 0;
  size_t count_ = 0;
  std::mutex m_;
};

}  // namespace lkrt
