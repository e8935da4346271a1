#include "host_arena.h"

#include <sys/mman.h>

#include <cstring>
#include <stdexcept>
#include <string>

namespace lkrt {

HostArena::HostArena(size_t capacity) {
  const size_t page = 2u << 20;  // round to 2 MiB so the whole mapping can use huge pages
  cap_ = (capacity + page - 1) / page * page;
  if (cap_ == 0) cap_ = page;
  void* p = mmap(nullptr, cap_, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  if (p == MAP_FAILED) throw std::runtime_error("HostArena: mmap of " + std::to_string(cap_) + " bytes failed");
#ifdef MADV_HUGEPAGE
  madvise(p, cap_, MADV_HUGEPAGE);  // advisory; ignored where THP is off
#endif
  std::memset(p, 0, cap_);  // first touch on the caller's (NUMA-pinned) thread
  base_ = p;
}

HostArena::~HostArena() {
  if (base_) munmap(base_, cap_);
}

void* HostArena::allocate(size_t bytes, size_t align) {
  if (align == 0 || (align & (align - 1))) throw std::invalid_argument("HostArena: alignment must be a power of two");
  std::lock_guard<std::mutex> g(m_);
  const uintptr_t b = (uintptr_t)base_;
  const uintptr_t start = (b + used_ + align - 1) & ~(uintptr_t)(align - 1);
  if (start + bytes > b + cap_) return nullptr;
  used_ = start + bytes - b;
  if (used_ > peak_) peak_ = used_;
  ++count_;
  return (void*)start;
}

void HostArena::reset() {
  std::lock_guard<std::mutex> g(m_);
  used_ = 0;
  count_ = 0;
}

}  // namespace lkrt
