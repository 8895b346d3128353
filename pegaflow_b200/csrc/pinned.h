// Pinned host memory (the reference's PinnedMemory, pegaflow-core/src/pinned_mem.rs)
// plus a registry of the ranges this library pinned, so zero-copy kernels are
// only ever pointed at memory the GPU can reach.
#pragma once

#include <cstddef>
#include <cstdint>

namespace pf {

enum class PinKind { kCudaHostAlloc, kHugePagesRegistered, kPlainHost };

class PinnedMemory {
 public:
  // kCudaHostAlloc: cudaHostAlloc(Portable | Mapped [| WriteCombined])
  //   (pinned_mem.rs:155-164 uses WriteCombined only; Portable+Mapped make the
  //   pool valid in every device context and addressable by kernels).
  // kHugePagesRegistered: mmap(MAP_HUGETLB) + cudaHostRegister(Portable|Mapped)
  //   (pinned_mem.rs:165-197).
  // kPlainHost: aligned pageable memory for host-logic tests; never handed to
  //   a GPU (the engine refuses transfers on it).
  PinnedMemory(size_t size, PinKind kind, bool write_combined);
  ~PinnedMemory();
  PinnedMemory(const PinnedMemory&) = delete;
  PinnedMemory& operator=(const PinnedMemory&) = delete;

  uint8_t* data() const { return ptr_; }
  size_t size() const { return size_; }
  PinKind kind() const { return kind_; }

 private:
  uint8_t* ptr_ = nullptr;
  size_t size_ = 0;
  PinKind kind_;
};

// Huge page size from /proc/meminfo (pinned_mem.rs:37-52), 0 if unknown.
size_t huge_page_size();

// Registry of device-reachable pinned ranges.
void pinned_register(const void* p, size_t bytes);
void pinned_unregister(const void* p);
bool pinned_contains(const void* p, size_t bytes);

}  // namespace pf
