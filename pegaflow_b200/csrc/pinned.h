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
  // numa_node >= 0 places the pages on that NUMA node (best effort): the
  // range is mmap'ed, bound with mbind(MPOL_PREFERRED), and then registered
  // with cudaHostRegister(Portable|Mapped) instead of cudaHostAlloc, which
  // has no placement control. Registered memory cannot be write-combined, so
  // write_combined is ignored then.
  PinnedMemory(size_t size, PinKind kind, bool write_combined, int numa_node = -1);
  ~PinnedMemory();
  PinnedMemory(const PinnedMemory&) = delete;
  PinnedMemory& operator=(const PinnedMemory&) = delete;

  uint8_t* data() const { return ptr_; }
  size_t size() const { return size_; }
  PinKind kind() const { return kind_; }
  // The node asked for, or -1; numa_bound() says whether mbind accepted it.
  int numa_node() const { return numa_node_; }
  bool numa_bound() const { return numa_bound_; }

 private:
  uint8_t* ptr_ = nullptr;
  size_t size_ = 0;
  PinKind kind_;
  int numa_node_ = -1;
  bool numa_bound_ = false;
  bool mapped_ = false;      // ptr_ came from mmap (munmap on destruction)
  bool registered_ = false;  // ptr_ was registered with cudaHostRegister
};

// Huge page size from /proc/meminfo (pinned_mem.rs:37-52), 0 if unknown.
size_t huge_page_size();
// NUMA node of the page at p (get_mempolicy), or -1 when unknown.
int numa_node_of(const void* p);
// NUMA node of a CUDA device from sysfs (via its PCI bus id), or -1.
int device_numa_node(int device);

// Registry of device-reachable pinned ranges.
void pinned_register(const void* p, size_t bytes);
void pinned_unregister(const void* p);
bool pinned_contains(const void* p, size_t bytes);

}  // namespace pf
