#include "pinned.h"

#include <cuda_runtime.h>
#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <map>
#include <mutex>
#include <sstream>
#include <string>

#include "common.h"

namespace pf {

namespace {
std::mutex g_reg_mu;
std::map<uintptr_t, size_t>& registry() {
  static std::map<uintptr_t, size_t> r;
  return r;
}
}  // namespace

void pinned_register(const void* p, size_t bytes) {
  std::lock_guard<std::mutex> g(g_reg_mu);
  registry()[reinterpret_cast<uintptr_t>(p)] = bytes;
}

void pinned_unregister(const void* p) {
  std::lock_guard<std::mutex> g(g_reg_mu);
  registry().erase(reinterpret_cast<uintptr_t>(p));
}

bool pinned_contains(const void* p, size_t bytes) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  std::lock_guard<std::mutex> g(g_reg_mu);
  auto& r = registry();
  auto it = r.upper_bound(a);
  if (it == r.begin()) return false;
  --it;
  return a >= it->first && a + bytes <= it->first + it->second && a + bytes >= a;
}

size_t huge_page_size() {
  std::ifstream f("/proc/meminfo");
  std::string line;
  while (std::getline(f, line)) {
    if (line.rfind("Hugepagesize:", 0) == 0) {
      std::istringstream is(line);
      std::string key, unit;
      size_t kb = 0;
      is >> key >> kb >> unit;
      if (unit == "kB") return kb * 1024;
    }
  }
  return 0;
}

namespace {

// Linux memory-policy modes and flags (uapi/linux/mempolicy.h).
constexpr int kMpolPreferred = 1;
constexpr int kMpolFNode = 1 << 0;
constexpr int kMpolFAddr = 1 << 1;
constexpr int kMaxNodes = 1024;

// mbind(MPOL_PREFERRED, {node}) on [p, p + bytes); false when refused.
bool bind_to_node(void* p, size_t bytes, int node) {
  if (node < 0 || node >= kMaxNodes) return false;
  unsigned long mask[kMaxNodes / (8 * sizeof(unsigned long))] = {};
  mask[node / (8 * sizeof(unsigned long))] = 1ul << (node % (8 * sizeof(unsigned long)));
  return syscall(SYS_mbind, p, bytes, kMpolPreferred, mask, static_cast<unsigned long>(kMaxNodes), 0u) == 0;
}

}  // namespace

int numa_node_of(const void* p) {
  int node = -1;
  if (syscall(SYS_get_mempolicy, &node, nullptr, 0ul, const_cast<void*>(p), kMpolFNode | kMpolFAddr) != 0) {
    return -1;
  }
  return node;
}

int device_numa_node(int device) {
  char bus[32] = {};
  if (cudaDeviceGetPCIBusId(bus, sizeof(bus), device) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  std::string id(bus);
  std::transform(id.begin(), id.end(), id.begin(), [](unsigned char c) { return std::tolower(c); });
  std::ifstream f("/sys/bus/pci/devices/" + id + "/numa_node");
  int node = -1;
  if (!(f >> node)) return -1;
  return node;
}

PinnedMemory::PinnedMemory(size_t size, PinKind kind, bool write_combined, int numa_node)
    : kind_(kind), numa_node_(numa_node) {
  if (size == 0) throw Error(PF_ERR_INVALID_ARGUMENT, "size must be greater than zero");
  if (numa_node >= 0 && kind != PinKind::kHugePagesRegistered) {
    // Placement needs memory this library maps itself: mmap, bind, then pin
    // in place (the page faults cudaHostRegister takes follow the binding).
    const size_t aligned = (size + 4095) & ~size_t(4095);
    void* p = mmap(nullptr, aligned, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
    if (p == MAP_FAILED) throw cuda_init("mmap failed for a pool on NUMA node " + std::to_string(numa_node));
    numa_bound_ = bind_to_node(p, aligned, numa_node);
    if (!numa_bound_) {
      fprintf(stderr, "pegaflow_b200: mbind to NUMA node %d refused (errno %d); pool pages are not placed\n",
              numa_node, errno);
    }
    ptr_ = static_cast<uint8_t*>(p);
    size_ = aligned;
    mapped_ = true;
    if (kind == PinKind::kCudaHostAlloc) {
      cudaError_t err = cudaHostRegister(p, aligned, cudaHostRegisterPortable | cudaHostRegisterMapped);
      if (err != cudaSuccess) {
        cudaGetLastError();
        munmap(p, aligned);
        ptr_ = nullptr;
        throw cuda_init(std::string("cudaHostRegister failed: ") + cudaGetErrorString(err));
      }
      registered_ = true;
      pinned_register(ptr_, size_);
    }
    return;
  }
  switch (kind) {
    case PinKind::kCudaHostAlloc: {
      unsigned flags = cudaHostAllocPortable | cudaHostAllocMapped;
      if (write_combined) flags |= cudaHostAllocWriteCombined;
      void* p = nullptr;
      cudaError_t err = cudaHostAlloc(&p, size, flags);
      if (err != cudaSuccess) {
        cudaGetLastError();
        throw cuda_init(std::string("cudaHostAlloc failed: ") + cudaGetErrorString(err));
      }
      ptr_ = static_cast<uint8_t*>(p);
      size_ = size;
      break;
    }
    case PinKind::kHugePagesRegistered: {
      const size_t hp = huge_page_size();
      if (hp == 0) {
        throw cuda_init("cannot determine huge page size: Hugepagesize not found in /proc/meminfo");
      }
      const size_t aligned = (size + hp - 1) & ~(hp - 1);
      void* p = mmap(nullptr, aligned, PROT_READ | PROT_WRITE,
                     MAP_PRIVATE | MAP_ANONYMOUS | MAP_HUGETLB, -1, 0);
      if (p == MAP_FAILED) throw cuda_init("mmap failed (MAP_HUGETLB)");
      if (numa_node >= 0) numa_bound_ = bind_to_node(p, aligned, numa_node);
      cudaError_t err = cudaHostRegister(p, aligned, cudaHostRegisterPortable | cudaHostRegisterMapped);
      if (err != cudaSuccess) {
        cudaGetLastError();
        munmap(p, aligned);
        throw cuda_init(std::string("cudaHostRegister failed: ") + cudaGetErrorString(err));
      }
      ptr_ = static_cast<uint8_t*>(p);
      size_ = aligned;
      break;
    }
    case PinKind::kPlainHost: {
      void* p = nullptr;
      if (posix_memalign(&p, 4096, size) != 0) throw std::bad_alloc();
      ptr_ = static_cast<uint8_t*>(p);
      size_ = size;
      break;
    }
  }
  if (kind != PinKind::kPlainHost) pinned_register(ptr_, size_);
}

PinnedMemory::~PinnedMemory() {
  if (!ptr_) return;
  if (mapped_ && kind_ != PinKind::kHugePagesRegistered) {  // placed on a NUMA node
    if (registered_) {
      pinned_unregister(ptr_);
      if (cudaHostUnregister(ptr_) != cudaSuccess) cudaGetLastError();
    }
    munmap(ptr_, size_);
    return;
  }
  if (kind_ != PinKind::kPlainHost) pinned_unregister(ptr_);
  switch (kind_) {
    case PinKind::kCudaHostAlloc:
      if (cudaFreeHost(ptr_) != cudaSuccess) {
        fprintf(stderr, "pegaflow_b200: cudaFreeHost failed\n");
        cudaGetLastError();
      }
      break;
    case PinKind::kHugePagesRegistered:
      if (cudaHostUnregister(ptr_) != cudaSuccess) cudaGetLastError();
      munmap(ptr_, size_);
      break;
    case PinKind::kPlainHost:
      free(ptr_);
      break;
  }
}

}  // namespace pf
