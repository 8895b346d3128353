// pf_save_blocks_noalloc: the save (pack) path without any device allocation.
//
// Who needs it: callers that cannot call cudaMalloc at the moment they save.
// Examples are an inference engine that hands all free HBM to its own caching
// allocator or KV pool (a stray cudaMalloc can then fail or fragment it), and
// code running under a memory-pool policy that forbids out-of-band
// allocations. The regular executor allocates its staging ring and plan
// buffer with cudaMalloc when it is created and grows the plan buffer on
// demand; this entry point allocates nothing.
//
// How: the scratch it needs lives in two file-scope __device__ arrays of fixed
// size, which every GPU that loads this library holds until the process
// exits:
//   - g_noalloc_plan     (kNoAllocPlanBytes = 1 MiB): layer table, block ids
//                         and staging offsets of one call;
//   - g_noalloc_staging  (kNoAllocStagingBytes = 8 MiB): one staging slot the
//                         pack kernel fills before a copy-engine D2H drains it.
// A save whose plan does not fit in 1 MiB, or which has a copy unit larger
// than the staging slot, is rejected with PF_ERR_INVALID_ARGUMENT.
//
// Set-up: the first call on a device (with that device current) resolves the
// arrays' device addresses with cudaGetSymbolAddress. Every call on a device shares the same arrays
// and leaves its contents behind: nothing in them needs to start at zero (the
// plan is written whole by each call and each staging range is written by the
// kernel before it is copied out). Calls that overlap on the GPU (on
// different streams, or from threads racing on one stream) race on the
// arrays; keep them ordered on one stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.h"
#include "executor.h"
#include "pegaflow.h"
#include "plan.h"

namespace pf {
namespace {

constexpr size_t kNoAllocPlanBytes = 1ull << 20;
constexpr size_t kNoAllocStagingBytes = 8ull << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_plan[kNoAllocPlanBytes];
static __device__ __align__(256) unsigned char g_noalloc_staging[kNoAllocStagingBytes];

struct DeviceScratch {
  bool ready = false;
  uint8_t* plan = nullptr;
  uint8_t* staging = nullptr;
  int sms = 0;
  int ctas = 1;  // resident CTAs per SM of the copy kernel
};
std::mutex g_mu;
DeviceScratch g_dev[kMaxDevices];

uint64_t up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// Resolves the device addresses of the scratch arrays once per device.
DeviceScratch& scratch_for(int device) {
  std::lock_guard<std::mutex> g(g_mu);
  DeviceScratch& d = g_dev[device];
  if (!d.ready) {
    void* p = nullptr;
    cuda_check(cudaGetSymbolAddress(&p, g_noalloc_plan), "cudaGetSymbolAddress(plan)");
    d.plan = static_cast<uint8_t*>(p);
    cuda_check(cudaGetSymbolAddress(&p, g_noalloc_staging), "cudaGetSymbolAddress(staging)");
    d.staging = static_cast<uint8_t*>(p);
    cuda_check(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device), "cudaDeviceGetAttribute");
    d.ctas = std::max(1, std::min(4, copy_kernel_resident_ctas()));
    d.ready = true;
  }
  return d;
}

void save_noalloc(int device, const pf_save_layer* layers, uint64_t n_layers, cudaStream_t stream) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    throw cuda_init("no CUDA device available");
  }
  if (device < 0 || device >= count || device >= kMaxDevices) {
    throw cuda_init("device " + std::to_string(device) + " out of range");
  }
  DeviceGuard on(device);
  DeviceScratch& sc = scratch_for(device);

  // The executor's staged save plan (same checks, geometry, dense layout and
  // host runs), bounded by the fixed scratch arrays.
  Built b;
  plan_save(layers, n_layers, /*staged=*/true, device, check_device_memory, &b);
  if (b.total_tiles == 0) return;
  for (const PlanLayer& p : b.layers) {
    if (p.unit_bytes > kNoAllocStagingBytes / 2) {
      throw invalid_argument("copy unit of " + std::to_string(p.unit_bytes) +
                             " bytes exceeds the no-allocation staging limit (" +
                             std::to_string(kNoAllocStagingBytes / 2) + " bytes)");
    }
  }

  // Serialise the plan into one host image and copy it into the plan array.
  const uint64_t sz_table = up(b.layers.size() * sizeof(PlanLayer), 16);
  const uint64_t sz_ids = up(b.ids.size() * sizeof(uint32_t), 16);
  const uint64_t sz_bases = up(b.side_base.size() * sizeof(uint64_t), 16);
  const uint64_t total = sz_table + sz_ids + sz_bases;
  if (total > kNoAllocPlanBytes) {
    throw invalid_argument("save plan of " + std::to_string(total) + " bytes exceeds the no-allocation limit (" +
                           std::to_string(kNoAllocPlanBytes) + " bytes); split the save");
  }
  std::vector<uint8_t> image(total, 0);
  std::memcpy(image.data(), b.layers.data(), b.layers.size() * sizeof(PlanLayer));
  std::memcpy(image.data() + sz_table, b.ids.data(), b.ids.size() * sizeof(uint32_t));
  std::memcpy(image.data() + sz_table + sz_ids, b.side_base.data(), b.side_base.size() * sizeof(uint64_t));
  // A pageable source: the call returns once the bytes are staged, so the
  // image may go out of scope afterwards.
  cuda_check(cudaMemcpyAsync(sc.plan, image.data(), total, cudaMemcpyHostToDevice, stream), "cudaMemcpyAsync(plan)");

  CopyArgs a{};
  a.layers = reinterpret_cast<const PlanLayer*>(sc.plan);
  a.ids = reinterpret_cast<const uint32_t*>(sc.plan + sz_table);
  a.side_base = reinterpret_cast<const uint64_t*>(sc.plan + sz_table + sz_ids);
  a.side_ptrs = nullptr;
  a.layer_tiles_done = nullptr;
  a.layer_done = nullptr;
  a.n_layers = static_cast<uint32_t>(b.layers.size());

  // Chunks of whole tiles that each fit the one staging slot (the executor's
  // cutter); each is packed, then drained by D2H copies of its own bytes
  // [dense_first, dense_end), in order on the caller's stream.
  std::vector<Chunk> chunks;
  cut_chunks(b.layers, b.total_tiles, kNoAllocStagingBytes, kNoAllocStagingBytes, &chunks);
  const uint64_t max_grid = static_cast<uint64_t>(sc.sms) * sc.ctas;
  for (const Chunk& c : chunks) {
    a.tile_begin = c.tile_begin;
    a.tile_end = c.tile_end;
    a.side_shift = static_cast<int64_t>(reinterpret_cast<uint64_t>(sc.staging)) - static_cast<int64_t>(c.dense_begin);
    const uint64_t grid = std::max<uint64_t>(1, std::min<uint64_t>((c.tile_end - c.tile_begin + 7) / 8, max_grid));
    cuda_check(launch_copy(kPack, false, a, static_cast<int>(grid), stream), "kernel launch");
    auto it = std::upper_bound(b.runs.begin(), b.runs.end(), c.dense_first,
                               [](uint64_t v, const Run& r) { return v < r.dense + r.bytes; });
    for (; it != b.runs.end() && it->dense < c.dense_end; ++it) {
      const uint64_t lo = std::max(it->dense, c.dense_first);
      const uint64_t hi = std::min(it->dense + it->bytes, c.dense_end);
      if (hi <= lo) continue;
      cuda_check(cudaMemcpyAsync(reinterpret_cast<void*>(it->host + (lo - it->dense)),
                                 sc.staging + (lo - c.dense_begin), hi - lo, cudaMemcpyDeviceToHost, stream),
                 "cudaMemcpyAsync D2H");
    }
  }
}

}  // namespace
}  // namespace pf

extern "C" int pf_save_blocks_noalloc(int32_t device_id, const pf_save_layer* layers, uint64_t n_layers,
                                      void* stream) {
  if (!layers && n_layers) {
    pf::set_last_error("invalid argument: null layers");
    return PF_ERR_INVALID_ARGUMENT;
  }
  return pf::guarded([&] { pf::save_noalloc(device_id, layers, n_layers, static_cast<cudaStream_t>(stream)); });
}
