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
// arrays' device addresses with cudaGetSymbolAddress; make that first call
// before any stream capture. Every call on a device shares the same arrays
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
constexpr uint64_t kAlign = 256;
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

struct Extent {  // one contiguous dense range and its host destination
  uint64_t dense, host, bytes;
};

void save_noalloc(int device, const pf_save_layer* layers, uint64_t n_layers, cudaStream_t stream) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    throw cuda_init("no CUDA device available");
  }
  if (device < 0 || device >= count || device >= kMaxDevices) {
    throw cuda_init("device " + std::to_string(device) + " out of range");
  }
  cuda_check(cudaSetDevice(device), "cudaSetDevice");
  DeviceScratch& sc = scratch_for(device);

  // Plan: the same per-layer geometry and checks as the executor's save.
  std::vector<PlanLayer> table;
  std::vector<uint32_t> ids;
  std::vector<uint64_t> bases;
  std::vector<Extent> extents;
  uint64_t tiles = 0, dense = 0;
  for (uint64_t li = 0; li < n_layers; ++li) {
    const pf_save_layer& s = layers[li];
    const pf_layer_desc& l = s.layer;
    const std::string name = "#" + std::to_string(li);
    validate_layout(l, name.c_str());
    if (s.n == 0) continue;
    if (!s.block_idx || !s.k_dst) throw invalid_argument("null block list or destination");
    if (l.num_blocks > 0xffffffffull) throw invalid_argument("too many blocks for one layer");
    for (uint64_t addr : {l.data_ptr, l.data_ptr + l.size_bytes - 1}) {
      cudaPointerAttributes attr{};
      if (cudaPointerGetAttributes(&attr, reinterpret_cast<const void*>(addr)) != cudaSuccess) {
        cudaGetLastError();
        throw invalid_argument("KV tensor address is not CUDA memory");
      }
      if ((attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) || attr.device != device) {
        throw invalid_argument("KV tensor is not device memory of device " + std::to_string(device));
      }
    }
    const UnitGeometry g = save_geometry(l);
    if (g.unit_bytes > kNoAllocStagingBytes / 2) {
      throw invalid_argument("copy unit of " + std::to_string(g.unit_bytes) +
                             " bytes exceeds the no-allocation staging limit (" +
                             std::to_string(kNoAllocStagingBytes / 2) + " bytes)");
    }
    for (uint64_t i = 0; i < s.n; ++i) {
      const int64_t b = s.block_idx[i];
      if (b < 0 || static_cast<uint64_t>(b) >= l.num_blocks) {
        throw invalid_argument("block " + std::to_string(b) + " out of range for layer " + name + " (" +
                               std::to_string(l.num_blocks) + " blocks registered)");
      }
      for (uint64_t sg = 0; sg < (is_split_layout(l) ? 2u : (is_contiguous_layout(l) ? 1u : l.segments)); ++sg) {
        segment_offset(l, static_cast<uint64_t>(b), sg);
      }
      for (uint32_t u = 0; u < g.units; ++u) {
        const uint64_t end = static_cast<uint64_t>(b) * l.bytes_per_block + u * g.unit_stride + g.unit_bytes;
        if (end > l.size_bytes) throw storage_error("Block " + std::to_string(b) + " exceeds registered memory");
      }
    }
    // Host destinations, as in Executor::build_save.
    std::vector<uint64_t> host(g.units);
    uint64_t pitch;
    const uint64_t k = reinterpret_cast<uint64_t>(s.k_dst);
    if (is_split_layout(l)) {
      host[0] = k;
      host[1] = s.v_dst ? reinterpret_cast<uint64_t>(s.v_dst) : k + l.bytes_per_block;
      pitch = s.v_dst ? l.bytes_per_block : 2 * l.bytes_per_block;
    } else if (is_contiguous_layout(l)) {
      host[0] = k;
      pitch = l.bytes_per_block * l.segments;
    } else {
      for (uint32_t u = 0; u < g.units; ++u) host[u] = k + u * l.bytes_per_block;
      pitch = l.bytes_per_block * l.segments;
    }
    PlanLayer p{};
    p.cache_base = l.data_ptr;
    p.block_pitch = l.bytes_per_block;
    p.unit_stride = g.unit_stride;
    p.side_pitch = g.unit_bytes;
    p.unit_bytes = static_cast<uint32_t>(g.unit_bytes);
    p.units = g.units;
    p.n = static_cast<uint32_t>(s.n);
    p.tiles_per_unit = static_cast<uint32_t>((g.unit_bytes + kTileBytes - 1) / kTileBytes);
    p.tile_start = tiles;
    p.tile_count = static_cast<uint64_t>(g.units) * s.n * p.tiles_per_unit;
    p.ids_off = static_cast<uint32_t>(ids.size());
    p.side_off = static_cast<uint32_t>(bases.size());
    p.done_index = static_cast<uint32_t>(li);
    const bool vec = (l.data_ptr | l.bytes_per_block | g.unit_stride | g.unit_bytes) % 16 == 0;
    p.flags = vec ? kFlagVector : 0u;
    dense = up(dense, kAlign);
    for (uint32_t u = 0; u < g.units; ++u) {
      bases.push_back(dense + static_cast<uint64_t>(u) * s.n * g.unit_bytes);
      for (uint64_t i = 0; i < s.n; ++i) {
        const uint64_t d = dense + (u * s.n + i) * g.unit_bytes;
        const uint64_t h = host[u] + i * pitch;
        if (!extents.empty() && extents.back().dense + extents.back().bytes == d &&
            extents.back().host + extents.back().bytes == h) {
          extents.back().bytes += g.unit_bytes;
        } else {
          extents.push_back({d, h, g.unit_bytes});
        }
      }
    }
    for (uint64_t i = 0; i < s.n; ++i) ids.push_back(static_cast<uint32_t>(s.block_idx[i]));
    dense += static_cast<uint64_t>(g.units) * s.n * g.unit_bytes;
    tiles += p.tile_count;
    table.push_back(p);
  }
  if (tiles == 0) return;

  // Serialise the plan into one host image and copy it into the plan array.
  const uint64_t sz_table = up(table.size() * sizeof(PlanLayer), 16);
  const uint64_t sz_ids = up(ids.size() * sizeof(uint32_t), 16);
  const uint64_t sz_bases = up(bases.size() * sizeof(uint64_t), 16);
  const uint64_t total = sz_table + sz_ids + sz_bases;
  if (total > kNoAllocPlanBytes) {
    throw invalid_argument("save plan of " + std::to_string(total) + " bytes exceeds the no-allocation limit (" +
                           std::to_string(kNoAllocPlanBytes) + " bytes); split the save");
  }
  std::vector<uint8_t> image(total, 0);
  std::memcpy(image.data(), table.data(), table.size() * sizeof(PlanLayer));
  std::memcpy(image.data() + sz_table, ids.data(), ids.size() * sizeof(uint32_t));
  std::memcpy(image.data() + sz_table + sz_ids, bases.data(), bases.size() * sizeof(uint64_t));
  cuda_check(cudaMemcpyAsync(sc.plan, image.data(), total, cudaMemcpyHostToDevice, stream), "cudaMemcpyAsync(plan)");

  CopyArgs a{};
  a.layers = reinterpret_cast<const PlanLayer*>(sc.plan);
  a.ids = reinterpret_cast<const uint32_t*>(sc.plan + sz_table);
  a.side_base = reinterpret_cast<const uint64_t*>(sc.plan + sz_table + sz_ids);
  a.side_ptrs = nullptr;
  a.layer_tiles_done = nullptr;
  a.layer_done = nullptr;
  a.n_layers = static_cast<uint32_t>(table.size());

  // Chunks of whole tiles whose dense span fits the staging slot; each chunk
  // is packed, then drained by D2H copies, in order on the caller's stream.
  const uint64_t slot = kNoAllocStagingBytes;
  // db: the chunk's slot base (its first byte rounded down to kAlign); df: its
  // first byte. Only [df, de) is copied out: the slot bytes before df were not
  // packed by this chunk and would overwrite the previous chunk's last bytes.
  auto flush = [&](uint64_t tb, uint64_t te, uint64_t db, uint64_t df, uint64_t de) {
    a.tile_begin = tb;
    a.tile_end = te;
    a.side_shift = static_cast<int64_t>(reinterpret_cast<uint64_t>(sc.staging)) - static_cast<int64_t>(db);
    const uint64_t grid = std::min<uint64_t>((te - tb + 7) / 8, static_cast<uint64_t>(sc.sms) * sc.ctas);
    cuda_check(launch_copy(kPack, false, a, static_cast<int>(std::max<uint64_t>(grid, 1)), stream), "kernel launch");
    for (const Extent& e : extents) {
      const uint64_t lo = std::max(e.dense, df), hi = std::min(e.dense + e.bytes, de);
      if (hi <= lo) continue;
      cuda_check(cudaMemcpyAsync(reinterpret_cast<void*>(e.host + (lo - e.dense)), sc.staging + (lo - db), hi - lo,
                                 cudaMemcpyDeviceToHost, stream),
                 "cudaMemcpyAsync D2H");
    }
  };
  uint64_t cur_tb = 0, cur_db = 0, cur_df = 0, last_end = 0;
  bool first = true;
  uint64_t d = 0;
  for (const PlanLayer& p : table) {
    d = up(d, kAlign);
    const uint64_t nunits = static_cast<uint64_t>(p.units) * p.n;
    for (uint64_t ul = 0; ul < nunits; ++ul) {
      const uint64_t ud = d + ul * p.unit_bytes, ue = ud + p.unit_bytes;
      const uint64_t ut = p.tile_start + ul * p.tiles_per_unit;
      if (first) {
        cur_tb = ut;
        cur_df = ud;
        cur_db = ud / kAlign * kAlign;
        first = false;
      }
      if (ue - cur_db <= slot) {
        last_end = ue;
        continue;
      }
      for (uint32_t t = 0; t < p.tiles_per_unit; ++t) {
        const uint64_t d0 = ud + static_cast<uint64_t>(t) * kTileBytes;
        const uint64_t d1 = std::min<uint64_t>(d0 + kTileBytes, ue);
        if (d1 - cur_db > slot) {
          flush(cur_tb, ut + t, cur_db, cur_df, last_end);
          cur_tb = ut + t;
          cur_df = d0;
          cur_db = d0 / kAlign * kAlign;
        }
        last_end = d1;
      }
    }
    d += nunits * p.unit_bytes;
  }
  flush(cur_tb, tiles, cur_db, cur_df, last_end);
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
