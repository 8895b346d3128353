// Transfer executor: plan building, validation, staging-ring pipeline.
//
// Save (staged):  pack kernel -> HBM slot  ==event==>  D2H DMA -> pinned pool
// Load (staged):  H2D DMA -> HBM slot  ==event==>  unpack kernel -> paged KV
// Slots form a ring; a slot is refilled only after the consumer of its last
// contents has finished (ev_drained). Several copy streams keep more than one
// DMA in flight on the host link. Saves and loads each have a lane of their
// own (streams, ring, plan buffers, host lock), so the two directions of the
// link are used at once. Direct mode skips the ring: the kernel reads/writes
// mapped pinned host memory itself. The chunks a transfer moves through the
// ring are cut by cut_chunks (chunks.cpp).
#include "executor.h"

#include <algorithm>
#include <chrono>
#include <cstring>
#include <memory>
#include <string>

#include "common.h"
#include "pinned.h"

namespace pf {

// ---------------------------------------------------------------------------
// Host timing, and the plans' one CUDA-side check (the plans themselves:
// plan_build.cpp)
// ---------------------------------------------------------------------------

namespace {

// Adds the calling thread's time in a save/load/p2p call to stats.host_ms,
// under the stats mutex, when the call returns or throws.
struct HostTimer {
  double* acc;
  std::mutex* mu;
  std::chrono::steady_clock::time_point t0 = std::chrono::steady_clock::now();
  ~HostTimer() {
    const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    std::lock_guard<std::mutex> g(*mu);
    *acc += ms;
  }
};

}  // namespace

void check_device_memory(int device, const pf_layer_desc& l) {
  for (uint64_t addr : {l.data_ptr, l.data_ptr + l.size_bytes - 1}) {
    cudaPointerAttributes attr{};
    cudaError_t err = cudaPointerGetAttributes(&attr, reinterpret_cast<const void*>(addr));
    if (err != cudaSuccess) {
      cudaGetLastError();
      throw invalid_argument("KV tensor address is not CUDA memory");
    }
    if ((attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) || attr.device != device) {
      throw invalid_argument("KV tensor is not device memory of device " + std::to_string(device));
    }
  }
}

// ---------------------------------------------------------------------------
// Executor lifecycle
// ---------------------------------------------------------------------------

Executor::Executor(int device, const pf_executor_config& cfg) : device_(device), cfg_(cfg) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    throw cuda_init("no CUDA device available");
  }
  if (device < 0 || device >= count) {
    throw cuda_init("device " + std::to_string(device) + " out of range (" + std::to_string(count) + " devices)");
  }
  DeviceGuard on(device);
  cuda_check(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device), "cudaDeviceGetAttribute");
  if (cfg_.staging_chunk_bytes == 0) cfg_.staging_chunk_bytes = kDefaultSlotBytes;
  if (cfg_.staging_slots == 0) cfg_.staging_slots = kDefaultSlots;
  if (cfg_.ctas_per_sm == 0) cfg_.ctas_per_sm = 4;
  // One full wave: never ask for more CTAs per SM than stay resident.
  cfg_.ctas_per_sm = std::min<uint32_t>(cfg_.ctas_per_sm, std::max(1, copy_kernel_resident_ctas()));
  if (cfg_.copy_streams == 0) cfg_.copy_streams = 2;
  if (cfg_.save_mode == PF_MODE_AUTO) cfg_.save_mode = PF_MODE_STAGED;
  if (cfg_.load_mode == PF_MODE_AUTO) cfg_.load_mode = PF_MODE_STAGED;
  // A slot must hold one tile plus the alignment slack of a chunk start.
  slot_bytes_ = align_up(std::max<uint64_t>(cfg_.staging_chunk_bytes, 2 * kTileBytes), kDenseAlign);
  slots_ = std::max<uint32_t>(cfg_.staging_slots, 1);
  if (cfg_.first_chunk_bytes == 0) cfg_.first_chunk_bytes = kDefaultFirstChunkBytes;
  first_chunk_ = std::min(slot_bytes_, std::max<uint64_t>(cfg_.first_chunk_bytes, 2 * kTileBytes));

  cuda_check(cudaStreamCreateWithFlags(&own_stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  cuda_check(cudaStreamCreateWithFlags(&save_stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  init_lane(save_lane_);
  init_lane(load_lane_);
  if (cfg_.copy_kernel != PF_COPY_KERNEL_REGISTERS) {
    bulk_ = bulk_copy_ready();
    if (!bulk_ && cfg_.copy_kernel == PF_COPY_KERNEL_BULK) {
      throw cuda_init("the bulk copy kernel cannot run on device " + std::to_string(device));
    }
  }
  void* st = nullptr;
  cuda_check(cudaHostAlloc(&st, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable), "cudaHostAlloc(status)");
  status_host_ = static_cast<volatile int*>(st);
  *status_host_ = 0;
  void* dev = nullptr;
  cuda_check(cudaHostGetDevicePointer(&dev, st, 0), "cudaHostGetDevicePointer(status)");
  status_dev_ = static_cast<int*>(dev);
}

bool Executor::use_bulk(const Built& b) const {
  if (!bulk_) return false;
  for (const PlanLayer& p : b.layers) {
    if ((p.flags & kFlagVector) == 0) return false;
  }
  return true;
}

void Executor::check_kernel_status() {
  if (status_host_ && *status_host_) {
    *status_host_ = 0;
    throw storage_error("a bulk copy kernel gave up waiting for a tile copy (1 s); the copies of that call "
                        "are incomplete");
  }
}

void Executor::init_lane(Lane& l) {
  cuda_check(cudaStreamCreateWithFlags(&l.kstream, cudaStreamNonBlocking), "cudaStreamCreate");
  l.cstreams.resize(cfg_.copy_streams);
  l.ev_copy_done.resize(cfg_.copy_streams);
  for (uint32_t i = 0; i < cfg_.copy_streams; ++i) {
    cuda_check(cudaStreamCreateWithFlags(&l.cstreams[i], cudaStreamNonBlocking), "cudaStreamCreate");
    cuda_check(cudaEventCreateWithFlags(&l.ev_copy_done[i], cudaEventDisableTiming), "cudaEventCreate");
  }
  l.ev_filled.resize(slots_);
  l.ev_drained.resize(slots_);
  for (uint32_t i = 0; i < slots_; ++i) {
    cuda_check(cudaEventCreateWithFlags(&l.ev_filled[i], cudaEventDisableTiming), "cudaEventCreate");
    cuda_check(cudaEventCreateWithFlags(&l.ev_drained[i], cudaEventDisableTiming), "cudaEventCreate");
  }
  cuda_check(cudaEventCreateWithFlags(&l.ev_start, cudaEventDisableTiming), "cudaEventCreate");
  cuda_check(cudaEventCreateWithFlags(&l.ev_plan, cudaEventDisableTiming), "cudaEventCreate");
  cuda_check(cudaEventCreateWithFlags(&l.ev_done, cudaEventDisableTiming), "cudaEventCreate");
  // Nothing is in flight yet: record the "previous call finished" events once.
  cuda_check(cudaEventRecord(l.ev_done, l.kstream), "cudaEventRecord");
  for (uint32_t i = 0; i < cfg_.copy_streams; ++i) {
    cuda_check(cudaEventRecord(l.ev_copy_done[i], l.cstreams[i]), "cudaEventRecord");
  }
}

uint8_t* Executor::lane_staging(Lane& l) {
  // Allocated on first use: a lane that only moves zero-copy transfers never
  // needs it, and a save-only caller holds one lane's worth.
  if (!l.staging) {
    cuda_check(cudaMalloc(reinterpret_cast<void**>(&l.staging), slot_bytes_ * slots_), "cudaMalloc(staging)");
  }
  return l.staging;
}

void Executor::destroy_lane(Lane& l) {
  for (auto e : l.ev_filled) cudaEventDestroy(e);
  for (auto e : l.ev_drained) cudaEventDestroy(e);
  for (auto e : l.ev_copy_done) cudaEventDestroy(e);
  if (l.ev_start) cudaEventDestroy(l.ev_start);
  if (l.ev_plan) cudaEventDestroy(l.ev_plan);
  if (l.ev_done) cudaEventDestroy(l.ev_done);
  for (auto s : l.cstreams) cudaStreamDestroy(s);
  if (l.kstream) cudaStreamDestroy(l.kstream);
  cudaFree(l.staging);
  cudaFree(l.d_plan);
  if (l.h_plan) cudaFreeHost(l.h_plan);
}

Executor::~Executor() {
  std::unique_ptr<DeviceGuard> on;
  try {
    on = std::make_unique<DeviceGuard>(device_);
  } catch (const Error&) {
    // Tear down in whatever context is current; nothing here may throw.
  }
  cudaDeviceSynchronize();
  for (auto& p : timed_) {
    cudaEventDestroy(p.first);
    cudaEventDestroy(p.second);
  }
  for (auto e : event_pool_) cudaEventDestroy(e);
  destroy_lane(save_lane_);
  destroy_lane(load_lane_);
  cudaStreamDestroy(own_stream_);
  cudaStreamDestroy(save_stream_);
  if (status_host_) cudaFreeHost(const_cast<int*>(status_host_));
  cudaFree(spans_);
  cudaGetLastError();
}

void Executor::reset_spans() {
  // {max, 0} so the kernels' atomicMin / atomicMax start from an empty span.
  std::vector<unsigned long long> init(2 * kSpanCap);
  for (uint64_t i = 0; i < kSpanCap; ++i) {
    init[2 * i] = ~0ull;
    init[2 * i + 1] = 0;
  }
  cuda_check(cudaMemcpy(spans_, init.data(), init.size() * sizeof(unsigned long long), cudaMemcpyHostToDevice),
             "cudaMemcpy(spans)");
  spans_used_ = 0;
}

// ---------------------------------------------------------------------------
// Plan building
// ---------------------------------------------------------------------------

void Executor::build_save(const pf_save_layer* layers, uint64_t n_layers, bool staged, Built* b) {
  plan_save(layers, n_layers, staged, device_, check_device_memory, b);
}

void Executor::build_load(const pf_load_layer* layers, uint64_t n_layers, bool staged, Built* b) {
  plan_load(layers, n_layers, staged, device_, check_device_memory, b);
}

void Executor::build_p2p(const pf_p2p_layer* layers, uint64_t n_layers, int peer, bool push, Built* b) {
  plan_p2p(layers, n_layers, device_, peer, push, check_device_memory, b);
}

void Executor::enable_peer(int peer) {
  if (peer == device_) return;  // same-device copies need no peer mapping
  if (std::find(peers_enabled_.begin(), peers_enabled_.end(), peer) != peers_enabled_.end()) return;
  int can = 0;
  cuda_check(cudaDeviceCanAccessPeer(&can, device_, peer), "cudaDeviceCanAccessPeer");
  if (!can) {
    throw invalid_argument("device " + std::to_string(device_) + " cannot access device " + std::to_string(peer));
  }
  const cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
  } else {
    cuda_check(e, "cudaDeviceEnablePeerAccess");
  }
  peers_enabled_.push_back(peer);
}

void Executor::p2p(const pf_p2p_layer* layers, uint64_t n_layers, int peer, bool push, cudaStream_t caller) {
  HostTimer timer{&stats_.host_ms, &stats_mu_};
  DeviceGuard on(device_);
  Lane& L = load_lane_;
  std::lock_guard<std::mutex> g(L.mu);
  enable_peer(peer);
  Built b;
  build_p2p(layers, n_layers, peer, push, &b);
  if (b.total_tiles == 0) return;
  cuda_check(cudaEventRecord(L.ev_start, caller), "cudaEventRecord");
  cuda_check(cudaStreamWaitEvent(L.kstream, L.ev_start, 0), "cudaStreamWaitEvent");
  const CopyArgs args = upload(L, b, false);
  launch(push ? kPack : kUnpack, true, args, 0, b.total_tiles, 0, L.kstream);
  cuda_check(cudaEventRecord(L.ev_done, L.kstream), "cudaEventRecord");
  cuda_check(cudaStreamWaitEvent(caller, L.ev_done, 0), "cudaStreamWaitEvent");
  // kernel bytes: the local HBM side; the other side crosses NVLink
  account(b.total_bytes, 0, 0, 0, b.total_bytes);
}

void Executor::p2p_sync(const pf_p2p_layer* layers, uint64_t n_layers, int peer, bool push) {
  DeviceGuard on(device_);
  p2p(layers, n_layers, peer, push, own_stream_);
  cuda_check(cudaStreamSynchronize(own_stream_), "cudaStreamSynchronize(p2p)");
}

namespace {
void CUDART_CB raise_flag(void* p) { *static_cast<volatile int64_t*>(p) = 1; }
}  // namespace

uint64_t Executor::issue_serial(const Built& b, cudaStream_t s, int64_t* layer_done) {
  // Copies in list order, merged into runs, exactly as batch_copy_segments_to_gpu
  // (transfer.rs:116-198): K list then V list for the split layout, one
  // block_size_bytes list otherwise.
  uint64_t copies = 0;
  for (const SerialLoad& sl : b.serial) {
    const pf_layer_desc& l = sl.layer;
    const bool split = is_split_layout(l);
    const uint64_t unit = split ? l.bytes_per_block : l.bytes_per_block * l.segments;
    for (int u = 0; u < (split ? 2 : 1); ++u) {
      const std::vector<uint64_t>& host = u == 0 ? sl.k : sl.v;
      size_t i = 0;
      while (i < sl.ids.size()) {
        const uint64_t g0 = static_cast<uint64_t>(sl.ids[i]) * l.bytes_per_block + u * l.kv_stride_bytes;
        size_t c = 1;
        while (i + c < sl.ids.size() &&
               static_cast<uint64_t>(sl.ids[i + c]) * l.bytes_per_block + u * l.kv_stride_bytes == g0 + c * unit &&
               host[i + c] == host[i] + c * unit) {
          ++c;
        }
        cuda_check(cudaMemcpyAsync(reinterpret_cast<void*>(l.data_ptr + g0), reinterpret_cast<void*>(host[i]),
                                   c * unit, cudaMemcpyHostToDevice, s),
                   "cudaMemcpyAsync H2D (ordered)");
        copies += 1;
        i += c;
      }
    }
    if (layer_done) cuda_check(cudaLaunchHostFunc(s, raise_flag, layer_done + sl.done_index), "cudaLaunchHostFunc");
  }
  return copies;
}

void Executor::make_chunks(const Built& b, uint64_t first_limit, std::vector<Chunk>* chunks) {
  cut_chunks(b.layers, b.total_tiles, slot_bytes_, first_limit, chunks);
}

CopyArgs Executor::upload(Lane& l, const Built& b, bool with_counters) {
  // The plan is copied on the lane's kernel stream, after the lane's
  // previous kernels (which read the previous plan) and before its own.
  const cudaStream_t s = l.kstream;
  auto a16 = [](size_t v) { return (v + 15) & ~size_t(15); };
  const size_t sz_layers = a16(b.layers.size() * sizeof(PlanLayer));
  const size_t sz_ids = a16(b.ids.size() * sizeof(uint32_t));
  const size_t sz_base = a16(b.side_base.size() * sizeof(uint64_t));
  const size_t sz_ptrs = a16(b.side_ptrs.size() * sizeof(uint64_t));
  const size_t sz_cnt = with_counters ? a16(b.layers.size() * sizeof(unsigned long long)) : 0;
  const size_t total = sz_layers + sz_ids + sz_base + sz_ptrs + sz_cnt;

  // The pinned staging of the previous plan may still be in flight.
  if (l.plan_pending) cuda_check(cudaEventSynchronize(l.ev_plan), "cudaEventSynchronize(plan)");
  if (total > l.h_plan_cap) {
    if (l.h_plan) cudaFreeHost(l.h_plan);
    l.h_plan = nullptr;
    l.h_plan_cap = 0;
    const size_t cap = std::max<size_t>(total * 2, 1 << 16);
    cuda_check(cudaHostAlloc(reinterpret_cast<void**>(&l.h_plan), cap, cudaHostAllocDefault), "cudaHostAlloc(plan)");
    l.h_plan_cap = cap;
  }
  if (total > l.d_plan_cap) {
    cuda_check(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    if (l.d_plan) cudaFree(l.d_plan);
    l.d_plan = nullptr;
    l.d_plan_cap = 0;
    const size_t cap = std::max<size_t>(total * 2, 1 << 16);
    cuda_check(cudaMalloc(reinterpret_cast<void**>(&l.d_plan), cap), "cudaMalloc(plan)");
    l.d_plan_cap = cap;
  }
  uint8_t* h = l.h_plan;
  size_t off = 0;
  std::memcpy(h + off, b.layers.data(), b.layers.size() * sizeof(PlanLayer));
  off += sz_layers;
  std::memcpy(h + off, b.ids.data(), b.ids.size() * sizeof(uint32_t));
  off += sz_ids;
  std::memcpy(h + off, b.side_base.data(), b.side_base.size() * sizeof(uint64_t));
  off += sz_base;
  if (!b.side_ptrs.empty()) std::memcpy(h + off, b.side_ptrs.data(), b.side_ptrs.size() * sizeof(uint64_t));
  off += sz_ptrs;
  if (sz_cnt) std::memset(h + off, 0, sz_cnt);
  cuda_check(cudaMemcpyAsync(l.d_plan, l.h_plan, total, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync(plan)");
  cuda_check(cudaEventRecord(l.ev_plan, s), "cudaEventRecord(plan)");
  l.plan_pending = true;

  uint8_t* d = l.d_plan;
  CopyArgs a{};
  off = 0;
  a.layers = reinterpret_cast<const PlanLayer*>(d + off);
  off += sz_layers;
  a.ids = reinterpret_cast<const uint32_t*>(d + off);
  off += sz_ids;
  a.side_base = reinterpret_cast<const uint64_t*>(d + off);
  off += sz_base;
  a.side_ptrs = reinterpret_cast<const uint64_t*>(d + off);
  off += sz_ptrs;
  a.layer_tiles_done = sz_cnt ? reinterpret_cast<unsigned long long*>(d + off) : nullptr;
  a.n_layers = static_cast<uint32_t>(b.layers.size());
  return a;
}

int Executor::grid_for(uint64_t tiles) const {
  const uint64_t max_grid = static_cast<uint64_t>(num_sms_) * cfg_.ctas_per_sm;
  const uint64_t need = (tiles + 7) / 8;
  return static_cast<int>(std::max<uint64_t>(1, std::min(need, max_grid)));
}

void Executor::launch(Dir dir, bool table, const CopyArgs& args0, uint64_t tile_begin, uint64_t tile_end,
                      int64_t shift, cudaStream_t s, bool bulk) {
  CopyArgs a = args0;
  a.tile_begin = tile_begin;
  a.tile_end = tile_end;
  a.side_shift = shift;
  a.status = status_dev_;
  a.stall_tile = ~0ull;
  const bool use_bulk = bulk && !table && a.layer_tiles_done == nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  {
    std::lock_guard<std::mutex> g(stats_mu_);
    stats_.kernel_launches += 1;
    if (timing_ && spans_ && spans_used_ < kSpanCap) a.span = spans_ + 2 * spans_used_++;
    if (use_bulk && stall_tile_ != ~0ull) {
      a.stall_tile = stall_tile_;
      stall_tile_ = ~0ull;
    }
    if (timing_) {
      auto take = [this]() {
        if (!event_pool_.empty()) {
          cudaEvent_t e = event_pool_.back();
          event_pool_.pop_back();
          return e;
        }
        cudaEvent_t e;
        cuda_check(cudaEventCreate(&e), "cudaEventCreate");
        return e;
      };
      e0 = take();
      e1 = take();
      // Until its events are in timed_, stats() must not read or reset the
      // spans: this launch may hold one and write it.
      ++unregistered_launches_;
    }
  }
  try {
    if (e0) cuda_check(cudaEventRecord(e0, s), "cudaEventRecord");
    if (use_bulk) {
      cuda_check(launch_bulk_copy(dir, a, num_sms_, s), "kernel launch");
    } else {
      cuda_check(launch_copy(dir, table, a, grid_for(tile_end - tile_begin), s, cfg_.cache_streaming != 0),
                 "kernel launch");
    }
    if (e1) cuda_check(cudaEventRecord(e1, s), "cudaEventRecord");
  } catch (...) {
    if (e1) {
      std::lock_guard<std::mutex> g(stats_mu_);
      --unregistered_launches_;
      event_pool_.push_back(e0);
      event_pool_.push_back(e1);
    }
    throw;
  }
  if (e1) {
    std::lock_guard<std::mutex> g(stats_mu_);
    timed_.emplace_back(e0, e1);
    --unregistered_launches_;
    // A caller that times without reading stats must not grow this list
    // without bound: spans that have finished are folded in as we go.
    if (timed_.size() >= 1024) fold_finished_timings();
  }
}

void Executor::fold_finished_timings() {
  size_t k = 0;
  for (; k < timed_.size(); ++k) {
    const auto& p = timed_[k];
    const cudaError_t q = cudaEventQuery(p.second);
    if (q == cudaErrorNotReady) {
      cudaGetLastError();
      break;
    }
    cuda_check(q, "cudaEventQuery");
    float ms = 0.f;
    cuda_check(cudaEventElapsedTime(&ms, p.first, p.second), "cudaEventElapsedTime");
    stats_.kernel_ms += ms;
    stats_.timed_launches += 1;
    event_pool_.push_back(p.first);
    event_pool_.push_back(p.second);
  }
  timed_.erase(timed_.begin(), timed_.begin() + static_cast<std::ptrdiff_t>(k));
}

void Executor::account(uint64_t kernel_bytes, uint64_t copies, uint64_t saved, uint64_t loaded, uint64_t p2p) {
  std::lock_guard<std::mutex> g(stats_mu_);
  stats_.kernel_bytes += kernel_bytes;
  stats_.copy_calls += copies;
  stats_.bytes_saved += saved;
  stats_.bytes_loaded += loaded;
  stats_.bytes_p2p += p2p;
}

uint64_t Executor::copy_runs(const Built& b, const Chunk& c, uint8_t* slot, bool d2h, cudaStream_t s) {
  // The chunk's own bytes only: from its first tile (dense_first), not from
  // the aligned slot base (dense_begin), whose leading bytes belong to the
  // previous chunk and are not in this slot. A save that copied them would
  // write stale slot bytes over the previous chunk's last bytes in the pool.
  // First run ending after the chunk start.
  auto it = std::upper_bound(b.runs.begin(), b.runs.end(), c.dense_first,
                             [](uint64_t v, const Run& r) { return v < r.dense + r.bytes; });
  uint64_t copies = 0;
  for (; it != b.runs.end() && it->dense < c.dense_end; ++it) {
    const uint64_t lo = std::max(it->dense, c.dense_first);
    const uint64_t hi = std::min(it->dense + it->bytes, c.dense_end);
    if (hi <= lo) continue;
    void* host = reinterpret_cast<void*>(it->host + (lo - it->dense));
    uint8_t* dev = slot + (lo - c.dense_begin);
    if (d2h) {
      cuda_check(cudaMemcpyAsync(host, dev, hi - lo, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync D2H");
    } else {
      cuda_check(cudaMemcpyAsync(dev, host, hi - lo, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync H2D");
    }
    copies += 1;
  }
  return copies;
}

// ---------------------------------------------------------------------------
// Save / load
// ---------------------------------------------------------------------------

void Executor::save(const pf_save_layer* layers, uint64_t n_layers, cudaStream_t caller) {
  HostTimer timer{&stats_.host_ms, &stats_mu_};
  DeviceGuard on(device_);
  check_kernel_status();
  const bool staged = cfg_.save_mode != PF_MODE_DIRECT;
  Built b;
  build_save(layers, n_layers, staged, &b);
  if (b.total_tiles == 0) return;
  if (!staged) {
    for (const Run& r : b.runs) {
      if (!pinned_contains(reinterpret_cast<void*>(r.host), r.bytes)) {
        throw invalid_argument("direct mode needs destinations in pinned memory allocated by this library");
      }
    }
  }
  // Order after the caller's work and after the save lane's previous call.
  Lane& L = save_lane_;
  std::lock_guard<std::mutex> g(L.mu);
  uint64_t kernel_bytes = b.total_bytes, copies = 0;
  cuda_check(cudaEventRecord(L.ev_start, caller), "cudaEventRecord");
  cuda_check(cudaStreamWaitEvent(L.kstream, L.ev_start, 0), "cudaStreamWaitEvent");
  for (auto e : L.ev_copy_done) cuda_check(cudaStreamWaitEvent(L.kstream, e, 0), "cudaStreamWaitEvent");
  for (auto cs : L.cstreams) {
    cuda_check(cudaStreamWaitEvent(cs, L.ev_start, 0), "cudaStreamWaitEvent");
    cuda_check(cudaStreamWaitEvent(cs, L.ev_done, 0), "cudaStreamWaitEvent");
  }
  uint8_t* staging = staged ? lane_staging(L) : nullptr;
  const CopyArgs args = upload(L, b, false);
  if (!staged) {
    launch(kPack, false, args, 0, b.total_tiles, 0, L.kstream);
  } else {
    // A save has no per-layer consumer waiting on its first chunk: starting
    // at half a slot only delays the first D2H by one larger pack (about
    // 0.1 ms for 256 MiB) and saves kernel launches.
    std::vector<Chunk> chunks;
    make_chunks(b, std::max(first_chunk_, slot_bytes_ / 2), &chunks);
    const bool bulk = use_bulk(b);
    for (size_t k = 0; k < chunks.size(); ++k) {
      const uint32_t si = static_cast<uint32_t>(k % slots_);
      uint8_t* slot = staging + static_cast<uint64_t>(si) * slot_bytes_;
      if (k >= slots_) cuda_check(cudaStreamWaitEvent(L.kstream, L.ev_drained[si], 0), "cudaStreamWaitEvent");
      const int64_t shift = static_cast<int64_t>(reinterpret_cast<uint64_t>(slot)) -
                            static_cast<int64_t>(chunks[k].dense_begin);
      launch(kPack, false, args, chunks[k].tile_begin, chunks[k].tile_end, shift, L.kstream, bulk);
      cuda_check(cudaEventRecord(L.ev_filled[si], L.kstream), "cudaEventRecord");
      cudaStream_t cs = L.cstreams[k % L.cstreams.size()];
      cuda_check(cudaStreamWaitEvent(cs, L.ev_filled[si], 0), "cudaStreamWaitEvent");
      copies += copy_runs(b, chunks[k], slot, true, cs);
      cuda_check(cudaEventRecord(L.ev_drained[si], cs), "cudaEventRecord");
    }
    kernel_bytes = 2 * b.total_bytes;  // into the slot, then out of it
  }
  cuda_check(cudaEventRecord(L.ev_done, L.kstream), "cudaEventRecord");
  cuda_check(cudaStreamWaitEvent(caller, L.ev_done, 0), "cudaStreamWaitEvent");
  for (size_t j = 0; j < L.cstreams.size(); ++j) {
    cuda_check(cudaEventRecord(L.ev_copy_done[j], L.cstreams[j]), "cudaEventRecord");
    cuda_check(cudaStreamWaitEvent(caller, L.ev_copy_done[j], 0), "cudaStreamWaitEvent");
  }
  account(kernel_bytes, copies, b.total_bytes, 0, 0);
}

void Executor::load(const pf_load_layer* layers, uint64_t n_layers, cudaStream_t caller, int64_t* layer_done) {
  HostTimer timer{&stats_.host_ms, &stats_mu_};
  DeviceGuard on(device_);
  check_kernel_status();
  const bool staged = cfg_.load_mode != PF_MODE_DIRECT;
  Built b;
  build_load(layers, n_layers, staged, &b);
  if (layer_done) {
    if (!pinned_contains(layer_done, n_layers * sizeof(int64_t))) {
      throw invalid_argument("layer_done must be pinned memory allocated by this library");
    }
    // Layers without blocks are complete at once.
    std::vector<bool> has(n_layers, false);
    for (const PlanLayer& p : b.layers) has[p.done_index] = true;
    for (const SerialLoad& sl : b.serial) has[sl.done_index] = true;
    for (uint64_t l = 0; l < n_layers; ++l) {
      if (!has[l]) reinterpret_cast<volatile int64_t*>(layer_done)[l] = 1;
    }
  }
  if (b.total_tiles == 0 && b.serial.empty()) return;
  if (!staged) {
    for (const Run& r : b.runs) {
      if (!pinned_contains(reinterpret_cast<void*>(r.host), r.bytes)) {
        throw invalid_argument("direct mode needs sources in pinned memory allocated by this library");
      }
    }
  }
  Lane& L = load_lane_;
  std::lock_guard<std::mutex> g(L.mu);
  uint64_t kernel_bytes = 0, copies = 0;
  cuda_check(cudaEventRecord(L.ev_start, caller), "cudaEventRecord");
  cuda_check(cudaStreamWaitEvent(L.kstream, L.ev_start, 0), "cudaStreamWaitEvent");
  for (auto e : L.ev_copy_done) cuda_check(cudaStreamWaitEvent(L.kstream, e, 0), "cudaStreamWaitEvent");
  for (auto cs : L.cstreams) {
    cuda_check(cudaStreamWaitEvent(cs, L.ev_start, 0), "cudaStreamWaitEvent");
    cuda_check(cudaStreamWaitEvent(cs, L.ev_done, 0), "cudaStreamWaitEvent");
  }
  uint8_t* staging = (staged && b.total_tiles > 0) ? lane_staging(L) : nullptr;
  CopyArgs args{};
  if (b.total_tiles > 0) {
    args = upload(L, b, layer_done != nullptr);
    if (layer_done) {
      // The kernel writes through the device view of the pinned words.
      void* dev = nullptr;
      cuda_check(cudaHostGetDevicePointer(&dev, layer_done, 0), "cudaHostGetDevicePointer(layer_done)");
      args.layer_done = static_cast<int64_t*>(dev);
    }
  }
  if (b.total_tiles == 0) {
    // only ordered copies below
  } else if (!staged) {
    launch(kUnpack, true, args, 0, b.total_tiles, 0, L.kstream);
    kernel_bytes = b.total_bytes;
  } else {
    // Small first chunk: the first layers of a layer-wise restore are ready
    // after one small DMA. When the caller waits on per-layer flags, the
    // first chunk holds layer 0 and the small layers listed right after it
    // (per-block scales beside their KV), at least 4 MiB, so layer 0's flags
    // rise after the DMA of those bytes alone; the chunks then double as usual.
    // Without per-layer flags nobody reads the first layers early, so the
    // load uses whole slots from the start: fewer launches (each pays a fixed
    // cost of tens of microseconds while DMA streams), and the remainder,
    // the smallest chunk, comes last, where its unpack is the only work
    // left after the final DMA.
    const uint64_t first = layer_done ? layerwise_first_limit(b.layers, first_chunk_, kLayerwiseMinFirstChunk)
                                      : slot_bytes_;
    std::vector<Chunk> chunks;
    make_chunks(b, first, &chunks);
    const bool bulk = layer_done == nullptr && use_bulk(b);
    for (size_t k = 0; k < chunks.size(); ++k) {
      const uint32_t si = static_cast<uint32_t>(k % slots_);
      uint8_t* slot = staging + static_cast<uint64_t>(si) * slot_bytes_;
      cudaStream_t cs = L.cstreams[k % L.cstreams.size()];
      if (k >= slots_) cuda_check(cudaStreamWaitEvent(cs, L.ev_drained[si], 0), "cudaStreamWaitEvent");
      copies += copy_runs(b, chunks[k], slot, false, cs);
      cuda_check(cudaEventRecord(L.ev_filled[si], cs), "cudaEventRecord");
      cuda_check(cudaStreamWaitEvent(L.kstream, L.ev_filled[si], 0), "cudaStreamWaitEvent");
      const int64_t shift = static_cast<int64_t>(reinterpret_cast<uint64_t>(slot)) -
                            static_cast<int64_t>(chunks[k].dense_begin);
      launch(kUnpack, false, args, chunks[k].tile_begin, chunks[k].tile_end, shift, L.kstream, bulk);
      cuda_check(cudaEventRecord(L.ev_drained[si], L.kstream), "cudaEventRecord");
    }
    kernel_bytes = 2 * b.total_bytes;  // into the slot, then out of it
  }
  copies += issue_serial(b, L.kstream, layer_done);
  cuda_check(cudaEventRecord(L.ev_done, L.kstream), "cudaEventRecord");
  cuda_check(cudaStreamWaitEvent(caller, L.ev_done, 0), "cudaStreamWaitEvent");
  for (size_t j = 0; j < L.cstreams.size(); ++j) {
    cuda_check(cudaEventRecord(L.ev_copy_done[j], L.cstreams[j]), "cudaEventRecord");
  }
  uint64_t loaded = b.total_bytes;
  for (const SerialLoad& sl : b.serial) {
    loaded += sl.ids.size() * load_geometry(sl.layer).unit_bytes * load_geometry(sl.layer).units;
  }
  account(kernel_bytes, copies, 0, loaded, 0);
}

void Executor::save_sync(const pf_save_layer* layers, uint64_t n_layers) {
  DeviceGuard on(device_);
  save(layers, n_layers, save_stream_);
  cuda_check(cudaStreamSynchronize(save_stream_), "cudaStreamSynchronize(save)");
  check_kernel_status();
}

void Executor::load_sync(const pf_load_layer* layers, uint64_t n_layers, int64_t* layer_done) {
  DeviceGuard on(device_);
  load(layers, n_layers, own_stream_, layer_done);
  cuda_check(cudaStreamSynchronize(own_stream_), "cudaStreamSynchronize(load)");
  check_kernel_status();
}

void Executor::stats(pf_executor_stats* out) {
  DeviceGuard on(device_);
  // Wait for the spans issued so far without holding the mutex, so that
  // calls on either lane keep launching meanwhile.
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending;
  {
    std::lock_guard<std::mutex> g(stats_mu_);
    pending.swap(timed_);
  }
  double ms_sum = 0.0;
  for (const auto& p : pending) {
    cuda_check(cudaEventSynchronize(p.second), "cudaEventSynchronize");
    float ms = 0.f;
    cuda_check(cudaEventElapsedTime(&ms, p.first, p.second), "cudaEventElapsedTime");
    ms_sum += ms;
  }
  std::lock_guard<std::mutex> g(stats_mu_);
  stats_.kernel_ms += ms_sum;
  stats_.timed_launches += pending.size();
  for (const auto& p : pending) {
    event_pool_.push_back(p.first);
    event_pool_.push_back(p.second);
  }
  if (spans_used_ > 0 && timed_.empty() && unregistered_launches_ == 0) {
    // Every span handed out so far belongs to a launch whose end event was
    // waited on above: spans are given out with a launch's events, and no
    // timed launch was added or is being added since (else the spans wait
    // for a later call).
    std::vector<unsigned long long> sp(2 * spans_used_);
    cuda_check(cudaMemcpy(sp.data(), spans_, sp.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost),
               "cudaMemcpy(spans)");
    for (uint64_t i = 0; i < spans_used_; ++i) {
      if (sp[2 * i + 1] > sp[2 * i]) {
        stats_.kernel_body_ms += static_cast<double>(sp[2 * i + 1] - sp[2 * i]) * 1e-6;
        stats_.body_launches += 1;
      }
    }
    reset_spans();
  }
  *out = stats_;
}

void Executor::reset_stats() {
  pf_executor_stats tmp;
  stats(&tmp);
  std::lock_guard<std::mutex> g(stats_mu_);
  stats_ = pf_executor_stats{};
}

void Executor::debug_stall_tile(uint64_t tile) {
  std::lock_guard<std::mutex> g(stats_mu_);
  stall_tile_ = tile;
}

void Executor::set_timing(bool on) {
  DeviceGuard dev(device_);
  std::lock_guard<std::mutex> g(stats_mu_);
  if (on && !spans_) {
    cuda_check(cudaMalloc(reinterpret_cast<void**>(&spans_), 2 * kSpanCap * sizeof(unsigned long long)),
               "cudaMalloc(spans)");
    reset_spans();
  }
  timing_ = on;
}

}  // namespace pf
