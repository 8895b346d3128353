// extern "C" entry points declared in include/pegaflow.h.
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "common.h"
#include "wire.h"
#include "engine.h"
#include "executor.h"
#include "offset_allocator.h"
#include "pegaflow.h"
#include "pinned.h"

namespace pf {
void refcopy_save(int device, const pf_save_layer* layers, uint64_t n);
uint64_t refcopy_load(int device, const pf_load_layer* layers, uint64_t n);

namespace {
thread_local std::string g_last_error;
}
void set_last_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }
}  // namespace pf

struct pf_executor {
  std::unique_ptr<pf::Executor> impl;
  pf::Executor* ref = nullptr;  // borrowed (engine-owned) executor
  pf::Executor& get() { return impl ? *impl : *ref; }
};

struct pf_engine {
  std::unique_ptr<pf::Engine> impl;
  std::mutex exec_mu;
  std::map<int, std::unique_ptr<pf_executor>> exec_handles;
};

struct pf_allocator {
  std::unique_ptr<pf::ScaledOffsetAllocator> impl;
  std::map<uint32_t, pf::ScaledOffsetAllocator::Allocation> live;
};

using pf::guarded;

namespace {
int null_arg(const char* what) {
  pf::set_last_error(std::string("invalid argument: null ") + what);
  return PF_ERR_INVALID_ARGUMENT;
}
std::string str(const char* s) { return s ? std::string(s) : std::string(); }
std::string bytes_str(const pf_bytes& b) {
  return b.len ? std::string(reinterpret_cast<const char*>(b.data), b.len) : std::string();
}
}  // namespace

extern "C" {

const char* pf_last_error(void) { return pf::last_error(); }
int pf_abi_version(void) { return PF_ABI_VERSION; }

int pf_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int pf_layer_validate(const pf_layer_desc* layer, const char* layer_name) {
  if (!layer) return null_arg("layer");
  return guarded([&] { pf::validate_layout(*layer, layer_name ? layer_name : ""); });
}

int pf_segment_offset(const pf_layer_desc* layer, uint64_t block_idx, uint64_t segment_idx, uint64_t* out_offset) {
  if (!layer || !out_offset) return null_arg("argument");
  return guarded([&] { *out_offset = pf::segment_offset(*layer, block_idx, segment_idx); });
}

// ----------------------------------------------------------------- executor

void pf_executor_config_default(pf_executor_config* cfg) {
  if (!cfg) return;
  std::memset(cfg, 0, sizeof(*cfg));
  cfg->staging_chunk_bytes = pf::kDefaultSlotBytes;
  cfg->staging_slots = pf::kDefaultSlots;
  cfg->save_mode = PF_MODE_AUTO;
  cfg->load_mode = PF_MODE_AUTO;
  cfg->ctas_per_sm = 4;
  cfg->copy_streams = 2;
  cfg->first_chunk_bytes = pf::kDefaultFirstChunkBytes;
}

int pf_executor_create(int32_t device_id, const pf_executor_config* cfg, pf_executor** out) {
  if (!out) return null_arg("out");
  return guarded([&] {
    pf_executor_config c;
    pf_executor_config_default(&c);
    if (cfg) c = *cfg;
    auto h = std::make_unique<pf_executor>();
    h->impl = std::make_unique<pf::Executor>(device_id, c);
    *out = h.release();
  });
}

void pf_executor_destroy(pf_executor* exec) {
  if (exec && exec->impl) delete exec;
}

int pf_save_blocks(pf_executor* exec, const pf_save_layer* layers, uint64_t n_layers) {
  if (!exec || (!layers && n_layers)) return null_arg("executor or layers");
  return guarded([&] { exec->get().save_sync(layers, n_layers); });
}

int pf_load_blocks(pf_executor* exec, const pf_load_layer* layers, uint64_t n_layers) {
  if (!exec || (!layers && n_layers)) return null_arg("executor or layers");
  return guarded([&] { exec->get().load_sync(layers, n_layers); });
}

int pf_save_blocks_async(pf_executor* exec, const pf_save_layer* layers, uint64_t n_layers, void* stream) {
  if (!exec || (!layers && n_layers)) return null_arg("executor or layers");
  return guarded([&] { exec->get().save(layers, n_layers, static_cast<cudaStream_t>(stream)); });
}

int pf_load_blocks_async(pf_executor* exec, const pf_load_layer* layers, uint64_t n_layers, void* stream,
                         int64_t* layer_done) {
  if (!exec || (!layers && n_layers)) return null_arg("executor or layers");
  return guarded([&] { exec->get().load(layers, n_layers, static_cast<cudaStream_t>(stream), layer_done); });
}

int pf_p2p_transfer(pf_executor* exec, int32_t peer_device, int push, const pf_p2p_layer* layers,
                    uint64_t n_layers, void* stream) {
  if (!exec || (!layers && n_layers)) return null_arg("executor or layers");
  return guarded([&] {
    if (stream) {
      exec->get().p2p(layers, n_layers, peer_device, push != 0, static_cast<cudaStream_t>(stream));
    } else {
      exec->get().p2p_sync(layers, n_layers, peer_device, push != 0);
    }
  });
}

int pf_executor_stats_get(pf_executor* exec, pf_executor_stats* out) {
  if (!exec || !out) return null_arg("argument");
  return guarded([&] { exec->get().stats(out); });
}

int pf_executor_stats_reset(pf_executor* exec) {
  if (!exec) return null_arg("executor");
  return guarded([&] { exec->get().reset_stats(); });
}

int pf_executor_set_timing(pf_executor* exec, int enabled) {
  if (!exec) return null_arg("executor");
  return guarded([&] { exec->get().set_timing(enabled != 0); });
}

int pf_executor_debug_stall_tile(pf_executor* exec, uint64_t tile) {
  if (!exec) return null_arg("executor");
  return guarded([&] { exec->get().debug_stall_tile(tile); });
}

int pf_refcopy_save(int32_t device_id, const pf_save_layer* layers, uint64_t n_layers) {
  if (!layers && n_layers) return null_arg("layers");
  return guarded([&] { pf::refcopy_save(device_id, layers, n_layers); });
}

int pf_refcopy_load(int32_t device_id, const pf_load_layer* layers, uint64_t n_layers, uint64_t* out_runs) {
  if (!layers && n_layers) return null_arg("layers");
  return guarded([&] {
    const uint64_t r = pf::refcopy_load(device_id, layers, n_layers);
    if (out_runs) *out_runs = r;
  });
}

// ------------------------------------------------------------------ pinned

int pf_pinned_alloc(uint64_t size, int write_combined, void** out) {
  if (!out) return null_arg("out");
  return guarded([&] {
    unsigned flags = cudaHostAllocPortable | cudaHostAllocMapped;
    if (write_combined) flags |= cudaHostAllocWriteCombined;
    if (size == 0) throw pf::invalid_argument("size must be greater than zero");
    void* p = nullptr;
    cudaError_t err = cudaHostAlloc(&p, size, flags);
    if (err != cudaSuccess) {
      cudaGetLastError();
      throw pf::cuda_init(std::string("cudaHostAlloc failed: ") + cudaGetErrorString(err));
    }
    pf::pinned_register(p, size);
    *out = p;
  });
}

int pf_pinned_free(void* ptr) {
  return guarded([&] {
    if (!ptr) return;
    pf::pinned_unregister(ptr);
    pf::cuda_check(cudaFreeHost(ptr), "cudaFreeHost");
  });
}

// --------------------------------------------------------------- allocator

int pf_allocator_create(uint64_t total_bytes, uint64_t unit_size, uint32_t max_allocs, pf_allocator** out) {
  if (!out) return null_arg("out");
  return guarded([&] {
    auto a = std::make_unique<pf_allocator>();
    a->impl = std::make_unique<pf::ScaledOffsetAllocator>(
        pf::ScaledOffsetAllocator::make(total_bytes, unit_size, unit_size == PF_ALLOCATOR_AUTO_UNIT,
                                           max_allocs));
    *out = a.release();
  });
}

void pf_allocator_destroy(pf_allocator* a) { delete a; }

int pf_allocator_alloc(pf_allocator* a, uint64_t size, uint64_t* out_offset, uint64_t* out_size,
                       uint32_t* out_handle) {
  if (!a) return null_arg("allocator");
  if (size == 0) {
    pf::set_last_error("invalid argument: size must be greater than zero");
    return PF_ERR_INVALID_ARGUMENT;
  }
  int rc = PF_OK;
  const int g = guarded([&] {
    pf::ScaledOffsetAllocator::Allocation al{};
    if (!a->impl->allocate(size, &al)) {
      pf::set_last_error("allocator has no space");
      rc = PF_ERR_NO_SPACE;
      return;
    }
    a->live[al.raw.metadata] = al;
    if (out_offset) *out_offset = al.offset_bytes;
    if (out_size) *out_size = al.size_bytes;
    if (out_handle) *out_handle = al.raw.metadata;
  });
  return g != PF_OK ? g : rc;
}

void pf_allocator_free(pf_allocator* a, uint32_t handle) {
  if (!a) return;
  auto it = a->live.find(handle);
  if (it == a->live.end()) return;
  a->impl->free(it->second);
  a->live.erase(it);
}

void pf_allocator_report(pf_allocator* a, uint64_t* total_free_bytes, uint64_t* largest_free_bytes,
                         uint64_t* total_bytes, uint64_t* unit_size) {
  if (!a) return;
  if (total_free_bytes) *total_free_bytes = a->impl->total_free_bytes();
  if (largest_free_bytes) *largest_free_bytes = a->impl->largest_free_bytes();
  if (total_bytes) *total_bytes = a->impl->total_bytes();
  if (unit_size) *unit_size = a->impl->unit_size();
}

// -------------------------------------------------------------- load state

int pf_load_state_create(pf_load_state** out) {
  if (!out) return null_arg("out");
  return guarded([&] { *out = pf::load_state_create(0); });
}

int pf_load_state_create_layers(uint32_t n_layers, pf_load_state** out) {
  if (!out) return null_arg("out");
  return guarded([&] { *out = pf::load_state_create(n_layers); });
}

int pf_load_state_attach(const char* shm_name, pf_load_state** out) {
  if (!out || !shm_name) return null_arg("argument");
  return guarded([&] { *out = pf::load_state_attach(shm_name); });
}

int64_t pf_load_state_get(const pf_load_state* s) { return s ? pf::load_state_get(s) : PF_LOAD_STATE_ERROR; }
void pf_load_state_set_completed(pf_load_state* s) {
  if (s) pf::load_state_set(s, PF_LOAD_STATE_SUCCESS);
}
void pf_load_state_set_error(pf_load_state* s) {
  if (s) pf::load_state_set(s, PF_LOAD_STATE_ERROR);
}
void pf_load_state_close(pf_load_state* s) { pf::load_state_close(s); }

// ------------------------------------------------------------------ engine

void pf_engine_config_default(pf_engine_config* cfg) {
  if (!cfg) return;
  std::memset(cfg, 0, sizeof(*cfg));
  cfg->pool_bytes = 30ull << 30;
  cfg->write_combined = 1;
  cfg->enable_lfu_admission = 1;
  cfg->pool_kind = PF_POOL_PINNED;
  cfg->pre_evict_threshold_bytes = 5ull << 30;
  cfg->pre_evict_target_bytes = 8ull << 30;
  cfg->pre_evict_interval_ms = 100;
  pf_executor_config_default(&cfg->executor);
}

int pf_engine_create(const pf_engine_config* cfg, pf_engine** out) {
  if (!out) return null_arg("out");
  return guarded([&] {
    pf_engine_config c;
    pf_engine_config_default(&c);
    if (cfg) c = *cfg;
    auto e = std::make_unique<pf_engine>();
    e->impl = std::make_unique<pf::Engine>(c);
    *out = e.release();
  });
}

void pf_engine_destroy(pf_engine* e) {
  if (!e) return;
  {
    std::lock_guard<std::mutex> g(e->exec_mu);
    e->exec_handles.clear();
  }
  e->impl.reset();
  delete e;
}

int pf_engine_register_context_layer(pf_engine* e, const char* instance_id, const char* ns, int32_t device_id,
                                     const char* layer_name, uint64_t data_ptr, uint64_t size_bytes,
                                     uint64_t num_blocks, uint64_t bytes_per_block, uint64_t kv_stride_bytes,
                                     uint64_t segments, uint64_t tp_rank, uint64_t tp_size, uint64_t num_layers) {
  if (!e) return null_arg("engine");
  return guarded([&] {
    pf_layer_desc reg{data_ptr, size_bytes, num_blocks, bytes_per_block, kv_stride_bytes, segments};
    e->impl->register_context_layer(str(instance_id), str(ns), device_id, str(layer_name), reg, tp_rank, tp_size,
                                    num_layers);
  });
}

int pf_engine_unregister_instance(pf_engine* e, const char* instance_id) {
  if (!e) return null_arg("engine");
  return guarded([&] { e->impl->unregister_instance(str(instance_id)); });
}

int pf_engine_batch_save_kv_blocks(pf_engine* e, const char* instance_id, uint64_t tp_rank, int32_t device_id,
                                   const pf_save_entry* saves, uint64_t n_saves) {
  if (!e || (!saves && n_saves)) return null_arg("engine or saves");
  return guarded([&] {
    std::vector<pf::Engine::SaveEntry> entries(n_saves);
    for (uint64_t i = 0; i < n_saves; ++i) {
      const pf_save_entry& s = saves[i];
      entries[i].layer_name = str(s.layer_name);
      if ((s.n_ids && !s.block_ids) || (s.n_hashes && !s.block_hashes)) {
        throw pf::invalid_argument("null block_ids or block_hashes");
      }
      entries[i].block_ids.assign(s.block_ids, s.block_ids + s.n_ids);
      if (i > 0 && s.block_hashes == saves[i - 1].block_hashes && s.n_hashes == saves[i - 1].n_hashes) {
        entries[i].hashes = entries[i - 1].hashes;  // the caller passed one array for both entries
        continue;
      }
      auto hashes = std::make_shared<std::vector<std::string>>();
      hashes->reserve(s.n_hashes);
      for (uint64_t k = 0; k < s.n_hashes; ++k) hashes->push_back(bytes_str(s.block_hashes[k]));
      entries[i].hashes = std::move(hashes);
    }
    e->impl->batch_save(str(instance_id), tp_rank, device_id, entries);
  });
}

int pf_engine_save_kv_blocks(pf_engine* e, const char* instance_id, uint64_t tp_rank, int32_t device_id,
                             const char* layer_name, const int32_t* block_ids, const pf_bytes* block_hashes,
                             uint64_t n) {
  pf_save_entry entry{layer_name, block_ids, n, block_hashes, n};
  return pf_engine_batch_save_kv_blocks(e, instance_id, tp_rank, device_id, &entry, 1);
}

int pf_engine_count_prefix_hit_blocks(pf_engine* e, const char* instance_id, const pf_bytes* block_hashes,
                                      uint64_t n, uint64_t* out_hits) {
  if (!e || !out_hits || (!block_hashes && n)) return null_arg("argument");
  return guarded([&] {
    std::vector<std::string> hashes;
    hashes.reserve(n);
    for (uint64_t k = 0; k < n; ++k) hashes.push_back(bytes_str(block_hashes[k]));
    *out_hits = e->impl->count_prefix_hit_blocks(str(instance_id), hashes);
  });
}

int pf_engine_query_prefetch(pf_engine* e, const char* instance_id, const pf_bytes* block_hashes, uint64_t n,
                             pf_prefetch_status* out) {
  if (!e || !out || (!block_hashes && n)) return null_arg("argument");
  return guarded([&] {
    std::vector<std::string> hashes;
    hashes.reserve(n);
    for (uint64_t k = 0; k < n; ++k) hashes.push_back(bytes_str(block_hashes[k]));
    const pf::PrefetchStatus s = e->impl->query_prefetch(str(instance_id), hashes);
    *out = pf_prefetch_status{};
    out->state = static_cast<uint32_t>(s.state);
    out->hit_blocks = s.hit_blocks;
    out->loading_blocks = s.loading_blocks;
    out->missing_blocks = s.missing_blocks;
  });
}

namespace {
pf::DfsTier* dfs_or_throw(pf_engine* e) {
  pf::DfsTier* t = e->impl->dfs();
  if (!t) throw pf::invalid_argument("the packed-file tier is off (no dfs_root)");
  return t;
}
}  // namespace

int pf_engine_dfs_stats(pf_engine* e, pf_dfs_stats* out) {
  if (!e || !out) return null_arg("argument");
  return guarded([&] {
    const pf::DfsStats s = dfs_or_throw(e)->stats();
    *out = pf_dfs_stats{s.files,          s.blocks,           s.usage_bytes,       s.written_files, s.written_blocks,
                        s.write_failures, s.prefetched_blocks, s.prefetch_failures, s.evicted_files};
  });
}

int pf_engine_dfs_flush(pf_engine* e, double timeout_s, int* out_idle) {
  if (!e || !out_idle) return null_arg("argument");
  return guarded([&] { *out_idle = dfs_or_throw(e)->flush(timeout_s) ? 1 : 0; });
}

int pf_engine_dfs_check_quota(pf_engine* e) {
  if (!e) return null_arg("engine");
  return guarded([&] { dfs_or_throw(e)->check_quota(); });
}

int pf_engine_batch_load_kv_blocks(pf_engine* e, const char* instance_id, uint64_t tp_rank, int32_t device_id,
                                   const char* load_state_shm, const char* const* layer_names, uint64_t n_layers,
                                   const int32_t* block_ids, const pf_bytes* block_hashes, uint64_t n_blocks) {
  if (!e || (!layer_names && n_layers) || (n_blocks && (!block_ids || !block_hashes))) {
    return null_arg("argument");
  }
  return guarded([&] {
    std::vector<std::string> names;
    for (uint64_t i = 0; i < n_layers; ++i) names.push_back(str(layer_names[i]));
    std::vector<int32_t> ids(block_ids, block_ids + n_blocks);
    std::vector<std::string> hashes;
    hashes.reserve(n_blocks);
    for (uint64_t k = 0; k < n_blocks; ++k) hashes.push_back(bytes_str(block_hashes[k]));
    e->impl->batch_load(str(instance_id), tp_rank, device_id, str(load_state_shm), names, ids, hashes);
  });
}

int pf_engine_save_request(pf_engine* e, const uint8_t* request, uint64_t len) {
  if (!e || (!request && len)) return null_arg("engine or request");
  return guarded([&] {
    pf::SaveRequestWire req;
    pf::decode_save_request(request, len, &req);
    e->impl->batch_save(req.instance_id, req.tp_rank, req.device_id, req.saves);
  });
}

int pf_engine_load_request(pf_engine* e, const uint8_t* request, uint64_t len) {
  if (!e || (!request && len)) return null_arg("engine or request");
  return guarded([&] {
    pf::LoadRequestWire req;
    pf::decode_load_request(request, len, &req);
    e->impl->batch_load(req.instance_id, req.tp_rank, req.device_id, req.load_state_shm, req.layer_names,
                        req.block_ids, req.block_hashes);
  });
}

int pf_request_instance_id(const uint8_t* request, uint64_t len, char* out, uint64_t cap, uint64_t* out_len) {
  if ((!request && len) || !out || !out_len) return null_arg("argument");
  return guarded([&] {
    const std::string id = pf::decode_request_instance_id(request, len);
    *out_len = id.size();
    if (id.size() + 1 > cap) throw pf::invalid_argument("instance_id longer than the output buffer");
    std::memcpy(out, id.data(), id.size());
    out[id.size()] = '\0';
  });
}

int pf_engine_wait_loads(pf_engine* e, int32_t device_id, double timeout_s) {
  if (!e) return null_arg("engine");
  if (!e->impl->wait_loads(device_id, timeout_s)) {
    pf::set_last_error("timed out waiting for loads on device " + std::to_string(device_id));
    return PF_ERR_TIMEOUT;
  }
  return PF_OK;
}

int pf_engine_pool_usage(pf_engine* e, uint64_t* used, uint64_t* total, uint64_t* largest_free) {
  if (!e) return null_arg("engine");
  return guarded([&] {
    uint64_t u = 0, t = 0;
    e->impl->storage().usage(&u, &t);  // all pools together
    if (used) *used = u;
    if (total) *total = t;
    if (largest_free) *largest_free = e->impl->storage().largest_free();
  });
}

int pf_engine_slot_info(pf_engine* e, const char* ns, const uint8_t* hash, uint64_t hash_len, uint64_t slot,
                        uint64_t* k_ptr, uint64_t* v_ptr, uint64_t* size) {
  if (!e) return null_arg("engine");
  return guarded([&] {
    const std::string h = hash_len ? std::string(reinterpret_cast<const char*>(hash), hash_len) : std::string();
    auto sb = e->impl->storage().cache_peek(str(ns), h);
    if (!sb) throw pf::storage_error("block not sealed in cache");
    if (slot >= sb->slots.size()) throw pf::storage_error("slot out of range");
    const auto& lb = sb->slots[slot];
    if (k_ptr) *k_ptr = reinterpret_cast<uint64_t>(lb->k_ptr);
    if (v_ptr) *v_ptr = reinterpret_cast<uint64_t>(lb->v_ptr);
    if (size) *size = lb->size;
  });
}

int pf_engine_metrics_get(pf_engine* e, pf_engine_metrics* out) {
  if (!e || !out) return null_arg("argument");
  return guarded([&] { e->impl->metrics(out); });
}

int pf_engine_executor(pf_engine* e, int32_t device_id, pf_executor** out) {
  if (!e || !out) return null_arg("argument");
  return guarded([&] {
    auto w = e->impl->device_worker(device_id);
    if (!w) throw pf::cuda_init("engine pool is plain host memory; no executor");
    std::lock_guard<std::mutex> g(e->exec_mu);
    auto& h = e->exec_handles[device_id];
    if (!h) {
      h = std::make_unique<pf_executor>();
      h->ref = &w->executor();
    }
    *out = h.get();
  });
}

}  // extern "C"
