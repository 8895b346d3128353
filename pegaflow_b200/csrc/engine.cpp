#include "engine.h"

#include <chrono>
#include <cstdio>
#include <unordered_set>
#include <utility>

#include "common.h"
#include "pinned.h"

namespace pf {

namespace {
using Clock = std::chrono::steady_clock;
double ms_since(Clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
}

// LoadState errors reach the engine caller as EngineError::Storage("LoadState: ...")
// (From<LoadStateError> for EngineError, lib.rs:87-91).
pf_load_state* attach_or_storage_error(const std::string& shm) {
  try {
    return load_state_attach(shm);
  } catch (const Error& e) {
    throw storage_error(std::string("LoadState: ") + e.what());
  }
}
}  // namespace

// ---------------------------------------------------------------------------
// DeviceWorker
// ---------------------------------------------------------------------------

DeviceWorker::DeviceWorker(int device, const pf_executor_config& cfg, EngineCounters* counters)
    : exec_(std::make_unique<Executor>(device, cfg)), counters_(counters) {
  thread_ = std::thread([this] { load_loop(); });
}

DeviceWorker::~DeviceWorker() {
  {
    std::lock_guard<std::mutex> g(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  if (thread_.joinable()) thread_.join();
  std::unique_ptr<DeviceGuard> on;
  try {
    on = std::make_unique<DeviceGuard>(exec_->device());
  } catch (const Error&) {
    // Destroy the streams in whatever context is current; nothing here may throw.
  }
  for (cudaStream_t s : all_save_streams_) cudaStreamDestroy(s);
}

cudaStream_t DeviceWorker::acquire_save_stream() {
  std::lock_guard<std::mutex> g(streams_mu_);
  if (!free_save_streams_.empty()) {
    cudaStream_t s = free_save_streams_.back();
    free_save_streams_.pop_back();
    return s;
  }
  DeviceGuard on(exec_->device());
  cudaStream_t s = nullptr;
  cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate(save)");
  all_save_streams_.push_back(s);
  return s;
}

void DeviceWorker::release_save_stream(cudaStream_t s) {
  std::lock_guard<std::mutex> g(streams_mu_);
  free_save_streams_.push_back(s);
}

void DeviceWorker::submit_load(LoadTask task) {
  {
    std::lock_guard<std::mutex> g(mu_);
    queue_.push_back(std::move(task));
  }
  cv_.notify_one();
}

bool DeviceWorker::wait_idle(double timeout_s) {
  std::unique_lock<std::mutex> lk(mu_);
  return idle_cv_.wait_for(lk, std::chrono::duration<double>(timeout_s),
                           [this] { return queue_.empty() && !busy_; });
}

void DeviceWorker::load_loop() {
  // load_worker_loop (gpu_worker.rs:141-181). This thread belongs to the
  // worker, so its device stays current for the thread's life (LoadState
  // polling and flag buffers run in that context).
  if (cudaSetDevice(exec_->device()) != cudaSuccess) cudaGetLastError();
  for (;;) {
    LoadTask task;
    {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [this] { return stop_ || !queue_.empty(); });
      if (queue_.empty()) return;  // stop requested and nothing left
      task = std::move(queue_.front());
      queue_.pop_front();
      busy_ = true;
    }
    process(task);
    {
      std::lock_guard<std::mutex> g(mu_);
      busy_ = false;
    }
    idle_cv_.notify_all();
  }
}

void DeviceWorker::process(LoadTask& task) {
  // process_load_task (gpu_worker.rs:205-317) followed by the LoadState signal.
  const auto t0 = Clock::now();
  bool ok = true;
  uint64_t bytes = 0;
  Clock::time_point t_setup = t0, t_first = t0, t_done = t0;
  // A LoadState with a per-layer extension covering every requested layer
  // gets its words raised as layers land (load_with_layer_words).
  pf_load_state* ls = nullptr;
  try {
    ls = load_state_attach(task.shm);
  } catch (const std::exception& e) {
    fprintf(stderr, "pegaflow_b200: failed to attach LoadState %s: %s\n", task.shm.c_str(), e.what());
  }
  int64_t* words = nullptr;
  if (ls && load_state_layers(ls) >= task.layers.size() && !task.layers.empty()) {
    words = load_state_layer_words(ls);
  }
  try {
    std::vector<pf_load_layer> layers;
    std::vector<std::vector<const void*>> ks(task.layers.size()), vs(task.layers.size());
    layers.reserve(task.layers.size());
    for (size_t l = 0; l < task.layers.size(); ++l) {
      LoadLayer& L = task.layers[l];
      ks[l].resize(L.blocks.size());
      vs[l].resize(L.blocks.size());
      for (size_t i = 0; i < L.blocks.size(); ++i) {
        ks[l][i] = L.blocks[i]->k_ptr;
        vs[l][i] = L.blocks[i]->v_ptr;
      }
      pf_load_layer pl{};
      pl.layer = L.reg;
      pl.block_idx = L.ids.data();
      pl.n = L.ids.size();
      pl.k_src = ks[l].data();
      pl.v_src = vs[l].data();
      layers.push_back(pl);
      bytes += load_geometry(L.reg).unit_bytes * load_geometry(L.reg).units * L.ids.size();
    }
    t_setup = Clock::now();
    if (words) {
      t_first = load_with_layer_words(layers.data(), layers.size(), words);
    } else {
      exec_->load_sync(layers.data(), layers.size(), nullptr);
      t_first = Clock::now();
    }
    t_done = Clock::now();
  } catch (const std::exception& e) {
    ok = false;
    fprintf(stderr, "pegaflow_b200: load task failed: %s\n", e.what());
  }
  if (!ls) {
    counters_->load_failures.fetch_add(1);
  } else {
    if (ok) {
      load_state_set(ls, PF_LOAD_STATE_SUCCESS);
    } else {
      counters_->load_failures.fetch_add(1);
      load_state_set(ls, PF_LOAD_STATE_ERROR);
    }
    load_state_close(ls);
  }
  if (ok && bytes > 0) {
    counters_->load_bytes.fetch_add(bytes);
    counters_->load_calls.fetch_add(1);
    auto ms = [](Clock::time_point a, Clock::time_point b) {
      return std::chrono::duration<double, std::milli>(b - a).count();
    };
    std::lock_guard<std::mutex> g(counters_->ms_mu);
    counters_->load_ms += ms_since(t0);
    counters_->load_queue_ms += ms(task.queued, t0);
    counters_->load_setup_ms += ms(t0, t_setup);
    counters_->load_transfer_ms += ms(t_setup, t_done);
    counters_->load_first_layer_ms += ms(task.queued, t_first);
  }
}

Clock::time_point DeviceWorker::load_with_layer_words(const pf_load_layer* layers, size_t n, int64_t* words) {
  // Registering the LoadState page with CUDA for every task would cost a
  // driver round trip on each side of every load (and unregistering can stall
  // other work), so the kernels raise flags in one mapped pinned array this
  // worker keeps, and this thread copies each newly raised flag into the
  // LoadState while the load runs.
  const size_t need = n * sizeof(int64_t);
  if (!flags_mem_ || flags_mem_->size() < need) {
    flags_mem_.reset();
    flags_mem_ = std::make_unique<PinnedMemory>(std::max<size_t>(need, 4096 * sizeof(int64_t)),
                                                PinKind::kCudaHostAlloc, /*write_combined=*/false);
  }
  volatile int64_t* flags = reinterpret_cast<volatile int64_t*>(flags_mem_->data());
  for (size_t l = 0; l < n; ++l) flags[l] = 0;
  cudaStream_t s = exec_->own_stream();
  exec_->load(layers, n, s, const_cast<int64_t*>(flags));
  std::vector<char> copied(n, 0);
  size_t left = n;
  Clock::time_point first{};
  bool any = false;
  for (;;) {
    const cudaError_t q = cudaStreamQuery(s);
    for (size_t l = 0; l < n && left; ++l) {
      if (!copied[l] && flags[l] == 1) {
        // The kernel fenced at system scope before raising the flag, so the
        // layer's bytes are visible to whoever sees the word.
        __atomic_store_n(&words[l], int64_t{1}, __ATOMIC_RELEASE);
        copied[l] = 1;
        --left;
        if (!any) {
          first = Clock::now();
          any = true;
        }
      }
    }
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) {
      cudaGetLastError();
      cuda_check(q, "load stream");
    }
    std::this_thread::yield();
  }
  // Every layer is in place once the stream is done.
  for (size_t l = 0; l < n; ++l) {
    if (!copied[l]) __atomic_store_n(&words[l], int64_t{1}, __ATOMIC_RELEASE);
  }
  return any ? first : Clock::now();
}

// ---------------------------------------------------------------------------
// Engine
// ---------------------------------------------------------------------------

Engine::Engine(const pf_engine_config& cfg) : cfg_(cfg) {
  if (cfg_.pool_bytes == 0) cfg_.pool_bytes = 30ull << 30;  // lib.rs:56
  PinKind kind = PinKind::kCudaHostAlloc;
  if (cfg_.pool_kind == PF_POOL_HOST) {
    kind = PinKind::kPlainHost;
  } else if (cfg_.use_hugepages) {
    kind = PinKind::kHugePagesRegistered;
  }
  if (cfg_.numa_pools != 0 && kind != PinKind::kPlainHost) {
    // Group the visible GPUs by NUMA node (numa_pools 1) or one per GPU (2);
    // each group gets a pool on its node, sized by its share of the GPUs.
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess) {
      cudaGetLastError();
      count = 0;
    }
    std::vector<int> group_node;
    std::vector<uint64_t> group_gpus;
    std::vector<size_t> group_of(static_cast<size_t>(count), 0);
    for (int d = 0; d < count; ++d) {
      const int node = device_numa_node(d);
      size_t g = group_node.size();
      if (cfg_.numa_pools == 1) {
        for (size_t i = 0; i < group_node.size(); ++i) {
          if (group_node[i] == node) g = i;
        }
      }
      if (g == group_node.size()) {
        group_node.push_back(node);
        group_gpus.push_back(0);
      }
      group_gpus[g] += 1;
      group_of[d] = g;
    }
    if (group_node.size() > 1) {
      uint64_t given = 0;
      for (size_t g = 0; g < group_node.size(); ++g) {
        const uint64_t bytes = g + 1 == group_node.size()
                                   ? cfg_.pool_bytes - given
                                   : cfg_.pool_bytes / static_cast<uint64_t>(count) * group_gpus[g];
        given += bytes;
        pools_.push_back(PinnedPool::create(bytes, kind, cfg_.write_combined != 0, cfg_.hint_value_size_bytes,
                                            group_node[g]));
      }
      device_pool_ = group_of;
    }
  }
  if (pools_.empty()) {
    pools_.push_back(PinnedPool::create(cfg_.pool_bytes, kind, cfg_.write_combined != 0, cfg_.hint_value_size_bytes));
  }
  StorageConfig sc;
  sc.enable_lfu_admission = cfg_.enable_lfu_admission != 0;
  sc.capacity_bytes = cfg_.pool_bytes;
  sc.hint_value_size_bytes = cfg_.hint_value_size_bytes;
  sc.pre_evict_enabled = cfg_.pre_evict_enabled != 0;
  if (cfg_.pre_evict_threshold_bytes) sc.pre_evict_threshold_bytes = cfg_.pre_evict_threshold_bytes;
  if (cfg_.pre_evict_target_bytes) sc.pre_evict_target_bytes = cfg_.pre_evict_target_bytes;
  if (cfg_.pre_evict_interval_ms) sc.pre_evict_interval_ms = cfg_.pre_evict_interval_ms;
  storage_ = std::make_unique<Storage>(pools_, sc);
  if (cfg_.dfs_root && cfg_.dfs_root[0]) {
    DfsConfig dc;
    dc.root = cfg_.dfs_root;
    if (cfg_.dfs_quota_bytes) dc.quota_bytes = cfg_.dfs_quota_bytes;
    if (cfg_.dfs_scan_interval_ms) dc.scan_interval_ms = cfg_.dfs_scan_interval_ms;
    if (cfg_.dfs_max_pack_size) dc.max_pack_size = cfg_.dfs_max_pack_size;
    dfs_ = std::make_unique<DfsTier>(storage_.get(), dc);
    DfsTier* tier = dfs_.get();
    storage_->set_seal_listener([tier](const BlockKey& k, const SealedBlockPtr& b) { tier->on_seal(k, b); });
  }
  cfg_.dfs_root = nullptr;  // the caller's string is not kept
}

Engine::~Engine() {
  // Finish queued loads before the blocks they read go away.
  std::map<int, std::shared_ptr<DeviceWorker>> devs;
  {
    std::lock_guard<std::mutex> g(dev_mu_);
    devs.swap(devices_);
  }
  for (auto& kv : devs) kv.second->wait_idle(600.0);
  {
    std::unique_lock<std::shared_mutex> g(inst_mu_);
    instances_.clear();
  }
  devs.clear();
  if (dfs_) {
    storage_->set_seal_listener(nullptr);
    dfs_.reset();  // stops its threads before the storage they use goes
  }
  storage_.reset();
  pools_.clear();
}

size_t Engine::pool_for_device(int device_id) const {
  if (device_id < 0 || static_cast<size_t>(device_id) >= device_pool_.size()) return 0;
  return device_pool_[static_cast<size_t>(device_id)];
}

std::shared_ptr<DeviceWorker> Engine::device_worker(int device_id) {
  std::lock_guard<std::mutex> g(dev_mu_);
  auto it = devices_.find(device_id);
  if (it != devices_.end()) return it->second;
  if (pools_.front()->kind() == PinKind::kPlainHost) return nullptr;
  auto w = std::make_shared<DeviceWorker>(device_id, cfg_.executor, &counters_);
  devices_[device_id] = w;
  return w;
}

std::shared_ptr<InstanceContext> Engine::get_instance(const std::string& id) {
  std::shared_lock<std::shared_mutex> g(inst_mu_);
  auto it = instances_.find(id);
  if (it == instances_.end()) throw instance_missing(id);
  return it->second;
}

std::shared_ptr<InstanceContext> Engine::get_or_create_instance(const std::string& id, const std::string& ns,
                                                                uint64_t num_layers, uint64_t tp_size) {
  // lib.rs:310-355
  auto mismatch = [&](const InstanceContext& inst) {
    return topology_mismatch("instance " + id + " exists with layers=" + std::to_string(inst.num_layers) +
                             ", tp=" + std::to_string(inst.tp_size) + "; requested layers=" +
                             std::to_string(num_layers) + ", tp=" + std::to_string(tp_size));
  };
  std::unique_lock<std::shared_mutex> g(inst_mu_);
  auto it = instances_.find(id);
  if (it != instances_.end()) {
    if (it->second->num_layers != num_layers || it->second->tp_size != tp_size) throw mismatch(*it->second);
    return it->second;
  }
  auto inst = std::make_shared<InstanceContext>();
  inst->id = id;
  inst->ns = ns;
  inst->num_layers = num_layers;
  inst->tp_size = tp_size;
  instances_[id] = inst;
  return inst;
}

std::shared_ptr<GpuContext> Engine::ensure_gpu(InstanceContext& inst, int device_id) {
  // InstanceContext::ensure_gpu (lib.rs:221-252). Workers are shared by all
  // instances on a device (one executor per GPU, with a save lane and a load
  // lane).
  if (device_id < 0) throw invalid_argument("device_id " + std::to_string(device_id) + " must be >= 0");
  {
    std::shared_lock<std::shared_mutex> g(inst.gpu_mu);
    auto it = inst.gpus.find(device_id);
    if (it != inst.gpus.end()) return it->second;
  }
  std::unique_lock<std::shared_mutex> g(inst.gpu_mu);
  auto it = inst.gpus.find(device_id);
  if (it != inst.gpus.end()) return it->second;
  auto ctx = std::make_shared<GpuContext>();
  ctx->device = device_id;
  try {
    ctx->worker = device_worker(device_id);
  } catch (const Error& e) {
    if (e.code() == PF_ERR_CUDA_INIT) throw;
    throw cuda_init(e.what());
  }
  inst.gpus[device_id] = ctx;
  return ctx;
}

void Engine::register_context_layer(const std::string& instance_id, const std::string& ns, int device_id,
                                    const std::string& layer_name, const pf_layer_desc& reg, uint64_t tp_rank,
                                    uint64_t tp_size, uint64_t num_layers) {
  (void)tp_rank;
  // lib.rs:389-403 then the overflow/bounds checks of :405-449.
  if (reg.bytes_per_block == 0 || reg.num_blocks == 0 || reg.segments == 0) {
    throw invalid_argument("invalid KV cache layout for layer " + layer_name);
  }
  if (reg.segments > 1 && reg.kv_stride_bytes == 0) {
    throw invalid_argument("kv_stride_bytes must be > 0 when segments > 1 for layer " + layer_name);
  }
  if (device_id < 0) throw invalid_argument("device_id must be >= 0");
  validate_layout(reg, layer_name.c_str());

  auto inst = get_or_create_instance(instance_id, ns, num_layers, tp_size);
  auto gpu = ensure_gpu(*inst, device_id);
  {
    std::lock_guard<std::mutex> g(inst->layer_mu);
    if (!inst->layer_ids.count(layer_name)) {
      inst->layer_ids[layer_name] = inst->layer_names.size();
      inst->layer_names.push_back(layer_name);
    }
  }
  std::lock_guard<std::mutex> g(gpu->mu);
  gpu->kv_caches[layer_name] = reg;
}

void Engine::unregister_instance(const std::string& instance_id) {
  std::unique_lock<std::shared_mutex> g(inst_mu_);
  if (instances_.erase(instance_id) == 0) throw instance_missing(instance_id);
}

namespace {

std::shared_ptr<GpuContext> get_gpu(InstanceContext& inst, int device_id) {
  std::shared_lock<std::shared_mutex> g(inst.gpu_mu);
  auto it = inst.gpus.find(device_id);
  return it == inst.gpus.end() ? nullptr : it->second;
}

bool get_layer_id(InstanceContext& inst, const std::string& name, uint64_t* out) {
  std::lock_guard<std::mutex> g(inst.layer_mu);
  auto it = inst.layer_ids.find(name);
  if (it == inst.layer_ids.end()) return false;
  *out = it->second;
  return true;
}

bool get_registration(GpuContext& gpu, const std::string& name, pf_layer_desc* out) {
  std::lock_guard<std::mutex> g(gpu.mu);
  auto it = gpu.kv_caches.find(name);
  if (it == gpu.kv_caches.end()) return false;
  *out = it->second;
  return true;
}

uint64_t slot_index(const InstanceContext& inst, uint64_t layer_id, uint64_t tp_rank) {
  // InstanceContext::get_slot_index (lib.rs:205-219)
  if (layer_id >= inst.num_layers) {
    throw invalid_argument("layer_id " + std::to_string(layer_id) + " out of range (" +
                           std::to_string(inst.num_layers) + " layers)");
  }
  if (tp_rank >= inst.tp_size) {
    throw invalid_argument("tp_rank " + std::to_string(tp_rank) + " out of range (tp_size " +
                           std::to_string(inst.tp_size) + ")");
  }
  return layer_id * inst.tp_size + tp_rank;
}

}  // namespace

void Engine::batch_save(const std::string& instance_id, uint64_t tp_rank, int device_id,
                        const std::vector<SaveEntry>& saves) {
  // batch_save_kv_blocks_from_ipc (lib.rs:497-520) + save_kv_blocks_from_ipc_inner
  // (lib.rs:553-782). The reference runs the entries one after another; here
  // every entry is planned first (same checks, same dedup, same allocations,
  // in the same order), then all planned layers move in one pipelined pass,
  // then slots are inserted in entry order. An error in entry k still leaves
  // entries 0..k-1 saved, as in the reference.
  auto inst = get_instance(instance_id);
  const std::string ns = inst->ns;

  struct Planned {
    std::string layer;
    pf_layer_desc reg;
    uint64_t slot, total_slots;
    bool split;
    std::vector<int64_t> ids;
    std::shared_ptr<const std::vector<std::string>> hashes;  // the entry's list when nothing was filtered
    std::shared_ptr<PoolAllocation> k_alloc, v_alloc;
    std::shared_ptr<DeviceWorker> worker;
  };
  std::vector<Planned> planned;
  std::unordered_map<uint64_t, std::unordered_set<std::string>> planned_slots;  // slot -> hashes planned
  std::exception_ptr pending;
  const auto t0 = Clock::now();
  // Entries usually carry the same hash list (one request, every layer): the
  // cache/inflight state of a list is probed once and reused while it repeats.
  SaveProbe probe;
  const std::vector<std::string>* probed = nullptr;
  // A layer listed again later in the batch must see this entry's hashes as
  // saved (the reference would have inserted them before reaching it).
  std::unordered_map<std::string, size_t> last_of_layer;
  for (size_t k = 0; k < saves.size(); ++k) last_of_layer[saves[k].layer_name] = k;

  for (size_t k_entry = 0; k_entry < saves.size(); ++k_entry) {
    const SaveEntry& e = saves[k_entry];
    try {
      static const std::vector<std::string> kNoHashes;
      const std::vector<std::string>& hashes = e.hashes ? *e.hashes : kNoHashes;
      if (e.block_ids.size() != hashes.size()) {
        throw invalid_argument("block_ids length " + std::to_string(e.block_ids.size()) +
                               " does not match block_hashes " + std::to_string(hashes.size()));
      }
      auto gpu = get_gpu(*inst, device_id);
      if (!gpu) throw worker_missing(instance_id, device_id);
      uint64_t layer_id = 0;
      if (!get_layer_id(*inst, e.layer_name, &layer_id)) {
        throw invalid_argument("layer " + e.layer_name + " unknown");
      }
      pf_layer_desc reg{};
      if (!get_registration(*gpu, e.layer_name, &reg)) {
        throw invalid_argument("layer " + e.layer_name + " not registered on device");
      }
      const uint64_t slot = slot_index(*inst, layer_id, tp_rank);
      const uint64_t total_slots = inst->num_layers * inst->tp_size;

      Planned p;
      p.layer = e.layer_name;
      p.reg = reg;
      p.slot = slot;
      p.total_slots = total_slots;
      p.split = is_split_layout(reg);
      std::vector<size_t> cand;
      cand.reserve(e.block_ids.size());
      for (size_t i = 0; i < e.block_ids.size(); ++i) {
        const int32_t id = e.block_ids[i];
        if (id < 0) continue;
        if (static_cast<uint64_t>(id) >= reg.num_blocks) {
          throw invalid_argument("block " + std::to_string(id) + " out of range for layer " + e.layer_name + " (" +
                                 std::to_string(reg.num_blocks) + " blocks registered)");
        }
        cand.push_back(i);
      }
      // Dedup (lib.rs:613-616): not sealed, not inflight for this slot, and
      // not planned for this slot by an earlier entry of this batch (which
      // the reference would already have inserted).
      if (probed == nullptr || (probed != &hashes && *probed != hashes)) {
        storage_->probe_save(ns, hashes, &probe);
        probed = &hashes;
      }
      const std::unordered_set<std::string>* earlier = nullptr;
      auto ps = planned_slots.find(slot);
      if (ps != planned_slots.end()) earlier = &ps->second;
      std::vector<size_t> keep;
      keep.reserve(cand.size());
      for (size_t j = 0; j < cand.size(); ++j) {
        if (!probe.needs(cand[j], slot) || (earlier && earlier->count(hashes[cand[j]]))) continue;
        keep.push_back(cand[j]);
      }
      if (keep.empty()) continue;
      p.ids.reserve(keep.size());
      for (size_t i : keep) p.ids.push_back(e.block_ids[i]);
      if (keep.size() == hashes.size()) {
        p.hashes = e.hashes;  // nothing filtered: share the caller's list
      } else {
        auto kept = std::make_shared<std::vector<std::string>>();
        kept->reserve(keep.size());
        for (size_t i : keep) kept->push_back(hashes[i]);
        p.hashes = std::move(kept);
      }
      const uint64_t n = p.ids.size();
      const size_t pool = pool_for_device(device_id);
      if (p.split) {
        const uint64_t bytes = reg.bytes_per_block * n;
        p.k_alloc = storage_->allocate(bytes, pool);
        if (!p.k_alloc) throw storage_error("pinned pool exhausted while allocating K segment buffer");
        p.v_alloc = storage_->allocate(bytes, pool);
        if (!p.v_alloc) throw storage_error("pinned pool exhausted while allocating V segment buffer");
      } else {
        const uint64_t bytes = reg.bytes_per_block * reg.segments * n;
        p.k_alloc = storage_->allocate(bytes, pool);
        if (!p.k_alloc) throw storage_error("pinned pool exhausted while allocating contiguous block buffer");
      }
      p.worker = gpu->worker;
      // Remember planned hashes only when another entry of this batch uses
      // the same slot (a layer listed twice); usually none does.
      if (last_of_layer[e.layer_name] > k_entry) planned_slots[slot].insert(p.hashes->begin(), p.hashes->end());
      planned.push_back(std::move(p));
    } catch (...) {
      pending = std::current_exception();
      break;
    }
  }

  if (!planned.empty()) {
    std::shared_ptr<DeviceWorker> worker = planned.front().worker;
    if (!worker) throw cuda_init("engine pool is plain host memory; transfers need a pinned pool");
    std::vector<pf_save_layer> layers(planned.size());
    for (size_t k = 0; k < planned.size(); ++k) {
      Planned& p = planned[k];
      pf_save_layer& s = layers[k];
      s.layer = p.reg;
      s.block_idx = p.ids.data();
      s.n = p.ids.size();
      s.k_dst = p.k_alloc->ptr;
      s.v_dst = p.split ? p.v_alloc->ptr : nullptr;
    }
    const auto t_plan = Clock::now();
    Executor& ex = worker->executor();
    // The call orders on a stream of its own, so concurrent saves on this
    // device (other instances, other RPC threads) each wait only for their
    // own copies; the executor's save lane still runs them in order.
    // The copy and its stream wait run with the save's device current; the
    // caller's own context is current again when the call returns.
    DeviceGuard on(ex.device());
    struct StreamLease {
      DeviceWorker* w;
      cudaStream_t s;
      ~StreamLease() { w->release_save_stream(s); }
    } lease{worker.get(), worker->acquire_save_stream()};
    ex.save(layers.data(), layers.size(), lease.s);

    // LayerBlocks (lib.rs:687-698, 755-763) are built while the copy runs,
    // one batch per entry sharing its pool allocations; their slots are
    // inserted once the bytes are in the pool.
    std::vector<std::shared_ptr<LayerBlockBatch>> built(planned.size());
    bool same_hashes = true;
    for (size_t k = 0; k < planned.size(); ++k) {
      Planned& p = planned[k];
      const uint64_t block_size = p.reg.bytes_per_block * p.reg.segments;
      auto batch = std::make_shared<LayerBlockBatch>();
      batch->k_alloc = p.k_alloc;
      batch->v_alloc = p.v_alloc;
      batch->blocks.resize(p.ids.size());
      for (size_t i = 0; i < p.ids.size(); ++i) {
        LayerBlock& lb = batch->blocks[i];
        if (p.split) {
          lb.k_ptr = p.k_alloc->ptr + i * p.reg.bytes_per_block;
          lb.v_ptr = p.v_alloc->ptr + i * p.reg.bytes_per_block;
        } else {
          lb.k_ptr = p.k_alloc->ptr + i * block_size;
          lb.v_ptr = nullptr;
        }
        lb.size = block_size;
      }
      built[k] = std::move(batch);
      if (k > 0 && same_hashes) same_hashes = p.hashes == planned[0].hashes || *p.hashes == *planned[0].hashes;
    }
    cuda_check(cudaStreamSynchronize(lease.s), "cudaStreamSynchronize(save)");
    const auto t_xfer = Clock::now();

    // insert_slot (lib.rs:700-705, 765-770): entry by entry, or in one
    // hash-major pass with the same outcome when every entry has the same list.
    auto count = [this](const Planned& p) {
      counters_.save_bytes.fetch_add(p.reg.bytes_per_block * p.reg.segments * p.ids.size());
      counters_.save_calls.fetch_add(1);
    };
    if (same_hashes && planned.size() > 1) {
      std::vector<SlotFill> fills(planned.size());
      for (size_t k = 0; k < planned.size(); ++k) fills[k] = SlotFill{planned[k].slot, built[k]};
      storage_->insert_slots_multi(ns, *planned[0].hashes, fills, planned[0].total_slots);
      for (const Planned& p : planned) count(p);
    } else {
      for (size_t k = 0; k < planned.size(); ++k) {
        Planned& p = planned[k];
        std::vector<LayerBlockPtr> blocks(p.ids.size());
        for (size_t i = 0; i < blocks.size(); ++i) blocks[i] = layer_block_at(built[k], i);
        storage_->insert_slots(ns, *p.hashes, p.slot, blocks, p.total_slots);
        count(p);
      }
    }
    std::lock_guard<std::mutex> g(counters_.ms_mu);
    counters_.save_ms += ms_since(t0);
    counters_.save_plan_ms += std::chrono::duration<double, std::milli>(t_plan - t0).count();
    counters_.save_transfer_ms += std::chrono::duration<double, std::milli>(t_xfer - t_plan).count();
    counters_.save_insert_ms += ms_since(t_xfer);
  }
  if (pending) std::rethrow_exception(pending);
}

uint64_t Engine::count_prefix_hit_blocks(const std::string& instance_id, const std::vector<std::string>& hashes) {
  // lib.rs:803-838
  auto inst = get_instance(instance_id);
  uint64_t hit = 0;
  for (const auto& h : hashes) {
    if (!storage_->cache_contains(inst->ns, h)) {
      counters_.misses.fetch_add(hashes.size() - hit);
      break;
    }
    ++hit;
  }
  if (hit) counters_.hits.fetch_add(hit);
  return hit;
}

PrefetchStatus Engine::query_prefetch(const std::string& instance_id, const std::vector<std::string>& hashes) {
  if (!dfs_) {
    // The server's query without the DFS tier (service.rs:307-319).
    PrefetchStatus st;
    st.hit_blocks = count_prefix_hit_blocks(instance_id, hashes);
    return st;
  }
  auto inst = get_instance(instance_id);
  return dfs_->query(inst->ns, hashes);
}

void Engine::batch_load(const std::string& instance_id, uint64_t tp_rank, int device_id, const std::string& shm,
                        const std::vector<std::string>& layer_names, const std::vector<int32_t>& block_ids,
                        const std::vector<std::string>& hashes) {
  // lib.rs:957-987: attach first so a failure before submission sets -1.
  pf_load_state* ls = attach_or_storage_error(shm);
  try {
    batch_load_inner(instance_id, tp_rank, device_id, shm, layer_names, block_ids, hashes);
  } catch (...) {
    fprintf(stderr, "pegaflow_b200: batch_load_kv_blocks_multi_layer failed before worker\n");
    load_state_set(ls, PF_LOAD_STATE_ERROR);
    load_state_close(ls);
    throw;
  }
  load_state_close(ls);
}

void Engine::batch_load_inner(const std::string& instance_id, uint64_t tp_rank, int device_id,
                              const std::string& shm, const std::vector<std::string>& layer_names,
                              const std::vector<int32_t>& block_ids, const std::vector<std::string>& hashes) {
  // lib.rs:990-1069
  const auto t0 = Clock::now();
  auto inst = get_instance(instance_id);
  auto gpu = get_gpu(*inst, device_id);
  if (!gpu) throw worker_missing(instance_id, device_id);
  std::vector<SealedBlockPtr> cache = storage_->cache_lookup_many(inst->ns, hashes);

  LoadTask task;
  task.shm = shm;
  for (const std::string& name : layer_names) {
    uint64_t layer_id = 0;
    if (!get_layer_id(*inst, name, &layer_id)) {
      throw invalid_argument("layer " + name + " unknown for instance " + instance_id);
    }
    pf_layer_desc reg{};
    if (!get_registration(*gpu, name, &reg)) {
      throw invalid_argument("layer " + name + " not registered on device " + std::to_string(device_id));
    }
    const uint64_t slot = slot_index(*inst, layer_id, tp_rank);
    LoadLayer L;
    L.name = name;
    L.reg = reg;
    const size_t n = std::min(block_ids.size(), cache.size());  // zip
    L.ids.reserve(n);
    L.blocks.reserve(n);
    for (size_t k = 0; k < n; ++k) {
      if (block_ids[k] < 0) continue;
      if (slot >= cache[k]->slots.size()) continue;
      L.ids.push_back(block_ids[k]);
      L.blocks.push_back(cache[k]->slots[slot]);
    }
    // Layers without blocks stay in the task (as empty entries) so per-layer
    // completion words line up with layer_names; the executor raises them at once.
    task.layers.push_back(std::move(L));
  }
  bool any = false;
  for (const LoadLayer& L : task.layers) any = any || !L.ids.empty();
  if (!any) {
    // lib.rs:1054-1060: nothing to load completes immediately.
    pf_load_state* ls = attach_or_storage_error(shm);
    const uint32_t nw = load_state_layers(ls);
    int64_t* w = load_state_layer_words(ls);
    for (uint32_t l = 0; l < nw && l < task.layers.size(); ++l) reinterpret_cast<volatile int64_t*>(w)[l] = 1;
    load_state_set(ls, PF_LOAD_STATE_SUCCESS);
    load_state_close(ls);
    return;
  }
  if (!gpu->worker) throw cuda_init("engine pool is plain host memory; transfers need a pinned pool");
  task.hold = std::move(cache);
  task.queued = Clock::now();
  {
    std::lock_guard<std::mutex> g(counters_.ms_mu);
    counters_.load_lookup_ms += std::chrono::duration<double, std::milli>(task.queued - t0).count();
  }
  gpu->worker->submit_load(std::move(task));
}

bool Engine::wait_loads(int device_id, double timeout_s) {
  std::shared_ptr<DeviceWorker> w;
  {
    std::lock_guard<std::mutex> g(dev_mu_);
    auto it = devices_.find(device_id);
    if (it == devices_.end()) return true;
    w = it->second;
  }
  return w->wait_idle(timeout_s);
}

void Engine::metrics(pf_engine_metrics* out) {
  *out = pf_engine_metrics{};
  out->save_bytes = counters_.save_bytes.load();
  out->save_calls = counters_.save_calls.load();
  out->load_bytes = counters_.load_bytes.load();
  out->load_calls = counters_.load_calls.load();
  out->load_failures = counters_.load_failures.load();
  out->cache_block_hits = counters_.hits.load();
  out->cache_block_misses = counters_.misses.load();
  {
    std::lock_guard<std::mutex> g(counters_.ms_mu);
    out->save_ms = counters_.save_ms;
    out->load_ms = counters_.load_ms;
    out->save_plan_ms = counters_.save_plan_ms;
    out->save_transfer_ms = counters_.save_transfer_ms;
    out->save_insert_ms = counters_.save_insert_ms;
    out->load_lookup_ms = counters_.load_lookup_ms;
    out->load_queue_ms = counters_.load_queue_ms;
    out->load_setup_ms = counters_.load_setup_ms;
    out->load_transfer_ms = counters_.load_transfer_ms;
    out->load_first_layer_ms = counters_.load_first_layer_ms;
  }
  auto& sc = storage_->counters();
  out->cache_block_insertions = sc.insertions.load();
  out->cache_block_admission_rejections = sc.admission_rejections.load();
  out->cache_block_evictions = sc.evictions.load();
  out->pool_alloc_failures = sc.pool_alloc_failures.load();
  out->inflight_dropped = sc.inflight_dropped.load();
  out->inflight_blocks = storage_->inflight_count();
  out->cached_blocks = storage_->cached_count();
}

}  // namespace pf
