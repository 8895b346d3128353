// PegaEngine (pegaflow-core/src/lib.rs:93-1069) over the B200 executor.
#pragma once

#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <shared_mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "dfs_tier.h"
#include "executor.h"
#include "pegaflow.h"
#include "storage.h"

struct pf_load_state;

namespace pf {

pf_load_state* load_state_create(uint32_t n_layers);
pf_load_state* load_state_attach(const std::string& name);
void load_state_close(pf_load_state* s);
int64_t load_state_get(const pf_load_state* s);
void load_state_set(pf_load_state* s, int64_t v);
uint32_t load_state_layers(const pf_load_state* s);
int64_t* load_state_layer_words(pf_load_state* s);
void* load_state_base(pf_load_state* s, size_t* len);

struct EngineCounters {
  std::atomic<uint64_t> save_bytes{0}, save_calls{0}, load_bytes{0}, load_calls{0}, load_failures{0};
  std::atomic<uint64_t> hits{0}, misses{0};
  std::mutex ms_mu;
  double save_ms = 0, load_ms = 0;
  double save_plan_ms = 0, save_transfer_ms = 0, save_insert_ms = 0;
  double load_lookup_ms = 0, load_queue_ms = 0, load_setup_ms = 0, load_transfer_ms = 0, load_first_layer_ms = 0;
};

// One load task (gpu_worker.rs:12-28): layers with the LayerBlocks they read,
// held until the copy has finished.
struct LoadLayer {
  std::string name;
  pf_layer_desc reg;
  std::vector<int64_t> ids;
  std::vector<const LayerBlock*> blocks;  // kept alive by LoadTask::hold
};
struct LoadTask {
  std::vector<LoadLayer> layers;
  std::string shm;
  std::vector<SealedBlockPtr> hold;  // the sealed blocks read by the task
  std::chrono::steady_clock::time_point queued;  // when the task was handed to the load thread
};

// Per-device worker: the executor plus the load thread of GpuWorkerPool
// (gpu_worker.rs:61-201). Saves run on the caller's thread (the reference
// caller awaits them too); loads are queued and completed through LoadState.
class DeviceWorker {
 public:
  DeviceWorker(int device, const pf_executor_config& cfg, EngineCounters* counters);
  ~DeviceWorker();
  Executor& executor() { return *exec_; }
  void submit_load(LoadTask task);
  bool wait_idle(double timeout_s);
  // A stream for one save call to order on and wait for, so that concurrent
  // saves on this device each wait only for their own copies. Return it with
  // release_save_stream once synchronised.
  cudaStream_t acquire_save_stream();
  void release_save_stream(cudaStream_t s);

 private:
  std::mutex streams_mu_;
  std::vector<cudaStream_t> free_save_streams_, all_save_streams_;
  void load_loop();
  void process(LoadTask& task);
  // Loads `layers`, raising `words[l]` (a LoadState's per-layer words) as
  // layer l lands: the kernels raise flags in this worker's own mapped
  // pinned array, and this thread copies each new one into `words` while the
  // load runs. The LoadState page itself is never registered with CUDA.
  // Returns when the first layer was marked ready.
  std::chrono::steady_clock::time_point load_with_layer_words(const pf_load_layer* layers, size_t n, int64_t* words);
  std::unique_ptr<Executor> exec_;
  std::unique_ptr<PinnedMemory> flags_mem_;  // per-layer flags the kernels raise (grown on demand)
  EngineCounters* counters_;
  std::mutex mu_;
  std::condition_variable cv_, idle_cv_;
  std::deque<LoadTask> queue_;
  bool busy_ = false;
  bool stop_ = false;
  std::thread thread_;
};

struct GpuContext {
  int device;
  std::mutex mu;
  std::unordered_map<std::string, pf_layer_desc> kv_caches;
  std::shared_ptr<DeviceWorker> worker;  // null for host-only engines
};

struct InstanceContext {
  std::string id, ns;
  uint64_t num_layers, tp_size;
  std::mutex layer_mu;
  std::unordered_map<std::string, uint64_t> layer_ids;
  std::vector<std::string> layer_names;
  std::shared_mutex gpu_mu;
  std::map<int, std::shared_ptr<GpuContext>> gpus;
};

class Engine {
 public:
  explicit Engine(const pf_engine_config& cfg);
  ~Engine();

  void register_context_layer(const std::string& instance_id, const std::string& ns, int device_id,
                              const std::string& layer_name, const pf_layer_desc& reg, uint64_t tp_rank,
                              uint64_t tp_size, uint64_t num_layers);
  void unregister_instance(const std::string& instance_id);

  struct SaveEntry {
    std::string layer_name;
    std::vector<int32_t> block_ids;
    // Entries of one call that pass the same hash array share one list.
    std::shared_ptr<const std::vector<std::string>> hashes;
  };
  void batch_save(const std::string& instance_id, uint64_t tp_rank, int device_id,
                  const std::vector<SaveEntry>& saves);
  uint64_t count_prefix_hit_blocks(const std::string& instance_id, const std::vector<std::string>& hashes);
  // count_prefix_hit_blocks_async (lib.rs:855-942) over the packed-file tier;
  // READY with the plain prefix count when the tier is off.
  PrefetchStatus query_prefetch(const std::string& instance_id, const std::vector<std::string>& hashes);
  DfsTier* dfs() { return dfs_.get(); }
  void batch_load(const std::string& instance_id, uint64_t tp_rank, int device_id, const std::string& shm,
                  const std::vector<std::string>& layer_names, const std::vector<int32_t>& block_ids,
                  const std::vector<std::string>& hashes);
  bool wait_loads(int device_id, double timeout_s);

  Storage& storage() { return *storage_; }
  std::shared_ptr<DeviceWorker> device_worker(int device_id);
  void metrics(pf_engine_metrics* out);

 private:
  std::shared_ptr<InstanceContext> get_instance(const std::string& id);
  std::shared_ptr<InstanceContext> get_or_create_instance(const std::string& id, const std::string& ns,
                                                          uint64_t num_layers, uint64_t tp_size);
  std::shared_ptr<GpuContext> ensure_gpu(InstanceContext& inst, int device_id);
  void batch_load_inner(const std::string& instance_id, uint64_t tp_rank, int device_id, const std::string& shm,
                        const std::vector<std::string>& layer_names, const std::vector<int32_t>& block_ids,
                        const std::vector<std::string>& hashes);

  // The pool a save on `device_id` allocates from.
  size_t pool_for_device(int device_id) const;

  pf_engine_config cfg_;
  std::vector<std::shared_ptr<PinnedPool>> pools_;
  std::vector<size_t> device_pool_;  // device -> index in pools_ (empty: one pool)
  std::unique_ptr<Storage> storage_;
  std::unique_ptr<DfsTier> dfs_;  // null when the packed-file tier is off
  std::shared_mutex inst_mu_;
  std::unordered_map<std::string, std::shared_ptr<InstanceContext>> instances_;
  std::mutex dev_mu_;
  std::map<int, std::shared_ptr<DeviceWorker>> devices_;
  EngineCounters counters_;
};

}  // namespace pf
