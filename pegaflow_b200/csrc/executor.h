// Per-device transfer executor: the B200 replacement for GpuWorkerPool's copy
// loops (pegaflow-core/src/gpu_worker.rs:205-390).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <utility>
#include <vector>

#include "chunks.h"
#include "pegaflow.h"
#include "plan.h"
#include "plan_build.h"

namespace pf {

// Staging defaults. While the copy engines stream a D2H/H2D, every kernel
// launch on the device pays a fixed latency of 30-45 microseconds (the kernel
// itself runs no slower), so the chunk schedule (first chunk, doubling to the
// slot size) spends HBM on few, large launches: two 1 GiB slots per lane move
// a 10 GiB direction in ten or eleven launches, and a 1.25 GiB direction in
// two. On a 180 GB B200 the two lanes' 4 GiB are 2.2% of HBM.
constexpr uint64_t kDefaultSlotBytes = 1024ull << 20;
constexpr uint32_t kDefaultSlots = 2;
// A layer-wise load's first chunk holds its first layer whole up to this
// size, so layer 0's flag waits for that layer's DMA only (a 128 MiB layer
// split at 64 MiB waited for 192 MiB).
constexpr uint64_t kDefaultFirstChunkBytes = 256ull << 20;
// Lower bound of a layer-wise load's first chunk (which holds layer 0 and
// the small layers listed right after it).
constexpr uint64_t kLayerwiseMinFirstChunk = 4ull << 20;

// Throws unless the KV tensor [data_ptr, data_ptr + size_bytes) is device
// (or managed) memory of `device`: the DeviceCheck the executor's and the
// no-allocation save's plans use.
void check_device_memory(int device, const pf_layer_desc& l);

class Executor {
 public:
  Executor(int device, const pf_executor_config& cfg);
  ~Executor();
  Executor(const Executor&) = delete;
  Executor& operator=(const Executor&) = delete;

  int device() const { return device_; }
  // The executor's private streams, used by the blocking wrappers: one for
  // loads and peer copies, one for saves, so the two can overlap.
  cudaStream_t own_stream() const { return own_stream_; }
  cudaStream_t save_stream() const { return save_stream_; }

  // Enqueue a save/load ordered after `caller`; `caller` waits for completion.
  void save(const pf_save_layer* layers, uint64_t n_layers, cudaStream_t caller);
  void load(const pf_load_layer* layers, uint64_t n_layers, cudaStream_t caller,
            int64_t* layer_done);
  // Paged-to-paged copy between this device and `peer` over NVLink. pull:
  // this device holds the destination; push: this device holds the source.
  void p2p(const pf_p2p_layer* layers, uint64_t n_layers, int peer, bool push, cudaStream_t caller);
  void p2p_sync(const pf_p2p_layer* layers, uint64_t n_layers, int peer, bool push);
  // Blocking wrappers on the executor's own stream.
  void save_sync(const pf_save_layer* layers, uint64_t n_layers);
  void load_sync(const pf_load_layer* layers, uint64_t n_layers, int64_t* layer_done = nullptr);

  void stats(pf_executor_stats* out);
  void reset_stats();
  void set_timing(bool on);
  // Test hook: the next bulk launch leaves `tile` uncopied (its wait runs out).
  void debug_stall_tile(uint64_t tile);

 private:
  // Plans (plan_build.h) with this executor's device check.
  void build_save(const pf_save_layer* layers, uint64_t n, bool staged, Built* b);
  void build_load(const pf_load_layer* layers, uint64_t n, bool staged, Built* b);
  void build_p2p(const pf_p2p_layer* layers, uint64_t n, int peer, bool push, Built* b);
  void enable_peer(int peer);
  // Chunks of at most `first` bytes, doubling per chunk up to the slot size.
  void make_chunks(const Built& b, uint64_t first, std::vector<Chunk>* chunks);

  // One transfer pipeline: its kernel stream, copy streams, staging slots,
  // plan buffers and events. Saves run on the save lane, loads and peer
  // copies on the load lane, so a save and a load on one GPU proceed at the
  // same time (the host link is full duplex, and each direction has its own
  // copy engine). Calls on one lane run in order; `mu` serialises them on
  // the host, so a call on one lane never waits for the other lane's host
  // work. Plans are built before the lane is taken.
  struct Lane {
    std::mutex mu;
    cudaStream_t kstream = nullptr;
    std::vector<cudaStream_t> cstreams;
    std::vector<cudaEvent_t> ev_filled, ev_drained, ev_copy_done;
    cudaEvent_t ev_start = nullptr, ev_plan = nullptr, ev_done = nullptr;
    uint8_t* staging = nullptr;  // allocated on the lane's first staged call
    uint8_t* d_plan = nullptr;
    size_t d_plan_cap = 0;
    uint8_t* h_plan = nullptr;
    size_t h_plan_cap = 0;
    bool plan_pending = false;
  };
  void init_lane(Lane& l);
  void destroy_lane(Lane& l);
  uint8_t* lane_staging(Lane& l);
  CopyArgs upload(Lane& l, const Built& b, bool with_counters);
  void launch(Dir dir, bool table, const CopyArgs& args, uint64_t tile_begin,
              uint64_t tile_end, int64_t shift, cudaStream_t s, bool bulk = false);
  // The bulk kernel applies: enabled, and every layer of the plan 16-byte aligned.
  bool use_bulk(const Built& b) const;
  // Throws if a bulk kernel gave up on a bounded wait since the last check.
  void check_kernel_status();
  int grid_for(uint64_t tiles) const;
  // Both return the number of copy-engine copies issued.
  uint64_t copy_runs(const Built& b, const Chunk& c, uint8_t* slot, bool d2h,
                     cudaStream_t s);
  uint64_t issue_serial(const Built& b, cudaStream_t s, int64_t* layer_done);
  // Adds one call's counters to stats_.
  void account(uint64_t kernel_bytes, uint64_t copies, uint64_t saved, uint64_t loaded, uint64_t p2p);

  int device_;
  pf_executor_config cfg_;
  int num_sms_ = 148;
  bool bulk_ = false;                  // the bulk (TMA) kernel is enabled and ready on this device
  uint64_t stall_tile_ = ~0ull;        // test hook, consumed by the next bulk launch (stats_mu_)
  volatile int* status_host_ = nullptr;  // set by a bulk kernel whose bounded wait ran out
  int* status_dev_ = nullptr;          // device view of the same word
  cudaStream_t own_stream_ = nullptr;   // blocking loads and peer copies
  cudaStream_t save_stream_ = nullptr;  // blocking saves
  uint64_t slot_bytes_ = 0;
  uint64_t first_chunk_ = 0;  // limit of a load's first chunk; doubles per chunk up to slot_bytes_
  uint32_t slots_ = 0;
  Lane save_lane_, load_lane_;

  std::vector<int> peers_enabled_;  // touched only by peer copies, under load_lane_.mu

  // Counters and kernel timing, shared by both lanes.
  std::mutex stats_mu_;
  bool timing_ = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> timed_;  // pending kernel spans
  // Adds the finished spans at the front of timed_ to stats_ (stats_mu_ held).
  void fold_finished_timings();
  std::vector<cudaEvent_t> event_pool_;
  pf_executor_stats stats_{};
  // Kernel-body spans ({start, end} %globaltimer ns per timed launch): a
  // device array of kSpanCap entries, handed out in launch order while
  // timing is on and read back by stats().
  static constexpr uint64_t kSpanCap = 8192;
  unsigned long long* spans_ = nullptr;
  uint64_t spans_used_ = 0;
  uint64_t unregistered_launches_ = 0;  // timed launches whose events are not yet in timed_
  void reset_spans();  // stats_mu_ held; no timed launch in flight
};

}  // namespace pf
