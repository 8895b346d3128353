// Pinned pool + block store (pegaflow-core/src/pinned_pool.rs, storage.rs, cache.rs).
//
// Lifecycle of a block (storage.rs:1-13): allocate -> write (inflight, one
// slot per (layer, tp_rank)) -> seal when every slot is filled -> cache
// (read-only, LRU with optional TinyLFU admission) -> evict. Sealing is a
// one-way gate. Pool memory is reference counted: a LayerBlock keeps its
// allocation alive, and an allocation is returned to the pool when the last
// LayerBlock sharing it is dropped.
#pragma once

#include <algorithm>
#include <array>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <functional>
#include <list>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "offset_allocator.h"
#include "pinned.h"

namespace pf {

class PinnedPool;

// RAII pool allocation (PinnedAllocation, pinned_pool.rs:16-52).
struct PoolAllocation {
  std::shared_ptr<PinnedPool> pool;
  ScaledOffsetAllocator::Allocation a;
  uint8_t* ptr;
  ~PoolAllocation();
};

class PinnedPool : public std::enable_shared_from_this<PinnedPool> {
 public:
  // PinnedMemoryPool::new (pinned_pool.rs:67-113). The allocator unit is
  // max(reference unit, 64 B) so every allocation starts 64-byte aligned.
  // numa_node >= 0 places the pool's pages on that node (PinnedMemory).
  static std::shared_ptr<PinnedPool> create(uint64_t bytes, PinKind kind, bool write_combined,
                                            uint64_t unit_hint, int numa_node = -1);
  std::shared_ptr<PoolAllocation> allocate(uint64_t size);  // null when it cannot fit
  void usage(uint64_t* used, uint64_t* total);
  uint64_t largest_free();
  uint8_t* base() const { return mem_->data(); }
  PinKind kind() const { return mem_->kind(); }
  const PinnedMemory& memory() const { return *mem_; }
  bool contains(const void* p) const {
    const uint8_t* q = static_cast<const uint8_t*>(p);
    return q >= mem_->data() && q < mem_->data() + mem_->size();
  }
  void free_internal(const ScaledOffsetAllocator::Allocation& a);

 private:
  PinnedPool(std::unique_ptr<PinnedMemory> mem, ScaledOffsetAllocator alloc)
      : mem_(std::move(mem)), alloc_(std::move(alloc)) {}
  std::unique_ptr<PinnedMemory> mem_;
  std::mutex mu_;
  ScaledOffsetAllocator alloc_;
};

// Host bytes of one (block, slot) (LayerBlock, storage.rs:249-310).
struct LayerBlock {
  uint8_t* k_ptr;
  uint8_t* v_ptr;  // null for contiguous blocks
  uint64_t size;   // block_size_bytes (memory_footprint)
};
// The blocks one save call wrote for one layer. They share the call's K (and
// V) pool allocations, which go back to the pool when no sealed or inflight
// block holds the batch any more (directly, or through the owner group of
// the call that wrote it; see SlotOwner): the lifetime the reference gets
// from one Arc<PinnedAllocation> per block (storage.rs:249-261), with one
// heap object per (call, layer) instead of one per block.
struct LayerBlockBatch {
  std::vector<LayerBlock> blocks;
  std::shared_ptr<PoolAllocation> k_alloc;
  std::shared_ptr<PoolAllocation> v_alloc;
};
// Points at one block of a batch and keeps the whole batch alive.
using LayerBlockPtr = std::shared_ptr<LayerBlock>;
inline LayerBlockPtr layer_block_at(const std::shared_ptr<LayerBlockBatch>& batch, size_t i) {
  return LayerBlockPtr(batch, &batch->blocks[i]);
}
// Keeps the batches that a block's slots point into alive: a LayerBlockPtr
// (its batch), or the group of every batch one multi-slot insert call wrote.
// A block holds one owner per call that filled any of its slots, so a TP
// block of L layers saved by T ranks holds T owners, not L x T batch
// references; dropping an evicted block is T reference-count decrements.
using SlotOwner = std::shared_ptr<const void>;

// One layer's share of a multi-slot insert: block i of `batch` goes into
// `slot` of hash i.
struct SlotFill {
  uint64_t slot;
  std::shared_ptr<LayerBlockBatch> batch;
};

// Cache and inflight state of one hash list, for the save-side dedup of
// several slots at once (lib.rs:613-616 per (hash, slot)).
struct SaveProbe {
  std::vector<char> cached;              // per hash: sealed in the cache
  std::vector<std::vector<char>> filled; // per hash: filled slots (empty when not inflight)
  bool needs(size_t i, uint64_t slot) const {
    return !cached[i] && !(slot < filled[i].size() && filled[i][slot]);
  }
};

struct SealedBlock {
  // Per slot, its host bytes (all set once sealed); valid while `owners` lives.
  std::vector<const LayerBlock*> slots;
  std::vector<SlotOwner> owners;
  uint64_t footprint = 0;
};
using SealedBlockPtr = std::shared_ptr<SealedBlock>;

struct BlockKey {
  std::string ns;
  std::string hash;
  bool operator==(const BlockKey& o) const { return ns == o.ns && hash == o.hash; }
};
struct BlockKeyHash {
  size_t operator()(const BlockKey& k) const;
};

struct StorageConfig {
  bool enable_lfu_admission = true;
  uint64_t capacity_bytes = 0;
  uint64_t hint_value_size_bytes = 0;
  bool pre_evict_enabled = false;
  uint64_t pre_evict_threshold_bytes = 5ull << 30;  // storage.rs:35
  uint64_t pre_evict_target_bytes = 8ull << 30;     // storage.rs:37
  uint64_t pre_evict_interval_ms = 100;             // storage.rs:39
  // An inflight block older than this is dropped with its pool memory (0 =
  // never). A block skipped for one layer because it was cached, then
  // evicted before its next layer is saved, becomes an inflight block whose
  // earlier slots never arrive (the race lib.rs:604-611 describes; the
  // reference proposes this cleanup but has none).
  uint64_t inflight_max_age_ms = 3600ull * 1000;
};

struct StorageCounters {
  std::atomic<uint64_t> insertions{0};
  std::atomic<uint64_t> admission_rejections{0};
  std::atomic<uint64_t> evictions{0};
  std::atomic<uint64_t> pool_alloc_failures{0};
  std::atomic<uint64_t> inflight_dropped{0};  // stale inflight blocks released
};

// Count-min-sketch TinyLFU (cache.rs:99-243), deterministic hashing.
class TinyLfu {
 public:
  explicit TinyLfu(uint64_t cache_size);
  uint8_t get(const BlockKey& k) const;
  uint8_t incr(const BlockKey& k);

 private:
  void age();
  uint64_t slots_;
  std::vector<std::vector<std::atomic<uint8_t>>> rows_;
  std::atomic<uint64_t> window_{0};
  uint64_t window_limit_;
};

class Storage {
 public:
  Storage(std::shared_ptr<PinnedPool> pool, const StorageConfig& cfg);
  // Several pools (one per NUMA node, say): every allocation names its pool,
  // and reclaim for a pool evicts, in LRU order, only the cached blocks that
  // hold memory in that pool. With one pool this is the reference's storage.
  Storage(std::vector<std::shared_ptr<PinnedPool>> pools, const StorageConfig& cfg);
  ~Storage();

  // StorageEngine::allocate (storage.rs:405-433): evicts LRU blocks until the
  // allocator reports a large enough free region. `pool` indexes the pools
  // (out-of-range values use the last one).
  std::shared_ptr<PoolAllocation> allocate(uint64_t size, size_t pool = 0);
  bool inflight_has_slot(const std::string& ns, const std::string& hash, uint64_t slot);
  // The save-side dedup answer, !cache_contains && !inflight_has_slot, for
  // every (hash, slot) of one hash list, from one cache and one inflight
  // lookup per hash under one acquisition of each lock (the reference checks
  // each block separately, lib.rs:613-616; the answers are the same).
  void probe_save(const std::string& ns, const std::vector<std::string>& hashes, SaveProbe* out);
  // insert_slot for many (hash, block) pairs of one slot, in order.
  void insert_slots(const std::string& ns, const std::vector<std::string>& hashes, uint64_t slot,
                    std::vector<LayerBlockPtr>& blocks, uint64_t total_slots);
  // The same end state, cache order and admission decisions as calling
  // insert_slots(ns, hashes, f.slot, <the blocks of f.batch>, total_slots)
  // for each fill in order, with one inflight lookup per hash instead of one
  // per (hash, fill).
  void insert_slots_multi(const std::string& ns, const std::vector<std::string>& hashes,
                          const std::vector<SlotFill>& fills, uint64_t total_slots);
  // StorageEngine::insert_slot (storage.rs:457-514). Throws pf::Error(Storage)
  // on SlotOutOfBounds / SlotCountMismatch.
  bool insert_slot(const std::string& ns, const std::string& hash, uint64_t slot, LayerBlockPtr block,
                   uint64_t total_slots);
  bool cache_contains(const std::string& ns, const std::string& hash);
  // Inserts a block that was not sealed here (a block read back from the
  // packed-file tier), with the same admission as a freshly sealed block.
  bool cache_insert(const std::string& ns, const std::string& hash, SealedBlockPtr block);
  // Called once for every block that seals, before it is offered to the
  // cache (the reference's seal notification, storage.rs:494-503). It runs on
  // the inserting thread outside the storage locks and must not block.
  using SealListener = std::function<void(const BlockKey&, const SealedBlockPtr&)>;
  void set_seal_listener(SealListener fn);
  // cache_lookup_many (storage.rs:529-547): bumps recency/frequency.
  std::vector<SealedBlockPtr> cache_lookup_many(const std::string& ns, const std::vector<std::string>& hashes);
  // Read-only peek (no LRU/frequency update), for introspection.
  SealedBlockPtr cache_peek(const std::string& ns, const std::string& hash);

  uint64_t inflight_count();
  uint64_t cached_count();
  // Drops every inflight block older than inflight_max_age_ms and returns
  // how many. Saves run it on their own, at most every few seconds.
  uint64_t drop_stale_inflight();
  // Read-only views (hash, slot block addresses; null = empty slot): the
  // cache from least to most recently used, and inflight blocks by hash.
  using BlockView = std::vector<std::pair<std::string, std::vector<const LayerBlock*>>>;
  BlockView cache_view();
  BlockView inflight_view();
  StorageCounters& counters() { return counters_; }
  PinnedPool& pool(size_t i = 0) { return *pools_[std::min(i, pools_.size() - 1)]; }
  size_t pool_count() const { return pools_.size(); }
  // Totals over all pools; largest_free is the largest of the pools'.
  void usage(uint64_t* used, uint64_t* total);
  uint64_t largest_free();

 private:
  bool cache_insert_locked(const BlockKey& key, SealedBlockPtr block);  // TinyLFU admission
  void reclaim_until_fits(uint64_t required, size_t pool, uint64_t* freed_blocks);
  // Evicts cached blocks in LRU order until `bytes` of footprint are gone,
  // taking only blocks that hold memory in `pool` when there are several.
  std::vector<SealedBlockPtr> evict_lru(uint64_t max_blocks, uint64_t bytes, size_t pool);
  // Drops what evict_lru returned (releasing pool memory) and ends its
  // dropping_ count. wait_for_drops waits (until `deadline`) until no thread
  // holds evicted blocks or `p` has room for `size`; false when no thread
  // held any or the deadline passed.
  void drop_evicted(std::vector<SealedBlockPtr>& evicted);
  bool wait_for_drops(PinnedPool& p, uint64_t size, std::chrono::steady_clock::time_point deadline);
  std::atomic<int> dropping_{0};  // evict_lru results not yet dropped
  bool holds_memory_in(const SealedBlock& b, size_t pool) const;
  void pre_evict_loop();

  struct Inflight {
    std::vector<const LayerBlock*> slots;  // null = not filled yet
    std::vector<SlotOwner> owners;
    uint64_t remaining;
    uint64_t total_slots;
    uint64_t footprint = 0;
    std::chrono::steady_clock::time_point created = std::chrono::steady_clock::now();
  };
  // Runs drop_stale_inflight when the last sweep is older than a quarter of
  // the age limit (at most once a minute), so a save pays for it rarely.
  void maybe_drop_stale_inflight();
  std::atomic<int64_t> last_sweep_ns_{0};
  using LruList = std::list<std::pair<BlockKey, SealedBlockPtr>>;

  std::vector<std::shared_ptr<PinnedPool>> pools_;
  StorageConfig cfg_;
  // Inflight blocks, split into shards by key, each with its own lock: the
  // saves of different TP ranks fill different slots of the same hashes at
  // the same time, and under one lock for all blocks they ran one after
  // another (the reference keeps inflight blocks in a sharded concurrent
  // map). A call takes one shard's lock at a time.
  static constexpr size_t kInflightShards = 64;
  struct InflightShard {
    std::mutex mu;
    std::unordered_map<BlockKey, Inflight, BlockKeyHash> map;
    // Entries per slot count, and a summary readable without the lock (0:
    // no entries, the slot count all entries share, or ~0 when they differ),
    // so that a call can tell that no entry here has a slot count other than
    // its own without a lookup per hash or waiting for the lock.
    std::unordered_map<uint64_t, uint32_t> totals;
    std::atomic<uint64_t> sole_total{0};
    void summarize() {
      sole_total.store(totals.empty() ? 0 : totals.size() == 1 ? totals.begin()->first : ~0ull,
                       std::memory_order_release);
    }
  };
  using InflightIt = std::unordered_map<BlockKey, Inflight, BlockKeyHash>::iterator;
  // Add an empty entry for `key` / remove one, with the shard's lock held;
  // both keep inflight_blocks_ and the shard's slot-count tally.
  InflightIt inflight_add(InflightShard& sh, const BlockKey& key, uint64_t total_slots);
  InflightIt inflight_remove(InflightShard& sh, InflightIt it);
  std::array<InflightShard, kInflightShards> inflight_;
  std::atomic<uint64_t> inflight_blocks_{0};  // entries over all shards
  static size_t shard_of(const BlockKey& k);
  static size_t shard_of_hash(uint64_t key_hash);  // shard_of from BlockKeyHash's value
  InflightShard& shard(const BlockKey& k) { return inflight_[shard_of(k)]; }
  std::mutex cache_mu_;
  LruList lru_;  // front = least recently used
  std::unordered_map<BlockKey, LruList::iterator, BlockKeyHash> index_;
  std::unique_ptr<TinyLfu> lfu_;
  StorageCounters counters_;

  void notify_sealed(const BlockKey& key, const SealedBlockPtr& block);
  std::mutex listener_mu_;
  SealListener seal_listener_;

  std::thread pre_evict_;
  std::mutex stop_mu_;
  std::condition_variable stop_cv_;
  bool stop_ = false;
};

}  // namespace pf
