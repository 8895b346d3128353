// Packed-file tier behind the pinned pool: sealed blocks are written through
// to files under a root directory, and blocks missing from the pool are read
// back (prefetched) from there. Restates the reference's DFS offload
// (pegaflow-core/src/seal_offload.rs) with its file format and per-block
// metadata records unchanged:
//
//   {root}/{namespace}/{uuid}.bin   blocks back to back; per block, per slot:
//                                   K half then V half (split) or the slot's
//                                   bytes (contiguous) (seal_offload.rs:379-448)
//   BlockMeta  {"file","offset","slots":[{"is_split","size"}],"total_slots"}
//   FileMeta   {"blocks":[hex hash...],"size"}
//
// The reference keeps the metadata in Redis (no Redis here); this tier keeps
// the same JSON records in memory and in a sidecar file next to each packed
// file ({uuid}.bin.meta), from which the index is rebuilt on start.
#pragma once

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <utility>
#include <vector>

#include "storage.h"

namespace pf {

struct DfsConfig {
  std::string root;                        // --dfs-root
  uint64_t quota_bytes = 50ull << 30;      // --dfs-quota (server default 50gb)
  uint64_t scan_interval_ms = 100;         // --dfs-scan-interval-ms
  uint32_t max_pack_size = 64;             // blocks per packed file (DfsOffloadConfig::default)
};

struct SlotMeta {
  bool is_split;
  uint64_t size;  // K + V bytes of the slot
};

// BlockMeta (seal_offload.rs:79-98).
struct BlockMeta {
  std::string file;
  uint64_t offset = 0;
  std::vector<SlotMeta> slots;
  uint64_t total_slots = 0;
  uint64_t total_size() const;
};

// serde_json's compact encoding of the reference structs, field order kept.
std::string block_meta_json(const BlockMeta& m);
bool parse_block_meta_json(const std::string& s, BlockMeta* out);
std::string file_meta_json(const std::vector<std::string>& hex_hashes, uint64_t size);
std::string hex_encode(const std::string& bytes);
bool hex_decode(const std::string& hex, std::string* out);

// PrefetchStatus (seal_offload.rs:584-601), numbered as engine.proto's PrefetchState.
enum class PrefetchState : uint32_t { kReady = 0, kLoading = 1, kPartialMiss = 2 };
struct PrefetchStatus {
  PrefetchState state = PrefetchState::kReady;
  uint64_t hit_blocks = 0;
  uint64_t loading_blocks = 0;
  uint64_t missing_blocks = 0;
};

struct DfsStats {
  uint64_t files, blocks, usage_bytes;
  uint64_t written_files, written_blocks, write_failures;
  uint64_t prefetched_blocks, prefetch_failures, evicted_files;
};

class DfsTier {
 public:
  // Rebuilds the index from the sidecar files under cfg.root, then starts the
  // writer, quota and prefetch threads. `storage` must outlive the tier.
  DfsTier(Storage* storage, DfsConfig cfg);
  ~DfsTier();
  DfsTier(const DfsTier&) = delete;
  DfsTier& operator=(const DfsTier&) = delete;

  // Seal notification (storage.rs:494-503): queued with a weak reference, so a
  // block evicted before its turn is skipped.
  void on_seal(const BlockKey& key, const SealedBlockPtr& block);

  // count_prefix_hit_blocks_async (lib.rs:855-942): counts the cached prefix
  // and blocks being prefetched; at the first block in neither, starts a
  // prefetch of the rest when that block is in the tier.
  PrefetchStatus query(const std::string& ns, const std::vector<std::string>& hashes);

  // Waits until queued writes and prefetches are done (false on timeout).
  bool flush(double timeout_s);
  // Runs one quota check now (the quota thread also runs it every interval).
  void check_quota();
  DfsStats stats();
  bool has_block(const std::string& ns, const std::string& hash);

 private:
  struct FileEntry {
    std::string ns, uuid, member;
    uint64_t ts_ms, size;
    std::vector<std::string> hashes;  // raw hash bytes
  };
  using Pending = std::pair<BlockKey, std::weak_ptr<SealedBlock>>;
  struct PrefetchTask {
    std::string ns;
    std::vector<std::pair<std::string, BlockMeta>> blocks;
  };

  void load_index();
  void writer_loop();
  void quota_loop();
  void prefetch_loop();
  void write_and_register(const std::string& ns, const std::vector<std::pair<BlockKey, SealedBlockPtr>>& blocks);
  void run_prefetch(PrefetchTask& task);
  static std::string index_key(const std::string& ns, const std::string& hash) { return ns + '\0' + hash; }

  Storage* storage_;
  DfsConfig cfg_;

  std::mutex mu_;  // index, files, usage, pending, queues
  std::condition_variable cv_;       // writer queue / stop
  std::condition_variable pcv_;      // prefetch queue / stop
  std::condition_variable idle_cv_;  // flush waiters
  std::condition_variable quota_cv_;
  std::deque<Pending> queue_;
  std::deque<PrefetchTask> prefetch_queue_;
  bool writer_busy_ = false, prefetch_busy_ = false, stop_ = false;
  std::map<std::pair<uint64_t, std::string>, FileEntry> files_;  // (timestamp, member): oldest first
  std::unordered_map<std::string, BlockMeta> index_;             // ns\0hash -> where the block lives
  std::unordered_set<std::string> pending_;                      // ns\0hash being prefetched
  uint64_t usage_ = 0;
  DfsStats st_{};

  std::thread writer_, quota_, prefetch_;
};

}  // namespace pf
