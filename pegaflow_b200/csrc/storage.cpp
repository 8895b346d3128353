#include "storage.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <string_view>
#include <unordered_set>

#include "common.h"

namespace pf {

namespace {

uint64_t fnv1a(const std::string& a, const std::string& b) {
  uint64_t h = 1469598103934665603ull;
  for (unsigned char c : a) {
    h ^= c;
    h *= 1099511628211ull;
  }
  h ^= 0xffu;
  h *= 1099511628211ull;
  for (unsigned char c : b) {
    h ^= c;
    h *= 1099511628211ull;
  }
  return h;
}

uint64_t splitmix64(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

constexpr uint64_t kDefaultBytesPerValue = 128ull << 20;  // cache.rs:14
constexpr uint64_t kReclaimBatch = 64;                      // storage.rs:41
constexpr int kMaxDropWaits = 64;  // allocate: waits for other threads' drops before failing
constexpr uint64_t kPoolMinUnit = 64;
constexpr uint32_t kPoolMaxAllocs = 4000000;  // pinned_pool.rs:61

}  // namespace

size_t BlockKeyHash::operator()(const BlockKey& k) const { return static_cast<size_t>(fnv1a(k.ns, k.hash)); }

size_t Storage::shard_of(const BlockKey& k) { return shard_of_hash(BlockKeyHash{}(k)); }

size_t Storage::shard_of_hash(uint64_t h) {
  // The top bits of a multiplicative mix of the key's hash, so a shard's own
  // map (which buckets by the same hash) still spreads its keys.
  return static_cast<size_t>((h * 0x9E3779B97F4A7C15ull) >> 58);
}

// ---------------------------------------------------------------------------
// Pool
// ---------------------------------------------------------------------------

PoolAllocation::~PoolAllocation() {
  if (pool) pool->free_internal(a);
}

std::shared_ptr<PinnedPool> PinnedPool::create(uint64_t bytes, PinKind kind, bool write_combined,
                                               uint64_t unit_hint, int numa_node) {
  if (bytes == 0) throw invalid_argument("Pinned memory pool size must be greater than zero");
  auto mem = std::make_unique<PinnedMemory>(bytes, kind, write_combined, numa_node);
  const uint64_t actual = mem->size();
  uint64_t unit = unit_hint;
  if (unit == 0) unit = actual > 0xffffffffull ? (actual + 0xfffffffeull) / 0xffffffffull : 1;
  unit = std::max(unit, kPoolMinUnit);
  auto alloc = ScaledOffsetAllocator::make(actual, unit, false, kPoolMaxAllocs);
  return std::shared_ptr<PinnedPool>(new PinnedPool(std::move(mem), std::move(alloc)));
}

std::shared_ptr<PoolAllocation> PinnedPool::allocate(uint64_t size) {
  ScaledOffsetAllocator::Allocation a{};
  {
    std::lock_guard<std::mutex> g(mu_);
    try {
      if (!alloc_.allocate(size, &a)) return nullptr;
    } catch (const Error&) {
      return nullptr;  // RequestTooLarge is logged and treated as exhaustion (pinned_pool.rs:130-138)
    }
  }
  auto out = std::make_shared<PoolAllocation>();
  out->pool = shared_from_this();
  out->a = a;
  out->ptr = mem_->data() + a.offset_bytes;
  return out;
}

void PinnedPool::free_internal(const ScaledOffsetAllocator::Allocation& a) {
  std::lock_guard<std::mutex> g(mu_);
  alloc_.free(a);
}

void PinnedPool::usage(uint64_t* used, uint64_t* total) {
  std::lock_guard<std::mutex> g(mu_);
  *total = alloc_.total_bytes();
  *used = *total - alloc_.total_free_bytes();
}

uint64_t PinnedPool::largest_free() {
  std::lock_guard<std::mutex> g(mu_);
  return alloc_.largest_free_bytes();
}

// ---------------------------------------------------------------------------
// TinyLFU
// ---------------------------------------------------------------------------

TinyLfu::TinyLfu(uint64_t cache_size) : window_limit_(cache_size * 8) {
  // Estimator::optimal_paras (cache.rs:105-122)
  const double items = static_cast<double>(cache_size);
  const double err = 1.0 / items;
  const double fail = 1.0 / items;
  slots_ = std::max<uint64_t>(static_cast<uint64_t>(std::ceil(M_E / err)), 16);
  const uint64_t hashes = std::max<uint64_t>(static_cast<uint64_t>(std::ceil(std::log(fail) / std::log(0.5))), 2);
  rows_.resize(hashes);
  for (auto& r : rows_) {
    std::vector<std::atomic<uint8_t>> v(slots_);
    for (auto& c : v) c.store(0, std::memory_order_relaxed);
    r.swap(v);
  }
}

uint8_t TinyLfu::get(const BlockKey& k) const {
  const uint64_t h = fnv1a(k.ns, k.hash);
  uint8_t m = 255;
  for (size_t r = 0; r < rows_.size(); ++r) {
    const uint64_t idx = splitmix64(h ^ (0x51ed2701ull * (r + 1))) % slots_;
    m = std::min<uint8_t>(m, rows_[r][idx].load(std::memory_order_relaxed));
  }
  return m;
}

uint8_t TinyLfu::incr(const BlockKey& k) {
  // TinyLfu::incr (cache.rs:217-224): age every window_limit increments.
  const uint64_t w = window_.fetch_add(1, std::memory_order_relaxed);
  if (w == window_limit_ || w > window_limit_ * 2) {
    window_.store(0, std::memory_order_relaxed);
    age();
  }
  const uint64_t h = fnv1a(k.ns, k.hash);
  uint8_t m = 255;
  for (size_t r = 0; r < rows_.size(); ++r) {
    const uint64_t idx = splitmix64(h ^ (0x51ed2701ull * (r + 1))) % slots_;
    auto& c = rows_[r][idx];
    uint8_t cur = c.load(std::memory_order_relaxed);
    uint8_t nv = cur;
    while (cur != 255) {  // saturating increment (cache.rs:185-204)
      nv = static_cast<uint8_t>(cur + 1);
      if (c.compare_exchange_weak(cur, nv, std::memory_order_acquire, std::memory_order_relaxed)) break;
      nv = cur;
    }
    if (cur == 255) nv = 255;
    m = std::min(m, nv);
  }
  return m;
}

void TinyLfu::age() {
  for (auto& r : rows_) {
    for (auto& c : r) c.store(static_cast<uint8_t>(c.load(std::memory_order_relaxed) >> 1), std::memory_order_relaxed);
  }
}

// ---------------------------------------------------------------------------
// Storage
// ---------------------------------------------------------------------------

Storage::Storage(std::shared_ptr<PinnedPool> pool, const StorageConfig& cfg)
    : Storage(std::vector<std::shared_ptr<PinnedPool>>{std::move(pool)}, cfg) {}

Storage::Storage(std::vector<std::shared_ptr<PinnedPool>> pools, const StorageConfig& cfg)
    : pools_(std::move(pools)), cfg_(cfg) {
  if (pools_.empty() || std::any_of(pools_.begin(), pools_.end(), [](const auto& p) { return !p; })) {
    throw invalid_argument("storage needs at least one pool");
  }
  if (cfg_.enable_lfu_admission) {
    const uint64_t per_value = cfg_.hint_value_size_bytes ? cfg_.hint_value_size_bytes : kDefaultBytesPerValue;
    const uint64_t items = std::max<uint64_t>(1, cfg_.capacity_bytes / per_value);  // cache.rs:39-42
    lfu_ = std::make_unique<TinyLfu>(items);
  }
  if (cfg_.pre_evict_enabled) pre_evict_ = std::thread([this] { pre_evict_loop(); });
}

Storage::~Storage() {
  {
    std::lock_guard<std::mutex> g(stop_mu_);
    stop_ = true;
  }
  stop_cv_.notify_all();
  if (pre_evict_.joinable()) pre_evict_.join();
}

std::shared_ptr<PoolAllocation> Storage::allocate(uint64_t size, size_t pool) {
  // The allocator succeeds exactly when its largest-free report covers the
  // request, so the retry below is taken at most once per reclaim that freed
  // something; a retry that frees nothing ends the loop (the reference would
  // spin if the allocator ran out of nodes). One exception: when concurrent
  // saves reclaim at once, another thread may hold the last evicted blocks
  // (taken from the LRU list, not yet dropped), so this thread finds nothing
  // to evict although their memory is about to come back. It waits for those
  // drops and tries again, at most kMaxDropWaits times within one second.
  pool = std::min(pool, pools_.size() - 1);
  PinnedPool& p = *pools_[pool];
  std::chrono::steady_clock::time_point deadline{};
  for (int waits = 0;;) {
    if (auto a = p.allocate(size)) return a;
    uint64_t freed = 0;
    reclaim_until_fits(size, pool, &freed);
    if (p.largest_free() >= size && freed > 0) continue;
    if (p.largest_free() >= size) {
      if (auto a = p.allocate(size)) return a;
    }
    if (waits == 0) deadline = std::chrono::steady_clock::now() + std::chrono::seconds(1);
    if (waits < kMaxDropWaits && wait_for_drops(p, size, deadline)) {
      ++waits;
      continue;
    }
    counters_.pool_alloc_failures.fetch_add(1);
    return nullptr;
  }
}

bool Storage::wait_for_drops(PinnedPool& p, uint64_t size, std::chrono::steady_clock::time_point deadline) {
  // Drops take microseconds to milliseconds.
  if (dropping_.load(std::memory_order_acquire) == 0) return false;
  while (dropping_.load(std::memory_order_acquire) != 0 && p.largest_free() < size) {
    if (std::chrono::steady_clock::now() > deadline) return false;
    std::this_thread::yield();
  }
  return true;
}

void Storage::drop_evicted(std::vector<SealedBlockPtr>& evicted) {
  if (evicted.empty()) return;
  evicted.clear();  // frees pool memory whose last holder this was
  dropping_.fetch_sub(1, std::memory_order_acq_rel);
}

bool Storage::holds_memory_in(const SealedBlock& b, size_t pool) const {
  // A slot's K and V come from one save call on one device, so one pool.
  const PinnedPool& p = *pools_[pool];
  for (const LayerBlock* s : b.slots) {
    if (s && p.contains(s->k_ptr)) return true;
  }
  return false;
}

std::vector<SealedBlockPtr> Storage::evict_lru(uint64_t max_blocks, uint64_t bytes, size_t pool) {
  std::vector<SealedBlockPtr> out;
  const bool any = pools_.size() == 1;
  uint64_t freed = 0;
  std::lock_guard<std::mutex> g(cache_mu_);
  for (auto it = lru_.begin(); it != lru_.end() && out.size() < max_blocks && freed < bytes;) {
    if (!any && !holds_memory_in(*it->second, pool)) {
      ++it;
      continue;
    }
    freed += it->second->footprint;
    out.push_back(std::move(it->second));
    index_.erase(it->first);
    it = lru_.erase(it);
  }
  // Dropped by the caller outside the cache lock, with drop_evicted; until
  // then dropping_ tells other reclaiming threads that memory is on its way.
  if (!out.empty()) dropping_.fetch_add(1, std::memory_order_acq_rel);
  return out;
}

void Storage::reclaim_until_fits(uint64_t required, size_t pool, uint64_t* freed_blocks) {
  // reclaim_until_allocator_can_allocate (storage.rs:565-608)
  *freed_blocks = 0;
  if (required == 0) return;
  while (pools_[pool]->largest_free() < required) {
    std::vector<SealedBlockPtr> evicted = evict_lru(kReclaimBatch, UINT64_MAX, pool);
    if (evicted.empty()) break;
    *freed_blocks += evicted.size();
    counters_.evictions.fetch_add(evicted.size());
    drop_evicted(evicted);
  }
}

void Storage::usage(uint64_t* used, uint64_t* total) {
  uint64_t u = 0, t = 0;
  for (const auto& p : pools_) {
    uint64_t pu = 0, pt = 0;
    p->usage(&pu, &pt);
    u += pu;
    t += pt;
  }
  *used = u;
  *total = t;
}

uint64_t Storage::largest_free() {
  uint64_t m = 0;
  for (const auto& p : pools_) m = std::max(m, p->largest_free());
  return m;
}

void Storage::pre_evict_loop() {
  // pre_evict_monitor (storage.rs:646-686). With several pools each keeps
  // its share (by size) of the threshold and target free.
  std::unique_lock<std::mutex> lk(stop_mu_);
  while (!stop_) {
    stop_cv_.wait_for(lk, std::chrono::milliseconds(cfg_.pre_evict_interval_ms));
    if (stop_) break;
    lk.unlock();
    uint64_t all_used = 0, all_total = 0;
    usage(&all_used, &all_total);
    for (size_t i = 0; i < pools_.size(); ++i) {
      uint64_t used = 0, total = 0;
      pools_[i]->usage(&used, &total);
      uint64_t threshold = cfg_.pre_evict_threshold_bytes, target = cfg_.pre_evict_target_bytes;
      if (pools_.size() > 1 && all_total > 0) {
        const double share = static_cast<double>(total) / static_cast<double>(all_total);
        threshold = static_cast<uint64_t>(static_cast<double>(threshold) * share);
        target = static_cast<uint64_t>(static_cast<double>(target) * share);
      }
      const uint64_t free_bytes = total > used ? total - used : 0;
      if (free_bytes < threshold) {
        const uint64_t need = target > free_bytes ? target - free_bytes : 0;
        std::vector<SealedBlockPtr> evicted = evict_lru(UINT64_MAX, need, i);
        counters_.evictions.fetch_add(evicted.size());
        drop_evicted(evicted);
      }
    }
    lk.lock();
  }
}

Storage::InflightIt Storage::inflight_add(InflightShard& sh, const BlockKey& key, uint64_t total_slots) {
  Inflight fresh;
  fresh.slots.assign(total_slots, nullptr);
  fresh.remaining = total_slots;
  fresh.total_slots = total_slots;
  auto it = sh.map.emplace(key, std::move(fresh)).first;
  if (++sh.totals[total_slots] == 1) sh.summarize();
  inflight_blocks_.fetch_add(1, std::memory_order_relaxed);
  return it;
}

Storage::InflightIt Storage::inflight_remove(InflightShard& sh, InflightIt it) {
  auto t = sh.totals.find(it->second.total_slots);
  if (t != sh.totals.end() && --t->second == 0) {
    sh.totals.erase(t);
    sh.summarize();
  }
  inflight_blocks_.fetch_sub(1, std::memory_order_relaxed);
  return sh.map.erase(it);
}

bool Storage::inflight_has_slot(const std::string& ns, const std::string& hash, uint64_t slot) {
  const BlockKey key{ns, hash};
  InflightShard& sh = shard(key);
  std::lock_guard<std::mutex> g(sh.mu);
  auto it = sh.map.find(key);
  if (it == sh.map.end()) return false;
  return slot < it->second.slots.size() && it->second.slots[slot] != nullptr;
}

void Storage::insert_slots(const std::string& ns, const std::vector<std::string>& hashes, uint64_t slot,
                           std::vector<LayerBlockPtr>& blocks, uint64_t total_slots) {
  // Same per-block steps as insert_slot (storage.rs:457-514), with the cache
  // lock taken once for the whole list; each block takes its shard's lock.
  maybe_drop_stale_inflight();
  std::vector<std::pair<BlockKey, SealedBlockPtr>> sealed;
  {
    std::vector<char> cached(hashes.size(), 0);
    {
      std::lock_guard<std::mutex> gc(cache_mu_);
      BlockKey probe{ns, std::string()};
      for (size_t i = 0; i < hashes.size(); ++i) {
        probe.hash = hashes[i];
        cached[i] = index_.count(probe) ? 1 : 0;
      }
    }
    std::unordered_map<std::string, bool> sealed_here;  // a repeated hash finds its block sealed
    for (size_t i = 0; i < hashes.size(); ++i) {
      if (cached[i]) continue;
      if (!sealed.empty() && sealed_here.count(hashes[i])) continue;
      BlockKey key{ns, hashes[i]};
      InflightShard& sh = shard(key);
      std::lock_guard<std::mutex> gi(sh.mu);
      auto it = sh.map.find(key);
      if (it == sh.map.end()) {
        it = inflight_add(sh, key, total_slots);
      }
      Inflight& ib = it->second;
      if (slot < ib.slots.size() && ib.slots[slot]) continue;
      if (total_slots != ib.total_slots) {
        throw storage_error("slot count mismatch: expected " + std::to_string(ib.total_slots) + ", got " +
                            std::to_string(total_slots));
      }
      if (slot >= ib.total_slots) {
        throw storage_error("slot_id " + std::to_string(slot) + " out of bounds (" +
                            std::to_string(ib.total_slots) + " slots)");
      }
      ib.footprint += blocks[i]->size;
      ib.slots[slot] = blocks[i].get();
      ib.owners.push_back(std::move(blocks[i]));
      ib.remaining -= 1;
      if (ib.remaining == 0) {
        auto sb = std::make_shared<SealedBlock>();
        sb->slots = std::move(ib.slots);
        sb->owners = std::move(ib.owners);
        sb->footprint = ib.footprint;
        inflight_remove(sh, it);
        sealed_here[key.hash] = true;
        sealed.emplace_back(std::move(key), std::move(sb));
      }
    }
  }
  if (!sealed.empty()) {
    for (const auto& kv : sealed) notify_sealed(kv.first, kv.second);
    std::lock_guard<std::mutex> g(cache_mu_);
    for (auto& kv : sealed) {
      if (cache_insert_locked(kv.first, std::move(kv.second))) {
        counters_.insertions.fetch_add(1);
      } else {
        counters_.admission_rejections.fetch_add(1);
      }
    }
  }
}

void Storage::probe_save(const std::string& ns, const std::vector<std::string>& hashes, SaveProbe* out) {
  const size_t n = hashes.size();
  out->cached.assign(n, 0);
  out->filled.assign(n, std::vector<char>());
  BlockKey key{ns, std::string()};
  {
    std::lock_guard<std::mutex> g(cache_mu_);
    for (size_t i = 0; i < n; ++i) {
      key.hash = hashes[i];
      if (index_.count(key)) out->cached[i] = 1;
    }
  }
  if (inflight_blocks_.load(std::memory_order_relaxed) == 0) return;
  for (size_t i = 0; i < n; ++i) {
    if (out->cached[i]) continue;
    key.hash = hashes[i];
    InflightShard& sh = shard(key);
    std::lock_guard<std::mutex> g(sh.mu);
    auto it = sh.map.find(key);
    if (it == sh.map.end()) continue;
    const std::vector<const LayerBlock*>& slots = it->second.slots;
    std::vector<char>& f = out->filled[i];
    f.resize(slots.size());
    for (size_t s = 0; s < slots.size(); ++s) f[s] = slots[s] ? 1 : 0;
  }
}

void Storage::insert_slots_multi(const std::string& ns, const std::vector<std::string>& hashes,
                                 const std::vector<SlotFill>& fills, uint64_t total_slots) {
  // Hash-major form of calling insert_slots once per fill (fill-major). Per
  // hash the fills are applied in order until the block seals; the sealed
  // blocks then enter the cache in fill-major order (by the fill that sealed
  // them, then by position), so LRU order and TinyLFU decisions match. A
  // block that admission refuses is gone from the cache and from inflight,
  // so fill-major would start a new inflight block from the later fills: the
  // second pass below does that. That new block cannot seal in this call: it
  // gets at most fills-1 < total_slots slots.
  //
  // The hashes are visited shard by shard, one shard lock at a time. The
  // saves of a block's TP ranks start at different shards (rank r of t at
  // shard r*64/t), so they sweep the shards side by side instead of queueing
  // on one lock.
  const size_t n = hashes.size();
  if (fills.empty() || n == 0) return;
  maybe_drop_stale_inflight();
  auto per_fill = [&] {
    for (const SlotFill& f : fills) {
      std::vector<LayerBlockPtr> blocks(n);
      for (size_t i = 0; i < n; ++i) blocks[i] = layer_block_at(f.batch, i);
      insert_slots(ns, hashes, f.slot, blocks, total_slots);
    }
  };
  {
    std::vector<char> seen(total_slots, 0);
    for (const SlotFill& f : fills) {
      if (f.slot >= total_slots || f.batch->blocks.size() != n || seen[f.slot]) return per_fill();
      seen[f.slot] = 1;
    }
  }
  std::vector<char> cached(n, 0);
  std::vector<BlockKey> keys;
  std::vector<uint64_t> key_hash(n);
  keys.reserve(n);
  for (size_t i = 0; i < n; ++i) {
    keys.push_back(BlockKey{ns, hashes[i]});
    key_hash[i] = BlockKeyHash{}(keys.back());
  }
  // A hash listed twice finds its block sealed by the first occurrence; only
  // a list with a repeat needs the set of hashes sealed so far. Equal keys
  // hash equally, so comparing the 64-bit hashes misses no repeat (a
  // collision only turns the set on).
  bool repeats = false;
  {
    std::vector<uint64_t> sorted(key_hash);
    std::sort(sorted.begin(), sorted.end());
    repeats = std::adjacent_find(sorted.begin(), sorted.end()) != sorted.end();
  }
  {
    std::lock_guard<std::mutex> g(cache_mu_);
    for (size_t i = 0; i < n; ++i) cached[i] = index_.count(keys[i]) ? 1 : 0;
  }
  std::vector<std::vector<uint32_t>> by_shard(kInflightShards);  // positions, in list order
  for (size_t i = 0; i < n; ++i) {
    if (!cached[i]) by_shard[shard_of_hash(key_hash[i])].push_back(static_cast<uint32_t>(i));
  }
  // An inflight block with another slot count makes fill-major throw part
  // way through its first fill; let it do exactly that. (A snapshot: such a
  // block created after this check meets the throw in the main pass.)
  if (inflight_blocks_.load(std::memory_order_relaxed) != 0) {
    bool mismatch = false;
    for (size_t sh_i = 0; sh_i < kInflightShards && !mismatch; ++sh_i) {
      if (by_shard[sh_i].empty()) continue;
      InflightShard& sh = inflight_[sh_i];
      const uint64_t sole = sh.sole_total.load(std::memory_order_acquire);
      if (sole == 0 || sole == total_slots) continue;  // every entry here has this call's slot count
      std::lock_guard<std::mutex> g(sh.mu);
      for (uint32_t i : by_shard[sh_i]) {
        auto it = sh.map.find(keys[i]);
        if (it != sh.map.end() && it->second.total_slots != total_slots) {
          mismatch = true;
          break;
        }
      }
    }
    if (mismatch) return per_fill();
  }
  struct Seal {
    size_t fill;
    size_t index;
    BlockKey key;
    SealedBlockPtr block;
  };
  std::vector<Seal> seals;
  seals.reserve(n);
  std::unordered_set<std::string_view> sealed_here;  // a repeated hash finds its block sealed
  if (repeats) sealed_here.reserve(n);
  // One owner for the batches of every fill: each block this call touches
  // holds it once (instead of one reference per slot).
  SlotOwner owner;
  {
    auto group = std::make_shared<std::vector<std::shared_ptr<LayerBlockBatch>>>();
    group->reserve(fills.size());
    for (const SlotFill& f : fills) group->push_back(f.batch);
    owner = std::move(group);
  }
  // Every slot filled by this call: a hash with no inflight block seals at
  // the last fill, so its block is built directly, without an inflight
  // entry that would be created and erased at once.
  const bool all_slots = fills.size() == total_slots;
  size_t start = 0;
  if (total_slots % fills.size() == 0) {
    const uint64_t tp = total_slots / fills.size();
    start = static_cast<size_t>((fills.front().slot % tp) * kInflightShards / tp);
  }
  // A block created with another slot count after the check above stops the
  // pass (fill-major would throw there); what sealed before it is still
  // published below, then the call throws.
  std::string mismatch;
  for (size_t step = 0; step < kInflightShards && mismatch.empty(); ++step) {
    const size_t sh_i = (start + step) % kInflightShards;
    if (by_shard[sh_i].empty()) continue;
    InflightShard& sh = inflight_[sh_i];
    std::lock_guard<std::mutex> g(sh.mu);
    for (uint32_t i : by_shard[sh_i]) {
      if (repeats && !sealed_here.empty() && sealed_here.count(hashes[i])) continue;
      const BlockKey& key = keys[i];
      auto it = sh.map.find(key);
      if (it == sh.map.end() && all_slots) {
        auto sb = std::make_shared<SealedBlock>();
        sb->slots.resize(total_slots);
        for (const SlotFill& f : fills) {
          sb->footprint += f.batch->blocks[i].size;
          sb->slots[f.slot] = &f.batch->blocks[i];
        }
        sb->owners.push_back(owner);
        if (repeats) sealed_here.insert(hashes[i]);
        seals.push_back({fills.size() - 1, i, key, std::move(sb)});
        continue;
      }
      if (it == sh.map.end()) {
        it = inflight_add(sh, key, total_slots);
      }
      Inflight& ib = it->second;
      if (ib.total_slots != total_slots) {
        mismatch = "slot count mismatch: expected " + std::to_string(ib.total_slots) + ", got " +
                   std::to_string(total_slots);
        break;
      }
      bool owned = false;
      for (size_t f = 0; f < fills.size(); ++f) {
        const uint64_t slot = fills[f].slot;
        if (ib.slots[slot]) continue;
        if (!owned) {
          ib.owners.push_back(owner);
          owned = true;
        }
        ib.footprint += fills[f].batch->blocks[i].size;
        ib.slots[slot] = &fills[f].batch->blocks[i];
        if (--ib.remaining == 0) {
          auto sb = std::make_shared<SealedBlock>();
          sb->slots = std::move(ib.slots);
          sb->owners = std::move(ib.owners);
          sb->footprint = ib.footprint;
          inflight_remove(sh, it);
          if (repeats) sealed_here.insert(hashes[i]);
          seals.push_back({f, i, key, std::move(sb)});
          break;
        }
      }
    }
  }
  if (seals.empty()) {
    if (!mismatch.empty()) throw storage_error(mismatch);
    return;
  }
  auto fill_major = [](const Seal& a, const Seal& b) { return a.fill != b.fill ? a.fill < b.fill : a.index < b.index; };
  if (!std::is_sorted(seals.begin(), seals.end(), fill_major)) std::sort(seals.begin(), seals.end(), fill_major);
  SealListener listener;
  {
    std::lock_guard<std::mutex> g(listener_mu_);
    listener = seal_listener_;
  }
  if (listener) {
    for (const Seal& s : seals) listener(s.key, s.block);
  }
  std::vector<const Seal*> refused;
  uint64_t inserted = 0, rejected = 0;
  {
    std::lock_guard<std::mutex> g(cache_mu_);
    for (Seal& s : seals) {
      // The key stays with the seal: a refused block restarts inflight below.
      if (cache_insert_locked(s.key, std::move(s.block))) {
        ++inserted;
      } else {
        ++rejected;
        if (s.fill + 1 < fills.size()) refused.push_back(&s);
      }
    }
  }
  counters_.insertions.fetch_add(inserted);
  counters_.admission_rejections.fetch_add(rejected);
  for (const Seal* s : refused) {
    InflightShard& sh = shard(s->key);
    std::lock_guard<std::mutex> g(sh.mu);
    auto it = sh.map.find(s->key);
    if (it == sh.map.end()) {
      it = inflight_add(sh, s->key, total_slots);
    }
    Inflight& ib = it->second;
    if (ib.total_slots != total_slots) continue;  // another call's block: fill-major would have thrown
    bool owned = false;
    for (size_t f = s->fill + 1; f < fills.size(); ++f) {
      const uint64_t slot = fills[f].slot;
      if (ib.slots[slot]) continue;
      if (!owned) {
        ib.owners.push_back(owner);
        owned = true;
      }
      ib.footprint += fills[f].batch->blocks[s->index].size;
      ib.slots[slot] = &fills[f].batch->blocks[s->index];
      --ib.remaining;
    }
  }
  if (!mismatch.empty()) throw storage_error(mismatch);
}

bool Storage::cache_insert_locked(const BlockKey& key, SealedBlockPtr block) {
  // TinyLfuCache::insert (cache.rs:66-90)
  if (lfu_) lfu_->incr(key);
  auto it = index_.find(key);
  if (it != index_.end()) {
    it->second->second = std::move(block);
    lru_.splice(lru_.end(), lru_, it->second);
    return true;
  }
  if (lfu_ && !lru_.empty()) {
    if (lfu_->get(key) < lfu_->get(lru_.front().first)) return false;
  }
  lru_.emplace_back(key, std::move(block));
  index_.emplace_hint(it, lru_.back().first, std::prev(lru_.end()));
  return true;
}

bool Storage::insert_slot(const std::string& ns, const std::string& hash, uint64_t slot, LayerBlockPtr block,
                          uint64_t total_slots) {
  maybe_drop_stale_inflight();
  BlockKey key{ns, hash};
  {
    std::lock_guard<std::mutex> g(cache_mu_);
    if (index_.count(key)) return false;
  }
  SealedBlockPtr sealed;
  {
    InflightShard& sh = shard(key);
    std::lock_guard<std::mutex> g(sh.mu);
    auto it = sh.map.find(key);
    if (it == sh.map.end()) {
      it = inflight_add(sh, key, total_slots);
    }
    Inflight& ib = it->second;
    if (slot < ib.slots.size() && ib.slots[slot]) return false;
    // InflightBlock::insert_slot (storage.rs:161-193)
    if (total_slots != ib.total_slots) {
      throw storage_error("slot count mismatch: expected " + std::to_string(ib.total_slots) + ", got " +
                          std::to_string(total_slots));
    }
    if (slot >= ib.total_slots) {
      throw storage_error("slot_id " + std::to_string(slot) + " out of bounds (" + std::to_string(ib.total_slots) +
                          " slots)");
    }
    ib.footprint += block->size;
    ib.slots[slot] = block.get();
    ib.owners.push_back(std::move(block));
    ib.remaining -= 1;
    if (ib.remaining == 0) {
      sealed = std::make_shared<SealedBlock>();
      sealed->slots = std::move(ib.slots);
      sealed->owners = std::move(ib.owners);
      sealed->footprint = ib.footprint;
      inflight_remove(sh, it);
    }
  }
  if (sealed) {
    notify_sealed(key, sealed);
    std::lock_guard<std::mutex> g(cache_mu_);
    if (cache_insert_locked(key, std::move(sealed))) {
      counters_.insertions.fetch_add(1);
    } else {
      counters_.admission_rejections.fetch_add(1);
    }
  }
  return true;
}

void Storage::set_seal_listener(SealListener fn) {
  std::lock_guard<std::mutex> g(listener_mu_);
  seal_listener_ = std::move(fn);
}

void Storage::notify_sealed(const BlockKey& key, const SealedBlockPtr& block) {
  SealListener fn;
  {
    std::lock_guard<std::mutex> g(listener_mu_);
    fn = seal_listener_;
  }
  if (fn) fn(key, block);
}

bool Storage::cache_insert(const std::string& ns, const std::string& hash, SealedBlockPtr block) {
  std::lock_guard<std::mutex> g(cache_mu_);
  const bool ok = cache_insert_locked(BlockKey{ns, hash}, std::move(block));
  if (ok) {
    counters_.insertions.fetch_add(1);
  } else {
    counters_.admission_rejections.fetch_add(1);
  }
  return ok;
}

bool Storage::cache_contains(const std::string& ns, const std::string& hash) {
  std::lock_guard<std::mutex> g(cache_mu_);
  return index_.count(BlockKey{ns, hash}) != 0;
}

std::vector<SealedBlockPtr> Storage::cache_lookup_many(const std::string& ns, const std::vector<std::string>& hashes) {
  std::vector<SealedBlockPtr> out;
  out.reserve(hashes.size());
  std::lock_guard<std::mutex> g(cache_mu_);
  for (size_t i = 0; i < hashes.size(); ++i) {
    BlockKey key{ns, hashes[i]};
    auto it = index_.find(key);
    if (it == index_.end()) {
      throw storage_error("missing KV block hash at index " + std::to_string(i) + " (namespace=" + ns +
                          ", hash_len=" + std::to_string(hashes[i].size()) + ")");
    }
    lru_.splice(lru_.end(), lru_, it->second);  // LruCache::get moves to MRU
    if (lfu_) lfu_->incr(key);
    out.push_back(it->second->second);
  }
  return out;
}

SealedBlockPtr Storage::cache_peek(const std::string& ns, const std::string& hash) {
  std::lock_guard<std::mutex> g(cache_mu_);
  auto it = index_.find(BlockKey{ns, hash});
  return it == index_.end() ? nullptr : it->second->second;
}

uint64_t Storage::inflight_count() { return inflight_blocks_.load(std::memory_order_relaxed); }

uint64_t Storage::drop_stale_inflight() {
  if (cfg_.inflight_max_age_ms == 0) return 0;
  const auto now = std::chrono::steady_clock::now();
  const auto max_age = std::chrono::milliseconds(cfg_.inflight_max_age_ms);
  std::vector<Inflight> dropped;  // their pool memory is released after the lock
  for (InflightShard& sh : inflight_) {
    std::lock_guard<std::mutex> g(sh.mu);
    for (auto it = sh.map.begin(); it != sh.map.end();) {
      if (now - it->second.created > max_age) {
        dropped.push_back(std::move(it->second));
        it = inflight_remove(sh, it);
      } else {
        ++it;
      }
    }
  }
  counters_.inflight_dropped.fetch_add(dropped.size());
  return dropped.size();
}

void Storage::maybe_drop_stale_inflight() {
  if (cfg_.inflight_max_age_ms == 0) return;
  const int64_t now = std::chrono::duration_cast<std::chrono::nanoseconds>(
                          std::chrono::steady_clock::now().time_since_epoch())
                          .count();
  const int64_t every = std::min<int64_t>(60'000'000'000ll, int64_t(cfg_.inflight_max_age_ms) * 250'000);
  int64_t last = last_sweep_ns_.load(std::memory_order_relaxed);
  if (now - last < every) return;
  if (!last_sweep_ns_.compare_exchange_strong(last, now)) return;  // another save sweeps
  drop_stale_inflight();
}

uint64_t Storage::cached_count() {
  std::lock_guard<std::mutex> g(cache_mu_);
  return lru_.size();
}

Storage::BlockView Storage::cache_view() {
  std::lock_guard<std::mutex> g(cache_mu_);
  BlockView out;
  out.reserve(lru_.size());
  for (const auto& kv : lru_) out.emplace_back(kv.first.ns + '\0' + kv.first.hash, kv.second->slots);
  return out;
}

Storage::BlockView Storage::inflight_view() {
  BlockView out;
  for (InflightShard& sh : inflight_) {
    std::lock_guard<std::mutex> g(sh.mu);
    for (const auto& kv : sh.map) {
      out.emplace_back(kv.first.ns + '\0' + kv.first.hash, kv.second.slots);
    }
  }
  std::sort(out.begin(), out.end());
  return out;
}

}  // namespace pf
