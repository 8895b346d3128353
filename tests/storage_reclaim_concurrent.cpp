// Concurrent TP saves into one Storage whose pool holds two steps: every
// step, `tp` threads (one per rank) each allocate their K and V regions for
// every layer, which evicts the previous step's blocks, then insert their
// slots (slot = layer * tp + rank) for the same hash list. Checks:
//   - no allocation fails: a thread that finds the LRU list empty while
//     another thread still holds the last evicted blocks must wait for their
//     memory instead of giving up;
//   - every step's blocks are sealed with every slot set, none left inflight;
//   - a sealed block holds one owner per rank (not one per slot), and its
//     slots point into the pool.
//
//   storage_reclaim_concurrent <tp> <steps>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "storage.h"

using namespace pf;

int main(int argc, char** argv) {
  const int tp = argc > 1 ? std::atoi(argv[1]) : 4;
  const int steps = argc > 2 ? std::atoi(argv[2]) : 10;
  const int layers = 80, n = 2048;
  const uint64_t seg = 1024;  // K and V bytes per block and layer; sizes do not change the bookkeeping
  const uint64_t per_rank = uint64_t(layers) * 2 * n * seg;
  auto pool = PinnedPool::create(2 * tp * per_rank + (64ull << 20), PinKind::kPlainHost, false, 0);
  StorageConfig cfg;
  cfg.enable_lfu_admission = false;
  cfg.capacity_bytes = 1ull << 40;
  Storage st(pool, cfg);
  const uint64_t total = uint64_t(layers) * tp;
  for (int step = 0; step < steps; ++step) {
    std::vector<std::string> hashes(n);
    for (int i = 0; i < n; ++i) hashes[i] = "s" + std::to_string(step) + "-b" + std::to_string(i);
    std::vector<int> failed(tp, 0);
    std::vector<std::thread> th;
    for (int r = 0; r < tp; ++r) {
      th.emplace_back([&, r] {
        std::vector<SlotFill> fills;
        for (int l = 0; l < layers; ++l) {
          auto k = st.allocate(seg * n, 0), v = st.allocate(seg * n, 0);
          if (!k || !v) {
            failed[r] = 1;
            return;
          }
          auto b = std::make_shared<LayerBlockBatch>();
          b->k_alloc = k;
          b->v_alloc = v;
          b->blocks.resize(n);
          for (int i = 0; i < n; ++i) b->blocks[i] = LayerBlock{k->ptr + i * seg, v->ptr + i * seg, 2 * seg};
          fills.push_back(SlotFill{uint64_t(l) * tp + r, b});
        }
        st.insert_slots_multi("ns", hashes, fills, total);
      });
    }
    for (auto& t : th) t.join();
    for (int r = 0; r < tp; ++r) {
      if (failed[r]) {
        uint64_t used = 0, cap = 0;
        st.usage(&used, &cap);
        std::printf("FAIL step %d rank %d: allocation failed (used %llu of %llu, %llu cached, %llu inflight)\n", step,
                    r, static_cast<unsigned long long>(used), static_cast<unsigned long long>(cap),
                    static_cast<unsigned long long>(st.cached_count()),
                    static_cast<unsigned long long>(st.inflight_count()));
        return 1;
      }
    }
    if (st.inflight_count() != 0) {
      std::printf("FAIL step %d: %llu blocks left inflight\n", step,
                  static_cast<unsigned long long>(st.inflight_count()));
      return 1;
    }
    for (int i = 0; i < n; ++i) {
      SealedBlockPtr sb = st.cache_peek("ns", hashes[i]);
      if (!sb || sb->slots.size() != total || sb->owners.size() != static_cast<size_t>(tp)) {
        std::printf("FAIL step %d: block %d not sealed with %llu slots and %d owners\n", step, i,
                    static_cast<unsigned long long>(total), tp);
        return 1;
      }
      for (const LayerBlock* s : sb->slots) {
        if (!s || !pool->contains(s->k_ptr) || !pool->contains(s->v_ptr)) {
          std::printf("FAIL step %d: block %d has a slot outside the pool\n", step, i);
          return 1;
        }
      }
    }
  }
  std::printf("ok tp=%d steps=%d evictions=%llu\n", tp, steps,
              static_cast<unsigned long long>(st.counters().evictions.load()));
  return 0;
}
