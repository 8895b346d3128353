// Storage releases inflight blocks whose missing slots never arrive, and
// only those. Such a block appears when a per-layer save skips a block that
// is cached, the block is evicted, and the next layer's save starts a fresh
// inflight block that lacks the skipped slot (pegaflow-core/src/lib.rs:604-611).
//
// Build and run (tests/test_storage_gc.py does this):
//   g++ -O1 -std=c++17 -I<repo>/include -I<repo>/pegaflow_b200/csrc -I<cuda>/include
//       tests/storage_gc.cpp <csrc>/storage.cpp <csrc>/offset_allocator.cpp
//       <csrc>/pinned.cpp -L<cuda>/lib64 -lcudart_static -ldl -lrt -lpthread
//   ./storage_gc
#include <chrono>
#include <cstdio>
#include <memory>
#include <thread>

#include "storage.h"

using namespace pf;

#define CHECK(c)                                                       \
  do {                                                                 \
    if (!(c)) {                                                        \
      std::printf("FAIL line %d: %s\n", __LINE__, #c);                 \
      return 1;                                                        \
    }                                                                  \
  } while (0)

namespace {

constexpr uint64_t kBlock = 4096;

// One block of `kBlock` bytes in its own pool allocation.
LayerBlockPtr block_from(const std::shared_ptr<PinnedPool>& pool) {
  auto b = std::make_shared<LayerBlockBatch>();
  b->k_alloc = pool->allocate(kBlock);
  if (!b->k_alloc) return nullptr;
  b->blocks.push_back(LayerBlock{b->k_alloc->ptr, nullptr, kBlock});
  return layer_block_at(b, 0);
}

uint64_t used(const std::shared_ptr<PinnedPool>& pool) {
  uint64_t u = 0, t = 0;
  pool->usage(&u, &t);
  return u;
}

}  // namespace

int main() {
  auto pool = PinnedPool::create(8 << 20, PinKind::kPlainHost, false, 0);
  StorageConfig cfg;
  cfg.enable_lfu_admission = false;
  cfg.capacity_bytes = 8 << 20;
  cfg.inflight_max_age_ms = 200;
  Storage st(pool, cfg);
  const uint64_t used0 = used(pool);

  // "a" gets slot 1 of 2 and nothing else: it can never seal.
  st.insert_slot("ns", "a", 1, block_from(pool), 2);
  CHECK(st.inflight_count() == 1);
  CHECK(used(pool) == used0 + kBlock);
  CHECK(st.drop_stale_inflight() == 0);  // young blocks stay

  std::this_thread::sleep_for(std::chrono::milliseconds(300));
  // The next save sweeps on its own: "a" is older than the limit, "b" new.
  st.insert_slot("ns", "b", 0, block_from(pool), 2);
  CHECK(st.counters().inflight_dropped.load() == 1);
  CHECK(st.inflight_count() == 1);
  CHECK(used(pool) == used0 + kBlock);  // a's memory is back, b holds one block

  // "b" completes normally.
  st.insert_slot("ns", "b", 1, block_from(pool), 2);
  CHECK(st.inflight_count() == 0);
  CHECK(st.cached_count() == 1);
  CHECK(used(pool) == used0 + 2 * kBlock);

  // A dropped hash can be saved again from scratch.
  st.insert_slot("ns", "a", 0, block_from(pool), 2);
  st.insert_slot("ns", "a", 1, block_from(pool), 2);
  CHECK(st.cached_count() == 2);
  CHECK(st.inflight_count() == 0);

  // A limit of 0 keeps inflight blocks forever.
  StorageConfig keep = cfg;
  keep.inflight_max_age_ms = 0;
  Storage st2(pool, keep);
  st2.insert_slot("ns", "c", 1, block_from(pool), 2);
  std::this_thread::sleep_for(std::chrono::milliseconds(250));
  CHECK(st2.drop_stale_inflight() == 0);
  st2.insert_slot("ns", "d", 0, block_from(pool), 2);
  CHECK(st2.inflight_count() == 2);
  CHECK(st2.counters().inflight_dropped.load() == 0);

  std::printf("ok\n");
  return 0;
}
