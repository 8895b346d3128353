// Storage over several pools (one per NUMA node): an allocation comes from
// the pool it names, reclaim for a pool evicts only cached blocks that hold
// memory in that pool (in LRU order, the other pools' blocks stay), usage
// sums the pools, and a pool placed on a node has its pages there.
//
// Build and run (tests/test_storage_pools.py does this):
//   g++ -O1 -std=c++17 -I<repo>/include -I<repo>/pegaflow_b200/csrc -I<cuda>/include
//       tests/storage_pools.cpp <csrc>/storage.cpp <csrc>/offset_allocator.cpp
//       <csrc>/pinned.cpp -L<cuda>/lib64 -lcudart_static -ldl -lrt -lpthread
//   ./storage_pools
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "storage.h"

using namespace pf;

#define CHECK(c)                                              \
  do {                                                        \
    if (!(c)) {                                               \
      std::printf("FAIL line %d: %s\n", __LINE__, #c);        \
      return 1;                                               \
    }                                                         \
  } while (0)

namespace {

constexpr uint64_t kBlock = 16 << 10;
constexpr uint64_t kPool = 4 * kBlock;

// Seals a one-slot block `hash` whose bytes come from `pool`.
bool seal(Storage& st, const std::string& hash, size_t pool) {
  auto a = st.allocate(kBlock, pool);
  if (!a) return false;
  auto b = std::make_shared<LayerBlockBatch>();
  b->k_alloc = a;
  b->blocks.push_back(LayerBlock{a->ptr, nullptr, kBlock});
  return st.insert_slot("ns", hash, 0, layer_block_at(b, 0), 1);
}

// Cached hashes from least to most recently used (view keys are ns, NUL, hash).
std::vector<std::string> cached(Storage& st) {
  std::vector<std::string> out;
  for (auto& kv : st.cache_view()) out.push_back(kv.first.substr(kv.first.find('\0') + 1));
  return out;
}

}  // namespace

int main() {
  // ---- routing and per-pool reclaim -----------------------------------
  {
    auto a = PinnedPool::create(kPool, PinKind::kPlainHost, false, 0);
    auto b = PinnedPool::create(kPool, PinKind::kPlainHost, false, 0);
    StorageConfig cfg;
    cfg.enable_lfu_admission = false;
    cfg.capacity_bytes = 2 * kPool;
    Storage st({a, b}, cfg);
    CHECK(st.pool_count() == 2);

    // LRU order a0 b0 a1 b1 a2 b2 a3 b3; each pool is then full.
    for (int i = 0; i < 4; ++i) {
      CHECK(seal(st, "a" + std::to_string(i), 0));
      CHECK(seal(st, "b" + std::to_string(i), 1));
    }
    uint64_t used = 0, total = 0;
    st.usage(&used, &total);
    CHECK(used == 2 * kPool && total == 2 * kPool);
    CHECK(st.largest_free() == 0);

    // A new block for pool 1 evicts pool 1's blocks only (one reclaim batch
    // takes every pool-1 block in LRU order), never pool 0's.
    CHECK(seal(st, "b4", 1));
    CHECK((cached(st) == std::vector<std::string>{"a0", "a1", "a2", "a3", "b4"}));
    CHECK(st.counters().evictions.load() == 4);

    // Pool 0 is still full; its next block evicts a0..a3, and b4 stays.
    CHECK(seal(st, "a4", 0));
    CHECK((cached(st) == std::vector<std::string>{"b4", "a4"}));

    // An out-of-range pool index uses the last pool.
    auto x = st.allocate(kBlock, 7);
    CHECK(x && b->contains(x->ptr));
  }

  // ---- one pool: reclaim evicts from the LRU front, as before ----------
  {
    auto p = PinnedPool::create(kPool, PinKind::kPlainHost, false, 0);
    StorageConfig cfg;
    cfg.enable_lfu_admission = false;
    cfg.capacity_bytes = kPool;
    Storage st(p, cfg);
    for (int i = 0; i < 4; ++i) CHECK(seal(st, "c" + std::to_string(i), 0));
    CHECK(seal(st, "c4", 0));
    CHECK((cached(st) == std::vector<std::string>{"c4"}));  // the whole batch went
  }

  // ---- placement --------------------------------------------------------
  {
    auto p = PinnedPool::create(kPool, PinKind::kPlainHost, false, 0, /*numa_node=*/0);
    const PinnedMemory& m = p->memory();
    CHECK(m.numa_node() == 0);
    std::memset(p->base(), 1, kPool);  // fault the pages in
    if (m.numa_bound()) {
      const int node = numa_node_of(p->base());
      CHECK(node == 0 || node == -1);  // -1: get_mempolicy refused here
      std::printf("placed on node %d\n", node);
    } else {
      std::printf("mbind refused here; placement not checked\n");
    }
    auto a = p->allocate(kBlock);
    CHECK(a && p->contains(a->ptr));
  }

  std::printf("ok\n");
  return 0;
}
