// Property test: Storage::insert_slots_multi (one hash-major pass) leaves
// exactly the state that calling Storage::insert_slots once per fill leaves:
// the same cached blocks in the same LRU order, the same inflight blocks with
// the same slot contents, the same admission counters, and the same error.
// Random pre-states cover sealed, partially inflight and foreign-slot-count
// blocks, repeated hashes, fills in any slot order, and TinyLFU on or off
// (with recency and frequency bumps, so admission refuses some blocks).
//
// Build and run (tests/test_storage_equiv.py does this):
//   g++ -O1 -std=c++17 -I<repo>/include -I<repo>/pegaflow_b200/csrc -I<cuda>/include
//       tests/storage_equiv.cpp <csrc>/storage.cpp <csrc>/offset_allocator.cpp
//       <csrc>/pinned.cpp -L<cuda>/lib64 -lcudart_static -ldl -lrt -lpthread
//   ./storage_equiv <scenarios>
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "storage.h"

using namespace pf;

namespace {

struct Op {  // one pre-state operation, replayed on both stores
  int kind;  // 0 insert_slot, 1 cache_lookup_many
  std::string hash;
  uint64_t slot, total;
  std::vector<std::string> lookups;
};

std::unique_ptr<Storage> make_store(bool lfu) {
  // The stores never allocate here; one pool (its allocator is sized for
  // millions of allocations) serves them all.
  static std::shared_ptr<PinnedPool> pool = PinnedPool::create(1 << 20, PinKind::kPlainHost, false, 0);
  StorageConfig cfg;
  cfg.enable_lfu_admission = lfu;
  cfg.capacity_bytes = 1 << 20;
  return std::make_unique<Storage>(pool, cfg);
}

std::shared_ptr<LayerBlockBatch> make_batch(size_t n) {
  auto b = std::make_shared<LayerBlockBatch>();
  b->blocks.resize(n);
  for (size_t i = 0; i < n; ++i) b->blocks[i] = LayerBlock{nullptr, nullptr, 100 + i};
  return b;
}

void replay(Storage& st, const std::string& ns, const std::vector<Op>& ops,
            const std::vector<std::shared_ptr<LayerBlockBatch>>& pre_blocks) {
  for (size_t k = 0; k < ops.size(); ++k) {
    const Op& op = ops[k];
    if (op.kind == 0) {
      try {
        st.insert_slot(ns, op.hash, op.slot, layer_block_at(pre_blocks[k], 0), op.total);
      } catch (const std::exception&) {
      }
    } else {
      try {
        st.cache_lookup_many(ns, op.lookups);
      } catch (const std::exception&) {
      }
    }
  }
}

bool same(Storage& a, Storage& b, std::string* why) {
  if (a.cache_view() != b.cache_view()) {
    *why = "cache contents or LRU order differ";
    return false;
  }
  if (a.inflight_view() != b.inflight_view()) {
    *why = "inflight blocks differ";
    return false;
  }
  if (a.counters().insertions.load() != b.counters().insertions.load() ||
      a.counters().admission_rejections.load() != b.counters().admission_rejections.load()) {
    *why = "admission counters differ";
    return false;
  }
  return true;
}

}  // namespace

int main(int argc, char** argv) {
  const int scenarios = argc > 1 ? atoi(argv[1]) : 2000;
  const std::string ns = "ns";
  int with_refusals = 0, with_seals = 0, with_errors = 0;
  for (int sc = 0; sc < scenarios; ++sc) {
    std::mt19937 rng(sc);
    auto pick = [&](int lo, int hi) { return std::uniform_int_distribution<int>(lo, hi)(rng); };
    const bool lfu = pick(0, 1) == 1;
    const uint64_t total = pick(2, 6);
    const int universe = pick(3, 10);
    auto name = [](int i) { return std::string("h") + std::to_string(i); };

    // Pre-state: random slot inserts (some complete a block, some use another
    // slot count), and lookups that bump recency and frequency.
    std::vector<Op> ops;
    const int n_ops = pick(0, 40);
    for (int k = 0; k < n_ops; ++k) {
      Op op;
      if (pick(0, 4) == 0) {
        op.kind = 1;
        for (int j = pick(1, 4); j > 0; --j) op.lookups.push_back(name(pick(0, universe - 1)));
      } else {
        op.kind = 0;
        op.hash = name(pick(0, universe - 1));
        op.total = pick(0, 15) == 0 ? total + 1 : total;
        op.slot = pick(0, static_cast<int>(op.total) - 1);
      }
      ops.push_back(op);
    }
    std::vector<std::shared_ptr<LayerBlockBatch>> pre_blocks;
    for (size_t k = 0; k < ops.size(); ++k) pre_blocks.push_back(make_batch(1));

    // The call: a hash list (repeats allowed) and fills of distinct slots.
    std::vector<std::string> hashes;
    for (int j = pick(1, 8); j > 0; --j) hashes.push_back(name(pick(0, universe - 1)));
    std::vector<uint64_t> slots(total);
    for (uint64_t s = 0; s < total; ++s) slots[s] = s;
    std::shuffle(slots.begin(), slots.end(), rng);
    slots.resize(pick(1, static_cast<int>(total)));
    std::vector<SlotFill> fills;
    for (uint64_t s : slots) fills.push_back(SlotFill{s, make_batch(hashes.size())});

    auto a = make_store(lfu);
    auto b = make_store(lfu);
    replay(*a, ns, ops, pre_blocks);
    replay(*b, ns, ops, pre_blocks);
    std::string err_a, err_b, why;
    if (!same(*a, *b, &why)) {
      printf("scenario %d: pre-states differ (%s)\n", sc, why.c_str());
      return 1;
    }
    const uint64_t ins0 = a->counters().insertions.load();
    const uint64_t rej0 = a->counters().admission_rejections.load();
    try {
      for (const SlotFill& f : fills) {
        std::vector<LayerBlockPtr> blocks(hashes.size());
        for (size_t i = 0; i < hashes.size(); ++i) blocks[i] = layer_block_at(f.batch, i);
        a->insert_slots(ns, hashes, f.slot, blocks, total);
      }
    } catch (const std::exception& e) {
      err_a = e.what();
    }
    try {
      b->insert_slots_multi(ns, hashes, fills, total);
    } catch (const std::exception& e) {
      err_b = e.what();
    }
    if (err_a != err_b) {
      printf("scenario %d: errors differ: '%s' vs '%s'\n", sc, err_a.c_str(), err_b.c_str());
      return 1;
    }
    if (!same(*a, *b, &why)) {
      printf("scenario %d: %s\n", sc, why.c_str());
      return 1;
    }
    with_errors += !err_a.empty();
    with_seals += a->counters().insertions.load() > ins0;
    with_refusals += a->counters().admission_rejections.load() > rej0;
  }
  printf("ok scenarios=%d seals=%d refusals=%d errors=%d\n", scenarios, with_seals, with_refusals, with_errors);
  return 0;
}
