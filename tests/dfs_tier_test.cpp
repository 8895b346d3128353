// Packed-file tier on a plain-memory pool (no GPU): write-through of sealed
// blocks, the file and record format, prefetch back into the pool, the query
// states, the index rebuilt on restart, and quota eviction of the oldest
// files. Expected bytes and records are computed here from the format of
// pegaflow-core/src/seal_offload.rs:379-448 and 785-909, independently of the
// tier's own code. Run by tests/test_dfs_tier.py; prints "ok ..." or the
// first failure.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "dfs_tier.h"
#include "storage.h"

using namespace pf;
namespace fs = std::filesystem;

namespace {

int failures = 0;
#define CHECK(cond)                                                     \
  do {                                                                  \
    if (!(cond)) {                                                      \
      printf("FAIL line %d: %s\n", __LINE__, #cond);                    \
      ++failures;                                                       \
      return;                                                           \
    }                                                                   \
  } while (0)

constexpr uint64_t kSeg = 1024;      // split slot: K and V of 1 KiB
constexpr uint64_t kContig = 1536;   // contiguous slot
constexpr int kBlocks = 7;
const std::string kNs = "ns0";

std::string hash_of(int i) { return std::string("\x01\x02", 2) + "block-" + std::to_string(i); }

// Deterministic bytes of (block, slot, part).
uint8_t byte_at(int block, int slot, int part, uint64_t i) {
  return static_cast<uint8_t>((block * 131 + slot * 17 + part * 7 + i * 13) & 0xff);
}

// What a packed file holds for block b: slot 0 K then V, slot 1's bytes.
std::string expected_block_bytes(int b) {
  std::string s;
  for (uint64_t i = 0; i < kSeg; ++i) s.push_back(static_cast<char>(byte_at(b, 0, 0, i)));
  for (uint64_t i = 0; i < kSeg; ++i) s.push_back(static_cast<char>(byte_at(b, 0, 1, i)));
  for (uint64_t i = 0; i < kContig; ++i) s.push_back(static_cast<char>(byte_at(b, 1, 0, i)));
  return s;
}

std::string expected_meta_json(const std::string& file, uint64_t offset) {
  return "{\"file\":\"" + file + "\",\"offset\":" + std::to_string(offset) +
         ",\"slots\":[{\"is_split\":true,\"size\":" + std::to_string(2 * kSeg) +
         "},{\"is_split\":false,\"size\":" + std::to_string(kContig) + "}],\"total_slots\":2}";
}

std::unique_ptr<Storage> make_storage(std::shared_ptr<PinnedPool> pool) {
  StorageConfig cfg;
  cfg.enable_lfu_admission = false;
  cfg.capacity_bytes = 8 << 20;
  return std::make_unique<Storage>(pool, cfg);
}

// Seals kBlocks two-slot blocks: slot 0 split, slot 1 contiguous.
void seal_blocks(Storage& st) {
  std::vector<std::string> hashes;
  for (int b = 0; b < kBlocks; ++b) hashes.push_back(hash_of(b));
  auto k = st.allocate(kSeg * kBlocks), v = st.allocate(kSeg * kBlocks), c = st.allocate(kContig * kBlocks);
  auto split = std::make_shared<LayerBlockBatch>(), contig = std::make_shared<LayerBlockBatch>();
  split->k_alloc = k;
  split->v_alloc = v;
  contig->k_alloc = c;
  for (int b = 0; b < kBlocks; ++b) {
    for (uint64_t i = 0; i < kSeg; ++i) {
      k->ptr[b * kSeg + i] = byte_at(b, 0, 0, i);
      v->ptr[b * kSeg + i] = byte_at(b, 0, 1, i);
    }
    for (uint64_t i = 0; i < kContig; ++i) c->ptr[b * kContig + i] = byte_at(b, 1, 0, i);
    split->blocks.push_back(LayerBlock{k->ptr + b * kSeg, v->ptr + b * kSeg, 2 * kSeg});
    contig->blocks.push_back(LayerBlock{c->ptr + b * kContig, nullptr, kContig});
  }
  std::vector<LayerBlockPtr> s0, s1;
  for (int b = 0; b < kBlocks; ++b) {
    s0.push_back(layer_block_at(split, b));
    s1.push_back(layer_block_at(contig, b));
  }
  st.insert_slots(kNs, hashes, 0, s0, 2);
  st.insert_slots(kNs, hashes, 1, s1, 2);
}

std::string read_file(const fs::path& p) {
  std::ifstream in(p, std::ios::binary);
  return std::string(std::istreambuf_iterator<char>(in), std::istreambuf_iterator<char>());
}

// The block's bytes as the pool now holds them (slot 0 K|V, slot 1).
std::string cached_bytes(Storage& st, int b) {
  SealedBlockPtr sb = st.cache_peek(kNs, hash_of(b));
  if (!sb || sb->slots.size() != 2) return "";
  std::string s(reinterpret_cast<const char*>(sb->slots[0]->k_ptr), kSeg);
  s.append(reinterpret_cast<const char*>(sb->slots[0]->v_ptr), kSeg);
  s.append(reinterpret_cast<const char*>(sb->slots[1]->k_ptr), kContig);
  return s;
}

void evict_everything(Storage& st) {
  // An allocation of the whole pool: reclaim-on-allocate evicts every cached
  // block (storage.rs:405-433); it is released at once.
  auto big = st.allocate(8 << 20);
}

void run(const fs::path& root) {
  auto pool = PinnedPool::create(8 << 20, PinKind::kPlainHost, false, 0);
  auto st = make_storage(pool);
  DfsConfig cfg;
  cfg.root = root.string();
  cfg.max_pack_size = 3;
  cfg.scan_interval_ms = 3600 * 1000;  // quota only when asked
  auto tier = std::make_unique<DfsTier>(st.get(), cfg);
  DfsTier* t = tier.get();
  st->set_seal_listener([t](const BlockKey& k, const SealedBlockPtr& b) { t->on_seal(k, b); });

  // 1. Write-through: 7 blocks, 3 per file.
  seal_blocks(*st);
  CHECK(tier->flush(30));
  DfsStats s = tier->stats();
  CHECK(s.written_blocks == kBlocks && s.files == 3 && s.write_failures == 0);
  CHECK(s.usage_bytes == kBlocks * (2 * kSeg + kContig));

  // 2. Format: every packed file's bytes and records.
  int seen = 0;
  for (const auto& f : fs::directory_iterator(root / kNs)) {
    const std::string name = f.path().filename().string();
    if (name.size() < 9 || name.substr(name.size() - 9) != ".bin.meta") continue;
    const std::string bin = name.substr(0, name.size() - 5);
    const std::string data = read_file(root / kNs / bin);
    std::ifstream in(f.path());
    std::string line;
    std::getline(in, line);
    CHECK(line == "pegaflow-packed-file 1");
    uint64_t expect_off = 0;
    std::vector<std::string> hexes;
    std::string file_meta;
    while (std::getline(in, line)) {
      if (line.rfind("file_meta\t", 0) == 0) file_meta = line.substr(10);
      if (line.rfind("block\t", 0) != 0) continue;
      const size_t tab = line.find('\t', 6);
      const std::string hex = line.substr(6, tab - 6), json = line.substr(tab + 1);
      std::string hash;
      CHECK(hex_decode(hex, &hash));
      const int b = std::atoi(hash.substr(8).c_str());
      CHECK(json == expected_meta_json(bin, expect_off));
      CHECK(data.compare(expect_off, 2 * kSeg + kContig, expected_block_bytes(b)) == 0);
      expect_off += 2 * kSeg + kContig;
      hexes.push_back(hex);
      ++seen;
    }
    CHECK(data.size() == expect_off);
    std::string fm = "{\"blocks\":[";
    for (size_t i = 0; i < hexes.size(); ++i) fm += (i ? ",\"" : "\"") + hexes[i] + "\"";
    fm += "],\"size\":" + std::to_string(expect_off) + "}";
    CHECK(file_meta == fm);
  }
  CHECK(seen == kBlocks);

  // 3. Prefetch: evicted from the pool, read back on a query miss.
  evict_everything(*st);
  CHECK(st->cached_count() == 0);
  std::vector<std::string> q;
  for (int b = 0; b < kBlocks; ++b) q.push_back(hash_of(b));
  q.push_back("not-saved-anywhere");
  PrefetchStatus p = tier->query(kNs, q);
  CHECK(p.state == PrefetchState::kLoading && p.hit_blocks == 0 && p.loading_blocks == q.size());
  CHECK(tier->flush(30));
  for (int b = 0; b < kBlocks; ++b) CHECK(cached_bytes(*st, b) == expected_block_bytes(b));
  CHECK(tier->stats().prefetched_blocks == kBlocks);
  // 4. The last block is nowhere: a partial miss after the cached prefix.
  p = tier->query(kNs, q);
  CHECK(p.state == PrefetchState::kPartialMiss && p.hit_blocks == kBlocks && p.missing_blocks == 1);
  // All cached: ready.
  q.pop_back();
  p = tier->query(kNs, q);
  CHECK(p.state == PrefetchState::kReady && p.hit_blocks == kBlocks);
  // Prefetched blocks are not written again.
  CHECK(tier->flush(30) && tier->stats().written_blocks == kBlocks);

  // 5. Restart: a new tier over the same root finds all three files.
  st->set_seal_listener(nullptr);
  tier.reset();
  cfg.quota_bytes = 3 * (2 * kSeg + kContig);  // one file's worth
  tier = std::make_unique<DfsTier>(st.get(), cfg);
  s = tier->stats();
  CHECK(s.files == 3 && s.blocks == kBlocks && s.usage_bytes == kBlocks * (2 * kSeg + kContig));

  // 6. Quota: the two oldest files go, with their records.
  tier->check_quota();
  s = tier->stats();
  CHECK(s.files == 1 && s.evicted_files == 2 && s.usage_bytes <= cfg.quota_bytes);
  int bins = 0;
  for (const auto& f : fs::directory_iterator(root / kNs)) bins += f.path().extension() == ".bin";
  CHECK(bins == 1);
  int still = 0;
  for (int b = 0; b < kBlocks; ++b) still += tier->has_block(kNs, hash_of(b));
  CHECK(still == static_cast<int>(s.blocks) && still >= 1 && still <= 3);
  // What is left still reads back.
  evict_everything(*st);
  for (int b = 0; b < kBlocks; ++b) {
    if (!tier->has_block(kNs, hash_of(b))) continue;
    p = tier->query(kNs, {hash_of(b)});
    CHECK(p.state == PrefetchState::kLoading);
    CHECK(tier->flush(30));
    CHECK(cached_bytes(*st, b) == expected_block_bytes(b));
  }
  tier.reset();
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    printf("usage: dfs_tier_test <empty directory>\n");
    return 2;
  }
  run(argv[1]);
  if (failures) return 1;
  printf("ok\n");
  return 0;
}
