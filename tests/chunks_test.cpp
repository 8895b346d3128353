// The staging-chunk cutter (pegaflow_b200/csrc/chunks.cpp) on random plans
// and on the schedules the benchmark uses. Each chunk is relocated into one
// staging slot by a kernel launch and drained or filled by copy-engine
// copies, so the invariants below keep those inside the slot:
//   - the chunks tile the plan: contiguous, non-empty, ending at total_tiles;
//   - every chunk's slot base is on a kDenseAlign boundary, less than one
//     step before its first byte, and the chunk spans at most a slot;
//   - every tile's dense bytes lie inside its chunk's [dense_first, dense_end),
//     and those ranges never overlap between chunks (a copy of one chunk must
//     not touch bytes another chunk moves);
//   - chunk k spans at most limit_k: the first limit (clamped to [2 tiles,
//     slot]) doubled k times, up to the slot.
//
// Build and run (tests/test_chunks.py does this):
//   g++ -O1 -std=c++17 -I<repo>/pegaflow_b200/csrc -I<cuda>/include
//       tests/chunks_test.cpp <csrc>/chunks.cpp
//   ./chunks_test
#include <algorithm>
#include <cstdio>
#include <random>
#include <vector>

#include "chunks.h"

using namespace pf;

namespace {

struct Case {
  std::vector<PlanLayer> layers;
  uint64_t total_tiles = 0;
};

Case make_case(const std::vector<std::pair<uint32_t, uint32_t>>& unit_bytes_and_units, uint32_t n) {
  Case c;
  for (auto [ub, units] : unit_bytes_and_units) {
    PlanLayer p{};
    p.unit_bytes = ub;
    p.units = units;
    p.n = n;
    p.tiles_per_unit = (ub + kTileBytes - 1) / kTileBytes;
    p.tile_start = c.total_tiles;
    p.tile_count = static_cast<uint64_t>(units) * n * p.tiles_per_unit;
    c.total_tiles += p.tile_count;
    c.layers.push_back(p);
  }
  return c;
}

// Returns an empty string when every invariant holds.
const char* check(const Case& c, uint64_t slot, uint64_t first, const std::vector<Chunk>& ch) {
  if (ch.empty()) return "no chunks";
  if (ch.front().tile_begin != 0 || ch.back().tile_end != c.total_tiles) return "chunks do not span the plan";
  uint64_t limit = std::min(slot, std::max<uint64_t>(first, 2 * kTileBytes));
  for (size_t k = 0; k < ch.size(); ++k) {
    if (ch[k].tile_end <= ch[k].tile_begin) return "empty chunk";
    if (k + 1 < ch.size() && ch[k].tile_end != ch[k + 1].tile_begin) return "chunks not contiguous";
    if (ch[k].dense_begin % kDenseAlign) return "chunk start not aligned";
    if (ch[k].dense_first < ch[k].dense_begin || ch[k].dense_first - ch[k].dense_begin >= kDenseAlign) {
      return "first byte not within one alignment step of the slot base";
    }
    // The chunks' own byte ranges never overlap: a copy of chunk k+1 must not
    // touch the bytes chunk k moves.
    if (k + 1 < ch.size() && ch[k].dense_end > ch[k + 1].dense_first) return "chunk byte ranges overlap";
    if (ch[k].dense_end < ch[k].dense_begin || ch[k].dense_end - ch[k].dense_begin > limit) return "chunk over its limit";
    if (limit > slot) return "limit above the slot";
    limit = std::min(slot, limit * 2);
  }
  // Every tile's dense bytes inside its chunk.
  size_t k = 0;
  uint64_t dense = 0;
  for (const PlanLayer& p : c.layers) {
    dense = align_up(dense, kDenseAlign);
    for (uint64_t t = 0; t < p.tile_count; ++t) {
      const uint64_t tile = p.tile_start + t;
      while (k < ch.size() && tile >= ch[k].tile_end) ++k;
      if (k == ch.size() || tile < ch[k].tile_begin) return "tile outside every chunk";
      const uint64_t ul = t / p.tiles_per_unit, tt = t % p.tiles_per_unit;
      const uint64_t d0 = dense + ul * p.unit_bytes + tt * kTileBytes;
      const uint64_t d1 = std::min<uint64_t>(d0 + kTileBytes, dense + (ul + 1) * p.unit_bytes);
      if (d0 < ch[k].dense_first || d1 > ch[k].dense_end) return "tile bytes outside its chunk";
    }
    dense += static_cast<uint64_t>(p.units) * p.n * p.unit_bytes;
  }
  return "";
}

std::vector<uint64_t> spans_mib(const std::vector<Chunk>& ch) {
  std::vector<uint64_t> out;
  for (const Chunk& c : ch) out.push_back((c.dense_end - c.dense_begin) >> 20);
  return out;
}

}  // namespace

int main() {
  std::mt19937_64 rng(7);
  const uint32_t sizes[] = {3, 4, 12, 45, 4096, 8192, 16384, 24576, 32768, 65536, 100000};
  long cases = 0;
  for (int it = 0; it < 50000; ++it) {
    std::vector<std::pair<uint32_t, uint32_t>> spec;
    const int nl = 1 + static_cast<int>(rng() % 6);
    for (int i = 0; i < nl; ++i) spec.push_back({sizes[rng() % 11], 1 + static_cast<uint32_t>(rng() % 2)});
    const Case c = make_case(spec, 1 + static_cast<uint32_t>(rng() % 50));
    const uint64_t slot = align_up(std::max<uint64_t>(2 * kTileBytes, 1 + rng() % (1 << 22)), kDenseAlign);
    const uint64_t first = rng() % (1 << 21);
    std::vector<Chunk> ch;
    cut_chunks(c.layers, c.total_tiles, slot, first, &ch);
    const char* why = check(c, slot, first, ch);
    if (*why) {
      std::printf("FAIL case %d: %s\n", it, why);
      return 1;
    }
    ++cases;
  }

  // The benchmark's schedules. configs[1]: one 1.25 GiB direction of 32
  // layers of 640 blocks x (K, V) x 32 KiB; configs[3] at TP1: 10 GiB of 80
  // layers of 2048 blocks x (K, V) x 32 KiB. Default 1 GiB slots, and the
  // earlier 512 MiB slots.
  const Case llama = make_case(std::vector<std::pair<uint32_t, uint32_t>>(32, {32768, 2}), 640);
  const Case llama70 = make_case(std::vector<std::pair<uint32_t, uint32_t>>(80, {32768, 2}), 2048);
  const uint64_t m512 = 512ull << 20, g1 = 1024ull << 20;
  struct Want {
    const Case* c;
    uint64_t slot;
    uint64_t first;
    std::vector<uint64_t> mib;
  };
  std::vector<uint64_t> tp1_loads(10, 1024), tp1_saves(9, 1024);
  tp1_saves.insert(tp1_saves.begin(), 512);
  tp1_saves.push_back(512);
  const Want wants[] = {
      {&llama, m512, 64ull << 20, {64, 128, 256, 512, 320}},     // growth from 64 MiB
      {&llama, m512, m512, {512, 512, 256}},                      // loads without per-layer flags: whole slots
      {&llama, m512, m512 / 2, {256, 512, 512}},                  // saves: half a slot first
      {&llama, m512, 40ull << 20, {40, 80, 160, 320, 512, 168}},  // layer-wise load: first chunk = one layer
      {&llama, g1, g1, {1024, 256}},                              // default slots: loads without flags
      {&llama, g1, g1 / 2, {512, 768}},                           // default slots: saves
      {&llama, g1, 40ull << 20, {40, 80, 160, 320, 640, 40}},     // default slots: layer-wise load
      {&llama70, g1, g1, tp1_loads},                              // configs[3] TP1 loads: ten whole slots
      {&llama70, g1, g1 / 2, tp1_saves},                          // configs[3] TP1 saves
  };
  for (const Want& w : wants) {
    std::vector<Chunk> ch;
    cut_chunks(w.c->layers, w.c->total_tiles, w.slot, w.first, &ch);
    if (*check(*w.c, w.slot, w.first, ch) || spans_mib(ch) != w.mib) {
      std::printf("FAIL schedule with slot %llu MiB, first chunk %llu MiB:",
                  static_cast<unsigned long long>(w.slot >> 20), static_cast<unsigned long long>(w.first >> 20));
      for (uint64_t m : spans_mib(ch)) std::printf(" %llu", static_cast<unsigned long long>(m));
      std::printf("\n");
      return 1;
    }
  }
  // Layer-wise loads: the first chunk ends where layer 0 (and the small
  // layers right after it) end, so layer 0's flags rise after chunk 0.
  const uint64_t kMin = 4ull << 20, kFirst = 64ull << 20;
  {
    // fp8 KV ([2, nb, 16, 8, 128] uint8: K and V units of 16 KiB) interleaved
    // with its fp32 per-block scales (4-byte units), 265 blocks per layer.
    std::vector<std::pair<uint32_t, uint32_t>> spec;
    for (int l = 0; l < 32; ++l) {
      spec.push_back({16384, 2});
      spec.push_back({4, 1});
    }
    const Case fp8 = make_case(spec, 265);
    const uint64_t first = layerwise_first_limit(fp8.layers, kFirst, kMin);
    std::vector<Chunk> ch;
    cut_chunks(fp8.layers, fp8.total_tiles, g1, first, &ch);
    if (*check(fp8, g1, first, ch) || ch[0].tile_end != fp8.layers[2].tile_start) {
      std::printf("FAIL fp8 first chunk: limit %llu, ends at tile %llu, layer 1 of KV starts at %llu\n",
                  static_cast<unsigned long long>(first), static_cast<unsigned long long>(ch[0].tile_end),
                  static_cast<unsigned long long>(fp8.layers[2].tile_start));
      return 1;
    }
  }
  {
    const uint64_t first = layerwise_first_limit(llama.layers, kFirst, kMin);  // one 40 MiB layer
    std::vector<Chunk> ch;
    cut_chunks(llama.layers, llama.total_tiles, g1, first, &ch);
    if (first != (40ull << 20) || ch[0].tile_end != llama.layers[1].tile_start) {
      std::printf("FAIL llama first chunk %llu\n", static_cast<unsigned long long>(first));
      return 1;
    }
  }
  {
    // configs[3] at TP1 with the default 256 MiB first-chunk limit: the first
    // chunk is the whole 128 MiB layer 0 (a 64 MiB limit split it, and layer
    // 0's flag then waited for the second chunk too).
    const uint64_t first = layerwise_first_limit(llama70.layers, 256ull << 20, kMin);
    std::vector<Chunk> ch;
    cut_chunks(llama70.layers, llama70.total_tiles, g1, first, &ch);
    std::vector<uint64_t> want = {128, 256, 512};
    for (int k = 0; k < 9; ++k) want.push_back(1024);
    want.push_back(128);
    if (first != (128ull << 20) || ch[0].tile_end != llama70.layers[1].tile_start || spans_mib(ch) != want) {
      std::printf("FAIL llama70 layer-wise first chunk %llu\n", static_cast<unsigned long long>(first));
      return 1;
    }
  }
  {
    // Layers of 1.5 MiB: the 4 MiB floor applies; a cap below the layer wins.
    const Case small = make_case(std::vector<std::pair<uint32_t, uint32_t>>(24, {24576, 1}), 64);
    if (layerwise_first_limit(small.layers, kFirst, kMin) != kMin ||
        layerwise_first_limit(llama.layers, 8ull << 20, kMin) != (8ull << 20) ||
        layerwise_first_limit({}, kFirst, kMin) != kFirst) {
      std::printf("FAIL first-chunk floor or cap\n");
      return 1;
    }
  }

  std::printf("ok %ld random plans\n", cases);
  return 0;
}
