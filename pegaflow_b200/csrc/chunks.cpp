#include "chunks.h"

#include <algorithm>

namespace pf {

void cut_chunks(const std::vector<PlanLayer>& layers, uint64_t total_tiles, uint64_t slot_bytes,
                uint64_t first_limit, std::vector<Chunk>* chunks) {
  chunks->clear();
  if (total_tiles == 0) return;
  // Walk units in order; a chunk is a tile range whose dense span fits the
  // current limit. The limit starts at first_limit and doubles with each
  // chunk up to the slot size: the first copy-engine transfer (and, for a
  // load, the first layer's completion) starts after a small kernel, while
  // the bulk moves in few launches. Every launch pays a fixed latency of tens
  // of microseconds while the copy engine is busy, so the launch count, not
  // the bytes, sets the kernel's cost. A chunk's dense start is rounded down
  // to kDenseAlign so the slot shift (slot - dense_begin) keeps every
  // 16-byte-aligned dense address aligned, even when the chunk starts inside
  // a layer of unaligned units.
  uint64_t cur_tb = 0, cur_db = 0, cur_df = 0, last_end = 0;
  uint64_t limit = std::min(slot_bytes, std::max<uint64_t>(first_limit, 2 * kTileBytes));
  bool first = true;
  uint64_t dense = 0;
  for (const PlanLayer& p : layers) {
    dense = align_up(dense, kDenseAlign);
    const uint64_t nunits = static_cast<uint64_t>(p.units) * p.n;
    for (uint64_t ul = 0; ul < nunits; ++ul) {
      const uint64_t ud = dense + ul * p.unit_bytes;
      const uint64_t ue = ud + p.unit_bytes;
      const uint64_t ut = p.tile_start + ul * p.tiles_per_unit;
      if (first) {
        cur_tb = ut;
        cur_df = ud;
        cur_db = ud / kDenseAlign * kDenseAlign;
        first = false;
      }
      if (ue - cur_db <= limit) {  // whole unit joins the current chunk ...
        // ... and so do the following units that end inside the limit
        // (units of a layer are uniform): skip to the last of them.
        const uint64_t fit = (cur_db + limit - ud) / p.unit_bytes;  // >= 1 units starting at ul
        const uint64_t last = std::min(nunits - 1, ul + fit - 1);
        ul = last;
        last_end = dense + (last + 1) * p.unit_bytes;
        continue;
      }
      for (uint32_t t = 0; t < p.tiles_per_unit; ++t) {
        const uint64_t d0 = ud + static_cast<uint64_t>(t) * kTileBytes;
        const uint64_t d1 = std::min<uint64_t>(d0 + kTileBytes, ue);
        if (d1 - cur_db > limit) {
          chunks->push_back({cur_tb, ut + t, cur_db, last_end, cur_df});
          cur_tb = ut + t;
          cur_df = d0;
          cur_db = d0 / kDenseAlign * kDenseAlign;
          limit = std::min(slot_bytes, limit * 2);
        }
        last_end = d1;
      }
    }
    dense += nunits * p.unit_bytes;
  }
  chunks->push_back({cur_tb, total_tiles, cur_db, last_end, cur_df});
}

uint64_t layerwise_first_limit(const std::vector<PlanLayer>& layers, uint64_t first_chunk, uint64_t min_first) {
  if (layers.empty()) return first_chunk;
  auto layer_bytes = [](const PlanLayer& p) { return static_cast<uint64_t>(p.units) * p.n * p.unit_bytes; };
  const uint64_t layer0 = layer_bytes(layers[0]);
  uint64_t span = align_up(layer0, kDenseAlign);  // dense bytes, as the chunks count them
  for (size_t i = 1; i < layers.size() && layer_bytes(layers[i]) * 8 <= layer0; ++i) {
    span += align_up(layer_bytes(layers[i]), kDenseAlign);
  }
  return std::min(first_chunk, std::max(min_first, span));
}

}  // namespace pf
