#include "plan_build.h"

#include <algorithm>
#include <string>

#include "chunks.h"
#include "common.h"

namespace pf {

// ---------------------------------------------------------------------------
// Layout helpers (reference semantics)
// ---------------------------------------------------------------------------

bool is_split_layout(const pf_layer_desc& l) {
  // lib.rs:636, gpu_worker.rs:218,326
  return l.segments == 2 && l.kv_stride_bytes > l.bytes_per_block;
}

bool is_contiguous_layout(const pf_layer_desc& l) {
  // transfer.rs:50-52
  return l.segments <= 1 || l.kv_stride_bytes == l.bytes_per_block;
}

UnitGeometry save_geometry(const pf_layer_desc& l) {
  if (is_split_layout(l)) return {2u, l.bytes_per_block, l.kv_stride_bytes};
  // copy_block_gpu_to_cpu (transfer.rs:200-239)
  if (is_contiguous_layout(l)) return {1u, l.bytes_per_block * l.segments, 0};
  return {static_cast<uint32_t>(l.segments), l.bytes_per_block, l.kv_stride_bytes};
}

UnitGeometry load_geometry(const pf_layer_desc& l) {
  if (is_split_layout(l)) return {2u, l.bytes_per_block, l.kv_stride_bytes};
  // gpu_worker.rs:260-282: one block_size_bytes copy at segment 0's offset.
  return {1u, l.bytes_per_block * l.segments, 0};
}

void validate_layout(const pf_layer_desc& l, const char* layer_name) {
  // register_context_layer (lib.rs:389-449), same order and messages.
  const std::string name = layer_name ? layer_name : "";
  if (l.bytes_per_block == 0 || l.num_blocks == 0 || l.segments == 0) {
    throw invalid_argument("invalid KV cache layout for layer " + name);
  }
  if (l.segments > 1 && l.kv_stride_bytes == 0) {
    throw invalid_argument("kv_stride_bytes must be > 0 when segments > 1 for layer " + name);
  }
  uint64_t block_size = 0;
  if (mul_ovf(l.bytes_per_block, l.segments, &block_size)) {
    throw invalid_argument("block size overflow: bytes_per_block=" + std::to_string(l.bytes_per_block) +
                           " segments=" + std::to_string(l.segments) + " for layer " + name);
  }
  uint64_t max_block_offset = 0;
  if (mul_ovf(l.num_blocks - 1, l.bytes_per_block, &max_block_offset)) {
    throw invalid_argument("num_blocks " + std::to_string(l.num_blocks) + " too large for layer " + name);
  }
  uint64_t max_segment_offset = 0;
  if (mul_ovf(l.segments - 1, l.kv_stride_bytes, &max_segment_offset)) {
    throw invalid_argument("segments/stride overflow for layer " + name + " (segments=" +
                           std::to_string(l.segments) + ", stride=" + std::to_string(l.kv_stride_bytes) + ")");
  }
  uint64_t max_offset = 0;
  if (add_ovf(max_block_offset, max_segment_offset, &max_offset)) {
    throw invalid_argument("layout offset overflow for layer " + name);
  }
  uint64_t end = 0;
  if (add_ovf(max_offset, l.bytes_per_block, &end)) {
    throw invalid_argument("layout end overflow for layer " + name);
  }
  if (end > l.size_bytes) {
    throw invalid_argument("registered memory too small for layer " + name + ": need at least " +
                           std::to_string(end) + " bytes, got " + std::to_string(l.size_bytes));
  }
}

uint64_t segment_offset(const pf_layer_desc& l, uint64_t block_idx, uint64_t segment_idx) {
  // transfer.rs:18-47
  if (segment_idx >= l.segments) throw storage_error("Segment index out of range");
  uint64_t base = 0, seg = 0, off = 0, end = 0;
  if (mul_ovf(block_idx, l.bytes_per_block, &base)) throw storage_error("Block offset overflow");
  if (mul_ovf(segment_idx, l.kv_stride_bytes, &seg)) throw storage_error("Segment offset overflow");
  if (add_ovf(base, seg, &off)) throw storage_error("Combined offset overflow");
  if (add_ovf(off, l.bytes_per_block, &end) || end > l.size_bytes) {
    throw storage_error("Block " + std::to_string(block_idx) + " segment " + std::to_string(segment_idx) +
                        " exceeds registered memory (offset " + std::to_string(off) + ", size " +
                        std::to_string(l.bytes_per_block) + ", limit " + std::to_string(l.size_bytes) + ")");
  }
  return off;
}

namespace {


constexpr uint64_t kMaxUnitBytes = 1ull << 31;

bool aligned16(uint64_t v) { return (v & 15u) == 0; }

// Plan offsets are 32-bit in PlanLayer and the kernel adds them in 32-bit
// arithmetic, so every array end (not only each start) must fit.
uint32_t plan_offset(uint64_t v) {
  if (v > 0xffffffffull) throw invalid_argument("transfer too large for one plan (more than 2^32 units)");
  return static_cast<uint32_t>(v);
}
void check_plan_ends(const std::vector<uint32_t>& ids, const std::vector<uint64_t>& side_base, uint64_t units) {
  plan_offset(ids.size());
  plan_offset(side_base.size());
  plan_offset(units);
}

// The copy of unit (b, u) must stay inside the registration. This is stricter
// than segment_offset for non-split loads, where the reference copies
// block_size_bytes after checking only bytes_per_block (transfer.rs:39-44 vs
// gpu_worker.rs:266-272); a copy past size_bytes is refused here instead of
// writing outside the registered tensor.
void check_unit_range(const pf_layer_desc& l, uint64_t b, uint32_t u, const UnitGeometry& g) {
  uint64_t off = 0, t = 0, end = 0;
  if (mul_ovf(b, l.bytes_per_block, &off) || mul_ovf(u, g.unit_stride, &t) || add_ovf(off, t, &off) ||
      add_ovf(off, g.unit_bytes, &end) || end > l.size_bytes) {
    throw storage_error("Block " + std::to_string(b) + " unit " + std::to_string(u) + " (" +
                        std::to_string(g.unit_bytes) + " bytes) exceeds registered memory (limit " +
                        std::to_string(l.size_bytes) + ")");
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Plan building
// ---------------------------------------------------------------------------

void plan_save(const pf_save_layer* layers, uint64_t n_layers, bool staged, int device,
               const DeviceCheck& check_device_range, Built* b) {
  uint64_t dense = 0;
  uint64_t unit_base = 0;
  for (uint64_t li = 0; li < n_layers; ++li) {
    const pf_save_layer& s = layers[li];
    const pf_layer_desc& l = s.layer;
    const std::string lname = "#" + std::to_string(li);
    validate_layout(l, lname.c_str());
    if (s.n == 0) continue;
    if (s.block_idx == nullptr || s.k_dst == nullptr) throw invalid_argument("null block list or destination");
    if (l.num_blocks > 0xffffffffull || s.n > 0xffffffffull) throw invalid_argument("too many blocks for one layer");
    check_device_range(device, l);
    const UnitGeometry g = save_geometry(l);
    if (g.unit_bytes > kMaxUnitBytes) throw invalid_argument("block larger than 2 GiB");
    const uint64_t block_size = l.bytes_per_block * l.segments;

    auto check_offsets = [&](uint64_t blk) {
      if (is_split_layout(l)) {
        segment_offset(l, blk, 0);
        segment_offset(l, blk, 1);
      } else if (is_contiguous_layout(l)) {
        segment_offset(l, blk, 0);
      } else {
        for (uint64_t sg = 0; sg < l.segments; ++sg) segment_offset(l, blk, sg);
      }
      for (uint32_t u = 0; u < g.units; ++u) check_unit_range(l, blk, u, g);
    };
    auto check_block = [&](uint64_t i) {
      const int64_t bi = s.block_idx[i];
      if (bi < 0 || static_cast<uint64_t>(bi) >= l.num_blocks) {
        // lib.rs:597-603
        throw invalid_argument("block " + std::to_string(bi) + " out of range for layer " + lname + " (" +
                               std::to_string(l.num_blocks) + " blocks registered)");
      }
      check_offsets(static_cast<uint64_t>(bi));
    };
    // Every offset and copy end grows with the block index, so when all ids
    // are in range, checking the largest id checks them all. Any failure
    // replays the per-block checks in list order, for the same first error.
    bool fast = true;
    uint64_t max_blk = 0;
    for (uint64_t i = 0; i < s.n && fast; ++i) {
      const int64_t bi = s.block_idx[i];
      fast = bi >= 0 && static_cast<uint64_t>(bi) < l.num_blocks;
      if (fast) max_blk = std::max(max_blk, static_cast<uint64_t>(bi));
    }
    if (fast) {
      try {
        check_offsets(max_blk);
      } catch (const std::exception&) {
        fast = false;
      }
    }
    if (!fast) {
      for (uint64_t i = 0; i < s.n; ++i) check_block(i);
    }

    // Host destinations (SaveBlock pointers, lib.rs:671-679 and 739-747).
    std::vector<uint64_t> host_base(g.units);
    uint64_t host_pitch;
    const uint64_t k = reinterpret_cast<uint64_t>(s.k_dst);
    if (is_split_layout(l)) {
      if (s.v_dst) {
        host_base[0] = k;
        host_base[1] = reinterpret_cast<uint64_t>(s.v_dst);
        host_pitch = l.bytes_per_block;
      } else {  // SaveBlock with v_dst_ptr None: V follows K (gpu_worker.rs:354-356)
        host_base[0] = k;
        host_base[1] = k + l.bytes_per_block;
        host_pitch = 2 * l.bytes_per_block;
      }
    } else if (is_contiguous_layout(l)) {
      host_base[0] = k;
      host_pitch = block_size;
    } else {  // strided: segment s at dst + s*bytes_per_block (transfer.rs:228-230)
      for (uint32_t u = 0; u < g.units; ++u) host_base[u] = k + u * l.bytes_per_block;
      host_pitch = block_size;
    }

    PlanLayer p{};
    p.cache_base = l.data_ptr;
    p.block_pitch = l.bytes_per_block;
    p.unit_stride = g.unit_stride;
    p.unit_bytes = static_cast<uint32_t>(g.unit_bytes);
    p.units = g.units;
    p.n = static_cast<uint32_t>(s.n);
    p.tiles_per_unit = static_cast<uint32_t>((g.unit_bytes + kTileBytes - 1) / kTileBytes);
    p.tile_start = b->total_tiles;
    p.tile_count = static_cast<uint64_t>(g.units) * s.n * p.tiles_per_unit;
    if (p.tile_count > 0xffffffffull) throw invalid_argument("layer transfer too large for one plan");
    p.ids_off = plan_offset(b->ids.size());
    p.side_off = plan_offset(b->side_base.size());
    p.unit_off = plan_offset(unit_base);
    p.done_index = static_cast<uint32_t>(li);
    bool vec = aligned16(l.data_ptr) && aligned16(l.bytes_per_block) && aligned16(g.unit_stride) &&
               aligned16(g.unit_bytes);
    dense = align_up(dense, kDenseAlign);
    const uint64_t dense_layer = dense;
    if (staged) {
      p.side_pitch = g.unit_bytes;
      for (uint32_t u = 0; u < g.units; ++u) b->side_base.push_back(dense_layer + u * s.n * g.unit_bytes);
    } else {
      p.side_pitch = host_pitch;
      vec = vec && aligned16(host_pitch);
      for (uint32_t u = 0; u < g.units; ++u) {
        vec = vec && aligned16(host_base[u]);
        b->side_base.push_back(host_base[u]);
      }
    }
    p.flags = vec ? kFlagVector : 0u;
    for (uint64_t i = 0; i < s.n; ++i) b->ids.push_back(static_cast<uint32_t>(s.block_idx[i]));

    // Host extents in unit order, merged where both sides are contiguous.
    for (uint32_t u = 0; u < g.units; ++u) {
      for (uint64_t i = 0; i < s.n; ++i) {
        const uint64_t d = dense_layer + (u * s.n + i) * g.unit_bytes;
        const uint64_t h = host_base[u] + i * host_pitch;
        if (!b->runs.empty()) {
          Run& r = b->runs.back();
          if (r.dense + r.bytes == d && r.host + r.bytes == h) {
            r.bytes += g.unit_bytes;
            continue;
          }
        }
        b->runs.push_back({d, h, g.unit_bytes});
      }
    }
    dense = dense_layer + static_cast<uint64_t>(g.units) * s.n * g.unit_bytes;
    b->total_tiles += p.tile_count;
    b->total_bytes += static_cast<uint64_t>(g.units) * s.n * g.unit_bytes;
    unit_base += static_cast<uint64_t>(g.units) * s.n;
    check_plan_ends(b->ids, b->side_base, unit_base);
    b->layers.push_back(p);
  }
}

void plan_load(const pf_load_layer* layers, uint64_t n_layers, bool staged, int device,
               const DeviceCheck& check_device_range, Built* b) {
  uint64_t dense = 0;
  uint64_t unit_base = 0;
  for (uint64_t li = 0; li < n_layers; ++li) {
    const pf_load_layer& s = layers[li];
    const pf_layer_desc& l = s.layer;
    const std::string lname = "#" + std::to_string(li);
    validate_layout(l, lname.c_str());
    if (s.n == 0) continue;
    if (s.block_idx == nullptr || s.k_src == nullptr) throw invalid_argument("null block list or source");
    if (l.num_blocks > 0xffffffffull || s.n > 0xffffffffull) throw invalid_argument("too many blocks for one layer");
    check_device_range(device, l);
    const UnitGeometry g = load_geometry(l);
    if (g.unit_bytes > kMaxUnitBytes) throw invalid_argument("block larger than 2 GiB");
    const bool split = is_split_layout(l);

    auto check_offsets = [&](uint64_t blk) {
      // process_load_task's checks (gpu_worker.rs:227-230, 266-267) ...
      segment_offset(l, blk, 0);
      if (split) segment_offset(l, blk, 1);
      // ... plus the copy's own end (see check_unit_range).
      for (uint32_t u = 0; u < g.units; ++u) check_unit_range(l, blk, u, g);
    };
    // As for saves: with no negative id and no null source, checking the
    // largest id checks every block; otherwise the per-block checks run in
    // list order for the same first error.
    uint64_t max_id = 0;
    bool fast = true;
    for (uint64_t i = 0; i < s.n && fast; ++i) {
      const int64_t bi = s.block_idx[i];
      fast = bi >= 0 && s.k_src[i] != nullptr;
      if (fast) max_id = std::max(max_id, static_cast<uint64_t>(bi));
    }
    if (fast) {
      try {
        check_offsets(max_id);
      } catch (const std::exception&) {
        fast = false;
      }
    }
    if (!fast) {
      for (uint64_t i = 0; i < s.n; ++i) {
        const int64_t bi = s.block_idx[i];
        if (bi < 0) throw invalid_argument("negative block index " + std::to_string(bi));
        check_offsets(static_cast<uint64_t>(bi));
        if (s.k_src[i] == nullptr) throw invalid_argument("null source pointer for block " + std::to_string(bi));
        max_id = std::max(max_id, static_cast<uint64_t>(bi));
      }
    }

    // The reference copies a layer's blocks in list order on one stream, so
    // where destinations coincide the later block wins (gpu_worker.rs:223-283).
    // Warps run in no order, so: in layouts where every block owns its bytes,
    // a repeated destination keeps only its last occurrence; in layouts whose
    // blocks share bytes (several segments without the split predicate, or a
    // K->V stride shorter than the K region) overlapping lists are copied in
    // list order by the copy engine instead of the kernel.
    std::vector<uint64_t> keep;
    keep.reserve(s.n);
    uint64_t k_region = 0;
    const bool owns_bytes = max_id < l.num_blocks &&
                            (split ? !mul_ovf(l.num_blocks, l.bytes_per_block, &k_region) &&
                                         l.kv_stride_bytes >= k_region
                                   : l.segments == 1);
    bool serial = false;
    if (owns_bytes) {
      std::vector<uint64_t> seen((max_id >> 6) + 1, 0);
      for (uint64_t i = s.n; i-- > 0;) {
        const uint64_t blk = static_cast<uint64_t>(s.block_idx[i]);
        if (seen[blk >> 6] & (1ull << (blk & 63))) continue;
        seen[blk >> 6] |= 1ull << (blk & 63);
        keep.push_back(i);
      }
      std::reverse(keep.begin(), keep.end());
    } else {
      std::vector<std::pair<uint64_t, uint64_t>> spans;  // [start, end) of every unit
      for (uint64_t i = 0; i < s.n; ++i) {
        const uint64_t blk = static_cast<uint64_t>(s.block_idx[i]);
        for (uint32_t u = 0; u < g.units; ++u) {
          const uint64_t st = blk * l.bytes_per_block + u * g.unit_stride;
          spans.emplace_back(st, st + g.unit_bytes);
        }
      }
      std::sort(spans.begin(), spans.end());
      for (size_t j = 1; j < spans.size() && !serial; ++j) serial = spans[j].first < spans[j - 1].second;
      for (uint64_t i = 0; i < s.n; ++i) keep.push_back(i);
    }
    if (serial) {
      SerialLoad sl;
      sl.layer = l;
      sl.done_index = static_cast<uint32_t>(li);
      for (uint64_t i = 0; i < s.n; ++i) {
        sl.ids.push_back(s.block_idx[i]);
        sl.k.push_back(reinterpret_cast<uint64_t>(s.k_src[i]));
        const void* v = s.v_src ? s.v_src[i] : nullptr;
        sl.v.push_back(v ? reinterpret_cast<uint64_t>(v) : reinterpret_cast<uint64_t>(s.k_src[i]) + l.bytes_per_block);
      }
      b->serial.push_back(std::move(sl));
      continue;
    }
    const uint64_t n = keep.size();

    PlanLayer p{};
    p.cache_base = l.data_ptr;
    p.block_pitch = l.bytes_per_block;
    p.unit_stride = g.unit_stride;
    p.unit_bytes = static_cast<uint32_t>(g.unit_bytes);
    p.units = g.units;
    p.n = static_cast<uint32_t>(n);
    p.tiles_per_unit = static_cast<uint32_t>((g.unit_bytes + kTileBytes - 1) / kTileBytes);
    p.tile_start = b->total_tiles;
    p.tile_count = static_cast<uint64_t>(g.units) * n * p.tiles_per_unit;
    if (p.tile_count > 0xffffffffull) throw invalid_argument("layer transfer too large for one plan");
    p.ids_off = plan_offset(b->ids.size());
    p.side_off = plan_offset(b->side_base.size());
    p.unit_off = plan_offset(unit_base);
    p.done_index = static_cast<uint32_t>(li);
    bool vec = aligned16(l.data_ptr) && aligned16(l.bytes_per_block) && aligned16(g.unit_stride) &&
               aligned16(g.unit_bytes);
    dense = align_up(dense, kDenseAlign);
    const uint64_t dense_layer = dense;
    p.side_pitch = g.unit_bytes;
    for (uint32_t u = 0; u < g.units; ++u) b->side_base.push_back(dense_layer + u * n * g.unit_bytes);
    for (uint64_t j = 0; j < n; ++j) b->ids.push_back(static_cast<uint32_t>(s.block_idx[keep[j]]));

    for (uint32_t u = 0; u < g.units; ++u) {
      for (uint64_t j = 0; j < n; ++j) {
        const uint64_t i = keep[j];
        uint64_t h;
        if (u == 0) {
          h = reinterpret_cast<uint64_t>(s.k_src[i]);
        } else {  // V: LayerBlock::v_ptr or K + bytes_per_block (gpu_worker.rs:233-236)
          const void* v = s.v_src ? s.v_src[i] : nullptr;
          h = v ? reinterpret_cast<uint64_t>(v) : reinterpret_cast<uint64_t>(s.k_src[i]) + l.bytes_per_block;
        }
        if (!staged) {
          b->side_ptrs.push_back(h);
          vec = vec && aligned16(h);
        }
        const uint64_t d = dense_layer + (u * n + j) * g.unit_bytes;
        if (!b->runs.empty()) {
          Run& r = b->runs.back();
          if (r.dense + r.bytes == d && r.host + r.bytes == h) {
            r.bytes += g.unit_bytes;
            continue;
          }
        }
        b->runs.push_back({d, h, g.unit_bytes});
      }
    }
    p.flags = vec ? kFlagVector : 0u;
    dense = dense_layer + static_cast<uint64_t>(g.units) * n * g.unit_bytes;
    b->total_tiles += p.tile_count;
    b->total_bytes += static_cast<uint64_t>(g.units) * n * g.unit_bytes;
    unit_base += static_cast<uint64_t>(g.units) * n;
    check_plan_ends(b->ids, b->side_base, unit_base);
    b->layers.push_back(p);
  }
}

void plan_p2p(const pf_p2p_layer* layers, uint64_t n_layers, int device, int peer, bool push,
              const DeviceCheck& check_device_range, Built* b) {
  uint64_t unit_base = 0;
  for (uint64_t li = 0; li < n_layers; ++li) {
    const pf_p2p_layer& s = layers[li];
    const std::string lname = "#" + std::to_string(li);
    validate_layout(s.src, (lname + ".src").c_str());
    validate_layout(s.dst, (lname + ".dst").c_str());
    if (s.n == 0) continue;
    if (!s.src_idx || !s.dst_idx) throw invalid_argument("null block list");
    if (s.src.bytes_per_block != s.dst.bytes_per_block || s.src.segments != s.dst.segments ||
        is_split_layout(s.src) != is_split_layout(s.dst)) {
      throw invalid_argument("source and destination layouts differ for layer " + lname);
    }
    if (!is_split_layout(s.src) && !is_contiguous_layout(s.src)) {
      throw invalid_argument("peer transfer needs split K/V or contiguous layouts (layer " + lname + ")");
    }
    if (s.src.num_blocks > 0xffffffffull || s.dst.num_blocks > 0xffffffffull || s.n > 0xffffffffull) {
      throw invalid_argument("too many blocks for one layer");
    }
    const pf_layer_desc& local = push ? s.src : s.dst;
    const pf_layer_desc& remote = push ? s.dst : s.src;
    const int64_t* local_ids = push ? s.src_idx : s.dst_idx;
    const int64_t* remote_ids = push ? s.dst_idx : s.src_idx;
    check_device_range(device, local);
    check_device_range(peer, remote);
    const UnitGeometry gl = save_geometry(local);
    const UnitGeometry gr = save_geometry(remote);
    if (gl.unit_bytes > kMaxUnitBytes) throw invalid_argument("block larger than 2 GiB");
    for (uint64_t i = 0; i < s.n; ++i) {
      for (int side = 0; side < 2; ++side) {
        const pf_layer_desc& l = side ? s.dst : s.src;
        const int64_t bi = side ? s.dst_idx[i] : s.src_idx[i];
        if (bi < 0 || static_cast<uint64_t>(bi) >= l.num_blocks) {
          throw invalid_argument("block " + std::to_string(bi) + " out of range for layer " + lname +
                                 (side ? ".dst" : ".src") + " (" + std::to_string(l.num_blocks) +
                                 " blocks registered)");
        }
        const UnitGeometry& g = (&l == &local) ? gl : gr;
        for (uint32_t u = 0; u < g.units; ++u) check_unit_range(l, static_cast<uint64_t>(bi), u, g);
      }
    }
    // A destination block listed twice keeps the later source block.
    const int64_t* dst_ids = s.dst_idx;
    std::vector<uint64_t> seen((s.dst.num_blocks >> 6) + 1, 0);
    std::vector<uint64_t> keep;
    for (uint64_t i = s.n; i-- > 0;) {
      const uint64_t d = static_cast<uint64_t>(dst_ids[i]);
      if (seen[d >> 6] & (1ull << (d & 63))) continue;
      seen[d >> 6] |= 1ull << (d & 63);
      keep.push_back(i);
    }
    std::reverse(keep.begin(), keep.end());
    const uint64_t n = keep.size();

    // Warps write destination units in no order, so the destination layout
    // must give every block its own bytes (the load path sends layouts that
    // share bytes through ordered copy-engine copies instead).
    uint64_t dst_k_region = 0;
    const bool dst_owns_bytes =
        is_split_layout(s.dst)
            ? !mul_ovf(s.dst.num_blocks, s.dst.bytes_per_block, &dst_k_region) && s.dst.kv_stride_bytes >= dst_k_region
            : s.dst.segments == 1;
    if (!dst_owns_bytes) {
      throw invalid_argument("peer transfer needs a destination layout whose blocks do not share bytes (layer " +
                             lname + ")");
    }
    // One device on both sides with overlapping tensors: a byte read by one
    // pair must not be written by another, or the result depends on timing.
    if (peer == device && s.src.data_ptr < s.dst.data_ptr + s.dst.size_bytes &&
        s.dst.data_ptr < s.src.data_ptr + s.src.size_bytes) {
      const UnitGeometry gs = save_geometry(s.src), gd = save_geometry(s.dst);
      std::vector<std::pair<uint64_t, uint64_t>> reads, writes;
      for (uint64_t j = 0; j < n; ++j) {
        const uint64_t sb = static_cast<uint64_t>(s.src_idx[keep[j]]);
        const uint64_t db = static_cast<uint64_t>(s.dst_idx[keep[j]]);
        for (uint32_t u = 0; u < gs.units; ++u) {
          const uint64_t r = s.src.data_ptr + sb * s.src.bytes_per_block + u * gs.unit_stride;
          const uint64_t w = s.dst.data_ptr + db * s.dst.bytes_per_block + u * gd.unit_stride;
          reads.emplace_back(r, r + gs.unit_bytes);
          writes.emplace_back(w, w + gd.unit_bytes);
        }
      }
      std::sort(reads.begin(), reads.end());
      std::sort(writes.begin(), writes.end());
      for (size_t i = 0, k = 0; i < reads.size() && k < writes.size();) {
        if (reads[i].second <= writes[k].first) {
          ++i;
        } else if (writes[k].second <= reads[i].first) {
          ++k;
        } else {
          throw invalid_argument("source and destination blocks overlap in layer " + lname);
        }
      }
    }

    PlanLayer p{};
    p.cache_base = local.data_ptr;
    p.block_pitch = local.bytes_per_block;
    p.unit_stride = gl.unit_stride;
    p.unit_bytes = static_cast<uint32_t>(gl.unit_bytes);
    p.units = gl.units;
    p.n = static_cast<uint32_t>(n);
    p.tiles_per_unit = static_cast<uint32_t>((gl.unit_bytes + kTileBytes - 1) / kTileBytes);
    p.tile_start = b->total_tiles;
    p.tile_count = static_cast<uint64_t>(gl.units) * n * p.tiles_per_unit;
    if (p.tile_count > 0xffffffffull) throw invalid_argument("layer transfer too large for one plan");
    p.ids_off = plan_offset(b->ids.size());
    p.side_off = plan_offset(b->side_base.size());
    p.unit_off = plan_offset(unit_base);
    p.done_index = static_cast<uint32_t>(li);
    p.side_pitch = gl.unit_bytes;
    bool vec = aligned16(local.data_ptr) && aligned16(local.bytes_per_block) && aligned16(gl.unit_stride) &&
               aligned16(gl.unit_bytes) && aligned16(remote.data_ptr) && aligned16(gr.unit_stride);
    for (uint32_t u = 0; u < gl.units; ++u) b->side_base.push_back(0);
    for (uint64_t j = 0; j < n; ++j) b->ids.push_back(static_cast<uint32_t>(local_ids[keep[j]]));
    for (uint32_t u = 0; u < gl.units; ++u) {
      for (uint64_t j = 0; j < n; ++j) {
        const uint64_t rb = static_cast<uint64_t>(remote_ids[keep[j]]);
        b->side_ptrs.push_back(remote.data_ptr + rb * remote.bytes_per_block + u * gr.unit_stride);
      }
    }
    p.flags = vec ? kFlagVector : 0u;
    b->total_tiles += p.tile_count;
    b->total_bytes += static_cast<uint64_t>(gl.units) * n * gl.unit_bytes;
    unit_base += static_cast<uint64_t>(gl.units) * n;
    check_plan_ends(b->ids, b->side_base, unit_base);
    b->layers.push_back(p);
  }
}

}  // namespace pf
