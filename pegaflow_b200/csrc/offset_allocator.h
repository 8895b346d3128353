// Offset allocator for the pinned pool.
//
// The reference wraps the third-party crate `offset-allocator` 0.2.0 (a Rust
// port of Sebastian Aaltonen's MIT-licensed OffsetAllocator) in a byte-scaling
// layer (pegaflow-core/src/allocator.rs). The crate is not vendored in the
// reference tree; this file restates its published algorithm in our own code:
//   - sizes are binned with a small float: 5-bit exponent, 3-bit mantissa,
//     256 bins in 32 top bins x 8 leaf bins, found with two bitmasks;
//   - allocation rounds the request up to a bin, takes the first free node of
//     the lowest non-empty bin at or above it, and returns the remainder to
//     its own (round-down) bin;
//   - free merges the node with free physical neighbours before re-binning;
//   - the storage report's "largest free region" is the size of the highest
//     non-empty bin, i.e. a lower bound of the largest node.
// It decides pool addresses only, never bytes.
#pragma once

#include <cstdint>
#include <vector>

namespace pf {

class OffsetAllocator {
 public:
  static constexpr uint32_t kNoSpace = 0xffffffffu;

  struct Allocation {
    uint32_t offset = kNoSpace;
    uint32_t metadata = kNoSpace;  // node index
  };
  struct Report {
    uint32_t total_free_space;
    uint32_t largest_free_region;
  };

  OffsetAllocator(uint32_t size, uint32_t max_allocs);
  Allocation allocate(uint32_t size);
  void free(Allocation a);
  uint32_t allocation_size(Allocation a) const;
  Report storage_report() const;

  static uint32_t uint_to_float_round_up(uint32_t size);
  static uint32_t uint_to_float_round_down(uint32_t size);
  static uint32_t float_to_uint(uint32_t f);

 private:
  struct Node {
    uint32_t data_offset = 0;
    uint32_t data_size = 0;
    uint32_t bin_list_prev = kNoSpace;
    uint32_t bin_list_next = kNoSpace;
    uint32_t neighbor_prev = kNoSpace;
    uint32_t neighbor_next = kNoSpace;
    bool used = false;
  };
  uint32_t insert_node_into_bin(uint32_t size, uint32_t data_offset);
  void remove_node_from_bin(uint32_t node_index);

  uint32_t size_;
  uint32_t max_allocs_;
  uint32_t free_storage_ = 0;
  uint32_t used_bins_top_ = 0;
  uint8_t used_bins_[32] = {};
  uint32_t bin_indices_[256];
  std::vector<Node> nodes_;
  std::vector<uint32_t> free_nodes_;
  uint32_t free_offset_;
};

// ScaledOffsetAllocator (allocator.rs:66-170): byte API over u32 units.
class ScaledOffsetAllocator {
 public:
  struct Allocation {
    uint64_t offset_bytes;
    uint64_t size_bytes;
    OffsetAllocator::Allocation raw;
  };
  // unit_size 0 selects ceil(total/u32::MAX) (allocator.rs:89-97).
  // Throws pf::Error(PF_ERR_INVALID_ARGUMENT) for unit 0 passed explicitly via
  // make() and when the unit count overflows u32 (allocator.rs:105-124).
  static ScaledOffsetAllocator make(uint64_t total_bytes, uint64_t unit_size, bool auto_unit,
                                    uint32_t max_allocs);

  // Returns false when nothing fits (Ok(None)); throws for a request beyond
  // u32 units (AllocatorError::RequestTooLarge). size 0 returns false.
  bool allocate(uint64_t size_bytes, Allocation* out);
  void free(const Allocation& a);
  uint64_t total_bytes() const { return unit_size_ * total_units_; }
  uint64_t unit_size() const { return unit_size_; }
  uint64_t total_free_bytes() const;
  uint64_t largest_free_bytes() const;

 private:
  ScaledOffsetAllocator(uint64_t unit, uint32_t units, uint32_t max_allocs)
      : unit_size_(unit), total_units_(units), inner_(units, max_allocs) {}
  uint64_t unit_size_;
  uint32_t total_units_;
  OffsetAllocator inner_;
};

}  // namespace pf
