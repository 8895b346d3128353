#include "offset_allocator.h"

#include <string>

#include "common.h"

namespace pf {

namespace {
constexpr uint32_t kMantissaBits = 3;
constexpr uint32_t kMantissaValue = 1u << kMantissaBits;
constexpr uint32_t kMantissaMask = kMantissaValue - 1;
constexpr uint32_t kNumLeafBins = 256;

inline uint32_t lzcnt32(uint32_t v) { return v ? static_cast<uint32_t>(__builtin_clz(v)) : 32u; }
inline uint32_t tzcnt32(uint32_t v) { return v ? static_cast<uint32_t>(__builtin_ctz(v)) : 32u; }

// Lowest set bit of `mask` at or after bit `start` (kNoSpace if none).
inline uint32_t lowest_bit_after(uint32_t mask, uint32_t start) {
  if (start >= 32) return OffsetAllocator::kNoSpace;
  const uint32_t after = mask & ~((1u << start) - 1u);
  return after ? tzcnt32(after) : OffsetAllocator::kNoSpace;
}
}  // namespace

uint32_t OffsetAllocator::uint_to_float_round_up(uint32_t size) {
  uint32_t exp = 0, mantissa = 0;
  if (size < kMantissaValue) {
    mantissa = size;
  } else {
    const uint32_t highest = 31 - lzcnt32(size);
    const uint32_t mantissa_start = highest - kMantissaBits;
    exp = mantissa_start + 1;
    mantissa = (size >> mantissa_start) & kMantissaMask;
    const uint32_t low_mask = (1u << mantissa_start) - 1u;
    if ((size & low_mask) != 0) mantissa += 1;  // may carry into the exponent
  }
  return (exp << kMantissaBits) + mantissa;
}

uint32_t OffsetAllocator::uint_to_float_round_down(uint32_t size) {
  uint32_t exp = 0, mantissa = 0;
  if (size < kMantissaValue) {
    mantissa = size;
  } else {
    const uint32_t highest = 31 - lzcnt32(size);
    const uint32_t mantissa_start = highest - kMantissaBits;
    exp = mantissa_start + 1;
    mantissa = (size >> mantissa_start) & kMantissaMask;
  }
  return (exp << kMantissaBits) | mantissa;
}

uint32_t OffsetAllocator::float_to_uint(uint32_t f) {
  const uint32_t exponent = f >> kMantissaBits;
  const uint32_t mantissa = f & kMantissaMask;
  if (exponent == 0) return mantissa;
  return (mantissa | kMantissaValue) << (exponent - 1);
}

OffsetAllocator::OffsetAllocator(uint32_t size, uint32_t max_allocs)
    : size_(size), max_allocs_(max_allocs < 2 ? 2 : max_allocs) {
  for (uint32_t i = 0; i < kNumLeafBins; ++i) bin_indices_[i] = kNoSpace;
  nodes_.assign(max_allocs_, Node{});
  free_nodes_.resize(max_allocs_);
  for (uint32_t i = 0; i < max_allocs_; ++i) free_nodes_[i] = max_allocs_ - i - 1;
  free_offset_ = max_allocs_ - 1;
  insert_node_into_bin(size_, 0);
}

uint32_t OffsetAllocator::insert_node_into_bin(uint32_t size, uint32_t data_offset) {
  const uint32_t bin = uint_to_float_round_down(size);
  const uint32_t top = bin >> 3, leaf = bin & 7;
  if (bin_indices_[bin] == kNoSpace) {
    used_bins_[top] |= static_cast<uint8_t>(1u << leaf);
    used_bins_top_ |= 1u << top;
  }
  const uint32_t head = bin_indices_[bin];
  const uint32_t node_index = free_nodes_[free_offset_];
  free_offset_ -= 1;
  Node n;
  n.data_offset = data_offset;
  n.data_size = size;
  n.bin_list_next = head;
  nodes_[node_index] = n;
  if (head != kNoSpace) nodes_[head].bin_list_prev = node_index;
  bin_indices_[bin] = node_index;
  free_storage_ += size;
  return node_index;
}

void OffsetAllocator::remove_node_from_bin(uint32_t node_index) {
  Node& node = nodes_[node_index];
  if (node.bin_list_prev != kNoSpace) {
    nodes_[node.bin_list_prev].bin_list_next = node.bin_list_next;
    if (node.bin_list_next != kNoSpace) nodes_[node.bin_list_next].bin_list_prev = node.bin_list_prev;
  } else {
    const uint32_t bin = uint_to_float_round_down(node.data_size);
    const uint32_t top = bin >> 3, leaf = bin & 7;
    bin_indices_[bin] = node.bin_list_next;
    if (node.bin_list_next != kNoSpace) nodes_[node.bin_list_next].bin_list_prev = kNoSpace;
    if (bin_indices_[bin] == kNoSpace) {
      used_bins_[top] &= static_cast<uint8_t>(~(1u << leaf));
      if (used_bins_[top] == 0) used_bins_top_ &= ~(1u << top);
    }
  }
  free_offset_ += 1;
  free_nodes_[free_offset_] = node_index;
  free_storage_ -= node.data_size;
}

OffsetAllocator::Allocation OffsetAllocator::allocate(uint32_t size) {
  Allocation none;
  if (free_offset_ == 0) return none;  // out of nodes
  const uint32_t min_bin = uint_to_float_round_up(size);
  const uint32_t min_top = min_bin >> 3, min_leaf = min_bin & 7;
  uint32_t top = min_top;
  uint32_t leaf = kNoSpace;
  if (top < 32 && (used_bins_top_ & (1u << top))) leaf = lowest_bit_after(used_bins_[top], min_leaf);
  if (leaf == kNoSpace) {
    top = lowest_bit_after(used_bins_top_, min_top + 1);
    if (top == kNoSpace) return none;
    leaf = tzcnt32(used_bins_[top]);
  }
  const uint32_t bin = (top << 3) | leaf;
  const uint32_t node_index = bin_indices_[bin];
  Node& node = nodes_[node_index];
  const uint32_t node_total = node.data_size;
  node.data_size = size;
  node.used = true;
  bin_indices_[bin] = node.bin_list_next;
  if (node.bin_list_next != kNoSpace) nodes_[node.bin_list_next].bin_list_prev = kNoSpace;
  free_storage_ -= node_total;
  if (bin_indices_[bin] == kNoSpace) {
    used_bins_[top] &= static_cast<uint8_t>(~(1u << leaf));
    if (used_bins_[top] == 0) used_bins_top_ &= ~(1u << top);
  }
  const uint32_t remainder = node_total - size;
  if (remainder > 0) {
    const uint32_t nn = insert_node_into_bin(remainder, node.data_offset + size);
    Node& n2 = nodes_[node_index];  // same storage; no reallocation happens
    if (n2.neighbor_next != kNoSpace) nodes_[n2.neighbor_next].neighbor_prev = nn;
    nodes_[nn].neighbor_prev = node_index;
    nodes_[nn].neighbor_next = n2.neighbor_next;
    n2.neighbor_next = nn;
  }
  Allocation a;
  a.offset = nodes_[node_index].data_offset;
  a.metadata = node_index;
  return a;
}

void OffsetAllocator::free(Allocation a) {
  if (a.metadata == kNoSpace) return;
  const uint32_t node_index = a.metadata;
  Node& node = nodes_[node_index];
  if (!node.used) return;  // double free: ignore
  uint32_t offset = node.data_offset;
  uint32_t size = node.data_size;
  if (node.neighbor_prev != kNoSpace && !nodes_[node.neighbor_prev].used) {
    const Node prev = nodes_[node.neighbor_prev];
    offset = prev.data_offset;
    size += prev.data_size;
    remove_node_from_bin(node.neighbor_prev);
    node.neighbor_prev = prev.neighbor_prev;
  }
  if (node.neighbor_next != kNoSpace && !nodes_[node.neighbor_next].used) {
    const Node next = nodes_[node.neighbor_next];
    size += next.data_size;
    remove_node_from_bin(node.neighbor_next);
    node.neighbor_next = next.neighbor_next;
  }
  const uint32_t neighbor_next = node.neighbor_next;
  const uint32_t neighbor_prev = node.neighbor_prev;
  node.used = false;
  free_offset_ += 1;
  free_nodes_[free_offset_] = node_index;
  const uint32_t combined = insert_node_into_bin(size, offset);
  if (neighbor_next != kNoSpace) {
    nodes_[combined].neighbor_next = neighbor_next;
    nodes_[neighbor_next].neighbor_prev = combined;
  }
  if (neighbor_prev != kNoSpace) {
    nodes_[combined].neighbor_prev = neighbor_prev;
    nodes_[neighbor_prev].neighbor_next = combined;
  }
}

uint32_t OffsetAllocator::allocation_size(Allocation a) const {
  if (a.metadata == kNoSpace) return 0;
  return nodes_[a.metadata].data_size;
}

OffsetAllocator::Report OffsetAllocator::storage_report() const {
  Report r{0, 0};
  if (free_offset_ > 0) {
    r.total_free_space = free_storage_;
    if (used_bins_top_) {
      const uint32_t top = 31 - lzcnt32(used_bins_top_);
      const uint32_t leaf = 31 - lzcnt32(used_bins_[top]);
      r.largest_free_region = float_to_uint((top << 3) | leaf);
    }
  }
  return r;
}

// ---------------------------------------------------------------------------

ScaledOffsetAllocator ScaledOffsetAllocator::make(uint64_t total_bytes, uint64_t unit_size, bool auto_unit,
                                                  uint32_t max_allocs) {
  const uint64_t max_units = 0xffffffffull;
  if (auto_unit) unit_size = total_bytes > max_units ? (total_bytes + max_units - 1) / max_units : 1;
  if (unit_size == 0) throw Error(PF_ERR_INVALID_ARGUMENT, "unit size must be greater than zero");
  const uint64_t units = (total_bytes + unit_size - 1) / unit_size;
  if (units > max_units) {
    throw Error(PF_ERR_INVALID_ARGUMENT, "capacity " + std::to_string(total_bytes) + " bytes with unit " +
                                             std::to_string(unit_size) + " overflows u32 backing allocator");
  }
  return ScaledOffsetAllocator(unit_size, static_cast<uint32_t>(units), max_allocs ? max_allocs : 128 * 1024);
}

bool ScaledOffsetAllocator::allocate(uint64_t size_bytes, Allocation* out) {
  if (size_bytes == 0) return false;
  const uint64_t units = (size_bytes + unit_size_ - 1) / unit_size_;
  if (units > 0xffffffffull) {
    throw Error(PF_ERR_INVALID_ARGUMENT, "request " + std::to_string(size_bytes) + " bytes with unit " +
                                             std::to_string(unit_size_) + " overflows u32 backing allocator");
  }
  const OffsetAllocator::Allocation raw = inner_.allocate(static_cast<uint32_t>(units));
  if (raw.offset == OffsetAllocator::kNoSpace) return false;
  out->raw = raw;
  out->offset_bytes = static_cast<uint64_t>(raw.offset) * unit_size_;
  out->size_bytes = static_cast<uint64_t>(inner_.allocation_size(raw)) * unit_size_;
  return true;
}

void ScaledOffsetAllocator::free(const Allocation& a) { inner_.free(a.raw); }

uint64_t ScaledOffsetAllocator::total_free_bytes() const {
  return static_cast<uint64_t>(inner_.storage_report().total_free_space) * unit_size_;
}

uint64_t ScaledOffsetAllocator::largest_free_bytes() const {
  return static_cast<uint64_t>(inner_.storage_report().largest_free_region) * unit_size_;
}

}  // namespace pf
