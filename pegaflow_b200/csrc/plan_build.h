// Host-side transfer plans: the layout rules of the reference, the checks a
// transfer passes before any byte moves, and the arrays the copy kernel and
// the copy engine follow (plan.h). No CUDA calls: the one check that needs
// the CUDA runtime (is this address device memory of that GPU?) is passed in.
#pragma once

#include <cstdint>
#include <functional>
#include <vector>

#include "pegaflow.h"
#include "plan.h"

namespace pf {

// Geometry of one layer of a transfer, derived from its registration the
// way the reference chooses its copy loop (gpu_worker.rs:218,326; transfer.rs:50-52).
struct UnitGeometry {
  uint32_t units;        // units per block
  uint64_t unit_bytes;   // bytes per unit
  uint64_t unit_stride;  // HBM distance between units of a block
};
UnitGeometry save_geometry(const pf_layer_desc& l);
UnitGeometry load_geometry(const pf_layer_desc& l);
bool is_split_layout(const pf_layer_desc& l);       // lib.rs:636
bool is_contiguous_layout(const pf_layer_desc& l);  // transfer.rs:50-52

// Layout checks of register_context_layer (lib.rs:389-449).
void validate_layout(const pf_layer_desc& l, const char* layer_name);
// transfer::segment_offset (transfer.rs:18-47).
uint64_t segment_offset(const pf_layer_desc& l, uint64_t block_idx, uint64_t segment_idx);

struct Run {  // one contiguous (dense offset, host address, bytes) extent
  uint64_t dense;
  uint64_t host;
  uint64_t bytes;
};
// A load layer whose destination blocks share bytes: copied in list order.
struct SerialLoad {
  pf_layer_desc layer;
  uint32_t done_index;
  std::vector<int64_t> ids;
  std::vector<uint64_t> k, v;
};
// A checked transfer plan: the kernel's layer table, block ids and dense
// (or host) addresses, the host extents the copy engine moves (staged mode),
// and the load layers that must be copied in list order instead.
struct Built {
  std::vector<PlanLayer> layers;
  std::vector<uint32_t> ids;
  std::vector<uint64_t> side_base;
  std::vector<uint64_t> side_ptrs;
  std::vector<Run> runs;  // staged mode only
  std::vector<SerialLoad> serial;
  uint64_t total_tiles = 0;
  uint64_t total_bytes = 0;
};

// Throws unless the layer's KV tensor is device memory of `device`.
using DeviceCheck = std::function<void(int device, const pf_layer_desc& layer)>;

// Plans of a save, a load, and a peer copy between `device` and `peer`
// (pull: device holds the destination; push: device holds the source).
// staged: the dense side is the HBM staging ring (copy-engine runs are
// planned); otherwise the kernel reads or writes the host side directly.
void plan_save(const pf_save_layer* layers, uint64_t n_layers, bool staged, int device,
               const DeviceCheck& check_device_range, Built* b);
void plan_load(const pf_load_layer* layers, uint64_t n_layers, bool staged, int device,
               const DeviceCheck& check_device_range, Built* b);
void plan_p2p(const pf_p2p_layer* layers, uint64_t n_layers, int device, int peer, bool push,
              const DeviceCheck& check_device_range, Built* b);

}  // namespace pf
