// Device-visible description of one block transfer (save or load).
//
// A transfer moves "units" between a paged KV tensor in HBM (the cache side)
// and a dense side (the HBM staging ring, or pinned host memory). A unit is
// the byte range the reference copies with one cudaMemcpy:
//   - split K/V layout (segments == 2 && kv_stride > bytes_per_block,
//     lib.rs:636, gpu_worker.rs:218,326): two units per block, K and V, each
//     bytes_per_block long, kv_stride apart in HBM;
//   - contiguous layout (transfer.rs:50-52): one unit of
//     bytes_per_block*segments per block;
//   - other strided layouts on save (transfer.rs:221-239): one unit per
//     segment, written back to back in the pool;
//   - other strided layouts on load: one unit of bytes_per_block*segments at
//     the block offset (gpu_worker.rs:260-282).
// Units are ordered layer-major, then unit-major (all K, then all V), then by
// position in the block list: the order in which the reference lays out the
// pool (lib.rs:671-679) and issues its copies (gpu_worker.rs:343-360).
//
// Units are cut into tiles of kTileBytes; the kernels schedule tiles, one warp
// per tile, so a 4 KiB TP-8 segment and a 64 KiB block both run full width.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace pf {

constexpr uint32_t kTileBytes = 4096;  // 32 lanes x 8 x 16 B

enum PlanFlags : uint32_t {
  kFlagVector = 1u,  // all addresses and unit_bytes are 16-byte multiples
};

struct PlanLayer {
  uint64_t cache_base;   // registration data_ptr (device address)
  uint64_t block_pitch;  // bytes_per_block: distance between blocks in HBM
  uint64_t unit_stride;  // distance between the units of one block in HBM
  uint64_t side_pitch;   // distance between blocks on the dense side (affine mode)
  uint64_t tile_start;   // global index of this layer's first tile
  uint64_t tile_count;   // units * n * tiles_per_unit
  uint32_t unit_bytes;   // bytes per unit
  uint32_t units;        // units per block
  uint32_t n;            // blocks in this layer
  uint32_t tiles_per_unit;
  uint32_t ids_off;      // first block index of this layer in the id array
  uint32_t side_off;     // first affine base of this layer (units entries)
  uint32_t unit_off;     // global index of this layer's first unit (table mode)
  uint32_t flags;        // PlanFlags
  uint32_t done_index;   // caller's layer index (per-layer completion flag)
  uint32_t pad[3];
};
static_assert(sizeof(PlanLayer) == 96, "PlanLayer layout");

// Kernel launch arguments (passed by value).
struct CopyArgs {
  const PlanLayer* layers;
  const uint32_t* ids;          // block indices, validated on the host
  const uint64_t* side_base;    // affine mode: per (layer, unit) base address
  const uint64_t* side_ptrs;    // table mode: per unit address
  unsigned long long* layer_tiles_done;  // per-layer completion counters, or null
  int64_t* layer_done;          // per-layer flags in mapped host memory, or null
  uint64_t tile_begin;
  uint64_t tile_end;
  int64_t side_shift;           // added to affine side addresses (staging slot)
  uint32_t n_layers;
  uint32_t pad;
  int* status;                  // bulk kernel: set to 1 when a bounded wait gave up, or null
  unsigned long long* span;     // {first CTA start, last CTA end} in %globaltimer ns, or null
  uint64_t stall_tile;          // bulk kernel test hook: tile (from tile_begin) whose copy is not issued
};

// Directions.
enum Dir : int { kPack = 0, kUnpack = 1 };

// Host entry: launch the copy kernel. table = side addresses come from
// side_ptrs (one per unit) instead of side_base + i*side_pitch; streaming =
// evict-first (.cs) loads and stores.
cudaError_t launch_copy(Dir dir, bool table, const CopyArgs& args, int grid,
                        cudaStream_t stream, bool streaming = false);

// The bulk-copy variant: tiles move through shared memory with TMA bulk
// copies (cp.async.bulk global -> shared -> global) instead of registers.
// Only for affine launches (no table) whose layers are all 16-byte aligned
// and that raise no per-layer flags; one CTA per SM.
cudaError_t launch_bulk_copy(Dir dir, const CopyArgs& args, int num_sms, cudaStream_t stream);
// Prepares the bulk kernels on the current device (their shared-memory
// size); false when the device cannot run them.
bool bulk_copy_ready();
// Tiles the bulk kernel keeps per CTA before it uses fewer CTAs.
uint64_t bulk_tiles_per_cta();

// CTAs of kv_copy_kernel resident per SM on the current device (the lowest
// over its instances); grids beyond SMs x this run as a partial second wave.
int copy_kernel_resident_ctas();

}  // namespace pf
