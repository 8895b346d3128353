// Staging chunks of a staged transfer: how a plan's tiles are cut into the
// pieces that pass through one HBM staging slot at a time (one kernel launch
// and one set of copy-engine copies each). Host-only, no CUDA.
#pragma once

#include <cstdint>
#include <vector>

#include "plan.h"

namespace pf {

// Each layer's units start at a multiple of this in the dense order (the
// order of the pool and the staging slots), and every chunk's dense start is
// rounded down to it, so relocating a chunk into a slot keeps 16-byte
// alignment.
constexpr uint64_t kDenseAlign = 256;

inline uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// Tiles [tile_begin, tile_end), whose dense bytes are [dense_first, dense_end).
// dense_begin is dense_first rounded down to kDenseAlign: the chunk is placed
// in a slot at (dense - dense_begin), which keeps 16-byte alignment, but the
// bytes in [dense_begin, dense_first) belong to the previous chunk. Copies
// between the slot and the host move [dense_first, dense_end) only.
struct Chunk {
  uint64_t tile_begin, tile_end;
  uint64_t dense_begin, dense_end;
  uint64_t dense_first;
};

// Cuts the plan's tiles, in order, into chunks whose dense span fits a limit
// that starts at first_limit (at least two tiles, at most slot_bytes) and
// doubles with each chunk up to slot_bytes. A unit may be split between
// chunks at a tile boundary. `layers` are the plan's layers in dense order,
// with units laid out back to back from each layer's kDenseAlign-aligned
// start; total_tiles is the plan's tile count.
void cut_chunks(const std::vector<PlanLayer>& layers, uint64_t total_tiles, uint64_t slot_bytes,
                uint64_t first_limit, std::vector<Chunk>* chunks);

// First-chunk limit for a load that raises per-layer flags: the dense span of
// layer 0 and of the layers listed right after it that are at most an eighth
// of its size (per-block scales beside their KV), so the first chunk ends
// where those layers end; at least min_first, at most first_chunk.
uint64_t layerwise_first_limit(const std::vector<PlanLayer>& layers, uint64_t first_chunk, uint64_t min_first);

}  // namespace pf
