// sm_100a pack/unpack kernels for paged-KV block transfers.
//
// One kernel, two directions:
//   kPack   : cache (paged KV in HBM) -> dense side   (save, replaces the
//             per-segment cuMemcpyDtoH loop of gpu_worker.rs:343-360)
//   kUnpack : dense side -> cache                      (load, replaces the
//             per-run cuMemcpyHtoDAsync loop of transfer.rs:116-198)
// The dense side is either the HBM staging ring (the copy engine moves it
// across the host link) or mapped pinned host memory (zero-copy).
//
// Work is split into 4 KiB tiles (plan.h). Each CTA owns a contiguous range
// of tiles and its 8 warps walk it interleaved, so neighbouring warps touch
// neighbouring bytes. Per tile, one warp decodes (layer, unit, block) with
// integer math, reads the block index once (a broadcast load), and moves the
// tile with 8 x 16-byte loads per lane in flight before the 8 stores.
// Sorted and shuffled block lists cost the same: the block index only picks
// the tile's base address.
//
// Bounds: the host validates every (block, unit) range against the layer's
// registered size before launch; the kernel does no unchecked indexing beyond
// the plan it is given.
#include <cuda_runtime.h>

#include <cstdint>

#include "plan.h"

namespace pf {
namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kThreads = kWarpsPerCta * 32;
constexpr int kMinCtasPerSm = 4;
constexpr int kVecPerLane = kTileBytes / (32 * 16);  // 8
static_assert(kVecPerLane == 8, "tile = 32 lanes x 8 x 16 B");
static_assert(sizeof(PlanLayer) % 16 == 0, "layer table is copied in 16-byte words");
// Layer tables up to 48 KiB (512 layers) go to shared memory without opt-in.
constexpr size_t kMaxSmemTableBytes = 48 * 1024;

// 16-byte load of data read exactly once: kept out of L1; with CS (cache
// streaming) also marked evict-first in L2.
template <bool CS>
__device__ __forceinline__ uint4 ld_v4(const char* p) {
  uint4 v;
  if (CS) {
    asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
  } else {
    asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
  }
  return v;
}

template <bool CS>
__device__ __forceinline__ void st_v4(char* p, const uint4& v) {
  if (CS) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
  } else {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
  }
}

template <bool CS>
__device__ __forceinline__ void copy_tile(char* dst, const char* src,
                                          uint32_t bytes, bool vec, int lane) {
  if (vec) {
    if (bytes == kTileBytes) {
      uint4 r[kVecPerLane];
#pragma unroll
      for (int k = 0; k < kVecPerLane; ++k) r[k] = ld_v4<CS>(src + (k * 32 + lane) * 16);
#pragma unroll
      for (int k = 0; k < kVecPerLane; ++k) st_v4<CS>(dst + (k * 32 + lane) * 16, r[k]);
    } else {
      // Tail of a unit: bytes is a multiple of 16 below one tile.
      for (uint32_t off = lane * 16u; off < bytes; off += 512u) st_v4<CS>(dst + off, ld_v4<CS>(src + off));
    }
  } else {
    // Unaligned layouts (e.g. 4-byte per-block scales): byte granularity.
    for (uint32_t off = lane; off < bytes; off += 32u) dst[off] = src[off];
  }
}

// Count `done` finished tiles of layer l; the warp that completes the layer
// raises its flag in host memory after a system-scope fence, so a host poller
// that sees the flag also sees every byte of the layer.
__device__ __forceinline__ void flush_layer(const CopyArgs& a, uint32_t l,
                                            uint64_t layer_tiles, uint32_t done_index,
                                            uint32_t done, int lane) {
  if (a.layer_tiles_done == nullptr || done == 0) return;
  __threadfence();
  __syncwarp();
  if (lane == 0) {
    const unsigned long long prev = atomicAdd(&a.layer_tiles_done[l], (unsigned long long)done);
    if (prev + done == layer_tiles) {
      __threadfence_system();
      *reinterpret_cast<volatile int64_t*>(a.layer_done + done_index) = 1;
      __threadfence_system();
    }
  }
  __syncwarp();
}

extern __shared__ __align__(16) unsigned char g_smem[];

// SMEM: the CTA first copies the plan's layer table into shared memory with
// coalesced 16-byte loads (one round trip), so the per-warp layer lookups
// below hit shared memory instead of chaining dependent global loads.
// Four CTAs per SM (64 registers): 32 warps x 4 KiB of loads in flight per SM,
// and the default grid of 4 x SMs runs as exactly one wave.
template <int DIR, bool TABLE, bool SMEM, bool CS>
__global__ void __launch_bounds__(kThreads, kMinCtasPerSm) kv_copy_kernel(const CopyArgs a) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;

  const PlanLayer* layers = a.layers;
  if (SMEM) {
    const uint32_t n16 = a.n_layers * (uint32_t)(sizeof(PlanLayer) / 16);
    const uint4* src = reinterpret_cast<const uint4*>(a.layers);
    uint4* dst = reinterpret_cast<uint4*>(g_smem);
    for (uint32_t i = threadIdx.x; i < n16; i += kThreads) dst[i] = src[i];
    __syncthreads();
    layers = reinterpret_cast<const PlanLayer*>(g_smem);
  }

  const uint64_t total = a.tile_end - a.tile_begin;
  const uint64_t per_cta = (total + gridDim.x - 1) / gridDim.x;
  const uint64_t cta_begin = a.tile_begin + (uint64_t)blockIdx.x * per_cta;
  uint64_t cta_end = cta_begin + per_cta;
  if (cta_end > a.tile_end) cta_end = a.tile_end;

  uint64_t tile = cta_begin + (uint64_t)warp;
  if (tile >= cta_end) return;

  // Layer of the first tile: last l with tile_start <= tile.
  uint32_t lo = 0, hi = a.n_layers;
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) >> 1;
    if (layers[mid].tile_start <= tile) lo = mid; else hi = mid;
  }
  uint32_t l = lo;
  // The layer entry is read in place (shared memory when SMEM) on every tile
  // rather than held in 24 registers: a few shared loads per 4 KiB moved keep
  // the kernel within 64 registers without spilling.
  const PlanLayer* Lp = &layers[l];
  uint32_t done_in_layer = 0;

  for (; tile < cta_end; tile += kWarpsPerCta) {
    while (tile >= Lp->tile_start + Lp->tile_count) {
      flush_layer(a, l, Lp->tile_count, Lp->done_index, done_in_layer, lane);
      done_in_layer = 0;
      ++l;
      Lp = &layers[l];
    }
    const PlanLayer& L = *Lp;
    const uint32_t local = (uint32_t)(tile - L.tile_start);
    const uint32_t unit_local = local / L.tiles_per_unit;
    const uint32_t t = local - unit_local * L.tiles_per_unit;
    const uint32_t u = unit_local / L.n;
    const uint32_t i = unit_local - u * L.n;
    const uint64_t b = a.ids[L.ids_off + i];
    const uint32_t in_unit = t * kTileBytes;
    const uint32_t rest = L.unit_bytes - in_unit;
    const uint32_t bytes = rest < kTileBytes ? rest : kTileBytes;

    char* cache = reinterpret_cast<char*>(L.cache_base + b * L.block_pitch +
                                          (uint64_t)u * L.unit_stride + in_unit);
    char* side;
    if (TABLE) {
      side = reinterpret_cast<char*>(a.side_ptrs[L.unit_off + unit_local] + in_unit);
    } else {
      side = reinterpret_cast<char*>(a.side_base[L.side_off + u] + (uint64_t)i * L.side_pitch +
                                     in_unit + a.side_shift);
    }
    if (DIR == kPack) {
      copy_tile<CS>(side, cache, bytes, (L.flags & kFlagVector) != 0, lane);
    } else {
      copy_tile<CS>(cache, side, bytes, (L.flags & kFlagVector) != 0, lane);
    }
    ++done_in_layer;
  }
  flush_layer(a, l, Lp->tile_count, Lp->done_index, done_in_layer, lane);
}

// Runtime flags -> template instance.
template <int DIR, bool TABLE, bool SMEM>
void launch_cs(bool cs, const CopyArgs& a, int grid, size_t shm, cudaStream_t s) {
  if (cs) {
    kv_copy_kernel<DIR, TABLE, SMEM, true><<<grid, kThreads, shm, s>>>(a);
  } else {
    kv_copy_kernel<DIR, TABLE, SMEM, false><<<grid, kThreads, shm, s>>>(a);
  }
}

template <int DIR, bool TABLE>
void launch_smem(bool smem, bool cs, const CopyArgs& a, int grid, size_t shm, cudaStream_t s) {
  if (smem) {
    launch_cs<DIR, TABLE, true>(cs, a, grid, shm, s);
  } else {
    launch_cs<DIR, TABLE, false>(cs, a, grid, shm, s);
  }
}

}  // namespace

int copy_kernel_resident_ctas() {
  // The fewest CTAs per SM any instance keeps resident, with a full 48 KiB
  // layer table in shared memory (the largest dynamic size launch_copy asks for).
  int lowest = kMinCtasPerSm * 4;
  auto take = [&](const void* fn, size_t shm) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kThreads, shm) != cudaSuccess) {
      cudaGetLastError();
      return;
    }
    if (n > 0 && n < lowest) lowest = n;
  };
  take(reinterpret_cast<const void*>(&kv_copy_kernel<kPack, false, true, false>), kMaxSmemTableBytes);
  take(reinterpret_cast<const void*>(&kv_copy_kernel<kUnpack, false, true, false>), kMaxSmemTableBytes);
  take(reinterpret_cast<const void*>(&kv_copy_kernel<kUnpack, true, true, false>), kMaxSmemTableBytes);
  take(reinterpret_cast<const void*>(&kv_copy_kernel<kPack, true, true, true>), kMaxSmemTableBytes);
  take(reinterpret_cast<const void*>(&kv_copy_kernel<kPack, false, false, false>), 0);
  return lowest;
}

cudaError_t launch_copy(Dir dir, bool table, const CopyArgs& args, int grid,
                        cudaStream_t stream, bool streaming) {
  if (args.tile_end <= args.tile_begin) return cudaSuccess;
  if (grid < 1) grid = 1;
  const size_t table_bytes = static_cast<size_t>(args.n_layers) * sizeof(PlanLayer);
  const bool smem = table_bytes <= kMaxSmemTableBytes;
  const size_t shm = smem ? table_bytes : 0;
  if (dir == kPack) {
    if (table) {
      launch_smem<kPack, true>(smem, streaming, args, grid, shm, stream);
    } else {
      launch_smem<kPack, false>(smem, streaming, args, grid, shm, stream);
    }
  } else {
    if (table) {
      launch_smem<kUnpack, true>(smem, streaming, args, grid, shm, stream);
    } else {
      launch_smem<kUnpack, false>(smem, streaming, args, grid, shm, stream);
    }
  }
  return cudaGetLastError();
}

}  // namespace pf
