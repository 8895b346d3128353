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
// of tiles and its warps walk it interleaved, so neighbouring warps touch
// neighbouring bytes. Two kernels move the tiles:
//   kv_copy_kernel: per tile, one warp decodes (layer, unit, block) with
//     integer math, reads the block index once (a broadcast load), and moves
//     the tile with 8 x 16-byte loads per lane in flight before the 8 stores.
//     Handles every layout: unaligned units, zero-copy and peer tables,
//     per-layer completion flags.
//   kv_bulk_kernel: TMA bulk copies (cp.async.bulk) move each tile from
//     global memory into a per-warp ring of shared-memory stages and back
//     out, several tiles in flight per warp; for staged, 16-byte aligned
//     transfers without per-layer flags.
// Sorted and shuffled block lists cost the same: the block index only picks
// the tile's base address.
//
// Bounds: the host validates every (block, unit) range against the layer's
// registered size before launch; the kernel does no unchecked indexing beyond
// the plan it is given.
#include <cuda_runtime.h>

#include <algorithm>
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
// Unaligned units below this size (one tile each) are copied one per lane.
constexpr uint32_t kTinyUnitBytes = 16;
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

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Kernel-body timing (only while the executor times launches, a.span set):
// the CTA's first thread stamps its start into span[0] (min over CTAs); the
// last of the CTA's warps to finish, after a fence that waits for its writes,
// stamps span[1] (max over CTAs).
__device__ __forceinline__ void span_start(const CopyArgs& a, unsigned int* warps_done) {
  if (threadIdx.x == 0) {
    *warps_done = 0;
    atomicMin(&a.span[0], global_ns());
  }
  __syncthreads();
}

__device__ __forceinline__ void span_warp_done(const CopyArgs& a, unsigned int* warps_done, int lane,
                                               unsigned int warps) {
  if (a.span == nullptr) return;
  __threadfence();
  __syncwarp();
  if (lane == 0 && atomicAdd(warps_done, 1u) == warps - 1) atomicMax(&a.span[1], global_ns());
}

// SMEM: the CTA first copies the plan's layer table into shared memory with
// coalesced 16-byte loads (one round trip), so the per-warp layer lookups
// below hit shared memory instead of chaining dependent global loads.
// Four CTAs per SM (64 registers): 32 warps x 4 KiB of loads in flight per SM,
// and the default grid of 4 x SMs runs as exactly one wave.
template <int DIR, bool TABLE, bool SMEM, bool CS>
__global__ void __launch_bounds__(kThreads, kMinCtasPerSm) kv_copy_kernel(const CopyArgs a) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  __shared__ unsigned int warps_done;
  if (a.span) span_start(a, &warps_done);

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
  if (tile >= cta_end) {
    span_warp_done(a, &warps_done, lane, kWarpsPerCta);
    return;
  }

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
    if ((L.flags & kFlagVector) == 0 && L.unit_bytes < kTinyUnitBytes) {
      // Tiny unaligned units (4-byte per-block scales): one unit per tile,
      // so the warp's next tiles of this layer (up to 32) go one to a lane
      // instead of one tile per warp iteration.
      uint64_t lim = L.tile_start + L.tile_count;
      if (lim > cta_end) lim = cta_end;
      uint64_t cnt = (lim - tile + kWarpsPerCta - 1) / kWarpsPerCta;
      const uint32_t count = cnt < 32 ? (uint32_t)cnt : 32u;
      if ((uint32_t)lane < count) {
        const uint32_t unit_local = (uint32_t)(tile + (uint64_t)lane * kWarpsPerCta - L.tile_start);
        const uint32_t u = unit_local / L.n;
        const uint32_t i = unit_local - u * L.n;
        const uint64_t b = a.ids[L.ids_off + i];
        char* cache = reinterpret_cast<char*>(L.cache_base + b * L.block_pitch + (uint64_t)u * L.unit_stride);
        char* side = TABLE ? reinterpret_cast<char*>(a.side_ptrs[L.unit_off + unit_local])
                           : reinterpret_cast<char*>(a.side_base[L.side_off + u] + (uint64_t)i * L.side_pitch +
                                                     a.side_shift);
        for (uint32_t k = 0; k < L.unit_bytes; ++k) {
          if (DIR == kPack) side[k] = cache[k]; else cache[k] = side[k];
        }
      }
      done_in_layer += count;
      tile += (uint64_t)(count - 1) * kWarpsPerCta;  // the loop adds the last step
      continue;
    }
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
  span_warp_done(a, &warps_done, lane, kWarpsPerCta);
}

// ---------------------------------------------------------------------------
// Bulk-copy variant (TMA engine, no registers in the data path)
// ---------------------------------------------------------------------------
// One CTA per SM, kBulkWarps warps. Each warp owns a ring of kBulkStages
// 4 KiB stages in shared memory with one mbarrier per stage, and walks its
// tiles (the same CTA ranges and warp interleave as kv_copy_kernel) as a
// software pipeline run by lane 0: the bulk load of tile j is issued
// kBulkAhead tiles before its bulk store, so kBulkAhead x 4 KiB per warp are
// in flight on the load side while earlier stores drain. The 32 lanes decode
// the tiles 32 at a time (layer, unit, block id -> addresses) into a
// double-buffered descriptor table in shared memory, so the block-id loads of
// a batch overlap instead of sitting in lane 0's issue loop.
//
// Every wait on an mbarrier is bounded by time; a wait that runs out sets
// *status and the warp stops issuing, waits (bounded) for the loads it has in
// flight and returns, so the host sees an error instead of a hung stream.
constexpr int kBulkWarps = 6;
constexpr int kBulkThreads = kBulkWarps * 32;
constexpr int kBulkStages = 8;
constexpr int kBulkAhead = 6;
static_assert(kBulkAhead < kBulkStages, "a stage is reloaded only after its store has read it");
constexpr unsigned long long kBulkWaitNs = 1000000000ull;  // 1 s per mbarrier wait

struct BulkDesc {
  uint64_t src;
  uint64_t dst;
  uint32_t bytes;
  uint32_t pad[3];
};
static_assert(sizeof(BulkDesc) == 32, "BulkDesc layout");

constexpr size_t kBulkStageBytes = size_t(kBulkWarps) * kBulkStages * kTileBytes;
constexpr size_t kBulkBarBytes = size_t(kBulkWarps) * kBulkStages * sizeof(uint64_t);
constexpr size_t kBulkDescBytes = size_t(kBulkWarps) * 64 * sizeof(BulkDesc);
constexpr size_t kBulkSmemBytes = kBulkStageBytes + kBulkBarBytes + kBulkDescBytes;
static_assert(kBulkSmemBytes <= 227 * 1024, "bulk kernel shared memory");

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// true once the phase with `parity` has completed; false after kBulkWaitNs.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = global_ns();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (global_ns() - t0 > kBulkWaitNs) return false;
  }
}

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int DIR>
__global__ void __launch_bounds__(kBulkThreads, 1) kv_bulk_kernel(const CopyArgs a) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  __shared__ unsigned int warps_done;
  if (a.span) span_start(a, &warps_done);
  unsigned char* stages = g_smem + size_t(warp) * kBulkStages * kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(g_smem + kBulkStageBytes) + warp * kBulkStages;
  BulkDesc* descs = reinterpret_cast<BulkDesc*>(g_smem + kBulkStageBytes + kBulkBarBytes) + warp * 64;

  const uint64_t total = a.tile_end - a.tile_begin;
  const uint64_t per_cta = (total + gridDim.x - 1) / gridDim.x;
  const uint64_t cta_begin = a.tile_begin + (uint64_t)blockIdx.x * per_cta;
  uint64_t cta_end = cta_begin + per_cta;
  if (cta_end > a.tile_end) cta_end = a.tile_end;
  const uint64_t first = cta_begin + (uint64_t)warp;
  if (first >= cta_end) {
    span_warp_done(a, &warps_done, lane, kBulkWarps);
    return;
  }
  const uint64_t n = (cta_end - first + kBulkWarps - 1) / kBulkWarps;  // this warp's tiles

  if (lane == 0) {
    for (int st = 0; st < kBulkStages; ++st) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[st])) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();

  // Lane i decodes this warp's tile k0 + i into descs[buf*32 + i].
  auto decode = [&](uint64_t k0, int buf) {
    const uint64_t k = k0 + (uint64_t)lane;
    BulkDesc d{};
    if (k < n) {
      const uint64_t tile = first + k * kBulkWarps;
      uint32_t lo = 0, hi = a.n_layers;
      while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (a.layers[mid].tile_start <= tile) lo = mid; else hi = mid;
      }
      const PlanLayer& L = a.layers[lo];
      const uint32_t local = (uint32_t)(tile - L.tile_start);
      const uint32_t unit_local = local / L.tiles_per_unit;
      const uint32_t t = local - unit_local * L.tiles_per_unit;
      const uint32_t u = unit_local / L.n;
      const uint32_t i = unit_local - u * L.n;
      const uint64_t b = a.ids[L.ids_off + i];
      const uint32_t in_unit = t * kTileBytes;
      const uint32_t rest = L.unit_bytes - in_unit;
      const uint64_t cache = L.cache_base + b * L.block_pitch + (uint64_t)u * L.unit_stride + in_unit;
      const uint64_t side = a.side_base[L.side_off + u] + (uint64_t)i * L.side_pitch + in_unit + a.side_shift;
      d.src = DIR == kPack ? cache : side;
      d.dst = DIR == kPack ? side : cache;
      d.bytes = rest < kTileBytes ? rest : kTileBytes;
    }
    descs[buf * 32 + lane] = d;
    __syncwarp();
  };

  decode(0, 0);
  uint64_t loads_issued = 0, stores_issued = 0;
  int bad = 0;
  for (uint64_t j = 0; j < n + kBulkAhead && !bad; ++j) {
    if (j < n && j > 0 && (j & 31) == 0) decode(j, (int)((j >> 5) & 1));
    if (lane == 0) {
      if (j < n) {
        // Stage j % S was last read by the store of tile j - S; at most
        // S - A - 1 newer stores may still be reading their stages.
        const BulkDesc& d = descs[((j >> 5) & 1) * 32 + (j & 31)];
        const uint32_t st = (uint32_t)(j % kBulkStages);
        const uint32_t bar = smem_u32(&bars[st]);
        bulk_wait_read<kBulkStages - kBulkAhead - 1>();
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(d.bytes) : "memory");
        // The test hook leaves one armed barrier without its copy, so the
        // bounded wait below runs out; nothing else ever skips a copy.
        if (first + j * kBulkWarps - a.tile_begin != a.stall_tile) {
          asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                       ::"r"(smem_u32(stages + (size_t)st * kTileBytes)), "l"(d.src), "r"(d.bytes), "r"(bar)
                       : "memory");
        }
        loads_issued = j + 1;
      }
      if (j >= kBulkAhead) {
        const uint64_t t = j - kBulkAhead;
        const BulkDesc& d = descs[((t >> 5) & 1) * 32 + (t & 31)];
        const uint32_t st = (uint32_t)(t % kBulkStages);
        if (mbar_wait(smem_u32(&bars[st]), (uint32_t)((t / kBulkStages) & 1))) {
          asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                       ::"l"(d.dst), "r"(smem_u32(stages + (size_t)st * kTileBytes)), "r"(d.bytes)
                       : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          stores_issued = t + 1;
        } else {
          bad = 1;
        }
      }
    }
    bad = __shfl_sync(0xffffffffu, bad, 0);
  }
  if (lane == 0) {
    if (bad) {
      if (a.status) {
        *reinterpret_cast<volatile int*>(a.status) = 1;
        __threadfence_system();
      }
      // Loads still in flight land in this warp's stages: wait for them
      // (bounded) before the CTA's shared memory can be reused.
      for (uint64_t t = stores_issued; t < loads_issued; ++t) {
        mbar_wait(smem_u32(&bars[t % kBulkStages]), (uint32_t)((t / kBulkStages) & 1));
      }
    }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  __syncwarp();
  span_warp_done(a, &warps_done, lane, kBulkWarps);
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

bool bulk_copy_ready() {
  for (const void* fn : {reinterpret_cast<const void*>(&kv_bulk_kernel<kPack>),
                         reinterpret_cast<const void*>(&kv_bulk_kernel<kUnpack>)}) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBulkSmemBytes) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kBulkThreads, kBulkSmemBytes) != cudaSuccess || n < 1) {
      cudaGetLastError();
      return false;
    }
  }
  return true;
}

uint64_t bulk_tiles_per_cta() { return uint64_t(kBulkWarps) * 2 * kBulkStages; }

cudaError_t launch_bulk_copy(Dir dir, const CopyArgs& args, int num_sms, cudaStream_t stream) {
  if (args.tile_end <= args.tile_begin) return cudaSuccess;
  const uint64_t tiles = args.tile_end - args.tile_begin;
  const uint64_t need = (tiles + bulk_tiles_per_cta() - 1) / bulk_tiles_per_cta();
  const int grid = static_cast<int>(std::max<uint64_t>(1, std::min<uint64_t>(need, (uint64_t)num_sms)));
  if (dir == kPack) {
    kv_bulk_kernel<kPack><<<grid, kBulkThreads, kBulkSmemBytes, stream>>>(args);
  } else {
    kv_bulk_kernel<kUnpack><<<grid, kBulkThreads, kBulkSmemBytes, stream>>>(args);
  }
  return cudaGetLastError();
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
