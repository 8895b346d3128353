/*
 * pegaflow.h — C ABI of the B200-native KV-cache block transfer path.
 *
 * This is the drop-in boundary for PegaFlow's GPU<->pinned-host block path.
 * Every entry point below names the reference interface it replaces
 * (paths are relative to the xiaguan/pegaflow source tree). All arguments are
 * plain pointers, sizes and C strings; no framework types cross this line.
 *
 * Conventions
 *   - Every function that can fail returns a pf_status (0 = PF_OK). The
 *     message of the last failure on the calling thread is returned by
 *     pf_last_error(); its text follows EngineError's Display impl
 *     (pegaflow-core/src/lib.rs:69-83), e.g. "instance X not found".
 *   - Device addresses are uint64_t (CUdeviceptr-like), host addresses are
 *     void*. Pinned pool memory is mapped into the unified address space, so a
 *     pool pointer is valid on every device.
 *   - Thread safety: a pf_engine may be called from many threads at once
 *     (the reference engine is Sync). A pf_executor may be too: it
 *     serialises the calls of each of its two lanes (saves; loads and peer
 *     copies) and runs the lanes side by side.
 */
#ifndef PEGAFLOW_B200_H
#define PEGAFLOW_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PF_ABI_VERSION 4

/* ------------------------------------------------------------------------ */
/* Status codes: one per EngineError variant (pegaflow-core/src/lib.rs:58-67) */
/* ------------------------------------------------------------------------ */
typedef enum pf_status {
  PF_OK = 0,
  PF_ERR_INSTANCE_MISSING = 1,  /* EngineError::InstanceMissing */
  PF_ERR_WORKER_MISSING = 2,    /* EngineError::WorkerMissing */
  PF_ERR_INVALID_ARGUMENT = 3,  /* EngineError::InvalidArgument */
  PF_ERR_CUDA_INIT = 4,         /* EngineError::CudaInit */
  PF_ERR_STORAGE = 5,           /* EngineError::Storage (copy failures included) */
  PF_ERR_POISONED = 6,          /* EngineError::Poisoned */
  PF_ERR_TOPOLOGY_MISMATCH = 7, /* EngineError::TopologyMismatch */
  PF_ERR_LOAD_STATE = 8,        /* LoadStateError (pegaflow-core/src/sync_state.rs:46-56) */
  PF_ERR_TIMEOUT = 9,           /* a bounded wait ran out (no reference counterpart) */
  PF_ERR_NO_SPACE = 10          /* allocator could not satisfy a request (allocator.rs:138-140) */
} pf_status;

/* Message of the last failed call on this thread ("" if none). */
const char* pf_last_error(void);
/* PF_ABI_VERSION of the loaded library. */
int pf_abi_version(void);
/* Number of CUDA devices visible to the library (0 when none). */
int pf_device_count(void);

/* ------------------------------------------------------------------------ */
/* Layer layout = KVCacheRegistration (pegaflow-core/src/lib.rs:100-112)     */
/* ------------------------------------------------------------------------ */
typedef struct pf_layer_desc {
  uint64_t data_ptr;        /* device address of the layer's KV tensor */
  uint64_t size_bytes;      /* bytes registered at data_ptr */
  uint64_t num_blocks;      /* paged blocks in the layer */
  uint64_t bytes_per_block; /* bytes of one segment of one block */
  uint64_t kv_stride_bytes; /* distance K->V for KV-first layouts, 0 otherwise */
  uint64_t segments;        /* 1 = blocks-first, 2 = KV-first */
} pf_layer_desc;

/* Layout checks of PegaEngine::register_context_layer
 * (pegaflow-core/src/lib.rs:389-449). PF_ERR_INVALID_ARGUMENT on failure. */
int pf_layer_validate(const pf_layer_desc* layer, const char* layer_name);

/* transfer::segment_offset (pegaflow-core/src/transfer.rs:18-47):
 * block_idx*bytes_per_block + segment_idx*kv_stride_bytes, checked against
 * size_bytes. PF_ERR_STORAGE with the reference's message on failure. */
int pf_segment_offset(const pf_layer_desc* layer, uint64_t block_idx,
                      uint64_t segment_idx, uint64_t* out_offset);

/* ------------------------------------------------------------------------ */
/* Transfer executor: replaces GpuWorkerPool's copy loops                    */
/* (pegaflow-core/src/gpu_worker.rs:52-390, transfer.rs:56-239)              */
/* ------------------------------------------------------------------------ */
typedef struct pf_executor pf_executor;

/* How the bytes cross the host link. */
typedef enum pf_transfer_mode {
  PF_MODE_AUTO = 0,   /* library default per direction */
  PF_MODE_STAGED = 1, /* sm_100a pack/unpack kernel <-> HBM staging ring <-> copy engine DMA */
  PF_MODE_DIRECT = 2  /* sm_100a kernel loads/stores mapped pinned host memory (zero-copy) */
} pf_transfer_mode;

/* How the pack/unpack kernels move a staged transfer's 4 KiB tiles:
 * REGISTERS: each warp loads a tile into registers (8 x 16 B per lane) and
 * stores it; BULK: TMA bulk copies (cp.async.bulk) move each tile from global
 * memory into a shared-memory ring and back out, several tiles in flight per
 * warp, no registers in the data path. AUTO picks BULK where it applies
 * (staged transfers whose layers are all 16-byte aligned and that raise no
 * per-layer flags) and REGISTERS elsewhere. */
typedef enum pf_copy_kernel {
  PF_COPY_KERNEL_AUTO = 0,
  PF_COPY_KERNEL_REGISTERS = 1,
  PF_COPY_KERNEL_BULK = 2
} pf_copy_kernel;

typedef struct pf_executor_config {
  /* Saves and loads each have their own staging slots (allocated on first
   * use), so a save and a load on two streams run at the same time. */
  uint64_t staging_chunk_bytes; /* slot size, 0 = default (1 GiB) */
  uint32_t staging_slots;       /* slots per direction, 0 = default (2) */
  uint32_t save_mode;           /* pf_transfer_mode */
  uint32_t load_mode;           /* pf_transfer_mode */
  uint32_t ctas_per_sm;         /* 0 = default */
  uint32_t copy_streams;        /* 0 = default (2) */
  uint32_t cache_streaming;     /* 1 = evict-first loads/stores in the kernels */
  uint32_t copy_kernel;         /* pf_copy_kernel: how staged tiles move through the SM */
  /* Size limit of the first staged chunk of a load; each later chunk may be
   * twice the previous one, up to staging_chunk_bytes. A small first chunk
   * raises the first per-layer flags early; large later chunks keep the
   * kernel launch count low. Saves start at the larger of this and half a
   * slot; loads without per-layer flags use whole slots. A load given
   * per-layer flags starts at the smaller of this and its first layer plus
   * the small layers listed right after it (at least 4 MiB), so its first
   * flag rises after that layer's DMA alone when the layer fits.
   * 0 = default (256 MiB: a whole first layer of the benchmark shapes,
   * 40 MiB for Llama-3.1-8B and 128 MiB for Llama-3-70B at TP1). */
  uint64_t first_chunk_bytes;
} pf_executor_config;

/* Fill *cfg with the library defaults. */
void pf_executor_config_default(pf_executor_config* cfg);

/* One executor per device (replaces GpuWorkerPool::spawn,
 * gpu_worker.rs:61-93, which starts a load thread and a save thread per GPU).
 * It has two lanes, each with its own streams, staging ring and plan buffers:
 * saves use one, loads and peer copies the other. Calls on one lane run in
 * the order they were made; a save and a load, issued from different threads
 * or on different streams, run at the same time, one per direction of the
 * host link. */
int pf_executor_create(int32_t device_id, const pf_executor_config* cfg,
                       pf_executor** out);
void pf_executor_destroy(pf_executor* exec);

/* One layer of a save task = SaveTask{registration, blocks} (gpu_worker.rs:32-44).
 * Block i of the list lands at  k_dst + i*pitch  (and v_dst + i*bytes_per_block
 * for the split K/V layout), which is exactly the SaveBlock pointers the
 * engine builds (lib.rs:671-679, 739-747): pitch = bytes_per_block for the
 * split layout, bytes_per_block*segments otherwise. */
typedef struct pf_save_layer {
  pf_layer_desc layer;
  const int64_t* block_idx; /* n block indices, each in [0, num_blocks) */
  uint64_t n;
  void* k_dst;              /* pinned host destination of block 0 (K region) */
  void* v_dst;              /* pinned host V region (split layout), else NULL */
} pf_save_layer;

/* One layer of a load task = LayerLoadData{registration, blocks}
 * (gpu_worker.rs:18-28). k_src[i]/v_src[i] are LayerBlock::k_ptr/v_ptr;
 * a NULL v_src (array or entry) means k_src[i] + bytes_per_block, as in
 * gpu_worker.rs:233-236. */
typedef struct pf_load_layer {
  pf_layer_desc layer;
  const int64_t* block_idx;
  uint64_t n;
  const void* const* k_src;
  const void* const* v_src;
} pf_load_layer;

/* GPU -> pinned host, blocking until the bytes are in host memory.
 * Replaces process_save_task (gpu_worker.rs:321-390): one pipelined pass over
 * all layers instead of one synchronous cuMemcpyDtoH per segment. */
int pf_save_blocks(pf_executor* exec, const pf_save_layer* layers,
                   uint64_t n_layers);

/* Pinned host -> GPU, blocking until the bytes are in HBM.
 * Replaces process_load_task (gpu_worker.rs:205-317). */
int pf_load_blocks(pf_executor* exec, const pf_load_layer* layers,
                   uint64_t n_layers);

/* Stream-ordered variants. The work starts after everything already queued
 * on `stream` (a cudaStream_t, NULL = legacy default stream) and `stream`
 * waits for its completion, so CUDA events on `stream` bracket the whole
 * transfer. Host buffers and index arrays may be reused when the call returns.
 * layer_done, if not NULL, must be mapped pinned host memory of n_layers
 * int64 words; word l is set to 1 once layer l's bytes are in place (the
 * per-layer signal that the reference lacks, worker.py:288-289). */
int pf_save_blocks_async(pf_executor* exec, const pf_save_layer* layers,
                         uint64_t n_layers, void* stream);
int pf_load_blocks_async(pf_executor* exec, const pf_load_layer* layers,
                         uint64_t n_layers, void* stream, int64_t* layer_done);

/* Prefill -> decode handoff between two GPUs over NVLink, paged cache to
 * paged cache (no reference counterpart: the reference hands P/D blocks over
 * through its host pool, docs/pd.md:20-27). For every layer, block
 * src_idx[i] of `src` (on the source GPU) lands in block dst_idx[i] of `dst`
 * (on the destination GPU); both layouts must have the same bytes_per_block,
 * segments and K/V split. One kernel moves the bytes with 16-byte peer loads
 * (pull: runs on the destination GPU, exec is its executor) or peer stores
 * (push: runs on the source GPU). A destination listed twice keeps the later
 * block. Work is ordered after `stream` and `stream` waits for it (NULL =
 * blocking call). Peer access between the two devices is enabled on first
 * use; PF_ERR_INVALID_ARGUMENT when the devices cannot reach each other. */
typedef struct pf_p2p_layer {
  pf_layer_desc src;
  pf_layer_desc dst;
  const int64_t* src_idx;
  const int64_t* dst_idx;
  uint64_t n;
} pf_p2p_layer;
int pf_p2p_transfer(pf_executor* exec, int32_t peer_device, int push,
                    const pf_p2p_layer* layers, uint64_t n_layers, void* stream);

/* Save without allocating: for callers that cannot call cudaMalloc while
 * they save, e.g. an inference engine whose caching allocator or KV pool owns
 * all free HBM, or code under a pool policy that forbids out-of-band device
 * allocations. No counterpart in the reference (its saves always go through
 * its worker threads). Same copies and pool bytes as pf_save_blocks, issued in
 * order on `stream` (a cudaStream_t; NULL = legacy default stream); the call
 * returns once they are queued. Scratch is two fixed file-scope device arrays
 * that every GPU loading this library holds until exit: a 1 MiB plan area and
 * an 8 MiB staging slot. A save whose plan (layer table + block ids + offsets)
 * exceeds 1 MiB, or with a copy unit above 4 MiB, fails with
 * PF_ERR_INVALID_ARGUMENT. The first call on a device resolves the arrays'
 * addresses (cudaGetSymbolAddress). The arrays are reserved in device memory when that first call loads the
 * library's device code on the device (CUDA loads modules lazily), so make
 * the first call before the caller's allocator claims HBM: the warm-up call
 * pf_save_blocks_noalloc(device, NULL, 0, stream) loads the code, reserves
 * the arrays and moves nothing. Later calls take no device memory.
 * All calls on a device share the arrays, so calls that overlap on the GPU
 * race; keep them ordered on one stream. Calls no cudaMalloc or cudaFree.
 * The caller's current device is current again when the call returns. */
int pf_save_blocks_noalloc(int32_t device_id, const pf_save_layer* layers,
                           uint64_t n_layers, void* stream);

/* Counters since creation (or the last reset). kernel_ms is the sum of the
 * pack/unpack kernels' CUDA-event durations, collected only while timing is
 * on; kernel_bytes counts the algorithmic HBM bytes those kernels moved
 * (payload read + payload written). */
typedef struct pf_executor_stats {
  uint64_t kernel_launches;
  uint64_t copy_calls;
  uint64_t bytes_saved;
  uint64_t bytes_loaded;
  uint64_t kernel_bytes;
  double kernel_ms;
  uint64_t timed_launches;
  uint64_t bytes_p2p;       /* payload moved by pf_p2p_transfer */
  double host_ms;           /* calling-thread time inside save/load/p2p: checks, plan, enqueue */
  /* While timing is on, each kernel also stamps %globaltimer when its first
   * CTA starts and its last CTA ends: kernel_body_ms sums those spans over
   * body_launches launches. The CUDA-event duration (kernel_ms) adds the
   * launch's own latency, which grows while the copy engines stream. */
  double kernel_body_ms;
  uint64_t body_launches;
} pf_executor_stats;
int pf_executor_stats_get(pf_executor* exec, pf_executor_stats* out);
int pf_executor_stats_reset(pf_executor* exec);
/* Record CUDA events around each kernel launch (on the kernel's stream). */
int pf_executor_set_timing(pf_executor* exec, int enabled);

/* Test hook for the bulk kernel's bounded waits (no counterpart in the
 * reference). The next bulk-kernel launch of this executor arms the mbarrier
 * of the launch's tile `tile` (counted from the launch's first tile) but
 * issues no copy into it, so the wait for that tile runs out after 1 s; the
 * warp then stops, the kernel returns, and the executor fails the call with
 * PF_ERR_STORAGE. No fault and no hang: the barrier is simply never
 * completed. UINT64_MAX (the default) disarms it. */
int pf_executor_debug_stall_tile(pf_executor* exec, uint64_t tile);

/* ------------------------------------------------------------------------ */
/* Reference copy strategy, restated for side-by-side timing on one box      */
/* ------------------------------------------------------------------------ */
/* Save exactly as process_save_task does: one synchronous cudaMemcpy D2H per
 * K segment, then per V segment (gpu_worker.rs:343-360; contiguous layouts
 * per block, transfer.rs:200-239). */
int pf_refcopy_save(int32_t device_id, const pf_save_layer* layers,
                    uint64_t n_layers);
/* Load exactly as process_load_task does: per layer, K then V lists merged
 * into maximal runs (transfer.rs:116-198), one async H2D per run on one
 * stream, one event synchronize at the end (gpu_worker.rs:286-291).
 * *out_runs (if not NULL) receives the number of copies issued. */
int pf_refcopy_load(int32_t device_id, const pf_load_layer* layers,
                    uint64_t n_layers, uint64_t* out_runs);

/* ------------------------------------------------------------------------ */
/* Pinned host memory (pegaflow-core/src/pinned_mem.rs:128-208)              */
/* ------------------------------------------------------------------------ */
/* Allocate pinned host memory that every device can reach (portable+mapped;
 * write_combined mirrors the reference default cudaHostAllocWriteCombined). */
int pf_pinned_alloc(uint64_t size, int write_combined, void** out);
int pf_pinned_free(void* ptr);

/* ------------------------------------------------------------------------ */
/* Offset allocator = ScaledOffsetAllocator over offset-allocator 0.2.0      */
/* (pegaflow-core/src/allocator.rs:66-170)                                    */
/* ------------------------------------------------------------------------ */
typedef struct pf_allocator pf_allocator;
/* unit_size PF_ALLOCATOR_AUTO_UNIT = smallest unit keeping the unit count
 * within u32 (ScaledOffsetAllocator::new, allocator.rs:77-86); an explicit 0
 * is rejected with PF_ERR_INVALID_ARGUMENT (AllocatorError::InvalidUnitSize).
 * max_allocs 0 = 128*1024 (allocator.rs:85). */
#define PF_ALLOCATOR_AUTO_UNIT UINT64_MAX
int pf_allocator_create(uint64_t total_bytes, uint64_t unit_size,
                        uint32_t max_allocs, pf_allocator** out);
void pf_allocator_destroy(pf_allocator* a);
/* PF_ERR_NO_SPACE when nothing fits (Ok(None) in the reference);
 * PF_ERR_INVALID_ARGUMENT for size 0 or a request beyond u32 units. */
int pf_allocator_alloc(pf_allocator* a, uint64_t size, uint64_t* out_offset,
                       uint64_t* out_size, uint32_t* out_handle);
void pf_allocator_free(pf_allocator* a, uint32_t handle);
void pf_allocator_report(pf_allocator* a, uint64_t* total_free_bytes,
                         uint64_t* largest_free_bytes, uint64_t* total_bytes,
                         uint64_t* unit_size);

/* ------------------------------------------------------------------------ */
/* LoadState: shared-memory completion flag, byte-compatible with            */
/* pegaflow-core/src/sync_state.rs (magic 'PFLD', version 1, i64 state)      */
/* ------------------------------------------------------------------------ */
#define PF_LOAD_STATE_PENDING 0
#define PF_LOAD_STATE_SUCCESS 1
#define PF_LOAD_STATE_ERROR (-1)

typedef struct pf_load_state pf_load_state;
/* LoadState::new (sync_state.rs:125-142): creates "pega_load_<uuid>". */
int pf_load_state_create(pf_load_state** out);
/* LoadState::attach (sync_state.rs:145-155) with the same checks. */
int pf_load_state_attach(const char* shm_name, pf_load_state** out);
/* LoadState with a per-layer extension (no reference counterpart; the
 * reference has no per-layer signal, worker.py:288-289). The first 32 bytes
 * are the version-1 mapping unchanged, so a reference reader still attaches;
 * after them: u32 'PFL2', u32 n_layers, 8 reserved bytes, then one i64 per
 * layer of the load request (in layer_names order): 0 pending, 1 in place. */
int pf_load_state_create_layers(uint32_t n_layers, pf_load_state** out);
/* Layers in the extension (0 for a version-1-only mapping). */
uint32_t pf_load_state_layer_count(const pf_load_state* s);
/* Word of one layer (PF_LOAD_STATE_ERROR when out of range). */
int64_t pf_load_state_layer_get(const pf_load_state* s, uint32_t layer);
const char* pf_load_state_name(const pf_load_state* s);
int64_t pf_load_state_get(const pf_load_state* s);
void pf_load_state_set_completed(pf_load_state* s);
void pf_load_state_set_error(pf_load_state* s);
/* Unmaps; the creating handle also unlinks the shm object (owner drop). */
void pf_load_state_close(pf_load_state* s);

/* ------------------------------------------------------------------------ */
/* Engine = PegaEngine (pegaflow-core/src/lib.rs:93-1069)                     */
/* ------------------------------------------------------------------------ */
typedef struct pf_engine pf_engine;

typedef enum pf_pool_kind {
  PF_POOL_PINNED = 0, /* cudaHostAlloc'd pool (the product path) */
  PF_POOL_HOST = 1    /* plain pageable host memory: host-logic tests only;
                         every save/load on it fails with PF_ERR_CUDA_INIT */
} pf_pool_kind;

typedef struct pf_engine_config {
  uint64_t pool_bytes;            /* 0 = 30 GiB (lib.rs:56) */
  int32_t use_hugepages;          /* mmap(MAP_HUGETLB)+register (pinned_mem.rs:165-197) */
  int32_t write_combined;         /* reference default 1 (pinned_mem.rs:159) */
  int32_t enable_lfu_admission;   /* StorageConfig default 1 (storage.rs:91) */
  int32_t pool_kind;              /* pf_pool_kind */
  uint64_t hint_value_size_bytes; /* allocator unit hint, 0 = none (storage.rs:84) */
  int32_t pre_evict_enabled;      /* PreEvictConfig (storage.rs:43-76) */
  /* Pool placement for an engine that drives several GPUs (no reference
   * counterpart; the reference allocates one pool): 0 = one pool (default);
   * 1 = one pool per NUMA node of the visible GPUs, each on its node, sized
   * by its GPU count; 2 = one pool per GPU, on that GPU's node. A save
   * allocates from its GPU's pool, and reclaim for a pool evicts only blocks
   * held there. With every GPU on one node, 1 is the same as 0. Placed
   * pools are page-locked with cudaHostRegister, so not write-combined. */
  int32_t numa_pools;
  uint64_t pre_evict_threshold_bytes;
  uint64_t pre_evict_target_bytes;
  uint64_t pre_evict_interval_ms;
  pf_executor_config executor;    /* used for every device the engine opens */
  /* Packed-file tier: sealed blocks are written through to packed files and
   * read back on a query miss (the reference's DFS offload, seal_offload.rs,
   * file format unchanged; the per-block metadata it keeps in Redis lives in
   * a sidecar file beside each packed file). NULL or "" = off. */
  const char* dfs_root;
  uint64_t dfs_quota_bytes;       /* 0 = 50 GiB (server --dfs-quota default) */
  uint64_t dfs_scan_interval_ms;  /* 0 = 100 */
  uint32_t dfs_max_pack_size;     /* blocks per packed file, 0 = 64 */
  uint32_t reserved1;
} pf_engine_config;

void pf_engine_config_default(pf_engine_config* cfg);
/* PegaEngine::new_with_config (lib.rs:294-308). */
int pf_engine_create(const pf_engine_config* cfg, pf_engine** out);
void pf_engine_destroy(pf_engine* e);

typedef struct pf_bytes {
  const uint8_t* data;
  uint64_t len;
} pf_bytes;

/* PegaEngine::register_context_layer (lib.rs:373-469). */
int pf_engine_register_context_layer(
    pf_engine* e, const char* instance_id, const char* ns, int32_t device_id,
    const char* layer_name, uint64_t data_ptr, uint64_t size_bytes,
    uint64_t num_blocks, uint64_t bytes_per_block, uint64_t kv_stride_bytes,
    uint64_t segments, uint64_t tp_rank, uint64_t tp_size,
    uint64_t num_layers);

/* PegaEngine::unregister_instance (lib.rs:473-484). */
int pf_engine_unregister_instance(pf_engine* e, const char* instance_id);

/* One (layer_name, block_ids, block_hashes) entry of a batch save
 * (lib.rs:502; engine.proto SaveLayer). The two lists carry their own
 * lengths; an entry whose lengths differ fails with the reference's
 * "block_ids length .. does not match block_hashes .." after the entries
 * before it have been saved (lib.rs:563-569). */
typedef struct pf_save_entry {
  const char* layer_name;
  const int32_t* block_ids;
  uint64_t n_ids;
  const pf_bytes* block_hashes;
  uint64_t n_hashes;
} pf_save_entry;

/* PegaEngine::batch_save_kv_blocks_from_ipc (lib.rs:497-520). Blocking. */
int pf_engine_batch_save_kv_blocks(pf_engine* e, const char* instance_id,
                                   uint64_t tp_rank, int32_t device_id,
                                   const pf_save_entry* saves,
                                   uint64_t n_saves);

/* PegaEngine::save_kv_blocks_from_ipc (lib.rs:528-550). Blocking. */
int pf_engine_save_kv_blocks(pf_engine* e, const char* instance_id,
                             uint64_t tp_rank, int32_t device_id,
                             const char* layer_name, const int32_t* block_ids,
                             const pf_bytes* block_hashes, uint64_t n);

/* PegaEngine::count_prefix_hit_blocks (lib.rs:803-838). */
int pf_engine_count_prefix_hit_blocks(pf_engine* e, const char* instance_id,
                                      const pf_bytes* block_hashes, uint64_t n,
                                      uint64_t* out_hits);

/* PrefetchStatus (seal_offload.rs:584-601) as engine.proto's QueryResponse
 * carries it (service.rs:283-297). */
typedef enum pf_prefetch_state {
  PF_PREFETCH_READY = 0,        /* hit_blocks are in the pool */
  PF_PREFETCH_LOADING = 1,      /* loading_blocks are being read back from packed files */
  PF_PREFETCH_PARTIAL_MISS = 2  /* missing_blocks are in neither */
} pf_prefetch_state;
typedef struct pf_prefetch_status {
  uint32_t state; /* pf_prefetch_state */
  uint32_t reserved;
  uint64_t hit_blocks;
  uint64_t loading_blocks;
  uint64_t missing_blocks;
} pf_prefetch_status;
/* PegaEngine::count_prefix_hit_blocks_async (lib.rs:855-942): with the
 * packed-file tier on, a miss that the tier holds starts a background read
 * of the rest of the prefix and reports LOADING (ask again later); with the
 * tier off it is count_prefix_hit_blocks reported as READY. */
int pf_engine_query_prefetch(pf_engine* e, const char* instance_id, const pf_bytes* block_hashes,
                             uint64_t n, pf_prefetch_status* out);

typedef struct pf_dfs_stats {
  uint64_t files;             /* packed files indexed */
  uint64_t blocks;            /* blocks indexed */
  uint64_t usage_bytes;       /* bytes in indexed packed files */
  uint64_t written_files;
  uint64_t written_blocks;
  uint64_t write_failures;
  uint64_t prefetched_blocks; /* blocks read back into the pool */
  uint64_t prefetch_failures;
  uint64_t evicted_files;     /* removed by the quota */
} pf_dfs_stats;
/* Tier counters (PF_ERR_INVALID_ARGUMENT when the tier is off). */
int pf_engine_dfs_stats(pf_engine* e, pf_dfs_stats* out);
/* Waits up to timeout_s for queued writes and reads; *out_idle = 1 if done. */
int pf_engine_dfs_flush(pf_engine* e, double timeout_s, int* out_idle);
/* Runs the quota check now (it also runs every dfs_scan_interval_ms). */
int pf_engine_dfs_check_quota(pf_engine* e);

/* PegaEngine::batch_load_kv_blocks_multi_layer (lib.rs:957-1069).
 * Returns after the task is queued; completion is written to the LoadState
 * named load_state_shm (1 = success, -1 = error). */
int pf_engine_batch_load_kv_blocks(pf_engine* e, const char* instance_id,
                                   uint64_t tp_rank, int32_t device_id,
                                   const char* load_state_shm,
                                   const char* const* layer_names,
                                   uint64_t n_layers, const int32_t* block_ids,
                                   const pf_bytes* block_hashes,
                                   uint64_t n_blocks);

/* The gRPC server's Save and Load RPCs (pegaflow-server/src/service.rs,
 * Save and Load handlers), taking the request's protobuf wire bytes
 * (engine.proto SaveRequest / LoadRequest) instead of decoded arguments. The
 * library decodes them (fields in any order, packed or unpacked ids, unknown
 * fields skipped) and runs batch_save_kv_blocks / batch_load_kv_blocks with
 * the same results and errors; a malformed request is
 * PF_ERR_INVALID_ARGUMENT. Layers of a Save whose hash lists are identical
 * share one list. A Load's block ids and hashes are paired up to the shorter
 * of the two lists (the reference zips them, lib.rs:1032-1033). */
int pf_engine_save_request(pf_engine* e, const uint8_t* request, uint64_t len);
int pf_engine_load_request(pf_engine* e, const uint8_t* request, uint64_t len);
/* Field 1 (instance_id) of a Save or Load request's wire bytes, copied into
 * out (NUL-terminated, at most cap bytes with the NUL); *out_len is its
 * length. PF_ERR_INVALID_ARGUMENT when it does not fit or the bytes are
 * malformed. */
int pf_request_instance_id(const uint8_t* request, uint64_t len, char* out, uint64_t cap,
                           uint64_t* out_len);

/* Block until every queued load on device_id has finished (bounded by
 * timeout_s; PF_ERR_TIMEOUT otherwise). No reference counterpart. */
int pf_engine_wait_loads(pf_engine* e, int32_t device_id, double timeout_s);

/* Pool usage (PinnedMemoryPool::usage / largest_free_allocation,
 * pinned_pool.rs:171-185); with numa_pools, used and total sum the pools and
 * largest_free is the largest of them. */
int pf_engine_pool_usage(pf_engine* e, uint64_t* used, uint64_t* total,
                         uint64_t* largest_free);

/* Host pointers of a sealed block's slot (LayerBlock k_ptr/v_ptr/size,
 * storage.rs:249-310); v_ptr = 0 for contiguous blocks. PF_ERR_STORAGE when
 * the block is not sealed in the cache. Does not touch LRU order. */
int pf_engine_slot_info(pf_engine* e, const char* ns, const uint8_t* hash,
                        uint64_t hash_len, uint64_t slot, uint64_t* k_ptr,
                        uint64_t* v_ptr, uint64_t* size);

/* Core counters (metrics.rs:7-99, kept as plain counters). */
typedef struct pf_engine_metrics {
  uint64_t save_bytes;
  uint64_t save_calls;
  double save_ms;
  uint64_t load_bytes;
  uint64_t load_calls;
  double load_ms;
  uint64_t load_failures;
  uint64_t cache_block_hits;
  uint64_t cache_block_misses;
  uint64_t cache_block_insertions;
  uint64_t cache_block_admission_rejections;
  uint64_t cache_block_evictions;
  uint64_t pool_alloc_failures;
  uint64_t inflight_blocks;
  uint64_t cached_blocks;
  double save_plan_ms;      /* dedup + pool allocation (host) */
  double save_transfer_ms;  /* pack kernels + D2H, waited on */
  double save_insert_ms;    /* slot bookkeeping after the copy (host) */
  uint64_t inflight_dropped; /* inflight blocks released after the age limit (ABI 3) */
  /* Load phases (ABI 4), summed over load calls: */
  double load_lookup_ms;      /* cache lookup + task build on the caller's thread */
  double load_queue_ms;       /* task queued until the device's load thread takes it */
  double load_setup_ms;       /* LoadState attach + pool pointer tables (load thread) */
  double load_transfer_ms;    /* executor load: plan, H2D + unpack, waited on */
  double load_first_layer_ms; /* task queued until its first layer is marked ready */
} pf_engine_metrics;
int pf_engine_metrics_get(pf_engine* e, pf_engine_metrics* out);

/* The executor the engine uses for device_id (created on first
 * registration), for stats/timing. */
int pf_engine_executor(pf_engine* e, int32_t device_id, pf_executor** out);

#ifdef __cplusplus
}
#endif

#endif /* PEGAFLOW_B200_H */
