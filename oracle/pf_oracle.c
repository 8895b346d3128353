/*
 * pf_oracle.c — CPU restatement of PegaFlow's KV block transfer path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the
 * B200 library and the timed CPU baseline; the product never links it.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use it.
 *
 * The "GPU memory" of a layer is a host byte array here; copies are memcpy.
 * Every function names the reference code it restates (paths relative to
 * the xiaguan/pegaflow tree). Parity status: KV-byte parity unpinned. The
 * reference ships no golden
 * vectors for KV bytes (its 13 unit tests cover LoadState headers, allocator
 * arithmetic and size parsing only), and its Rust sources cannot be built
 * here, so byte-level parity of this restatement is pinned by copy identity
 * and by the reference's own caller code (tests/golden), not by reference
 * outputs.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct or_layout {
  uint64_t size_bytes;
  uint64_t num_blocks;
  uint64_t bytes_per_block;
  uint64_t kv_stride_bytes;
  uint64_t segments;
} or_layout;

enum { OR_OK = 0, OR_INVALID_ARGUMENT = 3, OR_STORAGE = 5 };

static int set_err(char* err, size_t n, int code, const char* fmt, ...)
    __attribute__((format(printf, 4, 5)));
#include <stdarg.h>
static int set_err(char* err, size_t n, int code, const char* fmt, ...) {
  if (err && n) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, n, fmt, ap);
    va_end(ap);
  }
  return code;
}

/* register_context_layer layout checks (pegaflow-core/src/lib.rs:389-449). */
int or_validate_layout(const or_layout* l, const char* name, char* err, size_t errlen) {
  uint64_t block_size, max_block, max_seg, max_off, end;
  if (l->bytes_per_block == 0 || l->num_blocks == 0 || l->segments == 0)
    return set_err(err, errlen, OR_INVALID_ARGUMENT, "invalid argument: invalid KV cache layout for layer %s", name);
  if (l->segments > 1 && l->kv_stride_bytes == 0)
    return set_err(err, errlen, OR_INVALID_ARGUMENT,
                   "invalid argument: kv_stride_bytes must be > 0 when segments > 1 for layer %s", name);
  if (__builtin_mul_overflow(l->bytes_per_block, l->segments, &block_size))
    return set_err(err, errlen, OR_INVALID_ARGUMENT,
                   "invalid argument: block size overflow: bytes_per_block=%llu segments=%llu for layer %s",
                   (unsigned long long)l->bytes_per_block, (unsigned long long)l->segments, name);
  if (__builtin_mul_overflow(l->num_blocks - 1, l->bytes_per_block, &max_block))
    return set_err(err, errlen, OR_INVALID_ARGUMENT, "invalid argument: num_blocks %llu too large for layer %s",
                   (unsigned long long)l->num_blocks, name);
  if (__builtin_mul_overflow(l->segments - 1, l->kv_stride_bytes, &max_seg))
    return set_err(err, errlen, OR_INVALID_ARGUMENT,
                   "invalid argument: segments/stride overflow for layer %s (segments=%llu, stride=%llu)", name,
                   (unsigned long long)l->segments, (unsigned long long)l->kv_stride_bytes);
  if (__builtin_add_overflow(max_block, max_seg, &max_off))
    return set_err(err, errlen, OR_INVALID_ARGUMENT, "invalid argument: layout offset overflow for layer %s", name);
  if (__builtin_add_overflow(max_off, l->bytes_per_block, &end))
    return set_err(err, errlen, OR_INVALID_ARGUMENT, "invalid argument: layout end overflow for layer %s", name);
  if (end > l->size_bytes)
    return set_err(err, errlen, OR_INVALID_ARGUMENT,
                   "invalid argument: registered memory too small for layer %s: need at least %llu bytes, got %llu",
                   name, (unsigned long long)end, (unsigned long long)l->size_bytes);
  return OR_OK;
}

/* transfer::segment_offset (pegaflow-core/src/transfer.rs:18-47). */
int or_segment_offset(const or_layout* l, uint64_t block, uint64_t seg, uint64_t* out, char* err, size_t errlen) {
  uint64_t base, so, off, end;
  if (seg >= l->segments) return set_err(err, errlen, OR_STORAGE, "Segment index out of range");
  if (__builtin_mul_overflow(block, l->bytes_per_block, &base))
    return set_err(err, errlen, OR_STORAGE, "Block offset overflow");
  if (__builtin_mul_overflow(seg, l->kv_stride_bytes, &so))
    return set_err(err, errlen, OR_STORAGE, "Segment offset overflow");
  if (__builtin_add_overflow(base, so, &off)) return set_err(err, errlen, OR_STORAGE, "Combined offset overflow");
  if (__builtin_add_overflow(off, l->bytes_per_block, &end) || end > l->size_bytes)
    return set_err(err, errlen, OR_STORAGE,
                   "Block %llu segment %llu exceeds registered memory (offset %llu, size %llu, limit %llu)",
                   (unsigned long long)block, (unsigned long long)seg, (unsigned long long)off,
                   (unsigned long long)l->bytes_per_block, (unsigned long long)l->size_bytes);
  *out = off;
  return OR_OK;
}

/* Split K/V predicate (lib.rs:636; gpu_worker.rs:218,326). */
int or_is_split(const or_layout* l) { return l->segments == 2 && l->kv_stride_bytes > l->bytes_per_block; }

/* is_contiguous_layout (transfer.rs:50-52). */
int or_is_contiguous(const or_layout* l) { return l->segments <= 1 || l->kv_stride_bytes == l->bytes_per_block; }

/*
 * process_save_task (gpu_worker.rs:321-372) for the SaveBlock pointers the
 * engine builds (lib.rs:671-679, 739-747): block i of the list goes to
 * k_dst + i*seg and v_dst + i*seg (split), or k_dst + i*block_size.
 * Returns the number of copies the reference issues (>= 0) or -code.
 */
int64_t or_save_layer(const or_layout* l, const uint8_t* gpu, const int64_t* ids, uint64_t n, uint8_t* k_dst,
                      uint8_t* v_dst, char* err, size_t errlen) {
  const uint64_t seg = l->bytes_per_block;
  const uint64_t block_size = l->bytes_per_block * l->segments;
  int64_t copies = 0;
  uint64_t off, i, s;
  int rc;
  if (or_is_split(l)) {
    /* offsets first (gpu_worker.rs:334-341), then all K, then all V */
    uint64_t* ko = (uint64_t*)malloc(sizeof(uint64_t) * (n ? n : 1));
    uint64_t* vo = (uint64_t*)malloc(sizeof(uint64_t) * (n ? n : 1));
    for (i = 0; i < n; ++i) {
      if ((rc = or_segment_offset(l, (uint64_t)ids[i], 0, &ko[i], err, errlen)) ||
          (rc = or_segment_offset(l, (uint64_t)ids[i], 1, &vo[i], err, errlen))) {
        free(ko);
        free(vo);
        return -rc;
      }
    }
    for (i = 0; i < n; ++i, ++copies) memcpy(k_dst + i * seg, gpu + ko[i], seg);
    for (i = 0; i < n; ++i, ++copies) {
      uint8_t* dst = v_dst ? v_dst + i * seg : k_dst + i * seg + seg; /* gpu_worker.rs:354-356 */
      memcpy(dst, gpu + vo[i], seg);
    }
    free(ko);
    free(vo);
    return copies;
  }
  /* copy_block_gpu_to_cpu (transfer.rs:200-239) */
  for (i = 0; i < n; ++i) {
    uint8_t* dst = k_dst + i * block_size;
    if (or_is_contiguous(l)) {
      if ((rc = or_segment_offset(l, (uint64_t)ids[i], 0, &off, err, errlen))) return -rc;
      memcpy(dst, gpu + off, block_size);
      ++copies;
    } else {
      for (s = 0; s < l->segments; ++s) {
        if ((rc = or_segment_offset(l, (uint64_t)ids[i], s, &off, err, errlen))) return -rc;
        memcpy(dst + s * seg, gpu + off, seg);
        ++copies;
      }
    }
  }
  return copies;
}

/* batch_copy_segments_to_gpu (transfer.rs:116-198): merge maximal runs where
 * both the GPU offset and the host pointer advance by seg. */
static int64_t copy_runs(uint8_t* gpu, const uint64_t* goff, const uint8_t* const* host, uint64_t n, uint64_t seg) {
  int64_t runs = 0;
  uint64_t i = 0;
  while (i < n) {
    uint64_t count = 1;
    while (i + count < n && goff[i + count] == goff[i] + count * seg && host[i + count] == host[i] + count * seg)
      ++count;
    memmove(gpu + goff[i], host[i], seg * count);
    ++runs;
    i += count;
  }
  return runs;
}

/*
 * process_load_task (gpu_worker.rs:211-283) for one layer: K and V lists for
 * the split layout, one block_size_bytes list otherwise. Returns the number of
 * runs (copies) the reference issues, or -code. check_end enables the extra
 * "copy stays inside size_bytes" check the B200 library applies to non-split
 * loads (the reference only checks bytes_per_block there).
 */
int64_t or_load_layer(const or_layout* l, uint8_t* gpu, const int64_t* ids, uint64_t n, const uint8_t* const* k_src,
                      const uint8_t* const* v_src, int check_end, char* err, size_t errlen) {
  uint64_t i;
  int rc;
  int64_t runs = 0;
  if (n == 0) return 0;
  uint64_t* goff = (uint64_t*)malloc(sizeof(uint64_t) * n);
  const uint8_t** hp = (const uint8_t**)malloc(sizeof(uint8_t*) * n);
  if (or_is_split(l)) {
    for (i = 0; i < n; ++i) {
      if ((rc = or_segment_offset(l, (uint64_t)ids[i], 0, &goff[i], err, errlen))) goto fail;
      hp[i] = k_src[i];
    }
    uint64_t* voff = (uint64_t*)malloc(sizeof(uint64_t) * n);
    const uint8_t** vp = (const uint8_t**)malloc(sizeof(uint8_t*) * n);
    for (i = 0; i < n; ++i) {
      if ((rc = or_segment_offset(l, (uint64_t)ids[i], 1, &voff[i], err, errlen))) {
        free(voff);
        free(vp);
        goto fail;
      }
      vp[i] = (v_src && v_src[i]) ? v_src[i] : k_src[i] + l->bytes_per_block; /* gpu_worker.rs:233-236 */
    }
    runs += copy_runs(gpu, goff, hp, n, l->bytes_per_block);
    runs += copy_runs(gpu, voff, vp, n, l->bytes_per_block);
    free(voff);
    free(vp);
  } else {
    const uint64_t block_size = l->bytes_per_block * l->segments;
    for (i = 0; i < n; ++i) {
      if ((rc = or_segment_offset(l, (uint64_t)ids[i], 0, &goff[i], err, errlen))) goto fail;
      if (check_end && goff[i] + block_size > l->size_bytes) {
        rc = set_err(err, errlen, OR_STORAGE, "Block %llu exceeds registered memory", (unsigned long long)ids[i]);
        goto fail;
      }
      hp[i] = k_src[i];
    }
    runs += copy_runs(gpu, goff, hp, n, block_size);
  }
  free(goff);
  free(hp);
  return runs;
fail:
  free(goff);
  free(hp);
  return -rc;
}

/* ------------------------------------------------------------------------ */
/* Multi-threaded CPU gather/scatter of the same layout (the CPU baseline).  */
/* Work item = (layer, unit, block); threads take contiguous item ranges.    */
/* ------------------------------------------------------------------------ */

typedef struct or_mt_layer {
  or_layout layout;
  uint8_t* gpu;          /* host-resident "KV cache" of the layer */
  const int64_t* ids;
  uint64_t n;
  uint8_t* k_pool;       /* pool regions (save dst / load src) */
  uint8_t* v_pool;
} or_mt_layer;

typedef struct {
  const or_mt_layer* layers;
  uint64_t n_layers;
  int save;
  uint64_t begin, end; /* global item range */
  const uint64_t* item_start;
} or_mt_arg;

static void* mt_worker(void* p) {
  or_mt_arg* a = (or_mt_arg*)p;
  uint64_t li = 0;
  for (uint64_t g = a->begin; g < a->end; ++g) {
    while (g >= a->item_start[li + 1]) ++li;
    const or_mt_layer* L = &a->layers[li];
    const or_layout* l = &L->layout;
    const uint64_t local = g - a->item_start[li];
    const int split = or_is_split(l);
    const uint64_t seg = l->bytes_per_block;
    const uint64_t u = split ? local / L->n : 0;
    const uint64_t i = split ? local % L->n : local;
    const uint64_t b = (uint64_t)L->ids[i];
    const uint64_t unit = split ? seg : seg * l->segments;
    uint8_t* cache = L->gpu + b * seg + (split ? u * l->kv_stride_bytes : 0);
    uint8_t* pool = split ? (u ? L->v_pool : L->k_pool) + i * seg : L->k_pool + i * unit;
    if (a->save)
      memcpy(pool, cache, unit);
    else
      memcpy(cache, pool, unit);
  }
  return NULL;
}

/* Gather (save=1) or scatter (save=0) every layer with `threads` threads.
 * Layouts must be split or contiguous (the vLLM layouts). Returns bytes moved. */
uint64_t or_mt_transfer(const or_mt_layer* layers, uint64_t n_layers, int save, int threads) {
  if (threads < 1) threads = 1;
  uint64_t* start = (uint64_t*)malloc(sizeof(uint64_t) * (n_layers + 1));
  uint64_t bytes = 0;
  start[0] = 0;
  for (uint64_t l = 0; l < n_layers; ++l) {
    const int split = or_is_split(&layers[l].layout);
    start[l + 1] = start[l] + layers[l].n * (split ? 2 : 1);
    bytes += layers[l].n * layers[l].layout.bytes_per_block * (split ? 2 : layers[l].layout.segments);
  }
  const uint64_t total = start[n_layers];
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  or_mt_arg* args = (or_mt_arg*)malloc(sizeof(or_mt_arg) * (size_t)threads);
  for (int t = 0; t < threads; ++t) {
    args[t].layers = layers;
    args[t].n_layers = n_layers;
    args[t].save = save;
    args[t].begin = total * (uint64_t)t / (uint64_t)threads;
    args[t].end = total * (uint64_t)(t + 1) / (uint64_t)threads;
    args[t].item_start = start;
    pthread_create(&th[t], NULL, mt_worker, &args[t]);
  }
  for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
  free(th);
  free(args);
  free(start);
  return bytes;
}
