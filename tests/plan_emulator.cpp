// Byte parity of the library's transfer plans on the CPU. The plans come from
// the library itself (plan_save / plan_load in plan_build.cpp, cut_chunks in
// chunks.cpp). This harness replays them on host arrays: the copy kernel's
// per-tile addressing (kernels.cu), and the copy-engine runs between staging
// slot and pool. The bytes must equal the C oracle's restatement of the
// reference's copies (oracle/pf_oracle.c). Random layouts cover split K/V,
// blocks-first, contiguous two-segment and strided three-segment blocks;
// unit sizes from 4 bytes to over 64 KiB; staged mode with small slots, and
// direct mode; repeated destination ids; and layouts whose blocks share
// bytes (the ordered-copy path).
// The no-allocation save (noalloc.cu) runs the same plan, cutter and copies
// with a first chunk of a whole slot; a fifth of the cases cut that way.
// Peer copies (plan_p2p, the P/D handoff) are replayed too, as pulls and as
// pushes: every destination block must hold its source block's bytes, the
// last of repeated destinations winning. Copies within one tensor on one
// device must keep identity, and a pair that reads the block it writes must
// be refused.
//
// Build and run (tests/test_plan_emulator.py does this):
//   gcc -O1 -c oracle/pf_oracle.c -o pf_oracle.o
//   g++ -O1 -std=c++17 -I<repo>/include -I<csrc> -I<cuda>/include tests/plan_emulator.cpp
//       <csrc>/plan_build.cpp <csrc>/chunks.cpp pf_oracle.o -L<cuda>/lib64 -lcudart_static -ldl -lrt -lpthread
//   ./plan_emulator <cases>
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "chunks.h"
#include "common.h"
#include "plan_build.h"

extern "C" {
typedef struct or_layout {
  uint64_t size_bytes, num_blocks, bytes_per_block, kv_stride_bytes, segments;
} or_layout;
int64_t or_save_layer(const or_layout* l, const uint8_t* gpu, const int64_t* ids, uint64_t n, uint8_t* k_dst,
                      uint8_t* v_dst, char* err, size_t errlen);
int64_t or_load_layer(const or_layout* l, uint8_t* gpu, const int64_t* ids, uint64_t n,
                      const uint8_t* const* k_src, const uint8_t* const* v_src, int check_end, char* err,
                      size_t errlen);
}

using namespace pf;

namespace {

// The copy kernel's work for tiles [tb, te): kernels.cu, kv_copy_kernel.
// Warps run tiles in no fixed order; `backwards` replays them last to first,
// so a plan whose result depends on the order fails one of the two replays.
void run_tiles(const Built& b, bool pack, bool table, uint64_t tb, uint64_t te, int64_t shift,
               bool backwards = false) {
  for (uint64_t k = tb; k < te; ++k) {
    const uint64_t tile = backwards ? te - 1 - (k - tb) : k;
    size_t l = 0;
    while (l + 1 < b.layers.size() && b.layers[l + 1].tile_start <= tile) ++l;
    const PlanLayer& L = b.layers[l];
    const uint32_t local = static_cast<uint32_t>(tile - L.tile_start);
    const uint32_t unit_local = local / L.tiles_per_unit;
    const uint32_t t = local - unit_local * L.tiles_per_unit;
    const uint32_t u = unit_local / L.n;
    const uint32_t i = unit_local - u * L.n;
    const uint64_t blk = b.ids[L.ids_off + i];
    const uint32_t in_unit = t * kTileBytes;
    const uint32_t rest = L.unit_bytes - in_unit;
    const uint32_t bytes = rest < kTileBytes ? rest : kTileBytes;
    uint8_t* cache = reinterpret_cast<uint8_t*>(L.cache_base + blk * L.block_pitch + uint64_t(u) * L.unit_stride + in_unit);
    uint8_t* side = table ? reinterpret_cast<uint8_t*>(b.side_ptrs[L.unit_off + unit_local] + in_unit)
                          : reinterpret_cast<uint8_t*>(b.side_base[L.side_off + u] + uint64_t(i) * L.side_pitch +
                                                       in_unit + shift);
    if (pack) {
      std::memcpy(side, cache, bytes);
    } else {
      std::memcpy(cache, side, bytes);
    }
  }
}

// The copy-engine copies of one chunk (Executor::copy_runs): the chunk's own
// bytes [dense_first, dense_end), placed in the slot relative to dense_begin.
void run_copies(const Built& b, const Chunk& c, uint8_t* slot, bool d2h) {
  for (const Run& r : b.runs) {
    const uint64_t lo = std::max(r.dense, c.dense_first);
    const uint64_t hi = std::min(r.dense + r.bytes, c.dense_end);
    if (hi <= lo) continue;
    uint8_t* host = reinterpret_cast<uint8_t*>(r.host + (lo - r.dense));
    uint8_t* dev = slot + (lo - c.dense_begin);
    if (d2h) {
      std::memcpy(host, dev, hi - lo);
    } else {
      std::memcpy(dev, host, hi - lo);
    }
  }
}

// The ordered copies of loads whose blocks share bytes (Executor::issue_serial).
void run_serial(const Built& b) {
  for (const SerialLoad& sl : b.serial) {
    const pf_layer_desc& l = sl.layer;
    const bool split = is_split_layout(l);
    const uint64_t unit = split ? l.bytes_per_block : l.bytes_per_block * l.segments;
    for (int u = 0; u < (split ? 2 : 1); ++u) {
      const std::vector<uint64_t>& host = u == 0 ? sl.k : sl.v;
      for (size_t i = 0; i < sl.ids.size(); ++i) {
        const uint64_t g0 = static_cast<uint64_t>(sl.ids[i]) * l.bytes_per_block + u * l.kv_stride_bytes;
        std::memmove(reinterpret_cast<uint8_t*>(l.data_ptr + g0), reinterpret_cast<const uint8_t*>(host[i]), unit);
      }
    }
  }
}

// A staged or direct save / load as Executor::save / Executor::load run it.
void run_save(const Built& b, bool staged, uint64_t slot_bytes, uint64_t first, bool backwards) {
  if (!staged) return run_tiles(b, true, false, 0, b.total_tiles, 0, backwards);
  std::vector<uint8_t> slot(slot_bytes + 64);
  uint8_t* s = slot.data();
  std::vector<Chunk> chunks;
  cut_chunks(b.layers, b.total_tiles, slot_bytes, first, &chunks);
  for (const Chunk& c : chunks) {
    run_tiles(b, true, false, c.tile_begin, c.tile_end,
              static_cast<int64_t>(reinterpret_cast<uint64_t>(s)) - static_cast<int64_t>(c.dense_begin), backwards);
    run_copies(b, c, s, true);
  }
}

void run_load(const Built& b, bool staged, uint64_t slot_bytes, uint64_t first, bool backwards) {
  if (b.total_tiles) {
    if (!staged) {
      run_tiles(b, false, true, 0, b.total_tiles, 0, backwards);
    } else {
      std::vector<uint8_t> slot(slot_bytes + 64);
      uint8_t* s = slot.data();
      std::vector<Chunk> chunks;
      cut_chunks(b.layers, b.total_tiles, slot_bytes, first, &chunks);
      for (const Chunk& c : chunks) {
        run_copies(b, c, s, false);
        run_tiles(b, false, false, c.tile_begin, c.tile_end,
                  static_cast<int64_t>(reinterpret_cast<uint64_t>(s)) - static_cast<int64_t>(c.dense_begin),
                  backwards);
      }
    }
  }
  run_serial(b);
}

struct Layer {
  or_layout ol;
  std::vector<uint8_t> cache;  // the "KV tensor" of the layer
  pf_layer_desc desc() const {
    pf_layer_desc d{};
    d.data_ptr = reinterpret_cast<uint64_t>(cache.data());
    d.size_bytes = ol.size_bytes;
    d.num_blocks = ol.num_blocks;
    d.bytes_per_block = ol.bytes_per_block;
    d.kv_stride_bytes = ol.kv_stride_bytes;
    d.segments = ol.segments;
    return d;
  }
};

// Random bytes, eight per draw.
void fill(std::vector<uint8_t>& v, std::mt19937_64& rng) {
  size_t i = 0;
  for (; i + 8 <= v.size(); i += 8) {
    const uint64_t r = rng();
    std::memcpy(v.data() + i, &r, 8);
  }
  for (; i < v.size(); ++i) v[i] = static_cast<uint8_t>(rng());
}

Layer random_layer(std::mt19937_64& rng) {
  static const uint64_t bpbs[] = {4, 12, 45, 4096, 8196, 32768, 100000};
  const uint64_t bpb = bpbs[rng() % 7];
  const uint64_t nb = 1 + rng() % 40;
  Layer L;
  switch (rng() % 4) {
    case 0:  // split K/V: [2, nb, ...]
      L.ol = {2 * nb * bpb, nb, bpb, nb * bpb, 2};
      break;
    case 1:  // blocks-first, one segment
      L.ol = {nb * bpb, nb, bpb, 0, 1};
      break;
    case 2:  // two segments back to back in each block (contiguous)
      L.ol = {2 * nb * bpb, nb, bpb, bpb, 2};
      break;
    default:  // three segments a stride apart (neither split nor contiguous)
      L.ol = {(nb - 1) * bpb + 2 * (nb * bpb) + bpb, nb, bpb, nb * bpb, 3};
      break;
  }
  L.cache.resize(L.ol.size_bytes);
  fill(L.cache, rng);
  return L;
}

}  // namespace

int main(int argc, char** argv) {
  const int cases = argc > 1 ? std::atoi(argv[1]) : 3000;
  std::mt19937_64 rng(11);
  const DeviceCheck no_check = [](int, const pf_layer_desc&) {};
  char err[256];
  long saves = 0, loads = 0, serial = 0, peers = 0, within = 0;
  for (int c = 0; c < cases; ++c) {
    const int nl = 1 + static_cast<int>(rng() % 4);
    std::vector<Layer> layers;
    for (int i = 0; i < nl; ++i) layers.push_back(random_layer(rng));
    const bool staged = rng() % 4 != 0;
    const uint64_t slot_bytes = align_up(std::max<uint64_t>(2 * kTileBytes, rng() % (1 << 20)), kDenseAlign);
    uint64_t first = rng() % (1 << 19);
    if (c % 5 == 0) first = slot_bytes;  // whole slots from the start: the no-allocation save's cut

    // ---- save: every layer's chosen blocks into its own pool regions ----
    std::vector<std::vector<int64_t>> ids(nl);
    std::vector<std::vector<uint8_t>> pool_k(nl), pool_v(nl);
    std::vector<pf_save_layer> sl(nl);
    for (int i = 0; i < nl; ++i) {
      const Layer& L = layers[i];
      const uint64_t n = 1 + rng() % L.ol.num_blocks;
      for (uint64_t j = 0; j < n; ++j) ids[i].push_back(static_cast<int64_t>(rng() % L.ol.num_blocks));
      const bool split = L.ol.segments == 2 && L.ol.kv_stride_bytes > L.ol.bytes_per_block;
      const uint64_t per = split ? L.ol.bytes_per_block : L.ol.bytes_per_block * L.ol.segments;
      pool_k[i].assign(n * per + (split ? 0 : 0), 0);
      if (split) pool_v[i].assign(n * per, 0);
      sl[i] = pf_save_layer{L.desc(), ids[i].data(), n, pool_k[i].data(), split ? pool_v[i].data() : nullptr};
    }
    Built bs;
    plan_save(sl.data(), nl, staged, 0, no_check, &bs);
    run_save(bs, staged, slot_bytes, first, (c & 2) != 0);
    for (int i = 0; i < nl; ++i) {
      const Layer& L = layers[i];
      std::vector<uint8_t> k(pool_k[i].size()), v(pool_v[i].size());
      if (or_save_layer(&L.ol, L.cache.data(), ids[i].data(), ids[i].size(), k.data(), v.empty() ? nullptr : v.data(),
                        err, sizeof err) < 0) {
        std::printf("FAIL case %d: oracle save refused: %s\n", c, err);
        return 1;
      }
      if (k != pool_k[i] || v != pool_v[i]) {
        std::printf("FAIL case %d layer %d: pool bytes differ from the oracle's (segments %llu, bpb %llu)\n", c, i,
                    (unsigned long long)L.ol.segments, (unsigned long long)L.ol.bytes_per_block);
        return 1;
      }
    }
    ++saves;

    // ---- load: the saved blocks into other (possibly repeated) ids ----
    std::vector<Layer> dst = layers;  // same layouts, fresh bytes
    for (auto& L : dst) {
      fill(L.cache, rng);
    }
    std::vector<std::vector<int64_t>> dids(nl);
    std::vector<std::vector<const void*>> ksrc(nl), vsrc(nl);
    std::vector<pf_load_layer> ll(nl);
    for (int i = 0; i < nl; ++i) {
      const Layer& L = dst[i];
      const uint64_t n = ids[i].size();
      const bool split = L.ol.segments == 2 && L.ol.kv_stride_bytes > L.ol.bytes_per_block;
      const uint64_t per = split ? L.ol.bytes_per_block : L.ol.bytes_per_block * L.ol.segments;
      for (uint64_t j = 0; j < n; ++j) {
        dids[i].push_back(static_cast<int64_t>(rng() % L.ol.num_blocks));
        ksrc[i].push_back(pool_k[i].data() + j * per);
        vsrc[i].push_back(split ? static_cast<const void*>(pool_v[i].data() + j * per) : nullptr);
      }
      ll[i] = pf_load_layer{L.desc(), dids[i].data(), n, ksrc[i].data(), vsrc[i].data()};
    }
    std::vector<Layer> want = dst;
    Built bl;
    try {
      plan_load(ll.data(), nl, staged, 0, no_check, &bl);
    } catch (const std::exception& e) {
      // A non-split load copies a whole block at the block offset; in a
      // strided layout the last blocks reach past the registration, which the
      // library refuses before copying (the oracle's check_end does the same).
      bool refused = false;
      for (int i = 0; i < nl && !refused; ++i) {
        std::vector<const uint8_t*> kp(ksrc[i].size()), vp(vsrc[i].size());
        for (size_t j = 0; j < kp.size(); ++j) kp[j] = static_cast<const uint8_t*>(ksrc[i][j]);
        for (size_t j = 0; j < vp.size(); ++j) vp[j] = static_cast<const uint8_t*>(vsrc[i][j]);
        refused = or_load_layer(&want[i].ol, want[i].cache.data(), dids[i].data(), dids[i].size(), kp.data(),
                                vp.data(), 1, err, sizeof err) < 0;
      }
      if (!refused) {
        std::printf("FAIL case %d: library refused a load the oracle accepts: %s\n", c, e.what());
        return 1;
      }
      continue;
    }
    serial += bl.serial.empty() ? 0 : 1;
    run_load(bl, staged, slot_bytes, first, (c & 2) != 0);
    for (int i = 0; i < nl; ++i) {
      std::vector<const uint8_t*> kp(ksrc[i].size()), vp(vsrc[i].size());
      for (size_t j = 0; j < kp.size(); ++j) kp[j] = static_cast<const uint8_t*>(ksrc[i][j]);
      for (size_t j = 0; j < vp.size(); ++j) vp[j] = static_cast<const uint8_t*>(vsrc[i][j]);
      if (or_load_layer(&want[i].ol, want[i].cache.data(), dids[i].data(), dids[i].size(), kp.data(), vp.data(), 1,
                        err, sizeof err) < 0) {
        std::printf("FAIL case %d: the oracle refused a load the library accepted: %s\n", c, err);
        return 1;
      }
      if (want[i].cache != dst[i].cache) {
        std::printf("FAIL case %d layer %d: restored bytes differ from the oracle's (segments %llu, bpb %llu)\n", c,
                    i, (unsigned long long)dst[i].ol.segments, (unsigned long long)dst[i].ol.bytes_per_block);
        return 1;
      }
    }
    ++loads;

    // ---- peer copies (P/D handoff): pull and push between two "devices" ----
    // Copy identity: each destination block gets its source block's bytes,
    // and for a repeated destination the last occurrence wins.
    for (int push = 0; push < 2; ++push) {
      const int np = 1 + static_cast<int>(rng() % 3);
      std::vector<Layer> srcs, dsts;
      std::vector<std::vector<int64_t>> sidx(np), didx(np);
      std::vector<pf_p2p_layer> pl(np);
      for (int i = 0; i < np; ++i) {
        static const uint64_t bpbs[] = {4, 45, 4096, 32768, 100000};
        const uint64_t bpb = bpbs[rng() % 5];
        const bool split = rng() % 2;
        // At least two blocks a side: a split layout of one block is a contiguous one.
        const uint64_t nbs = 2 + rng() % 30, nbd = 2 + rng() % 30;
        Layer S, D;
        S.ol = split ? or_layout{2 * nbs * bpb, nbs, bpb, nbs * bpb, 2} : or_layout{nbs * bpb, nbs, bpb, 0, 1};
        D.ol = split ? or_layout{2 * nbd * bpb, nbd, bpb, nbd * bpb, 2} : or_layout{nbd * bpb, nbd, bpb, 0, 1};
        S.cache.resize(S.ol.size_bytes);
        D.cache.resize(D.ol.size_bytes);
        fill(S.cache, rng);
        fill(D.cache, rng);
        const uint64_t n = 1 + rng() % std::min(nbs, nbd);
        for (uint64_t j = 0; j < n; ++j) {
          sidx[i].push_back(static_cast<int64_t>(rng() % nbs));
          didx[i].push_back(static_cast<int64_t>(rng() % nbd));
        }
        srcs.push_back(std::move(S));
        dsts.push_back(std::move(D));
      }
      std::vector<Layer> want = dsts;
      for (int i = 0; i < np; ++i) {
        pl[i] = pf_p2p_layer{srcs[i].desc(), dsts[i].desc(), sidx[i].data(), didx[i].data(), sidx[i].size()};
        const uint64_t bpb = srcs[i].ol.bytes_per_block;
        const int units = srcs[i].ol.segments == 2 ? 2 : 1;
        for (size_t j = 0; j < sidx[i].size(); ++j) {
          for (int u = 0; u < units; ++u) {
            std::memcpy(want[i].cache.data() + didx[i][j] * bpb + u * want[i].ol.kv_stride_bytes,
                        srcs[i].cache.data() + sidx[i][j] * bpb + u * srcs[i].ol.kv_stride_bytes, bpb);
          }
        }
      }
      Built bp;
      plan_p2p(pl.data(), np, 0, 1, push != 0, no_check, &bp);
      run_tiles(bp, push != 0, true, 0, bp.total_tiles, 0, /*backwards=*/(c & 1) != 0);
      for (int i = 0; i < np; ++i) {
        if (want[i].cache != dsts[i].cache) {
          std::printf("FAIL case %d: peer %s layer %d differs from copy identity (segments %llu, bpb %llu)\n", c,
                      push ? "push" : "pull", i, (unsigned long long)dsts[i].ol.segments,
                      (unsigned long long)dsts[i].ol.bytes_per_block);
          return 1;
        }
      }
      ++peers;
    }

    // ---- one device, one tensor: blocks copied within it ----
    // Sources from the first half of the blocks, destinations from the second:
    // copy identity. A pair that reads the block it writes is refused, since
    // the result would depend on the order the warps run in.
    {
      const uint64_t bpb = (c & 4) ? 45 : 4096;
      const uint64_t nb = 4 + rng() % 40, half = nb / 2;
      const bool split = rng() % 2;
      Layer T;
      T.ol = split ? or_layout{2 * nb * bpb, nb, bpb, nb * bpb, 2} : or_layout{nb * bpb, nb, bpb, 0, 1};
      T.cache.resize(T.ol.size_bytes);
      fill(T.cache, rng);
      const uint64_t n = 1 + rng() % half;
      std::vector<int64_t> si, di;
      for (uint64_t j = 0; j < n; ++j) {
        si.push_back(static_cast<int64_t>(rng() % half));
        di.push_back(static_cast<int64_t>(half + rng() % (nb - half)));
      }
      std::vector<uint8_t> want = T.cache;
      for (uint64_t j = 0; j < n; ++j) {
        for (int u = 0; u < (split ? 2 : 1); ++u) {
          std::memcpy(want.data() + di[j] * bpb + u * T.ol.kv_stride_bytes,
                      T.cache.data() + si[j] * bpb + u * T.ol.kv_stride_bytes, bpb);
        }
      }
      pf_p2p_layer one{T.desc(), T.desc(), si.data(), di.data(), n};
      Built bt;
      plan_p2p(&one, 1, 0, 0, false, no_check, &bt);
      run_tiles(bt, false, true, 0, bt.total_tiles, 0, (c & 1) != 0);
      if (T.cache != want) {
        std::printf("FAIL case %d: copy within one tensor differs from copy identity\n", c);
        return 1;
      }
      si.back() = di.back();  // the last pair for a destination is always kept
      Built bo;
      bool refused = false;
      try {
        plan_p2p(&one, 1, 0, 0, false, no_check, &bo);
      } catch (const std::exception&) {
        refused = true;
      }
      if (!refused) {
        std::printf("FAIL case %d: a block read and written by one copy was not refused\n", c);
        return 1;
      }
      ++within;
    }
  }
  std::printf("ok saves=%ld loads=%ld serial=%ld peers=%ld within=%ld\n", saves, loads, serial, peers, within);
  return 0;
}
