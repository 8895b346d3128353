// LoadState: POSIX shared-memory completion flag, byte-compatible with
// pegaflow-core/src/sync_state.rs.
//
// Mapping layout (sync_state.rs:27-43, 186-242), little-endian x86_64:
//   [0, 8)            usize: offset of the aligned record from the base (8)
//   [off, off+4)      u32 magic 0x50464C44 ('PFLD')
//   [off+4, off+8)    u32 version 1
//   [off+8, off+16)   i64 state: 0 pending, 1 success, -1 error
// Allocation size = 8 + sizeof(record)=16 + align 8 = 32 bytes. The object is
// named "pega_load_<uuid v4, 32 lowercase hex>" (sync_state.rs:126) and the
// creating handle unlinks it when closed (owner drop).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <random>
#include <string>

#include "common.h"

namespace pf {

namespace {
constexpr uint32_t kMagic = 0x50464C44u;
constexpr uint32_t kVersion = 1;
constexpr size_t kMetaSize = 8;
constexpr size_t kRecordSize = 16;
constexpr size_t kRecordAlign = 8;
constexpr size_t kAllocSize = kMetaSize + kRecordSize + kRecordAlign;  // 32

struct Record {
  std::atomic<uint32_t> magic;
  std::atomic<uint32_t> version;
  std::atomic<int64_t> state;
};
static_assert(sizeof(Record) == kRecordSize, "record layout");

// Per-layer extension, placed after the 32 bytes a version-1 reader maps
// (a reader built against sync_state.rs only checks that the mapping is at
// least 32 bytes, so it still attaches):
//   [32, 36)  u32 magic 0x324C4650 ('PFL2')
//   [36, 40)  u32 layer count n
//   [40, 48)  reserved
//   [48, 48 + 8n)  i64 per layer: 0 pending, 1 bytes in place
constexpr uint32_t kLayerMagic = 0x324C4650u;
constexpr size_t kLayerHeader = 16;
struct LayerHeader {
  std::atomic<uint32_t> magic;
  std::atomic<uint32_t> count;
  uint64_t reserved;
};
static_assert(sizeof(LayerHeader) == kLayerHeader, "layer header layout");

std::string uuid_v4_simple() {
  unsigned char b[16];
  bool ok = false;
  {
    std::ifstream f("/dev/urandom", std::ios::binary);
    if (f.read(reinterpret_cast<char*>(b), 16)) ok = true;
  }
  if (!ok) {
    std::random_device rd;
    for (auto& x : b) x = static_cast<unsigned char>(rd());
  }
  b[6] = static_cast<unsigned char>((b[6] & 0x0f) | 0x40);  // version 4
  b[8] = static_cast<unsigned char>((b[8] & 0x3f) | 0x80);  // RFC 4122 variant
  static const char* hex = "0123456789abcdef";
  std::string s;
  for (unsigned char x : b) {
    s.push_back(hex[x >> 4]);
    s.push_back(hex[x & 15]);
  }
  return s;
}

Error ls_error(const std::string& msg) { return Error(PF_ERR_LOAD_STATE, msg); }
}  // namespace

}  // namespace pf

struct pf_load_state {
  std::string name;
  void* base = nullptr;
  size_t len = 0;
  pf::Record* rec = nullptr;
  bool owner = false;
  uint32_t layers = 0;              // per-layer extension size (0: version-1 only)
  int64_t* layer_words = nullptr;   // the extension's per-layer words
};

namespace pf {

pf_load_state* load_state_create(uint32_t n_layers) {
  const std::string name = "pega_load_" + uuid_v4_simple();
  const size_t size = n_layers ? kAllocSize + kLayerHeader + 8ull * n_layers : kAllocSize;
  const int fd = shm_open(name.c_str(), O_CREAT | O_EXCL | O_RDWR, S_IRUSR | S_IWUSR);
  if (fd < 0) throw ls_error("failed to create shared memory: " + std::string(strerror(errno)));
  if (ftruncate(fd, static_cast<off_t>(size)) != 0) {
    const int e = errno;
    close(fd);
    shm_unlink(name.c_str());
    throw ls_error("failed to create shared memory: " + std::string(strerror(e)));
  }
  void* base = mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (base == MAP_FAILED) {
    shm_unlink(name.c_str());
    throw ls_error("failed to create shared memory: mmap failed");
  }
  // init_new_mapping (sync_state.rs:201-242)
  const uintptr_t b = reinterpret_cast<uintptr_t>(base);
  const uintptr_t aligned = (b + kMetaSize + kRecordAlign - 1) & ~(uintptr_t)(kRecordAlign - 1);
  const uint64_t offset = aligned - b;
  std::memcpy(base, &offset, sizeof(offset));
  auto* rec = reinterpret_cast<Record*>(aligned);
  rec->magic.store(kMagic, std::memory_order_release);
  rec->version.store(kVersion, std::memory_order_release);
  rec->state.store(PF_LOAD_STATE_PENDING, std::memory_order_release);
  auto* s = new pf_load_state();
  s->name = name;
  s->base = base;
  s->len = size;
  s->rec = rec;
  s->owner = true;
  if (n_layers) {
    auto* lh = reinterpret_cast<LayerHeader*>(static_cast<uint8_t*>(base) + kAllocSize);
    s->layer_words = reinterpret_cast<int64_t*>(static_cast<uint8_t*>(base) + kAllocSize + kLayerHeader);
    for (uint32_t i = 0; i < n_layers; ++i) s->layer_words[i] = 0;
    lh->count.store(n_layers, std::memory_order_relaxed);
    lh->magic.store(kLayerMagic, std::memory_order_release);
    s->layers = n_layers;
  }
  return s;
}

pf_load_state* load_state_attach(const std::string& name) {
  const int fd = shm_open(name.c_str(), O_RDWR, 0);
  if (fd < 0) throw ls_error("failed to open shared memory: " + std::string(strerror(errno)));
  struct stat st {};
  if (fstat(fd, &st) != 0) {
    close(fd);
    throw ls_error("failed to open shared memory: fstat failed");
  }
  const size_t len = static_cast<size_t>(st.st_size);
  // attach_mapping (sync_state.rs:244-283)
  if (len < kAllocSize) {
    close(fd);
    throw ls_error("shared memory too small (actual=" + std::to_string(len) + " bytes, required=" +
                   std::to_string(kAllocSize) + " bytes)");
  }
  void* base = mmap(nullptr, len, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (base == MAP_FAILED) throw ls_error("failed to open shared memory: mmap failed");
  uint64_t offset = 0;
  std::memcpy(&offset, base, sizeof(offset));
  auto fail = [&](const std::string& m) {
    munmap(base, len);
    return ls_error(m);
  };
  if (offset < kMetaSize) {
    throw fail("invalid LoadState offset (offset=" + std::to_string(offset) + ", len=" + std::to_string(len) +
               ") recorded in shared memory");
  }
  if (offset > len || len - offset < kRecordSize) {
    throw fail("shared memory too small (actual=" + std::to_string(len) + " bytes, required=" +
               std::to_string(offset + kRecordSize) + " bytes)");
  }
  const uintptr_t addr = reinterpret_cast<uintptr_t>(base) + offset;
  if (addr % kRecordAlign != 0) throw fail("aligned pointer is not 8-byte aligned");
  auto* rec = reinterpret_cast<Record*>(addr);
  // validate_header (sync_state.rs:285-292)
  const uint32_t magic = rec->magic.load(std::memory_order_acquire);
  const uint32_t version = rec->version.load(std::memory_order_acquire);
  if (magic != kMagic || version != kVersion) {
    char buf[160];
    snprintf(buf, sizeof(buf),
             "invalid LoadState header (magic=%#x, version=%u, expected magic=%#x, version=%u)", magic, version,
             kMagic, kVersion);
    throw fail(buf);
  }
  auto* s = new pf_load_state();
  s->name = name;
  s->base = base;
  s->len = len;
  s->rec = rec;
  s->owner = false;
  if (len >= kAllocSize + kLayerHeader) {
    auto* lh = reinterpret_cast<LayerHeader*>(static_cast<uint8_t*>(base) + kAllocSize);
    const uint32_t n = lh->count.load(std::memory_order_relaxed);
    if (lh->magic.load(std::memory_order_acquire) == kLayerMagic && n > 0 &&
        kAllocSize + kLayerHeader + 8ull * n <= len) {
      s->layers = n;
      s->layer_words = reinterpret_cast<int64_t*>(static_cast<uint8_t*>(base) + kAllocSize + kLayerHeader);
    }
  }
  return s;
}

void load_state_close(pf_load_state* s) {
  if (!s) return;
  if (s->base) munmap(s->base, s->len);
  if (s->owner) shm_unlink(s->name.c_str());
  delete s;
}

int64_t load_state_get(const pf_load_state* s) { return s->rec->state.load(std::memory_order_acquire); }
void load_state_set(pf_load_state* s, int64_t v) { s->rec->state.store(v, std::memory_order_release); }
uint32_t load_state_layers(const pf_load_state* s) { return s->layers; }
int64_t* load_state_layer_words(pf_load_state* s) { return s->layer_words; }
void* load_state_base(pf_load_state* s, size_t* len) {
  *len = s->len;
  return s->base;
}

}  // namespace pf

extern "C" const char* pf_load_state_name(const pf_load_state* s) { return s ? s->name.c_str() : ""; }

extern "C" uint32_t pf_load_state_layer_count(const pf_load_state* s) { return s ? s->layers : 0; }

extern "C" int64_t pf_load_state_layer_get(const pf_load_state* s, uint32_t layer) {
  if (!s || layer >= s->layers) return PF_LOAD_STATE_ERROR;
  return reinterpret_cast<volatile const int64_t*>(s->layer_words)[layer];
}
