#include "dfs_tier.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <random>
#include <sstream>

#include "common.h"

namespace pf {

namespace fs = std::filesystem;

// ---------------------------------------------------------------------------
// Records
// ---------------------------------------------------------------------------

uint64_t BlockMeta::total_size() const {
  uint64_t s = 0;
  for (const SlotMeta& m : slots) s += m.size;
  return s;
}

std::string hex_encode(const std::string& bytes) {
  static const char* d = "0123456789abcdef";
  std::string out(bytes.size() * 2, '0');
  for (size_t i = 0; i < bytes.size(); ++i) {
    const unsigned char c = static_cast<unsigned char>(bytes[i]);
    out[2 * i] = d[c >> 4];
    out[2 * i + 1] = d[c & 15];
  }
  return out;
}

bool hex_decode(const std::string& hex, std::string* out) {
  if (hex.size() % 2) return false;
  auto nib = [](char c) -> int {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    return -1;
  };
  out->assign(hex.size() / 2, '\0');
  for (size_t i = 0; i < out->size(); ++i) {
    const int hi = nib(hex[2 * i]), lo = nib(hex[2 * i + 1]);
    if (hi < 0 || lo < 0) return false;
    (*out)[i] = static_cast<char>(hi << 4 | lo);
  }
  return true;
}

namespace {

void json_string(std::string* o, const std::string& s) {
  o->push_back('"');
  for (char c : s) {
    if (c == '"' || c == '\\') {
      o->push_back('\\');
      o->push_back(c);
    } else if (static_cast<unsigned char>(c) < 0x20) {
      char buf[8];
      snprintf(buf, sizeof(buf), "\\u%04x", static_cast<unsigned char>(c));
      o->append(buf);
    } else {
      o->push_back(c);
    }
  }
  o->push_back('"');
}

// A reader for the records above: objects, arrays, strings, unsigned
// integers and booleans, which is all they contain.
class JsonReader {
 public:
  explicit JsonReader(const std::string& s) : s_(s) {}
  bool object(const std::function<bool(const std::string&)>& field) {
    if (!eat('{')) return false;
    if (eat('}')) return true;
    do {
      std::string key;
      if (!string(&key) || !eat(':') || !field(key)) return false;
    } while (eat(','));
    return eat('}');
  }
  bool array(const std::function<bool()>& item) {
    if (!eat('[')) return false;
    if (eat(']')) return true;
    do {
      if (!item()) return false;
    } while (eat(','));
    return eat(']');
  }
  bool string(std::string* out) {
    ws();
    if (i_ >= s_.size() || s_[i_] != '"') return false;
    ++i_;
    out->clear();
    while (i_ < s_.size() && s_[i_] != '"') {
      char c = s_[i_++];
      if (c == '\\') {
        if (i_ >= s_.size()) return false;
        c = s_[i_++];
        if (c == 'u') {
          if (i_ + 4 > s_.size()) return false;
          c = static_cast<char>(std::stoi(s_.substr(i_, 4), nullptr, 16));
          i_ += 4;
        }
      }
      out->push_back(c);
    }
    return eat_raw('"');
  }
  bool number(uint64_t* out) {
    ws();
    const size_t start = i_;
    while (i_ < s_.size() && s_[i_] >= '0' && s_[i_] <= '9') ++i_;
    if (i_ == start) return false;
    *out = std::stoull(s_.substr(start, i_ - start));
    return true;
  }
  bool boolean(bool* out) {
    ws();
    if (s_.compare(i_, 4, "true") == 0) {
      i_ += 4;
      *out = true;
      return true;
    }
    if (s_.compare(i_, 5, "false") == 0) {
      i_ += 5;
      *out = false;
      return true;
    }
    return false;
  }
  bool done() {
    ws();
    return i_ == s_.size();
  }

 private:
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\t' || s_[i_] == '\r')) ++i_;
  }
  bool eat(char c) {
    ws();
    return eat_raw(c);
  }
  bool eat_raw(char c) {
    if (i_ < s_.size() && s_[i_] == c) {
      ++i_;
      return true;
    }
    return false;
  }
  const std::string& s_;
  size_t i_ = 0;
};

std::string uuid_v4() {
  static thread_local std::mt19937_64 rng(std::random_device{}() ^
                                          static_cast<uint64_t>(std::chrono::steady_clock::now().time_since_epoch().count()));
  unsigned char b[16];
  for (int i = 0; i < 16; i += 8) {
    const uint64_t r = rng();
    std::memcpy(b + i, &r, 8);
  }
  b[6] = static_cast<unsigned char>((b[6] & 0x0f) | 0x40);  // version 4
  b[8] = static_cast<unsigned char>((b[8] & 0x3f) | 0x80);  // RFC 4122 variant
  static const char* d = "0123456789abcdef";
  std::string s;
  for (int i = 0; i < 16; ++i) {
    if (i == 4 || i == 6 || i == 8 || i == 10) s.push_back('-');
    s.push_back(d[b[i] >> 4]);
    s.push_back(d[b[i] & 15]);
  }
  return s;
}

uint64_t now_ms() {
  return static_cast<uint64_t>(
      std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::system_clock::now().time_since_epoch())
          .count());
}

bool write_all(int fd, const uint8_t* p, uint64_t n) {
  while (n > 0) {
    const ssize_t w = ::write(fd, p, n);
    if (w < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    p += w;
    n -= static_cast<uint64_t>(w);
  }
  return true;
}

bool read_all_at(int fd, uint8_t* p, uint64_t n, uint64_t off) {
  while (n > 0) {
    const ssize_t r = ::pread(fd, p, n, static_cast<off_t>(off));
    if (r < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    if (r == 0) return false;  // file shorter than its metadata says
    p += r;
    n -= static_cast<uint64_t>(r);
    off += static_cast<uint64_t>(r);
  }
  return true;
}

constexpr const char* kSidecarMagic = "pegaflow-packed-file 1";

}  // namespace

std::string block_meta_json(const BlockMeta& m) {
  std::string o = "{\"file\":";
  json_string(&o, m.file);
  o += ",\"offset\":" + std::to_string(m.offset) + ",\"slots\":[";
  for (size_t i = 0; i < m.slots.size(); ++i) {
    if (i) o.push_back(',');
    o += std::string("{\"is_split\":") + (m.slots[i].is_split ? "true" : "false") +
         ",\"size\":" + std::to_string(m.slots[i].size) + "}";
  }
  o += "],\"total_slots\":" + std::to_string(m.total_slots) + "}";
  return o;
}

bool parse_block_meta_json(const std::string& s, BlockMeta* out) {
  JsonReader r(s);
  BlockMeta m;
  const bool ok = r.object([&](const std::string& k) {
    if (k == "file") return r.string(&m.file);
    if (k == "offset") return r.number(&m.offset);
    if (k == "total_slots") return r.number(&m.total_slots);
    if (k == "slots") {
      return r.array([&] {
        SlotMeta sm{false, 0};
        const bool good = r.object([&](const std::string& f) {
          if (f == "is_split") return r.boolean(&sm.is_split);
          if (f == "size") return r.number(&sm.size);
          return false;
        });
        m.slots.push_back(sm);
        return good;
      });
    }
    return false;
  });
  if (!ok || !r.done()) return false;
  *out = std::move(m);
  return true;
}

std::string file_meta_json(const std::vector<std::string>& hex_hashes, uint64_t size) {
  std::string o = "{\"blocks\":[";
  for (size_t i = 0; i < hex_hashes.size(); ++i) {
    if (i) o.push_back(',');
    json_string(&o, hex_hashes[i]);
  }
  o += "],\"size\":" + std::to_string(size) + "}";
  return o;
}

// ---------------------------------------------------------------------------
// Tier
// ---------------------------------------------------------------------------

DfsTier::DfsTier(Storage* storage, DfsConfig cfg) : storage_(storage), cfg_(std::move(cfg)) {
  if (cfg_.root.empty()) throw invalid_argument("dfs root must not be empty");
  if (cfg_.max_pack_size == 0) cfg_.max_pack_size = 64;
  if (cfg_.scan_interval_ms == 0) cfg_.scan_interval_ms = 100;
  std::error_code ec;
  fs::create_directories(cfg_.root, ec);
  if (ec) throw storage_error("cannot create dfs root " + cfg_.root + ": " + ec.message());
  load_index();
  writer_ = std::thread([this] { writer_loop(); });
  quota_ = std::thread([this] { quota_loop(); });
  prefetch_ = std::thread([this] { prefetch_loop(); });
}

DfsTier::~DfsTier() {
  {
    std::lock_guard<std::mutex> g(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  pcv_.notify_all();
  quota_cv_.notify_all();
  for (std::thread* t : {&writer_, &quota_, &prefetch_}) {
    if (t->joinable()) t->join();
  }
}

void DfsTier::load_index() {
  // The sidecar of each packed file carries the records the reference keeps
  // in Redis; a packed file without one cannot be found and is left alone.
  std::error_code ec;
  for (const auto& nsdir : fs::directory_iterator(cfg_.root, ec)) {
    if (!nsdir.is_directory()) continue;
    const std::string ns = nsdir.path().filename().string();
    for (const auto& f : fs::directory_iterator(nsdir.path(), ec)) {
      const std::string name = f.path().filename().string();
      const std::string suffix = ".bin.meta";
      if (name.size() <= suffix.size() || name.compare(name.size() - suffix.size(), suffix.size(), suffix) != 0) {
        continue;
      }
      const std::string bin = name.substr(0, name.size() - 5);  // "<uuid>.bin"
      if (!fs::exists(nsdir.path() / bin)) continue;
      std::ifstream in(f.path());
      std::string line;
      if (!std::getline(in, line) || line != kSidecarMagic) continue;
      FileEntry fe;
      fe.ns = ns;
      fe.uuid = bin.substr(0, bin.size() - 4);
      fe.member = ns + ":" + fe.uuid;
      fe.ts_ms = 0;
      fe.size = 0;
      std::vector<std::pair<std::string, BlockMeta>> blocks;
      bool good = true;
      try {
        while (std::getline(in, line)) {
          const size_t t1 = line.find('\t');
          if (t1 == std::string::npos) continue;
          const std::string tag = line.substr(0, t1);
          const std::string rest = line.substr(t1 + 1);
          if (tag == "timestamp_ms") {
            fe.ts_ms = std::stoull(rest);
          } else if (tag == "size") {
            fe.size = std::stoull(rest);
          } else if (tag == "block") {
            const size_t t2 = rest.find('\t');
            std::string hash;
            BlockMeta m;
            if (t2 == std::string::npos || !hex_decode(rest.substr(0, t2), &hash) ||
                !parse_block_meta_json(rest.substr(t2 + 1), &m)) {
              good = false;
              break;
            }
            blocks.emplace_back(std::move(hash), std::move(m));
          }
        }
      } catch (const std::exception&) {
        good = false;  // a damaged sidecar: its packed file is left unindexed
      }
      if (!good) continue;
      for (auto& hb : blocks) {
        fe.hashes.push_back(hb.first);
        index_[index_key(ns, hb.first)] = std::move(hb.second);
      }
      usage_ += fe.size;
      st_.blocks += blocks.size();
      files_.emplace(std::make_pair(fe.ts_ms, fe.member), std::move(fe));
    }
  }
  st_.files = files_.size();
}

void DfsTier::on_seal(const BlockKey& key, const SealedBlockPtr& block) {
  {
    std::lock_guard<std::mutex> g(mu_);
    queue_.emplace_back(key, std::weak_ptr<SealedBlock>(block));
  }
  cv_.notify_one();
}

void DfsTier::writer_loop() {
  // offload_loop (seal_offload.rs:231-290): take what has queued, up to one
  // packed file's worth, drop blocks already evicted, pack per namespace.
  for (;;) {
    std::vector<Pending> batch;
    {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [this] { return stop_ || !queue_.empty(); });
      if (stop_) return;
      while (!queue_.empty() && batch.size() < cfg_.max_pack_size) {
        batch.push_back(std::move(queue_.front()));
        queue_.pop_front();
      }
      writer_busy_ = true;
    }
    std::vector<std::string> order;
    std::unordered_map<std::string, std::vector<std::pair<BlockKey, SealedBlockPtr>>> by_ns;
    for (Pending& p : batch) {
      SealedBlockPtr b = p.second.lock();
      if (!b) continue;
      auto& v = by_ns[p.first.ns];
      if (v.empty()) order.push_back(p.first.ns);
      v.emplace_back(p.first, std::move(b));
    }
    for (const std::string& ns : order) {
      try {
        write_and_register(ns, by_ns[ns]);
      } catch (const std::exception& e) {
        fprintf(stderr, "pegaflow_b200: packed-file write failed: %s\n", e.what());
        std::lock_guard<std::mutex> g(mu_);
        st_.write_failures += 1;
      }
    }
    {
      std::lock_guard<std::mutex> g(mu_);
      writer_busy_ = false;
    }
    idle_cv_.notify_all();
  }
}

void DfsTier::write_and_register(const std::string& ns,
                                 const std::vector<std::pair<BlockKey, SealedBlockPtr>>& blocks) {
  // write_packed_file + write_and_register (seal_offload.rs:297-448).
  const fs::path dir = fs::path(cfg_.root) / ns;
  std::error_code ec;
  fs::create_directories(dir, ec);
  const std::string uuid = uuid_v4();
  const std::string file_name = uuid + ".bin";
  const fs::path path = dir / file_name;
  const uint64_t total_slots = blocks.front().second->slots.size();

  std::vector<BlockMeta> metas;
  uint64_t offset = 0, total_size = 0;
  for (const auto& kb : blocks) {
    BlockMeta m;
    m.file = file_name;
    m.offset = offset;
    m.total_slots = total_slots;
    for (const LayerBlock* s : kb.second->slots) m.slots.push_back(SlotMeta{s && s->v_ptr != nullptr, s ? s->size : 0});
    offset += m.total_size();
    total_size += kb.second->footprint;
    metas.push_back(std::move(m));
  }

  bool ok = true;
  const int fd = ::open(path.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
  if (fd < 0) ok = false;
  for (size_t b = 0; ok && b < blocks.size(); ++b) {
    for (const LayerBlock* s : blocks[b].second->slots) {
      if (!s) continue;
      if (s->v_ptr) {
        const uint64_t half = s->size / 2;
        ok = write_all(fd, s->k_ptr, half) && write_all(fd, s->v_ptr, half);
      } else {
        ok = write_all(fd, s->k_ptr, s->size);
      }
      if (!ok) break;
    }
  }
  if (fd >= 0) {
    if (ok && ::fsync(fd) != 0) ok = false;
    ::close(fd);
  }

  // The sidecar holds what the reference writes to Redis in one script
  // (LUA_WRITE_BATCH): the file's record, its timestamp and size, and every
  // block's record. Written to a temporary name and renamed into place.
  const uint64_t ts = now_ms();
  std::vector<std::string> hex;
  for (const auto& kb : blocks) hex.push_back(hex_encode(kb.first.hash));
  if (ok) {
    const fs::path side = dir / (file_name + ".meta");
    const fs::path tmp = dir / (file_name + ".meta.tmp");
    std::ofstream out(tmp, std::ios::trunc);
    out << kSidecarMagic << "\n"
        << "member\t" << ns << ":" << uuid << "\n"
        << "timestamp_ms\t" << ts << "\n"
        << "size\t" << total_size << "\n"
        << "file_meta\t" << file_meta_json(hex, total_size) << "\n";
    for (size_t b = 0; b < blocks.size(); ++b) out << "block\t" << hex[b] << "\t" << block_meta_json(metas[b]) << "\n";
    out.flush();
    ok = static_cast<bool>(out);
    out.close();
    if (ok) {
      fs::rename(tmp, side, ec);
      ok = !ec;
    }
    if (!ok) fs::remove(tmp, ec);
  }
  if (!ok) {
    fs::remove(path, ec);  // no orphaned packed file (seal_offload.rs:432-437)
    std::lock_guard<std::mutex> g(mu_);
    st_.write_failures += 1;
    return;
  }

  std::lock_guard<std::mutex> g(mu_);
  FileEntry fe{ns, uuid, ns + ":" + uuid, ts, total_size, {}};
  for (size_t b = 0; b < blocks.size(); ++b) {
    fe.hashes.push_back(blocks[b].first.hash);
    index_[index_key(ns, blocks[b].first.hash)] = metas[b];
  }
  usage_ += total_size;
  files_.emplace(std::make_pair(ts, fe.member), std::move(fe));
  st_.written_files += 1;
  st_.written_blocks += blocks.size();
}

void DfsTier::quota_loop() {
  std::unique_lock<std::mutex> lk(mu_);
  while (!stop_) {
    quota_cv_.wait_for(lk, std::chrono::milliseconds(cfg_.scan_interval_ms), [this] { return stop_; });
    if (stop_) return;
    lk.unlock();
    check_quota();
    lk.lock();
  }
}

void DfsTier::check_quota() {
  // check_quota + evict_oldest (seal_offload.rs:466-561): drop the oldest
  // packed files until usage is back under the quota.
  std::vector<FileEntry> gone;
  {
    std::lock_guard<std::mutex> g(mu_);
    if (usage_ <= cfg_.quota_bytes) return;
    const uint64_t target = usage_ - cfg_.quota_bytes;
    uint64_t freed = 0;
    while (freed < target && !files_.empty()) {
      FileEntry fe = std::move(files_.begin()->second);
      files_.erase(files_.begin());
      const std::string file_name = fe.uuid + ".bin";
      for (const std::string& h : fe.hashes) {
        // Only records that still point at this file: a block written again
        // later lives in a newer file.
        auto it = index_.find(index_key(fe.ns, h));
        if (it != index_.end() && it->second.file == file_name) index_.erase(it);
      }
      usage_ -= std::min(usage_, fe.size);
      freed += fe.size;
      st_.evicted_files += 1;
      gone.push_back(std::move(fe));
    }
  }
  std::error_code ec;
  for (const FileEntry& fe : gone) {
    const fs::path dir = fs::path(cfg_.root) / fe.ns;
    fs::remove(dir / (fe.uuid + ".bin.meta"), ec);
    fs::remove(dir / (fe.uuid + ".bin"), ec);
    fs::remove(dir, ec);  // only succeeds once the namespace directory is empty
  }
}

PrefetchStatus DfsTier::query(const std::string& ns, const std::vector<std::string>& hashes) {
  PrefetchStatus st;
  uint64_t ready = 0, loading = 0;
  size_t miss = hashes.size();
  for (size_t i = 0; i < hashes.size(); ++i) {
    if (storage_->cache_contains(ns, hashes[i])) {
      ++ready;
      continue;
    }
    std::lock_guard<std::mutex> g(mu_);
    if (pending_.count(index_key(ns, hashes[i]))) {
      ++loading;
      continue;
    }
    miss = i;
    break;
  }
  if (miss == hashes.size()) {
    st.state = loading ? PrefetchState::kLoading : PrefetchState::kReady;
    st.hit_blocks = ready;
    st.loading_blocks = loading;
    return st;
  }
  const uint64_t rest = hashes.size() - ready - loading;
  {
    std::lock_guard<std::mutex> g(mu_);
    if (!index_.count(index_key(ns, hashes[miss]))) {
      st.state = PrefetchState::kPartialMiss;
      st.hit_blocks = ready + loading;
      st.missing_blocks = rest;
      return st;
    }
    // Prefetch every later block the tier holds that is neither cached nor
    // already on its way (prefetch_blocks_inner, seal_offload.rs:676-720).
    PrefetchTask task;
    task.ns = ns;
    for (size_t i = miss; i < hashes.size(); ++i) {
      const std::string k = index_key(ns, hashes[i]);
      if (pending_.count(k)) continue;
      auto it = index_.find(k);
      if (it == index_.end()) continue;
      if (storage_->cache_contains(ns, hashes[i])) continue;
      pending_.insert(k);
      task.blocks.emplace_back(hashes[i], it->second);
    }
    if (!task.blocks.empty()) prefetch_queue_.push_back(std::move(task));
  }
  pcv_.notify_one();
  // As the reference reports it: everything from the first miss counts as loading.
  st.state = PrefetchState::kLoading;
  st.hit_blocks = ready;
  st.loading_blocks = loading + (hashes.size() - miss);
  return st;
}

void DfsTier::prefetch_loop() {
  for (;;) {
    PrefetchTask task;
    {
      std::unique_lock<std::mutex> lk(mu_);
      pcv_.wait(lk, [this] { return stop_ || !prefetch_queue_.empty(); });
      if (stop_) return;
      task = std::move(prefetch_queue_.front());
      prefetch_queue_.pop_front();
      prefetch_busy_ = true;
    }
    try {
      run_prefetch(task);
    } catch (const std::exception& e) {
      fprintf(stderr, "pegaflow_b200: packed-file prefetch failed: %s\n", e.what());
      std::lock_guard<std::mutex> g(mu_);
      st_.prefetch_failures += 1;
    }
    {
      std::lock_guard<std::mutex> g(mu_);
      for (const auto& hb : task.blocks) pending_.erase(index_key(task.ns, hb.first));
      prefetch_busy_ = false;
    }
    idle_cv_.notify_all();
  }
}

void DfsTier::run_prefetch(PrefetchTask& task) {
  // read_file_blocks + rebuild_sealed_block (seal_offload.rs:785-909): per
  // file, in offset order, read each block into one pool allocation and
  // rebuild it with its slots pointing into that allocation. The rebuilt
  // blocks enter the cache together once the task has read them all (the
  // reference inserts each at once): a pool allocation later in the task may
  // reclaim cached blocks in batches, and must not take back ones this task
  // has just read. They count as loading until then either way.
  std::vector<std::pair<std::string, SealedBlockPtr>> rebuilt;
  std::map<std::string, std::vector<size_t>> by_file;
  for (size_t i = 0; i < task.blocks.size(); ++i) by_file[task.blocks[i].second.file].push_back(i);
  uint64_t loaded = 0, failed = 0;
  for (auto& fb : by_file) {
    std::sort(fb.second.begin(), fb.second.end(),
              [&](size_t a, size_t b) { return task.blocks[a].second.offset < task.blocks[b].second.offset; });
    const fs::path path = fs::path(cfg_.root) / task.ns / fb.first;
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
      failed += fb.second.size();
      continue;
    }
    for (size_t i : fb.second) {
      const std::string& hash = task.blocks[i].first;
      const BlockMeta& m = task.blocks[i].second;
      const uint64_t size = m.total_size();
      if (m.total_slots == 0 || size == 0 || storage_->cache_contains(task.ns, hash)) continue;
      std::shared_ptr<PoolAllocation> alloc = storage_->allocate(size);
      if (!alloc || !read_all_at(fd, alloc->ptr, size, m.offset)) {
        failed += 1;
        continue;
      }
      auto batch = std::make_shared<LayerBlockBatch>();
      batch->k_alloc = alloc;
      batch->blocks.resize(m.slots.size());
      uint64_t off = 0;
      for (size_t s = 0; s < m.slots.size(); ++s) {
        uint8_t* base = alloc->ptr + off;
        batch->blocks[s] = LayerBlock{base, m.slots[s].is_split ? base + m.slots[s].size / 2 : nullptr, m.slots[s].size};
        off += m.slots[s].size;
      }
      auto sealed = std::make_shared<SealedBlock>();
      sealed->slots.resize(m.slots.size());
      for (size_t s = 0; s < m.slots.size(); ++s) sealed->slots[s] = &batch->blocks[s];
      sealed->owners.push_back(batch);
      sealed->footprint = size;
      rebuilt.emplace_back(hash, std::move(sealed));
    }
    ::close(fd);
  }
  for (auto& hb : rebuilt) {
    storage_->cache_insert(task.ns, hb.first, std::move(hb.second));
    loaded += 1;
  }
  std::lock_guard<std::mutex> g(mu_);
  st_.prefetched_blocks += loaded;
  st_.prefetch_failures += failed;
}

bool DfsTier::flush(double timeout_s) {
  std::unique_lock<std::mutex> lk(mu_);
  return idle_cv_.wait_for(lk, std::chrono::duration<double>(timeout_s), [this] {
    return queue_.empty() && prefetch_queue_.empty() && !writer_busy_ && !prefetch_busy_;
  });
}

DfsStats DfsTier::stats() {
  std::lock_guard<std::mutex> g(mu_);
  DfsStats s = st_;
  s.files = files_.size();
  s.blocks = index_.size();
  s.usage_bytes = usage_;
  return s;
}

bool DfsTier::has_block(const std::string& ns, const std::string& hash) {
  std::lock_guard<std::mutex> g(mu_);
  return index_.count(index_key(ns, hash)) != 0;
}

}  // namespace pf
