// Protobuf wire decoding of engine.proto's SaveRequest and LoadRequest (see
// wire.h for why the server decodes these two natively).
#include "wire.h"

#include <cstring>
#include <memory>
#include <string_view>

#include "common.h"

namespace pf {
namespace {

enum WireType : uint32_t { kVarint = 0, kFixed64 = 1, kLen = 2, kFixed32 = 5 };

class Reader {
 public:
  Reader(const uint8_t* p, size_t n) : p_(p), end_(p + n) {}
  bool done() const { return p_ >= end_; }

  uint64_t varint() {
    uint64_t v = 0;
    for (int shift = 0; shift < 70; shift += 7) {
      if (p_ >= end_) throw invalid_argument("truncated request (varint)");
      const uint8_t b = *p_++;
      v |= static_cast<uint64_t>(b & 0x7f) << shift;
      if ((b & 0x80) == 0) return v;
    }
    throw invalid_argument("malformed request (varint longer than 10 bytes)");
  }

  std::string_view bytes() {
    const uint64_t n = varint();
    if (n > static_cast<uint64_t>(end_ - p_)) throw invalid_argument("truncated request (length-delimited field)");
    std::string_view s(reinterpret_cast<const char*>(p_), static_cast<size_t>(n));
    p_ += n;
    return s;
  }

  void skip(uint32_t wire_type) {
    switch (wire_type) {
      case kVarint:
        varint();
        return;
      case kFixed64:
        advance(8);
        return;
      case kLen:
        bytes();
        return;
      case kFixed32:
        advance(4);
        return;
      default:
        throw invalid_argument("malformed request (wire type " + std::to_string(wire_type) + ")");
    }
  }

  // Reads a tag; returns false at the end of the message.
  bool tag(uint32_t* field, uint32_t* wire_type) {
    if (done()) return false;
    const uint64_t t = varint();
    *field = static_cast<uint32_t>(t >> 3);
    *wire_type = static_cast<uint32_t>(t & 7);
    if (*field == 0) throw invalid_argument("malformed request (field number 0)");
    return true;
  }

 private:
  void advance(size_t n) {
    if (n > static_cast<size_t>(end_ - p_)) throw invalid_argument("truncated request (fixed field)");
    p_ += n;
  }
  const uint8_t* p_;
  const uint8_t* end_;
};

std::string_view expect_len(Reader& r, uint32_t wt, const char* what) {
  if (wt != kLen) throw invalid_argument(std::string("malformed request (") + what + " is not length-delimited)");
  return r.bytes();
}

uint64_t expect_varint(Reader& r, uint32_t wt, const char* what) {
  if (wt != kVarint) throw invalid_argument(std::string("malformed request (") + what + " is not a varint)");
  return r.varint();
}

// A repeated int32, packed (one length-delimited run of varints) or not.
void read_int32s(Reader& r, uint32_t wt, std::vector<int32_t>* out) {
  if (wt == kVarint) {
    out->push_back(static_cast<int32_t>(r.varint()));
    return;
  }
  const std::string_view run = expect_len(r, wt, "block_ids");
  Reader pr(reinterpret_cast<const uint8_t*>(run.data()), run.size());
  while (!pr.done()) out->push_back(static_cast<int32_t>(pr.varint()));
}

}  // namespace

void decode_save_request(const uint8_t* data, size_t len, SaveRequestWire* out) {
  *out = SaveRequestWire{};
  Reader r(data, len);
  uint32_t field = 0, wt = 0;
  // Per layer, its hashes as views into `data` until the shared lists are built.
  std::vector<std::vector<std::string_view>> layer_hashes;
  while (r.tag(&field, &wt)) {
    switch (field) {
      case 1:
        out->instance_id = std::string(expect_len(r, wt, "instance_id"));
        break;
      case 2:
        out->tp_rank = static_cast<uint32_t>(expect_varint(r, wt, "tp_rank"));
        break;
      case 3:
        out->device_id = static_cast<int32_t>(expect_varint(r, wt, "device_id"));
        break;
      case 4: {
        const std::string_view msg = expect_len(r, wt, "saves");
        Reader lr(reinterpret_cast<const uint8_t*>(msg.data()), msg.size());
        Engine::SaveEntry entry;
        std::vector<std::string_view> hashes;
        uint32_t f = 0, w = 0;
        while (lr.tag(&f, &w)) {
          if (f == 1) {
            entry.layer_name = std::string(expect_len(lr, w, "layer_name"));
          } else if (f == 2) {
            read_int32s(lr, w, &entry.block_ids);
          } else if (f == 3) {
            hashes.push_back(expect_len(lr, w, "block_hashes"));
          } else {
            lr.skip(w);
          }
        }
        out->saves.push_back(std::move(entry));
        layer_hashes.push_back(std::move(hashes));
        break;
      }
      default:
        r.skip(wt);
    }
  }
  // One hash list per distinct content: a layer whose hashes equal the
  // previous layer's shares that layer's list.
  for (size_t i = 0; i < out->saves.size(); ++i) {
    if (i > 0 && layer_hashes[i] == layer_hashes[i - 1]) {
      out->saves[i].hashes = out->saves[i - 1].hashes;
      continue;
    }
    auto list = std::make_shared<std::vector<std::string>>();
    list->reserve(layer_hashes[i].size());
    for (std::string_view h : layer_hashes[i]) list->emplace_back(h);
    out->saves[i].hashes = std::move(list);
  }
}

void decode_load_request(const uint8_t* data, size_t len, LoadRequestWire* out) {
  *out = LoadRequestWire{};
  Reader r(data, len);
  uint32_t field = 0, wt = 0;
  while (r.tag(&field, &wt)) {
    switch (field) {
      case 1:
        out->instance_id = std::string(expect_len(r, wt, "instance_id"));
        break;
      case 2:
        out->tp_rank = static_cast<uint32_t>(expect_varint(r, wt, "tp_rank"));
        break;
      case 3:
        out->device_id = static_cast<int32_t>(expect_varint(r, wt, "device_id"));
        break;
      case 4:
        out->load_state_shm = std::string(expect_len(r, wt, "load_state_shm"));
        break;
      case 5:
        out->layer_names.emplace_back(expect_len(r, wt, "layer_names"));
        break;
      case 6:
        read_int32s(r, wt, &out->block_ids);
        break;
      case 7:
        out->block_hashes.emplace_back(expect_len(r, wt, "block_hashes"));
        break;
      default:
        r.skip(wt);
    }
  }
}

std::string decode_request_instance_id(const uint8_t* data, size_t len) {
  Reader r(data, len);
  uint32_t field = 0, wt = 0;
  std::string id;
  while (r.tag(&field, &wt)) {
    if (field == 1 && wt == kLen) {
      id = std::string(r.bytes());
    } else {
      r.skip(wt);
    }
  }
  return id;
}

}  // namespace pf
