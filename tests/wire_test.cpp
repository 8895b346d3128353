// The native decoder of engine.proto's Save and Load requests
// (pegaflow_b200/csrc/wire.cpp) on request files: prints each decoded field in
// a canonical text form that tests/test_wire.py compares with the protobuf
// library's own parse of the same bytes.
//
//   wire_test save|load|id <request file>
//
// Strings and bytes print as hex. A malformed request prints "error: <msg>"
// and exits 2.
#include <cstdio>
#include <fstream>
#include <iterator>
#include <string>
#include <vector>

#include "common.h"
#include "wire.h"

namespace {

std::string hex(const std::string& s) {
  static const char* d = "0123456789abcdef";
  std::string o;
  for (unsigned char c : s) {
    o += d[c >> 4];
    o += d[c & 15];
  }
  return o;
}

template <typename T>
std::string join(const std::vector<T>& v) {
  std::string o;
  for (size_t i = 0; i < v.size(); ++i) o += (i ? "," : "") + std::to_string(v[i]);
  return o;
}

std::string join_hex(const std::vector<std::string>& v) {
  std::string o;
  for (size_t i = 0; i < v.size(); ++i) o += (i ? "," : "") + hex(v[i]);
  return o;
}

}  // namespace

namespace pf {
void set_last_error(const std::string&) {}
}  // namespace pf

int main(int argc, char** argv) {
  if (argc != 3) {
    std::fprintf(stderr, "usage: wire_test save|load|id <file>\n");
    return 1;
  }
  std::ifstream f(argv[2], std::ios::binary);
  const std::string data((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  const auto* p = reinterpret_cast<const uint8_t*>(data.data());
  const std::string mode = argv[1];
  try {
    if (mode == "id") {
      std::printf("instance_id=%s\n", hex(pf::decode_request_instance_id(p, data.size())).c_str());
    } else if (mode == "save") {
      pf::SaveRequestWire r;
      pf::decode_save_request(p, data.size(), &r);
      std::printf("instance_id=%s\ntp_rank=%llu\ndevice_id=%d\nlayers=%zu\n", hex(r.instance_id).c_str(),
                  static_cast<unsigned long long>(r.tp_rank), r.device_id, r.saves.size());
      for (size_t i = 0; i < r.saves.size(); ++i) {
        const auto& s = r.saves[i];
        const bool shared = i > 0 && s.hashes.get() == r.saves[i - 1].hashes.get();
        std::printf("layer %zu name=%s ids=%s hashes=%s shared=%d\n", i, hex(s.layer_name).c_str(),
                    join(s.block_ids).c_str(), join_hex(*s.hashes).c_str(), shared ? 1 : 0);
      }
    } else if (mode == "load") {
      pf::LoadRequestWire r;
      pf::decode_load_request(p, data.size(), &r);
      std::printf("instance_id=%s\ntp_rank=%llu\ndevice_id=%d\nshm=%s\nnames=%s\nids=%s\nhashes=%s\n",
                  hex(r.instance_id).c_str(), static_cast<unsigned long long>(r.tp_rank), r.device_id,
                  hex(r.load_state_shm).c_str(), join_hex(r.layer_names).c_str(), join(r.block_ids).c_str(),
                  join_hex(r.block_hashes).c_str());
    } else {
      return 1;
    }
  } catch (const std::exception& e) {
    std::printf("error: %s\n", e.what());
    return 2;
  }
  return 0;
}
