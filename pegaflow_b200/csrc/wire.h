// Decoding of the engine.proto Save and Load requests (pegaflow-proto/proto/
// engine.proto:5-115) straight from their protobuf wire bytes, for the gRPC
// server's two data-path RPCs.
//
// A Save request for 80 layers x 2,048 blocks is about 6 MB of wire bytes.
// Turning it into per-layer Python lists and ctypes arrays costs tens of
// milliseconds of interpreter time per call, under the GIL, where the
// reference's Rust server decodes it natively. Here the server hands the raw
// bytes to the library, and the decoder builds the engine's arguments
// directly. Layers whose hash list is byte-for-byte the one of an earlier
// layer share a single list (the connector sends one list per request for all
// of its layers), which is also what lets the engine insert slots hash-major.
//
// The decoder follows the protobuf wire format: fields in any order, packed
// or unpacked repeated scalars, unknown fields skipped by wire type, and the
// last occurrence of a singular field wins. Malformed input throws
// invalid_argument.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "engine.h"

namespace pf {

struct SaveRequestWire {
  std::string instance_id;
  uint64_t tp_rank = 0;
  int32_t device_id = 0;
  std::vector<Engine::SaveEntry> saves;
};

struct LoadRequestWire {
  std::string instance_id;
  uint64_t tp_rank = 0;
  int32_t device_id = 0;
  std::string load_state_shm;
  std::vector<std::string> layer_names;
  std::vector<int32_t> block_ids;
  std::vector<std::string> block_hashes;
};

// SaveRequest {1: instance_id, 2: tp_rank, 3: device_id, 4: repeated SaveLayer
// {1: layer_name, 2: repeated int32 block_ids, 3: repeated bytes block_hashes}}.
void decode_save_request(const uint8_t* data, size_t len, SaveRequestWire* out);
// LoadRequest {1: instance_id, 2: tp_rank, 3: device_id, 4: load_state_shm,
// 5: repeated layer_names, 6: repeated int32 block_ids, 7: repeated bytes
// block_hashes}.
void decode_load_request(const uint8_t* data, size_t len, LoadRequestWire* out);
// Field 1 (instance_id) of a Save or Load request, without decoding the rest.
std::string decode_request_instance_id(const uint8_t* data, size_t len);

}  // namespace pf
