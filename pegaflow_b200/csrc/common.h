// Shared helpers: status + thread-local error message, CUDA error mapping.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

#include "pegaflow.h"

namespace pf {

// An error carrying one of the pf_status codes. Its message is the text the
// reference's EngineError Display impl would produce (lib.rs:69-83).
class Error : public std::runtime_error {
 public:
  Error(int code, const std::string& msg) : std::runtime_error(msg), code_(code) {}
  int code() const { return code_; }

 private:
  int code_;
};

inline Error instance_missing(const std::string& id) {
  return Error(PF_ERR_INSTANCE_MISSING, "instance " + id + " not found");
}
inline Error worker_missing(const std::string& id, int device) {
  return Error(PF_ERR_WORKER_MISSING,
               "device " + std::to_string(device) + " not found in instance " + id);
}
inline Error invalid_argument(const std::string& msg) {
  return Error(PF_ERR_INVALID_ARGUMENT, "invalid argument: " + msg);
}
inline Error cuda_init(const std::string& msg) {
  return Error(PF_ERR_CUDA_INIT, "failed to initialize CUDA: " + msg);
}
inline Error storage_error(const std::string& msg) {
  return Error(PF_ERR_STORAGE, "storage error: " + msg);
}
inline Error topology_mismatch(const std::string& msg) {
  return Error(PF_ERR_TOPOLOGY_MISMATCH, "topology mismatch: " + msg);
}

// Thread-local last-error slot behind pf_last_error().
void set_last_error(const std::string& msg);
const char* last_error();

// Throws storage_error("<what> failed: <cuda error>") on failure: copy and
// stream failures surface as EngineError::Storage in the reference
// (gpu_worker.rs:243-291).
inline void cuda_check(cudaError_t err, const char* what) {
  if (err != cudaSuccess) {
    throw storage_error(std::string(what) + " failed: " + cudaGetErrorString(err));
  }
}

// Runs f, converting exceptions into a status code + thread-local message.
template <typename F>
int guarded(F&& f) {
  try {
    f();
    return PF_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code();
  } catch (const std::bad_alloc&) {
    set_last_error("storage error: host allocation failed");
    return PF_ERR_STORAGE;
  } catch (const std::exception& e) {
    set_last_error(std::string("storage error: ") + e.what());
    return PF_ERR_STORAGE;
  }
}

// Checked arithmetic mirroring the reference's checked_mul/checked_add.
inline bool mul_ovf(uint64_t a, uint64_t b, uint64_t* out) {
  return __builtin_mul_overflow(a, b, out);
}
inline bool add_ovf(uint64_t a, uint64_t b, uint64_t* out) {
  return __builtin_add_overflow(a, b, out);
}

}  // namespace pf
