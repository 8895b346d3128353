// Shared helpers: status + thread-local error message, CUDA error mapping.
#pragma once

#include <cuda.h>
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

// The driver's current-context calls, resolved through the runtime so the
// library needs no libcuda at link time. Either pointer is null when the
// driver does not provide it.
struct CtxCalls {
  CUresult (*get)(CUcontext*) = nullptr;
  CUresult (*set)(CUcontext) = nullptr;
};

inline const CtxCalls& ctx_calls() {
  static const CtxCalls calls = [] {
    CtxCalls c;
    void* g = nullptr;
    void* s = nullptr;
    cudaDriverEntryPointQueryResult qg{}, qs{};
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &g, 4000, cudaEnableDefault, &qg) == cudaSuccess &&
        cudaGetDriverEntryPointByVersion("cuCtxSetCurrent", &s, 4000, cudaEnableDefault, &qs) == cudaSuccess &&
        qg == cudaDriverEntryPointSuccess && qs == cudaDriverEntryPointSuccess) {
      c.get = reinterpret_cast<CUresult (*)(CUcontext*)>(g);
      c.set = reinterpret_cast<CUresult (*)(CUcontext)>(s);
    }
    cudaGetLastError();
    return c;
  }();
  return calls;
}

// Makes `device` current on the calling thread for one scope, then puts the
// caller's own context back, including "no context": a caller working on
// device 1 that saves for device 0 finds device 1 current afterwards, and a
// thread that had no context gets none. With the runtime linked statically
// the current device is the driver's current context, which every other
// CUDA user in the process (torch included) sees.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    const CtxCalls& c = ctx_calls();
    if (c.get && c.set && c.get(&prev_) == CUDA_SUCCESS) restore_ = true;
    const cudaError_t err = cudaSetDevice(device);
    if (err != cudaSuccess) {
      if (restore_) c.set(prev_);
      cuda_check(err, "cudaSetDevice");
    }
  }
  ~DeviceGuard() {
    if (restore_) ctx_calls().set(prev_);
  }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;

 private:
  CUcontext prev_ = nullptr;
  bool restore_ = false;
};

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
