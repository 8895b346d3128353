// The reference's copy strategy, restated so it can be timed beside the
// kernels on the same GPU. It issues the same CUDA copies in the same order
// as pegaflow-core's worker; it is a measurement baseline, not a product path.
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "common.h"
#include "executor.h"

namespace pf {

namespace {

void refcopy_save_layer(const pf_save_layer& s) {
  const pf_layer_desc& l = s.layer;
  const uint64_t seg = l.bytes_per_block;
  const uint64_t block_size = l.bytes_per_block * l.segments;
  auto* k = static_cast<uint8_t*>(s.k_dst);
  auto* v = static_cast<uint8_t*>(s.v_dst);
  if (is_split_layout(l)) {
    // gpu_worker.rs:334-360: all K segments, then all V segments, one
    // synchronous device-to-host copy each.
    std::vector<uint64_t> koff(s.n), voff(s.n);
    for (uint64_t i = 0; i < s.n; ++i) {
      koff[i] = segment_offset(l, static_cast<uint64_t>(s.block_idx[i]), 0);
      voff[i] = segment_offset(l, static_cast<uint64_t>(s.block_idx[i]), 1);
    }
    for (uint64_t i = 0; i < s.n; ++i) {
      cuda_check(cudaMemcpy(k + i * seg, reinterpret_cast<void*>(l.data_ptr + koff[i]), seg, cudaMemcpyDeviceToHost),
                 "cuMemcpyDtoH (K)");
    }
    for (uint64_t i = 0; i < s.n; ++i) {
      uint8_t* dst = v ? v + i * seg : k + i * seg + seg;
      cuda_check(cudaMemcpy(dst, reinterpret_cast<void*>(l.data_ptr + voff[i]), seg, cudaMemcpyDeviceToHost),
                 "cuMemcpyDtoH (V)");
    }
    return;
  }
  // gpu_worker.rs:364-372 -> copy_block_gpu_to_cpu (transfer.rs:200-239)
  for (uint64_t i = 0; i < s.n; ++i) {
    const uint64_t b = static_cast<uint64_t>(s.block_idx[i]);
    uint8_t* dst = k + i * block_size;
    if (is_contiguous_layout(l)) {
      const uint64_t off = segment_offset(l, b, 0);
      cuda_check(cudaMemcpy(dst, reinterpret_cast<void*>(l.data_ptr + off), block_size, cudaMemcpyDeviceToHost),
                 "cuMemcpyDtoH");
    } else {
      for (uint64_t sg = 0; sg < l.segments; ++sg) {
        const uint64_t off = segment_offset(l, b, sg);
        cuda_check(cudaMemcpy(dst + sg * seg, reinterpret_cast<void*>(l.data_ptr + off), seg, cudaMemcpyDeviceToHost),
                   "cuMemcpyDtoH");
      }
    }
  }
}

// batch_copy_segments_to_gpu (transfer.rs:116-198): merge maximal runs where
// the GPU offset and the host pointer both advance by segment_size.
uint64_t refcopy_runs(const std::vector<std::pair<uint64_t, const uint8_t*>>& xfers, uint64_t seg,
                      const pf_layer_desc& l, cudaStream_t stream) {
  uint64_t runs = 0;
  size_t i = 0;
  while (i < xfers.size()) {
    const uint64_t g0 = xfers[i].first;
    const uint8_t* h0 = xfers[i].second;
    size_t count = 1;
    while (i + count < xfers.size() && xfers[i + count].first == g0 + count * seg &&
           xfers[i + count].second == h0 + count * seg) {
      ++count;
    }
    cuda_check(cudaMemcpyAsync(reinterpret_cast<void*>(l.data_ptr + g0), h0, seg * count, cudaMemcpyHostToDevice,
                               stream),
               "cuMemcpyHtoDAsync");
    ++runs;
    i += count;
  }
  return runs;
}

}  // namespace

void refcopy_save(int device, const pf_save_layer* layers, uint64_t n) {
  DeviceGuard on(device);
  for (uint64_t li = 0; li < n; ++li) {
    validate_layout(layers[li].layer, ("#" + std::to_string(li)).c_str());
    refcopy_save_layer(layers[li]);
  }
}

uint64_t refcopy_load(int device, const pf_load_layer* layers, uint64_t n) {
  DeviceGuard on(device);
  cudaStream_t stream;
  cuda_check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
  uint64_t runs = 0;
  try {
    // process_load_task (gpu_worker.rs:211-283)
    for (uint64_t li = 0; li < n; ++li) {
      const pf_load_layer& s = layers[li];
      const pf_layer_desc& l = s.layer;
      validate_layout(l, ("#" + std::to_string(li)).c_str());
      if (s.n == 0) continue;
      if (is_split_layout(l)) {
        std::vector<std::pair<uint64_t, const uint8_t*>> kx, vx;
        for (uint64_t i = 0; i < s.n; ++i) {
          const uint64_t b = static_cast<uint64_t>(s.block_idx[i]);
          const auto* kp = static_cast<const uint8_t*>(s.k_src[i]);
          const auto* vp = (s.v_src && s.v_src[i]) ? static_cast<const uint8_t*>(s.v_src[i]) : kp + l.bytes_per_block;
          kx.emplace_back(segment_offset(l, b, 0), kp);
          vx.emplace_back(segment_offset(l, b, 1), vp);
        }
        runs += refcopy_runs(kx, l.bytes_per_block, l, stream);
        runs += refcopy_runs(vx, l.bytes_per_block, l, stream);
      } else {
        const uint64_t block_size = l.bytes_per_block * l.segments;
        std::vector<std::pair<uint64_t, const uint8_t*>> x;
        for (uint64_t i = 0; i < s.n; ++i) {
          const uint64_t b = static_cast<uint64_t>(s.block_idx[i]);
          const uint64_t off = segment_offset(l, b, 0);
          if (off + block_size > l.size_bytes) {
            throw storage_error("Block " + std::to_string(b) + " exceeds registered memory");
          }
          x.emplace_back(off, static_cast<const uint8_t*>(s.k_src[i]));
        }
        runs += refcopy_runs(x, block_size, l, stream);
      }
    }
    cudaEvent_t ev;  // gpu_worker.rs:286-291
    cuda_check(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "cudaEventCreate");
    cuda_check(cudaEventRecord(ev, stream), "record_event");
    cudaError_t err = cudaEventSynchronize(ev);
    cudaEventDestroy(ev);
    cuda_check(err, "synchronize");
  } catch (...) {
    cudaStreamSynchronize(stream);
    cudaStreamDestroy(stream);
    throw;
  }
  cudaStreamDestroy(stream);
  return runs;
}

}  // namespace pf
