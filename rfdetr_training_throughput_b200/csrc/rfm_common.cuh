// Shared helpers of the rfm CUDA library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "rfm.h"

namespace rfm {

constexpr unsigned kFullMask = 0xffffffffu;

// Maps a CUDA launch-time error onto the library's return codes.
inline int launch_status() {
  const cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess) return RFM_OK;
  if (err == cudaErrorNoDevice || err == cudaErrorInsufficientDriver) return RFM_ERR_NO_DEVICE;
  return RFM_ERR_LAUNCH;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Waits until the grid this one was launched after (with programmatic stream
// serialization) has completed and its memory operations are visible; returns
// at once for a grid launched without that attribute.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// rfm_cost with `reset_word` (when not null, and the layout is target-major)
// set to 0 by the cost kernel: rfm_match uses it for the solver's counter.
int cost_run(const float* pred_logits, const float* pred_boxes, const int64_t* tgt_labels,
             const float* tgt_boxes, const int32_t* tgt_offsets, int num_layers, int num_images,
             int num_queries, int num_classes, int sum_targets, int64_t ld, int layout,
             float cost_class, float cost_bbox, float cost_giou, float focal_alpha, float* out,
             int* reset_word, void* stream);

// Unique id of the CUDA context current on the calling thread (the runtime's
// primary context of the current device once the runtime has initialised it),
// or 0 when no context is current or the driver cannot say.  Ids are never
// reused within a process, so state that belongs to one context (a kernel
// attribute, the device address of a module variable) is cached under this id
// and is looked up afresh after the context is destroyed and recreated
// (cudaDeviceReset).
unsigned long long current_context_id();

// SMs of the current device (1 if the runtime cannot say).
inline int device_sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) {
    cudaGetLastError();
    return 1;
  }
  return n;
}

}  // namespace rfm
