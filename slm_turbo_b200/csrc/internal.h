// internal.h -- host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "slm_turbo_b200.h"

namespace slmt {

inline bool valid_head_dim(int64_t d) { return d == 64 || d == 80 || d == 128; }

// Status of the launch just issued (clears the sticky-free launch error).
inline int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SLMT_OK : SLMT_ERR_CUDA;
}

// SM count of the current device, cached per device id.
int current_device_sms(int* device_out);

// Bytes at the start of a split-K workspace of `workspace_bytes` that hold
// the per-segment arrival counters (zero between calls).  Every entry point
// that lays out or resets a workspace uses this one definition.
int64_t counter_region(int64_t workspace_bytes);

}  // namespace slmt
