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

// M-tiled per-channel prefill (prefill.cu): 64 query rows per CTA over K/V
// chunks dequantized once into shared memory.  Arguments as
// slmt_per_channel_prefill (checked by the caller); out_dtype 0 f16, 1 bf16,
// 2 f32.
int prefill_pc_launch(const void* q, int q_bf16, int64_t q_head_stride, int64_t q_row_stride,
                      const uint8_t* k_packed, const uint8_t* v_packed, int64_t seq_len, const uint16_t* k_scale,
                      const uint16_t* k_zero, const uint16_t* v_scale, const uint16_t* v_zero, int use_quant,
                      int causal, int64_t num_rows, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                      float sm_scale, void* out, int out_dtype, int64_t out_head_stride, int64_t out_row_stride,
                      cudaStream_t st);

// M-tiled prefill over the paged per-token cache (prefill.cu): request r's
// query rows [qsl[r], qsl[r+1]) attend causally to its seq_lens[r] cached
// keys.  Arguments as slmt_paged_prefill (checked by the caller); bt_i64 0/1,
// out_dtype 0 f16, 1 bf16, 2 f32.
int prefill_paged_launch(const void* q, int q_bf16, int64_t q_row_stride, int64_t q_head_stride,
                         const uint8_t* kv_cache, int64_t num_blocks, int64_t block_size, int64_t num_kv_heads,
                         int64_t head_dim, const void* block_tables, int bt_i64, int64_t bt_seq_stride,
                         int64_t max_blocks_per_seq, const int32_t* query_start_loc, const int32_t* seq_lens,
                         int64_t num_reqs, int64_t max_query_len, int64_t num_q_heads, float sm_scale, void* out,
                         int out_dtype, int64_t out_row_stride, int64_t out_head_stride, int32_t* err_flag,
                         cudaStream_t st);

}  // namespace slmt
