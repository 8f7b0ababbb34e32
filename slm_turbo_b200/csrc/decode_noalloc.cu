// decode_noalloc.cu -- slmt_paged_decode_noalloc: the batched paged decode
// with its split-K scratch in a static device array of this library instead
// of a buffer the caller allocates.
//
// Who needs it: a serving engine that hands all of HBM to its page pool and
// activation arena before the first request has no spare device memory to
// give an attention op, and some hosts (plugin runtimes, custom allocators
// that refuse allocation while a step is running) give the op no allocator
// at all.  Those callers cannot provide the workspace slmt_paged_decode
// takes, and an op that allocated on their hot path would stall on the
// driver or fail outright.  This entry point allocates nothing: no
// cudaMalloc, no cudaFree, no allocating library call.  The scratch below is
// reserved when the CUDA module is loaded, and the call reaches it through
// cudaGetSymbolAddress.
#include <cuda_runtime.h>

#include <mutex>

#include "internal.h"
#include "slm_turbo_b200.h"

namespace {

// Zero-filled when the module is loaded.  It starts with the split-K
// segment arrival counters, which must be zero when a launch begins; every
// launch that completes without a device error leaves them at zero again.
static __device__ __align__(256) unsigned char g_decode_scratch[SLMT_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch[kMaxDevices] = {};

// Device address of g_decode_scratch in the context of device `dev` (the
// current device).  The lookup runs once per device, on the first call made
// there, and is cached for the life of the process: the cache assumes the
// device's primary context lives that long (after cudaDeviceReset the module
// is loaded again elsewhere and the cached address is stale).
int scratch_address(int dev, void** out) {
  if (dev >= 0 && dev < kMaxDevices) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || !p) return SLMT_ERR_CUDA;
      g_scratch[dev] = p;
    }
    *out = g_scratch[dev];
    return SLMT_OK;
  }
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || !p) return SLMT_ERR_CUDA;
  *out = p;
  return SLMT_OK;
}

}  // namespace

extern "C" int slmt_paged_decode_noalloc(
    const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
    const uint8_t* kv_cache, int64_t num_blocks, int64_t block_size,
    int64_t num_kv_heads, int64_t head_dim, const void* block_tables,
    int bt_dtype, int64_t bt_seq_stride, int64_t max_blocks_per_seq,
    const int32_t* seq_lens, int64_t seq_len_scalar, int64_t max_seq_len_hint,
    int64_t num_seqs, int64_t num_q_heads, float sm_scale, void* out,
    int out_dtype, int64_t out_seq_stride, int64_t out_head_stride,
    int reset_scratch, int32_t* err_flag, void* stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SLMT_ERR_CUDA;
  // Worst-case scratch of this request (the bound slmt_decode_workspace_bytes
  // gives); anything above the static array is refused before any launch.
  const int64_t need = slmt_decode_workspace_bytes(num_seqs, num_q_heads, num_kv_heads, head_dim, dev);
  if (need < 0) return (int)need;
  if (need > (int64_t)SLMT_NOALLOC_SCRATCH_BYTES) return SLMT_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  int rc = scratch_address(dev, &scratch);
  if (rc != SLMT_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (reset_scratch) {
    // the counter region of a workspace of the array's size
    const size_t zero = (size_t)slmt::counter_region((int64_t)SLMT_NOALLOC_SCRATCH_BYTES);
    if (cudaMemsetAsync(scratch, 0, zero, st) != cudaSuccess) return SLMT_ERR_CUDA;
  }
  return slmt_paged_decode(q, q_dtype, q_seq_stride, q_head_stride, kv_cache, num_blocks, block_size,
                           num_kv_heads, head_dim, block_tables, bt_dtype, bt_seq_stride,
                           max_blocks_per_seq, seq_lens, seq_len_scalar, max_seq_len_hint, num_seqs,
                           num_q_heads, sm_scale, out, out_dtype, out_seq_stride, out_head_stride,
                           scratch, (int64_t)SLMT_NOALLOC_SCRATCH_BYTES, err_flag, stream);
}
