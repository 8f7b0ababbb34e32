/*
 * slm_turbo_b200.h -- C ABI of the B200 (sm_100a) 4-bit KV-cache kernels.
 *
 * Every entry point takes plain device pointers, 64-bit sizes/strides (in
 * ELEMENTS unless the name says bytes), a dtype tag, an optional device error
 * word and a cudaStream_t passed as void*.  No entry point allocates device
 * memory: split-K scratch is owned by the caller and sized by
 * slmt_decode_workspace_bytes().  No entry point synchronises the host.
 * Every entry point returns SLMT_OK (0) or a negative SLMT_ERR_* status.
 * Argument checks happen before anything touches the GPU, so invalid calls
 * never launch a kernel.
 *
 * Each function names the reference interface it replaces.  "ref:" paths are
 * files of the slm-turbo project (kernels/kv_dequant.py is its Python API,
 * kernels/kv_dequant_cuda.cu its torch launchers, kernels/kv_dequant_kernels.cuh
 * its device kernels).
 *
 * Packed formats (kept bit-for-bit from the reference):
 *   paged per-token cache  uint8 [num_blocks, block_size, num_kv_heads, D+8];
 *                          slot = [K codes D/2][V codes D/2][k_min][k_step]
 *                          [v_min][v_step] (fp16 rulers), value = code*step+min,
 *                          dim 2j in the low nibble of byte j, 2j+1 in the high
 *                          nibble  (ref: kernels/kv_dequant_kernels.cuh:511-517).
 *   per-channel codes      uint8 [..., KV, S, D/2], same nibble order, fp16
 *                          scale/zero per (kv head, dim), value = (code-zero)*scale
 *                          (ref: kernels/benchmark/benchmark.py:26-66).
 */
#ifndef SLM_TURBO_B200_H
#define SLM_TURBO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- dtype tags ---------------------------------------------------------- */
#define SLMT_DTYPE_F16 0
#define SLMT_DTYPE_BF16 1
#define SLMT_DTYPE_F32 2
#define SLMT_DTYPE_I32 3
#define SLMT_DTYPE_I64 4

/* ---- status codes (return values) ---------------------------------------- */
#define SLMT_OK 0
#define SLMT_ERR_NULL (-1)        /* a required pointer is NULL               */
#define SLMT_ERR_HEAD_DIM (-2)    /* head_dim not in {64, 80, 128}            */
#define SLMT_ERR_SHAPE (-3)       /* inconsistent sizes (H % KV, slot != D+8) */
#define SLMT_ERR_DTYPE (-4)       /* dtype tag not accepted by this entry     */
#define SLMT_ERR_ALIGN (-5)       /* pointer/stride alignment not met         */
#define SLMT_ERR_WORKSPACE (-6)   /* workspace NULL or smaller than required  */
#define SLMT_ERR_UNSUPPORTED (-7) /* valid but unsupported (e.g. H/KV > 16)   */
#define SLMT_ERR_CUDA (-8)        /* CUDA runtime error at launch             */
#define SLMT_ERR_BLOCK (-9)       /* BLOCK_N / BLOCK_M value rejected         */
#define SLMT_ERR_SCRATCH_LIMIT (-10) /* request needs more than the static    */
                                    /* scratch of slmt_paged_decode_noalloc  */

/* ---- device error word bits (OR-ed into *err_flag by the kernels) -------- */
#define SLMT_DEVERR_BLOCK_ID 1u /* block-table entry outside [0, num_blocks)    */
#define SLMT_DEVERR_SLOT 2u     /* slot_mapping entry beyond the cache          */
#define SLMT_DEVERR_TIMEOUT 4u  /* a pipeline wait exceeded its time limit      */
#define SLMT_DEVERR_SEQ_LEN 8u  /* sequence length above the table capacity     */
#define SLMT_DEVERR_PLACEMENT 16u /* a decode grid that should hold two CTAs per SM
                                     did not (its SM-aware chunk ranges are incomplete) */

/* Library version (major*10000 + minor*100 + patch). */
int slmt_version(void);

/* Human-readable text for a status code (static storage). */
const char* slmt_status_string(int status);

/* Number of SMs of `device` (or a negative status). */
int slmt_device_sm_count(int device);

/*
 * Bound of every wait inside the decode kernels (pipeline barriers, the
 * split-K merge's wait for the other CTAs of a segment), in nanoseconds, for
 * launches issued after the call; ns <= 0 restores the default of 4 s.  A
 * wait that runs out sets SLMT_DEVERR_TIMEOUT in *err_flag and the kernel
 * returns (after its in-flight copies landed) instead of hanging; its
 * outputs are then undefined and the workspace must be zeroed again.
 * Process-wide; returns the previous value.  No counterpart in the reference
 * (its kernels have no waits).
 */
int64_t slmt_set_wait_limit_ns(int64_t ns);

/*
 * Test hook for failure detection, off by default: while on, the consumer
 * warps of CTA 0 of every decode launch wait on a barrier that nothing
 * completes, so that wait runs out after the wait limit above and the launch
 * reports SLMT_DEVERR_TIMEOUT without faulting or hanging.  Process-wide;
 * returns the previous setting.  No counterpart in the reference.
 */
int slmt_set_debug_stall(int on);

/*
 * Bytes of split-K scratch the decode entry points need for `num_seqs`
 * sequences (pseudo-sequences for prefill) on `device`; negative on error.
 * The first workspace_bytes/64 bytes (rounded up to 256) of the scratch hold
 * per-segment arrival counters: they must be zero before the first use, and
 * every completed call leaves them at zero again, so one scratch serves calls
 * of any batch size it is large enough for (pass the same workspace_bytes
 * each time).  It must be 256-byte aligned and must not be shared by calls
 * that overlap on the GPU.  If a call reports a device error, zero it again.
 */
int64_t slmt_decode_workspace_bytes(int64_t num_seqs, int64_t num_q_heads,
                                    int64_t num_kv_heads, int64_t head_dim,
                                    int device);

/*
 * Quantize-on-write into the paged per-token cache.
 * key/value: [num_tokens, num_kv_heads, head_dim] fp16 or bf16, head rows
 * contiguous, token stride `kv_token_stride` elements.  slot_mapping: int64
 * [num_tokens], flat slot = block*block_size + pos; negative slots are skipped.
 * Per (token, kv head): fp32 min/max, step=(max-min)/15 (1 if not >0),
 * code=(int)((x-min)/step+0.5f) clamped to [0,15], fp16 rulers (round to
 * nearest).  Codes and rulers are bit-exact to the reference kernel.
 * ref: kv_quantize_store_cuda, kernels/kv_dequant_cuda.cu:415-456
 *      (kernel kernels/kv_dequant_kernels.cuh:816-919;
 *       Python kv_quantize_store, kernels/kv_dequant.py:220-233).
 */
int slmt_kv_quantize_store(const void* key, const void* value, int kv_dtype,
                           int64_t kv_token_stride, int64_t num_tokens,
                           int64_t num_kv_heads, int64_t head_dim,
                           uint8_t* kv_cache, int64_t num_blocks,
                           int64_t block_size, const int64_t* slot_mapping,
                           int32_t* err_flag, void* stream);

/*
 * Batched ragged decode attention over the paged per-token cache.
 * q: [num_seqs, num_q_heads, head_dim] (fp16/bf16) with strides in elements.
 * block_tables: int32 or int64 [num_seqs, >= max_blocks_per_seq] (row stride
 * bt_seq_stride).  Lengths come from seq_lens (int32 device array) or, when
 * seq_lens is NULL, from seq_len_scalar for every sequence.  Query head h
 * reads kv head h / (num_q_heads / num_kv_heads).  Softmax scale sm_scale
 * (the reference always uses 1/sqrt(head_dim)).  out: [num_seqs, num_q_heads,
 * head_dim] in out_dtype (f32/f16/bf16) with strides in elements.  A sequence
 * of length 0 produces zeros.  max_seq_len_hint (0 = unknown) only sizes the
 * persistent grid.
 * ref: kv_dequant_decode_per_token_paged_attention_cuda,
 *      kernels/kv_dequant_cuda.cu:355-410 (kernel .cuh:671-801; Python
 *      kernels/kv_dequant.py:236-257; caller adapters/vllm_adapter.py:246-284).
 *      The reference decodes one request per call; this call decodes a batch.
 */
int slmt_paged_decode(const void* q, int q_dtype, int64_t q_seq_stride,
                      int64_t q_head_stride, const uint8_t* kv_cache,
                      int64_t num_blocks, int64_t block_size,
                      int64_t num_kv_heads, int64_t head_dim,
                      const void* block_tables, int bt_dtype,
                      int64_t bt_seq_stride, int64_t max_blocks_per_seq,
                      const int32_t* seq_lens, int64_t seq_len_scalar,
                      int64_t max_seq_len_hint, int64_t num_seqs,
                      int64_t num_q_heads, float sm_scale, void* out,
                      int out_dtype, int64_t out_seq_stride,
                      int64_t out_head_stride, void* workspace,
                      int64_t workspace_bytes, int32_t* err_flag,
                      void* stream);

/*
 * One decode step of a ragged batch in ONE launch: each sequence's new token
 * is quantized into the paged cache and then every sequence is decoded over
 * its whole context, the new token included.  new_key/new_value: [num_seqs,
 * num_kv_heads, head_dim] fp16 or bf16 (kv_dtype), head rows contiguous,
 * sequence stride new_seq_stride elements.  seq_lens (required) are the
 * lengths AFTER the append: the new token of sequence b goes to position
 * seq_lens[b]-1, i.e. slot block_tables[b][(len-1)/block_size]*block_size +
 * (len-1)%block_size, the slot vLLM's slot_mapping names for a decode token.
 * A sequence of length 0 appends nothing and produces zeros.  The slot's
 * bytes are those slmt_kv_quantize_store writes for the same row, and the
 * outputs are those of slmt_kv_quantize_store followed by slmt_paged_decode.
 * The warp that decodes a sequence's final chunk quantizes its kv head's new
 * row, so no separate store launch and no re-read of the new slot from HBM.
 * Every other argument as slmt_paged_decode.
 * ref: the decode step of adapters/vllm_adapter.py (do_kv_cache_update
 *      :185-203 then _decode_attention :246-284), i.e. kv_quantize_store_cuda
 *      (kernels/kv_dequant_cuda.cu:415-456) followed by one
 *      kv_dequant_decode_per_token_paged_attention_cuda (.cu:355-410) per
 *      request.
 */
int slmt_paged_append_decode(const void* q, int q_dtype, int64_t q_seq_stride,
                             int64_t q_head_stride, const void* new_key,
                             const void* new_value, int kv_dtype,
                             int64_t new_seq_stride, uint8_t* kv_cache,
                             int64_t num_blocks, int64_t block_size,
                             int64_t num_kv_heads, int64_t head_dim,
                             const void* block_tables, int bt_dtype,
                             int64_t bt_seq_stride, int64_t max_blocks_per_seq,
                             const int32_t* seq_lens, int64_t max_seq_len_hint,
                             int64_t num_seqs, int64_t num_q_heads, float sm_scale,
                             void* out, int out_dtype, int64_t out_seq_stride,
                             int64_t out_head_stride, void* workspace,
                             int64_t workspace_bytes, int32_t* err_flag,
                             void* stream);

/*
 * Batched decode attention over the standalone per-channel layout.
 * k_packed/v_packed: uint8 [num_seqs, num_kv_heads, s_cap, head_dim/2]; the
 * per-sequence stride is kv_seq_stride_rows rows of head_dim/2 bytes (use
 * num_kv_heads*s_cap for a dense batch, 0 to share one K/V among sequences).
 * k_scale/k_zero/v_scale/v_zero: fp16 [num_seqs, num_kv_heads, head_dim] with
 * per-sequence stride ruler_seq_stride elements (0 = shared).  use_quant=0
 * reads raw nibbles (ref `use_quant=False`).  causal_rows!=0 gives sequence b
 * the length min(seq_len_scalar, b+1) (causal prefill rows).
 * ref: kv_dequant_decode_attention_cuda, kernels/kv_dequant_cuda.cu:83-177
 *      (kernel .cuh:113-275; Python kernels/kv_dequant.py:92-123).
 */
int slmt_per_channel_decode(
    const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
    const uint8_t* k_packed, const uint8_t* v_packed,
    int64_t kv_seq_stride_rows, int64_t s_cap, const uint16_t* k_scale,
    const uint16_t* k_zero, const uint16_t* v_scale, const uint16_t* v_zero,
    int64_t ruler_seq_stride, int use_quant, const int32_t* seq_lens,
    int64_t seq_len_scalar, int causal_rows, int64_t num_seqs,
    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
    float sm_scale, void* out, int out_dtype, int64_t out_seq_stride,
    int64_t out_head_stride, void* workspace, int64_t workspace_bytes,
    int32_t* err_flag, void* stream);

/*
 * Batched decode attention over contiguous per-token codes with separate
 * rulers: k/v codes uint8 [num_seqs, KV, s_cap, D/2]; k_min/k_step/v_min/
 * v_step fp16 [num_seqs, KV, s_cap] (per-sequence stride kv_seq_stride_rows
 * rows / elements respectively).
 * ref: kv_dequant_decode_per_token_attention_cuda,
 *      kernels/kv_dequant_cuda.cu:277-350 (kernel .cuh:528-655; Python
 *      kernels/kv_dequant.py:189-217).
 */
int slmt_per_token_decode(
    const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
    const uint8_t* k_packed, const uint8_t* v_packed,
    int64_t kv_seq_stride_rows, int64_t s_cap, const uint16_t* k_min,
    const uint16_t* k_step, const uint16_t* v_min, const uint16_t* v_step,
    const int32_t* seq_lens, int64_t seq_len_scalar, int64_t num_seqs,
    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
    float sm_scale, void* out, int out_dtype, int64_t out_seq_stride,
    int64_t out_head_stride, void* workspace, int64_t workspace_bytes,
    int32_t* err_flag, void* stream);

/*
 * Per-channel prefill attention: q [num_q_heads, M, head_dim] against one
 * per-channel K/V of S tokens ([KV, S, D/2] codes, [KV, D] rulers).  causal!=0
 * lets query row m see keys 0..m (ref mask `m_idx >= n_abs`).  out
 * [num_q_heads, M, head_dim] in out_dtype.  M-tiled kernel (64 query rows
 * per CTA over 64-token K/V chunks dequantized once in shared memory);
 * workspace and err_flag are accepted and unused (may be NULL).  Codes must
 * be 8-byte aligned.  With seq_len 0 every row is zero and codes/rulers may
 * be NULL.
 * ref: kv_dequant_prefill_attention_cuda, kernels/kv_dequant_cuda.cu:182-272
 *      (kernel .cuh:293-502; Python kernels/kv_dequant.py:129-177).
 */
int slmt_per_channel_prefill(
    const void* q, int q_dtype, int64_t q_head_stride, int64_t q_row_stride,
    const uint8_t* k_packed, const uint8_t* v_packed, int64_t seq_len,
    const uint16_t* k_scale, const uint16_t* k_zero, const uint16_t* v_scale,
    const uint16_t* v_zero, int use_quant, int causal, int64_t num_rows,
    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
    float sm_scale, void* out, int out_dtype, int64_t out_head_stride,
    int64_t out_row_stride, void* workspace, int64_t workspace_bytes,
    int32_t* err_flag, void* stream);

/*
 * Prefill attention of query chunks over the paged per-token cache (the
 * layout of slmt_paged_decode).  Request r (r < num_reqs) owns query rows
 * [query_start_loc[r], query_start_loc[r+1]) of q (row m, head h at
 * q + m*q_row_stride + h*q_head_stride); those n rows are the LAST n of its
 * seq_lens[r] cached tokens (the step's new tokens already stored), so row i
 * attends causally to keys [0, seq_lens[r] - n + i + 1) read through
 * block_tables.  A request with seq_lens[r] <= 0 is skipped (its rows of out
 * are left as they are; a caller attends those rows some other way).
 * max_query_len bounds n of the other requests: the launch covers 64-row
 * tiles up to max_query_len, and a request with rows beyond them sets
 * SLMT_DEVERR_SEQ_LEN and those rows are not written.  out like q, in
 * out_dtype.  Bad block-table entries set SLMT_DEVERR_BLOCK_ID (the token
 * reads as zero), lengths above max_blocks_per_seq*block_size set
 * SLMT_DEVERR_SEQ_LEN (clamped).  No workspace, no host sync.  kv_cache must
 * be 8-byte aligned; num_reqs and num_q_heads at most 65535.
 * Replaces the reference adapter's prefill branch, which runs SDPA over the
 * step's raw K/V only (adapters/vllm_adapter.py:218-243), for chunks with a
 * cached prefix; same M-tiled kernel as slmt_per_channel_prefill
 * (ref kernel .cuh:293-502).
 */
int slmt_paged_prefill(
    const void* q, int q_dtype, int64_t q_row_stride, int64_t q_head_stride,
    const uint8_t* kv_cache, int64_t num_blocks, int64_t block_size,
    int64_t num_kv_heads, int64_t head_dim, const void* block_tables,
    int bt_dtype, int64_t bt_seq_stride, int64_t max_blocks_per_seq,
    const int32_t* query_start_loc, const int32_t* seq_lens, int64_t num_reqs,
    int64_t max_query_len, int64_t num_q_heads, float sm_scale, void* out,
    int out_dtype, int64_t out_row_stride, int64_t out_head_stride,
    int32_t* err_flag, void* stream);

/*
 * Per-channel rulers + codes of whole sequences, on the device:
 * x fp16 [num_seqs, KV, S, D] contiguous -> packed uint8 [num_seqs, KV, S, D/2],
 * scale/zero fp16 [num_seqs, KV, D].  Same fp16 arithmetic as the reference's
 * compute_scale_zero/quantize_tensor, codes and rulers bit-exact.
 * ref: kernels/benchmark/benchmark.py:26-56 (quantize_kv :69-74).
 */
int slmt_per_channel_quantize(const void* x, int x_dtype, int64_t num_seqs,
                              int64_t num_kv_heads, int64_t seq_len,
                              int64_t head_dim, uint8_t* packed,
                              uint16_t* scale, uint16_t* zero, void* stream);

/*
 * Append new tokens to a per-channel buffer with frozen rulers:
 * x fp16 [KV, N, D] (token stride x_token_stride, head stride x_head_stride
 * elements) -> packed rows [pos, pos+N) of uint8 [KV, s_cap, D/2];
 * code = clamp(round_half_even(fp16(x/scale)) + zero, 0, 15).
 * ref: incremental append, kernels/benchmark/benchmark.py:201-221
 *      (quantize_tensor :45-56).
 */
int slmt_per_channel_append(const void* x, int x_dtype, int64_t x_head_stride,
                            int64_t x_token_stride, int64_t num_new,
                            int64_t num_kv_heads, int64_t head_dim,
                            const uint16_t* scale, const uint16_t* zero,
                            uint8_t* packed, int64_t s_cap, int64_t pos,
                            void* stream);

/*
 * slmt_paged_decode with no workspace argument: its split-K scratch is a
 * static device array of SLMT_NOALLOC_SCRATCH_BYTES inside this library, so
 * the call allocates no device memory (no cudaMalloc/cudaFree, no allocating
 * library routine).  It is for callers that cannot allocate when they decode
 * -- an engine that gave all of HBM to its page pool and activation arena up
 * front, or a plugin host that offers the op no allocator -- and so cannot
 * pass slmt_paged_decode a workspace.  No counterpart in the reference (its
 * single-request decode needs no scratch).  Every other argument, the
 * results and the statuses are those of slmt_paged_decode.
 * Limit: a request whose worst-case scratch (slmt_decode_workspace_bytes of
 * num_seqs, num_q_heads, num_kv_heads, head_dim) exceeds the array returns
 * SLMT_ERR_SCRATCH_LIMIT before anything is launched; 8 MiB covers e.g. 64
 * sequences at 32 query heads x 128 dims on a 148-SM device.
 * Zero state: the array starts zero-filled when the module loads.  Its first
 * 1/64 holds arrival counters that must be zero when a launch starts; each
 * launch that completes without a device error bit leaves them at zero.
 * After a call that set a bit in *err_flag, pass reset_scratch != 0 on the
 * next call: that zeroes the counters with cudaMemsetAsync on `stream`
 * before the launch (0 skips it).
 * Set-up: the first call on each device (with that device current) looks up
 * the array's address with cudaGetSymbolAddress, which may load the module,
 * and the first decode call configures the kernel; make that first call
 * before any stream capture begins.  The address is cached per device for
 * the life of the process, which assumes the device's primary context lives
 * as long (no cudaDeviceReset in between).
 * Concurrency: all calls on one device share the one array, so two calls
 * whose executions overlap (different streams, or different host threads)
 * race on it and give wrong results; order them on one stream or with
 * events.
 */
#define SLMT_NOALLOC_SCRATCH_BYTES (8 * 1024 * 1024)
int slmt_paged_decode_noalloc(const void* q, int q_dtype, int64_t q_seq_stride,
                              int64_t q_head_stride, const uint8_t* kv_cache,
                              int64_t num_blocks, int64_t block_size,
                              int64_t num_kv_heads, int64_t head_dim,
                              const void* block_tables, int bt_dtype,
                              int64_t bt_seq_stride, int64_t max_blocks_per_seq,
                              const int32_t* seq_lens, int64_t seq_len_scalar,
                              int64_t max_seq_len_hint, int64_t num_seqs,
                              int64_t num_q_heads, float sm_scale, void* out,
                              int out_dtype, int64_t out_seq_stride,
                              int64_t out_head_stride, int reset_scratch,
                              int32_t* err_flag, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SLM_TURBO_B200_H */
