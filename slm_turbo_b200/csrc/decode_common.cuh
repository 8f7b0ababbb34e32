// decode_common.cuh -- shared definitions of the split-K decode kernel (its
// in-launch partial merge included) and the host launchers.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace slmt {

// A CTA has one consumer warp per kv head of its group (KVC of them, 1..8)
// and one producer warp.
__host__ __device__ constexpr int cta_threads(int kvc) { return (kvc + 1) * 32; }
// Resident CTAs per SM the kernels are built for: about 18 warps per SM with
// one n-tile (96 registers: a sub-partition holds up to 5 such warps), but 16
// (128 registers) with 1 or 2 kv heads per CTA, whose many small CTAs spill at
// 96; about 9 warps with two n-tiles.
__host__ __device__ constexpr int warps_per_sm_target(int kvc, int nt) {
  return nt == 1 ? (kvc <= 2 ? 16 : 18) : 9;
}
__host__ __device__ constexpr int ctas_per_sm(int kvc, int nt) {
  return warps_per_sm_target(kvc, nt) / (kvc + 1) > 0 ? warps_per_sm_target(kvc, nt) / (kvc + 1) : 1;
}
constexpr int kMaxStages = 8;
constexpr int kMaxEnds = 8;  // segment ends per range whose new token is quantized at the start
constexpr int kTileTokens = 16;   // one m16 tensor-core tile of tokens
constexpr int kChunkTokens = 32;  // one pipeline stage = two tiles
constexpr uint64_t kDefaultWaitLimitNs = 4000000000ull;  // 4 s per wait (host-settable)
constexpr uint64_t kDrainLimitNs = 200000000ull;  // 0.2 s per drain wait
constexpr float kRescaleSlack = 4.0f;  // lazy softmax rescale threshold (log2 units)
constexpr float kMaxFloor = -1e30f;    // running max before any score (finite on purpose)

enum Layout : int {
  LAYOUT_PAGED = 0,        // [num_blocks, block_size, KV, D+8] per-token slots
  LAYOUT_PER_CHANNEL = 1,  // [B, KV, S, D/2] codes + [B, KV, D] scale/zero
  LAYOUT_PER_TOKEN = 2,    // [B, KV, S, D/2] codes + [B, KV, S] min/step
};

// One descriptor per pipeline stage, written by the producer warp.
struct ChunkDesc {
  int seq;        // sequence index, -1 = no more work
  int kg;         // kv-head group
  int chunk;      // 32-token chunk index inside the sequence
  int nvalid;     // valid tokens in this chunk (1..32)
  int flags;      // bit0 first chunk of segment, bit1 last, bits2.. q buffer
  int slot;       // partial slot (cta + segment)
  int ncov;       // CTAs whose chunk ranges cover this segment
  int c_first;    // first of them
  int nmergers;   // how many of them end their range inside it (they merge it)
  int len;        // the sequence's length
  int pad[2];
};

// Descriptor flag bits.
constexpr int kFlagFirst = 1;     // first chunk of the segment in this CTA
constexpr int kFlagLast = 2;      // last chunk of the segment in this CTA
constexpr int kFlagQbuf = 4;      // q buffer index (0/1)
constexpr int kFlagRangeEnd = 8;  // last chunk of this CTA's range
constexpr int kFlagPatch = 16;  // fused append: the range's first segment end, whose new slot
                                // the consumers quantized at the start (hdr->newslot)

// The split segment this CTA helps merge after its main loop: the segment
// its range ends in.  Every CTA whose range ends inside a split segment
// merges a slice of its (head, dim-quad) items once all covering CTAs have
// published their partials.
struct MergeJob {
  int e_seg, seq, kg, c_first, ncov, nmergers;
};

struct SmemHeader {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t qfull[2];
  uint64_t qempty[2];
  uint64_t never;  // a barrier nothing arrives on (the stalled-consumer test hook)
  // fused append: the new token's slot of the range's first segment per
  // consumer warp (kv head), quantized when the launch starts and copied over
  // the stale staged row when the segment's final chunk arrives
  uint8_t newslot[8][136];
  // fused append: the producer publishes the segments whose final chunk lies
  // in this CTA's range (up to kMaxEnds, in range order); the consumer warps
  // quantize their new tokens when the launch starts and arrive on `appended`
  uint64_t prologue;
  uint64_t appended;
  int n_end;
  int end_seq[kMaxEnds], end_kg[kMaxEnds], end_len[kMaxEnds];
  ChunkDesc desc[kMaxStages];
  int has_job;
  int merge_ok;
  int spiece;  // SM-aware piece 2*sm + arrival (-1: none), set at the launch start
  int pidx;    // this CTA's piece of the partition (set by the producer)
  int abort;  // a consumer warp gave up on a wait: the others skip the merge
  MergeJob job;
};

// Per-segment word in the scratch's counter region: low 16 bits count the
// consumer warps that published their slice of a partial (KVC per covering
// CTA), high 16 bits the mergers that are done; the last merger resets the
// word to zero.
constexpr uint32_t kArriveOne = 1u, kDoneOne = 1u << 16;

constexpr int kHeaderBytes = (int)((sizeof(SmemHeader) + 127) / 128 * 128);

struct DecodeParams {
  // queries: element (seq, head, d) at q + seq*q_seq_stride + head*q_head_stride + d
  const void* q;
  int64_t q_seq_stride, q_head_stride;
  int q_bf16, q_bulk;  // q_bulk: a group's q rows are one 16-byte aligned span
  // paged cache
  const uint8_t* cache;
  int64_t num_blocks;
  int block_size, kv_total;
  const void* block_tables;
  int bt_i64;
  int64_t bt_seq_stride;
  int max_blocks;
  int paged_mode;  // 0: one bulk copy per 16-token tile, 1: bulk copy per row, 2: cp.async rows,
                   // 3: one 2-D tiled copy per 16-token tile of the group's heads (tmap_k),
                   // 4: one 3-D tiled copy per 16-token tile of whole rows, 64-byte swizzled
                   //    (tmap_k; the SWZ consumer reads through the swizzle)
  // contiguous layouts
  const uint8_t* k_codes;
  const uint8_t* v_codes;
  int64_t kv_seq_stride_rows, s_cap;
  const uint16_t* r0;  // per-channel k_scale | per-token k_min
  const uint16_t* r1;  // per-channel k_zero  | per-token k_step
  const uint16_t* r2;  // per-channel v_scale | per-token v_min
  const uint16_t* r3;  // per-channel v_zero  | per-token v_step
  int64_t ruler_seq_stride;
  int use_quant, contig_bulk_ok;
  int rul_bulk;  // per-channel rulers of a kv group: four 16-byte aligned spans
  // contiguous layouts: K and V codes [B, KV, S*D/2 bytes] as 3-D tensor
  // maps of 8-byte elements with a box of one chunk of a kv group, so a
  // chunk's K (or V) rows of every kv head of the group arrive with one
  // tiled TMA copy; used when tma_tensor is set.  Paged layout, mode 3:
  // tmap_k views the pool as [num_blocks*block_size token rows][kv_total*
  // (D+8) bytes as 8-byte elements] with a box of 16 rows x the group's heads
  int tma_tensor;
  CUtensorMap tmap_k, tmap_v;
  // lengths
  const int32_t* seq_lens;
  int seq_len_scalar, causal_rows, len_cap;
  // shape
  int num_seqs, hq, G, kvc, ngroups;
  float scale_log2;
  // pipeline geometry
  int stages, stage_bytes, qbuf_bytes, rbuf_bytes, nqbuf, stage_offset, num_ctas;
  // split-K scratch
  float* part_ml;      // [slots][kvc*G][2] (running max in log2 units, sum)
  float* part_acc;     // [slots][kvc*G][D]  (unnormalised output)
  int32_t* seg_count;  // [ngroups*B] arrivals per segment; zero between launches
  // SM-aware partition (full grids of two CTAs per SM, 8 kv heads per CTA,
  // one n-tile): the CTA that arrives second on its SM is the slower one
  // (its warps lose issue slots to the older CTA's), so chunk ranges are
  // given per (SM, arrival) with weights part_w0 : part_w1.  sm_ctr: one
  // arrival word per SM + a CTAs-done word; zero between launches.
  int sm_weighted, num_sms, part_w0, part_w1;
  int seg_cost;  // weighted partition: a segment start costs seg_cost/8 chunks
  int32_t* sm_ctr;
  int32_t* err;
  // fused append (paged layout): one new token per sequence at position
  // len-1, row (seq, kv head) at new_k/new_v + seq*new_seq_stride + head*D,
  // quantized into the cache by the warp that consumes the segment's final chunk
  int append, new_bf16;
  const void* new_k;
  const void* new_v;
  int64_t new_seq_stride;
  uint64_t wait_limit_ns;  // bound of every pipeline / merge wait
  int debug_stall;         // test hook: CTA 0's consumers wait on a flag nothing sets
  // output element (seq, head, d) at out + seq*out_seq_stride + head*out_head_stride + d
  void* out;
  int out_dtype;  // 0 f16, 1 bf16, 2 f32
  int out_pair;   // base and strides let adjacent (even, odd) dims be stored as one pair
  int64_t out_seq_stride, out_head_stride;
};

// Host-side handle of one decode kernel instantiation.
using DecodeFn = void (*)(const DecodeParams);

// Per head dim: the kernel for n-tiles nt, tile packing pk, kv heads per CTA
// kvc, and (paged) whether the launch appends or (contiguous) the layout.
// Defined in decode_d64.cu, decode_d80.cu, decode_d128.cu.
DecodeFn decode_fn_64_paged(int nt, bool pk, int kvc, bool append, bool swz);
DecodeFn decode_fn_80_paged(int nt, bool pk, int kvc, bool append, bool swz);
DecodeFn decode_fn_128_paged(int nt, bool pk, int kvc, bool append, bool swz);
DecodeFn decode_fn_64_contig(int nt, bool pk, int layout, int kvc);
DecodeFn decode_fn_80_contig(int nt, bool pk, int layout, int kvc);
DecodeFn decode_fn_128_contig(int nt, bool pk, int layout, int kvc);

__host__ __device__ inline int nchunks_of(int len) {
  return (len + kChunkTokens - 1) / kChunkTokens;
}

// Largest c with floor(c*T/NC) <= t: the persistent CTA that owns chunk t.
__host__ __device__ inline int64_t cta_of_unit(int64_t t, int64_t T, int64_t NC) {
  return ((t + 1) * NC + T - 1) / T - 1;
}

__host__ __device__ inline int64_t cta_start(int64_t c, int64_t T, int64_t NC) {
  return c * T / NC;
}

// The chunk partition of one launch: NC pieces over T chunks, uniform
// (piece c = CTA c) or weighted by SM arrival (piece 2*sm + arrival, weights
// w0 for the first CTA on an SM and w1 for the second).
struct Partition {
  int64_t T, NC;
  int weighted, w0, w1;
  __host__ __device__ int64_t start(int64_t c) const {
    if (!weighted) return cta_start(c, T, NC);
    const int64_t W = (NC / 2) * (w0 + w1);
    const int64_t cw = (c >> 1) * (w0 + w1) + ((c & 1) ? w0 : 0);
    return cw * T / W;
  }
  // the piece that owns chunk t (largest c with start(c) <= t)
  __host__ __device__ int64_t owner(int64_t t) const {
    if (!weighted) return cta_of_unit(t, T, NC);
    const int64_t W = (NC / 2) * (w0 + w1);
    const int64_t K = ((t + 1) * W + T - 1) / T - 1;  // largest cw with cw*T/W <= t
    int64_t c = 2 * (K / (w0 + w1)) + ((K % (w0 + w1)) >= w0 ? 1 : 0);
    return c < NC - 1 ? c : NC - 1;
  }
};

}  // namespace slmt
