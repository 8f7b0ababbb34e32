// decode_kernels.cuh -- split-K 4-bit decode attention for sm_100a.
//
// One persistent CTA per (SM x resident CTAs).  The work space is the list of
// 32-token chunks of every (kv-head group, sequence) segment, concatenated;
// CTA c owns the contiguous chunk range [c*T/NC, (c+1)*T/NC), so every CTA
// streams the same number of bytes whatever the length mix of the batch.
//
// Warp roles ((KVC + 1) x 32 threads, KVC = kv heads per group):
//   warp KVC    producer: walks its chunk range and stages each chunk with
//               1-D bulk copies (TMA unit; one per 16-token page tile, or per
//               row / cp.async when the layout is not 16-byte aligned) into a
//               STAGES-deep shared-memory ring guarded by mbarriers; stages
//               q (+ per-channel rulers) once per segment.
//   warps 0..KVC-1  consumers: warp w owns kv head w of the group.  Per
//               32-token chunk (two m16 tiles, independent tensor-core chains):
//                 S^T[16 tok x 8 heads] = codes(K) . q            (m16n8k16, fp32)
//                 s = k_step*S + k_min*sum(q)                      (per-token rulers)
//                 online softmax, log2 domain, lazy rescale (quad shuffles)
//                 P' = p*v_step -> fp16 -> movmatrix -> B operand
//                 O^T[D x 8 heads] += codes(V)^T . P'^T            (m16n8k16)
//                 sum_v += p*v_min
//               4-bit codes go straight from shared memory to biased fp16
//               operands in registers (1024+c, 64+c; the bias is taken off
//               per dot product); no dequantised K/V exists anywhere.
//   At a segment end: a segment that one CTA streamed alone is normalised and
//   written straight to the output; otherwise each consumer warp writes
//   (m, l, acc) to the split-K scratch slot cta+segment and the CTA counts
//   itself in the segment's arrival word.  After their ranges, the CTAs whose
//   ranges end inside the segment wait for every covering CTA to publish and
//   each merges a slice of its output rows (log-sum-exp weights); the last
//   of them resets the word -- no separate combine launch.
#pragma once

#include "decode_common.cuh"
#include "ptx.cuh"
#include "quant_store.cuh"

namespace slmt {

// ------------------------------------------------------------------ helpers --
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int warp_incl_scan(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

__device__ __forceinline__ long long warp_incl_scan_ll(long long v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    long long t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// Cost positions of the weighted partition: a non-empty segment costs SC
// units for its start and U8 per chunk; chunk t of the segment with ordinal e
// (among non-empty segments, in (group, sequence) order) sits at its last
// unit, SC*(e+1) + U8*(t+1) - 1.  SC = 0, U8 = 1 is the plain chunk index.
__device__ __forceinline__ long long cost_pos(long long t, long long e, int SC, int U8) {
  return (long long)SC * (e + 1) + (long long)U8 * (t + 1) - 1;
}

// Wait until the low 16 bits of `word` (published by other CTAs with a
// fence before their atomic add) reach n; false after limit_ns.
__device__ __forceinline__ bool spin_until_arrived(const unsigned int* word, unsigned int n,
                                                   uint64_t limit_ns) {
  auto arrived = [&]() {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(word) : "memory");
    return (v & 0xFFFFu) >= n;
  };
  if (arrived()) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i) {
      __nanosleep(100);
      if (arrived()) return true;
    }
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}

__device__ __forceinline__ void set_err(const DecodeParams& p, uint32_t bit) {
  if (p.err) atomicOr(reinterpret_cast<unsigned int*>(p.err), bit);
}

// Length of sequence b after clamping to what the layout can hold.
__device__ __forceinline__ int seq_len_of(const DecodeParams& p, int b) {
  int L;
  if (p.causal_rows)
    L = min(p.seq_len_scalar, b + 1);
  else if (p.seq_lens)
    L = p.seq_lens[b];
  else
    L = p.seq_len_scalar;
  L = max(L, 0);
  return min(L, p.len_cap);
}

// Raw (unclamped) length, used once by the producer to flag overflow.
__device__ __forceinline__ int seq_len_raw(const DecodeParams& p, int b) {
  if (p.causal_rows) return min(p.seq_len_scalar, b + 1);
  if (p.seq_lens) return p.seq_lens[b];
  return p.seq_len_scalar;
}

// First chunk (global index) whose cost position is >= x (the total chunk
// count if none): the start of the piece whose cost range begins at x.
__device__ inline long long chunk_at_cost(const DecodeParams& p, long long x, long long t_seq, int e_seq, int SC, int U8) {
  const int lane = threadIdx.x & 31;
  const int B = p.num_seqs;
  const long long Gc = (long long)SC * e_seq + (long long)U8 * t_seq;  // cost of one kv-head group
  if (Gc <= 0 || x >= Gc * p.ngroups) return t_seq * p.ngroups;
  const long long kg = x / Gc;
  const long long xr = x - kg * Gc;
  long long cb = 0, ps = 0;  // cost and chunks of the group's sequences before `base`
  for (int base = 0; base < B; base += 32) {
    const int b = base + lane;
    const int n = (b < B) ? nchunks_of(seq_len_of(p, b)) : 0;
    const long long cst = n > 0 ? (long long)SC + (long long)U8 * n : 0;
    const long long ci = warp_incl_scan_ll(cst);
    const int ni = warp_incl_scan(n);
    const long long ctot = __shfl_sync(0xffffffffu, ci, 31);
    const int ntot = __shfl_sync(0xffffffffu, ni, 31);
    if (cb + ctot > xr) {
      const unsigned m = __ballot_sync(0xffffffffu, cb + ci > xr);
      const int src = __ffs(m) - 1;
      const long long cbefore = cb + __shfl_sync(0xffffffffu, ci - cst, src);
      const long long nbefore = ps + __shfl_sync(0xffffffffu, ni - n, src);
      const int nb = __shfl_sync(0xffffffffu, n, src);
      // first chunk j of that sequence with cbefore + SC + U8*(j+1) - 1 >= xr
      long long j = xr - cbefore - SC + 1 - U8;
      j = j <= 0 ? 0 : (j + U8 - 1) / U8;
      if (j > nb) j = nb;
      return kg * t_seq + nbefore + j;
    }
    cb += ctot;
    ps += ntot;
  }
  return (kg + 1) * t_seq;
}


__device__ __forceinline__ int64_t block_entry(const DecodeParams& p, int s, int blk) {
  if (p.bt_i64)
    return reinterpret_cast<const int64_t*>(p.block_tables)[(int64_t)s * p.bt_seq_stride + blk];
  return reinterpret_cast<const int32_t*>(p.block_tables)[(int64_t)s * p.bt_seq_stride + blk];
}

// Load N bytes starting at shared-memory `ptr` into 32-bit words (little
// endian, zero padded).  ALIGN is the guaranteed alignment of ptr.
template <int N, int ALIGN>
__device__ __forceinline__ void load_bytes(const uint8_t* ptr, uint32_t* w) {
  constexpr int NW = (N + 3) / 4;
  if constexpr (N % 8 == 0 && ALIGN >= 8) {
#pragma unroll
    for (int i = 0; i < N / 8; ++i) {
      uint2 v = reinterpret_cast<const uint2*>(ptr)[i];
      w[2 * i] = v.x;
      w[2 * i + 1] = v.y;
    }
  } else if constexpr (N == 4 && ALIGN >= 4) {
    w[0] = *reinterpret_cast<const uint32_t*>(ptr);
  } else if constexpr (N % 2 == 0 && ALIGN >= 2) {
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = 0;
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      uint32_t h = reinterpret_cast<const uint16_t*>(ptr)[i];
      w[i >> 1] |= h << (16 * (i & 1));
    }
  } else {
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = 0;
#pragma unroll
    for (int i = 0; i < N; ++i) w[i >> 2] |= (uint32_t)ptr[i] << (8 * (i & 3));
  }
}

// Physical head dim held by k-slot `slot` (0:2r, 1:2r+1, 2:2r+8, 3:2r+9) of
// QK k-step `s` in thread r.  Thread r reads bytes [r*D/8, (r+1)*D/8) of a K
// row; one 32-bit word feeds two k-steps (low nibbles of bytes 0/2 and 1/3
// pair up in one f16x2), a trailing 2-byte word (D = 80) feeds one.
template <int D>
__device__ __forceinline__ int kword_byte(int r, int u) {
  constexpr int QB = D / 8;
  // D = 128: a lane's 16 bytes are [8r, 8r+8) and [32+8r, 40+8r), so each of
  // its two 8-byte loads covers 32 contiguous bytes across the 4 lanes of a row
  if constexpr (QB == 16) return 32 * (u >> 1) + 8 * r + 4 * (u & 1);
  return r * QB + 4 * u;
}

template <int D>
__device__ __forceinline__ int qk_dim(int s, int slot, int r) {
  constexpr int QB = D / 8;
  const int u = s >> 1, e = s & 1;
  const int base = kword_byte<D>(r, u);
  const int nib = (slot >> 1) & 1;
  int byte;
  if (4 * u + 4 <= QB)
    byte = base + e + ((slot & 1) ? 2 : 0);
  else
    byte = base + (slot & 1);
  return 2 * byte + nib;
}

// Shared-memory addresses of token row t (0..31) of kv head j in a stage.
// `base` already holds the warp's kv-head offset; paged rows are KVC*(D+8)
// bytes apart, contiguous layouts hold D/2-byte K and V rows.
template <int D, int LAYOUT, int KVC>
struct StageView {
  static constexpr int kRow = (LAYOUT == LAYOUT_PAGED) ? KVC * (D + 8) : D / 2;  // row stride
  // byte distance of rows t+8 / t+16 from row t
  static constexpr int d8 = 8 * kRow;
  static constexpr int d16 = 16 * kRow;
  static constexpr int r8 = (LAYOUT == LAYOUT_PAGED) ? d8 : 8 * KVC * 8;
  static constexpr int r16 = (LAYOUT == LAYOUT_PAGED) ? d16 : 16 * KVC * 8;
  const uint8_t* base;  // paged: st + j*(D+8); contiguous: st + j*32*(D/2) (the K block)
  const uint8_t* rul;   // contiguous per-token rulers: st + KVC*32*D + j*8
  __device__ __forceinline__ const uint8_t* k(int t) const {
    if (LAYOUT == LAYOUT_PAGED) return base + t * kRow;
    return base + t * (D / 2);
  }
  __device__ __forceinline__ const uint8_t* v(int t) const {
    if (LAYOUT == LAYOUT_PAGED) return base + t * kRow + D / 2;
    return base + KVC * kChunkTokens * (D / 2) + t * (D / 2);  // the V block follows the K block
  }
  __device__ __forceinline__ const uint8_t* rulers(int t) const {
    if (LAYOUT == LAYOUT_PAGED) return base + t * kRow + D;
    return rul + t * KVC * 8;
  }
};


// Swizzled stages (paged mode 4): the tiled copy stores each 64-byte piece of
// a stage with its 16-byte chunks permuted, chunk ^= bits 7-8 of the offset
// (CU_TENSOR_MAP_SWIZZLE_64B, stage bases 1024-byte aligned).  Byte offset o
// of the unswizzled stage lies at swz64(o); 8-byte reads never straddle a
// chunk.  Row offsets of 8 and 16 tokens are multiples of 512 bytes (a row is
// a multiple of 64), so they commute with the swizzle.
__device__ __forceinline__ uint32_t swz64(uint32_t o) { return o ^ (((o >> 7) & 3u) << 4); }

// With swizzled stages, MMA fragment row k of a 16-token tile holds token
// tok_perm(k) (bits 0 and 1 swapped): the 8 rows one shared load touches
// then spread over all 32 banks.  A permutation of the tokens of a tile
// changes nothing in the result as long as scores, masks, rulers and V rows
// all use it.
__device__ __forceinline__ int tok_perm(int k) { return (k & ~3) | ((k & 1) << 1) | ((k >> 1) & 1); }

// ------------------------------------------------------------------ producer --
// Page ids of 32 consecutive 16-token tiles of sequence s, one per lane.
__device__ __forceinline__ int64_t page_window(const DecodeParams& p, int s, int tile0, int ntile) {
  const int lane = threadIdx.x & 31;
  const int pt = tile0 + lane;
  return (pt < ntile) ? block_entry(p, s, (pt * kTileTokens) / p.block_size) : 0;
}

// Next non-empty segment after (s, kg): one warp-wide load of 32 lengths.
// Returns false when none of the next 32 sequences has tokens (caller loops).
__device__ __forceinline__ bool next_segment(const DecodeParams& p, int s, int kg, int& s2, int& kg2,
                                             int& L2) {
  const int lane = threadIdx.x & 31;
  const int B = p.num_seqs;
  const int raw = s + 1 + lane;
  const int ls = raw % B;
  const int Ll = seq_len_of(p, ls);
  const unsigned m = __ballot_sync(0xffffffffu, Ll > 0);
  if (m == 0) {
    s2 = (s + 32) % B;
    kg2 = kg + (s + 32) / B;
    L2 = 0;
    return false;
  }
  const int src = __ffs(m) - 1;
  const int r2 = s + 1 + src;
  s2 = r2 % B;
  kg2 = kg + r2 / B;
  L2 = __shfl_sync(0xffffffffu, Ll, src);
  return true;
}

// Fused append, done by the producer warp for a segment end beyond the
// kMaxEnds that the consumers quantize at the start (only ranges that hold
// more than kMaxEnds segment ends, i.e. very short sequences, get here):
// quantize the new token (position t) of sequence `seq` for every kv head of
// group kg into its cache slot before the copy of that final chunk is issued.
// One head at a time, to keep the producer's registers free.
template <int D>
__device__ __noinline__ void producer_append(const DecodeParams& p, int seq, int kg, int t) {
  const int lane = threadIdx.x & 31;
  const int64_t ph = block_entry(p, seq, t / p.block_size);
  const bool ok = ph >= 0 && ph < p.num_blocks;
  if (!ok && lane == 0) set_err(p, 1u);
  for (int j = 0; j < p.kvc; ++j) {
    const int h = kg * p.kvc + j;
    const int64_t off = ((int64_t)seq * p.new_seq_stride + (int64_t)h * D) * 2;  // bytes
    const SlotRow r = quantize_slot_row<D>(reinterpret_cast<const uint8_t*>(p.new_k) + off,
                                           reinterpret_cast<const uint8_t*>(p.new_v) + off, p.new_bf16);
    if (ok)
      write_slot_row<D>(const_cast<uint8_t*>(p.cache) +
                            ((ph * p.block_size + t % p.block_size) * p.kv_total + h) * (int64_t)(D + 8),
                        r);
  }
  fence_proxy_async_global();  // the copy about to be issued reads these bytes through the async proxy
  __syncwarp();
}

template <int D, int LAYOUT, bool APPEND>
__device__ void decode_producer(const DecodeParams& p, SmemHeader* hdr,
                                uint8_t* qbuf, uint8_t* rbuf, uint8_t* stg) {
  constexpr int SLOT = D + 8;
  constexpr int HALF = D / 2;
  const int lane = threadIdx.x & 31;
  const int B = p.num_seqs;

  // Chunks (and non-empty sequences) per kv-head group; flag lengths above
  // capacity once per grid.
  long long t_seq = 0;
  int e_seq = 0;
  for (int base = 0; base < B; base += 32) {
    const int b = base + lane;
    int n = 0;
    if (b < B) {
      n = nchunks_of(seq_len_of(p, b));
      if (blockIdx.x == 0 && seq_len_raw(p, b) > p.len_cap) set_err(p, 8u);
    }
    t_seq += warp_sum_i(n);
    e_seq += warp_sum_i(n > 0 ? 1 : 0);
  }
  const long long T = t_seq * p.ngroups;
  // SM-aware weighted pieces when the host enabled them and every piece gets
  // chunks, over cost positions that charge each segment start SC units
  // (8 per chunk); else piece = CTA index over plain chunk indices, never
  // more CTAs than chunks, so every working CTA owns at least one
  const bool use_w = p.sm_weighted && T >= 8LL * p.num_ctas;
  const long long nc_eff = use_w ? p.num_ctas : (T < p.num_ctas ? T : p.num_ctas);
  const int SC = use_w ? p.seg_cost : 0;
  const int U8 = use_w ? 8 : 1;
  const long long Ctot = (long long)SC * e_seq * p.ngroups + (long long)U8 * T;
  // (weights re-read from the kernel parameters at each use: no registers held)
  auto part = [&]() { return Partition{Ctot, nc_eff, use_w ? 1 : 0, p.part_w0, p.part_w1}; };
  int c = (int)blockIdx.x;
  if (use_w) {
    c = hdr->spiece;
    if (c < 0) {  // placement other than two CTAs per SM: this CTA works on nothing
      if (lane == 0) set_err(p, 16u);
      c = (int)nc_eff;
    }
  }
  if (lane == 0) hdr->pidx = c;  // read by the consumers after their main loop
  long long t_begin = 0, t_end = 0;
  if (c < nc_eff) {
    if (use_w) {
      t_begin = chunk_at_cost(p, part().start(c), t_seq, e_seq, SC, U8);
      t_end = chunk_at_cost(p, part().start(c + 1), t_seq, e_seq, SC, U8);
    } else {
      t_begin = part().start(c);
      t_end = part().start(c + 1);
    }
  }

  // sequences without tokens get zeros (no segment ever writes them)
  for (int b = (int)blockIdx.x; b < B; b += gridDim.x) {
    if (seq_len_of(p, b) != 0) continue;
    for (int i = lane; i < p.hq * D; i += 32) {
      const int64_t o = (int64_t)b * p.out_seq_stride + (int64_t)(i / D) * p.out_head_stride + i % D;
      if (p.out_dtype == 2)
        reinterpret_cast<float*>(p.out)[o] = 0.f;
      else
        reinterpret_cast<uint16_t*>(p.out)[o] = 0;
    }
  }

  const uint64_t policy = l2_evict_first_policy();
  uint32_t q_issued[2] = {0u, 0u};  // q (+ ruler) copies issued per q buffer
  uint32_t it = 0;
  int stage = 0;
  uint32_t phase = 0;
  bool failed = false;

  if (t_begin < t_end) {
    int kg = (int)(t_begin / t_seq);
    const long long tt = t_begin - (long long)kg * t_seq;
    // Locate the sequence holding chunk tt of group kg (second pass hits L1),
    // and its ordinal among the non-empty segments.
    int s = 0;
    long long ps = 0;
    long long eord = (long long)kg * e_seq;
    for (int base = 0; base < B; base += 32) {
      const int b = base + lane;
      const int n = (b < B) ? nchunks_of(seq_len_of(p, b)) : 0;
      const int incl = warp_incl_scan(n);
      const int eincl = warp_incl_scan(n > 0 ? 1 : 0);
      const int tot = __shfl_sync(0xffffffffu, incl, 31);
      if (ps + tot > tt) {
        const unsigned m = __ballot_sync(0xffffffffu, ps + incl > tt);
        const int src = __ffs(m) - 1;
        s = base + src;
        ps += __shfl_sync(0xffffffffu, incl - n, src);
        eord += __shfl_sync(0xffffffffu, eincl - (n > 0 ? 1 : 0), src);
        break;
      }
      ps += tot;
      eord += __shfl_sync(0xffffffffu, eincl, 31);
    }
    int chunk = (int)(tt - ps);
    int L = seq_len_of(p, s);
    int nch = nchunks_of(L);
    if constexpr (APPEND) {
      // publish the segments whose final chunk lies in this range: the
      // consumer warps quantize their new tokens now, while the first copies
      // are in flight
      int n_end = 0;
      int es = s, ekg = kg, eL = L;
      long long e_last = t_begin - chunk + nch - 1;  // global index of the segment's final chunk
      while (n_end < kMaxEnds && e_last < t_end) {
        if (lane == 0) {
          hdr->end_seq[n_end] = es;
          hdr->end_kg[n_end] = ekg;
          hdr->end_len[n_end] = eL;
        }
        ++n_end;
        int s2 = es, kg2 = ekg, L2 = 0;
        bool have = false;
        while (!have && kg2 < p.ngroups) have = next_segment(p, s2, kg2, s2, kg2, L2);
        if (!have || kg2 >= p.ngroups) break;
        es = s2;
        ekg = kg2;
        eL = L2;
        e_last += nchunks_of(L2);
      }
      __syncwarp();
      if (lane == 0) {
        hdr->n_end = n_end;
        mbar_arrive(&hdr->prologue);
      }
    }
    int ends_passed = 0;  // final chunks issued so far
    bool first = true;
    uint32_t seg = 0;  // segments started by this CTA
    int seg_ncov = 1, seg_cfirst = c, seg_mergers = 0;

    // prefetched state: page-id windows of this segment (current, next) and
    // the next segment's length and first window
    // whole 16-token tiles per copy (mode 0: contiguous bulk; mode 3: 2-D tiled)
    const bool pg_mode0 = (LAYOUT == LAYOUT_PAGED) && (p.paged_mode == 0 || p.paged_mode >= 3);
    int pg_base = 2 * chunk;
    int64_t pg_cur = 0, pg_nxt = 0, pg_seg = 0;
    int ns = 0, nkg = 0, nL = 0;
    bool have_next = false;
    if (pg_mode0) {
      const int ntile = (L + kTileTokens - 1) / kTileTokens;
      pg_cur = page_window(p, s, pg_base, ntile);
      pg_nxt = page_window(p, s, pg_base + 32, ntile);
    }
    auto prefetch_next_segment = [&]() {
      have_next = next_segment(p, s, kg, ns, nkg, nL);
      if (pg_mode0 && have_next && nkg < p.ngroups)
        pg_seg = page_window(p, ns, 0, (nL + kTileTokens - 1) / kTileTokens);
    };
    prefetch_next_segment();

    for (long long t = t_begin; t < t_end; ++t) {
      if (it >= (uint32_t)p.stages) {
        if (!mbar_wait(&hdr->empty[stage], phase ^ 1u, p.wait_limit_ns)) {
          failed = true;
          break;
        }
      }
      const int qb = (int)(seg % (uint32_t)p.nqbuf);
      if (first) {
        // CTAs whose ranges cover this segment (its chunk 0 is global chunk t - chunk)
        const long long p0 = t - chunk;
        seg_cfirst = (int)part().owner(cost_pos(p0, eord, SC, U8));
        const int c_last = (int)part().owner(cost_pos(p0 + nch - 1, eord, SC, U8));
        seg_ncov = c_last - seg_cfirst + 1;
        // CTAs c_first .. c_last-1 end their ranges inside the segment; c_last
        // does too when the segment ends exactly where its range ends (the
        // next chunk, the next segment's first, belongs to a later piece)
        const long long tn = p0 + nch;
        seg_mergers = seg_ncov - 1 +
                      ((tn >= T || part().owner(cost_pos(tn, eord + 1, SC, U8)) > c_last) ? 1 : 0);
      }
      const bool last = (chunk == nch - 1) || (t == t_end - 1);
      const int nvalid = min(kChunkTokens, L - chunk * kChunkTokens);
      int flags = (first ? kFlagFirst : 0) | (last ? kFlagLast : 0) | (qb ? kFlagQbuf : 0) |
                  (t == t_end - 1 ? kFlagRangeEnd : 0);
      if constexpr (APPEND) {
        if (chunk == nch - 1) {
          if (ends_passed == 0) {
            // the consumers quantized this one at the start, possibly after
            // the copy below reads the slot: they patch the staged row
            flags |= kFlagPatch;
          } else if (ends_passed < hdr->n_end) {
            // quantized at the start too: wait until those slots are written
            // before the copy below reads them
            if (ends_passed == 1 && !mbar_wait(&hdr->appended, 0u, p.wait_limit_ns)) {
              failed = true;
              break;
            }
          } else {
            // beyond the published ends: quantize it here
            producer_append<D>(p, s, kg, L - 1);
          }
          ++ends_passed;
        }
      }
      const int slot = (int)(c + (int64_t)kg * B + s);
      uint8_t* dst = stg + (size_t)stage * p.stage_bytes;
      uint64_t* fb = &hdr->full[stage];
      const int tok0 = chunk * kChunkTokens;

      if (LAYOUT == LAYOUT_PAGED) {
        const int bs = p.block_size;
        const int row_bytes = p.kvc * SLOT;
        if (pg_mode0) {
          // tiles 2*chunk, 2*chunk+1: page ids from the prefetched windows
          const int t0 = 2 * chunk;
          if (t0 - pg_base >= 32) {
            pg_base += 32;
            pg_cur = pg_nxt;
            pg_nxt = page_window(p, s, pg_base + 32, (L + kTileTokens - 1) / kTileTokens);
          }
          const int ntile = (L + kTileTokens - 1) / kTileTokens;
          const int64_t ph0 = __shfl_sync(0xffffffffu, pg_cur, t0 - pg_base);
          const int64_t ph1 = __shfl_sync(0xffffffffu, pg_cur, t0 + 1 - pg_base);
          const bool has1 = t0 + 1 < ntile;
          const bool ok0 = ph0 >= 0 && ph0 < p.num_blocks;
          const bool ok1 = has1 && ph1 >= 0 && ph1 < p.num_blocks;
          if (lane == 0 && (!ok0 || (has1 && !ok1))) set_err(p, 1u);
          const uint32_t tile_bytes = (uint32_t)(kTileTokens * row_bytes);
          const uint32_t tx = (ok0 ? tile_bytes : 0u) + (ok1 ? tile_bytes : 0u);
          if (lane == 0) {
            hdr->desc[stage] = ChunkDesc{s, kg, chunk, nvalid, flags, slot, seg_ncov, seg_cfirst, seg_mergers, APPEND ? L : 0, {0, 0}};
          }
          __syncwarp();
          if (lane == 0) {
            mbar_arrive_expect_tx(fb, tx);
            if (p.paged_mode == 4) {
              // whole rows of 16 tokens: 64-byte pieces x rows, swizzled
              if (ok0) tma_load_3d_hint(dst, &p.tmap_k, 0, 0, (int)(ph0 * bs + tok0 % bs), fb, policy);
              if (ok1)
                tma_load_3d_hint(dst + tile_bytes, &p.tmap_k, 0, 0, (int)(ph1 * bs + (tok0 + kTileTokens) % bs), fb,
                                 policy);
            } else if (p.paged_mode == 3) {
              // the group's heads of 16 token rows: x = first 8-byte element of
              // head kg*kvc in a row (a multiple of 16 bytes), y = token row
              const int x = kg * p.kvc * (SLOT / 8);
              if (ok0) tma_load_2d(dst, &p.tmap_k, x, (int)(ph0 * bs + tok0 % bs), fb);
              if (ok1) tma_load_2d(dst + tile_bytes, &p.tmap_k, x, (int)(ph1 * bs + (tok0 + kTileTokens) % bs), fb);
            } else {
              if (ok0)
                bulk_g2s(dst, p.cache + ((ph0 * bs + tok0 % bs) * p.kv_total) * (int64_t)SLOT, tile_bytes, fb,
                         policy);
              if (ok1)
                bulk_g2s(dst + tile_bytes,
                         p.cache + ((ph1 * bs + (tok0 + kTileTokens) % bs) * p.kv_total) * (int64_t)SLOT,
                         tile_bytes, fb, policy);
            }
          }
        } else {
          // one row (token) per lane
          const int row = lane;
          const int tok = tok0 + row;
          const int rows_alloc = ((L + bs - 1) / bs) * bs - tok0;  // rows whose page exists
          int64_t phys = -1;
          bool ok = false;
          if (row < rows_alloc) {
            phys = block_entry(p, s, tok / bs);
            ok = phys >= 0 && phys < p.num_blocks;
            if (!ok) set_err(p, 1u);
          }
          const unsigned okm = __ballot_sync(0xffffffffu, ok);
          if (lane == 0) {
            hdr->desc[stage] = ChunkDesc{s, kg, chunk, nvalid, flags, slot, seg_ncov, seg_cfirst, seg_mergers, APPEND ? L : 0, {0, 0}};
          }
          const uint8_t* src =
              p.cache + ((phys * bs + (tok % bs)) * p.kv_total + (int64_t)kg * p.kvc) * SLOT;
          if (p.paged_mode == 1) {
            const uint32_t tx = (uint32_t)(__popc(okm) * row_bytes);
            __syncwarp();
            if (lane == 0) mbar_arrive_expect_tx(fb, tx);
            __syncwarp();
            if (ok) bulk_g2s(dst + row * row_bytes, src, (uint32_t)row_bytes, fb, policy);
          } else {
            // cp.async, 8 bytes per op; each lane copies its own row
            if (ok) {
              for (int cc = 0; cc < row_bytes / 8; ++cc) cp_async8(dst + row * row_bytes + cc * 8, src + cc * 8);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_expect_tx(fb, 0u);
          }
        }
      } else {
        // contiguous layouts: per kv head of the group, nvalid rows of K and V
        const int64_t row0 = (int64_t)s * p.kv_seq_stride_rows + tok0;
        const int bytes = nvalid * HALF;
        const bool bulk = p.contig_bulk_ok && (bytes % 16 == 0);
        if (LAYOUT == LAYOUT_PER_TOKEN) {
          // rulers: 4 fp16 per (row, kv head) in slot-tail order
          uint16_t* rd = reinterpret_cast<uint16_t*>(dst + p.kvc * kChunkTokens * D);
          for (int i = lane; i < nvalid * p.kvc; i += 32) {
            const int rr = i / p.kvc, jj = i % p.kvc;
            const int64_t idx = row0 + (int64_t)(kg * p.kvc + jj) * p.s_cap + rr;
            uint16_t* o = rd + (rr * p.kvc + jj) * 4;
            o[0] = p.r0[idx];
            o[1] = p.r1[idx];
            o[2] = p.r2[idx];
            o[3] = p.r3[idx];
          }
        }
        if (lane == 0) {
          hdr->desc[stage] = ChunkDesc{s, kg, chunk, nvalid, flags, slot, seg_ncov, seg_cfirst, seg_mergers, APPEND ? L : 0, {0, 0}};
        }
        // stage: K block [kvc][32 rows][D/2] then V block of the same shape
        const int kblock = p.kvc * kChunkTokens * HALF;
        if (p.tma_tensor) {
          // one tiled copy per K / V: the chunk's 32 rows of every kv head of
          // the group (rows past the capacity arrive as zeros, past the
          // length as whatever is stored there; both are masked)
          __syncwarp();
          if (lane == 0) {
            const int x0 = tok0 * HALF / 8;  // 8-byte elements
            mbar_arrive_expect_tx(fb, (uint32_t)(2 * kblock));
            tma_load_3d(dst, &p.tmap_k, x0, kg * p.kvc, s, fb);
            tma_load_3d(dst + kblock, &p.tmap_v, x0, kg * p.kvc, s, fb);
          }
        } else {
          const uint32_t tx = bulk ? (uint32_t)(2 * p.kvc * bytes) : 0u;
          __syncwarp();
          if (lane == 0) mbar_arrive_expect_tx(fb, tx);
          __syncwarp();
          if (bulk) {
            if (lane < 2 * p.kvc) {
              const int jj = lane >> 1, isv = lane & 1;
              const int64_t roff = (row0 + (int64_t)(kg * p.kvc + jj) * p.s_cap) * HALF;
              const uint8_t* src = (isv ? p.v_codes : p.k_codes) + roff;
              bulk_g2s(dst + isv * kblock + jj * kChunkTokens * HALF, src, (uint32_t)bytes, fb, policy);
            }
          } else {
            const int cpr = bytes / 8;
            for (int i = lane; i < 2 * p.kvc * cpr; i += 32) {
              const int cp = i / cpr, cc = i % cpr;
              const int jj = cp >> 1, isv = cp & 1;
              const int64_t roff = (row0 + (int64_t)(kg * p.kvc + jj) * p.s_cap) * HALF + cc * 8;
              cp_async8(dst + isv * kblock + jj * kChunkTokens * HALF + cc * 8, (isv ? p.v_codes : p.k_codes) + roff);
            }
          }
        }
      }
      cp_async_arrive_noinc(fb);

      if (first) {
        // ---- q (raw fp16/bf16) and per-channel rulers of this segment, staged
        // after the segment's first chunk is already in flight ----
        const uint32_t use = seg / (uint32_t)p.nqbuf;
        if (use >= 1) {
          if (!mbar_wait(&hdr->qempty[qb], (use - 1) & 1u, p.wait_limit_ns)) {
            failed = true;
            ++it;
            break;
          }
        }
        const int hg = p.kvc * p.G;  // q heads of the group
        uint8_t* qd = qbuf + qb * p.qbuf_bytes;
        const int64_t qrow0 = (int64_t)s * p.q_seq_stride + (int64_t)kg * hg * p.q_head_stride;
        const uint16_t* qsrc = reinterpret_cast<const uint16_t*>(p.q) + qrow0;
        uint32_t qtx = 0;
        if (p.q_bulk)
          qtx = (uint32_t)(hg * D * 2);
        else
          for (int i = lane; i < hg * D; i += 32)
            reinterpret_cast<uint16_t*>(qd)[i] = qsrc[(int64_t)(i / D) * p.q_head_stride + i % D];
        // per-channel rulers (only read when use_quant): the group's kvc*D
        // values of k_scale, k_zero, v_scale, v_zero, one contiguous span each
        uint16_t* rd = reinterpret_cast<uint16_t*>(rbuf + qb * p.rbuf_bytes);
        const int64_t rsrc = (int64_t)s * p.ruler_seq_stride + (int64_t)kg * p.kvc * D;
        const int span = p.kvc * D;
        uint32_t rtx = 0;
        if (LAYOUT == LAYOUT_PER_CHANNEL && p.use_quant) {
          if (p.rul_bulk) {
            rtx = (uint32_t)(4 * span * 2);
          } else {
            for (int a = 0; a < 4; ++a) {
              const uint16_t* src = ((a == 0) ? p.r0 : (a == 1) ? p.r1 : (a == 2) ? p.r2 : p.r3) + rsrc;
              for (int i = lane; i < span; i += 32) rd[a * span + i] = src[i];
            }
          }
        }
        __syncwarp();
        ++q_issued[qb];
        if (lane == 0) {
          mbar_arrive_expect_tx(&hdr->qfull[qb], qtx + rtx);
          if (qtx) bulk_g2s(qd, qsrc, qtx, &hdr->qfull[qb], policy);
          if (rtx) {
            bulk_g2s(rd, p.r0 + rsrc, (uint32_t)(span * 2), &hdr->qfull[qb], policy);
            bulk_g2s(rd + span, p.r1 + rsrc, (uint32_t)(span * 2), &hdr->qfull[qb], policy);
            bulk_g2s(rd + 2 * span, p.r2 + rsrc, (uint32_t)(span * 2), &hdr->qfull[qb], policy);
            bulk_g2s(rd + 3 * span, p.r3 + rsrc, (uint32_t)(span * 2), &hdr->qfull[qb], policy);
          }
        }
      }

      ++it;
      if (++stage == p.stages) {
        stage = 0;
        phase ^= 1u;
      }
      first = false;
      ++chunk;
      if (chunk == nch && t + 1 < t_end) {
        // next non-empty segment (prefetched when this one started)
        if (!have_next) {  // 32 empty sequences in a row: keep scanning
          while (!have_next) {
            s = ns;
            kg = nkg;
            have_next = next_segment(p, s, kg, ns, nkg, nL);
          }
          if (pg_mode0) pg_seg = page_window(p, ns, 0, (nL + kTileTokens - 1) / kTileTokens);
        }
        s = ns;
        kg = nkg;
        L = nL;
        nch = nchunks_of(L);
        chunk = 0;
        first = true;
        ++seg;
        ++eord;
        if (pg_mode0) {
          const int ntile = (L + kTileTokens - 1) / kTileTokens;
          pg_base = 0;
          pg_cur = pg_seg;
          pg_nxt = page_window(p, s, 32, ntile);
        }
        prefetch_next_segment();
      }
    }
  }

  if constexpr (APPEND) {
    if (t_begin >= t_end && lane == 0) {  // empty range: nothing to publish
      hdr->n_end = 0;
      mbar_arrive(&hdr->prologue);
    }
  }
  if (!failed) {
    // terminal descriptor
    if (it >= (uint32_t)p.stages) {
      if (!mbar_wait(&hdr->empty[stage], phase ^ 1u, p.wait_limit_ns)) failed = true;
    }
    if (!failed) {
      if (lane == 0) hdr->desc[stage].seq = -1;
      __syncwarp();
      if (lane == 0) mbar_arrive(&hdr->full[stage]);
      cp_async_arrive_noinc(&hdr->full[stage]);
      ++it;
    }
  }
  if (failed && lane == 0) set_err(p, 4u);
  // Wait (bounded) until every copy this warp issued has landed, so that the
  // CTA never exits with a copy into its shared memory in flight -- also
  // when the consumers gave up early.  Stages the consumers already waited
  // for pass at once.
  const uint32_t n = it < (uint32_t)p.stages ? it : (uint32_t)p.stages;
  for (uint32_t k = 0; k < n; ++k) {
    const uint32_t i = it - 1 - k;
    const int st = (int)(i % (uint32_t)p.stages);
    const uint32_t ph = (i / (uint32_t)p.stages) & 1u;
    mbar_wait(&hdr->full[st], ph, kDrainLimitNs);
  }
  for (int b = 0; b < 2; ++b)
    if (q_issued[b]) mbar_wait(&hdr->qfull[b], (q_issued[b] - 1u) & 1u, kDrainLimitNs);
}

// Output element store in the requested dtype (0 f16, 1 bf16, 2 f32).
__device__ __forceinline__ void store_out(const DecodeParams& p, int64_t off, float v) {
  if (p.out_dtype == 2)
    reinterpret_cast<float*>(p.out)[off] = v;
  else if (p.out_dtype == 1)
    reinterpret_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<__half*>(p.out)[off] = __float2half_rn(v);
}

// Barrier of the CTA's consumer threads only (the producer warp never joins).
// Every consumer warp reaches each of these the same number of times: a warp
// that gives up on a wait leaves the main loop for the barrier after it (it
// never returns early), so no warp is left waiting here.
template <int NCW>
__device__ __forceinline__ void consumer_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
}

// The CTA's consumer threads merge segment `job` from the partials of CTAs
// c_first .. c_first+ncov-1 and write its output rows.  Work goes in passes
// over groups of heads and batches of partials sized to the scratch `scr`
// (the idle stage ring).  Per pass: one round of L2 reads (cp.async.cg for
// the partial rows, ld.global.cg for the (m, l) pairs -- coherent with the
// other CTAs' stores), then every thread folds the batch into the output
// quads it owns, computing the log-sum-exp weights of their heads itself.
template <int D, int KVC>
__device__ void merge_segment(const DecodeParams& p, const MergeJob& job, int i0, int i1, float* scr,
                              int scr_floats) {
  constexpr int NTHR = KVC * 32;
  constexpr int Q = D / 4;
  constexpr int IPT = 4;  // output quads per thread per pass
  const int tid = threadIdx.x;
  const int hg = p.kvc * p.G;
  const int np = job.ncov;
  // partials per pass: up to 64 (a segment split over many CTAs, e.g. one
  // long sequence over the whole grid, then merges in few dependent passes)
  int nb = min(np, 64);
  while (nb > 1 && nb * (D + 2) > scr_floats) nb >>= 1;
  const int hp = max(1, min(min(hg, scr_floats / (nb * (D + 2))), IPT * NTHR / Q));
  const int64_t row0 = (int64_t)(job.c_first + job.e_seg) * hg;  // partial i, head h: row0 + i*hg + h
  const float4* acc4 = reinterpret_cast<const float4*>(p.part_acc);
  const float2* ml2 = reinterpret_cast<const float2*>(p.part_ml);
  float* sRow = scr;                 // [nb][hp][D]
  float2* sMl = reinterpret_cast<float2*>(scr + nb * hp * D);  // [nb][hp]
  // items are (head, dim quad) pairs h*Q + q; this call owns [i0, i1)
  const int hlo = i0 / Q, hhi = (i1 + Q - 1) / Q;
  for (int h0 = hlo; h0 < hhi; h0 += hp) {
    const int hb = min(hp, hhi - h0);
    const int lo = max(i0 - h0 * Q, 0), hi = min(i1 - h0 * Q, hb * Q);  // local item range
    float4 a[IPT];
    float M[IPT], L[IPT];
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      a[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      M[k] = -INFINITY;
      L[k] = 0.f;
    }
    for (int p0 = 0; p0 < np; p0 += nb) {
      const int nbb = min(nb, np - p0);
      for (int i = 0; i < nbb; ++i) {
        const int64_t r = row0 + (int64_t)(p0 + i) * hg + h0;
        for (int t = lo + tid; t < hi; t += NTHR) cp_async16_cg(sRow + (i * hp * D + 4 * t), acc4 + r * Q + t);
      }
      // (m, l) pairs: two loads in flight per thread before either store, so
      // no thread serialises on one L2 round trip per partial.
      for (int t = tid; t < nbb * hb; t += 2 * NTHR) {
        const int t1 = t + NTHR;
        const int ia = t / hb, ib = t1 / hb;
        const float2 v0 = __ldcg(ml2 + row0 + (int64_t)(p0 + ia) * hg + h0 + (t - ia * hb));
        float2 v1 = make_float2(0.f, 0.f);
        if (t1 < nbb * hb) v1 = __ldcg(ml2 + row0 + (int64_t)(p0 + ib) * hg + h0 + (t1 - ib * hb));
        sMl[ia * hp + (t - ia * hb)] = v0;
        if (t1 < nbb * hb) sMl[ib * hp + (t1 - ib * hb)] = v1;
      }
      cp_async_wait_all();
      consumer_bar<KVC>();
#pragma unroll
      for (int k = 0; k < IPT; ++k) {
        const int item = lo + k * NTHR + tid;
        if (item < hi) {
          const int h = item / Q;
          float mx = M[k];
          for (int i = 0; i < nbb; ++i) mx = fmaxf(mx, sMl[i * hp + h].x);
          if (mx != -INFINITY) {
            const float sc = (M[k] == -INFINITY) ? 0.f : exp2_approx(M[k] - mx);
            float4 v = make_float4(a[k].x * sc, a[k].y * sc, a[k].z * sc, a[k].w * sc);
            float l = L[k] * sc;
            for (int i = 0; i < nbb; ++i) {
              const float2 ml = sMl[i * hp + h];
              const float w = (ml.x == -INFINITY) ? 0.f : exp2_approx(ml.x - mx);
              const float4 x = *reinterpret_cast<const float4*>(sRow + (i * hp * D + 4 * item));
              l += w * ml.y;
              v.x += w * x.x;
              v.y += w * x.y;
              v.z += w * x.z;
              v.w += w * x.w;
            }
            a[k] = v;
            L[k] = l;
            M[k] = mx;
          }
        }
      }
      consumer_bar<KVC>();
    }
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      const int item = lo + k * NTHR + tid;
      if (item < hi) {
        const int h = item / Q, q = item % Q;
        const float inv = (L[k] > 0.f) ? 1.f / L[k] : 0.f;
        const int64_t o = (int64_t)job.seq * p.out_seq_stride +
                          (int64_t)(job.kg * hg + h0 + h) * p.out_head_stride + 4 * q;
        store_out(p, o, a[k].x * inv);
        store_out(p, o + 1, a[k].y * inv);
        store_out(p, o + 2, a[k].z * inv);
        store_out(p, o + 3, a[k].w * inv);
      }
    }
  }
}

// ------------------------------------------------------------------ consumer --
// Both operands that carry codes keep the magic-number bias (low nibble
// 1024+c, high nibble 64+c).  QK: sum_d q_d*(bias_d + c_d) = q.c +
// sum_d q_d*bias_d, and the second term (one number per head) starts the
// accumulator negated.  PV: sum_t P'_t*(bias_d + c_td) = P'.c_d +
// bias_d*sum_t P'_t, and sum_t P'_t comes from the same P' against a ones
// tile, subtracted when the segment's rows are finalised.  No f16x2 op is
// spent per code.
// Per-thread state of one consumer warp (head columns 2r, 2r+1 of each
// 8-head n-tile; output rows = head dims 2*(g*D/16 + mt) + {0, 1}).
template <int D, int NT>
struct WarpState {
  static constexpr int KS = D / 16;
  uint4 qf[NT][(D / 8 + 3) / 4];  // q B-fragments: k-steps 2u (x, y) and 2u+1 (z, w)
  float qs[NT][2];         // log2e*scale * (sum q (per-token) | sum q'*zero (per-channel))
  float qb[NT][2];         // QK accumulator bias: sum_d q_d * (1024 | 64)
  float acc[KS][NT][4];     // O^T on biased V codes: rows g hold 1024 + c, rows g+8 hold 64 + c
  float ps[NT][2];          // sum over tokens of P' per head column, to take the V bias off
  float m[NT][2], l[NT][2], vs[NT][2];
};

// PK (one n-tile, at most 4 query heads per kv head): lanes of columns 4..7
// carry the same query heads as columns 0..3, so one score fragment holds
// tile 0's scores in columns 0..3 and tile 1's in columns 4..7 and the
// softmax runs on useful columns only; PV feeds each tile its own columns.
// The two column halves are two online-softmax streams over the even and
// odd tiles, combined at the segment end.
template <int D, int NT, int LAYOUT, int KVC, bool MASK, bool PK, bool SWZ>
__device__ __forceinline__ void consume_chunk(const DecodeParams& p, WarpState<D, NT>& w,
                                              const StageView<D, LAYOUT, KVC>& sv, int nvalid,
                                              uint64_t* empty_bar, bool release) {
  constexpr int KS = D / 16;  // QK k-steps == PV m-tiles
  constexpr int QB = D / 8;   // K bytes per thread per row
  constexpr int VB = D / 16;  // V bytes per thread per row
  constexpr int QW = (QB + 3) / 4;
  constexpr int VW = (VB + 3) / 4;
  constexpr int QALIGN = (QB % 8 == 0) ? 8 : 2;
  constexpr int VALIGN = (VB % 8 == 0) ? 8 : ((VB % 4 == 0) ? 4 : 1);
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, r = lane & 3;
  // QK / scores use token rows g and g+8 of each tile, PV rows 2r, 2r+1,
  // 2r+8, 2r+9
  using SV = StageView<D, LAYOUT, KVC>;
  static_assert(!SWZ || (LAYOUT == LAYOUT_PAGED && (D == 64 || D == 128) && SV::kRow % 64 == 0),
                "swizzled stages: whole 64-byte rows, 8-byte aligned reads");
  // fragment row -> token row of the tile (identity unless swizzled)
  const int tg = SWZ ? tok_perm(g) : g;
  const int tv0 = SWZ ? tok_perm(2 * r) : 2 * r;
  const int tv1 = SWZ ? tok_perm(2 * r + 1) : 2 * r + 1;
  const uint8_t* krow = sv.k(tg);  // + a*d16 + h*d8 -> row 16a + tg + 8h
  const uint8_t* rrow = sv.rulers(tg);
  const uint8_t* vrow0 = sv.v(tv0);
  const uint8_t* vrow1 = sv.v(tv1);
  // swizzled: sv.base is the stage base (1024-aligned); the warp's head and
  // every byte offset within a row go through swz64, and the reads use
  // 32-bit shared addresses
  uint32_t kq0 = 0, kq1 = 0, rq = 0, vq0 = 0, vq1 = 0;
  if constexpr (SWZ) {
    const uint32_t sb = smem_addr(sv.base);
    const uint32_t hb = (uint32_t)(threadIdx.x >> 5) * (D + 8);
    const uint32_t ok = (uint32_t)(tg * SV::kRow) + hb;
    kq0 = sb + swz64(ok + 8u * r);
    kq1 = sb + swz64(ok + 32u + 8u * r);
    rq = sb + swz64(ok + D);
    const uint32_t ov = (uint32_t)(tv0 * SV::kRow) + hb + D / 2 + (uint32_t)(g * (D / 16));
    vq0 = sb + swz64(ov);
    vq1 = sb + swz64(ov + 2 * SV::kRow);  // tok_perm(2r+1) = tok_perm(2r) + 2
  }
  static_assert(!PK || NT == 1, "tile packing needs one n-tile");
  constexpr int NA = PK ? 1 : 2;     // score tiles held per thread
  const int at = PK ? (r >> 1) : 0;  // PK: the tile of this thread's columns

  // ---- QK on biased codes: both tiles' codes loaded, then their two
  // accumulator chains advanced in turn (a second chain per tile would cost
  // registers the kernel does not have) ----
  float sacc[2][NT][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      sacc[a][nt][0] = sacc[a][nt][2] = -w.qb[nt][0];
      sacc[a][nt][1] = sacc[a][nt][3] = -w.qb[nt][1];
    }
  uint32_t ka[2][QW], kb[2][QW];
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    const uint8_t* k0 = krow + a * SV::d16;
    if constexpr (SWZ) {
      uint2 x = lds64(kq0 + a * SV::d16), y = lds64(kq0 + a * SV::d16 + SV::d8);
      ka[a][0] = x.x;
      ka[a][1] = x.y;
      kb[a][0] = y.x;
      kb[a][1] = y.y;
      if constexpr (QB == 16) {
        x = lds64(kq1 + a * SV::d16);
        y = lds64(kq1 + a * SV::d16 + SV::d8);
        ka[a][2] = x.x;
        ka[a][3] = x.y;
        kb[a][2] = y.x;
        kb[a][3] = y.y;
      }
    } else if constexpr (QB == 16) {
      load_bytes<8, 8>(k0 + 8 * r, ka[a]);
      load_bytes<8, 8>(k0 + 32 + 8 * r, ka[a] + 2);
      load_bytes<8, 8>(k0 + SV::d8 + 8 * r, kb[a]);
      load_bytes<8, 8>(k0 + SV::d8 + 32 + 8 * r, kb[a] + 2);
    } else {
      load_bytes<QB, QALIGN>(k0 + r * QB, ka[a]);
      load_bytes<QB, QALIGN>(k0 + SV::d8 + r * QB, kb[a]);
    }
  }
  // consecutive tensor-core ops belong to different tiles: independent
#pragma unroll
  for (int u = 0; u < QW; ++u) {
    uint4 qf[NT];  // B-fragments of k-steps 2u (x, y) and 2u+1 (z, w)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) qf[nt] = w.qf[nt][u];
    if (4 * u + 4 <= QB) {
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        const uint32_t a0 = codes_lo_biased(ka[a][u]), a1 = codes_lo_biased(kb[a][u]);
        const uint32_t a2 = codes_hi_biased(ka[a][u]), a3 = codes_hi_biased(kb[a][u]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816(sacc[a][nt], a0, a1, a2, a3, qf[nt].x, qf[nt].y);
      }
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        const uint32_t sa = ka[a][u] >> 8, sb = kb[a][u] >> 8;
        const uint32_t a0 = codes_lo_biased(sa), a1 = codes_lo_biased(sb);
        const uint32_t a2 = codes_hi_biased(sa), a3 = codes_hi_biased(sb);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816(sacc[a][nt], a0, a1, a2, a3, qf[nt].z, qf[nt].w);
      }
    } else {
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        const uint32_t sa = __byte_perm(ka[a][u], 0u, 0x3120), sb = __byte_perm(kb[a][u], 0u, 0x3120);
        const uint32_t a0 = codes_lo_biased(sa), a1 = codes_lo_biased(sb);
        const uint32_t a2 = codes_hi_biased(sa), a3 = codes_hi_biased(sb);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816(sacc[a][nt], a0, a1, a2, a3, qf[nt].x, qf[nt].y);
      }
    }
  }
  if constexpr (PK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) sacc[0][0][i] = at ? sacc[1][0][i] : sacc[0][0][i];
  }

  // ---- per-token rulers (k_min, k_step | v_min, v_step) ----
  auto tile = [&](int a) { return PK ? at : a; };
  // one 8-byte read per token row: (k_min, k_step, v_min, v_step)
  uint2 rr[NA][2];
  if (LAYOUT != LAYOUT_PER_CHANNEL) {
#pragma unroll
    for (int a = 0; a < NA; ++a)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if constexpr (SWZ)
          rr[a][h] = lds64(rq + tile(a) * SV::r16 + h * SV::r8);
        else
          rr[a][h] = *reinterpret_cast<const uint2*>(rrow + tile(a) * SV::r16 + h * SV::r8);
      }
  }
  auto ruler_k = [&](int a, int h) -> float2 {
    if (LAYOUT == LAYOUT_PER_CHANNEL) return make_float2(p.use_quant ? -1.f : 0.f, 1.f);
    return __half22float2(*reinterpret_cast<const __half2*>(&rr[PK ? 0 : a][h].x));
  };
  auto ruler_v = [&](int a, int h) -> float2 {
    if (LAYOUT == LAYOUT_PER_CHANNEL) return make_float2(0.f, 1.f);
    return __half22float2(*reinterpret_cast<const __half2*>(&rr[PK ? 0 : a][h].y));
  };
  bool val[NA][2];
#pragma unroll
  for (int a = 0; a < NA; ++a)
#pragma unroll
    for (int h = 0; h < 2; ++h) val[a][h] = !MASK || (16 * tile(a) + tg + 8 * h) < nvalid;

  // ---- scores + online softmax (log2 domain, lazy rescale) ----
  const float sl2 = p.scale_log2;
  float sc[NA][NT][4];
  float mx[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) mx[nt][0] = mx[nt][1] = -INFINITY;
#pragma unroll
  for (int a = 0; a < NA; ++a) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float2 kr = ruler_k(tile(a), h);
      const float kst = kr.y * sl2;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float v = fmaf(sacc[a][nt][2 * h + e], kst, kr.x * w.qs[nt][e]);
          if (MASK) v = val[a][h] ? v : -INFINITY;
          sc[a][nt][2 * h + e] = v;
          mx[nt][e] = fmaxf(mx[nt][e], v);
        }
      }
    }
  }
  // Each thread checks its own scores against the running max; only when
  // some score exceeds it by more than the slack is the head max reduced
  // across the 8 lanes that share the head column and the state rescaled.
  bool need = false;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
    need |= (mx[nt][0] > w.m[nt][0] + kRescaleSlack) || (mx[nt][1] > w.m[nt][1] + kRescaleSlack);
  if (__any_sync(0xffffffffu, need)) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        mx[nt][0] = fmaxf(mx[nt][0], __shfl_xor_sync(0xffffffffu, mx[nt][0], o));
        mx[nt][1] = fmaxf(mx[nt][1], __shfl_xor_sync(0xffffffffu, mx[nt][1], o));
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float mn = fmaxf(w.m[nt][e], mx[nt][e]);
        const float al = exp2_approx(w.m[nt][e] - mn);
        w.m[nt][e] = mn;
        w.l[nt][e] *= al;
        w.vs[nt][e] *= al;
        w.ps[nt][e] *= al;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          w.acc[mt][nt][e] *= al;
          w.acc[mt][nt][e + 2] *= al;
        }
      }
    }
  }

  uint32_t pb[NA][NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      float pp[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int h = i >> 1, e = i & 1;
        const float2 vr = ruler_v(tile(a), h);
        const float pe = exp2_approx(sc[a][nt][i] - w.m[nt][e]);  // 0 for masked rows
        w.l[nt][e] += pe;
        if (MASK) {
          w.vs[nt][e] += val[a][h] ? pe * vr.x : 0.f;
          pp[i] = val[a][h] ? pe * vr.y : 0.f;
        } else {
          w.vs[nt][e] = fmaf(pe, vr.x, w.vs[nt][e]);
          pp[i] = pe * vr.y;
        }
      }
      pb[a][nt][0] = movmatrix_t(pack_half2(pp[0], pp[1]));
      pb[a][nt][1] = movmatrix_t(pack_half2(pp[2], pp[3]));
    }
  }

  // ---- PV on biased codes: O^T[dims x heads] += (V^T + bias) . P'^T, one
  // k-step per tile; the same P' against a ones tile gives sum_t P'_t per
  // head, exactly as the tensor core sums it, to take the bias off later ----
  // thread (g, r) needs tokens 16a + {2r, 2r+1, 2r+8, 2r+9}, bytes [g*VB, +VB)
  constexpr uint32_t kOnes = 0x3C003C00u;  // fp16x2 (1, 1)
#pragma unroll
  for (int a = 0; a < NA; ++a)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      mma_16816_rows0(w.ps[nt][0], w.ps[nt][1], kOnes, kOnes, kOnes, kOnes, pb[a][nt][0], pb[a][nt][1]);
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    // B operand of tile a: PK keeps only the columns of tile a (B column = g)
    uint32_t pbt[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if constexpr (PK) {
        const bool mine = (g >= 4) == (a == 1);
        pbt[nt][0] = mine ? pb[0][nt][0] : 0u;
        pbt[nt][1] = mine ? pb[0][nt][1] : 0u;
      } else {
        pbt[nt][0] = pb[a][nt][0];
        pbt[nt][1] = pb[a][nt][1];
      }
    }
    uint32_t vw[4][VW];
    if constexpr (SWZ) {
      // VB = 8 (D=128) or 4 (D=64) bytes of rows tv0, tv1 (+8)
      const uint32_t ad[4] = {vq0 + a * SV::d16, vq1 + a * SV::d16, vq0 + a * SV::d16 + SV::d8,
                              vq1 + a * SV::d16 + SV::d8};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if constexpr (VB == 8) {
          const uint2 x = lds64(ad[i]);
          vw[i][0] = x.x;
          vw[i][1] = x.y;
        } else {
          vw[i][0] = lds32(ad[i]);
        }
      }
    } else {
      load_bytes<VB, VALIGN>(vrow0 + a * SV::d16 + g * VB, vw[0]);
      load_bytes<VB, VALIGN>(vrow1 + a * SV::d16 + g * VB, vw[1]);
      load_bytes<VB, VALIGN>(vrow0 + a * SV::d16 + SV::d8 + g * VB, vw[2]);
      load_bytes<VB, VALIGN>(vrow1 + a * SV::d16 + SV::d8 + g * VB, vw[3]);
    }
    if (a == 1 && release) {  // every shared-memory read of the stage is done: release it
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar);
    }
#pragma unroll
    for (int u = 0; u < VW; ++u) {
      const uint32_t x = __byte_perm(vw[0][u], vw[1][u], 0x5410);
      const uint32_t y = __byte_perm(vw[0][u], vw[1][u], 0x7632);
      const uint32_t x2 = __byte_perm(vw[2][u], vw[3][u], 0x5410);
      const uint32_t y2 = __byte_perm(vw[2][u], vw[3][u], 0x7632);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int mt = 4 * u + k;
        if (mt < KS) {
          const uint32_t w1 = (k == 0) ? x : (k == 1) ? (x >> 8) : (k == 2) ? y : (y >> 8);
          const uint32_t w2 = (k == 0) ? x2 : (k == 1) ? (x2 >> 8) : (k == 2) ? y2 : (y2 >> 8);
          const uint32_t a0 = codes_lo_biased(w1), a1 = codes_hi_biased(w1);
          const uint32_t a2 = codes_lo_biased(w2), a3 = codes_hi_biased(w2);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_16816(w.acc[mt][nt], a0, a1, a2, a3, pbt[nt][0], pbt[nt][1]);
        }
      }
    }
  }
}

// Take the V-code bias out of the PV accumulator: rows g hold 1024 + c,
// rows g+8 hold 64 + c, so acc -= bias * sum_t P'_t, and the sum restarts.
// Done every few chunks, not only at the segment end: the tensor core's
// fp32 accumulation errs by a fraction of the accumulator's magnitude, and
// the bias would otherwise grow that magnitude over a long segment.
template <int D, int NT>
__device__ __forceinline__ void fold_v_bias(WarpState<D, NT>& w) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        w.acc[mt][nt][e] = fmaf(-1024.f, w.ps[nt][e], w.acc[mt][nt][e]);
        w.acc[mt][nt][e + 2] = fmaf(-64.f, w.ps[nt][e], w.acc[mt][nt][e + 2]);
      }
      w.ps[nt][e] = 0.f;
    }
  }
}

// Fused append (paged layout): kv head h's new row of sequence `seq` (its
// newest token, position t = len-1) is quantized by this warp with the store
// kernel's arithmetic; the slot goes to the cache and, when `keep` (the
// range's first segment end, whose copy may already be in flight), to
// hdr->newslot[j], which replaces the stale staged copy of the slot when the
// segment's final chunk arrives.
template <int D, int KVC>
__device__ __forceinline__ void append_token(const DecodeParams& p, SmemHeader* hdr, int seq, int h, int t,
                                             int j, bool keep) {
  const int lane = threadIdx.x & 31;
  const int64_t ph = block_entry(p, seq, t / p.block_size);
  const int64_t off = ((int64_t)seq * p.new_seq_stride + (int64_t)h * D) * 2;  // bytes
  const SlotRow nr = quantize_slot_row<D>(reinterpret_cast<const uint8_t*>(p.new_k) + off,
                                          reinterpret_cast<const uint8_t*>(p.new_v) + off, p.new_bf16);
  if (ph >= 0 && ph < p.num_blocks)
    write_slot_row<D>(const_cast<uint8_t*>(p.cache) +
                          ((ph * p.block_size + t % p.block_size) * p.kv_total + h) * (int64_t)(D + 8),
                      nr);
  else if (lane == 0)
    set_err(p, 1u);
  if (keep) write_slot_row<D>(hdr->newslot[j], nr);
  __syncwarp();
}

template <int D, int NT, int LAYOUT, int KVC, bool PK, bool APPEND, bool SWZ>
__device__ void decode_consumer(const DecodeParams& p, SmemHeader* hdr,
                                const uint8_t* qbuf, const uint8_t* rbuf,
                                const uint8_t* stg) {
  constexpr int KS = D / 16;
  constexpr int VB = D / 16;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, r = lane & 3;
  constexpr int kvc = KVC;
  const int G = p.G;
  const int j = warp;  // one consumer warp per kv head of the group

  WarpState<D, NT> w;
  int stage = 0;
  uint32_t phase = 0, seg = 0;
  // A failed wait sets the error bit and the abort flag and leaves the loop
  // for the barrier after it.
  auto give_up = [&]() {
    if (lane == 0) {
      set_err(p, 4u);
      hdr->abort = 1;
    }
  };

  bool run = true;
  if (p.debug_stall && blockIdx.x == 0) {
    // Test hook (off unless the host sets it): CTA 0's consumer warps wait
    // for a barrier phase that nothing completes, so the wait runs out after
    // p.wait_limit_ns; the producer then times out on the ring and drains.
    if (!mbar_wait(&hdr->never, 0u, p.wait_limit_ns)) give_up();
    run = false;
  }

  if constexpr (APPEND) {
    // Fused append: quantize the new tokens of the segments whose final chunk
    // this CTA decodes (kv head j each), while the producer's first copies
    // are in flight; then let the producer copy those final chunks.
    if (run) {
      if (!mbar_wait(&hdr->prologue, 0u, p.wait_limit_ns)) {
        give_up();
        run = false;
      } else {
        const int n_end = hdr->n_end;
        for (int e = 0; e < n_end; ++e)
          append_token<D, KVC>(p, hdr, hdr->end_seq[e], hdr->end_kg[e] * kvc + j, hdr->end_len[e] - 1, j,
                               e == 0);
        fence_proxy_async_global();  // the producer's copies read these slots through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive(&hdr->appended);
      }
    }
  }

  while (run) {
    if (!mbar_wait(&hdr->full[stage], phase, p.wait_limit_ns)) {
      give_up();
      break;
    }
    const ChunkDesc& dsm = hdr->desc[stage];
    if (dsm.seq < 0) break;
    // fields needed after the stage is released are copied to registers
    const int flags = dsm.flags, slot = dsm.slot, nvalid = dsm.nvalid;
    const int qbi = (flags & kFlagQbuf) ? 1 : 0;

    if (flags & kFlagFirst) {
      // ---- segment start: q fragments, q sums, fresh softmax state ----
      if (!mbar_wait(&hdr->qfull[qbi], (seg / (uint32_t)p.nqbuf) & 1u, p.wait_limit_ns)) {
        give_up();
        break;
      }
      const __half* qh = reinterpret_cast<const __half*>(qbuf + qbi * p.qbuf_bytes) + (size_t)j * G * D;
      const __half* ksc = reinterpret_cast<const __half*>(rbuf + qbi * p.rbuf_bytes) + (size_t)j * D;
      const __half* kze = ksc + (size_t)kvc * D;
      float part[NT], bpart[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) part[nt] = bpart[nt] = 0.f;
#pragma unroll
      for (int s = 0; s < KS; ++s) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int n = PK ? (g & 3) : nt * 8 + g;  // PK: columns 4..7 repeat heads 0..3
          if constexpr (LAYOUT != LAYOUT_PER_CHANNEL && (D / 8) % 4 == 0) {
            if (!p.q_bf16) {
              // fp16 q, whole K words (D 64 / 128): k-slots 0 and 2 are the
              // adjacent dims 2b, 2b+1, slots 1 and 3 are 2b+4, 2b+5 (b =
              // this k-step's K byte): two 4-byte reads give the fragment
              // words by byte permutes, the sums take the same order as below
              uint32_t fa = 0u, fb = 0u;
              if (n < G) {
                const int b = kword_byte<D>(r, s >> 1) + (s & 1);
                const uint32_t w0 = *reinterpret_cast<const uint32_t*>(qh + n * D + 2 * b);
                const uint32_t w1 = *reinterpret_cast<const uint32_t*>(qh + n * D + 2 * b + 4);
                fa = __byte_perm(w0, w1, 0x5410);
                fb = __byte_perm(w0, w1, 0x7632);
                const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&w0));
                const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&w1));
                part[nt] += f0.x;
                part[nt] += f1.x;
                part[nt] += f0.y;
                part[nt] += f1.y;
                bpart[nt] += f0.x * 1024.f;
                bpart[nt] += f1.x * 1024.f;
                bpart[nt] += f0.y * 64.f;
                bpart[nt] += f1.y * 64.f;
              }
              if (s & 1) {
                w.qf[nt][s >> 1].z = fa;
                w.qf[nt][s >> 1].w = fb;
              } else {
                w.qf[nt][s >> 1].x = fa;
                w.qf[nt][s >> 1].y = fb;
              }
              continue;
            }
          }
          float x[4] = {0.f, 0.f, 0.f, 0.f};
          if (n < G) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int dd = qk_dim<D>(s, e, r);
              const uint16_t raw = reinterpret_cast<const uint16_t*>(qh)[n * D + dd];
              float v = p.q_bf16 ? __half2float(__float2half_rn(__bfloat162float(__ushort_as_bfloat16(raw))))
                                 : half_bits_to_float(raw);
              if (LAYOUT == LAYOUT_PER_CHANNEL) {
                if (p.use_quant) {
                  v = __half2float(__float2half_rn(v * __half2float(ksc[dd])));
                  part[nt] += v * __half2float(kze[dd]);
                }
              } else {
                part[nt] += v;
              }
              bpart[nt] += v * ((e < 2) ? 1024.f : 64.f);  // k-slots 0,1: low nibble
              x[e] = v;
            }
          }
          if (s & 1) {
            w.qf[nt][s >> 1].z = pack_half2(x[0], x[1]);
            w.qf[nt][s >> 1].w = pack_half2(x[2], x[3]);
          } else {
            w.qf[nt][s >> 1].x = pack_half2(x[0], x[1]);
            w.qf[nt][s >> 1].y = pack_half2(x[2], x[3]);
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float v = part[nt], bv = bpart[nt];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        bv += __shfl_xor_sync(0xffffffffu, bv, 1);
        bv += __shfl_xor_sync(0xffffffffu, bv, 2);
        w.qs[nt][0] = __shfl_sync(0xffffffffu, v, (2 * r) * 4) * p.scale_log2;
        w.qs[nt][1] = __shfl_sync(0xffffffffu, v, (2 * r + 1) * 4) * p.scale_log2;
        w.qb[nt][0] = __shfl_sync(0xffffffffu, bv, (2 * r) * 4);
        w.qb[nt][1] = __shfl_sync(0xffffffffu, bv, (2 * r + 1) * 4);
        // a finite floor (not -inf): a stream whose tokens in a chunk are all
        // masked must give exp2(-inf - m) = 0, not NaN
        w.m[nt][0] = w.m[nt][1] = kMaxFloor;
        w.l[nt][0] = w.l[nt][1] = 0.f;
        w.vs[nt][0] = w.vs[nt][1] = 0.f;
#pragma unroll
        for (int i = 0; i < 2; ++i) w.ps[nt][i] = 0.f;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) w.acc[mt][nt][i] = 0.f;
      }
      if (LAYOUT != LAYOUT_PER_CHANNEL) {
        // the q buffer is no longer needed: let the producer restage it
        __syncwarp();
        if (lane == 0) mbar_arrive(&hdr->qempty[qbi]);
      }
    }

    {
      const uint8_t* st = stg + (size_t)stage * p.stage_bytes;
      if constexpr (APPEND) {
        if (flags & kFlagPatch) {
          // the segment's newest token is the last valid row of this chunk:
          // its slot, quantized at the segment start, replaces the staged copy
          // (read from the cache before this launch wrote it)
          const uint32_t ro = (uint32_t)((nvalid - 1) * StageView<D, LAYOUT, KVC>::kRow + j * (D + 8));
          if (lane < (D + 8) / 8) {
            const uint32_t o = ro + 8u * lane;
            *reinterpret_cast<uint2*>(const_cast<uint8_t*>(st) + (SWZ ? swz64(o) : o)) =
                reinterpret_cast<const uint2*>(hdr->newslot[j])[lane];
          }
          fence_proxy_async_shared();  // before the producer's next copy reuses the stage
          __syncwarp();
        }
      }
      StageView<D, LAYOUT, KVC> sv;
      if (LAYOUT == LAYOUT_PAGED) {
        sv.base = SWZ ? st : st + j * (D + 8);  // swizzled: offsets are taken from the stage base
        sv.rul = nullptr;
      } else {
        sv.base = st + j * kChunkTokens * (D / 2);
        sv.rul = st + kvc * kChunkTokens * D + j * 8;
      }
      // a segment's last chunk keeps its stage (and descriptor) until the
      // segment's output or partial is written
      const bool rel = !(flags & kFlagLast);
      if (nvalid == kChunkTokens)
        consume_chunk<D, NT, LAYOUT, KVC, false, PK, SWZ>(p, w, sv, nvalid, &hdr->empty[stage], rel);
      else
        consume_chunk<D, NT, LAYOUT, KVC, true, PK, SWZ>(p, w, sv, nvalid, &hdr->empty[stage], rel);
    }

    if (flags & kFlagLast) {
      // ---- segment end: write the output, or a partial + maybe merge ----
      fold_v_bias(w);
      const ChunkDesc& dd = hdr->desc[stage];  // still owned: released below
      const int ncov = dd.ncov, c_first = dd.c_first;
      const int e_seg = dd.kg * p.num_seqs + dd.seq;
      const int seq = dd.seq, kgrp = dd.kg;
      const __half* vsc = reinterpret_cast<const __half*>(rbuf + qbi * p.rbuf_bytes) + (size_t)(2 * kvc + j) * D;
      const __half* vze = vsc + (size_t)kvc * D;
      const int hg = kvc * G;
      const bool direct = ncov == 1;
      const int64_t slotw = slot;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float l0 = w.l[nt][0], l1 = w.l[nt][1], u0 = w.vs[nt][0], u1 = w.vs[nt][1];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          l0 += __shfl_xor_sync(0xffffffffu, l0, o);
          l1 += __shfl_xor_sync(0xffffffffu, l1, o);
          u0 += __shfl_xor_sync(0xffffffffu, u0, o);
          u1 += __shfl_xor_sync(0xffffffffu, u1, o);
        }
        if constexpr (PK) {
          // lane r^2 holds the other tile parity's stream of the same heads
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float mo = __shfl_xor_sync(0xffffffffu, w.m[nt][e], 2);
            const float mn = fmaxf(w.m[nt][e], mo);
            const float s0 = exp2_approx(w.m[nt][e] - mn), s1 = exp2_approx(mo - mn);
            float& lr = e ? l1 : l0;
            float& ur = e ? u1 : u0;
            lr = lr * s0 + __shfl_xor_sync(0xffffffffu, lr, 2) * s1;
            ur = ur * s0 + __shfl_xor_sync(0xffffffffu, ur, 2) * s1;
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
              w.acc[mt][nt][e] = w.acc[mt][nt][e] * s0 + __shfl_xor_sync(0xffffffffu, w.acc[mt][nt][e], 2) * s1;
              w.acc[mt][nt][e + 2] =
                  w.acc[mt][nt][e + 2] * s0 + __shfl_xor_sync(0xffffffffu, w.acc[mt][nt][e + 2], 2) * s1;
            }
            w.m[nt][e] = mn;
          }
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int n = nt * 8 + 2 * r + e;
          const float lsum = e ? l1 : l0;
          const float vsum = e ? u1 : u0;
          if (n < G) {
            const int64_t row = slotw * hg + (int64_t)j * G + n;
            if (!direct && g == 0) {
              p.part_ml[row * 2 + 0] = w.m[nt][e];
              p.part_ml[row * 2 + 1] = lsum;
            }
            const float inv = (direct && lsum > 0.f) ? 1.f / lsum : 1.f;
            const int64_t obase = (int64_t)seq * p.out_seq_stride +
                                  (int64_t)(kgrp * hg + j * G + n) * p.out_head_stride + 2 * g * VB;
            float* dst = p.part_acc + row * D + 2 * g * VB;
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
              float o0 = w.acc[mt][nt][e] + vsum;
              float o1 = w.acc[mt][nt][e + 2] + vsum;
              if (LAYOUT == LAYOUT_PER_CHANNEL && p.use_quant) {
                const int d0 = 2 * (g * VB + mt);
                o0 = __half2float(vsc[d0]) * (o0 - __half2float(vze[d0]) * lsum);
                o1 = __half2float(vsc[d0 + 1]) * (o1 - __half2float(vze[d0 + 1]) * lsum);
              }
              if (direct) {
                // the two values are adjacent dims: one paired store when the
                // host found the output's element offsets even
                if (p.out_pair) {
                  if (p.out_dtype == 2)
                    *reinterpret_cast<float2*>(reinterpret_cast<float*>(p.out) + obase + 2 * mt) =
                        make_float2(o0 * inv, o1 * inv);
                  else if (p.out_dtype == 1)
                    *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(p.out) + obase + 2 * mt) =
                        __floats2bfloat162_rn(o0 * inv, o1 * inv);
                  else
                    *reinterpret_cast<uint32_t*>(reinterpret_cast<uint16_t*>(p.out) + obase + 2 * mt) =
                        pack_half2(o0 * inv, o1 * inv);
                } else {
                  store_out(p, obase + 2 * mt, o0 * inv);
                  store_out(p, obase + 2 * mt + 1, o1 * inv);
                }
              } else {
                reinterpret_cast<float2*>(dst)[mt] = make_float2(o0, o1);
              }
            }
          }
        }
      }
      if (!direct) {
        // publish this warp's slice of the partial (each consumer warp counts
        // itself); if this CTA's range ends in the segment it merges a slice
        // of it after its main loop
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(reinterpret_cast<unsigned int*>(p.seg_count) + e_seg, kArriveOne);
        if (threadIdx.x == 0 && (flags & kFlagRangeEnd)) {
          hdr->job = MergeJob{e_seg, seq, kgrp, c_first, ncov, dd.nmergers};
          hdr->has_job = 1;
        }
      }
      if (LAYOUT == LAYOUT_PER_CHANNEL) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&hdr->qempty[qbi]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&hdr->empty[stage]);
      ++seg;
    } else if (stage == 0 && phase == 0) {
      fold_v_bias(w);  // once per two turns of the stage ring
    }

    if (++stage == p.stages) {
      stage = 0;
      phase ^= 1u;
    }
  }

  // ---- this CTA's slice of the merge of the split segment its range ends
  // in (the stage ring is idle now: every copy has landed and been consumed) ----
  consumer_bar<KVC>();
  if (hdr->abort) return;  // every consumer warp returns here together
  if (hdr->has_job) {
    const MergeJob job = hdr->job;
    unsigned int* word = reinterpret_cast<unsigned int*>(p.seg_count) + job.e_seg;
    if (threadIdx.x == 0) {
      // every covering CTA publishes before it waits on anything, and a
      // cooperative launch makes all of them resident, so this wait ends;
      // it is bounded all the same
      const bool ok = spin_until_arrived(word, (unsigned)(job.ncov * KVC), p.wait_limit_ns);
      if (!ok) set_err(p, 4u);
      hdr->merge_ok = ok ? 1 : 0;
    }
    consumer_bar<KVC>();
    __threadfence();
    if (hdr->merge_ok) {
      const int items = kvc * G * (D / 4);
      const int k = hdr->pidx - job.c_first;
      const int i0 = (int)((int64_t)k * items / job.nmergers);
      const int i1 = (int)((int64_t)(k + 1) * items / job.nmergers);
      merge_segment<D, KVC>(p, job, i0, i1, reinterpret_cast<float*>(const_cast<uint8_t*>(stg)),
                            p.stages * p.stage_bytes / 4);
      consumer_bar<KVC>();
      if (threadIdx.x == 0) {
        const unsigned int old = atomicAdd(word, kDoneOne);
        if ((old >> 16) == (unsigned)job.nmergers - 1u) atomicExch(word, 0u);  // last merger: reset
      }
    }
  }
}

// -------------------------------------------------------------------- kernel --
// KVC consumer warps (one per kv head of the group) + 1 producer warp.  The
// CTAs per SM are chosen for about 18 warps per SM with one n-tile (96
// registers: a sub-partition holds up to 5 warps of its 16K registers) and
// about 9 with two n-tiles.
// APPEND (paged layout only): the launch also quantizes each sequence's new
// token into the cache (slmt_paged_append_decode); a separate instantiation,
// so the plain decode carries none of that code.
// SWZ (paged, whole rows, D 64/128): stages filled by the 64-byte swizzled
// tiled copy (paged mode 4) and read through the swizzle; the host reserves
// 1 KB more shared memory so the stage base can be rounded up to 1024 bytes.
template <int D, int NT, int LAYOUT, int KVC, bool PK, bool APPEND = false, bool SWZ = false>
__global__ void __launch_bounds__(cta_threads(KVC), ctas_per_sm(KVC, NT))
    decode_splitk_kernel(const __grid_constant__ DecodeParams p) {
  static_assert(!APPEND || LAYOUT == LAYOUT_PAGED, "the fused append writes the paged layout");
  extern __shared__ __align__(128) uint8_t smem[];
  SmemHeader* hdr = reinterpret_cast<SmemHeader*>(smem);
  uint8_t* qbuf = smem + kHeaderBytes;
  uint8_t* rbuf = qbuf + p.nqbuf * p.qbuf_bytes;
  uint8_t* stg = smem + p.stage_offset;
  if constexpr (SWZ) stg += (1024u - (smem_addr(stg) & 1023u)) & 1023u;
  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(&hdr->full[i], 33);  // producer lane 0 + 32 cp.async arrivals
      mbar_init(&hdr->empty[i], KVC);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&hdr->qfull[i], 1);
      mbar_init(&hdr->qempty[i], KVC);
    }
    mbar_init(&hdr->never, 1);
    mbar_init(&hdr->prologue, 1);
    mbar_init(&hdr->appended, KVC);
    hdr->has_job = 0;
    hdr->abort = 0;
    int sp = -1;
    if (p.sm_weighted) {
      unsigned smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      if ((int)smid < p.num_sms) {
        const int r = atomicAdd(p.sm_ctr + smid, 1);
        if (r < 2) sp = 2 * (int)smid + r;
      }
    }
    hdr->spiece = sp;
    hdr->pidx = (int)blockIdx.x;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x >= KVC * 32)
    decode_producer<D, LAYOUT, APPEND>(p, hdr, qbuf, rbuf, stg);
  else
    decode_consumer<D, NT, LAYOUT, KVC, PK, APPEND, SWZ>(p, hdr, qbuf, rbuf, stg);
  if (p.sm_weighted) {
    // the last CTA to finish zeroes the SM arrival words for the next launch
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const int done = atomicAdd(p.sm_ctr + p.num_sms, 1);
      if (done == (int)gridDim.x - 1)
        for (int i = 0; i <= p.num_sms; ++i) p.sm_ctr[i] = 0;
    }
  }
}

}  // namespace slmt
