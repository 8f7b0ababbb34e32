// decode_kernels.cuh -- split-K 4-bit decode attention for sm_100a.
//
// One persistent CTA per (SM x resident CTAs).  The work space is the list of
// 32-token chunks of every (kv-head group, sequence) segment, concatenated;
// CTA c owns the contiguous chunk range [c*T/NC, (c+1)*T/NC), so every CTA
// streams the same number of bytes whatever the length mix of the batch.
//
// Warp roles (288 threads):
//   warp 8      producer: walks its chunk range and stages each chunk with
//               1-D bulk copies (TMA unit; one per 16-token page tile, or per
//               row / cp.async when the layout is not 16-byte aligned) into a
//               STAGES-deep shared-memory ring guarded by mbarriers; stages
//               q (+ per-channel rulers) once per segment.
//   warps 0..7  consumers: warp w owns kv head w % KVC of the group and the
//               chunks with seg_chunk % WPK == w / KVC.  Per 32-token chunk
//               (two m16 tiles, independent tensor-core chains):
//                 S^T[16 tok x 8 heads] = codes(K) . q            (m16n8k16, fp32)
//                 s = k_step*S + k_min*sum(q)                      (per-token rulers)
//                 online softmax, log2 domain, lazy rescale (quad shuffles)
//                 P' = p*v_step -> fp16 -> movmatrix -> B operand
//                 O^T[D x 8 heads] += codes(V)^T . P'^T            (m16n8k16)
//                 sum_v += p*v_min
//               4-bit codes go straight from shared memory to exact fp16
//               integers in registers; no dequantised K/V exists anywhere.
//   At a segment end each consumer warp writes (m, l, acc) to the split-K
//   scratch slot cta+segment; decode_combine_kernel merges the slots.
#pragma once

#include "decode_common.cuh"
#include "ptx.cuh"

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
__device__ __forceinline__ int qk_dim(int s, int slot, int r) {
  constexpr int QB = D / 8;
  const int u = s >> 1, e = s & 1;
  const int base = r * QB + 4 * u;
  const int nib = (slot >> 1) & 1;
  int byte;
  if (4 * u + 4 <= QB)
    byte = base + e + ((slot & 1) ? 2 : 0);
  else
    byte = base + (slot & 1);
  return 2 * byte + nib;
}

// Shared-memory addresses of token row t (0..31) of kv head j in a stage.
// `base` already holds the warp's kv-head offset, so with a compile-time
// KVC every row address is base + immediate.
template <int D, int LAYOUT, int KVC>
struct StageView {
  const uint8_t* base;  // paged: st + j*(D+8); contiguous: st + j*32*D
  const uint8_t* rul;   // contiguous per-token rulers: st + kvc*32*D + j*8
  int kvc;              // runtime kv heads per stage row (used when KVC == 0)
  __device__ __forceinline__ int rs() const { return (KVC > 0 ? KVC : kvc) * (D + 8); }
  __device__ __forceinline__ const uint8_t* k(int t) const {
    if (LAYOUT == LAYOUT_PAGED) return base + t * rs();
    return base + t * (D / 2);
  }
  __device__ __forceinline__ const uint8_t* v(int t) const {
    if (LAYOUT == LAYOUT_PAGED) return base + t * rs() + D / 2;
    return base + (kChunkTokens / 2) * D + t * (D / 2);
  }
  __device__ __forceinline__ const uint8_t* rulers(int t) const {
    if (LAYOUT == LAYOUT_PAGED) return base + t * rs() + D;
    return rul + t * (KVC > 0 ? KVC : kvc) * 8;
  }
};

// ------------------------------------------------------------------ producer --
template <int D, int LAYOUT>
__device__ void decode_producer(const DecodeParams& p, SmemHeader* hdr,
                                uint8_t* qbuf, uint8_t* rbuf, uint8_t* stg) {
  constexpr int SLOT = D + 8;
  constexpr int HALF = D / 2;
  const int lane = threadIdx.x & 31;
  const int B = p.num_seqs;
  const int c = blockIdx.x;

  // Chunks per kv-head group; flag lengths above capacity once per grid.
  long long t_seq = 0;
  for (int base = 0; base < B; base += 32) {
    const int b = base + lane;
    int n = 0;
    if (b < B) {
      n = nchunks_of(seq_len_of(p, b));
      if (c == 0 && seq_len_raw(p, b) > p.len_cap) set_err(p, 8u);
    }
    t_seq += warp_sum_i(n);
  }
  const long long T = t_seq * p.ngroups;
  const long long t_begin = cta_start(c, T, p.num_ctas);
  const long long t_end = cta_start(c + 1, T, p.num_ctas);

  const uint64_t policy = l2_evict_first_policy();
  uint32_t it = 0;
  int stage = 0;
  uint32_t phase = 0;
  bool failed = false;

  if (t_begin < t_end) {
    int kg = (int)(t_begin / t_seq);
    const long long tt = t_begin - (long long)kg * t_seq;
    // Locate the sequence holding chunk tt of group kg.
    int s = 0;
    long long ps = 0;
    for (int base = 0; base < B; base += 32) {
      const int b = base + lane;
      const int n = (b < B) ? nchunks_of(seq_len_of(p, b)) : 0;
      const int incl = warp_incl_scan(n);
      const int tot = __shfl_sync(0xffffffffu, incl, 31);
      if (ps + tot > tt) {
        const unsigned m = __ballot_sync(0xffffffffu, ps + incl > tt);
        const int src = __ffs(m) - 1;
        s = base + src;
        ps += __shfl_sync(0xffffffffu, incl - n, src);
        break;
      }
      ps += tot;
    }
    int chunk = (int)(tt - ps);
    int L = seq_len_of(p, s);
    int nch = nchunks_of(L);
    bool first = true;
    int seg_chunk = 0;
    uint32_t seg = 0;   // segments started by this CTA
    int pg_base = 0;    // first tile whose page id lane 0 of pg_cache holds
    int64_t pg_cache = 0;

    for (long long t = t_begin; t < t_end; ++t) {
      if (it >= (uint32_t)p.stages) {
        if (!mbar_wait(&hdr->empty[stage], phase ^ 1u, kWaitLimitNs)) {
          failed = true;
          break;
        }
      }
      const int qb = (int)(seg % (uint32_t)p.nqbuf);
      if (first) {
        // ---- stage q (fp16) and per-channel rulers of this segment ----
        const uint32_t use = seg / (uint32_t)p.nqbuf;
        if (use >= 1) {
          if (!mbar_wait(&hdr->qempty[qb], (use - 1) & 1u, kWaitLimitNs)) {
            failed = true;
            break;
          }
        }
        const int hg = p.kvc * p.G;  // q heads of the group
        __half* qd = reinterpret_cast<__half*>(qbuf + qb * p.qbuf_bytes);
        const int64_t qrow0 = (int64_t)s * p.q_seq_stride + (int64_t)kg * hg * p.q_head_stride;
        if (p.q_vec16 && !p.q_bf16) {
          const int per_head = D / 8;
          for (int i = lane; i < hg * per_head; i += 32) {
            const int h = i / per_head, c8 = i % per_head;
            const __half* src = reinterpret_cast<const __half*>(p.q) + qrow0 +
                                (int64_t)h * p.q_head_stride + c8 * 8;
            reinterpret_cast<uint4*>(qd + h * D)[c8] = *reinterpret_cast<const uint4*>(src);
          }
        } else {
          for (int i = lane; i < hg * D; i += 32) {
            const int h = i / D, d = i % D;
            const int64_t off = qrow0 + (int64_t)h * p.q_head_stride + d;
            float v;
            if (p.q_bf16)
              v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.q)[off]);
            else
              v = __half2float(reinterpret_cast<const __half*>(p.q)[off]);
            qd[h * D + d] = __float2half_rn(v);
          }
        }
        if (LAYOUT == LAYOUT_PER_CHANNEL) {
          uint16_t* rd = reinterpret_cast<uint16_t*>(rbuf + qb * p.rbuf_bytes);
          for (int i = lane; i < 4 * p.kvc * D; i += 32) {
            const int a = i / (p.kvc * D), rem = i % (p.kvc * D);
            const int jj = rem / D, d = rem % D;
            const int kvh = kg * p.kvc + jj;
            uint16_t v;
            if (p.use_quant) {
              const uint16_t* src = (a == 0) ? p.r0 : (a == 1) ? p.r1 : (a == 2) ? p.r2 : p.r3;
              v = src[(int64_t)s * p.ruler_seq_stride + (int64_t)kvh * D + d];
            } else {
              v = (a & 1) ? (uint16_t)0 : (uint16_t)0x3C00u;  // scale 1, zero 0
            }
            rd[i] = v;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&hdr->qfull[qb]);
      }

      const bool last = (chunk == nch - 1) || (t == t_end - 1);
      const int nvalid = min(kChunkTokens, L - chunk * kChunkTokens);
      const int flags = (first ? 1 : 0) | (last ? 2 : 0) | (qb << 2);
      const int slot = (int)(c + (int64_t)kg * B + s);
      uint8_t* dst = stg + (size_t)stage * p.stage_bytes;
      uint64_t* fb = &hdr->full[stage];
      const int tok0 = chunk * kChunkTokens;

      if (LAYOUT == LAYOUT_PAGED) {
        const int bs = p.block_size;
        const int row_bytes = p.kvc * SLOT;
        if (p.paged_mode == 0) {
          // tiles 2*chunk, 2*chunk+1; page ids of 32 tiles per warp load
          const int t0 = 2 * chunk;
          const int ntile = (L + kTileTokens - 1) / kTileTokens;
          if (first || t0 + 1 - pg_base >= 32) {
            pg_base = t0;
            const int pt = t0 + lane;
            pg_cache = (pt < ntile) ? block_entry(p, s, (pt * kTileTokens) / bs) : 0;
          }
          const int64_t ph0 = __shfl_sync(0xffffffffu, pg_cache, t0 - pg_base);
          const int64_t ph1 = __shfl_sync(0xffffffffu, pg_cache, t0 + 1 - pg_base);
          const bool has1 = t0 + 1 < ntile;
          const bool ok0 = ph0 >= 0 && ph0 < p.num_blocks;
          const bool ok1 = has1 && ph1 >= 0 && ph1 < p.num_blocks;
          if (lane == 0 && (!ok0 || (has1 && !ok1))) set_err(p, 1u);
          const uint32_t tile_bytes = (uint32_t)(kTileTokens * row_bytes);
          const uint32_t tx = (ok0 ? tile_bytes : 0u) + (ok1 ? tile_bytes : 0u);
          if (lane == 0) {
            hdr->desc[stage] = ChunkDesc{s, kg, chunk, nvalid, flags, slot, seg_chunk, 0};
          }
          __syncwarp();
          if (lane == 0) {
            mbar_arrive_expect_tx(fb, tx);
            if (ok0) {
              const int tok = tok0;
              bulk_g2s(dst, p.cache + ((ph0 * bs + tok % bs) * p.kv_total) * (int64_t)SLOT, tile_bytes, fb,
                       policy);
            }
            if (ok1) {
              const int tok = tok0 + kTileTokens;
              bulk_g2s(dst + tile_bytes, p.cache + ((ph1 * bs + tok % bs) * p.kv_total) * (int64_t)SLOT,
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
            hdr->desc[stage] = ChunkDesc{s, kg, chunk, nvalid, flags, slot, seg_chunk, 0};
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
          hdr->desc[stage] = ChunkDesc{s, kg, chunk, nvalid, flags, slot, seg_chunk, 0};
        }
        const uint32_t tx = bulk ? (uint32_t)(2 * p.kvc * bytes) : 0u;
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(fb, tx);
        __syncwarp();
        if (bulk) {
          if (lane < 2 * p.kvc) {
            const int jj = lane >> 1, isv = lane & 1;
            const int64_t roff = (row0 + (int64_t)(kg * p.kvc + jj) * p.s_cap) * HALF;
            const uint8_t* src = (isv ? p.v_codes : p.k_codes) + roff;
            bulk_g2s(dst + jj * kChunkTokens * D + isv * (kChunkTokens / 2) * D, src, (uint32_t)bytes, fb,
                     policy);
          }
        } else {
          const int cpr = bytes / 8;
          for (int i = lane; i < 2 * p.kvc * cpr; i += 32) {
            const int cp = i / cpr, cc = i % cpr;
            const int jj = cp >> 1, isv = cp & 1;
            const int64_t roff = (row0 + (int64_t)(kg * p.kvc + jj) * p.s_cap) * HALF + cc * 8;
            cp_async8(dst + jj * kChunkTokens * D + isv * (kChunkTokens / 2) * D + cc * 8,
                      (isv ? p.v_codes : p.k_codes) + roff);
          }
        }
      }
      cp_async_arrive_noinc(fb);

      ++it;
      if (++stage == p.stages) {
        stage = 0;
        phase ^= 1u;
      }
      first = false;
      ++seg_chunk;
      ++chunk;
      if (chunk == nch && t + 1 < t_end) {
        // next non-empty segment
        do {
          if (++s == B) {
            s = 0;
            ++kg;
          }
          L = seq_len_of(p, s);
          nch = nchunks_of(L);
        } while (nch == 0);
        chunk = 0;
        first = true;
        seg_chunk = 0;
        ++seg;
      }
    }
  }

  if (!failed) {
    // terminal descriptor
    if (it >= (uint32_t)p.stages) {
      if (!mbar_wait(&hdr->empty[stage], phase ^ 1u, kWaitLimitNs)) failed = true;
    }
    if (!failed) {
      if (lane == 0) hdr->desc[stage].seq = -1;
      __syncwarp();
      if (lane == 0) mbar_arrive(&hdr->full[stage]);
      cp_async_arrive_noinc(&hdr->full[stage]);
      return;
    }
  }
  // failure: flag it and wait (bounded) for the copies this warp issued
  if (lane == 0) set_err(p, 4u);
  const uint32_t n = it < (uint32_t)p.stages ? it : (uint32_t)p.stages;
  for (uint32_t k = 0; k < n; ++k) {
    const uint32_t i = it - 1 - k;
    const int st = (int)(i % (uint32_t)p.stages);
    const uint32_t ph = (i / (uint32_t)p.stages) & 1u;
    mbar_wait(&hdr->full[st], ph, kDrainLimitNs);
  }
}

// ------------------------------------------------------------------ consumer --
// K codes enter QK with the magic-number bias left in: the low nibble as
// fp16 1024+c, the high nibble as 64+c (exponent 0x54, nibble in mantissa
// bits 4..7).  sum_d q_d*(bias_d + c_d) = q.c + sum_d q_d*bias_d, and the
// second term (one number per head) starts the accumulator negated, so the
// tensor core returns q.c directly and no f16x2 subtract is spent per code.
__device__ __forceinline__ uint32_t kcodes_lo(uint32_t w) { return lop_and_or(w, 0x000F000Fu, 0x64006400u); }
__device__ __forceinline__ uint32_t kcodes_hi(uint32_t w) { return lop_and_or(w, 0x00F000F0u, 0x54005400u); }

// Per-thread state of one consumer warp (head columns 2r, 2r+1 of each
// 8-head n-tile; output rows = head dims 2*(g*D/16 + mt) + {0, 1}).
template <int D, int NT>
struct WarpState {
  static constexpr int KS = D / 16;
  uint4 qf[NT][(D / 8 + 3) / 4];  // q B-fragments: k-steps 2u (x, y) and 2u+1 (z, w)
  float qs[NT][2];         // log2e*scale * (sum q (per-token) | sum q'*zero (per-channel))
  float qb[NT][2];         // QK accumulator bias: sum_d q_d * (1024 | 64)
  float acc[KS][NT][4];
  float m[NT][2], l[NT][2], vs[NT][2];
};

template <int D, int NT, int LAYOUT, int KVC, bool MASK>
__device__ __forceinline__ void consume_chunk(const DecodeParams& p, WarpState<D, NT>& w,
                                              const StageView<D, LAYOUT, KVC>& sv, int nvalid,
                                              uint64_t* empty_bar) {
  constexpr int KS = D / 16;  // QK k-steps == PV m-tiles
  constexpr int QB = D / 8;   // K bytes per thread per row
  constexpr int VB = D / 16;  // V bytes per thread per row
  constexpr int QW = (QB + 3) / 4;
  constexpr int VW = (VB + 3) / 4;
  constexpr int QALIGN = (QB % 8 == 0) ? 8 : 2;
  constexpr int VALIGN = (VB % 8 == 0) ? 8 : ((VB % 4 == 0) ? 4 : 1);
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, r = lane & 3;

  // ---- QK on biased codes, tile by tile; even/odd k-steps in two chains ----
  float sacc[2][NT][4];
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    float c[NT][4], c2[NT][4];
    asm volatile("" ::: "memory");  // keep the two tiles' loads from being hoisted together
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      c[nt][0] = c[nt][2] = -w.qb[nt][0];
      c[nt][1] = c[nt][3] = -w.qb[nt][1];
#pragma unroll
      for (int i = 0; i < 4; ++i) c2[nt][i] = 0.f;
    }
    uint32_t ka[QW], kb[QW];
    load_bytes<QB, QALIGN>(sv.k(16 * a + g) + r * QB, ka);
    load_bytes<QB, QALIGN>(sv.k(16 * a + g + 8) + r * QB, kb);
#pragma unroll
    for (int u = 0; u < QW; ++u) {
      uint4 qf[NT];  // B-fragments of k-steps 2u (x, y) and 2u+1 (z, w)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) qf[nt] = w.qf[nt][u];
      if (4 * u + 4 <= QB) {
        uint32_t a0 = kcodes_lo(ka[u]), a1 = kcodes_lo(kb[u]);
        uint32_t a2 = kcodes_hi(ka[u]), a3 = kcodes_hi(kb[u]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816(c[nt], a0, a1, a2, a3, qf[nt].x, qf[nt].y);
        const uint32_t sa = ka[u] >> 8, sb = kb[u] >> 8;
        a0 = kcodes_lo(sa);
        a1 = kcodes_lo(sb);
        a2 = kcodes_hi(sa);
        a3 = kcodes_hi(sb);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816(c2[nt], a0, a1, a2, a3, qf[nt].z, qf[nt].w);
      } else {
        const uint32_t sa = __byte_perm(ka[u], 0u, 0x3120), sb = __byte_perm(kb[u], 0u, 0x3120);
        const uint32_t a0 = kcodes_lo(sa), a1 = kcodes_lo(sb);
        const uint32_t a2 = kcodes_hi(sa), a3 = kcodes_hi(sb);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816(c[nt], a0, a1, a2, a3, qf[nt].x, qf[nt].y);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) sacc[a][nt][i] = c[nt][i] + c2[nt][i];
  }

  // ---- per-token rulers (k_min, k_step | v_min, v_step) are read from shared
  // memory where they are used, to keep registers free ----
  auto ruler_k = [&](int a, int h) -> float2 {
    if (LAYOUT == LAYOUT_PER_CHANNEL) return make_float2(p.use_quant ? -1.f : 0.f, 1.f);
    return __half22float2(*reinterpret_cast<const __half2*>(sv.rulers(16 * a + g + 8 * h)));
  };
  auto ruler_v = [&](int a, int h) -> float2 {
    if (LAYOUT == LAYOUT_PER_CHANNEL) return make_float2(0.f, 1.f);
    return __half22float2(*reinterpret_cast<const __half2*>(sv.rulers(16 * a + g + 8 * h) + 4));
  };
  bool val[2][2];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int h = 0; h < 2; ++h) val[a][h] = !MASK || (16 * a + g + 8 * h) < nvalid;

  // ---- scores + online softmax (log2 domain, lazy rescale) ----
  const float sl2 = p.scale_log2;
  float sc[2][NT][4];
  float mx[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) mx[nt][0] = mx[nt][1] = -INFINITY;
#pragma unroll
  for (int a = 0; a < 2; ++a) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float2 kr = ruler_k(a, h);
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
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx[nt][0] = fmaxf(mx[nt][0], __shfl_xor_sync(0xffffffffu, mx[nt][0], o));
      mx[nt][1] = fmaxf(mx[nt][1], __shfl_xor_sync(0xffffffffu, mx[nt][1], o));
    }
  }
  bool need = false;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
    need |= (mx[nt][0] > w.m[nt][0] + kRescaleSlack) || (mx[nt][1] > w.m[nt][1] + kRescaleSlack);
  if (__any_sync(0xffffffffu, need)) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float mn = fmaxf(w.m[nt][e], mx[nt][e]);
        const float al = exp2_approx(w.m[nt][e] - mn);
        w.m[nt][e] = mn;
        w.l[nt][e] *= al;
        w.vs[nt][e] *= al;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          w.acc[mt][nt][e] *= al;
          w.acc[mt][nt][e + 2] *= al;
        }
      }
    }
  }

  uint32_t pb[2][NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      float pp[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int h = i >> 1, e = i & 1;
        const float2 vr = ruler_v(a, h);
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

  // ---- PV on raw codes: O^T[dims x heads] += V^T . P'^T, one k-step per tile ----
  // thread (g, r) needs tokens 16a + {2r, 2r+1, 2r+8, 2r+9}, bytes [g*VB, +VB)
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    uint32_t vw[4][VW];
    load_bytes<VB, VALIGN>(sv.v(16 * a + 2 * r) + g * VB, vw[0]);
    load_bytes<VB, VALIGN>(sv.v(16 * a + 2 * r + 1) + g * VB, vw[1]);
    load_bytes<VB, VALIGN>(sv.v(16 * a + 2 * r + 8) + g * VB, vw[2]);
    load_bytes<VB, VALIGN>(sv.v(16 * a + 2 * r + 9) + g * VB, vw[3]);
    if (a == 1) {  // every shared-memory read of the stage is done: release it
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
          const uint32_t a0 = codes_lo(w1), a1 = codes_hi(w1);
          const uint32_t a2 = codes_lo(w2), a3 = codes_hi(w2);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_16816(w.acc[mt][nt], a0, a1, a2, a3, pb[a][nt][0], pb[a][nt][1]);
        }
      }
    }
  }
}

template <int D, int NT, int LAYOUT, int KVC>
__device__ void decode_consumer(const DecodeParams& p, SmemHeader* hdr,
                                const uint8_t* qbuf, const uint8_t* rbuf,
                                const uint8_t* stg) {
  constexpr int KS = D / 16;
  constexpr int VB = D / 16;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, r = lane & 3;
  const int kvc = KVC > 0 ? KVC : p.kvc, G = p.G;
  const int j = warp & (kvc - 1), wsub = warp / kvc;  // kvc and wpk are powers of two
  const int wmask = p.wpk - 1;

  WarpState<D, NT> w;
  int stage = 0;
  uint32_t phase = 0, seg = 0;

  while (true) {
    if (!mbar_wait(&hdr->full[stage], phase, kWaitLimitNs)) {
      if (lane == 0) set_err(p, 4u);
      return;
    }
    const ChunkDesc& dsm = hdr->desc[stage];
    if (dsm.seq < 0) break;
    // fields needed after the stage is released are copied to registers
    const int flags = dsm.flags, slot = dsm.slot, nvalid = dsm.nvalid, seg_chunk = dsm.seg_chunk;
    const int qbi = flags >> 2;

    if (flags & 1) {
      // ---- segment start: q fragments, q sums, fresh softmax state ----
      if (!mbar_wait(&hdr->qfull[qbi], (seg / (uint32_t)p.nqbuf) & 1u, kWaitLimitNs)) {
        if (lane == 0) set_err(p, 4u);
        return;
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
          const int n = nt * 8 + g;
          float x[4] = {0.f, 0.f, 0.f, 0.f};
          if (n < G) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int dd = qk_dim<D>(s, e, r);
              float v = __half2float(qh[n * D + dd]);
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
        w.m[nt][0] = w.m[nt][1] = -INFINITY;
        w.l[nt][0] = w.l[nt][1] = 0.f;
        w.vs[nt][0] = w.vs[nt][1] = 0.f;
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

    if ((seg_chunk & wmask) == wsub) {
      const uint8_t* st = stg + (size_t)stage * p.stage_bytes;
      StageView<D, LAYOUT, KVC> sv;
      sv.kvc = kvc;
      if (LAYOUT == LAYOUT_PAGED) {
        sv.base = st + j * (D + 8);
        sv.rul = nullptr;
      } else {
        sv.base = st + j * kChunkTokens * D;
        sv.rul = st + kvc * kChunkTokens * D + j * 8;
      }
      if (nvalid == kChunkTokens)
        consume_chunk<D, NT, LAYOUT, KVC, false>(p, w, sv, nvalid, &hdr->empty[stage]);
      else
        consume_chunk<D, NT, LAYOUT, KVC, true>(p, w, sv, nvalid, &hdr->empty[stage]);
    } else {
      __syncwarp();
      if (lane == 0) mbar_arrive(&hdr->empty[stage]);
    }

    if (flags & 2) {
      // ---- segment end: finish the sums and write the split-K partial ----
      const __half* vsc = reinterpret_cast<const __half*>(rbuf + qbi * p.rbuf_bytes) + (size_t)(2 * kvc + j) * D;
      const __half* vze = vsc + (size_t)kvc * D;
      const int hg = kvc * G;
      const int64_t slotw = (int64_t)slot * p.wpk + wsub;
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
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int n = nt * 8 + 2 * r + e;
          const float lsum = e ? l1 : l0;
          const float vsum = e ? u1 : u0;
          if (n < G) {
            const int64_t row = slotw * hg + (int64_t)j * G + n;
            if (g == 0) {
              p.part_ml[row * 2 + 0] = w.m[nt][e];
              p.part_ml[row * 2 + 1] = lsum;
            }
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
              reinterpret_cast<float2*>(dst)[mt] = make_float2(o0, o1);
            }
          }
        }
      }
      if (LAYOUT == LAYOUT_PER_CHANNEL) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&hdr->qempty[qbi]);
      }
      ++seg;
    }

    if (++stage == p.stages) {
      stage = 0;
      phase ^= 1u;
    }
  }
}

// -------------------------------------------------------------------- kernel --
// One n-tile: two CTAs (18 warps) per SM, which caps registers at 96 (a
// sub-partition holds up to 5 warps of its 16K registers); two n-tiles run one
// CTA per SM.
template <int D, int NT, int LAYOUT, int KVC>
__global__ void __launch_bounds__(kThreads, (NT == 1) ? 2 : 1)
    decode_splitk_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  SmemHeader* hdr = reinterpret_cast<SmemHeader*>(smem);
  uint8_t* qbuf = smem + kHeaderBytes;
  uint8_t* rbuf = qbuf + p.nqbuf * p.qbuf_bytes;
  uint8_t* stg = smem + p.stage_offset;
  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(&hdr->full[i], 33);  // producer lane 0 + 32 cp.async arrivals
      mbar_init(&hdr->empty[i], kConsumerWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&hdr->qfull[i], 1);
      mbar_init(&hdr->qempty[i], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x >= kConsumerWarps * 32)
    decode_producer<D, LAYOUT>(p, hdr, qbuf, rbuf, stg);
  else
    decode_consumer<D, NT, LAYOUT, KVC>(p, hdr, qbuf, rbuf, stg);
}

// ------------------------------------------------------------------- combine --
// One warp per (segment, q head): lanes load the (m, l) of up to 32 partials
// at once, reduce the log-sum-exp weights with shuffles, then accumulate the
// weighted partial rows (each lane owns D/32 dims) and write the output row.
template <int D>
__global__ void __launch_bounds__(256) decode_combine_kernel(
    const DecodeParams p, void* out, int out_dtype, int64_t out_seq_stride,
    int64_t out_head_stride) {
  const int B = p.num_seqs;
  const int hg = p.kvc * p.G;
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nsegs = (int64_t)p.ngroups * B;
  if (gw >= nsegs * hg) return;
  const int e = (int)(gw / hg), hl = (int)(gw % hg);
  const int kg = e / B, s = e % B;

  long long pre = 0, tot = 0;
  for (int b = lane; b < B; b += 32) {
    const int n = nchunks_of(seq_len_of(p, b));
    tot += n;
    if (b < s) pre += n;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    pre += __shfl_xor_sync(0xffffffffu, pre, o);
    tot += __shfl_xor_sync(0xffffffffu, tot, o);
  }
  const int n_s = nchunks_of(seq_len_of(p, s));
  const int64_t T = tot * p.ngroups;
  const int64_t P0 = (int64_t)kg * tot + pre;
  const int64_t NC = p.num_ctas;

  constexpr int DPL = (D + 31) / 32;  // dims per lane
  float o[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) o[i] = 0.f;
  float Lsum = 0.f;
  if (n_s > 0) {
    const int64_t c_first = cta_of_unit(P0, T, NC);
    const int64_t c_last = cta_of_unit(P0 + n_s - 1, T, NC);
    const int np = (int)(c_last - c_first + 1) * p.wpk;
    // pass 1: running max over all partials, 32 at a time
    float M = -INFINITY;
    for (int i0 = 0; i0 < np; i0 += 32) {
      const int i = i0 + lane;
      float m = -INFINITY;
      if (i < np) {
        const int64_t c = c_first + i / p.wpk;
        const int64_t a = cta_start(c, T, NC), b2 = cta_start(c + 1, T, NC);
        if (a < b2 && b2 > P0 && a < P0 + n_s) {
          const int64_t row = ((c + e) * p.wpk + i % p.wpk) * hg + hl;
          m = p.part_ml[row * 2];
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      M = fmaxf(M, m);
    }
    // pass 2: weights and weighted rows
    if (M != -INFINITY) {
      for (int i0 = 0; i0 < np; i0 += 32) {
        const int i = i0 + lane;
        float wgt = 0.f, lw = 0.f;
        int64_t row = -1;
        if (i < np) {
          const int64_t c = c_first + i / p.wpk;
          const int64_t a = cta_start(c, T, NC), b2 = cta_start(c + 1, T, NC);
          if (a < b2 && b2 > P0 && a < P0 + n_s) {
            row = ((c + e) * p.wpk + i % p.wpk) * hg + hl;
            wgt = exp2f(p.part_ml[row * 2] - M);
            lw = wgt * p.part_ml[row * 2 + 1];
          }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, off);
        Lsum += lw;
        const int cnt = min(32, np - i0);
        for (int k = 0; k < cnt; ++k) {
          const float wk = __shfl_sync(0xffffffffu, wgt, k);
          const int64_t rk = __shfl_sync(0xffffffffu, row, k);
          if (rk >= 0) {
            const float* src = p.part_acc + rk * D;
#pragma unroll
            for (int dd = 0; dd < DPL; ++dd) {
              const int d = lane + 32 * dd;
              if (d < D) o[dd] += wk * src[d];
            }
          }
        }
      }
    }
  }
  const float inv = (Lsum > 0.f) ? 1.f / Lsum : 0.f;
  const int64_t obase = (int64_t)s * out_seq_stride + (int64_t)(kg * hg + hl) * out_head_stride;
#pragma unroll
  for (int dd = 0; dd < DPL; ++dd) {
    const int d = lane + 32 * dd;
    if (d < D) {
      const float v = o[dd] * inv;
      if (out_dtype == 2)
        reinterpret_cast<float*>(out)[obase + d] = v;
      else if (out_dtype == 1)
        reinterpret_cast<__nv_bfloat16*>(out)[obase + d] = __float2bfloat16_rn(v);
      else
        reinterpret_cast<__half*>(out)[obase + d] = __float2half_rn(v);
    }
  }
}

}  // namespace slmt
