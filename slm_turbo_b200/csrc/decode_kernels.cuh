// decode_kernels.cuh -- split-K 4-bit decode attention for sm_100a.
//
// One persistent CTA per (SM x resident CTAs).  The work space is the list of
// 16-token tiles of every (kv-head group, sequence) segment, concatenated; CTA
// c owns the contiguous tile range [c*T/NC, (c+1)*T/NC), so every CTA streams
// the same number of bytes whatever the length mix of the batch.
//
// Warp roles (288 threads):
//   warp 8      producer: walks its tile range, stages each tile with one
//               1-D bulk copy (TMA unit) per tile (or per row / cp.async when
//               the layout is not 16-byte aligned) into a STAGES-deep ring,
//               and stages q (+ per-channel rulers) per segment.
//   warps 0..7  consumers: warp w owns kv head w % KVC of the group and the
//               tiles with seg_tile % WPK == w / KVC.  Per 16-token tile:
//                 S^T[16 tok x 8 heads] = codes(K) . q'     (m16n8k16, fp32 acc)
//                 s = k_step*S + k_min*sum(q)               (per-token rulers)
//                 online softmax in the log2 domain (quad shuffles)
//                 P'= p*v_step -> fp16 -> movmatrix -> B operand
//                 O^T[D x 8 heads] += codes(V)^T . P'^T     (m16n8k16)
//                 sum_v += p*v_min
//               The 4-bit codes go straight from shared memory to fp16
//               registers (exact), so no dequantised K/V exists anywhere.
//   At a segment end each consumer warp writes (m, l, acc) to the split-K
//   scratch slot cta+segment; combine_kernel merges the slots.
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

__device__ __forceinline__ int64_t block_entry(const DecodeParams& p, int s,
                                               int blk) {
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

// ------------------------------------------------------------------ producer --
template <int D, int LAYOUT>
__device__ void decode_producer(const DecodeParams& p, SmemHeader* hdr,
                                uint8_t* qbuf, uint8_t* rbuf, uint8_t* stg) {
  constexpr int SLOT = D + 8;
  constexpr int HALF = D / 2;
  const int lane = threadIdx.x & 31;
  const int B = p.num_seqs;
  const int c = blockIdx.x;

  // Tiles per kv-head group; flag lengths above capacity once per grid.
  long long t_seq = 0;
  for (int base = 0; base < B; base += 32) {
    const int b = base + lane;
    int n = 0;
    if (b < B) {
      n = ntiles_of(seq_len_of(p, b));
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
    // Locate the sequence holding tile tt of group kg.
    int s = 0;
    long long ps = 0;
    for (int base = 0; base < B; base += 32) {
      const int b = base + lane;
      const int n = (b < B) ? ntiles_of(seq_len_of(p, b)) : 0;
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
    int tile = (int)(tt - ps);
    int L = seq_len_of(p, s);
    int nts = ntiles_of(L);
    bool first = true;
    int seg_tile = 0;
    uint32_t seg = 0;  // segments started by this CTA

    for (long long t = t_begin; t < t_end; ++t) {
      if (it >= (uint32_t)p.stages) {
        if (!mbar_wait(&hdr->empty[stage], phase ^ 1u, kWaitLimitNs)) {
          failed = true;
          break;
        }
      }
      const int qpar = (int)(seg & 1u);
      if (first) {
        // ---- stage q (fp16) and per-channel rulers of this segment ----
        if (seg >= 2) {
          if (!mbar_wait(&hdr->qempty[qpar], ((seg >> 1) - 1) & 1u, kWaitLimitNs)) {
            failed = true;
            break;
          }
        }
        const int hg = p.kvc * p.G;  // q heads of the group
        __half* qd = reinterpret_cast<__half*>(qbuf + qpar * p.qbuf_bytes);
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
          uint16_t* rd = reinterpret_cast<uint16_t*>(rbuf + qpar * p.rbuf_bytes);
          const uint16_t* srcs[4] = {p.r0, p.r1, p.r2, p.r3};
          for (int i = lane; i < 4 * p.kvc * D; i += 32) {
            const int a = i / (p.kvc * D), rem = i % (p.kvc * D);
            const int jj = rem / D, d = rem % D;
            const int kvh = kg * p.kvc + jj;
            uint16_t v = 0x3C00u;  // 1.0 (scale) / also used for zero when !use_quant
            if (p.use_quant)
              v = srcs[a][(int64_t)s * p.ruler_seq_stride + (int64_t)kvh * D + d];
            else
              v = (a & 1) ? (uint16_t)0 : (uint16_t)0x3C00u;
            rd[i] = v;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&hdr->qfull[qpar]);
      }

      const bool last = (tile == nts - 1) || (t == t_end - 1);
      const int nvalid = min(kTileTokens, L - tile * kTileTokens);
      uint8_t* dst = stg + (size_t)stage * p.stage_bytes;
      uint64_t* fb = &hdr->full[stage];

      // ---- plan the copies of this tile (identical on every lane) ----
      uint32_t tx = 0;
      if (LAYOUT == LAYOUT_PAGED) {
        const int bs = p.block_size;
        const int row_bytes = p.kvc * SLOT;
        const int tok0 = tile * kTileTokens;
        // rows whose page exists: pages 0 .. ceil(L/bs)-1
        const int rows_alloc = min(kTileTokens, ((L + bs - 1) / bs) * bs - tok0);
        if (p.paged_mode == 0) {
          int64_t phys = 0;
          bool ok = false;
          if (lane == 0) {
            phys = block_entry(p, s, tok0 / bs);
            ok = phys >= 0 && phys < p.num_blocks;
            if (!ok) set_err(p, 1u);
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          tx = ok ? (uint32_t)(kTileTokens * row_bytes) : 0u;
          if (lane == 0) {
            hdr->desc[stage] = TileDesc{s, kg, tile, nvalid, (first ? 1 : 0) | (last ? 2 : 0) | (qpar << 2),
                                        (int)(c + (int64_t)kg * B + s), seg_tile, 0};
          }
          __syncwarp();
          if (lane == 0) {
            mbar_arrive_expect_tx(fb, tx);
            if (ok) {
              const uint8_t* src = p.cache + ((phys * bs + (tok0 % bs)) * p.kv_total) * (int64_t)SLOT;
              bulk_g2s(dst, src, tx, fb, policy);
            }
          }
        } else {
          // one row (token) per lane 0..15
          int64_t phys = -1;
          bool ok = false;
          const int row = lane;
          if (row < rows_alloc) {
            const int tok = tok0 + row;
            phys = block_entry(p, s, tok / bs);
            ok = phys >= 0 && phys < p.num_blocks;
            if (!ok) set_err(p, 1u);
          }
          const unsigned okm = __ballot_sync(0xffffffffu, ok);
          if (lane == 0) {
            hdr->desc[stage] = TileDesc{s, kg, tile, nvalid, (first ? 1 : 0) | (last ? 2 : 0) | (qpar << 2),
                                        (int)(c + (int64_t)kg * B + s), seg_tile, 0};
          }
          if (p.paged_mode == 1) {
            tx = (uint32_t)(__popc(okm) * row_bytes);
            __syncwarp();
            if (lane == 0) mbar_arrive_expect_tx(fb, tx);
            __syncwarp();
            if (ok) {
              const int tok = tok0 + row;
              const uint8_t* src =
                  p.cache + ((phys * bs + (tok % bs)) * p.kv_total + (int64_t)kg * p.kvc) * SLOT;
              bulk_g2s(dst + row * row_bytes, src, (uint32_t)row_bytes, fb, policy);
            }
          } else {
            // cp.async, 8 bytes per op, all lanes; each op looks up its row's page
            const int cpr = row_bytes / 8;
            for (int i = lane; i < kTileTokens * cpr; i += 32) {
              const int rr = i / cpr, cc = i % cpr;
              if (!((okm >> rr) & 1u)) continue;
              const int tok = tok0 + rr;
              const int64_t ph2 = block_entry(p, s, tok / bs);
              const uint8_t* src =
                  p.cache + ((ph2 * bs + (tok % bs)) * p.kv_total + (int64_t)kg * p.kvc) * SLOT + cc * 8;
              cp_async8(dst + rr * row_bytes + cc * 8, src);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_expect_tx(fb, 0u);
          }
        }
      } else {
        // contiguous layouts: per kv head of the group, nvalid rows of K and V
        const int64_t row0 = (int64_t)s * p.kv_seq_stride_rows + (int64_t)tile * kTileTokens;
        const int bytes = nvalid * HALF;
        const bool bulk = p.contig_bulk_ok && (bytes % 16 == 0);
        if (LAYOUT == LAYOUT_PER_TOKEN) {
          // rulers: 4 fp16 per (row, kv head) in slot-tail order
          uint16_t* rd = reinterpret_cast<uint16_t*>(dst + p.kvc * kTileTokens * D);
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
          hdr->desc[stage] = TileDesc{s, kg, tile, nvalid, (first ? 1 : 0) | (last ? 2 : 0) | (qpar << 2),
                                      (int)(c + (int64_t)kg * B + s), seg_tile, 0};
        }
        tx = bulk ? (uint32_t)(2 * p.kvc * bytes) : 0u;
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(fb, tx);
        __syncwarp();
        if (bulk) {
          if (lane < 2 * p.kvc) {
            const int jj = lane >> 1, isv = lane & 1;
            const int64_t roff = (row0 + (int64_t)(kg * p.kvc + jj) * p.s_cap) * HALF;
            const uint8_t* src = (isv ? p.v_codes : p.k_codes) + roff;
            bulk_g2s(dst + jj * kTileTokens * D + isv * 8 * D, src, (uint32_t)bytes, fb, policy);
          }
        } else {
          const int cpr = bytes / 8;
          for (int i = lane; i < 2 * p.kvc * cpr; i += 32) {
            const int cp = i / cpr, cc = i % cpr;
            const int jj = cp >> 1, isv = cp & 1;
            const int64_t roff = (row0 + (int64_t)(kg * p.kvc + jj) * p.s_cap) * HALF + cc * 8;
            cp_async8(dst + jj * kTileTokens * D + isv * 8 * D + cc * 8,
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
      ++seg_tile;
      ++tile;
      if (tile == nts && t + 1 < t_end) {
        // next non-empty segment
        do {
          if (++s == B) {
            s = 0;
            ++kg;
          }
          L = seq_len_of(p, s);
          nts = ntiles_of(L);
        } while (nts == 0);
        tile = 0;
        first = true;
        seg_tile = 0;
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
template <int D, int NT, int LAYOUT>
__device__ void decode_consumer(const DecodeParams& p, SmemHeader* hdr,
                                const uint8_t* qbuf, const uint8_t* rbuf,
                                const uint8_t* stg) {
  constexpr int KS = D / 16;  // QK k-steps == PV m-tiles
  constexpr int QB = D / 8;   // K bytes per thread per row
  constexpr int VB = D / 16;  // V bytes per thread per row
  constexpr int QW = (QB + 3) / 4;
  constexpr int VW = (VB + 3) / 4;
  constexpr int SLOT = D + 8;
  constexpr int QALIGN = (QB % 8 == 0) ? 8 : 2;
  constexpr int VALIGN = (VB % 8 == 0) ? 8 : ((VB % 4 == 0) ? 4 : 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, r = lane & 3;
  const int kvc = p.kvc, G = p.G;
  const int j = warp % kvc, wsub = warp / kvc;
  const float sl2 = p.scale_log2;

  uint32_t qf[KS][NT][2];
  float qs[NT][2];
  float acc[KS][NT][4];
  float mrun[NT][2], lrun[NT][2], vrun[NT][2];

  int stage = 0;
  uint32_t phase = 0, seg = 0;

  while (true) {
    if (!mbar_wait(&hdr->full[stage], phase, kWaitLimitNs)) {
      if (lane == 0) set_err(p, 4u);
      return;
    }
    const TileDesc d = hdr->desc[stage];
    if (d.seq < 0) break;
    const int qpar = (d.flags >> 2) & 1;

    if (d.flags & 1) {
      // ---- segment start: q fragments, q sums, fresh softmax state ----
      if (!mbar_wait(&hdr->qfull[qpar], (seg >> 1) & 1u, kWaitLimitNs)) {
        if (lane == 0) set_err(p, 4u);
        return;
      }
      const __half* qb = reinterpret_cast<const __half*>(qbuf + qpar * p.qbuf_bytes) + (size_t)j * G * D;
      const __half* ksc = reinterpret_cast<const __half*>(rbuf + qpar * p.rbuf_bytes) + (size_t)j * D;
      const __half* kze = ksc + (size_t)kvc * D;
      float part[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) part[nt] = 0.f;
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
              float v = __half2float(qb[n * D + dd]);
              if (LAYOUT == LAYOUT_PER_CHANNEL) {
                if (p.use_quant) {
                  v = __half2float(__float2half_rn(v * __half2float(ksc[dd])));
                  part[nt] += v * __half2float(kze[dd]);
                }
              } else {
                part[nt] += v;
              }
              x[e] = v;
            }
          }
          qf[s][nt][0] = pack_half2(x[0], x[1]);
          qf[s][nt][1] = pack_half2(x[2], x[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float v = part[nt];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        qs[nt][0] = __shfl_sync(0xffffffffu, v, (2 * r) * 4);
        qs[nt][1] = __shfl_sync(0xffffffffu, v, (2 * r + 1) * 4);
        mrun[nt][0] = mrun[nt][1] = -INFINITY;
        lrun[nt][0] = lrun[nt][1] = 0.f;
        vrun[nt][0] = vrun[nt][1] = 0.f;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[mt][nt][i] = 0.f;
      }
    }

    if ((d.seg_tile % p.wpk) == wsub) {
      const uint8_t* st = stg + (size_t)stage * p.stage_bytes;
      const uint8_t* kb0;
      const uint8_t* kb1;
      if (LAYOUT == LAYOUT_PAGED) {
        kb0 = st + (g * kvc + j) * SLOT;
        kb1 = st + ((g + 8) * kvc + j) * SLOT;
      } else {
        kb0 = st + j * kTileTokens * D + g * (D / 2);
        kb1 = kb0 + 8 * (D / 2);
      }
      // ---- QK on raw codes ----
      uint32_t ka[QW], kb[QW];
      load_bytes<QB, QALIGN>(kb0 + r * QB, ka);
      load_bytes<QB, QALIGN>(kb1 + r * QB, kb);
      float c[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) c[nt][i] = 0.f;
#pragma unroll
      for (int u = 0; u < QW; ++u) {
        if (4 * u + 4 <= QB) {
          uint32_t a0 = codes_lo(ka[u]), a1 = codes_lo(kb[u]);
          uint32_t a2 = codes_hi(ka[u]), a3 = codes_hi(kb[u]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            mma_16816(c[nt], a0, a1, a2, a3, qf[2 * u][nt][0], qf[2 * u][nt][1]);
          const uint32_t sa = ka[u] >> 8, sb = kb[u] >> 8;
          a0 = codes_lo(sa);
          a1 = codes_lo(sb);
          a2 = codes_hi(sa);
          a3 = codes_hi(sb);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            mma_16816(c[nt], a0, a1, a2, a3, qf[2 * u + 1][nt][0], qf[2 * u + 1][nt][1]);
        } else {
          const uint32_t sa = __byte_perm(ka[u], 0u, 0x3120), sb = __byte_perm(kb[u], 0u, 0x3120);
          const uint32_t a0 = codes_lo(sa), a1 = codes_lo(sb);
          const uint32_t a2 = codes_hi(sa), a3 = codes_hi(sb);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            mma_16816(c[nt], a0, a1, a2, a3, qf[2 * u][nt][0], qf[2 * u][nt][1]);
        }
      }

      // ---- rulers of tokens g and g+8 ----
      float kst0, kmn0, vst0, vmn0, kst1, kmn1, vst1, vmn1;
      if (LAYOUT == LAYOUT_PER_CHANNEL) {
        kst0 = kst1 = 1.f;
        kmn0 = kmn1 = p.use_quant ? -1.f : 0.f;
        vst0 = vst1 = 1.f;
        vmn0 = vmn1 = 0.f;
      } else {
        const uint8_t* rr0;
        const uint8_t* rr1;
        if (LAYOUT == LAYOUT_PAGED) {
          rr0 = kb0 + D;
          rr1 = kb1 + D;
        } else {
          const uint8_t* rbase = st + kvc * kTileTokens * D;
          rr0 = rbase + (g * kvc + j) * 8;
          rr1 = rbase + ((g + 8) * kvc + j) * 8;
        }
        const uint2 w0 = *reinterpret_cast<const uint2*>(rr0);
        const uint2 w1 = *reinterpret_cast<const uint2*>(rr1);
        kmn0 = half_bits_to_float((uint16_t)(w0.x & 0xFFFFu));
        kst0 = half_bits_to_float((uint16_t)(w0.x >> 16));
        vmn0 = half_bits_to_float((uint16_t)(w0.y & 0xFFFFu));
        vst0 = half_bits_to_float((uint16_t)(w0.y >> 16));
        kmn1 = half_bits_to_float((uint16_t)(w1.x & 0xFFFFu));
        kst1 = half_bits_to_float((uint16_t)(w1.x >> 16));
        vmn1 = half_bits_to_float((uint16_t)(w1.y & 0xFFFFu));
        vst1 = half_bits_to_float((uint16_t)(w1.y >> 16));
      }
      const bool v0 = g < d.nvalid, v1 = (g + 8) < d.nvalid;

      // ---- online softmax (log2 domain) + P' fragments ----
      uint32_t pb[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float s0 = v0 ? (c[nt][0] * kst0 + kmn0 * qs[nt][0]) * sl2 : -INFINITY;
        const float s1 = v0 ? (c[nt][1] * kst0 + kmn0 * qs[nt][1]) * sl2 : -INFINITY;
        const float s2 = v1 ? (c[nt][2] * kst1 + kmn1 * qs[nt][0]) * sl2 : -INFINITY;
        const float s3 = v1 ? (c[nt][3] * kst1 + kmn1 * qs[nt][1]) * sl2 : -INFINITY;
        float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
        }
        const float mn0 = fmaxf(mrun[nt][0], mx0), mn1 = fmaxf(mrun[nt][1], mx1);
        const float al0 = exp2_approx(mrun[nt][0] - mn0);
        const float al1 = exp2_approx(mrun[nt][1] - mn1);
        mrun[nt][0] = mn0;
        mrun[nt][1] = mn1;
        const float p0 = exp2_approx(s0 - mn0), p1 = exp2_approx(s1 - mn1);
        const float p2 = exp2_approx(s2 - mn0), p3 = exp2_approx(s3 - mn1);
        lrun[nt][0] = lrun[nt][0] * al0 + p0 + p2;
        lrun[nt][1] = lrun[nt][1] * al1 + p1 + p3;
        vrun[nt][0] = vrun[nt][0] * al0 + (v0 ? p0 * vmn0 : 0.f) + (v1 ? p2 * vmn1 : 0.f);
        vrun[nt][1] = vrun[nt][1] * al1 + (v0 ? p1 * vmn0 : 0.f) + (v1 ? p3 * vmn1 : 0.f);
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          acc[mt][nt][0] *= al0;
          acc[mt][nt][1] *= al1;
          acc[mt][nt][2] *= al0;
          acc[mt][nt][3] *= al1;
        }
        const uint32_t x0 = pack_half2(v0 ? p0 * vst0 : 0.f, v0 ? p1 * vst0 : 0.f);
        const uint32_t x1 = pack_half2(v1 ? p2 * vst1 : 0.f, v1 ? p3 * vst1 : 0.f);
        pb[nt][0] = movmatrix_t(x0);
        pb[nt][1] = movmatrix_t(x1);
      }

      // ---- PV on raw codes: O^T[dims x heads] += V^T . P'^T ----
      const uint8_t* vr[4];
      const int toks[4] = {2 * r, 2 * r + 1, 2 * r + 8, 2 * r + 9};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (LAYOUT == LAYOUT_PAGED)
          vr[k] = st + (toks[k] * kvc + j) * SLOT + D / 2 + g * VB;
        else
          vr[k] = st + j * kTileTokens * D + 8 * D + toks[k] * (D / 2) + g * VB;
      }
      uint32_t va[VW], vb[VW], vc[VW], vd[VW];
      load_bytes<VB, VALIGN>(vr[0], va);
      load_bytes<VB, VALIGN>(vr[1], vb);
      load_bytes<VB, VALIGN>(vr[2], vc);
      load_bytes<VB, VALIGN>(vr[3], vd);
#pragma unroll
      for (int u = 0; u < VW; ++u) {
        const uint32_t x = __byte_perm(va[u], vb[u], 0x5410), y = __byte_perm(va[u], vb[u], 0x7632);
        const uint32_t x2 = __byte_perm(vc[u], vd[u], 0x5410), y2 = __byte_perm(vc[u], vd[u], 0x7632);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int mt = 4 * u + k;
          if (mt < KS) {
            const uint32_t w1 = (k == 0) ? x : (k == 1) ? (x >> 8) : (k == 2) ? y : (y >> 8);
            const uint32_t w2 = (k == 0) ? x2 : (k == 1) ? (x2 >> 8) : (k == 2) ? y2 : (y2 >> 8);
            const uint32_t a0 = codes_lo(w1), a1 = codes_hi(w1);
            const uint32_t a2 = codes_lo(w2), a3 = codes_hi(w2);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
              mma_16816(acc[mt][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
          }
        }
      }
    }

    __syncwarp();
    if (lane == 0) mbar_arrive(&hdr->empty[stage]);

    if (d.flags & 2) {
      // ---- segment end: finish the sums and write the split-K partial ----
      const __half* vsc = reinterpret_cast<const __half*>(rbuf + qpar * p.rbuf_bytes) + (size_t)(2 * kvc + j) * D;
      const __half* vze = vsc + (size_t)kvc * D;
      const int hg = kvc * G;
      const int64_t slotw = (int64_t)d.slot * p.wpk + wsub;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float l0 = lrun[nt][0], l1 = lrun[nt][1], u0 = vrun[nt][0], u1 = vrun[nt][1];
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
              p.part_ml[row * 2 + 0] = mrun[nt][e];
              p.part_ml[row * 2 + 1] = lsum;
            }
            float* dst = p.part_acc + row * D + 2 * g * VB;
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
              float o0 = acc[mt][nt][e] + vsum;
              float o1 = acc[mt][nt][e + 2] + vsum;
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
      __syncwarp();
      if (lane == 0) mbar_arrive(&hdr->qempty[qpar]);
      ++seg;
    }

    if (++stage == p.stages) {
      stage = 0;
      phase ^= 1u;
    }
  }
}

// -------------------------------------------------------------------- kernel --
template <int D, int NT, int LAYOUT>
__global__ void __launch_bounds__(kThreads, (NT == 1) ? 2 : 1)
    decode_splitk_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  SmemHeader* hdr = reinterpret_cast<SmemHeader*>(smem);
  uint8_t* qbuf = smem + kHeaderBytes;
  uint8_t* rbuf = qbuf + 2 * p.qbuf_bytes;
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
    decode_consumer<D, NT, LAYOUT>(p, hdr, qbuf, rbuf, stg);
}

// ------------------------------------------------------------------- combine --
// One CTA per (kv group, sequence) segment: merges the partials of every CTA
// that streamed part of it (log-sum-exp weights) and writes the output row.
template <int D>
__global__ void __launch_bounds__(256) decode_combine_kernel(
    const DecodeParams p, void* out, int out_dtype, int64_t out_seq_stride,
    int64_t out_head_stride) {
  __shared__ long long red[2][8];
  const int B = p.num_seqs;
  const int e = blockIdx.x;
  const int kg = e / B, s = e % B;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  long long pre = 0, tot = 0;
  for (int b = tid; b < B; b += blockDim.x) {
    const int n = ntiles_of(seq_len_of(p, b));
    tot += n;
    if (b < s) pre += n;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    pre += __shfl_xor_sync(0xffffffffu, pre, o);
    tot += __shfl_xor_sync(0xffffffffu, tot, o);
  }
  if (lane == 0) {
    red[0][warp] = pre;
    red[1][warp] = tot;
  }
  __syncthreads();
  pre = 0;
  tot = 0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
    pre += red[0][w];
    tot += red[1][w];
  }

  const int hg = p.kvc * p.G;
  const int n_s = ntiles_of(seq_len_of(p, s));
  const int64_t T = tot * p.ngroups;
  const int64_t P0 = (int64_t)kg * tot + pre;
  const int64_t NC = p.num_ctas;
  int64_t c_first = 0, c_last = -1;
  if (n_s > 0) {
    c_first = cta_of_tile(P0, T, NC);
    c_last = cta_of_tile(P0 + n_s - 1, T, NC);
  }
  constexpr int DPL = (D + 31) / 32;  // dims per lane
  for (int hl = warp; hl < hg; hl += (int)(blockDim.x >> 5)) {
    float M = -INFINITY;
    for (int64_t c = c_first; c <= c_last; ++c) {
      const int64_t a = cta_start(c, T, NC), b2 = cta_start(c + 1, T, NC);
      if (a >= b2 || b2 <= P0 || a >= P0 + n_s) continue;
      for (int w = 0; w < p.wpk; ++w) {
        const int64_t row = ((c + e) * p.wpk + w) * hg + hl;
        M = fmaxf(M, p.part_ml[row * 2]);
      }
    }
    float Lsum = 0.f;
    float o[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) o[i] = 0.f;
    if (M != -INFINITY) {
      for (int64_t c = c_first; c <= c_last; ++c) {
        const int64_t a = cta_start(c, T, NC), b2 = cta_start(c + 1, T, NC);
        if (a >= b2 || b2 <= P0 || a >= P0 + n_s) continue;
        for (int w = 0; w < p.wpk; ++w) {
          const int64_t row = ((c + e) * p.wpk + w) * hg + hl;
          const float wgt = exp2f(p.part_ml[row * 2] - M);
          Lsum += wgt * p.part_ml[row * 2 + 1];
#pragma unroll
          for (int i = 0; i < DPL; ++i) {
            const int dd = lane + 32 * i;
            if (dd < D) o[i] += wgt * p.part_acc[row * D + dd];
          }
        }
      }
    }
    const float inv = (Lsum > 0.f) ? 1.f / Lsum : 0.f;
    const int64_t obase = (int64_t)s * out_seq_stride + (int64_t)(kg * hg + hl) * out_head_stride;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int dd = lane + 32 * i;
      if (dd < D) {
        const float v = o[i] * inv;
        if (out_dtype == 2)
          reinterpret_cast<float*>(out)[obase + dd] = v;
        else if (out_dtype == 1)
          reinterpret_cast<__nv_bfloat16*>(out)[obase + dd] = __float2bfloat16_rn(v);
        else
          reinterpret_cast<__half*>(out)[obase + dd] = __float2half_rn(v);
      }
    }
  }
}

}  // namespace slmt
