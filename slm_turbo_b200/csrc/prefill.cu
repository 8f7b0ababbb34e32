// prefill.cu -- M-tiled prefill attention over the packed 4-bit caches.
//
// Two layouts, one kernel template:
//   PF_PER_CHANNEL  the kv_dequant_prefill_attention entry (ref
//                   kernels/kv_dequant_kernels.cuh:293-502): codes [KV, S, D/2],
//                   per-(kv head, dim) rulers, k = (c - zero) * scale; row m of
//                   M attends to keys [0, causal ? min(S, m+1) : S).
//   PF_PAGED        query chunks of requests whose keys live in the paged
//                   per-token cache [NB, bs, KV, D+8] (codes, then k_min,
//                   k_step, v_min, v_step fp16; ref .cuh:671-801 reads the same
//                   slots), k = c * step + min; request r owns query rows
//                   [qsl[r], qsl[r+1]) at the last positions of its seq_lens[r]
//                   keys, so row i attends to keys [0, S - n + i + 1): a
//                   continuation chunk of a prompt over its cached prefix
//                   (chunked prefill, prefix caching).
//
// One CTA = 4 warps per query head x 64 query rows, for one or two query
// heads of a kv group (warp w owns rows m0+16(w%4) .. +15 of head w/4).  The CTA walks the keys in chunks of 64 tokens:
//   1. the chunk's packed K and V codes (and, paged, token rulers) arrive in
//      a raw shared-memory buffer by 8-byte cp.async, issued while the
//      previous chunk is dequantized and computed (the paged layout resolves
//      the slot rows through the block table one chunk further ahead); all
//      128 threads then dequantize them ONCE for all 64 rows into shared
//      memory as fp16 (rows padded to D+8 halves so ldmatrix rows fall in
//      distinct banks);
//   2. each warp: S[16 x 64] = Q K^T on the tensor core (m16n8k16, fp32
//      accumulation; Q A-fragments held in registers for the whole CTA, K
//      B-fragments by ldmatrix), causal / length mask, online softmax in the
//      log2 domain (rows g and g+8 of the fragment, quad shuffles),
//      O[16 x D] += P V with P taken straight from the score accumulators as
//      A-fragments and V B-fragments by ldmatrix.trans.
// K/V are read once per 64 query rows instead of once per row.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>
#include <type_traits>

#include "internal.h"
#include "ptx.cuh"

namespace slmt {

enum { PF_PER_CHANNEL = 0, PF_PAGED = 1 };

struct PrefillParams {
  const void* q;  // row m (absolute), head h at q + m*q_row_stride + h*q_head_stride
  int64_t q_head_stride, q_row_stride;
  int q_bf16;
  // PF_PER_CHANNEL
  const uint8_t* k_codes;  // [KV, S, D/2]
  const uint8_t* v_codes;
  const uint16_t* k_scale;  // [KV, D] fp16 bits
  const uint16_t* k_zero;
  const uint16_t* v_scale;
  const uint16_t* v_zero;
  int use_quant;  // 0: codes are the values (reference use_quant=False)
  int S, M;       // keys and query rows (per-channel: one problem)
  // PF_PAGED
  const uint8_t* cache;  // [num_blocks, block_size, KV, D+8]
  int64_t num_blocks;
  int block_size;
  const void* block_tables;
  int bt_i64;
  int64_t bt_seq_stride;
  int64_t len_cap;                 // max_blocks_per_seq * block_size
  const int32_t* query_start_loc;  // [R+1]
  const int32_t* seq_lens;         // [R]
  int32_t* err;
  // both
  int H, KV, G, causal;
  float scale_log2;
  void* out;  // row m, head h at out + m*out_row_stride + h*out_head_stride
  int out_dtype;  // 0 f16, 1 bf16, 2 f32
  int64_t out_head_stride, out_row_stride;
};

constexpr int kPfRows = 64;    // query rows per CTA
constexpr int kPfTokens = 64;  // key tokens per chunk

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_addr(p)));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_addr(p)));
}

__device__ __forceinline__ void store_elem(const PrefillParams& p, int64_t off, float v) {
  if (p.out_dtype == 2)
    reinterpret_cast<float*>(p.out)[off] = v;
  else if (p.out_dtype == 1)
    reinterpret_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<__half*>(p.out)[off] = __float2half_rn(v);
}

__device__ __forceinline__ void pf_set_err(const PrefillParams& p, uint32_t bit) {
  if (p.err) atomicOr(reinterpret_cast<unsigned int*>(p.err), bit);
}

// Paged layout: byte offset of token t's slot row of kv head kvh, or -1 when
// the block-table entry is outside the pool (flagged, the token reads as 0).
__device__ __forceinline__ int64_t pf_slot_row(const PrefillParams& p, int req, int t, int kvh, int D) {
  const int blk = t / p.block_size;
  const int64_t e = (int64_t)req * p.bt_seq_stride + blk;
  const int64_t ph = p.bt_i64 ? reinterpret_cast<const int64_t*>(p.block_tables)[e]
                              : (int64_t) reinterpret_cast<const int32_t*>(p.block_tables)[e];
  if (ph < 0 || ph >= p.num_blocks) {
    pf_set_err(p, SLMT_DEVERR_BLOCK_ID);
    return -1;
  }
  return ((ph * p.block_size + t % p.block_size) * p.KV + kvh) * (int64_t)(D + 8);
}

// Shared memory of one CTA (dynamic): the dequantized chunk (K and V rows
// padded to D+8 halves) and two raw-code buffers, chunk c+1 arriving by
// cp.async while chunk c is dequantized and computed.  A raw buffer holds
// the chunk's K codes [64][D/2], V codes [64][D/2] and, paged, the token
// rulers [64][8] (k_min, k_step, v_min, v_step).
template <int D, int LAYOUT>
constexpr int pf_raw_bytes() {
  return 2 * kPfTokens * (D / 2) + (LAYOUT == PF_PAGED ? kPfTokens * 8 : 0);
}
template <int D, int LAYOUT>
constexpr int pf_smem_bytes() {
  return 2 * kPfTokens * (D + 8) * 2 + 2 * pf_raw_bytes<D, LAYOUT>();
}

__device__ __forceinline__ void pf_cp_async8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}

// HPC query heads of one kv group per CTA (4 warps each, rows m0.. m0+63):
// the dequantized chunk is shared by all of them.
template <int D, int LAYOUT, int HPC>
__global__ void __launch_bounds__(128 * HPC, (D <= 80 && HPC == 2) ? 2 : 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
  constexpr int NTHR = 128 * HPC;
  constexpr int KS = D / 16;   // k-steps of QK
  constexpr int NTO = D / 8;   // n-tiles of O
  constexpr int LD = D + 8;    // smem row stride in halves (odd multiple of 16 bytes)
  constexpr int NTS = kPfTokens / 8;  // n-tiles of S per chunk
  constexpr int WPR = D / 8;          // 4-byte code words per token row
  constexpr int WORDS = kPfTokens * WPR;
  constexpr int PPR = D / 16;         // 8-byte pieces per token row of K (or V)
  constexpr int RAW = pf_raw_bytes<D, LAYOUT>();
  extern __shared__ __align__(16) uint8_t pf_smem[];
  __half* ksh = reinterpret_cast<__half*>(pf_smem);
  __half* vsh = ksh + kPfTokens * LD;
  uint8_t* raw = reinterpret_cast<uint8_t*>(vsh + kPfTokens * LD);  // [2][RAW]
  __shared__ __align__(16) __half rul[4][D];  // per-channel: k scale, k zero, v scale, v zero
  __shared__ int64_t slot_off[2][kPfTokens];  // paged: slot row of each chunk token (-1: none)

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, r = lane & 3;
  const int h = blockIdx.y * HPC + (warp >> 2), kvh = h / p.G;  // HPC divides G: one kv head per CTA
  const int m0 = blockIdx.x * kPfRows;

  // ---- this CTA's problem: rows [row0, row0+M), keys [0, S), row i
  // attends to keys below min(S, off + i + 1) when causal ----
  int row0 = 0, M = p.M, S = p.S, off = 0;
  const int req = blockIdx.z;
  if (LAYOUT == PF_PAGED) {
    row0 = p.query_start_loc[req];
    M = max(p.query_start_loc[req + 1] - row0, 0);
    const int sraw = p.seq_lens[req];
    if (sraw <= 0) return;  // a request without keys is skipped: its rows are left as they are
    S = (int)min((int64_t)sraw, p.len_cap);
    if (tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) {
      if ((int64_t)sraw > p.len_cap) pf_set_err(p, SLMT_DEVERR_SEQ_LEN);
      if (M > (int)gridDim.x * kPfRows) pf_set_err(p, SLMT_DEVERR_SEQ_LEN);  // rows past max_query_len
    }
    off = S - M;
  }
  if (m0 >= M) return;  // whole CTA: no row of this tile exists
  const int mw = m0 + (warp & 3) * 16;  // this warp's first row (relative)

  if (LAYOUT == PF_PER_CHANNEL && p.use_quant && S > 0) {  // rulers unused (and may be NULL) otherwise
    for (int i = tid; i < 4 * D; i += NTHR) {
      const uint16_t* src = (i < D) ? p.k_scale : (i < 2 * D) ? p.k_zero : (i < 3 * D) ? p.v_scale : p.v_zero;
      reinterpret_cast<uint16_t*>(&rul[0][0])[i] = src[(int64_t)kvh * D + (i % D)];
    }
  }
  // Per-channel rulers are folded out of the chunk: the chunk holds the raw
  // codes as exact fp16, the key scale is multiplied into q (the key zero
  // adds the same term to every score of a row, which the softmax drops),
  // and the value scale and zero are applied once to the normalised output.
  constexpr bool kPC = (LAYOUT == PF_PER_CHANNEL);
  const bool pcq = kPC && p.use_quant && S > 0;
  if (kPC) __syncthreads();  // rul is read by the q load below

  // ---- Q A-fragments of rows mw+g and mw+g+8 (zeros past M) ----
  uint32_t qa[KS][4];
  {
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = mw + g + ((i & 1) ? 8 : 0);
        const int col = 16 * ks + 2 * r + ((i & 2) ? 8 : 0);
        uint32_t w = 0u;
        if (row < M) {
          const int64_t qo = (int64_t)(row0 + row) * p.q_row_stride + (int64_t)h * p.q_head_stride + col;
          if (kPC && pcq) {  // fp16(q * key scale)
            float2 qf;
            if (p.q_bf16) {
              const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(p.q) + qo;
              qf = make_float2(__bfloat162float(qb[0]), __bfloat162float(qb[1]));
            } else {
              qf = __half22float2(*reinterpret_cast<const __half2*>(reinterpret_cast<const __half*>(p.q) + qo));
            }
            const float2 sc = __half22float2(*reinterpret_cast<const __half2*>(&rul[0][col]));
            const __half2 hv = __floats2half2_rn(qf.x * sc.x, qf.y * sc.y);
            w = *reinterpret_cast<const uint32_t*>(&hv);
          } else if (p.q_bf16) {
            const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(p.q) + qo;
            const __half2 hv = __floats2half2_rn(__bfloat162float(qb[0]), __bfloat162float(qb[1]));
            w = *reinterpret_cast<const uint32_t*>(&hv);
          } else {
            const uint16_t* qh = reinterpret_cast<const uint16_t*>(p.q) + qo;
            w = (uint32_t)qh[0] | ((uint32_t)qh[1] << 16);
          }
        }
        qa[ks][i] = w;
      }
    }
  }

  float o[NTO][4];
#pragma unroll
  for (int n = 0; n < NTO; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

  const int row_last = min(M, m0 + kPfRows) - 1;  // last row of this CTA
  const int kend = p.causal ? max(0, min(S, off + row_last + 1)) : S;
  const int64_t kvbase = (int64_t)kvh * S * (D / 2);  // per-channel codes of this kv head

  // paged: resolve a chunk's slot rows through the block table (threads 0..63)
  auto prep = [&](int t0, int buf) {
    if (LAYOUT == PF_PAGED && tid < kPfTokens) {
      const int t = t0 + tid;
      slot_off[buf][tid] = (t < S) ? pf_slot_row(p, req, t, kvh, D) : -1;
    }
  };
  // start the copies of chunk t0 into raw buffer `rb` (8-byte pieces; a
  // token that does not exist or whose page is bad is written as zeros)
  auto issue = [&](int t0, int rb) {
    uint8_t* dst = raw + rb * RAW;
    const uint32_t d0 = smem_addr(dst);
    constexpr int NPC = 2 * kPfTokens * PPR + (LAYOUT == PF_PAGED ? kPfTokens : 0);
    for (int i = tid; i < NPC; i += NTHR) {
      int tok, boff;
      const uint8_t* src = nullptr;
      if (i < 2 * kPfTokens * PPR) {
        const int isv = i >= kPfTokens * PPR;
        const int pc = isv ? i - kPfTokens * PPR : i;
        tok = pc / PPR;
        const int pp = pc % PPR;
        boff = isv * kPfTokens * (D / 2) + tok * (D / 2) + 8 * pp;
        if (LAYOUT == PF_PER_CHANNEL) {
          if (t0 + tok < S) src = (isv ? p.v_codes : p.k_codes) + kvbase + (int64_t)(t0 + tok) * (D / 2) + 8 * pp;
        } else {
          const int64_t so = slot_off[rb][tok];
          if (so >= 0) src = p.cache + so + (isv ? D / 2 : 0) + 8 * pp;
        }
      } else {  // paged token rulers
        tok = i - 2 * kPfTokens * PPR;
        boff = 2 * kPfTokens * (D / 2) + tok * 8;
        const int64_t so = slot_off[rb][tok];
        if (so >= 0) src = p.cache + so + D;
      }
      if (src)
        pf_cp_async8(d0 + boff, src);
      else
        *reinterpret_cast<uint2*>(dst + boff) = make_uint2(0u, 0u);
    }
  };
  prep(0, 0);
  prep(kPfTokens, 1);
  __syncthreads();
  if (kend > 0) issue(0, 0);

  int buf = 0;
  for (int t0 = 0; t0 < kend; t0 += kPfTokens, buf ^= 1) {
    // ---- 1. chunk t0 has landed; start chunk t0+64, resolve chunk t0+128 ----
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    if (t0 + kPfTokens < kend) issue(t0 + kPfTokens, buf ^ 1);  // its slot rows: slot_off[buf ^ 1]
    if (t0 + 2 * kPfTokens < kend) prep(t0 + 2 * kPfTokens, buf);  // slot_off[buf] was chunk t0's
    // ---- 2. dequantize the chunk's K and V into shared memory ----
    // a word holds the 8 codes of dims 8wr .. 8wr+7 (byte e/2, low nibble for
    // even dims); a token row is a whole number of words for every D
    const uint8_t* src = raw + buf * RAW;
    for (int i = tid; i < 2 * WORDS; i += NTHR) {
      const int isv = i >= WORDS;
      const int w = isv ? i - WORDS : i;
      const int tok = w / WPR, wr = w % WPR;
      const int d0 = 8 * wr;
      const uint32_t word =
          *reinterpret_cast<const uint32_t*>(src + isv * kPfTokens * (D / 2) + tok * (D / 2) + 4 * wr);
      // codes as exact fp16: nibble | 0x6400 is 1024 + c, minus 1024.
      // a/b/c/d hold dims (0,4)/(1,5)/(2,6)/(3,7) in their (low, high) halves.
      const uint32_t a = (word & 0x000F000Fu) | 0x64006400u;
      const uint32_t b = ((word >> 4) & 0x000F000Fu) | 0x64006400u;
      const uint32_t c = ((word >> 8) & 0x000F000Fu) | 0x64006400u;
      const uint32_t d = ((word >> 12) & 0x000F000Fu) | 0x64006400u;
      const uint32_t x[4] = {__byte_perm(a, b, 0x5410), __byte_perm(c, d, 0x5410), __byte_perm(a, b, 0x7632),
                             __byte_perm(c, d, 0x7632)};
      const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6400u));
      uint32_t y[4];
      if (kPC) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __half2 hv = __hsub2(*reinterpret_cast<const __half2*>(&x[e]), bias);
          y[e] = *reinterpret_cast<const uint32_t*>(&hv);
        }
      } else {  // c * step + min, one fp16 rounding (fused multiply-add on half pairs)
        const uint2 ru = *reinterpret_cast<const uint2*>(src + 2 * kPfTokens * (D / 2) + tok * 8);
        const uint32_t rp = isv ? ru.y : ru.x;  // (min, step)
        const __half2 ms = *reinterpret_cast<const __half2*>(&rp);
        const __half2 mn = __low2half2(ms), st = __high2half2(ms);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __half2 hv = __hfma2(__hsub2(*reinterpret_cast<const __half2*>(&x[e]), bias), st, mn);
          y[e] = *reinterpret_cast<const uint32_t*>(&hv);
        }
      }
      *reinterpret_cast<uint4*>((isv ? vsh : ksh) + tok * LD + d0) = make_uint4(y[0], y[1], y[2], y[3]);
    }
    __syncthreads();

    if (mw < M && (!p.causal || t0 <= off + mw + 15)) {
      // ---- 2. S = Q K^T for this warp's 16 rows x 64 tokens ----
      float s[NTS][4];
#pragma unroll
      for (int n = 0; n < NTS; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
      // k-steps outer, the 8 token tiles inner: consecutive tensor-core ops
      // update different accumulators instead of one dependent chain
#pragma unroll
      for (int ks = 0; ks < KS; ks += 2) {
        // matrices: (k-step ks, dims 0-7), (ks, 8-15), (ks+1, 0-7), (ks+1, 8-15) of tokens 8n..8n+7
        const int mi = lane >> 3, ri = lane & 7;
        const int kk = (ks + (mi >> 1) < KS) ? ks + (mi >> 1) : ks;
        uint32_t bb[NTS][4];
#pragma unroll
        for (int n = 0; n < NTS; ++n)
          ldsm_x4(bb[n][0], bb[n][1], bb[n][2], bb[n][3], ksh + (8 * n + ri) * LD + 16 * kk + 8 * (mi & 1));
#pragma unroll
        for (int n = 0; n < NTS; ++n) mma_16816(s[n], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], bb[n][0], bb[n][1]);
        if (ks + 1 < KS) {
#pragma unroll
          for (int n = 0; n < NTS; ++n)
            mma_16816(s[n], qa[ks + 1][0], qa[ks + 1][1], qa[ks + 1][2], qa[ks + 1][3], bb[n][2], bb[n][3]);
        }
      }
      // ---- 3. mask, online softmax (log2 domain) ----
      float mx[2] = {mrow[0], mrow[1]};
      // the mask only where some row of the warp does not see the whole
      // chunk (the causal diagonal, the sequence end); warp-uniform
      auto scale_scores = [&](auto masked) {
#pragma unroll
        for (int n = 0; n < NTS; ++n) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float v = s[n][i] * p.scale_log2;
            if constexpr (decltype(masked)::value) {
              const int row = mw + g + ((i & 2) ? 8 : 0);
              const int tok = t0 + 8 * n + 2 * r + (i & 1);
              const int lim = p.causal ? min(S, off + row + 1) : S;
              v = tok < lim ? v : -INFINITY;
            }
            s[n][i] = v;
            mx[i >> 1] = fmaxf(mx[i >> 1], v);
          }
        }
      };
      if (t0 + kPfTokens <= (p.causal ? min(S, off + mw + 1) : S))
        scale_scores(std::false_type{});
      else
        scale_scores(std::true_type{});
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 1));
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 2));
      }
      float al[2], msafe[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        msafe[e] = (mx[e] == -INFINITY) ? 0.f : mx[e];  // a row with no key yet
        al[e] = (mrow[e] == -INFINITY) ? 0.f : exp2_approx(mrow[e] - msafe[e]);
        mrow[e] = mx[e];
        lrow[e] *= al[e];
      }
#pragma unroll
      for (int n = 0; n < NTO; ++n) {
        o[n][0] *= al[0];
        o[n][1] *= al[0];
        o[n][2] *= al[1];
        o[n][3] *= al[1];
      }
      uint32_t pa[NTS][2];
#pragma unroll
      for (int n = 0; n < NTS; ++n) {
        const float p0 = exp2_approx(s[n][0] - msafe[0]), p1 = exp2_approx(s[n][1] - msafe[0]);
        const float p2 = exp2_approx(s[n][2] - msafe[1]), p3 = exp2_approx(s[n][3] - msafe[1]);
        pa[n][0] = pack_half2(p0, p1);
        pa[n][1] = pack_half2(p2, p3);
        if (kPC) {  // the sum of the fp16 weights the tensor core multiplies: o / l is then
                    // a convex combination of the codes, and (o / l - zero) * scale exact
          const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&pa[n][0]));
          const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&pa[n][1]));
          lrow[0] += f0.x + f0.y;
          lrow[1] += f1.x + f1.y;
        } else {
          lrow[0] += p0 + p1;
          lrow[1] += p2 + p3;
        }
      }
      // ---- 4. O += P V ----
#pragma unroll
      for (int kt = 0; kt < kPfTokens / 16; ++kt) {
        const uint32_t a0 = pa[2 * kt][0], a1 = pa[2 * kt][1], a2 = pa[2 * kt + 1][0], a3 = pa[2 * kt + 1][1];
#pragma unroll
        for (int n = 0; n < NTO; n += 2) {
          // matrices: tokens 16kt+0..7 / +8..15 of dims 8n..8n+7, then of dims 8n+8..
          const int mi = lane >> 3, ri = lane & 7;
          const int nn = (n + (mi >> 1) < NTO) ? n + (mi >> 1) : n;
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(b0, b1, b2, b3, vsh + (16 * kt + 8 * (mi & 1) + ri) * LD + 8 * nn);
          mma_16816(o[n], a0, a1, a2, a3, b0, b1);
          if (n + 1 < NTO) mma_16816(o[n + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
  }

  // ---- normalise and store rows mw+g, mw+g+8 ----
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    float l = lrow[e];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int row = mw + g + 8 * e;
    if (row >= M) continue;
    const float inv = l > 0.f ? 1.f / l : 0.f;  // a row with no key is written as zeros
    const int64_t base = (int64_t)(row0 + row) * p.out_row_stride + (int64_t)h * p.out_head_stride;
#pragma unroll
    for (int n = 0; n < NTO; ++n) {
      float v0 = o[n][2 * e] * inv, v1 = o[n][2 * e + 1] * inv;
      if (kPC && pcq && l > 0.f) {
        const int dd = 8 * n + 2 * r;
        const float2 vs = __half22float2(*reinterpret_cast<const __half2*>(&rul[2][dd]));
        const float2 vz = __half22float2(*reinterpret_cast<const __half2*>(&rul[3][dd]));
        v0 = (v0 - vz.x) * vs.x;
        v1 = (v1 - vz.y) * vs.y;
      }
      store_elem(p, base + 8 * n + 2 * r, v0);
      store_elem(p, base + 8 * n + 2 * r + 1, v1);
    }
  }
}

// One instantiation: opt it into its dynamic shared memory (more than the
// default 48 KB at D=128) the first time, then launch.
template <int D, int LAYOUT, int HPC>
int prefill_launch_d(const PrefillParams& p, dim3 grid, cudaStream_t st) {
  constexpr int smem = pf_smem_bytes<D, LAYOUT>();
  static std::atomic<int> opted{-1};  // device the attribute was last set for
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SLMT_ERR_CUDA;
  if (opted.load(std::memory_order_acquire) != dev) {
    if (cudaFuncSetAttribute(prefill_kernel<D, LAYOUT, HPC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem) != cudaSuccess) {
      (void)cudaGetLastError();
      return SLMT_ERR_CUDA;
    }
    opted.store(dev, std::memory_order_release);
  }
  grid.y /= HPC;
  prefill_kernel<D, LAYOUT, HPC><<<grid, 128 * HPC, smem, st>>>(p);
  return launch_status();
}

// Two query heads per CTA when the group has an even number of them (their
// shared chunk is dequantized once), else one.
template <int LAYOUT>
int prefill_launch(const PrefillParams& p, int head_dim, dim3 grid, cudaStream_t st) {
  const bool two = p.G % 2 == 0;
  if (head_dim == 64) return two ? prefill_launch_d<64, LAYOUT, 2>(p, grid, st) : prefill_launch_d<64, LAYOUT, 1>(p, grid, st);
  if (head_dim == 80) return two ? prefill_launch_d<80, LAYOUT, 2>(p, grid, st) : prefill_launch_d<80, LAYOUT, 1>(p, grid, st);
  return two ? prefill_launch_d<128, LAYOUT, 2>(p, grid, st) : prefill_launch_d<128, LAYOUT, 1>(p, grid, st);
}

int prefill_pc_launch(const void* q, int q_bf16, int64_t q_head_stride, int64_t q_row_stride,
                      const uint8_t* k_packed, const uint8_t* v_packed, int64_t seq_len, const uint16_t* k_scale,
                      const uint16_t* k_zero, const uint16_t* v_scale, const uint16_t* v_zero, int use_quant,
                      int causal, int64_t num_rows, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                      float sm_scale, void* out, int out_dtype, int64_t out_head_stride, int64_t out_row_stride,
                      cudaStream_t st) {
  PrefillParams p{};
  p.q = q;
  p.q_bf16 = q_bf16;
  p.q_head_stride = q_head_stride;
  p.q_row_stride = q_row_stride;
  p.k_codes = k_packed;
  p.v_codes = v_packed;
  p.k_scale = k_scale;
  p.k_zero = k_zero;
  p.v_scale = v_scale;
  p.v_zero = v_zero;
  p.use_quant = use_quant ? 1 : 0;
  p.S = (int)seq_len;
  p.M = (int)num_rows;
  p.H = (int)num_q_heads;
  p.KV = (int)num_kv_heads;
  p.G = (int)(num_q_heads / num_kv_heads);
  p.causal = causal ? 1 : 0;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.out = out;
  p.out_dtype = out_dtype;
  p.out_head_stride = out_head_stride;
  p.out_row_stride = out_row_stride;
  const dim3 grid((unsigned)((num_rows + kPfRows - 1) / kPfRows), (unsigned)num_q_heads, 1);
  return prefill_launch<PF_PER_CHANNEL>(p, (int)head_dim, grid, st);
}

int prefill_paged_launch(const void* q, int q_bf16, int64_t q_row_stride, int64_t q_head_stride,
                         const uint8_t* kv_cache, int64_t num_blocks, int64_t block_size, int64_t num_kv_heads,
                         int64_t head_dim, const void* block_tables, int bt_i64, int64_t bt_seq_stride,
                         int64_t max_blocks_per_seq, const int32_t* query_start_loc, const int32_t* seq_lens,
                         int64_t num_reqs, int64_t max_query_len, int64_t num_q_heads, float sm_scale, void* out,
                         int out_dtype, int64_t out_row_stride, int64_t out_head_stride, int32_t* err_flag,
                         cudaStream_t st) {
  PrefillParams p{};
  p.q = q;
  p.q_bf16 = q_bf16;
  p.q_row_stride = q_row_stride;
  p.q_head_stride = q_head_stride;
  p.cache = kv_cache;
  p.num_blocks = num_blocks;
  p.block_size = (int)block_size;
  p.block_tables = block_tables;
  p.bt_i64 = bt_i64;
  p.bt_seq_stride = bt_seq_stride;
  p.len_cap = max_blocks_per_seq * block_size;
  p.query_start_loc = query_start_loc;
  p.seq_lens = seq_lens;
  p.err = err_flag;
  p.H = (int)num_q_heads;
  p.KV = (int)num_kv_heads;
  p.G = (int)(num_q_heads / num_kv_heads);
  p.causal = 1;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.out = out;
  p.out_dtype = out_dtype;
  p.out_head_stride = out_head_stride;
  p.out_row_stride = out_row_stride;
  const dim3 grid((unsigned)((max_query_len + kPfRows - 1) / kPfRows), (unsigned)num_q_heads, (unsigned)num_reqs);
  return prefill_launch<PF_PAGED>(p, (int)head_dim, grid, st);
}

}  // namespace slmt
