// store.cu -- quantize-on-write kernels (sm_100a).
//
//  * kv_store_kernel: vLLM paged per-token layout.  One warp per (token, kv
//    head) through quantize_slot_row / write_slot_row (quant_store.cuh):
//    lanes hold 2-4 dims, warp-shuffle min/max, fp32 IEEE step and codes
//    exactly as the reference kernel computes them
//    (kernels/kv_dequant_kernels.cuh:838-918), then each lane stores its
//    packed bytes and lane 0 the four fp16 rulers with one 8-byte store.
//  * pc_rulers_kernel / pc_codes_kernel: the per-channel quantizer of
//    kernels/benchmark/benchmark.py:26-56 on the device, with the same
//    fp16 arithmetic (each op computed in fp32 and rounded to fp16, as torch
//    evaluates half tensors).
#include <cooperative_groups.h>

#include "internal.h"
#include "ptx.cuh"
#include "quant_store.cuh"

namespace slmt {

template <int D>
__global__ void __launch_bounds__(128) kv_store_kernel(
    const void* __restrict__ key, const void* __restrict__ value, int in_bf16,
    int64_t tok_stride, int num_tokens, int kv, uint8_t* __restrict__ cache,
    int64_t num_slots, const int64_t* __restrict__ slot_mapping,
    int32_t* err) {
  constexpr int SLOT = D + 8;
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (wid >= (int64_t)num_tokens * kv) return;
  const int tok = (int)(wid / kv), kvh = (int)(wid % kv);
  const int64_t slot = slot_mapping[tok];
  if (slot < 0) return;  // padding token (ref .cuh:902)
  if (slot >= num_slots) {
    if (lane == 0 && err) atomicOr(reinterpret_cast<unsigned int*>(err), 2u);
    return;
  }
  const int64_t row = (int64_t)tok * tok_stride + (int64_t)kvh * D;
  const size_t esz = in_bf16 ? sizeof(__nv_bfloat16) : sizeof(__half);
  const SlotRow r = quantize_slot_row<D>(reinterpret_cast<const uint8_t*>(key) + row * esz,
                                         reinterpret_cast<const uint8_t*>(value) + row * esz, in_bf16);
  write_slot_row<D>(cache + (slot * kv + kvh) * (int64_t)SLOT, r);
}

// fp16 tensor arithmetic as torch evaluates it: fp32 op, round to fp16.
__device__ __forceinline__ float h16(float x) { return __half2float(__float2half_rn(x)); }

// Per (seq*kv, dim): min/max over S, then scale/zero (benchmark.py:26-42).
__global__ void __launch_bounds__(256) pc_rulers_kernel(
    const __half* __restrict__ x, int64_t S, int D, uint16_t* __restrict__ scale,
    uint16_t* __restrict__ zero) {
  __shared__ float smn[8][32], smx[8][32];
  const int dl = threadIdx.x & 31, sg = threadIdx.x >> 5;
  const int d = blockIdx.y * 32 + dl;
  const int64_t row0 = (int64_t)blockIdx.x * S;
  float mn = INFINITY, mx = -INFINITY;
  if (d < D) {
    for (int64_t s = sg; s < S; s += 8) {
      const float v = __half2float(x[(row0 + s) * D + d]);
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
  }
  smn[sg][dl] = mn;
  smx[sg][dl] = mx;
  __syncthreads();
  if (sg == 0 && d < D) {
#pragma unroll
    for (int k = 1; k < 8; ++k) {
      mn = fminf(mn, smn[k][dl]);
      mx = fmaxf(mx, smx[k][dl]);
    }
    float sc = h16(__fdiv_rn(h16(__fsub_rn(mx, mn)), 15.0f));
    float zp = h16(__fsub_rn(0.0f, rintf(h16(__fdiv_rn(mn, sc)))));
    if (mx == mn) {
      sc = 1.0f;
      zp = 0.0f;
    }
    zp = fminf(fmaxf(zp, 0.0f), 15.0f);
    const int64_t o = (int64_t)blockIdx.x * D + d;
    scale[o] = __half_as_ushort(__float2half_rn(sc));
    zero[o] = __half_as_ushort(__float2half_rn(zp));
  }
}

__device__ __forceinline__ uint32_t pc_code(float x, float sc, float zp) {
  // q = clamp(round(x / scale) + zero, 0, 15) in fp16 steps (benchmark.py:50-52)
  float q = h16(__fadd_rn(rintf(h16(__fdiv_rn(x, sc))), zp));
  if (q != q) return 0u;  // NaN (scale underflow) -> 0, as the host cast gives
  q = fminf(fmaxf(q, 0.0f), 15.0f);
  return (uint32_t)q;
}

// codes of rows [row, row+1) for every byte: grid-stride over rows*D/2 bytes.
// x element (h, t, d) at x + h*xh + t*xt + d; packed byte (h, pos+t, j) at
// packed + (h*s_cap + pos + t)*D/2 + j; rulers (h, d) at scale/zero + h*D + d.
__global__ void __launch_bounds__(256) pc_codes_kernel(
    const __half* __restrict__ x, int64_t xh, int64_t xt, int64_t heads,
    int64_t ntok, int D, const uint16_t* __restrict__ scale,
    const uint16_t* __restrict__ zero, int64_t ruler_h, uint8_t* __restrict__ packed,
    int64_t s_cap, int64_t pos) {
  const int half = D / 2;
  const int64_t total = heads * ntok * half;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const int64_t t = (i / half) % ntok;
    const int64_t h = i / ((int64_t)half * ntok);
    const __half* xr = x + h * xh + t * xt;
    const int64_t ro = h * ruler_h;
    const uint32_t c0 = pc_code(__half2float(xr[2 * j]), half_bits_to_float(scale[ro + 2 * j]),
                                half_bits_to_float(zero[ro + 2 * j]));
    const uint32_t c1 = pc_code(__half2float(xr[2 * j + 1]), half_bits_to_float(scale[ro + 2 * j + 1]),
                                half_bits_to_float(zero[ro + 2 * j + 1]));
    packed[(h * s_cap + pos + t) * half + j] = (uint8_t)(c0 | (c1 << 4));
  }
}

// Vector path of the per-channel quantizer: rows of D fp16 values that start
// on 16 bytes (D = 64, 80, 128 are multiples of 8 values).
constexpr int kPcSplit = 8;  // CTAs (one cluster) per row of the rulers pass

// Rulers, one cluster of kPcSplit CTAs per (seq*kv) row: CTA k reduces tokens
// [k*S/split, (k+1)*S/split) with 16-byte loads (8 dims per thread), the
// cluster's rank 0 combines the 8 partial min/max sets through distributed
// shared memory and writes scale/zero exactly as pc_rulers_kernel does.
template <int D>
__global__ void __cluster_dims__(kPcSplit, 1, 1) __launch_bounds__(256)
    pc_rulers_vec_kernel(const __half* __restrict__ x, int64_t S, uint16_t* __restrict__ scale,
                         uint16_t* __restrict__ zero) {
  namespace cg = cooperative_groups;
  constexpr int LPR = D / 8;           // threads per token row
  constexpr int RPI = 256 / LPR;       // token rows per iteration
  __shared__ float smn[RPI][D], smx[RPI][D];
  __shared__ float cmn[D], cmx[D];
  cg::cluster_group cluster = cg::this_cluster();
  const int row = blockIdx.x / kPcSplit;
  const int part = (int)cluster.block_rank();
  const int tid = threadIdx.x;
  const int rs = tid / LPR, dg = tid % LPR;  // token-row slot, 8-dim group
  const int64_t s0 = part * S / kPcSplit, s1 = (part + 1) * S / kPcSplit;
  float mn[8], mx[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    mn[i] = INFINITY;
    mx[i] = -INFINITY;
  }
  if (rs < RPI) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + ((int64_t)row * S) * D) + dg;
#pragma unroll 4
    for (int64_t t = s0 + rs; t < s1; t += RPI) {
      const uint4 u = __ldg(xr + t * (D / 8));
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        mn[2 * i] = fminf(mn[2 * i], f.x);
        mx[2 * i] = fmaxf(mx[2 * i], f.x);
        mn[2 * i + 1] = fminf(mn[2 * i + 1], f.y);
        mx[2 * i + 1] = fmaxf(mx[2 * i + 1], f.y);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      smn[rs][dg * 8 + i] = mn[i];
      smx[rs][dg * 8 + i] = mx[i];
    }
  }
  __syncthreads();
  for (int d = tid; d < D; d += 256) {
    float a = INFINITY, b = -INFINITY;
    for (int k = 0; k < RPI; ++k) {
      a = fminf(a, smn[k][d]);
      b = fmaxf(b, smx[k][d]);
    }
    cmn[d] = a;
    cmx[d] = b;
  }
  cluster.sync();
  if (part == 0) {
    for (int d = tid; d < D; d += 256) {
      float a = cmn[d], b = cmx[d];
      for (int k = 1; k < kPcSplit; ++k) {
        a = fminf(a, cluster.map_shared_rank(cmn, k)[d]);
        b = fmaxf(b, cluster.map_shared_rank(cmx, k)[d]);
      }
      float sc = h16(__fdiv_rn(h16(__fsub_rn(b, a)), 15.0f));
      float zp = h16(__fsub_rn(0.0f, rintf(h16(__fdiv_rn(a, sc)))));
      if (b == a) {
        sc = 1.0f;
        zp = 0.0f;
      }
      zp = fminf(fmaxf(zp, 0.0f), 15.0f);
      const int64_t o = (int64_t)row * D + d;
      scale[o] = __half_as_ushort(__float2half_rn(sc));
      zero[o] = __half_as_ushort(__float2half_rn(zp));
    }
  }
  cluster.sync();  // keep every CTA's shared memory alive until rank 0 has read it
}

// Codes, 16 dims per thread: two 16-byte loads of x, the rulers of those
// dims, one 8-byte store of packed codes.  Item i = (h, t, g) with g the
// 16-dim group; x rows and rulers as pc_codes_kernel.
template <int D>
__global__ void __launch_bounds__(256) pc_codes_vec_kernel(
    const __half* __restrict__ x, int64_t xh, int64_t xt, int64_t heads, int64_t ntok,
    const uint16_t* __restrict__ scale, const uint16_t* __restrict__ zero, int64_t ruler_h,
    uint8_t* __restrict__ packed, int64_t s_cap, int64_t pos) {
  constexpr int G = D / 16;
  const int64_t total = heads * ntok * G;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(i % G);
    const int64_t ht = i / G;
    const int64_t t = ht % ntok, h = ht / ntok;
    const uint4* xr = reinterpret_cast<const uint4*>(x + h * xh + t * xt + 16 * g);
    const uint4 u0 = __ldg(xr), u1 = __ldg(xr + 1);
    const uint4* sr = reinterpret_cast<const uint4*>(scale + h * ruler_h + 16 * g);
    const uint4* zr = reinterpret_cast<const uint4*>(zero + h * ruler_h + 16 * g);
    const uint4 s0 = __ldg(sr), s1 = __ldg(sr + 1), z0 = __ldg(zr), z1 = __ldg(zr + 1);
    const __half* xv0 = reinterpret_cast<const __half*>(&u0);
    const __half* xv1 = reinterpret_cast<const __half*>(&u1);
    const uint16_t* sv0 = reinterpret_cast<const uint16_t*>(&s0);
    const uint16_t* sv1 = reinterpret_cast<const uint16_t*>(&s1);
    const uint16_t* zv0 = reinterpret_cast<const uint16_t*>(&z0);
    const uint16_t* zv1 = reinterpret_cast<const uint16_t*>(&z1);
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      w0 |= pc_code(__half2float(xv0[k]), half_bits_to_float(sv0[k]), half_bits_to_float(zv0[k])) << (4 * k);
      w1 |= pc_code(__half2float(xv1[k]), half_bits_to_float(sv1[k]), half_bits_to_float(zv1[k])) << (4 * k);
    }
    *reinterpret_cast<uint2*>(packed + (h * s_cap + pos + t) * (D / 2) + 8 * g) = make_uint2(w0, w1);
  }
}

template <int D>
int launch_pc_codes(const __half* x, int64_t xh, int64_t xt, int64_t heads, int64_t ntok,
                    const uint16_t* scale, const uint16_t* zero, uint8_t* packed, int64_t s_cap,
                    int64_t pos, cudaStream_t st) {
  const int64_t total = heads * ntok * (D / 16);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148LL * 32);
  pc_codes_vec_kernel<D><<<(unsigned)blocks, 256, 0, st>>>(x, xh, xt, heads, ntok, scale, zero, D, packed,
                                                           s_cap, pos);
  return launch_status();
}

int launch_pc_codes_any(int D, const __half* x, int64_t xh, int64_t xt, int64_t heads, int64_t ntok,
                        const uint16_t* scale, const uint16_t* zero, uint8_t* packed, int64_t s_cap,
                        int64_t pos, cudaStream_t st) {
  if (D == 64) return launch_pc_codes<64>(x, xh, xt, heads, ntok, scale, zero, packed, s_cap, pos, st);
  if (D == 80) return launch_pc_codes<80>(x, xh, xt, heads, ntok, scale, zero, packed, s_cap, pos, st);
  return launch_pc_codes<128>(x, xh, xt, heads, ntok, scale, zero, packed, s_cap, pos, st);
}

// 16-byte-aligned rows, rulers and packed codes (the vector kernels' needs).
bool pc_vec_ok(const void* x, int64_t xh, int64_t xt, const void* scale, const void* zero,
               const void* packed, int64_t s_cap, int64_t pos, int64_t D) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(scale) |
                      reinterpret_cast<uintptr_t>(zero);
  return a % 16 == 0 && (xh * 2) % 16 == 0 && (xt * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(packed) % 8 == 0 &&
         ((s_cap * (D / 2)) % 8 == 0) && ((pos * (D / 2)) % 8 == 0);
}

}  // namespace slmt

using namespace slmt;

extern "C" int slmt_kv_quantize_store(const void* key, const void* value,
                                      int kv_dtype, int64_t kv_token_stride,
                                      int64_t num_tokens, int64_t num_kv_heads,
                                      int64_t head_dim, uint8_t* kv_cache,
                                      int64_t num_blocks, int64_t block_size,
                                      const int64_t* slot_mapping,
                                      int32_t* err_flag, void* stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks < 0)
    return SLMT_ERR_SHAPE;
  if (!valid_head_dim(head_dim)) return SLMT_ERR_HEAD_DIM;
  if (kv_dtype != SLMT_DTYPE_F16 && kv_dtype != SLMT_DTYPE_BF16) return SLMT_ERR_DTYPE;
  if (num_tokens == 0) return SLMT_OK;
  if (!key || !value || !kv_cache || !slot_mapping) return SLMT_ERR_NULL;
  if (kv_token_stride < num_kv_heads * head_dim) return SLMT_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(kv_cache) % 8 != 0) return SLMT_ERR_ALIGN;
  if (reinterpret_cast<uintptr_t>(key) % 8 != 0 || reinterpret_cast<uintptr_t>(value) % 8 != 0 ||
      kv_token_stride % 4 != 0)
    return SLMT_ERR_ALIGN;
  const int64_t warps = num_tokens * num_kv_heads;
  if (warps > (int64_t)INT32_MAX) return SLMT_ERR_SHAPE;
  const dim3 grid((unsigned)((warps + 3) / 4));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t num_slots = num_blocks * block_size;
  const int bf = kv_dtype == SLMT_DTYPE_BF16;
  switch (head_dim) {
    case 64:
      kv_store_kernel<64><<<grid, 128, 0, st>>>(key, value, bf, kv_token_stride, (int)num_tokens,
                                                (int)num_kv_heads, kv_cache, num_slots, slot_mapping,
                                                err_flag);
      break;
    case 80:
      kv_store_kernel<80><<<grid, 128, 0, st>>>(key, value, bf, kv_token_stride, (int)num_tokens,
                                                (int)num_kv_heads, kv_cache, num_slots, slot_mapping,
                                                err_flag);
      break;
    default:
      kv_store_kernel<128><<<grid, 128, 0, st>>>(key, value, bf, kv_token_stride, (int)num_tokens,
                                                 (int)num_kv_heads, kv_cache, num_slots,
                                                 slot_mapping, err_flag);
      break;
  }
  return launch_status();
}

extern "C" int slmt_per_channel_quantize(const void* x, int x_dtype,
                                         int64_t num_seqs, int64_t num_kv_heads,
                                         int64_t seq_len, int64_t head_dim,
                                         uint8_t* packed, uint16_t* scale,
                                         uint16_t* zero, void* stream) {
  if (num_seqs < 0 || num_kv_heads <= 0 || seq_len < 0) return SLMT_ERR_SHAPE;
  if (!valid_head_dim(head_dim)) return SLMT_ERR_HEAD_DIM;
  if (x_dtype != SLMT_DTYPE_F16) return SLMT_ERR_DTYPE;
  if (num_seqs == 0 || seq_len == 0) return SLMT_OK;
  if (!x || !packed || !scale || !zero) return SLMT_ERR_NULL;
  const int64_t rows = num_seqs * num_kv_heads;
  if (rows > 65535LL * 32768LL) return SLMT_ERR_SHAPE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const __half* xh = reinterpret_cast<const __half*>(x);
  if (pc_vec_ok(x, seq_len * head_dim, head_dim, scale, zero, packed, seq_len, 0, head_dim) &&
      rows * kPcSplit <= (int64_t)INT32_MAX) {
    const unsigned grid = (unsigned)(rows * kPcSplit);
    if (head_dim == 64)
      pc_rulers_vec_kernel<64><<<grid, 256, 0, st>>>(xh, seq_len, scale, zero);
    else if (head_dim == 80)
      pc_rulers_vec_kernel<80><<<grid, 256, 0, st>>>(xh, seq_len, scale, zero);
    else
      pc_rulers_vec_kernel<128><<<grid, 256, 0, st>>>(xh, seq_len, scale, zero);
    int rc = launch_status();
    if (rc != SLMT_OK) return rc;
    return launch_pc_codes_any((int)head_dim, xh, seq_len * head_dim, head_dim, rows, seq_len, scale, zero,
                               packed, seq_len, 0, st);
  }
  const dim3 g1((unsigned)rows, (unsigned)((head_dim + 31) / 32));
  pc_rulers_kernel<<<g1, 256, 0, st>>>(xh, seq_len, (int)head_dim, scale, zero);
  int rc = launch_status();
  if (rc != SLMT_OK) return rc;
  const int64_t total = rows * seq_len * (head_dim / 2);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148LL * 16);
  pc_codes_kernel<<<(unsigned)blocks, 256, 0, st>>>(xh, seq_len * head_dim, head_dim, rows, seq_len,
                                                    (int)head_dim, scale, zero, head_dim, packed, seq_len, 0);
  return launch_status();
}

extern "C" int slmt_per_channel_append(const void* x, int x_dtype,
                                       int64_t x_head_stride,
                                       int64_t x_token_stride, int64_t num_new,
                                       int64_t num_kv_heads, int64_t head_dim,
                                       const uint16_t* scale,
                                       const uint16_t* zero, uint8_t* packed,
                                       int64_t s_cap, int64_t pos,
                                       void* stream) {
  if (num_new < 0 || num_kv_heads <= 0 || s_cap < 0 || pos < 0) return SLMT_ERR_SHAPE;
  if (!valid_head_dim(head_dim)) return SLMT_ERR_HEAD_DIM;
  if (x_dtype != SLMT_DTYPE_F16) return SLMT_ERR_DTYPE;
  if (pos + num_new > s_cap) return SLMT_ERR_SHAPE;
  if (num_new == 0) return SLMT_OK;
  if (!x || !packed || !scale || !zero) return SLMT_ERR_NULL;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (pc_vec_ok(x, x_head_stride, x_token_stride, scale, zero, packed, s_cap, pos, head_dim))
    return launch_pc_codes_any((int)head_dim, reinterpret_cast<const __half*>(x), x_head_stride, x_token_stride,
                               num_kv_heads, num_new, scale, zero, packed, s_cap, pos, st);
  const int64_t total = num_kv_heads * num_new * (head_dim / 2);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148LL * 16);
  pc_codes_kernel<<<(unsigned)blocks, 256, 0, st>>>(
      reinterpret_cast<const __half*>(x), x_head_stride, x_token_stride, num_kv_heads, num_new,
      (int)head_dim, scale, zero, head_dim, packed, s_cap, pos);
  return launch_status();
}
