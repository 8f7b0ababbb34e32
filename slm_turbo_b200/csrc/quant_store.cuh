// quant_store.cuh -- one warp quantizes one (token, kv head) row of K and V
// into a packed per-token slot [K codes D/2][V codes D/2][k_min k_step v_min
// v_step fp16].  The store kernel and the decode kernel's fused append both
// go through these two functions, so they write the same bytes.
//
// Arithmetic of the reference kernel (kernels/kv_dequant_kernels.cuh:838-918):
// fp32 min/max over the row, step = (max-min)/15 with IEEE division, step = 1
// when not positive, code = (int)((x-min)/step + 0.5f) clamped to [0, 15],
// dim 2j in the low nibble of byte j, rulers rounded to fp16 (nearest).
#pragma once

#include "ptx.cuh"

namespace slmt {

// Lanes of a warp hold VEC consecutive dims each (lanes >= LANES idle).
template <int D>
struct SlotGeom {
  static constexpr int VEC = (D == 64) ? 2 : 4;
  static constexpr int LANES = D / VEC;  // 32, 32, 20
};

// This lane's packed codes of the row and (lane 0) the row's rulers.
struct SlotRow {
  uint32_t kc, vc;  // VEC nibbles each
  uint2 rulers;     // (k_min | k_step << 16, v_min | v_step << 16), fp16 bits
};

// Quantize a row whose VEC values per lane are in xk / xv (lanes >= LANES
// hold zeros and take no part in the min/max).
template <int D>
__device__ __forceinline__ SlotRow quantize_slot_vals(const float (&xk)[SlotGeom<D>::VEC],
                                                      const float (&xv)[SlotGeom<D>::VEC]) {
  constexpr int VEC = SlotGeom<D>::VEC;
  const int lane = threadIdx.x & 31;
  const bool act = lane < SlotGeom<D>::LANES;
  float kmn = INFINITY, kmx = -INFINITY, vmn = INFINITY, vmx = -INFINITY;
  if (act) {
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      kmn = fminf(kmn, xk[i]);
      kmx = fmaxf(kmx, xk[i]);
      vmn = fminf(vmn, xv[i]);
      vmx = fmaxf(vmx, xv[i]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kmn = fminf(kmn, __shfl_xor_sync(0xffffffffu, kmn, o));
    kmx = fmaxf(kmx, __shfl_xor_sync(0xffffffffu, kmx, o));
    vmn = fminf(vmn, __shfl_xor_sync(0xffffffffu, vmn, o));
    vmx = fmaxf(vmx, __shfl_xor_sync(0xffffffffu, vmx, o));
  }
  float kst = __fdiv_rn(kmx - kmn, 15.0f);
  if (!(kst > 0.0f)) kst = 1.0f;  // constant row guard (ref .cuh:854)
  float vst = __fdiv_rn(vmx - vmn, 15.0f);
  if (!(vst > 0.0f)) vst = 1.0f;

  SlotRow r;
  r.kc = 0u;
  r.vc = 0u;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    int qk = (int)__fadd_rn(__fdiv_rn(__fsub_rn(xk[i], kmn), kst), 0.5f);
    int qv = (int)__fadd_rn(__fdiv_rn(__fsub_rn(xv[i], vmn), vst), 0.5f);
    qk = qk < 0 ? 0 : (qk > 15 ? 15 : qk);
    qv = qv < 0 ? 0 : (qv > 15 ? 15 : qv);
    r.kc |= (uint32_t)qk << (4 * i);
    r.vc |= (uint32_t)qv << (4 * i);
  }
  r.rulers.x = (uint32_t)__half_as_ushort(__float2half_rn(kmn)) |
               ((uint32_t)__half_as_ushort(__float2half_rn(kst)) << 16);
  r.rulers.y = (uint32_t)__half_as_ushort(__float2half_rn(vmn)) |
               ((uint32_t)__half_as_ushort(__float2half_rn(vst)) << 16);
  return r;
}

// This lane's VEC values of a row of D fp16 (or bf16, in_bf16) values.
template <int D>
__device__ __forceinline__ void load_row_vals(const void* row, int in_bf16, float (&x)[SlotGeom<D>::VEC]) {
  constexpr int VEC = SlotGeom<D>::VEC;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < VEC; ++i) x[i] = 0.f;
  if (lane < SlotGeom<D>::LANES) {
    if (in_bf16) {
      const __nv_bfloat16* rp = reinterpret_cast<const __nv_bfloat16*>(row) + lane * VEC;
#pragma unroll
      for (int i = 0; i < VEC; ++i) x[i] = __bfloat162float(rp[i]);
    } else {
      const __half* rp = reinterpret_cast<const __half*>(row) + lane * VEC;
#pragma unroll
      for (int i = 0; i < VEC; ++i) x[i] = __half2float(rp[i]);
    }
  }
}

// Quantize one (token, kv head): key_row / value_row are its D values.
template <int D>
__device__ __forceinline__ SlotRow quantize_slot_row(const void* key_row, const void* value_row,
                                                     int in_bf16) {
  float xk[SlotGeom<D>::VEC], xv[SlotGeom<D>::VEC];
  load_row_vals<D>(key_row, in_bf16, xk);
  load_row_vals<D>(value_row, in_bf16, xv);
  return quantize_slot_vals<D>(xk, xv);
}

// The VEC 16-bit values of this lane, packed (two per word), for rows that
// are 4-byte aligned at every lane's offset (D = 64: 2 values; else 4).
template <int D>
struct PackedRow {
  uint32_t w[SlotGeom<D>::VEC / 2];
};

template <int D>
__device__ __forceinline__ PackedRow<D> load_row_packed(const void* row) {
  constexpr int VEC = SlotGeom<D>::VEC;
  const int lane = threadIdx.x & 31;
  PackedRow<D> r;
#pragma unroll
  for (int i = 0; i < VEC / 2; ++i) r.w[i] = 0u;
  if (lane < SlotGeom<D>::LANES) {
    const uint32_t* rp = reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint16_t*>(row) + lane * VEC);
#pragma unroll
    for (int i = 0; i < VEC / 2; ++i) r.w[i] = rp[i];
  }
  return r;
}

template <int D>
__device__ __forceinline__ void unpack_row(const PackedRow<D>& r, int in_bf16, float (&x)[SlotGeom<D>::VEC]) {
#pragma unroll
  for (int i = 0; i < SlotGeom<D>::VEC / 2; ++i) {
    const uint16_t lo = (uint16_t)(r.w[i] & 0xFFFFu), hi = (uint16_t)(r.w[i] >> 16);
    x[2 * i] = in_bf16 ? __bfloat162float(__ushort_as_bfloat16(lo)) : __half2float(__ushort_as_half(lo));
    x[2 * i + 1] = in_bf16 ? __bfloat162float(__ushort_as_bfloat16(hi)) : __half2float(__ushort_as_half(hi));
  }
}

// Write the row's slot at `slot` (global or shared memory; 8-byte aligned,
// as every slot of the paged layout is when the cache base is).
template <int D>
__device__ __forceinline__ void write_slot_row(uint8_t* slot, const SlotRow& r) {
  constexpr int VEC = SlotGeom<D>::VEC;
  const int lane = threadIdx.x & 31;
  if (lane < SlotGeom<D>::LANES) {
    if (VEC == 4) {
      reinterpret_cast<uint16_t*>(slot)[lane] = (uint16_t)r.kc;
      reinterpret_cast<uint16_t*>(slot + D / 2)[lane] = (uint16_t)r.vc;
    } else {
      slot[lane] = (uint8_t)r.kc;
      slot[D / 2 + lane] = (uint8_t)r.vc;
    }
  }
  if (lane == 0) *reinterpret_cast<uint2*>(slot + D) = r.rulers;
}

}  // namespace slmt
