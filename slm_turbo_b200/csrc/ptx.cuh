// ptx.cuh -- thin inline-PTX wrappers used by the sm_100a kernels:
// mbarrier pipelines, bulk (TMA 1-D) and cp.async copies into shared memory,
// the m16n8k16 f16 tensor-core tile, movmatrix, and the 4-bit -> fp16 code
// conversion.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace slmt {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on phase `parity`: false once `limit_ns` of wall time passed.
// Every spin in these kernels goes through here, so no wait is endless.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}

// ------------------------------------------------------------ async copies --
// 1-D bulk copy global -> shared (TMA unit), completes `bytes` of tx on `bar`.
// src and dst 16-byte aligned, bytes a multiple of 16; the source is always
// this GPU's own memory and the destination this CTA's shared memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src,
                                         uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::"
      "cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Tiled 3-D TMA copy global -> shared of the box at (c0, c1, c2) of the
// tensor map `tmap` (the address of a __grid_constant__ kernel parameter),
// completing the box's bytes of tx on `bar`.  c0 (the innermost coordinate)
// times the element size is a multiple of 16 bytes.  No multicast.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
      : "memory");
}

// 8- and 4-byte shared-memory loads at a 32-bit shared address.  Volatile:
// they stay after the mbarrier wait that publishes the bytes.
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// As tma_load_3d with an L2 cache policy (createpolicy) for the loaded lines.
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const void* tmap, int c0, int c1, int c2,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Order this thread's earlier generic-proxy accesses to shared memory before
// later async-proxy (TMA) accesses of the same bytes.
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Order this thread's earlier generic-proxy writes to global memory before
// later async-proxy (TMA) reads of the same bytes.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Pull the 128-byte line holding `p` into L2 (no register result).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Tiled 2-D TMA copy global -> shared of the box at (c0, c1) of `tmap`, with
// the same rules as tma_load_3d.  No multicast.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

// L2 policy for data streamed once (the packed cache).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;"
               : "=l"(p));
  return p;
}

// 8-byte cp.async global -> shared (both 8-byte aligned).
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst)),
               "l"(src)
               : "memory");
}

// 16-byte cp.async global -> shared through L2 only (.cg: coherent with
// stores other CTAs made during the kernel).
__device__ __forceinline__ void cp_async16_cg(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Arrive on `bar` once all earlier cp.async of this thread landed; the
// barrier's expected count already includes this arrival (.noinc).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

// ------------------------------------------------------------ tensor cores --
// D = A(16x16 f16, row) * B(16x8 f16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0,
                                          uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// As mma_16816 for a tile whose C rows g and g+8 are known to be equal (an A
// tile of identical rows): only rows g are kept (c0, c1); rows g+8 land in
// temporaries that die here.
__device__ __forceinline__ void mma_16816_rows0(float& c0, float& c1, uint32_t a0, uint32_t a1,
                                                uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  float d2 __attribute__((unused)), d3 __attribute__((unused));
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%10,%10};"
      : "+f"(c0), "+f"(c1), "=f"(d2), "=f"(d3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// Transpose of an 8x8 b16 matrix held one row-pair per thread.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;"
               : "=r"(y)
               : "r"(x));
  return y;
}

// ------------------------------------------------------ 4-bit -> fp16 codes --
// IEEE fp16 1024 is 0x6400 and has ulp 1 on [1024, 2048), so OR-ing a nibble
// into the low mantissa bits gives 1024+c exactly; fp16 64 is 0x5400 and has
// ulp 1/16 on [64, 128), so OR-ing a nibble that sits in bits 4..7 gives
// 64+c exactly.  One LOP3 builds two such halves.  (The magic-number int4 ->
// fp16 conversion of the mixed-input GEMM literature, e.g. Kim et al. 2022,
// "Who Says Elephants Can't Run".)  The bias (1024 or 64 per nibble) is left
// in: the kernels take it off once per dot product instead of once per code.
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask,
                                               uint32_t orv) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));
  return d;
}

// halves = 1024 + (low nibble of byte 0, low nibble of byte 2)
__device__ __forceinline__ uint32_t codes_lo_biased(uint32_t w) {
  return lop_and_or(w, 0x000F000Fu, 0x64006400u);
}

// halves = 64 + (high nibble of byte 0, high nibble of byte 2)
__device__ __forceinline__ uint32_t codes_hi_biased(uint32_t w) {
  return lop_and_or(w, 0x00F000F0u, 0x54005400u);
}

__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float half_bits_to_float(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}

}  // namespace slmt
