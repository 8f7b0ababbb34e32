// decode.cu -- host launchers (C ABI) of the split-K decode kernels.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "decode_kernels.cuh"
#include "internal.h"

namespace slmt {

namespace {

// Chunk shares of the first and the second CTA on an SM (SM-aware pieces):
// 6:5 measured best on C3 (5:4, 4:3 and 1:1 beside it).
constexpr int kPartWeightFirst = 6;
constexpr int kPartWeightSecond = 5;
// Cost of a segment start in eighths of a chunk (q staging, fragments,
// output or partial and its publication), for the weighted partition: 24
// measured best on C3 (0, 8, 16, 32 beside it: 77.3, 76.5, 75.7, 74.9 vs 74.5 us).
constexpr int kSegStartCost = 24;
constexpr int kMinChunksPerCta = 4;    // do not split below ~128 tokens per CTA
constexpr int kSmemPerSm = 233472;     // 228 KB shared memory per SM (sm_100)
constexpr int kSmemPerCtaMax = 232448; // 227 KB opt-in per CTA
constexpr int kSmemReserved = 1024;    // reserved per resident CTA

inline int round_up(int x, int a) { return (x + a - 1) / a * a; }

// One translation unit per (head dim, layout family) instantiates the
// kernels and returns the one a call needs (decode_d*.cu); this file
// instantiates none, so the library's sources compile in parallel.
DecodeFn decode_fn(int D, int nt, bool pk, int layout, int kvc, bool append, bool swz) {
  const bool paged = layout == LAYOUT_PAGED;
  if (D == 64)
    return paged ? decode_fn_64_paged(nt, pk, kvc, append, swz) : decode_fn_64_contig(nt, pk, layout, kvc);
  if (D == 80) return paged ? decode_fn_80_paged(nt, pk, kvc, append, false) : decode_fn_80_contig(nt, pk, layout, kvc);
  return paged ? decode_fn_128_paged(nt, pk, kvc, append, swz) : decode_fn_128_contig(nt, pk, layout, kvc);
}

struct OccEntry {
  int device;
  const void* fn;
  int smem;
  int occ;
};

std::mutex g_occ_mu;
OccEntry g_occ[256];
int g_occ_n = 0;

// Resident CTAs per SM for `fn` at `smem` bytes (opts the kernel into large
// dynamic shared memory the first time it is seen on a device).
int occupancy(int device, const void* fn, int threads, int smem) {
  std::lock_guard<std::mutex> lk(g_occ_mu);
  for (int i = 0; i < g_occ_n; ++i)
    if (g_occ[i].device == device && g_occ[i].fn == fn && g_occ[i].smem == smem) return g_occ[i].occ;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemPerCtaMax) !=
      cudaSuccess)
    return -1;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, threads, smem) != cudaSuccess) return -1;
  if (g_occ_n < 256) g_occ[g_occ_n++] = OccEntry{device, fn, smem, occ};
  return occ;
}

std::mutex g_sm_mu;
int g_sms[64] = {0};

// Process-wide knobs read at every launch (slmt_set_wait_limit_ns,
// slmt_set_debug_stall).
std::atomic<uint64_t> g_wait_limit_ns{kDefaultWaitLimitNs};
std::atomic<int> g_debug_stall{0};

}  // namespace

int current_device_sms(int* device_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (device_out) *device_out = dev;
  if (dev >= 0 && dev < 64) {
    std::lock_guard<std::mutex> lk(g_sm_mu);
    if (g_sms[dev] > 0) return g_sms[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    g_sms[dev] = n;
    return n;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  return n;
}

namespace {

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime
// (the library links the runtime only).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Tensor map of packed codes [num_seqs, kv, s_cap, half bytes] (sequence
// stride seq_stride_rows rows) viewed as 8-byte elements [num_seqs, kv,
// s_cap*half/8]: the box [1, kvc, 32*half/8] is one 32-token chunk of `kvc`
// kv heads, i.e. kvc contiguous spans, the x coordinate tok0*half/8 of a
// chunk start is a multiple of 16 bytes.  False (and the bulk-copy path is
// used) unless every rule of the tiled copy holds: 16-byte aligned base and
// strides, box within 256 elements per dimension.
bool encode_codes_map(CUtensorMap* m, const uint8_t* base, int64_t num_seqs, int64_t kv, int64_t s_cap,
                      int64_t half, int64_t seq_stride_rows, int kvc) {
  auto enc = tensor_map_encoder();
  if (!enc || reinterpret_cast<uintptr_t>(base) % 16 != 0 || half % 8 != 0) return false;
  if (seq_stride_rows < kv * s_cap || s_cap < 1 || num_seqs < 1 || kvc > kv) return false;
  const int64_t box_x = kChunkTokens * half / 8;
  if (box_x > 256 || (kChunkTokens * half) % 16 != 0) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)(s_cap * half / 8), (cuuint64_t)kv, (cuuint64_t)num_seqs};
  const cuuint64_t strides[2] = {(cuuint64_t)(s_cap * half), (cuuint64_t)(seq_stride_rows * half)};
  for (cuuint64_t st : strides)
    if (st % 16 != 0 || st >= (1ull << 40)) return false;
  const cuuint32_t box[3] = {(cuuint32_t)box_x, (cuuint32_t)kvc, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<uint8_t*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor map of the paged pool [num_blocks*block_size rows][kv*(D+8) bytes]
// viewed as 8-byte elements, box = 16 rows x kvc heads: one tiled copy moves
// a 16-token page tile of a kv group whose heads are a part of each row.
// False unless every rule of the tiled copy holds (16-byte aligned base and
// row stride, box row a multiple of 16 bytes, box within 256 elements, row
// count within the 32-bit coordinate range).
bool encode_pool_map(CUtensorMap* m, const uint8_t* base, int64_t rows, int64_t kv, int64_t D, int kvc) {
  auto enc = tensor_map_encoder();
  const int64_t slot = D + 8;
  if (!enc || reinterpret_cast<uintptr_t>(base) % 16 != 0 || slot % 8 != 0) return false;
  if ((kv * slot) % 16 != 0 || (kvc * slot) % 16 != 0 || kvc * slot / 8 > 256) return false;
  if (rows < 16 || rows > INT32_MAX) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)(kv * slot / 8), (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(kv * slot)};
  const cuuint32_t box[2] = {(cuuint32_t)(kvc * slot / 8), (cuuint32_t)kTileTokens};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Swizzled variant of the whole-row page-tile copy (paged mode 4): the pool
// [rows][kv*(D+8) bytes] as 8-byte elements [rows][kv*(D+8)/64][8], box =
// 16 rows x all 64-byte pieces x 8 elements, CU_TENSOR_MAP_SWIZZLE_64B (the
// inner box is exactly the 64-byte swizzle span).  Same bytes as the bulk
// copy of mode 0, with the 16-byte chunks of each 64-byte piece permuted as
// swz64 undoes.  False unless the row is a whole number of 64-byte pieces
// (at most 256 of them), the base is 16-byte aligned and the row count fits
// the 32-bit coordinate.
bool encode_pool_map_swz(CUtensorMap* m, const uint8_t* base, int64_t rows, int64_t kv, int64_t D) {
  auto enc = tensor_map_encoder();
  const int64_t row = kv * (D + 8);
  if (!enc || reinterpret_cast<uintptr_t>(base) % 16 != 0 || row % 64 != 0 || row / 64 > 256) return false;
  if (rows < 16 || rows > INT32_MAX) return false;
  const cuuint64_t dims[3] = {8, (cuuint64_t)(row / 64), (cuuint64_t)rows};
  const cuuint64_t strides[2] = {64, (cuuint64_t)row};
  const cuuint32_t box[3] = {8, (cuuint32_t)(row / 64), (cuuint32_t)kTileTokens};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<uint8_t*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Geometry {
  int G, nt, kvc, ngroups;
  bool pk;  // two tiles share one n-tile (G <= 4)
};

int geometry(int64_t hq, int64_t kv, Geometry* g) {
  if (kv <= 0 || hq <= 0 || hq % kv != 0) return SLMT_ERR_SHAPE;
  const int64_t G = hq / kv;
  if (G > 16) return SLMT_ERR_UNSUPPORTED;
  int kvc = 1;
  for (int c : {8, 4, 2}) {
    if (kv % c == 0) {
      kvc = c;
      break;
    }
  }
  g->G = (int)G;
  g->nt = G <= 8 ? 1 : 2;
  g->pk = G <= 4;
  g->kvc = kvc;
  g->ngroups = (int)(kv / kvc);
  return SLMT_OK;
}

int64_t workspace_floats(int64_t slots, const Geometry& g, int D) {
  return slots * (int64_t)g.kvc * g.G * (D + 2);
}

}  // namespace

// Scratch layout: [segment arrival counters (int32, zero between calls)]
// [partial rows (float) D per head] [partial (m, l) pairs].  The counter
// region is the first workspace_bytes/64 (rounded up to 256) bytes whatever
// the call, so calls of different batch sizes can share one workspace: a
// call's partial rows never land where any call's counters live.  Every
// segment brings at least 264 bytes of partials (one head of D+2 >= 66
// floats), so a workspace that holds a call's partials holds its counters.
int64_t counter_region(int64_t workspace_bytes) { return (workspace_bytes / 64 + 255) / 256 * 256; }

namespace {

int64_t workspace_total(int64_t slots, int64_t segments, const Geometry& g, int D) {
  const int64_t pb = workspace_floats(slots, g, D) * 4;
  int64_t w = (pb + pb / 63 + 1024 + 255) / 256 * 256;
  while (w - counter_region(w) < pb || counter_region(w) < segments * 4) w += 256;
  return w;
}

// Fill pipeline geometry, grid size and scratch pointers; launch both kernels.
int launch_decode(DecodeParams& p, int layout, int D, const Geometry& geo,
                  int64_t chunks_upper, void* workspace, int64_t workspace_bytes,
                  void* out, int out_dtype, int64_t out_seq_stride,
                  int64_t out_head_stride, cudaStream_t st) {
  int dev = 0;
  const int sms = current_device_sms(&dev);
  if (sms <= 0) return SLMT_ERR_CUDA;
  p.G = geo.G;
  p.kvc = geo.kvc;
  // one bulk copy per (sequence, group) when the group's heads are contiguous
  p.q_bulk = (reinterpret_cast<uintptr_t>(p.q) % 16 == 0) && (p.q_head_stride == D) &&
             ((p.q_seq_stride * 2) % 16 == 0);
  p.ngroups = geo.ngroups;
  int stage_bytes;
  if (layout == LAYOUT_PER_CHANNEL)
    stage_bytes = geo.kvc * kChunkTokens * D;
  else
    stage_bytes = kChunkTokens * geo.kvc * (D + 8);
  stage_bytes = round_up(stage_bytes, 128);
  // q is read into registers at a segment start, so one buffer suffices; the
  // per-channel rulers are needed again at the segment end: double buffer.
  const int nqbuf = layout == LAYOUT_PER_CHANNEL ? 2 : 1;
  const int qbuf = round_up(geo.kvc * geo.G * D * 2, 128);
  const int rbuf = layout == LAYOUT_PER_CHANNEL ? round_up(4 * geo.kvc * D * 2, 128) : 0;
  const int stage_offset = round_up(kHeaderBytes + nqbuf * (qbuf + rbuf), 128);
  // swizzled stages start on a 1024-byte boundary: the kernel rounds the
  // stage base up inside 1 KB of extra shared memory (stage sizes are whole
  // KB there: 32 rows of 8*(D+8) bytes at D 64 / 128)
  const bool swz = layout == LAYOUT_PAGED && p.paged_mode == 4;
  if (swz && stage_bytes % 1024 != 0) return SLMT_ERR_UNSUPPORTED;
  const int slack = swz ? 1024 : 0;
  const int want_ctas = ctas_per_sm(geo.kvc, geo.nt);
  const int threads = cta_threads(geo.kvc);
  const int budget = std::min(kSmemPerCtaMax, kSmemPerSm / want_ctas - kSmemReserved);
  int stages = (budget - stage_offset - slack) / stage_bytes;
  stages = std::min(stages, 6);
  if (stages < 2) {
    stages = (kSmemPerCtaMax - stage_offset - slack) / stage_bytes;
    stages = std::min(stages, 6);
    if (stages < 2) return SLMT_ERR_UNSUPPORTED;
  }
  const int smem = stage_offset + stages * stage_bytes + slack;
  p.stages = stages;
  p.stage_bytes = stage_bytes;
  p.qbuf_bytes = qbuf;
  p.rbuf_bytes = rbuf;
  p.nqbuf = nqbuf;
  p.stage_offset = stage_offset;

  DecodeFn fn = decode_fn(D, geo.nt, geo.pk, layout, geo.kvc, p.append != 0, swz);
  const int occ = occupancy(dev, reinterpret_cast<const void*>(fn), threads, smem);
  if (occ <= 0) return SLMT_ERR_CUDA;
  const int64_t per_sm = std::min(occ, ctas_per_sm(geo.kvc, geo.nt));  // keeps the workspace bound
  int64_t nc = (int64_t)sms * per_sm;
  // about kMinChunksPerCta chunks per CTA, but at least one CTA per segment
  // while the grid has room: many short segments then start side by side
  // instead of one after another in a few CTAs
  const int64_t by_work = std::max<int64_t>(
      std::max<int64_t>(1, (chunks_upper + kMinChunksPerCta - 1) / kMinChunksPerCta),
      std::min<int64_t>((int64_t)geo.ngroups * p.num_seqs, chunks_upper));
  nc = std::max<int64_t>(1, std::min(nc, by_work));
  p.num_ctas = (int)nc;

  const int64_t segments = (int64_t)geo.ngroups * p.num_seqs;
  const int64_t slots = nc + segments - 1;
  if (!workspace) return SLMT_ERR_WORKSPACE;
  const int64_t creg = counter_region(workspace_bytes);
  if (creg < segments * 4 || workspace_bytes - creg < workspace_floats(slots, geo, D) * 4)
    return SLMT_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return SLMT_ERR_ALIGN;
  uint8_t* w = reinterpret_cast<uint8_t*>(workspace);
  p.seg_count = reinterpret_cast<int32_t*>(w);
  // SM-aware pieces need exactly two CTAs on every SM: a full grid of a
  // kernel whose registers allow no more than two per SM (8 kv heads, one
  // n-tile), and room for the arrival words after the segment words
  p.sm_weighted = (geo.kvc == 8 && geo.nt == 1 && nc == 2LL * sms && ctas_per_sm(geo.kvc, geo.nt) == 2 &&
                   creg >= (segments + sms + 1) * 4)
                      ? 1
                      : 0;
  p.num_sms = sms;
  p.part_w0 = kPartWeightFirst;
  p.part_w1 = kPartWeightSecond;
  p.seg_cost = kSegStartCost;
  p.sm_ctr = p.seg_count + segments;
  p.part_acc = reinterpret_cast<float*>(w + creg);
  p.part_ml = p.part_acc + slots * (int64_t)geo.kvc * geo.G * D;
  p.out = out;
  p.out_dtype = out_dtype;
  p.out_seq_stride = out_seq_stride;
  p.out_head_stride = out_head_stride;
  p.out_pair = reinterpret_cast<uintptr_t>(out) % (out_dtype == 2 ? 8 : 4) == 0 && out_seq_stride % 2 == 0 &&
               out_head_stride % 2 == 0;
  p.wait_limit_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
  p.debug_stall = g_debug_stall.load(std::memory_order_relaxed);

  // A CTA whose range ends inside a segment waits for the other CTAs that
  // cover it, so all nc CTAs must be resident at once: a cooperative launch
  // guarantees it (and fails up front, instead of stalling, if they cannot
  // be).  nc never exceeds SMs x resident CTAs per SM.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)nc);
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, fn, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return SLMT_ERR_CUDA;
  }
  return launch_status();
}

int check_q(const void* q, int q_dtype, int64_t seq_stride, int64_t head_stride,
            DecodeParams& p) {
  if (!q) return SLMT_ERR_NULL;
  if (q_dtype != SLMT_DTYPE_F16 && q_dtype != SLMT_DTYPE_BF16) return SLMT_ERR_DTYPE;
  if (reinterpret_cast<uintptr_t>(q) % 2 != 0) return SLMT_ERR_ALIGN;
  p.q = q;
  p.q_seq_stride = seq_stride;
  p.q_head_stride = head_stride;
  p.q_bf16 = q_dtype == SLMT_DTYPE_BF16;
  p.q_bulk = 0;  // decided once the head dim and group size are known
  return SLMT_OK;
}

int check_out(const void* out, int out_dtype) {
  if (!out) return SLMT_ERR_NULL;
  if (out_dtype != SLMT_DTYPE_F32 && out_dtype != SLMT_DTYPE_F16 && out_dtype != SLMT_DTYPE_BF16)
    return SLMT_ERR_DTYPE;
  return SLMT_OK;
}

int out_dtype_code(int out_dtype) {
  return out_dtype == SLMT_DTYPE_F32 ? 2 : (out_dtype == SLMT_DTYPE_BF16 ? 1 : 0);
}

int contig_decode(int layout, const void* q, int q_dtype, int64_t q_seq_stride,
                  int64_t q_head_stride, const uint8_t* k_packed,
                  const uint8_t* v_packed, int64_t kv_seq_stride_rows,
                  int64_t s_cap, const uint16_t* r0, const uint16_t* r1,
                  const uint16_t* r2, const uint16_t* r3,
                  int64_t ruler_seq_stride, int use_quant,
                  const int32_t* seq_lens, int64_t seq_len_scalar,
                  int causal_rows, int64_t num_seqs, int64_t hq, int64_t kv,
                  int64_t D, float sm_scale, void* out, int out_dtype,
                  int64_t out_seq_stride, int64_t out_head_stride,
                  void* workspace, int64_t workspace_bytes, int32_t* err_flag,
                  void* stream) {
  if (!valid_head_dim(D)) return SLMT_ERR_HEAD_DIM;
  if (num_seqs < 0 || s_cap < 0 || kv_seq_stride_rows < 0 || ruler_seq_stride < 0)
    return SLMT_ERR_SHAPE;
  Geometry geo;
  int rc = geometry(hq, kv, &geo);
  if (rc != SLMT_OK) return rc;
  if (num_seqs == 0) return SLMT_OK;
  if (num_seqs > INT32_MAX / 2 || s_cap > INT32_MAX / 2) return SLMT_ERR_SHAPE;
  DecodeParams p{};
  rc = check_q(q, q_dtype, q_seq_stride, q_head_stride, p);
  if (rc != SLMT_OK) return rc;
  rc = check_out(out, out_dtype);
  if (rc != SLMT_OK) return rc;
  if (!k_packed || !v_packed) return SLMT_ERR_NULL;
  if (layout == LAYOUT_PER_TOKEN || use_quant) {
    if (!r0 || !r1 || !r2 || !r3) return SLMT_ERR_NULL;
  }
  if (!seq_lens && seq_len_scalar < 0) return SLMT_ERR_SHAPE;
  if (!seq_lens && seq_len_scalar > s_cap) return SLMT_ERR_SHAPE;
  const uintptr_t ka = reinterpret_cast<uintptr_t>(k_packed), va = reinterpret_cast<uintptr_t>(v_packed);
  if (ka % 8 != 0 || va % 8 != 0) return SLMT_ERR_ALIGN;
  const int64_t half = D / 2;
  p.k_codes = k_packed;
  p.v_codes = v_packed;
  p.kv_seq_stride_rows = kv_seq_stride_rows;
  p.s_cap = s_cap;
  p.r0 = r0;
  p.r1 = r1;
  p.r2 = r2;
  p.r3 = r3;
  p.ruler_seq_stride = ruler_seq_stride;
  p.use_quant = use_quant ? 1 : 0;
  p.contig_bulk_ok = (ka % 16 == 0) && (va % 16 == 0) && ((s_cap * half) % 16 == 0) &&
                     ((kv_seq_stride_rows * half) % 16 == 0);
  p.tma_tensor = encode_codes_map(&p.tmap_k, k_packed, num_seqs, kv, s_cap, half, kv_seq_stride_rows, geo.kvc) &&
                 encode_codes_map(&p.tmap_v, v_packed, num_seqs, kv, s_cap, half, kv_seq_stride_rows, geo.kvc);
  // rulers [B, KV, D] fp16: a kv group's rows are one span of kvc*D values
  const bool rul_al = ((reinterpret_cast<uintptr_t>(r0) | reinterpret_cast<uintptr_t>(r1) |
                        reinterpret_cast<uintptr_t>(r2) | reinterpret_cast<uintptr_t>(r3)) % 16 == 0);
  p.rul_bulk = (layout == LAYOUT_PER_CHANNEL) && use_quant && rul_al && ((ruler_seq_stride * 2) % 16 == 0) &&
               ((geo.kvc * D * 2) % 16 == 0);
  p.seq_lens = seq_lens;
  p.seq_len_scalar = (int)seq_len_scalar;
  p.causal_rows = causal_rows ? 1 : 0;
  p.len_cap = (int)s_cap;
  p.num_seqs = (int)num_seqs;
  p.hq = (int)hq;
  p.kv_total = (int)kv;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.err = err_flag;
  const int64_t max_len = seq_lens ? s_cap : std::min<int64_t>(seq_len_scalar, s_cap);
  const int64_t chunks_upper = num_seqs * ((max_len + kChunkTokens - 1) / kChunkTokens) * geo.ngroups;
  return launch_decode(p, layout, (int)D, geo, chunks_upper, workspace, workspace_bytes, out,
                       out_dtype_code(out_dtype), out_seq_stride, out_head_stride,
                       reinterpret_cast<cudaStream_t>(stream));
}

}  // namespace
}  // namespace slmt

using namespace slmt;

extern "C" int slmt_version(void) { return 100; }

extern "C" const char* slmt_status_string(int status) {
  switch (status) {
    case SLMT_OK:
      return "ok";
    case SLMT_ERR_NULL:
      return "a required pointer is NULL";
    case SLMT_ERR_HEAD_DIM:
      return "head_dim must be 64/80/128";
    case SLMT_ERR_SHAPE:
      return "inconsistent sizes";
    case SLMT_ERR_DTYPE:
      return "dtype not accepted";
    case SLMT_ERR_ALIGN:
      return "pointer or stride alignment not met";
    case SLMT_ERR_WORKSPACE:
      return "workspace missing or too small";
    case SLMT_ERR_UNSUPPORTED:
      return "configuration not supported";
    case SLMT_ERR_CUDA:
      return "CUDA runtime error";
    case SLMT_ERR_BLOCK:
      return "BLOCK_N / BLOCK_M rejected";
    case SLMT_ERR_SCRATCH_LIMIT:
      return "request needs more scratch than slmt_paged_decode_noalloc's static array "
             "(SLMT_NOALLOC_SCRATCH_BYTES)";
    default:
      return "unknown status";
  }
}

extern "C" int64_t slmt_set_wait_limit_ns(int64_t ns) {
  const uint64_t v = ns > 0 ? (uint64_t)ns : kDefaultWaitLimitNs;
  return (int64_t)g_wait_limit_ns.exchange(v);
}

extern "C" int slmt_set_debug_stall(int on) { return g_debug_stall.exchange(on ? 1 : 0); }

extern "C" int slmt_device_sm_count(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return SLMT_ERR_CUDA;
  return n;
}

extern "C" int64_t slmt_decode_workspace_bytes(int64_t num_seqs, int64_t num_q_heads,
                                               int64_t num_kv_heads, int64_t head_dim,
                                               int device) {
  if (!valid_head_dim(head_dim)) return SLMT_ERR_HEAD_DIM;
  if (num_seqs < 0) return SLMT_ERR_SHAPE;
  Geometry geo;
  const int rc = geometry(num_q_heads, num_kv_heads, &geo);
  if (rc != SLMT_OK) return rc;
  const int sms = slmt_device_sm_count(device);
  if (sms <= 0) return SLMT_ERR_CUDA;
  const int64_t segments = (int64_t)geo.ngroups * num_seqs;
  const int64_t slots = (int64_t)sms * ctas_per_sm(geo.kvc, geo.nt) + segments;
  return workspace_total(slots, segments, geo, (int)head_dim);
}

namespace slmt {
namespace {

// Shared by slmt_paged_decode and slmt_paged_append_decode (append != 0: one
// new token per sequence, quantized into the cache at position len-1 by the
// decode launch itself).
int paged_decode_impl(
    const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
    const uint8_t* kv_cache, int64_t num_blocks, int64_t block_size,
    int64_t num_kv_heads, int64_t head_dim, const void* block_tables,
    int bt_dtype, int64_t bt_seq_stride, int64_t max_blocks_per_seq,
    const int32_t* seq_lens, int64_t seq_len_scalar, int64_t max_seq_len_hint,
    int64_t num_seqs, int64_t num_q_heads, float sm_scale, void* out,
    int out_dtype, int64_t out_seq_stride, int64_t out_head_stride,
    void* workspace, int64_t workspace_bytes, int32_t* err_flag, void* stream,
    const void* new_key, const void* new_value, int kv_dtype, int64_t new_seq_stride) {
  if (!valid_head_dim(head_dim)) return SLMT_ERR_HEAD_DIM;
  if (num_seqs < 0 || num_blocks < 0 || block_size <= 0 || max_blocks_per_seq < 0)
    return SLMT_ERR_SHAPE;
  Geometry geo;
  int rc = geometry(num_q_heads, num_kv_heads, &geo);
  if (rc != SLMT_OK) return rc;
  if (num_seqs == 0) return SLMT_OK;
  if (num_seqs > INT32_MAX / 2) return SLMT_ERR_SHAPE;
  DecodeParams p{};
  rc = check_q(q, q_dtype, q_seq_stride, q_head_stride, p);
  if (rc != SLMT_OK) return rc;
  rc = check_out(out, out_dtype);
  if (rc != SLMT_OK) return rc;
  if (!kv_cache || !block_tables) return SLMT_ERR_NULL;
  if (bt_dtype != SLMT_DTYPE_I32 && bt_dtype != SLMT_DTYPE_I64) return SLMT_ERR_DTYPE;
  if (num_seqs > 1 && bt_seq_stride < max_blocks_per_seq) return SLMT_ERR_SHAPE;
  const int64_t cap = max_blocks_per_seq * block_size;
  if (cap > INT32_MAX / 2) return SLMT_ERR_SHAPE;
  if (!seq_lens && (seq_len_scalar < 0 || seq_len_scalar > cap)) return SLMT_ERR_SHAPE;
  const uintptr_t ca = reinterpret_cast<uintptr_t>(kv_cache);
  if (ca % 8 != 0) return SLMT_ERR_ALIGN;
  const int64_t slot = head_dim + 8;
  p.cache = kv_cache;
  p.num_blocks = num_blocks;
  p.block_size = (int)block_size;
  p.kv_total = (int)num_kv_heads;
  p.block_tables = block_tables;
  p.bt_i64 = bt_dtype == SLMT_DTYPE_I64;
  p.bt_seq_stride = bt_seq_stride;
  p.max_blocks = (int)max_blocks_per_seq;
  if (geo.kvc == num_kv_heads && block_size % 16 == 0 && ca % 16 == 0)
    // whole rows per page tile; swizzled (bank-conflict-free reads) where the
    // SWZ kernels exist: 8 kv heads per CTA, head dim 64 or 128
    p.paged_mode = (geo.kvc == 8 && (head_dim == 64 || head_dim == 128) &&
                    encode_pool_map_swz(&p.tmap_k, kv_cache, num_blocks * block_size, num_kv_heads, head_dim))
                       ? 4
                       : 0;
  else if (block_size % 16 == 0 &&
           encode_pool_map(&p.tmap_k, kv_cache, num_blocks * block_size, num_kv_heads, head_dim, geo.kvc))
    p.paged_mode = 3;
  else if ((geo.kvc * slot) % 16 == 0 && (num_kv_heads * slot) % 16 == 0 && ca % 16 == 0)
    p.paged_mode = 1;
  else
    p.paged_mode = 2;
  if (new_key || new_value) {
    if (!new_key || !new_value || !seq_lens) return SLMT_ERR_NULL;
    if (kv_dtype != SLMT_DTYPE_F16 && kv_dtype != SLMT_DTYPE_BF16) return SLMT_ERR_DTYPE;
    if (new_seq_stride < num_kv_heads * head_dim) return SLMT_ERR_SHAPE;
    // rows are read two values per 32-bit word
    if ((reinterpret_cast<uintptr_t>(new_key) | reinterpret_cast<uintptr_t>(new_value)) % 4 != 0 ||
        new_seq_stride % 2 != 0)
      return SLMT_ERR_ALIGN;
    p.append = 1;
    p.new_bf16 = kv_dtype == SLMT_DTYPE_BF16;
    p.new_k = new_key;
    p.new_v = new_value;
    p.new_seq_stride = new_seq_stride;
  }
  p.seq_lens = seq_lens;
  p.seq_len_scalar = (int)seq_len_scalar;
  p.causal_rows = 0;
  p.len_cap = (int)cap;
  p.num_seqs = (int)num_seqs;
  p.hq = (int)num_q_heads;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.err = err_flag;
  int64_t max_len = seq_lens ? cap : seq_len_scalar;
  if (seq_lens && max_seq_len_hint > 0) max_len = std::min(max_len, max_seq_len_hint);
  const int64_t chunks_upper = num_seqs * ((max_len + kChunkTokens - 1) / kChunkTokens) * geo.ngroups;
  return launch_decode(p, LAYOUT_PAGED, (int)head_dim, geo, chunks_upper, workspace,
                       workspace_bytes, out, out_dtype_code(out_dtype), out_seq_stride,
                       out_head_stride, reinterpret_cast<cudaStream_t>(stream));
}

}  // namespace
}  // namespace slmt

extern "C" int slmt_paged_decode(
    const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
    const uint8_t* kv_cache, int64_t num_blocks, int64_t block_size,
    int64_t num_kv_heads, int64_t head_dim, const void* block_tables,
    int bt_dtype, int64_t bt_seq_stride, int64_t max_blocks_per_seq,
    const int32_t* seq_lens, int64_t seq_len_scalar, int64_t max_seq_len_hint,
    int64_t num_seqs, int64_t num_q_heads, float sm_scale, void* out,
    int out_dtype, int64_t out_seq_stride, int64_t out_head_stride,
    void* workspace, int64_t workspace_bytes, int32_t* err_flag, void* stream) {
  return paged_decode_impl(q, q_dtype, q_seq_stride, q_head_stride, kv_cache, num_blocks, block_size,
                           num_kv_heads, head_dim, block_tables, bt_dtype, bt_seq_stride, max_blocks_per_seq,
                           seq_lens, seq_len_scalar, max_seq_len_hint, num_seqs, num_q_heads, sm_scale, out,
                           out_dtype, out_seq_stride, out_head_stride, workspace, workspace_bytes, err_flag,
                           stream, nullptr, nullptr, SLMT_DTYPE_F16, 0);
}

extern "C" int slmt_paged_append_decode(
    const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
    const void* new_key, const void* new_value, int kv_dtype, int64_t new_seq_stride,
    uint8_t* kv_cache, int64_t num_blocks, int64_t block_size,
    int64_t num_kv_heads, int64_t head_dim, const void* block_tables,
    int bt_dtype, int64_t bt_seq_stride, int64_t max_blocks_per_seq,
    const int32_t* seq_lens, int64_t max_seq_len_hint, int64_t num_seqs,
    int64_t num_q_heads, float sm_scale, void* out, int out_dtype,
    int64_t out_seq_stride, int64_t out_head_stride, void* workspace,
    int64_t workspace_bytes, int32_t* err_flag, void* stream) {
  if (!new_key || !new_value || !seq_lens) return SLMT_ERR_NULL;
  return paged_decode_impl(q, q_dtype, q_seq_stride, q_head_stride, kv_cache, num_blocks, block_size,
                           num_kv_heads, head_dim, block_tables, bt_dtype, bt_seq_stride, max_blocks_per_seq,
                           seq_lens, 0, max_seq_len_hint, num_seqs, num_q_heads, sm_scale, out, out_dtype,
                           out_seq_stride, out_head_stride, workspace, workspace_bytes, err_flag, stream,
                           new_key, new_value, kv_dtype, new_seq_stride);
}

extern "C" int slmt_per_channel_decode(
    const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
    const uint8_t* k_packed, const uint8_t* v_packed, int64_t kv_seq_stride_rows,
    int64_t s_cap, const uint16_t* k_scale, const uint16_t* k_zero,
    const uint16_t* v_scale, const uint16_t* v_zero, int64_t ruler_seq_stride,
    int use_quant, const int32_t* seq_lens, int64_t seq_len_scalar,
    int causal_rows, int64_t num_seqs, int64_t num_q_heads, int64_t num_kv_heads,
    int64_t head_dim, float sm_scale, void* out, int out_dtype,
    int64_t out_seq_stride, int64_t out_head_stride, void* workspace,
    int64_t workspace_bytes, int32_t* err_flag, void* stream) {
  return contig_decode(LAYOUT_PER_CHANNEL, q, q_dtype, q_seq_stride, q_head_stride, k_packed,
                       v_packed, kv_seq_stride_rows, s_cap, k_scale, k_zero, v_scale, v_zero,
                       ruler_seq_stride, use_quant, seq_lens, seq_len_scalar, causal_rows,
                       num_seqs, num_q_heads, num_kv_heads, head_dim, sm_scale, out, out_dtype,
                       out_seq_stride, out_head_stride, workspace, workspace_bytes, err_flag,
                       stream);
}

extern "C" int slmt_per_token_decode(
    const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
    const uint8_t* k_packed, const uint8_t* v_packed, int64_t kv_seq_stride_rows,
    int64_t s_cap, const uint16_t* k_min, const uint16_t* k_step,
    const uint16_t* v_min, const uint16_t* v_step, const int32_t* seq_lens,
    int64_t seq_len_scalar, int64_t num_seqs, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, float sm_scale, void* out,
    int out_dtype, int64_t out_seq_stride, int64_t out_head_stride,
    void* workspace, int64_t workspace_bytes, int32_t* err_flag, void* stream) {
  // rulers share the codes' row indexing: [seq, kv, s_cap]
  return contig_decode(LAYOUT_PER_TOKEN, q, q_dtype, q_seq_stride, q_head_stride, k_packed,
                       v_packed, kv_seq_stride_rows, s_cap, k_min, k_step, v_min, v_step,
                       kv_seq_stride_rows, 1, seq_lens, seq_len_scalar, 0, num_seqs, num_q_heads,
                       num_kv_heads, head_dim, sm_scale, out, out_dtype, out_seq_stride,
                       out_head_stride, workspace, workspace_bytes, err_flag, stream);
}

extern "C" int slmt_per_channel_prefill(
    const void* q, int q_dtype, int64_t q_head_stride, int64_t q_row_stride,
    const uint8_t* k_packed, const uint8_t* v_packed, int64_t seq_len,
    const uint16_t* k_scale, const uint16_t* k_zero, const uint16_t* v_scale,
    const uint16_t* v_zero, int use_quant, int causal, int64_t num_rows,
    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, float sm_scale,
    void* out, int out_dtype, int64_t out_head_stride, int64_t out_row_stride,
    void* workspace, int64_t workspace_bytes, int32_t* err_flag, void* stream) {
  // M-tiled kernel (prefill.cu): needs no split-K workspace and sets no error
  // bits (every read is bounded by seq_len); both arguments are accepted for
  // the signature's sake.
  (void)workspace;
  (void)workspace_bytes;
  (void)err_flag;
  if (!valid_head_dim(head_dim)) return SLMT_ERR_HEAD_DIM;
  if (seq_len < 0 || num_rows < 0 || seq_len > INT32_MAX / 2 || num_rows > INT32_MAX / 2) return SLMT_ERR_SHAPE;
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads != 0) return SLMT_ERR_SHAPE;
  if (num_q_heads > 65535) return SLMT_ERR_UNSUPPORTED;
  if (num_rows == 0) return SLMT_OK;
  if (!q || !out) return SLMT_ERR_NULL;
  // with no keys (seq_len 0) every row is zero and codes/rulers are not read
  if (seq_len > 0 && (!k_packed || !v_packed)) return SLMT_ERR_NULL;
  if (seq_len > 0 && use_quant && (!k_scale || !k_zero || !v_scale || !v_zero)) return SLMT_ERR_NULL;
  if (q_dtype != SLMT_DTYPE_F16 && q_dtype != SLMT_DTYPE_BF16) return SLMT_ERR_DTYPE;
  if (out_dtype != SLMT_DTYPE_F32 && out_dtype != SLMT_DTYPE_F16 && out_dtype != SLMT_DTYPE_BF16)
    return SLMT_ERR_DTYPE;
  // codes are copied in 8-byte pieces (rows of D/2 bytes are whole pieces),
  // q read two elements at a time
  if (reinterpret_cast<uintptr_t>(k_packed) % 8 != 0 || reinterpret_cast<uintptr_t>(v_packed) % 8 != 0 ||
      reinterpret_cast<uintptr_t>(q) % 2 != 0)
    return SLMT_ERR_ALIGN;
  return prefill_pc_launch(q, q_dtype == SLMT_DTYPE_BF16, q_head_stride, q_row_stride, k_packed, v_packed,
                           seq_len, k_scale, k_zero, v_scale, v_zero, use_quant, causal, num_rows, num_q_heads,
                           num_kv_heads, head_dim, sm_scale, out, out_dtype_code(out_dtype), out_head_stride,
                           out_row_stride, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int slmt_paged_prefill(
    const void* q, int q_dtype, int64_t q_row_stride, int64_t q_head_stride,
    const uint8_t* kv_cache, int64_t num_blocks, int64_t block_size,
    int64_t num_kv_heads, int64_t head_dim, const void* block_tables,
    int bt_dtype, int64_t bt_seq_stride, int64_t max_blocks_per_seq,
    const int32_t* query_start_loc, const int32_t* seq_lens, int64_t num_reqs,
    int64_t max_query_len, int64_t num_q_heads, float sm_scale, void* out,
    int out_dtype, int64_t out_row_stride, int64_t out_head_stride,
    int32_t* err_flag, void* stream) {
  if (!valid_head_dim(head_dim)) return SLMT_ERR_HEAD_DIM;
  if (num_reqs < 0 || max_query_len < 0 || num_blocks < 0 || block_size <= 0 || max_blocks_per_seq < 0)
    return SLMT_ERR_SHAPE;
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads != 0) return SLMT_ERR_SHAPE;
  if (num_q_heads > 65535 || num_reqs > 65535) return SLMT_ERR_UNSUPPORTED;
  if (max_query_len > INT32_MAX / 2) return SLMT_ERR_SHAPE;
  if (num_reqs == 0 || max_query_len == 0) return SLMT_OK;
  if (!q || !out || !kv_cache || !block_tables || !query_start_loc || !seq_lens) return SLMT_ERR_NULL;
  if (q_dtype != SLMT_DTYPE_F16 && q_dtype != SLMT_DTYPE_BF16) return SLMT_ERR_DTYPE;
  if (out_dtype != SLMT_DTYPE_F32 && out_dtype != SLMT_DTYPE_F16 && out_dtype != SLMT_DTYPE_BF16)
    return SLMT_ERR_DTYPE;
  if (bt_dtype != SLMT_DTYPE_I32 && bt_dtype != SLMT_DTYPE_I64) return SLMT_ERR_DTYPE;
  if (num_reqs > 1 && bt_seq_stride < max_blocks_per_seq) return SLMT_ERR_SHAPE;
  if (max_blocks_per_seq * block_size > INT32_MAX / 2) return SLMT_ERR_SHAPE;
  // slot rows are read as 4-byte code words and one 8-byte ruler quad
  if (reinterpret_cast<uintptr_t>(kv_cache) % 8 != 0 || reinterpret_cast<uintptr_t>(q) % 2 != 0)
    return SLMT_ERR_ALIGN;
  return prefill_paged_launch(q, q_dtype == SLMT_DTYPE_BF16, q_row_stride, q_head_stride, kv_cache, num_blocks,
                              block_size, num_kv_heads, head_dim, block_tables, bt_dtype == SLMT_DTYPE_I64,
                              bt_seq_stride, max_blocks_per_seq, query_start_loc, seq_lens, num_reqs, max_query_len,
                              num_q_heads, sm_scale, out, out_dtype_code(out_dtype), out_row_stride, out_head_stride,
                              err_flag, reinterpret_cast<cudaStream_t>(stream));
}
