/*
 * kvq_oracle.c -- CPU restatement of slm-turbo's 4-bit KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py load this code, and only
 * as the checker (or as the timed CPU baseline).  The product path never
 * calls it.
 *
 * Every function restates one piece of the reference (paths inside the
 * slm-turbo project):
 *   oracle_kv_store          kv_quantize_store_kernel,
 *                            kernels/kv_dequant_kernels.cuh:816-919
 *   oracle_pc_scale_zero     compute_scale_zero,
 *                            kernels/benchmark/benchmark.py:26-42
 *   oracle_pc_codes          quantize_tensor, benchmark.py:45-56
 *   oracle_paged_decode      kv_dequant_decode_per_token_paged_kernel,
 *                            kernels/kv_dequant_kernels.cuh:671-801
 *   oracle_pc_decode         kv_dequant_decode_kernel .cuh:113-275 and, with
 *                            causal rows, kv_dequant_prefill_kernel .cuh:293-502
 *   oracle_pt_decode         kv_dequant_decode_per_token_kernel .cuh:528-655
 *
 * Quantizers are evaluated in IEEE fp32 / fp16 exactly as the reference
 * evaluates them (compile with -ffp-contract=off, no -ffast-math): codes and
 * rulers must be bit-exact.  Attention is evaluated in double precision from
 * the exact dequantized values (code*step+min, (code-zero)*scale), with scale
 * 1/sqrt(D) chosen by the caller, so it is a tighter answer than either
 * GPU implementation and is compared with a tolerance.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- fp16 / bf16 conversions (IEEE round-to-nearest-even) --------------- */
static inline float h2f(uint16_t b) {
  _Float16 h;
  memcpy(&h, &b, 2);
  return (float)h;
}
static inline uint16_t f2h(float f) {
  _Float16 h = (_Float16)f;
  uint16_t b;
  memcpy(&b, &h, 2);
  return b;
}
static inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
/* one fp16 tensor op as torch evaluates it: fp32 result rounded to fp16 */
static inline float h16(float x) { return h2f(f2h(x)); }

/* min/max as the GPU min.f32/max.f32 order signed zeros (-0 < +0) */
static inline float fmin0(float a, float b) {
  if (a < b) return a;
  if (b < a) return b;
  if (a != a) return b;
  if (b != b) return a;
  return signbit(a) ? a : b;
}
static inline float fmax0(float a, float b) {
  if (a > b) return a;
  if (b > a) return b;
  if (a != a) return b;
  if (b != b) return a;
  return signbit(a) ? b : a;
}

int oracle_version(void) { return 1; }

/* ---- per-token quantize-on-write (.cuh:816-919) -------------------------- */
void oracle_kv_store(const uint16_t* key, const uint16_t* value, int in_bf16,
                     int64_t tok_stride, int64_t n_tok, int64_t kv, int64_t d,
                     uint8_t* cache, int64_t num_slots,
                     const int64_t* slot_mapping) {
  const int64_t slot_bytes = d + 8;
  for (int64_t t = 0; t < n_tok; ++t) {
    const int64_t slot = slot_mapping[t];
    if (slot < 0 || slot >= num_slots) continue; /* ref: skip padding */
    for (int64_t h = 0; h < kv; ++h) {
      const uint16_t* rows[2] = {key + t * tok_stride + h * d, value + t * tok_stride + h * d};
      uint8_t* base = cache + (slot * kv + h) * slot_bytes;
      float mins[2], steps[2];
      for (int w = 0; w < 2; ++w) {
        float mn = INFINITY, mx = -INFINITY;
        for (int64_t i = 0; i < d; ++i) {
          const float x = in_bf16 ? bf2f(rows[w][i]) : h2f(rows[w][i]);
          mn = fmin0(mn, x);
          mx = fmax0(mx, x);
        }
        float step = (mx - mn) / 15.0f;
        if (!(step > 0.0f)) step = 1.0f;
        for (int64_t j = 0; j < d / 2; ++j) {
          const float x0 = in_bf16 ? bf2f(rows[w][2 * j]) : h2f(rows[w][2 * j]);
          const float x1 = in_bf16 ? bf2f(rows[w][2 * j + 1]) : h2f(rows[w][2 * j + 1]);
          const float f0 = (x0 - mn) / step + 0.5f;
          const float f1 = (x1 - mn) / step + 0.5f;
          int q0 = (int)f0, q1 = (int)f1;
          q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
          q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
          base[w * (d / 2) + j] = (uint8_t)(q0 | (q1 << 4));
        }
        mins[w] = mn;
        steps[w] = step;
      }
      uint16_t r[4] = {f2h(mins[0]), f2h(steps[0]), f2h(mins[1]), f2h(steps[1])};
      memcpy(base + d, r, 8);
    }
  }
}

/* ---- per-channel rulers (benchmark.py:26-42), fp16 tensor arithmetic ---- */
void oracle_pc_scale_zero(const uint16_t* x, int64_t rows, int64_t s_len,
                          int64_t d, uint16_t* scale, uint16_t* zero) {
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t c = 0; c < d; ++c) {
      float mn = INFINITY, mx = -INFINITY;
      for (int64_t s = 0; s < s_len; ++s) {
        const float v = h2f(x[(r * s_len + s) * d + c]);
        mn = fmin0(mn, v);
        mx = fmax0(mx, v);
      }
      float sc = h16(h16(mx - mn) / 15.0f);
      float zp = h16(0.0f - rintf(h16(mn / sc)));
      if (mx == mn) {
        sc = 1.0f;
        zp = 0.0f;
      }
      zp = fminf(fmaxf(zp, 0.0f), 15.0f);
      scale[r * d + c] = f2h(sc);
      zero[r * d + c] = f2h(zp);
    }
  }
}

static inline uint32_t pc_code(float x, float sc, float zp) {
  float q = h16(rintf(h16(x / sc)) + zp);
  if (q != q) return 0u;
  q = fminf(fmaxf(q, 0.0f), 15.0f);
  return (uint32_t)q;
}

/* ---- per-channel codes (benchmark.py:45-56); also the frozen-ruler append -- */
void oracle_pc_codes(const uint16_t* x, int64_t rows, int64_t s_len, int64_t d,
                     const uint16_t* scale, const uint16_t* zero,
                     uint8_t* packed) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t s = 0; s < s_len; ++s)
      for (int64_t j = 0; j < d / 2; ++j) {
        const uint16_t* xr = x + (r * s_len + s) * d;
        const uint32_t c0 = pc_code(h2f(xr[2 * j]), h2f(scale[r * d + 2 * j]), h2f(zero[r * d + 2 * j]));
        const uint32_t c1 =
            pc_code(h2f(xr[2 * j + 1]), h2f(scale[r * d + 2 * j + 1]), h2f(zero[r * d + 2 * j + 1]));
        packed[(r * s_len + s) * (d / 2) + j] = (uint8_t)(c0 | (c1 << 4));
      }
}

/* ---- attention over one kv head's dequantized rows, G query heads -------- */
static void attend(const float* kd, const float* vd, int64_t len, int64_t d,
                   const double* qv, int64_t g, double sm_scale, double* sc,
                   float* out, int64_t out_head_stride) {
  for (int64_t h = 0; h < g; ++h) {
    const double* qh = qv + h * d;
    double m = -INFINITY;
    for (int64_t t = 0; t < len; ++t) {
      double s = 0.0;
      const float* kr = kd + t * d;
      for (int64_t i = 0; i < d; ++i) s += qh[i] * (double)kr[i];
      s *= sm_scale;
      sc[t] = s;
      if (s > m) m = s;
    }
    double l = 0.0;
    for (int64_t t = 0; t < len; ++t) {
      sc[t] = exp(sc[t] - m);
      l += sc[t];
    }
    float* o = out + h * out_head_stride;
    for (int64_t i = 0; i < d; ++i) {
      double a = 0.0;
      for (int64_t t = 0; t < len; ++t) a += sc[t] * (double)vd[t * d + i];
      o[i] = (float)(a / l);
    }
  }
}

static inline double qval(const uint16_t* q, int q_bf16, int64_t off) {
  return q_bf16 ? (double)bf2f(q[off]) : (double)h2f(q[off]);
}

static inline int64_t bt_entry(const void* bt, int bt_i64, int64_t idx) {
  return bt_i64 ? ((const int64_t*)bt)[idx] : (int64_t)((const int32_t*)bt)[idx];
}

/* ---- paged per-token decode (.cuh:671-801), batched --------------------- */
void oracle_paged_decode(const uint16_t* q, int q_bf16, int64_t q_seq_stride,
                         int64_t q_head_stride, const uint8_t* cache,
                         int64_t block_size, int64_t kv, int64_t d,
                         const void* bt, int bt_i64, int64_t bt_stride,
                         const int32_t* seq_lens, int64_t n_seq, int64_t hq,
                         double sm_scale, float* out, int nthreads) {
  const int64_t g = hq / kv, slot_bytes = d + 8;
  int64_t lmax = 0;
  for (int64_t b = 0; b < n_seq; ++b)
    if (seq_lens[b] > lmax) lmax = seq_lens[b];
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    float* kd = (float*)malloc(sizeof(float) * (size_t)(lmax + 1) * d);
    float* vd = (float*)malloc(sizeof(float) * (size_t)(lmax + 1) * d);
    double* sc = (double*)malloc(sizeof(double) * (size_t)(lmax + 1));
    double* qv = (double*)malloc(sizeof(double) * (size_t)g * d);
#pragma omp for collapse(2) schedule(dynamic)
    for (int64_t b = 0; b < n_seq; ++b) {
      for (int64_t h = 0; h < kv; ++h) {
        const int64_t len = seq_lens[b];
        float* ob = out + (b * hq + h * g) * d;
        if (len <= 0) {
          memset(ob, 0, sizeof(float) * (size_t)(g * d));
          continue;
        }
        for (int64_t t = 0; t < len; ++t) {
          const int64_t phys = bt_entry(bt, bt_i64, b * bt_stride + t / block_size);
          const uint8_t* sl = cache + ((phys * block_size + t % block_size) * kv + h) * slot_bytes;
          uint16_t r[4];
          memcpy(r, sl + d, 8);
          const double kmin = h2f(r[0]), kstep = h2f(r[1]), vmin = h2f(r[2]), vstep = h2f(r[3]);
          for (int64_t j = 0; j < d / 2; ++j) {
            const uint8_t kb = sl[j], vb = sl[d / 2 + j];
            kd[t * d + 2 * j] = (float)((kb & 15) * kstep + kmin);
            kd[t * d + 2 * j + 1] = (float)((kb >> 4) * kstep + kmin);
            vd[t * d + 2 * j] = (float)((vb & 15) * vstep + vmin);
            vd[t * d + 2 * j + 1] = (float)((vb >> 4) * vstep + vmin);
          }
        }
        for (int64_t hh = 0; hh < g; ++hh)
          for (int64_t i = 0; i < d; ++i)
            qv[hh * d + i] = qval(q, q_bf16, b * q_seq_stride + (h * g + hh) * q_head_stride + i);
        attend(kd, vd, len, d, qv, g, sm_scale, sc, ob, d);
      }
    }
    free(kd);
    free(vd);
    free(sc);
    free(qv);
  }
}

/* ---- per-channel decode / prefill rows (.cuh:113-275, :293-502) ---------- */
/* codes [n_seq or 1, kv, s_cap, d/2] (seq stride kv_seq_rows rows), rulers
 * [., kv, d] (seq stride ruler_seq); q element (b, h, i) at
 * q[b*q_seq_stride + h*q_head_stride + i]; out (b, h, i) at
 * out[b*out_seq_stride + h*out_head_stride + i].  causal_rows: length of row
 * b is min(len, b+1).  use_quant=0 reads raw nibbles. */
void oracle_pc_decode(const uint16_t* q, int q_bf16, int64_t q_seq_stride,
                      int64_t q_head_stride, const uint8_t* kp,
                      const uint8_t* vp, int64_t kv_seq_rows, int64_t s_cap,
                      const uint16_t* ks, const uint16_t* kz,
                      const uint16_t* vs, const uint16_t* vz,
                      int64_t ruler_seq, int use_quant,
                      const int32_t* seq_lens, int64_t len_scalar,
                      int causal_rows, int64_t n_seq, int64_t hq, int64_t kv,
                      int64_t d, double sm_scale, float* out,
                      int64_t out_seq_stride, int64_t out_head_stride,
                      int nthreads) {
  const int64_t g = hq / kv;
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    float* kd = (float*)malloc(sizeof(float) * (size_t)(s_cap + 1) * d);
    float* vd = (float*)malloc(sizeof(float) * (size_t)(s_cap + 1) * d);
    double* sc = (double*)malloc(sizeof(double) * (size_t)(s_cap + 1));
    double* qv = (double*)malloc(sizeof(double) * (size_t)g * d);
#pragma omp for collapse(2) schedule(dynamic)
    for (int64_t b = 0; b < n_seq; ++b) {
      for (int64_t h = 0; h < kv; ++h) {
        int64_t len = seq_lens ? seq_lens[b] : len_scalar;
        if (causal_rows && b + 1 < len) len = b + 1;
        float* ob = out + b * out_seq_stride + h * g * out_head_stride;
        if (len <= 0) {
          for (int64_t hh = 0; hh < g; ++hh) memset(ob + hh * out_head_stride, 0, sizeof(float) * (size_t)d);
          continue;
        }
        const uint8_t* kr0 = kp + (b * kv_seq_rows + h * s_cap) * (d / 2);
        const uint8_t* vr0 = vp + (b * kv_seq_rows + h * s_cap) * (d / 2);
        const int64_t ro = b * ruler_seq + h * d;
        for (int64_t t = 0; t < len; ++t)
          for (int64_t j = 0; j < d; ++j) {
            const uint8_t kb = kr0[t * (d / 2) + j / 2], vb = vr0[t * (d / 2) + j / 2];
            const double kc = (j & 1) ? (kb >> 4) : (kb & 15);
            const double vc = (j & 1) ? (vb >> 4) : (vb & 15);
            if (use_quant) {
              kd[t * d + j] = (float)((kc - h2f(kz[ro + j])) * h2f(ks[ro + j]));
              vd[t * d + j] = (float)((vc - h2f(vz[ro + j])) * h2f(vs[ro + j]));
            } else {
              kd[t * d + j] = (float)kc;
              vd[t * d + j] = (float)vc;
            }
          }
        for (int64_t hh = 0; hh < g; ++hh)
          for (int64_t i = 0; i < d; ++i)
            qv[hh * d + i] = qval(q, q_bf16, b * q_seq_stride + (h * g + hh) * q_head_stride + i);
        attend(kd, vd, len, d, qv, g, sm_scale, sc, ob, out_head_stride);
      }
    }
    free(kd);
    free(vd);
    free(sc);
    free(qv);
  }
}

/* ---- contiguous per-token decode (.cuh:528-655) -------------------------- */
void oracle_pt_decode(const uint16_t* q, int q_bf16, int64_t q_seq_stride,
                      int64_t q_head_stride, const uint8_t* kp,
                      const uint8_t* vp, int64_t kv_seq_rows, int64_t s_cap,
                      const uint16_t* kmin, const uint16_t* kstep,
                      const uint16_t* vmin, const uint16_t* vstep,
                      const int32_t* seq_lens, int64_t len_scalar,
                      int64_t n_seq, int64_t hq, int64_t kv, int64_t d,
                      double sm_scale, float* out, int nthreads) {
  const int64_t g = hq / kv;
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    float* kd = (float*)malloc(sizeof(float) * (size_t)(s_cap + 1) * d);
    float* vd = (float*)malloc(sizeof(float) * (size_t)(s_cap + 1) * d);
    double* sc = (double*)malloc(sizeof(double) * (size_t)(s_cap + 1));
    double* qv = (double*)malloc(sizeof(double) * (size_t)g * d);
#pragma omp for collapse(2) schedule(dynamic)
    for (int64_t b = 0; b < n_seq; ++b) {
      for (int64_t h = 0; h < kv; ++h) {
        const int64_t len = seq_lens ? seq_lens[b] : len_scalar;
        float* ob = out + (b * hq + h * g) * d;
        if (len <= 0) {
          memset(ob, 0, sizeof(float) * (size_t)(g * d));
          continue;
        }
        const int64_t row0 = b * kv_seq_rows + h * s_cap;
        for (int64_t t = 0; t < len; ++t) {
          const double k0 = h2f(kmin[row0 + t]), k1 = h2f(kstep[row0 + t]);
          const double v0 = h2f(vmin[row0 + t]), v1 = h2f(vstep[row0 + t]);
          for (int64_t j = 0; j < d; ++j) {
            const uint8_t kb = kp[(row0 + t) * (d / 2) + j / 2], vb = vp[(row0 + t) * (d / 2) + j / 2];
            const double kc = (j & 1) ? (kb >> 4) : (kb & 15);
            const double vc = (j & 1) ? (vb >> 4) : (vb & 15);
            kd[t * d + j] = (float)(kc * k1 + k0);
            vd[t * d + j] = (float)(vc * v1 + v0);
          }
        }
        for (int64_t hh = 0; hh < g; ++hh)
          for (int64_t i = 0; i < d; ++i)
            qv[hh * d + i] = qval(q, q_bf16, b * q_seq_stride + (h * g + hh) * q_head_stride + i);
        attend(kd, vd, len, d, qv, g, sm_scale, sc, ob, d);
      }
    }
    free(kd);
    free(vd);
    free(sc);
    free(qv);
  }
}
