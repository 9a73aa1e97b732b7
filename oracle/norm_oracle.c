/*
 * norm_oracle.c -- CPU restatement of the reference's normalisation math.
 *
 * TEST INFRASTRUCTURE. This is the checker the CUDA kernels are compared
 * against, and the CPU baseline that bench.py times. Nothing in the shipped
 * package links or calls it.
 *
 * The math follows the reference's PyTorch oracle, sm120_rmsnorm/reference.py
 * (paths relative to the reference project), operation by operation, with the
 * rounding that PyTorch's CPU kernels apply:
 *   - every fp32 product / sum / difference is rounded to fp32 on its own
 *     (PyTorch evaluates x.float() * inv_rms * weight as separate tensor ops);
 *   - mean(v) is sum(v) / n (PyTorch's CPU mean), and rsqrt(v) is the IEEE
 *     fp32 1 / sqrt(v): correctly rounded sqrt and divide. PyTorch's
 *     vectorised CPU sqrt / rsqrt are not correctly rounded on every build
 *     (on AVX-512 about 0.5% of results differ from it in the last bit), so
 *     the IEEE form is the reproducible reading of the reference's formula;
 *   - fp32 -> bf16 / fp16 conversions round to nearest even;
 *   - the file is compiled with -ffp-contract=off and without fast-math, so
 *     no product is fused into an FMA and no sum is reassociated;
 *   - sums of squares accumulate in fp32. PyTorch's vectorised cascade sum has
 *     an ISA-dependent order that is not restated; this file sums in a
 *     16-lane x 4-accumulator tree, so the fp32 sum can differ from PyTorch's
 *     in its last bits and an output can differ by one ulp of its dtype.
 *
 * Threads: rows (or tokens) are split across OpenMP threads; see
 * oracle_set_threads().
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { ORACLE_F32 = 0, ORACLE_F16 = 1, ORACLE_BF16 = 2 };

static int g_threads = 1;

void oracle_set_threads(int n) { g_threads = n > 0 ? n : 1; }
int oracle_get_threads(void) { return g_threads; }

/* ---- element conversions -------------------------------------------------- */

static inline float bf16_bits_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

/* Round to nearest, ties to even; NaN maps to the canonical quiet NaN. */
static inline uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0u;
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float load_elem(const void* base, int64_t i, int dtype) {
  switch (dtype) {
    case ORACLE_F16: return (float)((const _Float16*)base)[i];
    case ORACLE_BF16: return bf16_bits_to_f32(((const uint16_t*)base)[i]);
    default: return ((const float*)base)[i];
  }
}

static inline void store_elem(void* base, int64_t i, int dtype, float v) {
  switch (dtype) {
    case ORACLE_F16: ((_Float16*)base)[i] = (_Float16)v; break;
    case ORACLE_BF16: ((uint16_t*)base)[i] = f32_to_bf16_bits(v); break;
    default: ((float*)base)[i] = v; break;
  }
}

/* Value after a round trip through the storage dtype ("tensor.to(dtype)"). */
static inline float round_to(float v, int dtype) {
  switch (dtype) {
    case ORACLE_F16: return (float)(_Float16)v;
    case ORACLE_BF16: return bf16_bits_to_f32(f32_to_bf16_bits(v));
    default: return v;
  }
}

static inline size_t elem_size(int dtype) { return dtype == ORACLE_F32 ? 4 : 2; }

/* fp32 sum of squares: 16 lanes x 4 accumulators, then a pairwise tree. The
 * squares are rounded before they are added (x.float().square() is its own
 * tensor op in the reference). */
static float sum_squares(const float* v, int64_t n) {
  enum { LANES = 16, ACCS = 4, BLOCK = LANES * ACCS };
  float acc[ACCS][LANES];
  memset(acc, 0, sizeof acc);
  int64_t full = n / BLOCK * BLOCK;
  for (int64_t i = 0; i < full; i += BLOCK)
    for (int a = 0; a < ACCS; ++a)
      for (int l = 0; l < LANES; ++l) {
        float sq = v[i + a * LANES + l] * v[i + a * LANES + l];
        acc[a][l] += sq;
      }
  float lane[LANES];
  for (int l = 0; l < LANES; ++l) {
    float s = acc[0][l];
    for (int a = 1; a < ACCS; ++a) s += acc[a][l];
    lane[l] = s;
  }
  for (int width = LANES / 2; width > 0; width /= 2)
    for (int l = 0; l < width; ++l) lane[l] += lane[l + width];
  float total = lane[0];
  for (int64_t i = full; i < n; ++i) {
    float sq = v[i] * v[i];
    total += sq;
  }
  return total;
}

/* rsqrt(mean(v^2) + eps) in IEEE fp32
 * (reference.py:10, :22; F.rms_norm at :38-40). */
static float inv_rms(const float* v, int64_t n, float eps) {
  float mean = sum_squares(v, n) / (float)n;
  float shifted = mean + eps;
  float root = sqrtf(shifted);
  return 1.0f / root;
}

/* ---- RMSNorm: reference.py:5-11 ------------------------------------------- */

int oracle_rms_norm(const void* x, const void* w, void* y, int64_t rows,
                    int64_t hidden, int dtype, float eps) {
  if (rows < 0 || hidden <= 0) return 1;
#pragma omp parallel num_threads(g_threads)
  {
    float* row = (float*)malloc(sizeof(float) * (size_t)hidden);
#pragma omp for schedule(static)
    for (int64_t i = 0; i < rows; ++i) {
      const int64_t base = i * hidden;
      for (int64_t j = 0; j < hidden; ++j) row[j] = load_elem(x, base + j, dtype);
      const float inv = inv_rms(row, hidden, eps);
      for (int64_t j = 0; j < hidden; ++j) {
        float scaled = row[j] * inv;        /* x.float() * inv_rms */
        float out = scaled * load_elem(w, j, dtype); /* ... * weight.float() */
        store_elem(y, base + j, dtype, out);         /* .to(x.dtype) */
      }
    }
    free(row);
  }
  return 0;
}

/* ---- residual add + RMSNorm: reference.py:14-24 --------------------------- */

int oracle_fused_add_rms_norm(const void* x, const void* r, const void* w,
                              void* out, void* r_out, int64_t rows,
                              int64_t hidden, int dtype, float eps) {
  if (rows < 0 || hidden <= 0) return 1;
#pragma omp parallel num_threads(g_threads)
  {
    float* row = (float*)malloc(sizeof(float) * (size_t)hidden);
#pragma omp for schedule(static)
    for (int64_t i = 0; i < rows; ++i) {
      const int64_t base = i * hidden;
      /* residual_out = x + residual, in the activation dtype (:20) */
      for (int64_t j = 0; j < hidden; ++j) {
        float s = load_elem(x, base + j, dtype) + load_elem(r, base + j, dtype);
        row[j] = round_to(s, dtype);
      }
      const float inv = inv_rms(row, hidden, eps);
      for (int64_t j = 0; j < hidden; ++j) {
        float scaled = row[j] * inv;
        float o = scaled * load_elem(w, j, dtype);
        store_elem(r_out, base + j, dtype, row[j]);
        store_elem(out, base + j, dtype, o);
      }
    }
    free(row);
  }
  return 0;
}

/* ---- per-head Q/K RMSNorm + half-split RoPE: reference.py:27-49 ----------- */

/* One head of head_dim values at `head`, in place. */
static void norm_rope_head(void* t, int64_t head, const void* w,
                           const float* cs_row, int64_t head_dim, int dtype,
                           float eps, float* tmp) {
  const int64_t half = head_dim / 2;
  for (int64_t j = 0; j < head_dim; ++j) tmp[j] = load_elem(t, head + j, dtype);
  const float inv = inv_rms(tmp, head_dim, eps);
  for (int64_t j = 0; j < head_dim; ++j) {
    /* F.rms_norm(x.float()).to(dtype) (:38-40), then * weight in dtype (:41) */
    float normed = tmp[j] * inv;
    float weighted = round_to(normed, dtype) * load_elem(w, j, dtype);
    tmp[j] = round_to(weighted, dtype);
  }
  for (int64_t j = 0; j < half; ++j) {
    const float c = cs_row[j], s = cs_row[half + j];
    float a = tmp[j] * c, b = tmp[half + j] * s;   /* first*cos, second*sin */
    float d = tmp[half + j] * c, e = tmp[j] * s;   /* second*cos, first*sin */
    float lo = a - b;                                       /* :45 */
    float hi = d + e;                                       /* :46 */
    store_elem(t, head + j, dtype, lo);
    store_elem(t, head + half + j, dtype, hi);
  }
}

static int qk_common(void* q, void* k, const void* v, const void* qw,
                     const void* kw, const int64_t* pos, const float* cs,
                     void* kc, void* vc, const int32_t* slots, int64_t tokens,
                     int64_t hq, int64_t hk, int64_t head_dim,
                     int64_t rope_positions, int64_t cache_slots, int dtype,
                     float eps) {
  if (tokens < 0 || hq < 0 || hk < 0 || head_dim <= 0 || (head_dim & 1)) return 1;
  const size_t es = elem_size(dtype);
#pragma omp parallel num_threads(g_threads)
  {
    float* tmp = (float*)malloc(sizeof(float) * (size_t)head_dim);
#pragma omp for schedule(static)
    for (int64_t t = 0; t < tokens; ++t) {
      const int64_t p = pos[t];
      /* Positions outside the cache leave the token untouched (the reference
       * CUDA kernel reads out of bounds there; torch indexing raises). */
      if (p < 0 || p >= rope_positions) continue;
      const float* row = cs + p * head_dim;
      for (int64_t h = 0; h < hq; ++h)
        norm_rope_head(q, (t * hq + h) * head_dim, qw, row, head_dim, dtype, eps, tmp);
      for (int64_t h = 0; h < hk; ++h)
        norm_rope_head(k, (t * hk + h) * head_dim, kw, row, head_dim, dtype, eps, tmp);
      if (kc == NULL) continue;
      const int64_t slot = slots[t];
      if (slot < 0 || slot >= cache_slots) continue;
      /* The reference kernel's KV store, csrc/rmsnorm_kernels.cu:425-435:
       * rotated K and unmodified V are copied bit for bit. */
      const size_t head_bytes = (size_t)(hk * head_dim) * es;
      memcpy((char*)kc + (size_t)slot * head_bytes, (const char*)k + (size_t)t * head_bytes, head_bytes);
      memcpy((char*)vc + (size_t)slot * head_bytes, (const char*)v + (size_t)t * head_bytes, head_bytes);
    }
    free(tmp);
  }
  return 0;
}

int oracle_qk_rms_norm_rope(void* q, void* k, const void* qw, const void* kw,
                            const int64_t* pos, const float* cs, int64_t tokens,
                            int64_t hq, int64_t hk, int64_t head_dim,
                            int64_t rope_positions, int dtype, float eps) {
  return qk_common(q, k, NULL, qw, kw, pos, cs, NULL, NULL, NULL, tokens, hq,
                   hk, head_dim, rope_positions, 0, dtype, eps);
}

int oracle_qk_rms_norm_rope_kv(void* q, void* k, const void* v, const void* qw,
                               const void* kw, const int64_t* pos,
                               const float* cs, void* kc, void* vc,
                               const int32_t* slots, int64_t tokens, int64_t hq,
                               int64_t hk, int64_t head_dim,
                               int64_t rope_positions, int64_t cache_slots,
                               int dtype, float eps) {
  if (kc == NULL || vc == NULL || slots == NULL || v == NULL) return 1;
  return qk_common(q, k, v, qw, kw, pos, cs, kc, vc, slots, tokens, hq, hk,
                   head_dim, rope_positions, cache_slots, dtype, eps);
}
