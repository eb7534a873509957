/*
 * astro_oracle.c -- CPU restatement of the reference's sorted-MoE block.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA path
 * (tests/, __graft_entry__.smoke(), and the CPU baseline leg of bench.py).  The
 * product library never links, loads or calls it.
 *
 * Parity status: the small-shape semantics are pinned by the reference's own
 * known-answer tests (ported in tests/test_oracle_kat.py).  The reference's
 * arithmetic runs inside MLX 0.32.1 (Apple Metal), which cannot run on this
 * machine, so reduction orders that MLX leaves open are DEFINED here (marked
 * "defined here") and the CUDA kernels follow the same definitions.
 *
 * Build: oracle/Makefile (gcc -O3 -ffp-contract=off -fopenmp).  fp contraction
 * is off so that every fused multiply-add below is an explicit fmaf().
 */
#include "astro_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* scalar numerics                                                           */
/* ------------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t ao_f32_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float ao_bf16_to_f32(uint16_t h) { return u2f(((uint32_t)h) << 16); }

static inline float rnd_bf16(float f) { return ao_bf16_to_f32(ao_f32_to_bf16(f)); }

/* Half precision helpers (only used to read/write f16 arrays in the small ops). */
static float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
  if (exp == 0) {
    if (man == 0) return u2f(sign);
    float v = ldexpf((float)man, -24);
    return (sign ? -v : v);
  }
  if (exp == 31) return u2f(sign | 0x7f800000u | (man << 13));
  return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

static uint16_t f32_to_f16(float f) {
  uint32_t u = f2u(f), sign = (u >> 16) & 0x8000u;
  float a = fabsf(f);
  if (a != a) return (uint16_t)(sign | 0x7e00u);
  if (a >= 65520.0f) return (uint16_t)(sign | 0x7c00u);
  if (a < 6.103515625e-05f) { /* subnormal: scale to integer units of 2^-24 */
    float s = a * 16777216.0f;
    float r = nearbyintf(s); /* round half even (default rounding mode) */
    return (uint16_t)(sign | (uint32_t)r);
  }
  uint32_t au = f2u(a);
  uint32_t exp = (au >> 23) - 112u, man = au & 0x7fffffu;
  uint32_t h = (exp << 10) | (man >> 13);
  uint32_t rest = man & 0x1fffu;
  if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h += 1u;
  return (uint16_t)(sign | h);
}

static inline float load_dt(const void* p, int dtype, int64_t i) {
  switch (dtype) {
    case AO_BF16: return ao_bf16_to_f32(((const uint16_t*)p)[i]);
    case AO_F16: return f16_to_f32(((const uint16_t*)p)[i]);
    default: return ((const float*)p)[i];
  }
}

static inline float round_dt(float v, int dtype) {
  if (dtype == AO_BF16) return rnd_bf16(v);
  if (dtype == AO_F16) return f16_to_f32(f32_to_f16(v));
  return v;
}

static inline void store_dt(void* p, int dtype, int64_t i, float v) {
  switch (dtype) {
    case AO_BF16: ((uint16_t*)p)[i] = ao_f32_to_bf16(v); break;
    case AO_F16: ((uint16_t*)p)[i] = f32_to_f16(v); break;
    default: ((float*)p)[i] = v; break;
  }
}

/* e^x, defined here (a published method, not a vendor routine): Cody-Waite
 * range reduction x = n*ln2 + r with ln2 split into a 12-significant-bit head
 * (so n*head is exact for |n| < 2^11) and a tail, then the degree-7 Taylor
 * polynomial of e^r on |r| <= ln2/2 evaluated by Horner's rule with fused
 * multiply-adds, then an exact scaling by 2^n.  Truncation error is below 0.1
 * ulp; the routing kernel evaluates the identical sequence so that bf16
 * router probabilities, and hence the selected experts, are bit-identical. */
#define AO_LOG2E 1.44269502162933349609375f       /* float(1/ln 2) */
#define AO_LN2_HI 0.693115234375f                 /* 0x3f317000 */
#define AO_LN2_LO 3.19461833714e-05f              /* 0x3805fdf4 = float(ln2 - hi) */
float ao_expf(float x) {
  if (x != x) return x;
  if (x > 88.72283172607421875f) return INFINITY;
  if (x < -87.0f) return 0.0f; /* results below ~1.6e-38 flush to zero (defined here) */
  float n = nearbyintf(x * AO_LOG2E);
  float r = fmaf(-n, AO_LN2_HI, x);
  r = fmaf(-n, AO_LN2_LO, r);
  float p = u2f(0x39500d01u);         /* 1/7! */
  p = fmaf(p, r, u2f(0x3ab60b61u));   /* 1/6! */
  p = fmaf(p, r, u2f(0x3c088889u));   /* 1/5! */
  p = fmaf(p, r, u2f(0x3d2aaaabu));   /* 1/4! */
  p = fmaf(p, r, u2f(0x3e2aaaabu));   /* 1/3! */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = (int)n;
  if (ni > 127) { p = p * 2.0f; ni -= 1; }
  return p * u2f((uint32_t)(ni + 127) << 23);
}

void ao_expf_batch(const float* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = ao_expf(x[i]);
}

/* MLX's sigmoid: y = 1 / (1 + e^-|x|), result y for x >= 0 and 1 - y for x < 0. */
float ao_sigmoidf(float x) {
  float y = 1.0f / (1.0f + ao_expf(-fabsf(x)));
  return (x < 0.0f) ? 1.0f - y : y;
}

/* ------------------------------------------------------------------------ */
/* accumulation arithmetic of a dot product                                  */
/* ------------------------------------------------------------------------ */

static inline int f_exp(float v) { return (int)((f2u(v) >> 23) & 0xffu) - 127; }

/* 2^e for -1022 <= e <= 1023 */
static inline double pow2d(int e) {
  const uint64_t u = (uint64_t)(e + 1023) << 52;
  double d;
  memcpy(&d, &u, 8);
  return d;
}

/* Tensor-core step (see the header): exact products truncated toward zero at
 * 2^(emax - 25), exact sum, the sum rounded toward zero to 24 bits.  Every term
 * is an integer multiple of the quantum below 2^27 of it, so the double sum of
 * the 17 terms is exact; clearing the low 29 of the sum's 52 stored mantissa
 * bits keeps its 24 leading bits (rounding toward zero).  idx (NULL: 0..15)
 * lists the 16 element positions the step takes. */
static float tc_step_idx(float c, const float* a, const float* b, const int* idx) {
  int emax = -100000;
  for (int i = 0; i < 16; ++i) {
    const int k = idx ? idx[i] : i;
    const int e = (a[k] != 0.0f && b[k] != 0.0f) ? f_exp(a[k]) + f_exp(b[k]) : -100000;
    emax = e > emax ? e : emax;
  }
  if (c != 0.0f && f_exp(c) > emax) emax = f_exp(c);
  if (emax == -100000) return 0.0f;
  const double up = pow2d(25 - emax);
  double sum = 0.0;
  for (int i = 0; i < 16; ++i) {
    const int k = idx ? idx[i] : i;
    sum += trunc((double)a[k] * (double)b[k] * up); /* zero products add 0 */
  }
  if (c != 0.0f) sum += trunc((double)c * up);
  uint64_t u;
  memcpy(&u, &sum, 8);
  u &= ~(((uint64_t)1 << 29) - 1u);
  memcpy(&sum, &u, 8);
  return (float)(sum * pow2d(emax - 25));
}

float ao_tc_step(float c, const float* a, const float* b) { return tc_step_idx(c, a, b, NULL); }

void ao_tc_chain_batch(const float* a, const float* b, const float* c, int64_t count, int64_t n,
                       float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < count; ++i) {
    float acc = c ? c[i] : 0.0f;
    for (int64_t k = 0; k + 16 <= n; k += 16)
      acc = tc_step_idx(acc, a + i * n + k, b + i * n + k, NULL);
    out[i] = acc;
  }
}

/* partial[0] after a butterfly over L lanes (partial[l] + partial[l ^ m]). */
static float butterfly(float* part, int L) {
  for (int m = L / 2; m >= 1; m >>= 1) {
    float nxt[32];
    for (int l = 0; l < L; ++l) nxt[l] = part[l] + part[l ^ m];
    for (int l = 0; l < L; ++l) part[l] = nxt[l];
  }
  return part[0];
}

float ao_dot(const float* a, const float* b, int64_t n, int mode) {
  switch (mode) {
    case AO_DOT_TC: {
      float acc = 0.0f;
      for (int64_t k = 0; k + 16 <= n; k += 16) acc = tc_step_idx(acc, a + k, b + k, NULL);
      return acc;
    }
    case AO_DOT_TC_QUARTERS: {
      static const int kSet[4][16] = {
          {0, 1, 4, 5, 16, 17, 20, 21, 32, 33, 36, 37, 48, 49, 52, 53},
          {2, 3, 6, 7, 18, 19, 22, 23, 34, 35, 38, 39, 50, 51, 54, 55},
          {8, 9, 12, 13, 24, 25, 28, 29, 40, 41, 44, 45, 56, 57, 60, 61},
          {10, 11, 14, 15, 26, 27, 30, 31, 42, 43, 46, 47, 58, 59, 62, 63}};
      const int64_t ql = n / 4;
      float v = 0.0f;
      for (int q = 0; q < 4; ++q) {
        float acc = 0.0f;
        for (int64_t g0 = q * ql; g0 < (q + 1) * ql; g0 += 64)
          for (int s = 0; s < 4; ++s) acc = tc_step_idx(acc, a + g0, b + g0, kSet[s]);
        v = v + acc;
      }
      return v;
    }
    case AO_DOT_SLICES8: {
      const int64_t slen = n / 8, svecs = slen / 8, per_lane = (svecs + 31) / 32;
      float v = 0.0f;
      for (int sl = 0; sl < 8; ++sl) {
        float part[32];
        for (int l = 0; l < 32; ++l) {
          float p = 0.0f;
          for (int64_t kk = 0; kk < per_lane; ++kk) {
            const int64_t vi = kk * 32 + l;
            if (vi >= svecs) continue;
            const int64_t base = sl * slen + vi * 8;
            for (int i = 0; i < 8; ++i) p = fmaf(a[base + i], b[base + i], p);
          }
          part[l] = p;
        }
        v = v + butterfly(part, 32);
      }
      return v;
    }
    case AO_DOT_LANES8: {
      float part[32];
      for (int l = 0; l < 32; ++l) {
        float p = 0.0f;
        for (int64_t c = l; c < n / 8; c += 32)
          for (int i = 0; i < 8; ++i) p = fmaf(a[c * 8 + i], b[c * 8 + i], p);
        part[l] = p;
      }
      return butterfly(part, 32);
    }
    case AO_DOT_DECODE32:
    case AO_DOT_DECODE16: {
      const int L = mode == AO_DOT_DECODE32 ? 32 : 16;
      const int64_t step = 32 * (int64_t)L;
      float part[32];
      for (int l = 0; l < L; ++l) {
        float p = 0.0f;
        for (int64_t s0 = 0; s0 + step <= n; s0 += step)
          for (int c = 0; c < 4; ++c) {
            const int64_t base = s0 + 32 * l + 8 * c;
            for (int i = 0; i < 4; ++i) {
              p = fmaf(a[base + i], b[base + i], p);
              p = fmaf(a[base + i + 4], b[base + i + 4], p);
            }
          }
        part[l] = p;
      }
      return butterfly(part, L);
    }
    case AO_DOT_CHUNK32: {
      const int64_t chunks = n / 32;
      int L = 32;
      while (L > chunks && L > 1) L >>= 1;
      float part[32];
      for (int l = 0; l < L; ++l) {
        float p = 0.0f;
        for (int64_t c = l; c < chunks; c += L)
          for (int j = 0; j < 32; ++j) p = fmaf(a[c * 32 + j], b[c * 32 + j], p);
        part[l] = p;
      }
      return butterfly(part, L);
    }
    default: {
      float acc = 0.0f;
      for (int64_t k = 0; k < n; ++k) acc = fmaf(a[k], b[k], acc);
      return acc;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* a1: dense bf16 projection                                                 */
/* ------------------------------------------------------------------------ */

/* out[r, c] = bf16( sum_k x[r, k] * w[c, k] ), sequential fp32 fmaf over k
 * (accumulation order defined here). */
void ao_matmul_bf16_nt(const uint16_t* x, const uint16_t* w, int64_t rows, int64_t cols,
                       int64_t depth, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t c = 0; c < cols; ++c) {
      float acc = 0.0f;
      for (int64_t k = 0; k < depth; ++k)
        acc = fmaf(ao_bf16_to_f32(x[r * depth + k]), ao_bf16_to_f32(w[c * depth + k]), acc);
      out[r * cols + c] = ao_f32_to_bf16(acc);
    }
  }
}

void ao_matmul_bf16_nt_mode(const uint16_t* x, const uint16_t* w, int64_t rows, int64_t cols,
                            int64_t depth, int mode, uint16_t* out) {
  if (mode == AO_DOT_SEQ) {
    ao_matmul_bf16_nt(x, w, rows, cols, depth, out);
    return;
  }
  float* wf = (float*)malloc(sizeof(float) * (size_t)(cols > 0 ? cols : 1) * (size_t)depth);
  for (int64_t i = 0; i < cols * depth; ++i) wf[i] = ao_bf16_to_f32(w[i]);
#pragma omp parallel
  {
    float* xf = (float*)malloc(sizeof(float) * (size_t)(depth > 0 ? depth : 1));
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      for (int64_t k = 0; k < depth; ++k) xf[k] = ao_bf16_to_f32(x[r * depth + k]);
      for (int64_t c = 0; c < cols; ++c)
        out[r * cols + c] = ao_f32_to_bf16(ao_dot(wf + c * depth, xf, depth, mode));
    }
    free(xf);
  }
  free(wf);
}

/* ------------------------------------------------------------------------ */
/* a2: routing                                                               */
/* ------------------------------------------------------------------------ */

/* One token.  softmax(precise) over E in fp32, probabilities rounded to the
 * logits dtype; top-K by (probability desc, expert id asc) -- MLX argpartition's
 * tie order and in-slice order are unspecified, the canonical order is defined
 * here; optional renormalisation by the dtype-rounded sum.
 * Reduction order (defined here, matches a 32-lane warp): lane l owns experts
 * [l*C, min(E,(l+1)*C)), C = ceil(E/32), sums them in index order, then the 32
 * partials are combined by a butterfly over xor distances 16, 8, 4, 2, 1. */
static void route_one(const void* logits, int dtype, int64_t t, int E, int K, int normalize,
                      float* e, float* p, uint32_t* ids, void* scores) {
  const int C = (E + 31) / 32;
  float mx = -INFINITY;
  for (int i = 0; i < E; ++i) {
    float v = load_dt(logits, dtype, t * E + i);
    mx = (v > mx) ? v : mx;
  }
  float part[32];
  for (int l = 0; l < 32; ++l) {
    float s = 0.0f;
    for (int i = l * C; i < (l + 1) * C && i < E; ++i) {
      e[i] = ao_expf(load_dt(logits, dtype, t * E + i) - mx);
      s = s + e[i];
    }
    part[l] = s;
  }
  for (int m = 16; m >= 1; m >>= 1) {
    float nxt[32];
    for (int l = 0; l < 32; ++l) nxt[l] = part[l] + part[l ^ m];
    memcpy(part, nxt, sizeof(part));
  }
  const float inv = 1.0f / part[0];
  for (int i = 0; i < E; ++i) p[i] = round_dt(e[i] * inv, dtype);

  float sel[64];
  for (int k = 0; k < K; ++k) {
    int best = -1;
    for (int i = 0; i < E; ++i) {
      if (p[i] != p[i]) continue;
      if (best < 0 || p[i] > p[best]) best = i; /* strict '>' keeps the lower id on ties */
    }
    if (best < 0) best = 0;
    ids[t * K + k] = (uint32_t)best;
    sel[k] = p[best];
    p[best] = -INFINITY;
  }
  if (normalize) {
    float s = 0.0f;
    for (int k = 0; k < K; ++k) s = s + sel[k];
    const float S = round_dt(s, dtype);
    for (int k = 0; k < K; ++k) store_dt(scores, dtype, t * K + k, sel[k] / S);
  } else {
    for (int k = 0; k < K; ++k) store_dt(scores, dtype, t * K + k, sel[k]);
  }
}

int ao_route_experts(const void* logits, int dtype, int64_t tokens, int experts, int top_k,
                     int normalize, uint32_t* out_ids, void* out_scores) {
  /* validate_router_arguments, routing.rs:123-153 */
  if (tokens < 0 || experts <= 0 || top_k <= 0 || top_k > experts || top_k > 64)
    return AO_ERR_INVALID_ARGUMENT;
  if (dtype != AO_BF16 && dtype != AO_F16 && dtype != AO_F32) return AO_ERR_INVALID_ARGUMENT;
#pragma omp parallel
  {
    float* e = (float*)malloc(sizeof(float) * (size_t)experts);
    float* p = (float*)malloc(sizeof(float) * (size_t)experts);
#pragma omp for schedule(static)
    for (int64_t t = 0; t < tokens; ++t)
      route_one(logits, dtype, t, experts, top_k, normalize, e, p,
                out_ids, out_scores);
    free(e);
    free(p);
  }
  return AO_OK;
}

/* ------------------------------------------------------------------------ */
/* f4: Laguna router                                                         */
/* ------------------------------------------------------------------------ */

float ao_sigmoid_plainf(float x) { return 1.0f / (1.0f + ao_expf(-x)); }

float ao_tanhf(float x) {
  const float a = fabsf(x);
  const float t = 1.0f - 2.0f / (ao_expf(2.0f * a) + 1.0f);
  return x < 0.0f ? -t : t;
}

/* IEEE total order of fp32 as an unsigned key (Rust's f32::total_cmp) */
static inline uint32_t ordered_bits(float v) {
  const uint32_t u = f2u(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

int ao_route_laguna_experts(const void* logits, int dtype, int64_t tokens, int experts, int top_k,
                            const float* bias, float softcap, int normalize, uint32_t* out_ids,
                            float* out_scores) {
  /* validate_router_geometry, router_selection.rs:127-150 */
  if (tokens < 0 || experts <= 0 || top_k <= 0 || top_k > experts || softcap != softcap ||
      softcap < 0.0f)
    return AO_ERR_INVALID_ARGUMENT;
  if (dtype != AO_BF16 && dtype != AO_F16 && dtype != AO_F32) return AO_ERR_INVALID_ARGUMENT;
#pragma omp parallel
  {
    float* sc = (float*)malloc(sizeof(float) * (size_t)experts);
    uint64_t* key = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)experts);
#pragma omp for schedule(static)
    for (int64_t t = 0; t < tokens; ++t) {
      for (int e = 0; e < experts; ++e) {
        float l = load_dt(logits, dtype, t * experts + e);
        if (softcap > 0.0f) l = ao_tanhf(l / softcap) * softcap;
        sc[e] = ao_sigmoid_plainf(l);
        const float sel = bias ? sc[e] + bias[e] : sc[e];
        key[e] = ((uint64_t)ordered_bits(sel) << 32) | (uint64_t)(0xffffffffu - (uint32_t)e);
      }
      float sum = 0.0f;
      for (int k = 0; k < top_k; ++k) {
        int best = 0;
        for (int e = 1; e < experts; ++e) best = key[e] > key[best] ? e : best;
        out_ids[t * top_k + k] = (uint32_t)best;
        out_scores[t * top_k + k] = sc[best];
        sum = sum + sc[best];
        key[best] = 0;
      }
      if (normalize && sum > 0.0f)
        for (int k = 0; k < top_k; ++k) out_scores[t * top_k + k] = out_scores[t * top_k + k] / sum;
    }
    free(key);
    free(sc);
  }
  return AO_OK;
}

/* ------------------------------------------------------------------------ */
/* a3: stable sort of assignments by expert                                  */
/* ------------------------------------------------------------------------ */

/* argsort(flat ids) is taken as STABLE (defined here: MLX's stability is assumed
 * by the reference, whose tests only use distinct ids); inverse = argsort of the
 * order; sorted token = order / K; sorted ids = ids[order]; offsets = exclusive
 * scan of the per-expert histogram (implicit inside MLX gather_qmm, explicit here). */
int ao_sort_expert_assignments(const uint32_t* ids, int64_t tokens, int top_k, int experts,
                               uint32_t* sorted_order, uint32_t* inverse_order,
                               uint32_t* sorted_ids, uint32_t* sorted_tokens,
                               uint32_t* expert_offsets) {
  if (tokens < 0 || top_k < 0 || experts <= 0) return AO_ERR_INVALID_ARGUMENT;
  const int64_t n = tokens * (int64_t)top_k;
  if (n > 0xffffffffLL) return AO_ERR_INVALID_ARGUMENT;
  int64_t* cursor = (int64_t*)calloc((size_t)experts + 1, sizeof(int64_t));
  if (!cursor) return AO_ERR_INVALID_ARGUMENT;
  for (int64_t i = 0; i < n; ++i) {
    if (ids[i] >= (uint32_t)experts) { free(cursor); return AO_ERR_INVALID_ARGUMENT; }
    cursor[ids[i] + 1]++;
  }
  for (int e = 0; e < experts; ++e) cursor[e + 1] += cursor[e];
  if (expert_offsets)
    for (int e = 0; e <= experts; ++e) expert_offsets[e] = (uint32_t)cursor[e];
  for (int64_t i = 0; i < n; ++i) {
    const uint32_t e = ids[i];
    const int64_t pos = cursor[e]++;
    if (sorted_order) sorted_order[pos] = (uint32_t)i;
    if (inverse_order) inverse_order[i] = (uint32_t)pos;
    if (sorted_ids) sorted_ids[pos] = e;
    if (sorted_tokens) sorted_tokens[pos] = (uint32_t)(i / top_k);
  }
  free(cursor);
  return AO_OK;
}

int ao_invert_assignment_order(const uint32_t* sorted_order, int64_t n, uint32_t* inverse_order) {
  if (n < 0 || n > 0xffffffffLL) return AO_ERR_INVALID_ARGUMENT;
  unsigned char* seen = (unsigned char*)calloc((size_t)(n > 0 ? n : 1), 1);
  if (!seen) return AO_ERR_INVALID_ARGUMENT;
  for (int64_t s = 0; s < n; ++s) {
    const uint32_t o = sorted_order[s];
    if ((int64_t)o >= n) { free(seen); return AO_ERR_OUT_OF_RANGE_SLOT; }
    if (seen[o]) { free(seen); return AO_ERR_DUPLICATE_SLOT; }
    seen[o] = 1;
    inverse_order[o] = (uint32_t)s;
  }
  free(seen);
  return AO_OK;
}

/* ------------------------------------------------------------------------ */
/* affine quantisation                                                       */
/* ------------------------------------------------------------------------ */

static int valid_affine(int in_features, int group, int bits) {
  if (group != 32 && group != 64 && group != 128) return 0;
  if (!(bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8)) return 0;
  if (in_features <= 0 || in_features % group != 0) return 0;
  if (((int64_t)in_features * bits) % 32 != 0) return 0;
  return 1;
}

/* Element j of a packed row sits at bit j*bits of the row's little-endian bit
 * stream (for 4 bits: nibble j%8 of word j/8, bits 4*(j%8)); MLX's packing. */
static inline uint32_t unpack_q(const uint32_t* row, int64_t j, int bits) {
  const int64_t bit = j * bits;
  const int64_t w = bit >> 5;
  const int b = (int)(bit & 31);
  uint64_t v = row[w];
  if (b + bits > 32) v |= ((uint64_t)row[w + 1]) << 32;
  return (uint32_t)((v >> b) & ((1u << bits) - 1u));
}

/* Dequantised weight, defined here as bf16(fma(scale, q, bias)) computed in fp32
 * (exact for scale/bias of comparable magnitude) and rounded once to bf16. */
static void dequant_rows_f32(const uint32_t* packed, const uint16_t* scales,
                             const uint16_t* biases, int64_t row0, int64_t rows, int in_features,
                             int group, int bits, float* out /* [rows][in] */) {
  const int64_t words = (int64_t)in_features * bits / 32;
  const int groups = in_features / group;
  for (int64_t r = 0; r < rows; ++r) {
    const uint32_t* prow = packed + (row0 + r) * words;
    for (int g = 0; g < groups; ++g) {
      const float s = ao_bf16_to_f32(scales[(row0 + r) * groups + g]);
      const float b = ao_bf16_to_f32(biases[(row0 + r) * groups + g]);
      for (int j = g * group; j < (g + 1) * group; ++j)
        out[r * in_features + j] = rnd_bf16(fmaf(s, (float)unpack_q(prow, j, bits), b));
    }
  }
}

int ao_dequantize_affine(const uint32_t* packed, const uint16_t* scales, const uint16_t* biases,
                         int64_t rows, int in_features, int group, int bits, uint16_t* out) {
  if (rows < 0 || !valid_affine(in_features, group, bits)) return AO_ERR_INVALID_ARGUMENT;
  float* tmp = (float*)malloc(sizeof(float) * (size_t)in_features);
  for (int64_t r = 0; r < rows; ++r) {
    dequant_rows_f32(packed, scales, biases, r, 1, in_features, group, bits, tmp);
    for (int j = 0; j < in_features; ++j) out[r * in_features + j] = ao_f32_to_bf16(tmp[j]);
  }
  free(tmp);
  return AO_OK;
}

/* y[n, o] = bf16( sum_k x[k] * W[o, k] ), sequential fmaf in k order (defined
 * here).  wt is the dequantised weight transposed to [in][out] so the loop over
 * o vectorises without changing any output's accumulation order. */
static void rows_times_wt(const uint16_t* xrow, const float* wt, int in_features,
                          int out_features, float* acc, uint16_t* yrow) {
  for (int o = 0; o < out_features; ++o) acc[o] = 0.0f;
  for (int k = 0; k < in_features; ++k) {
    const float xk = ao_bf16_to_f32(xrow[k]);
    const float* w = wt + (int64_t)k * out_features;
    for (int o = 0; o < out_features; ++o) acc[o] = fmaf(xk, w[o], acc[o]);
  }
  for (int o = 0; o < out_features; ++o) yrow[o] = ao_f32_to_bf16(acc[o]);
}

static float* dequant_expert_transposed(const uint32_t* packed, const uint16_t* scales,
                                        const uint16_t* biases, int e, int out_features,
                                        int in_features, int group, int bits) {
  float* w = (float*)malloc(sizeof(float) * (size_t)out_features * in_features);
  float* wt = (float*)malloc(sizeof(float) * (size_t)out_features * in_features);
  dequant_rows_f32(packed, scales, biases, (int64_t)e * out_features, out_features, in_features,
                   group, bits, w);
  for (int o = 0; o < out_features; ++o)
    for (int k = 0; k < in_features; ++k)
      wt[(int64_t)k * out_features + o] = w[(int64_t)o * in_features + k];
  free(w);
  return wt;
}

int ao_gather_qmm(const uint16_t* x, const uint32_t* lhs_rows, const uint32_t* rhs_experts,
                  int64_t n_rows, int in_features, const uint32_t* packed,
                  const uint16_t* scales, const uint16_t* biases, int experts,
                  int out_features, int group, int bits, uint16_t* y) {
  if (n_rows < 0 || experts <= 0 || out_features <= 0 || !valid_affine(in_features, group, bits))
    return AO_ERR_INVALID_ARGUMENT;
  for (int64_t n = 0; n < n_rows; ++n)
    if (rhs_experts && rhs_experts[n] >= (uint32_t)experts) return AO_ERR_INVALID_ARGUMENT;
#pragma omp parallel for schedule(dynamic, 1)
  for (int e = 0; e < experts; ++e) {
    int64_t used = 0;
    for (int64_t n = 0; n < n_rows; ++n)
      if ((rhs_experts ? (int)rhs_experts[n] : 0) == e) { used = 1; break; }
    if (!used) continue;
    float* wt = dequant_expert_transposed(packed, scales, biases, e, out_features, in_features,
                                          group, bits);
    float* acc = (float*)malloc(sizeof(float) * (size_t)out_features);
    for (int64_t n = 0; n < n_rows; ++n) {
      if ((rhs_experts ? (int)rhs_experts[n] : 0) != e) continue;
      const int64_t r = lhs_rows ? (int64_t)lhs_rows[n] : n;
      rows_times_wt(x + r * in_features, wt, in_features, out_features, acc,
                    y + n * out_features);
    }
    free(acc);
    free(wt);
  }
  return AO_OK;
}

/* ------------------------------------------------------------------------ */
/* a5: SwiGLU                                                                */
/* ------------------------------------------------------------------------ */

/* gate * sigmoid(gate) * up as three bf16 ops (the compiled graph keeps each
 * intermediate in the activation dtype). */
static inline float swiglu_bf16(float g, float u) {
  const float s = rnd_bf16(ao_sigmoidf(g));
  const float a = rnd_bf16(g * s);
  return rnd_bf16(a * u);
}

void ao_swiglu(const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i)
    out[i] = ao_f32_to_bf16(swiglu_bf16(ao_bf16_to_f32(gate[i]), ao_bf16_to_f32(up[i])));
}

/* ------------------------------------------------------------------------ */
/* a7: weighted sums                                                         */
/* ------------------------------------------------------------------------ */

/* Kernel source weighted_sum.rs:16-33: per output element, in slot order,
 * weighted_sum += float(out[inverse[t*K+k]]) * float(score[t*K+k]); the update is
 * one fused multiply-add (defined here); the result is cast to the output dtype. */
int ao_sorted_expert_weighted_sum(const void* sorted_outputs, int out_dtype,
                                  const uint32_t* inverse_order, const void* scores,
                                  int score_dtype, int64_t tokens, int top_k, int64_t dim,
                                  void* out) {
  if (tokens < 0 || top_k < 0 || dim < 0) return AO_ERR_INVALID_ARGUMENT;
  const int64_t n = tokens * top_k;
  for (int64_t i = 0; i < n; ++i)
    if ((int64_t)inverse_order[i] >= n) return AO_ERR_INVALID_ARGUMENT;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < tokens; ++t) {
    for (int64_t d = 0; d < dim; ++d) {
      float acc = 0.0f;
      for (int k = 0; k < top_k; ++k) {
        const int64_t a = t * top_k + k;
        acc = fmaf(load_dt(sorted_outputs, out_dtype, (int64_t)inverse_order[a] * dim + d),
                   load_dt(scores, score_dtype, a), acc);
      }
      store_dt(out, out_dtype, t * dim + d, acc);
    }
  }
  return AO_OK;
}

/* weighted_sum.rs:94-120: multiply(outputs, scores[..., None]) in the promoted
 * dtype (bf16 x bf16 -> bf16, anything x f32 -> f32), sum over K accumulated in
 * fp32 in slot order (defined here), cast to the output dtype. */
int ao_unsorted_expert_weighted_sum(const void* outputs, int out_dtype, const void* scores,
                                    int score_dtype, int64_t tokens, int top_k, int64_t dim,
                                    void* out) {
  if (tokens < 0 || top_k < 0 || dim < 0) return AO_ERR_INVALID_ARGUMENT;
  const int prod_dtype = (out_dtype == AO_F32 || score_dtype == AO_F32) ? AO_F32
                         : (out_dtype == score_dtype ? out_dtype : AO_F32);
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < tokens; ++t) {
    for (int64_t d = 0; d < dim; ++d) {
      float acc = 0.0f;
      for (int k = 0; k < top_k; ++k) {
        const float pr = load_dt(outputs, out_dtype, (t * top_k + k) * dim + d) *
                         load_dt(scores, score_dtype, t * top_k + k);
        acc = acc + round_dt(pr, prod_dtype);
      }
      store_dt(out, out_dtype, t * dim + d, acc);
    }
  }
  return AO_OK;
}

/* ------------------------------------------------------------------------ */
/* a8: combination                                                           */
/* ------------------------------------------------------------------------ */

void ao_combine_sparse_and_shared(const void* sparse, const void* shared, const void* gate_logits,
                                  int dtype, int64_t tokens, int64_t dim, void* out) {
  for (int64_t t = 0; t < tokens; ++t) {
    const float g = round_dt(ao_sigmoidf(load_dt(gate_logits, dtype, t)), dtype);
    for (int64_t d = 0; d < dim; ++d) {
      const float prod = round_dt(load_dt(shared, dtype, t * dim + d) * g, dtype);
      store_dt(out, dtype, t * dim + d, load_dt(sparse, dtype, t * dim + d) + prod);
    }
  }
}

/* ------------------------------------------------------------------------ */
/* a9: whole block                                                           */
/* ------------------------------------------------------------------------ */

typedef struct {
  const uint32_t* q;
  const uint16_t* s;
  const uint16_t* b;
  int bits, group;
} proj_t;

/* projection `which` (0 gate, 1 up, 2 down, 3 shared gate, 4 shared up, 5 shared
 * down) with its own quantisation (qwen3_5/model/decoder_layer_weights.rs:15-26) */
static proj_t proj_of(const ao_block_weights* w, int which) {
  proj_t p;
  switch (which) {
    case 0: p.q = w->gate_q; p.s = w->gate_s; p.b = w->gate_b; break;
    case 1: p.q = w->up_q; p.s = w->up_s; p.b = w->up_b; break;
    case 2: p.q = w->down_q; p.s = w->down_s; p.b = w->down_b; break;
    case 3: p.q = w->sgate_q; p.s = w->sgate_s; p.b = w->sgate_b; break;
    case 4: p.q = w->sup_q; p.s = w->sup_s; p.b = w->sup_b; break;
    default: p.q = w->sdown_q; p.s = w->sdown_s; p.b = w->sdown_b; break;
  }
  p.bits = w->proj_bits[which] > 0 ? w->proj_bits[which] : w->bits;
  p.group = w->proj_group[which] > 0 ? w->proj_group[which] : w->group;
  return p;
}

/* y[r] = bf16(x_row(r) . dequant(W[e])^T) for n rows of one expert, in `mode`. */
static void expert_rows(const proj_t* P, int e, int out_features, int in_features,
                        const uint16_t* const* xrows, int64_t n, int mode, uint16_t* y,
                        int64_t ldy) {
  if (n == 0) return;
  if (mode == AO_DOT_SEQ) {
    float* acc = (float*)malloc(sizeof(float) * (size_t)out_features);
    float* wt = dequant_expert_transposed(P->q, P->s, P->b, e, out_features, in_features,
                                          P->group, P->bits);
    for (int64_t r = 0; r < n; ++r) rows_times_wt(xrows[r], wt, in_features, out_features, acc, y + r * ldy);
    free(wt);
    free(acc);
    return;
  }
  float* wf = (float*)malloc(sizeof(float) * (size_t)out_features * in_features);
  float* xf = (float*)malloc(sizeof(float) * (size_t)in_features);
  dequant_rows_f32(P->q, P->s, P->b, (int64_t)e * out_features, out_features, in_features,
                   P->group, P->bits, wf);
  for (int64_t r = 0; r < n; ++r) {
    for (int k = 0; k < in_features; ++k) xf[k] = ao_bf16_to_f32(xrows[r][k]);
    for (int o = 0; o < out_features; ++o)
      y[r * ldy + o] = ao_f32_to_bf16(ao_dot(wf + (int64_t)o * in_features, xf, in_features, mode));
  }
  free(xf);
  free(wf);
}

/* bf16 [rows, in] weight of a dense-or-affine projection (the affine one
 * dequantised: the weight MLX's quantized matmul multiplies); caller frees. */
static uint16_t* dense_or_affine(const uint16_t* dense, const uint32_t* q, const uint16_t* sc,
                                 const uint16_t* bi, int bits, int group, int64_t rows, int in) {
  uint16_t* out = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)rows * in);
  if (bits > 0) ao_dequantize_affine(q, sc, bi, rows, in, group, bits, out);
  else memcpy(out, dense, sizeof(uint16_t) * (size_t)rows * in);
  return out;
}

/* Laguna combination (laguna/moe/resident.rs:89-100): routed = multiply_scalar(
 * sparse, factor) with the scalar cast to bf16 first (mlx_operations.rs:234-242),
 * rounded to bf16; out = bf16(routed + shared) (shared NULL: routed). */
static void laguna_finish(const uint16_t* sparse, const uint16_t* shared, int64_t nt, int H,
                          float factor, uint16_t* out) {
  const float f = rnd_bf16(factor > 0.0f ? factor : 1.0f);
  for (int64_t i = 0; i < nt * H; ++i) {
    float y = rnd_bf16(ao_bf16_to_f32(sparse[i]) * f);
    if (shared) y = y + ao_bf16_to_f32(shared[i]);
    out[i] = ao_f32_to_bf16(y);
  }
}

int ao_moe_block_forward(const ao_block_weights* w, const uint16_t* x, int64_t tokens,
                         const int64_t* token_subset, int64_t n_subset,
                         const uint16_t* logits_override, uint16_t* out,
                         uint32_t* out_ids, void* out_scores, int num_threads) {
  return ao_moe_block_forward_terms(w, x, tokens, token_subset, n_subset, logits_override, out,
                                    out_ids, out_scores, NULL, NULL, num_threads);
}

int ao_moe_block_forward_terms(const ao_block_weights* w, const uint16_t* x, int64_t tokens,
                               const int64_t* token_subset, int64_t n_subset,
                               const uint16_t* logits_override, uint16_t* out,
                               uint32_t* out_ids, void* out_scores, uint16_t* out_sparse,
                               uint16_t* out_shared_gated, int num_threads) {
  const int H = w->hidden, E = w->experts, K = w->top_k, I = w->intermediate;
  const int Is = w->shared_intermediate;
  if (tokens < 0 || H <= 0 || E <= 0 || K <= 0 || K > E || I <= 0 || Is < 0)
    return AO_ERR_INVALID_ARGUMENT;
  proj_t P[6];
  for (int i = 0; i < 6; ++i) P[i] = proj_of(w, i);
  if (!valid_affine(H, P[0].group, P[0].bits) || !valid_affine(H, P[1].group, P[1].bits) ||
      !valid_affine(I, P[2].group, P[2].bits))
    return AO_ERR_INVALID_ARGUMENT;
  if (Is > 0 && (!valid_affine(H, P[3].group, P[3].bits) || !valid_affine(H, P[4].group, P[4].bits) ||
                 !valid_affine(Is, P[5].group, P[5].bits)))
    return AO_ERR_INVALID_ARGUMENT;
  if (w->router_bits > 0 && !valid_affine(H, w->router_group, w->router_bits))
    return AO_ERR_INVALID_ARGUMENT;
  if (Is > 0 && w->shared_gate_bits > 0 && !valid_affine(H, w->shared_gate_group, w->shared_gate_bits))
    return AO_ERR_INVALID_ARGUMENT;
#ifdef _OPENMP
  if (num_threads > 0) omp_set_num_threads(num_threads);
#else
  (void)num_threads;
#endif
  const int64_t nt = token_subset ? n_subset : tokens;
  /* routing.rs:13 / resident_execution.rs:86-96: sorted iff T*K >= 64 */
  const int sorted = tokens * (int64_t)K >= 64;
  const int m_router = w->arith[0], m_glogit = w->arith[1], m_gu = w->arith[2],
            m_down = w->arith[3], m_sgu = w->arith[4], m_sdown = w->arith[5];

  uint16_t* xs = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(nt > 0 ? nt : 1) * H);
  uint16_t* logits = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(nt > 0 ? nt : 1) * E);
  for (int64_t i = 0; i < nt; ++i) {
    const int64_t t = token_subset ? token_subset[i] : i;
    memcpy(xs + i * H, x + t * H, sizeof(uint16_t) * H);
    if (logits_override) memcpy(logits + i * E, logits_override + t * E, sizeof(uint16_t) * E);
  }
  /* a1: router projection (forward.rs:52-93; an affine router goes through
   * quantized_linear, :53-58) */
  if (!logits_override) {
    uint16_t* wr = dense_or_affine(w->router_w, w->router_q, w->router_s, w->router_b,
                                   w->router_bits, w->router_group, E, H);
    ao_matmul_bf16_nt_mode(xs, wr, nt, E, H, m_router, logits);
    free(wr);
  }
  /* a2: route (routing.rs:16-49), or the Laguna router (f4) with fp32 scores */
  const int laguna = w->router_kind == 1;
  uint32_t* ids = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(nt > 0 ? nt : 1) * K);
  uint16_t* scores = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(nt > 0 ? nt : 1) * K);
  float* fscores = (float*)malloc(sizeof(float) * (size_t)(nt > 0 ? nt : 1) * K);
  if (laguna)
    ao_route_laguna_experts(logits, AO_BF16, nt, E, K, w->router_correction_bias,
                            w->router_logit_softcap, w->normalize, ids, fscores);
  else
    ao_route_experts(logits, AO_BF16, nt, E, K, w->normalize, ids, scores);
  /* a3: sort (assignment_sort.rs:79-91) */
  const int64_t n = nt * K;
  uint32_t* order = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(n > 0 ? n : 1));
  uint32_t* inv = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(n > 0 ? n : 1));
  uint32_t* sids = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(n > 0 ? n : 1));
  uint32_t* stok = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(n > 0 ? n : 1));
  uint32_t* offs = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(E + 1));
  ao_sort_expert_assignments(ids, nt, K, E, order, inv, sids, stok, offs);

  /* a4-a6: per expert: gate, up, SwiGLU, down over the expert's sorted rows
   * (resident_execution.rs:98-116 with gather_qmm, sorted_indices=true). */
  uint16_t* yrows = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(n > 0 ? n : 1) * H);
#pragma omp parallel for schedule(dynamic, 1)
  for (int e = 0; e < E; ++e) {
    const int64_t r0 = offs[e], r1 = offs[e + 1], m = r1 - r0;
    if (m == 0) continue;
    const uint16_t** xr = (const uint16_t**)malloc(sizeof(uint16_t*) * (size_t)m);
    const uint16_t** ar = (const uint16_t**)malloc(sizeof(uint16_t*) * (size_t)m);
    uint16_t* g = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)m * I);
    uint16_t* u = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)m * I);
    uint16_t* a = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)m * I);
    for (int64_t r = 0; r < m; ++r) {
      xr[r] = xs + (int64_t)stok[r0 + r] * H;
      ar[r] = a + r * I;
    }
    expert_rows(&P[0], e, I, H, xr, m, m_gu, g, I);
    expert_rows(&P[1], e, I, H, xr, m, m_gu, u, I);
    ao_swiglu(g, u, m * I, a);
    expert_rows(&P[2], e, H, I, ar, m, m_down, yrows + r0 * H, H);
    free(a); free(u); free(g); free(ar); free(xr);
  }

  /* a7: weighted sum (sorted kernel, or unsorted multiply+sum for N < 64) */
  uint16_t* sparse = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(nt > 0 ? nt : 1) * H);
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < nt; ++t) {
    for (int d = 0; d < H; ++d) {
      float acc = 0.0f;
      for (int k = 0; k < K; ++k) {
        const float yv = ao_bf16_to_f32(yrows[(int64_t)inv[t * K + k] * H + d]);
        const float sv = laguna ? fscores[t * K + k] : ao_bf16_to_f32(scores[t * K + k]);
        if (sorted) acc = fmaf(yv, sv, acc);
        else if (laguna) acc = acc + yv * sv; /* bf16 x f32 promotes to f32 */
        else acc = acc + rnd_bf16(yv * sv);
      }
      sparse[t * H + d] = ao_f32_to_bf16(acc);
    }
  }

  /* a8: shared expert + sigmoid gate (resident_execution.rs:352-400) */
  if (Is > 0) {
    const int64_t nn = nt > 0 ? nt : 1;
    uint16_t* sg = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)nn * Is);
    uint16_t* su = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)nn * Is);
    uint16_t* sa = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)nn * Is);
    uint16_t* so = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)nn * H);
    uint16_t* gl = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)nn);
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t t0 = 0; t0 < nt; t0 += 64) {
      const int64_t m = (nt - t0 < 64) ? nt - t0 : 64;
      const uint16_t* xr[64];
      const uint16_t* ar[64];
      for (int64_t r = 0; r < m; ++r) {
        xr[r] = xs + (t0 + r) * H;
        ar[r] = sa + (t0 + r) * Is;
      }
      expert_rows(&P[3], 0, Is, H, xr, m, m_sgu, sg + t0 * Is, Is);
      expert_rows(&P[4], 0, Is, H, xr, m, m_sgu, su + t0 * Is, Is);
      ao_swiglu(sg + t0 * Is, su + t0 * Is, m * Is, sa + t0 * Is);
      expert_rows(&P[5], 0, H, Is, ar, m, m_sdown, so + t0 * H, H);
    }
    if (laguna) {
      laguna_finish(sparse, so, nt, H, w->routed_scaling_factor, out);
      if (out_shared_gated) memcpy(out_shared_gated, so, sizeof(uint16_t) * (size_t)nt * H);
    } else {
    uint16_t* wg = dense_or_affine(w->shared_gate_w, w->shared_gate_q, w->shared_gate_s,
                                   w->shared_gate_b, w->shared_gate_bits, w->shared_gate_group, 1, H);
    ao_matmul_bf16_nt_mode(xs, wg, nt, 1, H, m_glogit, gl);
    free(wg);
    ao_combine_sparse_and_shared(sparse, so, gl, AO_BF16, nt, H, out);
    }
    if (out_shared_gated && !laguna) {
      for (int64_t t = 0; t < nt; ++t) {
        const float g = rnd_bf16(ao_sigmoidf(ao_bf16_to_f32(gl[t])));
        for (int d = 0; d < H; ++d)
          out_shared_gated[t * H + d] = ao_f32_to_bf16(ao_bf16_to_f32(so[t * H + d]) * g);
      }
    }
    free(gl); free(so); free(sa); free(su); free(sg);
  } else {
    if (laguna) laguna_finish(sparse, NULL, nt, H, w->routed_scaling_factor, out);
    else memcpy(out, sparse, sizeof(uint16_t) * (size_t)nt * H);
    if (out_shared_gated) memset(out_shared_gated, 0, sizeof(uint16_t) * (size_t)nt * H);
  }
  if (out_sparse) memcpy(out_sparse, sparse, sizeof(uint16_t) * (size_t)nt * H);
  if (out_ids) memcpy(out_ids, ids, sizeof(uint32_t) * (size_t)n);
  if (out_scores) {
    if (laguna) memcpy(out_scores, fscores, sizeof(float) * (size_t)n);
    else memcpy(out_scores, scores, sizeof(uint16_t) * (size_t)n);
  }
  free(sparse); free(yrows); free(offs); free(stok); free(sids); free(inv); free(order);
  free(fscores); free(scores); free(ids); free(logits); free(xs);
  return AO_OK;
}
