/*
 * dcr_oracle.c — CPU restatement of DCR-Attention's per-step sparse decode attention.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for libdcr_b200: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load it. The product path never
 * calls it and has no CPU fallback.
 *
 * It restates the reference algorithm (Seqev/dcr-attention_v3,
 * dcr_attention/kernel/qaxis_topk_reference.py) step by step. The floating-point sums are
 * written in the fixed order the CUDA kernels use, so the bf16 scores and the selected
 * index sets can be compared bit for bit:
 *
 *   oracle_unit_query   _compute_u_Q                qaxis_topk_reference.py:42-55
 *   oracle_scores       _compute_projection_scores  qaxis_topk_reference.py:58-88
 *   oracle_select       _select_topk_indices        qaxis_topk_reference.py:91-108
 *   oracle_attend       _gather_kv + _fused_softmax_attention
 *                                                   qaxis_topk_reference.py:111-193
 *
 * Projected-score mode (no counterpart in the reference; the rank-R projection P of the
 * keys is written at cache-append time and the unit query is projected with the same P):
 *
 *   oracle_project_keys      KP = round_dtype(K . P), fmaf chain over d = 0..63
 *   oracle_query_projection  qp = u . P (fp32), fmaf chain over d = 0..63
 *   oracle_scores_projected  bf16_rne(even + odd): two fmaf chains of KP . qp, one over
 *                            the even j, one over the odd j, added at the end
 *
 * Their parity is pinned against this restatement only (the reference has no such mode).
 *
 * Pinning: tests/test_oracle_golden.py checks these functions against golden vectors the
 * reference itself produced (tests/golden/make_golden.py).
 *
 * Build: see oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off; fmaf is exact in any
 * ISA, the target_clones only pick the hardware instruction when the host has it).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_D 64

enum { ORACLE_BF16 = 0, ORACLE_F16 = 1, ORACLE_F32 = 2 };

#if defined(__x86_64__)
#define HOT __attribute__((target_clones("fma", "default")))
#else
#define HOT
#endif

/* ---------------------------------------------------------------------------------- */
/* element widening (exact)                                                            */
/* ---------------------------------------------------------------------------------- */
static inline float bits_to_f32(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}
static inline uint32_t f32_to_bits(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
}

static inline float bf16_to_f32(uint16_t h) { return bits_to_f32((uint32_t)h << 16); }

static inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  const uint32_t man = h & 0x3ffu;
  if (exp == 0) {
    if (man == 0) return bits_to_f32(sign);
    /* subnormal: man * 2^-24, exact in fp32 */
    float v = (float)man * 5.9604644775390625e-08f;
    return sign ? -v : v;
  }
  if (exp == 31) return bits_to_f32(sign | 0x7f800000u | (man << 13));
  return bits_to_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

static inline float load_elem(const void* base, int dtype, int64_t i) {
  switch (dtype) {
    case ORACLE_BF16: return bf16_to_f32(((const uint16_t*)base)[i]);
    case ORACLE_F16: return f16_to_f32(((const uint16_t*)base)[i]);
    default: return ((const float*)base)[i];
  }
}

/* bf16 round-to-nearest-even (torch's Tensor.to(torch.bfloat16)); NaN -> 0x7fc0. */
static inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t b = f32_to_bits(f);
  if ((b & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((b >> 16) | 0x40u);
  b += 0x7fffu + ((b >> 16) & 1u);
  return (uint16_t)(b >> 16);
}

/* fp32 -> fp16, IEEE round-to-nearest-even (overflow to inf, subnormals, quiet NaN). */
static inline uint16_t f32_to_f16_rne(float f) {
  const uint32_t x = f32_to_bits(f);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
  if (ax < 0x38800000u) {                                   /* below 2^-14: subnormal   */
    if (ax <= 0x33000000u) return (uint16_t)sign;           /* <= 2^-25 rounds to zero  */
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - e; /* value = m * 2^(e-150); units of 2^-24 */
    uint32_t q = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
  }
  uint32_t q = (((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13);
  const uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
  return (uint16_t)(sign | q);
}

static inline void store_elem(void* base, int dtype, int64_t i, float v) {
  switch (dtype) {
    case ORACLE_BF16: ((uint16_t*)base)[i] = f32_to_bf16_rne(v); break;
    case ORACLE_F16: ((uint16_t*)base)[i] = f32_to_f16_rne(v); break;
    default: ((float*)base)[i] = v;
  }
}

/* ---------------------------------------------------------------------------------- */
/* u = q / max(||q||, eps)                                                             */
/* The 64-element sum of squares follows the kernel's warp layout: lane l holds         */
/* fmaf(q[2l+1]^2 + q[2l]*q[2l]), then an xor butterfly with offsets 16, 8, 4, 2, 1.   */
/* ---------------------------------------------------------------------------------- */
void oracle_unit_query(const void* q, int dtype, int rows, float eps, float* u) {
  for (int r = 0; r < rows; ++r) {
    float x[ORACLE_D];
    for (int d = 0; d < ORACLE_D; ++d) x[d] = load_elem(q, dtype, (int64_t)r * ORACLE_D + d);
    float part[32], nxt[32];
    for (int l = 0; l < 32; ++l) {
      const float sq0 = x[2 * l] * x[2 * l];
      part[l] = fmaf(x[2 * l + 1], x[2 * l + 1], sq0);
    }
    for (int off = 16; off >= 1; off >>= 1) {
      for (int l = 0; l < 32; ++l) nxt[l] = part[l] + part[l ^ off];
      memcpy(part, nxt, sizeof(part));
    }
    float norm = sqrtf(part[0]);
    norm = fmaxf(norm, eps);
    for (int d = 0; d < ORACLE_D; ++d) u[(int64_t)r * ORACLE_D + d] = x[d] / norm;
  }
}

/* ---------------------------------------------------------------------------------- */
/* scores[b*H + h, n] = bf16_rne( sum_{d=0..63} fmaf chain of K[b, h/G, n, d] * u[b, h, d] ) */
/* ---------------------------------------------------------------------------------- */
HOT static void score_group(const void* K, int dtype, int64_t kbase, const float* ug, int G,
                            int N, uint16_t* out, int64_t s_stride) {
  float kr[ORACLE_D];
  for (int n = 0; n < N; ++n) {
    const int64_t rb = kbase + (int64_t)n * ORACLE_D;
    for (int d = 0; d < ORACLE_D; ++d) kr[d] = load_elem(K, dtype, rb + d);
    for (int j = 0; j < G; ++j) {
      const float* uj = ug + (int64_t)j * ORACLE_D;
      float acc = 0.0f;
      for (int d = 0; d < ORACLE_D; ++d) acc = fmaf(kr[d], uj[d], acc);
      out[(int64_t)j * s_stride + n] = f32_to_bf16_rne(acc);
    }
  }
}

void oracle_scores(const void* K, int dtype, int64_t k_stride_b, int64_t k_stride_h,
                   const float* u, int B, int H, int H_kv, int N, uint16_t* scores,
                   int64_t s_stride) {
  const int G = H / H_kv;
#pragma omp parallel for schedule(dynamic, 1)
  for (int g = 0; g < B * H_kv; ++g) {
    const int b = g / H_kv, hk = g % H_kv;
    score_group(K, dtype, (int64_t)b * k_stride_b + (int64_t)hk * k_stride_h,
                u + (int64_t)g * G * ORACLE_D, G, N, scores + (int64_t)g * G * s_stride, s_stride);
  }
}

/* ---------------------------------------------------------------------------------- */
/* projected-score mode                                                                 */
/* ---------------------------------------------------------------------------------- */
HOT void oracle_project_keys(const void* K, int dtype, int64_t k_stride_b, int64_t k_stride_h,
                             int B, int H_kv, int N, const float* P, int R, void* KP,
                             int64_t p_stride_b, int64_t p_stride_h) {
#pragma omp parallel for schedule(static)
  for (int g = 0; g < B * H_kv; ++g) {
    const int b = g / H_kv, hk = g % H_kv;
    const int64_t kb = (int64_t)b * k_stride_b + (int64_t)hk * k_stride_h;
    const int64_t pb = (int64_t)b * p_stride_b + (int64_t)hk * p_stride_h;
    float kr[ORACLE_D];
    for (int n = 0; n < N; ++n) {
      for (int d = 0; d < ORACLE_D; ++d) kr[d] = load_elem(K, dtype, kb + (int64_t)n * ORACLE_D + d);
      for (int j = 0; j < R; ++j) {
        float acc = 0.0f;
        for (int d = 0; d < ORACLE_D; ++d) acc = fmaf(kr[d], P[d * R + j], acc);
        store_elem(KP, dtype, pb + (int64_t)n * R + j, acc);
      }
    }
  }
}

void oracle_query_projection(const float* u, int rows, const float* P, int R, float* qp) {
  for (int r = 0; r < rows; ++r)
    for (int j = 0; j < R; ++j) {
      float acc = 0.0f;
      for (int d = 0; d < ORACLE_D; ++d) acc = fmaf(u[(int64_t)r * ORACLE_D + d], P[d * R + j], acc);
      qp[(int64_t)r * R + j] = acc;
    }
}

HOT void oracle_scores_projected(const void* KP, int dtype, int64_t p_stride_b,
                                 int64_t p_stride_h, const float* qp, int R, int B, int H,
                                 int H_kv, int N, uint16_t* scores, int64_t s_stride) {
  const int G = H / H_kv;
#pragma omp parallel for schedule(static)
  for (int g = 0; g < B * H_kv; ++g) {
    const int b = g / H_kv, hk = g % H_kv;
    const int64_t pb = (int64_t)b * p_stride_b + (int64_t)hk * p_stride_h;
    float kr[64];
    for (int n = 0; n < N; ++n) {
      for (int j = 0; j < R; ++j) kr[j] = load_elem(KP, dtype, pb + (int64_t)n * R + j);
      for (int h = 0; h < G; ++h) {
        const float* q = qp + ((int64_t)g * G + h) * R;
        float even = 0.0f, odd = 0.0f;
        for (int j = 0; j < R; j += 2) {
          even = fmaf(kr[j], q[j], even);
          odd = fmaf(kr[j + 1], q[j + 1], odd);
        }
        scores[((int64_t)g * G + h) * s_stride + n] = f32_to_bf16_rne(even + odd);
      }
    }
  }
}

/* ---------------------------------------------------------------------------------- */
/* top-K: the k largest bf16 scores, ties to the lower index, ascending index order.     */
/* Equal to a stable descending argsort of f32(score) cut at k then sorted ascending:    */
/* -0 == +0, and NaN ranks above every number (torch's descending sort order).           */
/* ---------------------------------------------------------------------------------- */
static inline uint32_t order_key(uint16_t b) {
  uint32_t x = b;
  if ((x & 0x7fffu) > 0x7f80u) return 0xffffu;
  if (x == 0x8000u) x = 0;
  return (x & 0x8000u) ? (~x & 0xffffu) : (x | 0x8000u);
}

int oracle_select(const uint16_t* scores, int64_t s_stride, int rows, int N, int k,
                  int32_t* idx) {
  if (k <= 0 || k > N) return 1;
  int bad = 0;
#pragma omp parallel
  {
    uint32_t* hist = (uint32_t*)malloc(sizeof(uint32_t) * 65536);
#pragma omp for schedule(dynamic, 1)
    for (int r = 0; r < rows; ++r) {
      const uint16_t* s = scores + (int64_t)r * s_stride;
      memset(hist, 0, sizeof(uint32_t) * 65536);
      for (int n = 0; n < N; ++n) hist[order_key(s[n])]++;
      /* threshold T: #{key > T} < k <= #{key >= T} */
      int64_t above = 0;
      int T = 65535;
      for (; T >= 0; --T) {
        if (above + hist[T] >= (int64_t)k) break;
        above += hist[T];
      }
      int64_t need = (int64_t)k - above; /* equal keys to take, lowest indices first */
      int32_t* out = idx + (int64_t)r * k;
      int64_t pos = 0;
      for (int n = 0; n < N; ++n) {
        const uint32_t key = order_key(s[n]);
        if ((int)key > T || ((int)key == T && need > 0)) {
          if ((int)key == T) --need;
          out[pos++] = n;
        }
      }
      if (pos != k) {
#pragma omp atomic write
        bad = 1;
      }
    }
    free(hist);
  }
  return bad;
}

/* ---------------------------------------------------------------------------------- */
/* attention over the selected rows: 64-key tiles, fp32 running (m, l, o),              */
/* z = (K . f32(Q)) / sqrt(D) with the UNNORMALISED query, one final o / l.              */
/* ---------------------------------------------------------------------------------- */
HOT void oracle_attend(const void* Q, const void* K, const void* V, int dtype,
                       int64_t k_stride_b, int64_t k_stride_h, int64_t v_stride_b,
                       int64_t v_stride_h, const int32_t* idx, int B, int H, int H_kv, int N,
                       int k, int tile, float* O) {
  const int G = H / H_kv;
  const float scale = 1.0f / sqrtf((float)ORACLE_D);
  if (tile <= 0) tile = 64;
#pragma omp parallel for schedule(dynamic, 1)
  for (int row = 0; row < B * H; ++row) {
    const int b = row / H, h = row % H, hk = h / G;
    float q[ORACLE_D], o[ORACLE_D];
    for (int d = 0; d < ORACLE_D; ++d) {
      q[d] = load_elem(Q, dtype, (int64_t)row * ORACLE_D + d);
      o[d] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    const int64_t kb = (int64_t)b * k_stride_b + (int64_t)hk * k_stride_h;
    const int64_t vb = (int64_t)b * v_stride_b + (int64_t)hk * v_stride_h;
    const int32_t* ir = idx + (int64_t)row * k;
    float* z = (float*)malloc(sizeof(float) * (size_t)tile);
    for (int t0 = 0; t0 < k; t0 += tile) {
      const int t1 = t0 + tile < k ? t0 + tile : k;
      float tmax = -INFINITY;
      for (int t = t0; t < t1; ++t) {
        const int64_t n = ir[t];
        float acc = 0.0f;
        if (n >= 0 && n < N)
          for (int d = 0; d < ORACLE_D; ++d)
            acc = fmaf(load_elem(K, dtype, kb + n * ORACLE_D + d), q[d], acc);
        z[t - t0] = acc * scale;
        if (z[t - t0] > tmax) tmax = z[t - t0];
      }
      const float m_new = m > tmax ? m : tmax;
      const float alpha = expf(m - m_new);
      float psum = 0.0f;
      for (int d = 0; d < ORACLE_D; ++d) o[d] *= alpha;
      for (int t = t0; t < t1; ++t) {
        const float p = expf(z[t - t0] - m_new);
        psum += p;
        const int64_t n = ir[t];
        if (n >= 0 && n < N)
          for (int d = 0; d < ORACLE_D; ++d)
            o[d] = fmaf(p, load_elem(V, dtype, vb + n * ORACLE_D + d), o[d]);
      }
      l = alpha * l + psum;
      m = m_new;
    }
    free(z);
    for (int d = 0; d < ORACLE_D; ++d) O[(int64_t)row * ORACLE_D + d] = o[d] / l;
  }
}

/* k_eff = min(N, max(k_min, floor(N * c))), odd -> +1 capped at N
 * (adaptive_k_window, dcr_attention/models/llama/adaptive.py:85-105). */
int oracle_adaptive_k_window(int k_window_min, int n_kv, double coverage_floor) {
  if (n_kv <= 0 || !(coverage_floor >= 0.0 && coverage_floor <= 1.0)) return -1;
  long long f = (long long)((double)n_kv * coverage_floor);
  long long k = f > k_window_min ? f : k_window_min;
  if (k > n_kv) k = n_kv;
  if (k % 2 == 1) k = (k + 1 < n_kv) ? k + 1 : n_kv;
  return (int)k;
}
