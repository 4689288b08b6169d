/*
 * bwpp_oracle.c -- CPU checker for the BW++ hot path.  TEST INFRASTRUCTURE
 * ONLY: the CUDA runtime never links or calls this file.
 *
 * Parity pin: the restatements in section 1 are compared bit-for-bit with the
 * reference's runtime/cpu/bwpp_cpu_ref.c, compiled from the reference sources
 * into oracle/_ref/ by oracle/Makefile, and against the reference tests' known
 * answers (runtime/cpu/test_metal_parity.c, test_norm.c, test_reduce_max.c);
 * see tests/test_oracle.py.  Section 2 is unpinned by the reference (it has
 * no such functions) and is checked against float64 numpy restatements.
 */
#include "bwpp_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* 1. restatements of runtime/cpu/bwpp_cpu_ref.c                            */
/* ------------------------------------------------------------------------ */

/* runtime/cpu/bwpp_cpu_ref.c:4-6 */
static float oracle_silu(float x) { return x / (1.0f + expf(-x)); }

void bwpp_oracle_matmul_f32(const float *a, const float *b, float *c,
                            uint32_t M, uint32_t N, uint32_t K,
                            uint32_t lda, uint32_t ldb, uint32_t ldc,
                            const float *bias, int apply_silu, int apply_bias) {
  if (!a || !b || !c) return;
  for (uint32_t row = 0; row < M; ++row) {
    float *crow = c + (size_t)row * ldc;
    const float *arow = a + (size_t)row * lda;
    for (uint32_t col = 0; col < N; ++col) crow[col] = 0.0f;
    /* k outer, col inner: element (row,col) still accumulates k = 0..K-1 in
     * order, starting from 0.0f, exactly as bwpp_cpu_ref.c:22-25. */
    for (uint32_t k = 0; k < K; ++k) {
      const float av = arow[k];
      const float *brow = b + (size_t)k * ldb;
      for (uint32_t col = 0; col < N; ++col) crow[col] += av * brow[col];
    }
    for (uint32_t col = 0; col < N; ++col) {
      float acc = crow[col];
      if (apply_bias && bias) acc += bias[col]; /* bias before SiLU (:26-31) */
      if (apply_silu) acc = oracle_silu(acc);
      crow[col] = acc;
    }
  }
}

void bwpp_oracle_softmax_f32(const float *x, float *y, uint32_t rows,
                             uint32_t cols, uint32_t ld) {
  if (!x || !y) return;
  for (uint32_t r = 0; r < rows; ++r) {
    const float *xr = x + (size_t)r * ld;
    float *yr = y + (size_t)r * ld;
    float m = -INFINITY;
    for (uint32_t c = 0; c < cols; ++c)
      if (xr[c] > m) m = xr[c];
    float s = 0.0f;
    for (uint32_t c = 0; c < cols; ++c) {
      const float e = expf(xr[c] - m);
      yr[c] = e;
      s += e;
    }
    const float inv = s > 0.0f ? 1.0f / s : 0.0f;
    for (uint32_t c = 0; c < cols; ++c) yr[c] *= inv;
  }
}

void bwpp_oracle_rmsnorm_f32(const float *x, float *y, const float *gamma,
                             const float *beta, uint32_t rows, uint32_t cols,
                             uint32_t ld, float eps) {
  if (!x || !y) return;
  for (uint32_t r = 0; r < rows; ++r) {
    const float *xr = x + (size_t)r * ld;
    float *yr = y + (size_t)r * ld;
    float ss = 0.0f;
    for (uint32_t c = 0; c < cols; ++c) ss += xr[c] * xr[c];
    const float inv = 1.0f / sqrtf(ss / (float)cols + eps);
    for (uint32_t c = 0; c < cols; ++c) {
      float v = xr[c] * inv;
      if (gamma) v *= gamma[c];
      if (beta) v += beta[c];
      yr[c] = v;
    }
  }
}

/* one query row of the reference's three-pass attention */
static void oracle_attention_row(const float *qr, const float *k,
                                 const float *v, float *orow, uint32_t N,
                                 uint32_t K, uint32_t D, uint32_t ldk,
                                 uint32_t ldv) {
  float m = -INFINITY;
  for (uint32_t n = 0; n < N; ++n) {
    const float *kr = k + (size_t)n * ldk;
    float s = 0.0f;
    for (uint32_t i = 0; i < K; ++i) s += qr[i] * kr[i];
    if (s > m) m = s;
  }
  float sum = 0.0f;
  for (uint32_t n = 0; n < N; ++n) {
    const float *kr = k + (size_t)n * ldk;
    float s = 0.0f;
    for (uint32_t i = 0; i < K; ++i) s += qr[i] * kr[i];
    sum += expf(s - m);
  }
  const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
  for (uint32_t d = 0; d < D; ++d) {
    float out = 0.0f;
    for (uint32_t n = 0; n < N; ++n) {
      const float *kr = k + (size_t)n * ldk;
      float s = 0.0f;
      for (uint32_t i = 0; i < K; ++i) s += qr[i] * kr[i];
      out += expf(s - m) * inv * v[(size_t)n * ldv + d];
    }
    orow[d] = out;
  }
}

void bwpp_oracle_attention_f32(const float *q, const float *k, const float *v,
                               float *o, uint32_t M, uint32_t N, uint32_t K,
                               uint32_t D, uint32_t ldq, uint32_t ldk,
                               uint32_t ldv, uint32_t ldo) {
  if (!q || !k || !v || !o) return;
  for (uint32_t m = 0; m < M; ++m)
    oracle_attention_row(q + (size_t)m * ldq, k, v, o + (size_t)m * ldo, N, K,
                         D, ldk, ldv);
}

void bwpp_oracle_reduce_max_mask_f32(const float *x, float *mask,
                                     uint32_t rows, uint32_t cols, int axis) {
  if (!x || !mask) return;
  memset(mask, 0, sizeof(float) * (size_t)rows * cols);
  if (axis == 0) {
    for (uint32_t c = 0; c < cols; ++c) {
      float m = -INFINITY;
      for (uint32_t r = 0; r < rows; ++r)
        if (x[(size_t)r * cols + c] > m) m = x[(size_t)r * cols + c];
      for (uint32_t r = 0; r < rows; ++r)
        if (x[(size_t)r * cols + c] == m) mask[(size_t)r * cols + c] = 1.0f;
    }
  } else {
    for (uint32_t r = 0; r < rows; ++r) {
      const float *xr = x + (size_t)r * cols;
      float m = -INFINITY;
      for (uint32_t c = 0; c < cols; ++c)
        if (xr[c] > m) m = xr[c];
      for (uint32_t c = 0; c < cols; ++c)
        if (xr[c] == m) mask[(size_t)r * cols + c] = 1.0f;
    }
  }
}

void bwpp_oracle_reduce_max_grad_f32(const float *mask, const float *dy,
                                     float *dx, uint32_t rows, uint32_t cols,
                                     int axis) {
  if (!mask || !dy || !dx) return;
  for (uint32_t r = 0; r < rows; ++r)
    for (uint32_t c = 0; c < cols; ++c) {
      const size_t i = (size_t)r * cols + c;
      dx[i] = mask[i] * (axis == 0 ? dy[c] : dy[r]);
    }
}

/* ------------------------------------------------------------------------ */
/* 2. extensions                                                            */
/* ------------------------------------------------------------------------ */

void bwpp_oracle_reduce_max_argmax_f32(const float *x, float *maxv,
                                       uint32_t *argmax, uint32_t rows,
                                       uint32_t cols, uint32_t ld) {
  for (uint32_t r = 0; r < rows; ++r) {
    const float *xr = x + (size_t)r * ld;
    float m = -INFINITY;
    uint32_t idx = 0;
    for (uint32_t c = 0; c < cols; ++c)
      if (xr[c] > m) {
        m = xr[c];
        idx = c;
      }
    if (maxv) maxv[r] = m;
    if (argmax) argmax[r] = idx;
  }
}

void bwpp_oracle_reduce_max_bwd_f32(const uint32_t *argmax, const float *dy,
                                    float *dx, uint32_t rows, uint32_t cols,
                                    uint32_t ld) {
  for (uint32_t r = 0; r < rows; ++r) {
    float *dr = dx + (size_t)r * ld;
    for (uint32_t c = 0; c < cols; ++c) dr[c] = 0.0f;
    if (argmax[r] < cols) dr[argmax[r]] = dy[r];
  }
}

void bwpp_oracle_layernorm_f32(const float *x, float *y, const float *gamma,
                               const float *beta, uint32_t rows, uint32_t cols,
                               uint32_t ld, float eps) {
  for (uint32_t r = 0; r < rows; ++r) {
    const float *xr = x + (size_t)r * ld;
    float *yr = y + (size_t)r * ld;
    double s = 0.0;
    for (uint32_t c = 0; c < cols; ++c) s += xr[c];
    const double mean = s / cols;
    double v = 0.0;
    for (uint32_t c = 0; c < cols; ++c) v += (xr[c] - mean) * (xr[c] - mean);
    const double rstd = 1.0 / sqrt(v / cols + (double)eps);
    for (uint32_t c = 0; c < cols; ++c) {
      double t = (xr[c] - mean) * rstd;
      if (gamma) t *= gamma[c];
      if (beta) t += beta[c];
      yr[c] = (float)t;
    }
  }
}

/* shared body of the two norm backward passes; `centered` selects layernorm */
static void oracle_norm_bwd(const float *x, const float *gamma, const float *dy,
                            float *dx, float *dgamma, float *dbeta,
                            uint32_t rows, uint32_t cols, uint32_t ld,
                            float eps, int centered) {
  double *dg = dgamma ? (double *)calloc(cols, sizeof(double)) : NULL;
  double *db = dbeta ? (double *)calloc(cols, sizeof(double)) : NULL;
  for (uint32_t r = 0; r < rows; ++r) {
    const float *xr = x + (size_t)r * ld;
    const float *gr = dy + (size_t)r * ld;
    double mean = 0.0;
    if (centered) {
      for (uint32_t c = 0; c < cols; ++c) mean += xr[c];
      mean /= cols;
    }
    double ss = 0.0;
    for (uint32_t c = 0; c < cols; ++c) ss += (xr[c] - mean) * (xr[c] - mean);
    const double rs = 1.0 / sqrt(ss / cols + (double)eps);
    double mg = 0.0, mgx = 0.0;
    for (uint32_t c = 0; c < cols; ++c) {
      const double g = (gamma ? gamma[c] : 1.0) * gr[c];
      const double xh = (xr[c] - mean) * rs;
      mg += g;
      mgx += g * xh;
      if (dg) dg[c] += gr[c] * xh;
      if (db) db[c] += gr[c];
    }
    mg /= cols;
    mgx /= cols;
    float *dxr = dx + (size_t)r * ld;
    for (uint32_t c = 0; c < cols; ++c) {
      const double g = (gamma ? gamma[c] : 1.0) * gr[c];
      const double xh = (xr[c] - mean) * rs;
      dxr[c] = (float)(rs * (g - (centered ? mg : 0.0) - xh * mgx));
    }
  }
  for (uint32_t c = 0; c < cols; ++c) {
    if (dg) dgamma[c] = (float)dg[c];
    if (db) dbeta[c] = (float)db[c];
  }
  free(dg);
  free(db);
}

void bwpp_oracle_rmsnorm_bwd_f32(const float *x, const float *gamma,
                                 const float *dy, float *dx, float *dgamma,
                                 float *dbeta, uint32_t rows, uint32_t cols,
                                 uint32_t ld, float eps) {
  oracle_norm_bwd(x, gamma, dy, dx, dgamma, dbeta, rows, cols, ld, eps, 0);
}

void bwpp_oracle_layernorm_bwd_f32(const float *x, const float *gamma,
                                   const float *dy, float *dx, float *dgamma,
                                   float *dbeta, uint32_t rows, uint32_t cols,
                                   uint32_t ld, float eps) {
  oracle_norm_bwd(x, gamma, dy, dx, dgamma, dbeta, rows, cols, ld, eps, 1);
}

static void oracle_attention_bhsd(const float *q, const float *k, const float *v,
                                  float *o, uint32_t B, uint32_t H, uint32_t Sq,
                                  uint32_t Skv, uint32_t D, float scale,
                                  int causal, uint32_t row_begin,
                                  uint32_t row_end, int fast) {
  if (row_end > Sq) row_end = Sq;
  float *qs = (float *)malloc(sizeof(float) * D);
  float *sc = fast ? (float *)malloc(sizeof(float) * (Skv ? Skv : 1)) : NULL;
  for (uint32_t bh = 0; bh < B * H; ++bh) {
    const float *qb = q + (size_t)bh * Sq * D;
    const float *kb = k + (size_t)bh * Skv * D;
    const float *vb = v + (size_t)bh * Skv * D;
    float *ob = o + (size_t)bh * Sq * D;
    for (uint32_t m = row_begin; m < row_end; ++m) {
      for (uint32_t i = 0; i < D; ++i) qs[i] = qb[(size_t)m * D + i] * scale;
      uint32_t n_keys = Skv;
      if (causal && m + 1 < Skv) n_keys = m + 1;
      float *orow = ob + (size_t)m * D;
      if (!fast) {
        oracle_attention_row(qs, kb, vb, orow, n_keys, D, D, D, D);
        continue;
      }
      float mx = -INFINITY;
      for (uint32_t n = 0; n < n_keys; ++n) {
        const float *kr = kb + (size_t)n * D;
        float s = 0.0f;
        for (uint32_t i = 0; i < D; ++i) s += qs[i] * kr[i];
        sc[n] = s;
        if (s > mx) mx = s;
      }
      float sum = 0.0f;
      for (uint32_t n = 0; n < n_keys; ++n) {
        sc[n] = expf(sc[n] - mx);
        sum += sc[n];
      }
      const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
      for (uint32_t d = 0; d < D; ++d) orow[d] = 0.0f;
      for (uint32_t n = 0; n < n_keys; ++n) {
        const float w = sc[n] * inv;
        const float *vr = vb + (size_t)n * D;
        for (uint32_t d = 0; d < D; ++d) orow[d] += w * vr[d];
      }
    }
  }
  free(qs);
  free(sc);
}

void bwpp_oracle_attention_bhsd_f32(const float *q, const float *k,
                                    const float *v, float *o, uint32_t B,
                                    uint32_t H, uint32_t Sq, uint32_t Skv,
                                    uint32_t D, float scale, int causal,
                                    uint32_t row_begin, uint32_t row_end) {
  oracle_attention_bhsd(q, k, v, o, B, H, Sq, Skv, D, scale, causal, row_begin,
                        row_end, 0);
}

void bwpp_oracle_attention_bhsd_fast_f32(const float *q, const float *k,
                                         const float *v, float *o, uint32_t B,
                                         uint32_t H, uint32_t Sq, uint32_t Skv,
                                         uint32_t D, float scale, int causal,
                                         uint32_t row_begin, uint32_t row_end) {
  oracle_attention_bhsd(q, k, v, o, B, H, Sq, Skv, D, scale, causal, row_begin,
                        row_end, 1);
}

void bwpp_oracle_f32_to_bf16(const float *src, uint16_t *dst, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    uint32_t u;
    memcpy(&u, &src[i], 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
      dst[i] = (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
      continue;
    }
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    dst[i] = (uint16_t)(u >> 16);
  }
}

void bwpp_oracle_bf16_to_f32(const uint16_t *src, float *dst, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    const uint32_t u = (uint32_t)src[i] << 16;
    memcpy(&dst[i], &u, 4);
  }
}

/* ---- autodiff-internal graph ops ----------------------------------------- */

void bwpp_oracle_silu_grad_f32(const float *x, const float *dy, float *dx, size_t n) {
  if (!x || !dy || !dx) return;
  for (size_t i = 0; i < n; ++i) {
    const double s = 1.0 / (1.0 + exp(-(double)x[i]));
    dx[i] = (float)((double)dy[i] * s * (1.0 + (double)x[i] * (1.0 - s)));
  }
}

void bwpp_oracle_softmax_grad_f32(const float *y, const float *dy, float *dx,
                                  uint32_t rows, uint32_t cols, uint32_t ld) {
  if (!y || !dy || !dx) return;
  for (uint32_t r = 0; r < rows; ++r) {
    const float *yr = y + (size_t)r * ld, *gr = dy + (size_t)r * ld;
    double dot = 0.0;
    for (uint32_t c = 0; c < cols; ++c) dot += (double)yr[c] * (double)gr[c];
    float *dr = dx + (size_t)r * ld;
    for (uint32_t c = 0; c < cols; ++c) dr[c] = (float)((double)yr[c] * ((double)gr[c] - dot));
  }
}

void bwpp_oracle_reduce_sum_f32(const float *x, float *out, uint32_t rows,
                                uint32_t cols, uint32_t ld, int axis) {
  if (!out) return;
  if (axis == 1) {
    for (uint32_t r = 0; r < rows; ++r) {
      double s = 0.0;
      for (uint32_t c = 0; c < cols; ++c) s += x[(size_t)r * ld + c];
      out[r] = (float)s;
    }
  } else {
    for (uint32_t c = 0; c < cols; ++c) {
      double s = 0.0;
      for (uint32_t r = 0; r < rows; ++r) s += x[(size_t)r * ld + c];
      out[c] = (float)s;
    }
  }
}

void bwpp_oracle_broadcast_f32(const float *src, float *dst, uint32_t rows,
                               uint32_t cols, uint32_t ld, int axis) {
  if (!src || !dst) return;
  for (uint32_t r = 0; r < rows; ++r)
    for (uint32_t c = 0; c < cols; ++c) dst[(size_t)r * ld + c] = axis == 1 ? src[r] : src[c];
}
