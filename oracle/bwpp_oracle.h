/*
 * bwpp_oracle.h -- CPU restatement of the BW++ hot path, used ONLY as a
 * test / benchmark checker.  Nothing in the shipped CUDA runtime links or
 * calls this code; only tests/, __graft_entry__.smoke() and the cpu_baseline
 * leg of bench.py load it.
 *
 * Two groups of functions:
 *
 *  1. Restatements of runtime/cpu/bwpp_cpu_ref.c (reference project).  They
 *     keep the reference's fp32 operation order, so at the same compiler
 *     flags they are bit-identical to the reference library built from the
 *     reference sources by oracle/Makefile (oracle/_ref/).  tests/test_oracle.py
 *     checks that bit-exactness and the reference tests' known answers.
 *
 *  2. Extensions the reference lacks (layernorm, norm backward, first-index
 *     argmax, batched scaled/causal attention).  "Parity unpinned by the
 *     reference": they are checked against float64 numpy restatements.
 */
#ifndef BWPP_ORACLE_H
#define BWPP_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- 1. restatements of runtime/cpu/bwpp_cpu_ref.c ---------------------- */

/* runtime/cpu/bwpp_cpu_ref.c:8-35.  Loop order is row / k / col, which keeps
 * each output element's accumulation order (k ascending from 0.0f) identical
 * to the reference's row / col / k loop, so results are bit-identical. */
void bwpp_oracle_matmul_f32(const float *a, const float *b, float *c,
                            uint32_t M, uint32_t N, uint32_t K,
                            uint32_t lda, uint32_t ldb, uint32_t ldc,
                            const float *bias, int apply_silu, int apply_bias);

/* runtime/cpu/bwpp_cpu_ref.c:37-61 */
void bwpp_oracle_softmax_f32(const float *x, float *y, uint32_t rows,
                             uint32_t cols, uint32_t ld);

/* runtime/cpu/bwpp_cpu_ref.c:63-90 */
void bwpp_oracle_rmsnorm_f32(const float *x, float *y, const float *gamma,
                             const float *beta, uint32_t rows, uint32_t cols,
                             uint32_t ld, float eps);

/* runtime/cpu/bwpp_cpu_ref.c:92-144 (three passes over the keys per row) */
void bwpp_oracle_attention_f32(const float *q, const float *k, const float *v,
                               float *o, uint32_t M, uint32_t N, uint32_t K,
                               uint32_t D, uint32_t ldq, uint32_t ldk,
                               uint32_t ldv, uint32_t ldo);

/* runtime/cpu/bwpp_cpu_ref.c:146-190 (every tied maximum gets mask 1) */
void bwpp_oracle_reduce_max_mask_f32(const float *x, float *mask,
                                     uint32_t rows, uint32_t cols, int axis);

/* runtime/cpu/bwpp_cpu_ref.c:192-219 */
void bwpp_oracle_reduce_max_grad_f32(const float *mask, const float *dy,
                                     float *dx, uint32_t rows, uint32_t cols,
                                     int axis);

/* ---- 2. extensions (parity unpinned by the reference) ------------------- */

/* Row-wise max and FIRST index of the max (strict '>' scan from -INF, index 0
 * when no element exceeds -INF).  Same scan rule as
 * runtime/cpu/bwpp_cpu_ref.c:174-181, but it keeps one index instead of a
 * mask with every tie set. */
void bwpp_oracle_reduce_max_argmax_f32(const float *x, float *maxv,
                                       uint32_t *argmax, uint32_t rows,
                                       uint32_t cols, uint32_t ld);

/* dx[r, argmax[r]] = dy[r]; every other element 0. */
void bwpp_oracle_reduce_max_bwd_f32(const uint32_t *argmax, const float *dy,
                                    float *dx, uint32_t rows, uint32_t cols,
                                    uint32_t ld);

/* y = (x - mean) * rstd * gamma + beta, rstd = 1/sqrt(var + eps); float64
 * accumulation.  gamma / beta may be NULL (1 / 0). */
void bwpp_oracle_layernorm_f32(const float *x, float *y, const float *gamma,
                               const float *beta, uint32_t rows, uint32_t cols,
                               uint32_t ld, float eps);

/* RMSNorm backward (rule of compiler/graph_ir.c:1735-1789, dgamma computed
 * directly as sum(dy * x * r) instead of through (y - beta) / gamma):
 *   r = 1/sqrt(mean(x^2) + eps), xhat = x*r, g = gamma*dy
 *   dx = r * (g - xhat * mean(g*xhat)); dgamma = sum_rows dy*xhat;
 *   dbeta = sum_rows dy.
 * dgamma / dbeta may be NULL; gamma NULL means 1. float64 accumulation. */
void bwpp_oracle_rmsnorm_bwd_f32(const float *x, const float *gamma,
                                 const float *dy, float *dx, float *dgamma,
                                 float *dbeta, uint32_t rows, uint32_t cols,
                                 uint32_t ld, float eps);

/* LayerNorm backward: g = gamma*dy,
 *   dx = rstd * (g - mean(g) - xhat * mean(g*xhat)),
 *   dgamma = sum_rows dy*xhat, dbeta = sum_rows dy. */
void bwpp_oracle_layernorm_bwd_f32(const float *x, const float *gamma,
                                   const float *dy, float *dx, float *dgamma,
                                   float *dbeta, uint32_t rows, uint32_t cols,
                                   uint32_t ld, float eps);

/* Batched attention on [B,H,S,D] contiguous tensors, rows [row_begin,
 * row_end) of every (b,h) only.  Each query row is pre-scaled by `scale` in
 * fp32 and handed to the three-pass restatement above with M=1; causal rows
 * use N = m+1 keys (key n visible iff n <= m).  Rows outside the range are
 * left untouched. */
void bwpp_oracle_attention_bhsd_f32(const float *q, const float *k,
                                    const float *v, float *o, uint32_t B,
                                    uint32_t H, uint32_t Sq, uint32_t Skv,
                                    uint32_t D, float scale, int causal,
                                    uint32_t row_begin, uint32_t row_end);

/* Same contract as bwpp_oracle_attention_bhsd_f32, but two-pass: the row's
 * scores are computed once into a scratch row (the three-pass form recomputes
 * them D+2 times).  Used for sampled checks at full size. */
void bwpp_oracle_attention_bhsd_fast_f32(const float *q, const float *k,
                                         const float *v, float *o, uint32_t B,
                                         uint32_t H, uint32_t Sq, uint32_t Skv,
                                         uint32_t D, float scale, int causal,
                                         uint32_t row_begin, uint32_t row_end);

/* Autodiff-internal graph ops (compiler/include/graph_ir.h:42-55; the
 * reference has rules, compiler/graph_ir.c:1414-1470,1709-1733,1791-1796,
 * but no kernels).  float64 arithmetic, rounded to fp32 once. */

/* dx = dy * s * (1 + x * (1 - s)), s = 1 / (1 + exp(-x)) over n elements. */
void bwpp_oracle_silu_grad_f32(const float *x, const float *dy, float *dx, size_t n);

/* dx[r, c] = y[r, c] * (dy[r, c] - sum_j dy[r, j] * y[r, j]). */
void bwpp_oracle_softmax_grad_f32(const float *y, const float *dy, float *dx,
                                  uint32_t rows, uint32_t cols, uint32_t ld);

/* axis 1: out[r] = sum_c x[r, c]; axis 0: out[c] = sum_r x[r, c]. */
void bwpp_oracle_reduce_sum_f32(const float *x, float *out, uint32_t rows,
                                uint32_t cols, uint32_t ld, int axis);

/* dst[r, c] = src[axis == 1 ? r : c]. */
void bwpp_oracle_broadcast_f32(const float *src, float *dst, uint32_t rows,
                               uint32_t cols, uint32_t ld, int axis);

/* Host float -> bf16 bits, round to nearest even (NaN kept quiet). */
void bwpp_oracle_f32_to_bf16(const float *src, uint16_t *dst, size_t n);
/* bf16 bits -> float (exact). */
void bwpp_oracle_bf16_to_f32(const uint16_t *src, float *dst, size_t n);

#ifdef __cplusplus
}
#endif

#endif
