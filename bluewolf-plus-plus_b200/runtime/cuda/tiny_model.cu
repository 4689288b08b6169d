// tiny_model training step (the block of
// examples/tiny_model.bwpp:4-58 with the config's changes): L pre-RMSNorm
// decoder layers, each
//   n1 = rmsnorm(h, g1);  [q k v] = n1 Wqkv;  o = causal_attention(q, k, v)
//   h  = h + o Wo;  n2 = rmsnorm(h, g2);  [g u] = n2 W13;  a = silu(g) * u
//   h  = h + a W2
// then loss = mean((h - target)^2).  Forward, backward (autodiff rules of
// compiler/graph_ir.c:1529-1583 matmul, 1709-1720 silu, 1735-1789 rmsnorm,
// plus the attention backward), optional NCCL allreduce of the gradients
// (one bucket per layer, on a side stream, overlapped with the backward of
// the layers below),
// and an SGD update of the fp32 master weights with bf16 compute copies.
//
// Every product runs on the tcgen05 GEMM / attention kernels; the transposed
// products of the backward use the GEMM's MN-major / K-major operand forms,
// so nothing is transposed in memory.  Parameters and gradients are single
// flat fp32 buffers (one allreduce bucket per layer).
#include <stdlib.h>
#include <string.h>

#include "bwpp_cuda_internal.cuh"

int bwpp_gemm_launch_ex(BwppCudaCtx *ctx, const uint16_t *a, int a_mn, uint32_t lda,
                        const uint16_t *b, int b_mn, uint32_t ldb, void *c, uint32_t ldc,
                        uint32_t M, uint32_t N, uint32_t K, const float *bias, int silu,
                        const float *residual, uint32_t ldr, int out_bf16, int force_simt);
int bwpp_gemm_launch_glu_bwd(BwppCudaCtx *ctx, const uint16_t *a, int a_mn, uint32_t lda,
                             const uint16_t *b, int b_mn, uint32_t ldb, const uint16_t *gu,
                             uint16_t *dgu, uint32_t ldgu, uint32_t M, uint32_t F, uint32_t K);
int bwpp_cast_launch(BwppCudaCtx *ctx, const float *src, uint16_t *dst, uint32_t rows,
                     uint32_t cols, uint32_t ld_src, uint32_t ld_dst);
int bwpp_rmsnorm_bf16out(BwppCudaCtx *ctx, const float *x, const float *gamma, uint16_t *y,
                         uint32_t rows, uint32_t cols, float eps);
int bwpp_norm_bwd_with_scratch(BwppCudaCtx *ctx, int centered, const float *x,
                               const float *gamma, const float *dy, float *dx, float *dgamma,
                               float *dbeta, uint32_t rows, uint32_t cols, uint32_t ld,
                               float eps, float *scratch);
int bwpp_swiglu_fwd(BwppCudaCtx *ctx, const uint16_t *gu, uint16_t *a, uint32_t rows, uint32_t F);
int bwpp_swiglu_bwd(BwppCudaCtx *ctx, const uint16_t *gu, const float *da, uint16_t *dgu,
                    uint32_t rows, uint32_t F);
int bwpp_mse(BwppCudaCtx *ctx, const float *h, const float *t, float *dh, uint16_t *dh16,
             float *part, float *loss, size_t n);
int bwpp_attn_delta(BwppCudaCtx *ctx, const uint16_t *dO, const uint16_t *O, float *delta,
                    uint32_t B, uint32_t S, uint32_t H, uint32_t Dh);
int bwpp_sgd(BwppCudaCtx *ctx, float *w, const float *g, uint16_t *w16, size_t n, float lr);
int bwpp_add(BwppCudaCtx *ctx, float *a, const float *b, size_t n);
int bwpp_norm_bwd_accumulate(BwppCudaCtx *ctx, int centered, const float *x,
                             const float *gamma, const float *dy, float *acc,
                             uint16_t *acc16, float *dgamma, float *dbeta,
                             uint32_t rows, uint32_t cols, uint32_t ld, float eps,
                             float *scratch);
int bwpp_fill_normal(BwppCudaCtx *ctx, float *w, size_t n, uint64_t seed, float mean,
                     float stddev);
int bwpp_attention_fwd_train(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                             const uint16_t *v, uint32_t ld_in, uint32_t B, uint32_t H,
                             uint32_t S, uint32_t D, float scale, int causal, uint16_t *o,
                             uint32_t ldo, float *lse);
int bwpp_attention_bwd_train(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                             const uint16_t *v, uint32_t ld_in, const uint16_t *dout,
                             uint32_t ld_do, const float *lse, const float *delta,
                             uint32_t B, uint32_t H, uint32_t S, float scale, int causal,
                             uint16_t *dq, uint16_t *dk, uint16_t *dv, uint32_t ldd);
int bwpp_comm_nranks(const BwppCudaComm *c);

namespace {

struct LayerParams {
  size_t g1, wqkv, wo, g2, w13, w2;  // offsets into the flat parameter buffer
};

struct LayerActs {
  float *h_in, *h_mid, *lse;
  uint16_t *n1, *qkv, *o, *n2, *gu, *a;
};

}  // namespace

struct BwppCudaTinyModel {
  BwppCudaCtx *ctx;
  BwppCudaTinyModelConfig cfg;
  size_t nparams;
  float *params, *grads;
  uint16_t *params16;
  LayerParams lp[16];
  LayerActs act[16];
  float *h_out;      // final hidden state [T, D]
  float *target;     // staged regression target [T, D]
  float *dh, *dtmp;  // fp32 [T, D]
  uint16_t *dh16;    // bf16 [T, D]
  float *da;         // fp32 [T, F]
  uint16_t *dgu;     // bf16 [T, 2F]
  uint16_t *dout;    // bf16 [T, D]
  uint16_t *dqkv;    // bf16 [T, 3D]
  float *delta;      // [B*H, S]
  float *part, *loss;
  float *norm_scratch;
  void *arena;       // one cudaMalloc for everything above
  // gradient allreduce overlapped with the backward: one bucket per layer
  cudaStream_t comm_stream;
  // two gradient buckets per layer (FFN part, then attention part)
  cudaEvent_t grad_ready[32], bucket_done[32];
};

namespace {

size_t align_up(size_t v) { return (v + 255) & ~(size_t)255; }

// Sums gradient bucket b (count floats at g) over the ranks on the comm
// stream once the backward has produced it; every rank issues the buckets
// in the same order.
int allreduce_bucket(BwppCudaCtx *ctx, BwppCudaTinyModel *m, BwppCudaComm *comm, uint32_t b,
                     float *g, size_t count) {
  int rc = bwpp_check_cuda(ctx, cudaEventRecord(m->grad_ready[b], ctx->stream), "grad event");
  if (!rc)
    rc = bwpp_check_cuda(ctx, cudaStreamWaitEvent(m->comm_stream, m->grad_ready[b], 0),
                         "comm wait");
  if (!rc) rc = bwpp_cuda_comm_allreduce_sum_f32(comm, g, count, m->comm_stream);
  if (!rc)
    rc = bwpp_check_cuda(ctx, cudaEventRecord(m->bucket_done[b], m->comm_stream), "bucket event");
  return rc;
}

// dh += rmsnorm_bwd(x, gamma, dtmp) and dgamma; dh16 = bf16(dh) when given.
// One pass (the norm backward adds its dx into dh) when the row fits the
// register-resident kernel; else the norm backward, an add and a cast.
int norm_bwd_into_dh(BwppCudaCtx *ctx, BwppCudaTinyModel *m, const float *x,
                     const float *gamma, float *dgamma, uint32_t T, uint32_t D, float eps,
                     uint16_t *dh16) {
  int rc = bwpp_norm_bwd_accumulate(ctx, 0, x, gamma, m->dtmp, m->dh, dh16, dgamma, nullptr, T,
                                    D, D, eps, m->norm_scratch);
  if (rc != BWPP_CUDA_ERR_UNSUPPORTED) return rc;
  rc = bwpp_norm_bwd_with_scratch(ctx, 0, x, gamma, m->dtmp, m->dtmp, dgamma, nullptr, T, D, D,
                                  eps, m->norm_scratch);
  if (!rc) rc = bwpp_add(ctx, m->dh, m->dtmp, (size_t)T * D);
  if (!rc && dh16) rc = bwpp_cast_launch(ctx, m->dh, dh16, T, D, D, D);
  return rc;
}

}  // namespace

extern "C" {

int bwpp_cuda_tiny_model_create(BwppCudaCtx *ctx, const BwppCudaTinyModelConfig *cfg,
                                uint64_t seed, BwppCudaTinyModel **out) {
  if (!ctx || !cfg || !out) return BWPP_CUDA_ERR_ARG;
  *out = nullptr;
  const BwppCudaTinyModelConfig c = *cfg;
  if (c.layers == 0 || c.layers > 16 || c.head_dim != 128 || c.d_model != c.heads * c.head_dim ||
      c.seq % 128 || c.d_model % 64 || c.ffn % 64 || c.batch == 0)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED,
                          "tiny_model: needs head_dim 128, d_model = heads*128, seq %% 128 == 0");
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  BwppCudaTinyModel *m = (BwppCudaTinyModel *)calloc(1, sizeof(BwppCudaTinyModel));
  if (!m) return BWPP_CUDA_ERR;
  m->ctx = ctx;
  m->cfg = c;
  const size_t D = c.d_model, F = c.ffn, T = (size_t)c.batch * c.seq;
  // parameter layout per layer: g1, wqkv [D,3D], wo [D,D], g2, w13 [D,2F], w2 [F,D]
  size_t off = 0;
  for (uint32_t l = 0; l < c.layers; ++l) {
    LayerParams &p = m->lp[l];
    p.g1 = off; off += D;
    p.wqkv = off; off += D * 3 * D;
    p.wo = off; off += D * D;
    p.g2 = off; off += D;
    p.w13 = off; off += D * 2 * F;
    p.w2 = off; off += F * D;
  }
  m->nparams = off;
  // one arena: params, grads, bf16 params, activations, gradient temporaries
  size_t bytes = 0;
  auto take = [&](size_t b) { size_t o = bytes; bytes += align_up(b); return o; };
  const size_t o_params = take(off * 4), o_grads = take(off * 4), o_p16 = take(off * 2);
  size_t o_act[16][9];
  for (uint32_t l = 0; l < c.layers; ++l) {
    o_act[l][0] = take(T * D * 4);                         // h_in
    o_act[l][1] = take(T * D * 4);                         // h_mid
    o_act[l][2] = take((size_t)c.batch * c.heads * c.seq * 4);  // lse
    o_act[l][3] = take(T * D * 2);                         // n1
    o_act[l][4] = take(T * 3 * D * 2);                     // qkv
    o_act[l][5] = take(T * D * 2);                         // o
    o_act[l][6] = take(T * D * 2);                         // n2
    o_act[l][7] = take(T * 2 * F * 2);                     // gu
    o_act[l][8] = take(T * F * 2);                         // a
  }
  const size_t o_tgt = take(T * D * 4);
  const size_t o_hout = take(T * D * 4), o_dh = take(T * D * 4), o_dtmp = take(T * D * 4),
               o_dh16 = take(T * D * 2), o_da = take(T * F * 4), o_dgu = take(T * 2 * F * 2),
               o_dout = take(T * D * 2), o_dqkv = take(T * 3 * D * 2),
               o_delta = take((size_t)c.batch * c.heads * c.seq * 4),
               o_part = take((size_t)ctx->num_sms * 4 * 4), o_loss = take(4),
               o_ns = take(bwpp_cuda_norm_bwd_workspace_size(ctx, (uint32_t)T, (uint32_t)D));
  rc = bwpp_check_cuda(ctx, cudaMalloc(&m->arena, bytes), "tiny_model arena");
  if (rc) {
    free(m);
    return rc;
  }
  uint8_t *A = (uint8_t *)m->arena;
  m->params = (float *)(A + o_params);
  m->grads = (float *)(A + o_grads);
  m->params16 = (uint16_t *)(A + o_p16);
  for (uint32_t l = 0; l < c.layers; ++l) {
    LayerActs &a = m->act[l];
    a.h_in = (float *)(A + o_act[l][0]);
    a.h_mid = (float *)(A + o_act[l][1]);
    a.lse = (float *)(A + o_act[l][2]);
    a.n1 = (uint16_t *)(A + o_act[l][3]);
    a.qkv = (uint16_t *)(A + o_act[l][4]);
    a.o = (uint16_t *)(A + o_act[l][5]);
    a.n2 = (uint16_t *)(A + o_act[l][6]);
    a.gu = (uint16_t *)(A + o_act[l][7]);
    a.a = (uint16_t *)(A + o_act[l][8]);
  }
  m->h_out = (float *)(A + o_hout);
  m->target = (float *)(A + o_tgt);
  m->dh = (float *)(A + o_dh);
  m->dtmp = (float *)(A + o_dtmp);
  m->dh16 = (uint16_t *)(A + o_dh16);
  m->da = (float *)(A + o_da);
  m->dgu = (uint16_t *)(A + o_dgu);
  m->dout = (uint16_t *)(A + o_dout);
  m->dqkv = (uint16_t *)(A + o_dqkv);
  m->delta = (float *)(A + o_delta);
  m->part = (float *)(A + o_part);
  m->loss = (float *)(A + o_loss);
  m->norm_scratch = (float *)(A + o_ns);
  // init: matrices ~ N(0, 0.02), norm gains 1; bf16 copies
  for (uint32_t l = 0; l < c.layers && !rc; ++l) {
    const LayerParams &p = m->lp[l];
    rc = bwpp_fill_normal(ctx, m->params + p.g1, D, seed * 16 + 6 * l + 0, 1.0f, 0.0f);
    if (!rc) rc = bwpp_fill_normal(ctx, m->params + p.wqkv, D * 3 * D, seed * 16 + 6 * l + 1, 0.0f, 0.02f);
    if (!rc) rc = bwpp_fill_normal(ctx, m->params + p.wo, D * D, seed * 16 + 6 * l + 2, 0.0f, 0.02f);
    if (!rc) rc = bwpp_fill_normal(ctx, m->params + p.g2, D, seed * 16 + 6 * l + 3, 1.0f, 0.0f);
    if (!rc) rc = bwpp_fill_normal(ctx, m->params + p.w13, D * 2 * F, seed * 16 + 6 * l + 4, 0.0f, 0.02f);
    if (!rc) rc = bwpp_fill_normal(ctx, m->params + p.w2, F * D, seed * 16 + 6 * l + 5, 0.0f, 0.02f);
  }
  if (!rc) rc = bwpp_sgd(ctx, m->params, m->grads, m->params16, off, 0.0f);  // bf16 copies
  if (!rc)
    rc = bwpp_check_cuda(ctx, cudaMemsetAsync(m->grads, 0, off * 4, ctx->stream), "grads");
  if (!rc)
    rc = bwpp_check_cuda(ctx, cudaStreamCreateWithFlags(&m->comm_stream, cudaStreamNonBlocking),
                         "comm stream");
  for (uint32_t b = 0; b < 2 * c.layers && !rc; ++b) {
    rc = bwpp_check_cuda(ctx, cudaEventCreateWithFlags(&m->grad_ready[b], cudaEventDisableTiming),
                         "grad event");
    if (!rc)
      rc = bwpp_check_cuda(ctx, cudaEventCreateWithFlags(&m->bucket_done[b], cudaEventDisableTiming),
                           "bucket event");
  }
  if (rc) {
    for (uint32_t b = 0; b < 2 * c.layers; ++b) {
      if (m->grad_ready[b]) cudaEventDestroy(m->grad_ready[b]);
      if (m->bucket_done[b]) cudaEventDestroy(m->bucket_done[b]);
    }
    if (m->comm_stream) cudaStreamDestroy(m->comm_stream);
    cudaFree(m->arena);
    free(m);
    return rc;
  }
  *out = m;
  return BWPP_CUDA_OK;
}

int bwpp_cuda_tiny_model_destroy(BwppCudaTinyModel *m) {
  if (!m) return BWPP_CUDA_ERR_ARG;
  bwpp_ctx_enter(m->ctx);
  cudaStreamSynchronize(m->ctx->stream);
  cudaStreamSynchronize(m->comm_stream);
  for (uint32_t b = 0; b < 2 * m->cfg.layers; ++b) {
    cudaEventDestroy(m->grad_ready[b]);
    cudaEventDestroy(m->bucket_done[b]);
  }
  cudaStreamDestroy(m->comm_stream);
  cudaFree(m->arena);
  free(m);
  return BWPP_CUDA_OK;
}

size_t bwpp_cuda_tiny_model_param_count(const BwppCudaTinyModel *m) { return m ? m->nparams : 0; }

int bwpp_cuda_tiny_model_get(BwppCudaTinyModel *m, float *params_out, float *grads_out) {
  if (!m) return BWPP_CUDA_ERR_ARG;
  int rc = bwpp_ctx_enter(m->ctx);
  if (rc) return rc;
  if (params_out)
    rc = bwpp_check_cuda(m->ctx, cudaMemcpyAsync(params_out, m->params, m->nparams * 4,
                                                 cudaMemcpyDefault, m->ctx->stream),
                         "params out");
  if (!rc && grads_out)
    rc = bwpp_check_cuda(m->ctx, cudaMemcpyAsync(grads_out, m->grads, m->nparams * 4,
                                                 cudaMemcpyDefault, m->ctx->stream),
                         "grads out");
  if (rc) return rc;
  return bwpp_cuda_sync(m->ctx);
}

int bwpp_cuda_tiny_model_input_grad(BwppCudaTinyModel *m, float *dx_out) {
  if (!m || !dx_out) return BWPP_CUDA_ERR_ARG;
  int rc = bwpp_ctx_enter(m->ctx);
  if (rc) return rc;
  // after the backward of layer 0, dh holds d loss / d h_in(0) = d loss / d x
  const size_t n = (size_t)m->cfg.batch * m->cfg.seq * m->cfg.d_model;
  rc = bwpp_check_cuda(m->ctx, cudaMemcpyAsync(dx_out, m->dh, n * 4, cudaMemcpyDefault,
                                               m->ctx->stream),
                       "input grad out");
  if (rc) return rc;
  return bwpp_cuda_sync(m->ctx);
}

int bwpp_cuda_tiny_model_set_params(BwppCudaTinyModel *m, const float *params_in) {
  if (!m || !params_in) return BWPP_CUDA_ERR_ARG;
  int rc = bwpp_ctx_enter(m->ctx);
  if (rc) return rc;
  rc = bwpp_check_cuda(m->ctx, cudaMemcpyAsync(m->params, params_in, m->nparams * 4,
                                               cudaMemcpyDefault, m->ctx->stream),
                       "params in");
  if (!rc) rc = bwpp_sgd(m->ctx, m->params, m->grads, m->params16, m->nparams, 0.0f);
  if (rc) return rc;
  return bwpp_cuda_sync(m->ctx);
}

int bwpp_cuda_tiny_model_step(BwppCudaTinyModel *m, const float *x, const float *target,
                              float lr, BwppCudaComm *comm, float *loss_out) {
  if (!m || !x || !target) return BWPP_CUDA_ERR_ARG;
  BwppCudaCtx *ctx = m->ctx;
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  const BwppCudaTinyModelConfig &c = m->cfg;
  const uint32_t D = c.d_model, F = c.ffn, H = c.heads, S = c.seq, B = c.batch;
  const uint32_t T = B * S;
  const float scale = 1.0f / sqrtf((float)c.head_dim);
  float *P = m->params;
  float *G = m->grads;
  uint16_t *P16 = m->params16;
#define TRY(expr)      \
  do {                 \
    rc = (expr);       \
    if (rc) return rc; \
  } while (0)
  // ---------------- forward
  // x and target may be host or device memory
  TRY(bwpp_check_cuda(ctx, cudaMemcpyAsync(m->act[0].h_in, x, (size_t)T * D * 4,
                                           cudaMemcpyDefault, ctx->stream),
                      "input copy"));
  TRY(bwpp_check_cuda(ctx, cudaMemcpyAsync(m->target, target, (size_t)T * D * 4,
                                           cudaMemcpyDefault, ctx->stream),
                      "target copy"));
  for (uint32_t l = 0; l < c.layers; ++l) {
    const LayerParams &p = m->lp[l];
    LayerActs &a = m->act[l];
    float *h_next = l + 1 < c.layers ? m->act[l + 1].h_in : m->h_out;
    TRY(bwpp_rmsnorm_bf16out(ctx, a.h_in, P + p.g1, a.n1, T, D, c.eps));
    TRY(bwpp_gemm_launch_ex(ctx, a.n1, 0, D, P16 + p.wqkv, 1, 3 * D, a.qkv, 3 * D, T, 3 * D, D,
                            nullptr, 0, nullptr, 0, 1, 0));
    TRY(bwpp_attention_fwd_train(ctx, a.qkv, a.qkv + D, a.qkv + 2 * D, 3 * D, B, H, S,
                                 c.head_dim, scale, 1, a.o, D, a.lse));
    TRY(bwpp_gemm_launch_ex(ctx, a.o, 0, D, P16 + p.wo, 1, D, a.h_mid, D, T, D, D, nullptr, 0,
                            a.h_in, D, 0, 0));
    TRY(bwpp_rmsnorm_bf16out(ctx, a.h_mid, P + p.g2, a.n2, T, D, c.eps));
    TRY(bwpp_gemm_launch_ex(ctx, a.n2, 0, D, P16 + p.w13, 1, 2 * F, a.gu, 2 * F, T, 2 * F, D,
                            nullptr, 0, nullptr, 0, 1, 0));
    TRY(bwpp_swiglu_fwd(ctx, a.gu, a.a, T, F));
    TRY(bwpp_gemm_launch_ex(ctx, a.a, 0, F, P16 + p.w2, 1, D, h_next, D, T, D, F, nullptr, 0,
                            a.h_mid, D, 0, 0));
  }
  TRY(bwpp_mse(ctx, m->h_out, m->target, m->dh, m->dh16, m->part, m->loss, (size_t)T * D));
  // ---------------- backward (dh holds d loss / d h of the current level)
  for (int l = (int)c.layers - 1; l >= 0; --l) {
    const LayerParams &p = m->lp[l];
    LayerActs &a = m->act[l];
    // h_out = h_mid + a W2
    TRY(bwpp_gemm_launch_ex(ctx, a.a, 1, F, m->dh16, 1, D, G + p.w2, D, F, D, T, nullptr, 0,
                            nullptr, 0, 0, 0));  // dW2 = a^T dh
    // da = dh W2^T and the SwiGLU backward into dgu in one GEMM (its epilogue
    // reads gu); unfused through fp32 da where that path cannot be taken
    rc = bwpp_gemm_launch_glu_bwd(ctx, m->dh16, 0, D, P16 + p.w2, 0, D, a.gu, m->dgu, 2 * F, T, F,
                                  D);
    if (rc == BWPP_CUDA_ERR_UNSUPPORTED) {
      TRY(bwpp_gemm_launch_ex(ctx, m->dh16, 0, D, P16 + p.w2, 0, D, m->da, F, T, F, D, nullptr, 0,
                              nullptr, 0, 0, 0));
      TRY(bwpp_swiglu_bwd(ctx, a.gu, m->da, m->dgu, T, F));
    } else if (rc) {
      return rc;
    }
    TRY(bwpp_gemm_launch_ex(ctx, a.n2, 1, D, m->dgu, 1, 2 * F, G + p.w13, 2 * F, D, 2 * F, T,
                            nullptr, 0, nullptr, 0, 0, 0));  // dW13 = n2^T dgu
    TRY(bwpp_gemm_launch_ex(ctx, m->dgu, 0, 2 * F, P16 + p.w13, 0, 2 * F, m->dtmp, D, T, D,
                            2 * F, nullptr, 0, nullptr, 0, 0, 0));  // dn2 = dgu W13^T
    // h_mid feeds rmsnorm(g2) and the residual: dh += rmsnorm_bwd(dn2), dh16 = bf16(dh)
    TRY(norm_bwd_into_dh(ctx, m, a.h_mid, P + p.g2, G + p.g2, T, D, c.eps, m->dh16));
    // the FFN half of layer l's gradients (g2, w13, w2) is final: its sum over
    // the ranks overlaps the attention backward of this layer
    if (comm) TRY(allreduce_bucket(ctx, m, comm, 2 * l, G + p.g2, p.w2 + (size_t)F * D - p.g2));
    // h_mid = h_in + o Wo
    TRY(bwpp_gemm_launch_ex(ctx, a.o, 1, D, m->dh16, 1, D, G + p.wo, D, D, D, T, nullptr, 0,
                            nullptr, 0, 0, 0));  // dWo = o^T dh
    TRY(bwpp_gemm_launch_ex(ctx, m->dh16, 0, D, P16 + p.wo, 0, D, m->dout, D, T, D, D, nullptr,
                            0, nullptr, 0, 1, 0));  // do = dh Wo^T (bf16)
    TRY(bwpp_attn_delta(ctx, m->dout, a.o, m->delta, B, S, H, c.head_dim));
    TRY(bwpp_attention_bwd_train(ctx, a.qkv, a.qkv + D, a.qkv + 2 * D, 3 * D, m->dout, D,
                                 a.lse, m->delta, B, H, S, scale, 1, m->dqkv, m->dqkv + D,
                                 m->dqkv + 2 * D, 3 * D));
    TRY(bwpp_gemm_launch_ex(ctx, a.n1, 1, D, m->dqkv, 1, 3 * D, G + p.wqkv, 3 * D, D, 3 * D, T,
                            nullptr, 0, nullptr, 0, 0, 0));  // dWqkv = n1^T dqkv
    TRY(bwpp_gemm_launch_ex(ctx, m->dqkv, 0, 3 * D, P16 + p.wqkv, 0, 3 * D, m->dtmp, D, T, D,
                            3 * D, nullptr, 0, nullptr, 0, 0, 0));  // dn1 = dqkv Wqkv^T
    // h_in feeds rmsnorm(g1) and the residual: dh += rmsnorm_bwd(dn1) (dh16 only
    // when a lower layer still reads it)
    TRY(norm_bwd_into_dh(ctx, m, a.h_in, P + p.g1, G + p.g1, T, D, c.eps,
                         l > 0 ? m->dh16 : nullptr));
    // and the attention half (g1, wqkv, wo), overlapping the backward of
    // layer l-1 (buckets in the same order on every rank)
    if (comm) TRY(allreduce_bucket(ctx, m, comm, 2 * l + 1, G + p.g1, p.g2 - p.g1));
  }
  // ---------------- data-parallel gradient sum (overlapped above), SGD on
  // the mean gradient once every bucket has been summed
  const int nr = comm ? bwpp_comm_nranks(comm) : 1;
  if (comm)
    for (uint32_t b = 0; b < 2 * c.layers; ++b)
      TRY(bwpp_check_cuda(ctx, cudaStreamWaitEvent(ctx->stream, m->bucket_done[b], 0),
                          "bucket wait"));
  if (lr != 0.0f) TRY(bwpp_sgd(ctx, P, G, P16, m->nparams, lr / (float)nr));
  if (loss_out)
    TRY(bwpp_check_cuda(ctx, cudaMemcpyAsync(loss_out, m->loss, 4, cudaMemcpyDefault, ctx->stream),
                        "loss readback"));
#undef TRY
  return BWPP_CUDA_OK;
}

}  // extern "C"
