// Attention entry point: O = softmax(scale * Q K^T [causal]) V on [B,H,S,D]:
// dispatch between the tcgen05 kernel (attention_tc.cu) and the CUDA-core
// kernel (attention_simt.cu).
#include "bwpp_cuda_internal.cuh"

int bwpp_attention_simt_launch(BwppCudaCtx *ctx, const uint16_t *q,
                               const uint16_t *k, const uint16_t *v, void *o,
                               uint32_t BH, uint32_t Sq, uint32_t Skv,
                               uint32_t Kd, uint32_t Dv, uint64_t q_bh,
                               uint64_t k_bh, uint64_t v_bh, uint64_t o_bh,
                               uint32_t ldq, uint32_t ldk, uint32_t ldv,
                               uint32_t ldo, float scale, int causal, int f16);

int bwpp_attention_tc_launch_f16(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                                 const uint16_t *v, uint16_t *o, uint32_t BH, uint32_t Sq,
                                 uint32_t Skv, uint32_t D, float scale, int causal);

int bwpp_attention_tc_launch(BwppCudaCtx *ctx, const uint16_t *q,
                             const uint16_t *k, const uint16_t *v, float *o,
                             uint32_t BH, uint32_t Sq, uint32_t Skv, uint32_t D,
                             float scale, int causal);

// Chooses the kernel for a batch of BH independent (Sq x Kd, Skv x Kd,
// Skv x Dv) problems with the given strides: the tcgen05 kernel for dense
// [BH, S, D] tensors with D in {64, 128}, the CUDA-core kernel otherwise.
// f16 = 0: bf16 Q/K/V, fp32 O; f16 = 1: f16 Q/K/V and f16 O.
int bwpp_attention_launch(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                          const uint16_t *v, void *o, uint32_t BH, uint32_t Sq,
                          uint32_t Skv, uint32_t Kd, uint32_t Dv, uint64_t q_bh,
                          uint64_t k_bh, uint64_t v_bh, uint64_t o_bh,
                          uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo,
                          float scale, int causal, int f16) {
  const bool dense = Kd == Dv && ldq == Kd && ldk == Kd && ldv == Dv && ldo == Dv &&
                     q_bh == (uint64_t)Sq * Kd && k_bh == (uint64_t)Skv * Kd &&
                     v_bh == (uint64_t)Skv * Dv && o_bh == (uint64_t)Sq * Dv;
  if (dense && (Kd == 64 || Kd == 128) && Skv > 0) {
    int rc = f16 ? bwpp_attention_tc_launch_f16(ctx, q, k, v, static_cast<uint16_t *>(o), BH, Sq,
                                                Skv, Kd, scale, causal)
                 : bwpp_attention_tc_launch(ctx, q, k, v, static_cast<float *>(o), BH, Sq, Skv,
                                            Kd, scale, causal);
    if (rc != BWPP_CUDA_ERR_UNSUPPORTED) return rc;
  }
  return bwpp_attention_simt_launch(ctx, q, k, v, o, BH, Sq, Skv, Kd, Dv, q_bh,
                                    k_bh, v_bh, o_bh, ldq, ldk, ldv, ldo, scale,
                                    causal, f16);
}

extern "C" int bwpp_cuda_attention_bf16(BwppCudaCtx *ctx, const uint16_t *q,
                                        const uint16_t *k, const uint16_t *v,
                                        float *o, uint32_t B, uint32_t H,
                                        uint32_t Sq, uint32_t Skv, uint32_t D,
                                        float scale, int causal) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!q || !k || !v || !o) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "attention: NULL buffer");
  const uint64_t BH = (uint64_t)B * H;
  if (BH == 0 || Sq == 0 || D == 0) return BWPP_CUDA_OK;
  if (BH > 0xFFFFFFFFull) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "attention: B*H too large");
  return bwpp_attention_launch(ctx, q, k, v, o, (uint32_t)BH, Sq, Skv, D, D,
                               (uint64_t)Sq * D, (uint64_t)Skv * D,
                               (uint64_t)Skv * D, (uint64_t)Sq * D, D, D, D, D,
                               scale, causal, 0);
}

// The half ABI (compiler/codegen_metal.c:457-556 takes half Q/K/V/O):
// f16 [B,H,S,D] in, f16 [B,H,Sq,D] out, fp32 softmax and accumulation.
extern "C" int bwpp_cuda_attention_f16(BwppCudaCtx *ctx, const uint16_t *q,
                                       const uint16_t *k, const uint16_t *v,
                                       uint16_t *o, uint32_t B, uint32_t H,
                                       uint32_t Sq, uint32_t Skv, uint32_t D,
                                       float scale, int causal) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!q || !k || !v || !o) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "attention f16: NULL buffer");
  const uint64_t BH = (uint64_t)B * H;
  if (BH == 0 || Sq == 0 || D == 0) return BWPP_CUDA_OK;
  if (BH > 0xFFFFFFFFull) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "attention: B*H too large");
  return bwpp_attention_launch(ctx, q, k, v, o, (uint32_t)BH, Sq, Skv, D, D,
                               (uint64_t)Sq * D, (uint64_t)Skv * D,
                               (uint64_t)Skv * D, (uint64_t)Sq * D, D, D, D, D,
                               scale, causal, 1);
}
