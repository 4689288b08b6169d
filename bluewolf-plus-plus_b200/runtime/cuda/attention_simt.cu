// Attention on CUDA cores for the shapes the tcgen05 kernel does not take
// (head dims other than 64/128, Kd != Dv, strided 2-D views from the Metal /
// CPU mirrors).  One warp per query row, single-pass online softmax
// (compiler/codegen_metal.c:534-548): running max m, running sum l, output
// accumulator rescaled by exp(m_old - m_new) whenever the max grows.
#include <math.h>

#include "bwpp_cuda_internal.cuh"

namespace {

constexpr int kMaxPerLane = 8;  // head dims up to 256

// F16 = false: bf16 Q/K/V, fp32 O.  F16 = true (the half ABI): f16 Q/K/V and
// f16 O (rounded to nearest even once, at the end).
template <bool F16>
__global__ void __launch_bounds__(128)
    attention_simt_kernel(const uint16_t *__restrict__ q,
                          const uint16_t *__restrict__ k,
                          const uint16_t *__restrict__ v, void *__restrict__ o,
                          uint32_t BH, uint32_t Sq, uint32_t Skv, uint32_t Kd,
                          uint32_t Dv, uint64_t q_bh, uint64_t k_bh,
                          uint64_t v_bh, uint64_t o_bh, uint32_t ldq,
                          uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale,
                          int causal) {
  const int lane = threadIdx.x & 31;
  const uint64_t row_id = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row_id >= (uint64_t)BH * Sq) return;
  const uint32_t bh = (uint32_t)(row_id / Sq), m = (uint32_t)(row_id % Sq);
  const uint16_t *qr = q + bh * q_bh + (uint64_t)m * ldq;
  const uint16_t *kb = k + bh * k_bh;
  const uint16_t *vb = v + bh * v_bh;
  float qv[kMaxPerLane], acc[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const uint32_t d = lane + 32 * i;
    qv[i] = d < Kd ? load16<F16>(qr[d]) : 0.0f;
    acc[i] = 0.0f;
  }
  uint32_t nk = Skv;
  if (causal && m + 1 < Skv) nk = m + 1;
  float mx = -INFINITY, l = 0.0f;
  for (uint32_t n = 0; n < nk; ++n) {
    const uint16_t *kr = kb + (uint64_t)n * ldk;
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const uint32_t d = lane + 32 * i;
      if (d < Kd) s += qv[i] * load16<F16>(kr[d]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    s *= scale;
    const float mn = fmaxf(mx, s);
    const float corr = expf(mx - mn);
    const float p = expf(s - mn);
    l = l * corr + p;
    const uint16_t *vr = vb + (uint64_t)n * ldv;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const uint32_t d = lane + 32 * i;
      const float vv = d < Dv ? load16<F16>(vr[d]) : 0.0f;
      acc[i] = acc[i] * corr + p * vv;
    }
    mx = mn;
  }
  const float inv = l > 0.0f ? 1.0f / l : 0.0f;
  const uint64_t ob = bh * o_bh + (uint64_t)m * ldo;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const uint32_t d = lane + 32 * i;
    if (d < Dv) {
      if (F16) static_cast<uint16_t *>(o)[ob + d] = (uint16_t)pack2_16<true>(acc[i] * inv, 0.0f);
      else static_cast<float *>(o)[ob + d] = acc[i] * inv;
    }
  }
}

}  // namespace

// o: fp32 (f16 == 0, bf16 inputs) or f16 (f16 == 1, f16 inputs)
int bwpp_attention_simt_launch(BwppCudaCtx *ctx, const uint16_t *q,
                               const uint16_t *k, const uint16_t *v, void *o,
                               uint32_t BH, uint32_t Sq, uint32_t Skv,
                               uint32_t Kd, uint32_t Dv, uint64_t q_bh,
                               uint64_t k_bh, uint64_t v_bh, uint64_t o_bh,
                               uint32_t ldq, uint32_t ldk, uint32_t ldv,
                               uint32_t ldo, float scale, int causal, int f16) {
  if (Kd > 32 * kMaxPerLane || Dv > 32 * kMaxPerLane)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED,
                          "attention: head dims above 256 are not supported");
  const uint64_t rows = (uint64_t)BH * Sq;
  if (rows == 0 || Dv == 0) return BWPP_CUDA_OK;
  const uint64_t blocks = (rows + 3) / 4;
  if (blocks > 0x7fffffffull)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "attention: too many rows");
  if (f16)
    attention_simt_kernel<true><<<(unsigned)blocks, 128, 0, ctx->stream>>>(
        q, k, v, o, BH, Sq, Skv, Kd, Dv, q_bh, k_bh, v_bh, o_bh, ldq, ldk, ldv, ldo, scale, causal);
  else
    attention_simt_kernel<false><<<(unsigned)blocks, 128, 0, ctx->stream>>>(
        q, k, v, o, BH, Sq, Skv, Kd, Dv, q_bh, k_bh, v_bh, o_bh, ldq, ldk, ldv, ldo, scale, causal);
  BWPP_LAUNCH_CHECK(ctx, "attention simt");
  return BWPP_CUDA_OK;
}
