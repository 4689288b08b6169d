// Helpers shared by the attention forward (attention_tc.cu) and backward
// (attention_bwd.cu) kernels: TMA row tiles in head-major or token-major
// layout, base-2 exponent, bf16 packing, paired fp32 arithmetic.
#pragma once

#include "bwpp_cuda_internal.cuh"

namespace bwpp_attn {

constexpr int BM = 128;              // rows per Q tile
constexpr int BN = 128;              // keys per K/V block
constexpr int BOX = 128 * 64 * 2;    // one TMA box: 128 rows x 64 bf16 (16 KB)
constexpr int P_TILE = BM * BN * 2;  // a 128 x 128 bf16 tile (32 KB)

// Where the inputs come from and where the results go.
//   tok = 0: Q/K/V head-major [B*H, S, D] (tensor maps {D, S, B*H})
//   tok = 1: token-major rows t = b*S + s with head h at column h*D
//            (tensor maps {D, H, B*S}; e.g. straight out of a QKV projection)
//   out_f32: head-major fp32 [B*H, Sq, D]   (either or both outputs)
//   out_bf16: token-major 16-bit (bf16, or f16 in the f16 kernels), row
//             b*Sq + m, column h*D, pitch ldo (H = 1: head-major, pitch D)
//   lse: base-2 log-sum-exp of the scaled scores per query, [B*H, Sq]
struct AttnIO {
  float *out_f32;
  uint16_t *out_bf16;
  uint32_t ldo;
  float *lse;
  int tok;
  uint32_t H;
};

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map,
                                            uint64_t *bar, int32_t x, int32_t y,
                                            int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z),
      "r"(smem_u32(bar))
      : "memory");
}

// One tile of 128 rows (s0 .. s0+127 of head bh) as D/64 boxes of 16 KB.
template <int BOXES>
__device__ __forceinline__ void load_rows(uint8_t *dst, const CUtensorMap *map, uint64_t *bar,
                                          const AttnIO &io, uint32_t bh, uint32_t S,
                                          uint32_t s0) {
#pragma unroll
  for (int b = 0; b < BOXES; ++b) {
    if (io.tok)
      tma_load_3d(dst + b * (128 * 64 * 2), map, bar, b * 64, (int32_t)(bh % io.H),
                  (int32_t)((bh / io.H) * S + s0));
    else
      tma_load_3d(dst + b * (128 * 64 * 2), map, bar, b * 64, (int32_t)s0, (int32_t)bh);
  }
}

// TMA store of one box from this CTA's shared memory (bulk async group).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, const void *src, int32_t x,
                                             int32_t y, int32_t z, int32_t w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for two lanes on the FMA pipe, to take load off the MUFU unit
// (ex2): x = n + f with n = round(x) (magic-constant add: 1.5 * 2^23 leaves
// round(x) in the low mantissa bits), f in [-0.5, 0.5]; 2^f from a cubic
// fitted for relative error on that interval by weighted least squares on
// Chebyshev nodes (max relative error 1.4e-4, far below the 2^-9 of the bf16
// P it feeds); 2^n is added to the exponent bits.  x is clamped at -126 (the
// cubic may return just under 1, whose exponent field 126 must stay >= 126
// after adding n), so -inf (a masked score) gives about 2^-126, i.e. 0 for
// all purposes.
__device__ __forceinline__ void exp2_fma2(float x0, float x1, float &y0, float &y1) {
  const uint64_t magic = f2pack(12582912.0f, 12582912.0f);
  const uint64_t nmagic = f2pack(-12582912.0f, -12582912.0f);
  const uint64_t neg1 = f2pack(-1.0f, -1.0f);
  const uint64_t x = f2pack(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
  const uint64_t j = f2add(x, magic);
  const uint64_t n = f2add(j, nmagic);
  const uint64_t f = f2fma(n, neg1, x);  // x - n
  uint64_t p = f2fma(f, f2pack(0.05546907f, 0.05546907f), f2pack(0.24239302f, 0.24239302f));
  p = f2fma(p, f, f2pack(0.69318938f, 0.69318938f));
  p = f2fma(p, f, f2pack(0.99993980f, 0.99993980f));
  float p0, p1, j0, j1;
  f2unpack(p, p0, p1);
  f2unpack(j, j0, j1);
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(j0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(j1) << 23));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Number of 128-key blocks tile X (first row r0) needs.
__device__ __forceinline__ int blocks_for(uint32_t r0, uint32_t Sq, uint32_t Skv,
                                          int causal) {
  if (r0 >= Sq) return 0;
  int n = (int)((Skv + BN - 1) / BN);
  if (causal) {
    const uint32_t last = min(r0 + BM - 1, Sq - 1);
    n = min(n, (int)(last / BN) + 1);
  }
  return n;
}

// 10 warps: two SM sub-partitions host three warps each, which caps the
// kernel at 168 registers per thread (16384 / (3 * 32), rounded down to 8).

// Writes 16 packed bf16 pairs (32 values: columns c*32 .. c*32+31 of a row
// within a 128-column tile) into a K-major 128-byte-swizzle tile: two 64-column
// atoms of 16 KB, row r at r*128, 16-byte chunk q at (q ^ (r & 7)) * 16.
__device__ __forceinline__ void store_swizzled_chunk(uint8_t *tile, int row, int c,
                                                     const uint32_t (&pk)[16]) {
  uint8_t *atom = tile + (c >> 1) * BOX + row * 128;
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) {
    const int q = (c & 1) * 4 + q4;
    *reinterpret_cast<uint4 *>(atom + ((q ^ (row & 7)) << 4)) =
        make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
  }
}

}  // namespace bwpp_attn
