// Row-kernel helpers shared by the HBM-bound row operations (norms, the
// autodiff row kernels): 128-bit or scalar element access and a block-wide
// sum of several values at once.
#pragma once

#include "bwpp_cuda_internal.cuh"

namespace bwpp_row {

template <bool V4>
struct Vec;
template <>
struct Vec<true> {
  static constexpr int W = 4;
  __device__ static void load(const float *p, uint32_t i, float (&o)[4]) {
    float4 t = __ldg(reinterpret_cast<const float4 *>(p) + i);
    o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
  }
  __device__ static void load_stream(const float *p, uint32_t i,
                                     float (&o)[4]) {
    float4 t = __ldcs(reinterpret_cast<const float4 *>(p) + i);
    o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
  }
  __device__ static void store(float *p, uint32_t i, const float (&v)[4]) {
    __stcs(reinterpret_cast<float4 *>(p) + i,
           make_float4(v[0], v[1], v[2], v[3]));
  }
};
template <>
struct Vec<false> {
  static constexpr int W = 1;
  __device__ static void load(const float *p, uint32_t i, float (&o)[1]) {
    o[0] = __ldg(p + i);
  }
  __device__ static void load_stream(const float *p, uint32_t i,
                                     float (&o)[1]) {
    o[0] = __ldcs(p + i);
  }
  __device__ static void store(float *p, uint32_t i, const float (&v)[1]) {
    __stcs(p + i, v[0]);
  }
};

// Sums NV values over the block; every thread gets the totals.
template <int NV>
__device__ __forceinline__ void block_sum(float (&v)[NV], float *red) {
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  __syncthreads();  // `red` may still be read from the previous row
  if (lane == 0)
#pragma unroll
    for (int j = 0; j < NV; ++j) red[j * 32 + warp] = v[j];
  __syncthreads();
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float t = lane < nwarps ? red[j * 32 + lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    v[j] = t;
  }
}

}  // namespace bwpp_row
