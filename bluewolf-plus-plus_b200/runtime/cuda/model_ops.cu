// Elementwise and row kernels of the tiny_model training step (BASELINE
// configs[4]): a pre-RMSNorm decoder block with causal attention and a
// SiLU-gated MLP.  All HBM-bound; 128-bit loads where the layout allows.
//
// bf16 values travel as uint16_t bit patterns; conversions round to nearest
// even (cvt.rn.bf16x2.f32).
#include <math.h>

#include "bwpp_cuda_internal.cuh"

namespace {


__device__ __forceinline__ uint32_t f2bf2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float sigmoidf_(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

template <int NV>
__device__ __forceinline__ void block_sum_n(float (&v)[NV], float *red) {
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0)
#pragma unroll
    for (int j = 0; j < NV; ++j) red[j * 32 + warp] = v[j];
  __syncthreads();
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float t = lane < (int)(blockDim.x >> 5) ? red[j * 32 + lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    v[j] = t;
  }
}

// y(bf16) = x * rsqrt(mean(x^2) + eps) * gamma, one CTA (256 threads) per row,
// cols a multiple of 4 and at most 256 * 4 * 8.
__global__ void __launch_bounds__(256)
    rmsnorm_bf16out_kernel(const float *__restrict__ x, const float *__restrict__ gamma,
                           uint16_t *__restrict__ y, uint32_t rows, uint32_t cols, float eps) {
  __shared__ float red[32];
  const uint32_t nv = cols / 4;
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)r * cols);
    float4 v[8];
    float ss[1] = {0.0f};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t idx = threadIdx.x + i * 256;
      v[i] = idx < nv ? xr[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
      ss[0] += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    block_sum_n<1>(ss, red);
    const float inv = 1.0f / sqrtf(ss[0] / (float)cols + eps);
    uint2 *yr = reinterpret_cast<uint2 *>(y + (size_t)r * cols);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t idx = threadIdx.x + i * 256;
      if (idx >= nv) continue;
      const float4 g = reinterpret_cast<const float4 *>(gamma)[idx];
      yr[idx] = make_uint2(f2bf2(v[i].x * inv * g.x, v[i].y * inv * g.y),
                           f2bf2(v[i].z * inv * g.z, v[i].w * inv * g.w));
    }
  }
}

// The same with one warp per row (cols % 128 == 0, cols <= 2048): the row
// stays in the warp's registers (up to 16 float4 per lane) and the sum of
// squares needs only shuffles, so many rows are in flight per SM and no
// block barrier stalls a CTA between load and store.
template <int NV4>  // float4 per lane
__global__ void __launch_bounds__(256)
    rmsnorm_bf16out_warp_kernel(const float *__restrict__ x, const float *__restrict__ gamma,
                                uint16_t *__restrict__ y, uint32_t rows, uint32_t cols, float eps) {
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;
  for (uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += nwarps) {
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)r * cols);
    float4 v[NV4];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
      v[i] = __ldcs(xr + lane + 32 * i);
      ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss / (float)cols + eps);
    uint2 *yr = reinterpret_cast<uint2 *>(y + (size_t)r * cols);
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
      const float4 g = __ldg(reinterpret_cast<const float4 *>(gamma) + lane + 32 * i);
      yr[lane + 32 * i] = make_uint2(f2bf2(v[i].x * inv * g.x, v[i].y * inv * g.y),
                                     f2bf2(v[i].z * inv * g.z, v[i].w * inv * g.w));
    }
  }
}

// a[t, f] = silu(gu[t, f]) * gu[t, F + f]   (gate | up halves)
__global__ void swiglu_fwd_kernel(const uint16_t *__restrict__ gu, uint16_t *__restrict__ a,
                                  uint32_t rows, uint32_t F) {
  const size_t n = (size_t)rows * F / 2;  // pairs
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t e = 2 * i, t = e / F, f = e % F;
    const uint32_t g2 = *reinterpret_cast<const uint32_t *>(gu + t * 2 * F + f);
    const uint32_t u2 = *reinterpret_cast<const uint32_t *>(gu + t * 2 * F + F + f);
    const float g0 = __uint_as_float(g2 << 16), g1 = __uint_as_float(g2 & 0xFFFF0000u);
    const float u0 = __uint_as_float(u2 << 16), u1 = __uint_as_float(u2 & 0xFFFF0000u);
    *reinterpret_cast<uint32_t *>(a + e) =
        f2bf2(g0 * sigmoidf_(g0) * u0, g1 * sigmoidf_(g1) * u1);
  }
}

// The same, 8 columns per thread (128-bit loads and stores, 32-bit index
// arithmetic): F % 8 == 0, rows * F / 8 < 2^32, 16-byte aligned rows.
__global__ void swiglu_fwd_v8_kernel(const uint16_t *__restrict__ gu, uint16_t *__restrict__ a,
                                     uint32_t rows, uint32_t F) {
  const uint32_t fv = F / 8, n = rows * fv;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint32_t t = i / fv, f = (i - t * fv) * 8;
    const uint4 g4 = __ldcs(reinterpret_cast<const uint4 *>(gu + (size_t)t * 2 * F + f));
    const uint4 u4 = __ldcs(reinterpret_cast<const uint4 *>(gu + (size_t)t * 2 * F + F + f));
    const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w}, uw[4] = {u4.x, u4.y, u4.z, u4.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g0 = __uint_as_float(gw[k] << 16), g1 = __uint_as_float(gw[k] & 0xFFFF0000u);
      const float u0 = __uint_as_float(uw[k] << 16), u1 = __uint_as_float(uw[k] & 0xFFFF0000u);
      o[k] = f2bf2(g0 * sigmoidf_(g0) * u0, g1 * sigmoidf_(g1) * u1);
    }
    __stcs(reinterpret_cast<uint4 *>(a + (size_t)t * F + f), make_uint4(o[0], o[1], o[2], o[3]));
  }
}

// dgu[t, f] = da * up * silu'(gate), dgu[t, F + f] = da * silu(gate)
// silu'(g) = s (1 + g (1 - s)), s = sigmoid(g); da is fp32 [rows, F].
__global__ void swiglu_bwd_kernel(const uint16_t *__restrict__ gu, const float *__restrict__ da,
                                  uint16_t *__restrict__ dgu, uint32_t rows, uint32_t F) {
  const size_t n = (size_t)rows * F / 2;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t e = 2 * i, t = e / F, f = e % F;
    const uint32_t g2 = *reinterpret_cast<const uint32_t *>(gu + t * 2 * F + f);
    const uint32_t u2 = *reinterpret_cast<const uint32_t *>(gu + t * 2 * F + F + f);
    const float2 d = *reinterpret_cast<const float2 *>(da + e);
    const float g[2] = {__uint_as_float(g2 << 16), __uint_as_float(g2 & 0xFFFF0000u)};
    const float u[2] = {__uint_as_float(u2 << 16), __uint_as_float(u2 & 0xFFFF0000u)};
    const float dd[2] = {d.x, d.y};
    float dg[2], du[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float s = sigmoidf_(g[k]);
      dg[k] = dd[k] * u[k] * s * (1.0f + g[k] * (1.0f - s));
      du[k] = dd[k] * g[k] * s;
    }
    *reinterpret_cast<uint32_t *>(dgu + t * 2 * F + f) = f2bf2(dg[0], dg[1]);
    *reinterpret_cast<uint32_t *>(dgu + t * 2 * F + F + f) = f2bf2(du[0], du[1]);
  }
}

// diff = h - target; dh = 2 diff / n (fp32 and bf16 copies); per-CTA sum of
// squares into part[blockIdx.x] (summed by loss_sum_kernel in a fixed order).
__global__ void __launch_bounds__(256)
    mse_kernel(const float *__restrict__ h, const float *__restrict__ tgt, float *__restrict__ dh,
               uint16_t *__restrict__ dh16, float *__restrict__ part, size_t n, float scale) {
  __shared__ float red[32];
  float s[1] = {0.0f};
  const size_t n4 = n / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4 *>(h)[i];
    const float4 b = reinterpret_cast<const float4 *>(tgt)[i];
    const float4 d = make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w);
    s[0] += d.x * d.x + d.y * d.y + d.z * d.z + d.w * d.w;
    const float4 g = make_float4(scale * d.x, scale * d.y, scale * d.z, scale * d.w);
    reinterpret_cast<float4 *>(dh)[i] = g;
    reinterpret_cast<uint2 *>(dh16)[i] = make_uint2(f2bf2(g.x, g.y), f2bf2(g.z, g.w));
  }
  block_sum_n<1>(s, red);
  if (threadIdx.x == 0) part[blockIdx.x] = s[0];
}

__global__ void loss_sum_kernel(const float *__restrict__ part, uint32_t nparts, float inv_n,
                                float *__restrict__ loss) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    double s = 0.0;
    for (uint32_t i = 0; i < nparts; ++i) s += part[i];
    *loss = (float)(s * inv_n);
  }
}

// delta[(b*H + h) * S + s] = sum_d dO[t, h*Dh + d] * O[t, h*Dh + d], t = b*S + s
// (token-major bf16 [T, H*Dh]); one warp per (t, h), Dh = 128.
// delta[b, h, s] = sum_d dO[t, h, d] * O[t, h, d] for head dim 128: a half
// warp per (token, head), 16-byte loads, 32-bit indices, grid-stride.
__global__ void attn_delta128_kernel(const uint16_t *__restrict__ dO,
                                     const uint16_t *__restrict__ Ot, float *__restrict__ delta,
                                     uint32_t S, uint32_t H, uint32_t items) {
  const uint32_t lane16 = threadIdx.x & 15;
  for (uint32_t w = (blockIdx.x * blockDim.x + threadIdx.x) >> 4; w < items;
       w += (gridDim.x * blockDim.x) >> 4) {
    const size_t off = (size_t)w * 128 + lane16 * 8;  // token-major, head h at column 128 h
    const uint4 x = __ldcs(reinterpret_cast<const uint4 *>(dO + off));
    const uint4 y = __ldcs(reinterpret_cast<const uint4 *>(Ot + off));
    const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, yw[4] = {y.x, y.y, y.z, y.w};
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      s += __uint_as_float(xw[k] << 16) * __uint_as_float(yw[k] << 16) +
           __uint_as_float(xw[k] & 0xFFFF0000u) * __uint_as_float(yw[k] & 0xFFFF0000u);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane16 == 0) {
      const uint32_t t = w / H, h = w - t * H;
      const uint32_t b_ = t / S, s_ = t - b_ * S;
      delta[((size_t)b_ * H + h) * S + s_] = s;
    }
  }
}

__global__ void attn_delta_kernel(const uint16_t *__restrict__ dO, const uint16_t *__restrict__ Ot,
                                  float *__restrict__ delta, uint32_t B, uint32_t S, uint32_t H,
                                  uint32_t Dh) {
  const uint64_t w = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (uint64_t)B * S * H) return;
  const uint32_t t = (uint32_t)(w / H), h = (uint32_t)(w % H);
  const uint16_t *a = dO + (size_t)t * H * Dh + h * Dh;
  const uint16_t *b = Ot + (size_t)t * H * Dh + h * Dh;
  float s = 0.0f;
  for (uint32_t d = lane * 4; d < Dh; d += 128) {
    const uint2 x = *reinterpret_cast<const uint2 *>(a + d);
    const uint2 y = *reinterpret_cast<const uint2 *>(b + d);
    s += __uint_as_float(x.x << 16) * __uint_as_float(y.x << 16) +
         __uint_as_float(x.x & 0xFFFF0000u) * __uint_as_float(y.x & 0xFFFF0000u) +
         __uint_as_float(x.y << 16) * __uint_as_float(y.y << 16) +
         __uint_as_float(x.y & 0xFFFF0000u) * __uint_as_float(y.y & 0xFFFF0000u);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    const uint32_t b_ = t / S, s_ = t % S;
    delta[((size_t)b_ * H + h) * S + s_] = s;
  }
}

// w -= lr * g (fp32 master), then w16 = bf16(w)
// w -= lr * g, w16 = bf16(w): four values per thread and step (16-byte
// loads and stores, 8 bytes of bf16) where w, g and w16 allow it.
__global__ void sgd_kernel(float *__restrict__ w, const float *__restrict__ g,
                           uint16_t *__restrict__ w16, size_t n, float lr) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t first = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(g)) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(w16) & 7) == 0;
  const size_t n4 = vec ? n / 4 : 0;
  for (size_t i = first; i < n4; i += stride) {
    float4 v = reinterpret_cast<const float4 *>(w)[i];
    const float4 d = reinterpret_cast<const float4 *>(g)[i];
    v.x -= lr * d.x;
    v.y -= lr * d.y;
    v.z -= lr * d.z;
    v.w -= lr * d.w;
    reinterpret_cast<float4 *>(w)[i] = v;
    uint32_t lo, hi;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(v.y), "f"(v.x));
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(v.w), "f"(v.z));
    reinterpret_cast<uint2 *>(w16)[i] = make_uint2(lo, hi);
  }
  for (size_t i = n4 * 4 + first; i < n; i += stride) {
    const float v = w[i] - lr * g[i];
    w[i] = v;
    uint32_t u;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(u) : "f"(0.0f), "f"(v));
    w16[i] = (uint16_t)(u & 0xFFFFu);
  }
}

// a += b (fp32)
__global__ void add_kernel(float *__restrict__ a, const float *__restrict__ b, size_t n) {
  const size_t n4 = n / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x) {
    float4 x = reinterpret_cast<float4 *>(a)[i];
    const float4 y = reinterpret_cast<const float4 *>(b)[i];
    x.x += y.x; x.y += y.y; x.z += y.z; x.w += y.w;
    reinterpret_cast<float4 *>(a)[i] = x;
  }
  for (size_t i = n4 * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    a[i] += b[i];
}

// Counter-based normal samples (SplitMix64 hash of (seed, index), Box-Muller)
__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__global__ void fill_normal_kernel(float *__restrict__ w, size_t n, uint64_t seed, float mean,
                                   float stddev) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint64_t r = splitmix64(seed * 0x100000001B3ull + i);
    const float u1 = ((float)(r >> 40) + 1.0f) * (1.0f / 16777217.0f);  // (0, 1]
    const float u2 = (float)((r >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
    w[i] = mean + stddev * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
  }
}

unsigned grid_for(BwppCudaCtx *ctx, size_t n, int threads) {
  size_t b = (n + threads - 1) / threads;
  const size_t cap = (size_t)ctx->num_sms * 16;
  return (unsigned)(b < cap ? (b ? b : 1) : cap);
}

}  // namespace

int bwpp_rmsnorm_bf16out(BwppCudaCtx *ctx, const float *x, const float *gamma, uint16_t *y,
                         uint32_t rows, uint32_t cols, float eps) {
  if (cols % 4 || cols > 256 * 4 * 8)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "rmsnorm bf16: cols");
  if (cols % 128 == 0 && cols <= 2048 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(gamma) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 7) == 0) {
    const unsigned grid = grid_for(ctx, (size_t)rows * 32, 256);
#define BWPP_RMSW(N) \
  rmsnorm_bf16out_warp_kernel<N><<<grid, 256, 0, ctx->stream>>>(x, gamma, y, rows, cols, eps)
    switch (cols / 128) {
      case 1: BWPP_RMSW(1); break;
      case 2: BWPP_RMSW(2); break;
      case 3: BWPP_RMSW(3); break;
      case 4: BWPP_RMSW(4); break;
      case 5: BWPP_RMSW(5); break;
      case 6: BWPP_RMSW(6); break;
      case 7: BWPP_RMSW(7); break;
      case 8: BWPP_RMSW(8); break;
      case 9: BWPP_RMSW(9); break;
      case 10: BWPP_RMSW(10); break;
      case 11: BWPP_RMSW(11); break;
      case 12: BWPP_RMSW(12); break;
      case 13: BWPP_RMSW(13); break;
      case 14: BWPP_RMSW(14); break;
      case 15: BWPP_RMSW(15); break;
      default: BWPP_RMSW(16); break;
    }
#undef BWPP_RMSW
    BWPP_LAUNCH_CHECK(ctx, "rmsnorm bf16");
    return BWPP_CUDA_OK;
  }
  const unsigned cap = (unsigned)ctx->num_sms * 8;
  const unsigned grid = rows < cap ? (rows ? rows : 1) : cap;
  rmsnorm_bf16out_kernel<<<grid, 256, 0, ctx->stream>>>(x, gamma, y, rows, cols, eps);
  BWPP_LAUNCH_CHECK(ctx, "rmsnorm bf16");
  return BWPP_CUDA_OK;
}

int bwpp_swiglu_fwd(BwppCudaCtx *ctx, const uint16_t *gu, uint16_t *a, uint32_t rows, uint32_t F) {
  if (F % 2) return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "swiglu: odd F");
  if (F % 8 == 0 && (size_t)rows * (F / 8) < (1ull << 31) &&
      (reinterpret_cast<uintptr_t>(gu) & 15) == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0) {
    swiglu_fwd_v8_kernel<<<grid_for(ctx, (size_t)rows * F / 8, 256), 256, 0, ctx->stream>>>(
        gu, a, rows, F);
    BWPP_LAUNCH_CHECK(ctx, "swiglu fwd");
    return BWPP_CUDA_OK;
  }
  swiglu_fwd_kernel<<<grid_for(ctx, (size_t)rows * F / 2, 256), 256, 0, ctx->stream>>>(gu, a, rows, F);
  BWPP_LAUNCH_CHECK(ctx, "swiglu fwd");
  return BWPP_CUDA_OK;
}

int bwpp_swiglu_bwd(BwppCudaCtx *ctx, const uint16_t *gu, const float *da, uint16_t *dgu,
                    uint32_t rows, uint32_t F) {
  if (F % 2) return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "swiglu: odd F");
  swiglu_bwd_kernel<<<grid_for(ctx, (size_t)rows * F / 2, 256), 256, 0, ctx->stream>>>(gu, da, dgu,
                                                                                      rows, F);
  BWPP_LAUNCH_CHECK(ctx, "swiglu bwd");
  return BWPP_CUDA_OK;
}

// loss = mean((h - t)^2) into *loss (device); dh = 2 (h - t) / n.
// part needs num_sms * 4 floats.
int bwpp_mse(BwppCudaCtx *ctx, const float *h, const float *t, float *dh, uint16_t *dh16,
             float *part, float *loss, size_t n) {
  if (n % 4) return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "mse: n % 4");
  const unsigned g = (unsigned)ctx->num_sms * 4;
  mse_kernel<<<g, 256, 0, ctx->stream>>>(h, t, dh, dh16, part, n, 2.0f / (float)n);
  loss_sum_kernel<<<1, 32, 0, ctx->stream>>>(part, g, 1.0 / (double)n, loss);
  BWPP_LAUNCH_CHECK(ctx, "mse");
  return BWPP_CUDA_OK;
}

int bwpp_attn_delta(BwppCudaCtx *ctx, const uint16_t *dO, const uint16_t *O, float *delta,
                    uint32_t B, uint32_t S, uint32_t H, uint32_t Dh) {
  const uint64_t warps = (uint64_t)B * S * H;
  if (Dh == 128 && warps < (1ull << 31) && (reinterpret_cast<uintptr_t>(dO) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(O) & 15) == 0) {
    attn_delta128_kernel<<<grid_for(ctx, warps * 16, 256), 256, 0, ctx->stream>>>(
        dO, O, delta, S, H, (uint32_t)warps);
    BWPP_LAUNCH_CHECK(ctx, "attention delta");
    return BWPP_CUDA_OK;
  }
  attn_delta_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, ctx->stream>>>(dO, O, delta, B,
                                                                                   S, H, Dh);
  BWPP_LAUNCH_CHECK(ctx, "attention delta");
  return BWPP_CUDA_OK;
}

int bwpp_sgd(BwppCudaCtx *ctx, float *w, const float *g, uint16_t *w16, size_t n, float lr) {
  sgd_kernel<<<grid_for(ctx, n / 4 + 1, 256), 256, 0, ctx->stream>>>(w, g, w16, n, lr);
  BWPP_LAUNCH_CHECK(ctx, "sgd");
  return BWPP_CUDA_OK;
}

int bwpp_add(BwppCudaCtx *ctx, float *a, const float *b, size_t n) {
  add_kernel<<<grid_for(ctx, n / 4 + 1, 256), 256, 0, ctx->stream>>>(a, b, n);
  BWPP_LAUNCH_CHECK(ctx, "add");
  return BWPP_CUDA_OK;
}

int bwpp_fill_normal(BwppCudaCtx *ctx, float *w, size_t n, uint64_t seed, float mean,
                     float stddev) {
  fill_normal_kernel<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(w, n, seed, mean, stddev);
  BWPP_LAUNCH_CHECK(ctx, "fill normal");
  return BWPP_CUDA_OK;
}
