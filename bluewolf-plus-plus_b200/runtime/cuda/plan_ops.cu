// Storage-generic kernels for the launch-plan executor (plan.cu): the graph
// ops of compiler/include/graph_ir.h:39-57 that are not a contraction, on
// values stored as f16, bf16 or f32 (the graph's declared dtype), computing
// in fp32.  Each is a plain HBM-streaming kernel; the contractions and the
// fused attention go to the tcgen05 kernels instead.
//   binary   add / sub / mul / div, b broadcast as the graph allows:
//            same shape, a row vector [C] (or [1, C]), a column [R, 1], or a
//            scalar
//   unary    silu, copy (reshape into another buffer), dtype conversion
//   row ops  softmax_grad, rmsnorm_grad (compiler/graph_ir.c:1735-1789 rule
//            for dX), rmsnorm / softmax for f32 or bf16 storage
//   reduce   reduce_sum over axis 0 or 1; broadcast back
//   layout   batched 2-D transpose; permute of up to 4 dims
//   max      reduce_max over one axis (values), and its mask (1 at every
//            element equal to the max along the axis: all ties, as
//            runtime/cpu/bwpp_cpu_ref.c:146-190 marks them)
//   fused    swiglu: silu(a) * b in one pass (the `swiglu` pattern of
//            spec/llm-primitives.md:17-22 when a is not a GEMM output);
//            residual + norm: h = a + b and y = rmsnorm(h) per row in one
//            kernel (h stored only when something else reads it)
#include <math.h>

#include "bwpp_cuda_internal.cuh"

namespace {

constexpr int kThreads = 256;

// dtype codes: 0 f16, 1 bf16, 2 f32 (the executor's BwppPlanDType)
template <int DT>
struct St;
template <>
struct St<0> {
  using T = uint16_t;
  __device__ static float ld(const T *p, size_t i) { return load16<true>(p[i]); }
  __device__ static void st(T *p, size_t i, float v) {
    p[i] = (uint16_t)(pack2_16<true>(v, 0.0f) & 0xFFFFu);
  }
};
template <>
struct St<1> {
  using T = uint16_t;
  __device__ static float ld(const T *p, size_t i) { return load16<false>(p[i]); }
  __device__ static void st(T *p, size_t i, float v) {
    p[i] = (uint16_t)(pack2_16<false>(v, 0.0f) & 0xFFFFu);
  }
};
template <>
struct St<2> {
  using T = float;
  __device__ static float ld(const T *p, size_t i) { return p[i]; }
  __device__ static void st(T *p, size_t i, float v) { p[i] = v; }
};

__device__ __forceinline__ float silu1(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// op: 0 add, 1 sub, 2 mul, 3 div, 4 broadcast (o = b; a unread), 5 b - a,
// 6 b / a; bmode: 0 same, 1 row vector [C], 2 column [R], 3 scalar.  a and o
// are [R, C] dense.
template <int DT>
__global__ void binary_kernel(const void *a_, const void *b_, void *o_, uint32_t R, uint32_t C,
                              int op, int bmode) {
  using S = St<DT>;
  const auto *a = static_cast<const typename S::T *>(a_);
  const auto *b = static_cast<const typename S::T *>(b_);
  auto *o = static_cast<typename S::T *>(o_);
  const size_t n = (size_t)R * C;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t bi = bmode == 0 ? i : bmode == 1 ? i % C : bmode == 2 ? i / C : 0;
    const float y = S::ld(b, bi);
    const float x = op == 4 ? 0.0f : S::ld(a, i);
    const float r = op == 0 ? x + y : op == 1 ? x - y : op == 2 ? x * y : op == 3 ? x / y
                  : op == 4 ? y : op == 5 ? y - x : y / x;
    S::st(o, i, r);
  }
}

// op: 0 copy, 1 silu
template <int DT>
__global__ void unary_kernel(const void *x_, void *o_, size_t n, int op) {
  using S = St<DT>;
  const auto *x = static_cast<const typename S::T *>(x_);
  auto *o = static_cast<typename S::T *>(o_);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const float v = S::ld(x, i);
    S::st(o, i, op == 1 ? silu1(v) : v);
  }
}

template <int DI, int DO>
__global__ void convert_kernel(const void *x_, void *o_, size_t n) {
  const auto *x = static_cast<const typename St<DI>::T *>(x_);
  auto *o = static_cast<typename St<DO>::T *>(o_);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    St<DO>::st(o, i, St<DI>::ld(x, i));
}

template <int DT>
__global__ void silu_grad_kernel(const void *x_, const void *dy_, void *dx_, size_t n) {
  using S = St<DT>;
  const auto *x = static_cast<const typename S::T *>(x_);
  const auto *dy = static_cast<const typename S::T *>(dy_);
  auto *dx = static_cast<typename S::T *>(dx_);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const float v = S::ld(x, i), g = S::ld(dy, i);
    const float s = __fdividef(1.0f, 1.0f + __expf(-v));
    S::st(dx, i, g * s * (1.0f + v * (1.0f - s)));
  }
}

__device__ __forceinline__ float block_sum(float v, float *sv) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sv[warp] = v;
  __syncthreads();
  v = lane < (int)(blockDim.x >> 5) ? sv[lane] : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float block_max(float v, float *sv) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sv[warp] = v;
  __syncthreads();
  v = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// one CTA per row (grid-stride): dx = y * (dy - sum(dy * y))
template <int DT>
__global__ void __launch_bounds__(kThreads)
    softmax_grad_kernel(const void *y_, const void *dy_, void *dx_, uint32_t R, uint32_t C) {
  using S = St<DT>;
  const auto *y = static_cast<const typename S::T *>(y_);
  const auto *dy = static_cast<const typename S::T *>(dy_);
  auto *dx = static_cast<typename S::T *>(dx_);
  __shared__ float sv[32];
  for (uint32_t r = blockIdx.x; r < R; r += gridDim.x) {
    const size_t o = (size_t)r * C;
    float s = 0.0f;
    for (uint32_t c = threadIdx.x; c < C; c += kThreads) s += S::ld(y, o + c) * S::ld(dy, o + c);
    s = block_sum(s, sv);
    for (uint32_t c = threadIdx.x; c < C; c += kThreads)
      S::st(dx, o + c, S::ld(y, o + c) * (S::ld(dy, o + c) - s));
  }
}

// RMSNorm dX (compiler/graph_ir.c:1735-1789): r = rsqrt(mean(x^2) + eps),
// g = gamma * dy, dx = r * g - x * r^3 * mean(g * x).  gamma NULL = 1.
template <int DT>
__global__ void __launch_bounds__(kThreads)
    rmsnorm_grad_kernel(const void *x_, const void *gamma_, const void *dy_, void *dx_,
                        uint32_t R, uint32_t C, float eps) {
  using S = St<DT>;
  const auto *x = static_cast<const typename S::T *>(x_);
  const auto *gm = static_cast<const typename S::T *>(gamma_);
  const auto *dy = static_cast<const typename S::T *>(dy_);
  auto *dx = static_cast<typename S::T *>(dx_);
  __shared__ float sv[32];
  for (uint32_t r = blockIdx.x; r < R; r += gridDim.x) {
    const size_t o = (size_t)r * C;
    float ss = 0.0f, gx = 0.0f;
    for (uint32_t c = threadIdx.x; c < C; c += kThreads) {
      const float xv = S::ld(x, o + c);
      const float g = (gm ? S::ld(gm, c) : 1.0f) * S::ld(dy, o + c);
      ss = fmaf(xv, xv, ss);
      gx = fmaf(g, xv, gx);
    }
    ss = block_sum(ss, sv);
    gx = block_sum(gx, sv);
    const float rs = rsqrtf(ss / (float)C + eps);
    const float k = rs * rs * rs * gx / (float)C;
    for (uint32_t c = threadIdx.x; c < C; c += kThreads) {
      const float xv = S::ld(x, o + c);
      const float g = (gm ? S::ld(gm, c) : 1.0f) * S::ld(dy, o + c);
      S::st(dx, o + c, rs * g - xv * k);
    }
  }
}

// Row softmax / RMSNorm for f32 and bf16 storage (f16 uses half_ops.cu).
template <int DT>
__global__ void __launch_bounds__(kThreads)
    softmax_rows_kernel(const void *x_, void *y_, uint32_t R, uint32_t C) {
  using S = St<DT>;
  const auto *x = static_cast<const typename S::T *>(x_);
  auto *y = static_cast<typename S::T *>(y_);
  __shared__ float sv[32];
  for (uint32_t r = blockIdx.x; r < R; r += gridDim.x) {
    const size_t o = (size_t)r * C;
    float m = -INFINITY;
    for (uint32_t c = threadIdx.x; c < C; c += kThreads) {
      const float t = S::ld(x, o + c);
      if (t > m) m = t;
    }
    m = block_max(m, sv);
    float s = 0.0f;
    for (uint32_t c = threadIdx.x; c < C; c += kThreads) s += expf(S::ld(x, o + c) - m);
    s = block_sum(s, sv);
    const float inv = s > 0.0f ? 1.0f / s : 0.0f;
    for (uint32_t c = threadIdx.x; c < C; c += kThreads)
      S::st(y, o + c, expf(S::ld(x, o + c) - m) * inv);
  }
}

template <int DT>
__global__ void __launch_bounds__(kThreads)
    rmsnorm_rows_kernel(const void *x_, const void *gamma_, const void *beta_, void *y_,
                        uint32_t R, uint32_t C, float eps) {
  using S = St<DT>;
  const auto *x = static_cast<const typename S::T *>(x_);
  const auto *gm = static_cast<const typename S::T *>(gamma_);
  const auto *bt = static_cast<const typename S::T *>(beta_);
  auto *y = static_cast<typename S::T *>(y_);
  __shared__ float sv[32];
  for (uint32_t r = blockIdx.x; r < R; r += gridDim.x) {
    const size_t o = (size_t)r * C;
    float ss = 0.0f;
    for (uint32_t c = threadIdx.x; c < C; c += kThreads) {
      const float t = S::ld(x, o + c);
      ss = fmaf(t, t, ss);
    }
    ss = block_sum(ss, sv);
    const float inv = rsqrtf(ss / (float)C + eps);
    for (uint32_t c = threadIdx.x; c < C; c += kThreads) {
      const float g = gm ? S::ld(gm, c) : 1.0f, b = bt ? S::ld(bt, c) : 0.0f;
      S::st(y, o + c, S::ld(x, o + c) * inv * g + b);
    }
  }
}

// o[i0, i1, i2, i3] = x[...] with output dim d taken from input dim perm[d]
// (rank <= 4, dense row-major; unused dims are 1).  Thread per output element.
struct PermDims {
  uint32_t out[4];      // output dims
  uint64_t in_stride[4];  // input stride of the input dim each output dim reads
};

template <int DT>
__global__ void permute_kernel(const void *x_, void *o_, size_t n, const PermDims pd) {
  using S = St<DT>;
  const auto *x = static_cast<const typename S::T *>(x_);
  auto *o = static_cast<typename S::T *>(o_);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    size_t r = i, src = 0;
#pragma unroll
    for (int d = 3; d >= 0; --d) {
      const uint32_t c = (uint32_t)(r % pd.out[d]);
      r /= pd.out[d];
      src += (size_t)c * pd.in_stride[d];
    }
    o[i] = x[src];
  }
}

// reduce_max over the middle dim of x viewed as [outer, n, inner]: mode 0
// writes the maxima [outer, inner]; mode 1 the mask [outer, n, inner] (1 where
// x equals its maximum, all ties).  Strict '>' scan from -INF.
// inner == 1 (the last axis): one CTA per row, block reduction.
template <int DT>
__global__ void __launch_bounds__(kThreads)
    max_rows_kernel(const void *x_, void *o_, uint32_t outer, uint32_t n, int mode) {
  using S = St<DT>;
  const auto *x = static_cast<const typename S::T *>(x_);
  auto *o = static_cast<typename S::T *>(o_);
  __shared__ float sv[32];
  for (uint32_t r = blockIdx.x; r < outer; r += gridDim.x) {
    const size_t base = (size_t)r * n;
    float m = -INFINITY;
    for (uint32_t c = threadIdx.x; c < n; c += kThreads) {
      const float t = S::ld(x, base + c);
      if (t > m) m = t;
    }
    m = block_max(m, sv);
    if (mode == 0) {
      if (threadIdx.x == 0) S::st(o, r, m);
    } else {
      for (uint32_t c = threadIdx.x; c < n; c += kThreads)
        S::st(o, base + c, S::ld(x, base + c) == m ? 1.0f : 0.0f);
    }
  }
}

// inner > 1: thread per (outer, inner) column, coalesced over inner
template <int DT>
__global__ void max_cols_kernel(const void *x_, void *o_, uint32_t outer, uint32_t n,
                                uint32_t inner, int mode) {
  using S = St<DT>;
  const auto *x = static_cast<const typename S::T *>(x_);
  auto *o = static_cast<typename S::T *>(o_);
  const size_t cols = (size_t)outer * inner;
  for (size_t k = blockIdx.x * (size_t)blockDim.x + threadIdx.x; k < cols;
       k += (size_t)gridDim.x * blockDim.x) {
    const size_t ob = k / inner, ib = k % inner;
    const size_t base = ob * (size_t)n * inner + ib;
    float m = -INFINITY;
    for (uint32_t c = 0; c < n; ++c) {
      const float t = S::ld(x, base + (size_t)c * inner);
      if (t > m) m = t;
    }
    if (mode == 0) {
      S::st(o, k, m);
    } else {
      for (uint32_t c = 0; c < n; ++c)
        S::st(o, base + (size_t)c * inner, S::ld(x, base + (size_t)c * inner) == m ? 1.0f : 0.0f);
    }
  }
}

// o = silu(a) * b, elementwise; a, b, o dense, same shape
template <int DT>
__global__ void swiglu_kernel(const void *a_, const void *b_, void *o_, size_t n) {
  using S = St<DT>;
  const auto *a = static_cast<const typename S::T *>(a_);
  const auto *b = static_cast<const typename S::T *>(b_);
  auto *o = static_cast<typename S::T *>(o_);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    S::st(o, i, silu1(S::ld(a, i)) * S::ld(b, i));
}

// Residual + RMSNorm, one CTA per row (grid-stride): h = a + b rounded to the
// storage type (as the unfused add would store it), y = rmsnorm(h) * gamma +
// beta; h is written when h_out != NULL.  The row's sum of squares is taken
// over the rounded h, as the unfused add -> rmsnorm would read it.
template <int DT>
__global__ void __launch_bounds__(kThreads)
    add_rmsnorm_kernel(const void *a_, const void *b_, const void *gamma_, const void *beta_,
                       void *h_, void *y_, uint32_t R, uint32_t C, float eps) {
  using S = St<DT>;
  const auto *a = static_cast<const typename S::T *>(a_);
  const auto *b = static_cast<const typename S::T *>(b_);
  const auto *gm = static_cast<const typename S::T *>(gamma_);
  const auto *bt = static_cast<const typename S::T *>(beta_);
  auto *h = static_cast<typename S::T *>(h_);
  auto *y = static_cast<typename S::T *>(y_);
  __shared__ float sv[32];
  // the rounded sum, as the storage type holds it
  auto hsum = [&](size_t i) {
    typename S::T t[1];
    S::st(t, 0, S::ld(a, i) + S::ld(b, i));
    return S::ld(t, 0);
  };
  for (uint32_t r = blockIdx.x; r < R; r += gridDim.x) {
    const size_t o = (size_t)r * C;
    float ss = 0.0f;
    for (uint32_t c = threadIdx.x; c < C; c += kThreads) {
      const float t = hsum(o + c);
      ss = fmaf(t, t, ss);
      if (h) S::st(h, o + c, t);
    }
    ss = block_sum(ss, sv);
    const float inv = rsqrtf(ss / (float)C + eps);
    // each thread re-reads only the elements it wrote (h may alias a or b)
    for (uint32_t c = threadIdx.x; c < C; c += kThreads) {
      const float g = gm ? S::ld(gm, c) : 1.0f, bb = bt ? S::ld(bt, c) : 0.0f;
      const float t = h ? S::ld(h, o + c) : hsum(o + c);
      S::st(y, o + c, t * inv * g + bb);
    }
  }
}

// axis 1: out[r] = sum_c x[r, c] (CTA per row); axis 0: out[c] = sum_r x[r, c]
// (thread per column, rows in order: deterministic)
template <int DT>
__global__ void __launch_bounds__(kThreads)
    reduce_rows_kernel(const void *x_, void *o_, uint32_t R, uint32_t C) {
  using S = St<DT>;
  const auto *x = static_cast<const typename S::T *>(x_);
  auto *out = static_cast<typename S::T *>(o_);
  __shared__ float sv[32];
  for (uint32_t r = blockIdx.x; r < R; r += gridDim.x) {
    float s = 0.0f;
    for (uint32_t c = threadIdx.x; c < C; c += kThreads) s += S::ld(x, (size_t)r * C + c);
    s = block_sum(s, sv);
    if (threadIdx.x == 0) S::st(out, r, s);
  }
}

template <int DT>
__global__ void reduce_cols_kernel(const void *x_, void *o_, uint32_t R, uint32_t C) {
  using S = St<DT>;
  const auto *x = static_cast<const typename S::T *>(x_);
  auto *out = static_cast<typename S::T *>(o_);
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float s = 0.0f;
  for (uint32_t r = 0; r < R; ++r) s += S::ld(x, (size_t)r * C + c);
  S::st(out, c, s);
}

// out[b, c, r] = x[b, r, c] through a 32 x 33 smem tile
template <int DT>
__global__ void transpose_kernel(const void *x_, void *o_, uint32_t R, uint32_t C) {
  using S = St<DT>;
  const auto *x = static_cast<const typename S::T *>(x_) + (size_t)blockIdx.z * R * C;
  auto *o = static_cast<typename S::T *>(o_) + (size_t)blockIdx.z * R * C;
  __shared__ float tile[32][33];
  const uint32_t c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (uint32_t i = threadIdx.y; i < 32; i += blockDim.y) {
    const uint32_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = S::ld(x, (size_t)r * C + c);
  }
  __syncthreads();
  for (uint32_t i = threadIdx.y; i < 32; i += blockDim.y) {
    const uint32_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) S::st(o, (size_t)c * R + r, tile[threadIdx.x][i]);
  }
}

uint32_t grid_flat(BwppCudaCtx *ctx, size_t n) {
  const size_t blocks = (n + 255) / 256;
  const size_t cap = (size_t)ctx->num_sms * 16;
  return (uint32_t)(blocks < cap ? (blocks ? blocks : 1) : cap);
}

uint32_t grid_rows(BwppCudaCtx *ctx, uint32_t rows) {
  const uint32_t g = (uint32_t)ctx->num_sms * 8;
  return rows < g ? (rows ? rows : 1) : g;
}

}  // namespace

#define BWPP_PLAN_DT(dt, KERNEL, ...)                                          \
  do {                                                                         \
    if ((dt) == 0) KERNEL<0>__VA_ARGS__;                                       \
    else if ((dt) == 1) KERNEL<1>__VA_ARGS__;                                  \
    else KERNEL<2>__VA_ARGS__;                                                 \
  } while (0)

// Host launchers (plan.cu).  Every pointer is a device pointer; all dense.
int bwpp_plan_binary(BwppCudaCtx *ctx, int dt, const void *a, const void *b, void *o, uint32_t R,
                     uint32_t C, int op, int bmode) {
  const size_t n = (size_t)R * C;
  if (n == 0) return BWPP_CUDA_OK;
  const uint32_t g = grid_flat(ctx, n);
  BWPP_PLAN_DT(dt, binary_kernel, <<<g, 256, 0, ctx->stream>>>(a, b, o, R, C, op, bmode));
  BWPP_LAUNCH_CHECK(ctx, "plan binary");
  return BWPP_CUDA_OK;
}

int bwpp_plan_unary(BwppCudaCtx *ctx, int dt, const void *x, void *o, size_t n, int op) {
  if (n == 0) return BWPP_CUDA_OK;
  const uint32_t g = grid_flat(ctx, n);
  BWPP_PLAN_DT(dt, unary_kernel, <<<g, 256, 0, ctx->stream>>>(x, o, n, op));
  BWPP_LAUNCH_CHECK(ctx, "plan unary");
  return BWPP_CUDA_OK;
}

int bwpp_plan_convert(BwppCudaCtx *ctx, int di, int dout, const void *x, void *o, size_t n) {
  if (n == 0) return BWPP_CUDA_OK;
  const uint32_t g = grid_flat(ctx, n);
  cudaStream_t s = ctx->stream;
  if (di == 0 && dout == 2) convert_kernel<0, 2><<<g, 256, 0, s>>>(x, o, n);
  else if (di == 1 && dout == 2) convert_kernel<1, 2><<<g, 256, 0, s>>>(x, o, n);
  else if (di == 2 && dout == 0) convert_kernel<2, 0><<<g, 256, 0, s>>>(x, o, n);
  else if (di == 2 && dout == 1) convert_kernel<2, 1><<<g, 256, 0, s>>>(x, o, n);
  else if (di == 0 && dout == 1) convert_kernel<0, 1><<<g, 256, 0, s>>>(x, o, n);
  else if (di == 1 && dout == 0) convert_kernel<1, 0><<<g, 256, 0, s>>>(x, o, n);
  else return bwpp_check_cuda(ctx, cudaMemcpyAsync(o, x, n * (di == 2 ? 4 : 2),
                                                   cudaMemcpyDeviceToDevice, s), "plan copy");
  BWPP_LAUNCH_CHECK(ctx, "plan convert");
  return BWPP_CUDA_OK;
}

int bwpp_plan_silu_grad(BwppCudaCtx *ctx, int dt, const void *x, const void *dy, void *dx,
                        size_t n) {
  if (n == 0) return BWPP_CUDA_OK;
  const uint32_t g = grid_flat(ctx, n);
  BWPP_PLAN_DT(dt, silu_grad_kernel, <<<g, 256, 0, ctx->stream>>>(x, dy, dx, n));
  BWPP_LAUNCH_CHECK(ctx, "plan silu_grad");
  return BWPP_CUDA_OK;
}

int bwpp_plan_softmax_grad(BwppCudaCtx *ctx, int dt, const void *y, const void *dy, void *dx,
                           uint32_t R, uint32_t C) {
  if (!R || !C) return BWPP_CUDA_OK;
  BWPP_PLAN_DT(dt, softmax_grad_kernel, <<<grid_rows(ctx, R), kThreads, 0, ctx->stream>>>(y, dy, dx, R, C));
  BWPP_LAUNCH_CHECK(ctx, "plan softmax_grad");
  return BWPP_CUDA_OK;
}

int bwpp_plan_rmsnorm_grad(BwppCudaCtx *ctx, int dt, const void *x, const void *gamma,
                           const void *dy, void *dx, uint32_t R, uint32_t C, float eps) {
  if (!R || !C) return BWPP_CUDA_OK;
  BWPP_PLAN_DT(dt, rmsnorm_grad_kernel,
               <<<grid_rows(ctx, R), kThreads, 0, ctx->stream>>>(x, gamma, dy, dx, R, C, eps));
  BWPP_LAUNCH_CHECK(ctx, "plan rmsnorm_grad");
  return BWPP_CUDA_OK;
}

int bwpp_plan_softmax(BwppCudaCtx *ctx, int dt, const void *x, void *y, uint32_t R, uint32_t C) {
  if (!R || !C) return BWPP_CUDA_OK;
  BWPP_PLAN_DT(dt, softmax_rows_kernel, <<<grid_rows(ctx, R), kThreads, 0, ctx->stream>>>(x, y, R, C));
  BWPP_LAUNCH_CHECK(ctx, "plan softmax");
  return BWPP_CUDA_OK;
}

int bwpp_plan_rmsnorm(BwppCudaCtx *ctx, int dt, const void *x, const void *gamma,
                      const void *beta, void *y, uint32_t R, uint32_t C, float eps) {
  if (!R || !C) return BWPP_CUDA_OK;
  BWPP_PLAN_DT(dt, rmsnorm_rows_kernel,
               <<<grid_rows(ctx, R), kThreads, 0, ctx->stream>>>(x, gamma, beta, y, R, C, eps));
  BWPP_LAUNCH_CHECK(ctx, "plan rmsnorm");
  return BWPP_CUDA_OK;
}

int bwpp_plan_reduce_sum(BwppCudaCtx *ctx, int dt, const void *x, void *o, uint32_t R, uint32_t C,
                         int axis) {
  if (axis == 1) {
    if (!R) return BWPP_CUDA_OK;
    BWPP_PLAN_DT(dt, reduce_rows_kernel, <<<grid_rows(ctx, R), kThreads, 0, ctx->stream>>>(x, o, R, C));
  } else {
    if (!C) return BWPP_CUDA_OK;
    BWPP_PLAN_DT(dt, reduce_cols_kernel, <<<(C + 255) / 256, 256, 0, ctx->stream>>>(x, o, R, C));
  }
  BWPP_LAUNCH_CHECK(ctx, "plan reduce_sum");
  return BWPP_CUDA_OK;
}

int bwpp_plan_transpose(BwppCudaCtx *ctx, int dt, const void *x, void *o, uint32_t batch,
                        uint32_t R, uint32_t C) {
  if (!batch || !R || !C) return BWPP_CUDA_OK;
  if (batch > 65535) return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "plan transpose: batch");
  dim3 grid((C + 31) / 32, (R + 31) / 32, batch);
  BWPP_PLAN_DT(dt, transpose_kernel, <<<grid, dim3(32, 8), 0, ctx->stream>>>(x, o, R, C));
  BWPP_LAUNCH_CHECK(ctx, "plan transpose");
  return BWPP_CUDA_OK;
}

int bwpp_plan_swiglu(BwppCudaCtx *ctx, int dt, const void *a, const void *b, void *o, size_t n) {
  if (n == 0) return BWPP_CUDA_OK;
  const uint32_t g = grid_flat(ctx, n);
  BWPP_PLAN_DT(dt, swiglu_kernel, <<<g, 256, 0, ctx->stream>>>(a, b, o, n));
  BWPP_LAUNCH_CHECK(ctx, "plan swiglu");
  return BWPP_CUDA_OK;
}

int bwpp_plan_add_rmsnorm(BwppCudaCtx *ctx, int dt, const void *a, const void *b,
                          const void *gamma, const void *beta, void *h, void *y, uint32_t R,
                          uint32_t C, float eps) {
  if (!R || !C) return BWPP_CUDA_OK;
  BWPP_PLAN_DT(dt, add_rmsnorm_kernel,
               <<<grid_rows(ctx, R), kThreads, 0, ctx->stream>>>(a, b, gamma, beta, h, y, R, C,
                                                                 eps));
  BWPP_LAUNCH_CHECK(ctx, "plan add_rmsnorm");
  return BWPP_CUDA_OK;
}

// perm[d]: the input dim output dim d reads; dims: the input's dims (rank <= 4)
int bwpp_plan_permute(BwppCudaCtx *ctx, int dt, const void *x, void *o, int rank,
                      const int64_t *dims, const int *perm) {
  if (rank < 1 || rank > 4) return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "plan permute: rank");
  uint64_t stride[4];
  uint64_t st = 1;
  for (int d = rank - 1; d >= 0; --d) {
    stride[d] = st;
    st *= (uint64_t)dims[d];
  }
  PermDims pd;
  const int pad = 4 - rank;  // leading unit dims
  size_t n = 1;
  for (int d = 0; d < 4; ++d) {
    if (d < pad) {
      pd.out[d] = 1;
      pd.in_stride[d] = 0;
    } else {
      const int p = perm[d - pad];
      pd.out[d] = (uint32_t)dims[p];
      pd.in_stride[d] = stride[p];
      n *= (size_t)dims[p];
    }
  }
  if (n == 0) return BWPP_CUDA_OK;
  BWPP_PLAN_DT(dt, permute_kernel, <<<grid_flat(ctx, n), 256, 0, ctx->stream>>>(x, o, n, pd));
  BWPP_LAUNCH_CHECK(ctx, "plan permute");
  return BWPP_CUDA_OK;
}

// x viewed as [outer, n, inner]; mode 0: maxima, 1: the tie mask
int bwpp_plan_reduce_max(BwppCudaCtx *ctx, int dt, const void *x, void *o, uint32_t outer,
                         uint32_t n, uint32_t inner, int mode) {
  if (!outer || !n || !inner) return BWPP_CUDA_OK;
  if (inner == 1) {
    BWPP_PLAN_DT(dt, max_rows_kernel,
                 <<<grid_rows(ctx, outer), kThreads, 0, ctx->stream>>>(x, o, outer, n, mode));
  } else {
    BWPP_PLAN_DT(dt, max_cols_kernel,
                 <<<grid_flat(ctx, (size_t)outer * inner), 256, 0, ctx->stream>>>(x, o, outer, n,
                                                                                  inner, mode));
  }
  BWPP_LAUNCH_CHECK(ctx, "plan reduce_max");
  return BWPP_CUDA_OK;
}
