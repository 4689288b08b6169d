// Kernels for the autodiff-internal ops of the compiler's gradient graph,
// fp32, HBM-bound.  The reference emits these graph ops
// (compiler/include/graph_ir.h:42-55: BROADCAST, REDUCE_SUM, SILU_GRAD,
// SOFTMAX_GRAD) from its backward rules but has no kernel for any of them:
//   silu_grad(x, dy)     compiler/graph_ir.c:1709-1720  dx = dy * silu'(x),
//                        silu'(x) = s (1 + x (1 - s)), s = sigmoid(x)
//   softmax_grad(y, dy)  compiler/graph_ir.c:1722-1733  dx = y (dy - sum(dy y))
//                        over the softmax axis (the last one, as the
//                        softmax kernels runtime/cpu/bwpp_cpu_ref.c:37-61 and
//                        compiler/codegen_metal.c:567-598)
//   reduce_sum(x, axis)  compiler/graph_ir.c:1414-1443 (reduce-to-shape):
//                        axis 1 -> [R, 1] row sums, axis 0 -> [1, C] column sums
//   broadcast(v, axis)   compiler/graph_ir.c:1457-1470, the reduce_sum grad
//                        (1791-1796): [R, 1] (axis 1) or [1, C] (axis 0)
//                        replicated to [R, C]
//
// Elementwise kernels stream with 128-bit accesses; the row kernels hold a
// row in registers (one HBM read of each input); column sums use per-CTA
// partial rows summed in a fixed order afterwards (deterministic).
#include "bwpp_cuda_internal.cuh"
#include "rowwise.cuh"

namespace {

using bwpp_row::Vec;
using bwpp_row::block_sum;

constexpr int kThreads = 256;

inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__device__ __forceinline__ float silu_grad_1(float x, float dy) {
  const float s = __fdividef(1.0f, 1.0f + __expf(-x));
  return dy * s * (1.0f + x * (1.0f - s));
}

template <bool V4>
__global__ void __launch_bounds__(kThreads)
    silu_grad_kernel(const float *__restrict__ x, const float *__restrict__ dy,
                     float *__restrict__ dx, size_t n) {
  if (V4) {
    const size_t n4 = n / 4;
    for (size_t i = blockIdx.x * (size_t)kThreads + threadIdx.x; i < n4;
         i += (size_t)gridDim.x * kThreads) {
      const float4 a = __ldcs(reinterpret_cast<const float4 *>(x) + i);
      const float4 g = __ldcs(reinterpret_cast<const float4 *>(dy) + i);
      __stcs(reinterpret_cast<float4 *>(dx) + i,
             make_float4(silu_grad_1(a.x, g.x), silu_grad_1(a.y, g.y), silu_grad_1(a.z, g.z),
                         silu_grad_1(a.w, g.w)));
    }
  } else {
    for (size_t i = blockIdx.x * (size_t)kThreads + threadIdx.x; i < n;
         i += (size_t)gridDim.x * kThreads)
      dx[i] = silu_grad_1(x[i], dy[i]);
  }
}

// softmax_grad, the row (y and dy) held in registers: MAXV vectors of W
// floats per thread and array.
template <int MAXV, bool V4>
__global__ void __launch_bounds__(kThreads)
    softmax_grad_kernel(const float *__restrict__ y, const float *__restrict__ dy,
                        float *dx, uint32_t rows, uint32_t cols, uint32_t ld) {
  using V = Vec<V4>;
  constexpr int W = V::W;
  __shared__ float red[32];
  const uint32_t nv = cols / W;
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *yr = y + (size_t)r * ld;
    const float *gr = dy + (size_t)r * ld;
    float yv[MAXV][W], gv[MAXV][W];
    float dot[1] = {0.0f};
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const uint32_t idx = threadIdx.x + i * kThreads;
      if (idx < nv) {
        V::load_stream(yr, idx, yv[i]);
        V::load_stream(gr, idx, gv[i]);
      } else {
#pragma unroll
        for (int w = 0; w < W; ++w) yv[i][w] = gv[i][w] = 0.0f;
      }
#pragma unroll
      for (int w = 0; w < W; ++w) dot[0] = fmaf(yv[i][w], gv[i][w], dot[0]);
    }
    block_sum<1>(dot, red);
    float *dr = dx + (size_t)r * ld;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const uint32_t idx = threadIdx.x + i * kThreads;
      if (idx < nv) {
        float o[W];
#pragma unroll
        for (int w = 0; w < W; ++w) o[w] = yv[i][w] * (gv[i][w] - dot[0]);
        V::store(dr, idx, o);
      }
    }
  }
}

// softmax_grad for rows wider than the register budget: two passes over the
// row (the second from L2).
__global__ void __launch_bounds__(kThreads)
    softmax_grad_looped_kernel(const float *__restrict__ y, const float *__restrict__ dy,
                               float *dx, uint32_t rows, uint32_t cols, uint32_t ld) {
  __shared__ float red[32];
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *yr = y + (size_t)r * ld;
    const float *gr = dy + (size_t)r * ld;
    float dot[1] = {0.0f};
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads) dot[0] = fmaf(yr[c], gr[c], dot[0]);
    block_sum<1>(dot, red);
    float *dr = dx + (size_t)r * ld;
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads) dr[c] = yr[c] * (gr[c] - dot[0]);
  }
}

// Row sums (axis 1): one CTA per row, grid-stride.
template <bool V4>
__global__ void __launch_bounds__(kThreads)
    row_sum_kernel(const float *__restrict__ x, float *__restrict__ out, uint32_t rows,
                   uint32_t cols, uint32_t ld) {
  using V = Vec<V4>;
  constexpr int W = V::W;
  __shared__ float red[32];
  const uint32_t nv = cols / W;
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *xr = x + (size_t)r * ld;
    float s[1] = {0.0f};
    for (uint32_t i = threadIdx.x; i < nv; i += kThreads) {
      float v[W];
      V::load_stream(xr, i, v);
#pragma unroll
      for (int w = 0; w < W; ++w) s[0] += v[w];
    }
    block_sum<1>(s, red);
    if (threadIdx.x == 0) out[r] = s[0];
  }
}

// Column sums (axis 0), pass 1: a 2-D grid of (column chunk, row group).
// Thread t of CTA (cx, g) owns one 4-column vector (or one column) of chunk
// cx and sums rows g, g + G, ... of it, eight loads in flight; the CTA writes
// partial row g of its chunk.
template <bool V4>
__global__ void __launch_bounds__(kThreads)
    col_partial_kernel(const float *__restrict__ x, float *__restrict__ part, uint32_t rows,
                       uint32_t cols, uint32_t ld) {
  constexpr uint32_t W = V4 ? 4 : 1;
  const uint32_t cv = blockIdx.x * kThreads + threadIdx.x;  // vector index in the row
  if (cv * W >= cols) return;
  const uint32_t G = gridDim.y;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  uint32_t r = blockIdx.y;
  for (; r + 7 * G < rows; r += 8 * G) {
    float4 t[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float *p = x + (size_t)(r + u * G) * ld;
      t[u] = V4 ? __ldcs(reinterpret_cast<const float4 *>(p) + cv)
                : make_float4(__ldcs(p + cv), 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      a.x += t[u].x;
      a.y += t[u].y;
      a.z += t[u].z;
      a.w += t[u].w;
    }
  }
  for (; r < rows; r += G) {
    const float *p = x + (size_t)r * ld;
    const float4 t = V4 ? __ldcs(reinterpret_cast<const float4 *>(p) + cv)
                        : make_float4(__ldcs(p + cv), 0.f, 0.f, 0.f);
    a.x += t.x;
    a.y += t.y;
    a.z += t.z;
    a.w += t.w;
  }
  float *dst = part + (size_t)blockIdx.y * cols;
  if (V4) reinterpret_cast<float4 *>(dst)[cv] = a;
  else dst[cv] = a.x;
}

// Column sums, pass 2: out[c] = sum over the G partial rows, in order.
__global__ void col_finish_kernel(const float *__restrict__ part, float *__restrict__ out,
                                  uint32_t g, uint32_t cols) {
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.0f;
  for (uint32_t i = 0; i < g; ++i) s += part[(size_t)i * cols + c];
  out[c] = s;
}

// dst[r, c] = src[axis == 1 ? r : c]
template <bool V4>
__global__ void __launch_bounds__(kThreads)
    broadcast_kernel(const float *__restrict__ src, float *__restrict__ dst, uint32_t rows,
                     uint32_t cols, uint32_t ld, int axis) {
  constexpr uint32_t W = V4 ? 4 : 1;
  const uint32_t nv = cols / W;
  const size_t n = (size_t)rows * nv;
  for (size_t i = blockIdx.x * (size_t)kThreads + threadIdx.x; i < n;
       i += (size_t)gridDim.x * kThreads) {
    const uint32_t r = (uint32_t)(i / nv), cv = (uint32_t)(i % nv);
    if (V4) {
      const float4 v = axis == 1 ? make_float4(src[r], src[r], src[r], src[r])
                                 : __ldg(reinterpret_cast<const float4 *>(src) + cv);
      __stcs(reinterpret_cast<float4 *>(dst + (size_t)r * ld) + cv, v);
    } else {
      __stcs(dst + (size_t)r * ld + cv, axis == 1 ? src[r] : src[cv]);
    }
  }
}

uint32_t grid_rows(BwppCudaCtx *ctx, uint32_t rows, int per_sm) {
  const uint32_t g = (uint32_t)ctx->num_sms * per_sm;
  return rows < g ? (rows ? rows : 1) : g;
}

uint32_t grid_flat(BwppCudaCtx *ctx, size_t n) {
  const size_t blocks = (n + kThreads - 1) / kThreads;
  const size_t cap = (size_t)ctx->num_sms * 8;
  return (uint32_t)(blocks < cap ? (blocks ? blocks : 1) : cap);
}

}  // namespace

extern "C" {

int bwpp_cuda_silu_grad_f32(BwppCudaCtx *ctx, const float *x, const float *dy, float *dx,
                            size_t n) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (n && (!x || !dy || !dx)) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "silu_grad: NULL");
  if (n == 0) return BWPP_CUDA_OK;
  if (n % 4 == 0 && al16(x) && al16(dy) && al16(dx))
    silu_grad_kernel<true><<<grid_flat(ctx, n / 4), kThreads, 0, ctx->stream>>>(x, dy, dx, n);
  else
    silu_grad_kernel<false><<<grid_flat(ctx, n), kThreads, 0, ctx->stream>>>(x, dy, dx, n);
  BWPP_LAUNCH_CHECK(ctx, "silu_grad");
  return BWPP_CUDA_OK;
}

int bwpp_cuda_softmax_grad_f32(BwppCudaCtx *ctx, const float *y, const float *dy, float *dx,
                               uint32_t rows, uint32_t cols, uint32_t ld) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (ld < cols || (rows && cols && (!y || !dy || !dx)))
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "softmax_grad: bad args");
  if (rows == 0 || cols == 0) return BWPP_CUDA_OK;
  const bool v4 = cols % 4 == 0 && ld % 4 == 0 && al16(y) && al16(dy) && al16(dx);
  const uint32_t nv = v4 ? cols / 4 : cols;
  const uint32_t per = (nv + kThreads - 1) / kThreads;
  const uint32_t grid = grid_rows(ctx, rows, 8);
  cudaStream_t s = ctx->stream;
#define BWPP_SMG(MV)                                                                        \
  (v4 ? softmax_grad_kernel<MV, true><<<grid, kThreads, 0, s>>>(y, dy, dx, rows, cols, ld)  \
      : softmax_grad_kernel<MV, false><<<grid, kThreads, 0, s>>>(y, dy, dx, rows, cols, ld))
  if (per <= 1) BWPP_SMG(1);
  else if (per <= 2) BWPP_SMG(2);
  else if (per <= 4) BWPP_SMG(4);
  else if (per <= 8) BWPP_SMG(8);
  else softmax_grad_looped_kernel<<<grid, kThreads, 0, s>>>(y, dy, dx, rows, cols, ld);
#undef BWPP_SMG
  BWPP_LAUNCH_CHECK(ctx, "softmax_grad");
  return BWPP_CUDA_OK;
}

int bwpp_cuda_reduce_sum_f32(BwppCudaCtx *ctx, const float *x, float *out, uint32_t rows,
                             uint32_t cols, uint32_t ld, int axis) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if ((axis != 0 && axis != 1) || ld < cols)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "reduce_sum: bad axis or ld");
  const uint32_t outn = axis == 1 ? rows : cols;
  if (outn == 0) return BWPP_CUDA_OK;
  if (!out || (rows && cols && !x)) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "reduce_sum: NULL");
  cudaStream_t s = ctx->stream;
  if (rows == 0 || cols == 0)  // sums over nothing
    return bwpp_check_cuda(ctx, cudaMemsetAsync(out, 0, (size_t)outn * 4, s), "reduce_sum zero");
  const bool v4 = cols % 4 == 0 && ld % 4 == 0 && al16(x);
  if (axis == 1) {
    if (v4) row_sum_kernel<true><<<grid_rows(ctx, rows, 8), kThreads, 0, s>>>(x, out, rows, cols, ld);
    else row_sum_kernel<false><<<grid_rows(ctx, rows, 8), kThreads, 0, s>>>(x, out, rows, cols, ld);
    BWPP_LAUNCH_CHECK(ctx, "reduce_sum rows");
    return BWPP_CUDA_OK;
  }
  // about 4 CTAs per SM in total, split between column chunks and row groups
  const uint32_t chunks = (cols + (v4 ? 4 : 1) * kThreads - 1) / ((v4 ? 4 : 1) * kThreads);
  const uint32_t want = (uint32_t)ctx->num_sms * 4;
  uint32_t g = want / chunks;
  if (g < 1) g = 1;
  if (g > rows) g = rows;
  if (g > 65535) g = 65535;
  float *part = static_cast<float *>(bwpp_ctx_workspace(ctx, (size_t)g * cols * 4));
  if (!part) return BWPP_CUDA_ERR_NOMEM;
  if (v4 && al16(part))
    col_partial_kernel<true><<<dim3(chunks, g), kThreads, 0, s>>>(x, part, rows, cols, ld);
  else
    col_partial_kernel<false><<<dim3((cols + kThreads - 1) / kThreads, g), kThreads, 0, s>>>(
        x, part, rows, cols, ld);
  col_finish_kernel<<<(cols + 255) / 256, 256, 0, s>>>(part, out, g, cols);
  BWPP_LAUNCH_CHECK(ctx, "reduce_sum cols");
  return BWPP_CUDA_OK;
}

int bwpp_cuda_broadcast_f32(BwppCudaCtx *ctx, const float *src, float *dst, uint32_t rows,
                            uint32_t cols, uint32_t ld, int axis) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if ((axis != 0 && axis != 1) || ld < cols)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "broadcast: bad axis or ld");
  if (rows == 0 || cols == 0) return BWPP_CUDA_OK;
  if (!src || !dst) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "broadcast: NULL");
  const bool v4 = cols % 4 == 0 && ld % 4 == 0 && al16(dst) && (axis == 1 || al16(src));
  const size_t n = (size_t)rows * (v4 ? cols / 4 : cols);
  if (v4)
    broadcast_kernel<true><<<grid_flat(ctx, n), kThreads, 0, ctx->stream>>>(src, dst, rows, cols, ld, axis);
  else
    broadcast_kernel<false><<<grid_flat(ctx, n), kThreads, 0, ctx->stream>>>(src, dst, rows, cols, ld, axis);
  BWPP_LAUNCH_CHECK(ctx, "broadcast");
  return BWPP_CUDA_OK;
}

}  // extern "C"
