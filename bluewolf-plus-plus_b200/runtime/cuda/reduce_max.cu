// reduce_max forward (max + first-index argmax), its argmax-routed gradient,
// the reference's tie-mask form and its gradient, and row softmax.  fp32,
// HBM-bound: 128-bit coalesced loads / streaming stores, one CTA per row
// (grid-stride), warp-shuffle reductions.
//
// Reference: runtime/cpu/bwpp_cpu_ref.c:37-61 (softmax), :146-190 (mask),
// :192-219 (mask gradient); autodiff rule compiler/graph_ir.c:1798-1821.
#include <math.h>

#include "bwpp_cuda_internal.cuh"
#include "rowwise.cuh"

namespace {

constexpr int kThreads = 256;
constexpr uint32_t kNoIndex = 0xFFFFFFFFu;

inline bool aligned16(const void *p) {
  return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// (value, index) pair order: larger value wins; equal values -> smaller index.
__device__ __forceinline__ void arg_combine(float &v, uint32_t &i, float ov,
                                            uint32_t oi) {
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}

__device__ __forceinline__ void block_argmax(float &v, uint32_t &i,
                                             float *sv, uint32_t *si) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
    arg_combine(v, i, ov, oi);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = i;
  }
  __syncthreads();
  const int nw = blockDim.x >> 5;
  v = lane < nw ? sv[lane] : -INFINITY;
  i = lane < nw ? si[lane] : kNoIndex;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
    arg_combine(v, i, ov, oi);
  }
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

__device__ __forceinline__ float block_sum1(float v, float *sv) {
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

// Each thread scans its elements in increasing index order with a strict '>'
// (so it keeps its first maximum); the block combine prefers smaller indices
// on equal values.  A row with no element > -INF yields (-INF, 0), matching
// the serial scan.  NaN never compares greater, as in the serial scan.
template <bool V4>
__global__ void __launch_bounds__(kThreads)
    argmax_kernel(const float *__restrict__ x, float *__restrict__ maxv,
                  uint32_t *__restrict__ argmax, uint32_t rows, uint32_t cols,
                  uint32_t ld) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *xr = x + (size_t)r * ld;
    float best = -INFINITY;
    uint32_t bi = kNoIndex;
    if (V4) {
      const float4 *x4 = reinterpret_cast<const float4 *>(xr);
      const uint32_t nv = cols >> 2;
      uint32_t idx = threadIdx.x;
      for (; idx + 3 * kThreads < nv; idx += 4 * kThreads) {
        float4 t[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) t[u] = __ldcs(x4 + idx + u * kThreads);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t e = (idx + u * kThreads) * 4;
          if (t[u].x > best) { best = t[u].x; bi = e; }
          if (t[u].y > best) { best = t[u].y; bi = e + 1; }
          if (t[u].z > best) { best = t[u].z; bi = e + 2; }
          if (t[u].w > best) { best = t[u].w; bi = e + 3; }
        }
      }
      for (; idx < nv; idx += kThreads) {
        const float4 t = __ldcs(x4 + idx);
        const uint32_t e = idx * 4;
        if (t.x > best) { best = t.x; bi = e; }
        if (t.y > best) { best = t.y; bi = e + 1; }
        if (t.z > best) { best = t.z; bi = e + 2; }
        if (t.w > best) { best = t.w; bi = e + 3; }
      }
    } else {
      for (uint32_t c = threadIdx.x; c < cols; c += kThreads) {
        const float t = xr[c];
        if (t > best) { best = t; bi = c; }
      }
    }
    block_argmax(best, bi, sv, si);
    if (threadIdx.x == 0) {
      if (maxv) maxv[r] = best;
      if (argmax) argmax[r] = bi == kNoIndex ? 0u : bi;
    }
  }
}

// dx[r, c] = c == argmax[r] ? dy[r] : 0   (write-only pass over dx)
template <bool V4>
__global__ void __launch_bounds__(kThreads)
    argmax_bwd_kernel(const uint32_t *__restrict__ argmax,
                      const float *__restrict__ dy, float *__restrict__ dx,
                      uint32_t rows, uint32_t cols, uint32_t ld) {
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint32_t a = __ldg(argmax + r);
    const float g = __ldg(dy + r);
    float *dr = dx + (size_t)r * ld;
    if (V4) {
      float4 *d4 = reinterpret_cast<float4 *>(dr);
      const uint32_t nv = cols >> 2;
      for (uint32_t idx = threadIdx.x; idx < nv; idx += kThreads) {
        const uint32_t e = idx * 4;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (a - e < 4u) {
          if (a == e) o.x = g;
          else if (a == e + 1) o.y = g;
          else if (a == e + 2) o.z = g;
          else o.w = g;
        }
        __stcs(d4 + idx, o);
      }
    } else {
      for (uint32_t c = threadIdx.x; c < cols; c += kThreads)
        dr[c] = c == a ? g : 0.0f;
    }
  }
}

// mask along rows (axis 1): mask = x == rowmax (every tie set)
__global__ void __launch_bounds__(kThreads)
    mask_rows_kernel(const float *__restrict__ x, float *__restrict__ mask,
                     uint32_t rows, uint32_t cols) {
  __shared__ float sv[32];
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *xr = x + (size_t)r * cols;
    float m = -INFINITY;
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads) {
      const float t = xr[c];
      if (t > m) m = t;
    }
    m = block_max(m, sv);
    float *mr = mask + (size_t)r * cols;
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads)
      mr[c] = xr[c] == m ? 1.0f : 0.0f;
  }
}

// mask along columns (axis 0): thread per column
__global__ void mask_cols_kernel(const float *__restrict__ x,
                                 float *__restrict__ mask, uint32_t rows,
                                 uint32_t cols) {
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float m = -INFINITY;
  for (uint32_t r = 0; r < rows; ++r) {
    const float t = x[(size_t)r * cols + c];
    if (t > m) m = t;
  }
  for (uint32_t r = 0; r < rows; ++r)
    mask[(size_t)r * cols + c] = x[(size_t)r * cols + c] == m ? 1.0f : 0.0f;
}

__global__ void mask_grad_kernel(const float *__restrict__ mask,
                                 const float *__restrict__ dy,
                                 float *__restrict__ dx, uint32_t rows,
                                 uint32_t cols, int axis) {
  const size_t n = (size_t)rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t r = (uint32_t)(i / cols), c = (uint32_t)(i % cols);
    dx[i] = mask[i] * (axis == 0 ? dy[c] : dy[r]);
  }
}

// Row softmax with the row held in registers (one HBM read, one write):
// max by strict '>' from -INF (NaN never wins, as the serial scan of
// runtime/cpu/bwpp_cpu_ref.c:43-49), e = expf(x - max) kept in registers,
// sum, inv = sum > 0 ? 1/sum : 0 (line 56), y = e * inv.
template <int MAXV, bool V4>
__global__ void __launch_bounds__(kThreads)
    softmax_rows_kernel(const float *__restrict__ x, float *__restrict__ y, uint32_t rows,
                        uint32_t cols, uint32_t ld) {
  using V = bwpp_row::Vec<V4>;
  constexpr int W = V::W;
  __shared__ float sv[32];
  const uint32_t nv = cols / W;
  // The next row's loads are issued before this row's two block reductions,
  // so a CTA keeps a second row in flight through its serial phases.
  float xv[MAXV][W];
  auto load_row = [&](uint32_t r, float (&dst)[MAXV][W]) {
    const float *xr = x + (size_t)r * ld;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const uint32_t idx = threadIdx.x + i * kThreads;
      if (idx < nv) V::load_stream(xr, idx, dst[i]);
    }
  };
  if (blockIdx.x < rows) load_row(blockIdx.x, xv);
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    float nx[MAXV][W];
    const uint32_t rn = r + gridDim.x;
    if (rn < rows) load_row(rn, nx);
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const uint32_t idx = threadIdx.x + i * kThreads;
#pragma unroll
      for (int w = 0; w < W; ++w)
        if (idx < nv && xv[i][w] > m) m = xv[i][w];
    }
    m = block_max(m, sv);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const uint32_t idx = threadIdx.x + i * kThreads;
      if (idx < nv)
#pragma unroll
        for (int w = 0; w < W; ++w) {
          xv[i][w] = expf(xv[i][w] - m);
          s += xv[i][w];
        }
    }
    s = block_sum1(s, sv);
    const float inv = s > 0.0f ? 1.0f / s : 0.0f;
    float *yr = y + (size_t)r * ld;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const uint32_t idx = threadIdx.x + i * kThreads;
      if (idx < nv) {
#pragma unroll
        for (int w = 0; w < W; ++w) xv[i][w] *= inv;
        V::store(yr, idx, xv[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
#pragma unroll
      for (int w = 0; w < W; ++w) xv[i][w] = nx[i][w];
  }
}

// Row softmax for rows wider than the register budget: three passes as
// runtime/cpu/bwpp_cpu_ref.c:37-61 (the second and third from L2).
__global__ void __launch_bounds__(kThreads)
    softmax_kernel(const float *__restrict__ x, float *__restrict__ y,
                   uint32_t rows, uint32_t cols, uint32_t ld) {
  __shared__ float sv[32];
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *xr = x + (size_t)r * ld;
    float *yr = y + (size_t)r * ld;
    float m = -INFINITY;
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads) {
      const float t = xr[c];
      if (t > m) m = t;
    }
    m = block_max(m, sv);
    float s = 0.0f;
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads) s += expf(xr[c] - m);
    s = block_sum1(s, sv);
    const float inv = s > 0.0f ? 1.0f / s : 0.0f;
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads)
      yr[c] = expf(xr[c] - m) * inv;
  }
}

uint32_t grid_for(BwppCudaCtx *ctx, uint32_t rows, int per_sm) {
  const uint32_t g = (uint32_t)ctx->num_sms * per_sm;
  return rows < g ? (rows ? rows : 1) : g;
}

}  // namespace

extern "C" {

int bwpp_cuda_reduce_max_fwd_f32(BwppCudaCtx *ctx, const float *x, float *maxv,
                                 uint32_t *argmax, uint32_t rows,
                                 uint32_t cols, uint32_t ld) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!x || ld < cols || cols == 0)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "reduce_max fwd: bad args");
  if (rows == 0) return BWPP_CUDA_OK;
  const bool v4 = cols % 4 == 0 && ld % 4 == 0 && aligned16(x);
  const uint32_t grid = grid_for(ctx, rows, 8);
  if (v4)
    argmax_kernel<true><<<grid, kThreads, 0, ctx->stream>>>(x, maxv, argmax, rows, cols, ld);
  else
    argmax_kernel<false><<<grid, kThreads, 0, ctx->stream>>>(x, maxv, argmax, rows, cols, ld);
  BWPP_LAUNCH_CHECK(ctx, "reduce_max fwd");
  return BWPP_CUDA_OK;
}

int bwpp_cuda_reduce_max_bwd_f32(BwppCudaCtx *ctx, const uint32_t *argmax,
                                 const float *dy, float *dx, uint32_t rows,
                                 uint32_t cols, uint32_t ld) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!argmax || !dy || !dx || ld < cols)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "reduce_max bwd: bad args");
  if (rows == 0 || cols == 0) return BWPP_CUDA_OK;
  const bool v4 = cols % 4 == 0 && ld % 4 == 0 && aligned16(dx);
  const uint32_t grid = grid_for(ctx, rows, 8);
  if (v4)
    argmax_bwd_kernel<true><<<grid, kThreads, 0, ctx->stream>>>(argmax, dy, dx, rows, cols, ld);
  else
    argmax_bwd_kernel<false><<<grid, kThreads, 0, ctx->stream>>>(argmax, dy, dx, rows, cols, ld);
  BWPP_LAUNCH_CHECK(ctx, "reduce_max bwd");
  return BWPP_CUDA_OK;
}

int bwpp_cuda_reduce_max_mask_ex(BwppCudaCtx *ctx, const float *x, float *mask,
                                 uint32_t rows, uint32_t cols, int axis) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!x || !mask) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "mask: NULL");
  if (rows == 0 || cols == 0) return BWPP_CUDA_OK;
  if (axis == 0)
    mask_cols_kernel<<<(cols + 255) / 256, 256, 0, ctx->stream>>>(x, mask, rows, cols);
  else
    mask_rows_kernel<<<grid_for(ctx, rows, 8), kThreads, 0, ctx->stream>>>(x, mask, rows, cols);
  BWPP_LAUNCH_CHECK(ctx, "reduce_max mask");
  return BWPP_CUDA_OK;
}

int bwpp_cuda_reduce_max_grad_ex(BwppCudaCtx *ctx, const float *mask,
                                 const float *dy, float *dx, uint32_t rows,
                                 uint32_t cols, int axis) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!mask || !dy || !dx) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "mask grad: NULL");
  if (rows == 0 || cols == 0) return BWPP_CUDA_OK;
  mask_grad_kernel<<<(uint32_t)ctx->num_sms * 8, 256, 0, ctx->stream>>>(mask, dy, dx, rows, cols, axis);
  BWPP_LAUNCH_CHECK(ctx, "reduce_max mask grad");
  return BWPP_CUDA_OK;
}

int bwpp_cuda_softmax_fwd_f32(BwppCudaCtx *ctx, const float *x, float *y,
                              uint32_t rows, uint32_t cols, uint32_t ld) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!x || !y || ld < cols) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "softmax: bad args");
  if (rows == 0 || cols == 0) return BWPP_CUDA_OK;
  const bool v4 = cols % 4 == 0 && ld % 4 == 0 && aligned16(x) && aligned16(y);
  const uint32_t per = ((v4 ? cols / 4 : cols) + kThreads - 1) / kThreads;
  const uint32_t grid = grid_for(ctx, rows, 8);
  cudaStream_t s = ctx->stream;
#define BWPP_SMX(MV)                                                                   \
  (v4 ? softmax_rows_kernel<MV, true><<<grid, kThreads, 0, s>>>(x, y, rows, cols, ld)  \
      : softmax_rows_kernel<MV, false><<<grid, kThreads, 0, s>>>(x, y, rows, cols, ld))
  if (per <= 1) BWPP_SMX(1);
  else if (per <= 2) BWPP_SMX(2);
  else if (per <= 4) BWPP_SMX(4);
  else if (per <= 8) BWPP_SMX(8);
  else if (per <= 16) BWPP_SMX(16);
  else softmax_kernel<<<grid, kThreads, 0, s>>>(x, y, rows, cols, ld);
#undef BWPP_SMX
  BWPP_LAUNCH_CHECK(ctx, "softmax");
  return BWPP_CUDA_OK;
}

}  // extern "C"
