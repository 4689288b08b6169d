// RMSNorm / LayerNorm forward and backward, fp32, HBM-bound.
//
// Row kernels: one CTA per row (grid-stride), the row held in registers as
// 128-bit vectors (thread t owns vectors t, t+T, t+2T, ...: every load and
// store instruction of a warp touches 512 contiguous bytes), warp-shuffle +
// shared-memory block reductions.  Rows wider than the register budget use a
// looped variant that re-reads the row (from L2) instead.
//
// Backward: a persistent grid; each CTA walks rows blockIdx.x, +gridDim.x, ...
// and accumulates its dgamma / dbeta partial for the columns its threads own
// in shared memory, then writes one partial row to scratch.  A second kernel
// sums the partials over CTAs in a fixed order, so results are deterministic.
//
// Reference: runtime/cpu/bwpp_cpu_ref.c:63-90 (rmsnorm fwd); backward rule
// compiler/graph_ir.c:1735-1789; layernorm has no reference counterpart.
#include <pthread.h>

#include "bwpp_cuda_internal.cuh"
#include "rowwise.cuh"

namespace {

using bwpp_row::Vec;
using bwpp_row::block_sum;

constexpr int kThreads = 256;
constexpr int kMaxVecFwd = 16;  // fwd: up to 256*16 vectors in registers
constexpr int kMaxVecBwd = 8;   // bwd: x and dy both resident

// ---------------------------------------------------------------------------
// forward, row held in registers
// ---------------------------------------------------------------------------
template <int MAXV, bool V4, bool CENTERED>
__global__ void __launch_bounds__(kThreads)
    norm_fwd_kernel(const float *__restrict__ x, float *__restrict__ y,
                    const float *__restrict__ gamma,
                    const float *__restrict__ beta, uint32_t rows,
                    uint32_t cols, uint32_t ld, float eps) {
  using V = Vec<V4>;
  constexpr int W = V::W;
  __shared__ float red[3 * 32];
  const uint32_t nv = cols / W;
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *xr = x + (size_t)r * ld;
    float *yr = y + (size_t)r * ld;
    float xv[MAXV][W];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const uint32_t idx = threadIdx.x + i * kThreads;
      if (idx < nv) V::load_stream(xr, idx, xv[i]);
      else
#pragma unroll
        for (int w = 0; w < W; ++w) xv[i][w] = 0.0f;
    }
    float mean = 0.0f;
    if (CENTERED) {
      float s[1] = {0.0f};
#pragma unroll
      for (int i = 0; i < MAXV; ++i)
#pragma unroll
        for (int w = 0; w < W; ++w) s[0] += xv[i][w];
      block_sum<1>(s, red);
      mean = s[0] / (float)cols;
    }
    float ss[1] = {0.0f};
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const uint32_t idx = threadIdx.x + i * kThreads;
      if (idx < nv)
#pragma unroll
        for (int w = 0; w < W; ++w) {
          const float d = xv[i][w] - mean;
          ss[0] += d * d;
        }
    }
    block_sum<1>(ss, red);
    const float inv = 1.0f / sqrtf(ss[0] / (float)cols + eps);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const uint32_t idx = threadIdx.x + i * kThreads;
      if (idx >= nv) continue;
      float g[W], b[W], o[W];
      if (gamma) V::load(gamma, idx, g);
      if (beta) V::load(beta, idx, b);
#pragma unroll
      for (int w = 0; w < W; ++w) {
        float v = (xv[i][w] - mean) * inv;
        if (gamma) v *= g[w];
        if (beta) v += b[w];
        o[w] = v;
      }
      V::store(yr, idx, o);
    }
  }
}

// forward, any width: re-reads the row
template <bool CENTERED>
__global__ void __launch_bounds__(kThreads)
    norm_fwd_looped_kernel(const float *__restrict__ x, float *__restrict__ y,
                           const float *__restrict__ gamma,
                           const float *__restrict__ beta, uint32_t rows,
                           uint32_t cols, uint32_t ld, float eps) {
  __shared__ float red[3 * 32];
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *xr = x + (size_t)r * ld;
    float *yr = y + (size_t)r * ld;
    float mean = 0.0f;
    if (CENTERED) {
      float s[1] = {0.0f};
      for (uint32_t c = threadIdx.x; c < cols; c += kThreads) s[0] += xr[c];
      block_sum<1>(s, red);
      mean = s[0] / (float)cols;
    }
    float ss[1] = {0.0f};
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads) {
      const float d = xr[c] - mean;
      ss[0] += d * d;
    }
    block_sum<1>(ss, red);
    const float inv = 1.0f / sqrtf(ss[0] / (float)cols + eps);
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads) {
      float v = (xr[c] - mean) * inv;
      if (gamma) v *= gamma[c];
      if (beta) v += beta[c];
      yr[c] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
// Per row (CENTERED = layernorm, else rmsnorm), with g = gamma * dy:
//   mu = CENTERED ? mean(x) : 0;  r = 1/sqrt(mean((x-mu)^2) + eps)
//   xhat = (x - mu) r;  dx = r (g - CENTERED*mean(g) - xhat mean(g xhat))
//   dgamma += dy xhat;  dbeta += dy
// One block reduction per row.  For layernorm the statistics come from sums
// shifted by the row's first element k (broadcast load):
//   s1 = sum(x-k), s2 = sum((x-k)^2), sg = sum g, sgx = sum g (x-k)
//   mean = k + s1/C, var = s2/C - (s1/C)^2, sum g xhat = r (sgx - (s1/C) sg)
// which keeps var well conditioned when |mean| >> std.  The CTA's dgamma /
// dbeta partials live in shared memory (each thread owns fixed columns, so
// there are no conflicts), leaving registers for more resident CTAs.
// ACC: the residual-gradient form (acc += dx, acc16 = bf16(acc)), a separate
// instantiation so the plain kernels keep their register count (they fill an
// SM with 4 CTAs at <= 64 registers).
template <int MAXV, bool V4, bool CENTERED, bool ACC = false>
__global__ void __launch_bounds__(kThreads)
    norm_bwd_kernel(const float *__restrict__ x, const float *__restrict__ gamma,
                    const float *__restrict__ dy, float *__restrict__ dx,
                    float *__restrict__ part_g, float *__restrict__ part_b,
                    uint32_t rows, uint32_t cols, uint32_t ld, float eps,
                    float *__restrict__ acc, uint16_t *__restrict__ acc16) {
  using V = Vec<V4>;
  constexpr int W = V::W;
  __shared__ float red[4 * 32];
  extern __shared__ float sacc[];  // [2][cols] when part_g != nullptr
  float *acc_g = sacc, *acc_b = sacc + cols;
  const uint32_t nv = cols / W;
  if (part_g)
    for (uint32_t c = threadIdx.x; c < 2 * cols; c += kThreads) sacc[c] = 0.0f;
  // (each thread only ever touches its own columns of sacc: no barrier needed)
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *xr = x + (size_t)r * ld;
    const float *gr = dy + (size_t)r * ld;
    float xv[MAXV][W], dv[MAXV][W];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const uint32_t idx = threadIdx.x + i * kThreads;
      if (idx < nv) {
        V::load_stream(xr, idx, xv[i]);
        V::load_stream(gr, idx, dv[i]);
      } else {
#pragma unroll
        for (int w = 0; w < W; ++w) xv[i][w] = dv[i][w] = 0.0f;
      }
    }
    const float k = CENTERED ? __ldg(xr) : 0.0f;
    // t = {sum (x-k)^2, sum g, sum g (x-k), sum (x-k)}
    float t[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const uint32_t idx = threadIdx.x + i * kThreads;
      if (idx >= nv) continue;
      float gm[W];
      if (gamma) V::load(gamma, idx, gm);
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const float d = xv[i][w] - k;
        const float g = (gamma ? gm[w] : 1.0f) * dv[i][w];
        t[0] += d * d;
        t[1] += g;
        t[2] += g * d;
        t[3] += d;
      }
    }
    block_sum<4>(t, red);
    const float inv_c = 1.0f / (float)cols;
    const float m1 = CENTERED ? t[3] * inv_c : 0.0f;            // mean - k
    const float var = CENTERED ? fmaxf(t[0] * inv_c - m1 * m1, 0.0f) : t[0] * inv_c;
    const float rs = 1.0f / sqrtf(var + eps);
    const float mg = CENTERED ? t[1] * inv_c : 0.0f;
    const float mgx = rs * (t[2] - m1 * t[1]) * inv_c;           // mean(g * xhat)
    const float mu = k + m1;
    float *dxr = dx + (size_t)r * ld;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const uint32_t idx = threadIdx.x + i * kThreads;
      if (idx >= nv) continue;
      float gm[W], o[W];
      if (gamma) V::load(gamma, idx, gm);
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const float xh = (xv[i][w] - mu) * rs;
        const float g = (gamma ? gm[w] : 1.0f) * dv[i][w];
        o[w] = rs * (g - mg - xh * mgx);
        xv[i][w] = xh;  // keep xhat for the partials below
      }
      if constexpr (ACC) {
        // residual-gradient form: acc += dx (and acc16 = bf16(acc)); dx
        // itself is not written
        float *ar = acc + (size_t)r * ld;
        float h[W];
        V::load_stream(ar, idx, h);
#pragma unroll
        for (int w = 0; w < W; ++w) h[w] += o[w];
        V::store(ar, idx, h);
        if (acc16) {
          uint16_t *hr = acc16 + (size_t)r * ld;
          if constexpr (W == 4) {
            *reinterpret_cast<uint2 *>(hr + 4 * (size_t)idx) =
                make_uint2(pack2_16<false>(h[0], h[1]), pack2_16<false>(h[2], h[3]));
          } else {
            hr[idx] = (uint16_t)(pack2_16<false>(h[0], 0.0f) & 0xFFFFu);
          }
        }
      } else {
        V::store(dxr, idx, o);
      }
      if (part_g) {
        // 128-bit shared accesses: a warp touches 512 contiguous bytes
        if constexpr (W == 4) {
          float4 *ag = reinterpret_cast<float4 *>(acc_g) + idx;
          float4 *ab = reinterpret_cast<float4 *>(acc_b) + idx;
          float4 tg = *ag, tb = *ab;
          tg.x += dv[i][0] * xv[i][0]; tg.y += dv[i][1] * xv[i][1];
          tg.z += dv[i][2] * xv[i][2]; tg.w += dv[i][3] * xv[i][3];
          tb.x += dv[i][0]; tb.y += dv[i][1]; tb.z += dv[i][2]; tb.w += dv[i][3];
          *ag = tg;
          *ab = tb;
        } else {
          acc_g[idx] += dv[i][0] * xv[i][0];
          acc_b[idx] += dv[i][0];
        }
      }
    }
  }
  if (part_g) {
    __syncthreads();
    float *pg = part_g + (size_t)blockIdx.x * cols;
    float *pb = part_b + (size_t)blockIdx.x * cols;
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads) {
      // column c was accumulated by the thread that owns vector c / W
      pg[c] = acc_g[c];
      pb[c] = acc_b[c];
    }
  }
}

// backward, any width (re-reads x and dy)
template <bool CENTERED>
__global__ void __launch_bounds__(kThreads)
    norm_bwd_looped_kernel(const float *__restrict__ x,
                           const float *__restrict__ gamma,
                           const float *__restrict__ dy, float *__restrict__ dx,
                           float *__restrict__ part_g, float *__restrict__ part_b,
                           uint32_t rows, uint32_t cols, uint32_t ld,
                           float eps) {
  __shared__ float red[3 * 32];
  float *pg = part_g ? part_g + (size_t)blockIdx.x * cols : nullptr;
  float *pb = part_b ? part_b + (size_t)blockIdx.x * cols : nullptr;
  if (pg)
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads) pg[c] = pb[c] = 0.0f;
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *xr = x + (size_t)r * ld;
    const float *gr = dy + (size_t)r * ld;
    float mean = 0.0f;
    if (CENTERED) {
      float s[1] = {0.0f};
      for (uint32_t c = threadIdx.x; c < cols; c += kThreads) s[0] += xr[c];
      block_sum<1>(s, red);
      mean = s[0] / (float)cols;
    }
    float t[3] = {0.0f, 0.0f, 0.0f};
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads) {
      const float d = xr[c] - mean;
      const float g = (gamma ? gamma[c] : 1.0f) * gr[c];
      t[0] += d * d;
      t[1] += g;
      t[2] += g * d;
    }
    block_sum<3>(t, red);
    const float rs = 1.0f / sqrtf(t[0] / (float)cols + eps);
    const float mg = CENTERED ? t[1] / (float)cols : 0.0f;
    const float mgx = t[2] * rs / (float)cols;
    float *dxr = dx + (size_t)r * ld;
    for (uint32_t c = threadIdx.x; c < cols; c += kThreads) {
      const float xh = (xr[c] - mean) * rs;
      const float g = (gamma ? gamma[c] : 1.0f) * gr[c];
      dxr[c] = rs * (g - mg - xh * mgx);
      if (pg) {
        pg[c] += gr[c] * xh;
        pb[c] += gr[c];
      }
    }
  }
}

// dgamma / dbeta from the backward's per-CTA partial rows:
// out_y[c] = sum over p < nparts of part_y[p * cols + c] (blockIdx.y = y; a
// NULL out_y is skipped).  A CTA takes 32 column groups (one per lane: four
// columns with V4, else one) and its 32 warps split the partial rows: warp w
// adds rows w, w + 32, w + 64, ... in that order, four loads in flight, and
// then one thread per column adds the 32 warp sums in warp order, so the
// order of the sum is fixed.  (One thread per column summing every row in
// turn kept only cols / 256 CTAs busy: ~25 us per output for 592 x 4096.)
constexpr int kColWarps = 32;
template <bool V4>
__global__ void __launch_bounds__(32 * kColWarps)
    column_sums_kernel(const float *__restrict__ part0, float *__restrict__ out0,
                       const float *__restrict__ part1, float *__restrict__ out1,
                       uint32_t nparts, uint32_t cols) {
  constexpr int W = V4 ? 4 : 1;  // columns per lane
  const float *part = blockIdx.y ? part1 : part0;
  float *out = blockIdx.y ? out1 : out0;
  if (!out) return;  // the whole block returns together
  __shared__ float sums[kColWarps][32 * W];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t c0 = (blockIdx.x * 32 + lane) * W;
  float acc[W];
#pragma unroll
  for (int e = 0; e < W; ++e) acc[e] = 0.0f;
  if (c0 < cols) {
    auto row = [&](uint32_t p, float (&v)[W]) {
      if constexpr (V4) {
        const float4 t = __ldg(reinterpret_cast<const float4 *>(part + (size_t)p * cols + c0));
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
      } else {
        v[0] = __ldg(part + (size_t)p * cols + c0);
      }
    };
    uint32_t p = (uint32_t)warp;
    for (; p + 3 * kColWarps < nparts; p += 4 * kColWarps) {
      float v[4][W];
#pragma unroll
      for (int u = 0; u < 4; ++u) row(p + u * kColWarps, v[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int e = 0; e < W; ++e) acc[e] += v[u][e];
    }
    for (; p < nparts; p += kColWarps) {
      float v[W];
      row(p, v);
#pragma unroll
      for (int e = 0; e < W; ++e) acc[e] += v[e];
    }
  }
#pragma unroll
  for (int e = 0; e < W; ++e) sums[warp][lane * W + e] = acc[e];
  __syncthreads();
  const uint32_t t = threadIdx.x;
  const uint32_t c = blockIdx.x * 32 * W + t;
  if (t < 32 * W && c < cols) {
    float total = sums[0][t];
    for (int w = 1; w < kColWarps; ++w) total += sums[w][t];
    out[c] = total;
  }
}

inline bool aligned16(const void *p) {
  return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Both column sums in one launch (either output may be NULL).
void launch_column_sums(cudaStream_t s, const float *pg, float *dgamma, const float *pb,
                        float *dbeta, uint32_t nparts, uint32_t cols) {
  if (cols % 4 == 0 && aligned16(pg) && aligned16(pb)) {
    const dim3 grid((cols / 4 + 31) / 32, 2);
    column_sums_kernel<true><<<grid, 32 * kColWarps, 0, s>>>(pg, dgamma, pb, dbeta, nparts, cols);
  } else {
    const dim3 grid((cols + 31) / 32, 2);
    column_sums_kernel<false><<<grid, 32 * kColWarps, 0, s>>>(pg, dgamma, pb, dbeta, nparts, cols);
  }
}


int pick_maxv(uint32_t nv, int limit) {
  uint32_t per = (nv + kThreads - 1) / kThreads;
  int m = 1;
  while ((uint32_t)m < per) m <<= 1;
  return m <= limit ? m : 0;  // 0: use the looped kernel
}

uint32_t row_grid(BwppCudaCtx *ctx, uint32_t rows, int ctas_per_sm) {
  uint32_t g = (uint32_t)ctx->num_sms * (uint32_t)ctas_per_sm;
  return rows < g ? (rows ? rows : 1) : g;
}

template <bool CENTERED>
int norm_fwd(BwppCudaCtx *ctx, const float *x, float *y, const float *gamma,
             const float *beta, uint32_t rows, uint32_t cols, uint32_t ld,
             float eps) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!x || !y || ld < cols) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "norm fwd: bad args");
  if (rows == 0 || cols == 0) return BWPP_CUDA_OK;
  const bool v4 = cols % 4 == 0 && ld % 4 == 0 && aligned16(x) && aligned16(y) &&
                  aligned16(gamma) && aligned16(beta);
  const uint32_t nv = v4 ? cols / 4 : cols;
  const int mv = pick_maxv(nv, kMaxVecFwd);
  const uint32_t grid = row_grid(ctx, rows, mv > 8 ? 4 : 8);
  cudaStream_t s = ctx->stream;
#define BWPP_FWD(MV, V4)                                                         \
  norm_fwd_kernel<MV, V4, CENTERED><<<grid, kThreads, 0, s>>>(x, y, gamma, beta, \
                                                              rows, cols, ld, eps)
  if (mv == 0) {
    norm_fwd_looped_kernel<CENTERED><<<grid, kThreads, 0, s>>>(x, y, gamma, beta,
                                                               rows, cols, ld, eps);
  } else if (v4) {
    switch (mv) {
      case 1: BWPP_FWD(1, true); break;
      case 2: BWPP_FWD(2, true); break;
      case 4: BWPP_FWD(4, true); break;
      case 8: BWPP_FWD(8, true); break;
      default: BWPP_FWD(16, true); break;
    }
  } else {
    switch (mv) {
      case 1: BWPP_FWD(1, false); break;
      case 2: BWPP_FWD(2, false); break;
      case 4: BWPP_FWD(4, false); break;
      case 8: BWPP_FWD(8, false); break;
      default: BWPP_FWD(16, false); break;
    }
  }
#undef BWPP_FWD
  BWPP_LAUNCH_CHECK(ctx, "norm fwd");
  return BWPP_CUDA_OK;
}

uint32_t bwd_grid(BwppCudaCtx *ctx, uint32_t rows) { return row_grid(ctx, rows, 4); }

// acc != NULL: instead of writing dx, add it into acc (and write bf16(acc) to
// acc16 when given); only rows held in registers (cols <= 8192 with dgamma).
template <bool CENTERED>
int norm_bwd(BwppCudaCtx *ctx, const float *x, const float *gamma,
             const float *dy, float *dx, float *dgamma, float *dbeta,
             uint32_t rows, uint32_t cols, uint32_t ld, float eps,
             float *scratch /* may be NULL: ctx workspace */,
             float *acc = nullptr, uint16_t *acc16 = nullptr) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (!x || !dy || (!dx && !acc) || ld < cols)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "norm bwd: bad args");
  if (cols == 0) return BWPP_CUDA_OK;
  cudaStream_t s = ctx->stream;
  if (rows == 0) {
    if (dgamma) cudaMemsetAsync(dgamma, 0, sizeof(float) * cols, s);
    if (dbeta) cudaMemsetAsync(dbeta, 0, sizeof(float) * cols, s);
    return BWPP_CUDA_OK;
  }
  const uint32_t grid = bwd_grid(ctx, rows);
  float *pg = nullptr, *pb = nullptr;
  if (dgamma || dbeta) {
    if (!scratch) {
      scratch = (float *)bwpp_ctx_workspace(ctx, sizeof(float) * 2 * (size_t)grid * cols);
      if (!scratch) return BWPP_CUDA_ERR_NOMEM;
    }
    pg = scratch;
    pb = scratch + (size_t)grid * cols;
  }
  const bool v4 = cols % 4 == 0 && ld % 4 == 0 && aligned16(x) && aligned16(dy) &&
                  aligned16(dx) && aligned16(gamma) && aligned16(acc) &&
                  (reinterpret_cast<uintptr_t>(acc16) & 7u) == 0;
  const uint32_t nv = v4 ? cols / 4 : cols;
  int mv = pick_maxv(nv, kMaxVecBwd);
  // partials in shared memory: 2 * cols floats per CTA
  const size_t acc_bytes = pg ? sizeof(float) * 2 * (size_t)cols : 0;
  if (acc_bytes > 48 * 1024) mv = 0;  // wide rows: looped kernel (global partials)
  if (acc && mv == 0)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_UNSUPPORTED, "norm bwd accumulate: row too wide");
#define BWPP_BWD(MV, V4)                                                           \
  (acc ? norm_bwd_kernel<MV, V4, CENTERED, true><<<grid, kThreads, acc_bytes, s>>>(  \
             x, gamma, dy, dx, pg, pb, rows, cols, ld, eps, acc, acc16)              \
       : norm_bwd_kernel<MV, V4, CENTERED, false><<<grid, kThreads, acc_bytes, s>>>( \
             x, gamma, dy, dx, pg, pb, rows, cols, ld, eps, nullptr, nullptr))
  if (mv == 0) {
    norm_bwd_looped_kernel<CENTERED><<<grid, kThreads, 0, s>>>(
        x, gamma, dy, dx, pg, pb, rows, cols, ld, eps);
  } else if (v4) {
    switch (mv) {
      case 1: BWPP_BWD(1, true); break;
      case 2: BWPP_BWD(2, true); break;
      case 4: BWPP_BWD(4, true); break;
      default: BWPP_BWD(8, true); break;
    }
  } else {
    switch (mv) {
      case 1: BWPP_BWD(1, false); break;
      case 2: BWPP_BWD(2, false); break;
      case 4: BWPP_BWD(4, false); break;
      default: BWPP_BWD(8, false); break;
    }
  }
#undef BWPP_BWD
  BWPP_LAUNCH_CHECK(ctx, "norm bwd");
  if (pg) {
    launch_column_sums(s, pg, dgamma, pb, dbeta, grid, cols);
    BWPP_LAUNCH_CHECK(ctx, "norm bwd column sum");
  }
  return BWPP_CUDA_OK;
}

}  // namespace

// Backward with caller-provided scratch (2 * grid * cols floats); used by the
// tiny_model step to keep scratch inside its arena.
int bwpp_norm_bwd_with_scratch(BwppCudaCtx *ctx, int centered, const float *x,
                               const float *gamma, const float *dy, float *dx,
                               float *dgamma, float *dbeta, uint32_t rows,
                               uint32_t cols, uint32_t ld, float eps,
                               float *scratch) {
  return centered ? norm_bwd<true>(ctx, x, gamma, dy, dx, dgamma, dbeta, rows,
                                   cols, ld, eps, scratch)
                  : norm_bwd<false>(ctx, x, gamma, dy, dx, dgamma, dbeta, rows,
                                    cols, ld, eps, scratch);
}

// Backward folded into a residual gradient: acc += dx, acc16 = bf16(acc)
// (acc16 may be NULL), dx never stored.  Rows must fit the register-resident
// kernel (BWPP_CUDA_ERR_UNSUPPORTED otherwise, with nothing launched).
int bwpp_norm_bwd_accumulate(BwppCudaCtx *ctx, int centered, const float *x,
                             const float *gamma, const float *dy, float *acc,
                             uint16_t *acc16, float *dgamma, float *dbeta,
                             uint32_t rows, uint32_t cols, uint32_t ld, float eps,
                             float *scratch) {
  return centered ? norm_bwd<true>(ctx, x, gamma, dy, nullptr, dgamma, dbeta, rows, cols, ld,
                                   eps, scratch, acc, acc16)
                  : norm_bwd<false>(ctx, x, gamma, dy, nullptr, dgamma, dbeta, rows, cols, ld,
                                    eps, scratch, acc, acc16);
}

extern "C" {

size_t bwpp_cuda_norm_bwd_workspace_size(BwppCudaCtx *ctx, uint32_t rows,
                                         uint32_t cols) {
  if (!ctx) return 0;
  return sizeof(float) * 2 * (size_t)bwd_grid(ctx, rows) * cols;
}

int bwpp_cuda_rmsnorm_fwd_f32(BwppCudaCtx *ctx, const float *x, float *y,
                              const float *gamma, const float *beta,
                              uint32_t rows, uint32_t cols, uint32_t ld,
                              float eps) {
  return norm_fwd<false>(ctx, x, y, gamma, beta, rows, cols, ld, eps);
}

int bwpp_cuda_layernorm_fwd_f32(BwppCudaCtx *ctx, const float *x, float *y,
                                const float *gamma, const float *beta,
                                uint32_t rows, uint32_t cols, uint32_t ld,
                                float eps) {
  return norm_fwd<true>(ctx, x, y, gamma, beta, rows, cols, ld, eps);
}

int bwpp_cuda_rmsnorm_bwd_f32(BwppCudaCtx *ctx, const float *x,
                              const float *gamma, const float *dy, float *dx,
                              float *dgamma, float *dbeta, uint32_t rows,
                              uint32_t cols, uint32_t ld, float eps) {
  return norm_bwd<false>(ctx, x, gamma, dy, dx, dgamma, dbeta, rows, cols, ld,
                         eps, nullptr);
}

int bwpp_cuda_layernorm_bwd_f32(BwppCudaCtx *ctx, const float *x,
                                const float *gamma, const float *dy, float *dx,
                                float *dgamma, float *dbeta, uint32_t rows,
                                uint32_t cols, uint32_t ld, float eps) {
  return norm_bwd<true>(ctx, x, gamma, dy, dx, dgamma, dbeta, rows, cols, ld,
                        eps, nullptr);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// RMSNorm backward without any allocation
// ---------------------------------------------------------------------------
// For callers that cannot allocate device memory themselves: code embedded in
// a host framework that owns the whole device-memory budget through its own
// pool and forbids allocations outside it, or latency-critical loops where a
// cudaMalloc / cudaFree (which can synchronize the device) is not acceptable.
// The dgamma / dbeta partials of this variant live in the fixed array below
// instead of a context workspace; it needs no BwppCudaCtx (creating one
// allocates).  Limits and sharing rules are stated at the declaration in
// include/bwpp_cuda.h.

namespace {

constexpr size_t kNoAllocScratchFloats = (size_t)1 << 20;  // 4 MiB

// Lives in the module of this file on every GPU that loads it, until exit.
// Host code must not pass this name to a kernel (on the host it is only a
// stand-in symbol); the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) float g_norm_bwd_scratch[kNoAllocScratchFloats];

// Per-device cache of the array's device address, keyed on the CUDA context
// that was current when it was looked up: a cudaDeviceReset (or anything else
// that recreates the primary context) reloads the module at a new address, so
// a changed context redoes the look-up instead of using a stale pointer.
typedef int (*cu_ctx_get_current_fn)(void **);

struct NoAllocDev {
  void *cu_ctx;
  float *scratch;
  int sms;
};

NoAllocDev g_noalloc[64];
pthread_mutex_t g_noalloc_mu = PTHREAD_MUTEX_INITIALIZER;
cu_ctx_get_current_fn g_ctx_get_current = nullptr;

void *current_cu_ctx() {
  cu_ctx_get_current_fn f = __atomic_load_n(&g_ctx_get_current, __ATOMIC_ACQUIRE);
  if (!f) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      cudaGetLastError();
      return nullptr;
    }
    f = (cu_ctx_get_current_fn)fn;
    __atomic_store_n(&g_ctx_get_current, f, __ATOMIC_RELEASE);
  }
  void *c = nullptr;
  return f(&c) == 0 ? c : nullptr;
}

// With device `dev` current: the array's address and the SM count, looked up
// again whenever the current context is not the one cached.
int noalloc_setup(int dev, float **scratch, int *sms) {
  if (dev < 0 || dev >= 64) return BWPP_CUDA_ERR_ARG;
  // cudaGetSymbolAddress makes the primary context current if none is yet
  float *p = nullptr;
  void *cc = current_cu_ctx();
  pthread_mutex_lock(&g_noalloc_mu);
  NoAllocDev &d = g_noalloc[dev];
  if (cc && d.cu_ctx == cc && d.scratch) {
    *scratch = d.scratch;
    *sms = d.sms;
    pthread_mutex_unlock(&g_noalloc_mu);
    return BWPP_CUDA_OK;
  }
  int n = 0;
  if (cudaGetSymbolAddress((void **)&p, g_norm_bwd_scratch) != cudaSuccess || !p ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    pthread_mutex_unlock(&g_noalloc_mu);
    return BWPP_CUDA_ERR_CUDA;
  }
  d.cu_ctx = cc ? cc : current_cu_ctx();
  d.scratch = p;
  d.sms = n;
  *scratch = p;
  *sms = n;
  pthread_mutex_unlock(&g_noalloc_mu);
  return BWPP_CUDA_OK;
}

}  // namespace

extern "C" int bwpp_cuda_rmsnorm_bwd_f32_noalloc(
    const float *x, const float *gamma, const float *dy, float *dx, float *dgamma,
    float *dbeta, uint32_t rows, uint32_t cols, uint32_t ld, float eps, void *stream) {
  if (!x || !dy || !dx || ld < cols) return BWPP_CUDA_ERR_ARG;
  if (cols == 0) return BWPP_CUDA_OK;
  const bool partials = dgamma || dbeta;
  // One CTA needs 2 * cols floats of partials: wider rows are rejected.
  if (partials && 2 * (size_t)cols > kNoAllocScratchFloats) return BWPP_CUDA_ERR_ARG;
  // An error left pending by earlier work of the caller is not this call's:
  // leave it in place for the caller and launch nothing.
  if (cudaPeekAtLastError() != cudaSuccess) return BWPP_CUDA_ERR_CUDA;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return BWPP_CUDA_ERR_CUDA;
  }
  float *scratch = nullptr;
  int sms = 0;
  int rc = noalloc_setup(dev, &scratch, &sms);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  if (rows == 0) {
    // dgamma = dbeta = 0 (sums over no rows) with one small kernel each; the
    // kernel skips a NULL output
    if (partials) {
      launch_column_sums(s, scratch, dgamma, scratch, dbeta, 0, cols);
    }
    return cudaGetLastError() == cudaSuccess ? BWPP_CUDA_OK : BWPP_CUDA_ERR_CUDA;
  }
  uint32_t grid = (uint32_t)sms * 4;
  if (rows < grid) grid = rows;
  float *pg = nullptr, *pb = nullptr;
  if (partials) {
    const size_t fit = kNoAllocScratchFloats / (2 * (size_t)cols);  // CTAs whose partials fit
    if (grid > fit) grid = (uint32_t)fit;
    // Each CTA overwrites its whole partial row before it is read, so nothing
    // left over from an earlier call leaks into this one.
    pg = scratch;
    pb = pg + (size_t)grid * cols;
  }
  const bool v4 = cols % 4 == 0 && ld % 4 == 0 && aligned16(x) && aligned16(dy) &&
                  aligned16(dx) && aligned16(gamma);
  const uint32_t nv = v4 ? cols / 4 : cols;
  int mv = pick_maxv(nv, kMaxVecBwd);
  const size_t acc_bytes = pg ? sizeof(float) * 2 * (size_t)cols : 0;
  if (acc_bytes > 48 * 1024) mv = 0;
#define BWPP_NA_BWD(MV, V4)                                                     \
  norm_bwd_kernel<MV, V4, false><<<grid, kThreads, acc_bytes, s>>>(             \
      x, gamma, dy, dx, pg, pb, rows, cols, ld, eps, nullptr, nullptr)
  if (mv == 0) {
    norm_bwd_looped_kernel<false><<<grid, kThreads, 0, s>>>(x, gamma, dy, dx, pg, pb, rows,
                                                            cols, ld, eps);
  } else if (v4) {
    switch (mv) {
      case 1: BWPP_NA_BWD(1, true); break;
      case 2: BWPP_NA_BWD(2, true); break;
      case 4: BWPP_NA_BWD(4, true); break;
      default: BWPP_NA_BWD(8, true); break;
    }
  } else {
    switch (mv) {
      case 1: BWPP_NA_BWD(1, false); break;
      case 2: BWPP_NA_BWD(2, false); break;
      case 4: BWPP_NA_BWD(4, false); break;
      default: BWPP_NA_BWD(8, false); break;
    }
  }
#undef BWPP_NA_BWD
  if (pg) launch_column_sums(s, pg, dgamma, pb, dbeta, grid, cols);
  return cudaGetLastError() == cudaSuccess ? BWPP_CUDA_OK : BWPP_CUDA_ERR_CUDA;
}
