// Drop-in mirrors of the reference's runtime/cpu and runtime/metal entry
// points on top of the ctx API.
//
// CPU mirrors (runtime/cpu/bwpp_cpu_ref.h:6-58): same argument lists, void,
// synchronous.  Each buffer may be host or device memory: device buffers are
// used in place, host buffers are staged through the calling thread's
// per-device context scratch.  fp32 matmul / attention operands are rounded
// to bf16 on the device before the tensor-core kernels run.  Like the
// reference, NULL required buffers make a call a silent no-op.
//
// Metal mirrors (runtime/metal/dispatch_stub.h:42-74): same param structs; a
// call only runs when `source` carries the kernel's bwpp.meta tag, as in
// runtime/metal/dispatch_stub.m:74-79.
#include <string.h>

#include "bwpp_cuda_internal.cuh"

int bwpp_gemm_launch(BwppCudaCtx *ctx, const uint16_t *a, const uint16_t *b,
                     float *c, uint32_t M, uint32_t N, uint32_t K, uint32_t lda,
                     uint32_t ldb, uint32_t ldc, const float *bias,
                     int apply_silu, int apply_bias, int force_simt);
int bwpp_cast_launch(BwppCudaCtx *ctx, const float *src, uint16_t *dst,
                     uint32_t rows, uint32_t cols, uint32_t ld_src,
                     uint32_t ld_dst);
int bwpp_comm_nranks(const BwppCudaComm *c);
int bwpp_comm_rank(const BwppCudaComm *c);
int bwpp_comm_device(const BwppCudaComm *c);
int bwpp_comm_allgather_bytes(BwppCudaComm *c, void *buf, size_t bytes, cudaStream_t stream);
int bwpp_attention_launch(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                          const uint16_t *v, void *o, uint32_t BH, uint32_t Sq,
                          uint32_t Skv, uint32_t Kd, uint32_t Dv, uint64_t q_bh,
                          uint64_t k_bh, uint64_t v_bh, uint64_t o_bh,
                          uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo,
                          float scale, int causal, int f16);

namespace {

thread_local BwppCudaCtx *tl_ctx[64];
thread_local int tl_status = BWPP_CUDA_OK;

BwppCudaCtx *mirror_ctx() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return nullptr;
  }
  if (!tl_ctx[dev] && bwpp_cuda_ctx_create(&tl_ctx[dev], dev, nullptr) != BWPP_CUDA_OK)
    tl_ctx[dev] = nullptr;
  return tl_ctx[dev];
}

bool is_device_ptr(const void *p) {
  if (!p) return false;
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

inline uint32_t round_up(uint32_t v, uint32_t m) { return (v + m - 1) / m * m; }

// Carves 256-byte-aligned pieces out of one workspace request.
struct Carver {
  size_t total = 0;
  size_t take(size_t bytes) {
    size_t off = total;
    total += (bytes + 255) & ~(size_t)255;
    return off;
  }
};

// A fp32 matrix view (rows x cols, leading dim ld) made device-resident:
// device buffers are used as they are, host buffers copied densely.
struct DevF32 {
  const float *src;
  uint32_t rows, cols, ld;
  bool dev;
  size_t off;
  const float *ptr;
  uint32_t dld;
};

void plan_f32(Carver &cv, DevF32 &m, const float *src, uint32_t rows,
              uint32_t cols, uint32_t ld) {
  m.src = src;
  m.rows = rows;
  m.cols = cols;
  m.ld = ld;
  m.dev = is_device_ptr(src);
  m.off = m.dev ? 0 : cv.take(sizeof(float) * (size_t)rows * cols);
  m.ptr = m.dev ? src : nullptr;
  m.dld = m.dev ? ld : cols;
}

int upload_f32(BwppCudaCtx *ctx, uint8_t *ws, DevF32 &m) {
  if (m.dev || !m.src) return BWPP_CUDA_OK;
  float *d = reinterpret_cast<float *>(ws + m.off);
  m.ptr = d;
  if ((size_t)m.rows * m.cols == 0) return BWPP_CUDA_OK;
  return bwpp_check_cuda(ctx,
                         cudaMemcpy2DAsync(d, sizeof(float) * m.cols, m.src,
                                           sizeof(float) * m.ld,
                                           sizeof(float) * m.cols, m.rows,
                                           cudaMemcpyHostToDevice, ctx->stream),
                         "mirror upload");
}

// Output view: written in place when it is device memory with a usable
// layout, else into dense scratch and copied back with the caller's ld.
struct OutF32 {
  float *dst;
  uint32_t rows, cols, ld;
  bool direct;
  size_t off;
  float *ptr;
  uint32_t dld;
};

void plan_out(Carver &cv, OutF32 &m, float *dst, uint32_t rows, uint32_t cols,
              uint32_t ld, uint32_t need_ld_mult) {
  m.dst = dst;
  m.rows = rows;
  m.cols = cols;
  m.ld = ld;
  m.direct = is_device_ptr(dst) && ld % need_ld_mult == 0 &&
             (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
  m.dld = m.direct ? ld : round_up(cols ? cols : 1, need_ld_mult);
  m.off = m.direct ? 0 : cv.take(sizeof(float) * (size_t)rows * m.dld);
  m.ptr = m.direct ? dst : nullptr;
}

void bind_out(uint8_t *ws, OutF32 &m) {
  if (!m.direct) m.ptr = reinterpret_cast<float *>(ws + m.off);
}

int download(BwppCudaCtx *ctx, OutF32 &m) {
  if (m.direct || (size_t)m.rows * m.cols == 0) return BWPP_CUDA_OK;
  return bwpp_check_cuda(ctx,
                         cudaMemcpy2DAsync(m.dst, sizeof(float) * m.ld, m.ptr,
                                           sizeof(float) * m.dld,
                                           sizeof(float) * m.cols, m.rows,
                                           cudaMemcpyDefault, ctx->stream),
                         "mirror download");
}

int finish(BwppCudaCtx *ctx, int rc) {
  if (rc == BWPP_CUDA_OK) rc = bwpp_cuda_sync(ctx);
  else bwpp_cuda_sync(ctx);
  tl_status = rc;
  return rc;
}

bool has_tag(const char *src, const char *tag) {
  return src && tag && strstr(src, tag) != nullptr;
}

void parse_epilogue(const char *src, int *ep_add, int *ep_silu) {
  // Same vocabulary as runtime/cpu/test_metal_parity.c:48-76.
  *ep_add = has_tag(src, "#define BWPP_EPILOGUE_ADD 1");
  *ep_silu = has_tag(src, "#define BWPP_EPILOGUE_SILU 1");
  if (*ep_add || *ep_silu) return;
  const char *p = src ? strstr(src, "bwpp.meta: epilogue=") : nullptr;
  if (!p) return;
  p += strlen("bwpp.meta: epilogue=");
  if (strncmp(p, "add_silu", 8) == 0) {
    *ep_add = 1;
    *ep_silu = 1;
  } else if (strncmp(p, "add", 3) == 0) {
    *ep_add = 1;
  } else if (strncmp(p, "silu", 4) == 0) {
    *ep_silu = 1;
  }
}

int bwpp_cuda_last_status_impl() { return tl_status; }

// Row-wise ops (softmax, rmsnorm) read x and write y with one leading dim.
// Device x and y that share ld run in place; otherwise both go through dense
// scratch (ld = cols).
struct RowOp {
  const float *x;
  float *y;
  uint32_t ld;
  bool staged;
  size_t off_x, off_y;
};

void plan_rowop(Carver &cv, RowOp &r, const float *x, float *y, uint32_t rows,
                uint32_t cols, uint32_t ld) {
  r.staged = !(is_device_ptr(x) && is_device_ptr(y));
  r.x = x;
  r.y = y;
  r.ld = r.staged ? cols : ld;
  r.off_x = r.staged ? cv.take(sizeof(float) * (size_t)rows * cols) : 0;
  r.off_y = r.staged ? cv.take(sizeof(float) * (size_t)rows * cols) : 0;
}

int rowop_upload(BwppCudaCtx *ctx, uint8_t *ws, RowOp &r, const float *x,
                 uint32_t rows, uint32_t cols, uint32_t ld) {
  if (!r.staged) return BWPP_CUDA_OK;
  float *dx = reinterpret_cast<float *>(ws + r.off_x);
  r.x = dx;
  r.y = reinterpret_cast<float *>(ws + r.off_y);
  if ((size_t)rows * cols == 0) return BWPP_CUDA_OK;
  return bwpp_check_cuda(ctx,
                         cudaMemcpy2DAsync(dx, sizeof(float) * cols, x, sizeof(float) * ld,
                                           sizeof(float) * cols, rows, cudaMemcpyDefault,
                                           ctx->stream),
                         "row op upload");
}

int rowop_download(BwppCudaCtx *ctx, RowOp &r, float *y, uint32_t rows,
                   uint32_t cols, uint32_t ld) {
  if (!r.staged || (size_t)rows * cols == 0) return BWPP_CUDA_OK;
  return bwpp_check_cuda(ctx,
                         cudaMemcpy2DAsync(y, sizeof(float) * ld, r.y, sizeof(float) * cols,
                                           sizeof(float) * cols, rows, cudaMemcpyDefault,
                                           ctx->stream),
                         "row op download");
}

// ---------------------------------------------------------------------------
// Host-operand matmul, pipelined.  When A, B and C all live in host memory the
// call is bound by the PCIe copies (about 0.3 GB in and 0.36 GB out at the
// 8192x4096x11008 config against well under a millisecond of tensor-core
// work).  A is cut into row chunks and B into column chunks.  Step k uploads
// A chunk k and B chunk k on an upload stream; the ctx stream casts them to
// bf16 and runs the GEMMs of the L-shaped region that just became computable
// (row block k over column chunks 0..k, column block k over row chunks
// 0..k-1); a download stream sends each finished region back with a strided
// 2-D copy.  Uploads, math and downloads of different steps overlap, and the
// two copy directions run concurrently, so the call approaches
// max(bytes in, bytes out) / PCIe bandwidth instead of their sum.

constexpr int kMaxChunks = 8;

struct CopyLanes {
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t uploaded[kMaxChunks] = {}, computed[kMaxChunks] = {};
  cudaEvent_t drained = nullptr;
  bool ready = false;
};

// Copy streams and events of the calling thread's mirror context, one set per
// device, created on first use and kept for the life of the thread.
thread_local CopyLanes tl_lanes[64];

int lanes_for(BwppCudaCtx *ctx, CopyLanes **out) {
  CopyLanes &l = tl_lanes[ctx->device];
  if (!l.ready) {
    int rc = bwpp_check_cuda(ctx, cudaStreamCreateWithFlags(&l.in, cudaStreamNonBlocking),
                             "copy stream");
    if (!rc)
      rc = bwpp_check_cuda(ctx, cudaStreamCreateWithFlags(&l.out, cudaStreamNonBlocking),
                           "copy stream");
    for (int i = 0; !rc && i < kMaxChunks; ++i) {
      rc = bwpp_check_cuda(ctx, cudaEventCreateWithFlags(&l.uploaded[i], cudaEventDisableTiming),
                           "copy event");
      if (!rc)
        rc = bwpp_check_cuda(ctx,
                             cudaEventCreateWithFlags(&l.computed[i], cudaEventDisableTiming),
                             "copy event");
    }
    if (!rc)
      rc = bwpp_check_cuda(ctx, cudaEventCreateWithFlags(&l.drained, cudaEventDisableTiming),
                           "copy event");
    if (rc) return rc;  // partially created handles are kept for the next try
    l.ready = true;
  }
  *out = &l;
  return BWPP_CUDA_OK;
}

// Chunk count and chunk size for `n` items: about `unit` items per chunk, at
// most kMaxChunks chunks, chunk sizes a multiple of `mult`.
void chunking(uint32_t n, uint32_t unit, uint32_t mult, uint32_t *count, uint32_t *size) {
  uint32_t c = n / unit;
  if (c < 1) c = 1;
  if (c > (uint32_t)kMaxChunks) c = kMaxChunks;
  uint32_t s = round_up((n + c - 1) / c, mult);
  *size = s;
  *count = (n + s - 1) / s;
}

// Returns 1 when the call is not a candidate (then nothing was done),
// otherwise the status of the pipelined run.
int matmul_f32_host_pipelined(BwppCudaCtx *ctx, const float *a, const float *b, float *c,
                              uint32_t M, uint32_t N, uint32_t K, uint32_t lda,
                              uint32_t ldb, uint32_t ldc, const float *bias,
                              int apply_silu, bool use_bias, bool *ran) {
  *ran = false;
  if (M == 0 || N == 0 || K == 0) return BWPP_CUDA_OK;
  if (is_device_ptr(a) || is_device_ptr(b) || is_device_ptr(c)) return BWPP_CUDA_OK;
  if (lda < K || ldb < N || ldc < N) return BWPP_CUDA_OK;  // left to the plain path
  uint32_t nr, mr, nc, cs;
  chunking(M, 1024, 128, &nr, &mr);
  chunking(N, 1024, 16, &nc, &cs);
  if (nr * nc < 2) return BWPP_CUDA_OK;  // too small to overlap anything
  CopyLanes *l = nullptr;
  *ran = true;
  int rc = lanes_for(ctx, &l);
  if (rc) return rc;

  const uint32_t K8 = round_up(K, 8), N8 = round_up(N, 8), ldC = round_up(N, 4);
  Carver cv;
  const size_t off_a = cv.take(sizeof(float) * (size_t)M * K);
  const size_t off_b = cv.take(sizeof(float) * (size_t)K * N);
  const size_t off_bias = cv.take(use_bias ? sizeof(float) * (size_t)N : 0);
  const size_t off_a16 = cv.take(2 * (size_t)M * K8);
  const size_t off_b16 = cv.take(2 * (size_t)K * N8);
  const size_t off_c = cv.take(sizeof(float) * (size_t)M * ldC);
  uint8_t *ws = (uint8_t *)bwpp_ctx_workspace(ctx, cv.total);
  if (!ws) return BWPP_CUDA_ERR_NOMEM;
  float *dA = reinterpret_cast<float *>(ws + off_a);
  float *dB = reinterpret_cast<float *>(ws + off_b);
  float *dBias = use_bias ? reinterpret_cast<float *>(ws + off_bias) : nullptr;
  uint16_t *a16 = reinterpret_cast<uint16_t *>(ws + off_a16);
  uint16_t *b16 = reinterpret_cast<uint16_t *>(ws + off_b16);
  float *dC = reinterpret_cast<float *>(ws + off_c);

  // The copy streams start after whatever the ctx stream already holds.
  rc = bwpp_check_cuda(ctx, cudaEventRecord(l->drained, ctx->stream), "event");
  if (!rc) rc = bwpp_check_cuda(ctx, cudaStreamWaitEvent(l->in, l->drained, 0), "wait");
  if (!rc) rc = bwpp_check_cuda(ctx, cudaStreamWaitEvent(l->out, l->drained, 0), "wait");
  if (!rc && use_bias)
    rc = bwpp_check_cuda(ctx, cudaMemcpyAsync(dBias, bias, sizeof(float) * N,
                                              cudaMemcpyHostToDevice, l->in),
                         "bias upload");

  const uint32_t steps = nr > nc ? nr : nc;
  for (uint32_t k = 0; k < steps && !rc; ++k) {
    const uint32_t r0 = k * mr, rows = k < nr ? (M - r0 < mr ? M - r0 : mr) : 0;
    const uint32_t c0 = k * cs, cols = k < nc ? (N - c0 < cs ? N - c0 : cs) : 0;
    if (rows)
      rc = bwpp_check_cuda(ctx,
                           cudaMemcpy2DAsync(dA + (size_t)r0 * K, sizeof(float) * K,
                                             a + (size_t)r0 * lda, sizeof(float) * lda,
                                             sizeof(float) * K, rows, cudaMemcpyHostToDevice,
                                             l->in),
                           "A chunk upload");
    if (!rc && cols)
      rc = bwpp_check_cuda(ctx,
                           cudaMemcpy2DAsync(dB + c0, sizeof(float) * N, b + c0,
                                             sizeof(float) * ldb, sizeof(float) * cols, K,
                                             cudaMemcpyHostToDevice, l->in),
                           "B chunk upload");
    if (!rc) rc = bwpp_check_cuda(ctx, cudaEventRecord(l->uploaded[k], l->in), "event");
    if (!rc) rc = bwpp_check_cuda(ctx, cudaStreamWaitEvent(ctx->stream, l->uploaded[k], 0), "wait");
    if (!rc && rows)
      rc = bwpp_cast_launch(ctx, dA + (size_t)r0 * K, a16 + (size_t)r0 * K8, rows, K, K, K8);
    if (!rc && cols) rc = bwpp_cast_launch(ctx, dB + c0, b16 + c0, K, cols, N, N8);
    // row block k over the column chunks that have arrived (0..k)
    const uint32_t ncov = (k + 1 < nc ? (k + 1) * cs : N);
    if (!rc && rows)
      rc = bwpp_gemm_launch(ctx, a16 + (size_t)r0 * K8, b16, dC + (size_t)r0 * ldC, rows, ncov,
                            K, K8, N8, ldC, dBias, apply_silu, use_bias, 0);
    // column block k over the row chunks that arrived before this step
    const uint32_t rcov = (k < nr ? k * mr : M);
    if (!rc && cols && rcov)
      rc = bwpp_gemm_launch(ctx, a16, b16 + c0, dC + c0, rcov, cols, K, K8, N8, ldC,
                            use_bias ? dBias + c0 : nullptr, apply_silu, use_bias, 0);
    if (!rc) rc = bwpp_check_cuda(ctx, cudaEventRecord(l->computed[k], ctx->stream), "event");
    if (!rc) rc = bwpp_check_cuda(ctx, cudaStreamWaitEvent(l->out, l->computed[k], 0), "wait");
    if (!rc && rows)
      rc = bwpp_check_cuda(ctx,
                           cudaMemcpy2DAsync(c + (size_t)r0 * ldc, sizeof(float) * ldc,
                                             dC + (size_t)r0 * ldC, sizeof(float) * ldC,
                                             sizeof(float) * ncov, rows,
                                             cudaMemcpyDeviceToHost, l->out),
                           "C row block download");
    if (!rc && cols && rcov)
      rc = bwpp_check_cuda(ctx,
                           cudaMemcpy2DAsync(c + c0, sizeof(float) * ldc, dC + c0,
                                             sizeof(float) * ldC, sizeof(float) * cols, rcov,
                                             cudaMemcpyDeviceToHost, l->out),
                           "C column block download");
  }
  // The ctx stream ends after the last download, so the caller's sync covers
  // all three streams.  On an error part way, the streams are drained before
  // returning so no copy still targets the workspace.
  cudaError_t e = cudaEventRecord(l->drained, l->out);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->stream, l->drained, 0);
  if (rc) {
    cudaStreamSynchronize(l->in);
    cudaStreamSynchronize(l->out);
    return rc;
  }
  return bwpp_check_cuda(ctx, e, "copy stream join");
}

// ---------------------------------------------------------------------------
// The same host-operand matmul across the ranks of a communicator, each rank
// holding its own rows of A and C and the whole B in host memory.  B is the
// large shared operand (4096 x 11008 fp32 = 180 MB at the benchmark config),
// so no rank copies all of it over PCIe: rank r uploads its 1/n of B's K rows,
// rounds them to bf16 into its slot of the bf16 B, and one in-place NCCL
// all-gather over NVLink assembles the whole bf16 B on every GPU.  Meanwhile
// A's row chunks go up on the upload stream; each chunk's GEMM (on the ctx
// stream, after the all-gather) sends its C rows back on the download stream.
int matmul_f32_dist(BwppCudaCtx *ctx, BwppCudaComm *comm, const float *a, const float *b,
                    float *c, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb,
                    uint32_t ldc, const float *bias, int apply_silu, bool use_bias) {
  if (N == 0 || K == 0) return BWPP_CUDA_OK;
  if (lda < K || ldb < N || ldc < N) return BWPP_CUDA_ERR_ARG;
  if (bwpp_comm_device(comm) != ctx->device) return BWPP_CUDA_ERR_ARG;
  CopyLanes *l = nullptr;
  int rc = lanes_for(ctx, &l);
  if (rc) return rc;
  const uint32_t n = (uint32_t)bwpp_comm_nranks(comm), r = (uint32_t)bwpp_comm_rank(comm);
  const uint32_t K8 = round_up(K, 8), N8 = round_up(N, 8), ldC = round_up(N, 4);
  const uint32_t kc = (K + n - 1) / n;                       // B rows per rank
  const uint32_t k0 = r * kc < K ? r * kc : K, k1 = k0 + kc < K ? k0 + kc : K;
  const size_t slot = (size_t)kc * N8 * 2;                   // bytes of one rank's bf16 rows
  uint32_t nr = 1, mr = M ? M : 1;
  if (M) chunking(M, 256, 128, &nr, &mr);
  Carver cv;
  const size_t off_b = cv.take(sizeof(float) * (size_t)kc * N);
  const size_t off_b16 = cv.take(slot * n);
  const size_t off_bias = cv.take(use_bias ? sizeof(float) * (size_t)N : 0);
  const size_t off_a = cv.take(sizeof(float) * (size_t)M * K);
  const size_t off_a16 = cv.take(2 * (size_t)M * K8);
  const size_t off_c = cv.take(sizeof(float) * (size_t)M * ldC);
  uint8_t *ws = (uint8_t *)bwpp_ctx_workspace(ctx, cv.total);
  if (!ws) return BWPP_CUDA_ERR_NOMEM;
  float *dB = reinterpret_cast<float *>(ws + off_b);
  uint16_t *b16 = reinterpret_cast<uint16_t *>(ws + off_b16);
  float *dBias = use_bias ? reinterpret_cast<float *>(ws + off_bias) : nullptr;
  float *dA = reinterpret_cast<float *>(ws + off_a);
  uint16_t *a16 = reinterpret_cast<uint16_t *>(ws + off_a16);
  float *dC = reinterpret_cast<float *>(ws + off_c);
  // this rank's K rows of B first (upload, then bf16 into its slot), then
  // the all-gather; the copy streams start after the ctx stream's earlier work
  rc = bwpp_check_cuda(ctx, cudaEventRecord(l->drained, ctx->stream), "event");
  if (!rc) rc = bwpp_check_cuda(ctx, cudaStreamWaitEvent(l->in, l->drained, 0), "wait");
  if (!rc) rc = bwpp_check_cuda(ctx, cudaStreamWaitEvent(l->out, l->drained, 0), "wait");
  if (!rc && k1 > k0)
    rc = bwpp_check_cuda(ctx,
                         cudaMemcpy2DAsync(dB, sizeof(float) * N, b + (size_t)k0 * ldb,
                                           sizeof(float) * ldb, sizeof(float) * N, k1 - k0,
                                           cudaMemcpyHostToDevice, l->in),
                         "B rows upload");
  if (!rc && use_bias)
    rc = bwpp_check_cuda(ctx, cudaMemcpyAsync(dBias, bias, sizeof(float) * N,
                                              cudaMemcpyHostToDevice, l->in),
                         "bias upload");
  if (!rc) rc = bwpp_check_cuda(ctx, cudaEventRecord(l->uploaded[0], l->in), "event");
  if (!rc) rc = bwpp_check_cuda(ctx, cudaStreamWaitEvent(ctx->stream, l->uploaded[0], 0), "wait");
  if (!rc && k1 > k0)
    rc = bwpp_cast_launch(ctx, dB, b16 + (size_t)r * kc * N8, k1 - k0, N, N, N8);
  if (!rc) rc = bwpp_comm_allgather_bytes(comm, b16, slot, ctx->stream);
  // A's row chunks: upload, cast, GEMM over all of N, download
  for (uint32_t k = 0; k < nr && M && !rc; ++k) {
    const uint32_t r0 = k * mr, rows = M - r0 < mr ? M - r0 : mr;
    const int ev = 1 + (int)(k % (kMaxChunks - 1));
    rc = bwpp_check_cuda(ctx,
                         cudaMemcpy2DAsync(dA + (size_t)r0 * K, sizeof(float) * K,
                                           a + (size_t)r0 * lda, sizeof(float) * lda,
                                           sizeof(float) * K, rows, cudaMemcpyHostToDevice, l->in),
                         "A chunk upload");
    if (!rc) rc = bwpp_check_cuda(ctx, cudaEventRecord(l->uploaded[ev], l->in), "event");
    if (!rc) rc = bwpp_check_cuda(ctx, cudaStreamWaitEvent(ctx->stream, l->uploaded[ev], 0), "wait");
    if (!rc) rc = bwpp_cast_launch(ctx, dA + (size_t)r0 * K, a16 + (size_t)r0 * K8, rows, K, K, K8);
    if (!rc)
      rc = bwpp_gemm_launch(ctx, a16 + (size_t)r0 * K8, b16, dC + (size_t)r0 * ldC, rows, N, K,
                            K8, N8, ldC, dBias, apply_silu, use_bias, 0);
    if (!rc) rc = bwpp_check_cuda(ctx, cudaEventRecord(l->computed[ev], ctx->stream), "event");
    if (!rc) rc = bwpp_check_cuda(ctx, cudaStreamWaitEvent(l->out, l->computed[ev], 0), "wait");
    if (!rc)
      rc = bwpp_check_cuda(ctx,
                           cudaMemcpy2DAsync(c + (size_t)r0 * ldc, sizeof(float) * ldc,
                                             dC + (size_t)r0 * ldC, sizeof(float) * ldC,
                                             sizeof(float) * N, rows, cudaMemcpyDeviceToHost,
                                             l->out),
                           "C chunk download");
  }
  cudaError_t e = cudaEventRecord(l->drained, l->out);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->stream, l->drained, 0);
  if (rc) {
    cudaStreamSynchronize(l->in);
    cudaStreamSynchronize(l->out);
    return rc;
  }
  return bwpp_check_cuda(ctx, e, "copy stream join");
}

}  // namespace

extern "C" {

int bwpp_cuda_matmul_f32_dist(BwppCudaComm *comm, const float *a, const float *b, float *c,
                              uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb,
                              uint32_t ldc, const float *bias, int apply_silu, int apply_bias) {
  tl_status = BWPP_CUDA_OK;
  if (!comm || !b || (M && (!a || !c))) return tl_status = BWPP_CUDA_ERR_ARG;
  BwppCudaCtx *ctx = mirror_ctx();
  if (!ctx) return tl_status = BWPP_CUDA_ERR_CUDA;
  if (is_device_ptr(a) || is_device_ptr(b) || is_device_ptr(c)) return tl_status = BWPP_CUDA_ERR_ARG;
  const int rc = matmul_f32_dist(ctx, comm, a, b, c, M, N, K, lda, ldb, ldc, bias, apply_silu,
                                 apply_bias && bias);
  return finish(ctx, rc);
}

int bwpp_cuda_last_status(void) { return bwpp_cuda_last_status_impl(); }

void bwpp_cuda_matmul_f32(const float *a, const float *b, float *c, uint32_t M,
                          uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb,
                          uint32_t ldc, const float *bias, int apply_silu,
                          int apply_bias) {
  tl_status = BWPP_CUDA_OK;
  if (!a || !b || !c) return;
  BwppCudaCtx *ctx = mirror_ctx();
  if (!ctx) { tl_status = BWPP_CUDA_ERR_CUDA; return; }
  const bool use_bias = apply_bias && bias;
  bool pipelined = false;
  int prc = matmul_f32_host_pipelined(ctx, a, b, c, M, N, K, lda, ldb, ldc, bias, apply_silu,
                                      use_bias, &pipelined);
  if (pipelined) {
    finish(ctx, prc);
    return;
  }
  const uint32_t K8 = round_up(K ? K : 1, 8), N8 = round_up(N ? N : 1, 8);
  Carver cv;
  DevF32 da, db, dbias;
  plan_f32(cv, da, a, M, K, lda);
  plan_f32(cv, db, b, K, N, ldb);
  plan_f32(cv, dbias, use_bias ? bias : nullptr, 1, use_bias ? N : 0, N);
  const size_t off_a16 = cv.take(2 * (size_t)M * K8);
  const size_t off_b16 = cv.take(2 * (size_t)K * N8);
  OutF32 oc;
  plan_out(cv, oc, c, M, N, ldc, 4);
  uint8_t *ws = (uint8_t *)bwpp_ctx_workspace(ctx, cv.total);
  if (!ws) { tl_status = BWPP_CUDA_ERR_NOMEM; return; }
  bind_out(ws, oc);
  uint16_t *a16 = reinterpret_cast<uint16_t *>(ws + off_a16);
  uint16_t *b16 = reinterpret_cast<uint16_t *>(ws + off_b16);
  int rc = upload_f32(ctx, ws, da);
  if (!rc) rc = upload_f32(ctx, ws, db);
  if (!rc && use_bias) rc = upload_f32(ctx, ws, dbias);
  if (!rc) rc = bwpp_cast_launch(ctx, da.ptr, a16, M, K, da.dld, K8);
  if (!rc) rc = bwpp_cast_launch(ctx, db.ptr, b16, K, N, db.dld, N8);
  if (!rc)
    rc = bwpp_gemm_launch(ctx, a16, b16, oc.ptr, M, N, K, K8, N8, oc.dld,
                          use_bias ? dbias.ptr : nullptr, apply_silu, use_bias, 0);
  if (!rc) rc = download(ctx, oc);
  finish(ctx, rc);
}

void bwpp_cuda_softmax_f32(const float *x, float *y, uint32_t rows,
                           uint32_t cols, uint32_t ld) {
  tl_status = BWPP_CUDA_OK;
  if (!x || !y) return;
  BwppCudaCtx *ctx = mirror_ctx();
  if (!ctx) { tl_status = BWPP_CUDA_ERR_CUDA; return; }
  Carver cv;
  RowOp r;
  plan_rowop(cv, r, x, y, rows, cols, ld);
  uint8_t *ws = (uint8_t *)bwpp_ctx_workspace(ctx, cv.total);
  if (!ws) { tl_status = BWPP_CUDA_ERR_NOMEM; return; }
  int rc = rowop_upload(ctx, ws, r, x, rows, cols, ld);
  if (!rc) rc = bwpp_cuda_softmax_fwd_f32(ctx, r.x, r.y, rows, cols, r.ld);
  if (!rc) rc = rowop_download(ctx, r, y, rows, cols, ld);
  finish(ctx, rc);
}

void bwpp_cuda_rmsnorm_f32(const float *x, float *y, const float *gamma,
                           const float *beta, uint32_t rows, uint32_t cols,
                           uint32_t ld, float eps) {
  tl_status = BWPP_CUDA_OK;
  if (!x || !y) return;
  BwppCudaCtx *ctx = mirror_ctx();
  if (!ctx) { tl_status = BWPP_CUDA_ERR_CUDA; return; }
  Carver cv;
  RowOp r;
  plan_rowop(cv, r, x, y, rows, cols, ld);
  DevF32 dg, db;
  plan_f32(cv, dg, gamma, 1, gamma ? cols : 0, cols);
  plan_f32(cv, db, beta, 1, beta ? cols : 0, cols);
  uint8_t *ws = (uint8_t *)bwpp_ctx_workspace(ctx, cv.total);
  if (!ws) { tl_status = BWPP_CUDA_ERR_NOMEM; return; }
  int rc = rowop_upload(ctx, ws, r, x, rows, cols, ld);
  if (!rc && gamma) rc = upload_f32(ctx, ws, dg);
  if (!rc && beta) rc = upload_f32(ctx, ws, db);
  if (!rc)
    rc = bwpp_cuda_rmsnorm_fwd_f32(ctx, r.x, r.y, gamma ? dg.ptr : nullptr,
                                   beta ? db.ptr : nullptr, rows, cols, r.ld, eps);
  if (!rc) rc = rowop_download(ctx, r, y, rows, cols, ld);
  finish(ctx, rc);
}

void bwpp_cuda_attention_f32(const float *q, const float *k, const float *v,
                             float *o, uint32_t M, uint32_t N, uint32_t K,
                             uint32_t D, uint32_t ldq, uint32_t ldk,
                             uint32_t ldv, uint32_t ldo) {
  tl_status = BWPP_CUDA_OK;
  if (!q || !k || !v || !o) return;
  BwppCudaCtx *ctx = mirror_ctx();
  if (!ctx) { tl_status = BWPP_CUDA_ERR_CUDA; return; }
  Carver cv;
  DevF32 dq, dk, dv;
  plan_f32(cv, dq, q, M, K, ldq);
  plan_f32(cv, dk, k, N, K, ldk);
  plan_f32(cv, dv, v, N, D, ldv);
  const size_t oq = cv.take(2 * (size_t)M * K), ok_ = cv.take(2 * (size_t)N * K),
               ov = cv.take(2 * (size_t)N * D);
  OutF32 oo;
  plan_out(cv, oo, o, M, D, ldo, 1);
  uint8_t *ws = (uint8_t *)bwpp_ctx_workspace(ctx, cv.total);
  if (!ws) { tl_status = BWPP_CUDA_ERR_NOMEM; return; }
  bind_out(ws, oo);
  uint16_t *q16 = reinterpret_cast<uint16_t *>(ws + oq);
  uint16_t *k16 = reinterpret_cast<uint16_t *>(ws + ok_);
  uint16_t *v16 = reinterpret_cast<uint16_t *>(ws + ov);
  int rc = upload_f32(ctx, ws, dq);
  if (!rc) rc = upload_f32(ctx, ws, dk);
  if (!rc) rc = upload_f32(ctx, ws, dv);
  if (!rc) rc = bwpp_cast_launch(ctx, dq.ptr, q16, M, K, dq.dld, K);
  if (!rc) rc = bwpp_cast_launch(ctx, dk.ptr, k16, N, K, dk.dld, K);
  if (!rc) rc = bwpp_cast_launch(ctx, dv.ptr, v16, N, D, dv.dld, D);
  if (!rc)
    rc = bwpp_attention_launch(ctx, q16, k16, v16, oo.ptr, 1, M, N, K, D,
                               (uint64_t)M * K, (uint64_t)N * K, (uint64_t)N * D,
                               (uint64_t)M * oo.dld, K, K, D, oo.dld, 1.0f, 0, 0);
  if (!rc) rc = download(ctx, oo);
  finish(ctx, rc);
}

void bwpp_cuda_reduce_max_mask_f32(const float *x, float *mask, uint32_t rows,
                                   uint32_t cols, int axis) {
  tl_status = BWPP_CUDA_OK;
  if (!x || !mask) return;
  BwppCudaCtx *ctx = mirror_ctx();
  if (!ctx) { tl_status = BWPP_CUDA_ERR_CUDA; return; }
  Carver cv;
  DevF32 dx;
  plan_f32(cv, dx, x, rows, cols, cols);
  OutF32 om;
  plan_out(cv, om, mask, rows, cols, cols, 1);
  uint8_t *ws = (uint8_t *)bwpp_ctx_workspace(ctx, cv.total);
  if (!ws) { tl_status = BWPP_CUDA_ERR_NOMEM; return; }
  bind_out(ws, om);
  int rc = upload_f32(ctx, ws, dx);
  if (!rc) rc = bwpp_cuda_reduce_max_mask_ex(ctx, dx.ptr, om.ptr, rows, cols, axis);
  if (!rc) rc = download(ctx, om);
  finish(ctx, rc);
}

void bwpp_cuda_reduce_max_grad_f32(const float *mask, const float *dy,
                                   float *dx, uint32_t rows, uint32_t cols,
                                   int axis) {
  tl_status = BWPP_CUDA_OK;
  if (!mask || !dy || !dx) return;
  BwppCudaCtx *ctx = mirror_ctx();
  if (!ctx) { tl_status = BWPP_CUDA_ERR_CUDA; return; }
  Carver cv;
  DevF32 dm, dd;
  plan_f32(cv, dm, mask, rows, cols, cols);
  plan_f32(cv, dd, dy, 1, axis == 0 ? cols : rows, axis == 0 ? cols : rows);
  OutF32 od;
  plan_out(cv, od, dx, rows, cols, cols, 1);
  uint8_t *ws = (uint8_t *)bwpp_ctx_workspace(ctx, cv.total);
  if (!ws) { tl_status = BWPP_CUDA_ERR_NOMEM; return; }
  bind_out(ws, od);
  int rc = upload_f32(ctx, ws, dm);
  if (!rc) rc = upload_f32(ctx, ws, dd);
  if (!rc) rc = bwpp_cuda_reduce_max_grad_ex(ctx, dm.ptr, dd.ptr, od.ptr, rows, cols, axis);
  if (!rc) rc = download(ctx, od);
  finish(ctx, rc);
}

// ---- Metal dispatch mirrors ----------------------------------------------

int bwpp_cuda_dispatch_matmul(BwppCudaCtx *ctx, const uint16_t *a,
                              const uint16_t *b, float *c, const float *bias,
                              BwppCudaMatmulParams p, const char *source) {
  if (!ctx || !a || !b || !c || !source) return BWPP_CUDA_ERR_ARG;
  if (has_tag(source, "bwpp.meta: kernel=none") ||
      !has_tag(source, "bwpp.meta: kernel=matmul_f16"))
    return BWPP_CUDA_OK;
  int ep_add = 0, ep_silu = 0;
  parse_epilogue(source, &ep_add, &ep_silu);
  return bwpp_cuda_matmul_bf16(ctx, a, b, c, p.M, p.N, p.K, p.lda, p.ldb, p.ldc,
                               bias, ep_silu, ep_add);
}

int bwpp_cuda_dispatch_softmax(BwppCudaCtx *ctx, const float *x, float *y,
                               BwppCudaSoftmaxParams p, const char *source) {
  if (!ctx || !x || !y || !source) return BWPP_CUDA_ERR_ARG;
  if (!has_tag(source, "softmax_f16")) return BWPP_CUDA_OK;
  return bwpp_cuda_softmax_fwd_f32(ctx, x, y, p.rows, p.cols, p.ld);
}

int bwpp_cuda_dispatch_rmsnorm(BwppCudaCtx *ctx, const float *x,
                               const float *gamma, const float *beta, float *y,
                               BwppCudaRmsnormParams p, const char *source) {
  if (!ctx || !x || !y || !source) return BWPP_CUDA_ERR_ARG;
  if (!has_tag(source, "rmsnorm_f16")) return BWPP_CUDA_OK;
  // A missing gamma / beta acts as ones / zeros (dispatch_stub.m:225-243).
  return bwpp_cuda_rmsnorm_fwd_f32(ctx, x, y, gamma, beta, p.rows, p.cols, p.ld,
                                   p.eps);
}

int bwpp_cuda_dispatch_attention(BwppCudaCtx *ctx, const uint16_t *q,
                                 const uint16_t *k, const uint16_t *v, float *o,
                                 BwppCudaAttentionParams p,
                                 const char *source) {
  if (!ctx || !q || !k || !v || !o || !source) return BWPP_CUDA_ERR_ARG;
  if (!has_tag(source, "bwpp.meta: kernel=attention_f16")) return BWPP_CUDA_OK;
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  return bwpp_attention_launch(ctx, q, k, v, o, 1, p.M, p.N, p.K, p.D, 0, 0, 0, 0,
                               p.ldq, p.ldk, p.ldv, p.ldo, 1.0f, 0, 0);
}

}  // extern "C"
