// Context, status word, workspace, arena and TMA-descriptor plumbing.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include "bwpp_cuda_internal.cuh"

extern "C" {

const char *bwpp_cuda_status_string(int status) {
  switch (status) {
    case BWPP_CUDA_OK: return "ok";
    case BWPP_CUDA_ERR: return "error";
    case BWPP_CUDA_ERR_ARG: return "invalid argument";
    case BWPP_CUDA_ERR_CUDA: return "CUDA error";
    case BWPP_CUDA_ERR_TIMEOUT: return "device wait timed out";
    case BWPP_CUDA_ERR_NOMEM: return "out of device memory";
    case BWPP_CUDA_ERR_UNSUPPORTED: return "unsupported shape or option";
  }
  return "unknown status";
}

}  // extern "C"

int bwpp_set_error(BwppCudaCtx *ctx, int code, const char *fmt, ...) {
  if (ctx) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(ctx->last_error, sizeof(ctx->last_error), fmt, ap);
    va_end(ap);
  }
  return code;
}

int bwpp_check_cuda(BwppCudaCtx *ctx, cudaError_t err, const char *what) {
  if (err == cudaSuccess) return BWPP_CUDA_OK;
  return bwpp_set_error(ctx, err == cudaErrorMemoryAllocation
                                 ? BWPP_CUDA_ERR_NOMEM
                                 : BWPP_CUDA_ERR_CUDA,
                        "%s: %s", what, cudaGetErrorString(err));
}

int bwpp_ctx_enter(BwppCudaCtx *ctx) {
  if (!ctx) return BWPP_CUDA_ERR_ARG;
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != ctx->device)
    return bwpp_check_cuda(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  return BWPP_CUDA_OK;
}

void *bwpp_ctx_workspace(BwppCudaCtx *ctx, size_t bytes) {
  if (bytes == 0) bytes = 16;
  if (ctx->workspace && ctx->workspace_bytes >= bytes) return ctx->workspace;
  if (ctx->user_workspace) {
    bwpp_set_error(ctx, BWPP_CUDA_ERR_NOMEM,
                   "workspace too small: need %zu bytes, have %zu", bytes,
                   ctx->workspace_bytes);
    return NULL;
  }
  if (ctx->workspace) {
    // The old buffer may still be read by queued kernels on this stream.
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->workspace);
    ctx->workspace = NULL;
    ctx->workspace_bytes = 0;
  }
  size_t cap = (bytes + 0xFFFFF) & ~(size_t)0xFFFFF;  // round to 1 MiB
  if (bwpp_check_cuda(ctx, cudaMalloc(&ctx->workspace, cap), "workspace") !=
      BWPP_CUDA_OK) {
    ctx->workspace = NULL;
    return NULL;
  }
  ctx->workspace_bytes = cap;
  return ctx->workspace;
}

static bwpp_encode_tiled_fn g_encode = NULL;

bwpp_encode_tiled_fn bwpp_get_encode_tiled(void) {
  if (g_encode) return g_encode;
  void *fn = NULL;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn,
                              cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return NULL;
  g_encode = (bwpp_encode_tiled_fn)fn;
  return g_encode;
}

int bwpp_make_tmap_2d(BwppCudaCtx *ctx, CUtensorMap *map, const void *base,
                      CUtensorMapDataType dtype, uint64_t inner,
                      uint64_t outer, uint64_t pitch_bytes, uint32_t box_inner,
                      uint32_t box_outer, CUtensorMapSwizzle swz) {
  bwpp_encode_tiled_fn enc = bwpp_get_encode_tiled();
  if (!enc)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_CUDA,
                          "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void *>(base), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_CUDA,
                          "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu "
                          "pitch %llu box %u x %u",
                          (int)r, (unsigned long long)inner,
                          (unsigned long long)outer,
                          (unsigned long long)pitch_bytes, box_inner,
                          box_outer);
  return BWPP_CUDA_OK;
}

extern "C" {

int bwpp_cuda_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

int bwpp_cuda_ctx_create(BwppCudaCtx **out, int device, void *stream) {
  if (!out) return BWPP_CUDA_ERR_ARG;
  *out = NULL;
  int n = bwpp_cuda_device_count();
  if (device < 0 || device >= n) return BWPP_CUDA_ERR_ARG;
  BwppCudaCtx *ctx = (BwppCudaCtx *)calloc(1, sizeof(BwppCudaCtx));
  if (!ctx) return BWPP_CUDA_ERR;
  ctx->device = device;
  ctx->stream = (cudaStream_t)stream;
  int rc = bwpp_check_cuda(ctx, cudaSetDevice(device), "cudaSetDevice");
  if (rc == BWPP_CUDA_OK)
    rc = bwpp_check_cuda(
        ctx,
        cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount,
                               device),
        "cudaDeviceGetAttribute");
  if (rc == BWPP_CUDA_OK)
    rc = bwpp_check_cuda(ctx, cudaMalloc(&ctx->status_word, 4 * sizeof(int)),
                         "status word");
  if (rc == BWPP_CUDA_OK)
    rc = bwpp_check_cuda(ctx, cudaMemset(ctx->status_word, 0, 4 * sizeof(int)),
                         "status word");
  if (rc == BWPP_CUDA_OK) ctx->sched_counter = ctx->status_word + 1;
  if (rc != BWPP_CUDA_OK) {
    if (ctx->status_word) cudaFree(ctx->status_word);
    free(ctx);
    return rc;
  }
  *out = ctx;
  return BWPP_CUDA_OK;
}

int bwpp_cuda_ctx_destroy(BwppCudaCtx *ctx) {
  if (!ctx) return BWPP_CUDA_ERR_ARG;
  bwpp_ctx_enter(ctx);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->workspace && !ctx->user_workspace) cudaFree(ctx->workspace);
  if (ctx->gemm_partials) cudaFree(ctx->gemm_partials);
  if (ctx->status_word) cudaFree(ctx->status_word);
  free(ctx);
  return BWPP_CUDA_OK;
}

int bwpp_cuda_ctx_set_stream(BwppCudaCtx *ctx, void *stream) {
  if (!ctx) return BWPP_CUDA_ERR_ARG;
  ctx->stream = (cudaStream_t)stream;
  return BWPP_CUDA_OK;
}

int bwpp_cuda_ctx_set_workspace(BwppCudaCtx *ctx, void *device_ptr,
                                size_t bytes) {
  if (!ctx) return BWPP_CUDA_ERR_ARG;
  if (ctx->workspace && !ctx->user_workspace) {
    bwpp_ctx_enter(ctx);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->workspace);
  }
  ctx->workspace = device_ptr;
  ctx->workspace_bytes = device_ptr ? bytes : 0;
  ctx->user_workspace = device_ptr != NULL;
  return BWPP_CUDA_OK;
}

int bwpp_cuda_sync(BwppCudaCtx *ctx) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  rc = bwpp_check_cuda(ctx, cudaStreamSynchronize(ctx->stream),
                       "cudaStreamSynchronize");
  if (rc) return rc;
  int word = 0;
  rc = bwpp_check_cuda(ctx,
                       cudaMemcpy(&word, ctx->status_word, sizeof(int),
                                  cudaMemcpyDeviceToHost),
                       "status readback");
  if (rc) return rc;
  if (word != 0) {
    cudaMemset(ctx->status_word, 0, sizeof(int));
    return bwpp_set_error(ctx, word, "device reported: %s",
                          bwpp_cuda_status_string(word));
  }
  return BWPP_CUDA_OK;
}

int bwpp_cuda_copy(BwppCudaCtx *ctx, void *dst, const void *src, size_t bytes) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (bytes == 0) return BWPP_CUDA_OK;
  if (!dst || !src) return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "copy: NULL");
  rc = bwpp_check_cuda(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, ctx->stream),
                       "copy");
  if (rc) return rc;
  return bwpp_check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "copy sync");
}

const char *bwpp_cuda_ctx_last_error(const BwppCudaCtx *ctx) {
  return ctx ? ctx->last_error : "no context";
}

// ---- bounded-wait self test ----------------------------------------------

}  // extern "C"

namespace {
// One thread waits on an mbarrier that nothing ever arrives on, through the
// same bounded wait the pipelined kernels use.  The wait expires after
// limit_ns, records BWPP_CUDA_ERR_TIMEOUT and the kernel returns normally.
__global__ void selftest_wait_kernel(uint64_t limit_ns, int *status) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  fence_mbar_init();
  mbar_wait(&bar, 0, status, limit_ns);
}
// Holds an SM slot for `busy_ns` of %globaltimer (no memory traffic).
__global__ void selftest_occupy_kernel(uint64_t busy_ns) {
  extern __shared__ uint8_t held[];
  const uint64_t t0 = bwpp_globaltimer();
  while (bwpp_globaltimer() - t0 < busy_ns) __nanosleep(1000);
  if (threadIdx.x == 0 && busy_ns == ~0ull) held[0] = 0;  // keeps the smem request
}
}  // namespace

extern "C" {

int bwpp_cuda_selftest_occupy(BwppCudaCtx *ctx, void *stream, uint32_t ctas,
                              uint32_t smem_bytes, uint32_t busy_ms) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (ctas == 0 || ctas > 4096 || busy_ms == 0 || busy_ms > 3000 || smem_bytes > 227 * 1024)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG,
                          "selftest_occupy: 1..4096 CTAs, 1..3000 ms, <= 227 KB shared memory");
  rc = bwpp_check_cuda(ctx,
                       cudaFuncSetAttribute(selftest_occupy_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)smem_bytes),
                       "selftest_occupy smem attribute");
  if (rc) return rc;
  selftest_occupy_kernel<<<ctas, 32, smem_bytes, (cudaStream_t)stream>>>(
      (uint64_t)busy_ms * 1000000ull);
  BWPP_LAUNCH_CHECK(ctx, "selftest occupy");
  return BWPP_CUDA_OK;
}

int bwpp_cuda_selftest_wait_timeout(BwppCudaCtx *ctx, uint32_t limit_ms) {
  int rc = bwpp_ctx_enter(ctx);
  if (rc) return rc;
  if (limit_ms == 0 || limit_ms > 2000)
    return bwpp_set_error(ctx, BWPP_CUDA_ERR_ARG, "selftest: limit must be 1..2000 ms");
  selftest_wait_kernel<<<1, 1, 0, ctx->stream>>>((uint64_t)limit_ms * 1000000ull,
                                                 ctx->status_word);
  BWPP_LAUNCH_CHECK(ctx, "selftest wait");
  return BWPP_CUDA_OK;
}

// ---- arena (runtime/core/arena.c semantics, device memory) -----------------

int bwpp_cuda_arena_init(BwppCudaArena *arena, size_t capacity, int device) {
  if (!arena) return 0;
  arena->buffer = NULL;
  arena->capacity = 0;
  arena->offset = 0;
  if (cudaSetDevice(device) != cudaSuccess) return 0;
  void *p = NULL;
  if (cudaMalloc(&p, capacity ? capacity : 1) != cudaSuccess) return 0;
  arena->buffer = (unsigned char *)p;
  arena->capacity = capacity;
  return 1;
}

void *bwpp_cuda_arena_alloc(BwppCudaArena *arena, size_t size, size_t align) {
  if (!arena || !arena->buffer) return NULL;
  if (align == 0) align = 1;
  if (align & (align - 1)) return NULL;  // must be a power of two
  // Align the device address, not just the offset (cudaMalloc is 256-aligned,
  // so both agree for align <= 256).
  uintptr_t base = (uintptr_t)arena->buffer;
  uintptr_t start = (base + arena->offset + (align - 1)) & ~(uintptr_t)(align - 1);
  size_t off = (size_t)(start - base);
  if (off + size > arena->capacity || off + size < off) return NULL;
  arena->offset = off + size;
  return (void *)start;
}

void bwpp_cuda_arena_reset(BwppCudaArena *arena) {
  if (arena) arena->offset = 0;
}

void bwpp_cuda_arena_destroy(BwppCudaArena *arena) {
  if (!arena) return;
  if (arena->buffer) cudaFree(arena->buffer);
  arena->buffer = NULL;
  arena->capacity = 0;
  arena->offset = 0;
}

}  // extern "C"
