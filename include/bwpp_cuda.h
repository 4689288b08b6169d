/*
 * bwpp_cuda.h -- C ABI of the BW++ B200 (sm_100a) runtime, runtime/cuda.
 *
 * Drop-in boundary for the reference project's kernel runtimes:
 *   - runtime/cpu/bwpp_cpu_ref.h:6-58     (bwpp_cpu_*_f32 entry points)
 *   - runtime/metal/dispatch_stub.h:9-74  (param structs + dispatch calls)
 *   - runtime/core/arena.h:6-15, tensor.h:7-25 (arena / tensor metadata)
 *   - compiler/include/bwpp.h:8-11        (BwppStatus: 0 ok, 1 error)
 *
 * Plain C, no CUDA or torch types in any signature: streams are passed as
 * `void *` (a cudaStream_t), every buffer is a plain pointer.
 *
 * Three families of entry points:
 *   1. ctx entry points (bwpp_cuda_*(BwppCudaCtx *ctx, ...)): device
 *      pointers, asynchronous on the ctx's stream, return a status code.
 *      bwpp_cuda_sync(ctx) waits and reports device-side errors (a bounded
 *      wait that expired inside a kernel comes back as
 *      BWPP_CUDA_ERR_TIMEOUT).
 *   2. exact mirrors of the CPU reference signatures (void, synchronous).
 *      Pointers may be host or device memory; host buffers are staged through
 *      the device.  bwpp_cuda_last_status() gives the status of the calling
 *      thread's last mirror call (the reference returns nothing and silently
 *      ignores NULL inputs; so do these).
 *   3. mirrors of the Metal dispatch calls with the same param structs.
 *
 * Numerics: contractions (matmul, attention) run on tcgen05 tensor cores with
 * bf16 operands and fp32 accumulation; fp32 inputs of the mirrors are rounded
 * to bf16 (nearest even) on the device first.  Norms, softmax and reduce_max
 * run in fp32.
 */
#ifndef BWPP_CUDA_H
#define BWPP_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---- status codes (0 / 1 agree with BwppStatus, compiler/include/bwpp.h:8-11) */
#define BWPP_CUDA_OK 0
#define BWPP_CUDA_ERR 1             /* generic failure */
#define BWPP_CUDA_ERR_ARG 2         /* invalid argument (NULL, size, alignment) */
#define BWPP_CUDA_ERR_CUDA 3        /* CUDA runtime / launch error */
#define BWPP_CUDA_ERR_TIMEOUT 4     /* a bounded device-side wait expired */
#define BWPP_CUDA_ERR_NOMEM 5       /* device allocation failed */
#define BWPP_CUDA_ERR_UNSUPPORTED 6 /* shape / option not supported */

/* ---- arena + tensor metadata ------------------------------------------- */

/* Same layout as BwppArena (runtime/core/arena.h:6-10); a BwppArena* may be
 * passed where a BwppCudaArena* is expected.  `buffer` is device memory. */
typedef struct {
  unsigned char *buffer;
  size_t capacity;
  size_t offset;
} BwppCudaArena;

/* Same enumerators / layout as runtime/core/tensor.h:7-25; `buffer` holds a
 * device pointer (typically from bwpp_cuda_arena_alloc). */
typedef enum {
  BWPP_CUDA_DTYPE_F16 = 0,
  BWPP_CUDA_DTYPE_BF16 = 1,
  BWPP_CUDA_DTYPE_F32 = 2
} BwppCudaDType;

typedef enum {
  BWPP_CUDA_LAYOUT_ROW_MAJOR = 0,
  BWPP_CUDA_LAYOUT_COL_MAJOR = 1
} BwppCudaLayout;

typedef struct {
  BwppCudaDType dtype;
  BwppCudaLayout layout;
  uint32_t rank;
  uint64_t shape[4];
  uint64_t stride[4];
  void *buffer;
} BwppCudaTensor;

/* Replaces bwpp_arena_init (runtime/core/arena.c:9-17): ONE cudaMalloc of
 * `capacity` bytes on `device`.  Returns 1 on success, 0 on failure (the
 * reference's convention). */
int bwpp_cuda_arena_init(BwppCudaArena *arena, size_t capacity, int device);
/* Same bump semantics as bwpp_arena_alloc (runtime/core/arena.c:23-31):
 * `align` a power of two (0 means 1), NULL when the arena is full. */
void *bwpp_cuda_arena_alloc(BwppCudaArena *arena, size_t size, size_t align);
/* runtime/core/arena.c:19-21 */
void bwpp_cuda_arena_reset(BwppCudaArena *arena);
/* runtime/core/arena.c:33-38, with cudaFree */
void bwpp_cuda_arena_destroy(BwppCudaArena *arena);

/* ---- context ------------------------------------------------------------ */

typedef struct BwppCudaCtx BwppCudaCtx;

/* New context on `device`, launching on `stream` (a cudaStream_t; NULL means
 * the legacy default stream).  One context per host thread per GPU. */
int bwpp_cuda_ctx_create(BwppCudaCtx **out, int device, void *stream);
int bwpp_cuda_ctx_destroy(BwppCudaCtx *ctx);
int bwpp_cuda_ctx_set_stream(BwppCudaCtx *ctx, void *stream);
/* Hands the context caller-owned device scratch (e.g. an arena slice).  With
 * a workspace set the context never allocates; a call that needs more than
 * `bytes` fails with BWPP_CUDA_ERR_NOMEM.  NULL / 0 returns to ctx-owned
 * scratch.  (Without one, the first tensor-core GEMM whose last round is cut
 * into K parts allocates a fixed split-tail scratch, 2 x SM count tiles of
 * 128 x 256 fp32, about 38 MB on a B200, kept until the context is
 * destroyed, which non-causal attention also uses for a half-empty last
 * round of its items; with one set beforehand, GEMMs run that round as
 * whole tiles or N halves and attention runs it whole instead.) */
int bwpp_cuda_ctx_set_workspace(BwppCudaCtx *ctx, void *device_ptr,
                                size_t bytes);
/* Copies `bytes` between any two host / device buffers (e.g. filling arena
 * buffers from a plain C caller), ordered on the ctx stream; synchronous. */
int bwpp_cuda_copy(BwppCudaCtx *ctx, void *dst, const void *src, size_t bytes);
/* Scratch bytes the norm backward passes need for `rows` x `cols`. */
size_t bwpp_cuda_norm_bwd_workspace_size(BwppCudaCtx *ctx, uint32_t rows,
                                         uint32_t cols);
/* Waits for the ctx's stream; returns the first device-side error recorded
 * since the previous sync (then clears it), or a CUDA error. */
int bwpp_cuda_sync(BwppCudaCtx *ctx);
const char *bwpp_cuda_status_string(int status);
const char *bwpp_cuda_ctx_last_error(const BwppCudaCtx *ctx);
int bwpp_cuda_device_count(void);
/* Failure-path self test (no reference counterpart): launches a kernel whose
 * bounded device wait never completes and expires after `limit_ms` (1..2000);
 * the next bwpp_cuda_sync returns BWPP_CUDA_ERR_TIMEOUT and the context stays
 * usable.  Nothing faults or traps. */
int bwpp_cuda_selftest_wait_timeout(BwppCudaCtx *ctx, uint32_t limit_ms);
/* Co-residency self test (no reference counterpart): launches `ctas` CTAs on
 * `stream` (a cudaStream_t other than the ctx's), each holding `smem_bytes`
 * of shared memory (<= 227 KB) and an SM slot for `busy_ms` (1..3000) of
 * %globaltimer, then returning.  A kernel launched meanwhile on the ctx's
 * stream gets only the SMs left over, which tests that no kernel here waits
 * on a CTA that has not started (the GEMM's split tail).  Nothing faults. */
int bwpp_cuda_selftest_occupy(BwppCudaCtx *ctx, void *stream, uint32_t ctas,
                              uint32_t smem_bytes, uint32_t busy_ms);

/* ---- 1. ctx entry points (device pointers, async) ---------------------- */

/* C[M,N] = A[M,K] * B[K,N] (+ bias[N] if apply_bias && bias) (then SiLU if
 * apply_silu), row-major with leading dims; A, B bf16 bits, bias / C fp32.
 * The fused matmul+bias+SiLU and matmul+bias(+reshape) epilogues of
 * runtime/cpu/bwpp_cpu_ref.c:8-35 and compiler/codegen_metal.c:392-434
 * (bias before SiLU).  tcgen05 path when lda, ldb are multiples of 8, ldc of
 * 4 and the pointers 16-byte aligned; otherwise a CUDA-core kernel. */
int bwpp_cuda_matmul_bf16(BwppCudaCtx *ctx, const uint16_t *a,
                          const uint16_t *b, float *c, uint32_t M, uint32_t N,
                          uint32_t K, uint32_t lda, uint32_t ldb, uint32_t ldc,
                          const float *bias, int apply_silu, int apply_bias);

/* General form of the matmul above (no single reference counterpart: it
 * covers the transposed products of the autodiff rule for matmul,
 * compiler/graph_ir.c:1529-1583, dA = dY B^T and dB = A^T dY, plus the
 * residual add of a decoder block).
 *   A[m,k] = a_mn_major ? a[k*lda + m] : a[m*lda + k]
 *   B[k,n] = b_mn_major ? b[k*ldb + n] : b[n*ldb + k]
 *   v = A*B (+ bias[n]) (SiLU) (+ residual[m*ldr + n]); C = v as fp32 or bf16
 * residual may alias C when C is fp32 (C += A*B). */
typedef struct {
  uint32_t M, N, K;
  uint32_t lda, ldb, ldc, ldr;
  int a_mn_major;
  int b_mn_major;
  int out_bf16;
  int apply_silu;
  const float *bias;
  const float *residual;
} BwppCudaGemmParams;

int bwpp_cuda_gemm_bf16_ex(BwppCudaCtx *ctx, const uint16_t *a,
                           const uint16_t *b, void *c,
                           const BwppCudaGemmParams *params);

/* O = softmax(scale * Q K^T [+ causal mask]) V on contiguous [B,H,S,D]
 * tensors: Q [B,H,Sq,D], K and V [B,H,Skv,D] bf16 bits, O [B,H,Sq,D] fp32.
 * causal: key n visible to query m iff n <= m.  Single-pass online softmax
 * (compiler/codegen_metal.c:534-548); the reference's 2-D, unscaled, unmasked
 * form (runtime/cpu/bwpp_cpu_ref.c:92-144) is B=H=1, scale=1, causal=0.
 * tcgen05 path for D in {64, 128}; other D up to 256 on CUDA cores. */
int bwpp_cuda_attention_bf16(BwppCudaCtx *ctx, const uint16_t *q,
                             const uint16_t *k, const uint16_t *v, float *o,
                             uint32_t B, uint32_t H, uint32_t Sq, uint32_t Skv,
                             uint32_t D, float scale, int causal);

/* Attention for training (no reference counterpart: the reference has no
 * attention backward).  Token-major bf16 tensors: row b*S + s, head h at
 * column h*128 (row pitches ld_*), head dim 128, Sq == Skv == S.
 * Forward writes O (bf16, pitch ldo) and the base-2 log-sum-exp of the
 * scaled scores per query, lse [B*H, S] fp32.  Backward takes O, dO and lse
 * and writes dQ, dK, dV (bf16, pitch ldd); it uses ctx scratch
 * (4 * B*H*S bytes).  Every pitch must be a multiple of 8 elements and the
 * dQ, dK, dV bases 16-byte aligned, else BWPP_CUDA_ERR_UNSUPPORTED. */
int bwpp_cuda_attention_fwd_lse_bf16(BwppCudaCtx *ctx, const uint16_t *q,
                                     const uint16_t *k, const uint16_t *v,
                                     uint32_t ld_qkv, uint32_t B, uint32_t H,
                                     uint32_t S, float scale, int causal,
                                     uint16_t *o, uint32_t ldo, float *lse);
int bwpp_cuda_attention_bwd_bf16(BwppCudaCtx *ctx, const uint16_t *q,
                                 const uint16_t *k, const uint16_t *v,
                                 uint32_t ld_qkv, const uint16_t *o,
                                 uint32_t ldo, const uint16_t *dout,
                                 uint32_t ld_do, const float *lse, uint32_t B,
                                 uint32_t H, uint32_t S, float scale,
                                 int causal, uint16_t *dq, uint16_t *dk,
                                 uint16_t *dv, uint32_t ldd);

/* RMSNorm forward, runtime/cpu/bwpp_cpu_ref.c:63-90: y = x / sqrt(mean(x^2) +
 * eps) * gamma + beta; gamma / beta may be NULL. */
int bwpp_cuda_rmsnorm_fwd_f32(BwppCudaCtx *ctx, const float *x, float *y,
                              const float *gamma, const float *beta,
                              uint32_t rows, uint32_t cols, uint32_t ld,
                              float eps);

/* RMSNorm backward (rule of compiler/graph_ir.c:1735-1789):
 * dx = r*(g - xhat*mean(g*xhat)), g = gamma*dy, r = 1/sqrt(mean(x^2)+eps),
 * dgamma = sum_rows dy*xhat, dbeta = sum_rows dy.  dgamma / dbeta may be
 * NULL (not computed); gamma NULL means 1.  Uses ctx scratch
 * (bwpp_cuda_norm_bwd_workspace_size). */
int bwpp_cuda_rmsnorm_bwd_f32(BwppCudaCtx *ctx, const float *x,
                              const float *gamma, const float *dy, float *dx,
                              float *dgamma, float *dbeta, uint32_t rows,
                              uint32_t cols, uint32_t ld, float eps);

/* RMSNorm backward that allocates nothing (no counterpart in the reference):
 * same math and outputs as bwpp_cuda_rmsnorm_bwd_f32, for callers that cannot
 * allocate device memory themselves -- code inside a host framework that owns
 * the whole device-memory budget and forbids allocations outside its pool, or
 * latency-critical loops where cudaMalloc / cudaFree (which may synchronize
 * the device) is not acceptable.  It takes no BwppCudaCtx (creating one
 * allocates) and runs on `stream` (a cudaStream_t, NULL = default stream) of
 * the current device.
 *   - Scratch: the dgamma / dbeta partials live in a fixed 4 MiB array
 *     (1,048,576 floats) inside the library, held on every GPU that loads it
 *     until the process exits.  The first call on a device does the set-up:
 *     it looks up that array's device address (once per device, with the
 *     device current).  Make that first call before any stream capture.  The
 *     look-up is tied to the device's CUDA context: after a cudaDeviceReset
 *     (or anything else that creates a new context) the next call looks the
 *     address up again.
 *   - Limit: with dgamma or dbeta requested, cols may be at most 524,288
 *     (2 * cols floats per CTA); larger cols return BWPP_CUDA_ERR_ARG.  Wide
 *     rows run on fewer CTAs (the partials of all CTAs must fit).
 *   - Sharing: every call uses the same array.  Calls whose work overlaps on
 *     the GPU (different streams, or other host threads) race on it and give
 *     wrong dgamma / dbeta; serialize them.  Each call overwrites the part of
 *     the array it reads, so leftovers of earlier calls do not matter.
 *   - Calls no cudaMalloc, cudaFree or other allocating routine.
 *   - Errors: BWPP_CUDA_ERR_ARG for bad arguments; BWPP_CUDA_ERR_CUDA when one
 *     of its own launches fails, or, without launching anything, when a CUDA
 *     error from earlier work on this thread is still pending (that error is
 *     left in place for the caller to read).  Device-side errors surface at
 *     the caller's next synchronization. */
int bwpp_cuda_rmsnorm_bwd_f32_noalloc(const float *x, const float *gamma,
                                      const float *dy, float *dx, float *dgamma,
                                      float *dbeta, uint32_t rows, uint32_t cols,
                                      uint32_t ld, float eps, void *stream);

/* LayerNorm forward (no reference counterpart; signature follows
 * bwpp_cpu_rmsnorm_f32): y = (x - mean) * rstd * gamma + beta. */
int bwpp_cuda_layernorm_fwd_f32(BwppCudaCtx *ctx, const float *x, float *y,
                                const float *gamma, const float *beta,
                                uint32_t rows, uint32_t cols, uint32_t ld,
                                float eps);

/* LayerNorm backward: dx = rstd*(g - mean(g) - xhat*mean(g*xhat)),
 * dgamma = sum_rows dy*xhat, dbeta = sum_rows dy. */
int bwpp_cuda_layernorm_bwd_f32(BwppCudaCtx *ctx, const float *x,
                                const float *gamma, const float *dy, float *dx,
                                float *dgamma, float *dbeta, uint32_t rows,
                                uint32_t cols, uint32_t ld, float eps);

/* Row max over the last dim and the FIRST index attaining it (strict '>'
 * scan from -INF as in runtime/cpu/bwpp_cpu_ref.c:174-181; index 0 when no
 * element exceeds -INF).  maxv or argmax may be NULL. */
int bwpp_cuda_reduce_max_fwd_f32(BwppCudaCtx *ctx, const float *x, float *maxv,
                                 uint32_t *argmax, uint32_t rows,
                                 uint32_t cols, uint32_t ld);

/* Argmax-routed gradient: dx[r, argmax[r]] = dy[r], 0 elsewhere (the
 * reduce_max rule of compiler/graph_ir.c:1798-1821 with first-index ties). */
int bwpp_cuda_reduce_max_bwd_f32(BwppCudaCtx *ctx, const uint32_t *argmax,
                                 const float *dy, float *dx, uint32_t rows,
                                 uint32_t cols, uint32_t ld);

/* runtime/cpu/bwpp_cpu_ref.c:146-190: mask = 1 at EVERY position equal to the
 * max along `axis` (0: down columns, else along rows), dense rows x cols. */
int bwpp_cuda_reduce_max_mask_ex(BwppCudaCtx *ctx, const float *x, float *mask,
                                 uint32_t rows, uint32_t cols, int axis);

/* runtime/cpu/bwpp_cpu_ref.c:192-219: dx = mask * dy[axis == 0 ? c : r]. */
int bwpp_cuda_reduce_max_grad_ex(BwppCudaCtx *ctx, const float *mask,
                                 const float *dy, float *dx, uint32_t rows,
                                 uint32_t cols, int axis);

/* runtime/cpu/bwpp_cpu_ref.c:37-61: row softmax, 1/sum guarded at 0. */
int bwpp_cuda_softmax_fwd_f32(BwppCudaCtx *ctx, const float *x, float *y,
                              uint32_t rows, uint32_t cols, uint32_t ld);

/* Autodiff-internal ops of the gradient graph (compiler/include/graph_ir.h:
 * 42-55).  The reference emits them from its backward rules but has no
 * kernel for them; fp32, stream-async. */

/* compiler/graph_ir.c:1709-1720 SILU_GRAD: dx = dy * s * (1 + x * (1 - s)),
 * s = sigmoid(x), over n dense elements (dx may alias dy). */
int bwpp_cuda_silu_grad_f32(BwppCudaCtx *ctx, const float *x, const float *dy,
                            float *dx, size_t n);

/* compiler/graph_ir.c:1722-1733 SOFTMAX_GRAD over the last axis:
 * dx[r, c] = y[r, c] * (dy[r, c] - sum_j dy[r, j] * y[r, j]) (dx may alias dy). */
int bwpp_cuda_softmax_grad_f32(BwppCudaCtx *ctx, const float *y, const float *dy,
                               float *dx, uint32_t rows, uint32_t cols, uint32_t ld);

/* compiler/graph_ir.c:1414-1443 REDUCE_SUM: axis 1 -> out[rows] row sums,
 * axis 0 -> out[cols] column sums (deterministic; column sums use ctx
 * scratch).  An empty reduction writes zeros. */
int bwpp_cuda_reduce_sum_f32(BwppCudaCtx *ctx, const float *x, float *out,
                             uint32_t rows, uint32_t cols, uint32_t ld, int axis);

/* compiler/graph_ir.c:1457-1470 BROADCAST (the reduce_sum gradient,
 * 1791-1796): dst[r, c] = src[axis == 1 ? r : c]. */
int bwpp_cuda_broadcast_f32(BwppCudaCtx *ctx, const float *src, float *dst,
                            uint32_t rows, uint32_t cols, uint32_t ld, int axis);

/* fp32 -> bf16 bits, round to nearest even (dst dense rows x cols, src with
 * leading dim ld_src). */
int bwpp_cuda_cast_f32_bf16(BwppCudaCtx *ctx, const float *src, uint16_t *dst,
                            uint32_t rows, uint32_t cols, uint32_t ld_src);

/* ---- data-parallel communicator (NCCL) ----------------------------------- */
/* The gradient allreduce of the tiny_model training step (no reference
 * counterpart: the reference has no multi-device code).  NCCL is loaded at
 * run time (libnccl.so.2, or the file $BWPP_NCCL_LIBRARY names), sharing a
 * copy the process already has.
 * Every wait on a communicator is bounded by its timeout: it is created
 * non-blocking, and before a collective is queued (and in
 * bwpp_cuda_comm_wait) a host watchdog waits for the previous one.  A peer
 * that stops taking part (a rank that left between steps) makes that wait
 * expire: the watchdog aborts the communicator (ncclCommAbort ends the NCCL
 * kernels waiting on the peer), and the call returns BWPP_CUDA_ERR_TIMEOUT
 * (BWPP_CUDA_ERR for an asynchronous NCCL error).  An aborted communicator
 * refuses further collectives; destroy it. */
typedef struct BwppCudaComm BwppCudaComm;
/* Rank 0 creates the 128-byte id and hands it to every rank. */
int bwpp_cuda_comm_unique_id(unsigned char *id128);
/* Creation waits (bounded by timeout_ms) for every rank to join. */
int bwpp_cuda_comm_create_timeout(BwppCudaComm **out, const unsigned char *id128,
                                  int rank, int nranks, int device,
                                  uint32_t timeout_ms);
/* bwpp_cuda_comm_create_timeout with a 120 s timeout. */
int bwpp_cuda_comm_create(BwppCudaComm **out, const unsigned char *id128,
                          int rank, int nranks, int device);
int bwpp_cuda_comm_set_timeout(BwppCudaComm *comm, uint32_t timeout_ms);
/* In-place sum over ranks, asynchronous on `stream` (after a bounded wait
 * for the communicator's previous collective). */
int bwpp_cuda_comm_allreduce_sum_f32(BwppCudaComm *comm, float *buf,
                                     size_t count, void *stream);
/* Waits (bounded) for the latest collective. */
int bwpp_cuda_comm_wait(BwppCudaComm *comm);
/* 1 once the communicator was aborted (then only destroy it). */
int bwpp_cuda_comm_aborted(const BwppCudaComm *comm);
int bwpp_cuda_comm_destroy(BwppCudaComm *comm);
/* Multi-GPU form of bwpp_cuda_matmul_f32 (no reference counterpart): a
 * collective over the communicator's ranks (one process or thread per GPU,
 * the communicator's device current).  Rank r passes its own M rows of A and
 * C and the whole B and bias, all in HOST memory, with the argument meaning
 * of bwpp_cpu_matmul_f32 (runtime/cpu/bwpp_cpu_ref.c:8-35).  Each rank uploads
 * only its 1/n of B's K rows and rounds them to bf16; an NCCL all-gather
 * over NVLink assembles the bf16 B on every GPU; A's row chunks go up, their
 * GEMMs run and their C rows come back, copies overlapping the math.
 * Synchronous; returns a status (also left in bwpp_cuda_last_status). */
int bwpp_cuda_matmul_f32_dist(BwppCudaComm *comm, const float *a, const float *b,
                              float *c, uint32_t M, uint32_t N, uint32_t K,
                              uint32_t lda, uint32_t ldb, uint32_t ldc,
                              const float *bias, int apply_silu, int apply_bias);
/* The host watchdog the communicator uses, driven by callbacks (a caller's
 * own collectives, or tests with a fake communicator): polls done(user)
 * (1 finished, 0 not yet, < 0 failed) and error(user) (0 fine, 1 in
 * progress, else failed; may be NULL) with a growing interval (10 us to
 * 160 us) until done, a failure or timeout_ms.  On failure or timeout it calls
 * abort_fn(user) once and returns BWPP_CUDA_ERR (error), BWPP_CUDA_ERR_CUDA
 * (done < 0) or BWPP_CUDA_ERR_TIMEOUT; BWPP_CUDA_OK when done. */
int bwpp_cuda_comm_watch(int (*done)(void *), int (*error)(void *),
                         void (*abort_fn)(void *), void *user,
                         uint32_t timeout_ms);

/* ---- tiny_model training step ------------------------------------------- */
/* The decoder block of examples/tiny_model.bwpp:4-58 in the shape of the
 * benchmark config: `layers` pre-RMSNorm blocks, causal attention with
 * `heads` x 128, SiLU-gated MLP of width `ffn`, MSE loss.  Forward and
 * backward follow the autodiff rules of compiler/graph_ir.c:1485-1839
 * (matmul, silu, rmsnorm) plus the attention backward; weights are fp32
 * masters with bf16 compute copies, initialised N(0, 0.02) (norm gains 1)
 * from `seed`. */
typedef struct {
  uint32_t layers, d_model, heads, head_dim, ffn, batch, seq;
  float eps;
} BwppCudaTinyModelConfig;

typedef struct BwppCudaTinyModel BwppCudaTinyModel;

int bwpp_cuda_tiny_model_create(BwppCudaCtx *ctx,
                                const BwppCudaTinyModelConfig *cfg,
                                uint64_t seed, BwppCudaTinyModel **out);
int bwpp_cuda_tiny_model_destroy(BwppCudaTinyModel *model);
/* Parameters form one flat fp32 vector; per layer the order is g1 [D],
 * Wqkv [D,3D], Wo [D,D], g2 [D], W13 [D,2F] (gate | up), W2 [F,D]. */
size_t bwpp_cuda_tiny_model_param_count(const BwppCudaTinyModel *model);
/* Copies the fp32 parameters and / or the gradients of the last step out
 * (host or device destinations; NULL skips).  Synchronous. */
int bwpp_cuda_tiny_model_get(BwppCudaTinyModel *model, float *params_out,
                             float *grads_out);
/* Copies d loss / d x [batch*seq, d_model] fp32 of the last step (the
 * gradient that reaches the input embeddings) to `dx_out` (host or device).
 * Synchronous. */
int bwpp_cuda_tiny_model_input_grad(BwppCudaTinyModel *model, float *dx_out);
/* Replaces the fp32 parameters (host or device source) and re-derives the
 * bf16 compute copies.  Synchronous. */
int bwpp_cuda_tiny_model_set_params(BwppCudaTinyModel *model,
                                    const float *params_in);
/* One training step on inputs x, target [batch*seq, d_model] fp32 (host or
 * device memory; both are staged into the model's arena):
 * forward, loss, backward into the gradient buffer, then (comm != NULL) the
 * gradient sum over ranks and (lr != 0) w -= lr * mean gradient.  The loss
 * is copied to *loss_out (host or device) when loss_out != NULL.
 * Asynchronous on the ctx stream. */
int bwpp_cuda_tiny_model_step(BwppCudaTinyModel *model, const float *x,
                              const float *target, float lr,
                              BwppCudaComm *comm, float *loss_out);

/* ---- 2. mirrors of runtime/cpu/bwpp_cpu_ref.h:6-58 ---------------------- */
/* Same argument lists; host or device pointers; synchronous; the calling
 * thread's context on the current device is created on first use.
 * bwpp_cuda_matmul_f32 with A, B and C all in host memory (and at least two
 * chunks of 1024 rows or columns) overlaps its copies with the GEMMs: A goes
 * up in row chunks and B in column chunks on one stream, each newly complete
 * L-shaped region of C is computed on the context stream and comes back on a
 * third; both streams belong to the calling thread and live as long as it. */

void bwpp_cuda_matmul_f32(const float *a, const float *b, float *c, uint32_t M,
                          uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb,
                          uint32_t ldc, const float *bias, int apply_silu,
                          int apply_bias);
void bwpp_cuda_softmax_f32(const float *x, float *y, uint32_t rows,
                           uint32_t cols, uint32_t ld);
void bwpp_cuda_rmsnorm_f32(const float *x, float *y, const float *gamma,
                           const float *beta, uint32_t rows, uint32_t cols,
                           uint32_t ld, float eps);
void bwpp_cuda_attention_f32(const float *q, const float *k, const float *v,
                             float *o, uint32_t M, uint32_t N, uint32_t K,
                             uint32_t D, uint32_t ldq, uint32_t ldk,
                             uint32_t ldv, uint32_t ldo);
void bwpp_cuda_reduce_max_mask_f32(const float *x, float *mask, uint32_t rows,
                                   uint32_t cols, int axis);
void bwpp_cuda_reduce_max_grad_f32(const float *mask, const float *dy,
                                   float *dx, uint32_t rows, uint32_t cols,
                                   int axis);
/* Status of the calling thread's last mirror call (BWPP_CUDA_OK when none). */
int bwpp_cuda_last_status(void);

/* ---- 3. mirrors of runtime/metal/dispatch_stub.h:9-74 -------------------- */
/* Param structs with the Metal layouts.  Buffers are device pointers; A/B/Q/
 * K/V are bf16 (the Metal kernels take half: an f16 variant is not built),
 * C/O/bias/x/y/gamma/beta fp32.  `source` is the compiler output text: like
 * the Metal shim (dispatch_stub.m:74-79) a call is a no-op returning
 * BWPP_CUDA_OK unless `source` carries the matching `bwpp.meta:` kernel tag;
 * `bwpp.meta: epilogue=add|silu|add_silu` selects the matmul epilogue. */

typedef struct {
  uint32_t M, N, K, lda, ldb, ldc;
} BwppCudaMatmulParams;

typedef struct {
  uint32_t rows, cols, ld;
} BwppCudaSoftmaxParams;

typedef struct {
  uint32_t rows, cols, ld;
  float eps;
} BwppCudaRmsnormParams;

typedef struct {
  uint32_t M, N, K, D, ldq, ldk, ldv, ldo;
} BwppCudaAttentionParams;

/* runtime/metal/dispatch_stub.h:42-49 */
int bwpp_cuda_dispatch_matmul(BwppCudaCtx *ctx, const uint16_t *a,
                              const uint16_t *b, float *c, const float *bias,
                              BwppCudaMatmulParams params, const char *source);
/* runtime/metal/dispatch_stub.h:51-56 */
int bwpp_cuda_dispatch_softmax(BwppCudaCtx *ctx, const float *x, float *y,
                               BwppCudaSoftmaxParams params,
                               const char *source);
/* runtime/metal/dispatch_stub.h:58-65 */
int bwpp_cuda_dispatch_rmsnorm(BwppCudaCtx *ctx, const float *x,
                               const float *gamma, const float *beta, float *y,
                               BwppCudaRmsnormParams params,
                               const char *source);
/* runtime/metal/dispatch_stub.h:67-74 (2-D, unscaled, unmasked; ld strides) */
int bwpp_cuda_dispatch_attention(BwppCudaCtx *ctx, const uint16_t *q,
                                 const uint16_t *k, const uint16_t *v, float *o,
                                 BwppCudaAttentionParams params,
                                 const char *source);

/* ---- 4. f16 variants: the half ABI of the MSL kernels --------------------
 * compiler/codegen_metal.c:392-434 (matmul), 457-556 (attention), 567-598
 * (softmax), 609-636 (rmsnorm) read and write half; these take IEEE half
 * bits (uint16_t) everywhere, compute in fp32 (tensor-core f16 operands with
 * fp32 accumulation for the contractions) and round each result to half
 * once, nearest even.  Stream-async like the bf16 / fp32 entry points. */

/* C = epilogue(A * B) with bias[N] (half, added when apply_bias && bias),
 * then SiLU when apply_silu; A [M, lda], B [K, ldb], C [M, ldc] row-major. */
int bwpp_cuda_matmul_f16(BwppCudaCtx *ctx, const uint16_t *a, const uint16_t *b,
                         uint16_t *c, uint32_t M, uint32_t N, uint32_t K,
                         uint32_t lda, uint32_t ldb, uint32_t ldc,
                         const uint16_t *bias, int apply_silu, int apply_bias);

/* Q [B,H,Sq,D], K / V [B,H,Skv,D], O [B,H,Sq,D], all half. */
int bwpp_cuda_attention_f16(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                            const uint16_t *v, uint16_t *o, uint32_t B, uint32_t H,
                            uint32_t Sq, uint32_t Skv, uint32_t D, float scale,
                            int causal);

/* Row softmax of runtime/cpu/bwpp_cpu_ref.c:37-61 on half rows. */
int bwpp_cuda_softmax_f16(BwppCudaCtx *ctx, const uint16_t *x, uint16_t *y,
                          uint32_t rows, uint32_t cols, uint32_t ld);

/* RMSNorm of runtime/cpu/bwpp_cpu_ref.c:63-90 on half rows (gamma / beta
 * half or NULL). */
int bwpp_cuda_rmsnorm_f16(BwppCudaCtx *ctx, const uint16_t *x, uint16_t *y,
                          const uint16_t *gamma, const uint16_t *beta, uint32_t rows,
                          uint32_t cols, uint32_t ld, float eps);

/* Dense conversions between half bits and fp32 (nearest even to half). */
int bwpp_cuda_cast_f16_f32(BwppCudaCtx *ctx, const uint16_t *src, float *dst, size_t n);
int bwpp_cuda_cast_f32_f16(BwppCudaCtx *ctx, const float *src, uint16_t *dst, size_t n);

/* Half mirrors of runtime/metal/dispatch_stub.h:42-74: every buffer half,
 * same bwpp.meta gating and epilogue tags as the calls above. */
int bwpp_cuda_dispatch_matmul_f16(BwppCudaCtx *ctx, const uint16_t *a, const uint16_t *b,
                                  uint16_t *c, const uint16_t *bias,
                                  BwppCudaMatmulParams params, const char *source);
int bwpp_cuda_dispatch_softmax_f16(BwppCudaCtx *ctx, const uint16_t *x, uint16_t *y,
                                   BwppCudaSoftmaxParams params, const char *source);
int bwpp_cuda_dispatch_rmsnorm_f16(BwppCudaCtx *ctx, const uint16_t *x, const uint16_t *gamma,
                                   const uint16_t *beta, uint16_t *y,
                                   BwppCudaRmsnormParams params, const char *source);
int bwpp_cuda_dispatch_attention_f16(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                                     const uint16_t *v, uint16_t *o,
                                     BwppCudaAttentionParams params, const char *source);

/* ---- 5. launch-plan executor ----------------------------------------------
 * Runs a graph built by the reference compiler, from the launch plan that
 * `bwppc --target cuda` writes (bwpp_cuda_plan_create_launch below) or from
 * the compiler's own dumps:
 *   bwppc in.bwpp out.metal --entry fn --dot graph.dot [--mem-plan plan.txt]
 *   (or --grad-dot for the gradient graph).
 * graph_dot: the text of the graph dump (compiler/graph_ir.c:1326-1358);
 * mem_plan: the text of the memory-plan dump (compiler/mem_plan.c:176-193) or
 * NULL (every value then gets its own buffer); dims: "T=128,D=256,..." binds
 * the symbolic dims; options: NULL or "eps=1e-5,fuse=1".
 * With ctx == NULL the plan is parsed and lowered only (no device memory):
 * bwpp_cuda_plan_describe shows the lowered steps.  Fusions: matmul ->
 * softmax attention patterns into the attention kernel, transposes into GEMM
 * operand layouts, matmul -> add(bias by dataflow) -> silu -> mul(gate) or
 * add(residual) into the GEMM epilogue, mul(silu(x), y) into one swiglu pass,
 * rmsnorm(add(a, b)) into one residual + norm pass; every other graph op
 * (permute and the reduce_max family included) is one kernel.  A dump does
 * not carry a permute's axes: they are read off the symbolic dims, and a
 * permute they do not determine is refused (the launch plan carries them).
 * No counterpart in the
 * reference (it has no executor for its graphs); the op vocabulary is
 * compiler/include/graph_ir.h:39-57. */
typedef struct BwppCudaPlan BwppCudaPlan;
int bwpp_cuda_plan_create(BwppCudaCtx *ctx, const char *graph_dot, const char *mem_plan,
                          const char *dims, const char *options, BwppCudaPlan **out);
/* The same executor on the text of a launch plan written by
 *   bwppc in.bwpp out.plan --entry fn --target cuda --dims T=128,D=256
 * (this package's compiler/codegen_cuda.c, selected by the --target flag the
 * patch compiler/main_target_cuda.patch adds to compiler/main.c:49-85,186).
 * The plan carries the compiler's fusion decisions, operand value ids, bound
 * shapes and arena offsets (one cudaMalloc, compiler/mem_plan.c's buffers
 * sized in bytes); nothing is re-lowered.  options: NULL or "fuse=1" (eps
 * comes from each launch line). */
int bwpp_cuda_plan_create_launch(BwppCudaCtx *ctx, const char *launch_plan, const char *options,
                                 BwppCudaPlan **out);
/* Message of the last failed bwpp_cuda_plan_create on this thread. */
const char *bwpp_cuda_plan_last_error(void);
/* Writes the lowered steps as text; returns the bytes needed (incl. NUL). */
int bwpp_cuda_plan_describe(const BwppCudaPlan *plan, char *buf, size_t len);
/* Value id of the value named `name` in the graph, or -1. */
int bwpp_cuda_plan_find(const BwppCudaPlan *plan, const char *name);
int bwpp_cuda_plan_value_count(const BwppCudaPlan *plan);
/* dtype: 0 f16, 1 bf16, 2 f32; dims8 receives up to 8 dims; flags: bit 0
 * graph input, bit 1 graph output, bit 2 held in the plan's memory. */
int bwpp_cuda_plan_value_info(const BwppCudaPlan *plan, int id, int *dtype, int *rank,
                              int64_t *dims8, int *flags);
/* Binds a graph input (required before run) or output (optional: written
 * there instead of the plan's memory) to caller device memory. */
int bwpp_cuda_plan_bind(BwppCudaPlan *plan, int id, void *dev_ptr);
/* Device address of a value held in the plan's memory (or bound). */
void *bwpp_cuda_plan_value_ptr(const BwppCudaPlan *plan, int id);
/* Enqueues every step on the ctx stream (stream-async, like the kernels). */
int bwpp_cuda_plan_run(BwppCudaPlan *plan);
/* Kernel launches the last run enqueued. */
size_t bwpp_cuda_plan_launches(const BwppCudaPlan *plan);
int bwpp_cuda_plan_destroy(BwppCudaPlan *plan);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* BWPP_CUDA_H */
