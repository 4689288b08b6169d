// Internal helpers of the BW++ CUDA runtime (sm_100a only).
//
//  * BwppCudaCtx: device, stream, device status word, workspace.
//  * Bounded device waits: every spin in a kernel gives up after
//    BWPP_WAIT_LIMIT_NS of %globaltimer, records BWPP_CUDA_ERR_TIMEOUT in the
//    ctx's status word and lets the kernel unwind; nothing traps.
//  * Thin inline-PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor, no
//    cluster-wide copies: every load lands in the issuing CTA) and tcgen05
//    (alloc / mma / commit / ld), in one-CTA and CTA-pair forms.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "bwpp_cuda.h"

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

struct BwppCudaCtx {
  int device;
  cudaStream_t stream;
  int *status_word;        // device int, 0 = ok, else a BWPP_CUDA_ERR_* code
  int *sched_counter;      // device int next to it: work counter of persistent kernels
  void *workspace;         // device scratch (owned unless user_workspace)
  size_t workspace_bytes;
  int user_workspace;      // 1: set by bwpp_cuda_ctx_set_workspace, not freed
  int num_sms;
  // Split-tail scratch of the tensor-core GEMM (allocated on first use, not
  // when the caller owns the workspace): fp32 partial sums of tiles cut into
  // K parts, and per-(slot, CTA, lane quarter) ready flags that hold the
  // epoch of the launch that last published them.
  float *gemm_partials;
  unsigned long long *gemm_counters;
  uint32_t gemm_epoch;
  int gemm_scratch_failed;
  char last_error[256];
};

// Split-work scratch of ctx (gemm.cu): fp32 partials and epoch-tagged
// counters shared by kernels that cut their last work items in two.
bool bwpp_split_scratch(BwppCudaCtx *ctx, float **partials, size_t *partial_floats,
                        unsigned long long **counters, size_t *ncounters, uint32_t *epoch);

// Records a message in ctx->last_error (if ctx) and returns `code`.
int bwpp_set_error(BwppCudaCtx *ctx, int code, const char *fmt, ...);

// Checks a CUDA runtime return code; on failure records it and returns
// BWPP_CUDA_ERR_CUDA.
int bwpp_check_cuda(BwppCudaCtx *ctx, cudaError_t err, const char *what);

// Makes ctx's device current; returns BWPP_CUDA_OK or an error.
int bwpp_ctx_enter(BwppCudaCtx *ctx);

// Returns a device pointer to at least `bytes` of scratch owned by ctx,
// growing the ctx-owned buffer if needed (a user-provided workspace is never
// grown: a too-small one is an error).  NULL on failure (error recorded).
void *bwpp_ctx_workspace(BwppCudaCtx *ctx, size_t bytes);

// Launch-error check after a kernel launch.
#define BWPP_LAUNCH_CHECK(ctx, name)                                        \
  do {                                                                     \
    cudaError_t e_ = cudaGetLastError();                                   \
    if (e_ != cudaSuccess) return bwpp_check_cuda((ctx), e_, (name));      \
  } while (0)

// TMA descriptor encoding through the driver entry point (no -lcuda link).
typedef CUresult (*bwpp_encode_tiled_fn)(
    CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
    CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
    CUtensorMapFloatOOBfill);
bwpp_encode_tiled_fn bwpp_get_encode_tiled(void);

// 2-D tensor map: dims {inner, outer}, row pitch in bytes, box {bi, bo}.
int bwpp_make_tmap_2d(BwppCudaCtx *ctx, CUtensorMap *map, const void *base,
                      CUtensorMapDataType dtype, uint64_t inner,
                      uint64_t outer, uint64_t pitch_bytes, uint32_t box_inner,
                      uint32_t box_outer, CUtensorMapSwizzle swz);

// ---------------------------------------------------------------------------
// device side
// ---------------------------------------------------------------------------

#define BWPP_WAIT_LIMIT_NS (2ull * 1000ull * 1000ull * 1000ull)  // 2 s

__device__ __forceinline__ uint64_t bwpp_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void bwpp_report(int *status, int code) {
  if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ---- mbarrier ---------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with `parity` to complete.  Gives up after `limit_ns`
// (default BWPP_WAIT_LIMIT_NS), reports BWPP_CUDA_ERR_TIMEOUT and returns
// false; the caller then unwinds instead of waiting on.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          int *status,
                                          uint64_t limit_ns = BWPP_WAIT_LIMIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = bwpp_globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (bwpp_globaltimer() - t0 > limit_ns) {
      bwpp_report(status, BWPP_CUDA_ERR_TIMEOUT);
      return false;
    }
  }
}

// ---- flags in global memory between CTAs of one launch ---------------------

__device__ __forceinline__ void st_release_gpu(uint32_t *p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits until *p == want (acquire: the publisher's earlier writes are then
// visible to this thread).  Bounded like mbar_wait.
__device__ __forceinline__ bool flag_wait(const uint32_t *p, uint32_t want, int *status,
                                          uint64_t limit_ns = BWPP_WAIT_LIMIT_NS) {
  if (ld_acquire_gpu(p) == want) return true;
  const uint64_t t0 = bwpp_globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i) {
      if (ld_acquire_gpu(p) == want) return true;
      __nanosleep(100);
    }
    if (bwpp_globaltimer() - t0 > limit_ns) {
      bwpp_report(status, BWPP_CUDA_ERR_TIMEOUT);
      return false;
    }
  }
}

// ---- epoch-tagged counters in global memory (split work items) ----------

// Counts one arrival on an epoch-tagged counter (high word: epoch, low word:
// count; a word from an earlier launch reads as a count of 0) and returns the
// count before it.  At most the parts of one split tile contend, so the loop
// ends.
__device__ __forceinline__ uint32_t epoch_arrive(unsigned long long *p, uint32_t epoch) {
  unsigned long long cur = *reinterpret_cast<volatile unsigned long long *>(p);
  while (true) {
    const unsigned long long base =
        (uint32_t)(cur >> 32) == epoch ? cur : ((unsigned long long)epoch << 32);
    const unsigned long long prev = atomicCAS(p, cur, base + 1);
    if (prev == cur) return (uint32_t)base;
    cur = prev;
  }
}

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Waits (bounded) until the counter reads `count` in this epoch; acquire, so
// the counted writers' partials are then visible.
__device__ __forceinline__ bool epoch_wait(const unsigned long long *p, uint32_t epoch,
                                           uint32_t count, int *status) {
  const unsigned long long want = ((unsigned long long)epoch << 32) | count;
  if (ld_acquire_gpu_u64(p) == want) return true;
  const uint64_t t0 = bwpp_globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i) {
      if (ld_acquire_gpu_u64(p) == want) return true;
      __nanosleep(64);
    }
    if (bwpp_globaltimer() - t0 > BWPP_WAIT_LIMIT_NS) {
      bwpp_report(status, BWPP_CUDA_ERR_TIMEOUT);
      return false;
    }
  }
}

// ---- TMA: each copy targets the issuing CTA only --------------------------

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map,
                                            uint64_t *bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
      "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map,
                                             const void *src, int32_t x,
                                             int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], "
      "[%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- per-thread asynchronous 16-byte copies global -> shared ---------------

__device__ __forceinline__ void cp_async_16(uint32_t dst_smem, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst_smem), "l"(src)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Waits until at most `pending` (0..7) of this thread's committed groups are
// still in flight.
__device__ __forceinline__ void cp_async_wait_pending(int pending) {
  switch (pending) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
  }
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map))
               : "memory");
}

// ---- tcgen05 ----------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst_smem)),
      "r"(ncols)
      : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc), kind::f16, one CTA.
__device__ __forceinline__ void tc_mma_f16_ss(uint32_t d_tmem, uint64_t adesc,
                                              uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem desc), kind::f16, one CTA.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem,
                                              uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The same wait for a 16-register load.
__device__ __forceinline__ void tc_wait_ld16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])::"memory");
}

// tcgen05.ld writes its destination registers asynchronously, but the
// compiler sees them defined at the load.  Waiting through this helper makes
// the 32 registers operands of the wait, so no use can be scheduled above it.
__device__ __forceinline__ void tc_wait_ld(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
        "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
        "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]),
        "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
        "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]),
        "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

__device__ __forceinline__ void tc_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 columns of 32-bit: thread t gets lane (base lane + t),
// columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr,
                                                   uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 columns of 32-bit: thread t gets lane (base lane + t).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 16 columns of 32-bit, from registers into TMEM.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr,
                                                   const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
      "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]),
      "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 16 lanes x 256 bits, repeated 8 times along the columns (64 columns):
// thread t holds, for k = 0..7, registers 4k..4k+3 = (lane L + t/4, column
// 8k + 2(t%4)), (L + t/4, 8k + 2(t%4) + 1), (L + 8 + t/4, 8k + 2(t%4)),
// (L + 8 + t/4, 8k + 2(t%4) + 1), L the address's lane.
__device__ __forceinline__ void tmem_ld_16x256b_x8(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// The same layout from registers into TMEM.
__device__ __forceinline__ void tmem_st_16x256b_x8(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x8.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 16 lanes x 128 bits, repeated 8 times (32 columns), into TMEM: thread t
// supplies, for k = 0..7, registers 2k, 2k+1 = (lane L + t/4, column
// 4k + t%4), (L + 8 + t/4, 4k + t%4).
__device__ __forceinline__ void tmem_st_16x128b_x8(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x128b.x8.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// 32 lanes x 8 columns of 32-bit, from registers into TMEM.
__device__ __forceinline__ void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}

// Shared-memory matrix descriptor for tcgen05 (sm_100 layout: start >> 4 in
// bits 0-13, leading byte offset >> 4 in 16-29, stride byte offset >> 4 in
// 32-45, version 1 in 46-47, swizzle mode in 61-63).
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr,
                                                   uint32_t lbo_bytes,
                                                   uint32_t sbo_bytes,
                                                   uint32_t swizzle_mode) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)(swizzle_mode & 7u) << 61;
  return d;
}

#define BWPP_SWIZZLE_128B 2u

// The same descriptor as two 32-bit words, for issue loops that step the
// address: the low word holds (address >> 4) in bits 0-13 and LBO >> 4 in
// bits 16-29, the high word SBO >> 4, the fixed version bit and the swizzle.
// Shared-memory addresses stay below 2^18, so stepping the low word by
// (offset >> 4) never carries into the LBO field: one add per operand.
__device__ __forceinline__ uint32_t smem_desc_lo(uint32_t saddr, uint32_t lbo_bytes) {
  return ((saddr >> 4) & 0x3FFFu) | (((lbo_bytes >> 4) & 0x3FFFu) << 16);
}
__host__ __device__ constexpr uint32_t smem_desc_hi(uint32_t sbo_bytes, uint32_t swizzle_mode) {
  return ((sbo_bytes >> 4) & 0x3FFFu) | (1u << 14) | ((swizzle_mode & 7u) << 29);
}

// D(tmem) (+)= A(smem) * B(smem) from descriptor words (see smem_desc_lo).
__device__ __forceinline__ void tc_mma_f16_ss_w(uint32_t d_tmem, uint32_t alo, uint32_t ahi,
                                                uint32_t blo, uint32_t bhi, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
      "mov.b64 da, {%1, %2};\n\t"
      "mov.b64 db, {%3, %4};\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, p;\n\t}" ::"r"(d_tmem),
      "r"(alo), "r"(ahi), "r"(blo), "r"(bhi), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem) from descriptor words.
__device__ __forceinline__ void tc_mma_f16_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint32_t blo,
                                                uint32_t bhi, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(blo), "r"(bhi), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The descriptor of the shared-memory address `bytes` past the one `d`
// describes.  The start address is d's low 14 bits (address >> 4); callers
// keep the sum below 256 KB, so only the low word changes.
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t bytes) {
  uint32_t lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(d));
  lo += bytes >> 4;
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}

// Instruction descriptor, kind::f16 with fp32 D and A/B both bf16 (ab_f16 =
// 0) or both f16 (ab_f16 = 1): A/B format fields 0 = f16, 1 = bf16.
__host__ __device__ constexpr uint32_t make_idesc_f32acc(uint32_t M, uint32_t N,
                                                         uint32_t a_mn_major,
                                                         uint32_t b_mn_major,
                                                         uint32_t ab_f16) {
  return (1u << 4)                          // D format: f32
         | ((ab_f16 ? 0u : 1u) << 7)        // A format
         | ((ab_f16 ? 0u : 1u) << 10)       // B format
         | (a_mn_major << 15)               // A major: 0 = K-major
         | (b_mn_major << 16)               // B major: 1 = MN-major
         | ((N >> 3) << 17)                 // N / 8
         | ((M >> 4) << 24);                // M / 16
}

__host__ __device__ constexpr uint32_t make_idesc_bf16_f32(uint32_t M, uint32_t N,
                                                           uint32_t a_mn_major,
                                                           uint32_t b_mn_major) {
  return make_idesc_f32acc(M, N, a_mn_major, b_mn_major, 0u);
}

// Two fp32 values to a packed pair of 16-bit floats (lo in the low half),
// round to nearest even: bf16 or, with F16, IEEE half.
template <bool F16>
__device__ __forceinline__ uint32_t pack2_16(float lo, float hi) {
  uint32_t r;
  if (F16) asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// One 16-bit float (bf16 or, with F16, IEEE half bits) to fp32, exact.
template <bool F16>
__device__ __forceinline__ float load16(uint16_t h) {
  if (F16) {
    float f;
    asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
    return f;
  }
  return __uint_as_float((uint32_t)h << 16);
}

// ---- CTA pairs (cluster of 2, tcgen05 cta_group::2) -------------------------
// A kernel that uses these must use cta_group::2 for every tcgen05 alloc /
// dealloc / mma / commit.  Rank 0 of the pair issues the MMAs; each CTA
// holds half of A (M/2 rows), half of B (N/2 columns) and its M/2 x N slice
// of the accumulator.  Every copy still lands in the issuing CTA's shared
// memory; only the mbarrier that counts its bytes may be the peer's.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

// shared::cluster address of the object at `p` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// All threads of both CTAs; orders prior shared-memory work cluster-wide.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (may be the peer's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}

// 2-D tile load into this CTA's shared memory whose completed bytes are
// counted on `cluster_bar`, an mbarrier of either CTA of the pair.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map,
                                                 uint32_t cluster_bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(cluster_bar)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D (both CTAs' TMEM) (+)= A (both CTAs' smem) * B (both CTAs' smem); the
// descriptors hold this CTA's addresses, the peer's halves sit at the same
// offsets in its shared memory.
__device__ __forceinline__ void tc_mma_f16_ss_pair(uint32_t d_tmem, uint64_t adesc,
                                                   uint64_t bdesc, uint32_t idesc,
                                                   uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at shared::cluster address `cluster_bar` once the
// pair MMAs issued so far by this thread are done.
__device__ __forceinline__ void tc_commit_pair(uint32_t cluster_bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          cluster_bar)
      : "memory");
}

// Two fp32 lanes in one 64-bit register: Blackwell issues one FMA / ADD for
// both (fma.rn.f32x2 / add.rn.f32x2).
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void f2unpack(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ uint64_t f2add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint64_t f2mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// x * sigmoid(x).  __fdividef (2 ulp, no special-case branch) instead of the
// IEEE divide: the divide's slow-path branch serialises the 32 independent
// columns an epilogue thread holds.  Limits are kept: for x -> -inf the
// denominator overflows to inf (or exceeds 2^126) and the result is -0 / 0.
__device__ __forceinline__ float bwpp_silu_f(float x) {
  return __fdividef(x, 1.0f + __expf(-x));
}

// SiLU of two columns at once, as x * (1 / (1 + 2^(-x log2 e))): the scaling,
// the 1 + e and the final product are paired fp32 operations (one issue slot
// for both columns), the power of two and the reciprocal are the MUFU
// approximations (ex2.approx, rcp.approx; flush-to-zero, so x -> -inf gives
// 1/inf = 0 and a result of -0).
__device__ __forceinline__ uint64_t bwpp_silu_f2(uint64_t x) {
  const uint64_t t = f2mul(x, f2pack(-1.44269504f, -1.44269504f));
  float t0, t1, e0, e1, y0, y1, r0, r1;
  f2unpack(t, t0, t1);
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(t0));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(t1));
  f2unpack(f2add(f2pack(e0, e1), f2pack(1.0f, 1.0f)), y0, y1);
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(y0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(y1));
  return f2mul(x, f2pack(r0, r1));
}
