// NCCL communicator for the data-parallel gradient allreduce of the
// tiny_model training step -- the only collective of the hot path.
//
// NCCL is resolved at run time with dlopen("libnccl.so.2"): when the process
// already has NCCL loaded (torch.distributed does), the same copy is used, so
// there is never a second NCCL in the process.  Only the handful of symbols
// below are used; their signatures (and the config struct's layout) are
// NCCL's public C API.
//
// Failure handling: the communicator is created non-blocking and every wait
// on it is bounded.  Each collective records a CUDA event after it; before
// the next one is enqueued (and in bwpp_cuda_comm_wait) a host watchdog polls
// that event and ncclCommGetAsyncError.  A peer that never joins a
// collective (a rank that died between steps) leaves the event pending: after
// the communicator's timeout the watchdog calls ncclCommAbort, which ends the
// NCCL kernels waiting on the peer, and the call returns
// BWPP_CUDA_ERR_TIMEOUT (an asynchronous NCCL error returns BWPP_CUDA_ERR).
// An aborted communicator refuses further collectives.
#include <dlfcn.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "bwpp_cuda_internal.cuh"

namespace {

typedef struct ncclComm *ncclComm_t;
typedef struct {
  char internal[128];
} ncclUniqueId;
typedef int ncclResult_t;  // 0 = ncclSuccess
constexpr int kNcclUint8 = 1;
constexpr int kNcclFloat32 = 7;
constexpr int kNcclSum = 0;
constexpr int kNcclInProgress = 7;

// ncclConfig_t as NCCL 2.28 lays it out (fields are only ever appended;
// `size` and `version` tell the library which of them this struct has).
struct NcclConfig {
  size_t size;
  unsigned int magic;
  unsigned int version;
  int blocking, cgaClusterSize, minCTAs, maxCTAs;
  const char *netName;
  int splitShare, trafficClass;
  const char *commName;
  int collnetEnable, CTAPolicy, shrinkShare, nvlsCTAs, nChannelsPerNetPeer, nvlinkCentricSched;
};
constexpr int kUndefInt = (int)0x80000000;  // NCCL_CONFIG_UNDEF_INT

struct Nccl {
  void *h = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, int, int, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, int, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t *) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
  ncclResult_t (*comm_init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, NcclConfig *) = nullptr;
  ncclResult_t (*comm_finalize)(ncclComm_t) = nullptr;
  ncclResult_t (*get_version)(int *) = nullptr;
};

Nccl g_nccl;

int nccl_load() {
  if (g_nccl.h) return BWPP_CUDA_OK;
  const char *lib = getenv("BWPP_NCCL_LIBRARY");  // another NCCL build, if the caller names one
  void *h = dlopen(lib && *lib ? lib : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return BWPP_CUDA_ERR_UNSUPPORTED;
  Nccl n;
  n.h = h;
  n.get_unique_id = (decltype(n.get_unique_id))dlsym(h, "ncclGetUniqueId");
  n.comm_init_rank = (decltype(n.comm_init_rank))dlsym(h, "ncclCommInitRank");
  n.all_reduce = (decltype(n.all_reduce))dlsym(h, "ncclAllReduce");
  n.all_gather = (decltype(n.all_gather))dlsym(h, "ncclAllGather");
  n.comm_destroy = (decltype(n.comm_destroy))dlsym(h, "ncclCommDestroy");
  n.comm_abort = (decltype(n.comm_abort))dlsym(h, "ncclCommAbort");
  n.get_async_error = (decltype(n.get_async_error))dlsym(h, "ncclCommGetAsyncError");
  n.error_string = (decltype(n.error_string))dlsym(h, "ncclGetErrorString");
  n.comm_init_rank_config =
      (decltype(n.comm_init_rank_config))dlsym(h, "ncclCommInitRankConfig");
  n.comm_finalize = (decltype(n.comm_finalize))dlsym(h, "ncclCommFinalize");
  n.get_version = (decltype(n.get_version))dlsym(h, "ncclGetVersion");
  if (!n.get_unique_id || !n.comm_init_rank || !n.all_reduce || !n.comm_destroy)
    return BWPP_CUDA_ERR_UNSUPPORTED;
  g_nccl = n;
  return BWPP_CUDA_OK;
}

}  // namespace

struct BwppCudaComm {
  ncclComm_t comm;
  int rank, nranks, device;
  uint32_t timeout_ms;  // bound of every wait on the communicator
  cudaEvent_t last;     // recorded after the latest collective
  int pending;          // `last` not yet seen complete
  int aborted;
};

namespace {

uint64_t now_ns() {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
}

void sleep_us(long us) {
  struct timespec ts = {0, us * 1000};
  nanosleep(&ts, nullptr);
}

// Watchdog callbacks of a live communicator: the last collective's event and
// NCCL's asynchronous error state.
int comm_done(void *u) {
  BwppCudaComm *c = (BwppCudaComm *)u;
  const cudaError_t e = cudaEventQuery(c->last);
  if (e == cudaSuccess) return 1;
  if (e == cudaErrorNotReady) return 0;
  cudaGetLastError();
  return -1;
}

int comm_error(void *u) {
  BwppCudaComm *c = (BwppCudaComm *)u;
  if (!g_nccl.get_async_error) return 0;
  ncclResult_t r = 0;
  if (g_nccl.get_async_error(c->comm, &r) != 0) return 2;
  return r == 0 ? 0 : r == kNcclInProgress ? 1 : 2;
}

void comm_abort(void *u) {
  BwppCudaComm *c = (BwppCudaComm *)u;
  if (c->aborted) return;
  c->aborted = 1;
  if (g_nccl.comm_abort) g_nccl.comm_abort(c->comm);
  else g_nccl.comm_destroy(c->comm);
  c->comm = nullptr;
}

// Polls NCCL's async state until it leaves "in progress" (non-blocking init
// and enqueue), bounded.
int comm_settle(BwppCudaComm *c) {
  const uint64_t t0 = now_ns();
  while (true) {
    const int e = comm_error(c);
    if (e == 0) return BWPP_CUDA_OK;
    if (e == 2) {
      comm_abort(c);
      return BWPP_CUDA_ERR;
    }
    if (now_ns() - t0 > (uint64_t)c->timeout_ms * 1000000ull) {
      comm_abort(c);
      return BWPP_CUDA_ERR_TIMEOUT;
    }
    sleep_us(100);
  }
}

int comm_wait_last(BwppCudaComm *c) {
  if (c->aborted) return BWPP_CUDA_ERR;
  if (!c->pending) return BWPP_CUDA_OK;
  const int rc = bwpp_cuda_comm_watch(comm_done, comm_error, comm_abort, c, c->timeout_ms);
  if (rc == BWPP_CUDA_OK) c->pending = 0;
  return rc;
}

}  // namespace

extern "C" {

int bwpp_cuda_comm_watch(int (*done)(void *), int (*error)(void *), void (*abort_fn)(void *),
                         void *user, uint32_t timeout_ms) {
  if (!done || !abort_fn) return BWPP_CUDA_ERR_ARG;
  const uint64_t t0 = now_ns(), limit = (uint64_t)timeout_ms * 1000000ull;
  long nap = 10;  // polling interval: 10 us, growing to 160 us (a late wake-up only delays
                  // queueing the next collective, which the GPU is usually still busy before)
  while (true) {
    const int e = error ? error(user) : 0;
    if (e != 0 && e != 1) {
      abort_fn(user);
      return BWPP_CUDA_ERR;
    }
    const int d = done(user);
    if (d > 0) return BWPP_CUDA_OK;
    if (d < 0) {
      abort_fn(user);
      return BWPP_CUDA_ERR_CUDA;
    }
    if (now_ns() - t0 >= limit) {
      abort_fn(user);
      return BWPP_CUDA_ERR_TIMEOUT;
    }
    sleep_us(nap);
    if (nap < 160) nap *= 2;
  }
}

int bwpp_cuda_comm_unique_id(unsigned char *id128) {
  if (!id128) return BWPP_CUDA_ERR_ARG;
  int rc = nccl_load();
  if (rc) return rc;
  ncclUniqueId id;
  if (g_nccl.get_unique_id(&id) != 0) return BWPP_CUDA_ERR;
  memcpy(id128, id.internal, 128);
  return BWPP_CUDA_OK;
}

int bwpp_cuda_comm_create_timeout(BwppCudaComm **out, const unsigned char *id128, int rank,
                                  int nranks, int device, uint32_t timeout_ms) {
  if (!out || !id128 || nranks < 1 || rank < 0 || rank >= nranks || timeout_ms == 0)
    return BWPP_CUDA_ERR_ARG;
  *out = nullptr;
  int rc = nccl_load();
  if (rc) return rc;
  if (cudaSetDevice(device) != cudaSuccess) return BWPP_CUDA_ERR_CUDA;
  BwppCudaComm *bc = (BwppCudaComm *)calloc(1, sizeof(BwppCudaComm));
  if (!bc) return BWPP_CUDA_ERR;
  bc->rank = rank;
  bc->nranks = nranks;
  bc->device = device;
  bc->timeout_ms = timeout_ms;
  if (cudaEventCreateWithFlags(&bc->last, cudaEventDisableTiming) != cudaSuccess) {
    cudaGetLastError();
    free(bc);
    return BWPP_CUDA_ERR_CUDA;
  }
  ncclUniqueId id;
  memcpy(id.internal, id128, 128);
  ncclResult_t r;
  if (g_nccl.comm_init_rank_config) {
    // non-blocking: init proceeds in the background; a rank that never
    // joins ends it after the timeout instead of blocking this thread
    NcclConfig cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.size = sizeof(NcclConfig);
    cfg.magic = 0xcafebeef;
    cfg.version = 22809;  // the layout above (NCCL 2.28.9)
    int lib_version = 0;
    if (g_nccl.get_version && g_nccl.get_version(&lib_version) == 0 && lib_version > 0 &&
        lib_version < 22809)
      cfg.version = (unsigned)lib_version;  // an older library reads its own prefix
    cfg.blocking = 0;
    cfg.cgaClusterSize = cfg.minCTAs = cfg.maxCTAs = kUndefInt;
    cfg.netName = nullptr;
    cfg.splitShare = cfg.trafficClass = kUndefInt;
    cfg.commName = nullptr;
    cfg.collnetEnable = cfg.CTAPolicy = cfg.shrinkShare = cfg.nvlsCTAs = kUndefInt;
    cfg.nChannelsPerNetPeer = cfg.nvlinkCentricSched = kUndefInt;
    r = g_nccl.comm_init_rank_config(&bc->comm, nranks, id, rank, &cfg);
    if (r != 0 && r != kNcclInProgress) {
      cudaEventDestroy(bc->last);
      free(bc);
      return BWPP_CUDA_ERR;
    }
    rc = comm_settle(bc);
    if (rc) {
      cudaEventDestroy(bc->last);
      free(bc);
      return rc;
    }
  } else {
    r = g_nccl.comm_init_rank(&bc->comm, nranks, id, rank);
    if (r != 0) {
      cudaEventDestroy(bc->last);
      free(bc);
      return BWPP_CUDA_ERR;
    }
  }
  *out = bc;
  return BWPP_CUDA_OK;
}

int bwpp_cuda_comm_create(BwppCudaComm **out, const unsigned char *id128, int rank,
                          int nranks, int device) {
  return bwpp_cuda_comm_create_timeout(out, id128, rank, nranks, device, 120000u);
}

int bwpp_cuda_comm_set_timeout(BwppCudaComm *c, uint32_t timeout_ms) {
  if (!c || timeout_ms == 0) return BWPP_CUDA_ERR_ARG;
  c->timeout_ms = timeout_ms;
  return BWPP_CUDA_OK;
}

int bwpp_cuda_comm_allreduce_sum_f32(BwppCudaComm *c, float *buf, size_t count, void *stream) {
  if (!c || (!buf && count)) return BWPP_CUDA_ERR_ARG;
  if (c->aborted) return BWPP_CUDA_ERR;
  if (count == 0) return BWPP_CUDA_OK;
  // the previous collective has finished (bounded) before the next is queued
  int rc = comm_wait_last(c);
  if (rc) return rc;
  const ncclResult_t r = g_nccl.all_reduce(buf, buf, count, kNcclFloat32, kNcclSum, c->comm,
                                           (cudaStream_t)stream);
  if (r == kNcclInProgress) {
    rc = comm_settle(c);
    if (rc) return rc;
  } else if (r != 0) {
    comm_abort(c);
    return BWPP_CUDA_ERR;
  }
  if (cudaEventRecord(c->last, (cudaStream_t)stream) != cudaSuccess) {
    cudaGetLastError();
    return BWPP_CUDA_ERR_CUDA;
  }
  c->pending = 1;
  return BWPP_CUDA_OK;
}

int bwpp_cuda_comm_wait(BwppCudaComm *c) {
  if (!c) return BWPP_CUDA_ERR_ARG;
  return comm_wait_last(c);
}

int bwpp_cuda_comm_aborted(const BwppCudaComm *c) { return c ? c->aborted : 1; }

int bwpp_cuda_comm_destroy(BwppCudaComm *c) {
  if (!c) return BWPP_CUDA_ERR_ARG;
  if (c->comm && !c->aborted) {
    // a collective still running has a bounded time to end; then the
    // communicator is finalized (non-blocking: settled, bounded) or aborted
    if (comm_wait_last(c) == BWPP_CUDA_OK && g_nccl.comm_finalize) {
      const ncclResult_t r = g_nccl.comm_finalize(c->comm);
      if (r == kNcclInProgress) comm_settle(c);
      else if (r != 0) comm_abort(c);
    }
    if (c->comm && !c->aborted) g_nccl.comm_destroy(c->comm);
  }
  cudaEventDestroy(c->last);
  free(c);
  return BWPP_CUDA_OK;
}

}  // extern "C"

// Ranks of the communicator (for the training step's gradient averaging).
int bwpp_comm_nranks(const BwppCudaComm *c) { return c ? c->nranks : 1; }
int bwpp_comm_rank(const BwppCudaComm *c) { return c ? c->rank : 0; }
int bwpp_comm_device(const BwppCudaComm *c) { return c ? c->device : -1; }

// In-place all-gather of `bytes` per rank on `stream`: rank r's part sits at
// buf + r * bytes.  Same bounded hand-off as the allreduce.
int bwpp_comm_allgather_bytes(BwppCudaComm *c, void *buf, size_t bytes, cudaStream_t stream) {
  if (!c || (!buf && bytes)) return BWPP_CUDA_ERR_ARG;
  if (c->aborted) return BWPP_CUDA_ERR;
  if (!g_nccl.all_gather) return BWPP_CUDA_ERR_UNSUPPORTED;
  if (bytes == 0) return BWPP_CUDA_OK;
  int rc = comm_wait_last(c);
  if (rc) return rc;
  uint8_t *base = static_cast<uint8_t *>(buf);
  const ncclResult_t r = g_nccl.all_gather(base + (size_t)c->rank * bytes, base, bytes, kNcclUint8,
                                           c->comm, stream);
  if (r == kNcclInProgress) {
    rc = comm_settle(c);
    if (rc) return rc;
  } else if (r != 0) {
    comm_abort(c);
    return BWPP_CUDA_ERR;
  }
  if (cudaEventRecord(c->last, stream) != cudaSuccess) {
    cudaGetLastError();
    return BWPP_CUDA_ERR_CUDA;
  }
  c->pending = 1;
  return BWPP_CUDA_OK;
}
