// NCCL communicator for the data-parallel gradient allreduce of the
// tiny_model training step -- the only collective of the hot path.
//
// NCCL is resolved at run time with dlopen("libnccl.so.2"): when the process
// already has NCCL loaded (torch.distributed does), the same copy is used, so
// there is never a second NCCL in the process.  Only the handful of symbols
// below are used; their signatures are NCCL's public C API.
#include <dlfcn.h>
#include <stdlib.h>
#include <string.h>

#include "bwpp_cuda_internal.cuh"

namespace {

typedef struct ncclComm *ncclComm_t;
typedef struct {
  char internal[128];
} ncclUniqueId;
typedef int ncclResult_t;  // 0 = ncclSuccess
constexpr int kNcclFloat32 = 7;
constexpr int kNcclSum = 0;

struct Nccl {
  void *h = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, int, int, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t *) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
};

Nccl g_nccl;

int nccl_load() {
  if (g_nccl.h) return BWPP_CUDA_OK;
  void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return BWPP_CUDA_ERR_UNSUPPORTED;
  Nccl n;
  n.h = h;
  n.get_unique_id = (decltype(n.get_unique_id))dlsym(h, "ncclGetUniqueId");
  n.comm_init_rank = (decltype(n.comm_init_rank))dlsym(h, "ncclCommInitRank");
  n.all_reduce = (decltype(n.all_reduce))dlsym(h, "ncclAllReduce");
  n.comm_destroy = (decltype(n.comm_destroy))dlsym(h, "ncclCommDestroy");
  n.comm_abort = (decltype(n.comm_abort))dlsym(h, "ncclCommAbort");
  n.get_async_error = (decltype(n.get_async_error))dlsym(h, "ncclCommGetAsyncError");
  n.error_string = (decltype(n.error_string))dlsym(h, "ncclGetErrorString");
  if (!n.get_unique_id || !n.comm_init_rank || !n.all_reduce || !n.comm_destroy)
    return BWPP_CUDA_ERR_UNSUPPORTED;
  g_nccl = n;
  return BWPP_CUDA_OK;
}

}  // namespace

struct BwppCudaComm {
  ncclComm_t comm;
  int rank, nranks, device;
};

extern "C" {

int bwpp_cuda_comm_unique_id(unsigned char *id128) {
  if (!id128) return BWPP_CUDA_ERR_ARG;
  int rc = nccl_load();
  if (rc) return rc;
  ncclUniqueId id;
  if (g_nccl.get_unique_id(&id) != 0) return BWPP_CUDA_ERR;
  memcpy(id128, id.internal, 128);
  return BWPP_CUDA_OK;
}

int bwpp_cuda_comm_create(BwppCudaComm **out, const unsigned char *id128, int rank,
                          int nranks, int device) {
  if (!out || !id128 || nranks < 1 || rank < 0 || rank >= nranks) return BWPP_CUDA_ERR_ARG;
  *out = nullptr;
  int rc = nccl_load();
  if (rc) return rc;
  if (cudaSetDevice(device) != cudaSuccess) return BWPP_CUDA_ERR_CUDA;
  ncclUniqueId id;
  memcpy(id.internal, id128, 128);
  ncclComm_t c = nullptr;
  if (g_nccl.comm_init_rank(&c, nranks, id, rank) != 0) return BWPP_CUDA_ERR;
  BwppCudaComm *bc = (BwppCudaComm *)calloc(1, sizeof(BwppCudaComm));
  if (!bc) {
    g_nccl.comm_destroy(c);
    return BWPP_CUDA_ERR;
  }
  bc->comm = c;
  bc->rank = rank;
  bc->nranks = nranks;
  bc->device = device;
  *out = bc;
  return BWPP_CUDA_OK;
}

int bwpp_cuda_comm_allreduce_sum_f32(BwppCudaComm *c, float *buf, size_t count, void *stream) {
  if (!c || (!buf && count)) return BWPP_CUDA_ERR_ARG;
  if (count == 0) return BWPP_CUDA_OK;
  return g_nccl.all_reduce(buf, buf, count, kNcclFloat32, kNcclSum, c->comm,
                           (cudaStream_t)stream) == 0
             ? BWPP_CUDA_OK
             : BWPP_CUDA_ERR;
}

int bwpp_cuda_comm_destroy(BwppCudaComm *c) {
  if (!c) return BWPP_CUDA_ERR_ARG;
  if (c->comm) g_nccl.comm_destroy(c->comm);
  free(c);
  return BWPP_CUDA_OK;
}

}  // extern "C"

// Ranks of the communicator (for the training step's gradient averaging).
int bwpp_comm_nranks(const BwppCudaComm *c) { return c ? c->nranks : 1; }
