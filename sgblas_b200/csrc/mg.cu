// Multi-GPU column-sharded SGEMM (include/sgblas/sgblas_mg.h).
//
// No counterpart in the reference (single-GPU library). One process or thread
// per GPU; A travels from the root to every rank with one in-place
// ncclBroadcast over NVLink/NVSwitch, then each rank runs the single-GPU
// sgblasSgemm on its column block of B and C. NCCL is resolved with dlopen at
// the first sgblasMgCreate, so libsgblas.so itself has no NCCL dependency.
// The remote data always lands in local HBM before a kernel reads it; no
// kernel reads peer memory.
#include "context.hpp"
#include "validation.hpp"

#include <sgblas/sgblas_mg.h>

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <new>

namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
};

template <typename F>
bool resolve(void *dl, const char *name, F *fn) {
  *fn = reinterpret_cast<F>(dlsym(dl, name));
  return *fn != nullptr;
}

const NcclApi *nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *dl = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (dl == nullptr) dl = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (dl == nullptr) return;
    api.ok = resolve(dl, "ncclGetUniqueId", &api.getUniqueId) &&
             resolve(dl, "ncclCommInitRank", &api.commInitRank) &&
             resolve(dl, "ncclCommDestroy", &api.commDestroy) &&
             resolve(dl, "ncclCommAbort", &api.commAbort) &&
             resolve(dl, "ncclBroadcast", &api.broadcast) &&
             resolve(dl, "ncclAllGather", &api.allGather);
  });
  return api.ok ? &api : nullptr;
}

}  // namespace

struct sgblasMgContext {
  ncclComm_t comm = nullptr;
  int rank = 0;
  int nranks = 1;
  int device = 0;
  sgblasHandle_t inner = nullptr;
  cudaStream_t stream = nullptr;
};

extern "C" sgblasStatus_t sgblasMgGetUniqueId(unsigned char id[SGBLAS_MG_UNIQUE_ID_BYTES]) {
  if (id == nullptr) return SGBLAS_STATUS_INVALID_VALUE;
  const NcclApi *api = nccl();
  if (api == nullptr) return SGBLAS_STATUS_NOT_SUPPORTED;
  static_assert(sizeof(ncclUniqueId) == SGBLAS_MG_UNIQUE_ID_BYTES, "NCCL id size");
  ncclUniqueId uid;
  if (api->getUniqueId(&uid) != ncclSuccess) return SGBLAS_STATUS_INTERNAL_ERROR;
  std::memcpy(id, &uid, sizeof(uid));
  return SGBLAS_STATUS_SUCCESS;
}

extern "C" sgblasStatus_t sgblasMgCreate(sgblasMgHandle_t *handle, int nranks, int rank,
                                         const unsigned char id[SGBLAS_MG_UNIQUE_ID_BYTES],
                                         int device) {
  if (handle == nullptr || id == nullptr || nranks < 1 || rank < 0 || rank >= nranks ||
      device < 0)
    return SGBLAS_STATUS_INVALID_VALUE;
  *handle = nullptr;
  const NcclApi *api = nccl();
  if (api == nullptr) return SGBLAS_STATUS_NOT_SUPPORTED;
  if (cudaSetDevice(device) != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_INVALID_VALUE;
  }
  auto *ctx = new (std::nothrow) sgblasMgContext{};
  if (ctx == nullptr) return SGBLAS_STATUS_ALLOC_FAILED;
  ctx->rank = rank;
  ctx->nranks = nranks;
  ctx->device = device;
  if (sgblasCreate(&ctx->inner) != SGBLAS_STATUS_SUCCESS) {
    delete ctx;
    return SGBLAS_STATUS_ALLOC_FAILED;
  }
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  if (api->commInitRank(&ctx->comm, nranks, uid, rank) != ncclSuccess) {
    sgblasDestroy(ctx->inner);
    delete ctx;
    return SGBLAS_STATUS_INTERNAL_ERROR;
  }
  *handle = ctx;
  return SGBLAS_STATUS_SUCCESS;
}

extern "C" sgblasStatus_t sgblasMgDestroy(sgblasMgHandle_t handle) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  const NcclApi *api = nccl();
  sgblasStatus_t status = SGBLAS_STATUS_SUCCESS;
  if (api != nullptr && handle->comm != nullptr && api->commDestroy(handle->comm) != ncclSuccess)
    status = SGBLAS_STATUS_INTERNAL_ERROR;
  sgblasDestroy(handle->inner);
  delete handle;
  return status;
}

extern "C" sgblasStatus_t sgblasMgSetStream(sgblasMgHandle_t handle, sgblasStream_t stream) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  handle->stream = static_cast<cudaStream_t>(stream);
  return sgblasSetStream(handle->inner, stream);
}

extern "C" sgblasStatus_t sgblasMgSetMathMode(sgblasMgHandle_t handle, sgblasMathMode_t mode) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  return sgblasSetMathMode(handle->inner, mode);
}

extern "C" sgblasStatus_t sgblasMgGetRank(sgblasMgHandle_t handle, int *rank, int *nranks) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  if (rank == nullptr || nranks == nullptr) return SGBLAS_STATUS_INVALID_VALUE;
  *rank = handle->rank;
  *nranks = handle->nranks;
  return SGBLAS_STATUS_SUCCESS;
}

extern "C" sgblasStatus_t sgblasMgSgemm(sgblasMgHandle_t handle, sgblasOperation_t transa,
                                        sgblasOperation_t transb, int m, int n_local, int k,
                                        const float *alpha, float *a, int lda, int root,
                                        const float *b, int ldb, const float *beta, float *c,
                                        int ldc) {
  using namespace sgblas::detail;
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  if (root < 0 || root >= handle->nranks) return SGBLAS_STATUS_INVALID_VALUE;
  SgemmPlan plan;
  const sgblasStatus_t status =
      validate(transa, transb, m, n_local, k, alpha, a, lda, b, ldb, beta, c, ldc, &plan);
  if (status != SGBLAS_STATUS_SUCCESS) return status;
  // Whether A is needed is a property of the whole problem (identical on every
  // rank), not of this rank's shard, so every rank takes the same collective.
  const bool product = m > 0 && k > 0 && alpha != nullptr && *alpha != 0.0F;
  if (product) {
    if (a == nullptr) return SGBLAS_STATUS_INVALID_VALUE;
    const NcclApi *api = nccl();
    if (api == nullptr) return SGBLAS_STATUS_NOT_SUPPORTED;
    const size_t count = static_cast<size_t>(lda) *
                         static_cast<size_t>(transa == SGBLAS_OP_N ? k : m);
    if (api->broadcast(a, a, count, ncclFloat32, root, handle->comm, handle->stream) !=
        ncclSuccess)
      return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  if (plan.work == Work::kNothing) return SGBLAS_STATUS_SUCCESS;
  return sgblasSgemm(handle->inner, transa, transb, m, n_local, k, alpha, a, lda, b, ldb, beta, c,
                     ldc);
}

extern "C" sgblasStatus_t sgblasMgAllGather(sgblasMgHandle_t handle, const float *send,
                                            float *recv, size_t count) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  if (count > 0 && (send == nullptr || recv == nullptr)) return SGBLAS_STATUS_INVALID_VALUE;
  const NcclApi *api = nccl();
  if (api == nullptr) return SGBLAS_STATUS_NOT_SUPPORTED;
  if (api->allGather(send, recv, count, ncclFloat32, handle->comm, handle->stream) != ncclSuccess)
    return SGBLAS_STATUS_EXECUTION_FAILED;
  return SGBLAS_STATUS_SUCCESS;
}
