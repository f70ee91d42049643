// Multi-GPU column-sharded SGEMM (include/sgblas/sgblas_mg.h).
//
// No counterpart in the reference, which is a single-GPU library (its
// docs/design.md:102 lists distributed execution as a non-goal).
//
// Rank p computes C_p = alpha * op(A) * op(B)_p + beta * C_p on its column
// block; A travels from the root to every rank. The broadcast runs on the
// GPUs' copy engines, not in NCCL kernels, so that it overlaps the local
// products: the persistent SGEMM kernel holds every SM, and a collective
// kernel queued behind it would wait for it to finish.
//
//   - The ranks form a chain that starts at the root (position (rank - root)
//     mod nranks). Each rank pushes A, one panel of rows of op(A) at a time,
//     into its child's staging buffer (library-owned device memory, mapped
//     into the parent with CUDA IPC) with cudaMemcpy2DAsync -- a copy engine
//     over NVLink -- and then writes the call's sequence number into the
//     child's flag for that panel.
//   - The child's compute stream waits for the flag (cuStreamWaitValue32; no
//     SM is involved) and computes that panel's rows of C while later panels
//     are still on their way. Panels grow (512, 1024, 2048 rows, then about
//     4096), so the last rank of the chain starts after a few hops of a small
//     panel, and later products are large. Row panels keep each output's
//     whole k sum in one kernel: no extra pass over C.
//   - A parent pushes call s into its child's staging only after the child
//     has announced, at the start of its own call s, that its staging is
//     free (every earlier use of it is done).
//   - The flags live in one small block of host shared memory per
//     communicator, registered with CUDA. Stream memory operations write and
//     wait on it; the host can read and write it directly. That is what lets
//     sgblasMgAbort release every wait without a stream of its own, and it
//     carries the start-up exchange of IPC handles. All ranks therefore run
//     on one host.
// Remote data always lands in local HBM before a kernel reads it: no kernel
// reads peer memory, and nothing uses TMA multicast. NCCL is loaded at run
// time for the communicator (sgblasMgAllGather); its initialisation runs
// non-blocking under a deadline.
#include "context.hpp"
#include "validation.hpp"

#include <sgblas/sgblas_mg.h>

#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <fcntl.h>
#include <nccl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

namespace {

using Clock = std::chrono::steady_clock;

constexpr int kMaxPanels = 16;
constexpr int kMaxRanks = 64;
constexpr int kDefaultTimeoutMs = 300000;
constexpr uint32_t kShmMagic = 0x53474d47u;    // "SGMG"
constexpr uint32_t kReleaseDistance = 1u << 30; // an abort moves every flag this far ahead

// ---- NCCL, resolved at run time ---------------------------------------------
struct NcclApi {
  bool ok = false;
  ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*commInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int,
                                     ncclConfig_t *) = nullptr;
  ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*commFinalize)(ncclComm_t) = nullptr;   // optional
  ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
};

template <typename F>
bool resolve(void *dl, const char *name, F *fn) {
  *fn = reinterpret_cast<F>(dlsym(dl, name));
  return *fn != nullptr;
}

// SGBLAS_NCCL_LIBRARY names another NCCL build (or a stand-in the tests use
// to make initialisation fail or never finish).
const NcclApi *nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    const char *path = std::getenv("SGBLAS_NCCL_LIBRARY");
    void *dl = nullptr;
    if (path != nullptr && *path != '\0') {
      dl = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    } else {
      dl = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
      if (dl == nullptr) dl = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    }
    if (dl == nullptr) return;
    api.ok = resolve(dl, "ncclGetUniqueId", &api.getUniqueId) &&
             resolve(dl, "ncclCommInitRankConfig", &api.commInitRankConfig) &&
             resolve(dl, "ncclCommGetAsyncError", &api.commGetAsyncError) &&
             resolve(dl, "ncclCommDestroy", &api.commDestroy) &&
             resolve(dl, "ncclCommAbort", &api.commAbort) &&
             resolve(dl, "ncclAllGather", &api.allGather);
    (void)resolve(dl, "ncclCommFinalize", &api.commFinalize);
  });
  return api.ok ? &api : nullptr;
}

// A non-blocking communicator reports ncclInProgress while an operation
// (initialisation, an enqueue) is still running. Polls until it settles or
// the deadline passes (*expired).
ncclResult_t settle(const NcclApi *api, ncclComm_t comm, ncclResult_t first,
                    Clock::time_point deadline, bool *expired) {
  *expired = false;
  ncclResult_t r = first;
  while (r == ncclInProgress) {
    if (Clock::now() >= deadline) {
      *expired = true;
      return r;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
    if (api->commGetAsyncError(comm, &r) != ncclSuccess) return ncclInternalError;
  }
  return r;
}

// ---- stream memory operations (driver API, fetched through the runtime) ------
using WaitValue32Fn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
using WriteValue32Fn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

struct MemOps {
  WaitValue32Fn wait = nullptr;
  WriteValue32Fn write = nullptr;
};

const MemOps *memOps() {
  static MemOps ops;
  static std::once_flag once;
  std::call_once(once, [] {
    auto get = [](const char *name) -> void * {
      void *f = nullptr;
      cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
      if (cudaGetDriverEntryPointByVersion(name, &f, 12000, cudaEnableDefault, &q) !=
              cudaSuccess ||
          q != cudaDriverEntryPointSuccess) {
        (void)cudaGetLastError();
        return nullptr;
      }
      return f;
    };
    ops.wait = reinterpret_cast<WaitValue32Fn>(get("cuStreamWaitValue32"));
    ops.write = reinterpret_cast<WriteValue32Fn>(get("cuStreamWriteValue32"));
  });
  return ops.wait != nullptr && ops.write != nullptr ? &ops : nullptr;
}

// ---- the shared signal block --------------------------------------------------
// What a rank publishes about one of its device buffers.
struct PeerRecord {
  cudaIpcMemHandle_t handle;
  uint64_t ptr;      // the raw address (used by peers in the same process)
  uint64_t bytes;
  int64_t pid;
  int32_t device;
  int32_t valid;
};

struct alignas(256) ShmSlot {
  // Written by stream memory operations, waited on by this rank's streams.
  volatile uint32_t panel[kMaxPanels];   // panel p of call s is in my staging: s
  volatile uint32_t ready;               // my child's staging is free for call s: s
  // Host-only: the start-up / growth exchange (double-buffered by generation).
  volatile uint32_t gen;
  PeerRecord rec[2];
};

struct ShmBlock {
  volatile uint32_t magic;
  volatile uint32_t nranks;
  volatile uint32_t aborted;
  ShmSlot slot[kMaxRanks];
};

// Name of the communicator's block: a hash of its NCCL unique id.
void shmName(const unsigned char *id, char *out, size_t size) {
  uint64_t h = 1469598103934665603ULL;
  for (int i = 0; i < SGBLAS_MG_UNIQUE_ID_BYTES; ++i) {
    h ^= id[i];
    h *= 1099511628211ULL;
  }
  std::snprintf(out, size, "/sgblas-mg-%016llx", static_cast<unsigned long long>(h));
}

int timeoutMs() {
  const char *v = std::getenv("SGBLAS_MG_TIMEOUT_MS");
  if (v == nullptr) return kDefaultTimeoutMs;
  const long t = std::strtol(v, nullptr, 10);
  return t > 0 && t < (1L << 30) ? static_cast<int>(t) : kDefaultTimeoutMs;
}

}  // namespace

struct sgblasMgContext {
  ncclComm_t comm = nullptr;
  int rank = 0;
  int nranks = 1;
  int device = 0;
  int timeout_ms = kDefaultTimeoutMs;
  sgblasHandle_t inner = nullptr;
  cudaStream_t stream = nullptr;     // the caller's stream (products, signals)
  cudaStream_t copy = nullptr;       // the chain's copies and their waits
  cudaEvent_t ev_start = nullptr;    // caller stream -> copy stream, per call
  cudaEvent_t ev_copies = nullptr;   // copy stream -> caller stream, per call
  ShmBlock *shm = nullptr;           // host address of the signal block
  size_t shm_bytes = 0;
  char *shm_dev = nullptr;           // device address of the signal block
  bool flush = false;                // waits flush remote writes first
  uint32_t seq = 0;                  // calls that used the chain
  uint32_t gen = 0;                  // exchanges
  float *staging = nullptr;          // where the parent pushes A
  size_t staging_bytes = 0;
  std::vector<float *> peer_staging;   // every rank's staging, mapped here
  std::vector<char> peer_ipc;          // 1 when mapped with cudaIpcOpenMemHandle
  bool aborted = false;
};

namespace {

bool deadlinePassed(Clock::time_point deadline) { return Clock::now() >= deadline; }

// Publishes `mine` and collects every rank's record (host shared memory; the
// generation counter doubles as a barrier). False when a rank did not arrive
// before the deadline, or the communicator was aborted.
bool exchange(sgblasMgContext *ctx, const PeerRecord &mine, std::vector<PeerRecord> *all) {
  const uint32_t gen = ++ctx->gen;
  ShmSlot &me = ctx->shm->slot[ctx->rank];
  std::memcpy(const_cast<PeerRecord *>(&me.rec[gen & 1]), &mine, sizeof(mine));
  __atomic_store_n(&me.gen, gen, __ATOMIC_RELEASE);
  const auto deadline = Clock::now() + std::chrono::milliseconds(ctx->timeout_ms);
  all->assign(ctx->nranks, PeerRecord{});
  for (int r = 0; r < ctx->nranks; ++r) {
    const ShmSlot &s = ctx->shm->slot[r];
    while (static_cast<int32_t>(__atomic_load_n(&s.gen, __ATOMIC_ACQUIRE) - gen) < 0) {
      if (ctx->shm->aborted != 0 || deadlinePassed(deadline)) return false;
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    std::memcpy(&(*all)[r], const_cast<const PeerRecord *>(&s.rec[gen & 1]), sizeof(PeerRecord));
  }
  return true;
}

// Waits for `stream` to drain, at most until the deadline.
bool drain(cudaStream_t stream, Clock::time_point deadline) {
  for (;;) {
    const cudaError_t e = cudaStreamQuery(stream);
    if (e == cudaSuccess) return true;
    if (e != cudaErrorNotReady) {
      (void)cudaGetLastError();
      return false;
    }
    if (deadlinePassed(deadline)) return false;
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

void unmapPeers(sgblasMgContext *ctx) {
  for (size_t r = 0; r < ctx->peer_staging.size(); ++r) {
    if (ctx->peer_ipc[r] != 0 && ctx->peer_staging[r] != nullptr)
      (void)cudaIpcCloseMemHandle(ctx->peer_staging[r]);
  }
  ctx->peer_staging.assign(ctx->nranks, nullptr);
  ctx->peer_ipc.assign(ctx->nranks, 0);
  (void)cudaGetLastError();
}

// Maps another rank's buffer: its raw address in the same process, else
// through CUDA IPC.
float *mapPeer(const sgblasMgContext *ctx, const PeerRecord &rec, char *ipc) {
  *ipc = 0;
  if (rec.valid == 0) return nullptr;
  if (rec.pid == static_cast<int64_t>(getpid())) {
    if (rec.device != ctx->device) {
      const cudaError_t e = cudaDeviceEnablePeerAccess(rec.device, 0);
      if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) {
        (void)cudaGetLastError();
        return nullptr;
      }
      (void)cudaGetLastError();
    }
    return reinterpret_cast<float *>(rec.ptr);
  }
  void *p = nullptr;
  if (cudaIpcOpenMemHandle(&p, rec.handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  *ipc = 1;
  return static_cast<float *>(p);
}

// Staging of at least `bytes` on every rank, mapped by every other rank.
// Collective: every rank reaches it on the same call, since the size depends
// only on arguments all ranks share. Growing drains this rank's streams
// (blocking the host, at most the timeout).
sgblasStatus_t ensureStaging(sgblasMgContext *ctx, size_t bytes) {
  if (ctx->staging_bytes >= bytes) return SGBLAS_STATUS_SUCCESS;
  const auto deadline = Clock::now() + std::chrono::milliseconds(ctx->timeout_ms);
  if (!drain(ctx->stream, deadline) || !drain(ctx->copy, deadline))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  unmapPeers(ctx);
  if (ctx->staging != nullptr) (void)cudaFree(ctx->staging);
  ctx->staging = nullptr;
  ctx->staging_bytes = 0;
  const size_t want = (bytes + bytes / 4 + (size_t{2} << 20) - 1) / (size_t{2} << 20) *
                      (size_t{2} << 20);
  PeerRecord mine = {};
  void *p = nullptr;
  if (cudaMalloc(&p, want) == cudaSuccess && cudaIpcGetMemHandle(&mine.handle, p) == cudaSuccess) {
    ctx->staging = static_cast<float *>(p);
    ctx->staging_bytes = want;
    mine.ptr = reinterpret_cast<uint64_t>(p);
    mine.bytes = want;
    mine.valid = 1;
  } else {
    (void)cudaGetLastError();
    if (p != nullptr) (void)cudaFree(p);
    ctx->staging = nullptr;
  }
  mine.pid = getpid();
  mine.device = ctx->device;
  std::vector<PeerRecord> all;
  // Every rank takes part in the exchange even after a failed allocation, so
  // that all of them learn of it.
  if (!exchange(ctx, mine, &all)) return SGBLAS_STATUS_EXECUTION_FAILED;
  bool ok = true;
  for (int r = 0; r < ctx->nranks; ++r) {
    if (all[r].valid == 0 || all[r].bytes < bytes) ok = false;
    if (r == ctx->rank || !ok) continue;
    ctx->peer_staging[r] = mapPeer(ctx, all[r], &ctx->peer_ipc[r]);
    if (ctx->peer_staging[r] == nullptr) ok = false;
  }
  if (!ok) {
    unmapPeers(ctx);
    if (ctx->staging != nullptr) (void)cudaFree(ctx->staging);
    ctx->staging = nullptr;
    ctx->staging_bytes = 0;
    return SGBLAS_STATUS_ALLOC_FAILED;
  }
  return SGBLAS_STATUS_SUCCESS;
}

// Row panels of op(A): [first, first + rows). A small A goes in one piece;
// otherwise 512, 1024 and 2048 rows, then the rest in at most
// kMaxPanels - 3 near-equal panels of about 4096 rows (multiples of 128).
struct Panel {
  int first, rows;
};

std::vector<Panel> planPanels(int m, size_t a_bytes, int nranks) {
  std::vector<Panel> out;
  constexpr size_t kSplitBytes = size_t{32} << 20;
  if (nranks == 1 || a_bytes < kSplitBytes || m < 1024) {
    out.push_back({0, m});
    return out;
  }
  int at = 0;
  for (int rows = 512; rows <= 2048 && m - at >= 2 * rows; rows *= 2) {
    out.push_back({at, rows});
    at += rows;
  }
  const int rest = m - at;
  const int count = std::max(1, std::min(kMaxPanels - static_cast<int>(out.size()),
                                          (rest + 4095) / 4096));
  const int step = (rest / count + 127) / 128 * 128;
  for (int i = 0; i < count && at < m; ++i) {
    const int rows = i == count - 1 ? m - at : std::min(step, m - at);
    out.push_back({at, rows});
    at += rows;
  }
  return out;
}

// Moves every flag of every rank far ahead of any call in flight (so that
// every wait returns) and marks the communicator aborted.
void releaseAll(sgblasMgContext *ctx) {
  ShmBlock *shm = ctx->shm;
  if (shm == nullptr) return;
  const uint32_t value = ctx->seq + kReleaseDistance;
  __atomic_store_n(&shm->aborted, 1u, __ATOMIC_RELEASE);
  for (int r = 0; r < ctx->nranks; ++r) {
    for (int p = 0; p < kMaxPanels; ++p)
      __atomic_store_n(&shm->slot[r].panel[p], value, __ATOMIC_RELEASE);
    __atomic_store_n(&shm->slot[r].ready, value, __ATOMIC_RELEASE);
  }
}

CUdeviceptr devAddr(const volatile uint32_t *p) {
  return static_cast<CUdeviceptr>(reinterpret_cast<uintptr_t>(p));
}

void destroyContext(sgblasMgContext *ctx, bool abort_comm) {
  const NcclApi *api = nccl();
  // After an abort anywhere in the communicator a peer may be gone: abort
  // rather than finalize (which waits for the other ranks' operations).
  if (ctx->shm != nullptr && ctx->shm->aborted != 0) abort_comm = true;
  if (api != nullptr && ctx->comm != nullptr && !abort_comm && api->commFinalize != nullptr) {
    bool expired = false;
    const auto deadline = Clock::now() + std::chrono::milliseconds(ctx->timeout_ms);
    const ncclResult_t started = api->commFinalize(ctx->comm);
    if (settle(api, ctx->comm, started, deadline, &expired) != ncclSuccess) abort_comm = true;
  }
  unmapPeers(ctx);
  if (ctx->staging != nullptr) (void)cudaFree(ctx->staging);
  if (ctx->shm != nullptr) {
    (void)cudaHostUnregister(ctx->shm);
    munmap(ctx->shm, ctx->shm_bytes);
  }
  if (ctx->ev_start != nullptr) (void)cudaEventDestroy(ctx->ev_start);
  if (ctx->ev_copies != nullptr) (void)cudaEventDestroy(ctx->ev_copies);
  if (ctx->copy != nullptr) (void)cudaStreamDestroy(ctx->copy);
  if (api != nullptr && ctx->comm != nullptr) {
    if (abort_comm) (void)api->commAbort(ctx->comm);
    else (void)api->commDestroy(ctx->comm);
  }
  if (ctx->inner != nullptr) sgblasDestroy(ctx->inner);
  (void)cudaGetLastError();
  delete ctx;
}

}  // namespace

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
  if (handle == nullptr || id == nullptr || nranks < 1 || nranks > kMaxRanks || rank < 0 ||
      rank >= nranks || device < 0)
    return SGBLAS_STATUS_INVALID_VALUE;
  *handle = nullptr;
  const NcclApi *api = nccl();
  if (api == nullptr) return SGBLAS_STATUS_NOT_SUPPORTED;
  if (cudaSetDevice(device) != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_INVALID_VALUE;
  }
  const MemOps *ops = memOps();
  if (ops == nullptr) return SGBLAS_STATUS_NOT_SUPPORTED;
  auto *ctx = new (std::nothrow) sgblasMgContext{};
  if (ctx == nullptr) return SGBLAS_STATUS_ALLOC_FAILED;
  ctx->rank = rank;
  ctx->nranks = nranks;
  ctx->device = device;
  ctx->timeout_ms = timeoutMs();
  ctx->peer_staging.assign(nranks, nullptr);
  ctx->peer_ipc.assign(nranks, 0);
  const auto deadline = Clock::now() + std::chrono::milliseconds(ctx->timeout_ms);
  if (sgblasCreate(&ctx->inner) != SGBLAS_STATUS_SUCCESS) {
    delete ctx;
    return SGBLAS_STATUS_ALLOC_FAILED;
  }
  // The communicator, initialised non-blocking: a rank that never joins ends
  // in an error at the deadline (the communicator is aborted), not a hang.
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  bool expired = false;
  const ncclResult_t started = api->commInitRankConfig(&ctx->comm, nranks, uid, rank, &config);
  const ncclResult_t init = started == ncclInProgress
                                ? settle(api, ctx->comm, started, deadline, &expired)
                                : started;
  if (init != ncclSuccess) {
    const bool have_comm = ctx->comm != nullptr;
    destroyContext(ctx, have_comm);
    return expired ? SGBLAS_STATUS_EXECUTION_FAILED : SGBLAS_STATUS_INTERNAL_ERROR;
  }
  // The signal block: every rank maps the same host pages and registers them.
  char name[64];
  shmName(id, name, sizeof(name));
  ctx->shm_bytes = (sizeof(ShmBlock) + 4095) / 4096 * 4096;
  const int fd = shm_open(name, O_CREAT | O_RDWR, 0600);
  bool ok = fd >= 0 && ftruncate(fd, static_cast<off_t>(ctx->shm_bytes)) == 0;
  void *map = ok ? mmap(nullptr, ctx->shm_bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0)
                 : MAP_FAILED;
  if (fd >= 0) close(fd);
  ok = map != MAP_FAILED;
  if (ok) {
    ctx->shm = static_cast<ShmBlock *>(map);
    ok = cudaHostRegister(map, ctx->shm_bytes, cudaHostRegisterMapped | cudaHostRegisterPortable) ==
         cudaSuccess;
    if (!ok) {
      (void)cudaGetLastError();
      munmap(map, ctx->shm_bytes);
      ctx->shm = nullptr;
    }
  }
  void *shm_dev = nullptr;
  ok = ok && cudaHostGetDevicePointer(&shm_dev, ctx->shm, 0) == cudaSuccess;
  ok = ok && cudaStreamCreateWithFlags(&ctx->copy, cudaStreamNonBlocking) == cudaSuccess &&
       cudaEventCreateWithFlags(&ctx->ev_start, cudaEventDisableTiming) == cudaSuccess &&
       cudaEventCreateWithFlags(&ctx->ev_copies, cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    (void)cudaGetLastError();
    if (fd >= 0 && rank == 0) shm_unlink(name);
    destroyContext(ctx, true);
    return SGBLAS_STATUS_ALLOC_FAILED;
  }
  ctx->shm_dev = static_cast<char *>(shm_dev);
  int flush = 0;
  if (cudaDeviceGetAttribute(&flush, cudaDevAttrCanFlushRemoteWrites, device) != cudaSuccess) {
    (void)cudaGetLastError();
    flush = 0;
  }
  ctx->flush = flush != 0;
  if (rank == 0) {
    ctx->shm->magic = kShmMagic;
    ctx->shm->nranks = static_cast<uint32_t>(nranks);
  }
  // Every rank has mapped the block once this exchange completes; then the
  // name can go (the mappings stay valid).
  PeerRecord hello = {};
  hello.pid = getpid();
  hello.device = device;
  hello.valid = 1;
  std::vector<PeerRecord> all;
  if (!exchange(ctx, hello, &all)) {
    if (rank == 0) shm_unlink(name);
    destroyContext(ctx, true);
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  if (rank == 0) shm_unlink(name);
  if (ctx->shm->magic != kShmMagic || ctx->shm->nranks != static_cast<uint32_t>(nranks)) {
    destroyContext(ctx, true);   // ranks disagree on the communicator size
    return SGBLAS_STATUS_INVALID_VALUE;
  }
  *handle = ctx;
  return SGBLAS_STATUS_SUCCESS;
}

extern "C" sgblasStatus_t sgblasMgDestroy(sgblasMgHandle_t handle) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  // Finish this rank's enqueued work before its buffers go. Work still
  // waiting for a peer at the deadline is released (every rank's waits),
  // which ends its products with undefined values.
  const auto deadline = Clock::now() + std::chrono::milliseconds(handle->timeout_ms);
  bool clean = !handle->aborted;
  clean = drain(handle->copy, deadline) && drain(handle->stream, deadline) && clean;
  if (!clean) {
    releaseAll(handle);
    const auto grace = Clock::now() + std::chrono::milliseconds(handle->timeout_ms);
    (void)drain(handle->copy, grace);
    (void)drain(handle->stream, grace);
  }
  destroyContext(handle, !clean);
  return clean ? SGBLAS_STATUS_SUCCESS : SGBLAS_STATUS_EXECUTION_FAILED;
}

extern "C" sgblasStatus_t sgblasMgAbort(sgblasMgHandle_t handle) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  handle->aborted = true;
  releaseAll(handle);
  const NcclApi *api = nccl();
  if (api != nullptr && handle->comm != nullptr) {
    (void)api->commAbort(handle->comm);
    handle->comm = nullptr;
  }
  return SGBLAS_STATUS_SUCCESS;
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
  sgblasMgContext *ctx = handle;
  if (ctx->aborted || (ctx->shm != nullptr && ctx->shm->aborted != 0))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  // Problem-wide arguments: identical on every rank, so every rank returns
  // the same error here, before any collective step.
  const bool op_ok = (transa == SGBLAS_OP_N || transa == SGBLAS_OP_T) &&
                     (transb == SGBLAS_OP_N || transb == SGBLAS_OP_T);
  if (!op_ok || m < 0 || k < 0 || root < 0 || root >= ctx->nranks ||
      lda < std::max(1, transa == SGBLAS_OP_N ? m : k))
    return SGBLAS_STATUS_INVALID_VALUE;
  if (m > 0 && (alpha == nullptr || beta == nullptr)) return SGBLAS_STATUS_INVALID_VALUE;
  const bool product = m > 0 && k > 0 && *alpha != 0.0F;
  const bool is_root = ctx->rank == root;

  // This rank's own arguments. A rank whose arguments are wrong still takes
  // its part in the broadcast (so that no other rank waits for it forever),
  // computes nothing and returns the error.
  static const float kNonNull = 0.0F;
  const float *a_check = is_root ? a : &kNonNull;   // elsewhere A comes from staging
  SgemmPlan plan;
  sgblasStatus_t status = validate(transa, transb, m, n_local, k, alpha, a_check, lda, b, ldb,
                                   beta, c, ldc, &plan);
  if (!product) {
    if (status != SGBLAS_STATUS_SUCCESS || plan.work == Work::kNothing) return status;
    return sgblasSgemm(ctx->inner, transa, transb, m, n_local, k, alpha, a, lda, b, ldb, beta, c,
                       ldc);
  }
  const bool compute = status == SGBLAS_STATUS_SUCCESS && plan.work == Work::kProduct;
  if (ctx->nranks == 1) {
    if (!compute) return status;
    return sgblasSgemm(ctx->inner, transa, transb, m, n_local, k, alpha, a, lda, b, ldb, beta, c,
                       ldc);
  }

  // Staging: op(A) row r, column kk at staging[r + kk*lds] (transa N) or
  // staging[kk + r*lds] (transa T); lds keeps columns 128-byte aligned.
  const bool tn = transa == SGBLAS_OP_N;
  const int lds = ((tn ? m : k) + 31) / 32 * 32;
  const size_t cols = static_cast<size_t>(tn ? k : m);
  const size_t a_bytes = static_cast<size_t>(lds) * cols * sizeof(float);
  const sgblasStatus_t grown = ensureStaging(ctx, a_bytes);
  if (grown != SGBLAS_STATUS_SUCCESS) {
    sgblasMgAbort(ctx);   // the chain cannot run on any rank
    return grown;
  }
  const MemOps *ops = memOps();
  const std::vector<Panel> panels =
      planPanels(m, static_cast<size_t>(m) * static_cast<size_t>(k) * sizeof(float), ctx->nranks);
  const int n = ctx->nranks;
  const int pos = (ctx->rank - root + n) % n;
  const int parent = (ctx->rank - 1 + n) % n;
  const int child = (ctx->rank + 1) % n;
  const bool has_parent = pos > 0;
  const bool has_child = pos < n - 1;
  const uint32_t seq = ++ctx->seq;
  const unsigned wait_flags = CU_STREAM_WAIT_VALUE_GEQ | (ctx->flush ? CU_STREAM_WAIT_VALUE_FLUSH : 0);
  // Device addresses of the slots (same offsets as in the host mapping).
  auto slotDev = [&](int r) {
    const size_t off = reinterpret_cast<const char *>(&ctx->shm->slot[r]) -
                       reinterpret_cast<const char *>(ctx->shm);
    return reinterpret_cast<ShmSlot *>(ctx->shm_dev + off);
  };
  ShmSlot *me = slotDev(ctx->rank);
  ShmSlot *parent_slot = has_parent ? slotDev(parent) : nullptr;
  ShmSlot *child_slot = has_child ? slotDev(child) : nullptr;
  const auto hs = reinterpret_cast<CUstream>(ctx->stream);
  const auto cs = reinterpret_cast<CUstream>(ctx->copy);
  bool enq = true;   // every chain step was enqueued
  auto check = [&](bool ok) {
    if (!ok) {
      (void)cudaGetLastError();
      enq = false;
    }
  };
  // 1. My staging is free for this call: everything before it on my stream
  //    (earlier products, and earlier forwards, which the stream waited
  //    for) is done with it.
  if (has_parent) check(ops->write(hs, devAddr(&parent_slot->ready), seq, 0) == CUDA_SUCCESS);
  check(cudaEventRecord(ctx->ev_start, ctx->stream) == cudaSuccess);
  check(cudaStreamWaitEvent(ctx->copy, ctx->ev_start, 0) == cudaSuccess);
  // 2. The child's staging is free.
  if (has_child) check(ops->wait(cs, devAddr(&me->ready), seq, CU_STREAM_WAIT_VALUE_GEQ) == CUDA_SUCCESS);
  // Source of my pushes and of my products: the caller's A on the root (its
  // staging if the root passed none: the other ranks then get undefined
  // values, and the root its error), the staging elsewhere.
  const bool from_caller = is_root && a != nullptr;
  const float *src = from_caller ? a : ctx->staging;
  const int src_ld = from_caller ? lda : lds;
  auto offset = [&](int row, int ld) {
    return tn ? static_cast<size_t>(row) : static_cast<size_t>(row) * static_cast<size_t>(ld);
  };
  sgblasStatus_t gemm_status = SGBLAS_STATUS_SUCCESS;
  for (size_t pi = 0; pi < panels.size(); ++pi) {
    const Panel &pn = panels[pi];
    const size_t width = (tn ? static_cast<size_t>(pn.rows) : static_cast<size_t>(k)) * 4;
    const size_t height = tn ? static_cast<size_t>(k) : static_cast<size_t>(pn.rows);
    // 3. Forward panel pi once it is here, then flag it to the child; give
    //    the caller's buffer its copy on a non-root rank that passed one.
    if (has_parent)
      check(ops->wait(cs, devAddr(&me->panel[pi]), seq, wait_flags) == CUDA_SUCCESS);
    if (has_child) {
      check(cudaMemcpy2DAsync(ctx->peer_staging[child] + offset(pn.first, lds),
                              static_cast<size_t>(lds) * 4, src + offset(pn.first, src_ld),
                              static_cast<size_t>(src_ld) * 4, width, height, cudaMemcpyDefault,
                              ctx->copy) == cudaSuccess);
      check(ops->write(cs, devAddr(&child_slot->panel[pi]), seq, 0) == CUDA_SUCCESS);
    }
    if (!is_root && a != nullptr)
      check(cudaMemcpy2DAsync(a + offset(pn.first, lda), static_cast<size_t>(lda) * 4,
                              ctx->staging + offset(pn.first, lds), static_cast<size_t>(lds) * 4,
                              width, height, cudaMemcpyDeviceToDevice, ctx->copy) == cudaSuccess);
    // 4. This panel's rows of C.
    if (compute && gemm_status == SGBLAS_STATUS_SUCCESS) {
      if (has_parent)
        check(ops->wait(hs, devAddr(&me->panel[pi]), seq, wait_flags) == CUDA_SUCCESS);
      gemm_status = sgblasSgemm(ctx->inner, transa, transb, pn.rows, n_local, k, alpha,
                                src + offset(pn.first, src_ld), src_ld, b, ldb, beta,
                                c + pn.first, ldc);
    }
  }
  // 5. The call ends on the caller's stream once the forwards are done too.
  check(cudaEventRecord(ctx->ev_copies, ctx->copy) == cudaSuccess);
  check(cudaStreamWaitEvent(ctx->stream, ctx->ev_copies, 0) == cudaSuccess);
  if (!enq) {
    sgblasMgAbort(ctx);   // a step is missing: release every rank's waits
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  if (status != SGBLAS_STATUS_SUCCESS) return status;
  if (is_root && a == nullptr) return SGBLAS_STATUS_INVALID_VALUE;
  return gemm_status;
}

extern "C" sgblasStatus_t sgblasMgAllGather(sgblasMgHandle_t handle, const float *send,
                                            float *recv, size_t count) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  if (handle->aborted || handle->comm == nullptr) return SGBLAS_STATUS_EXECUTION_FAILED;
  if (count > 0 && (send == nullptr || recv == nullptr)) return SGBLAS_STATUS_INVALID_VALUE;
  const NcclApi *api = nccl();
  if (api == nullptr) return SGBLAS_STATUS_NOT_SUPPORTED;
  bool expired = false;
  const auto deadline = Clock::now() + std::chrono::milliseconds(handle->timeout_ms);
  const ncclResult_t r =
      settle(api, handle->comm,
             api->allGather(send, recv, count, ncclFloat32, handle->comm, handle->stream),
             deadline, &expired);
  if (r != ncclSuccess) {
    if (expired) sgblasMgAbort(handle);
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  return SGBLAS_STATUS_SUCCESS;
}
