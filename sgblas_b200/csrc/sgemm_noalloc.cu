// sgblasSgemmNoAlloc: sgblasSgemm for callers that cannot allocate device memory.
//
// Who needs this: code that runs where cudaMalloc / cudaMallocAsync are not
// available or not allowed -- e.g. a host that has pre-reserved all device
// memory for its own pool, a plugin loaded into a process whose allocator
// owns the device, or code with a hard rule of no allocation after start-up.
// sgblasSgemm may allocate a stream-K workspace on the handle the first time a
// problem needs one; this entry point never does. Instead it uses one
// fixed-size scratch array compiled into the library (kScratchBytes below),
// which every GPU that loads the library holds until the process exits.
//
// Same arguments, validation, results and status codes as sgblasSgemm, with
// three differences:
//   - The first call on a device looks up the scratch array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it. Make
//     that first call before any stream capture.
//   - All calls on a device share the one scratch array, and it keeps what the
//     last call left in it. Calls whose kernels can overlap on the GPU (e.g.
//     issued on two streams without ordering) race on it: order them.
//   - A problem whose stream-K schedule needs more scratch than the array
//     holds is rejected with SGBLAS_STATUS_NOT_SUPPORTED (on B200, with 148
//     SMs, every problem fits: the need grows with the SM count, not with
//     m, n or k).
// It calls no cudaMalloc, cudaFree or other allocating routine. The kernel is
// the same persistent tile kernel sgblasSgemm launches (sgemm_tile.cuh).
#include "context.hpp"
#include "device.hpp"
#include "sgemm_tile.cuh"
#include "validation.hpp"

#include <sgblas/sgblas_ext.h>

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdint>

namespace {

using sgblas::kern::Beta;
using sgblas::kern::GemmParams;
using sgblas::kern::Src;

// Scratch layout: [arrival counters | partial-tile slots]. 38 MiB holds the
// counters of up to 1024 split tiles and two 128 KiB partial slots for each of
// up to 151 persistent CTAs (one per SM).
constexpr size_t kCounterBytes = 4096;
constexpr size_t kSlotBytes = size_t{sgblas::kern::kThreads} * sgblas::kern::kSlotFloat4 * sizeof(float4);
constexpr size_t kScratchBytes = size_t{38} << 20;

}  // namespace

// The scratch itself, at file scope (zero-initialised when the module loads).
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

namespace {

// Device address of g_scratch per device. In host code `g_scratch` only names
// a host-side stand-in, so its address must come from cudaGetSymbolAddress.
std::atomic<unsigned char *> g_scratch_address[sgblas::detail::kMaxDevices];

unsigned char *scratchAddress(int device) {
  if (device < 0 || device >= sgblas::detail::kMaxDevices) return nullptr;
  unsigned char *ptr = g_scratch_address[device].load(std::memory_order_acquire);
  if (ptr != nullptr) return ptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void **>(&ptr), g_scratch) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  g_scratch_address[device].store(ptr, std::memory_order_release);
  return ptr;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encodeTiled() {
  static const EncodeTiledFn fn = [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      return static_cast<EncodeTiledFn>(nullptr);
    }
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

bool encodeMatrix(CUtensorMap *map, const float *ptr, int rows, int cols, int ld, int box_rows,
                  int box_cols, bool swizzle64) {
  const EncodeTiledFn fn = encodeTiled();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(cols)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * sizeof(float)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_rows), static_cast<cuuint32_t>(box_cols)};
  const cuuint32_t elem_strides[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(ptr), dims, strides, box,
            elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swizzle64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

sgblasStatus_t launchStatus(cudaError_t e) {
  if (e == cudaSuccess) return SGBLAS_STATUS_SUCCESS;
  (void)cudaGetLastError();
  return SGBLAS_STATUS_EXECUTION_FAILED;
}

// The same persistent schedule sgblasSgemm uses (whole tiles, then stream-K
// for a partial last wave or for problems with fewer tiles than SMs).
constexpr int kMinSkIters = 8;

template <bool kTA, bool kTB, Beta kBeta, Src kSrc>
sgblasStatus_t launch(GemmParams p, int device, cudaStream_t stream) {
  using Plan = sgblas::kern::Plan<kTA, kTB, kSrc>;
  auto kernel = sgblas::kern::sgemmKernel<kTA, kTB, kBeta, kSrc>;
  static std::atomic<uint64_t> configured{0};
  if (!sgblas::detail::configureKernel(reinterpret_cast<const void *>(kernel), device,
                                       sgblas::kern::kSmemBytes, &configured))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  p.tiles_m = (p.m + Plan::kBM - 1) / Plan::kBM;
  p.tiles_n = (p.n + Plan::kBN - 1) / Plan::kBN;
  p.group_m = 8;
  p.kiters = (p.k + sgblas::kern::kBK - 1) / sgblas::kern::kBK;
  const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n;
  if (tiles > INT_MAX / 2 || static_cast<long long>(p.kiters) * tiles > INT_MAX)
    return SGBLAS_STATUS_NOT_SUPPORTED;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  const int t = static_cast<int>(tiles);
  p.dp_tiles = p.sk_tiles = p.sk_q = p.sk_r = 0;
  if (t >= sms) {
    p.grid = sms;
    const int waves = t / sms, rem = t % sms;
    if (rem == 0 || p.kiters < 2 * kMinSkIters) {
      p.dp_tiles = t;
    } else {
      p.dp_tiles = (waves - 1) * sms;
      p.sk_tiles = t - p.dp_tiles;
    }
  } else {
    p.grid = static_cast<int>(std::min<long long>(
        sms, std::max<long long>(tiles, tiles * p.kiters / kMinSkIters)));
    if (p.grid == t) p.dp_tiles = t;
    else p.sk_tiles = t;
  }
  if (p.sk_tiles > 0) {
    const long long it = static_cast<long long>(p.sk_tiles) * p.kiters;
    p.sk_q = static_cast<int>(it / p.grid);
    p.sk_r = static_cast<int>(it % p.grid);
    // The fixed scratch must hold this schedule: refuse rather than allocate.
    if (static_cast<size_t>(p.sk_tiles) * sizeof(int) > kCounterBytes ||
        kCounterBytes + 2 * static_cast<size_t>(p.grid) * kSlotBytes > kScratchBytes)
      return SGBLAS_STATUS_NOT_SUPPORTED;
    unsigned char *scratch = scratchAddress(device);
    if (scratch == nullptr) return SGBLAS_STATUS_EXECUTION_FAILED;
    // The counters must start at zero; a previous call normally leaves them
    // so, but one that did not finish might not have.
    if (cudaMemsetAsync(scratch, 0, static_cast<size_t>(p.sk_tiles) * sizeof(int), stream) !=
        cudaSuccess)
      return launchStatus(cudaErrorUnknown);
    p.counters = reinterpret_cast<int *>(scratch);
    p.ws = reinterpret_cast<float4 *>(scratch + kCounterBytes);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.grid));
  cfg.blockDim = dim3(sgblas::kern::kBlockThreads);
  cfg.dynamicSmemBytes = sgblas::kern::kSmemBytes;
  cfg.stream = stream;
  return launchStatus(cudaLaunchKernelEx(&cfg, kernel, p));
}

template <bool kTA, bool kTB, Src kSrc>
sgblasStatus_t launchByBeta(const GemmParams &p, int device, cudaStream_t stream) {
  if (p.beta == 0.0F) return launch<kTA, kTB, Beta::kZero, kSrc>(p, device, stream);
  if (p.beta == 1.0F) return launch<kTA, kTB, Beta::kOne, kSrc>(p, device, stream);
  return launch<kTA, kTB, Beta::kGeneral, kSrc>(p, device, stream);
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <bool kTA, bool kTB>
sgblasStatus_t launchBySource(GemmParams &p, int device, cudaStream_t stream) {
  if constexpr (!(kTA && !kTB)) {
    using Plan = sgblas::kern::Plan<kTA, kTB, Src::kTma>;
    if (aligned16(p.a) && aligned16(p.b) && p.lda % 4 == 0 && p.ldb % 4 == 0) {
      const int a_ext = Plan::kPairIsA ? sgblas::kern::kBP : sgblas::kern::kBD;
      const int b_ext = Plan::kPairIsA ? sgblas::kern::kBD : sgblas::kern::kBP;
      const bool a_kx = Plan::kA == sgblas::kern::Layout::kKX;
      const bool b_kx = Plan::kB == sgblas::kern::Layout::kKX;
      const int bk = sgblas::kern::kBK;
      if (encodeMatrix(&p.tma_a, p.a, kTA ? p.k : p.m, kTA ? p.m : p.k, p.lda,
                       a_kx ? bk : a_ext, a_kx ? a_ext : bk, a_kx) &&
          encodeMatrix(&p.tma_b, p.b, kTB ? p.n : p.k, kTB ? p.k : p.n, p.ldb,
                       b_kx ? bk : b_ext, b_kx ? b_ext : bk, b_kx))
        return launchByBeta<kTA, kTB, Src::kTma>(p, device, stream);
    }
  }
  return launchByBeta<kTA, kTB, Src::kCopy>(p, device, stream);
}

}  // namespace

extern "C" sgblasStatus_t sgblasSgemmNoAlloc(sgblasHandle_t handle, sgblasOperation_t transa,
                                             sgblasOperation_t transb, int m, int n, int k,
                                             const float *alpha, const float *a, int lda,
                                             const float *b, int ldb, const float *beta,
                                             float *c, int ldc) {
  using namespace sgblas::detail;
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  SgemmPlan plan;
  const sgblasStatus_t status =
      validate(transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc, &plan);
  if (status != SGBLAS_STATUS_SUCCESS) return status;
  if (plan.work != Work::kProduct) {
    // Quick returns and C = beta*C never use a workspace: sgblasSgemm does
    // exactly that without allocating.
    return sgblasSgemm(handle, transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc);
  }
  if (handle->math_mode != SGBLAS_MATH_FP32) return SGBLAS_STATUS_NOT_SUPPORTED;
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  unsigned *err = deviceErrorWord(device);
  if (err == nullptr) return SGBLAS_STATUS_EXECUTION_FAILED;
  GemmParams p = {};
  p.a = a;
  p.b = b;
  p.c = c;
  p.m = m;
  p.n = n;
  p.k = k;
  p.lda = lda;
  p.ldb = ldb;
  p.ldc = ldc;
  p.alpha = plan.alpha;
  p.beta = plan.beta;
  p.err = err;
  const auto stream = static_cast<cudaStream_t>(handle->stream);
  const bool tA = transa == SGBLAS_OP_T, tB = transb == SGBLAS_OP_T;
  if (!tA && !tB) return launchBySource<false, false>(p, device, stream);
  if (!tA && tB) return launchBySource<false, true>(p, device, stream);
  if (tA && !tB) return launchBySource<true, false>(p, device, stream);
  return launchBySource<true, true>(p, device, stream);
}
