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
//     that first call before any stream capture. The cache is keyed on the
//     current CUDA context, so after cudaDeviceReset the next call looks the
//     address up again (make it, too, before any capture).
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
#include "sgemm_launch.hpp"
#include "validation.hpp"

#include <sgblas/sgblas_ext.h>

#include <cuda_runtime.h>

#include <atomic>

namespace {

// Scratch layout (sgemm_launch.hpp): [arrival counters | partial-tile slots].
// 38 MiB holds the 4 KiB counter region and two 128 KiB partial slots for each
// of up to 151 persistent CTAs (one per SM).
constexpr size_t kScratchBytes = size_t{38} << 20;
static_assert(sgblas::detail::kCounterRegionBytes + 2 * 151 * sgblas::detail::kSlotBytes <=
                  kScratchBytes,
              "scratch sized for 151 SMs");

}  // namespace

// The scratch itself, at file scope (zero-initialised when the module loads).
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

namespace {

// Device address of g_scratch per device (and per context: looked up again
// after cudaDeviceReset). In host code `g_scratch` only names a host-side
// stand-in, so its address must come from cudaGetSymbolAddress, called with
// the device current.
sgblas::detail::SymbolCache g_scratch_address;

unsigned char *scratchAddress(int device) {
  return static_cast<unsigned char *>(
      sgblas::detail::symbolAddress(&g_scratch_address, device, &g_scratch));
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
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  const int arch = isSm100(device);
  if (arch < 0) return SGBLAS_STATUS_EXECUTION_FAILED;
  if (arch == 0) return SGBLAS_STATUS_ARCH_MISMATCH;
  unsigned *err = deviceErrorWord(device);
  if (err == nullptr) return SGBLAS_STATUS_EXECUTION_FAILED;
  unsigned char *scratch = scratchAddress(device);
  if (scratch == nullptr) return SGBLAS_STATUS_EXECUTION_FAILED;
  sgblas::kern::GemmParams p = {};
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
  p.batch = 1;
  const auto stream = static_cast<cudaStream_t>(handle->stream);
  Scratch fixed;
  fixed.fixed = scratch;
  fixed.fixed_bytes = kScratchBytes;
  const bool tA = transa == SGBLAS_OP_T, tB = transb == SGBLAS_OP_T;
  // The TF32 lane takes its stream-K scratch from the same fixed array;
  // operands it cannot read with TMA are computed in FP32 instead (more
  // accurate than TF32 asks).
  if (handle->math_mode == SGBLAS_MATH_TF32 && tf32Eligible(a, lda, b, ldb))
    return launchTf32(tA, tB, p, fixed, device, stream);
  // Small products: the cluster kernel (scratch only when several clusters
  // share a tile).
  const int sms = smCount(device);
  if (sms <= 0) return SGBLAS_STATUS_EXECUTION_FAILED;
  if (smallEligible(p, sms)) return launchSmall(tA, tB, p, fixed, device, sms, stream);
  if (!tA && !tB) return launchMode<false, false>(p, fixed, device, stream);
  if (!tA && tB) return launchMode<false, true>(p, fixed, device, stream);
  if (tA && !tB) return launchMode<true, false>(p, fixed, device, stream);
  return launchMode<true, true>(p, fixed, device, stream);
}
