// Device error word and the diagnostics entry point that reads it.
#include "device.hpp"
#include "ptx.cuh"

#include <cuda.h>

#include <new>

#include <sgblas/sgblas_ext.h>

namespace sgblas::detail {
namespace {

__device__ unsigned g_device_error;

SymbolCache g_error_word;

struct SymbolEntry {
  void *context;
  void *address;
};

using CtxGetCurrentFn = CUresult (*)(CUcontext *);

// The calling thread's current context, or nullptr (none yet, or the driver
// entry point is unavailable).
void *currentContext() {
  static const CtxGetCurrentFn fn = [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      return static_cast<CtxGetCurrentFn>(nullptr);
    }
    return reinterpret_cast<CtxGetCurrentFn>(f);
  }();
  CUcontext ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

}  // namespace

void *symbolAddress(SymbolCache *cache, int device, const void *symbol) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  const void *context = currentContext();
  const auto *entry =
      static_cast<const SymbolEntry *>(cache->entry[device].load(std::memory_order_acquire));
  if (entry != nullptr && context != nullptr && entry->context == context) return entry->address;
  void *address = nullptr;
  if (cudaGetSymbolAddress(&address, symbol) != cudaSuccess) {   // makes the context current
    (void)cudaGetLastError();
    return nullptr;
  }
  context = currentContext();
  if (context != nullptr) {
    // Published once per (device, context); an entry replaced by a newer
    // one is left allocated (a few bytes per context change), so a reader
    // holding it never sees freed memory.
    auto *fresh = new (std::nothrow) SymbolEntry{const_cast<void *>(context), address};
    if (fresh != nullptr) cache->entry[device].store(fresh, std::memory_order_release);
  }
  return address;
}

unsigned *deviceErrorWord(int device) {
  return static_cast<unsigned *>(symbolAddress(&g_error_word, device, &g_device_error));
}

namespace {

// Waits on an mbarrier that nothing will ever complete, with a short poll
// limit: the wait must give up, raise the error flag and let the kernel
// return normally. Reports whether the wait returned false.
__global__ void waitTimeoutKernel(unsigned *err, unsigned polls, int *gave_up) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    kern::mbarInit(&bar, 1);
    kern::fenceBarrierInit();
  }
  __syncthreads();
  if (threadIdx.x == 0) *gave_up = kern::mbarWait(&bar, 0, err, polls) ? 0 : 1;
}

}  // namespace

}  // namespace sgblas::detail

extern "C" sgblasStatus_t sgblasSelfTestWaitTimeout(unsigned polls, int *timed_out) {
  if (timed_out == nullptr || polls == 0) return SGBLAS_STATUS_INVALID_VALUE;
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  unsigned *err = sgblas::detail::deviceErrorWord(device);
  if (err == nullptr) return SGBLAS_STATUS_EXECUTION_FAILED;
  int *flag = nullptr;
  if (cudaMallocManaged(&flag, sizeof(int)) != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_ALLOC_FAILED;
  }
  *flag = -1;
  sgblas::detail::waitTimeoutKernel<<<1, 32>>>(err, polls, flag);
  const cudaError_t e = cudaDeviceSynchronize();
  *timed_out = *flag;
  (void)cudaFree(flag);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  return SGBLAS_STATUS_SUCCESS;
}

extern "C" sgblasStatus_t sgblasGetDeviceErrors(unsigned *flags, int clear) {
  if (flags == nullptr) return SGBLAS_STATUS_INVALID_VALUE;
  if (cudaDeviceSynchronize() != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  unsigned value = 0;
  if (cudaMemcpyFromSymbol(&value, sgblas::detail::g_device_error, sizeof(value)) != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  *flags = value;
  if (clear != 0) {
    const unsigned zero = 0;
    if (cudaMemcpyToSymbol(sgblas::detail::g_device_error, &zero, sizeof(zero)) != cudaSuccess) {
      (void)cudaGetLastError();
      return SGBLAS_STATUS_EXECUTION_FAILED;
    }
  }
  return SGBLAS_STATUS_SUCCESS;
}
