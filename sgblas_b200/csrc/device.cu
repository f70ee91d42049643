// Device error word and the diagnostics entry point that reads it.
#include "device.hpp"
#include "ptx.cuh"

#include <sgblas/sgblas_ext.h>

namespace sgblas::detail {
namespace {

__device__ unsigned g_device_error;

std::atomic<unsigned *> g_error_word[kMaxDevices];

}  // namespace

unsigned *deviceErrorWord(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  unsigned *cached = g_error_word[device].load(std::memory_order_acquire);
  if (cached != nullptr) return cached;
  void *address = nullptr;
  if (cudaGetSymbolAddress(&address, g_device_error) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  g_error_word[device].store(static_cast<unsigned *>(address), std::memory_order_release);
  return static_cast<unsigned *>(address);
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
