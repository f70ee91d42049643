// Device error word and the diagnostics entry point that reads it.
#include "device.hpp"

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

}  // namespace sgblas::detail

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
