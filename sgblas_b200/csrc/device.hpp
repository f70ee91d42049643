// Per-device state of the library: the device error word and the one-time
// kernel attribute set-up. Both are cached per device without locks
// (std::atomic), matching the reference's lock-free call path
// (src/sgemm_cuda.cu:443-472 caches device capabilities per thread).
#ifndef SGBLAS_B200_DEVICE_HPP_
#define SGBLAS_B200_DEVICE_HPP_

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

namespace sgblas::detail {

constexpr int kMaxDevices = 64;

// A device address of a __device__ symbol, cached per device and keyed on
// the CUDA context that was current when it was looked up: after the
// context is replaced (cudaDeviceReset, then the next runtime call makes a
// new primary context with the modules loaded again) the address is looked
// up anew instead of pointing into freed memory.
struct SymbolCache {
  std::atomic<const void *> entry[kMaxDevices];   // a SymbolEntry, never freed
};
// Address of `symbol` on `device` (the current device), or nullptr.
void *symbolAddress(SymbolCache *cache, int device, const void *symbol);

// Address of the device error word on `device` (the current device), or
// nullptr if it cannot be resolved. Kernels OR error codes into it
// (kern::kErrBarrierTimeout, ...); the host reads it with
// sgblasGetDeviceErrors.
unsigned *deviceErrorWord(int device);

// Sets the dynamic shared-memory limit of `kernel` on `device` once; `done`
// must be a per-kernel static bitmask.
inline bool configureKernel(const void *kernel, int device, int smem_bytes,
                            std::atomic<uint64_t> *done) {
  if (device < 0 || device >= kMaxDevices) return false;
  const uint64_t bit = uint64_t{1} << device;
  if (done->load(std::memory_order_acquire) & bit) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) !=
      cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  done->fetch_or(bit, std::memory_order_acq_rel);
  return true;
}

}  // namespace sgblas::detail

#endif  // SGBLAS_B200_DEVICE_HPP_
