// Handle life cycle, stream and math-mode accessors, status strings.
//
// Status semantics follow the reference host layer one for one
// (src/handle.cpp:5-92 of AG0708/sgBLAS): a NULL handle is NOT_INITIALIZED, a
// NULL output pointer or an out-of-range enum is INVALID_VALUE, and nothing
// here ever aborts or touches the GPU (Destroy only frees the workspace).
#include "context.hpp"

#include <new>

extern "C" sgblasStatus_t sgblasCreate(sgblasHandle_t *handle) {
  if (handle == nullptr) return SGBLAS_STATUS_INVALID_VALUE;
  *handle = new (std::nothrow) sgblasContext{};
  return *handle == nullptr ? SGBLAS_STATUS_ALLOC_FAILED : SGBLAS_STATUS_SUCCESS;
}

extern "C" sgblasStatus_t sgblasDestroy(sgblasHandle_t handle) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  sgblas::detail::releaseWorkspace(handle);
  delete handle;
  return SGBLAS_STATUS_SUCCESS;
}

extern "C" sgblasStatus_t sgblasSetStream(sgblasHandle_t handle,
                                          sgblasStream_t stream) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  handle->stream = stream;
  return SGBLAS_STATUS_SUCCESS;
}

extern "C" sgblasStatus_t sgblasGetStream(sgblasHandle_t handle,
                                          sgblasStream_t *stream) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  if (stream == nullptr) return SGBLAS_STATUS_INVALID_VALUE;
  *stream = handle->stream;
  return SGBLAS_STATUS_SUCCESS;
}

extern "C" sgblasStatus_t sgblasSetMathMode(sgblasHandle_t handle,
                                            sgblasMathMode_t mode) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  switch (mode) {
    case SGBLAS_MATH_FP32:
    case SGBLAS_MATH_TF32:
      handle->math_mode = mode;
      return SGBLAS_STATUS_SUCCESS;
    default:
      return SGBLAS_STATUS_INVALID_VALUE;
  }
}

extern "C" sgblasStatus_t sgblasGetMathMode(sgblasHandle_t handle,
                                            sgblasMathMode_t *mode) {
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  if (mode == nullptr) return SGBLAS_STATUS_INVALID_VALUE;
  *mode = handle->math_mode;
  return SGBLAS_STATUS_SUCCESS;
}

extern "C" const char *sgblasGetStatusString(sgblasStatus_t status) {
  // The strings are part of the observable interface: same text as the
  // reference (src/handle.cpp:70-92).
  switch (status) {
    case SGBLAS_STATUS_SUCCESS: return "success";
    case SGBLAS_STATUS_NOT_INITIALIZED: return "not initialized";
    case SGBLAS_STATUS_ALLOC_FAILED: return "allocation failed";
    case SGBLAS_STATUS_INVALID_VALUE: return "invalid value";
    case SGBLAS_STATUS_ARCH_MISMATCH: return "architecture mismatch";
    case SGBLAS_STATUS_EXECUTION_FAILED: return "execution failed";
    case SGBLAS_STATUS_INTERNAL_ERROR: return "internal error";
    case SGBLAS_STATUS_NOT_SUPPORTED: return "not supported";
    default: return "unknown status";
  }
}
