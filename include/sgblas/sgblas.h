/*
 * sgblas-b200 public C API: strict-FP32 column-major SGEMM for NVIDIA B200.
 *
 * This header is ABI-compatible with the reference sgBLAS interface
 * (include/sgblas/sgblas.h:1-69 of AG0708/sgBLAS): the same opaque handle, the
 * same enum values (including the FORCE_INT sentinels) and the same function
 * signatures, so a program built against the reference header links against
 * libsgblas.so from this project unchanged.
 *
 * Entry points and the reference interface each one replaces:
 *   sgblasCreate / sgblasDestroy          src/handle.cpp:5-23
 *   sgblasSetStream / sgblasGetStream     src/handle.cpp:25-44
 *   sgblasSetMathMode / sgblasGetMathMode src/handle.cpp:46-68
 *   sgblasSgemm                           src/sgemm_cuda.cu:699-730
 *   sgblasGetStatusString                 src/handle.cpp:70-92
 */
#ifndef SGBLAS_SGBLAS_H_
#define SGBLAS_SGBLAS_H_

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque library context: holds the stream and the math mode. */
typedef struct sgblasContext *sgblasHandle_t;

/* A cudaStream_t carried as void* so that host-only code can include this
 * header without the CUDA toolkit. NULL selects the legacy default stream. */
typedef void *sgblasStream_t;

typedef enum sgblasStatus_t {
  SGBLAS_STATUS_SUCCESS = 0,
  SGBLAS_STATUS_NOT_INITIALIZED = 1,
  SGBLAS_STATUS_ALLOC_FAILED = 2,
  SGBLAS_STATUS_INVALID_VALUE = 3,
  SGBLAS_STATUS_ARCH_MISMATCH = 4,
  SGBLAS_STATUS_EXECUTION_FAILED = 5,
  SGBLAS_STATUS_INTERNAL_ERROR = 6,
  SGBLAS_STATUS_NOT_SUPPORTED = 7,
  SGBLAS_STATUS_FORCE_INT = 0x7fffffff
} sgblasStatus_t;

typedef enum sgblasOperation_t {
  SGBLAS_OP_N = 0,
  SGBLAS_OP_T = 1,
  SGBLAS_OP_FORCE_INT = 0x7fffffff
} sgblasOperation_t;

typedef enum sgblasMathMode_t {
  SGBLAS_MATH_FP32 = 0,
  SGBLAS_MATH_TF32 = 1,
  SGBLAS_MATH_FORCE_INT = 0x7fffffff
} sgblasMathMode_t;

/* Allocates a context (stream NULL, math mode FP32). NULL output pointer:
 * INVALID_VALUE. Out of host memory: ALLOC_FAILED. */
sgblasStatus_t sgblasCreate(sgblasHandle_t *handle);

/* Releases a context and any device workspace it owns. NULL: NOT_INITIALIZED. */
sgblasStatus_t sgblasDestroy(sgblasHandle_t handle);

/* Stores the caller-owned stream later calls enqueue on. */
sgblasStatus_t sgblasSetStream(sgblasHandle_t handle, sgblasStream_t stream);
sgblasStatus_t sgblasGetStream(sgblasHandle_t handle, sgblasStream_t *stream);

/* FP32 (default) or TF32. FP32 computes strict FP32 on CUDA cores (FP32
 * multiply, FP32 accumulate, no tensor cores). TF32 selects the tensor-core
 * lane: operands rounded to TF32 (10-bit mantissa), FP32 accumulation, error
 * within (2^-9 + (k+2) * 2^-22) * (|alpha| sum|a*b| + |beta*c|) per element;
 * operands the tensor-core lane cannot read in place (and pointer-array
 * batches) are computed in strict FP32 instead. The reference returns
 * NOT_SUPPORTED for work in TF32 mode. */
sgblasStatus_t sgblasSetMathMode(sgblasHandle_t handle, sgblasMathMode_t mode);
sgblasStatus_t sgblasGetMathMode(sgblasHandle_t handle, sgblasMathMode_t *mode);

/*
 *   C = (*alpha) * op(A) * op(B) + (*beta) * C        (column-major, FP32)
 *
 * op(X) is X (SGBLAS_OP_N) or its transpose (SGBLAS_OP_T); op(A) is m x k,
 * op(B) is k x n, C is m x n. lda >= max(1, N ? m : k), ldb >= max(1, N ? k :
 * n), ldc >= max(1, m). alpha and beta are host pointers read once during the
 * call; A, B and C are device pointers on the current device and must not
 * overlap. The call enqueues on the handle's stream and never synchronizes.
 *   - m == 0 or n == 0: returns SUCCESS without reading any pointer.
 *   - k == 0 or *alpha == 0: A and B are not read; C = beta*C (nothing at all
 *     when beta == 1).
 *   - *beta == 0: C is written without being read (NaN/Inf in C vanish).
 *   - Rows [m, ldc) of every column of C are never written.
 */
sgblasStatus_t sgblasSgemm(sgblasHandle_t handle, sgblasOperation_t transa,
                           sgblasOperation_t transb, int m, int n, int k,
                           const float *alpha, const float *a, int lda,
                           const float *b, int ldb, const float *beta, float *c,
                           int ldc);

/* Static, human-readable name of a status ("unknown status" otherwise). */
const char *sgblasGetStatusString(sgblasStatus_t status);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SGBLAS_SGBLAS_H_ */
