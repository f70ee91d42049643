/*
 * sgblas-b200 extensions that have no counterpart in the reference API.
 */
#ifndef SGBLAS_SGBLAS_EXT_H_
#define SGBLAS_SGBLAS_EXT_H_

#include <sgblas/sgblas.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Device error flags raised by the kernels on the current device (bit 0: a
 * bounded wait for a tile copy ran out, the kernel stopped early and its
 * output is not valid). Synchronizes the current device first; clear != 0
 * resets the flags. Diagnostics only: the SGEMM call path never reads them.
 * No counterpart in the reference (it has no device-side waits). */
sgblasStatus_t sgblasGetDeviceErrors(unsigned *flags, int clear);

/* Self-test of the kernels' bounded waits: a one-thread kernel waits on a
 * barrier that nothing completes, giving up after `polls` polls. On return
 * *timed_out is 1 when the wait gave up (and the device error flags then hold
 * bit 0, which sgblasGetDeviceErrors reads and may clear); the device stays
 * usable. Synchronizes the current device. No counterpart in the reference. */
sgblasStatus_t sgblasSelfTestWaitTimeout(unsigned polls, int *timed_out);

/* Test hook for split-tile recovery. Leaves the handle workspace's arrival
 * counters in the state a split launch that stopped early (a bounded wait
 * that timed out) leaves behind -- every counter holding one arrival of the
 * handle's latest launch -- so that a test can check that the next split
 * product on the handle is still exact. Enqueued on the handle's stream, on
 * the current device, which must be the workspace's. Returns
 * SGBLAS_STATUS_NOT_SUPPORTED while the handle has no workspace.
 * No counterpart in the reference (it splits no tile across CTAs). */
sgblasStatus_t sgblasTestInterruptScratch(sgblasHandle_t handle);

/* sgblasSgemm for callers that cannot allocate device memory (their process
 * or host owns the allocator, or forbids allocation after start-up). Same
 * arguments, semantics and status codes as sgblasSgemm, but instead of the
 * handle's lazily allocated workspace it uses one fixed 38 MiB scratch array
 * built into the library, which every GPU that loads the library holds until
 * exit. It never calls cudaMalloc, cudaFree or any allocating routine.
 *   - The first call on a device resolves the scratch address; make it
 *     before any stream capture. After cudaDeviceReset the next call
 *     resolves it again (make that one before any capture too).
 *   - All calls on a device share the scratch and it keeps the last call's
 *     contents: calls that may overlap on the GPU race, so order them.
 *   - A schedule that needs more scratch than 38 MiB (only possible on a GPU
 *     with more than 151 SMs) returns SGBLAS_STATUS_NOT_SUPPORTED.
 * No counterpart in the reference API (the reference allocates nothing in
 * the first place: it has no split-k workspace). */
sgblasStatus_t sgblasSgemmNoAlloc(sgblasHandle_t handle, sgblasOperation_t transa,
                                  sgblasOperation_t transb, int m, int n, int k,
                                  const float *alpha, const float *a, int lda,
                                  const float *b, int ldb, const float *beta,
                                  float *c, int ldc);

/* Batched SGEMM: batch_count products C_i = alpha*op(A_i)*op(B_i) + beta*C_i
 * that share transa/transb, m, n, k, the leading dimensions and the scalars,
 * in one launch on the handle's stream. Each matrix follows sgblasSgemm's
 * semantics (beta == 0 never reads C, padding rows stay untouched) and
 * accuracy bound; the split of k across CTAs, and so the rounding, may differ
 * from a single sgblasSgemm call on the same matrix. The arguments
 * are validated as sgblasSgemm validates them, in the same order, and then
 * batch_count < 0 gives SGBLAS_STATUS_INVALID_VALUE; batch_count == 0, like
 * m == 0, is a successful no-op. The C matrices must not overlap each other.
 * No counterpart in the reference API (its design lists batched GEMM as a v1
 * non-goal, docs/design.md:102); the argument order is cuBLAS's
 * cublasSgemmStridedBatched / cublasSgemmBatched.
 *
 * Strided: matrix i is a + i*stride_a (b, c alike; strides in elements, any
 * sign; stride_a or stride_b 0 reuses one matrix for every product). In
 * SGBLAS_MATH_TF32 mode a strided batch runs on the tensor cores when its
 * strides are positive multiples of 4 floats (and A, B are 16-byte aligned
 * with leading dimensions that are multiples of 4); otherwise, and for
 * pointer arrays, it computes in FP32. */
sgblasStatus_t sgblasSgemmStridedBatched(sgblasHandle_t handle, sgblasOperation_t transa,
                                         sgblasOperation_t transb, int m, int n, int k,
                                         const float *alpha, const float *a, int lda,
                                         long long stride_a, const float *b, int ldb,
                                         long long stride_b, const float *beta, float *c,
                                         int ldc, long long stride_c, int batch_count);

/* Pointer arrays: a_array, b_array and c_array are DEVICE arrays of
 * batch_count device pointers (read by the kernels, never by the host). */
sgblasStatus_t sgblasSgemmBatched(sgblasHandle_t handle, sgblasOperation_t transa,
                                  sgblasOperation_t transb, int m, int n, int k,
                                  const float *alpha, const float *const a_array[], int lda,
                                  const float *const b_array[], int ldb, const float *beta,
                                  float *const c_array[], int ldc, int batch_count);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SGBLAS_SGBLAS_EXT_H_ */
