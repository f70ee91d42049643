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

/* sgblasSgemm for callers that cannot allocate device memory (their process
 * or host owns the allocator, or forbids allocation after start-up). Same
 * arguments, semantics and status codes as sgblasSgemm, but instead of the
 * handle's lazily allocated workspace it uses one fixed 38 MiB scratch array
 * built into the library, which every GPU that loads the library holds until
 * exit. It never calls cudaMalloc, cudaFree or any allocating routine.
 *   - The first call on a device resolves the scratch address; make it
 *     before any stream capture.
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

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SGBLAS_SGBLAS_EXT_H_ */
