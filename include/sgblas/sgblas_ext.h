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

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SGBLAS_SGBLAS_EXT_H_ */
