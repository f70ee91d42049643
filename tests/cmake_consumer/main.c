/* Calls the installed C API without touching device memory, so it runs on a
 * machine with or without a GPU: handle life cycle, math-mode accessors, an
 * argument error, a quick return and the status strings. Exit status 0 means
 * every check held; any other value names the first check that failed. */
#include <sgblas/sgblas.h>
#include <sgblas/sgblas_ext.h>
#include <sgblas/sgblas_mg.h>

#include <stdio.h>
#include <string.h>

int main(void) {
  sgblasHandle_t handle = NULL;
  sgblasMathMode_t mode = SGBLAS_MATH_FP32;
  const float one = 1.0f;

  if (sgblasCreate(&handle) != SGBLAS_STATUS_SUCCESS || handle == NULL) return 1;
  if (sgblasSetMathMode(handle, SGBLAS_MATH_TF32) != SGBLAS_STATUS_SUCCESS) return 2;
  if (sgblasGetMathMode(handle, &mode) != SGBLAS_STATUS_SUCCESS || mode != SGBLAS_MATH_TF32)
    return 3;
  /* lda < m is an argument error, reported before any device work. */
  if (sgblasSgemm(handle, SGBLAS_OP_N, SGBLAS_OP_N, 4, 4, 4, &one, (const float *)0x1000, 3,
                  (const float *)0x1000, 4, &one, (float *)0x2000, 4) !=
      SGBLAS_STATUS_INVALID_VALUE)
    return 4;
  /* m == 0 is a quick return: success with no pointer read. */
  if (sgblasSgemm(handle, SGBLAS_OP_N, SGBLAS_OP_T, 0, 4, 4, NULL, NULL, 1, NULL, 4, NULL, NULL,
                  1) != SGBLAS_STATUS_SUCCESS)
    return 5;
  if (sgblasSgemm(NULL, SGBLAS_OP_N, SGBLAS_OP_N, 0, 0, 0, NULL, NULL, 1, NULL, 1, NULL, NULL,
                  1) != SGBLAS_STATUS_NOT_INITIALIZED)
    return 6;
  if (strcmp(sgblasGetStatusString(SGBLAS_STATUS_SUCCESS), "success") != 0) return 7;
  /* The extension and multi-GPU headers link too (their symbols resolve). */
  if ((void *)&sgblasSgemmStridedBatched == NULL || (void *)&sgblasMgCreate == NULL) return 8;
  if (sgblasDestroy(handle) != SGBLAS_STATUS_SUCCESS) return 9;
  printf("sgblas consumer: %s\n", sgblasGetStatusString(SGBLAS_STATUS_INVALID_VALUE));
  return 0;
}
