/*
 * CPU oracle for strict-FP32 SGEMM -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library; the product (libsgblas.so) never links or calls it.
 *
 * What it restates from the reference (AG0708/sgBLAS):
 *   - input generation: std::mt19937 seeded per case, values drawn in storage
 *     order from uniform_real_distribution<float>(-1, 1)
 *     (tests/cuda/correctness.cu:170-174) or normal_distribution<float>(0, 1);
 *   - the FP64 triple-loop oracle of tests/cuda/correctness.cu:373-392: FP32
 *     inputs widened to double, products summed in k order, result
 *     alpha*dot (+ beta*c unless beta == 0) and the error magnitude
 *     |alpha|*sum|a*b| (+ |beta*c| unless beta == 0).
 * The reference has no CPU SGEMM (src/sgemm_host.cpp:26-27 returns
 * NOT_SUPPORTED), so this loop is also the timed CPU baseline.
 */
#ifndef SGBLAS_ORACLE_H_
#define SGBLAS_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A std::mt19937 stream; successive fills continue the same sequence, the
 * way the reference's correctness test fills A, then B, then C. */
void *oracle_rng_new(uint32_t seed);
void oracle_rng_free(void *rng);
void oracle_rng_uniform(void *rng, float *out, size_t count);
void oracle_rng_normal(void *rng, float *out, size_t count);

/* FP64 reference for the columns [j0, j1) of C: ref and mag are m x (j1-j0),
 * column-major, leading dimension m. c0 is the initial C (ignored, and may be
 * NULL, when beta == 0). threads <= 0 uses all hardware threads. */
void oracle_sgemm_f64(int transa, int transb, int m, int n, int k, float alpha,
                      const float *a, int lda, const float *b, int ldb,
                      float beta, const float *c0, int ldc, int j0, int j1,
                      double *ref, double *mag, int threads);

/* Same arithmetic at count chosen entries (rows[i], cols[i]). */
void oracle_sgemm_f64_points(int transa, int transb, int k, float alpha,
                             const float *a, int lda, const float *b, int ldb,
                             float beta, const float *c0, int ldc,
                             const int *rows, const int *cols, int count,
                             double *ref, double *mag, int threads);

/* The CPU baseline: the oracle loop writing float results into c (ldc) for
 * the columns [j0, j1), over `threads` host threads split by column. */
void oracle_sgemm_cpu(int transa, int transb, int m, int k, float alpha,
                      const float *a, int lda, const float *b, int ldb,
                      float beta, float *c, int ldc, int j0, int j1,
                      int threads);

int oracle_hardware_threads(void);

#ifdef __cplusplus
}
#endif

#endif /* SGBLAS_ORACLE_H_ */
