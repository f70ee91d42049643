// SGEMM argument validation and work classification.
//
// Same rules and the same order of checks as the reference
// (src/sgemm_validation.cpp:14-66 of AG0708/sgBLAS), because the order is
// observable: e.g. m == 0 succeeds even with NULL alpha, and NULL C is only an
// error once it is known that C will be written.
#ifndef SGBLAS_B200_VALIDATION_HPP_
#define SGBLAS_B200_VALIDATION_HPP_

#include <sgblas/sgblas.h>

namespace sgblas::detail {

enum class Work {
  kNothing,   // quick return: no pointer is touched
  kScale,     // C = beta * C (k == 0 or alpha == 0, beta != 1)
  kProduct,   // C = alpha * op(A) op(B) + beta * C
};

struct SgemmPlan {
  Work work = Work::kNothing;
  float alpha = 0.0F;
  float beta = 0.0F;
};

sgblasStatus_t validate(sgblasOperation_t transa, sgblasOperation_t transb,
                        int m, int n, int k, const float *alpha, const float *a,
                        int lda, const float *b, int ldb, const float *beta,
                        const float *c, int ldc, SgemmPlan *plan);

}  // namespace sgblas::detail

#endif  // SGBLAS_B200_VALIDATION_HPP_
