// See validation.hpp. Reference: src/sgemm_validation.cpp:14-66.
#include "validation.hpp"

namespace sgblas::detail {
namespace {

bool isOp(sgblasOperation_t op) { return op == SGBLAS_OP_N || op == SGBLAS_OP_T; }

int atLeastOne(int v) { return v < 1 ? 1 : v; }

}  // namespace

sgblasStatus_t validate(sgblasOperation_t transa, sgblasOperation_t transb,
                        int m, int n, int k, const float *alpha, const float *a,
                        int lda, const float *b, int ldb, const float *beta,
                        const float *c, int ldc, SgemmPlan *plan) {
  if (plan == nullptr) return SGBLAS_STATUS_INTERNAL_ERROR;
  *plan = SgemmPlan{};

  if (!isOp(transa) || !isOp(transb) || m < 0 || n < 0 || k < 0)
    return SGBLAS_STATUS_INVALID_VALUE;

  // Leading-dimension minima of column-major storage: op(A) is m x k, so A is
  // stored m x k (N) or k x m (T); likewise B is k x n (N) or n x k (T).
  const int need_lda = atLeastOne(transa == SGBLAS_OP_N ? m : k);
  const int need_ldb = atLeastOne(transb == SGBLAS_OP_N ? k : n);
  const int need_ldc = atLeastOne(m);
  if (lda < need_lda || ldb < need_ldb || ldc < need_ldc)
    return SGBLAS_STATUS_INVALID_VALUE;

  // Empty C: a true quick return, neither scalars nor matrices are read.
  if (m == 0 || n == 0) return SGBLAS_STATUS_SUCCESS;

  if (alpha == nullptr || beta == nullptr) return SGBLAS_STATUS_INVALID_VALUE;
  plan->alpha = *alpha;
  plan->beta = *beta;

  const bool product = k > 0 && plan->alpha != 0.0F;
  if (!product) {
    if (plan->beta == 1.0F) return SGBLAS_STATUS_SUCCESS;  // C unchanged
    if (c == nullptr) return SGBLAS_STATUS_INVALID_VALUE;
    plan->work = Work::kScale;
    return SGBLAS_STATUS_SUCCESS;
  }
  if (a == nullptr || b == nullptr || c == nullptr)
    return SGBLAS_STATUS_INVALID_VALUE;
  plan->work = Work::kProduct;
  return SGBLAS_STATUS_SUCCESS;
}

}  // namespace sgblas::detail
