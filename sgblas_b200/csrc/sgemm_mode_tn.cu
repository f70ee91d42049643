// launchMode<true, false>: the TN kernels (both orientations, both staging
// paths, three beta modes), in a translation unit of their own so that the
// four transpose modes compile in parallel.
#include "sgemm_launch.cuh"

namespace sgblas::detail {
template sgblasStatus_t launchMode<true, false>(kern::GemmParams, const Scratch &, int, cudaStream_t);
}  // namespace sgblas::detail
