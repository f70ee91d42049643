// launchMode<false, true>: the NT kernels (both orientations, both staging
// paths, three beta modes), in a translation unit of their own so that the
// four transpose modes compile in parallel.
#include "sgemm_launch.cuh"

namespace sgblas::detail {
template sgblasStatus_t launchMode<false, true>(kern::GemmParams, const Scratch &, int, cudaStream_t);
}  // namespace sgblas::detail
