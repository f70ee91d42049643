// Library context behind the opaque sgblasHandle_t.
//
// Mirrors the reference's two-field context (src/handle_internal.hpp:6-9 of
// AG0708/sgBLAS: stream + math mode) and adds the device workspace used by
// the split-K reduction, which the reference does not have. The workspace is
// grow-only, owned by the context, allocated stream-ordered on the handle's
// stream and released in sgblasDestroy.
#ifndef SGBLAS_B200_CONTEXT_HPP_
#define SGBLAS_B200_CONTEXT_HPP_

#include <sgblas/sgblas.h>

#include <cstddef>

struct sgblasContext {
  sgblasStream_t stream = nullptr;
  sgblasMathMode_t math_mode = SGBLAS_MATH_FP32;

  // Stream-K workspace: arrival counters, then FP32 partial-tile slots.
  // device == -1 means nothing allocated. `workspace_event` (a cudaEvent_t)
  // marks the last launch that used the workspace, so that a launch on a
  // different stream is ordered after it.
  void *workspace = nullptr;
  std::size_t workspace_bytes = 0;
  int workspace_device = -1;
  void *workspace_event = nullptr;
  // Epoch of the last launch that used the workspace's arrival counters
  // (each such launch takes the next one; see kern::arriveCounter).
  unsigned workspace_epoch = 0;
};

namespace sgblas::detail {
// Releases the context's device workspace (defined with the CUDA code; a
// no-op when nothing was allocated).
void releaseWorkspace(sgblasContext *context);
}  // namespace sgblas::detail

#endif  // SGBLAS_B200_CONTEXT_HPP_
