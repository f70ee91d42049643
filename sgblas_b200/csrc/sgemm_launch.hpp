// Host-side launch of the tile kernel: schedule, operand orientation, staging
// path and stream-K scratch. Shared by sgblasSgemm (sgemm.cu), which takes
// its scratch from the handle's workspace, and sgblasSgemmNoAlloc
// (sgemm_noalloc.cu), which uses a fixed array. The per-mode templates are
// instantiated in sgemm_mode_{nn,nt,tn,tt}.cu so that they compile in
// parallel.
#ifndef SGBLAS_B200_SGEMM_LAUNCH_HPP_
#define SGBLAS_B200_SGEMM_LAUNCH_HPP_

#include "context.hpp"
#include "sgemm_tile.cuh"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>

namespace sgblas::detail {

sgblasStatus_t launchStatus(cudaError_t e);

// 3-D tensor map of `batch` column-major rows x cols FP32 matrices (leading
// dimension ld, matrix i at ptr + i*stride floats) read in boxes of
// box_rows x box_cols of one matrix; swizzle64 for k-contiguous tiles whose
// rows are exactly 64 bytes. False if the stride or the driver refuses it.
bool encodeMatrix(CUtensorMap *map, const float *ptr, int rows, int cols, int ld, int batch,
                  long long stride, int box_rows, int box_cols, bool swizzle64);

// 3-D tensor map of `batch` dim0 x dim1 FP32 matrices (dim0 contiguous, rows
// stride1_bytes apart, matrix i at ptr + i * stride_elems floats) read in
// box0 x box1 boxes of one matrix, with the given swizzle. False if the batch
// stride or the driver refuses it.
bool encodeTiled3d(CUtensorMap *map, const float *ptr, unsigned long long dim0,
                   unsigned long long dim1, unsigned long long stride1_bytes, int batch,
                   long long stride_elems, unsigned box0, unsigned box1,
                   CUtensorMapSwizzle swizzle);

bool aligned16(const void *p);



int smCount(int device);

// 1 if `device` is compute capability 10.0 (what the kernels are built for),
// 0 if not (callers return SGBLAS_STATUS_ARCH_MISMATCH), -1 on an error.
int isSm100(int device);

// Persistent schedule: one CTA per SM. Whole tiles are dealt round-robin;
// when the tile count leaves a partial last wave, the last (full wave +
// remainder) tiles are split by k iterations over all CTAs (stream-K), so every
// SM finishes at the same time. Problems with fewer tiles than SMs are split
// the same way, down to kMinSkIters k slices per CTA, or into the same whole
// number of pieces per tile when that costs less (see makeSchedule).
struct Schedule {
  int grid = 0, dp_tiles = 0, sk_tiles = 0, sk_q = 0, sk_r = 0;
};
constexpr int kMinSkIters = 4;
constexpr int kItemCostIters = 3;   // a stream-K part's fix-up and epilogue, in k iterations
Schedule makeSchedule(long long tiles, int kiters, int sms);

// Scratch layout: [arrival counters (kCounterRegionBytes) | partial slots].
// The counter region holds kMaxCounters 8-byte arrival counters (epoch and
// count, kern::arriveCounter); sk_tiles <= 2 * grid <= 2 * SMs, so they cover
// any GPU with up to 512 SMs. The region has a fixed size so that the layout
// is the same for every call (one launch's counters must never be overlapped
// by another launch's slots).
constexpr size_t kSlotBytes = kern::Geo<16>::kSlotBytes;  // the largest slot (128 KiB)
constexpr size_t kCounterRegionBytes = 8192;
using Counter = unsigned long long;
constexpr size_t kMaxCounters = kCounterRegionBytes / sizeof(Counter);   // 1024

// A batch of products sharing sizes, leading dimensions and scalars: matrix
// i is A + i*stride_a (B, C alike), or a_ptrs[i] etc. when the caller passed
// device arrays of pointers. One matrix: count 1, no arrays.
struct Batch {
  int count = 1;
  long long stride_a = 0, stride_b = 0, stride_c = 0;
  const float *const *a_ptrs = nullptr;
  const float *const *b_ptrs = nullptr;
  float *const *c_ptrs = nullptr;
};

// Where a launch takes its stream-K scratch from.
struct Scratch {
  sgblasContext *ctx = nullptr;      // the handle's workspace (may allocate), or
  unsigned char *fixed = nullptr;    // a fixed device array of fixed_bytes
  size_t fixed_bytes = 0;
};

// Operand staging copies in the handle workspace (sgemm_pack.cu). The
// workspace layout with packed operands is [counters | 2*SMs slots | packed
// A | packed B], so the stream-K part keeps the same offsets on every call.
constexpr size_t kPackAlign = 256;
constexpr int kPackLdMultiple = 32;  // floats: 128-byte aligned columns
// A k-contiguous operand that TMA could read in place is still copied to the
// x-contiguous layout when the product is large: the kernel then runs without
// in-kernel transposes (about 2-3 % faster at 4096^3 and 8192^3, measured),
// and the copy -- 8 bytes of HBM traffic per element -- is repaid when the
// other dimension of C reuses each element at least kPackReuse times. Copies
// above kPackMaxBytes are not made (the workspace keeps its size).
constexpr long long kPackReuse = 3072;
constexpr size_t kPackMaxBytes = size_t{512} << 20;
inline size_t streamKRegionBytes(int sms) {
  return kCounterRegionBytes + 2 * static_cast<size_t>(sms) * kSlotBytes;
}
// Writes the operand whose element (x, k) is at src[x + k*ld]
// (k_contiguous false) or src[k + x*ld] (k_contiguous true) to dst as an
// rows_x x cols_k column-major matrix with leading dimension ldp (a multiple
// of 4; dst 16-byte aligned).
sgblasStatus_t launchPack(const float *src, int ld, bool k_contiguous, int rows_x, int cols_k,
                          float *dst, int ldp, int sms, cudaStream_t stream);

// Provides [counters | 2*grid slots] for a stream-K launch on `stream`.
// The handle workspace is grow-only and allocated stream-ordered; false when
// it cannot be provided (the caller then schedules whole tiles only). While
// `stream` is being captured into a CUDA graph it is never allocated or
// grown, and launches are not ordered by its event (the graph orders them).
bool ensureWorkspace(sgblasContext *ctx, size_t bytes, int device, cudaStream_t stream);
// Marks the end of a launch that used the handle workspace.
bool markWorkspaceUse(sgblasContext *ctx, cudaStream_t stream);
// Counter epoch for the next launch that uses the handle workspace's arrival
// counters: one more than the last (never 0). When the 32-bit epoch wraps,
// every counter is first cleared on `stream`, so that no value an earlier
// launch left can match. 0 if that clear could not be enqueued.
unsigned nextCounterEpoch(sgblasContext *ctx, cudaStream_t stream);
// Clears `count` counters of a fixed scratch array on `stream` (launches on
// a fixed array use epoch 1 after the clear). False if it cannot be enqueued.
bool clearFixedCounters(unsigned char *fixed, size_t count, cudaStream_t stream);

// The TF32 lane (tf32.cu): the tensor-core kernel reads both operands with
// TMA, so their bases must be 16-byte aligned and their leading dimensions
// multiples of 4 floats.
inline bool tf32Eligible(const float *a, int lda, const float *b, int ldb) {
  return aligned16(a) && aligned16(b) && lda % 4 == 0 && ldb % 4 == 0;
}
// One product, or a strided batch, in TF32 (p carries pointers, sizes,
// scalars, batch strides and the error word). Pointer-array batches are not
// handled here.
sgblasStatus_t launchTf32(bool ta, bool tb, const kern::GemmParams &p, const Scratch &scratch,
                          int device, cudaStream_t stream);

// The small-problem kernel (sgemm_small.cu): 64 x 64 tiles of C, each computed
// by one or more clusters of 1-8 CTAs that split its k range and sum their
// partial tiles through distributed shared memory (and, with several
// clusters per tile, through the stream-K scratch); any alignment, leading
// dimension, transpose or batch form. Chosen when the persistent kernel's
// 128 x 128 tiles number at most SMs / kSmallTileShare and the busiest SM
// of the cluster kernel has at most kSmallMaxFmaPerSm multiply-adds.
constexpr long long kSmallTileShare = 4;
constexpr double kSmallMaxFmaPerSm = 2097152.0;   // 2^21 (512^3: 2^20 on 148 SMs)
bool smallEligible(const kern::GemmParams &p, int sms);
// p carries pointers, sizes, scalars and the batch (strides or arrays).
sgblasStatus_t launchSmall(bool ta, bool tb, const kern::GemmParams &p, const Scratch &scratch,
                           int device, int sms, cudaStream_t stream);

// Launches one product of transpose mode (kTA, kTB). p carries the problem
// (pointers, sizes, alpha, beta, error word); the launcher fills in the rest.
template <bool kTA, bool kTB>
sgblasStatus_t launchMode(kern::GemmParams p, const Scratch &scratch, int device,
                          cudaStream_t stream);

extern template sgblasStatus_t launchMode<false, false>(kern::GemmParams, const Scratch &, int,
                                                        cudaStream_t);
extern template sgblasStatus_t launchMode<false, true>(kern::GemmParams, const Scratch &, int,
                                                       cudaStream_t);
extern template sgblasStatus_t launchMode<true, false>(kern::GemmParams, const Scratch &, int,
                                                       cudaStream_t);
extern template sgblasStatus_t launchMode<true, true>(kern::GemmParams, const Scratch &, int,
                                                      cudaStream_t);

}  // namespace sgblas::detail

#endif  // SGBLAS_B200_SGEMM_LAUNCH_HPP_
