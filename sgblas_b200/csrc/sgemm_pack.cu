// Operand staging copies: an operand that TMA cannot read in place (its base
// is not 16-byte aligned or its leading dimension is not a multiple of 4
// floats) is first copied into the handle's workspace as an X x K
// column-major matrix whose leading dimension is a multiple of 32 floats --
// x (the operand's side of C: m for A, n for B) contiguous, the layout the
// tile kernel's compute warps read. The copy is HBM-bound (read once, write
// once) and replaces the tile kernel's 4- or 8-byte cp.async staging, which
// saturates the producer warpgroup, and any in-kernel transposition of that
// operand.
#include "ptx.cuh"
#include "sgemm_launch.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

namespace sgblas::detail {

namespace {

constexpr int kPackThreads = 256;

// x-contiguous source: element (x, k) at src[x + k * ld]. One tile is 1024
// consecutive x of one column; each thread moves four x with scalar loads
// (the source may be unaligned) and one aligned float4 store.
__global__ __launch_bounds__(kPackThreads) void packColumnsKernel(const float *__restrict__ src,
                                                                 int ld, int rows_x, int cols_k,
                                                                 float *__restrict__ dst, int ldp,
                                                                 int tiles_x, long long tiles) {
  kern::gridDependencyWait();
  kern::allowDependentLaunch();
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int k = static_cast<int>(t / tiles_x);
    const int x = static_cast<int>(t % tiles_x) * (4 * kPackThreads) + 4 * threadIdx.x;
    if (x >= rows_x) continue;
    const float *sp = src + static_cast<size_t>(k) * ld + x;
    float4 v;
    v.x = sp[0];
    v.y = x + 1 < rows_x ? sp[1] : 0.0F;
    v.z = x + 2 < rows_x ? sp[2] : 0.0F;
    v.w = x + 3 < rows_x ? sp[3] : 0.0F;
    *reinterpret_cast<float4 *>(dst + static_cast<size_t>(k) * ldp + x) = v;
  }
  (void)cols_k;
}

// k-contiguous source: element (x, k) at src[k + x * ld]. Tiles of 32 x by
// 64 k through shared memory: warps read 32 consecutive k of one x (eight
// independent loads per thread, issued together) and write 32 consecutive x
// of one k; the padded row makes both shared accesses conflict-free.
constexpr int kTile = 32;
constexpr int kTileK = 64;
__global__ __launch_bounds__(kPackThreads) void packTransposeKernel(const float *__restrict__ src,
                                                                   int ld, int rows_x, int cols_k,
                                                                   float *__restrict__ dst,
                                                                   int ldp, int tiles_x,
                                                                   long long tiles) {
  __shared__ float tile[kTile][kTileK + 1];
  const int lane = threadIdx.x % 32, row = threadIdx.x / 32;
  constexpr int kRowsPerPass = kPackThreads / 32;
  kern::gridDependencyWait();
  kern::allowDependentLaunch();
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int x0 = static_cast<int>(t % tiles_x) * kTile;
    const int k0 = static_cast<int>(t / tiles_x) * kTileK;
    float v[kTile / kRowsPerPass][2];
#pragma unroll
    for (int i = 0; i < kTile / kRowsPerPass; ++i) {
      const int x = x0 + row + i * kRowsPerPass;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int k = k0 + lane + 32 * h;
        v[i][h] = (x < rows_x && k < cols_k) ? src[static_cast<size_t>(x) * ld + k] : 0.0F;
      }
    }
#pragma unroll
    for (int i = 0; i < kTile / kRowsPerPass; ++i)
#pragma unroll
      for (int h = 0; h < 2; ++h) tile[row + i * kRowsPerPass][lane + 32 * h] = v[i][h];
    __syncthreads();
#pragma unroll
    for (int r = row; r < kTileK; r += kRowsPerPass) {
      const int k = k0 + r, x = x0 + lane;
      if (k < cols_k && x < rows_x) dst[static_cast<size_t>(k) * ldp + x] = tile[lane][r];
    }
    __syncthreads();
  }
}

}  // namespace

sgblasStatus_t launchPack(const float *src, int ld, bool k_contiguous, int rows_x, int cols_k,
                          float *dst, int ldp, int sms, cudaStream_t stream) {
  int tiles_x;
  long long tiles;
  const void *kernel;
  if (k_contiguous) {
    tiles_x = (rows_x + kTile - 1) / kTile;
    tiles = static_cast<long long>(tiles_x) * ((cols_k + kTileK - 1) / kTileK);
    kernel = reinterpret_cast<const void *>(packTransposeKernel);
  } else {
    tiles_x = (rows_x + 4 * kPackThreads - 1) / (4 * kPackThreads);
    tiles = static_cast<long long>(tiles_x) * cols_k;
    kernel = reinterpret_cast<const void *>(packColumnsKernel);
  }
  // Eight resident 256-thread blocks per SM cover the latency of the loads.
  const long long grid = std::min<long long>(tiles, static_cast<long long>(sms) * 8);
  void *args[] = {&src, &ld, &rows_x, &cols_k, &dst, &ldp, &tiles_x, &tiles};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kPackThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1] = {};
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return launchStatus(cudaLaunchKernelExC(&cfg, kernel, args));
}

}  // namespace sgblas::detail
