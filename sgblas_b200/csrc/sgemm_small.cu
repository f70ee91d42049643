// The small-problem kernel: products too small to fill the GPU with the
// persistent tile kernel's 128 x 128 tiles (256^3, 512^3, deep-k products
// with a small C, a few small batched matrices).
//
// Replaces the reference's small kernel family (64-row tiles,
// src/sgemm_cuda.cu:598-640, sgemm_async_sm80_small.hpp) with a design for
// 148 SMs:
//   - C is cut into 64- or 128-row x 64-column tiles. Each tile's k range is
//     divided among `groups` thread-block clusters of `split` CTAs (split 1,
//     2, 4 or 8; groups > 1 only for deep k), chosen to give as many SMs as
//     possible one CTA: a 256^3 product runs on 128 SMs instead of 16. The
//     extra clusters of a deep-k product may put two 64-row CTAs on an SM.
//     Without a split (split 1) the kernel is launched without clusters.
//   - Every CTA stages its k slices (32 deep) with 4-byte cp.async into a
//     4-stage ring, any alignment, leading dimension or transpose, with zero
//     fill outside the matrix; 256 threads each compute a 4 x 4 (or 8 x 4)
//     block of the tile with paired FMAs (fma.rn.f32x2), reading the next
//     k step's fragments while the current one computes.
//   - The cluster's partial tiles are summed through distributed shared
//     memory: CTA r reads its 1/split share of the tile from every CTA of the
//     cluster in rank order. With one cluster per tile it then applies the
//     alpha/beta epilogue and writes C: no workspace, counters or atomics, so
//     the kernel runs the same way from sgblasSgemm, sgblasSgemmNoAlloc and
//     inside a CUDA graph. With several clusters per tile, each stores its
//     sum in the stream-K scratch and the last cluster to arrive (an arrival
//     counter per tile and share) adds the stored sums in cluster order.
//     Either way the summation order is fixed: results are deterministic.
//   - Programmatic dependent launch: the prologue overlaps the previous
//     kernel on the stream, and global memory is first read after
//     griddepcontrol.wait.
// Results obey the same bound as every other path (the reference's error
// model: the k products are summed in FP32 in some order).
#include "device.hpp"
#include "ptx.cuh"
#include "sgemm_launch.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdint>

namespace sgblas::kern::small {

constexpr int kBN = 64;         // tile columns (n)
constexpr int kBK = 32;         // k slice per stage
constexpr int kStages = 4;
constexpr int kThreads = 256;   // a 16 x 16 grid of threads over the tile
constexpr int kTN = kBN / 16;   // columns per thread
constexpr int kRowB = kBN + 4;  // floats per staged k row (padding: no bank conflicts)
constexpr int kMaxSplit = 8;    // portable cluster size
static_assert(kTN == 4, "4 columns per thread");

// Tiles of kBM (64 or 128) rows x kBN columns.
template <int kBM>
struct Tile {
  static constexpr int kTM = kBM / 16;       // rows per thread
  static constexpr int kRowA = kBM + 4;
  static constexpr int kTileA = kBK * kRowA;
  static constexpr int kStageFloats = kTileA + kBK * kRowB;
  static constexpr int kSmemBytes = kStages * kStageFloats * 4;
  static constexpr int kColGroups = kBM / 4;  // float4 groups per tile column
  static constexpr int kGroups = kBM * kBN / 4;
  static_assert(kTM % 4 == 0, "whole float4s of rows per thread");
  static_assert(kBN * kRowA <= kStages * kStageFloats, "the partial tile fits in the ring");
  static_assert(kGroups % kThreads == 0, "whole groups per thread");
};

struct Params {
  const float *a, *b;
  float *c;
  const float *const *a_ptrs;   // pointer-array batches (else nullptr)
  const float *const *b_ptrs;
  float *const *c_ptrs;
  long long stride_a, stride_b, stride_c;
  int m, n, k, lda, ldb, ldc;
  float alpha, beta;
  int tiles_m;
  int split;      // CTAs per cluster
  int groups;     // clusters per tile
  int slices;     // kBK slices of k
  int per_cta;    // slices per CTA: CTA r of cluster g owns chunk g*split + r
  int c_vec;      // C columns can be read and written as float4
  float4 *ws;     // groups > 1: one partial tile per (tile, cluster)
  unsigned long long *counters;  // groups > 1: arrivals per (tile, rank) (arriveCounter)
  unsigned epoch;                // this launch's counter epoch
  unsigned *err;                 // device error word
};

// Issues the copies of one operand's kX x kBK slice into a [k][x] buffer
// (row stride kX + 4). Element (x, k) of the operand is at src[x + k*ld]
// (kKContig false) or src[k + x*ld] (kKContig true). Within a warp the
// lanes read 32 consecutive floats (x-contiguous) or four runs of 8 (k-
// contiguous), and write 32 different banks.
template <int kX, bool kKContig>
__device__ __forceinline__ void loadSlice(float *dst, const float *src, int ld, int x0, int xlim,
                                          int k0, int klim, int tid) {
  constexpr int kRow = kX + 4;
#pragma unroll
  for (int j = 0; j < kX * kBK / kThreads; ++j) {
    const int idx = tid + j * kThreads;
    int xl, kl;
    if constexpr (kKContig) {
      const int lane = idx & 31, w = idx >> 5;
      kl = (w & 3) * 8 + (lane & 7);
      xl = (w >> 2) * 4 + (lane >> 3);
    } else {
      xl = idx & (kX - 1);
      kl = idx / kX;
    }
    const int x = x0 + xl, kk = k0 + kl;
    const bool ok = x < xlim && kk < klim;
    const long long off = kKContig ? static_cast<long long>(x) * ld + kk
                                   : static_cast<long long>(kk) * ld + x;
    cpAsync4(dst + kl * kRow + xl, ok ? src + off : src, ok ? 4u : 0u);
  }
}

template <Beta kBeta>
__device__ __forceinline__ float4 loadC(const float *cp, int rows, bool vec) {
  float4 v = make_float4(0.F, 0.F, 0.F, 0.F);
  if constexpr (kBeta != Beta::kZero) {
    if (vec && rows >= 4) {
      v = *reinterpret_cast<const float4 *>(cp);
    } else {
      if (rows > 0) v.x = cp[0];
      if (rows > 1) v.y = cp[1];
      if (rows > 2) v.z = cp[2];
      if (rows > 3) v.w = cp[3];
    }
  }
  return v;
}

template <int kBM, bool kTA, bool kTB, Beta kBeta>
__global__ void __launch_bounds__(kThreads, kBM == 64 ? 2 : 1)
    smallKernel(const __grid_constant__ Params p) {
  using T = Tile<kBM>;
  constexpr int kTM = T::kTM, kRowA = T::kRowA, kTileA = T::kTileA;
  constexpr int kStageFloats = T::kStageFloats, kColGroups = T::kColGroups;
  constexpr int kGroups = T::kGroups;
  extern __shared__ __align__(16) float smem[];
  __shared__ int last_arrival;
  const int tid = static_cast<int>(threadIdx.x);
  const int split = p.split, groups = p.groups;
  // split 1 is launched without clusters: the CTA's index is its tile's.
  const int rank = split > 1 ? static_cast<int>(clusterRank()) : 0;
  const int cluster = split > 1 ? static_cast<int>(clusterIdX()) : static_cast<int>(blockIdx.x);
  const int tile_m = cluster / groups, grp = cluster - tile_m * groups;
  const int m0 = tile_m * kBM;
  const int n0 = static_cast<int>(blockIdx.y) * kBN;
  const int bi = static_cast<int>(blockIdx.z);
  const int t0 = (grp * split + rank) * p.per_cta;
  const int nt = max(0, min(p.slices - t0, p.per_cta));

  gridDependencyWait();   // A, B, C (and pointer arrays) may come from the previous kernel
  const float *A = p.a_ptrs != nullptr ? p.a_ptrs[bi] : p.a + bi * p.stride_a;
  const float *B = p.b_ptrs != nullptr ? p.b_ptrs[bi] : p.b + bi * p.stride_b;
  float *C = p.c_ptrs != nullptr ? p.c_ptrs[bi] : p.c + bi * p.stride_c;

  auto load = [&](int stage, int t) {
    float *as = smem + stage * kStageFloats;
    const int k0 = t * kBK;
    loadSlice<kBM, kTA>(as, A, p.lda, m0, p.m, k0, p.k, tid);             // op(A)(m, k)
    loadSlice<kBN, !kTB>(as + kTileA, B, p.ldb, n0, p.n, k0, p.k, tid);   // op(B)(k, n)
  };

  const int tx = tid & 15, ty = tid >> 4;   // the thread's kTN columns / kTM rows of the tile
  float2 acc[kTM][kTN / 2];
#pragma unroll
  for (int i = 0; i < kTM; ++i) acc[i][0] = acc[i][1] = make_float2(0.F, 0.F);

#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < nt) load(s, t0 + s);
    cpAsyncCommit();
  }
  for (int i = 0; i < nt; ++i) {
    cpAsyncWait<kStages - 2>();
    __syncthreads();   // slice i landed; every thread is done with slice i - 1's stage
    if (i + kStages - 1 < nt) load((i + kStages - 1) % kStages, t0 + i + kStages - 1);
    cpAsyncCommit();
    const float *as = smem + (i % kStages) * kStageFloats + ty * kTM;
    const float *bs = smem + (i % kStages) * kStageFloats + kTileA + tx * kTN;
    // Fragments of step kk + 1 are read while step kk computes. The 64-row
    // loop is unrolled 4 steps deep, not 32: a small product runs this code
    // once per SM from a cold instruction cache, and the shorter loop took
    // 256^3 from 8.3 to 6.2 us per call (back to back, B200).
    float4 a[kTM / 4], b;
#pragma unroll
    for (int v = 0; v < kTM / 4; ++v) a[v] = *reinterpret_cast<const float4 *>(as + 4 * v);
    b = *reinterpret_cast<const float4 *>(bs);
#pragma unroll (kBM == 64 ? 4 : kBK)
    for (int kk = 0; kk < kBK; ++kk) {
      float4 an[kTM / 4], bn = b;
#pragma unroll
      for (int v = 0; v < kTM / 4; ++v) an[v] = a[v];
      if (kk + 1 < kBK) {
#pragma unroll
        for (int v = 0; v < kTM / 4; ++v)
          an[v] = *reinterpret_cast<const float4 *>(as + (kk + 1) * kRowA + 4 * v);
        bn = *reinterpret_cast<const float4 *>(bs + (kk + 1) * kRowB);
      }
      const float2 b01 = make_float2(b.x, b.y), b23 = make_float2(b.z, b.w);
#pragma unroll
      for (int v = 0; v < kTM / 4; ++v) {
        const float av[4] = {a[v].x, a[v].y, a[v].z, a[v].w};
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const float2 ar = make_float2(av[r], av[r]);
          acc[4 * v + r][0] = __ffma2_rn(ar, b01, acc[4 * v + r][0]);
          acc[4 * v + r][1] = __ffma2_rn(ar, b23, acc[4 * v + r][1]);
        }
      }
#pragma unroll
      for (int v = 0; v < kTM / 4; ++v) a[v] = an[v];
      b = bn;
    }
  }
  cpAsyncWait<0>();
  allowDependentLaunch();

  // This CTA's share of the tile: float4 groups [lo, hi) in column-major
  // order (group q holds rows 4*(q % kColGroups) .. +3 of column
  // q / kColGroups).
  const int lo = rank * kGroups / split, hi = (rank + 1) * kGroups / split;
  constexpr int kPerThread = kGroups / kThreads;
  auto rowsAt = [&](int q) { return p.m - (m0 + (q % kColGroups) * 4); };
  auto colAt = [&](int q) { return n0 + q / kColGroups; };
  auto cAt = [&](int q) {
    return C + static_cast<long long>(colAt(q)) * p.ldc + m0 + (q % kColGroups) * 4;
  };
  float4 cold[kPerThread];
#pragma unroll
  for (int u = 0; u < kPerThread; ++u) {
    const int q = lo + tid + u * kThreads;
    cold[u] = make_float4(0.F, 0.F, 0.F, 0.F);
    if (groups == 1 && q < hi && rowsAt(q) > 0 && colAt(q) < p.n)
      cold[u] = loadC<kBeta>(cAt(q), rowsAt(q), p.c_vec != 0);
  }

  // Partial tile, column-major with row stride kRowA, over the ring.
  __syncthreads();   // every thread's last reads of the ring are done
  float *part = smem;
#pragma unroll
  for (int j = 0; j < kTN; ++j) {
#pragma unroll
    for (int v = 0; v < kTM / 4; ++v) {
      const float4 val =
          (j & 1) == 0
              ? make_float4(acc[4 * v][j >> 1].x, acc[4 * v + 1][j >> 1].x,
                            acc[4 * v + 2][j >> 1].x, acc[4 * v + 3][j >> 1].x)
              : make_float4(acc[4 * v][j >> 1].y, acc[4 * v + 1][j >> 1].y,
                            acc[4 * v + 2][j >> 1].y, acc[4 * v + 3][j >> 1].y);
      *reinterpret_cast<float4 *>(part + (tx * kTN + j) * kRowA + ty * kTM + 4 * v) = val;
    }
  }
  // Every CTA's partial tile is written and visible to the cluster (a CTA
  // launched alone only needs its own threads).
  if (split == 1) __syncthreads();
  else clusterSync();

  // The cluster's sum of this CTA's share, CTA by CTA in rank order.
  const uint32_t part_addr = smemAddr(part);
  float4 sum[kPerThread];
#pragma unroll
  for (int u = 0; u < kPerThread; ++u) {
    const int q = lo + tid + u * kThreads;
    sum[u] = make_float4(0.F, 0.F, 0.F, 0.F);
    if (q >= hi) continue;
    const uint32_t off =
        static_cast<uint32_t>(((q / kColGroups) * kRowA + (q % kColGroups) * 4) * 4);
    if (split == 1) {
      sum[u] = *reinterpret_cast<const float4 *>(reinterpret_cast<const char *>(part) + off);
      continue;
    }
    // All of the cluster's reads are issued before the first add.
    float4 v[kMaxSplit];
#pragma unroll
    for (int r = 0; r < kMaxSplit; ++r)
      if (r < split) v[r] = ldCluster4(clusterAddr(part_addr + off, static_cast<uint32_t>(r)));
    sum[u] = v[0];
#pragma unroll
    for (int r = 1; r < kMaxSplit; ++r) {
      if (r < split) {
        sum[u].x += v[r].x;
        sum[u].y += v[r].y;
        sum[u].z += v[r].z;
        sum[u].w += v[r].w;
      }
    }
  }
  // The other CTAs have read this CTA's partial tile before it may exit. The
  // arrive has release semantics so that each CTA's distributed-shared-memory
  // reads are complete before it counts as arrived, whatever order the
  // compiler gives the adds that consume them.
  if (split > 1) clusterSync();

  if (groups > 1) {
    // Several clusters share the tile: each stores its sum, and for every
    // share the last of them to arrive adds the stored sums in cluster
    // order and writes C (same result whatever the arrival order).
    const long long tile =
        (static_cast<long long>(bi) * gridDim.y + blockIdx.y) * p.tiles_m + tile_m;
    float4 *slots = p.ws + tile * groups * kGroups;
#pragma unroll
    for (int u = 0; u < kPerThread; ++u) {
      const int q = lo + tid + u * kThreads;
      if (q < hi) __stcg(slots + grp * kGroups + q, sum[u]);
    }
    __threadfence();
    __syncthreads();
    unsigned long long *counter = p.counters + tile * split + rank;
    if (tid == 0)
      last_arrival = arriveCounter(counter, p.epoch, p.err) == static_cast<unsigned>(groups);
    __syncthreads();
    if (!last_arrival) return;
    __threadfence();
#pragma unroll
    for (int u = 0; u < kPerThread; ++u) {
      const int q = lo + tid + u * kThreads;
      if (q >= hi) continue;
      sum[u] = __ldcg(slots + q);
      for (int g = 1; g < groups; ++g) {
        const float4 v = __ldcg(slots + g * kGroups + q);
        sum[u].x += v.x;
        sum[u].y += v.y;
        sum[u].z += v.z;
        sum[u].w += v.w;
      }
      if (rowsAt(q) > 0 && colAt(q) < p.n)
        cold[u] = loadC<kBeta>(cAt(q), rowsAt(q), p.c_vec != 0);
    }
    if (tid == 0) *counter = 0;   // every cluster of the tile has arrived
  }

  const float alpha = p.alpha, beta = p.beta;
#pragma unroll
  for (int u = 0; u < kPerThread; ++u) {
    const int q = lo + tid + u * kThreads;
    const int rows = rowsAt(q);
    if (q >= hi || rows <= 0 || colAt(q) >= p.n) continue;
    float *cp = cAt(q);
    float4 out;
    out.x = epilogueValue<kBeta>(sum[u].x, alpha, beta, cold[u].x);
    out.y = epilogueValue<kBeta>(sum[u].y, alpha, beta, cold[u].y);
    out.z = epilogueValue<kBeta>(sum[u].z, alpha, beta, cold[u].z);
    out.w = epilogueValue<kBeta>(sum[u].w, alpha, beta, cold[u].w);
    if (p.c_vec != 0 && rows >= 4) {
      *reinterpret_cast<float4 *>(cp) = out;
    } else {
      cp[0] = out.x;
      if (rows > 1) cp[1] = out.y;
      if (rows > 2) cp[2] = out.z;
      if (rows > 3) cp[3] = out.w;
    }
  }
}

}  // namespace sgblas::kern::small

namespace sgblas::detail {

namespace {

using kern::Beta;
namespace sm = kern::small;

long long ceilDiv(long long a, long long b) { return (a + b - 1) / b; }

template <int kBM, bool kTA, bool kTB, Beta kBeta>
sgblasStatus_t launchTyped(const sm::Params &p, dim3 grid, int device, cudaStream_t stream) {
  auto kernel = sm::smallKernel<kBM, kTA, kTB, kBeta>;
  constexpr int kSmem = sm::Tile<kBM>::kSmemBytes;
  static std::atomic<uint64_t> configured{0};
  if (!configureKernel(reinterpret_cast<const void *>(kernel), device, kSmem, &configured))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(sm::kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  // Without a split each CTA is its own (implicit) cluster: no cluster
  // attribute, which launches faster (0.56 against 0.97 us per empty launch
  // back to back on B200).
  cudaLaunchAttribute attr[2] = {};
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(p.split);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.split > 1 ? 2 : 1;
  return launchStatus(cudaLaunchKernelEx(&cfg, kernel, p));
}

template <int kBM, bool kTA, bool kTB>
sgblasStatus_t launchByBeta(const sm::Params &p, dim3 grid, int device, cudaStream_t stream) {
  if (p.beta == 0.0F) return launchTyped<kBM, kTA, kTB, Beta::kZero>(p, grid, device, stream);
  if (p.beta == 1.0F) return launchTyped<kBM, kTA, kTB, Beta::kOne>(p, grid, device, stream);
  return launchTyped<kBM, kTA, kTB, Beta::kGeneral>(p, grid, device, stream);
}

template <int kBM>
sgblasStatus_t launchByMode(bool ta, bool tb, const sm::Params &p, dim3 grid, int device,
                            cudaStream_t stream) {
  if (!ta && !tb) return launchByBeta<kBM, false, false>(p, grid, device, stream);
  if (!ta && tb) return launchByBeta<kBM, false, true>(p, grid, device, stream);
  if (ta && !tb) return launchByBeta<kBM, true, false>(p, grid, device, stream);
  return launchByBeta<kBM, true, true>(p, grid, device, stream);
}

// CTAs per cluster: the largest power of two up to kMaxSplit that keeps the
// CTAs within `slots` (resident CTAs the GPU holds at once) and at least one
// k slice per CTA.
int chooseSplit(long long tiles, int slices, long long slots) {
  int split = 1;
  while (split * 2 <= sm::kMaxSplit && split * 2 <= slices && tiles * split * 2 <= slots)
    split *= 2;
  return split;
}

// Clusters per tile: more than one only when the tiles' clusters would
// leave over half the slots empty and k is deep enough to give every CTA
// kMinSlicesPerCta slices.
constexpr int kMinSlicesPerCta = 4;
int chooseGroups(long long tiles, int split, int slices, long long slots) {
  const long long ctas = tiles * split;
  if (ctas * 2 > slots) return 1;
  const long long by_slots = slots / ctas;
  const long long by_k = slices / (static_cast<long long>(split) * kMinSlicesPerCta);
  return static_cast<int>(std::max(1LL, std::min(by_slots, by_k)));
}

// Resident CTAs per SM: two of the 64-row kernel (at most 128 registers per
// thread and 70 KB of shared memory each), one of the 128-row kernel.
constexpr int ctasPerSm(int bm) { return bm == 64 ? 2 : 1; }

struct SmallPlan {
  int bm;   // tile rows: 64 or 128
  long long tiles_m, tiles_n, tiles;
  int slices, split, groups, per_cta;
  long long ctas() const { return tiles * split * groups; }
};

SmallPlan planFor(const kern::GemmParams &p, int sms, int bm) {
  SmallPlan s;
  s.bm = bm;
  s.tiles_m = ceilDiv(p.m, bm);
  s.tiles_n = ceilDiv(p.n, sm::kBN);
  s.tiles = s.tiles_m * s.tiles_n * p.batch;
  s.slices = static_cast<int>(ceilDiv(p.k, sm::kBK));
  // Clusters are sized for one CTA per SM; extra clusters for deep k may
  // fill every slot (measured on B200: two CTAs per SM took 128 x 128 x 8192
  // from 25.1 to 19.3 us, but slowed 384^3 from 10.7 to 12.8 us when used
  // for larger clusters).
  s.split = chooseSplit(s.tiles, s.slices, sms);
  s.groups = chooseGroups(s.tiles, s.split, s.slices,
                          static_cast<long long>(sms) * ctasPerSm(bm));
  s.per_cta = static_cast<int>(ceilDiv(s.slices, static_cast<long long>(s.split) * s.groups));
  return s;
}

// 128-row tiles halve the shared-memory reads per FMA, but double each
// cluster's partial-tile traffic and halve the CTA count: they are used
// when they still give over half the SMs a CTA, every CTA at least
// kMinSlicesPerCta k slices and clusters of at most 4 (measured on B200:
// 512^3 12.4 us against 13.7 us with 64-row tiles; with clusters of 8 the
// larger partial tiles cost more than they save); otherwise 64-row tiles.
SmallPlan planSmall(const kern::GemmParams &p, int sms) {
  const SmallPlan tall = planFor(p, sms, 128);
  if (p.m > 64 && tall.ctas() * 2 > sms && tall.per_cta >= kMinSlicesPerCta &&
      tall.split <= 4)
    return tall;
  return planFor(p, sms, 64);
}

}  // namespace

bool smallEligible(const kern::GemmParams &p, int sms) {
  if (p.batch > 65535 || ceilDiv(p.n, sm::kBN) > 65535 ||
      ceilDiv(p.m, 64) * sm::kMaxSplit * sms > INT_MAX)
    return false;
  // The persistent kernel's 128 x 128 tiles would leave most SMs without a
  // whole tile, and each CTA here has little enough work that latency, not
  // FMA throughput, decides the time.
  const long long tiles128 = ceilDiv(p.m, 128) * ceilDiv(p.n, 128) * p.batch;
  if (tiles128 * kSmallTileShare > sms) return false;
  const SmallPlan s = planSmall(p, sms);
  // Multiply-adds on the busiest SM (CTAs are spread over the SMs first).
  const long long ctas = s.ctas();
  const double fma_per_sm = static_cast<double>(p.m) * p.n * p.k * p.batch /
                            static_cast<double>(ctas) * static_cast<double>(ceilDiv(ctas, sms));
  return fma_per_sm <= kSmallMaxFmaPerSm;
}

sgblasStatus_t launchSmall(bool ta, bool tb, const kern::GemmParams &gp, const Scratch &scratch,
                           int device, int sms, cudaStream_t stream) {
  sm::Params p = {};
  p.a = gp.a;
  p.b = gp.b;
  p.c = gp.c;
  p.a_ptrs = gp.a_ptrs;
  p.b_ptrs = gp.b_ptrs;
  p.c_ptrs = gp.c_ptrs;
  p.stride_a = gp.batch > 1 ? gp.stride_a : 0;
  p.stride_b = gp.batch > 1 ? gp.stride_b : 0;
  p.stride_c = gp.batch > 1 ? gp.stride_c : 0;
  p.m = gp.m;
  p.n = gp.n;
  p.k = gp.k;
  p.lda = gp.lda;
  p.ldb = gp.ldb;
  p.ldc = gp.ldc;
  p.alpha = gp.alpha;
  p.beta = gp.beta;
  p.err = gp.err;
  SmallPlan s = planSmall(gp, sms);
  p.tiles_m = static_cast<int>(s.tiles_m);
  p.slices = s.slices;
  p.split = s.split;
  p.groups = s.groups;
  bool used_handle_workspace = false;
  if (p.groups > 1) {
    // [arrival counters | one partial tile per (tile, cluster)], the layout
    // of the tile kernel's stream-K scratch; without it, one cluster per tile.
    const size_t counters = static_cast<size_t>(s.tiles) * s.split;
    const size_t tile_bytes = static_cast<size_t>(s.bm) * sm::kBN * sizeof(float);
    const size_t need =
        kCounterRegionBytes + static_cast<size_t>(s.tiles) * p.groups * tile_bytes;
    unsigned char *base = nullptr;
    if (counters > kMaxCounters) {
      base = nullptr;
    } else if (scratch.fixed != nullptr) {
      if (need <= scratch.fixed_bytes) {
        if (!clearFixedCounters(scratch.fixed, counters, stream))
          return SGBLAS_STATUS_EXECUTION_FAILED;
        base = scratch.fixed;
        p.epoch = 1;
      }
    } else if (ensureWorkspace(scratch.ctx, need, device, stream)) {
      p.epoch = nextCounterEpoch(scratch.ctx, stream);
      if (p.epoch == 0) return SGBLAS_STATUS_EXECUTION_FAILED;
      base = static_cast<unsigned char *>(scratch.ctx->workspace);
      used_handle_workspace = true;
    }
    if (base != nullptr) {
      p.counters = reinterpret_cast<Counter *>(base);
      p.ws = reinterpret_cast<float4 *>(base + kCounterRegionBytes);
    } else {
      p.groups = 1;
    }
  }
  p.per_cta = static_cast<int>(ceilDiv(p.slices, static_cast<long long>(p.split) * p.groups));
  p.c_vec = gp.c_ptrs == nullptr && aligned16(gp.c) && p.ldc % 4 == 0 &&
            (gp.batch == 1 || gp.stride_c % 4 == 0);
  const dim3 grid(static_cast<unsigned>(s.tiles_m * p.groups * p.split),
                  static_cast<unsigned>(s.tiles_n), static_cast<unsigned>(gp.batch));
  const sgblasStatus_t st = s.bm == 128
                                ? launchByMode<128>(ta, tb, p, grid, device, stream)
                                : launchByMode<64>(ta, tb, p, grid, device, stream);
  if (st == SGBLAS_STATUS_SUCCESS && used_handle_workspace &&
      !markWorkspaceUse(scratch.ctx, stream))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  return st;
}

}  // namespace sgblas::detail
