// Host launch of the TF32 lane (tf32_tile.cuh): tensor maps, persistent grid,
// one kernel per (A major, B major, beta mode).
#include "device.hpp"
#include "sgemm_launch.hpp"
#include "tf32_tile.cuh"

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>

namespace sgblas::detail {

namespace {

namespace t = kern::tf32;

// Shortest tile depth, in 32-deep k slices, whose partial last wave is split.
constexpr int kMinTailSplitIters = 96;
Schedule makeScheduleTf32(long long tiles, int kiters, int sms, bool batched);

// Persistent schedule of `units` workers (CTAs, or CTA pairs) with the FP32
// kernel's item structure and workspace layout ([counters | slots]), filled
// into q; the workspace holds `slots` piece slots and `counters_per_tile`
// counters per split tile. A tensor-core tile computes about ten times
// faster than a CUDA-core one, so the piece fix-up costs relatively more:
// only a partial last wave that leaves more than 30 % of the workers idle is
// split (over all workers, each taking less than one tile), and a small
// problem only into pieces of 1024 k or more. Without scratch, whole tiles
// only. grid == 0 on failure.
Schedule scheduleTf32(t::Tf32Params &q, long long tiles, int slots, int units,
                      const Scratch &scratch, int device, cudaStream_t stream,
                      bool *used_handle_workspace, int counters_per_tile = 1) {
  Schedule s = makeScheduleTf32(tiles, q.kiters, units, q.batch > 1);
  *used_handle_workspace = false;
  if (s.sk_tiles > 0) {
    const size_t need = kCounterRegionBytes + static_cast<size_t>(slots) * kSlotBytes;
    const size_t counters = static_cast<size_t>(s.sk_tiles) * counters_per_tile;
    const bool counters_fit = counters <= kMaxCounters;
    unsigned char *base = nullptr;
    if (scratch.fixed != nullptr) {
      if (counters_fit && need <= scratch.fixed_bytes) {
        if (!clearFixedCounters(scratch.fixed, counters, stream)) return Schedule{};
        base = scratch.fixed;
        q.epoch = 1;
      }
    } else if (counters_fit && ensureWorkspace(scratch.ctx, need, device, stream)) {
      q.epoch = nextCounterEpoch(scratch.ctx, stream);
      if (q.epoch == 0) return Schedule{};
      base = static_cast<unsigned char *>(scratch.ctx->workspace);
      *used_handle_workspace = true;
    }
    if (base != nullptr) {
      q.counters = reinterpret_cast<Counter *>(base);
      q.ws = reinterpret_cast<float *>(base + kCounterRegionBytes);
    } else {
      s = Schedule{};
      s.grid = static_cast<int>(std::min<long long>(tiles, units));
      s.dp_tiles = static_cast<int>(tiles);
    }
  }
  q.grid = s.grid;
  q.dp_tiles = s.dp_tiles;
  q.sk_tiles = s.sk_tiles;
  q.sk_q = s.sk_q;
  q.sk_r = s.sk_r;
  return s;
}

constexpr int kMinSmallPieceIters = 32;   // 1024 of k

Schedule makeScheduleTf32(long long tiles, int kiters, int sms, bool batched) {
  Schedule s;
  const int t = static_cast<int>(tiles);
  const bool splittable = kiters >= 2 * kMinSkIters;
  // A tail split pays only for deep tiles (measured with pair tiles: k = 4096
  // +3 %, k = 2048 -3 %), and not at all in the batched instantiation.
  const bool tail_splittable = kiters >= kMinTailSplitIters && !batched;
  if (t >= sms) {
    const int rem = t % sms;
    s.grid = sms;
    if (rem == 0 || 10 * rem >= 7 * sms || !tail_splittable ||
        static_cast<long long>(rem) * kiters < static_cast<long long>(sms) * kMinSkIters) {
      s.dp_tiles = t;
    } else {
      s.dp_tiles = t - rem;
      s.sk_tiles = rem;
    }
  } else {
    // Fewer tiles than workers: split each tile into pieces of at least
    // kMinSmallPieceIters k-iterations, as many as the idle workers allow.
    // Shallower pieces cost more in the fix-up than they gain (measured on
    // B200: 1024^3 23.1 us split over all 148 CTAs, 18.7 us unsplit;
    // 1024 x 1024 x 4096 37.1 us split over all, 34.2 us in two pieces).
    const long long pieces = std::min<long long>(kiters / kMinSmallPieceIters, sms / t);
    if (pieces <= 1 || !splittable) {
      s.grid = t;
      s.dp_tiles = t;
    } else {
      s.grid = static_cast<int>(t * pieces);
      s.sk_tiles = t;
    }
  }
  if (s.sk_tiles > 0) {
    const long long it = static_cast<long long>(s.sk_tiles) * kiters;
    s.sk_q = static_cast<int>(it / s.grid);
    s.sk_r = static_cast<int>(it % s.grid);
  }
  return s;
}

template <int kBN, bool kAMN, bool kBMN, kern::Beta kBeta, bool kBatch>
sgblasStatus_t launchTyped(t::Tf32Params &q, const Scratch &scratch, int sms, int device,
                           cudaStream_t stream) {
  using G = t::Cfg<kBN>;
  static_assert(static_cast<size_t>(t::kBM) * kBN * 4 <= kSlotBytes, "piece slot size");
  auto kernel = t::tf32Kernel<kBN, kAMN, kBMN, kBeta, kBatch>;
  static std::atomic<uint64_t> configured{0};
  if (!configureKernel(reinterpret_cast<const void *>(kernel), device, G::kSmemBytes,
                       &configured))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  const long long tiles = static_cast<long long>(q.tiles_m) * q.tiles_n * q.batch;
  bool used_handle_workspace = false;
  const Schedule s = scheduleTf32(q, tiles, 2 * sms, sms, scratch, device, stream,
                                  &used_handle_workspace);
  if (s.grid == 0) return SGBLAS_STATUS_EXECUTION_FAILED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(s.grid));
  cfg.blockDim = dim3(t::kThreads);
  cfg.dynamicSmemBytes = G::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1] = {};
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const sgblasStatus_t st = launchStatus(cudaLaunchKernelEx(&cfg, kernel, q));
  if (st == SGBLAS_STATUS_SUCCESS && used_handle_workspace &&
      !markWorkspaceUse(scratch.ctx, stream))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  return st;
}

template <int kBN, bool kAMN, bool kBMN, kern::Beta kBeta>
sgblasStatus_t launchByBatch(t::Tf32Params &q, const Scratch &scratch, int sms, int device,
                             cudaStream_t stream) {
  if (q.batch > 1) return launchTyped<kBN, kAMN, kBMN, kBeta, true>(q, scratch, sms, device, stream);
  return launchTyped<kBN, kAMN, kBMN, kBeta, false>(q, scratch, sms, device, stream);
}

template <int kBN, bool kAMN, bool kBMN>
sgblasStatus_t launchByBeta(t::Tf32Params &q, const Scratch &scratch, int sms, int device,
                            cudaStream_t stream) {
  using kern::Beta;
  if (q.beta == 0.0F)
    return launchByBatch<kBN, kAMN, kBMN, Beta::kZero>(q, scratch, sms, device, stream);
  if (q.beta == 1.0F)
    return launchByBatch<kBN, kAMN, kBMN, Beta::kOne>(q, scratch, sms, device, stream);
  return launchByBatch<kBN, kAMN, kBMN, Beta::kGeneral>(q, scratch, sms, device, stream);
}

// The pair-CTA kernel: clusters of two, whole 256 x 256 tiles over the pairs.
template <bool kAMN, bool kBMN, kern::Beta kBeta, bool kBatch>
sgblasStatus_t launchPairTyped(t::Tf32Params &q, const Scratch &scratch, int sms, int device,
                               cudaStream_t stream) {
  static_assert(static_cast<size_t>(t::kBM) * t::Pair::kBN * 4 <= kSlotBytes, "piece slot size");
  auto kernel = t::tf32PairKernel<kAMN, kBMN, kBeta, kBatch>;
  static std::atomic<uint64_t> configured{0};
  if (!configureKernel(reinterpret_cast<const void *>(kernel), device, t::Pair::kSmemBytes,
                       &configured))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  const long long tiles = static_cast<long long>(q.tiles_m) * q.tiles_n * q.batch;
  // Workers are CTA pairs; each CTA of a pair owns two slots and each split
  // tile has a counter per half.
  bool used_handle_workspace = false;
  const Schedule s = scheduleTf32(q, tiles, 2 * 2 * (sms / 2), sms / 2, scratch, device, stream,
                                  &used_handle_workspace, 2);
  if (s.grid == 0) return SGBLAS_STATUS_EXECUTION_FAILED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * s.grid));
  cfg.blockDim = dim3(t::kThreads);
  cfg.dynamicSmemBytes = t::Pair::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2] = {};
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const sgblasStatus_t st = launchStatus(cudaLaunchKernelEx(&cfg, kernel, q));
  if (st == SGBLAS_STATUS_SUCCESS && used_handle_workspace &&
      !markWorkspaceUse(scratch.ctx, stream))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  return st;
}

template <bool kAMN, bool kBMN>
sgblasStatus_t launchPair(const kern::GemmParams &p, t::Tf32Params &q, const Scratch &scratch,
                          int sms, int device, cudaStream_t stream) {
  q.tiles_m = (p.m + 2 * t::kBM - 1) / (2 * t::kBM);
  q.tiles_n = (p.n + t::Pair::kBN - 1) / t::Pair::kBN;
  // Per CTA: A boxes of 128 rows (K-major) or 32 x 32 chunks (MN-major); B
  // boxes of 128 columns (K-major) or 32 x 32 chunks (MN-major).
  const auto sw_k = CU_TENSOR_MAP_SWIZZLE_128B;
  const auto sw_mn = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  const unsigned long long lda_b = static_cast<unsigned long long>(p.lda) * 4;
  const unsigned long long ldb_b = static_cast<unsigned long long>(p.ldb) * 4;
  const bool ok_a = kAMN ? encodeTiled3d(&q.tma_a, p.a, p.m, p.k, lda_b, p.batch, p.stride_a, 32, 32, sw_mn)
                         : encodeTiled3d(&q.tma_a, p.a, p.k, p.m, lda_b, p.batch, p.stride_a, 32, t::kBM, sw_k);
  const bool ok_b = kBMN ? encodeTiled3d(&q.tma_b, p.b, p.n, p.k, ldb_b, p.batch, p.stride_b, 32, 32, sw_mn)
                         : encodeTiled3d(&q.tma_b, p.b, p.k, p.n, ldb_b, p.batch,
                                         p.stride_b, 32, t::Pair::kBNHalf, sw_k);
  if (!ok_a || !ok_b) return SGBLAS_STATUS_EXECUTION_FAILED;
  using kern::Beta;
  const bool batched = q.batch > 1;
  if (q.beta == 0.0F)
    return batched ? launchPairTyped<kAMN, kBMN, Beta::kZero, true>(q, scratch, sms, device, stream)
                   : launchPairTyped<kAMN, kBMN, Beta::kZero, false>(q, scratch, sms, device,
                                                                      stream);
  if (q.beta == 1.0F)
    return batched ? launchPairTyped<kAMN, kBMN, Beta::kOne, true>(q, scratch, sms, device, stream)
                   : launchPairTyped<kAMN, kBMN, Beta::kOne, false>(q, scratch, sms, device,
                                                                     stream);
  return batched
             ? launchPairTyped<kAMN, kBMN, Beta::kGeneral, true>(q, scratch, sms, device, stream)
             : launchPairTyped<kAMN, kBMN, Beta::kGeneral, false>(q, scratch, sms, device, stream);
}

template <int kBN>
sgblasStatus_t launchSized(const kern::GemmParams &p, bool a_mn, bool b_mn, t::Tf32Params &q,
                           const Scratch &scratch, int sms, int device, cudaStream_t stream) {
  q.tiles_n = (p.n + kBN - 1) / kBN;
  // K-major tiles: 128-byte swizzle; MN-major tiles: 128-byte swizzle of
  // 32-byte atoms (what the tensor core requires for MN-major TF32).
  const auto sw_k = CU_TENSOR_MAP_SWIZZLE_128B;
  const auto sw_mn = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  const unsigned long long lda_b = static_cast<unsigned long long>(p.lda) * 4;
  const unsigned long long ldb_b = static_cast<unsigned long long>(p.ldb) * 4;
  const bool ok_a = a_mn ? encodeTiled3d(&q.tma_a, p.a, p.m, p.k, lda_b, p.batch, p.stride_a, 32, 32, sw_mn)
                         : encodeTiled3d(&q.tma_a, p.a, p.k, p.m, lda_b, p.batch, p.stride_a, 32, t::kBM, sw_k);
  const bool ok_b = b_mn ? encodeTiled3d(&q.tma_b, p.b, p.n, p.k, ldb_b, p.batch, p.stride_b, 32, 32, sw_mn)
                         : encodeTiled3d(&q.tma_b, p.b, p.k, p.n, ldb_b, p.batch, p.stride_b, 32, kBN, sw_k);
  if (!ok_a || !ok_b) return SGBLAS_STATUS_EXECUTION_FAILED;
  if (a_mn && b_mn) return launchByBeta<kBN, true, true>(q, scratch, sms, device, stream);
  if (a_mn) return launchByBeta<kBN, true, false>(q, scratch, sms, device, stream);
  if (b_mn) return launchByBeta<kBN, false, true>(q, scratch, sms, device, stream);
  return launchByBeta<kBN, false, false>(q, scratch, sms, device, stream);
}

}  // namespace

sgblasStatus_t launchTf32(bool ta, bool tb, const kern::GemmParams &p, const Scratch &scratch,
                          int device, cudaStream_t stream) {
  t::Tf32Params q = {};
  q.c = p.c;
  q.stride_c = p.stride_c;
  q.batch = p.batch;
  q.m = p.m;
  q.n = p.n;
  q.k = p.k;
  q.ldc = p.ldc;
  q.alpha = p.alpha;
  q.beta = p.beta;
  q.err = p.err;
  q.tiles_m = (p.m + t::kBM - 1) / t::kBM;
  q.kiters = (p.k + t::kBK - 1) / t::kBK;
  q.group_m = 8;
  const int sms = smCount(device);
  if (sms <= 0) return SGBLAS_STATUS_EXECUTION_FAILED;
  // Tile width: 256, whose partial last wave stream-K balances, once there
  // are at least as many 256-wide tiles as SMs. Below that, the one with the
  // shorter estimated run, waves x tile time: a 128-wide tile takes 0.77 of a
  // 256-wide tile's time (measured: its operand traffic per FLOP is higher).
  auto waves = [&](long long bn) {
    const long long tiles = static_cast<long long>(q.tiles_m) * ((p.n + bn - 1) / bn) * p.batch;
    return (tiles + sms - 1) / sms;
  };
  if (static_cast<long long>(q.tiles_m) * ((p.n + 127) / 128) * p.batch > INT_MAX)
    return SGBLAS_STATUS_NOT_SUPPORTED;
  // A: op N keeps m contiguous (MN-major), op T keeps k contiguous (K-major);
  // B: op N keeps k contiguous (K-major), op T keeps n contiguous (MN-major).
  const bool a_mn = !ta, b_mn = tb;
  // Pair-CTA 256 x 256 tiles (half the B traffic per FLOP) once there is at
  // least one tile per pair; the stream-K rule balances a partial last wave.
  const int pairs = sms / 2;
  const long long pair_tiles =
      static_cast<long long>((p.m + 255) / 256) * ((p.n + 255) / 256) * p.batch;
  if (pairs > 0 && pair_tiles >= pairs && pair_tiles <= INT_MAX) {
    if (a_mn && b_mn) return launchPair<true, true>(p, q, scratch, sms, device, stream);
    if (a_mn) return launchPair<true, false>(p, q, scratch, sms, device, stream);
    if (b_mn) return launchPair<false, true>(p, q, scratch, sms, device, stream);
    return launchPair<false, false>(p, q, scratch, sms, device, stream);
  }
  const long long wide_tiles = static_cast<long long>(q.tiles_m) * ((p.n + 255) / 256) * p.batch;
  // 64-wide tiles when 128-wide ones would leave over half the SMs idle and
  // the 128-wide schedule (with its k pieces) would run on fewer CTAs: each
  // CTA then streams a quarter less operand data per k slice, and more SMs
  // take part (measured on B200: 1024^3 19.1 -> 18.5 us, 256^3 12.2 -> 10.6
  // us; 1024 x 1024 x 2048, where 128-wide tiles in two pieces fill as many
  // SMs, 24.8 -> 28.3 us, so it keeps the 128-wide tiles).
  const long long tiles_128 = static_cast<long long>(q.tiles_m) * ((p.n + 127) / 128) * p.batch;
  const long long tiles_64 = static_cast<long long>(q.tiles_m) * ((p.n + 63) / 64) * p.batch;
  if (wide_tiles < sms && 2 * tiles_128 <= sms && p.n > 64 &&
      makeScheduleTf32(tiles_64, q.kiters, sms, p.batch > 1).grid >
          makeScheduleTf32(tiles_128, q.kiters, sms, p.batch > 1).grid)
    return launchSized<64>(p, a_mn, b_mn, q, scratch, sms, device, stream);
  if (wide_tiles < sms && waves(128) * 77 < waves(256) * 100)
    return launchSized<128>(p, a_mn, b_mn, q, scratch, sms, device, stream);
  return launchSized<256>(p, a_mn, b_mn, q, scratch, sms, device, stream);
}

}  // namespace sgblas::detail
