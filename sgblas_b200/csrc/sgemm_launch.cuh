// Definition of launchMode<kTA, kTB> (declared in sgemm_launch.hpp); included
// only by the per-mode translation units sgemm_mode_*.cu.
#ifndef SGBLAS_B200_SGEMM_LAUNCH_CUH_
#define SGBLAS_B200_SGEMM_LAUNCH_CUH_

#include "device.hpp"
#include "sgemm_launch.hpp"

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdint>

namespace sgblas::detail {

template <int kTP, bool kTA, bool kTB, bool kPairIsA, kern::Beta kBeta, kern::Src kSrc>
sgblasStatus_t launchTiles(kern::GemmParams p, const Scratch &scratch, int device,
                           cudaStream_t stream) {
  using Plan = kern::Plan<kTA, kTB, kPairIsA, kTP>;
  using G = kern::Geo<kTP>;
  auto kernel = kern::sgemmKernel<kTP, kTA, kTB, kPairIsA, kBeta, kSrc>;
  static std::atomic<uint64_t> configured{0};
  if (!configureKernel(reinterpret_cast<const void *>(kernel), device, G::kSmemBytes,
                       &configured))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  p.tiles_m = (p.m + Plan::kBM - 1) / Plan::kBM;
  p.tiles_n = (p.n + Plan::kBN - 1) / Plan::kBN;
  p.group_m = 8;
  p.kiters = (p.k + kern::kBK - 1) / kern::kBK;
  const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n * p.batch;
  if (tiles > INT_MAX / 2 || static_cast<long long>(p.kiters) * tiles > INT_MAX)
    return SGBLAS_STATUS_NOT_SUPPORTED;
  const int sms = smCount(device);
  if (sms <= 0) return SGBLAS_STATUS_EXECUTION_FAILED;
  Schedule s = makeSchedule(tiles, p.kiters, sms);
  bool used_handle_workspace = false;
  if (s.sk_tiles > 0) {
    const size_t need = kCounterRegionBytes + 2 * static_cast<size_t>(s.grid) * G::kSlotBytes;
    const bool counters_fit = static_cast<size_t>(s.sk_tiles) <= kMaxCounters;
    unsigned char *base = nullptr;
    if (scratch.fixed != nullptr) {
      // Fixed scratch: refuse rather than allocate. The counters are cleared
      // in case an earlier launch did not finish.
      if (!counters_fit || need > scratch.fixed_bytes) return SGBLAS_STATUS_NOT_SUPPORTED;
      if (!clearFixedCounters(scratch.fixed, static_cast<size_t>(s.sk_tiles), stream))
        return SGBLAS_STATUS_EXECUTION_FAILED;
      base = scratch.fixed;
      p.epoch = 1;
    } else if (counters_fit && ensureWorkspace(scratch.ctx, need, device, stream)) {
      p.epoch = nextCounterEpoch(scratch.ctx, stream);
      if (p.epoch == 0) return SGBLAS_STATUS_EXECUTION_FAILED;
      base = static_cast<unsigned char *>(scratch.ctx->workspace);
      used_handle_workspace = true;
    }
    if (base != nullptr) {
      p.counters = reinterpret_cast<Counter *>(base);
      p.ws = reinterpret_cast<float4 *>(base + kCounterRegionBytes);
    } else {  // no workspace: whole tiles only
      s = Schedule{};
      s.grid = static_cast<int>(std::min<long long>(tiles, sms));
      s.dp_tiles = static_cast<int>(tiles);
    }
  }
  p.grid = s.grid;
  p.dp_tiles = s.dp_tiles;
  p.sk_tiles = s.sk_tiles;
  p.sk_q = s.sk_q;
  p.sk_r = s.sk_r;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(s.grid));
  cfg.blockDim = dim3(kern::kBlockThreads);
  cfg.dynamicSmemBytes = G::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1] = {};
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const sgblasStatus_t st = launchStatus(cudaLaunchKernelEx(&cfg, kernel, p));
  if (st == SGBLAS_STATUS_SUCCESS && used_handle_workspace &&
      !markWorkspaceUse(scratch.ctx, stream))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  return st;
}

template <int kTP, bool kTA, bool kTB, bool kPairIsA, kern::Src kSrc>
sgblasStatus_t launchByBeta(const kern::GemmParams &p, const Scratch &scratch, int device,
                            cudaStream_t stream) {
  using kern::Beta;
  if (p.beta == 0.0F)
    return launchTiles<kTP, kTA, kTB, kPairIsA, Beta::kZero, kSrc>(p, scratch, device, stream);
  if (p.beta == 1.0F)
    return launchTiles<kTP, kTA, kTB, kPairIsA, Beta::kOne, kSrc>(p, scratch, device, stream);
  return launchTiles<kTP, kTA, kTB, kPairIsA, Beta::kGeneral, kSrc>(p, scratch, device, stream);
}

// TMA when both bases are 16-byte aligned and both leading dimensions are a
// multiple of 16 bytes (and the driver accepts the descriptors); otherwise
// cp.async, per operand in the widest size (16, 8 or 4 bytes) its base and
// leading dimension allow. Each operand is staged in its natural layout.
template <int kTP, bool kTA, bool kTB, bool kPairIsA>
sgblasStatus_t launchOriented(kern::GemmParams p, const Scratch &scratch, int device,
                              cudaStream_t stream) {
  using Plan = kern::Plan<kTA, kTB, kPairIsA, kTP>;
  using kern::Layout;
  const bool arrays = p.a_ptrs != nullptr;   // pointer arrays: no tensor maps
  auto strideOk = [&](long long stride, int q) { return p.batch == 1 || stride % q == 0; };
  if (!arrays && aligned16(p.a) && aligned16(p.b) && p.lda % 4 == 0 && p.ldb % 4 == 0 &&
      strideOk(p.stride_a, 4) && strideOk(p.stride_b, 4)) {
    const bool a_kx = Plan::kA == Layout::kKX;
    const bool b_kx = Plan::kB == Layout::kKX;
    const int bk = kern::kBK;
    if (encodeMatrix(&p.tma_a, p.a, kTA ? p.k : p.m, kTA ? p.m : p.k, p.lda, p.batch,
                     p.stride_a, a_kx ? bk : Plan::kAExt, a_kx ? Plan::kAExt : bk, a_kx) &&
        encodeMatrix(&p.tma_b, p.b, kTB ? p.n : p.k, kTB ? p.k : p.n, p.ldb, p.batch,
                     p.stride_b, b_kx ? bk : Plan::kBExt, b_kx ? Plan::kBExt : bk, b_kx))
      return launchByBeta<kTP, kTA, kTB, kPairIsA, kern::Src::kTma>(p, scratch, device, stream);
  }
  // Widest cp.async the operand's alignment allows (for every matrix of a
  // strided batch; 4 bytes for pointer arrays, whose entries are unknown here).
  auto vec = [&](const float *ptr, int ld, long long stride) {
    if (arrays) return 1;
    const uintptr_t addr = reinterpret_cast<uintptr_t>(ptr);
    if (addr % 16 == 0 && ld % 4 == 0 && strideOk(stride, 4)) return 4;
    if (addr % 8 == 0 && ld % 2 == 0 && strideOk(stride, 2)) return 2;
    return 1;
  };
  p.a_vec = vec(p.a, p.lda, p.stride_a);
  p.b_vec = vec(p.b, p.ldb, p.stride_b);
  return launchByBeta<kTP, kTA, kTB, kPairIsA, kern::Src::kCopy>(p, scratch, device, stream);
}

// Tile size and orientation. The pair operand spans 256 (kTP = 16) or 128
// (kTP = 8) rows of its side of C, the broadcast operand 128. Large tiles are
// used when they give at least one tile per SM; otherwise 128 x 128 tiles
// spread a small problem over more SMs with less stream-K splitting. Among
// orientations: less padded tile area, then fewer transposed elements per k
// step.
template <int kTP, bool kTA, bool kTB>
sgblasStatus_t launchSized(kern::GemmParams p, const Scratch &scratch, int device,
                           cudaStream_t stream) {
  using PA = kern::Plan<kTA, kTB, true, kTP>;
  using PB = kern::Plan<kTA, kTB, false, kTP>;
  auto padded = [](long long x, long long t) { return (x + t - 1) / t * t; };
  const long long area_a = padded(p.m, PA::kBM) * padded(p.n, PA::kBN);
  const long long area_b = padded(p.m, PB::kBM) * padded(p.n, PB::kBN);
  constexpr int trans_a = (PA::kTransP ? PA::kBP : 0) + (PA::kTransD ? kern::kBD : 0);
  constexpr int trans_b = (PB::kTransP ? PB::kBP : 0) + (PB::kTransD ? kern::kBD : 0);
  const bool pair_is_a = area_a < area_b || (area_a == area_b && trans_a <= trans_b);
  if (pair_is_a) return launchOriented<kTP, kTA, kTB, true>(p, scratch, device, stream);
  return launchOriented<kTP, kTA, kTB, false>(p, scratch, device, stream);
}

template <bool kTA, bool kTB>
sgblasStatus_t launchMode(kern::GemmParams p, const Scratch &scratch, int device,
                          cudaStream_t stream) {
  auto tiles = [&](long long bm, long long bn) {
    return ((p.m + bm - 1) / bm) * ((p.n + bn - 1) / bn) * p.batch;
  };
  const long long large = std::min(tiles(256, 128), tiles(128, 256));
  if (large >= smCount(device)) return launchSized<16, kTA, kTB>(p, scratch, device, stream);
  return launchSized<8, kTA, kTB>(p, scratch, device, stream);
}

}  // namespace sgblas::detail

#endif  // SGBLAS_B200_SGEMM_LAUNCH_CUH_
