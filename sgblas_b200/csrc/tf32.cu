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

template <int kBN, bool kAMN, bool kBMN, kern::Beta kBeta>
sgblasStatus_t launchTyped(t::Tf32Params &q, int sms, int device, cudaStream_t stream) {
  using G = t::Cfg<kBN>;
  auto kernel = t::tf32Kernel<kBN, kAMN, kBMN, kBeta>;
  static std::atomic<uint64_t> configured{0};
  if (!configureKernel(reinterpret_cast<const void *>(kernel), device, G::kSmemBytes,
                       &configured))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  const long long tiles = static_cast<long long>(q.tiles_m) * q.tiles_n;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(std::min<long long>(tiles, sms)));
  cfg.blockDim = dim3(t::kThreads);
  cfg.dynamicSmemBytes = G::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1] = {};
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return launchStatus(cudaLaunchKernelEx(&cfg, kernel, q));
}

template <int kBN, bool kAMN, bool kBMN>
sgblasStatus_t launchByBeta(t::Tf32Params &q, int sms, int device, cudaStream_t stream) {
  using kern::Beta;
  if (q.beta == 0.0F) return launchTyped<kBN, kAMN, kBMN, Beta::kZero>(q, sms, device, stream);
  if (q.beta == 1.0F) return launchTyped<kBN, kAMN, kBMN, Beta::kOne>(q, sms, device, stream);
  return launchTyped<kBN, kAMN, kBMN, Beta::kGeneral>(q, sms, device, stream);
}

template <int kBN>
sgblasStatus_t launchSized(const kern::GemmParams &p, bool a_mn, bool b_mn, t::Tf32Params &q,
                           int sms, int device, cudaStream_t stream) {
  q.tiles_n = (p.n + kBN - 1) / kBN;
  // K-major tiles: 128-byte swizzle; MN-major tiles: 128-byte swizzle of
  // 32-byte atoms (what the tensor core requires for MN-major TF32).
  const auto sw_k = CU_TENSOR_MAP_SWIZZLE_128B;
  const auto sw_mn = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  const unsigned long long lda_b = static_cast<unsigned long long>(p.lda) * 4;
  const unsigned long long ldb_b = static_cast<unsigned long long>(p.ldb) * 4;
  const bool ok_a = a_mn ? encodeTiled2d(&q.tma_a, p.a, p.m, p.k, lda_b, 32, 32, sw_mn)
                         : encodeTiled2d(&q.tma_a, p.a, p.k, p.m, lda_b, 32, t::kBM, sw_k);
  const bool ok_b = b_mn ? encodeTiled2d(&q.tma_b, p.b, p.n, p.k, ldb_b, 32, 32, sw_mn)
                         : encodeTiled2d(&q.tma_b, p.b, p.k, p.n, ldb_b, 32, kBN, sw_k);
  if (!ok_a || !ok_b) return SGBLAS_STATUS_EXECUTION_FAILED;
  if (a_mn && b_mn) return launchByBeta<kBN, true, true>(q, sms, device, stream);
  if (a_mn) return launchByBeta<kBN, true, false>(q, sms, device, stream);
  if (b_mn) return launchByBeta<kBN, false, true>(q, sms, device, stream);
  return launchByBeta<kBN, false, false>(q, sms, device, stream);
}

}  // namespace

sgblasStatus_t launchTf32(bool ta, bool tb, const kern::GemmParams &p, int device,
                          cudaStream_t stream) {
  t::Tf32Params q = {};
  q.c = p.c;
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
  // Tile width: the one with the shorter estimated run, waves x tile time.
  // A 128-wide tile takes 0.77 of a 256-wide tile's time (measured: its
  // operand traffic per FLOP is higher), so it wins only where the 256-wide
  // tiles leave most of a wave idle.
  auto waves = [&](long long bn) {
    const long long tiles = static_cast<long long>(q.tiles_m) * ((p.n + bn - 1) / bn);
    return (tiles + sms - 1) / sms;
  };
  if (static_cast<long long>(q.tiles_m) * ((p.n + 127) / 128) > INT_MAX)
    return SGBLAS_STATUS_NOT_SUPPORTED;
  // A: op N keeps m contiguous (MN-major), op T keeps k contiguous (K-major);
  // B: op N keeps k contiguous (K-major), op T keeps n contiguous (MN-major).
  const bool a_mn = !ta, b_mn = tb;
  if (waves(128) * 77 < waves(256) * 100)
    return launchSized<128>(p, a_mn, b_mn, q, sms, device, stream);
  return launchSized<256>(p, a_mn, b_mn, q, sms, device, stream);
}

}  // namespace sgblas::detail
