// sgblasSgemm for B200: validation -> dispatch -> sm_100a kernels.
//
// Entry-point semantics follow the reference CUDA build
// (src/sgemm_cuda.cu:699-730 of AG0708/sgBLAS): NULL handle -> NOT_INITIALIZED;
// validation errors as returned by validate(); no work -> SUCCESS; work in
// TF32 mode -> NOT_SUPPORTED; otherwise enqueue on the handle's stream and
// return without synchronizing. Unlike the reference, a launch clears only an
// error it caused itself (cudaLaunchKernelEx returns the launch's own status),
// so an error the caller left pending is not swallowed.
#include "context.hpp"
#include "sgemm_tile.cuh"
#include "validation.hpp"
#include "device.hpp"

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdint>

namespace sgblas::detail {

using kern::Beta;
using kern::GemmParams;
using kern::Src;

namespace {

// ---------------------------------------------------------------------------
// C = beta * C (or C = 0 without reading C when beta == 0) for the k == 0 /
// alpha == 0 case. Reference: scaleKernel, src/sgemm_cuda.cu:64-84.
// Rows are the fast grid axis so that a warp touches one contiguous column run.
template <bool kZero>
__global__ void scaleKernel(int m, int n, float beta, float *c, int ldc) {
  for (int col = blockIdx.y; col < n; col += gridDim.y) {
    float *column = c + static_cast<size_t>(col) * ldc;
    for (int row = blockIdx.x * blockDim.x + threadIdx.x; row < m;
         row += gridDim.x * blockDim.x) {
      column[row] = kZero ? 0.0F : beta * column[row];
    }
  }
}

sgblasStatus_t launchStatus(cudaError_t e) {
  if (e == cudaSuccess) return SGBLAS_STATUS_SUCCESS;
  (void)cudaGetLastError();  // clear the error this launch produced
  return SGBLAS_STATUS_EXECUTION_FAILED;
}

sgblasStatus_t launchScale(int m, int n, float beta, float *c, int ldc, cudaStream_t stream) {
  const unsigned row_blocks = static_cast<unsigned>((m + 255) / 256);
  const dim3 grid(row_blocks < 1024u ? row_blocks : 1024u,
                  static_cast<unsigned>(n < 65535 ? n : 65535));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  const cudaError_t e = beta == 0.0F
                            ? cudaLaunchKernelEx(&cfg, scaleKernel<true>, m, n, beta, c, ldc)
                            : cudaLaunchKernelEx(&cfg, scaleKernel<false>, m, n, beta, c, ldc);
  return launchStatus(e);
}

// ---------------------------------------------------------------------------
// TMA descriptors. cuTensorMapEncodeTiled is a host-side driver function; it
// is fetched once through the runtime so that the library needs no -lcuda.
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encodeTiled() {
  static const EncodeTiledFn fn = [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      return static_cast<EncodeTiledFn>(nullptr);
    }
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// Tensor map of a column-major rows x cols FP32 matrix (leading dimension ld)
// read in boxes of box_rows x box_cols; swizzle64 for k-contiguous tiles whose
// rows are exactly 64 bytes.
bool encodeMatrix(CUtensorMap *map, const float *ptr, int rows, int cols, int ld, int box_rows,
                  int box_cols, bool swizzle64) {
  const EncodeTiledFn fn = encodeTiled();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(cols)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * sizeof(float)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_rows), static_cast<cuuint32_t>(box_cols)};
  const cuuint32_t elem_strides[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(ptr), dims, strides, box,
            elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swizzle64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// Persistent schedule: one CTA per SM. Whole tiles are dealt round-robin;
// when the tile count leaves a partial last wave, the last (full wave +
// remainder) tiles are split by k iterations over all CTAs (stream-K), so every
// SM finishes at the same time. Small problems with fewer tiles than SMs are
// split the same way, down to kMinSkIters k slices per CTA.
struct Schedule {
  int grid = 0, dp_tiles = 0, sk_tiles = 0, sk_q = 0, sk_r = 0;
};

constexpr int kMinSkIters = 8;

Schedule makeSchedule(long long tiles, int kiters, int sms) {
  Schedule s;
  const int t = static_cast<int>(tiles);
  if (t >= sms) {
    s.grid = sms;
    const int waves = t / sms, rem = t % sms;
    if (rem == 0 || kiters < 2 * kMinSkIters) {
      s.dp_tiles = t;
    } else {
      s.dp_tiles = (waves - 1) * sms;
      s.sk_tiles = t - s.dp_tiles;
    }
  } else {
    const long long iters = tiles * kiters;
    s.grid = static_cast<int>(
        std::min<long long>(sms, std::max<long long>(tiles, iters / kMinSkIters)));
    if (s.grid == t) s.dp_tiles = t;
    else s.sk_tiles = t;
  }
  if (s.sk_tiles > 0) {
    const long long it = static_cast<long long>(s.sk_tiles) * kiters;
    s.sk_q = static_cast<int>(it / s.grid);
    s.sk_r = static_cast<int>(it % s.grid);
  }
  return s;
}

int smCount(int device) {
  static std::atomic<int> cached[kMaxDevices];
  if (device < 0 || device >= kMaxDevices) return 0;
  int v = cached[device].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
      (void)cudaGetLastError();
      return 0;
    }
    cached[device].store(v, std::memory_order_relaxed);
  }
  return v;
}

constexpr size_t kSlotBytes = size_t{kern::kThreads} * kern::kSlotFloat4 * sizeof(float4);
// Arrival counters: sk_tiles <= 2 * grid <= 2 * SMs, so 1024 counters cover
// any GPU with up to 512 SMs.
constexpr size_t kCounterRegionBytes = 4096;

// Grow-only, stream-ordered workspace of the handle: [counters | slots].
// Returns false (and the caller falls back to whole-tile scheduling) when it
// cannot be provided.
bool ensureWorkspace(sgblasContext *ctx, size_t counter_bytes, size_t slot_bytes, int device,
                     cudaStream_t stream) {
  const size_t need = counter_bytes + slot_bytes;
  if (ctx->workspace != nullptr && ctx->workspace_device == device &&
      ctx->workspace_bytes >= need) {
    if (ctx->workspace_event != nullptr &&
        cudaStreamWaitEvent(stream, static_cast<cudaEvent_t>(ctx->workspace_event), 0) !=
            cudaSuccess) {
      (void)cudaGetLastError();
      return false;
    }
    return true;
  }
  releaseWorkspace(ctx);
  if (cudaSetDevice(device) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  const size_t bytes = std::max(need, size_t{64} << 20);  // room for later, larger calls
  void *ws = nullptr;
  cudaEvent_t ev = nullptr;
  if (cudaMallocAsync(&ws, bytes, stream) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  // Counters must start at zero; every launch leaves them at zero again.
  if (cudaMemsetAsync(ws, 0, bytes, stream) != cudaSuccess ||
      cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
    (void)cudaGetLastError();
    (void)cudaFreeAsync(ws, stream);
    return false;
  }
  ctx->workspace = ws;
  ctx->workspace_bytes = bytes;
  ctx->workspace_device = device;
  ctx->workspace_event = ev;
  return true;
}

template <bool kTA, bool kTB, Beta kBeta, Src kSrc>
sgblasStatus_t launchTiles(GemmParams p, sgblasContext *ctx, int device, cudaStream_t stream) {
  using Plan = kern::Plan<kTA, kTB, kSrc>;
  auto kernel = kern::sgemmKernel<kTA, kTB, kBeta, kSrc>;
  static std::atomic<uint64_t> configured{0};
  if (!configureKernel(reinterpret_cast<const void *>(kernel), device, kern::kSmemBytes,
                       &configured))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  p.tiles_m = (p.m + Plan::kBM - 1) / Plan::kBM;
  p.tiles_n = (p.n + Plan::kBN - 1) / Plan::kBN;
  p.group_m = 8;
  p.kiters = (p.k + kern::kBK - 1) / kern::kBK;
  const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n;
  if (tiles > INT_MAX / 2 || static_cast<long long>(p.kiters) * tiles > INT_MAX)
    return SGBLAS_STATUS_NOT_SUPPORTED;
  const int sms = smCount(device);
  if (sms <= 0) return SGBLAS_STATUS_EXECUTION_FAILED;
  Schedule s = makeSchedule(tiles, p.kiters, sms);
  if (s.sk_tiles > 0) {
    // The counter region has a fixed size so that the layout of the workspace
    // is the same for every call: counters left at zero by one launch must not
    // be overlapped by another launch's partial slots.
    const size_t counter_bytes = kCounterRegionBytes;
    if (static_cast<size_t>(s.sk_tiles) * sizeof(int) <= counter_bytes &&
        ensureWorkspace(ctx, counter_bytes, 2 * static_cast<size_t>(s.grid) * kSlotBytes, device,
                        stream)) {
      p.counters = static_cast<int *>(ctx->workspace);
      p.ws = reinterpret_cast<float4 *>(static_cast<char *>(ctx->workspace) + counter_bytes);
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
  cfg.dynamicSmemBytes = kern::kSmemBytes;
  cfg.stream = stream;
  const sgblasStatus_t st = launchStatus(cudaLaunchKernelEx(&cfg, kernel, p));
  if (st == SGBLAS_STATUS_SUCCESS && s.sk_tiles > 0 &&
      cudaEventRecord(static_cast<cudaEvent_t>(ctx->workspace_event), stream) != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  return st;
}

template <bool kTA, bool kTB, Src kSrc>
sgblasStatus_t launchByBeta(const GemmParams &p, sgblasContext *ctx, int device,
                            cudaStream_t stream) {
  if (p.beta == 0.0F) return launchTiles<kTA, kTB, Beta::kZero, kSrc>(p, ctx, device, stream);
  if (p.beta == 1.0F) return launchTiles<kTA, kTB, Beta::kOne, kSrc>(p, ctx, device, stream);
  return launchTiles<kTA, kTB, Beta::kGeneral, kSrc>(p, ctx, device, stream);
}

// TMA descriptors for the operand tiles the kernel stages: a [k][x] tile is a
// box of (x extent) x BK elements of a x-contiguous matrix, a [x][k] tile a
// BK x (x extent) box of a k-contiguous matrix with the 64B swizzle.
template <bool kTA, bool kTB>
bool encodeOperands(GemmParams &p) {
  using Plan = kern::Plan<kTA, kTB, Src::kTma>;
  const int a_ext = Plan::kPairIsA ? kern::kBP : kern::kBD;
  const int b_ext = Plan::kPairIsA ? kern::kBD : kern::kBP;
  const int a_rows = kTA ? p.k : p.m, a_cols = kTA ? p.m : p.k;
  const int b_rows = kTB ? p.n : p.k, b_cols = kTB ? p.k : p.n;
  const bool a_kx = Plan::kA == kern::Layout::kKX;
  const bool b_kx = Plan::kB == kern::Layout::kKX;
  return encodeMatrix(&p.tma_a, p.a, a_rows, a_cols, p.lda, a_kx ? kern::kBK : a_ext,
                      a_kx ? a_ext : kern::kBK, a_kx) &&
         encodeMatrix(&p.tma_b, p.b, b_rows, b_cols, p.ldb, b_kx ? kern::kBK : b_ext,
                      b_kx ? b_ext : kern::kBK, b_kx);
}

template <bool kTA, bool kTB>
sgblasStatus_t launchBySource(GemmParams &p, sgblasContext *ctx, int device, cudaStream_t stream) {
  // TMA needs 16-byte aligned bases and leading dimensions that are a
  // multiple of 16 bytes; TN has no [k][x] operand for TMA to deliver.
  if constexpr (!(kTA && !kTB)) {
    if (aligned16(p.a) && aligned16(p.b) && p.lda % 4 == 0 && p.ldb % 4 == 0 &&
        encodeOperands<kTA, kTB>(p)) {
      return launchByBeta<kTA, kTB, Src::kTma>(p, ctx, device, stream);
    }
  }
  return launchByBeta<kTA, kTB, Src::kCopy>(p, ctx, device, stream);
}

sgblasStatus_t launchProduct(sgblasContext *ctx, sgblasOperation_t ta, sgblasOperation_t tb,
                             int m, int n, int k, float alpha, const float *a, int lda,
                             const float *b, int ldb, float beta, float *c, int ldc,
                             cudaStream_t stream) {
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  unsigned *err = deviceErrorWord(device);
  if (err == nullptr) return SGBLAS_STATUS_EXECUTION_FAILED;

  GemmParams p = {};
  p.a = a;
  p.b = b;
  p.c = c;
  p.m = m;
  p.n = n;
  p.k = k;
  p.lda = lda;
  p.ldb = ldb;
  p.ldc = ldc;
  p.alpha = alpha;
  p.beta = beta;
  p.err = err;

  const bool tA = ta == SGBLAS_OP_T, tB = tb == SGBLAS_OP_T;
  if (!tA && !tB) return launchBySource<false, false>(p, ctx, device, stream);
  if (!tA && tB) return launchBySource<false, true>(p, ctx, device, stream);
  if (tA && !tB) return launchBySource<true, false>(p, ctx, device, stream);
  return launchBySource<true, true>(p, ctx, device, stream);
}

}  // namespace

void releaseWorkspace(sgblasContext *context) {
  if (context->workspace != nullptr) {
    int current = -1;
    const bool restore = cudaGetDevice(&current) == cudaSuccess;
    if (cudaSetDevice(context->workspace_device) == cudaSuccess) {
      (void)cudaFree(context->workspace);  // synchronizes with the launches using it
      if (context->workspace_event != nullptr)
        (void)cudaEventDestroy(static_cast<cudaEvent_t>(context->workspace_event));
    }
    context->workspace_event = nullptr;
    if (restore) (void)cudaSetDevice(current);
    (void)cudaGetLastError();
    context->workspace = nullptr;
    context->workspace_bytes = 0;
    context->workspace_device = -1;
  }
}

}  // namespace sgblas::detail

extern "C" sgblasStatus_t sgblasSgemm(sgblasHandle_t handle, sgblasOperation_t transa,
                                      sgblasOperation_t transb, int m, int n, int k,
                                      const float *alpha, const float *a, int lda, const float *b,
                                      int ldb, const float *beta, float *c, int ldc) {
  using namespace sgblas::detail;
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  SgemmPlan plan;
  const sgblasStatus_t status =
      validate(transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc, &plan);
  if (status != SGBLAS_STATUS_SUCCESS) return status;
  if (plan.work == Work::kNothing) return SGBLAS_STATUS_SUCCESS;
  if (handle->math_mode != SGBLAS_MATH_FP32) return SGBLAS_STATUS_NOT_SUPPORTED;
  const auto stream = static_cast<cudaStream_t>(handle->stream);
  if (plan.work == Work::kScale) return launchScale(m, n, plan.beta, c, ldc, stream);
  return launchProduct(handle, transa, transb, m, n, k, plan.alpha, a, lda, b, ldb, plan.beta, c,
                       ldc, stream);
}
