// sgblasSgemm for B200: validation -> dispatch -> sm_100a kernels.
//
// Entry-point semantics follow the reference CUDA build
// (src/sgemm_cuda.cu:699-730 of AG0708/sgBLAS): NULL handle -> NOT_INITIALIZED;
// validation errors as returned by validate(); no work -> SUCCESS; otherwise
// enqueue on the handle's stream and return without synchronizing (the
// reference returns NOT_SUPPORTED for TF32 mode; here it selects the TF32
// tensor-core lane). Unlike the reference, a launch clears only an
// error it caused itself (cudaLaunchKernelEx returns the launch's own status),
// so an error the caller left pending is not swallowed.
#include "context.hpp"
#include "device.hpp"
#include "sgemm_launch.hpp"
#include "validation.hpp"

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdint>

namespace sgblas::detail {

using kern::GemmParams;

namespace {

// ---------------------------------------------------------------------------
// C = beta * C (or C = 0 without reading C when beta == 0) for the k == 0 /
// alpha == 0 case. Reference: scaleKernel, src/sgemm_cuda.cu:64-84.
// Rows are the fast grid axis so that a warp touches one contiguous column run.
// Batches run along grid z: matrix i is c + i*stride_c, or c_ptrs[i].
template <bool kZero>
__global__ void scaleKernel(int m, int n, float beta, float *c, int ldc, int batch,
                            long long stride_c, float *const *c_ptrs) {
  for (int bi = blockIdx.z; bi < batch; bi += gridDim.z) {
    float *matrix = c_ptrs != nullptr ? c_ptrs[bi] : c + bi * stride_c;
    for (int col = blockIdx.y; col < n; col += gridDim.y) {
      float *column = matrix + static_cast<size_t>(col) * ldc;
      for (int row = blockIdx.x * blockDim.x + threadIdx.x; row < m;
           row += gridDim.x * blockDim.x) {
        column[row] = kZero ? 0.0F : beta * column[row];
      }
    }
  }
}

}  // namespace

sgblasStatus_t launchStatus(cudaError_t e) {
  if (e == cudaSuccess) return SGBLAS_STATUS_SUCCESS;
  (void)cudaGetLastError();  // clear the error this launch produced
  return SGBLAS_STATUS_EXECUTION_FAILED;
}

namespace {

sgblasStatus_t launchScale(int m, int n, float beta, float *c, int ldc, const Batch &batch,
                           cudaStream_t stream) {
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  const int arch = isSm100(device);
  if (arch < 0) return SGBLAS_STATUS_EXECUTION_FAILED;
  if (arch == 0) return SGBLAS_STATUS_ARCH_MISMATCH;
  const unsigned row_blocks = static_cast<unsigned>((m + 255) / 256);
  const dim3 grid(row_blocks < 1024u ? row_blocks : 1024u,
                  static_cast<unsigned>(n < 65535 ? n : 65535),
                  static_cast<unsigned>(batch.count < 65535 ? batch.count : 65535));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  const cudaError_t e =
      beta == 0.0F ? cudaLaunchKernelEx(&cfg, scaleKernel<true>, m, n, beta, c, ldc, batch.count,
                                        batch.stride_c, batch.c_ptrs)
                   : cudaLaunchKernelEx(&cfg, scaleKernel<false>, m, n, beta, c, ldc, batch.count,
                                        batch.stride_c, batch.c_ptrs);
  return launchStatus(e);
}

}  // namespace

// ---------------------------------------------------------------------------
// TMA descriptors. cuTensorMapEncodeTiled is a host-side driver function; it
// is fetched once through the runtime so that the library needs no -lcuda.
namespace {

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

}  // namespace

bool encodeMatrix(CUtensorMap *map, const float *ptr, int rows, int cols, int ld, int batch,
                  long long stride, int box_rows, int box_cols, bool swizzle64) {
  const EncodeTiledFn fn = encodeTiled();
  if (fn == nullptr) return false;
  // A single matrix is a batch of one; its (unused) batch stride is the
  // matrix size rounded up to 16 bytes.
  const long long stride_bytes = batch == 1
                                     ? (static_cast<long long>(ld) * cols * 4 + 15) / 16 * 16
                                     : stride * 4;
  if (stride_bytes <= 0 || stride_bytes % 16 != 0 || stride_bytes >= (1LL << 40)) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(cols),
                              static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * sizeof(float),
                                 static_cast<cuuint64_t>(stride_bytes)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(box_rows), static_cast<cuuint32_t>(box_cols),
                             1};
  const cuuint32_t elem_strides[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(ptr), dims, strides, box,
            elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swizzle64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encodeTiled3d(CUtensorMap *map, const float *ptr, unsigned long long dim0,
                   unsigned long long dim1, unsigned long long stride1_bytes, int batch,
                   long long stride_elems, unsigned box0, unsigned box1,
                   CUtensorMapSwizzle swizzle) {
  const EncodeTiledFn fn = encodeTiled();
  if (fn == nullptr) return false;
  // A single matrix is a batch of one with an unused, valid batch stride.
  const long long stride2 = batch == 1
                                ? static_cast<long long>((dim1 * stride1_bytes + 15) / 16 * 16)
                                : stride_elems * 4;
  if (stride2 <= 0 || stride2 % 16 != 0 || stride2 >= (1LL << 40)) return false;
  const cuuint64_t dims[3] = {dim0, dim1, static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[2] = {stride1_bytes, static_cast<cuuint64_t>(stride2)};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t elem_strides[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(ptr), dims, strides, box,
            elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
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
    // Fewer tiles than SMs. Stream-K over (nearly) every SM gives each CTA
    // the fewest k iterations, but most CTAs then hold parts of two tiles,
    // and each part costs a fix-up and an epilogue (about kItemCostIters
    // iterations' worth, measured on B200). Splitting every tile into the
    // same whole number of pieces gives each CTA one part: used when its
    // longer k range still costs less (640^3: 29.4 -> 25.6 us, 768^3: 33.6
    // -> 30.0 us; 1024^3 and wider shapes keep stream-K).
    const long long iters = tiles * kiters;
    const long long sk_grid =
        std::min<long long>(sms, std::max<long long>(tiles, iters / kMinSkIters));
    const long long pieces =
        std::max<long long>(1, std::min<long long>(sms / tiles, kiters / kMinSkIters));
    const long long whole_iters = (kiters + pieces - 1) / pieces;
    const long long sk_iters = (iters + sk_grid - 1) / sk_grid;
    s.grid = static_cast<int>(whole_iters < sk_iters + kItemCostIters ? tiles * pieces : sk_grid);
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

namespace {

// True while `stream` is being captured into a CUDA graph (or when that
// cannot be told, to be safe). During a capture the workspace is neither
// allocated nor ordered by its event: the graph's own edges order it, and an
// allocation made inside a capture would belong to the graph.
bool capturing(cudaStream_t stream) {
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &status) != cudaSuccess) {
    (void)cudaGetLastError();
    return true;
  }
  return status != cudaStreamCaptureStatusNone;
}

}  // namespace

namespace {

// The handle moved to another device: its workspace is freed on the device
// it lives on, stream-ordered after its last user there (the legacy stream
// of that device waits for the workspace event), so that the call does not
// block the host. False if that cannot be enqueued.
bool retireOnOwnDevice(sgblasContext *ctx) {
  int current = -1;
  if (cudaGetDevice(&current) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  const auto ev = static_cast<cudaEvent_t>(ctx->workspace_event);
  const bool ok = cudaSetDevice(ctx->workspace_device) == cudaSuccess &&
                  (ev == nullptr || cudaStreamWaitEvent(cudaStreamLegacy, ev, 0) == cudaSuccess) &&
                  cudaFreeAsync(ctx->workspace, cudaStreamLegacy) == cudaSuccess;
  if (ok) {
    if (ev != nullptr) (void)cudaEventDestroy(ev);   // released once it completes
    ctx->workspace = nullptr;
    ctx->workspace_bytes = 0;
    ctx->workspace_device = -1;
    ctx->workspace_event = nullptr;
  }
  (void)cudaGetLastError();
  (void)cudaSetDevice(current);
  return ok;
}

}  // namespace

bool ensureWorkspace(sgblasContext *ctx, size_t need, int device, cudaStream_t stream) {
  const bool in_capture = capturing(stream);
  if (ctx->workspace != nullptr && ctx->workspace_device == device &&
      ctx->workspace_bytes >= need) {
    if (!in_capture && ctx->workspace_event != nullptr &&
        cudaStreamWaitEvent(stream, static_cast<cudaEvent_t>(ctx->workspace_event), 0) !=
            cudaSuccess) {
      (void)cudaGetLastError();
      return false;
    }
    return true;
  }
  if (in_capture) return false;   // the caller falls back to a path without it
  if (ctx->workspace != nullptr && ctx->workspace_device == device) {
    // Growing: free the old buffer stream-ordered after its last user, so the
    // call does not block the host.
    const auto ev = static_cast<cudaEvent_t>(ctx->workspace_event);
    const bool ordered = ev == nullptr || cudaStreamWaitEvent(stream, ev, 0) == cudaSuccess;
    if (!ordered || cudaFreeAsync(ctx->workspace, stream) != cudaSuccess) {
      (void)cudaGetLastError();
      releaseWorkspace(ctx);
    } else {
      if (ev != nullptr) (void)cudaEventDestroy(ev);  // released once it completes
      ctx->workspace = nullptr;
      ctx->workspace_bytes = 0;
      ctx->workspace_device = -1;
      ctx->workspace_event = nullptr;
    }
  } else if (ctx->workspace != nullptr && !retireOnOwnDevice(ctx)) {
    releaseWorkspace(ctx);
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  // Room for later, larger calls: at least 64 MiB, and a quarter more than
  // asked when growing past that.
  const size_t bytes = std::max(need + need / 4, size_t{64} << 20);
  void *ws = nullptr;
  cudaEvent_t ev = nullptr;
  if (cudaMallocAsync(&ws, bytes, stream) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  // Counters start at zero: epoch 0, which no launch uses.
  if (cudaMemsetAsync(ws, 0, std::min(bytes, kCounterRegionBytes), stream) != cudaSuccess ||
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

unsigned nextCounterEpoch(sgblasContext *ctx, cudaStream_t stream) {
  unsigned epoch = ctx->workspace_epoch + 1;
  if (epoch == 0) {
    if (cudaMemsetAsync(ctx->workspace, 0, kCounterRegionBytes, stream) != cudaSuccess) {
      (void)cudaGetLastError();
      return 0;
    }
    epoch = 1;
  }
  ctx->workspace_epoch = epoch;
  return epoch;
}

bool clearFixedCounters(unsigned char *fixed, size_t count, cudaStream_t stream) {
  if (cudaMemsetAsync(fixed, 0, count * sizeof(Counter), stream) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return true;
}

bool markWorkspaceUse(sgblasContext *ctx, cudaStream_t stream) {
  if (capturing(stream)) return true;
  if (cudaEventRecord(static_cast<cudaEvent_t>(ctx->workspace_event), stream) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return true;
}

// The kernels are built for sm_100a only: 1 if `device` is compute
// capability 10.0, 0 if not, -1 if it cannot be told. Cached per device.
int isSm100(int device) {
  static std::atomic<int> cached[kMaxDevices];   // 0 unknown, 1 yes, 2 no
  if (device < 0 || device >= kMaxDevices) return -1;
  int v = cached[device].load(std::memory_order_relaxed);
  if (v == 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) {
      (void)cudaGetLastError();
      return -1;
    }
    v = (major == 10 && minor == 0) ? 1 : 2;
    cached[device].store(v, std::memory_order_relaxed);
  }
  return v == 1 ? 1 : 0;
}

namespace {

sgblasStatus_t launchProduct(sgblasContext *ctx, sgblasOperation_t ta, sgblasOperation_t tb,
                             int m, int n, int k, float alpha, const float *a, int lda,
                             const float *b, int ldb, float beta, float *c, int ldc,
                             const Batch &batch, cudaStream_t stream) {
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_EXECUTION_FAILED;
  }
  const int arch = isSm100(device);
  if (arch < 0) return SGBLAS_STATUS_EXECUTION_FAILED;
  if (arch == 0) return SGBLAS_STATUS_ARCH_MISMATCH;
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
  p.batch = batch.count;
  p.stride_a = batch.stride_a;
  p.stride_b = batch.stride_b;
  p.stride_c = batch.stride_c;
  p.a_ptrs = batch.a_ptrs;
  p.b_ptrs = batch.b_ptrs;
  p.c_ptrs = batch.c_ptrs;
  Scratch scratch;
  scratch.ctx = ctx;

  bool tA = ta == SGBLAS_OP_T, tB = tb == SGBLAS_OP_T;
  // Small FP32 products: the cluster kernel, which stages any layout itself.
  if (ctx->math_mode != SGBLAS_MATH_TF32) {
    const int sms = smCount(device);
    if (sms <= 0) return SGBLAS_STATUS_EXECUTION_FAILED;
    if (smallEligible(p, sms)) return launchSmall(tA, tB, p, scratch, device, sms, stream);
  }
  // An operand TMA cannot read in place (base not 16-byte aligned, or ld not
  // a multiple of 4 floats) is copied into the workspace as an x-contiguous
  // matrix (A: m x k, as for op N; B: n x k, as for op T) with an aligned
  // leading dimension, and the product runs on TMA staging. Without a
  // workspace, and for batches, the tile kernel stages it with cp.async.
  // In a large FP32 product a k-contiguous operand (A transposed, B not) is
  // copied the same way so that the kernel needs no transposes, when the
  // other side of C is at least kPackReuse long (see sgemm_launch.hpp).
  const bool single = batch.count == 1 && batch.a_ptrs == nullptr;
  const bool fp32 = ctx->math_mode != SGBLAS_MATH_TF32;
  auto worthCopy = [&](long long reuse, long long rows_x) {
    return fp32 && reuse >= kPackReuse &&
           static_cast<size_t>(rows_x) * static_cast<size_t>(k) * sizeof(float) <= kPackMaxBytes;
  };
  const bool pack_a = single && (!(aligned16(a) && lda % 4 == 0) || (tA && worthCopy(n, m)));
  const bool pack_b = single && (!(aligned16(b) && ldb % 4 == 0) || (!tB && worthCopy(m, n)));
  bool packed = false;
  if (pack_a || pack_b) {
    const int sms = smCount(device);
    if (sms <= 0) return SGBLAS_STATUS_EXECUTION_FAILED;
    auto roundUp = [](size_t v, size_t q) { return (v + q - 1) / q * q; };
    const int ldp_a = static_cast<int>(roundUp(static_cast<size_t>(m), kPackLdMultiple));
    const int ldp_b = static_cast<int>(roundUp(static_cast<size_t>(n), kPackLdMultiple));
    const size_t off_a = roundUp(streamKRegionBytes(sms), kPackAlign);
    const size_t bytes_a = pack_a ? static_cast<size_t>(ldp_a) * k * sizeof(float) : 0;
    const size_t off_b = roundUp(off_a + bytes_a, kPackAlign);
    const size_t bytes_b = pack_b ? static_cast<size_t>(ldp_b) * k * sizeof(float) : 0;
    if (ldp_a >= m && ldp_b >= n && ensureWorkspace(ctx, off_b + bytes_b, device, stream)) {
      auto *ws = static_cast<unsigned char *>(ctx->workspace);
      if (pack_a) {
        auto *dst = reinterpret_cast<float *>(ws + off_a);
        const sgblasStatus_t st = launchPack(a, lda, tA, m, k, dst, ldp_a, sms, stream);
        if (st != SGBLAS_STATUS_SUCCESS) return st;
        p.a = dst;
        p.lda = ldp_a;
        tA = false;
      }
      if (pack_b) {
        auto *dst = reinterpret_cast<float *>(ws + off_b);
        const sgblasStatus_t st = launchPack(b, ldb, !tB, n, k, dst, ldp_b, sms, stream);
        if (st != SGBLAS_STATUS_SUCCESS) return st;
        p.b = dst;
        p.ldb = ldp_b;
        tB = true;
      }
      packed = true;
    }
  }
  sgblasStatus_t st;
  // TF32 for one matrix or a strided batch whose matrices TMA can all read
  // (positive strides, multiples of 4 floats); otherwise FP32, which is
  // more accurate than TF32 mode asks.
  auto tf32Stride = [](long long stride) {
    return stride > 0 && stride % 4 == 0 && stride < (1LL << 38);
  };
  if (ctx->math_mode == SGBLAS_MATH_TF32 && batch.a_ptrs == nullptr &&
      tf32Eligible(p.a, p.lda, p.b, p.ldb) &&
      (batch.count == 1 || (tf32Stride(batch.stride_a) && tf32Stride(batch.stride_b)))) {
    st = launchTf32(tA, tB, p, scratch, device, stream);
  } else if (!tA && !tB) st = launchMode<false, false>(p, scratch, device, stream);
  else if (!tA && tB) st = launchMode<false, true>(p, scratch, device, stream);
  else if (tA && !tB) st = launchMode<true, false>(p, scratch, device, stream);
  else st = launchMode<true, true>(p, scratch, device, stream);
  // The product read the packed operands: later users of the workspace wait.
  if (st == SGBLAS_STATUS_SUCCESS && packed && !markWorkspaceUse(ctx, stream))
    return SGBLAS_STATUS_EXECUTION_FAILED;
  return st;
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
  const auto stream = static_cast<cudaStream_t>(handle->stream);
  const Batch one;
  if (plan.work == Work::kScale) return launchScale(m, n, plan.beta, c, ldc, one, stream);
  return launchProduct(handle, transa, transb, m, n, k, plan.alpha, a, lda, b, ldb, plan.beta, c,
                       ldc, one, stream);
}

// Test hook: the counter state a split launch that stopped early leaves
// behind (one arrival of the handle's latest epoch on every counter).
namespace sgblas::detail {
namespace {
__global__ void interruptedCountersKernel(Counter *counters, int count, Counter value) {
  for (int i = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x); i < count;
       i += static_cast<int>(gridDim.x * blockDim.x))
    counters[i] = value;
}
}  // namespace
}  // namespace sgblas::detail

extern "C" sgblasStatus_t sgblasTestInterruptScratch(sgblasHandle_t handle) {
  using namespace sgblas::detail;
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  if (handle->workspace == nullptr) return SGBLAS_STATUS_NOT_SUPPORTED;
  int current = -1;
  if (cudaGetDevice(&current) != cudaSuccess || current != handle->workspace_device) {
    (void)cudaGetLastError();
    return SGBLAS_STATUS_INVALID_VALUE;
  }
  const auto stream = static_cast<cudaStream_t>(handle->stream);
  const Counter value = (static_cast<Counter>(handle->workspace_epoch) << 32) | 1ULL;
  constexpr int kCount = static_cast<int>(kCounterRegionBytes / sizeof(Counter));
  interruptedCountersKernel<<<4, 256, 0, stream>>>(static_cast<Counter *>(handle->workspace),
                                                   kCount, value);
  return launchStatus(cudaGetLastError());
}

// Batched forms (no counterpart in the reference, whose v1 design lists
// batched GEMM as a non-goal): every matrix of the batch is validated and
// computed exactly as sgblasSgemm would, in one launch. The pointers checked
// for NULL are the base pointers (strided) or the device pointer arrays.
namespace {

sgblasStatus_t sgemmBatch(sgblasHandle_t handle, sgblasOperation_t transa,
                          sgblasOperation_t transb, int m, int n, int k, const float *alpha,
                          const float *a, int lda, const float *b, int ldb, const float *beta,
                          float *c, int ldc, const sgblas::detail::Batch &batch) {
  using namespace sgblas::detail;
  if (handle == nullptr) return SGBLAS_STATUS_NOT_INITIALIZED;
  SgemmPlan plan;
  const sgblasStatus_t status =
      validate(transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc, &plan);
  if (status != SGBLAS_STATUS_SUCCESS) return status;
  if (batch.count < 0) return SGBLAS_STATUS_INVALID_VALUE;
  if (plan.work == Work::kNothing || batch.count == 0) return SGBLAS_STATUS_SUCCESS;
  const auto stream = static_cast<cudaStream_t>(handle->stream);
  if (plan.work == Work::kScale) return launchScale(m, n, plan.beta, c, ldc, batch, stream);
  return launchProduct(handle, transa, transb, m, n, k, plan.alpha, a, lda, b, ldb, plan.beta, c,
                       ldc, batch, stream);
}

}  // namespace

extern "C" sgblasStatus_t sgblasSgemmStridedBatched(
    sgblasHandle_t handle, sgblasOperation_t transa, sgblasOperation_t transb, int m, int n,
    int k, const float *alpha, const float *a, int lda, long long stride_a, const float *b,
    int ldb, long long stride_b, const float *beta, float *c, int ldc, long long stride_c,
    int batch_count) {
  sgblas::detail::Batch batch;
  batch.count = batch_count;
  batch.stride_a = stride_a;
  batch.stride_b = stride_b;
  batch.stride_c = stride_c;
  return sgemmBatch(handle, transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc, batch);
}

extern "C" sgblasStatus_t sgblasSgemmBatched(sgblasHandle_t handle, sgblasOperation_t transa,
                                             sgblasOperation_t transb, int m, int n, int k,
                                             const float *alpha, const float *const a_array[],
                                             int lda, const float *const b_array[], int ldb,
                                             const float *beta, float *const c_array[], int ldc,
                                             int batch_count) {
  sgblas::detail::Batch batch;
  batch.count = batch_count;
  batch.a_ptrs = a_array;
  batch.b_ptrs = b_array;
  batch.c_ptrs = c_array;
  // validate() checks the arrays for NULL where sgblasSgemm checks matrices.
  return sgemmBatch(handle, transa, transb, m, n, k, alpha,
                    reinterpret_cast<const float *>(a_array), lda,
                    reinterpret_cast<const float *>(b_array), ldb, beta,
                    reinterpret_cast<float *>(const_cast<float **>(c_array)), ldc, batch);
}
