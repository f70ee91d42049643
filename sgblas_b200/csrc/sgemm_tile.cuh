// The strict-FP32 tile kernel: C tile += op(A) panel * op(B) panel on CUDA
// cores with the sm_100 packed FP32 FMA (FFMA2, fma.rn.f32x2).
//
// Replaces the reference's SIMT FFMA kernels (src/sgemm_cuda.cu:86-395 and
// src/sgemm_async_sm80*.cu of AG0708/sgBLAS) with one family covering all four
// transpose modes, tails and any leading dimension.
//
// Arithmetic. Each FFMA2 performs two independent IEEE fma.rn operations, so
// every output is a chain of FP32 fused multiply-adds in k order -- the
// arithmetic of the reference's fmaf loops (no TF32, no tensor cores). The
// epilogue is the reference's: p = alpha*acc; beta == 0: c = p; beta == 1:
// c = c + p; otherwise c = fmaf(beta, c, p) (src/sgemm_cuda.cu:116-123).
//
// Operand roles. FFMA2 multiplies a register pair by a register pair. The
// "pair" operand P feeds two elements adjacent along its free dimension (half
// of a 16-byte shared-memory load); the "broadcast" operand D feeds one element
// to both lanes. Either A or B can be P (a template parameter): the
// orientation with the smaller padded tile area is chosen per call.
//
// Shared-memory tile layouts:
//   kXK : [BK][BX] floats, x contiguous -- what TMA writes when x is the
//         contiguous global dimension (A not transposed, B transposed).
//   kKX : [BX][BK] floats, k contiguous, 64-byte rows with the TMA 64B swizzle
//         (16-byte chunk index ^= (row >> 1) & 3).
// Operands are staged in their natural layout; the compute warps read both P
// and D as [k][x] (reads from [x][k] rows measured ~10% slower in the inner
// loop), so the producer warpgroup transposes every [x][k]-staged operand into
// a [k][x] buffer a few iterations ahead of its use.
//
// CTA: three warpgroups, one CTA per SM.
//   - Warpgroups 0-1 (256 threads, 8 warps) compute a 256 (P) x 128 (D) tile
//     (kTP = 16); each thread owns a 16 (P) x 8 (D) block of C (64 FFMA2 per
//     k step against 4+2 shared loads). Warps form 2 (P) x 4 (D); lane bits
//     lp = lane % 8, ld = lane / 8.
//       P coordinates: 128*wp + 4*lp + {0..3} + 32*q, q = 0..3.
//       D coordinates: 32*wd + 4*ld + {0..3} + {0, 16}.
//     The kTP = 8 variant (small problems) computes 128 x 128 tiles with an
//     8 x 8 block per thread.
//   - Warpgroup 2 (128 threads) is the producer: one thread issues the TMA
//     tile loads (or all 128 issue cp.async copies), and all 128 transpose
//     [x][k] tiles into [k][x] buffers. With beta != 0 it also prefetches
//     each whole tile's block of C into L2. It gives registers to the compute
//     warpgroups (setmaxnreg), so that those keep 232.
//   Tiles of a strided or pointer-array batch are numbered batch-major in the
//   same schedule; TMA tensor maps are 3-D (x, k, matrix).
//   Producer and consumers meet only at mbarriers (stage full/empty,
//   transposed buffer full/empty), so no warp ever waits on a CTA-wide
//   barrier inside the main loop.
#ifndef SGBLAS_B200_SGEMM_TILE_CUH_
#define SGBLAS_B200_SGEMM_TILE_CUH_

#include "ptx.cuh"

#include <cstddef>
#include <cstdint>

namespace sgblas::kern {

constexpr int kBD = 128;   // broadcast-operand tile extent
constexpr int kBK = 16;    // k slice per pipeline stage
constexpr int kStages = 6;
constexpr int kTransBufs = 3;   // ring of transposed [k][x] tiles
constexpr int kTD = 8;          // broadcast-operand elements per thread
constexpr int kWarpsP = 2;      // warps along P (8 lanes x kTP each)
constexpr int kWarpsD = kBD / 32;          // warps along D (4 lanes x 8 each)
constexpr int kThreads = 32 * kWarpsP * kWarpsD;   // compute threads (256)
constexpr int kConsumerWarps = kThreads / 32;
constexpr int kProducerThreads = 128;               // one warpgroup
constexpr int kBlockThreads = kThreads + kProducerThreads;
// With TMA staging and a transposed operand, warp 0 of the producer issues the
// loads and the other three warps transpose.
constexpr int kTransposers = kProducerThreads - 32;
constexpr int kSplitMinIters = 16;
// Register split: the block is launched with kLaunchRegs per thread (what
// __launch_bounds__(384, 1) leaves ptxas); setmaxnreg then moves registers
// from the producer warpgroup to the compute warpgroups.
constexpr int kLaunchRegs = 168;
constexpr int kConsumerRegs = 232;
constexpr int kProducerRegs = 40;
static_assert(kThreads * kConsumerRegs + kProducerThreads * kProducerRegs <=
                  kBlockThreads * kLaunchRegs,
              "register split exceeds the launch allocation");
constexpr int kDupFloats = kBD * kBK;
constexpr int kDupBytes = kDupFloats * 4;     // 8 KiB
constexpr int kBarrierBytes = 8 * (2 * kStages + 2 * kTransBufs);
constexpr int kSmemAlign = 1024;

// Tile geometry by pair-operand elements per thread: kTP = 16 gives the
// 256 (P) x 128 (D) tile used for large problems, kTP = 8 a 128 x 128 tile for
// problems with too few large tiles to fill the GPU.
template <int kTP_>
struct Geo {
  static constexpr int kTP = kTP_;
  static constexpr int kBP = kWarpsP * 8 * kTP;   // pair-operand tile extent
  static constexpr int kPairFloats = kBP * kBK;
  static constexpr int kPairBytes = kPairFloats * 4;
  static constexpr int kStageBytes = kPairBytes + kDupBytes;
  static constexpr int kTransBytes = kTransBufs * kStageBytes;  // room for both operands
  static constexpr int kSmemBytes =
      kStages * kStageBytes + kTransBytes + kBarrierBytes + kSmemAlign;
  static constexpr int kSlotFloat4 = kTP * kTD / 4;  // float4s per thread in a partial slot
  static constexpr size_t kSlotBytes = size_t{kThreads} * kSlotFloat4 * 16;
  static_assert(kTP == 8 || kTP == 16, "per-thread pair extent");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
};

enum class Beta { kZero, kOne, kGeneral };
enum class Src { kTma, kCopy };
enum class Layout { kXK, kKX };

struct GemmParams {
  CUtensorMap tma_a;  // valid when the kernel stages tiles with TMA (3-D: x, k, batch)
  CUtensorMap tma_b;
  const float *a;
  const float *b;
  float *c;
  // Batches: matrix i is A + i*stride_a (B, C alike), or a_ptrs[i] when the
  // caller passed device arrays of pointers (then a/b/c are unused).
  int batch;
  long long stride_a, stride_b, stride_c;
  const float *const *a_ptrs;
  const float *const *b_ptrs;
  float *const *c_ptrs;
  int m, n, k;
  int lda, ldb, ldc;
  float alpha, beta;
  int tiles_m, tiles_n;
  int group_m;        // raster: tile rows per CTA group
  unsigned *err;      // device error word
  // Persistent schedule (see the kernel comment): tiles [0, dp_tiles) are
  // whole-tile work dealt round-robin to the CTAs; tiles [dp_tiles,
  // dp_tiles + sk_tiles) are split by k iterations ("stream-K"): CTA c owns
  // iterations [c*sk_q + min(c, sk_r), (c+1)*sk_q + min(c+1, sk_r)).
  int kiters;         // k iterations (BK slices) per tile
  int grid;           // persistent CTAs
  int dp_tiles;
  int sk_tiles;
  int sk_q, sk_r;
  float4 *ws;         // 2 * grid partial-tile slots of Geo::kSlotBytes
  unsigned long long *counters;   // sk_tiles arrival counters (see arriveCounter)
  unsigned epoch;                 // this launch's counter epoch (non-zero)
  // cp.async path: floats per copy (1, 2 or 4) allowed by each operand's base
  // alignment and leading dimension.
  int a_vec, b_vec;
};

// One unit of a CTA's work: k iterations [kb, ke) of tile `tile`.
struct Item {
  int tile, kb, ke;
};

// Schedule helpers; Sched is any parameter block with the schedule fields of
// GemmParams (grid, dp_tiles, sk_tiles, sk_q, sk_r, kiters; tiles_m,
// tiles_n, group_m for the raster).
template <class Sched>
__device__ __forceinline__ int skBegin(const Sched &p, int c) {
  return c * p.sk_q + min(c, p.sk_r);
}

// The CTA owning stream-K iteration x (inverse of skBegin).
template <class Sched>
__device__ __forceinline__ int skOwner(const Sched &p, int x) {
  const int head = p.sk_r * (p.sk_q + 1);
  return x < head ? x / (p.sk_q + 1) : p.sk_r + (x - head) / p.sk_q;
}

template <class Sched>
__device__ __forceinline__ int dpItems(const Sched &p, int c) {
  return c < p.dp_tiles ? (p.dp_tiles - 1 - c) / p.grid + 1 : 0;
}

template <class Sched>
__device__ __forceinline__ int numItems(const Sched &p, int c) {
  int n = dpItems(p, c);
  if (p.sk_tiles > 0) {
    const int s = skBegin(p, c), e = skBegin(p, c + 1);
    if (e > s) n += (e - 1) / p.kiters - s / p.kiters + 1;
  }
  return n;
}

template <class Sched>
__device__ __forceinline__ Item itemAt(const Sched &p, int c, int idx) {
  const int ndp = dpItems(p, c);
  if (idx < ndp) return {c + idx * p.grid, 0, p.kiters};
  const int s = skBegin(p, c), e = skBegin(p, c + 1);
  const int u = s / p.kiters + (idx - ndp);
  const int base = u * p.kiters;
  return {p.dp_tiles + u, max(s, base) - base, min(e, base + p.kiters) - base};
}

// Workspace slot of CTA c's piece of stream-K tile u: slot 2c holds the piece
// of the first tile c touches, slot 2c+1 the piece of its last one.
template <class Sched>
__device__ __forceinline__ int skSlot(const Sched &p, int c, int u) {
  return 2 * c + (u == skBegin(p, c) / p.kiters ? 0 : 1);
}

// Byte offset of element (x, k) inside a kKX tile.
__device__ __forceinline__ uint32_t kxOffset(int x, int k) {
  return static_cast<uint32_t>(x * 64 + ((((k >> 2) ^ (x >> 1)) & 3) << 4) + ((k & 3) << 2));
}

// Operand roles, staged layouts and the tile shape that follows.
template <bool kTA, bool kTB, bool kPairIsA_, int kTP>
struct Plan {
  using G = Geo<kTP>;
  static constexpr int kBP = G::kBP;
  static constexpr bool kPairIsA = kPairIsA_;
  // Natural staged layout: [k][x] when x is the contiguous global dimension.
  static constexpr Layout kA = kTA ? Layout::kKX : Layout::kXK;
  static constexpr Layout kB = kTB ? Layout::kXK : Layout::kKX;
  static constexpr int kAExt = kPairIsA ? kBP : kBD;  // tile extent along m
  static constexpr int kBExt = kPairIsA ? kBD : kBP;  // tile extent along n
  static constexpr Layout kP = kPairIsA ? kA : kB;
  static constexpr Layout kD = kPairIsA ? kB : kA;
  static constexpr bool kTransP = (kP == Layout::kKX);
  static constexpr bool kTransD = (kD == Layout::kKX);
  static constexpr bool kTrans = kTransP || kTransD;
  static constexpr int kBM = kAExt;
  static constexpr int kBN = kBExt;
};

// Tile index -> (tile_m, tile_n): groups of group_m tile rows are walked
// column by column so that concurrently running CTAs share panels in L2.
template <class Sched>
__device__ __forceinline__ void rasterTile(const Sched &p, int t, int *tm, int *tn) {
  const int per_group = p.group_m * p.tiles_n;
  const int group = t / per_group;
  const int first = group * p.group_m;
  const int rows = min(p.tiles_m - first, p.group_m);
  const int in = t - group * per_group;
  *tm = first + in % rows;
  *tn = in / rows;
}

// ---- cp.async staging (any alignment, any leading dimension, tails) --------
// One operand tile in its natural layout (the layout TMA would write), by the
// producer warpgroup, in copies of kVec floats along the contiguous dimension
// (4 or 8 bytes when the operand's alignment forbids 16), zero-filled outside
// the matrix: a copy that straddles the matrix edge reads only its in-range
// floats. Global reads are coalesced along the contiguous dimension. Element
// (x, k) of the stored matrix is src[x + k*ld] for an [k][x] tile and
// src[k + x*ld] for an [x][k] tile; x0/k0 are the tile origin, x_limit/k_limit
// the matrix extents. Requires src and ld to be multiples of kVec floats.
template <int kExt, bool kKx, int kVec>
__device__ __forceinline__ void copyOperandVec(const float *src, int ld, int x_limit, int k_limit,
                                               float *dst, int x0, int k0, int tid) {
  constexpr int kN = kProducerThreads;
  constexpr int kRun = kKx ? kBK / kVec : kExt / kVec;  // copies along the contiguous dim
#pragma unroll 4
  for (int r = 0; r < kExt * kBK / (kVec * kN); ++r) {
    const int e = tid + r * kN;
    const int x = kKx ? e / kRun : (e % kRun) * kVec;
    const int kk = kKx ? (e % kRun) * kVec : e / kRun;
    const int gx = x0 + x, gk = k0 + kk;
    int valid;
    if constexpr (kKx) valid = gx < x_limit ? min(max(k_limit - gk, 0), kVec) : 0;
    else valid = gk < k_limit ? min(max(x_limit - gx, 0), kVec) : 0;
    const float *s = src;
    if (valid > 0) {
      s = kKx ? src + static_cast<size_t>(gk) + static_cast<size_t>(gx) * ld
              : src + static_cast<size_t>(gx) + static_cast<size_t>(gk) * ld;
    }
    float *d = kKx ? reinterpret_cast<float *>(reinterpret_cast<char *>(dst) + kxOffset(x, kk))
                   : dst + kk * kExt + x;
    cpAsyncN<4 * kVec>(d, s, static_cast<uint32_t>(4 * valid));
  }
}

template <int kExt, bool kKx>
__device__ __forceinline__ void copyOperand(const float *src, int ld, int x_limit, int k_limit,
                                            float *dst, int x0, int k0, int tid, int vec) {
  if (vec == 4) copyOperandVec<kExt, kKx, 4>(src, ld, x_limit, k_limit, dst, x0, k0, tid);
  else if (vec == 2) copyOperandVec<kExt, kKx, 2>(src, ld, x_limit, k_limit, dst, x0, k0, tid);
  else copyOperandVec<kExt, kKx, 1>(src, ld, x_limit, k_limit, dst, x0, k0, tid);
}

// [x][k] tile of kRows rows (64-byte swizzled) -> [k][x] (kRows floats per k),
// by kN producer threads: thread t moves rows t, t + kN, ... A warp reads 32
// consecutive rows at one chunk -- conflict-free thanks to the swizzle -- and
// writes 32 consecutive floats per k.
template <int kRows, int kN = kProducerThreads>
__device__ __forceinline__ void transposeKX(const float *src, float *dst, int tid) {
  static_assert(kBK == 16, "64-byte rows");
#pragma unroll
  for (int r = tid; r < kRows; r += kN) {
    const char *row = reinterpret_cast<const char *>(src) + r * 64;
    const int phase = (r >> 1) & 3;
    float *d = dst + r;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float4 v = *reinterpret_cast<const float4 *>(row + ((c ^ phase) << 4));
      d[(4 * c + 0) * kRows] = v.x;
      d[(4 * c + 1) * kRows] = v.y;
      d[(4 * c + 2) * kRows] = v.z;
      d[(4 * c + 3) * kRows] = v.w;
    }
  }
}

// ---- the FFMA2 micro-kernel over one BK slice ------------------------------
// sp: [k][kBP] pair tile, sd: [k][kBD] broadcast tile.
template <int kTP>
__device__ __forceinline__ void computeStage(const float *sp, const float *sd, int p_base,
                                             int d_base, float2 (&acc)[kTP / 2][kTD]) {
  constexpr int kBP = Geo<kTP>::kBP;
#pragma unroll
  for (int k = 0; k < kBK; k += 2) {
    float dv[2][kTD];
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const float4 d0 = *reinterpret_cast<const float4 *>(sd + (k + kk) * kBD + d_base);
      const float4 d1 = *reinterpret_cast<const float4 *>(sd + (k + kk) * kBD + d_base + 16);
      dv[kk][0] = d0.x; dv[kk][1] = d0.y; dv[kk][2] = d0.z; dv[kk][3] = d0.w;
      dv[kk][4] = d1.x; dv[kk][5] = d1.y; dv[kk][6] = d1.z; dv[kk][7] = d1.w;
    }
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      float2 pv[kTP / 2];
#pragma unroll
      for (int q = 0; q < kTP / 4; ++q) {
        const float4 v = *reinterpret_cast<const float4 *>(sp + (k + kk) * kBP + p_base + 32 * q);
        pv[2 * q] = make_float2(v.x, v.y);
        pv[2 * q + 1] = make_float2(v.z, v.w);
      }
#pragma unroll
      for (int i = 0; i < kTP / 2; ++i) {
#pragma unroll
        for (int j = 0; j < kTD; ++j) {
          acc[i][j] = __ffma2_rn(pv[i], make_float2(dv[kk][j], dv[kk][j]), acc[i][j]);
        }
      }
    }
  }
}

template <Beta kBeta>
__device__ __forceinline__ float epilogueValue(float acc, float alpha, float beta, float c) {
  const float prod = alpha * acc;
  if constexpr (kBeta == Beta::kZero) {
    return prod;
  } else if constexpr (kBeta == Beta::kOne) {
    return c + prod;
  } else {
    return fmaf(beta, c, prod);
  }
}

// ---- the persistent, warp-specialized kernel ----------------------------------
// Each CTA walks its items in order (whole tiles first, then its stream-K
// range); the k iterations of consecutive items form one flat stream, so the
// producer keeps prefetching the next tile while the compute warps finish the
// current one. A stream-K piece that does not cover its whole tile is
// published to the workspace; the CTA that publishes the last piece of a tile
// (an atomic arrival count, no waiting) sums every piece in piece order -- an
// order fixed by the schedule, so results do not depend on timing -- and
// writes C.
//
// Synchronisation (all mbarriers, all waits bounded):
//   full[s]     stage s holds iteration i's tiles   (TMA bytes / cp.async)
//   empty[s]    the 8 compute warps are done with stage s
//   tfull[t]    transposed buffer t is written (128 producer threads)
//   tempty[t]   the 8 compute warps are done with buffer t
// A wait that times out raises the device error flag; from then on that
// thread skips its waits (results are garbage and flagged) but still runs
// every loop to its end, so that no thread is left behind at a barrier.
template <int kTP, bool kTA, bool kTB, bool kPairIsA, Beta kBeta, Src kSrc>
__global__ void __launch_bounds__(kBlockThreads, 1)
    sgemmKernel(const __grid_constant__ GemmParams p) {
  using P = Plan<kTA, kTB, kPairIsA, kTP>;
  using G = typename P::G;
  constexpr int kBP = G::kBP;
  constexpr int kPairBytes = G::kPairBytes;
  constexpr int kStageBytes = G::kStageBytes;
  constexpr int kTransBytes = G::kTransBytes;
  constexpr int kSlotFloat4 = G::kSlotFloat4;
  extern __shared__ unsigned char smem_raw[];
  __shared__ int last_arrival;
  // Align within the shared window by offsetting smem_raw itself: pointers
  // derived from the __shared__ array stay in the shared address space, so the
  // compiler emits 32-bit shared loads (a uintptr_t round trip would turn them
  // into 64-bit generic loads and double the address registers).
  unsigned char *smem = smem_raw + ((kSmemAlign - (smemAddr(smem_raw) & (kSmemAlign - 1))) &
                                    (kSmemAlign - 1));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes + kTransBytes);
  uint64_t *empty = full + kStages;
  uint64_t *tfull = empty + kStages;
  uint64_t *tempty = tfull + kTransBufs;
  // Stage s: the pair tile at offset 0, the broadcast tile after it; the
  // transposed buffers use the same split.
  auto stageP = [&](int s) { return reinterpret_cast<float *>(smem + s * kStageBytes); };
  auto stageD = [&](int s) {
    return reinterpret_cast<float *>(smem + s * kStageBytes + kPairBytes);
  };
  auto tbufP = [&](int t) {
    return reinterpret_cast<float *>(smem + kStages * kStageBytes + t * kStageBytes);
  };
  auto tbufD = [&](int t) {
    return reinterpret_cast<float *>(smem + kStages * kStageBytes + t * kStageBytes + kPairBytes);
  };
  auto stageA = [&](int s) { return P::kPairIsA ? stageP(s) : stageD(s); };
  auto stageB = [&](int s) { return P::kPairIsA ? stageD(s) : stageP(s); };
  // Tiles are numbered batch-major; within a matrix they follow rasterTile.
  const int tiles_per_matrix = p.tiles_m * p.tiles_n;
  auto origin = [&](int tile, int *m0, int *n0, int *bi) {
    int tm, tn;
    *bi = tile / tiles_per_matrix;
    rasterTile(p, tile - *bi * tiles_per_matrix, &tm, &tn);
    *m0 = tm * P::kBM;
    *n0 = tn * P::kBN;
  };
  auto matrixA = [&](int bi) {
    return p.a_ptrs != nullptr ? p.a_ptrs[bi] : p.a + bi * p.stride_a;
  };
  auto matrixB = [&](int bi) {
    return p.b_ptrs != nullptr ? p.b_ptrs[bi] : p.b + bi * p.stride_b;
  };
  auto matrixC = [&](int bi) {
    return p.c_ptrs != nullptr ? p.c_ptrs[bi] : p.c + bi * p.stride_c;
  };

  const int cta = blockIdx.x;
  const int nitems = numItems(p, cta);
  if (nitems == 0) return;  // whole CTA, before any barrier
  int total = 0;            // k iterations over all items
  for (int i = 0; i < nitems; ++i) {
    const Item it = itemAt(p, cta, i);
    total += it.ke - it.kb;
  }
  const int tid = threadIdx.x;
  // Transposing plans staged by TMA split the producer into a loading warp
  // and three transposing warps when the CTA has enough iterations (measured:
  // faster from 896^3 up, slower for a single short piece, e.g. 768^3).
  const bool split_producer = P::kTrans && kSrc == Src::kTma && total >= kSplitMinIters;

  if (tid == 0) {
    if constexpr (kSrc == Src::kTma) {
      prefetchTensorMap(&p.tma_a);
      prefetchTensorMap(&p.tma_b);
    }
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbarInit(&full[s], kSrc == Src::kTma ? 1 : kProducerThreads);
      mbarInit(&empty[s], kConsumerWarps);
    }
#pragma unroll
    for (int t = 0; t < kTransBufs; ++t) {
      mbarInit(&tfull[t], split_producer ? kTransposers : kProducerThreads);
      mbarInit(&tempty[t], kConsumerWarps);
    }
    fenceBarrierInit();
  }
  __syncthreads();
  // Launched with programmatic stream serialization: the set-up above may
  // overlap the previous kernel in the stream; nothing below runs before it
  // has finished.
  gridDependencyWait();
  allowDependentLaunch();

  // ======================= producer warpgroup ===============================
  if (tid >= kThreads) {
    regDealloc<kProducerRegs>();
    const int pt = tid - kThreads;
    bool ok = true;
    auto wait = [&](uint64_t *bar, int parity) {
      if (ok) ok = mbarWait(bar, static_cast<uint32_t>(parity), p.err);
    };
    // With beta != 0 the epilogue of a tile reads its block of C. The
    // producer prefetches that block into L2 when it starts loading the item
    // that will most likely run that epilogue, a whole main loop before the
    // read: a whole tile, or the first piece (k from 0) of a split tile --
    // the CTA owning it reaches that piece at the end of its range, after
    // the owners of the later pieces have started theirs, so it is the last
    // to arrive. One column per thread, the 16-byte aligned interior of the
    // in-range rows (never outside C).
    auto prefetchC = [&](const Item &it, int tm0, int tn0, int bi, int first = -1,
                         int stride = kProducerThreads) {
      if constexpr (kBeta != Beta::kZero) {
        if (it.kb != 0) return;
        const int r1 = min(tm0 + P::kBM, p.m);
        const float *cbase = matrixC(bi);
#pragma unroll 1
        for (int cc = first < 0 ? pt : first; cc < P::kBN; cc += stride) {
          const int col = tn0 + cc;
          if (col >= p.n) break;
          const float *colp = cbase + static_cast<size_t>(col) * p.ldc;
          const uintptr_t lo = (reinterpret_cast<uintptr_t>(colp + tm0) + 15) & ~uintptr_t{15};
          const uintptr_t hi = reinterpret_cast<uintptr_t>(colp + r1) & ~uintptr_t{15};
          if (hi > lo)
            prefetchL2Bulk(reinterpret_cast<const void *>(lo), static_cast<uint32_t>(hi - lo));
        }
      }
    };
    // Three producer variants follow: per-item loads (no transposes), a
    // loading warp beside three transposing warps (TMA, enough iterations),
    // and one coupled loop (cp.async staging, or a CTA with a short piece).
    // Each writes its TMA issue out in full: sharing it through a lambda
    // changed the code generated for the transposing plans and measured
    // 0.3-0.6 % slower.
    if constexpr (!P::kTrans) {
      // No transposes: one item at a time, its loads in a loop of their own
      // (measured faster than the flat loop below for these plans, slower
      // for the transposing ones).
      int i = 0;   // iterations loaded so far, over all items
      for (int idx = 0; idx < nitems; ++idx) {
        const Item it = itemAt(p, cta, idx);
        int m0, n0, bi;
        origin(it.tile, &m0, &n0, &bi);
        const float *a_src = nullptr, *b_src = nullptr;  // cp.async: this item's matrices
        if constexpr (kSrc == Src::kCopy) {
          a_src = matrixA(bi);
          b_src = matrixB(bi);
        }
        prefetchC(it, m0, n0, bi);
#pragma unroll 1
        for (int kt = it.kb; kt < it.ke; ++kt, ++i) {
          const int s = i % kStages;
          const int k0 = kt * kBK;
          if constexpr (kSrc == Src::kTma) {
            if (pt == 0) {
              if (i >= kStages) {
                wait(&empty[s], (i / kStages - 1) & 1);
                fenceProxyAsyncShared();   // the compute warps read stage s with ld.shared
              }
              mbarArriveExpectTx(&full[s], kStageBytes);
              if (P::kA == Layout::kXK) tmaLoad3d(stageA(s), &p.tma_a, &full[s], m0, k0, bi);
              else tmaLoad3d(stageA(s), &p.tma_a, &full[s], k0, m0, bi);
              if (P::kB == Layout::kXK) tmaLoad3d(stageB(s), &p.tma_b, &full[s], n0, k0, bi);
              else tmaLoad3d(stageB(s), &p.tma_b, &full[s], k0, n0, bi);
            }
          } else {
            if (i >= kStages) wait(&empty[s], (i / kStages - 1) & 1);
            copyOperand<P::kAExt, P::kA == Layout::kKX>(a_src, p.lda, p.m, p.k, stageA(s), m0,
                                                         k0, pt, p.a_vec);
            copyOperand<P::kBExt, P::kB == Layout::kKX>(b_src, p.ldb, p.n, p.k, stageB(s), n0,
                                                         k0, pt, p.b_vec);
            cpAsyncArrive(&full[s]);
          }
        }
      }
    } else if (split_producer) {
      // Transposing plans staged by TMA: warp 0 loads (lane 0 issues the
      // TMA, its 32 lanes prefetch C), one item at a time; warps 1-3
      // transpose every landed stage into the transposed ring. Deadlock-free:
      // a load waits for the compute warps to release the stage it refills,
      // a transpose for the stage to land and for the compute warps to
      // release the buffer it overwrites, and the compute warps only for
      // transposed buffers -- no role waits on one that waits on it.
      if (pt < 32) {
        int i = 0;   // iterations loaded so far, over all items
        for (int idx = 0; idx < nitems; ++idx) {
          const Item it = itemAt(p, cta, idx);
          int m0, n0, bi;
          origin(it.tile, &m0, &n0, &bi);
          prefetchC(it, m0, n0, bi, pt, 32);
          if (pt != 0) continue;
#pragma unroll 1
          for (int kt = it.kb; kt < it.ke; ++kt, ++i) {
            const int s = i % kStages;
            const int k0 = kt * kBK;
            if (i >= kStages) {
              wait(&empty[s], (i / kStages - 1) & 1);
              fenceProxyAsyncShared();   // the compute warps read stage s with ld.shared
            }
            mbarArriveExpectTx(&full[s], kStageBytes);
            if (P::kA == Layout::kXK) tmaLoad3d(stageA(s), &p.tma_a, &full[s], m0, k0, bi);
            else tmaLoad3d(stageA(s), &p.tma_a, &full[s], k0, m0, bi);
            if (P::kB == Layout::kXK) tmaLoad3d(stageB(s), &p.tma_b, &full[s], n0, k0, bi);
            else tmaLoad3d(stageB(s), &p.tma_b, &full[s], k0, n0, bi);
          }
        }
      } else {
        const int xt = pt - 32;
#pragma unroll 1
        for (int j = 0; j < total; ++j) {
          const int t = j % kTransBufs;
          wait(&full[j % kStages], (j / kStages) & 1);
          if (j >= kTransBufs) wait(&tempty[t], (j / kTransBufs - 1) & 1);
          if constexpr (P::kTransP)
            transposeKX<kBP, kTransposers>(stageP(j % kStages), tbufP(t), xt);
          if constexpr (P::kTransD)
            transposeKX<kBD, kTransposers>(stageD(j % kStages), tbufD(t), xt);
          mbarArrive(&tfull[t]);
        }
      }
    } else {
      int idx = 0, kt, ke, m0, n0, bi;
      const float *a_src = nullptr, *b_src = nullptr;  // cp.async: this item's matrices
      auto startItem = [&](const Item &it) {
        kt = it.kb;
        ke = it.ke;
        origin(it.tile, &m0, &n0, &bi);
        if constexpr (kSrc == Src::kCopy) {
          a_src = matrixA(bi);
          b_src = matrixB(bi);
        }
        prefetchC(it, m0, n0, bi);
      };
      startItem(itemAt(p, cta, 0));
      // Transposes trail the loads by kLag iterations: far enough behind for the
      // data to have landed, early enough to stay up to two iterations ahead of
      // the compute warps. Deadlock-free: the load of iteration i waits for the
      // consumers to release iteration i - kStages, and the transpose of
      // iteration j = i - kLag waits for them to release j - kTransBufs; with
      // kTransBufs >= kStages - kLag both point at iterations the consumers can
      // finish without this transpose.
      constexpr int kLag = P::kTrans ? kStages - 3 : 0;
      static_assert(!P::kTrans || kTransBufs >= kStages - kLag, "transposed ring too small");
      for (int i = 0; i < total + kLag; ++i) {
        if (i < total) {
          const int s = i % kStages;
          const int k0 = kt * kBK;
          if constexpr (kSrc == Src::kTma) {
            if (pt == 0) {
              if (i >= kStages) {
                wait(&empty[s], (i / kStages - 1) & 1);
                fenceProxyAsyncShared();   // the compute warps read stage s with ld.shared
              }
              mbarArriveExpectTx(&full[s], kStageBytes);
              if (P::kA == Layout::kXK) tmaLoad3d(stageA(s), &p.tma_a, &full[s], m0, k0, bi);
              else tmaLoad3d(stageA(s), &p.tma_a, &full[s], k0, m0, bi);
              if (P::kB == Layout::kXK) tmaLoad3d(stageB(s), &p.tma_b, &full[s], n0, k0, bi);
              else tmaLoad3d(stageB(s), &p.tma_b, &full[s], k0, n0, bi);
            }
          } else {
            if (i >= kStages) wait(&empty[s], (i / kStages - 1) & 1);
            copyOperand<P::kAExt, P::kA == Layout::kKX>(a_src, p.lda, p.m, p.k, stageA(s), m0, k0,
                                                         pt, p.a_vec);
            copyOperand<P::kBExt, P::kB == Layout::kKX>(b_src, p.ldb, p.n, p.k, stageB(s), n0, k0,
                                                         pt, p.b_vec);
            cpAsyncArrive(&full[s]);
          }
          if (++kt == ke && ++idx < nitems) startItem(itemAt(p, cta, idx));
        }
        if constexpr (P::kTrans) {
          const int j = i - kLag;
          if (j >= 0) {
            const int t = j % kTransBufs;
            wait(&full[j % kStages], (j / kStages) & 1);
            if (j >= kTransBufs) wait(&tempty[t], (j / kTransBufs - 1) & 1);
            if constexpr (P::kTransP) transposeKX<kBP>(stageP(j % kStages), tbufP(t), pt);
            if constexpr (P::kTransD) transposeKX<kBD>(stageD(j % kStages), tbufD(t), pt);
            mbarArrive(&tfull[t]);
          }
        }
      }
    }
    if constexpr (kSrc == Src::kCopy) cpAsyncWait<0>();
    return;
  }

  // ======================= compute warpgroups ===============================
  regAlloc<kConsumerRegs>();
  const int warp = tid / 32, lane = tid % 32;
  const int wp = warp % kWarpsP, wd = warp / kWarpsP;
  const int lp = lane % 8, ld = lane / 8;
  const int p_base = wp * (8 * kTP) + lp * 4;
  const int d_base = wd * 32 + ld * 4;
  bool ok = true;
  auto wait = [&](uint64_t *bar, int parity) {
    if (ok) ok = mbarWait(bar, static_cast<uint32_t>(parity), p.err);
  };

  float2 acc[kTP / 2][kTD];
#pragma unroll
  for (int i = 0; i < kTP / 2; ++i)
#pragma unroll
    for (int j = 0; j < kTD; ++j) acc[i][j] = make_float2(0.0F, 0.0F);

  const float alpha = p.alpha, beta = p.beta;
  bool c_vec = false;  // float4 access to C: set per tile (batches may differ)
  // C = alpha * acc (+ beta * C) for the tile at (m0, n0). The thread's
  // values come in kGroups groups of four consecutive rows of one column
  // (P = A: four consecutive P coordinates; P = B: four consecutive D
  // coordinates); a group inside the matrix is one float4 access when C
  // allows it. With beta != 0 the C reads of a batch of groups are all issued
  // before any of its stores (the compiler cannot move a load of C past a
  // store to C), so their latencies overlap; the producer has prefetched the
  // block into L2 during the tile's main loop.
  constexpr int kGroups = kTP * kTD / 4;
  constexpr int kBatch = 8;
  static_assert(kGroups % kBatch == 0, "epilogue batches");
  auto groupAt = [&](int g, int m0, int n0, int *row, int *col, float v[4]) {
    if constexpr (P::kPairIsA) {
      const int j = g / (kTP / 4), q = g % (kTP / 4);
      *col = n0 + d_base + (j & 3) + 16 * (j >> 2);
      *row = m0 + p_base + 32 * q;
      v[0] = acc[2 * q][j].x;
      v[1] = acc[2 * q][j].y;
      v[2] = acc[2 * q + 1][j].x;
      v[3] = acc[2 * q + 1][j].y;
    } else {
      const int i = g / 2, h = g % 2;
      *col = n0 + p_base + (i & 3) + 32 * (i >> 2);
      *row = m0 + d_base + 16 * h;
#pragma unroll
      for (int e = 0; e < 4; ++e)
        v[e] = (i & 1) ? acc[i >> 1][4 * h + e].y : acc[i >> 1][4 * h + e].x;
    }
  };
  auto loadGroup = [&](const float *cbase, int row, int col) {
    float4 cv = make_float4(0.0F, 0.0F, 0.0F, 0.0F);
    if (col >= p.n || row >= p.m) return cv;
    const float *cp = cbase + static_cast<size_t>(col) * p.ldc + row;
    if (c_vec && row + 3 < p.m) return *reinterpret_cast<const float4 *>(cp);
    cv.x = cp[0];
    if (row + 1 < p.m) cv.y = cp[1];
    if (row + 2 < p.m) cv.z = cp[2];
    if (row + 3 < p.m) cv.w = cp[3];
    return cv;
  };
  auto storeGroup = [&](float *cbase, int row, int col, const float v[4], float4 cv) {
    if (col >= p.n || row >= p.m) return;
    float *cp = cbase + static_cast<size_t>(col) * p.ldc + row;
    float4 out;
    out.x = epilogueValue<kBeta>(v[0], alpha, beta, cv.x);
    out.y = epilogueValue<kBeta>(v[1], alpha, beta, cv.y);
    out.z = epilogueValue<kBeta>(v[2], alpha, beta, cv.z);
    out.w = epilogueValue<kBeta>(v[3], alpha, beta, cv.w);
    if (c_vec && row + 3 < p.m) {
      *reinterpret_cast<float4 *>(cp) = out;
      return;
    }
    cp[0] = out.x;
    if (row + 1 < p.m) cp[1] = out.y;
    if (row + 2 < p.m) cp[2] = out.z;
    if (row + 3 < p.m) cp[3] = out.w;
  };
  auto storeTile = [&](int m0, int n0, int bi) {
    float *cbase = matrixC(bi);
    c_vec = (p.ldc % 4 == 0) && (reinterpret_cast<uintptr_t>(cbase) % 16 == 0);
#pragma unroll
    for (int g0 = 0; g0 < kGroups; g0 += kBatch) {
      float4 cv[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        cv[b] = make_float4(0.0F, 0.0F, 0.0F, 0.0F);
        if constexpr (kBeta != Beta::kZero) {
          int row, col;
          float v[4];
          groupAt(g0 + b, m0, n0, &row, &col, v);
          cv[b] = loadGroup(cbase, row, col);
        }
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        int row, col;
        float v[4];
        groupAt(g0 + b, m0, n0, &row, &col, v);
        storeGroup(cbase, row, col, v, cv[b]);
      }
    }
  };

  // Workspace slot layout: float4 e of thread tid at slot[e * kThreads + tid].
  auto publish = [&](int slot) {
    float4 *w = p.ws + static_cast<size_t>(slot) * (kThreads * kSlotFloat4) + tid;
#pragma unroll
    for (int i = 0; i < kTP / 2; ++i)
#pragma unroll
      for (int j = 0; j < kTD; j += 2)
        __stcg(w + (i * (kTD / 2) + j / 2) * kThreads,
               make_float4(acc[i][j].x, acc[i][j].y, acc[i][j + 1].x, acc[i][j + 1].y));
  };
  auto gather = [&](int slot) {
    const float4 *w = p.ws + static_cast<size_t>(slot) * (kThreads * kSlotFloat4) + tid;
#pragma unroll
    for (int i = 0; i < kTP / 2; ++i)
#pragma unroll
      for (int j = 0; j < kTD; j += 2) {
        const float4 v = __ldcg(w + (i * (kTD / 2) + j / 2) * kThreads);
        acc[i][j].x += v.x;
        acc[i][j].y += v.y;
        acc[i][j + 1].x += v.z;
        acc[i][j + 1].y += v.w;
      }
  };

  // One item at a time: its k iterations in a tight loop, then its epilogue.
  // g counts iterations over all items (stage g % kStages, transposed buffer
  // g % kTransBufs).
  int g = 0;
  for (int c_idx = 0; c_idx < nitems; ++c_idx) {
    const Item c_item = itemAt(p, cta, c_idx);
    const int g_end = g + (c_item.ke - c_item.kb);
#pragma unroll 1
    for (; g < g_end; ++g) {
      const int s = g % kStages;
      const int t = g % kTransBufs;
      // With a transposed operand, tfull[t] implies full[s]: every producer
      // thread waited for stage s to land before transposing it and arriving
      // on tfull[t] (release), so acquiring tfull[t] also makes the stage's
      // TMA or cp.async data visible. One wait per iteration instead of two.
      if constexpr (P::kTrans) wait(&tfull[t], (g / kTransBufs) & 1);
      else wait(&full[s], (g / kStages) & 1);
      computeStage<kTP>(P::kTransP ? tbufP(t) : stageP(s), P::kTransD ? tbufD(t) : stageD(s),
                        p_base, d_base, acc);
      __syncwarp();
      if (lane == 0) {
        mbarArrive(&empty[s]);
        if constexpr (P::kTrans) mbarArrive(&tempty[t]);
      }
    }

    int c_m0, c_n0, c_bi;
    origin(c_item.tile, &c_m0, &c_n0, &c_bi);
    if (c_item.kb == 0 && c_item.ke == p.kiters) {
      storeTile(c_m0, c_n0, c_bi);
    } else {
      // Stream-K piece: publish, count the arrival, and let the last
      // arriving piece reduce all pieces in piece order.
      const int u = c_item.tile - p.dp_tiles;
      const int first = skOwner(p, u * p.kiters);
      const int last = skOwner(p, (u + 1) * p.kiters - 1);
      publish(skSlot(p, cta, u));
      __threadfence();
      namedBarrier<1, kThreads>();
      if (tid == 0)
        last_arrival = arriveCounter(p.counters + u, p.epoch, p.err) ==
                       static_cast<unsigned>(last - first + 1);
      namedBarrier<1, kThreads>();
      if (last_arrival) {
        __threadfence();
#pragma unroll
        for (int i = 0; i < kTP / 2; ++i)
#pragma unroll
          for (int j = 0; j < kTD; ++j) acc[i][j] = make_float2(0.0F, 0.0F);
#pragma unroll 1
        for (int c = first; c <= last; ++c) gather(skSlot(p, c, u));
        storeTile(c_m0, c_n0, c_bi);
        if (tid == 0) p.counters[u] = 0;  // ready for the next launch
      }
    }
#pragma unroll
    for (int i = 0; i < kTP / 2; ++i)
#pragma unroll
      for (int j = 0; j < kTD; ++j) acc[i][j] = make_float2(0.0F, 0.0F);
  }
}

}  // namespace sgblas::kern

#endif  // SGBLAS_B200_SGEMM_TILE_CUH_
