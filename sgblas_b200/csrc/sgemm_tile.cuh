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
// to both lanes. P must sit in shared memory as [k][x] (x contiguous); D may be
// [k][x] or [x][k].
//
// Shared-memory tile layouts (a pipeline stage holds one P and one D tile):
//   kXK : [BK][BX] floats, x contiguous -- what TMA writes when x is the
//         contiguous global dimension.
//   kKX : [BX][BK] floats, k contiguous, 64-byte rows with the TMA 64B swizzle
//         (16-byte chunk index ^= (row >> 1) & 3).
//
// CTA: three warpgroups, one CTA per SM.
//   - Warpgroups 0-1 (256 threads, 8 warps) compute a 256 (P) x 128 (D) tile;
//     each thread owns a 16 (P) x 8 (D) block of C (64 FFMA2 per k step against
//     4+2 shared loads). Warps form 2 (P) x 4 (D); lane bits lp = lane % 8,
//     ld = lane / 8.
//       P coordinates: 128*wp + 4*lp + {0..3} + 32*q, q = 0..3.
//       D coordinates ([k][x] tile): 32*wd + 4*ld + {0..3} + {0, 16}.
//   - Warpgroup 2 (128 threads) is the producer: one thread issues the TMA
//     tile loads (or all 128 issue cp.async copies), and all 128 transpose
//     [x][k] broadcast tiles into [k][x] buffers. It gives registers to the
//     compute warpgroups (setmaxnreg), so that those keep 232.
//   Producer and consumers meet only at mbarriers (stage full/empty,
//   transposed buffer full/empty), so no warp ever waits on a CTA-wide
//   barrier inside the main loop.
#ifndef SGBLAS_B200_SGEMM_TILE_CUH_
#define SGBLAS_B200_SGEMM_TILE_CUH_

#include "ptx.cuh"

#include <cstddef>
#include <cstdint>

namespace sgblas::kern {

constexpr int kBP = 256;   // pair-operand tile extent
constexpr int kBD = 128;   // broadcast-operand tile extent
constexpr int kBK = 16;    // k slice per pipeline stage
constexpr int kStages = 6;
constexpr int kTransBufs = 3;   // ring of transposed [k][x] broadcast tiles
constexpr int kTP = 16;         // pair-operand elements per thread
constexpr int kTD = 8;          // broadcast-operand elements per thread
constexpr int kWarpsP = kBP / (8 * kTP);   // warps along P (8 lanes x kTP each)
constexpr int kWarpsD = kBD / 32;          // warps along D (4 lanes x 8 each)
constexpr int kThreads = 32 * kWarpsP * kWarpsD;   // compute threads (256)
constexpr int kConsumerWarps = kThreads / 32;
constexpr int kProducerThreads = 128;               // one warpgroup
constexpr int kBlockThreads = kThreads + kProducerThreads;
// Register split: the block is launched with kLaunchRegs per thread (what
// __launch_bounds__(384, 1) leaves ptxas); setmaxnreg then moves registers
// from the producer warpgroup to the compute warpgroups.
constexpr int kLaunchRegs = 168;
constexpr int kConsumerRegs = 232;
constexpr int kProducerRegs = 40;
static_assert(kThreads * kConsumerRegs + kProducerThreads * kProducerRegs <=
                  kBlockThreads * kLaunchRegs,
              "register split exceeds the launch allocation");
constexpr int kSlotFloat4 = kTP * kTD / 4;  // float4s per thread in a partial slot
constexpr int kPairFloats = kBP * kBK;
constexpr int kDupFloats = kBD * kBK;
constexpr int kPairBytes = kPairFloats * 4;   // 16 KiB
constexpr int kDupBytes = kDupFloats * 4;     // 8 KiB
constexpr int kStageBytes = kPairBytes + kDupBytes;
constexpr int kTransBytes = kTransBufs * kDupBytes;
constexpr int kBarrierBytes = 8 * (2 * kStages + 2 * kTransBufs);
constexpr int kSmemAlign = 1024;
constexpr int kSmemBytes = kStages * kStageBytes + kTransBytes + kBarrierBytes + kSmemAlign;

enum class Beta { kZero, kOne, kGeneral };
enum class Src { kTma, kCopy };
enum class Layout { kXK, kKX };

struct GemmParams {
  CUtensorMap tma_a;  // valid when the kernel stages tiles with TMA
  CUtensorMap tma_b;
  const float *a;
  const float *b;
  float *c;
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
  float4 *ws;         // 2 * grid partial-tile slots of kThreads * kSlotFloat4 float4
  int *counters;      // sk_tiles arrival counters, zero between launches
};

// One unit of a CTA's work: k iterations [kb, ke) of tile `tile`.
struct Item {
  int tile, kb, ke;
};


__device__ __forceinline__ int skBegin(const GemmParams &p, int c) {
  return c * p.sk_q + min(c, p.sk_r);
}

// The CTA owning stream-K iteration x (inverse of skBegin).
__device__ __forceinline__ int skOwner(const GemmParams &p, int x) {
  const int head = p.sk_r * (p.sk_q + 1);
  return x < head ? x / (p.sk_q + 1) : p.sk_r + (x - head) / p.sk_q;
}

__device__ __forceinline__ int dpItems(const GemmParams &p, int c) {
  return c < p.dp_tiles ? (p.dp_tiles - 1 - c) / p.grid + 1 : 0;
}

__device__ __forceinline__ int numItems(const GemmParams &p, int c) {
  int n = dpItems(p, c);
  if (p.sk_tiles > 0) {
    const int s = skBegin(p, c), e = skBegin(p, c + 1);
    if (e > s) n += (e - 1) / p.kiters - s / p.kiters + 1;
  }
  return n;
}

__device__ __forceinline__ Item itemAt(const GemmParams &p, int c, int idx) {
  const int ndp = dpItems(p, c);
  if (idx < ndp) return {c + idx * p.grid, 0, p.kiters};
  const int s = skBegin(p, c), e = skBegin(p, c + 1);
  const int u = s / p.kiters + (idx - ndp);
  const int base = u * p.kiters;
  return {p.dp_tiles + u, max(s, base) - base, min(e, base + p.kiters) - base};
}

// Workspace slot of CTA c's piece of stream-K tile u: slot 2c holds the piece
// of the first tile c touches, slot 2c+1 the piece of its last one.
__device__ __forceinline__ int skSlot(const GemmParams &p, int c, int u) {
  return 2 * c + (u == skBegin(p, c) / p.kiters ? 0 : 1);
}

// Byte offset of element (x, k) inside a kKX tile.
__device__ __forceinline__ uint32_t kxOffset(int x, int k) {
  return static_cast<uint32_t>(x * 64 + ((((k >> 2) ^ (x >> 1)) & 3) << 4) + ((k & 3) << 2));
}

// Which operand plays which role, and the tile shape that follows.
template <bool kTA, bool kTB, Src kSrc>
struct Plan {
  // Shared-memory layout of each operand. The cp.async path may transpose A
  // while staging it, so it always stages A as [k][m].
  static constexpr Layout kA = (kSrc == Src::kTma && kTA) ? Layout::kKX : Layout::kXK;
  static constexpr Layout kB = kTB ? Layout::kXK : Layout::kKX;
  static constexpr bool kPairIsA = (kA == Layout::kXK);
  static constexpr Layout kD = kPairIsA ? kB : kA;
  static_assert(kPairIsA || kB == Layout::kXK, "one operand must be staged as [k][x]");
  // A broadcast tile staged as [x][k] is transposed into [k][x] before use:
  // broadcast reads from [x][k] rows measured ~10% slower in the inner loop.
  static constexpr bool kTransD = (kD == Layout::kKX);
  static constexpr Layout kCompD = Layout::kXK;
  static constexpr int kBM = kPairIsA ? kBP : kBD;
  static constexpr int kBN = kPairIsA ? kBD : kBP;
};

// Tile index -> (tile_m, tile_n): groups of group_m tile rows are walked
// column by column so that concurrently running CTAs share panels in L2.
__device__ __forceinline__ void rasterTile(const GemmParams &p, int t, int *tm, int *tn) {
  const int per_group = p.group_m * p.tiles_n;
  const int group = t / per_group;
  const int first = group * p.group_m;
  const int rows = min(p.tiles_m - first, p.group_m);
  const int in = t - group * per_group;
  *tm = first + in % rows;
  *tn = in / rows;
}

// ---- cp.async staging (any alignment, any leading dimension, tails) --------
// Writes the layouts the kernel reads: A as [k][m] (P, kBP wide), B as [k][n]
// or swizzled [n][k] (D, kBD wide), zero-filled outside the matrix. Global
// reads are coalesced along each operand's contiguous dimension.
template <bool kTA, bool kTB>
__device__ __forceinline__ void copyTile(const GemmParams &p, float *sa, float *sb, int m0, int n0,
                                         int k0, int tid) {
  constexpr int kN = kProducerThreads;
#pragma unroll 4
  for (int r = 0; r < kPairFloats / kN; ++r) {
    const int e = tid + r * kN;
    const int mm = kTA ? e / kBK : e % kBP;
    const int kk = kTA ? e % kBK : e / kBP;
    const int gm = m0 + mm, gk = k0 + kk;
    const bool ok = gm < p.m && gk < p.k;
    const float *src = p.a;
    if (ok) {
      src = kTA ? p.a + static_cast<size_t>(gk) + static_cast<size_t>(gm) * p.lda
                : p.a + static_cast<size_t>(gm) + static_cast<size_t>(gk) * p.lda;
    }
    cpAsync4(sa + kk * kBP + mm, src, ok ? 4u : 0u);
  }
#pragma unroll 4
  for (int r = 0; r < kDupFloats / kN; ++r) {
    const int e = tid + r * kN;
    const int nn = kTB ? e % kBD : e / kBK;
    const int kk = kTB ? e / kBD : e % kBK;
    const int gn = n0 + nn, gk = k0 + kk;
    const bool ok = gn < p.n && gk < p.k;
    const float *src = p.b;
    if (ok) {
      src = kTB ? p.b + static_cast<size_t>(gn) + static_cast<size_t>(gk) * p.ldb
                : p.b + static_cast<size_t>(gk) + static_cast<size_t>(gn) * p.ldb;
    }
    float *dst = kTB ? sb + kk * kBD + nn
                     : reinterpret_cast<float *>(reinterpret_cast<char *>(sb) + kxOffset(nn, kk));
    cpAsync4(dst, src, ok ? 4u : 0u);
  }
}

// Per-thread addressing of the broadcast tile.
struct DupAddr {
  uint32_t base;        // kXK: float index of the first column; kKX: byte offset of row 0
  uint32_t chunk[4];    // kKX: swizzled byte offset of each 16-byte k chunk
};

// [x][k] broadcast tile (64-byte swizzled rows) -> [k][x] (kBD floats per k),
// by the producer warpgroup: thread t moves row t. A warp reads 32
// consecutive rows at one chunk -- conflict-free thanks to the swizzle -- and
// writes 32 consecutive floats per k.
__device__ __forceinline__ void transposeDup(const float *src, float *dst, int tid) {
  static_assert(kProducerThreads == kBD && kBK == 16, "one row per producer thread");
  const char *row = reinterpret_cast<const char *>(src) + tid * 64;
  const int phase = (tid >> 1) & 3;
  float *d = dst + tid;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 v = *reinterpret_cast<const float4 *>(row + ((c ^ phase) << 4));
    d[(4 * c + 0) * kBD] = v.x;
    d[(4 * c + 1) * kBD] = v.y;
    d[(4 * c + 2) * kBD] = v.z;
    d[(4 * c + 3) * kBD] = v.w;
  }
}

// ---- the FFMA2 micro-kernel over one BK slice ------------------------------
template <Layout kD>
__device__ __forceinline__ void computeStage(const float *sp, const float *sd, int p_base,
                                             const DupAddr &da, float2 (&acc)[kTP / 2][kTD]) {
#pragma unroll
  for (int k = 0; k < kBK; k += 2) {
    float dv[2][kTD];
    if constexpr (kD == Layout::kXK) {
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const float4 d0 = *reinterpret_cast<const float4 *>(sd + (k + kk) * kBD + da.base);
        const float4 d1 = *reinterpret_cast<const float4 *>(sd + (k + kk) * kBD + da.base + 16);
        dv[kk][0] = d0.x; dv[kk][1] = d0.y; dv[kk][2] = d0.z; dv[kk][3] = d0.w;
        dv[kk][4] = d1.x; dv[kk][5] = d1.y; dv[kk][6] = d1.z; dv[kk][7] = d1.w;
      }
    } else {
      const char *row0 = reinterpret_cast<const char *>(sd) + da.base + da.chunk[k >> 2] +
                         ((k & 3) << 2);
#pragma unroll
      for (int j = 0; j < kTD; ++j) {
        const float2 v = *reinterpret_cast<const float2 *>(row0 + 512 * j);
        dv[0][j] = v.x;
        dv[1][j] = v.y;
      }
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
//   empty[s]    the 8 compute warps are done with stage s's pair tile
//   tfull[t]    transposed broadcast buffer t is written (128 producer threads)
//   tempty[t]   the 8 compute warps are done with buffer t
// A wait that times out raises the device error flag; from then on that
// thread skips its waits (results are garbage and flagged) but still runs
// every loop to its end, so that no thread is left behind at a barrier.
template <bool kTA, bool kTB, Beta kBeta, Src kSrc>
__global__ void __launch_bounds__(kBlockThreads, 1)
    sgemmKernel(const __grid_constant__ GemmParams p) {
  using P = Plan<kTA, kTB, kSrc>;
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
  auto tbuf = [&](int i) {
    return reinterpret_cast<float *>(smem + kStages * kStageBytes + i * kDupBytes);
  };
  // Stage s: the pair tile at offset 0, the broadcast tile after it.
  auto stageP = [&](int s) { return reinterpret_cast<float *>(smem + s * kStageBytes); };
  auto stageD = [&](int s) {
    return reinterpret_cast<float *>(smem + s * kStageBytes + kPairBytes);
  };
  auto stageA = [&](int s) { return P::kPairIsA ? stageP(s) : stageD(s); };
  auto stageB = [&](int s) { return P::kPairIsA ? stageD(s) : stageP(s); };
  auto origin = [&](int tile, int *m0, int *n0) {
    int tm, tn;
    rasterTile(p, tile, &tm, &tn);
    *m0 = tm * P::kBM;
    *n0 = tn * P::kBN;
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
      mbarInit(&tfull[t], kProducerThreads);
      mbarInit(&tempty[t], kConsumerWarps);
    }
    fenceBarrierInit();
  }
  __syncthreads();

  // ======================= producer warpgroup ===============================
  if (tid >= kThreads) {
    regDealloc<kProducerRegs>();
    const int pt = tid - kThreads;
    bool ok = true;
    auto wait = [&](uint64_t *bar, int parity) {
      if (ok) ok = mbarWait(bar, static_cast<uint32_t>(parity), p.err);
    };
    int idx = 0, kt, ke, m0, n0;
    {
      const Item it = itemAt(p, cta, 0);
      kt = it.kb;
      ke = it.ke;
      origin(it.tile, &m0, &n0);
    }
    // Transposes trail the loads by kLag iterations: far enough behind for the
    // data to have landed, early enough to stay ahead of the compute warps.
    constexpr int kLag = P::kTransD ? kStages - 2 : 0;
    for (int i = 0; i < total + kLag; ++i) {
      if (i < total) {
        const int s = i % kStages;
        const int k0 = kt * kBK;
        if constexpr (kSrc == Src::kTma) {
          if (pt == 0) {
            if (i >= kStages) wait(&empty[s], (i / kStages - 1) & 1);
            mbarArriveExpectTx(&full[s], kStageBytes);
            if (P::kA == Layout::kXK) tmaLoad2d(stageA(s), &p.tma_a, &full[s], m0, k0);
            else tmaLoad2d(stageA(s), &p.tma_a, &full[s], k0, m0);
            if (P::kB == Layout::kXK) tmaLoad2d(stageB(s), &p.tma_b, &full[s], n0, k0);
            else tmaLoad2d(stageB(s), &p.tma_b, &full[s], k0, n0);
          }
        } else {
          if (i >= kStages) wait(&empty[s], (i / kStages - 1) & 1);
          copyTile<kTA, kTB>(p, stageA(s), stageB(s), m0, n0, k0, pt);
          cpAsyncArrive(&full[s]);
        }
        if (++kt == ke && ++idx < nitems) {
          const Item it = itemAt(p, cta, idx);
          kt = it.kb;
          ke = it.ke;
          origin(it.tile, &m0, &n0);
        }
      }
      if constexpr (P::kTransD) {
        const int j = i - kLag;
        if (j >= 0) {
          const int t = j % kTransBufs;
          wait(&full[j % kStages], (j / kStages) & 1);
          if (j >= kTransBufs) wait(&tempty[t], (j / kTransBufs - 1) & 1);
          transposeDup(stageD(j % kStages), tbuf(t), pt);
          mbarArrive(&tfull[t]);
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
  DupAddr da;
  const int d_row0 = wd * 32 + ld * 4;  // [k][x] broadcast tile: first column
  da.base = static_cast<uint32_t>(d_row0);
#pragma unroll
  for (int c = 0; c < 4; ++c) da.chunk[c] = 0;
  static_assert(P::kCompD == Layout::kXK, "compute reads [k][x] broadcast tiles");
  auto dCoord = [&](int j) { return d_row0 + (j & 3) + 16 * (j >> 2); };
  auto pCoord = [&](int i) { return p_base + (i & 3) + 32 * (i >> 2); };
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
  // C = alpha * acc (+ beta * C) for the tile at (m0, n0).
  auto storeTile = [&](int m0, int n0) {
    if constexpr (P::kPairIsA) {
      const bool vec = m0 + P::kBM <= p.m && n0 + P::kBN <= p.n && (p.ldc % 4 == 0) &&
                       (reinterpret_cast<uintptr_t>(p.c) % 16 == 0);
      if (vec) {
#pragma unroll
        for (int j = 0; j < kTD; ++j) {
          float *col = p.c + static_cast<size_t>(n0 + dCoord(j)) * p.ldc + m0 + p_base;
#pragma unroll
          for (int q = 0; q < kTP / 4; ++q) {
            const float2 lo = acc[2 * q][j], hi = acc[2 * q + 1][j];
            float4 cv = make_float4(0.0F, 0.0F, 0.0F, 0.0F);
            if constexpr (kBeta != Beta::kZero) cv = *reinterpret_cast<const float4 *>(col + 32 * q);
            float4 out;
            out.x = epilogueValue<kBeta>(lo.x, alpha, beta, cv.x);
            out.y = epilogueValue<kBeta>(lo.y, alpha, beta, cv.y);
            out.z = epilogueValue<kBeta>(hi.x, alpha, beta, cv.z);
            out.w = epilogueValue<kBeta>(hi.y, alpha, beta, cv.w);
            *reinterpret_cast<float4 *>(col + 32 * q) = out;
          }
        }
        return;
      }
    }
#pragma unroll
    for (int j = 0; j < kTD; ++j) {
#pragma unroll
      for (int i = 0; i < kTP; ++i) {
        const int row = P::kPairIsA ? m0 + pCoord(i) : m0 + dCoord(j);
        const int col = P::kPairIsA ? n0 + dCoord(j) : n0 + pCoord(i);
        if (row < p.m && col < p.n) {
          float *cp = p.c + static_cast<size_t>(col) * p.ldc + row;
          const float a = (i & 1) ? acc[i >> 1][j].y : acc[i >> 1][j].x;
          const float cv = kBeta == Beta::kZero ? 0.0F : *cp;
          *cp = epilogueValue<kBeta>(a, alpha, beta, cv);
        }
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

  int c_idx = 0;
  int c_kt, c_ke;
  {
    const Item it = itemAt(p, cta, 0);
    c_kt = it.kb;
    c_ke = it.ke;
  }
  for (int g = 0; g < total; ++g) {
    const int s = g % kStages;
    const int t = g % kTransBufs;
    wait(&full[s], (g / kStages) & 1);
    if constexpr (P::kTransD) wait(&tfull[t], (g / kTransBufs) & 1);
    computeStage<P::kCompD>(stageP(s), P::kTransD ? tbuf(t) : stageD(s), p_base, da, acc);
    __syncwarp();
    if (lane == 0) {
      mbarArrive(&empty[s]);
      if constexpr (P::kTransD) mbarArrive(&tempty[t]);
    }

    if (++c_kt == c_ke) {
      const Item c_item = itemAt(p, cta, c_idx);
      int c_m0, c_n0;
      origin(c_item.tile, &c_m0, &c_n0);
      if (c_item.kb == 0 && c_item.ke == p.kiters) {
        storeTile(c_m0, c_n0);
      } else {
        // Stream-K piece: publish, count the arrival, and let the last
        // arriving piece reduce all pieces in piece order.
        const int u = c_item.tile - p.dp_tiles;
        const int first = skOwner(p, u * p.kiters);
        const int last = skOwner(p, (u + 1) * p.kiters - 1);
        publish(skSlot(p, cta, u));
        __threadfence();
        namedBarrier<1, kThreads>();
        if (tid == 0) last_arrival = atomicAdd(p.counters + u, 1) == last - first;
        namedBarrier<1, kThreads>();
        if (last_arrival) {
          __threadfence();
#pragma unroll
          for (int i = 0; i < kTP / 2; ++i)
#pragma unroll
            for (int j = 0; j < kTD; ++j) acc[i][j] = make_float2(0.0F, 0.0F);
#pragma unroll 1
          for (int c = first; c <= last; ++c) gather(skSlot(p, c, u));
          storeTile(c_m0, c_n0);
          if (tid == 0) p.counters[u] = 0;  // ready for the next launch
        }
      }
#pragma unroll
      for (int i = 0; i < kTP / 2; ++i)
#pragma unroll
        for (int j = 0; j < kTD; ++j) acc[i][j] = make_float2(0.0F, 0.0F);
      if (++c_idx < nitems) {
        const Item it = itemAt(p, cta, c_idx);
        c_kt = it.kb;
        c_ke = it.ke;
      }
    }
  }
}

}  // namespace sgblas::kern

#endif  // SGBLAS_B200_SGEMM_TILE_CUH_
