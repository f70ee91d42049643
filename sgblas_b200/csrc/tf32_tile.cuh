// The TF32 lane (math mode SGBLAS_MATH_TF32): C = alpha * op(A) * op(B) +
// beta * C on the 5th-generation tensor cores. Inputs are read as TF32 (the
// tensor core uses the top 19 bits of each FP32 word: sign, 8-bit exponent,
// 10-bit mantissa), products are accumulated in FP32 in tensor memory. This
// is outside the strict-FP32 contract of the default math mode and is only
// used when the caller selects SGBLAS_MATH_TF32.
//
// One persistent CTA per SM walks 128 x N tiles of C (N = 256, or 128 or 64
// when that fills the GPU better). Warp roles:
//   warp 0   TMA producer: 128x32 A and Nx32 B tiles into a stage ring,
//            128-byte swizzled (16-byte atoms for K-major tiles, 32-byte
//            atoms for MN-major ones: the canonical UMMA layouts);
//   warp 1   MMA issuer: per 32-deep k slice, four tcgen05.mma kind::tf32
//            (M = 128, N, K = 8) into one of two TMEM accumulators;
//   warp 2   allocates / frees the TMEM columns (2 x N);
//   warps 4-7 epilogue: TMEM -> registers (tcgen05.ld, one row of C per
//            thread) -> alpha/beta -> C, overlapping the next tile's MMAs.
// Operands may be K-major (k contiguous) or MN-major (m or n contiguous) in
// global memory; both are staged as TMA writes them and described to the
// tensor core accordingly, so nothing is transposed.
//
// Synchronisation (mbarriers, all waits bounded):
//   full[s]      stage s loaded (TMA transaction bytes)
//   empty[s]     the MMAs reading stage s completed (tcgen05.commit)
//   acc_full[b]  accumulator b holds a finished tile (tcgen05.commit)
//   acc_empty[b] the 128 epilogue threads have read accumulator b
#ifndef SGBLAS_B200_TF32_TILE_CUH_
#define SGBLAS_B200_TF32_TILE_CUH_

#include "ptx.cuh"
#include "sgemm_tile.cuh"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace sgblas::kern::tf32 {

constexpr int kBM = 128;             // UMMA M
constexpr int kBK = 32;              // k per stage: one 128-byte swizzle row of FP32
constexpr int kMmaK = 8;             // k per tcgen05.mma kind::tf32
constexpr int kAccums = 2;           // TMEM accumulators (double buffered)
constexpr int kABytes = kBM * kBK * 4;        // 16 KiB
constexpr int kChunkBytes = 32 * kBK * 4;     // one 32-wide MN chunk of an MN-major tile (4 KiB)
constexpr int kThreads = 256;
constexpr int kEpilogueWarp0 = 4;
// Split-tile fix-up: 32-column chunks summed per pass (two pieces are loaded
// per round trip to L2 in each pass).
constexpr int kGatherChunks = 2;

// Tile width N (UMMA N): 256, 128 where the 256-wide tiles would leave a
// poorly filled last wave, or 64 where even 128-wide tiles would leave over
// half the SMs without one. The stage ring fills about 192 KiB each way.
template <int kBN_>
struct Cfg {
  static constexpr int kBN = kBN_;
  static constexpr int kBBytes = kBN * kBK * 4;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = kBN == 256 ? 4 : kBN == 128 ? 6 : 8;
  static constexpr int kTmemColumns = kAccums * kBN;   // 512 or 256
  static constexpr int kBarrierBytes = 8 * (2 * kStages + 2 * kAccums);
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarrierBytes + 1024;
  static_assert(kBN == 64 || kBN == 128 || kBN == 256, "tile width");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
};

struct Tf32Params {
  // 3-D tensor maps, the third coordinate selecting the matrix of a strided
  // batch. A: K-major (k, m) boxes 32 x 128; MN-major (m, k) boxes 32 x 32.
  // B: K-major (k, n) boxes 32 x N; MN-major (n, k) boxes 32 x 32.
  CUtensorMap tma_a;
  CUtensorMap tma_b;
  float *c;
  long long stride_c;   // C of matrix i at c + i * stride_c; tiles are batch-major
  int batch;
  int m, n, k, ldc;
  float alpha, beta;
  int tiles_m, tiles_n, kiters, group_m;
  unsigned *err;
  // Persistent schedule, as in the FP32 kernel: whole tiles [0, dp_tiles)
  // round-robin, then tiles [dp_tiles, dp_tiles + sk_tiles) split by k slices
  // over all CTAs (stream-K), pieces summed in order by the last arriver.
  int grid, dp_tiles, sk_tiles, sk_q, sk_r;
  float *ws;          // 2 * grid piece slots of 128 x N floats
  unsigned long long *counters;   // sk_tiles arrival counters (see arriveCounter)
  unsigned epoch;                 // this launch's counter epoch (non-zero)
};

// Shared-memory matrix descriptor (tcgen05), version 1.
// K-major (128-byte swizzle, 16-byte atoms): rows of 128 bytes (32 k), 8-row
//   groups 1024 bytes apart (SBO); LBO unused.
// MN-major (128-byte swizzle with 32-byte atoms, the only MN-major layout
//   TF32 operands support): 128-byte rows of 32 consecutive m (or n) per k,
//   4-row groups 512 bytes apart (SBO), 32-wide MN chunks kChunkBytes apart
//   (LBO).
template <bool kMN>
__device__ __forceinline__ uint64_t smemDesc(uint32_t addr) {
  constexpr uint32_t lbo = kMN ? kChunkBytes : 16;
  constexpr uint32_t sbo = kMN ? 512 : 1024;
  constexpr uint64_t layout = kMN ? 1 : 2;   // SWIZZLE_128B_BASE32B : SWIZZLE_128B
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;   // version
  d |= layout << 61;
  return d;
}

// Instruction descriptor: FP32 accumulator, TF32 A and B, majors, N, M.
template <int kBN, bool kAMN, bool kBMN>
__host__ __device__ constexpr uint32_t instrDesc() {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(kAMN) << 15) |
         (static_cast<uint32_t>(kBMN) << 16) | (static_cast<uint32_t>(kBN >> 3) << 17) |
         (static_cast<uint32_t>(kBM >> 4) << 24);
}

// kBatch: tiles of a strided batch (p.batch > 1); the single-matrix
// instantiation keeps the matrix index out of the epilogue, whose split-tile
// fix-up runs at the edge of the register budget.
template <int kBN, bool kAMN, bool kBMN, Beta kBeta, bool kBatch>
__global__ void __launch_bounds__(kThreads, 1) tf32Kernel(const __grid_constant__ Tf32Params p) {
  using G = Cfg<kBN>;
  constexpr int kStages = G::kStages;
  constexpr int kStageBytes = G::kStageBytes;
  constexpr int kTmemColumns = G::kTmemColumns;
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint32_t tmem_base_slot;
  unsigned char *smem = smem_raw + ((1024 - (smemAddr(smem_raw) & 1023)) & 1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes);
  uint64_t *empty = full + kStages;
  uint64_t *acc_full = empty + kStages;
  uint64_t *acc_empty = acc_full + kAccums;

  __shared__ int last_arrival;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int cta = blockIdx.x;
  const int nitems = numItems(p, cta);
  if (nitems == 0) return;  // whole CTA, before any barrier

  if (threadIdx.x == 0) {
    prefetchTensorMap(&p.tma_a);
    prefetchTensorMap(&p.tma_b);
    for (int s = 0; s < kStages; ++s) {
      mbarInit(&full[s], 1);
      mbarInit(&empty[s], 1);
    }
    for (int b = 0; b < kAccums; ++b) {
      mbarInit(&acc_full[b], 1);
      mbarInit(&acc_empty[b], 32 * (kThreads / 32 - kEpilogueWarp0));
    }
    fenceBarrierInit();
  }
  if (warp == 2) {
    tmemAlloc(&tmem_base_slot, kTmemColumns);
    tmemRelinquish();
  }
  tcgenFenceBefore();
  __syncthreads();
  tcgenFenceAfter();
  const uint32_t tmem_base = tmem_base_slot;
  gridDependencyWait();
  allowDependentLaunch();

  const int tiles_per_matrix = p.tiles_m * p.tiles_n;
  auto tileOrigin = [&](int tile, int *m0, int *n0, int *bi) {
    int tm, tn;
    *bi = kBatch ? tile / tiles_per_matrix : 0;
    rasterTile(p, tile - *bi * tiles_per_matrix, &tm, &tn);
    *m0 = tm * kBM;
    *n0 = tn * kBN;
  };
  bool ok = true;
  auto wait = [&](uint64_t *bar, int parity) {
    if (ok) ok = mbarWait(bar, static_cast<uint32_t>(parity), p.err);
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int g = 0;  // k slices issued so far
      for (int i = 0; i < nitems; ++i) {
        const Item it = itemAt(p, cta, i);
        int m0, n0, bi;
        tileOrigin(it.tile, &m0, &n0, &bi);
        for (int kb = it.kb; kb < it.ke; ++kb, ++g) {
          const int s = g % kStages;
          if (g >= kStages) wait(&empty[s], (g / kStages - 1) & 1);
          unsigned char *sa = smem + s * kStageBytes;
          unsigned char *sb = sa + kABytes;
          const int k0 = kb * kBK;
          mbarArriveExpectTx(&full[s], kStageBytes);
          if constexpr (kAMN) {
            for (int j = 0; j < kBM / 32; ++j)
              tmaLoad3d(sa + j * kChunkBytes, &p.tma_a, &full[s], m0 + 32 * j, k0, bi);
          } else {
            tmaLoad3d(sa, &p.tma_a, &full[s], k0, m0, bi);
          }
          if constexpr (kBMN) {
            for (int j = 0; j < kBN / 32; ++j)
              tmaLoad3d(sb + j * kChunkBytes, &p.tma_b, &full[s], n0 + 32 * j, k0, bi);
          } else {
            tmaLoad3d(sb, &p.tma_b, &full[s], k0, n0, bi);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = instrDesc<kBN, kAMN, kBMN>();
      int g = 0;
      for (int i = 0; i < nitems; ++i) {
        const Item it = itemAt(p, cta, i);
        const int b = i % kAccums;
        if (i >= kAccums) wait(&acc_empty[b], (i / kAccums - 1) & 1);
        tcgenFenceAfter();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * kBN);
        for (int kb = it.kb; kb < it.ke; ++kb, ++g) {
          const int s = g % kStages;
          wait(&full[s], (g / kStages) & 1);
          tcgenFenceAfter();
          const uint32_t sa = smemAddr(smem + s * kStageBytes);
          const uint32_t sb = sa + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / kMmaK; ++kk) {
            // K-major: the next 8 k are 32 bytes further along each row;
            // MN-major: the next 8 k rows are one 1024-byte group further.
            const uint32_t koff = kAMN ? kk * 1024u : kk * 32u;
            const uint32_t koff_b = kBMN ? kk * 1024u : kk * 32u;
            const uint64_t ad = smemDesc<kAMN>(sa + koff);
            const uint64_t bd = smemDesc<kBMN>(sb + koff_b);
            mmaTf32(d_tmem, ad, bd, idesc, kb > it.kb || kk > 0);
          }
          mmaCommit(&empty[s]);  // the stage is free once these MMAs completed
        }
        mmaCommit(&acc_full[b]);
      }
    }
  } else if (warp >= kEpilogueWarp0) {
    // ---------------- epilogue ----------------
    const int quarter = warp % 4;   // TMEM lanes [32*quarter, 32*quarter + 32)
    const int r = quarter * 32 + lane;   // this thread's row of the tile
    const int etid = threadIdx.x - 32 * kEpilogueWarp0;   // 0..127
    constexpr size_t kSlotFloats = static_cast<size_t>(kBM) * kBN;
    // C = alpha * acc + beta * C for 32 columns of this thread's row.
    auto storeChunk = [&](float *cbase, int row, int col0, const float (&acc)[32]) {
      const bool row_ok = row < p.m;
      float *cp = cbase + static_cast<size_t>(col0) * p.ldc + row;
      float cv[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        cv[j] = 0.0F;
        if constexpr (kBeta != Beta::kZero)
          if (row_ok && col0 + j < p.n) cv[j] = cp[static_cast<size_t>(j) * p.ldc];
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (row_ok && col0 + j < p.n)
          cp[static_cast<size_t>(j) * p.ldc] = epilogueValue<kBeta>(acc[j], p.alpha, p.beta, cv[j]);
      }
    };
    for (int i = 0; i < nitems; ++i) {
      const Item it = itemAt(p, cta, i);
      const int b = i % kAccums;
      int m0, n0, bi;
      tileOrigin(it.tile, &m0, &n0, &bi);
      wait(&acc_full[b], (i / kAccums) & 1);
      tcgenFenceAfter();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(b * kBN);
      if (it.kb == 0 && it.ke == p.kiters) {
#pragma unroll 1
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t v[32];
          tmemLoad32(taddr + c * 32, v);
          float acc[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] = __uint_as_float(v[j]);
          storeChunk(kBatch ? p.c + bi * p.stride_c : p.c, m0 + r, n0 + c * 32, acc);
        }
        tcgenFenceBefore();
        mbarArrive(&acc_empty[b]);
        continue;
      }
      // Stream-K piece: publish it, free the accumulator, count the arrival;
      // the last arriving piece sums every piece in piece order and writes C.
      // Slot layout: float4 q of chunk c of thread r at [(c*8 + q)*128 + r],
      // so each warp access is 512 contiguous bytes.
      const int u = it.tile - p.dp_tiles;
      float4 *slot = reinterpret_cast<float4 *>(p.ws) +
                     static_cast<size_t>(skSlot(p, cta, u)) * (kSlotFloats / 4);
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t v[32];
        tmemLoad32(taddr + c * 32, v);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          __stcg(slot + (c * 8 + q) * kBM + r,
                 make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                             __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3])));
      }
      tcgenFenceBefore();
      mbarArrive(&acc_empty[b]);
      const int first = skOwner(p, u * p.kiters);
      const int last = skOwner(p, (u + 1) * p.kiters - 1);
      __threadfence();
      namedBarrier<1, 128>();
      if (etid == 0)
        last_arrival = arriveCounter(p.counters + u, p.epoch, p.err) ==
                       static_cast<unsigned>(last - first + 1);
      namedBarrier<1, 128>();
      if (last_arrival) {
        __threadfence();
        auto piece = [&](int pc) {
          return reinterpret_cast<const float4 *>(p.ws) +
                 static_cast<size_t>(skSlot(p, pc, u)) * (kSlotFloats / 4);
        };
        // kGatherChunks chunks per pass, two pieces per round trip to L2
        // (the sum order per element stays piece order).
#pragma unroll 1
        for (int c = 0; c < kBN / 32; c += kGatherChunks) {
          float4 acc[8 * kGatherChunks];
#pragma unroll
          for (int e = 0; e < 8 * kGatherChunks; ++e) acc[e] = make_float4(0.0F, 0.0F, 0.0F, 0.0F);
#pragma unroll 1
          for (int pc = first; pc <= last; pc += 2) {
            const bool two = pc + 1 <= last;
            const float4 *s0 = piece(pc) + c * 8 * kBM + r;
            const float4 *s1 = piece(two ? pc + 1 : pc) + c * 8 * kBM + r;
            float4 v0[8 * kGatherChunks], v1[8 * kGatherChunks];
#pragma unroll
            for (int e = 0; e < 8 * kGatherChunks; ++e) {
              v0[e] = __ldcg(s0 + e * kBM);
              v1[e] = two ? __ldcg(s1 + e * kBM) : make_float4(0.0F, 0.0F, 0.0F, 0.0F);
            }
#pragma unroll
            for (int e = 0; e < 8 * kGatherChunks; ++e) {
              acc[e].x += v0[e].x;
              acc[e].y += v0[e].y;
              acc[e].z += v0[e].z;
              acc[e].w += v0[e].w;
              if (two) {
                acc[e].x += v1[e].x;
                acc[e].y += v1[e].y;
                acc[e].z += v1[e].z;
                acc[e].w += v1[e].w;
              }
            }
          }
#pragma unroll
          for (int h = 0; h < kGatherChunks; ++h) {
            float out[32];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              out[4 * q] = acc[h * 8 + q].x;
              out[4 * q + 1] = acc[h * 8 + q].y;
              out[4 * q + 2] = acc[h * 8 + q].z;
              out[4 * q + 3] = acc[h * 8 + q].w;
            }
            storeChunk(kBatch ? p.c + bi * p.stride_c : p.c, m0 + r, n0 + (c + h) * 32, out);
          }
        }
        if (etid == 0) p.counters[u] = 0;  // ready for the next launch
      }
      namedBarrier<1, 128>();   // last_arrival is reused by the next piece
    }
  }

  tcgenFenceBefore();
  __syncthreads();
  if (warp == 2) {
    tcgenFenceAfter();
    tmemDealloc(tmem_base, kTmemColumns);
  }
}

// ---- pair-CTA variant: cta_group::2, 256 x 256 tiles ---------------------------
// Two CTAs of a cluster share each 256 x 256 tile: CTA r (r = 0, 1) loads rows
// [128 r, 128 r + 128) of the A tile and columns [128 r, 128 r + 128) of the B
// tile into its own shared memory; the even CTA issues tcgen05.mma
// cta_group::2 (M = 256, N = 256, K = 8), which reads A and B from both CTAs
// and accumulates rows [128 r, 128 r + 128) in CTA r's TMEM. Per CTA this
// moves half the B operand per FLOP of the single-CTA kernel. Both CTAs' TMA
// loads complete on the even CTA's full[s]; the even CTA's MMA thread commits
// each stage to both CTAs' empty[s] and each tile to both CTAs' acc_full[b];
// both CTAs' epilogue threads arrive on the even CTA's acc_empty[b]. The
// schedule is the single-CTA kernel's over pairs; each CTA publishes and sums
// the stream-K pieces of its own half.
struct Pair {
  static constexpr int kBN = 256;             // tile width (UMMA N)
  static constexpr int kBNHalf = 128;         // B columns per CTA
  static constexpr int kBBytes = kBNHalf * kBK * 4;
  static constexpr int kStageBytes = kABytes + kBBytes;   // 32 KiB
  static constexpr int kStages = 6;
  static constexpr int kTmemColumns = kAccums * kBN;      // 512
  static constexpr int kBarrierBytes = 8 * (2 * kStages + 2 * kAccums);
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarrierBytes + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
};

// M = 256 (two CTAs), N = 256.
template <bool kAMN, bool kBMN>
__host__ __device__ constexpr uint32_t instrDescPair() {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(kAMN) << 15) |
         (static_cast<uint32_t>(kBMN) << 16) | (static_cast<uint32_t>(Pair::kBN >> 3) << 17) |
         (static_cast<uint32_t>(256 >> 4) << 24);
}

template <bool kAMN, bool kBMN, Beta kBeta, bool kBatch>
__global__ void __launch_bounds__(kThreads, 1)
    tf32PairKernel(const __grid_constant__ Tf32Params p) {
  constexpr int kStages = Pair::kStages;
  constexpr int kStageBytes = Pair::kStageBytes;
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint32_t tmem_base_slot;
  __shared__ int last_arrival;
  unsigned char *smem = smem_raw + ((1024 - (smemAddr(smem_raw) & 1023)) & 1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes);
  uint64_t *empty = full + kStages;
  uint64_t *acc_full = empty + kStages;
  uint64_t *acc_empty = acc_full + kAccums;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = blockIdx.x & 1;      // position in the CTA pair (cluster of 2)
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int nitems = numItems(p, pair);      // the schedule is over pairs
  // Both CTAs of a pair have the same items, so both leave here or neither.
  if (nitems == 0) return;

  if (threadIdx.x == 0) {
    prefetchTensorMap(&p.tma_a);
    prefetchTensorMap(&p.tma_b);
    for (int s = 0; s < kStages; ++s) {
      mbarInit(&full[s], 1);
      mbarInit(&empty[s], 1);
    }
    for (int b = 0; b < kAccums; ++b) {
      mbarInit(&acc_full[b], 1);
      mbarInit(&acc_empty[b], 2 * 32 * (kThreads / 32 - kEpilogueWarp0));
    }
    fenceBarrierInit();
  }
  if (warp == 2) {
    tmemAllocPair(&tmem_base_slot, Pair::kTmemColumns);
    tmemRelinquishPair();
  }
  tcgenFenceBefore();
  __syncthreads();
  clusterSync();   // both CTAs' barriers and TMEM exist before either uses the other's
  tcgenFenceAfter();
  const uint32_t tmem_base = tmem_base_slot;
  gridDependencyWait();
  allowDependentLaunch();

  const int tiles_per_matrix = p.tiles_m * p.tiles_n;
  auto tileOrigin = [&](int tile, int *m0, int *n0, int *bi) {
    int tm, tn;
    *bi = kBatch ? tile / tiles_per_matrix : 0;
    rasterTile(p, tile - *bi * tiles_per_matrix, &tm, &tn);
    *m0 = tm * (2 * kBM);
    *n0 = tn * Pair::kBN;
  };
  bool ok = true;
  auto wait = [&](uint64_t *bar, int parity) {
    if (ok) ok = mbarWait(bar, static_cast<uint32_t>(parity), p.err);
  };
  int total = 0;   // k slices of this pair
  for (int i = 0; i < nitems; ++i) {
    const Item it = itemAt(p, pair, i);
    total += it.ke - it.kb;
  }

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int g = 0;
      for (int i = 0; i < nitems; ++i) {
        const Item it = itemAt(p, pair, i);
        int m0, n0, bi;
        tileOrigin(it.tile, &m0, &n0, &bi);
        const int am0 = m0 + static_cast<int>(rank) * kBM;
        const int bn0 = n0 + static_cast<int>(rank) * Pair::kBNHalf;
        for (int kb = it.kb; kb < it.ke; ++kb, ++g) {
          const int s = g % kStages;
          if (g >= kStages) wait(&empty[s], (g / kStages - 1) & 1);
          unsigned char *sa = smem + s * kStageBytes;
          unsigned char *sb = sa + kABytes;
          const int k0 = kb * kBK;
          const uint32_t bar0 = clusterAddr(smemAddr(&full[s]), 0);   // the even CTA's
          if (rank == 0) mbarArriveExpectTx(&full[s], 2 * kStageBytes);
          if constexpr (kAMN) {
            for (int j = 0; j < kBM / 32; ++j)
              tmaLoad3dPair(sa + j * kChunkBytes, &p.tma_a, bar0, am0 + 32 * j, k0, bi);
          } else {
            tmaLoad3dPair(sa, &p.tma_a, bar0, k0, am0, bi);
          }
          if constexpr (kBMN) {
            for (int j = 0; j < Pair::kBNHalf / 32; ++j)
              tmaLoad3dPair(sb + j * kChunkBytes, &p.tma_b, bar0, bn0 + 32 * j, k0, bi);
          } else {
            tmaLoad3dPair(sb, &p.tma_b, bar0, k0, bn0, bi);
          }
        }
      }
      // Drain: every commit the even CTA sent to this CTA's empty[s] has
      // landed before the pair tears down.
      for (int s = 0; s < kStages && s < total; ++s) {
        const int g_last = total - 1 - ((total - 1 - s) % kStages);
        wait(&empty[g_last % kStages], (g_last / kStages) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA) ----------------
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = instrDescPair<kAMN, kBMN>();
      int g = 0;
      for (int i = 0; i < nitems; ++i) {
        const Item it = itemAt(p, pair, i);
        const int b = i % kAccums;
        if (i >= kAccums) wait(&acc_empty[b], (i / kAccums - 1) & 1);
        tcgenFenceAfter();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * Pair::kBN);
        for (int kb = it.kb; kb < it.ke; ++kb, ++g) {
          const int s = g % kStages;
          wait(&full[s], (g / kStages) & 1);
          tcgenFenceAfter();
          const uint32_t sa = smemAddr(smem + s * kStageBytes);
          const uint32_t sb = sa + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / kMmaK; ++kk) {
            const uint32_t koff = kAMN ? kk * 1024u : kk * 32u;
            const uint32_t koff_b = kBMN ? kk * 1024u : kk * 32u;
            mmaTf32Pair(d_tmem, smemDesc<kAMN>(sa + koff), smemDesc<kBMN>(sb + koff_b), idesc,
                        kb > it.kb || kk > 0);
          }
          const uint32_t e = smemAddr(&empty[s]);
          mmaCommitPair(clusterAddr(e, 0));
          mmaCommitPair(clusterAddr(e, 1));
        }
        const uint32_t f = smemAddr(&acc_full[b]);
        mmaCommitPair(clusterAddr(f, 0));
        mmaCommitPair(clusterAddr(f, 1));
      }
    }
  } else if (warp >= kEpilogueWarp0) {
    // ---------------- epilogue (both CTAs: 128 rows each) ----------------
    const int quarter = warp % 4;
    const int r = quarter * 32 + lane;
    const int etid = threadIdx.x - 32 * kEpilogueWarp0;   // 0..127
    constexpr size_t kSlotFloat4 = static_cast<size_t>(kBM) * Pair::kBN / 4;
    auto storeChunk = [&](float *cbase, int row, int col0, const float (&acc)[32]) {
      const bool row_ok = row < p.m;
      float *cp = cbase + static_cast<size_t>(col0) * p.ldc + row;
      float cv[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        cv[j] = 0.0F;
        if constexpr (kBeta != Beta::kZero)
          if (row_ok && col0 + j < p.n) cv[j] = cp[static_cast<size_t>(j) * p.ldc];
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (row_ok && col0 + j < p.n)
          cp[static_cast<size_t>(j) * p.ldc] = epilogueValue<kBeta>(acc[j], p.alpha, p.beta, cv[j]);
      }
    };
    // This CTA's half of the slots: slot 2 * skSlot + rank.
    auto slotOf = [&](int worker, int u) {
      return reinterpret_cast<float4 *>(p.ws) +
             static_cast<size_t>(2 * skSlot(p, worker, u) + static_cast<int>(rank)) * kSlotFloat4;
    };
    for (int i = 0; i < nitems; ++i) {
      const Item it = itemAt(p, pair, i);
      const int b = i % kAccums;
      int m0, n0, bi;
      tileOrigin(it.tile, &m0, &n0, &bi);
      wait(&acc_full[b], (i / kAccums) & 1);
      tcgenFenceAfter();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(b * Pair::kBN);
      const int row = m0 + static_cast<int>(rank) * kBM + r;
      if (it.kb == 0 && it.ke == p.kiters) {
#pragma unroll 1
        for (int c = 0; c < Pair::kBN / 32; ++c) {
          uint32_t v[32];
          tmemLoad32(taddr + c * 32, v);
          float acc[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] = __uint_as_float(v[j]);
          storeChunk(kBatch ? p.c + bi * p.stride_c : p.c, row, n0 + c * 32, acc);
        }
        tcgenFenceBefore();
        mbarArriveCluster(clusterAddr(smemAddr(&acc_empty[b]), 0));
        continue;
      }
      // Stream-K piece of this CTA's half: as in the single-CTA kernel, with
      // a slot and an arrival counter per half.
      const int u = it.tile - p.dp_tiles;
      float4 *slot = slotOf(pair, u);
#pragma unroll 1
      for (int c = 0; c < Pair::kBN / 32; ++c) {
        uint32_t v[32];
        tmemLoad32(taddr + c * 32, v);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          __stcg(slot + (c * 8 + q) * kBM + r,
                 make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                             __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3])));
      }
      tcgenFenceBefore();
      mbarArriveCluster(clusterAddr(smemAddr(&acc_empty[b]), 0));
      const int first = skOwner(p, u * p.kiters);
      const int last = skOwner(p, (u + 1) * p.kiters - 1);
      unsigned long long *counter = p.counters + 2 * u + static_cast<int>(rank);
      __threadfence();
      namedBarrier<1, 128>();
      if (etid == 0)
        last_arrival = arriveCounter(counter, p.epoch, p.err) ==
                       static_cast<unsigned>(last - first + 1);
      namedBarrier<1, 128>();
      if (last_arrival) {
        __threadfence();
#pragma unroll 1
        for (int c = 0; c < Pair::kBN / 32; c += kGatherChunks) {
          float4 acc[8 * kGatherChunks];
#pragma unroll
          for (int e = 0; e < 8 * kGatherChunks; ++e) acc[e] = make_float4(0.0F, 0.0F, 0.0F, 0.0F);
#pragma unroll 1
          for (int pc = first; pc <= last; pc += 2) {
            const bool two = pc + 1 <= last;
            const float4 *s0 = slotOf(pc, u) + c * 8 * kBM + r;
            const float4 *s1 = slotOf(two ? pc + 1 : pc, u) + c * 8 * kBM + r;
            float4 v0[8 * kGatherChunks], v1[8 * kGatherChunks];
#pragma unroll
            for (int e = 0; e < 8 * kGatherChunks; ++e) {
              v0[e] = __ldcg(s0 + e * kBM);
              v1[e] = two ? __ldcg(s1 + e * kBM) : make_float4(0.0F, 0.0F, 0.0F, 0.0F);
            }
#pragma unroll
            for (int e = 0; e < 8 * kGatherChunks; ++e) {
              acc[e].x += v0[e].x;
              acc[e].y += v0[e].y;
              acc[e].z += v0[e].z;
              acc[e].w += v0[e].w;
              if (two) {
                acc[e].x += v1[e].x;
                acc[e].y += v1[e].y;
                acc[e].z += v1[e].z;
                acc[e].w += v1[e].w;
              }
            }
          }
#pragma unroll
          for (int h = 0; h < kGatherChunks; ++h) {
            float out[32];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              out[4 * q] = acc[h * 8 + q].x;
              out[4 * q + 1] = acc[h * 8 + q].y;
              out[4 * q + 2] = acc[h * 8 + q].z;
              out[4 * q + 3] = acc[h * 8 + q].w;
            }
            storeChunk(kBatch ? p.c + bi * p.stride_c : p.c, row, n0 + (c + h) * 32, out);
          }
        }
        if (etid == 0) *counter = 0;  // ready for the next launch
      }
      namedBarrier<1, 128>();   // last_arrival is reused by the next piece
    }
  }

  tcgenFenceBefore();
  __syncthreads();
  clusterSync();   // neither CTA frees TMEM or exits while the pair still works
  if (warp == 2) {
    tcgenFenceAfter();
    tmemDeallocPair(tmem_base, Pair::kTmemColumns);
  }
}

}  // namespace sgblas::kern::tf32

#endif  // SGBLAS_B200_TF32_TILE_CUH_
