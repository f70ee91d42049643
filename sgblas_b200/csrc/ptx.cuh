// Thin inline-PTX wrappers for sm_100a: mbarriers, TMA tile loads, cp.async.
//
// Every wait on an mbarrier is bounded (kSpinLimit polls of try_wait, each of
// which itself suspends for a hardware-defined slice); a wait that runs out
// records an error code in the library's device error word and returns false,
// so that a kernel never spins forever on a copy that did not arrive.
#ifndef SGBLAS_B200_PTX_CUH_
#define SGBLAS_B200_PTX_CUH_

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace sgblas::kern {

// Poll budget of one bounded mbarrier wait (each try_wait suspends the
// thread for up to a hardware time slice, so this is well above a second).
constexpr uint32_t kSpinLimit = 1u << 24;

// Device error word codes (OR-ed together).
constexpr unsigned kErrBarrierTimeout = 1u;
constexpr unsigned kErrCounter = 2u;   // an arrival counter could not be updated

// ---- split-tile arrival counters --------------------------------------------
// A tile split into pieces is finished by the CTA whose piece arrives last.
// Its counter holds (epoch << 32) | arrivals; the host gives every launch
// that uses a scratch buffer's counters an epoch that no earlier launch on
// that buffer used. Zero is the clean state: the last arrival resets its
// counter to zero, so the next launch -- or the next replay of a CUDA graph,
// which reuses its epoch -- starts clean. A value of another non-zero epoch
// is what a launch that stopped early (a wait that timed out) left behind:
// the arrival first swaps it back to zero, so an interrupted launch cannot
// make a later one pick the wrong last piece.
//
// Arrivals use atomicAdd: many pieces of one tile may arrive at once, and a
// compare-and-swap loop would serialise them into one L2 round trip each. The
// first arrival stamps the epoch with a second add; arrivals between the two
// see epoch 0 and count the same way.
//
// Returns the arrival's number (1 for the first piece).
__device__ __forceinline__ unsigned arriveCounter(unsigned long long *counter, unsigned epoch,
                                                  unsigned *err) {
  unsigned long long seen;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(seen) : "l"(counter) : "memory");
  const unsigned seen_epoch = static_cast<unsigned>(seen >> 32);
  if (seen_epoch != 0 && seen_epoch != epoch) {
    // Left by an interrupted launch: one of the arrivals that saw it clears
    // it (the others' swaps fail: the value has moved on).
    (void)atomicCAS(counter, seen, 0ULL);
  }
  const unsigned long long old = atomicAdd(counter, 1ULL);
  const unsigned old_epoch = static_cast<unsigned>(old >> 32);
  if (old_epoch != 0 && old_epoch != epoch && err != nullptr) atomicOr(err, kErrCounter);
  if (old == 0ULL) atomicAdd(counter, static_cast<unsigned long long>(epoch) << 32);
  return static_cast<unsigned>(old & 0xffffffffULL) + 1U;
}

__device__ __forceinline__ uint32_t smemAddr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbarInit(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smemAddr(bar)), "r"(count)
               : "memory");
}

// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fenceBarrierInit() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's view of shared memory in the generic proxy before
// its later async-proxy operations. A stage that the compute warps read with
// ordinary loads and TMA then refills is a write-after-read across proxies:
// the empty-barrier hand-off orders the reads only in the generic proxy, so
// the producer issues this fence after acquiring the stage and before the
// TMA that overwrites it (without it a refill can land while a lagging warp
// is still reading the previous contents).
__device__ __forceinline__ void fenceProxyAsyncShared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbarArriveExpectTx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smemAddr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbarTryWait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smemAddr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Non-blocking test of phase completion.
__device__ __forceinline__ bool mbarTestWait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smemAddr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for the phase with the given parity to complete. The common
// case -- the phase completed long ago -- costs one non-blocking test.
__device__ __forceinline__ bool mbarWait(uint64_t *bar, uint32_t parity, unsigned *err,
                                         uint32_t limit = kSpinLimit) {
  if (mbarTestWait(bar, parity)) return true;
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbarTryWait(bar, parity)) return true;
  }
  if (err != nullptr) atomicOr(err, kErrBarrierTimeout);
  return false;
}

// Plain arrive (release semantics at CTA scope).
__device__ __forceinline__ void mbarArrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smemAddr(bar)) : "memory");
}

// Arrive on `bar` once every cp.async this thread issued so far has landed.
__device__ __forceinline__ void cpAsyncArrive(uint64_t *bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smemAddr(bar))
               : "memory");
}

// Named barrier kId for kCount threads, whole warps (id 0 is the one
// __syncthreads uses).
template <int kId, int kCount>
__device__ __forceinline__ void namedBarrier() {
  asm volatile("bar.sync %0, %1;" ::"n"(kId), "n"(kCount) : "memory");
}

// Warpgroup register reallocation (all 128 threads of the warpgroup execute
// it). The block's launch allocation bounds the sum over warpgroups.
template <int kRegs>
__device__ __forceinline__ void regAlloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegs));
}
template <int kRegs>
__device__ __forceinline__ void regDealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegs));
}

// 2-D TMA tile load global -> shared, completion signalled on `bar`.
// x is the innermost (contiguous) coordinate in elements.
__device__ __forceinline__ void tmaLoad2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x,
                                          int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smemAddr(dst)),
      "l"(map), "r"(smemAddr(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3-D form: x, y within one matrix, z selects the matrix of a strided batch.
__device__ __forceinline__ void tmaLoad3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x,
                                          int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smemAddr(dst)),
      "l"(map), "r"(smemAddr(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void prefetchTensorMap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Programmatic dependent launch. A kernel launched with programmatic stream
// serialization may start while the previous kernel in the stream is still
// running; gridDependencyWait blocks until that kernel has completed and its
// memory operations are visible, so it must precede every global memory
// access. allowDependentLaunch lets the next kernel in the stream begin its
// own launch (it still waits in gridDependencyWait for this one to finish).
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void gridDependencyWait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void allowDependentLaunch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- tcgen05: tensor memory and the 5th-generation tensor cores ------------
// Tensor memory (TMEM) is allocated in columns (a power of two, 32..512) by
// one whole warp; the allocated base address is written to shared memory.
__device__ __forceinline__ void tmemAlloc(uint32_t *dst_smem, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smemAddr(dst_smem)),
               "r"(columns)
               : "memory");
}
__device__ __forceinline__ void tmemRelinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmemDealloc(uint32_t taddr, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns)
               : "memory");
}
// Orders tcgen05 operations against thread synchronisation (barriers,
// mbarrier waits) on either side.
__device__ __forceinline__ void tcgenFenceBefore() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tcgenFenceAfter() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], TF32 inputs, FP32 accumulate;
// one thread issues it for the CTA.
__device__ __forceinline__ void mmaTf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}
// Arrives (once) on `bar` when every tcgen05.mma this thread issued so far
// has completed.
__device__ __forceinline__ void mmaCommit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smemAddr(bar))
               : "memory");
}
// 32 consecutive TMEM columns of the warp's 32 lanes (lane i of the warp
// reads TMEM lane (warp % 4) * 32 + i); then wait for the load.
__device__ __forceinline__ void tmemLoad32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- CTA pairs (clusters of two) and cta_group::2 ---------------------------
// Shared-memory address of the same location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t clusterAddr(uint32_t local_smem, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem), "r"(rank));
  return r;
}
// This CTA's rank in its cluster, and the cluster's index along x.
__device__ __forceinline__ uint32_t clusterRank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t clusterIdX() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
// 16-byte load from distributed shared memory (a cluster address).
__device__ __forceinline__ float4 ldCluster4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}
// Whole-cluster barrier (every thread of every CTA), release / acquire.
__device__ __forceinline__ void clusterSync() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier in any CTA of the cluster (cluster address).
__device__ __forceinline__ void mbarArriveCluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}
// TMA 2-D load into this CTA's shared memory whose completion is counted on
// an mbarrier of either CTA of the pair (cluster address).
__device__ __forceinline__ void tmaLoad2dPair(void *dst, const CUtensorMap *map,
                                              uint32_t cluster_bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smemAddr(dst)),
      "l"(map), "r"(cluster_bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmaLoad3dPair(void *dst, const CUtensorMap *map,
                                              uint32_t cluster_bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smemAddr(dst)),
      "l"(map), "r"(cluster_bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tmemAllocPair(uint32_t *dst_smem, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smemAddr(dst_smem)),
               "r"(columns)
               : "memory");
}
__device__ __forceinline__ void tmemRelinquishPair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmemDeallocPair(uint32_t taddr, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns)
               : "memory");
}
// The pair's MMA (M = 256 over both CTAs' TMEM), issued by the even CTA.
__device__ __forceinline__ void mmaTf32Pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}
// Arrives once on the mbarrier at `cluster_bar` (either CTA of the pair)
// when every pair MMA this thread issued so far has completed.
__device__ __forceinline__ void mmaCommitPair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   cluster_bar)
               : "memory");
}

// Asynchronous prefetch of [ptr, ptr + bytes) from global memory into L2.
// ptr 16-byte aligned, bytes a non-zero multiple of 16; the range must lie
// inside one allocation.
__device__ __forceinline__ void prefetchL2Bulk(const void *ptr, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"(bytes) : "memory");
}

// 4-byte cp.async with zero fill: copies `bytes` (0 or 4) and zero-fills the
// rest of the 4-byte destination, so a predicated-off element reads as 0.
__device__ __forceinline__ void cpAsync4(void *dst, const void *src, uint32_t bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smemAddr(dst)), "l"(src),
               "r"(bytes)
               : "memory");
}

// cp.async of kBytes (4, 8 or 16) with zero fill: copies `bytes` (<= kBytes)
// and zero-fills the rest of the kBytes destination. Both addresses must be
// kBytes-aligned.
template <int kBytes>
__device__ __forceinline__ void cpAsyncN(void *dst, const void *src, uint32_t bytes) {
  static_assert(kBytes == 4 || kBytes == 8 || kBytes == 16, "cp.async size");
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(smemAddr(dst)), "l"(src),
               "n"(kBytes), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void cpAsyncCommit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cpAsyncWait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace sgblas::kern

#endif  // SGBLAS_B200_PTX_CUH_
