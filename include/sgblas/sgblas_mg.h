/*
 * sgblas-b200 multi-GPU extension: column-sharded SGEMM.
 *
 * No counterpart in the reference API (AG0708/sgBLAS is single-GPU; its
 * docs/design.md:102 lists distributed execution as a non-goal). The split is
 * by columns of C and B, which are contiguous column blocks in column-major
 * storage, so no reduction is needed: rank p computes
 *
 *   C_p = alpha * op(A) * op(B)_p + beta * C_p,  op(B)_p = columns of op(B)
 *
 * with A sent from the root rank to every rank during the call. The transfer
 * runs on the GPUs' copy engines over NVLink, in panels of rows of op(A)
 * passed along a chain of ranks, and each rank computes a panel's rows of C
 * as soon as that panel has arrived, so the transfer overlaps the products.
 * C stays sharded unless the caller gathers it (sgblasMgAllGather).
 *
 * One process (or thread) per GPU, all on one host (the ranks share a small
 * block of host shared memory for their signals). NCCL is loaded at run time
 * (libnccl.so.2, or the file SGBLAS_NCCL_LIBRARY names) for the
 * communicator; without it sgblasMgCreate returns SGBLAS_STATUS_NOT_SUPPORTED
 * and the single-GPU API is unaffected. Waits on other ranks during set-up
 * (and during a call that grows the staging) give up after
 * SGBLAS_MG_TIMEOUT_MS milliseconds (default 300000).
 */
#ifndef SGBLAS_SGBLAS_MG_H_
#define SGBLAS_SGBLAS_MG_H_

#include <stddef.h>
#include <sgblas/sgblas.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SGBLAS_MG_UNIQUE_ID_BYTES 128

typedef struct sgblasMgContext *sgblasMgHandle_t;

/* Fills id with a fresh NCCL unique id; call on one rank and pass the bytes
 * to every rank out of band. */
sgblasStatus_t sgblasMgGetUniqueId(unsigned char id[SGBLAS_MG_UNIQUE_ID_BYTES]);

/* Joins the communicator of nranks (at most 64) ranks as `rank`, on CUDA
 * device `device` (which becomes the calling thread's current device).
 * Collective: every rank must call it. NCCL initialises non-blocking; a rank
 * that has not joined when the deadline passes ends the call with
 * EXECUTION_FAILED (the half-made communicator is aborted) instead of a hang.
 * Errors: INVALID_VALUE (bad rank/size/pointer, or ranks disagree on
 * nranks), NOT_SUPPORTED (NCCL or stream memory operations unavailable),
 * INTERNAL_ERROR (NCCL initialisation failed), EXECUTION_FAILED (deadline),
 * ALLOC_FAILED. */
sgblasStatus_t sgblasMgCreate(sgblasMgHandle_t *handle, int nranks, int rank,
                              const unsigned char id[SGBLAS_MG_UNIQUE_ID_BYTES],
                              int device);

/* Waits (at most the deadline) for this rank's enqueued work, then releases
 * the communicator, the staging buffer and the inner SGEMM handle. Work still
 * waiting for another rank at the deadline is released as by sgblasMgAbort
 * and EXECUTION_FAILED is returned. */
sgblasStatus_t sgblasMgDestroy(sgblasMgHandle_t handle);

/* Failure handling, called from the host of any rank, e.g. when the host
 * learns that another rank has left: releases every wait that any rank's
 * enqueued sgblasMgSgemm has on another rank (their products finish with
 * undefined values) and aborts the NCCL communicator. Every later call on
 * any rank of the communicator returns EXECUTION_FAILED; sgblasMgDestroy
 * still frees the handle. */
sgblasStatus_t sgblasMgAbort(sgblasMgHandle_t handle);

/* Stream for the broadcast and the local SGEMM (NULL: legacy stream). */
sgblasStatus_t sgblasMgSetStream(sgblasMgHandle_t handle, sgblasStream_t stream);

sgblasStatus_t sgblasMgGetRank(sgblasMgHandle_t handle, int *rank, int *nranks);

/* Math mode of the local products (SGBLAS_MATH_FP32, the default, or
 * SGBLAS_MATH_TF32 for the tensor-core lane); same values and statuses as
 * sgblasSetMathMode. Set it to the same value on every rank. */
sgblasStatus_t sgblasMgSetMathMode(sgblasMgHandle_t handle, sgblasMathMode_t mode);

/*
 * Collective, column-sharded SGEMM. On `root`, `a` holds A (lda * (transa ==
 * N ? k : m) floats of device memory). On the other ranks `a` may be NULL;
 * if it is not, A is also copied there (lda as on the root). b and c hold
 * this rank's column block: n_local columns of op(B) (stored as for
 * sgblasSgemm with ldb) and of C (ldc). Every rank passes the same transa,
 * transb, m, k, lda, root and the same alpha and beta values (non-NULL when
 * m > 0); n_local may differ between ranks (0 is allowed: the rank then only
 * passes A on). Ranks that disagree on these shared arguments make the call
 * undefined, possibly never finishing (check them on the host first).
 *
 * The shared arguments are checked first and give every rank the same error.
 * A rank whose own arguments (n_local, b, ldb, c, ldc) are invalid still
 * passes A on, computes nothing and returns the error; the other ranks are
 * unaffected. With no work anywhere (m == 0, k == 0 or alpha == 0) nothing is
 * sent and each rank scales its C block as sgblasSgemm would.
 *
 * Enqueues on the handle's stream and returns without synchronizing, except
 * that a call needing more staging than earlier calls (the first one with a
 * product, or a larger A) first waits for this rank's earlier work, then
 * allocates the staging on every rank (about the size of A, one per rank)
 * and exchanges it -- at most the deadline. A holds its values until the call
 * has completed on the root's stream.
 */
sgblasStatus_t sgblasMgSgemm(sgblasMgHandle_t handle, sgblasOperation_t transa,
                             sgblasOperation_t transb, int m, int n_local, int k,
                             const float *alpha, float *a, int lda, int root,
                             const float *b, int ldb, const float *beta, float *c,
                             int ldc);

/* Gathers every rank's `count` floats of `send` into `recv` (nranks * count
 * floats, rank order). With ldc == m and equal shards this assembles C. */
sgblasStatus_t sgblasMgAllGather(sgblasMgHandle_t handle, const float *send,
                                 float *recv, size_t count);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SGBLAS_SGBLAS_MG_H_ */
