/*
 * sgblas-b200 multi-GPU extension: column-sharded SGEMM over NCCL.
 *
 * No counterpart in the reference API (AG0708/sgBLAS is single-GPU; its
 * docs/design.md:102 lists distributed execution as a non-goal). The split is
 * by columns of C and B, which are contiguous column blocks in column-major
 * storage, so no reduction is needed: rank p computes
 *
 *   C_p = alpha * op(A) * op(B)_p + beta * C_p,  op(B)_p = columns of op(B)
 *
 * after A has been broadcast from the root rank over NVLink by NCCL. C stays
 * sharded unless the caller gathers it (sgblasMgAllGather).
 *
 * One process (or thread) per GPU. NCCL is loaded at run time (libnccl.so.2);
 * without it sgblasMgCreate returns SGBLAS_STATUS_NOT_SUPPORTED and the
 * single-GPU API is unaffected.
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

/* Joins the communicator of nranks ranks as `rank`, on CUDA device `device`
 * (which becomes the calling thread's current device). Collective: every rank
 * must call it. Errors: INVALID_VALUE (bad rank/size/pointer), NOT_SUPPORTED
 * (NCCL not loadable), INTERNAL_ERROR (NCCL initialisation failed). */
sgblasStatus_t sgblasMgCreate(sgblasMgHandle_t *handle, int nranks, int rank,
                              const unsigned char id[SGBLAS_MG_UNIQUE_ID_BYTES],
                              int device);

/* Releases the communicator (ncclCommDestroy) and the inner SGEMM handle. */
sgblasStatus_t sgblasMgDestroy(sgblasMgHandle_t handle);

/* Stream for the broadcast and the local SGEMM (NULL: legacy stream). */
sgblasStatus_t sgblasMgSetStream(sgblasMgHandle_t handle, sgblasStream_t stream);

sgblasStatus_t sgblasMgGetRank(sgblasMgHandle_t handle, int *rank, int *nranks);

/* Math mode of the local products (SGBLAS_MATH_FP32, the default, or
 * SGBLAS_MATH_TF32 for the tensor-core lane); same values and statuses as
 * sgblasSetMathMode. Set it to the same value on every rank. */
sgblasStatus_t sgblasMgSetMathMode(sgblasMgHandle_t handle, sgblasMathMode_t mode);

/*
 * Collective, column-sharded SGEMM. On every rank `a` points to lda * (transa
 * == N ? k : m) floats of device memory: on `root` it holds A, on the others
 * it is the buffer A is broadcast into (overwritten). b and c hold this rank's
 * column block: n_local columns of op(B) (stored as for sgblasSgemm with ldb)
 * and of C (ldc). Every rank passes the same transa, transb, m, k, alpha,
 * beta, lda and root; n_local may differ between ranks (0 is allowed: the rank
 * only takes part in the broadcast).
 *
 * Validation follows sgblasSgemm on the local problem; with no work anywhere
 * (m == 0, k == 0 or alpha == 0) the broadcast is skipped. Enqueues on the
 * handle's stream and returns without synchronizing.
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
