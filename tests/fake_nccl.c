/*
 * A stand-in for libnccl.so.2 that the multi-GPU failure tests load through
 * SGBLAS_NCCL_LIBRARY, to make communicator initialisation fail on the host
 * without any real peer or any GPU work:
 *
 *   FAKE_NCCL_MODE=fail   ncclCommInitRankConfig returns ncclSystemError
 *   FAKE_NCCL_MODE=hang   initialisation never finishes (ncclInProgress for
 *                         ever), as when a rank never joins
 *   otherwise             initialisation succeeds at once
 *
 * Every ncclCommAbort / ncclCommDestroy appends a line to the file
 * FAKE_NCCL_LOG names, so a test can check what the library called.
 * Only the entry points libsgblas.so resolves are provided.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef enum {
  ncclSuccess = 0,
  ncclSystemError = 2,
  ncclInProgress = 7
} ncclResult_t;

typedef struct {
  char internal[128];
} ncclUniqueId;

typedef struct fakeComm {
  int hang;
} *ncclComm_t;

static void note(const char *what) {
  const char *path = getenv("FAKE_NCCL_LOG");
  if (path == NULL) return;
  FILE *f = fopen(path, "a");
  if (f == NULL) return;
  fprintf(f, "%s\n", what);
  fclose(f);
}

static int mode_is(const char *m) {
  const char *v = getenv("FAKE_NCCL_MODE");
  return v != NULL && strcmp(v, m) == 0;
}

ncclResult_t ncclGetUniqueId(ncclUniqueId *id) {
  memset(id, 7, sizeof(*id));
  return ncclSuccess;
}

ncclResult_t ncclCommInitRankConfig(ncclComm_t *comm, int nranks, ncclUniqueId id, int rank,
                                    void *config) {
  (void)nranks; (void)id; (void)rank; (void)config;
  note("init");
  if (mode_is("fail")) {
    *comm = NULL;
    return ncclSystemError;
  }
  *comm = (ncclComm_t)calloc(1, sizeof(struct fakeComm));
  (*comm)->hang = mode_is("hang");
  return (*comm)->hang ? ncclInProgress : ncclSuccess;
}

ncclResult_t ncclCommGetAsyncError(ncclComm_t comm, ncclResult_t *state) {
  *state = comm != NULL && comm->hang ? ncclInProgress : ncclSuccess;
  return ncclSuccess;
}

ncclResult_t ncclCommAbort(ncclComm_t comm) {
  note("abort");
  free(comm);
  return ncclSuccess;
}

ncclResult_t ncclCommDestroy(ncclComm_t comm) {
  note("destroy");
  free(comm);
  return ncclSuccess;
}

ncclResult_t ncclAllGather(const void *send, void *recv, size_t count, int type, ncclComm_t comm,
                           void *stream) {
  (void)send; (void)recv; (void)count; (void)type; (void)comm; (void)stream;
  return ncclSuccess;
}
