/*
 * A stand-in for libnccl.so.2, test infrastructure only: the NCCL entry points that
 * libgsampler's vocabulary-sharded exchange resolves (gs_nccl_*, gs_shard_sample), with a
 * behaviour chosen by the environment variable FAKE_NCCL_MODE at each call, so that the
 * host-side waits, timeouts and aborts are tested without a second rank and without a
 * GPU that waits on anything:
 *   ok            set-up completes; ncclAllGather copies the send buffer into every
 *                 rank's slot of the receive buffer (cudaMemcpyAsync on the stream);
 *   init_hang     set-up never completes (ncclCommGetAsyncError stays ncclInProgress);
 *   init_error    set-up fails at once (ncclInvalidArgument);
 *   gather_hang   ncclAllGather is accepted but never issued (stays ncclInProgress);
 *   gather_error  ncclAllGather reports a remote error afterwards.
 * fake_nccl_aborts() counts ncclCommAbort calls.  Built by the tests with gcc.
 */
#include <dlfcn.h>
#include <stdlib.h>
#include <string.h>

typedef struct { char internal[128]; } ncclUniqueId;
typedef int ncclResult_t;
enum { kSuccess = 0, kInvalidArgument = 4, kRemoteError = 6, kInProgress = 7 };

struct fake_comm {
  int nranks;
  int state; /* what ncclCommGetAsyncError reports */
};

static int g_aborts = 0;

static int mode_is(const char* m) {
  const char* v = getenv("FAKE_NCCL_MODE");
  return v && strcmp(v, m) == 0;
}

int fake_nccl_aborts(void) { return g_aborts; }

ncclResult_t ncclGetUniqueId(ncclUniqueId* id) {
  memset(id->internal, 'F', sizeof(id->internal));
  return kSuccess;
}

ncclResult_t ncclCommInitRankConfig(void** comm, int nranks, ncclUniqueId id, int rank, void* config) {
  (void)id;
  (void)rank;
  (void)config;
  if (mode_is("init_error")) return kInvalidArgument;
  struct fake_comm* c = (struct fake_comm*)calloc(1, sizeof(struct fake_comm));
  c->nranks = nranks;
  c->state = mode_is("init_hang") ? kInProgress : kSuccess;
  *comm = c;
  return c->state;
}

ncclResult_t ncclCommGetAsyncError(void* comm, ncclResult_t* state) {
  *state = ((struct fake_comm*)comm)->state;
  return kSuccess;
}

ncclResult_t ncclAllGather(const void* send, void* recv, size_t count, int type, void* comm, void* stream) {
  (void)type;
  struct fake_comm* c = (struct fake_comm*)comm;
  if (mode_is("gather_hang")) {
    c->state = kInProgress;
    return kInProgress;
  }
  if (mode_is("gather_error")) {
    c->state = kRemoteError;
    return kSuccess;
  }
  typedef int (*memcpy_async_t)(void*, const void*, size_t, int, void*);
  memcpy_async_t cp = (memcpy_async_t)dlsym(RTLD_DEFAULT, "cudaMemcpyAsync");
  if (!cp) return kInvalidArgument;
  for (int r = 0; r < c->nranks; ++r)
    if (cp((char*)recv + (size_t)r * count, send, count, 3 /* device to device */, stream) != 0) return kRemoteError;
  return kSuccess;
}

ncclResult_t ncclCommAbort(void* comm) {
  ++g_aborts;
  free(comm);
  return kSuccess;
}

ncclResult_t ncclCommFinalize(void* comm) {
  (void)comm;
  return kSuccess;
}

ncclResult_t ncclCommDestroy(void* comm) {
  free(comm);
  return kSuccess;
}

const char* ncclGetErrorString(ncclResult_t r) { return r == kRemoteError ? "fake remote error" : "fake error"; }

const char* ncclGetLastError(void* comm) {
  (void)comm;
  return "";
}
