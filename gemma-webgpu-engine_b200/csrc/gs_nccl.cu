// Vocabulary-sharded sampling with its own NCCL exchange: gs_nccl_* and gs_shard_sample.
//
// gs_shard_partials / gs_shard_merge leave the exchange of the per-shard records to the
// caller's framework.  A host without one (the Node addon of the reference's TypeScript
// session) gets the whole step here: the records of the local shard, one ncclAllGather of
// them over the communicator, and the merge, all on the caller's stream.
//
// NCCL is found at run time (dlopen of the library the process already has loaded, else
// libnccl.so.2, or the path in GS_NCCL_LIBRARY), so libgsampler itself does not depend on
// it.  Communicators are non-blocking (ncclConfig_t.blocking = 0): every NCCL call returns
// at once and its progress is polled on the host with ncclCommGetAsyncError, so a rank that
// never joins costs a bounded wait: after timeout_ms the communicator is aborted and the
// call returns GS_ETIMEOUT (the communicator is then unusable; destroy it).  Other NCCL
// failures return GS_ENCCL with NCCL's message.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>

#include "gs_internal.cuh"
#include "../../include/gsampler.h"

static_assert(sizeof(gs_nccl_id) == sizeof(ncclUniqueId), "gs_nccl_id holds an ncclUniqueId");

namespace gs {
namespace {

// The NCCL entry points this file uses, resolved once per process.
struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*finalize)(ncclComm_t) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  const char* (*last_error)(ncclComm_t) = nullptr;
};

std::mutex g_api_mu;
NcclApi g_api;
bool g_api_tried = false;
thread_local std::string g_nccl_err;

const NcclApi& nccl_api() {
  std::lock_guard<std::mutex> lock(g_api_mu);
  if (g_api_tried) return g_api;
  g_api_tried = true;
  void* h = nullptr;
  const char* path = std::getenv("GS_NCCL_LIBRARY");
  if (path && *path) {
    h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
  } else {
    h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // (the copy the process already uses)
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  }
  if (!h) {
    const char* e = dlerror();
    g_api.why = std::string("NCCL library not found: ") + (e ? e : "dlopen failed");
    return g_api;
  }
  bool all = true;
  auto sym = [&](auto& fn, const char* name) {
    fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
    if (!fn) {
      all = false;
      g_api.why = std::string("NCCL library lacks ") + name;
    }
  };
  sym(g_api.get_unique_id, "ncclGetUniqueId");
  sym(g_api.init_rank_config, "ncclCommInitRankConfig");
  sym(g_api.get_async_error, "ncclCommGetAsyncError");
  sym(g_api.all_gather, "ncclAllGather");
  sym(g_api.abort, "ncclCommAbort");
  sym(g_api.finalize, "ncclCommFinalize");
  sym(g_api.destroy, "ncclCommDestroy");
  sym(g_api.error_string, "ncclGetErrorString");
  sym(g_api.last_error, "ncclGetLastError");
  g_api.ok = all;
  return g_api;
}

using Clock = std::chrono::steady_clock;

}  // namespace
}  // namespace gs

using namespace gs;

struct gs_nccl {
  ncclComm_t comm = nullptr;
  int nranks = 0;
  int rank = 0;
  bool broken = false;                // aborted after a timeout or an error
  std::string err;
  unsigned char* local = nullptr;     // this rank's records [rows][record]
  unsigned char* gathered = nullptr;  // [nranks][rows][record]
  size_t local_bytes = 0;
  cudaEvent_t done = nullptr;
};

namespace {

gs_status nfail(gs_nccl* c, gs_status s, const std::string& msg) {
  if (c) c->err = msg;
  g_nccl_err = msg;
  return s;
}

// Aborts the communicator (which frees it) and marks the handle unusable.
void abort_comm(gs_nccl* c, const NcclApi& api) {
  if (c->comm) api.abort(c->comm);
  c->comm = nullptr;
  c->broken = true;
}

std::string nccl_msg(const NcclApi& api, ncclComm_t comm, ncclResult_t r, const char* what) {
  std::string m = std::string(what) + ": " + (api.error_string ? api.error_string(r) : "NCCL error");
  const char* last = api.last_error ? api.last_error(comm) : nullptr;
  if (last && *last) m += std::string(" (") + last + ")";
  return m;
}

// Polls the communicator until its pending operation has been issued (ncclInProgress gone).
// timeout_ms <= 0: no limit.
gs_status wait_issued(gs_nccl* c, const NcclApi& api, int32_t timeout_ms, Clock::time_point t0, const char* what) {
  for (;;) {
    ncclResult_t st = ncclInProgress;
    const ncclResult_t r = api.get_async_error(c->comm, &st);
    if (r != ncclSuccess) return nfail(c, GS_ENCCL, nccl_msg(api, c->comm, r, what));
    if (st == ncclSuccess) return GS_OK;
    if (st != ncclInProgress) {
      const gs_status e = nfail(c, GS_ENCCL, nccl_msg(api, c->comm, st, what));
      abort_comm(c, api);
      return e;
    }
    if (timeout_ms > 0 && Clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      abort_comm(c, api);
      return nfail(c, GS_ETIMEOUT, std::string(what) + ": no progress within the timeout; the communicator was aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

}  // namespace

extern "C" {

gs_status gs_nccl_unique_id(gs_nccl_id* id) {
  if (!id) return GS_EINVAL;
  const NcclApi& api = nccl_api();
  if (!api.ok) return nfail(nullptr, GS_ENCCL, api.why);
  ncclUniqueId u;
  const ncclResult_t r = api.get_unique_id(&u);
  if (r != ncclSuccess) return nfail(nullptr, GS_ENCCL, nccl_msg(api, nullptr, r, "ncclGetUniqueId"));
  std::memcpy(id, &u, sizeof(u));
  return GS_OK;
}

gs_status gs_nccl_create(int device, const gs_nccl_id* id, int32_t nranks, int32_t rank, int32_t timeout_ms,
                         gs_nccl** out) {
  if (!id || !out || nranks < 1 || rank < 0 || rank >= nranks) return nfail(nullptr, GS_EINVAL, "bad arguments");
  *out = nullptr;
  const NcclApi& api = nccl_api();
  if (!api.ok) return nfail(nullptr, GS_ENCCL, api.why);
  if (device >= 0) {
    const cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return nfail(nullptr, GS_ECUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  }
  gs_nccl* c = new gs_nccl();
  c->nranks = nranks;
  c->rank = rank;
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  const auto t0 = Clock::now();
  const ncclResult_t r = api.init_rank_config(&c->comm, nranks, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    const gs_status s = nfail(nullptr, GS_ENCCL, nccl_msg(api, c->comm, r, "ncclCommInitRankConfig"));
    abort_comm(c, api);
    delete c;
    return s;
  }
  const gs_status s = wait_issued(c, api, timeout_ms, t0, "communicator set-up");
  if (s != GS_OK) {
    g_nccl_err = c->err;
    abort_comm(c, api);
    delete c;
    return s;
  }
  *out = c;
  return GS_OK;
}

gs_status gs_nccl_destroy(gs_nccl* c) {
  if (!c) return GS_EINVAL;
  const NcclApi& api = nccl_api();
  if (c->comm && api.ok) {
    api.finalize(c->comm);
    const gs_status s = wait_issued(c, api, 10000, Clock::now(), "communicator finalize");
    if (s == GS_OK) {
      api.destroy(c->comm);
      c->comm = nullptr;
    } else {
      abort_comm(c, api);
    }
  }
  if (c->local) cudaFree(c->local);
  if (c->gathered) cudaFree(c->gathered);
  if (c->done) cudaEventDestroy(c->done);
  delete c;
  return GS_OK;
}

const char* gs_nccl_last_error(const gs_nccl* c) { return c ? c->err.c_str() : g_nccl_err.c_str(); }

gs_status gs_shard_sample(gs_ctx* ctx, gs_nccl* c, const gs_batch* shard, int64_t vocab_offset, int64_t vocab_total,
                          const gs_outputs* out, int32_t timeout_ms, void* stream) {
  if (!ctx || !c || !shard || !out) return nfail(c, GS_EINVAL, "ctx, communicator, shard batch and outputs are required");
  if (c->broken || !c->comm) return nfail(c, GS_ENCCL, "the communicator was aborted by an earlier failure; destroy it");
  const NcclApi& api = nccl_api();
  if (!api.ok) return nfail(c, GS_ENCCL, api.why);
  if (shard->rows == 0) return GS_OK;
  const int64_t rec = gs_shard_record_bytes(shard->params, shard->params_count, vocab_total,
                                            shard->history ? shard->history_stride : 0);
  if (rec < 0) return nfail(c, GS_EINVAL, "invalid shard geometry");
  int prev = -1;
  cudaGetDevice(&prev);
  const int dev = ctx_device(ctx);
  if (prev != dev) cudaSetDevice(dev);
  auto done = [&](gs_status s) {
    if (prev >= 0 && prev != dev) cudaSetDevice(prev);
    return s;
  };
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the communicator's record buffers (grown on demand: the first call of a larger batch allocates)
  const size_t lb = static_cast<size_t>(shard->rows) * static_cast<size_t>(rec);
  if (lb > c->local_bytes) {
    cudaStreamSynchronize(st);
    if (c->local) cudaFree(c->local);
    if (c->gathered) cudaFree(c->gathered);
    c->local = c->gathered = nullptr;
    c->local_bytes = 0;
    if (cudaMalloc(&c->local, lb) != cudaSuccess ||
        cudaMalloc(&c->gathered, lb * static_cast<size_t>(c->nranks)) != cudaSuccess)
      return done(nfail(c, GS_ENOMEM, "record buffers"));
    c->local_bytes = lb;
  }
  if (!c->done && cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming) != cudaSuccess)
    return done(nfail(c, GS_ECUDA, "event"));
  gs_status s = gs_shard_partials(ctx, shard, vocab_offset, vocab_total, out->logprob != nullptr, c->local, stream);
  if (s != GS_OK) return done(nfail(c, s, std::string("partials: ") + gs_last_error(ctx)));
  const auto t0 = Clock::now();
  const ncclResult_t r = api.all_gather(c->local, c->gathered, lb, ncclUint8, c->comm, st);
  if (r != ncclSuccess && r != ncclInProgress) {
    const gs_status e = nfail(c, GS_ENCCL, nccl_msg(api, c->comm, r, "ncclAllGather"));
    abort_comm(c, api);
    return done(e);
  }
  s = wait_issued(c, api, timeout_ms, t0, "record exchange");
  if (s != GS_OK) return done(s);
  gs_batch full = *shard;
  full.logits = nullptr;
  full.vocab = vocab_total;
  full.row_stride = vocab_total;
  s = gs_shard_merge(ctx, &full, c->nranks, c->gathered, out, stream);
  if (s != GS_OK) return done(nfail(c, s, std::string("merge: ") + gs_last_error(ctx)));
  if (timeout_ms > 0) {
    // the exchange completes on the stream: wait for it with a bound (a peer that never
    // joins would keep the collective waiting)
    cudaEventRecord(c->done, st);
    for (;;) {
      const cudaError_t q = cudaEventQuery(c->done);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) return done(nfail(c, GS_ECUDA, std::string("exchange: ") + cudaGetErrorString(q)));
      ncclResult_t as = ncclSuccess;
      api.get_async_error(c->comm, &as);
      if (as != ncclSuccess && as != ncclInProgress) {
        const gs_status e = nfail(c, GS_ENCCL, nccl_msg(api, c->comm, as, "record exchange"));
        abort_comm(c, api);
        return done(e);
      }
      if (Clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
        abort_comm(c, api);
        return done(nfail(c, GS_ETIMEOUT, "record exchange: not complete within the timeout; the communicator was aborted"));
      }
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
  }
  return done(GS_OK);
}

}  // extern "C"
