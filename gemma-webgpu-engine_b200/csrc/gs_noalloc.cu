// gs_sample_noalloc: gs_sample for callers that must not allocate device memory.
//
// Some hosts of this sampler cannot call cudaMalloc: a serving runtime that has already
// handed the whole device to its own memory pool, a real-time token loop where the
// implicit device synchronisation of cudaMalloc/cudaFree is not acceptable, or an
// embedding that only lends the sampler the caller's input and output buffers.  This
// entry point runs the same kernels as gs_sample, but its per-call scratch (the per-row
// plans, the streaming units' partial statistics and candidates) lives in the fixed
// device array below instead of a context's workspace.
//
// The array is a file-scope __device__ object: every GPU that loads this library keeps
// GS_NOALLOC_SCRATCH_BYTES of it until the process exits.  Host code cannot pass the
// array's name to a kernel (on the host that name is only a stand-in, not a device
// address), so every call looks the device address up with cudaGetSymbolAddress, with
// the call's device current.  The first call on a device also loads the module there
// (make it before any stream capture); later lookups are host-side only.  Looking the
// address up on every call, instead of caching it, keeps the call correct after the
// device's primary context is reset and created again, when the array can move.
//
// Every call writes each scratch byte it later reads, so nothing has to start at zero;
// the array keeps the previous call's contents.  The exception is the single-launch
// decode step's per-row counters (g_noalloc_done): they start at zero when the module
// loads, and the step's last CTA of each row sets its counter back to zero.  All calls share the one array: two
// calls whose kernels overlap on the GPU (different streams, no ordering between them)
// race on it and produce undefined results.
#include <string>

#include "gs_plan.cuh"

namespace gs {
namespace {

static_assert(GS_NOALLOC_SCRATCH_BYTES % 256 == 0, "scratch size must keep 256-byte alignment");

__device__ __align__(256) unsigned char g_noalloc_scratch[GS_NOALLOC_SCRATCH_BYTES];
__device__ unsigned g_noalloc_done[kStepDoneRows];

thread_local std::string g_noalloc_err;

gs_status set_error(gs_status s, const std::string& msg) {
  g_noalloc_err = msg;
  return s;
}

// Device address of g_noalloc_scratch on the current device, looked up on every call
// (see the file comment).
gs_status scratch_address(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr)
    return set_error(GS_ECUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
  *out = p;
  return GS_OK;
}

__global__ void plans_from_params(const gs_params* params, int n, int64_t vocab, RowPlan* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = make_plan(params[i], vocab);
}

}  // namespace

const char* noalloc_last_error() { return g_noalloc_err.c_str(); }

}  // namespace gs

using namespace gs;

extern "C" gs_status gs_sample_noalloc(const gs_batch* b, const gs_outputs* o, void* stream) {
  std::string err;
  gs_status s = check_batch(b, o, &err);
  if (s != GS_OK) return set_error(s, err);
  if (b->rows == 0) return GS_OK;
  PlanSummary ps;
  for (int i = 0; i < b->params_count; ++i) ps.add(make_plan(b->params[i], b->vocab));
  if (ps.any_sample && !b->rng_state && !b->uniforms) return set_error(GS_EINVAL, "rng_state or uniforms is required");
  Layout L;
  s = plan_layout(b, ps, &L, &err);
  if (s != GS_OK) return set_error(s, err);
  // scratch: [gs_params of every row, when per-row] [layout: plans | unit stats | candidates |
  //          histogram-path rows' workspace]
  const int np = b->params_count;
  const size_t params_bytes = np > 1 ? align_up(static_cast<size_t>(np) * sizeof(gs_params), 256) : 0;
  const size_t need = params_bytes + L.total;
  if (need > GS_NOALLOC_SCRATCH_BYTES)
    return set_error(GS_EUNSUPPORTED, "request needs " + std::to_string(need) + " bytes of scratch; the allocation-free "
                                      "entry point has " + std::to_string(GS_NOALLOC_SCRATCH_BYTES) +
                                      " (reduce rows or topK, or use gs_sample)");
  void* base = nullptr;
  s = scratch_address(&base);
  if (s != GS_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned char* scratch = static_cast<unsigned char*>(base);
  const RowPlan plan0 = make_plan(b->params[0], b->vocab);
  const RowPlan* dplans = nullptr;
  if (np > 1) {
    gs_params* dparams = reinterpret_cast<gs_params*>(scratch);
    RowPlan* plans = reinterpret_cast<RowPlan*>(scratch + params_bytes + L.plans_off);
    cudaError_t e = cudaMemcpyAsync(dparams, b->params, static_cast<size_t>(np) * sizeof(gs_params),
                                    cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return set_error(GS_ECUDA, std::string("params upload: ") + cudaGetErrorString(e));
    plans_from_params<<<(np + 127) / 128, 128, 0, st>>>(dparams, np, b->vocab, plans);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(GS_ECUDA, std::string("plan kernel: ") + cudaGetErrorString(e));
    dplans = plans;
  }
  void* done = nullptr;
  if (L.step) {
    const cudaError_t e = cudaGetSymbolAddress(&done, g_noalloc_done);
    if (e != cudaSuccess) return set_error(GS_ECUDA, std::string("cudaGetSymbolAddress(counters): ") + cudaGetErrorString(e));
  }
  s = launch_sampling(b, o, L, plan0, dplans, scratch + params_bytes, st, nullptr, &err, nullptr,
                      static_cast<unsigned*>(done));
  if (s != GS_OK) return set_error(s, err);
  return GS_OK;
}
