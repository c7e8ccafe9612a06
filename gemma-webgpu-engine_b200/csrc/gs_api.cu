// Host side of the C ABI declared in include/gsampler.h.
#include "gs_internal.cuh"
#include "gs_plan.cuh"
#include "../../include/gsampler.h"

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <array>
#include <vector>

using namespace gs;

struct gs_ctx {
  int device = 0;
  std::string err;
  // device workspace (plans | unit stats | unit candidates)
  unsigned char* ws = nullptr;
  size_t ws_bytes = 0;
  // pinned staging for per-row plans: a ring of buffers, each with the event guarding its
  // reuse, so that a call waits only for the upload issued kPlanSlots calls earlier
  static constexpr int kPlanSlots = 4;
  RowPlan* plans_host[kPlanSlots] = {};
  size_t plans_cap[kPlanSlots] = {};
  cudaEvent_t plans_ev[kPlanSlots] = {};
  bool plans_ev_live[kPlanSlots] = {};
  int plans_next = 0;
  // device staging of gs_sample_host
  unsigned char* io = nullptr;
  size_t io_bytes = 0;
  unsigned long long* digest = nullptr;
  unsigned* step_done = nullptr;  // [kStepDoneRows] counters of the single-launch decode step (zeroed once)
  int32_t* tok_dev = nullptr;
  double* lp_dev = nullptr;
  size_t tok_cap = 0;
  // kernel timing: events around the streaming pass and the merge of each gs_sample
  bool profile = false;
  std::vector<cudaEvent_t> ev_pool;
  std::vector<std::array<cudaEvent_t, 3>> ev_live;
};

namespace {

gs_status fail(gs_ctx* c, gs_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  return s;
}

gs_status cuda_fail(gs_ctx* c, cudaError_t e, const char* what) {
  return fail(c, GS_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int d) {
    cudaGetDevice(&prev);
    if (prev != d) cudaSetDevice(d);
  }
  ~DeviceGuard() {
    int cur;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

gs_status ensure_ws(gs_ctx* c, size_t bytes) {
  if (bytes <= c->ws_bytes) return GS_OK;
  if (c->ws) {
    cudaDeviceSynchronize();
    cudaFree(c->ws);
    c->ws = nullptr;
    c->ws_bytes = 0;
  }
  const size_t want = align_up(bytes + bytes / 4, 1 << 20);
  cudaError_t e = cudaMalloc(&c->ws, want);
  if (e != cudaSuccess) return fail(c, GS_ENOMEM, "workspace allocation of %zu bytes failed: %s", want, cudaGetErrorString(e));
  c->ws_bytes = want;
  return GS_OK;
}

gs_status ensure_io(gs_ctx* c, size_t bytes) {
  if (bytes <= c->io_bytes) return GS_OK;
  if (c->io) {
    cudaDeviceSynchronize();
    cudaFree(c->io);
    c->io = nullptr;
    c->io_bytes = 0;
  }
  const size_t want = align_up(bytes, 1 << 20);
  cudaError_t e = cudaMalloc(&c->io, want);
  if (e != cudaSuccess) return fail(c, GS_ENOMEM, "staging allocation of %zu bytes failed: %s", want, cudaGetErrorString(e));
  c->io_bytes = want;
  return GS_OK;
}

// Staging slot k for n plans, once the upload that last used it has completed.
gs_status ensure_plans_slot(gs_ctx* c, int k, size_t n) {
  if (c->plans_ev_live[k]) {
    cudaEventSynchronize(c->plans_ev[k]);
    c->plans_ev_live[k] = false;
  }
  if (n <= c->plans_cap[k]) return GS_OK;
  if (c->plans_host[k]) cudaFreeHost(c->plans_host[k]);
  c->plans_host[k] = nullptr;
  c->plans_cap[k] = 0;
  cudaError_t e = cudaMallocHost(&c->plans_host[k], n * sizeof(RowPlan));
  if (e != cudaSuccess) return cuda_fail(c, e, "pinned plan staging");
  c->plans_cap[k] = n;
  return GS_OK;
}

}  // namespace

namespace gs {
int ctx_device(const gs_ctx* c) { return c->device; }
void ctx_set_error(gs_ctx* c, const char* msg) { c->err = msg; }
}  // namespace gs

extern "C" {

gs_status gs_create(int device, gs_ctx** out) {
  if (!out) return GS_EINVAL;
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || device < 0 || device >= n) return GS_ECUDA;
  gs_ctx* c = new gs_ctx();
  c->device = device;
  DeviceGuard g(device);
  for (int k = 0; k < gs_ctx::kPlanSlots && e == cudaSuccess; ++k)
    e = cudaEventCreateWithFlags(&c->plans_ev[k], cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaMalloc(&c->digest, sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMalloc(&c->step_done, kStepDoneRows * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(c->step_done, 0, kStepDoneRows * sizeof(unsigned));
  if (e != cudaSuccess) {
    delete c;
    return GS_ECUDA;
  }
  *out = c;
  return GS_OK;
}

gs_status gs_destroy(gs_ctx* c) {
  if (!c) return GS_OK;
  DeviceGuard g(c->device);
  cudaDeviceSynchronize();
  if (c->ws) cudaFree(c->ws);
  if (c->io) cudaFree(c->io);
  if (c->digest) cudaFree(c->digest);
  if (c->step_done) cudaFree(c->step_done);
  if (c->tok_dev) cudaFree(c->tok_dev);
  if (c->lp_dev) cudaFree(c->lp_dev);
  for (int k = 0; k < gs_ctx::kPlanSlots; ++k) {
    if (c->plans_host[k]) cudaFreeHost(c->plans_host[k]);
    if (c->plans_ev[k]) cudaEventDestroy(c->plans_ev[k]);
  }
  for (auto& evs : c->ev_live)
    for (auto ev : evs) cudaEventDestroy(ev);
  for (auto ev : c->ev_pool) cudaEventDestroy(ev);
  delete c;
  return GS_OK;
}

const char* gs_last_error(const gs_ctx* c) { return c ? c->err.c_str() : noalloc_last_error(); }

gs_status gs_reserve(gs_ctx* c, int32_t rows, int64_t vocab, int32_t max_top_k, int64_t history_stride) {
  if (!c || rows < 0 || vocab <= 0) return GS_EINVAL;
  DeviceGuard g(c->device);
  gs_params p{};
  p.temperature = 1.0;
  p.top_k = std::max(1, std::min(max_top_k, GS_MAX_TOP_K));
  p.top_p = 1;
  p.repetition_penalty = 1;
  gs_batch b{};
  b.rows = rows;
  b.vocab = vocab;
  b.row_stride = vocab;
  b.params = &p;
  b.params_count = 1;
  b.history_stride = history_stride;
  PlanSummary ps;
  ps.add(make_plan(p, vocab));
  Layout L;
  const int32_t dummy = 0;
  if (history_stride > 0) b.history = &dummy;
  gs_status s = plan_layout(&b, ps, &L, &c->err);
  if (s != GS_OK) return s;
  size_t total = L.total;
  if ((max_top_k == 0 || max_top_k > GS_MAX_TOP_K) && vocab > GS_MAX_TOP_K) {
    // rows on the histogram path also need its per-row workspace
    gs_params pl = p;
    pl.top_k = 0;
    PlanSummary pls;
    pls.add(make_plan(pl, vocab));
    Layout LL;
    b.params = &pl;
    s = plan_layout(&b, pls, &LL, &c->err);
    if (s != GS_OK) return s;
    total = std::max(total, LL.total);
  }
  s = ensure_ws(c, total);
  if (s != GS_OK) return s;
  for (int k = 0; k < gs_ctx::kPlanSlots; ++k) {
    s = ensure_plans_slot(c, k, std::max<size_t>(rows, 1));
    if (s != GS_OK) return s;
  }
  return GS_OK;
}

}  // extern "C"

namespace {

// One sampling call: per-row plans (made against `plan_vocab`, the full vocabulary for
// a shard), the work layout, the plan upload and the launches.  `sh` selects a
// vocabulary-sharded mode (nullptr: an ordinary call).
gs_status run_call(gs_ctx* c, const gs_batch* b, const gs_outputs* o, void* stream, const ShardInfo* sh,
                   int64_t plan_vocab) {
  if (b->rows == 0) return GS_OK;
  DeviceGuard g(c->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int np = b->params_count;
  PlanSummary ps;
  for (int i = 0; i < np; ++i) ps.add(make_plan(b->params[i], plan_vocab));
  const int smode = sh ? sh->mode : 0;
  if (smode != 1 && ps.any_sample && !b->rng_state && !b->uniforms)
    return fail(c, GS_EINVAL, "rng_state or uniforms is required");
  if (smode && ps.any_large)
    return fail(c, GS_EUNSUPPORTED, "vocabulary-sharded mode needs 1 <= topK <= %d (or temperature 0)", GS_MAX_TOP_K);
  Layout L;
  gs_status s = smode == 2 ? plan_merge_layout(b, ps, *sh, &L, &c->err) : plan_layout(b, ps, &L, &c->err);
  if (s != GS_OK) return s;
  s = ensure_ws(c, L.total);
  if (s != GS_OK) return s;
  const RowPlan plan0 = make_plan(b->params[0], plan_vocab);
  const RowPlan* dplans = nullptr;
  if (np > 1) {
    const int k = c->plans_next;
    c->plans_next = (k + 1) % gs_ctx::kPlanSlots;
    s = ensure_plans_slot(c, k, np);
    if (s != GS_OK) return s;
    RowPlan* staged = c->plans_host[k];
    for (int i = 0; i < np; ++i) staged[i] = make_plan(b->params[i], plan_vocab);
    dplans = reinterpret_cast<const RowPlan*>(c->ws + L.plans_off);
    cudaError_t e = cudaMemcpyAsync(const_cast<RowPlan*>(dplans), staged, np * sizeof(RowPlan),
                                    cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(c, e, "plan upload");
    cudaEventRecord(c->plans_ev[k], st);
    c->plans_ev_live[k] = true;
  }
  std::array<cudaEvent_t, 3> evs{};
  if (c->profile) {
    for (auto& ev : evs) {
      if (c->ev_pool.empty()) {
        cudaEvent_t ne;
        if (cudaEventCreate(&ne) != cudaSuccess) return fail(c, GS_ECUDA, "event creation");
        c->ev_pool.push_back(ne);
      }
      ev = c->ev_pool.back();
      c->ev_pool.pop_back();
    }
  }
  gs_outputs none{};
  s = launch_sampling(b, o ? o : &none, L, plan0, dplans, c->ws, st, c->profile ? evs.data() : nullptr, &c->err, sh,
                      c->step_done);
  if (s != GS_OK) return s;
  if (c->profile) c->ev_live.push_back(evs);
  return GS_OK;
}

// Record geometry of a vocabulary-sharded batch: packs = the largest k of its rows,
// penalised slots = the history stride.
void shard_geometry(const gs_batch* b, int64_t vocab_total, ShardInfo* sh) {
  int k = 1;
  for (int i = 0; i < b->params_count; ++i) k = std::max(k, make_plan(b->params[i], vocab_total).k_eff);
  sh->rec_kcap = k;
  sh->rec_hcap = b->history ? static_cast<int>(b->history_stride) : 0;
  sh->rec_bytes = shard_record_bytes(sh->rec_kcap, sh->rec_hcap);
}

}  // namespace

extern "C" {

gs_status gs_sample(gs_ctx* c, const gs_batch* b, const gs_outputs* o, void* stream) {
  if (!c) return GS_EINVAL;
  gs_status s = check_batch(b, o, &c->err);
  if (s != GS_OK) return s;
  return run_call(c, b, o, stream, nullptr, b->vocab);
}

gs_status gs_sample_host(gs_ctx* c, const gs_batch* hb, const gs_outputs* ho, void* stream) {
  if (!c) return GS_EINVAL;
  gs_status s = check_batch(hb, ho, &c->err);
  if (s != GS_OK) return s;
  if (hb->rows == 0) return GS_OK;
  DeviceGuard g(c->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t rows = hb->rows;
  const size_t esz = hb->dtype == GS_DTYPE_F32 ? 4 : 2;
  // staging layout
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  const size_t o_logits = take(static_cast<size_t>(rows) * hb->row_stride * esz);
  const size_t o_hist = hb->history ? take(static_cast<size_t>(rows) * hb->history_stride * 4) : 0;
  const size_t o_hlen = hb->history ? take(static_cast<size_t>(rows) * 4) : 0;
  const bool hcounts = hb->history && hb->history_count;
  const size_t o_hcnt = hcounts ? take(static_cast<size_t>(rows) * hb->history_stride * 4) : 0;
  const size_t o_mstate = hb->mask_table ? take(static_cast<size_t>(rows) * 4) : 0;
  const size_t o_rng = hb->rng_state ? take(static_cast<size_t>(rows) * 8) : 0;
  const size_t o_uni = hb->uniforms ? take(static_cast<size_t>(rows) * 8) : 0;
  const size_t o_ids = take(static_cast<size_t>(rows) * 4);
  const size_t o_lp = ho->logprob ? take(static_cast<size_t>(rows) * 8) : 0;
  const size_t o_fl = take(static_cast<size_t>(rows) * 4);
  const size_t o_cid = ho->cand_ids ? take(static_cast<size_t>(rows) * ho->cand_cap * 4) : 0;
  const size_t o_cp = ho->cand_probs ? take(static_cast<size_t>(rows) * ho->cand_cap * 8) : 0;
  const size_t o_cc = ho->cand_count ? take(static_cast<size_t>(rows) * 4) : 0;
  s = ensure_io(c, off);
  if (s != GS_OK) return s;
  unsigned char* io = c->io;
  auto h2d = [&](size_t at, const void* src, size_t bytes) {
    return cudaMemcpyAsync(io + at, src, bytes, cudaMemcpyHostToDevice, st);
  };
  cudaError_t e = h2d(o_logits, hb->logits, static_cast<size_t>(rows) * hb->row_stride * esz);
  if (hb->history && e == cudaSuccess) e = h2d(o_hist, hb->history, static_cast<size_t>(rows) * hb->history_stride * 4);
  if (hb->history && e == cudaSuccess) e = h2d(o_hlen, hb->history_len, static_cast<size_t>(rows) * 4);
  if (hcounts && e == cudaSuccess) e = h2d(o_hcnt, hb->history_count, static_cast<size_t>(rows) * hb->history_stride * 4);
  if (hb->mask_table && e == cudaSuccess) e = h2d(o_mstate, hb->mask_state, static_cast<size_t>(rows) * 4);
  if (hb->rng_state && e == cudaSuccess) e = h2d(o_rng, hb->rng_state, static_cast<size_t>(rows) * 8);
  if (hb->uniforms && e == cudaSuccess) e = h2d(o_uni, hb->uniforms, static_cast<size_t>(rows) * 8);
  if (e != cudaSuccess) return cuda_fail(c, e, "input upload");
  gs_batch db = *hb;
  db.logits = io + o_logits;
  db.history = hb->history ? reinterpret_cast<const int32_t*>(io + o_hist) : nullptr;
  db.history_len = hb->history ? reinterpret_cast<const int32_t*>(io + o_hlen) : nullptr;
  db.history_count = hcounts ? reinterpret_cast<const int32_t*>(io + o_hcnt) : nullptr;
  db.mask_state = hb->mask_table ? reinterpret_cast<const int32_t*>(io + o_mstate) : nullptr;
  db.rng_state = hb->rng_state ? reinterpret_cast<double*>(io + o_rng) : nullptr;
  db.uniforms = hb->uniforms ? reinterpret_cast<const double*>(io + o_uni) : nullptr;
  gs_outputs dout{};
  dout.ids = reinterpret_cast<int32_t*>(io + o_ids);
  dout.logprob = ho->logprob ? reinterpret_cast<double*>(io + o_lp) : nullptr;
  dout.flags = reinterpret_cast<uint32_t*>(io + o_fl);
  dout.cand_ids = ho->cand_ids ? reinterpret_cast<int32_t*>(io + o_cid) : nullptr;
  dout.cand_probs = ho->cand_probs ? reinterpret_cast<double*>(io + o_cp) : nullptr;
  dout.cand_count = ho->cand_count ? reinterpret_cast<int32_t*>(io + o_cc) : nullptr;
  dout.cand_cap = ho->cand_cap;
  s = gs_sample(c, &db, &dout, stream);
  if (s != GS_OK) return s;
  std::vector<uint32_t> flags_local;
  uint32_t* flags_host = ho->flags;
  if (!flags_host) {
    flags_local.resize(rows);
    flags_host = flags_local.data();
  }
  auto d2h = [&](void* dst, size_t at, size_t bytes) {
    return cudaMemcpyAsync(dst, io + at, bytes, cudaMemcpyDeviceToHost, st);
  };
  e = d2h(ho->ids, o_ids, rows * 4);
  if (e == cudaSuccess) e = d2h(flags_host, o_fl, rows * 4);
  if (ho->logprob && e == cudaSuccess) e = d2h(ho->logprob, o_lp, rows * 8);
  if (ho->cand_ids && e == cudaSuccess) e = d2h(ho->cand_ids, o_cid, rows * ho->cand_cap * 4);
  if (ho->cand_probs && e == cudaSuccess) e = d2h(ho->cand_probs, o_cp, rows * ho->cand_cap * 8);
  if (ho->cand_count && e == cudaSuccess) e = d2h(ho->cand_count, o_cc, rows * 4);
  if (hb->rng_state && e == cudaSuccess) e = d2h(hb->rng_state, o_rng, rows * 8);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(c, e, "sampling");
  for (int64_t r = 0; r < rows; ++r) {
    const uint32_t f = flags_host[r];
    if (f & GS_FLAG_ERR_DEADEND) return fail(c, GS_EDEADEND, "Generation constraint reached a tokenization dead end");
    if (f & GS_FLAG_ERR_NONFINITE) return fail(c, GS_ENONFINITE, "row %lld: logits contain NaN or +Infinity", static_cast<long long>(r));
    if (f & GS_FLAG_ERR_INVALID) return fail(c, GS_EINVAL, "row %lld: mask state out of range", static_cast<long long>(r));
    if (f & GS_FLAG_ERR_UNSUPPORTED) return fail(c, GS_EUNSUPPORTED, "row %lld: request outside the histogram path", static_cast<long long>(r));
    if (f & GS_FLAG_ERR_TIMEOUT) return fail(c, GS_ETIMEOUT, "row %lld: device wait timed out", static_cast<long long>(r));
  }
  return GS_OK;
}

gs_status gs_token_log_probability(gs_ctx* c, const void* logits, int32_t dtype, int32_t rows, int64_t vocab,
                                   int64_t row_stride, float softcap, const int32_t* tokens, double* out, void* stream) {
  if (!c) return GS_EINVAL;
  if (rows < 0 || (rows > 0 && (!logits || !tokens || !out))) return fail(c, GS_EINVAL, "bad arguments");
  if (row_stride < vocab) return fail(c, GS_EINVAL, "row_stride must be >= vocab");
  DeviceGuard g(c->device);
  for (int r = 0; r < rows; ++r)
    if (tokens[r] < 0 || tokens[r] >= vocab)
      return fail(c, GS_EINVAL, "Token %d is outside logits length %lld", tokens[r], static_cast<long long>(vocab));
  if (rows == 0) return GS_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (static_cast<size_t>(rows) > c->tok_cap) {
    if (c->tok_dev) cudaFree(c->tok_dev);
    if (c->lp_dev) cudaFree(c->lp_dev);
    c->tok_dev = nullptr;
    c->lp_dev = nullptr;
    c->tok_cap = 0;
    if (cudaMalloc(&c->tok_dev, rows * 4) != cudaSuccess || cudaMalloc(&c->lp_dev, rows * 8) != cudaSuccess)
      return fail(c, GS_ENOMEM, "log-probability staging");
    c->tok_cap = rows;
  }
  cudaError_t e = cudaMemcpyAsync(c->tok_dev, tokens, rows * 4, cudaMemcpyHostToDevice, st);
  const float inv = softcap != 0.0f ? static_cast<float>(1.0 / static_cast<double>(softcap)) : 0.0f;
  if (e == cudaSuccess) e = launch_logprob(logits, dtype, rows, vocab, row_stride, softcap, inv, c->tok_dev, c->lp_dev, nullptr, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, c->lp_dev, rows * 8, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(c, e, "log probability");
  return GS_OK;
}

gs_status gs_mask_constraint_logits(gs_ctx* c, const float* raw, int64_t vocab, const int32_t* legal, int64_t n_legal,
                                    const int32_t* term, int64_t n_term, float* out, void* stream) {
  if (!c) return GS_EINVAL;
  if (vocab < 0 || (vocab > 0 && (!raw || !out)) || (n_legal > 0 && !legal) || (n_term > 0 && !term))
    return fail(c, GS_EINVAL, "bad arguments");
  DeviceGuard g(c->device);
  cudaError_t e = launch_mask_logits(raw, vocab, legal, n_legal, term, n_term, out, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GS_OK : cuda_fail(c, e, "mask");
}

gs_status gs_build_mask_row(gs_ctx* c, int64_t vocab, const int32_t* legal, int64_t n_legal, const int32_t* term,
                            int64_t n_term, uint32_t* row_out, void* stream) {
  if (!c) return GS_EINVAL;
  if (vocab <= 0 || !row_out || (n_legal > 0 && !legal) || (n_term > 0 && !term)) return fail(c, GS_EINVAL, "bad arguments");
  DeviceGuard g(c->device);
  cudaError_t e = launch_build_mask_row(vocab, legal, n_legal, term, n_term, row_out, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GS_OK : cuda_fail(c, e, "mask row");
}

gs_status gs_build_reasoning_mask_rows(gs_ctx* c, int64_t vocab, const uint8_t* has_bytes, int32_t end_channel_id,
                                       uint32_t* rows_out, int64_t mask_words, void* stream) {
  if (!c) return GS_EINVAL;
  if (vocab <= 0 || !has_bytes || !rows_out || mask_words < (vocab + 31) / 32) return fail(c, GS_EINVAL, "bad arguments");
  DeviceGuard g(c->device);
  cudaError_t e = launch_reasoning_rows(vocab, has_bytes, end_channel_id, rows_out, mask_words,
                                        static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GS_OK : cuda_fail(c, e, "reasoning mask rows");
}

gs_status gs_softcap(gs_ctx* c, const float* in, float* out, int64_t n, float cap, void* stream) {
  if (!c) return GS_EINVAL;
  if (n < 0 || (n > 0 && (!in || !out)) || !(cap > 0) || !std::isfinite(cap)) return fail(c, GS_EINVAL, "bad arguments");
  DeviceGuard g(c->device);
  const float inv = static_cast<float>(1.0 / static_cast<double>(cap));
  cudaError_t e = launch_softcap(in, out, n, cap, inv, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GS_OK : cuda_fail(c, e, "softcap");
}

gs_status gs_softcap_digest(gs_ctx* c, uint64_t lo, uint64_t hi, float cap, uint64_t* digest_host) {
  if (!c) return GS_EINVAL;
  if (!digest_host || hi < lo || hi > (1ull << 32) || !(cap > 0)) return fail(c, GS_EINVAL, "bad arguments");
  DeviceGuard g(c->device);
  const float inv = static_cast<float>(1.0 / static_cast<double>(cap));
  cudaError_t e = launch_softcap_digest(lo, hi, cap, inv, c->digest, nullptr);
  unsigned long long v = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&v, c->digest, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(c, e, "softcap digest");
  *digest_host = v;
  return GS_OK;
}

gs_status gs_profile_enable(gs_ctx* c, int32_t enable) {
  if (!c) return GS_EINVAL;
  c->profile = enable != 0;
  return GS_OK;
}

gs_status gs_profile_read(gs_ctx* c, double* stream_ms, int64_t* stream_launches, double* merge_ms,
                          int64_t* merge_launches) {
  if (!c) return GS_EINVAL;
  DeviceGuard g(c->device);
  double s_ms = 0, m_ms = 0;
  int64_t n = 0;
  for (auto& evs : c->ev_live) {
    cudaError_t e = cudaEventSynchronize(evs[2]);
    if (e != cudaSuccess) return cuda_fail(c, e, "profile read");
    float a = 0, b = 0;
    cudaEventElapsedTime(&a, evs[0], evs[1]);
    cudaEventElapsedTime(&b, evs[1], evs[2]);
    s_ms += a;
    m_ms += b;
    ++n;
    for (auto ev : evs) c->ev_pool.push_back(ev);
  }
  c->ev_live.clear();
  if (stream_ms) *stream_ms = s_ms;
  if (stream_launches) *stream_launches = n;
  if (merge_ms) *merge_ms = m_ms;
  if (merge_launches) *merge_launches = n;
  return GS_OK;
}

int64_t gs_shard_record_bytes(const gs_params* params, int32_t params_count, int64_t vocab_total,
                              int64_t history_stride) {
  if (!params || params_count <= 0 || vocab_total <= 0 || history_stride < 0) return -1;
  gs_batch b{};
  b.params = params;
  b.params_count = params_count;
  b.history_stride = history_stride;
  const int32_t dummy = 0;
  if (history_stride > 0) b.history = &dummy;
  ShardInfo sh;
  shard_geometry(&b, vocab_total, &sh);
  return sh.rec_bytes;
}

gs_status gs_shard_partials(gs_ctx* c, const gs_batch* shard, int64_t vocab_offset, int64_t vocab_total,
                            int32_t want_logprob, void* records, void* stream) {
  if (!c) return GS_EINVAL;
  gs_status s = check_batch(shard, nullptr, &c->err, kCheckNoOutputs);
  if (s != GS_OK) return s;
  if (!records && shard->rows > 0) return fail(c, GS_EINVAL, "records is NULL");
  if (vocab_offset < 0 || vocab_offset % 4096 != 0 || vocab_offset + shard->vocab > vocab_total ||
      vocab_total >= (1ll << 31))
    return fail(c, GS_EINVAL, "a shard starts at a multiple of 4096 ids inside [0, vocab_total)");
  if (shard->mask_table && shard->mask_words * 32 < vocab_total)
    return fail(c, GS_EINVAL, "mask_words must cover the whole vocabulary (>= ceil(vocab_total/32))");
  ShardInfo sh;
  sh.mode = 1;
  sh.vocab_offset = vocab_offset;
  shard_geometry(shard, vocab_total, &sh);
  sh.records = static_cast<unsigned char*>(records);
  sh.want_raw = want_logprob != 0;
  return run_call(c, shard, nullptr, stream, &sh, vocab_total);
}

gs_status gs_shard_merge(gs_ctx* c, const gs_batch* full, int32_t shards, const void* gathered,
                         const gs_outputs* out, void* stream) {
  if (!c) return GS_EINVAL;
  gs_status s = check_batch(full, out, &c->err, kCheckNoLogits);
  if (s != GS_OK) return s;
  if (shards < 1 || (!gathered && full->rows > 0)) return fail(c, GS_EINVAL, "shards >= 1 and gathered records are required");
  ShardInfo sh;
  sh.mode = 2;
  sh.shards = shards;
  shard_geometry(full, full->vocab, &sh);
  sh.records = static_cast<unsigned char*>(const_cast<void*>(gathered));
  return run_call(c, full, out, stream, &sh, full->vocab);
}

}  // extern "C"
