// Host-side planning shared by gs_sample, gs_sample_host and gs_sample_noalloc.
#include "gs_plan.cuh"

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <vector>

namespace gs {

int pipe_max_k();
int sm_count();
int64_t pipe_max_chunk();

namespace {

gs_status fmt(std::string* err, gs_status s, const char* f, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, sizeof(buf), f, ap);
  va_end(ap);
  if (err) *err = buf;
  return s;
}

int pow2ceil(int64_t n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

}  // namespace

bool valid_params(const gs_params& p, std::string* why) {
  std::vector<std::string> errors;
  if (!std::isfinite(p.temperature) || p.temperature < 0) errors.push_back("temperature must be >= 0");
  if (p.top_k < 0) errors.push_back("topK must be a non-negative integer");
  const double v3[3] = {p.top_p, p.min_p, p.typical_p};
  const char* n3[3] = {"topP", "minP", "typicalP"};
  for (int i = 0; i < 3; ++i)
    if (!std::isfinite(v3[i]) || v3[i] < 0 || v3[i] > 1) errors.push_back(std::string(n3[i]) + " must be between 0 and 1");
  if (!std::isfinite(p.repetition_penalty) || p.repetition_penalty <= 0) errors.push_back("repetitionPenalty must be > 0");
  if (!std::isfinite(p.frequency_penalty) || p.frequency_penalty < 0)
    errors.push_back("frequencyPenalty must be finite and non-negative");
  if (!std::isfinite(p.presence_penalty) || p.presence_penalty < 0)
    errors.push_back("presencePenalty must be finite and non-negative");
  if (errors.empty()) return true;
  std::string s = "Invalid Gemma decoding config: ";
  for (size_t i = 0; i < errors.size(); ++i) s += (i ? "; " : "") + errors[i];
  if (why) *why = s;
  return false;
}

gs_status check_batch(const gs_batch* b, const gs_outputs* o, std::string* err, unsigned what) {
  if (!b || (!o && !(what & kCheckNoOutputs))) return fmt(err, GS_EINVAL, "batch and outputs are required");
  if (b->rows < 0) return fmt(err, GS_EINVAL, "rows must be >= 0");
  if (b->vocab <= 0) return fmt(err, GS_EEMPTY, "Cannot sample empty logits");
  if (b->vocab >= (1ll << 31)) return fmt(err, GS_EINVAL, "vocab must be below 2^31");
  if (b->row_stride < b->vocab) return fmt(err, GS_EINVAL, "row_stride must be >= vocab");
  if (b->dtype != GS_DTYPE_F32 && b->dtype != GS_DTYPE_BF16) return fmt(err, GS_EINVAL, "unknown dtype %d", b->dtype);
  if (b->rows > 0 && !b->logits && !(what & kCheckNoLogits)) return fmt(err, GS_EINVAL, "logits is NULL");
  if (!(b->softcap >= 0) || !std::isfinite(b->softcap)) return fmt(err, GS_EINVAL, "softcap must be finite and >= 0");
  if (!b->params || (b->params_count != 1 && b->params_count != b->rows))
    return fmt(err, GS_EINVAL, "params_count must be 1 or rows");
  if (b->history && (b->history_stride < 0 || b->history_stride > GS_MAX_HISTORY))
    return fmt(err, GS_EUNSUPPORTED, "history_stride must be in [0, %d]", GS_MAX_HISTORY);
  if (b->history && !b->history_len) return fmt(err, GS_EINVAL, "history_len is required with history");
  if (b->mask_table) {
    if (!b->mask_state) return fmt(err, GS_EINVAL, "mask_state is required with mask_table");
    if (b->mask_words < (b->vocab + 31) / 32) return fmt(err, GS_EINVAL, "mask_words must be >= ceil(vocab/32)");
    if (b->mask_states <= 0) return fmt(err, GS_EINVAL, "mask_states must be > 0");
  }
  if (o) {
    if (b->rows > 0 && !o->ids) return fmt(err, GS_EINVAL, "outputs.ids is NULL");
    if (o->cand_ids && o->cand_cap <= 0) return fmt(err, GS_EINVAL, "cand_cap must be > 0 with cand_ids");
  }
  for (int i = 0; i < b->params_count; ++i)
    if (!valid_params(b->params[i], err)) return GS_EINVAL;
  return GS_OK;
}

gs_status plan_layout(const gs_batch* b, const PlanSummary& ps, Layout* L, std::string* err) {
  const int rows = b->rows;
  const int kmax = ps.kmax;
  // Vocabulary splits.  The warp-per-unit streaming kernels (small topK, aligned rows)
  // want one wave of units: the most units per row (a power of two) that keep the batch
  // within the GPU's warp slots (16 per SM), since a unit has fixed costs (its penalised
  // list, the first sub-tile's threshold, its candidate list and statistics) that longer
  // units spread.  (Measured at C3's 256 masked rows: 8 units a row 139 us a step, 64 units
  // 201 us; C4's 4096 rows: one unit a row 773 us, four 827 us.)  A unit keeps at most 256
  // penalised ids in its sorted list (more: a per-tile scan of the history), so a history
  // of more than 256 ids is spread at about 128 ids a unit.  The general kernel wants
  // about four CTAs per SM and chunks of >= 4096 ids.  Both keep at most 16384 streamed
  // candidates per row for the merge.
  const int64_t V = b->vocab;
  const int esz = b->dtype == GS_DTYPE_F32 ? 4 : 2;
  const bool aligned = (reinterpret_cast<uintptr_t>(b->logits) & 15) == 0 && ((b->row_stride * esz) & 15) == 0 &&
                       (!b->mask_table || ((reinterpret_cast<uintptr_t>(b->mask_table) & 15) == 0 && (b->mask_words & 3) == 0));
  const bool warp_kernel = kmax <= pipe_max_k() && aligned;
  const int sms = sm_count();  // (cached per device)
  const int64_t min_chunk = warp_kernel ? 2048 : 4096;
  const int64_t granule = warp_kernel ? 1024 : 4096;
  auto can_split = [&](int s) { return V / (2 * s) >= min_chunk && 2 * s * std::max(kmax, 1) <= 16384 && s < 1024; };
  int S = 1;
  if (warp_kernel) {
    const int64_t slots = static_cast<int64_t>(sms) * 16;
    while (static_cast<int64_t>(rows) * S * 2 <= slots && can_split(S)) S *= 2;
    const int64_t hs = b->history ? b->history_stride : 0;
    if (hs > 256)
      while (hs > 128 * static_cast<int64_t>(S) && can_split(S)) S *= 2;
    const int64_t need = (V + pipe_max_chunk() - 1) / pipe_max_chunk();
    while (S < need) S *= 2;
  } else {
    while (static_cast<int64_t>(rows) * S < static_cast<int64_t>(sms) * 4 && can_split(S)) S *= 2;
  }
  int64_t chunk = (V + S - 1) / S;
  chunk = (chunk + granule - 1) / granule * granule;
  S = static_cast<int>((V + chunk - 1) / chunk);
  const int kcap = std::max(kmax, 1);
  int kc = 256;
  while (kc < 2 * kmax) kc <<= 1;
  if (kc > 4096) return fmt(err, GS_EUNSUPPORTED, "topK above %d is not supported by the streaming buffer", GS_MAX_TOP_K);
  L->splits = S;
  L->chunk = chunk;
  L->kcap = kcap;
  L->kc = kc;
  L->kmax = kmax;
  L->any_large = ps.any_large;
  L->any_typical_large = ps.any_typical_large;
  L->any_small = ps.any_small;
  L->any_sample = ps.any_sample;
  const int64_t units = static_cast<int64_t>(rows) * S;
  L->plans_off = 0;
  L->stats_off = align_up(static_cast<size_t>(rows) * sizeof(RowPlan), 256);
  L->cands_off = align_up(L->stats_off + static_cast<size_t>(units) * sizeof(UnitStat), 256);
  L->rowtau_off = align_up(L->cands_off + static_cast<size_t>(units) * kcap * 8, 256);
  L->large_off = align_up(L->rowtau_off + static_cast<size_t>(rows) * 8, 256);
  L->large_row = ps.any_large ? large_row_bytes(b->history ? b->history_stride : 0) : 0;
  L->total = L->large_off + static_cast<size_t>(rows) * L->large_row;
  L->stream_smem = stream_smem_bytes(chunk, kc);
  const int64_t hs = b->history ? b->history_stride : 0;
  L->hist_cap = pow2ceil(std::max<int64_t>(hs, 1));
  L->pack_cap = S > 1 ? S * kcap : 0;
  L->ent_cap = pow2ceil(std::max<int64_t>(std::min<int64_t>(static_cast<int64_t>(S) * kcap, kmax) + hs, 1));
  L->work_cap = std::min(pow2ceil(std::max(kmax, 1)), 1024);
  // (with history counts the block merge sorts 64-bit (id, count) words: twice the bytes)
  L->fin_smem = finalize_smem_bytes(L->hist_cap * (b->history && b->history_count ? 2 : 1), L->ent_cap, L->pack_cap,
                                    L->work_cap);
  if (L->fin_smem > 220 * 1024)
    return fmt(err, GS_EUNSUPPORTED, "merge needs %zu bytes of shared memory (topK %d, history %lld)", L->fin_smem, kmax,
               static_cast<long long>(hs));
  L->large_smem = ps.any_large ? large_select_smem_bytes(hs) : 0;
  L->step = step_eligible(b, kmax, ps.any_large, rows);
  L->step_off = 0;
  if (L->step) {
    L->step_off = align_up(L->total, 256);
    L->total = L->step_off + step_ws_bytes(rows, V, kmax);
  }
  return GS_OK;
}

gs_status plan_merge_layout(const gs_batch* b, const PlanSummary& ps, const ShardInfo& sh, Layout* L,
                            std::string* err) {
  const int rows = b->rows;
  L->splits = sh.shards;
  L->chunk = 0;
  L->kcap = sh.rec_kcap;
  L->kc = 0;
  L->kmax = ps.kmax;
  L->any_large = ps.any_large;
  L->any_typical_large = false;
  L->any_small = ps.any_small;
  L->any_sample = ps.any_sample;
  L->plans_off = 0;
  L->stats_off = align_up(static_cast<size_t>(rows) * sizeof(RowPlan), 256);
  L->cands_off = L->stats_off;
  L->rowtau_off = L->stats_off;
  L->large_off = L->stats_off;
  L->large_row = 0;
  L->step = false;
  L->step_off = 0;
  L->total = L->stats_off;
  L->stream_smem = 0;
  L->hist_cap = 1;
  L->pack_cap = sh.shards * sh.rec_kcap;
  L->ent_cap = pow2ceil(std::max<int64_t>(static_cast<int64_t>(sh.shards) * sh.rec_hcap + ps.kmax, 1));
  L->work_cap = std::min(pow2ceil(std::max(ps.kmax, 1)), 1024);
  L->fin_smem = finalize_smem_bytes(L->hist_cap, L->ent_cap, L->pack_cap, L->work_cap);
  L->large_smem = 0;
  if (L->fin_smem > 220 * 1024)
    return fmt(err, GS_EUNSUPPORTED, "merge of %d shards needs %zu bytes of shared memory", sh.shards, L->fin_smem);
  return GS_OK;
}

gs_status launch_sampling(const gs_batch* b, const gs_outputs* o, const Layout& L, const RowPlan& plan0,
                          const RowPlan* dplans, unsigned char* ws, cudaStream_t st, cudaEvent_t* events,
                          std::string* err, const ShardInfo* shard, unsigned* step_done) {
  if (L.step && step_done && !shard) {
    // one launch: streaming, merge, filters and draw (gs_step.cu)
    if (events) cudaEventRecord(events[0], st);
    const cudaError_t e = launch_step(b, o, plan0, dplans, L.kmax, ws + L.step_off, step_done, st);
    if (e != cudaSuccess) return fmt(err, GS_ECUDA, "decode step launch: %s", cudaGetErrorString(e));
    if (events) {
      cudaEventRecord(events[1], st);
      cudaEventRecord(events[2], st);
    }
    return GS_OK;
  }
  UnitStat* stats = reinterpret_cast<UnitStat*>(ws + L.stats_off);
  unsigned long long* cands = reinterpret_cast<unsigned long long*>(ws + L.cands_off);
  const int smode = shard ? shard->mode : 0;
  const int rows = b->rows;
  const float cap = b->softcap;
  const float inv_cap = cap != 0.0f ? static_cast<float>(1.0 / static_cast<double>(cap)) : 0.0f;
  StreamArgs sa{};
  sa.logits = b->logits;
  sa.vocab = b->vocab;
  sa.row_stride = b->row_stride;
  sa.vocab_offset = smode == 1 ? shard->vocab_offset : 0;
  sa.softcap = cap;
  sa.inv_softcap = inv_cap;
  sa.want_raw = smode == 1 ? shard->want_raw : o->logprob != nullptr;
  sa.splits = L.splits;
  sa.chunk = L.chunk;
  sa.kcap = L.kcap;
  sa.kc = L.kc;
  sa.kmax = L.kmax;
  sa.plans = dplans;
  sa.plan0 = plan0;
  sa.history = b->history;
  sa.history_len = b->history ? b->history_len : nullptr;
  sa.history_stride = b->history ? b->history_stride : 0;
  // (a shard reads its own words of each state's row: the table pointer moves, the row
  // stride stays)
  sa.mask_table = b->mask_table && smode == 1 ? b->mask_table + (shard->vocab_offset >> 5) : b->mask_table;
  sa.mask_states = b->mask_states;
  sa.mask_words = b->mask_words;
  sa.mask_state = b->mask_table ? b->mask_state : nullptr;
  sa.stats = stats;
  sa.cands = cands;
  sa.row_tau = nullptr;
  // (rows on the histogram path take no streaming pass: the histogram kernel computes
  // their statistics; with no other rows the pass is not launched)
  const bool stream_pass = smode != 2 && L.any_small;
  if (stream_pass && L.kmax > 1) {
    sa.row_tau = reinterpret_cast<unsigned long long*>(ws + L.rowtau_off);
    cudaMemsetAsync(sa.row_tau, 0, static_cast<size_t>(rows) * 8, st);
  }
  if (events) cudaEventRecord(events[0], st);
  cudaError_t e = cudaSuccess;
  if (stream_pass) {
    e = launch_stream(sa, b->dtype, rows, L.stream_smem, st);
    if (e != cudaSuccess) return fmt(err, GS_ECUDA, "streaming pass launch: %s", cudaGetErrorString(e));
  }
  if (events) cudaEventRecord(events[1], st);

  FinalizeArgs fa{};
  fa.logits = b->logits;
  fa.vocab = b->vocab;
  fa.row_stride = b->row_stride;
  fa.softcap = cap;
  fa.inv_softcap = inv_cap;
  fa.want_raw = sa.want_raw;
  fa.splits = L.splits;
  fa.kcap = L.kcap;
  fa.hist_cap = L.hist_cap;
  fa.ent_cap = L.ent_cap;
  fa.pack_cap = L.pack_cap;
  fa.work_cap = L.work_cap;
  fa.plans = dplans;
  fa.plan0 = plan0;
  fa.history = sa.history;
  fa.history_len = sa.history_len;
  // (the merge of gathered shard records reads no history: its records hold the scores)
  fa.history_count = smode == 2 || !b->history ? nullptr : b->history_count;
  fa.history_stride = sa.history_stride;
  fa.mask_table = sa.mask_table;
  fa.mask_states = b->mask_states;
  fa.mask_words = b->mask_words;
  fa.mask_state = sa.mask_state;
  fa.stats = stats;
  fa.cands = cands;
  fa.rng_state = b->rng_state;
  fa.uniforms = b->uniforms;
  fa.ids = o->ids;
  fa.logprob = o->logprob;
  fa.flags = o->flags;
  fa.cand_ids = o->cand_ids;
  fa.cand_probs = o->cand_probs;
  fa.cand_count = o->cand_count;
  fa.cand_cap = o->cand_cap;
  fa.lws = ws + L.large_off;
  fa.lrow_bytes = static_cast<int64_t>(L.large_row);
  fa.lslots = static_cast<int32_t>(sa.history_stride);
  fa.lmoments = L.any_typical_large ? 1 : 0;
  if (smode) {
    fa.shard_mode = smode;
    fa.shards = shard->shards;
    fa.vocab_offset = smode == 1 ? shard->vocab_offset : 0;
    fa.rec_bytes = shard->rec_bytes;
    fa.rec_kcap = shard->rec_kcap;
    fa.rec_hcap = shard->rec_hcap;
    fa.records = shard->records;
    if (smode == 1) {  // partials: the merge writes only the records
      fa.ids = nullptr;
      fa.logprob = nullptr;
      fa.flags = nullptr;
      fa.cand_ids = nullptr;
      fa.cand_probs = nullptr;
      fa.cand_count = nullptr;
      fa.rng_state = nullptr;
      fa.uniforms = nullptr;
    }
  }
  if (L.any_small) {
    // One warp per row pays off when the rows fill the GPU several times over; fewer rows
    // merge faster with a CTA each (C4's settings on one B200, merge time, warp / CTA per
    // row: 512 rows 51.6 / 37.4 us, 1024 rows 56.7 / 66.7 us, 4096 rows 105 / 183 us).
    size_t wsmem = 0;
    if (rows >= 5 * sm_count() && finalize_warp_eligible(fa, L.kmax, &wsmem)) {
      e = launch_finalize_warp(fa, b->dtype, rows, L.kmax, st);
    } else {
      e = launch_finalize(fa, b->dtype, rows, L.fin_smem, st);
    }
    if (e != cudaSuccess) return fmt(err, GS_ECUDA, "merge launch: %s", cudaGetErrorString(e));
  }
  if (L.any_large) {
    e = launch_large(fa, b->dtype, rows, L.large_smem, st);
    if (e != cudaSuccess) return fmt(err, GS_ECUDA, "histogram path launch: %s", cudaGetErrorString(e));
  }
  if (events) cudaEventRecord(events[2], st);
  return GS_OK;
}

}  // namespace gs
