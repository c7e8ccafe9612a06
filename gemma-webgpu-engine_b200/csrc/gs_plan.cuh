// Planning shared by the entry points: per-row plans, work layout, argument checks and
// the launch sequence of one sampling call.
#pragma once
#include <cfloat>
#include <cstddef>
#include <string>

#include "gs_internal.cuh"
#include "../../include/gsampler.h"

namespace gs {

// Per-row plan from one DecodingConfig (the fields sampleToken reads).
__host__ __device__ inline RowPlan make_plan(const gs_params& p, int64_t vocab) {
  RowPlan r{};
  r.temperature = p.temperature;
  r.top_p = p.top_p;
  r.min_p = p.min_p;
  r.typical_p = p.typical_p;
  r.repetition_penalty = p.repetition_penalty;
  r.presence_penalty = p.presence_penalty;
  r.frequency_penalty = p.frequency_penalty;
  r.top_k = p.top_k;
  if (p.temperature == 0) {
    r.mode = kModeGreedy;
    r.k_eff = 1;
    r.a2 = 0;
    r.a2_hi = 0;
    r.a2_lo = FLT_MIN;
  } else {
    r.a2 = 1.4426950408889634 / p.temperature;
    float hi = static_cast<float>(r.a2);
    if (static_cast<double>(hi) > r.a2) hi = nextafterf(hi, 0.0f);
    float lo = static_cast<float>(r.a2 - static_cast<double>(hi));
    if (!(lo >= FLT_MIN)) lo = FLT_MIN;
    r.a2_hi = hi;
    r.a2_lo = lo;
    // topK 0 (disabled) or topK >= V keeps the whole vocabulary (sampling.ts:44), which is
    // the same as topK = V; small vocabularies therefore stay on the exact candidate path.
    const int64_t k = (p.top_k == 0 || p.top_k > vocab) ? vocab : p.top_k;
    if (k <= GS_MAX_TOP_K) {
      r.mode = kModeSmallK;
      r.top_k = static_cast<int32_t>(k);
      r.k_eff = static_cast<int32_t>(k);
    } else {
      r.mode = kModeLarge;
      r.k_eff = 0;
    }
  }
  return r;
}

struct Layout {
  int splits;
  int64_t chunk;
  int kcap;
  int kc;
  int kmax;
  bool any_large;
  bool any_typical_large;  // a histogram-path row with typical-p
  bool any_small;
  bool any_sample;
  size_t plans_off, stats_off, cands_off, rowtau_off, large_off, total;
  size_t large_row;  // per-row workspace of the histogram path (0: no such row)
  bool step;         // the single-launch decode step serves the batch (gs_step.cu)
  size_t step_off;   // its records and sort scratch
  size_t stream_smem, fin_smem, large_smem;
  int hist_cap, ent_cap, pack_cap, work_cap;
};

// Summary of the rows' plans that the layout depends on.
struct PlanSummary {
  int kmax = 0;
  bool any_large = false;
  bool any_typical_large = false;
  bool any_small = false;
  bool any_sample = false;
  void add(const RowPlan& p) {
    kmax = p.k_eff > kmax ? p.k_eff : kmax;
    any_large |= p.mode == kModeLarge;
    any_typical_large |= p.mode == kModeLarge && p.typical_p < 1;
    any_small |= p.mode != kModeLarge;
    any_sample |= p.mode != kModeGreedy;
  }
};

// validateDecodingConfig (src/runtime/decoding.ts:31-59) for the fields sampleToken reads.
bool valid_params(const gs_params& p, std::string* why);
enum : unsigned { kCheckNoOutputs = 1u, kCheckNoLogits = 2u };
gs_status check_batch(const gs_batch* b, const gs_outputs* o, std::string* err, unsigned what = 0);
gs_status plan_layout(const gs_batch* b, const PlanSummary& ps, Layout* L, std::string* err);

// Vocabulary-sharded calls: mode 1 streams a shard and writes its per-row records,
// mode 2 merges the gathered records (no streaming pass).
struct ShardInfo {
  int mode = 0;
  int64_t vocab_offset = 0;
  int shards = 1;
  int rec_kcap = 1, rec_hcap = 0;
  int64_t rec_bytes = 0;
  unsigned char* records = nullptr;
  bool want_raw = false;  // mode 1: record the raw sums (log-probabilities)
};

// Layout of a merge of `shards` gathered records per row (mode 2).
gs_status plan_merge_layout(const gs_batch* b, const PlanSummary& ps, const ShardInfo& sh, Layout* L,
                            std::string* err);

// Launches the streaming pass, the merge and (when a row needs it) the histogram path.
// `events` (3 entries or nullptr) are recorded before the stream pass, before the
// merge, and at the end.  `shard` (nullptr: an ordinary call) selects a sharded mode.
// `ws` is the call's workspace (the layout's offsets are relative to it).
// Single-launch decode step (gs_step.cu): a few rows without a constraint table or a
// penalty history, topK <= 64; `done` holds kStepDoneRows per-row counters that start at
// zero (the kernel resets them).
bool step_eligible(const gs_batch* b, int kmax, bool any_large, int rows);
size_t step_ws_bytes(int rows, int64_t vocab, int kmax);
cudaError_t launch_step(const gs_batch* b, const gs_outputs* o, const RowPlan& plan0, const RowPlan* dplans, int kmax,
                        unsigned char* ws, unsigned* done, cudaStream_t st);

gs_status launch_sampling(const gs_batch* b, const gs_outputs* o, const Layout& L, const RowPlan& plan0,
                          const RowPlan* dplans, unsigned char* ws, cudaStream_t st, cudaEvent_t* events,
                          std::string* err, const ShardInfo* shard = nullptr, unsigned* step_done = nullptr);

// Message of this thread's last failed gs_sample_noalloc call.
const char* noalloc_last_error();

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace gs
