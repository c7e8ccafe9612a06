// Internal types shared by the kernels and the host side of libgsampler.
#pragma once
#include <atomic>
#include <cstdint>
#include <cuda_runtime.h>

struct gs_ctx;

namespace gs {

enum RowMode : int32_t { kModeSmallK = 0, kModeGreedy = 1, kModeLarge = 2 };

constexpr int kStepDoneRows = 8;  // rows the single-launch decode step serves (one counter each)

// Per-row plan, derived on the host from gs_params (one DecodingConfig per row).
struct RowPlan {
  double temperature;
  double top_p;
  double min_p;
  double typical_p;
  double repetition_penalty;
  double presence_penalty;
  double frequency_penalty;
  double a2;        // log2(e) / temperature (double); 2^(x·a2) = e^(x/T)
  float a2_hi;      // a2 rounded toward zero to float
  float a2_lo;      // a2 - a2_hi (>= FLT_MIN, so (-inf)·a2_lo stays -inf)
  int32_t top_k;
  int32_t k_eff;    // candidates each streaming unit keeps: 1 greedy, topK small-K, 0 large
  int32_t mode;     // RowMode
  int32_t pad;
};

// Partial statistics of one streaming unit (row, vocabulary chunk).
struct UnitStat {
  float m;          // max over live ids (allowed and not in the penalty history), -inf if none
  float raw_m;      // max over every id of the chunk (log-probability)
  double s;         // sum 2^((x - m)·a2) over live ids
  double raw_s;     // sum e^(x - raw_m) over every id
  int32_t n_allowed;
  int32_t n_cand;
  uint32_t flags;
  int32_t pad;
};

struct StreamArgs {
  const void* logits;
  int64_t vocab;
  int64_t row_stride;
  int64_t vocab_offset;   // global id of local id 0 (vocabulary-sharded mode)
  float softcap;
  float inv_softcap;
  int32_t want_raw;
  int32_t splits;
  int64_t chunk;
  int32_t kcap;           // candidate slots per unit in `cands`
  int32_t kc;             // shared-memory candidate buffer entries (power of two)
  int32_t kmax;           // largest k_eff of the batch
  const RowPlan* plans;   // per-row plans or nullptr (then plan0)
  RowPlan plan0;
  const int32_t* history;
  const int32_t* history_len;
  int64_t history_stride;
  const uint32_t* mask_table;
  int64_t mask_states;
  int64_t mask_words;
  const int32_t* mask_state;
  UnitStat* stats;
  unsigned long long* cands;
  // per-row bound shared by the row's units (zeroed per call, or nullptr): every unit's
  // k-th best pack, and its first-tile threshold, bound the row's k-th best from below
  unsigned long long* row_tau;
};

struct FinalizeArgs {
  const void* logits;
  const int32_t* history_count;  // [rows, history_stride] occurrences per entry, or nullptr (one each)
  int64_t vocab;          // ids are [0, vocab) of this call
  int64_t row_stride;
  float softcap;
  float inv_softcap;
  int32_t want_raw;
  int32_t splits;
  int32_t kcap;
  int32_t hist_cap;       // power-of-two shared buffer for the sorted history
  int32_t ent_cap;        // power-of-two shared buffer for candidate entries
  int32_t pack_cap;       // shared buffer for unit packs (0 when units already hold <= k)
  int32_t work_cap;       // entries of the filter work arrays (power of two >= the batch's topK)
  const RowPlan* plans;
  RowPlan plan0;
  const int32_t* history;
  const int32_t* history_len;
  int64_t history_stride;
  const uint32_t* mask_table;
  int64_t mask_states;
  int64_t mask_words;
  const int32_t* mask_state;
  const UnitStat* stats;
  const unsigned long long* cands;
  double* rng_state;
  const double* uniforms;
  int32_t* ids;
  double* logprob;
  uint32_t* flags;
  int32_t* cand_ids;
  double* cand_probs;
  int32_t* cand_count;
  int32_t cand_cap;
  // vocabulary-sharded mode (0: sample the row here)
  int32_t shard_mode;     // 1: write this shard's per-row record; 2: merge gathered records
  int32_t shards;         // mode 2: records per row (one per shard)
  int64_t vocab_offset;   // mode 1: global id of local id 0
  int64_t rec_bytes;      // bytes per record (ShardRecord layout)
  int32_t rec_kcap;       // candidate packs per record
  int32_t rec_hcap;       // penalised-entry slots per record
  unsigned char* records; // mode 1: out [rows] records; mode 2: in [shards][rows] records
  // histogram path (topK 0 or > GS_MAX_TOP_K): per-row workspace
  unsigned char* lws;     // [rows] blocks of lrow_bytes
  int64_t lrow_bytes;
  int32_t lslots;         // penalised-entry slots per row (the history stride)
  int32_t lmoments;       // some histogram-path row has typical-p (its bins' first moments)
};

// Per-row record of one vocabulary shard (gs_shard_partials writes, gs_shard_merge reads):
//   UnitStat (the shard's combined statistics; n_cand packs follow),
//   packs[rec_kcap]   top-k candidate packs of the shard (global ids),
//   pen_key[rec_hcap] penalised entries' exact keys (double), pen_id[rec_hcap] their
//   global ids (0xffffffff: empty slot), pen_raw[rec_hcap] their soft-capped logits.
inline int64_t shard_record_bytes(int kcap, int hcap) {
  const int64_t b = static_cast<int64_t>(sizeof(UnitStat)) + 8ll * kcap + 16ll * hcap;
  return (b + 15) & ~15ll;
}

// Launch helpers implemented in gs_kernels.cu.
cudaError_t launch_stream(const StreamArgs& a, int dtype, int rows, size_t smem, cudaStream_t st);
int sm_count();  // SMs of the current device
// True until mark_device_done(seen) has run on the current device: a kernel's dynamic
// shared-memory attribute is a per-device setting, so a process that drives several
// GPUs sets it once on each (devices 0..63).
inline bool device_todo(const std::atomic<uint64_t>& seen) {
  int d = 0;
  cudaGetDevice(&d);
  return !((seen.load(std::memory_order_acquire) >> (d & 63)) & 1u);
}
inline void mark_device_done(std::atomic<uint64_t>& seen) {
  int d = 0;
  cudaGetDevice(&d);
  seen.fetch_or(1ull << (d & 63), std::memory_order_release);
}
int ctx_device(const gs_ctx* c);                 // the device a context is bound to
void ctx_set_error(gs_ctx* c, const char* msg);  // the message gs_last_error returns
size_t stream_smem_bytes(int64_t chunk, int kc);
cudaError_t launch_finalize(const FinalizeArgs& a, int dtype, int rows, size_t smem, cudaStream_t st);
// Warp-per-row merge (topK <= 128, history stride <= 512, not a shard call).
bool finalize_warp_eligible(const FinalizeArgs& a, int kmax, size_t* smem);
cudaError_t launch_finalize_warp(const FinalizeArgs& a, int dtype, int rows, int kmax, cudaStream_t st);
size_t finalize_smem_bytes(int hist_cap, int ent_cap, int pack_cap, int work_cap);
// Histogram path: hist (clusters of 8 CTAs), select, gather and resolve launches.
cudaError_t launch_large(const FinalizeArgs& a, int dtype, int rows, size_t select_smem, cudaStream_t st);
size_t large_row_bytes(int64_t slots);                  // per-row workspace of the histogram path
size_t large_select_smem_bytes(int64_t history_stride); // shared memory of its select kernel
cudaError_t launch_logprob(const void* logits, int dtype, int rows, int64_t vocab, int64_t stride,
                           float softcap, float inv_softcap, const int32_t* tokens, double* out,
                           int32_t* bad, cudaStream_t st);
cudaError_t launch_mask_logits(const float* raw, int64_t vocab, const int32_t* legal, int64_t nl,
                               const int32_t* term, int64_t nt, float* out, cudaStream_t st);
cudaError_t launch_build_mask_row(int64_t vocab, const int32_t* legal, int64_t nl, const int32_t* term,
                                  int64_t nt, uint32_t* row, cudaStream_t st);
cudaError_t launch_reasoning_rows(int64_t vocab, const uint8_t* has_bytes, int32_t end_id, uint32_t* rows,
                                  int64_t words, cudaStream_t st);
cudaError_t launch_softcap(const float* in, float* out, int64_t n, float cap, float inv_cap, cudaStream_t st);
cudaError_t launch_softcap_digest(uint64_t lo, uint64_t hi, float cap, float inv_cap,
                                  unsigned long long* acc, cudaStream_t st);

constexpr int kStreamThreads = 512;
constexpr int kFinalizeThreads = 256;
constexpr int kFinalizeMaxThreads = 1024;  // merge threads per row when rows are few

}  // namespace gs
