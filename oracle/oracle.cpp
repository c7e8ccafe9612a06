// ORACLE — test infrastructure only. Not part of the product.
//
// A plain C++17 restatement, in IEEE double arithmetic, of the reference's CPU
// decode sampler so that the CUDA path can be checked against it on identical
// inputs.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
// --impl reference legs may load this file's shared object.
//
// Reference (aribornstein/gemma-webgpu-engine, TypeScript):
//   src/runtime/sampling.ts:3-16     SeededRandom (Mulberry32 over a JS number state)
//   src/runtime/sampling.ts:18-65    sampleToken
//   src/runtime/sampling.ts:67-80    tokenLogProbability
//   src/runtime/sampling.ts:82-90    cumulativeCut
//   src/runtime/sampling.ts:92-96    argmax
//   src/runtime/constraints.ts:159-173 maskConstraintLogits
//   src/runtime/gemma-session.ts:1331-1345 maskReasoningLogits
//   src/webgpu/decode-lm-head.ts:176-256 int2 LM head (the producer of the logits)
//
// Parity pins: tests/test_oracle_golden.py checks this file against every
// known-answer test of tests/sampling.spec.ts and tests/constraints.spec.ts:158-161
// (restated as fixtures in tests/golden/reference_spec_cases.json).  The reference
// itself cannot run in this container (no Node); see the header of that fixture.
//
// JS semantics that matter and how they are restated here:
//  * Array.prototype.sort is stable (ES2019); a comparator that returns NaN is read as
//    +0 ("equal").  `right.logit - left.logit` is therefore the strict weak order
//    "a before b iff a.logit > b.logit" for every non-NaN input (-inf/-inf and +inf/+inf
//    give NaN = equal).  std::stable_sort with that predicate gives the same order.
//  * Math.imul / >>> / ^ / | wrap to 32 bits; the SeededRandom state itself is a JS
//    number that grows by 0x6d2b79f5 per draw without wrapping (sampling.ts:11), so it
//    is kept here as a double and converted with ToUint32 at each use.
//  * Float32Array -> Array.from widens exactly (sampling.ts:20).
//  * NaN logits make the reference's comparator inconsistent (implementation-defined
//    order); they are outside the domain of this oracle and of the CUDA path.
//
// Build: oracle/Makefile (g++ -O2 -ffp-contract=off, so no FMA contraction changes a
// rounding).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <vector>
#include <thread>

namespace {

// ---------------------------------------------------------------- SeededRandom
// JS ToUint32 of an integral double (state never holds a fraction).
inline uint32_t to_uint32(double v) {
  double m = std::fmod(v, 4294967296.0);
  if (m < 0) m += 4294967296.0;
  return static_cast<uint32_t>(m);
}

// sampling.ts:7  `seed >>> 0 || 0x6d2b79f5`
inline double seeded_init(double seed) {
  uint32_t s = to_uint32(std::trunc(seed));
  return s == 0 ? static_cast<double>(0x6d2b79f5u) : static_cast<double>(s);
}

// sampling.ts:10-15
inline double seeded_next(double* state) {
  *state = *state + 1831565813.0;  // 0x6d2b79f5 added to a JS number: no wrap
  uint32_t v = to_uint32(*state);
  v = static_cast<uint32_t>(static_cast<uint64_t>(v ^ (v >> 15)) * static_cast<uint64_t>(v | 1u));
  v ^= v + static_cast<uint32_t>(static_cast<uint64_t>(v ^ (v >> 7)) * static_cast<uint64_t>(v | 61u));
  return static_cast<double>(v ^ (v >> 14)) / 4294967296.0;
}

struct Item {
  int32_t token;
  double logit;
  double probability;
  double surprise;
};

}  // namespace

extern "C" {

// Same field order and meaning as DecodingConfig (src/runtime/decoding.ts:1-14),
// minus maxNewTokens / seed / stopTokenIds which sampleToken does not read.
struct OracleConfig {
  double temperature;
  double top_p;
  double min_p;
  double typical_p;
  double repetition_penalty;
  double presence_penalty;
  double frequency_penalty;
  int32_t top_k;
  int32_t repetition_window;
};

// Diagnostic margins of the decisions sampleToken took (all relative, >= 0; +inf when
// the decision did not happen).  Used by tests to count boundary cases.
struct OracleTrace {
  double total;          // full-vocabulary normaliser (sampling.ts:37-41)
  double max_key;        // scaled[0].logit
  double candidate_total;
  double uniform;        // the random() value consumed (NaN when none)
  double margin_top_p;   // |cumulative - topP| / topP at the cut index and the one before
  double margin_draw;    // distance of the cursor to the chosen CDF step, / candidateTotal
  double margin_min_p;   // min |p - threshold| / threshold over candidates
  double margin_typical; // |cumulative - typicalP| / typicalP at the typical cut
  int32_t n_after_top_k;
  int32_t n_after_min_p;
  int32_t n_after_typical;
  int32_t n_final;
  int32_t fell_through;  // draw loop ended without cursor <= 0 (sampling.ts:64)
  int32_t greedy;
};

double oracle_seeded_init(double seed) { return seeded_init(seed); }
double oracle_seeded_next(double* state) { return seeded_next(state); }

// sampling.ts:82-90, returning the kept length and the decision margin.
static size_t cumulative_cut(const std::vector<Item>& items, double threshold, double* margin) {
  double cumulative = 0;
  size_t end = 0;
  double prev = 0;
  do {
    prev = cumulative;
    cumulative += items[end].probability;
    end += 1;
  } while (end < items.size() && cumulative < threshold);
  if (margin) {
    double m = std::fabs(cumulative - threshold);
    if (end >= 2) m = std::min(m, std::fabs(prev - threshold));
    *margin = threshold > 0 ? m / threshold : m;
  }
  return std::max<size_t>(1, end);
}

// sampleToken (sampling.ts:18-65).  `uniform` is the value random() returns; it is
// read only when temperature != 0 (sampling.ts:31, 59).  Returns the token, or -1 for
// empty logits (the reference throws "Cannot sample empty logits").
// cand_ids/cand_probs (capacity cand_cap) receive the final candidate list in draw order.
int32_t oracle_sample_token(const float* raw_logits, int64_t vocab,
                            const int32_t* history, int64_t history_len,
                            const OracleConfig* config, double uniform,
                            int32_t* cand_ids, double* cand_probs, int32_t* cand_count,
                            int64_t cand_cap, OracleTrace* trace) {
  OracleTrace tr;
  tr.total = tr.max_key = tr.candidate_total = NAN;
  tr.uniform = NAN;
  tr.margin_top_p = tr.margin_draw = tr.margin_min_p = tr.margin_typical = INFINITY;
  tr.n_after_top_k = tr.n_after_min_p = tr.n_after_typical = tr.n_final = 0;
  tr.fell_through = 0;
  tr.greedy = 0;
  if (cand_count) *cand_count = 0;
  if (vocab <= 0) {
    if (trace) *trace = tr;
    return -1;
  }
  // sampling.ts:20
  std::vector<double> logits(static_cast<size_t>(vocab));
  for (int64_t i = 0; i < vocab; ++i) logits[i] = static_cast<double>(raw_logits[i]);
  // sampling.ts:21-25 (Map keeps first-insertion order; the per-token updates are
  // independent, so a sorted map gives the same values)
  std::map<int32_t, int64_t> counts;
  if (config->repetition_window != 0) {
    int64_t start = history_len - config->repetition_window;
    if (start < 0) start = 0;
    for (int64_t i = start; i < history_len; ++i) counts[history[i]] += 1;
  }
  // sampling.ts:26-30
  for (const auto& kv : counts) {
    int32_t token = kv.first;
    if (token < 0 || token >= vocab) continue;
    double v = logits[token];
    v = v < 0 ? v * config->repetition_penalty : v / config->repetition_penalty;
    v -= config->presence_penalty + static_cast<double>(kv.second) * config->frequency_penalty;
    logits[token] = v;
  }
  // sampling.ts:31, 92-96
  if (config->temperature == 0) {
    int64_t best = 0;
    for (int64_t i = 1; i < vocab; ++i)
      if (logits[i] > logits[best]) best = i;
    tr.greedy = 1;
    tr.n_final = 1;
    if (cand_count && cand_cap > 0) {
      cand_ids[0] = static_cast<int32_t>(best);
      cand_probs[0] = 1.0;
      *cand_count = 1;
    }
    if (trace) *trace = tr;
    return static_cast<int32_t>(best);
  }
  // sampling.ts:33-35
  std::vector<Item> scaled(static_cast<size_t>(vocab));
  for (int64_t i = 0; i < vocab; ++i)
    scaled[i] = Item{static_cast<int32_t>(i), logits[i] / config->temperature, 0.0, 0.0};
  std::stable_sort(scaled.begin(), scaled.end(),
                   [](const Item& a, const Item& b) { return a.logit > b.logit; });
  // sampling.ts:36-42
  const double maximum = scaled[0].logit;
  double total = 0;
  for (auto& item : scaled) {
    item.probability = std::exp(item.logit - maximum);
    total += item.probability;
  }
  for (auto& item : scaled) item.probability /= total;
  tr.total = total;
  tr.max_key = maximum;
  // sampling.ts:44
  std::vector<Item> candidates;
  if (config->top_k > 0) {
    size_t k = std::min<size_t>(static_cast<size_t>(config->top_k), scaled.size());
    candidates.assign(scaled.begin(), scaled.begin() + k);
  } else {
    candidates = scaled;
  }
  tr.n_after_top_k = static_cast<int32_t>(candidates.size());
  // sampling.ts:45-48
  if (config->min_p > 0) {
    const double threshold = candidates[0].probability * config->min_p;
    std::vector<Item> kept;
    double m = INFINITY;
    for (const auto& item : candidates) {
      if (threshold > 0) m = std::min(m, std::fabs(item.probability - threshold) / threshold);
      if (item.probability >= threshold) kept.push_back(item);
    }
    tr.margin_min_p = m;
    candidates.swap(kept);
  }
  tr.n_after_min_p = static_cast<int32_t>(candidates.size());
  // sampling.ts:49-55
  if (config->typical_p < 1) {
    double entropy = 0;
    for (const auto& item : candidates) entropy = entropy - item.probability * std::log(item.probability);
    for (auto& item : candidates) item.surprise = std::fabs(-std::log(item.probability) - entropy);
    std::stable_sort(candidates.begin(), candidates.end(),
                     [](const Item& a, const Item& b) { return a.surprise < b.surprise; });
    size_t keep = cumulative_cut(candidates, config->typical_p, &tr.margin_typical);
    candidates.resize(keep);
    std::stable_sort(candidates.begin(), candidates.end(),
                     [](const Item& a, const Item& b) { return a.probability > b.probability; });
  }
  tr.n_after_typical = static_cast<int32_t>(candidates.size());
  // sampling.ts:56
  if (config->top_p < 1) {
    size_t keep = cumulative_cut(candidates, config->top_p, &tr.margin_top_p);
    candidates.resize(keep);
  }
  tr.n_final = static_cast<int32_t>(candidates.size());
  // sampling.ts:58-64
  double candidate_total = 0;
  for (const auto& item : candidates) candidate_total += item.probability;
  tr.candidate_total = candidate_total;
  tr.uniform = uniform;
  double cursor = uniform * candidate_total;
  int32_t chosen = -1;
  for (const auto& item : candidates) {
    double before = cursor;
    cursor -= item.probability;
    if (cursor <= 0) {
      chosen = item.token;
      double m = std::min(std::fabs(before), std::fabs(cursor));
      tr.margin_draw = candidate_total > 0 ? m / candidate_total : m;
      break;
    }
  }
  if (chosen < 0) {
    chosen = candidates.back().token;
    tr.fell_through = 1;
    tr.margin_draw = candidate_total > 0 ? std::fabs(cursor) / candidate_total : std::fabs(cursor);
  }
  if (cand_count) {
    int64_t n = std::min<int64_t>(cand_cap, static_cast<int64_t>(candidates.size()));
    for (int64_t i = 0; i < n; ++i) {
      cand_ids[i] = candidates[i].token;
      cand_probs[i] = candidates[i].probability;
    }
    *cand_count = static_cast<int32_t>(candidates.size());
  }
  if (trace) *trace = tr;
  return chosen;
}

// Same as oracle_sample_token, with random() = SeededRandom.next() over *rng_state
// (a JS-number state, see seeded_next).  The state advances only when a draw happens.
int32_t oracle_sample_token_seeded(const float* raw_logits, int64_t vocab,
                                   const int32_t* history, int64_t history_len,
                                   const OracleConfig* config, double* rng_state,
                                   int32_t* cand_ids, double* cand_probs, int32_t* cand_count,
                                   int64_t cand_cap, OracleTrace* trace) {
  double u = NAN;
  if (vocab > 0 && config->temperature != 0) u = seeded_next(rng_state);
  return oracle_sample_token(raw_logits, vocab, history, history_len, config, u,
                             cand_ids, cand_probs, cand_count, cand_cap, trace);
}

// tokenLogProbability (sampling.ts:67-80).  *error = 1 when the token is outside
// [0, length) (the reference throws `Token ${token} is outside logits length ${n}`).
double oracle_token_log_probability(const float* raw_logits, int64_t vocab, int64_t token,
                                    int32_t* error) {
  *error = 0;
  if (token < 0 || token >= vocab) {
    *error = 1;
    return NAN;
  }
  double maximum = -INFINITY;
  for (int64_t i = 0; i < vocab; ++i) maximum = std::max(maximum, static_cast<double>(raw_logits[i]));
  double denominator = 0;
  for (int64_t i = 0; i < vocab; ++i) denominator += std::exp(static_cast<double>(raw_logits[i]) - maximum);
  return static_cast<double>(raw_logits[token]) - maximum - std::log(denominator);
}

// maskConstraintLogits (constraints.ts:159-173).
void oracle_mask_constraint_logits(const float* raw_logits, int64_t vocab,
                                   const int32_t* legal, int64_t n_legal,
                                   const int32_t* termination, int64_t n_termination,
                                   float* out) {
  for (int64_t i = 0; i < vocab; ++i) out[i] = -INFINITY;
  for (int64_t i = 0; i < n_legal; ++i)
    if (legal[i] >= 0 && legal[i] < vocab) out[legal[i]] = raw_logits[legal[i]];
  for (int64_t i = 0; i < n_termination; ++i)
    if (termination[i] >= 0 && termination[i] < vocab) out[termination[i]] = raw_logits[termination[i]];
}

// ------------------------------------------------------------------ softcap
// 30·tanh(x/30) style logit soft cap in float32, stated as an exact sequence of
// IEEE single operations so that every compliant implementation gives the same bits.
// The reference runtime never applies it (the Gemma manifest declares 30, the LM head
// writes uncapped logits); the benchmark configurations apply it when making inputs.
// Method: y = x * fl(1/c), z = fl(y·y).  z < 1 (exactly |y| < 1) uses the odd
// polynomial evaluated on the signed y, c·fma(y·z, Q(z), y) with Q of degree 6 (a
// least-squares/Lawson minimax fit, coefficients below; a zero y gives +0); otherwise
// 1 <= |y| < 9 uses t = 1 - 2/(e^{2|y|} + 1) with e^z by Cody–Waite reduction
// z = n·ln2 + r and a degree-6 polynomial for e^r, |y| >= 9 gives t = 1, and the result
// is c·copysign(t, y).
static const float kTanhQ[7] = {-0.33333296f, 0.13332345f, -0.0538798f, 0.021486657f,
                                -0.007946107f, 0.0023013647f, -0.00035845203f};
static const float kExpB[5] = {0.49999994f, 0.1666652f, 0.04166841f, 0.00836891f, 0.00138142f};
static const float kLn2Hi = 0.693145751953125f;     // 0x3f317200
static const float kLn2Lo = 1.428606765330187e-06f; // ln2 - kLn2Hi
static const float kLog2e = 1.44269502162933349609375f;

static inline float f_exp_reduced(float z) {
  float n = std::rint(z * kLog2e);
  float r = std::fmaf(-n, kLn2Hi, z);
  r = std::fmaf(-n, kLn2Lo, r);
  float p = kExpB[4];
  p = std::fmaf(p, r, kExpB[3]);
  p = std::fmaf(p, r, kExpB[2]);
  p = std::fmaf(p, r, kExpB[1]);
  p = std::fmaf(p, r, kExpB[0]);
  float r2 = r * r;
  float e = std::fmaf(p, r2, r) + 1.0f;
  int32_t ni = static_cast<int32_t>(n);
  uint32_t bits = static_cast<uint32_t>(ni + 127) << 23;
  float scale;
  std::memcpy(&scale, &bits, 4);
  return e * scale;
}

float oracle_softcap(float x, float cap, float inv_cap) {
  if (x != x) return x;
  float y = x * inv_cap;
  float z = y * y;
  if (z < 1.0f) {
    float q = kTanhQ[6];
    q = std::fmaf(q, z, kTanhQ[5]);
    q = std::fmaf(q, z, kTanhQ[4]);
    q = std::fmaf(q, z, kTanhQ[3]);
    q = std::fmaf(q, z, kTanhQ[2]);
    q = std::fmaf(q, z, kTanhQ[1]);
    q = std::fmaf(q, z, kTanhQ[0]);
    return cap * std::fmaf(y * z, q, y);
  }
  float a = std::fabs(y);
  float t;
  if (a < 9.0f) {
    float e = f_exp_reduced(a + a);
    t = 1.0f - 2.0f / (e + 1.0f);
  } else {
    t = 1.0f;
  }
  return cap * std::copysign(t, y);
}

void oracle_softcap_array(const float* in, float* out, int64_t n, float cap, float inv_cap) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_softcap(in[i], cap, inv_cap);
}

// Exhaustive check of softcap over every positive float32 input (the routine is odd):
// the largest error in ulps of the float32 result against c·tanh(x/c) in double (where
// x/c is a normal float), and the number of adjacent inputs whose results decrease
// (0: monotone).
void oracle_softcap_check(float cap, int threads, double* max_ulp, uint64_t* decreases) {
  const float inv = static_cast<float>(1.0 / static_cast<double>(cap));
  if (threads < 1) threads = 1;
  const uint64_t lo = 0, hi = 0x7f800000ull;  // +0 .. largest finite
  std::vector<double> worst(static_cast<size_t>(threads), 0.0);
  std::vector<uint64_t> dec(static_cast<size_t>(threads), 0);
  std::vector<std::thread> pool;
  const uint64_t span = (hi - lo + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([&, t] {
      const uint64_t a = lo + span * t, b = std::min(hi, a + span);
      double w = 0.0;
      uint64_t d = 0;
      float prev = 0.0f;
      for (uint64_t u = a; u <= b && u < hi; ++u) {  // (b: the next chunk's first input)
        const uint32_t xb = static_cast<uint32_t>(u);
        float x;
        std::memcpy(&x, &xb, 4);
        const float y = oracle_softcap(x, cap, inv);
        if (u > a && y < prev) ++d;
        prev = y;
        if (x < 1e-30f) continue;
        const double ref = static_cast<double>(cap) * std::tanh(static_cast<double>(x) / static_cast<double>(cap));
        const float rf = static_cast<float>(ref);
        const double ulp = static_cast<double>(std::nextafter(std::fabs(rf), INFINITY) - std::fabs(rf));
        const double e = std::fabs(static_cast<double>(y) - ref) / ulp;
        if (e > w) w = e;
      }
      worst[t] = w;
      dec[t] = d;
    });
  }
  for (auto& th : pool) th.join();
  *max_ulp = 0.0;
  *decreases = 0;
  for (int t = 0; t < threads; ++t) {
    *max_ulp = std::max(*max_ulp, worst[t]);
    *decreases += dec[t];
  }
}

// Order-independent 64-bit digest of softcap over the bit patterns [lo, hi) (used to
// compare the CUDA routine with this one exhaustively without moving 16 GB).
uint64_t oracle_softcap_digest(uint64_t lo, uint64_t hi, float cap, float inv_cap, int threads) {
  if (threads < 1) threads = 1;
  std::vector<uint64_t> part(static_cast<size_t>(threads), 0);
  std::vector<std::thread> pool;
  uint64_t span = (hi - lo + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([&, t] {
      uint64_t a = lo + span * t, b = std::min(hi, a + span), acc = 0;
      for (uint64_t u = a; u < b; ++u) {
        uint32_t xb = static_cast<uint32_t>(u);
        float x;
        std::memcpy(&x, &xb, 4);
        float y = oracle_softcap(x, cap, inv_cap);
        uint32_t yb;
        std::memcpy(&yb, &y, 4);
        if (y != y) yb = 0x7fc00000u;  // canonical NaN
        uint64_t h = (static_cast<uint64_t>(xb) << 32) | yb;
        h ^= h >> 33; h *= 0xff51afd7ed558ccdULL; h ^= h >> 33; h *= 0xc4ceb9fe1a85ec53ULL; h ^= h >> 33;
        acc += h;
      }
      part[t] = acc;
    });
  }
  for (auto& th : pool) th.join();
  uint64_t s = 0;
  for (auto p : part) s += p;
  return s;
}

// maskReasoningLogits (src/runtime/gemma-session.ts:1331-1345): a copy of the logits
// with -inf at every id whose tokenBytes is null (has_bytes[id] == 0); with allow_end the
// end-of-channel id keeps its raw value (a write outside the array is a no-op in JS).
void oracle_mask_reasoning_logits(const float* raw_logits, int64_t vocab, const uint8_t* has_bytes,
                                  int32_t allow_end, int64_t end_id, float* out) {
  for (int64_t i = 0; i < vocab; ++i) out[i] = has_bytes[i] ? raw_logits[i] : -INFINITY;
  if (allow_end && end_id >= 0 && end_id < vocab) out[end_id] = raw_logits[end_id];
}

// Batched driver used for the timed CPU baseline: rows are independent, so rows are
// split over `threads` host threads.  history is [rows, history_stride] with per-row
// lengths; mask_table/mask_state optional (state < 0 = unconstrained): masked ids are
// -inf before penalties exactly as selectConstrainedToken does
// (src/runtime/gemma-session.ts:1327-1328).  softcap 0 = off.  With cand_count, each
// row's final candidate list (at most cand_cap entries of [rows, cand_cap]) and its length
// are written as oracle_sample_token writes them.
void oracle_sample_rows(const float* logits, int64_t rows, int64_t vocab, int64_t row_stride,
                        float softcap,
                        const int32_t* history, int64_t history_stride, const int32_t* history_len,
                        const uint32_t* mask_table, int64_t mask_words, const int32_t* mask_state,
                        const OracleConfig* configs, int32_t per_row_config,
                        double* rng_state, const double* uniforms,
                        int32_t* out_ids, OracleTrace* traces, int threads,
                        int32_t* cand_ids, double* cand_probs, int32_t* cand_count, int64_t cand_cap) {
  if (threads < 1) threads = 1;
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([=] {
      std::vector<float> row(static_cast<size_t>(vocab));
      float inv = softcap != 0 ? static_cast<float>(1.0 / static_cast<double>(softcap)) : 0.0f;
      for (int64_t r = t; r < rows; r += threads) {
        const float* src = logits + r * row_stride;
        for (int64_t i = 0; i < vocab; ++i) row[i] = softcap != 0 ? oracle_softcap(src[i], softcap, inv) : src[i];
        if (mask_table && mask_state && mask_state[r] >= 0) {
          const uint32_t* m = mask_table + static_cast<int64_t>(mask_state[r]) * mask_words;
          for (int64_t i = 0; i < vocab; ++i)
            if (!((m[i >> 5] >> (i & 31)) & 1u)) row[i] = -INFINITY;
        }
        const OracleConfig* c = configs + (per_row_config ? r : 0);
        int64_t hl = history_len ? history_len[r] : 0;
        const int32_t* h = history ? history + r * history_stride : nullptr;
        OracleTrace tr;
        int32_t id;
        int32_t* ci = cand_count ? cand_ids + r * cand_cap : nullptr;
        double* cp = cand_count ? cand_probs + r * cand_cap : nullptr;
        int32_t* cc = cand_count ? cand_count + r : nullptr;
        const int64_t cap = cand_count ? cand_cap : 0;
        if (uniforms) {
          id = oracle_sample_token(row.data(), vocab, h, hl, c, uniforms[r], ci, cp, cc, cap, &tr);
        } else {
          id = oracle_sample_token_seeded(row.data(), vocab, h, hl, c, rng_state + r, ci, cp, cc, cap, &tr);
        }
        out_ids[r] = id;
        if (traces) traces[r] = tr;
      }
    });
  }
  for (auto& th : pool) th.join();
}

}  // extern "C"

// ------------------------------------------------------------------ constraint masks
// Restates CompiledGenerationConstraint.legalTokenIds (src/runtime/constraints.ts:56-92)
// with its helpers transitionByte (:222-247), transitionCharacter (:249-252),
// isViableConstraintState (:254-267), pendingUtf8CompletionRange (:269-292),
// decodeUtf8CodePoint (:294-300) and findViableStates (:302-321), over the token-byte
// trie of src/runtime/token-byte-trie.ts:16-40, then the legal-set rule of
// selectConstrainedToken (src/runtime/gemma-session.ts:1315-1326).  The DFA is given as
// per-node code-point ranges (range_lo..range_hi inclusive -> target), the form a refa
// DFA node's `out` CharMap takes.
namespace {

struct OState {
  int32_t node;
  std::vector<int> pending;
};

struct ODfa {
  const int32_t* off;
  const uint32_t* lo;
  const uint32_t* hi;
  const int32_t* target;
  std::vector<char> viable;
};

int o_transition_character(const ODfa& d, int32_t node, uint32_t ch) {
  for (int64_t r = d.off[node]; r < d.off[node + 1]; ++r)
    if (d.lo[r] <= ch && ch <= d.hi[r]) return d.target[r];
  return -1;
}

uint32_t o_decode(const std::vector<int>& bytes) {
  const size_t n = bytes.size();
  uint32_t cp = static_cast<uint32_t>(bytes[0]) & (n == 2 ? 0x1f : n == 3 ? 0x0f : 0x07);
  for (size_t i = 1; i < n; ++i) cp = (cp << 6) | (static_cast<uint32_t>(bytes[i]) & 0x3f);
  return cp;
}

bool o_transition_byte(const ODfa& d, const OState& s, int byte, OState* out) {
  if (s.pending.empty()) {
    if (byte <= 0x7f) {
      const int t = o_transition_character(d, s.node, static_cast<uint32_t>(byte));
      if (t < 0) return false;
      *out = OState{t, {}};
      return true;
    }
    if ((byte >= 0xc2 && byte <= 0xdf) || (byte >= 0xe0 && byte <= 0xef) || (byte >= 0xf0 && byte <= 0xf4)) {
      *out = OState{s.node, {byte}};
      return true;
    }
    return false;
  }
  if (byte < 0x80 || byte > 0xbf) return false;
  std::vector<int> bytes = s.pending;
  bytes.push_back(byte);
  const size_t expected = s.pending[0] <= 0xdf ? 2 : s.pending[0] <= 0xef ? 3 : 4;
  if (bytes.size() < expected) {
    *out = OState{s.node, bytes};
    return true;
  }
  if ((bytes[0] == 0xe0 && bytes[1] < 0xa0) || (bytes[0] == 0xed && bytes[1] > 0x9f) ||
      (bytes[0] == 0xf0 && bytes[1] < 0x90) || (bytes[0] == 0xf4 && bytes[1] > 0x8f))
    return false;
  const int t = o_transition_character(d, s.node, o_decode(bytes));
  if (t < 0) return false;
  *out = OState{t, {}};
  return true;
}

bool o_completion(const std::vector<int>& pending, uint32_t* mn, uint32_t* mx) {
  if (pending.empty()) return false;
  const int lead = pending[0];
  const size_t length = lead <= 0xdf ? 2 : lead <= 0xef ? 3 : 4;
  if (pending.size() >= length) return false;
  const int second_min = lead == 0xe0 ? 0xa0 : lead == 0xf0 ? 0x90 : 0x80;
  const int second_max = lead == 0xed ? 0x9f : lead == 0xf4 ? 0x8f : 0xbf;
  if (pending.size() > 1 && (pending[1] < second_min || pending[1] > second_max)) return false;
  for (size_t i = 2; i < pending.size(); ++i)
    if (pending[i] < 0x80 || pending[i] > 0xbf) return false;
  std::vector<int> lo = pending, hi = pending;
  while (lo.size() < length) {
    const size_t i = lo.size();
    lo.push_back(i == 1 ? second_min : 0x80);
    hi.push_back(i == 1 ? second_max : 0xbf);
  }
  *mn = o_decode(lo);
  *mx = o_decode(hi);
  return true;
}

bool o_viable_state(const ODfa& d, const OState& s) {
  if (s.pending.empty()) return d.viable[s.node] != 0;
  uint32_t mn, mx;
  if (!o_completion(s.pending, &mn, &mx)) return false;
  for (int64_t r = d.off[s.node]; r < d.off[s.node + 1]; ++r)
    if (d.viable[d.target[r]] && d.lo[r] <= mx && d.hi[r] >= mn) return true;
  return false;
}

struct OTrieNode {
  std::map<int, int> children;  // byte -> node index
  std::vector<int32_t> tokens;
};

}  // namespace

extern "C" {

void oracle_constraint_masks(int32_t nodes, const int32_t* range_off, const uint32_t* range_lo,
                             const uint32_t* range_hi, const int32_t* range_target, const uint8_t* final,
                             int64_t vocab, const int64_t* tok_off, const uint8_t* tok_bytes, int32_t n_states,
                             const int32_t* node, const uint8_t* pending_len, const uint8_t* pending_bytes,
                             const int32_t* term, int64_t n_term, const int32_t* extra, int64_t n_extra,
                             uint32_t* table, int64_t mask_words, int32_t* dead_end) {
  ODfa d{range_off, range_lo, range_hi, range_target, std::vector<char>(static_cast<size_t>(nodes), 0)};
  // findViableStates: the finals and their predecessors, transitively
  std::vector<std::vector<int32_t>> reverse(static_cast<size_t>(nodes));
  for (int32_t n = 0; n < nodes; ++n)
    for (int64_t r = range_off[n]; r < range_off[n + 1]; ++r) reverse[range_target[r]].push_back(n);
  std::vector<int32_t> stack;
  for (int32_t n = 0; n < nodes; ++n)
    if (final[n]) {
      d.viable[n] = 1;
      stack.push_back(n);
    }
  while (!stack.empty()) {
    const int32_t t = stack.back();
    stack.pop_back();
    for (int32_t p : reverse[t])
      if (!d.viable[p]) {
        d.viable[p] = 1;
        stack.push_back(p);
      }
  }
  // TokenByteTrie: every non-empty token under the path of its bytes
  std::vector<OTrieNode> trie(1);
  for (int64_t v = 0; v < vocab; ++v) {
    if (tok_off[v + 1] == tok_off[v]) continue;
    int cur = 0;
    for (int64_t i = tok_off[v]; i < tok_off[v + 1]; ++i) {
      const int b = tok_bytes[i];
      auto it = trie[cur].children.find(b);
      if (it == trie[cur].children.end()) {
        trie.push_back(OTrieNode{});
        const int nn = static_cast<int>(trie.size()) - 1;
        trie[cur].children[b] = nn;
        cur = nn;
      } else {
        cur = it->second;
      }
    }
    trie[cur].tokens.push_back(static_cast<int32_t>(v));
  }
  for (int32_t s = 0; s < n_states; ++s) {
    OState start{node[s], {}};
    const int pl = pending_len ? pending_len[s] : 0;
    for (int i = 0; i < pl; ++i) start.pending.push_back(pending_bytes[3 * s + i]);
    // legalTokenIds: depth-first over the trie, children only through viable states
    std::vector<int32_t> legal;
    std::vector<std::pair<int, OState>> dfs{{0, start}};
    while (!dfs.empty()) {
      auto cur = dfs.back();
      dfs.pop_back();
      if (!trie[cur.first].tokens.empty() && o_viable_state(d, cur.second))
        legal.insert(legal.end(), trie[cur.first].tokens.begin(), trie[cur.first].tokens.end());
      for (const auto& kv : trie[cur.first].children) {
        OState next;
        if (o_transition_byte(d, cur.second, kv.first, &next) && o_viable_state(d, next))
          dfs.push_back({kv.second, next});
      }
    }
    // selectConstrainedToken: (legal ∪ extra) − termination, + termination when accepting
    std::vector<char> allow(static_cast<size_t>(vocab), 0);
    for (int32_t v : legal) allow[v] = 1;
    for (int64_t i = 0; i < n_extra; ++i)
      if (extra[i] >= 0 && extra[i] < vocab) allow[extra[i]] = 1;
    for (int64_t i = 0; i < n_term; ++i)
      if (term[i] >= 0 && term[i] < vocab) allow[term[i]] = 0;
    const bool accepting = start.pending.empty() && final[start.node];
    if (accepting)
      for (int64_t i = 0; i < n_term; ++i)
        if (term[i] >= 0 && term[i] < vocab) allow[term[i]] = 1;
    uint32_t* row = table + static_cast<int64_t>(s) * mask_words;
    bool any = false;
    for (int64_t w = 0; w < mask_words; ++w) row[w] = 0;
    for (int64_t v = 0; v < vocab; ++v)
      if (allow[v]) {
        row[v >> 5] |= 1u << (v & 31);
        any = true;
      }
    if (dead_end) dead_end[s] = any ? 0 : 1;
  }
}

// ------------------------------------------------------------------ LM head
// The int2 LM head of src/webgpu/decode-lm-head.ts.  Packed weights: V rows of hidden/16
// u32 words; code j of word w (bits 2j..2j+1 — unpack4x8unorm of (word >> 2P) & 0x03030303
// gives the codes of elements 4k + P, k = byte) multiplies activation element 16w + j, and
// the weight is (code - 2)·scale[v]:
//   sum   = Σ_j (code_j / 255)·a_j                        (f32, decode-lm-head.ts:219-235)
//   logit = srq(scale[v]·fma(sum, 255, -(2·sumA)), outputScale)   (:239-247)
//   srq(x, s) = s == 0 ? x : clamp(round(x / s), -128, 127)·s      (:196-199; round: half
//               to even)
// sumA is the sum of the activations the producing kernel writes beside them
// (decode-ple-proj-norm-codes.ts:251-258).

static float o_srq(float x, float s) {
  if (s == 0.0f) return x;
  float r = std::nearbyint(x / s);  // (default rounding mode: nearest, ties to even)
  r = std::fmin(std::fmax(r, -128.0f), 127.0f);
  return r * s;
}

static inline int o_code(const uint32_t* row, int j) { return static_cast<int>((row[j >> 4] >> (2 * (j & 15))) & 3u); }

// The row-major-subgroups shader (decode-lm-head.ts:176-256) in its own f32 association:
// lane l of a 32-wide subgroup adds the words l, l+32, ... ((dot0 + dot1) + (dot2 + dot3),
// each dot summed left to right), then a butterfly subgroupAdd.  WGSL leaves the order of
// dot() and subgroupAdd open, so this is one legal evaluation, not the only one.
void oracle_lm_head_shader_f32(const uint32_t* packed, const float* scales, int64_t vocab, int hidden,
                               const float* act, const float* act_sum, int rows, float out_scale,
                               float* logits, int64_t ld_logits) {
  const int words = hidden / 16;
  for (int b = 0; b < rows; ++b) {
    const float* a = act + static_cast<int64_t>(b) * hidden;
    for (int64_t v = 0; v < vocab; ++v) {
      const uint32_t* row = packed + v * words;
      float lane[32];
      for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int w = l; w < words; w += 32) {
          float d[4];
          for (int c = 0; c < 4; ++c) {  // values[c] = a[16w + 4c .. 16w + 4c + 3]
            float t = 0.0f;
            for (int p = 0; p < 4; ++p) {
              const float code = static_cast<float>((row[w] >> (8 * c + 2 * p)) & 3u) / 255.0f;
              t = t + code * a[16 * w + 4 * c + p];
            }
            d[c] = t;
          }
          acc = acc + ((d[0] + d[1]) + (d[2] + d[3]));
        }
        lane[l] = acc;
      }
      for (int o = 16; o > 0; o >>= 1) {
        float nx[32];
        for (int l = 0; l < 32; ++l) nx[l] = lane[l] + lane[l ^ o];
        for (int l = 0; l < 32; ++l) lane[l] = nx[l];
      }
      const float t = std::fmaf(lane[0], 255.0f, -(2.0f * act_sum[b]));
      logits[static_cast<int64_t>(b) * ld_logits + v] = o_srq(scales[v] * t, out_scale);
    }
  }
}

// The same logits computed exactly, as the CUDA path does.
//   in_scale != 0: the activations are read as their int8 codes q = clamp(rint(a / in_scale),
//     -128, 127) (the srq grid the producing kernel writes them on), the dot product
//     Σ code·q is an exact integer, and t = fma(in_scale, Σ code·q, -2·sumA) rounds once.
//   in_scale == 0: Σ code·a accumulates in double, element by element in order (every
//     product is exact), and t = (float)(Σ - 2·sumA).
// logit = srq(scale[v]·t, outputScale).
void oracle_lm_head_exact(const uint32_t* packed, const float* scales, int64_t vocab, int hidden,
                          const float* act, const float* act_sum, int rows, float in_scale, float out_scale,
                          float* logits, int64_t ld_logits) {
  const int words = hidden / 16;
  std::vector<int> q(static_cast<size_t>(hidden));
  for (int b = 0; b < rows; ++b) {
    const float* a = act + static_cast<int64_t>(b) * hidden;
    if (in_scale != 0.0f)
      for (int j = 0; j < hidden; ++j) {
        float r = std::nearbyint(a[j] / in_scale);
        r = std::fmin(std::fmax(r, -128.0f), 127.0f);
        q[j] = static_cast<int>(r);
      }
    for (int64_t v = 0; v < vocab; ++v) {
      const uint32_t* row = packed + v * words;
      float t;
      if (in_scale != 0.0f) {
        int64_t s = 0;
        for (int j = 0; j < hidden; ++j) s += static_cast<int64_t>(o_code(row, j)) * q[j];
        t = std::fmaf(in_scale, static_cast<float>(s), -(2.0f * act_sum[b]));
      } else {
        double s = 0.0;
        for (int j = 0; j < hidden; ++j) s = s + static_cast<double>(o_code(row, j)) * static_cast<double>(a[j]);
        t = static_cast<float>(s - 2.0 * static_cast<double>(act_sum[b]));
      }
      logits[static_cast<int64_t>(b) * ld_logits + v] = o_srq(scales[v] * t, out_scale);
    }
  }
}

}  // extern "C"
