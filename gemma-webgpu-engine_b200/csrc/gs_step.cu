// Single-launch decode step: sampleToken (src/runtime/sampling.ts:18-65) for a few rows
// without a constraint table or a penalty history (a decode step with penalties off,
// C1's setting), in one kernel instead of a streaming pass plus a merge.
//
// One CTA per 2048-id unit of a row (512 threads, four ids each, one 16-byte load):
//   1. the unit's soft-capped logits, their maximum m and the sums of 2^((x - m)·log2e/T)
//      and e^(x - m);
//   2. a bound on the unit's k-th best key: each warp sorts its threads' best keys, and
//      the least of the warps' ceil(k/16)-th largest has 16·ceil(k/16) >= k threads, so
//      at least k values, at or above it.  Every pack (key32(x) << 32 | ~id: logit
//      descending, lower id first) at or above it goes to the unit's record, in no
//      order; warp 0 takes the record's best four (the head).  More ties at the bound
//      than the record holds: the unit's exact k2 best instead (warps sort their packs in
//      registers, the sixteen lists merge pairwise);
//   3. a release fence and a ticket on the row's counter; the last CTA of the row merges:
//      one record per thread, a bound on the row's k-th best pack (units' bests in groups
//      of 32, the least of the groups' ceil(k/g)-th largest), each unit's head packs at
//      or above it (a unit whose whole head reaches the bound is read in full), exact
//      order by rank counting; then one warp computes the probabilities and runs min-p,
//      typical-p, top-p and the seeded draw (gs_warp_filter.cuh, the warp merge's code;
//      one prefix scan when only top-p and the draw apply), writes the outputs and resets
//      the counter for the next call.
// The merge's arithmetic is the other merges' (same double operations, same order of the
// filters' prefix sums); only the order in which the normaliser's unit terms are added
// differs (a few ulp, far inside the 1e-6 parity bar).
#include "gs_device.cuh"
#include "gs_block.cuh"
#include "gs_warp_filter.cuh"
#include "gs_internal.cuh"
#include "gs_plan.cuh"
#include "../../include/gsampler.h"

namespace gs {

namespace {

constexpr int kStepIds = 2048;                   // ids per unit (one CTA)
constexpr int kStepThreads = 512;                // four ids per thread
constexpr int kStepWarps = kStepThreads / 32;    // sixteen sorted lists of 128 packs
constexpr int kStepMaxK = 64;                    // topK the step handles
constexpr int kStepMaxHist = 512;                // penalty history ids per row
constexpr int kStepHashLg = 10, kStepHash = 1 << kStepHashLg;  // the last CTA's history hash
constexpr int kStepMaxUnits = 512;               // vocabularies up to 1 M ids
constexpr int kStepRecPacks = 4;                  // record capacity: kStepRecPacks x k2 packs
constexpr int kStepMaxPacks = kStepMaxK * kStepRecPacks * kStepMaxK;  // packs at or above the bound: k units' records
constexpr int kStepSortSmem = 1024;              // candidate packs sorted in shared memory
// shared memory: the exact fallback's lists at k2 = 64, or the last CTA's arrays
constexpr int kStepSmemLast = kStepMaxUnits * (8 + 4 + 4) + 2 * kStepSortSmem * 8;
// with a penalty history, after those: the hash (keys, first positions, counts), the
// penalised entries, and the entries to order and their order
constexpr int kStepSmemHist =
    kStepSmemLast + 3 * kStepHash * 4 + kStepMaxHist * 16 + 2 * (kStepMaxHist + kStepMaxK) * 16;
constexpr int kStepSmemMax = kStepSmemHist;
static_assert(kStepSmemLast >= 2 * kStepWarps * kStepMaxK * 8, "the exact fallback's lists fit the last CTA's space");
static_assert(2 * kStepMaxHist <= kStepHash && kStepMaxHist <= kStepThreads, "history hash load and one slot per thread");

struct StepArgs {
  const void* logits;
  int64_t vocab;
  int64_t row_stride;
  float softcap;
  float inv_softcap;
  int32_t want_raw;
  int32_t units;        // CTAs per row
  int32_t k2;           // packs per unit record (power of two >= the batch's largest k)
  int32_t rec_bytes;
  const RowPlan* plans;  // per-row plans or nullptr (then plan0)
  RowPlan plan0;
  const double* uniforms;
  double* rng_state;
  int32_t* ids;
  double* logprob;
  uint32_t* flags;
  int32_t* cand_ids;
  double* cand_probs;
  int32_t* cand_count;
  int32_t cand_cap;
  unsigned char* recs;               // [rows][units] records
  unsigned long long* sort_scratch;  // [rows][kStepMaxPacks] (a row with many packs above the bound)
  unsigned* done;                    // [rows] CTAs of the row finished
  const int32_t* history;            // [rows][history_stride] penalty history ids, or nullptr
  const int32_t* history_len;
  const int32_t* history_count;      // [rows][history_stride] occurrences per entry, or nullptr (one each)
  int64_t history_stride;            // <= kStepMaxHist
  const uint32_t* mask_table;        // [mask_states][mask_words] allowed-id bitmask rows, or nullptr
  int32_t mask_states;
  int64_t mask_words;
  const int32_t* mask_state;         // [rows] row of the table (< 0: unconstrained)
};

constexpr int kStepHead = 4;  // a unit's best packs kept sorted in its record

struct StepRec {  // one unit's record; n packs follow (in no order)
  float m;        // max over the unit's live capped logits (not in the penalty history), -inf if none
  float raw_m;    // max over every id of the unit
  double s;       // sum 2^((x - m)·a2) over live ids
  double raw_s;   // sum e^(x - raw_m) over every id
  unsigned long long head[kStepHead];  // the unit's best live packs, descending (0: none)
  int32_t n;      // packs that follow: every live pack at or above the unit's bound (its k best among them)
  uint32_t flags;
  int32_t n_allowed;  // ids the constraint row allows
  int32_t pad;
};
static_assert(sizeof(StepRec) == 72, "record header");

// The warp's kStepHead best of the packs its lanes hold (every lane gets them, descending).
__device__ __forceinline__ void warp_head(const unsigned long long* v, int nv, unsigned long long* out) {
  unsigned long long c[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) c[q] = q < nv ? v[q] : 0ull;
#pragma unroll
  for (int r = 0; r < kStepHead; ++r) {
    unsigned long long lm = c[0];
#pragma unroll
    for (int q = 1; q < 4; ++q) lm = c[q] > lm ? c[q] : lm;
    unsigned long long wm = lm;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(kFullMask, wm, o);
      wm = t > wm ? t : wm;
    }
    out[r] = wm;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (wm != 0ull && c[q] == wm) c[q] = 0ull;  // (packs are distinct: one lane holds it)
  }
}

// Descending bitonic sort of 128 packs held four per lane (element lane·4 + q in v[q]).
__device__ __forceinline__ void warp_sort128_desc(unsigned long long (&v)[4], int lane) {
#pragma unroll
  for (int k = 2; k <= 128; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 4) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int i = lane * 4 + q;
          const unsigned long long p = __shfl_xor_sync(kFullMask, v[q], j >> 2);
          const bool lower = (i & j) == 0, desc = (i & k) == 0;
          const unsigned long long hi = v[q] > p ? v[q] : p, lo = v[q] > p ? p : v[q];
          v[q] = lower == desc ? hi : lo;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (q & j) continue;
          const int i = lane * 4 + q;
          const bool desc = (i & k) == 0;
          const unsigned long long a = v[q], b = v[q ^ j];
          if (desc ? a < b : a > b) {
            v[q] = b;
            v[q ^ j] = a;
          }
        }
      }
    }
  }
}

// The K2 (a power of two, <= 64) best of two descending lists a and b of K2 packs, sorted
// descending, by one warp: c[i] = max(a[i], b[K2-1-i]) is a bitonic sequence holding them,
// then half-cleaners sort it.  Element i sits in lane i & 31, register i >> 5.
__device__ __forceinline__ void warp_merge_top(const unsigned long long* a, const unsigned long long* b, int K2,
                                               unsigned long long* out, int lane) {
  unsigned long long c[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int i = q * 32 + lane;
    c[q] = 0ull;
    if (i < K2) {
      const unsigned long long x = a[i], y = b[K2 - 1 - i];
      c[q] = x > y ? x : y;
    }
  }
  if (K2 == 64) {  // h = 32: the two registers of a lane
    if (c[0] < c[1]) {
      const unsigned long long t = c[0];
      c[0] = c[1];
      c[1] = t;
    }
  }
  for (int h = (K2 < 32 ? K2 : 32) >> 1; h > 0; h >>= 1) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const unsigned long long p = __shfl_xor_sync(kFullMask, c[q], h);
      c[q] = (lane & h) == 0 ? (c[q] > p ? c[q] : p) : (c[q] > p ? p : c[q]);
    }
  }
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int i = q * 32 + lane;
    if (i < K2) out[i] = c[q];
  }
}

__device__ __forceinline__ double warp_max_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(kFullMask, v, o));
  return v;
}

// Descending block-wide bitonic sort of n2 (a power of two) packs in shared or global
// memory (this CTA's own: __syncthreads orders both).
__device__ void block_sort_desc(unsigned long long* v, int n2) {
  for (int k = 2; k <= n2; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n2; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long a = v[i], b = v[l];
          if ((i & k) == 0 ? a < b : a > b) {
            v[i] = b;
            v[l] = a;
          }
        }
      }
      __syncthreads();
    }
}

// The row's allowed-id bitmask (maskConstraintLogits: disallowed ids are -inf), or
// nullptr when the row has no constraint (no table, or a state of -1 / past the table:
// the latter is flagged invalid by the units).
__device__ __forceinline__ const uint32_t* step_mask_row(const StepArgs& A, int row) {
  if (A.mask_table == nullptr || A.mask_state == nullptr) return nullptr;
  const int32_t state = A.mask_state[row];
  return state >= 0 && state < A.mask_states ? A.mask_table + static_cast<int64_t>(state) * A.mask_words : nullptr;
}

// Fewer allowed ids than topK: the slots after the ordered entries' finite ones are the
// -inf ids (masked ones and -inf logits) in ascending id order, as the reference's
// stable descending sort leaves them (gemma-webgpu-engine/src/sampling.js:41-58 sorts the
// masked logits of maskConstraintLogits, :88-103).  One warp; returns the new count.
__device__ __noinline__ int step_fill_masked(Ent* sents, int ne, int k, const uint32_t* mrow, int64_t vocab,
                                             int* mids, Ent* tail) {
  const int lane = threadIdx.x & 31;
  const int nwords = static_cast<int>((vocab + 31) >> 5);
  int fill = 0;
  for (int w0 = 0; w0 < nwords && fill < k; w0 += 32) {  // (warp-uniform)
    const int wi = w0 + lane;
    uint32_t zero = 0u;
    if (wi < nwords) {
      zero = ~__ldg(mrow + wi);
      if (wi == nwords - 1 && (vocab & 31)) zero &= (1u << (vocab & 31)) - 1u;
    }
    const int c = __popc(zero);
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(kFullMask, incl, o);
      if (lane >= o) incl += u;
    }
    int base = fill + incl - c;
    for (uint32_t z = zero; z; z &= z - 1u) {
      if (base < k) mids[base] = wi * 32 + __ffs(z) - 1;
      ++base;
    }
    fill += __shfl_sync(kFullMask, incl, 31);
  }
  __syncwarp();
  const int n_masked = fill < k ? fill : k;
  int j0 = 0;  // the -inf tail of the ordered entries, merged with the masked ids by id
  while (j0 < ne && sents[j0].key > -INFINITY) ++j0;
  int t = 0;
  if (lane == 0) {
    int a = j0, b = 0;
    while (j0 + t < k && (a < ne || b < n_masked)) {
      if (b >= n_masked || (a < ne && sents[a].id < static_cast<uint32_t>(mids[b]))) tail[t++] = sents[a++];
      else tail[t++] = Ent{-INFINITY, static_cast<uint32_t>(mids[b++]), 2u};
    }
    for (int i = 0; i < t; ++i) sents[j0 + i] = tail[i];
  }
  t = __shfl_sync(kFullMask, t, 0);
  __syncwarp();
  return j0 + t;
}

// MINB: CTAs per SM the register budget allows (1: up to 128 registers a thread, for
// grids of at most one CTA per SM; 2: 64 registers, for batches of several rows).
template <int DT, int MINB>
__global__ void __launch_bounds__(kStepThreads, MINB) step_kernel(const __grid_constant__ StepArgs A) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ float s_wmax[kStepWarps], s_wrmax[kStepWarps];
  __shared__ uint32_t s_dead[kStepIds / 32];
  __shared__ double s_wsum[kStepWarps], s_wraw[kStepWarps];
  __shared__ uint32_t s_wkey[kStepWarps];
  __shared__ unsigned long long s_head[kStepHead], s_gtop[kStepWarps];
  __shared__ unsigned long long spk[kStepRecPacks * kStepMaxK];  // the record's packs
  __shared__ double s_r, s_st;
  __shared__ unsigned s_flags, s_wbad;
  __shared__ int s_last, s_n, s_nq;
  __shared__ int red_i[kStepWarps];
  __shared__ int s_pre[kStepMaxUnits + 1];
  const int S = A.units;
  const int row = blockIdx.x / S, unit = blockIdx.x - row * S;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const RowPlan* pp = A.plans ? A.plans + row : &A.plan0;
  const bool greedy = pp->mode == kModeGreedy;
  const int k = greedy ? 1 : pp->k_eff;
  const int K2 = A.k2;
  constexpr int ESZ = DT == GS_DTYPE_F32 ? 4 : 2;
  const unsigned char* rowbase = static_cast<const unsigned char*>(A.logits) + static_cast<int64_t>(row) * A.row_stride * ESZ;
  const float cap = A.softcap, inv_cap = A.inv_softcap;
  const float lim = cap != 0.0f ? INFINITY : 3.40282347e38f;  // raw x is an error when !(x <= lim)
  unsigned char* rec_row = A.recs + static_cast<int64_t>(row) * S * A.rec_bytes;

  // ---- 1. four ids per thread: capped logits; the unit maximum ----
  // (the history's length and this thread's history position load with the logits)
  int hl = 0;
  int32_t hid = -1;
  uint32_t hcn = 1u;  // occurrences the entry stands for
  if (A.history) {
    hl = A.history_len[row];
    if (tid < A.history_stride) {
      hid = A.history[static_cast<int64_t>(row) * A.history_stride + tid];
      if (A.history_count) hcn = static_cast<uint32_t>(max(A.history_count[static_cast<int64_t>(row) * A.history_stride + tid], 1));
    }
  }
  // the constraint row (sampling over maskConstraintLogits: disallowed ids are -inf)
  const int64_t id0 = static_cast<int64_t>(unit) * kStepIds + tid * 4;
  uint32_t allow4 = 0xfu;
  {
    const uint32_t* mrow = step_mask_row(A, row);
    if (mrow != nullptr && id0 < A.vocab) allow4 = (__ldg(mrow + (id0 >> 5)) >> (id0 & 31)) & 0xfu;
  }
  float x[4];
  bool valid[4];
  if (id0 + 3 < A.vocab) {
    if (DT == GS_DTYPE_F32) {
      const float4 v = ld_stream_f4(reinterpret_cast<const float4*>(rowbase + id0 * 4));
      x[0] = v.x;
      x[1] = v.y;
      x[2] = v.z;
      x[3] = v.w;
    } else {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(rowbase + id0 * 2));
      x[0] = bf16_lo(v.x);
      x[1] = bf16_hi(v.x);
      x[2] = bf16_lo(v.y);
      x[3] = bf16_hi(v.y);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) valid[q] = true;
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      valid[q] = id0 + q < A.vocab;
      x[q] = valid[q] ? load_logit(rowbase, DT, id0 + q) : 0.0f;
    }
  }
  // the row's penalty history ids in this unit are not live (the last CTA scores them)
  hl = hl < 0 ? 0 : (hl > A.history_stride ? static_cast<int>(A.history_stride) : hl);
  bool live[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) live[q] = valid[q] && ((allow4 >> q) & 1u);
  if (hl > 0) {  // (block-uniform; hl <= kStepMaxHist: one history position per thread)
    if (tid < kStepIds / 32) s_dead[tid] = 0u;
    __syncthreads();
    const int64_t off = static_cast<int64_t>(hid) - static_cast<int64_t>(unit) * kStepIds;
    if (tid < hl && off >= 0 && off < kStepIds) atomicOr(&s_dead[off >> 5], 1u << (off & 31));
    __syncthreads();
    const uint32_t dw = s_dead[tid >> 3] >> ((tid & 7) * 4);  // this thread's four ids
#pragma unroll
    for (int q = 0; q < 4; ++q) live[q] = live[q] && !((dw >> q) & 1u);
  }
  bool bad = false;
  float mx = -INFINITY, mraw = -INFINITY;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (!valid[q]) continue;
    bad |= !(x[q] <= lim);
    if (cap != 0.0f) x[q] = softcap(x[q], cap, inv_cap);
    mraw = fmaxf(mraw, x[q]);
    if (live[q]) mx = fmaxf(mx, x[q]);
  }
  {
    const float wm = warp_max(mx), wr = warp_max(mraw);
    if (lane == 0) {
      s_wmax[warp] = wm;
      s_wrmax[warp] = wr;
    }
  }
  if (tid == 0) {
    s_flags = 0u;
    s_wbad = 0u;
    s_n = 0;
  }
  __syncthreads();
  float m = s_wmax[0], mr = s_wrmax[0];
#pragma unroll
  for (int w = 1; w < kStepWarps; ++w) {
    m = fmaxf(m, s_wmax[w]);
    mr = fmaxf(mr, s_wrmax[w]);
  }

  // ---- 2. the sums; the packs; each warp's head and its threads' best keys ----
  float sa = 0.0f, sr = 0.0f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (!valid[q] || !(x[q] > -INFINITY)) continue;
    if (live[q] && m > -INFINITY) {
      const float d = x[q] - m;
      sa += ex2_approx(fmaf(d, pp->a2_lo, d * pp->a2_hi));
    }
    if (A.want_raw && mr > -INFINITY) {
      const float g = x[q] - mr;
      sr += ex2_approx(fmaf(g, kL2eLo, g * kL2eHi));
    }
  }
  unsigned long long v[4], tbest = 0ull;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    v[q] = live[q] ? make_pack(x[q], static_cast<uint32_t>(id0 + q)) : 0ull;
    tbest = v[q] > tbest ? v[q] : tbest;
  }
  // a bound on the unit's k-th best value: each warp's c-th largest thread best key
  // (c = ceil(k / 16)), the least of the sixteen (16·c >= k threads hold a value at or above it)
  uint32_t kk = static_cast<uint32_t>(tbest >> 32);  // (0: no value)
#pragma unroll
  for (int kw = 2; kw <= 32; kw <<= 1) {
#pragma unroll
    for (int j = kw >> 1; j > 0; j >>= 1) {
      const uint32_t p = __shfl_xor_sync(kFullMask, kk, j);
      kk = ((lane & j) == 0) == ((lane & kw) == 0) ? max(kk, p) : min(kk, p);
    }
  }
  const int cw = (k + kStepWarps - 1) / kStepWarps;  // <= 4
  if (lane == cw - 1) s_wkey[warp] = kk;
  {
    const double ws = warp_sum(static_cast<double>(sa)), wr = A.want_raw ? warp_sum(static_cast<double>(sr)) : 0.0;
    int na = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) na += valid[q] && ((allow4 >> q) & 1u);
    na = warp_sum_i(na);
    if (lane == 0) {
      s_wsum[warp] = ws;
      s_wraw[warp] = wr;
      red_i[warp] = na;
    }
  }
  if (__any_sync(kFullMask, bad) && lane == 0) atomicOr(&s_wbad, 1u);
  __syncthreads();
  kk = s_wkey[0];
#pragma unroll
  for (int w = 1; w < kStepWarps; ++w) kk = min(kk, s_wkey[w]);
  // the record keeps every pack whose key reaches the bound (at most kStepRecPacks·k2; a copy
  // stays in shared memory for the head)
  unsigned char* rec = rec_row + static_cast<int64_t>(unit) * A.rec_bytes;
  unsigned long long* rpk = reinterpret_cast<unsigned long long*>(rec + sizeof(StepRec));
  const int cap_rec = kStepRecPacks * K2;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const bool take = v[q] != 0ull && static_cast<uint32_t>(v[q] >> 32) >= kk;
    const unsigned bal = __ballot_sync(kFullMask, take);
    if (!bal) continue;
    const int leader = __ffs(bal) - 1;
    int at = 0;
    if (lane == leader) at = atomicAdd(&s_n, __popc(bal));
    at = __shfl_sync(kFullMask, at, leader) + __popc(bal & ((1u << lane) - 1u));
    if (take && at < cap_rec) {
      rpk[at] = v[q];
      spk[at] = v[q];
    }
  }
  __syncthreads();
  int n_rec = s_n;
  // the head: the best four of the record (the unit's best four when it holds four or more:
  // they all reach the bound then), by warp 0
  if (warp == 0 && n_rec <= cap_rec) {
    unsigned long long cur[kStepHead] = {0ull, 0ull, 0ull, 0ull};  // (the same in every lane)
    for (int b0 = 0; b0 < n_rec; b0 += 128) {
      unsigned long long hv[4], h[kStepHead];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int i = b0 + q * 32 + lane;
        hv[q] = i < n_rec ? spk[i] : 0ull;
      }
      warp_head(hv, 4, h);
      // the best four of two descending lists of four: the larger of cur[i] and h[3 - i]
      // (a bitonic sequence), then a sorting network
#pragma unroll
      for (int i = 0; i < kStepHead; ++i) cur[i] = cur[i] > h[kStepHead - 1 - i] ? cur[i] : h[kStepHead - 1 - i];
      auto cs = [](unsigned long long& x, unsigned long long& y) {
        if (x < y) {
          const unsigned long long t = x;
          x = y;
          y = t;
        }
      };
      cs(cur[0], cur[2]);
      cs(cur[1], cur[3]);
      cs(cur[0], cur[1]);
      cs(cur[2], cur[3]);
    }
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < kStepHead; ++i) s_head[i] = cur[i];
    }
    __syncwarp();
  }
  if (n_rec > cap_rec) {
    // ties at the bound beyond the record: the unit's exact k2 best, sorted (each warp
    // sorts its 128 packs, then the lists merge pairwise)
    warp_sort128_desc(v, lane);
    unsigned long long* la = reinterpret_cast<unsigned long long*>(dsm);  // [kStepWarps][K2], twice
    unsigned long long* lb = la + kStepWarps * K2;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int i = lane * 4 + q;
      if (i < K2) la[warp * K2 + i] = v[q];
    }
    __syncthreads();
    for (int nl = kStepWarps; nl > 1; nl >>= 1) {
      if (warp < (nl >> 1)) warp_merge_top(la + (2 * warp) * K2, la + (2 * warp + 1) * K2, K2, lb + warp * K2, lane);
      __syncthreads();
      unsigned long long* t = la;
      la = lb;
      lb = t;
    }
    for (int i = tid; i < K2; i += kStepThreads) rpk[i] = la[i];
    if (tid < kStepHead) s_head[tid] = tid < K2 ? la[tid] : 0ull;
    n_rec = K2;
    __syncthreads();
  }

  // ---- 3. the record, then a ticket ----
  if (tid == 0) {
    double su = 0.0, ru = 0.0;
    for (int w = 0; w < kStepWarps; ++w) {
      su = __dadd_rn(su, s_wsum[w]);
      ru = __dadd_rn(ru, s_wraw[w]);
    }
    StepRec r{};
    int na = 0;
    for (int w = 0; w < kStepWarps; ++w) na += red_i[w];
    r.n_allowed = na;
    r.m = m;
    r.raw_m = mr;
    r.s = m > -INFINITY ? su : 0.0;
    r.raw_s = mr > -INFINITY ? ru : 0.0;
    r.flags = (s_wbad ? GS_FLAG_ERR_NONFINITE : 0u) |
              (A.mask_table != nullptr && A.mask_state != nullptr && A.mask_state[row] >= A.mask_states
                   ? GS_FLAG_ERR_INVALID
                   : 0u);
#pragma unroll
    for (int i = 0; i < kStepHead; ++i) r.head[i] = s_head[i];
    r.n = n_rec;
    *reinterpret_cast<StepRec*>(rec) = r;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(A.done + row, 1u) == static_cast<unsigned>(S - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const uint32_t* mrow = step_mask_row(A, row);
  const bool has_mask = mrow != nullptr;
  // the history ids and their capped logits, early (random loads that overlap the records')
  uint32_t hv = 0xffffffffu;
  float hx = 0.0f;
  bool hallow = true;  // the history id is allowed by the constraint row
  if (tid < hl) {
    hv = static_cast<uint32_t>(hid);  // (negative ids are >= 2^31 here)
    if (hv < static_cast<uint64_t>(A.vocab)) {
      hx = load_logit(rowbase, DT, hv);
      if (cap != 0.0f) hx = softcap(hx, cap, inv_cap);
      if (has_mask) hallow = (__ldg(mrow + (hv >> 5)) >> (hv & 31)) & 1u;
    } else {
      hv = 0xffffffffu;
    }
  }
  if (tid == kStepThreads - 1 && !greedy) {  // the draw's uniform, early (its load overlaps the records')
    if (A.uniforms) {
      s_r = A.uniforms[row];
    } else {
      double st = A.rng_state[row];
      s_r = seeded_next(&st);
      s_st = st;
    }
  }

  // ---- 4. the last CTA of the row: one unit's record per thread; the bound; the
  //      candidates ----
  unsigned char* wwork = dsm;                                   // [4096] the warp filters' work
  int* un = reinterpret_cast<int*>(dsm + 4096);                 // [kStepMaxUnits] record sizes
  int* qlist = un + kStepMaxUnits;                              // [kStepMaxUnits] units read in full
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(qlist + kStepMaxUnits);  // [kStepSortSmem]
  unsigned long long* srt = cand + kStepSortSmem;                                          // [kStepSortSmem]
  unsigned long long* scratch = A.sort_scratch + static_cast<int64_t>(row) * kStepMaxPacks;
  float mu = -INFINITY, rmu = -INFINITY;
  double su = 0.0, ru = 0.0;
  int na_u = 0;
  unsigned long long hd[kStepHead] = {0ull, 0ull, 0ull, 0ull};
  if (tid < S) {
    const StepRec* st = reinterpret_cast<const StepRec*>(rec_row + static_cast<int64_t>(tid) * A.rec_bytes);
    mu = __ldcg(&st->m);
    rmu = __ldcg(&st->raw_m);
    su = __ldcg(&st->s);
    ru = __ldcg(&st->raw_s);
    const unsigned f = __ldcg(&st->flags);
#pragma unroll
    for (int i = 0; i < kStepHead; ++i) hd[i] = __ldcg(&st->head[i]);
    un[tid] = __ldcg(&st->n);
    na_u = __ldcg(&st->n_allowed);
    if (f) atomicOr(&s_flags, f);
  }
  if (tid == 0) {
    s_n = 0;
    s_nq = 0;
  }
  // the bound: the units' best keys in groups of 32, each group sorted by one warp; with g
  // groups, the least of the groups' c-th largest key (c = ceil(k / g)) has g·c >= k unit
  // bests at or above it (none when c > 32 or a group holds fewer than c)
  const int g = (S + 31) >> 5, cg = (k + g - 1) / g;
  if (warp < g) {
    const unsigned long long b = hd[0];  // (thread u holds unit u's record)
    uint32_t key = static_cast<uint32_t>(b >> 32);
#pragma unroll
    for (int kw = 2; kw <= 32; kw <<= 1) {
#pragma unroll
      for (int j = kw >> 1; j > 0; j >>= 1) {
        const uint32_t p = __shfl_xor_sync(kFullMask, key, j);
        key = ((lane & j) == 0) == ((lane & kw) == 0) ? max(key, p) : min(key, p);
      }
    }
    unsigned long long wt = b;
    float wr = rmu;
    int wn = na_u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(kFullMask, wt, o);
      wt = t > wt ? t : wt;
      wr = fmaxf(wr, __shfl_xor_sync(kFullMask, wr, o));
      wn += __shfl_xor_sync(kFullMask, wn, o);
    }
    const uint32_t kc = __shfl_sync(kFullMask, key, cg <= 32 ? cg - 1 : 0);
    if (lane == 0) {
      s_wkey[warp] = cg <= 32 ? kc : 0u;
      s_gtop[warp] = wt;
      s_wrmax[warp] = wr;
      red_i[warp] = wn;
    }
  }
  __syncthreads();
  int64_t na_row = 0;  // ids the constraint row allows
  for (int w = 0; w < g; ++w) na_row += red_i[w];
  uint32_t tk = s_wkey[0];
  unsigned long long top = s_gtop[0];
  float Mx = s_wrmax[0];  // the row's raw maximum (every id)
  for (int w = 1; w < g; ++w) {
    tk = min(tk, s_wkey[w]);
    top = s_gtop[w] > top ? s_gtop[w] : top;
    Mx = fmaxf(Mx, s_wrmax[w]);
  }
  unsigned fl = s_flags;
  if (greedy) fl |= GS_FLAG_GREEDY;
  if (has_mask && na_row == 0) fl |= GS_FLAG_ERR_DEADEND;
  const double T = pp->temperature;
  const double xtop = static_cast<double>(pack_value(top));
  double M = top == 0ull ? -INFINITY : (greedy ? xtop : __ddiv_rn(xtop, T));
  // penalised entries (sampling.ts:21-30): the distinct history ids, counted in a shared
  // hash, each scored exactly in double at its first position's slot
  Ent* pent = reinterpret_cast<Ent*>(dsm + kStepSmemLast + 3 * kStepHash * 4);  // [kStepMaxHist]
  if (hl > 0) {  // (block-uniform; hl <= kStepMaxHist: one history position per thread)
    int lg = 6;  // a table of at least twice the history's length
    while ((1 << lg) < 2 * hl) ++lg;
    const uint32_t nslot = 1u << lg;
    uint32_t* hk = reinterpret_cast<uint32_t*>(dsm + kStepSmemLast);
    uint32_t* hfirst = hk + kStepHash;
    uint32_t* hcnt = hfirst + kStepHash;
    for (uint32_t i = tid; i < nslot; i += kStepThreads) {
      hk[i] = 0xffffffffu;
      hfirst[i] = 0xffffffffu;
      hcnt[i] = 0u;
    }
    __syncthreads();
    auto slot_of = [&](uint32_t v, bool insert) {
      uint32_t sl = (v * 2654435761u) >> (32 - lg);
      for (;;) {  // at most hl distinct ids in >= 2·hl slots: a free slot exists
        const uint32_t kv = insert ? atomicCAS(&hk[sl], 0xffffffffu, v) : hk[sl];
        if (kv == 0xffffffffu || kv == v) return sl;
        sl = (sl + 1) & (nslot - 1);
      }
    };
    uint32_t sl = 0;
    if (hv != 0xffffffffu) {
      sl = slot_of(hv, true);
      atomicAdd(&hcnt[sl], hcn);
      atomicMin(&hfirst[sl], static_cast<uint32_t>(tid));
    }
    __syncthreads();
    double pmax = -INFINITY;
    const double rp = pp->repetition_penalty, pres = pp->presence_penalty, freq = pp->frequency_penalty;
    if (tid < hl) {
      Ent e{-INFINITY, 0xffffffffu, 0xffffffffu};
      if (hv != 0xffffffffu && hallow && hfirst[sl] == static_cast<uint32_t>(tid)) {
        const double xp = penalise(static_cast<double>(hx), static_cast<double>(hcnt[sl]), rp, pres, freq);
        e = Ent{greedy ? xp : __ddiv_rn(xp, T), hv, 1u};
        pmax = e.key;
      }
      pent[tid] = e;
    }
    pmax = warp_max_d(pmax);
    if (lane == 0) s_wsum[warp] = pmax;
    __syncthreads();
    for (int w = 0; w < kStepWarps; ++w) M = fmax(M, s_wsum[w]);
    __syncthreads();
  }
  // per unit: the normaliser's and the raw sum's terms; its head packs whose key reaches the
  // bound, or, when its whole head does (it may hold more), the unit for a full read
  {
    double part = 0.0, rpart = 0.0;
    if (tid < S && mu > -INFINITY && !greedy && M > -INFINITY)
      part = __dmul_rn(su, exp(__dsub_rn(__ddiv_rn(static_cast<double>(mu), T), M)));
    if (tid < S && rmu > -INFINITY && A.want_raw) rpart = __dmul_rn(ru, exp(static_cast<double>(rmu) - static_cast<double>(Mx)));
    if (tid < hl && !greedy && M > -INFINITY && pent[tid].id != 0xffffffffu)
      part = __dadd_rn(part, exp(__dsub_rn(pent[tid].key, M)));  // (hl <= kStepMaxHist = the block's threads)
    part = warp_sum(part);
    rpart = warp_sum(rpart);
    if (lane == 0) {
      s_wsum[warp] = part;
      s_wraw[warp] = rpart;
    }
  }
  auto append = [&](bool take, unsigned long long p) {
    const unsigned bal = __ballot_sync(kFullMask, take);
    if (!bal) return;
    const int leader = __ffs(bal) - 1;
    int at = 0;
    if (lane == leader) at = atomicAdd(&s_n, __popc(bal));
    at = __shfl_sync(kFullMask, at, leader) + __popc(bal & ((1u << lane) - 1u));
    if (take) {
      if (at < kStepSortSmem) cand[at] = p;
      if (at < kStepMaxPacks) scratch[at] = p;
    }
  };
  auto reaches = [&](unsigned long long p) { return p != 0ull && static_cast<uint32_t>(p >> 32) >= tk; };
  {
    const bool over = tid < S && reaches(hd[kStepHead - 1]);
#pragma unroll
    for (int i = 0; i < kStepHead; ++i) append(tid < S && !over && reaches(hd[i]), hd[i]);
    const unsigned bal = __ballot_sync(kFullMask, over);
    if (bal) {
      const int leader = __ffs(bal) - 1;
      int at = 0;
      if (lane == leader) at = atomicAdd(&s_nq, __popc(bal));
      at = __shfl_sync(kFullMask, at, leader) + __popc(bal & ((1u << lane) - 1u));
      if (over) qlist[at] = tid;
    }
  }
  __syncthreads();
  double total = 0.0, rs = 0.0;
  for (int w = 0; w < kStepWarps; ++w) {
    total = __dadd_rn(total, s_wsum[w]);
    rs = __dadd_rn(rs, s_wraw[w]);
  }
  const int nq = s_nq;
  if (nq > 0) {
    // the full records of those units, flattened (an exclusive prefix of their sizes), four
    // loads per thread in flight
    const int cu = tid < nq ? un[qlist[tid]] : 0;
    int incl = cu;
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(kFullMask, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) red_i[warp] = incl;
    __syncthreads();
    int before = 0, tot = 0;
    for (int w = 0; w < kStepWarps; ++w) {
      if (w < warp) before += red_i[w];
      tot += red_i[w];
    }
    if (tid < nq) s_pre[tid] = before + incl - cu;
    if (tid == 0) s_pre[nq] = tot;
    __syncthreads();
    const int P = s_pre[nq];
    for (int f0 = 0; f0 < P; f0 += 4 * kStepThreads) {
      unsigned long long p[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int f = f0 + q * kStepThreads + tid;
        p[q] = 0ull;
        if (f < P) {
          int lo = 0, hi = nq - 1;  // the last qi with s_pre[qi] <= f
          while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (s_pre[mid] <= f) lo = mid;
            else hi = mid - 1;
          }
          p[q] = __ldcg(reinterpret_cast<const unsigned long long*>(rec_row + static_cast<int64_t>(qlist[lo]) * A.rec_bytes +
                                                                     sizeof(StepRec)) + (f - s_pre[lo]));
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) append(reaches(p[q]), p[q]);
    }
    __syncthreads();
  }
  const int N = s_n < kStepMaxPacks ? s_n : kStepMaxPacks;
  const unsigned long long* sorted;
  if (N <= 512) {
    // exact order by rank counting (the packs are distinct)
    for (int i = tid; i < N; i += kStepThreads) {
      const unsigned long long p = cand[i];
      int r = 0;
      for (int j = 0; j < N; ++j) r += cand[j] > p;
      srt[r] = p;
    }
    sorted = srt;
  } else {
    unsigned long long* cbuf = N <= kStepSortSmem ? cand : scratch;
    const int n2 = pow2_ceil(N);
    for (int i = N + tid; i < n2; i += kStepThreads) cbuf[i] = 0ull;
    __syncthreads();
    block_sort_desc(cbuf, n2);
    sorted = cbuf;
  }
  __syncthreads();
  // with penalised entries: the k best live packs and the penalised entries in the
  // reference's order (key descending, lower id first), by rank counting
  Ent* sents = nullptr;
  int ne = 0;
  if (hl > 0 || has_mask) {  // (block-uniform)
    Ent* ents = pent + kStepMaxHist;        // [kStepMaxHist + kStepMaxK]
    Ent* sw = ents + kStepMaxHist + kStepMaxK;  // [kStepMaxHist + kStepMaxK]
    const int nL = N < k ? N : k;
    for (int i = tid; i < nL; i += kStepThreads) {
      const unsigned long long p = sorted[i];
      const double xv = static_cast<double>(pack_value(p));
      ents[i] = Ent{greedy ? xv : __ddiv_rn(xv, T), pack_id(p), 0u};
    }
    if (tid == 0) s_nq = 0;
    __syncthreads();
    {
      const bool take = tid < hl && hl > 0 && pent[tid].id != 0xffffffffu;
      const unsigned bal = __ballot_sync(kFullMask, take);
      if (bal) {
        const int leader = __ffs(bal) - 1;
        int at = 0;
        if (lane == leader) at = atomicAdd(&s_nq, __popc(bal));
        at = __shfl_sync(kFullMask, at, leader) + __popc(bal & ((1u << lane) - 1u));
        if (take) ents[nL + at] = pent[tid];
      }
    }
    __syncthreads();
    ne = nL + s_nq;
    for (int i = tid; i < ne; i += kStepThreads) {
      const Ent e = ents[i];
      int r = 0;
      for (int j = 0; j < ne; ++j) r += ent_before(ents[j], e);
      sw[r] = e;
    }
    __syncthreads();
    sents = sw;
  }
  if (warp != 0) return;

  // ---- 5. one warp: probabilities, filters, draw, outputs ----
  const int nAll = sents ? ne : N;
  int nC = nAll < k ? nAll : k;
  if (sents && has_mask && !greedy && ne < k && na_row < A.vocab)
    nC = step_fill_masked(sents, ne, k, mrow, A.vocab, reinterpret_cast<int*>(wwork + 2560),
                          reinterpret_cast<Ent*>(wwork + 2816));
  WWork w;
  {
    unsigned char* p = wwork;
    const int kc2 = K2;
    w.cp = reinterpret_cast<double*>(p);
    p += kc2 * 8;
    w.cum = reinterpret_cast<double*>(p);
    p += kc2 * 8;
    w.skey = reinterpret_cast<unsigned long long*>(p);
    p += kc2 * 8;
    w.cid = reinterpret_cast<uint32_t*>(p);
    p += kc2 * 4;
    w.sval = reinterpret_cast<uint32_t*>(p);
    p += kc2 * 4;
    w.pos = reinterpret_cast<int*>(p);
    p += kc2 * 4;
    w.flg = p;
  }
  uint32_t tok = 0xffffffffu;
  int n_final = 0;
  if (!(fl & GS_FLAG_ERRORS)) {
    if (greedy) {
      // argmax over the whole vocabulary: all -inf -> id 0 (sampling.ts:92-96)
      if (sents) tok = (ne == 0 || !(sents[0].key > -INFINITY)) ? 0u : sents[0].id;
      else tok = (top == 0ull || !(xtop > -INFINITY)) ? 0u : pack_id(top);
      if (lane == 0) {
        w.cid[0] = tok;
        w.cp[0] = 1.0;
      }
      n_final = 1;
    } else {
      if (!(M > -INFINITY)) {
        fl |= GS_FLAG_ERR_NONFINITE;  // every logit -inf: outside the domain
      } else {
#pragma unroll
        for (int q = 0; q < kStepMaxK / 32; ++q) {  // (independent chains)
          const int i = q * 32 + lane;
          if (i < nC) {
            double key;
            uint32_t id;
            if (sents) {
              key = sents[i].key;
              id = sents[i].id;
            } else {
              const unsigned long long pk = sorted[i];
              key = __ddiv_rn(static_cast<double>(pack_value(pk)), T);
              id = pack_id(pk);
            }
            w.cid[i] = id;
            w.cp[i] = __ddiv_rn(exp(__dsub_rn(key, M)), total);
          }
        }
        const double r = s_r;
        if (!A.uniforms && lane == 0) A.rng_state[row] = s_st;
        __syncwarp();
        if (!(pp->min_p > 0) && !(pp->typical_p < 1)) {
          // top-p and the draw only: the draw's running sums over the kept prefix are the
          // first entries of the top-p cut's (same prefix-sum order), so one scan serves both
          warp_scan4_d(w.cp, w.cum, nC, lane);
          int n = nC;
          if (pp->top_p < 1) {
            const double t = pp->top_p;
            const int below = warp_count_below(w.cum, nC, t, lane);
            n = below + 1 < nC ? below + 1 : nC;
            double m = fabs(w.cum[n - 1] - t);
            if (n >= 2) m = fmin(m, fabs(w.cum[n - 2] - t));
            if (m <= kBoundaryRel * t) fl |= GS_FLAG_BOUNDARY_TOP_P;
          }
          const double ct = w.cum[n - 1];
          const double cursor = __dmul_rn(r, ct);
          const int below = warp_count_below(w.cum, n, cursor, lane);
          if (below < n) {
            tok = w.cid[below];
          } else {
            tok = w.cid[n - 1];
            fl |= GS_FLAG_FELL_THROUGH;
          }
          const int j = below < n ? below : n - 1;
          double m = fabs(w.cum[j] - cursor);
          if (j >= 1) m = fmin(m, fabs(w.cum[j - 1] - cursor));
          if (m <= kBoundaryRel * ct) fl |= GS_FLAG_BOUNDARY_DRAW;
          n_final = n;
        } else {
          tok = warp_filter_and_draw(w, nC, pp->min_p, pp->typical_p, pp->top_p, r, &n_final, &fl, lane);
        }
      }
    }
  }
  __syncwarp();
  const bool err = (fl & GS_FLAG_ERRORS) != 0;
  if (lane == 0) {
    A.ids[row] = err ? -1 : static_cast<int32_t>(tok);
    if (A.flags) A.flags[row] = fl;
    if (A.cand_count) A.cand_count[row] = err ? 0 : n_final;
    if (A.logprob) {
      double lp = NAN;
      if (!err) {
        float xv = load_logit(rowbase, DT, tok);
        if (cap != 0.0f) xv = softcap(xv, cap, inv_cap);
        lp = __dsub_rn(__dsub_rn(static_cast<double>(xv), static_cast<double>(Mx)), log(rs));
      }
      A.logprob[row] = lp;
    }
    A.done[row] = 0u;  // ready for the next call (stream order)
  }
  if (A.cand_ids) {
    const int nw = err ? 0 : (n_final < A.cand_cap ? n_final : A.cand_cap);
    for (int i = lane; i < A.cand_cap; i += 32) {
      A.cand_ids[static_cast<int64_t>(row) * A.cand_cap + i] = i < nw ? static_cast<int32_t>(w.cid[i]) : -1;
      if (A.cand_probs) A.cand_probs[static_cast<int64_t>(row) * A.cand_cap + i] = i < nw ? w.cp[i] : 0.0;
    }
  }
}

int pow2_at_least(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

}  // namespace

bool step_eligible(const gs_batch* b, int kmax, bool any_large, int rows) {
  if (rows < 1 || rows > kStepDoneRows || any_large || kmax < 1 || kmax > kStepMaxK) return false;
  if (b->history && b->history_stride > kStepMaxHist) return false;
  if (b->dtype != GS_DTYPE_F32 && b->dtype != GS_DTYPE_BF16) return false;
  const int64_t esz = b->dtype == GS_DTYPE_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(b->logits) & 15) != 0 || (b->row_stride * esz) % 16 != 0) return false;
  const int64_t units = (b->vocab + kStepIds - 1) / kStepIds;
  return units <= kStepMaxUnits;
}

size_t step_ws_bytes(int rows, int64_t vocab, int kmax) {
  const int64_t units = (vocab + kStepIds - 1) / kStepIds;
  const size_t rec = sizeof(StepRec) + 8 * static_cast<size_t>(kStepRecPacks) * pow2_at_least(kmax);
  return align_up(static_cast<size_t>(rows) * units * rec, 256) + static_cast<size_t>(rows) * kStepMaxPacks * 8;
}

cudaError_t launch_step(const gs_batch* b, const gs_outputs* o, const RowPlan& plan0, const RowPlan* dplans, int kmax,
                        unsigned char* ws, unsigned* done, cudaStream_t st) {
  StepArgs a{};
  a.logits = b->logits;
  a.vocab = b->vocab;
  a.row_stride = b->row_stride;
  a.softcap = b->softcap;
  a.inv_softcap = b->softcap != 0.0f ? static_cast<float>(1.0 / static_cast<double>(b->softcap)) : 0.0f;
  a.want_raw = o->logprob != nullptr;
  a.plans = dplans;
  a.plan0 = plan0;
  a.uniforms = b->uniforms;
  a.rng_state = b->rng_state;
  a.ids = o->ids;
  a.logprob = o->logprob;
  a.flags = o->flags;
  a.cand_ids = o->cand_ids;
  a.cand_probs = o->cand_probs;
  a.cand_count = o->cand_count;
  a.cand_cap = o->cand_cap;
  a.units = static_cast<int32_t>((b->vocab + kStepIds - 1) / kStepIds);
  a.k2 = pow2_at_least(kmax);
  a.rec_bytes = static_cast<int32_t>(sizeof(StepRec) + 8 * static_cast<size_t>(kStepRecPacks) * a.k2);
  a.recs = ws;
  a.sort_scratch = reinterpret_cast<unsigned long long*>(ws + align_up(static_cast<size_t>(b->rows) * a.units * a.rec_bytes, 256));
  a.done = done;
  a.history = b->history;
  a.history_len = b->history ? b->history_len : nullptr;
  a.history_count = b->history ? b->history_count : nullptr;
  a.history_stride = b->history ? b->history_stride : 0;
  a.mask_table = b->mask_table;
  a.mask_states = b->mask_states;
  a.mask_words = b->mask_words;
  a.mask_state = b->mask_table ? b->mask_state : nullptr;
  // shared memory: the merge tree's two list sets, or the last CTA's arrays
  const size_t tree = 2 * static_cast<size_t>(kStepWarps) * a.k2 * 8;
  const size_t last = (b->history || b->mask_table) ? kStepSmemHist : kStepSmemLast;
  const size_t smem = tree > last ? tree : last;
  const int grid = b->rows * a.units;
  static std::atomic<uint64_t> attr{0};  // (set on each device's first call)
  if (device_todo(attr)) {
    cudaFuncSetAttribute(step_kernel<GS_DTYPE_F32, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStepSmemMax);
    cudaFuncSetAttribute(step_kernel<GS_DTYPE_BF16, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStepSmemMax);
    cudaFuncSetAttribute(step_kernel<GS_DTYPE_F32, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStepSmemMax);
    cudaFuncSetAttribute(step_kernel<GS_DTYPE_BF16, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStepSmemMax);
    mark_device_done(attr);
  }
  // one CTA per SM at most (a B = 1 call at V = 262144: 128 units): the larger register
  // budget (no spills); more: two CTAs per SM, halving the waves of an 8-row batch
  const bool one = grid <= sm_count();
  if (b->dtype == GS_DTYPE_F32) {
    if (one) step_kernel<GS_DTYPE_F32, 1><<<grid, kStepThreads, smem, st>>>(a);
    else step_kernel<GS_DTYPE_F32, 2><<<grid, kStepThreads, smem, st>>>(a);
  } else {
    if (one) step_kernel<GS_DTYPE_BF16, 1><<<grid, kStepThreads, smem, st>>>(a);
    else step_kernel<GS_DTYPE_BF16, 2><<<grid, kStepThreads, smem, st>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace gs
