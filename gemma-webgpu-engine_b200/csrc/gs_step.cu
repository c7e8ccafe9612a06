// Single-launch decode step: sampleToken (src/runtime/sampling.ts:18-65) for a few rows
// without a constraint table or a penalty history (a decode step with penalties off,
// C1's setting), in one kernel instead of a streaming pass plus a merge.
//
// One CTA per 2048-id unit of a row (512 threads, four ids each, one 16-byte load):
//   1. the unit's soft-capped logits, their maximum m and the sums of 2^((x - m)·log2e/T)
//      and e^(x - m) (block reductions in a fixed order);
//   2. the unit's best packs (key32(x) << 32 | ~id: logit descending, lower id first):
//      each warp sorts its 128 packs in registers (a bitonic network over the lanes), and
//      the sixteen sorted lists are merged pairwise down to the unit's k2 best, sorted;
//   3. the unit's record (statistics and sorted packs) goes to the workspace and the CTA
//      takes a ticket from the row's counter; the last CTA of the row merges the records:
//      the k-th largest unit maximum bounds the row's k-th best pack (k units hold a
//      pack at or above it), so only each unit's packs at or above that bound are read
//      (a handful per row) and sorted; then the maximum, the full-vocabulary normaliser,
//      probabilities, min-p, typical-p, top-p and the seeded draw run in one warp
//      (gs_warp_filter.cuh, the warp merge's code), and the counter is reset for the next
//      call.
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
constexpr int kStepMaxUnits = 512;               // vocabularies up to 1 M ids
constexpr int kStepMaxPacks = 8192;              // units x k2 (the bound's worst case)
constexpr int kStepSortSmem = 1024;              // candidate packs sorted in shared memory

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
};

struct StepRec {  // one unit's record; k2 packs follow (sorted, descending; 0 = none)
  float m;        // max over the unit's capped logits, -inf if none
  float pad0;
  double s;       // sum 2^((x - m)·a2)
  double raw_s;   // sum e^(x - m) (every id is live: m is also the raw maximum)
  uint32_t flags;
  int32_t pad1;
};
static_assert(sizeof(StepRec) == 32, "record header");

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

template <int DT>
__global__ void __launch_bounds__(kStepThreads) step_kernel(const __grid_constant__ StepArgs A) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ float red_f[kStepWarps];
  __shared__ double red_d[32];
  __shared__ int red_i[32];
  __shared__ unsigned s_flags;
  __shared__ int s_last, s_n;
  __shared__ unsigned long long s_tau;
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

  // ---- 1. four ids per thread: capped logits, maximum, sums ----
  const int64_t id0 = static_cast<int64_t>(unit) * kStepIds + tid * 4;
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
  int bad = 0;
  float mx = -INFINITY;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (!valid[q]) continue;
    bad |= !(x[q] <= lim);
    if (cap != 0.0f) x[q] = softcap(x[q], cap, inv_cap);
    mx = fmaxf(mx, x[q]);
  }
  if (tid == 0) s_flags = 0u;
  const float m = block_max_f(mx, red_f);
  bad = __syncthreads_or(bad);
  float sa = 0.0f, sr = 0.0f;
  if (m > -INFINITY) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (!valid[q] || !(x[q] > -INFINITY)) continue;
      const float d = x[q] - m;
      sa += ex2_approx(fmaf(d, pp->a2_lo, d * pp->a2_hi));
      if (A.want_raw) sr += ex2_approx(fmaf(d, kL2eLo, d * kL2eHi));
    }
  }
  const double s_unit = block_sum_d(static_cast<double>(sa), red_d);
  const double r_unit = A.want_raw ? block_sum_d(static_cast<double>(sr), red_d) : 0.0;

  // ---- 2. the unit's k2 best packs, sorted ----
  unsigned long long v[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) v[q] = valid[q] ? make_pack(x[q], static_cast<uint32_t>(id0 + q)) : 0ull;
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
    // lists 2j and 2j+1 -> list j: the larger of A[i] and B[K2-1-i] is a bitonic sequence
    // holding the K2 best of both, then half-cleaners sort it
    for (int t = tid; t < (nl >> 1) * K2; t += kStepThreads) {
      const int j = t / K2, i = t - j * K2;
      const unsigned long long a = la[(2 * j) * K2 + i], b = la[(2 * j + 1) * K2 + (K2 - 1 - i)];
      lb[j * K2 + i] = a > b ? a : b;
    }
    __syncthreads();
    for (int h = K2 >> 1; h > 0; h >>= 1) {
      for (int t = tid; t < (nl >> 1) * (K2 >> 1); t += kStepThreads) {
        const int j = t / (K2 >> 1), r = t - j * (K2 >> 1);
        const int i = ((r / h) * 2 * h) + (r % h);  // lower element of the pair (i, i + h)
        unsigned long long* c = lb + j * K2;
        const unsigned long long a = c[i], b = c[i + h];
        if (a < b) {
          c[i] = b;
          c[i + h] = a;
        }
      }
      __syncthreads();
    }
    unsigned long long* t = la;
    la = lb;
    lb = t;
  }

  // ---- 3. the record, then a ticket ----
  unsigned char* rec = rec_row + static_cast<int64_t>(unit) * A.rec_bytes;
  unsigned long long* rpk = reinterpret_cast<unsigned long long*>(rec + sizeof(StepRec));
  for (int i = tid; i < K2; i += kStepThreads) rpk[i] = la[i];
  if (tid == 0) {
    StepRec r{};
    r.m = m;
    r.s = m > -INFINITY ? s_unit : 0.0;
    r.raw_s = m > -INFINITY ? r_unit : 0.0;
    r.flags = bad ? GS_FLAG_ERR_NONFINITE : 0u;
    *reinterpret_cast<StepRec*>(rec) = r;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(A.done + row, 1u) == static_cast<unsigned>(S - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // ---- 4. the last CTA of the row: statistics over the units ----
  unsigned fl = 0;
  float um = -INFINITY;
  unsigned long long* umax = reinterpret_cast<unsigned long long*>(dsm);  // [S] each unit's best pack
  int* ucnt = reinterpret_cast<int*>(umax + kStepMaxUnits);              // [S + 1] packs above the bound, prefix
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(ucnt + kStepMaxUnits + 8);  // [kStepSortSmem]
  for (int u = tid; u < S; u += kStepThreads) {
    const unsigned char* r = rec_row + static_cast<int64_t>(u) * A.rec_bytes;
    const StepRec* st = reinterpret_cast<const StepRec*>(r);
    fl |= __ldcg(&st->flags);
    um = fmaxf(um, __ldcg(&st->m));
    umax[u] = __ldcg(reinterpret_cast<const unsigned long long*>(r + sizeof(StepRec)));
  }
  if (fl) atomicOr(&s_flags, fl);
  const float Mx = block_max_f(um, red_f);  // (the raw maximum too)
  if (tid == 0) s_tau = 0ull;
  __syncthreads();
  fl = s_flags;
  if (greedy) fl |= GS_FLAG_GREEDY;
  // the bound: the k-th largest unit maximum (none when fewer than k units hold packs)
  for (int u = tid; u < S; u += kStepThreads) {
    const unsigned long long mu = umax[u];
    int above = 0;
    for (int q = 0; q < S; ++q) above += umax[q] > mu;
    if (mu != 0ull && above == k - 1) s_tau = mu;
  }
  __syncthreads();
  const unsigned long long tau = s_tau;
  // each unit's packs at or above the bound (its list is sorted: a binary search)
  int c = 0;
  if (tid < S) {
    const unsigned long long* pk = reinterpret_cast<const unsigned long long*>(rec_row + static_cast<int64_t>(tid) * A.rec_bytes + sizeof(StepRec));
    int lo = 0, hi = K2;  // first index whose pack is below the bound (or empty)
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      const unsigned long long p = __ldcg(pk + mid);
      if (p != 0ull && p >= tau) lo = mid + 1;
      else hi = mid;
    }
    c = lo;
  }
  {
    int incl = c;
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
    if (tid < S) ucnt[tid] = before + incl - c;
    if (tid == 0) s_n = tot;
    __syncthreads();
  }
  const int N = s_n;
  unsigned long long* cbuf = N <= kStepSortSmem ? cand : A.sort_scratch + static_cast<int64_t>(row) * kStepMaxPacks;
  const int n2 = pow2_ceil(N > 0 ? N : 1);
  if (tid < S) {
    const unsigned long long* pk = reinterpret_cast<const unsigned long long*>(rec_row + static_cast<int64_t>(tid) * A.rec_bytes + sizeof(StepRec));
    for (int i = 0; i < c; ++i) cbuf[ucnt[tid] + i] = __ldcg(pk + i);
  }
  for (int i = N + tid; i < n2; i += kStepThreads) cbuf[i] = 0ull;
  __syncthreads();
  unsigned long long best[4] = {0ull, 0ull, 0ull, 0ull};  // warp 0: the row's best packs, lane·4 + q
  if (n2 <= 128) {
    if (warp == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) best[q] = lane * 4 + q < n2 ? cbuf[lane * 4 + q] : 0ull;
      warp_sort128_desc(best, lane);
    }
  } else {
    block_sort_desc(cbuf, n2);
    if (warp == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) best[q] = lane * 4 + q < N ? cbuf[lane * 4 + q] : 0ull;
    }
  }
  __syncthreads();
  if (warp != 0) return;

  // ---- 5. one warp: probabilities, filters, draw, outputs ----
  const double T = pp->temperature;
  const int nC = N < k ? N : k;
  WWork w;
  {
    unsigned char* p = reinterpret_cast<unsigned char*>(cand);  // (the candidates now sit in registers)
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
  double rs = 0.0;
  if (A.want_raw && Mx > -INFINITY) {
    for (int u = lane; u < S; u += 32) {
      const StepRec* st = reinterpret_cast<const StepRec*>(rec_row + static_cast<int64_t>(u) * A.rec_bytes);
      const float mu = __ldcg(&st->m);
      if (mu > -INFINITY) rs = __dadd_rn(rs, __dmul_rn(__ldcg(&st->raw_s), exp(static_cast<double>(mu) - static_cast<double>(Mx))));
    }
    rs = warp_sum(rs);
  }
  if (!(fl & GS_FLAG_ERRORS)) {
    const unsigned long long top = __shfl_sync(kFullMask, best[0], 0);
    const double xtop = static_cast<double>(pack_value(top));
    if (greedy) {
      // argmax over the whole vocabulary: all -inf -> id 0 (sampling.ts:92-96)
      tok = (top == 0ull || !(xtop > -INFINITY)) ? 0u : pack_id(top);
      if (lane == 0) {
        w.cid[0] = tok;
        w.cp[0] = 1.0;
      }
      n_final = 1;
    } else {
      const double M = __ddiv_rn(xtop, T);
      if (!(M > -INFINITY)) {
        fl |= GS_FLAG_ERR_NONFINITE;  // every logit -inf: outside the domain
      } else {
        double part = 0.0;
        for (int u = lane; u < S; u += 32) {
          const StepRec* st = reinterpret_cast<const StepRec*>(rec_row + static_cast<int64_t>(u) * A.rec_bytes);
          const float mu = __ldcg(&st->m);
          if (mu > -INFINITY) part = __dadd_rn(part, __dmul_rn(__ldcg(&st->s), exp(__dsub_rn(__ddiv_rn(static_cast<double>(mu), T), M))));
        }
        const double total = warp_sum(part);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int i = lane * 4 + q;
          if (i < nC) {
            const double key = __ddiv_rn(static_cast<double>(pack_value(best[q])), T);
            w.cid[i] = pack_id(best[q]);
            w.cp[i] = __ddiv_rn(exp(__dsub_rn(key, M)), total);
          }
        }
        double r;
        if (A.uniforms) {
          r = A.uniforms[row];
        } else {
          double st = A.rng_state[row];
          r = seeded_next(&st);
          if (lane == 0) A.rng_state[row] = st;
        }
        __syncwarp();
        tok = warp_filter_and_draw(w, nC, pp->min_p, pp->typical_p, pp->top_p, r, &n_final, &fl, lane);
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
  if (b->mask_table || b->history) return false;
  if (b->dtype != GS_DTYPE_F32 && b->dtype != GS_DTYPE_BF16) return false;
  const int64_t esz = b->dtype == GS_DTYPE_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(b->logits) & 15) != 0 || (b->row_stride * esz) % 16 != 0) return false;
  const int64_t units = (b->vocab + kStepIds - 1) / kStepIds;
  if (units > kStepMaxUnits) return false;
  return units * pow2_at_least(kmax) <= kStepMaxPacks;
}

size_t step_ws_bytes(int rows, int64_t vocab, int kmax) {
  const int64_t units = (vocab + kStepIds - 1) / kStepIds;
  const size_t rec = sizeof(StepRec) + 8 * static_cast<size_t>(pow2_at_least(kmax));
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
  a.rec_bytes = static_cast<int32_t>(sizeof(StepRec) + 8 * static_cast<size_t>(a.k2));
  a.recs = ws;
  a.sort_scratch = reinterpret_cast<unsigned long long*>(ws + align_up(static_cast<size_t>(b->rows) * a.units * a.rec_bytes, 256));
  a.done = done;
  // shared memory: the merge tree's two list sets, or the last CTA's arrays
  const size_t tree = 2 * static_cast<size_t>(kStepWarps) * a.k2 * 8;
  const size_t last = static_cast<size_t>(kStepMaxUnits) * 8 + (kStepMaxUnits + 8) * 4 + static_cast<size_t>(kStepSortSmem) * 8;
  const size_t smem = tree > last ? tree : last;
  const int grid = b->rows * a.units;
  if (b->dtype == GS_DTYPE_F32) {
    cudaFuncSetAttribute(step_kernel<GS_DTYPE_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    step_kernel<GS_DTYPE_F32><<<grid, kStepThreads, smem, st>>>(a);
  } else {
    cudaFuncSetAttribute(step_kernel<GS_DTYPE_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    step_kernel<GS_DTYPE_BF16><<<grid, kStepThreads, smem, st>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace gs
