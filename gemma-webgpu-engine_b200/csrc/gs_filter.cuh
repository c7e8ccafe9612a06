// The candidate filters and the draw of sampleToken over a short, already ordered
// candidate list (at most kMaxCand entries), one CTA per row, in IEEE double.
//
// Reference (aribornstein/gemma-webgpu-engine, src/runtime/sampling.ts):
//   45-48  min-p: keep p >= p[0]·minP (a filter, order kept)
//   49-55  typical-p: entropy, stable sort by |−ln p − H|, cumulativeCut, stable re-sort by p
//   56     top-p: cumulativeCut(topP)
//   58-64  draw: cursor = r·Σp; first candidate where the running cursor reaches <= 0,
//          else the last one
//   82-90  cumulativeCut: smallest prefix whose running sum reaches the threshold, >= 1
// Running sums are block prefix sums instead of the reference's left-to-right loop; the
// two differ only in the last bits, so a decision whose margin is below 1e-6 (relative)
// is flagged (GS_FLAG_BOUNDARY_*) instead of being claimed exact.
#pragma once
#include "gs_block.cuh"
#include "../../include/gsampler.h"

namespace gs {

constexpr int kMaxCand = 1024;
constexpr double kBoundaryRel = 1e-6;

struct FilterWork {
  uint32_t* cid;            // [kMaxCand] candidate ids, draw order
  double* cp;               // [kMaxCand] probabilities
  double* cum;              // [kMaxCand] scratch
  unsigned long long* skey; // [kMaxCand] scratch
  uint32_t* sval;           // [kMaxCand] scratch
  int* pos;                 // [kMaxCand] scratch
  unsigned char* flg;       // [kMaxCand] scratch
  double* red_d;            // [32]
  int* red_i;               // [32]
  int* s_int;               // [4] shared scalars
  unsigned* s_flags;        // shared flags word (atomicOr target)
};

// Keeps entries with keep[i] != 0, preserving order.  Returns the new length.
__device__ inline int compact_keep(FilterWork& w, int n) {
  const int total = block_exclusive_count(w.flg, w.pos, n, w.red_i);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    if (w.flg[i]) {
      w.sval[w.pos[i]] = w.cid[i];
      w.cum[w.pos[i]] = w.cp[i];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    w.cid[i] = w.sval[i];
    w.cp[i] = w.cum[i];
  }
  __syncthreads();
  return total;
}

// cumulativeCut over w.cp[0, n): returns the kept length (>= 1).  Flags a boundary when
// the running sum at the cut (or just before it) is within 1e-6·threshold.
__device__ inline int cumulative_cut(FilterWork& w, int n, double threshold, unsigned boundary_flag) {
  block_inclusive_scan_d(w.cp, w.cum, n, w.red_d);
  int below = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) below += w.cum[i] < threshold ? 1 : 0;
  below = block_sum_i(below, w.red_i);
  const int keep = below + 1 < n ? below + 1 : n;
  if (threadIdx.x == 0) {
    const double tol = kBoundaryRel * threshold;
    double m = fabs(w.cum[keep - 1] - threshold);
    if (keep >= 2) m = fmin(m, fabs(w.cum[keep - 2] - threshold));
    if (m <= tol) atomicOr(w.s_flags, boundary_flag);
  }
  __syncthreads();
  return keep;
}

// Runs min-p, typical-p, top-p and the draw on the ordered candidates
// (w.cid, w.cp)[0, n).  `uniform` is the random() value.  Returns the token; the final
// candidate list is left in (w.cid, w.cp)[0, *n_final).
__device__ inline uint32_t filter_and_draw(FilterWork& w, int n, double min_p, double typical_p, double top_p,
                                           double uniform, int* n_final) {
  // ---- min-p (sampling.ts:45-48) ----
  if (min_p > 0) {
    const double thr = __dmul_rn(w.cp[0], min_p);
    const double tol = kBoundaryRel * thr;
    int near = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      w.flg[i] = w.cp[i] >= thr ? 1 : 0;
      if (fabs(w.cp[i] - thr) <= tol) near = 1;
    }
    if (__syncthreads_or(near) && threadIdx.x == 0) atomicOr(w.s_flags, GS_FLAG_BOUNDARY_MIN_P);
    n = compact_keep(w, n);
  }
  // ---- typical-p (sampling.ts:49-55) ----
  if (typical_p < 1) {
    double t = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) t = __dadd_rn(t, __dmul_rn(w.cp[i], log(w.cp[i])));
    const double entropy = -block_sum_d(t, w.red_d);
    const bool ordered = entropy == entropy;
    const int n2 = pow2_ceil(n);
    // surprise of original index i -> w.cum[i]; surprise order -> w.sval
    for (int i = threadIdx.x; i < n2; i += blockDim.x) {
      if (i < n) {
        const double s = ordered ? fabs(__dsub_rn(-log(w.cp[i]), entropy)) : 0.0;
        w.cum[i] = s;
        w.skey[i] = key64(s);
      } else {
        w.skey[i] = ~0ull;
      }
      w.sval[i] = static_cast<uint32_t>(i);
    }
    __syncthreads();
    // A zero probability makes the entropy NaN; the reference's comparator then returns
    // NaN for every pair, which Array.prototype.sort reads as "equal" (order kept).
    if (ordered) bitonic_sort_kv(w.skey, w.sval, n2);  // ties keep the current order
    // running sums in surprise order (in w.skey, reused as doubles)
    double* ps = reinterpret_cast<double*>(w.skey);
    for (int j = threadIdx.x; j < n; j += blockDim.x) ps[j] = w.cp[w.sval[j]];
    __syncthreads();
    block_inclusive_scan_d(ps, ps, n, w.red_d);
    int below = 0;
    for (int j = threadIdx.x; j < n; j += blockDim.x) below += ps[j] < typical_p ? 1 : 0;
    below = block_sum_i(below, w.red_i);
    const int keep = below + 1 < n ? below + 1 : n;
    if (threadIdx.x == 0) {
      double m = fabs(ps[keep - 1] - typical_p);
      if (keep >= 2) m = fmin(m, fabs(ps[keep - 2] - typical_p));
      bool flag = m <= kBoundaryRel * typical_p;
      if (keep < n && ordered) {
        const double s0 = w.cum[w.sval[keep - 1]], s1 = w.cum[w.sval[keep]];
        if (fabs(s1 - s0) <= kBoundaryRel * fmax(fabs(s0), fabs(s1))) flag = true;
      }
      if (flag) atomicOr(w.s_flags, GS_FLAG_BOUNDARY_TYPICAL);
    }
    __syncthreads();
    // stable re-sort of the kept ones by probability descending (ties: surprise order)
    const int k2 = pow2_ceil(keep);
    for (int j = threadIdx.x; j < k2; j += blockDim.x) {
      if (j < keep) {
        w.pos[j] = static_cast<int>(w.sval[j]);
        w.skey[j] = ~key64(w.cp[w.sval[j]]);
        w.sval[j] = static_cast<uint32_t>(j);
      } else {
        w.skey[j] = ~0ull;
        w.sval[j] = 0xffffffffu;
      }
    }
    __syncthreads();
    bitonic_sort_kv(w.skey, w.sval, k2);
    uint32_t* ids_tmp = reinterpret_cast<uint32_t*>(w.skey);
    for (int j = threadIdx.x; j < keep; j += blockDim.x) {
      const int src = w.pos[w.sval[j]];
      w.cum[j] = w.cp[src];
      ids_tmp[j] = w.cid[src];
    }
    __syncthreads();
    for (int j = threadIdx.x; j < keep; j += blockDim.x) {
      w.cp[j] = w.cum[j];
      w.cid[j] = ids_tmp[j];
    }
    __syncthreads();
    n = keep;
  }
  // ---- top-p (sampling.ts:56) ----
  if (top_p < 1) n = cumulative_cut(w, n, top_p, GS_FLAG_BOUNDARY_TOP_P);
  // ---- draw (sampling.ts:58-64) ----
  block_inclusive_scan_d(w.cp, w.cum, n, w.red_d);
  const double total = w.cum[n - 1];
  const double cursor = __dmul_rn(uniform, total);
  int below = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) below += w.cum[i] < cursor ? 1 : 0;
  below = block_sum_i(below, w.red_i);
  uint32_t tok;
  if (below < n) {
    tok = w.cid[below];
  } else {
    tok = w.cid[n - 1];
    if (threadIdx.x == 0) atomicOr(w.s_flags, GS_FLAG_FELL_THROUGH);
  }
  if (threadIdx.x == 0) {
    const double tol = kBoundaryRel * total;
    const int j = below < n ? below : n - 1;
    double m = fabs(w.cum[j] - cursor);
    if (j >= 1) m = fmin(m, fabs(w.cum[j - 1] - cursor));
    if (m <= tol) atomicOr(w.s_flags, GS_FLAG_BOUNDARY_DRAW);
  }
  __syncthreads();
  *n_final = n;
  return tok;
}

}  // namespace gs
