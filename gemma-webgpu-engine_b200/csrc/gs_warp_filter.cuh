// One-warp forms of the filters and the draw (src/runtime/sampling.ts:45-64, 82-90) over
// at most kWFilterMax ordered candidates, shared by the warp-per-row merge and the
// single-launch decode step.  Same IEEE double operations and prefix-sum order as the
// block versions in gs_filter.cuh.
#pragma once
#include "gs_device.cuh"
#include "gs_block.cuh"
#include "gs_filter.cuh"
#include "../../include/gsampler.h"

namespace gs {

constexpr int kWFilterMax = 128;  // candidates the warp filters handle

// Ascending bitonic sort of (key, payload) pairs by (key, payload), one warp.
__device__ inline void warp_sort_kv(unsigned long long* key, uint32_t* val, int n2, int lane) {
  for (int k = 2; k <= n2; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = lane; i < n2; i += 32) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long ka = key[i], kb = key[ixj];
          const uint32_t va = val[i], vb = val[ixj];
          const bool a_gt_b = ka > kb || (ka == kb && va > vb);
          const bool up = (i & k) == 0;
          if (up ? a_gt_b : !a_gt_b) {
            key[i] = kb;
            key[ixj] = ka;
            val[i] = vb;
            val[ixj] = va;
          }
        }
      }
      __syncwarp();
    }
}

// Inclusive prefix sums out[i] = in[0] + ... + in[i], i < n <= 128: lane l sums items
// 4l..4l+3, then a shuffle scan over the lanes (block_inclusive_scan_d's order for n <= 128).
__device__ inline void warp_scan4_d(const double* in, double* out, int n, int lane) {
  double v[4];
  double run = 0.0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = 4 * lane + j;
    run = __dadd_rn(run, i < n ? in[i] : 0.0);
    v[j] = run;
  }
  double incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double u = __shfl_up_sync(kFullMask, incl, o);
    if (lane >= o) incl = __dadd_rn(incl, u);
  }
  double excl = __shfl_up_sync(kFullMask, incl, 1);
  if (lane == 0) excl = 0.0;
  const double base = __dadd_rn(0.0, excl);
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = 4 * lane + j;
    if (i < n) out[i] = __dadd_rn(base, v[j]);
  }
  __syncwarp();
}

__device__ __forceinline__ int warp_count_below(const double* a, int n, double thr, int lane) {
  int c = 0;
  for (int i = lane; i < n; i += 32) c += a[i] < thr ? 1 : 0;
  return static_cast<int>(__reduce_add_sync(kFullMask, static_cast<unsigned>(c)));
}

struct WWork {
  uint32_t* cid;
  double* cp;
  double* cum;
  unsigned long long* skey;
  uint32_t* sval;
  int* pos;
  unsigned char* flg;
};

// Order-preserving compaction of (cid, cp)[0, n) to the entries with flg set.
__device__ inline int warp_compact_keep(WWork& w, int n, int lane) {
  int base = 0;
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int i = i0 + lane;
    const bool keep = i < n && w.flg[i];
    uint32_t id = 0;
    double p = 0.0;
    if (keep) {
      id = w.cid[i];
      p = w.cp[i];
    }
    const unsigned b = __ballot_sync(kFullMask, keep);
    __syncwarp();
    if (keep) {
      const int at = base + __popc(b & ((1u << lane) - 1u));
      w.cid[at] = id;
      w.cp[at] = p;
    }
    base += __popc(b);
    __syncwarp();
  }
  return base;
}

// cumulativeCut (src/runtime/sampling.ts:82-90) over w.cp[0, n); flags a boundary when the
// running sum at the cut or just before it is within 1e-6·threshold.
__device__ inline int warp_cumulative_cut(WWork& w, int n, double threshold, unsigned flag, unsigned* fl, int lane) {
  warp_scan4_d(w.cp, w.cum, n, lane);
  const int below = warp_count_below(w.cum, n, threshold, lane);
  const int keep = below + 1 < n ? below + 1 : n;
  double m = fabs(w.cum[keep - 1] - threshold);
  if (keep >= 2) m = fmin(m, fabs(w.cum[keep - 2] - threshold));
  if (m <= kBoundaryRel * threshold) *fl |= flag;
  return keep;
}

// min-p, typical-p, top-p and the draw (src/runtime/sampling.ts:45-64) over the ordered
// candidates (w.cid, w.cp)[0, n); the final list is left in (w.cid, w.cp)[0, *n_final).
__device__ inline uint32_t warp_filter_and_draw(WWork& w, int n, double min_p, double typical_p, double top_p,
                                         double uniform, int* n_final, unsigned* fl, int lane) {
  if (min_p > 0) {
    const double thr = __dmul_rn(w.cp[0], min_p);
    const double tol = kBoundaryRel * thr;
    bool near = false;
    for (int i = lane; i < n; i += 32) {
      w.flg[i] = w.cp[i] >= thr ? 1 : 0;
      if (fabs(w.cp[i] - thr) <= tol) near = true;
    }
    if (__any_sync(kFullMask, near)) *fl |= GS_FLAG_BOUNDARY_MIN_P;
    __syncwarp();
    n = warp_compact_keep(w, n, lane);
  }
  if (typical_p < 1) {
    double t = 0.0;
    for (int i = lane; i < n; i += 32) t = __dadd_rn(t, __dmul_rn(w.cp[i], log(w.cp[i])));
    const double entropy = -warp_sum(t);
    const bool ordered = entropy == entropy;
    const int n2 = pow2_ceil(n);
    for (int i = lane; i < n2; i += 32) {
      if (i < n) {
        const double s = ordered ? fabs(__dsub_rn(-log(w.cp[i]), entropy)) : 0.0;
        w.cum[i] = s;
        w.skey[i] = key64(s);
      } else {
        w.skey[i] = ~0ull;
      }
      w.sval[i] = static_cast<uint32_t>(i);
    }
    __syncwarp();
    // a zero probability makes the entropy NaN: the reference's comparator then calls
    // every pair equal and the order is kept
    if (ordered) warp_sort_kv(w.skey, w.sval, n2, lane);
    double* ps = reinterpret_cast<double*>(w.skey);
    double tmp[kWFilterMax / 32];
#pragma unroll
    for (int q = 0; q < kWFilterMax / 32; ++q) {
      const int j = q * 32 + lane;
      tmp[q] = j < n ? w.cp[w.sval[j]] : 0.0;
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < kWFilterMax / 32; ++q) {
      const int j = q * 32 + lane;
      if (j < n) ps[j] = tmp[q];
    }
    __syncwarp();
    warp_scan4_d(ps, ps, n, lane);
    const int below = warp_count_below(ps, n, typical_p, lane);
    const int keep = below + 1 < n ? below + 1 : n;
    double m = fabs(ps[keep - 1] - typical_p);
    if (keep >= 2) m = fmin(m, fabs(ps[keep - 2] - typical_p));
    bool flag = m <= kBoundaryRel * typical_p;
    if (keep < n && ordered) {
      const double s0 = w.cum[w.sval[keep - 1]], s1 = w.cum[w.sval[keep]];
      if (fabs(s1 - s0) <= kBoundaryRel * fmax(fabs(s0), fabs(s1))) flag = true;
    }
    if (flag) *fl |= GS_FLAG_BOUNDARY_TYPICAL;
    __syncwarp();
    // stable re-sort of the kept ones by probability descending (ties: surprise order)
    const int k2 = pow2_ceil(keep);
    for (int j = lane; j < k2; j += 32) {
      if (j < keep) {
        w.pos[j] = static_cast<int>(w.sval[j]);
        w.skey[j] = ~key64(w.cp[w.sval[j]]);
        w.sval[j] = static_cast<uint32_t>(j);
      } else {
        w.skey[j] = ~0ull;
        w.sval[j] = 0xffffffffu;
      }
    }
    __syncwarp();
    warp_sort_kv(w.skey, w.sval, k2, lane);
    double pt[kWFilterMax / 32];
    uint32_t it[kWFilterMax / 32];
#pragma unroll
    for (int q = 0; q < kWFilterMax / 32; ++q) {
      const int j = q * 32 + lane;
      if (j < keep) {
        const int src = w.pos[w.sval[j]];
        pt[q] = w.cp[src];
        it[q] = w.cid[src];
      }
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < kWFilterMax / 32; ++q) {
      const int j = q * 32 + lane;
      if (j < keep) {
        w.cp[j] = pt[q];
        w.cid[j] = it[q];
      }
    }
    __syncwarp();
    n = keep;
  }
  if (top_p < 1) n = warp_cumulative_cut(w, n, top_p, GS_FLAG_BOUNDARY_TOP_P, fl, lane);
  warp_scan4_d(w.cp, w.cum, n, lane);
  const double total = w.cum[n - 1];
  const double cursor = __dmul_rn(uniform, total);
  const int below = warp_count_below(w.cum, n, cursor, lane);
  uint32_t tok;
  if (below < n) {
    tok = w.cid[below];
  } else {
    tok = w.cid[n - 1];
    *fl |= GS_FLAG_FELL_THROUGH;
  }
  const int j = below < n ? below : n - 1;
  double m = fabs(w.cum[j] - cursor);
  if (j >= 1) m = fmin(m, fabs(w.cum[j - 1] - cursor));
  if (m <= kBoundaryRel * total) *fl |= GS_FLAG_BOUNDARY_DRAW;
  *n_final = n;
  return tok;
}

}  // namespace gs
