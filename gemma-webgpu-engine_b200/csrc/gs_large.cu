// Kernel 3: the histogram path, for rows whose candidate list is not bounded by a small
// topK (topK == 0 or topK > GS_MAX_TOP_K with V > GS_MAX_TOP_K).  One CTA per row.
//
// The reference keeps the whole sorted vocabulary as candidates (src/runtime/sampling.ts:44)
// and then cuts prefixes of it: min-p (:45-48, a prefix because p falls along the order),
// top-p (:56, cumulativeCut :82-90) and the draw (:58-64).  Every one of these is a
// position in the sorted order where a running count or a running probability crosses a
// value.  Instead of sorting 262144 entries, this kernel:
//   1. builds a histogram of count and probability mass over 2048 bins of logit distance
//      below the row maximum (monotone in the sort key, so bins hold contiguous ranges of
//      the reference's order);
//   2. finds the bin where the running value crosses the target;
//   3. gathers only that bin's elements, sorts them exactly (logit/T desc, id asc) and
//      resolves the crossing with exact double probabilities.
// Masses are accumulated in 2^-44 fixed point so that the sums are order-independent and
// the result is bit-reproducible.  Decisions within 1e-6 of a boundary are flagged.
#include "gs_device.cuh"
#include "gs_block.cuh"
#include "gs_internal.cuh"
#include "../../include/gsampler.h"

namespace gs {

namespace {

constexpr int kNB = 2048;             // histogram bins
constexpr double kRangeKeys = 48.0;   // bins span 48 units of logit/T below the maximum
constexpr double kFix = 17592186044416.0;  // 2^44
constexpr double kBoundary = 1e-6;

struct LShared {
  unsigned flags;
  int n_allowed;
  int n_pen;
  int g_n;
  int g_lo;
  int g_hi;
  int n_neginf;
  float Mx;
  float raw_m;
  double raw_s;
  double M;
  double total;
  double f0;
  double uniform;
  int sres[8];
  double sresd[4];
  double red_d[32];
  int red_i[32];
  unsigned long long red_u[32];
};

struct LArgs {
  int nwords;
  int pen_cap;
  int gcap;
};

__device__ __forceinline__ int bin_of(float x, float Mx, float scale) {
  const float d = Mx - x;
  if (!(d > 0.0f)) return 0;
  const float b = d * scale;
  return b >= static_cast<float>(kNB - 1) ? kNB - 1 : static_cast<int>(b);
}

}  // namespace

size_t large_smem_bytes(int64_t vocab, int hist_cap) {
  const size_t nwords = (static_cast<size_t>((vocab + 31) / 32) + 3) & ~static_cast<size_t>(3);
  const size_t pen = static_cast<size_t>(hist_cap) * sizeof(Ent);
  const size_t bins = (kNB + 1) * 4 + (kNB + 1) * 8;
  const size_t gather = static_cast<size_t>(kLargeGatherCap) * (sizeof(Ent) + 8);
  return nwords * 4 + ((bins + 15) & ~static_cast<size_t>(15)) + pen + gather + 64;
}

template <int DT>
__global__ void __launch_bounds__(kLargeThreads) large_kernel(const __grid_constant__ FinalizeArgs A) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ LShared Z;
  const int row = blockIdx.x, tid = threadIdx.x, bs = blockDim.x;
  const RowPlan* pp = A.plans ? A.plans + row : &A.plan0;
  if (pp->mode != kModeLarge) return;
  const double T = pp->temperature;
  const int S = A.splits;
  const int64_t V = A.vocab;
  const int nwords = static_cast<int>((V + 31) / 32);
  const int nwords_pad = (nwords + 3) & ~3;
  const int GCAP = kLargeGatherCap;

  // ---- shared memory carve-up ----
  unsigned char* p = dsm;
  uint32_t* live = reinterpret_cast<uint32_t*>(p);
  p += static_cast<size_t>(nwords_pad) * 4;
  unsigned long long* bmass = reinterpret_cast<unsigned long long*>(p);  // [kNB + 1]
  p += (kNB + 1) * 8;
  uint32_t* bcnt = reinterpret_cast<uint32_t*>(p);  // [kNB + 1]
  p += (kNB + 1) * 4;
  p = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 15) & ~static_cast<uintptr_t>(15));
  Ent* pen = reinterpret_cast<Ent*>(p);
  p += static_cast<size_t>(A.hist_cap) * sizeof(Ent);
  Ent* G = reinterpret_cast<Ent*>(p);
  p += static_cast<size_t>(GCAP) * sizeof(Ent);
  double* gp = reinterpret_cast<double*>(p);  // exact probabilities of G, then running sums

  const int32_t state = A.mask_state ? A.mask_state[row] : -1;
  const bool has_mask = A.mask_table != nullptr && state >= 0 && state < A.mask_states;
  const uint32_t* mrow = has_mask ? A.mask_table + static_cast<int64_t>(state) * A.mask_words : nullptr;
  const unsigned char* rowbase =
      static_cast<const unsigned char*>(A.logits) + static_cast<int64_t>(row) * A.row_stride * (DT == GS_DTYPE_F32 ? 4 : 2);
  const float cap = A.softcap, inv_cap = A.inv_softcap;

  // ---- 0. unit partials ----
  if (tid == 0) {
    unsigned fl = GS_FLAG_LARGE_PATH;
    int na = 0;
    float mx = -INFINITY, rm = -INFINITY;
    for (int u = 0; u < S; ++u) {
      const UnitStat& st = A.stats[static_cast<int64_t>(row) * S + u];
      fl |= st.flags;
      na += st.n_allowed;
      mx = fmaxf(mx, st.m);
      rm = fmaxf(rm, st.raw_m);
    }
    double rs = 0.0;
    if (A.want_raw)
      for (int u = 0; u < S; ++u) {
        const UnitStat& st = A.stats[static_cast<int64_t>(row) * S + u];
        if (st.raw_m > -INFINITY) rs = __dadd_rn(rs, __dmul_rn(st.raw_s, exp(static_cast<double>(st.raw_m) - static_cast<double>(rm))));
      }
    if (has_mask && na == 0) fl |= GS_FLAG_ERR_DEADEND;
    if (pp->typical_p < 1) fl |= GS_FLAG_ERR_UNSUPPORTED;  // typical-p over > 1024 candidates
    Z.flags = fl;
    Z.n_allowed = na;
    Z.Mx = mx;
    Z.raw_m = rm;
    Z.raw_s = rs;
    Z.n_pen = 0;
    Z.n_neginf = 0;
  }
  __syncthreads();

  // ---- 1. live bitmap: allowed and not penalised ----
  for (int w = tid; w < nwords; w += bs) {
    uint32_t m = has_mask ? __ldg(mrow + w) : 0xffffffffu;
    if (w == nwords - 1 && (V & 31)) m &= (1u << (V & 31)) - 1u;
    live[w] = m;
  }
  __syncthreads();
  int64_t hl = A.history_len ? A.history_len[row] : 0;
  if (hl > A.history_stride) hl = A.history_stride;
  if (hl < 0) hl = 0;
  const int32_t* hrow = A.history + static_cast<int64_t>(row) * A.history_stride;
  for (int64_t j = tid; j < hl; j += bs) {
    const int32_t h = hrow[j];
    if (h >= 0 && h < V) atomicAnd(&live[h >> 5], ~(1u << (h & 31)));
  }
  // ---- 2. penalised ids: distinct, with counts, scored exactly ----
  if (hl > 0) {
    uint32_t* hs = reinterpret_cast<uint32_t*>(G);  // the gather area is free until step 4
    const int h2 = pow2_ceil(static_cast<int>(hl));
    for (int i = tid; i < h2; i += bs) hs[i] = i < hl ? static_cast<uint32_t>(hrow[i]) : 0xffffffffu;
    __syncthreads();
    bitonic_sort_u32(hs, h2);
    const double rp = pp->repetition_penalty, pres = pp->presence_penalty, freq = pp->frequency_penalty;
    for (int i = tid; i < hl; i += bs) {
      const uint32_t v = hs[i];
      if (v >= static_cast<uint64_t>(V)) continue;
      if (i > 0 && hs[i - 1] == v) continue;
      int cnt = 1;
      while (i + cnt < hl && hs[i + cnt] == v) ++cnt;
      if (has_mask && !((__ldg(mrow + (v >> 5)) >> (v & 31)) & 1u)) continue;
      float x = load_logit(rowbase, DT, v);
      if (cap != 0.0f) x = softcap(x, cap, inv_cap);
      if (!(x < INFINITY)) atomicOr(&Z.flags, GS_FLAG_ERR_NONFINITE);
      double xp = static_cast<double>(x);
      xp = xp < 0 ? __dmul_rn(xp, rp) : __ddiv_rn(xp, rp);
      xp = __dsub_rn(xp, __dadd_rn(pres, __dmul_rn(static_cast<double>(cnt), freq)));
      const int slot = atomicAdd(&Z.n_pen, 1);
      // kind holds the float32 rounding of the penalised logit, used only for binning
      pen[slot] = Ent{__ddiv_rn(xp, T), v, __float_as_uint(static_cast<float>(xp))};
    }
  }
  __syncthreads();

  const int n_pen = Z.n_pen;
  // ---- 3. maximum key and full-vocabulary normaliser ----
  {
    double pm = -INFINITY;
    for (int i = tid; i < n_pen; i += bs) pm = fmax(pm, pen[i].key);
    for (int o = 16; o > 0; o >>= 1) pm = fmax(pm, __shfl_xor_sync(kFullMask, pm, o));
    if ((tid & 31) == 0) Z.red_d[tid >> 5] = pm;
    __syncthreads();
    if (tid == 0) {
      double m = Z.Mx > -INFINITY ? __ddiv_rn(static_cast<double>(Z.Mx), T) : -INFINITY;
      for (int w = 0; w < (bs >> 5); ++w) m = fmax(m, Z.red_d[w]);
      Z.M = m;
      if (m == -INFINITY) Z.flags |= GS_FLAG_ERR_NONFINITE;
      Z.f0 = Z.Mx > -INFINITY ? exp(__dsub_rn(__ddiv_rn(static_cast<double>(Z.Mx), T), m)) : 0.0;
    }
    __syncthreads();
  }
  const double M = Z.M;
  if (!(Z.flags & GS_FLAG_ERRORS)) {
    double part = 0.0;
    for (int u = tid; u < S; u += bs) {
      const UnitStat& st = A.stats[static_cast<int64_t>(row) * S + u];
      if (st.m > -INFINITY) part = __dadd_rn(part, __dmul_rn(st.s, exp(__dsub_rn(__ddiv_rn(static_cast<double>(st.m), T), M))));
    }
    for (int i = tid; i < n_pen; i += bs) part = __dadd_rn(part, exp(__dsub_rn(pen[i].key, M)));
    const double total = block_sum_d(part, Z.red_d);
    if (tid == 0) Z.total = total;
    __syncthreads();
  }

  const float Mx = Z.Mx;
  const float scale = static_cast<float>(static_cast<double>(kNB) / (kRangeKeys * T));
  const float f0 = static_cast<float>(Z.f0);
  const float a2_hi = pp->a2_hi, a2_lo = pp->a2_lo;
  const double total = Z.total;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(rowbase) & 15) == 0 && DT == GS_DTYPE_F32;

  // Visits every live (allowed, unpenalised) id of the row with its soft-capped logit.
  auto for_each_live = [&](auto&& fn) {
    if (vec_ok) {
      const float4* r4 = reinterpret_cast<const float4*>(rowbase);
      const int64_t nv = V / 4;
      for (int64_t vi = tid; vi < nv; vi += bs) {
        const int64_t id0 = vi * 4;
        const uint32_t bits = (live[id0 >> 5] >> (id0 & 31)) & 15u;
        if (!bits) continue;
        const float4 v = __ldg(r4 + vi);
        const float xs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if ((bits >> i) & 1u) fn(cap != 0.0f ? softcap(xs[i], cap, inv_cap) : xs[i], static_cast<uint32_t>(id0 + i));
      }
      for (int64_t id = nv * 4 + tid; id < V; id += bs)
        if ((live[id >> 5] >> (id & 31)) & 1u) {
          float x = load_logit(rowbase, DT, id);
          fn(cap != 0.0f ? softcap(x, cap, inv_cap) : x, static_cast<uint32_t>(id));
        }
    } else {
      for (int64_t id = tid; id < V; id += bs)
        if ((live[id >> 5] >> (id & 31)) & 1u) {
          float x = load_logit(rowbase, DT, id);
          fn(cap != 0.0f ? softcap(x, cap, inv_cap) : x, static_cast<uint32_t>(id));
        }
    }
  };

  // ---- 4. histogram of count and mass ----
  if (!(Z.flags & GS_FLAG_ERRORS)) {
    for (int b = tid; b <= kNB; b += bs) {
      bcnt[b] = 0;
      bmass[b] = 0;
    }
    __syncthreads();
    int neginf = 0;
    for_each_live([&](float x, uint32_t) {
      if (x == -INFINITY) {
        ++neginf;
        return;
      }
      const int b = bin_of(x, Mx, scale);
      const float d = x - Mx;
      const float e = ex2_approx(fmaf(d, a2_lo, d * a2_hi)) * f0;
      atomicAdd(&bcnt[b], 1u);
      atomicAdd(&bmass[b], static_cast<unsigned long long>(__fmul_rn(e, 17592186044416.0f) + 0.5f));
    });
    for (int i = tid; i < n_pen; i += bs) {
      if (pen[i].key == -INFINITY) {
        ++neginf;
        continue;
      }
      const int b = bin_of(__uint_as_float(pen[i].kind), Mx, scale);
      const double e = exp(__dsub_rn(pen[i].key, M));
      atomicAdd(&bcnt[b], 1u);
      atomicAdd(&bmass[b], static_cast<unsigned long long>(e * kFix + 0.5));
    }
    neginf = block_sum_i(neginf, Z.red_i);
    // exclusive prefix over the bins (2 per thread; kNB == 2 * 1024)
    {
      const int b0 = 2 * tid;
      const uint32_t c0 = bcnt[b0], c1 = bcnt[b0 + 1];
      const unsigned long long m0 = bmass[b0], m1 = bmass[b0 + 1];
      uint32_t ci = c0 + c1;
      unsigned long long mi = m0 + m1;
      const int lane = tid & 31, warp = tid >> 5;
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t uc = __shfl_up_sync(kFullMask, ci, o);
        const unsigned long long um = __shfl_up_sync(kFullMask, mi, o);
        if (lane >= o) {
          ci += uc;
          mi += um;
        }
      }
      __syncthreads();
      if (lane == 31) {
        Z.red_i[warp] = static_cast<int>(ci);
        Z.red_u[warp] = mi;
      }
      __syncthreads();
      uint32_t cb = 0;
      unsigned long long mb = 0;
      for (int w = 0; w < warp; ++w) {
        cb += static_cast<uint32_t>(Z.red_i[w]);
        mb += Z.red_u[w];
      }
      const uint32_t ce = cb + ci - (c0 + c1);
      const unsigned long long me = mb + mi - (m0 + m1);
      __syncthreads();
      bcnt[b0] = ce;
      bcnt[b0 + 1] = ce + c0;
      bmass[b0] = me;
      bmass[b0 + 1] = me + m0;
      if (tid == bs - 1) {
        bcnt[kNB] = ce + c0 + c1;
        bmass[kNB] = me + m0 + m1;
      }
      __syncthreads();
    }
    if (tid == 0) Z.n_neginf = neginf;
    __syncthreads();
  }

  const int n_fin = static_cast<int>(bcnt[kNB]);
  const double inv_fix_total = 1.0 / (kFix * total);
  auto massP = [&](int b) { return static_cast<double>(bmass[b]) * inv_fix_total; };  // p-units before bin b

  // Gathers bins [lo, hi] into G (exact keys), sorts them in the reference order and sets
  // gp[i] = p_i.  Leaves Z.g_n = count (or flags unsupported when it exceeds GCAP).
  auto gather = [&](int lo, int hi) {
    if (Z.g_lo == lo && Z.g_hi == hi) return;
    __syncthreads();
    if (tid == 0) Z.g_n = 0;
    __syncthreads();
    for_each_live([&](float x, uint32_t id) {
      if (x == -INFINITY) return;
      const int b = bin_of(x, Mx, scale);
      if (b < lo || b > hi) return;
      const int slot = atomicAdd(&Z.g_n, 1);
      if (slot < GCAP) G[slot] = Ent{__ddiv_rn(static_cast<double>(x), T), id, 0u};
    });
    for (int i = tid; i < n_pen; i += bs) {
      if (pen[i].key == -INFINITY) continue;
      const int b = bin_of(__uint_as_float(pen[i].kind), Mx, scale);
      if (b < lo || b > hi) continue;
      const int slot = atomicAdd(&Z.g_n, 1);
      if (slot < GCAP) G[slot] = Ent{pen[i].key, pen[i].id, 1u};
    }
    __syncthreads();
    int n = Z.g_n;
    if (n > GCAP) {
      if (tid == 0) Z.flags |= GS_FLAG_ERR_UNSUPPORTED;  // more than GCAP ids in one bin
      n = GCAP;
    }
    const int n2 = pow2_ceil(n > 0 ? n : 1);
    for (int i = n + tid; i < n2; i += bs) G[i] = Ent{-INFINITY, 0xffffffffu, 0xffffffffu};
    __syncthreads();
    bitonic_sort_ent(G, n2);
    for (int i = tid; i < n; i += bs) gp[i] = __ddiv_rn(exp(__dsub_rn(G[i].key, M)), total);
    __syncthreads();
    if (tid == 0) {
      Z.g_lo = lo;
      Z.g_hi = hi;
      Z.g_n = n;
    }
    __syncthreads();
  };
  if (tid == 0) {
    Z.g_lo = -1;
    Z.g_hi = -1;
  }
  __syncthreads();

  // First rank j < limit with (running probability through j) >= target; -1 if none.
  // Writes the running sums at j and j-1 to Z.sresd[0..1].
  auto locate_mass = [&](double target, int limit) -> int {
    // first bin whose end reaches the target
    int cand = kNB;
    for (int b = tid; b < kNB; b += bs)
      if (massP(b + 1) >= target && massP(b) < target) cand = min(cand, b);
    for (int o = 16; o > 0; o >>= 1) cand = min(cand, __shfl_xor_sync(kFullMask, cand, o));
    __syncthreads();
    if ((tid & 31) == 0) Z.red_i[tid >> 5] = cand;
    __syncthreads();
    int b = kNB;
    for (int w = 0; w < (bs >> 5); ++w) b = min(b, Z.red_i[w]);
    __syncthreads();
    if (massP(0) >= target) b = 0;
    // The exact running sum inside the bin may fall just short of the binned estimate;
    // then the crossing is in one of the following bins.  Such a target is within ~1e-7
    // of a bin edge; after a few bins the search stops and flags a draw boundary.
    int tries = 0;
    for (; b < kNB; ++b) {
      if (static_cast<int>(bcnt[b]) >= limit) return -1;
      if (bcnt[b + 1] == bcnt[b]) continue;
      if (++tries > 4) {
        if (tid == 0) Z.flags |= GS_FLAG_BOUNDARY_DRAW;
        return -1;
      }
      gather(b, b);
      const int n = Z.g_n;
      if (tid == 0) {
        double c = massP(b);
        int found = -1;
        double prev = c;
        for (int i = 0; i < n && static_cast<int>(bcnt[b]) + i < limit; ++i) {
          prev = c;
          c = __dadd_rn(c, gp[i]);
          if (c >= target) {
            found = i;
            break;
          }
        }
        Z.sres[0] = found;
        Z.sresd[0] = c;
        Z.sresd[1] = prev;
      }
      __syncthreads();
      const int f = Z.sres[0];
      if (f >= 0) return static_cast<int>(bcnt[b]) + f;
      __syncthreads();
    }
    return -1;
  };

  // Id and running sum (through it) of rank r (0 <= r < n_fin).
  auto rank_info = [&](int r, uint32_t* id, double* cum_through) {
    int cand = kNB;
    for (int b = tid; b < kNB; b += bs)
      if (static_cast<int>(bcnt[b]) <= r && r < static_cast<int>(bcnt[b + 1])) cand = b;
    for (int o = 16; o > 0; o >>= 1) cand = min(cand, __shfl_xor_sync(kFullMask, cand, o));
    __syncthreads();
    if ((tid & 31) == 0) Z.red_i[tid >> 5] = cand;
    __syncthreads();
    int b = kNB;
    for (int w = 0; w < (bs >> 5); ++w) b = min(b, Z.red_i[w]);
    __syncthreads();
    gather(b, b);
    if (tid == 0) {
      const int i = r - static_cast<int>(bcnt[b]);
      double c = massP(b);
      for (int j = 0; j <= i && j < Z.g_n; ++j) c = __dadd_rn(c, gp[j]);
      Z.sres[1] = static_cast<int>(G[i < Z.g_n ? i : Z.g_n - 1].id);
      Z.sresd[2] = c;
    }
    __syncthreads();
    *id = static_cast<uint32_t>(Z.sres[1]);
    *cum_through = Z.sresd[2];
  };

  uint32_t tok = 0xffffffffu;
  int L = 0;
  if (!(Z.flags & GS_FLAG_ERRORS)) {
    const int K = pp->top_k;
    const int64_t klim64 = (K > 0 && K < V) ? K : V;
    int L1 = static_cast<int>(klim64);
    // ---- min-p (sampling.ts:45-48): p_i >= p_0·minP, with p_0 = 1/total ----
    if (pp->min_p > 0) {
      const double theta = __dmul_rn(__ddiv_rn(1.0, total), pp->min_p);
      const float xth = static_cast<float>(T * (M + log(pp->min_p)));
      const int bt = bin_of(xth, Mx, scale);
      const int lo = bt > 0 ? bt - 1 : 0, hi = bt < kNB - 1 ? bt + 1 : kNB - 1;
      gather(lo, hi);
      int kept = 0, near = 0;
      for (int i = tid; i < Z.g_n; i += bs) {
        kept += gp[i] >= theta ? 1 : 0;
        if (fabs(gp[i] - theta) <= kBoundary * theta) near = 1;
      }
      kept = block_sum_i(kept, Z.red_i);
      if (__syncthreads_or(near) && tid == 0) Z.flags |= GS_FLAG_BOUNDARY_MIN_P;
      const int Lm = static_cast<int>(bcnt[lo]) + kept;
      L1 = L1 < Lm ? L1 : Lm;
    }
    // ---- top-p (sampling.ts:56) ----
    L = L1;
    if (pp->top_p < 1) {
      const int j = locate_mass(pp->top_p, L1);
      if (j >= 0) {
        L = j + 1;
        if (tid == 0) {
          const double m = fmin(fabs(Z.sresd[0] - pp->top_p), j > 0 ? fabs(Z.sresd[1] - pp->top_p) : INFINITY);
          if (m <= kBoundary * pp->top_p) Z.flags |= GS_FLAG_BOUNDARY_TOP_P;
        }
      }
    }
    __syncthreads();
    // ---- candidate total C(L) ----
    double CT;
    uint32_t last_id = 0;
    if (L <= n_fin) {
      rank_info(L - 1, &last_id, &CT);
    } else {
      CT = massP(kNB);
      last_id = 0xffffffffu;  // in the -inf group: resolved below if the draw falls through
    }
    // ---- draw (sampling.ts:58-64) ----
    if (tid == 0) {
      double r;
      if (A.uniforms) {
        r = A.uniforms[row];
      } else {
        double st = A.rng_state[row];
        r = seeded_next(&st);
        A.rng_state[row] = st;
      }
      Z.uniform = r;
    }
    __syncthreads();
    const double cursor = __dmul_rn(Z.uniform, CT);
    const int lim = L < n_fin ? L : n_fin;
    const int j = locate_mass(cursor, lim);
    if (j >= 0) {
      tok = G[j - static_cast<int>(bcnt[Z.g_lo])].id;
      if (tid == 0) {
        const double m = fmin(fabs(Z.sresd[0] - cursor), j > 0 ? fabs(Z.sresd[1] - cursor) : INFINITY);
        if (m <= kBoundary * CT) Z.flags |= GS_FLAG_BOUNDARY_DRAW;
      }
    } else {
      if (tid == 0) Z.flags |= GS_FLAG_FELL_THROUGH;
      if (last_id != 0xffffffffu) {
        tok = last_id;
      } else {
        // the (L - 1 - n_fin)-th id, in ascending order, of the ids whose key is -inf
        const int want = L - 1 - n_fin;
        if (tid == 0) Z.sres[2] = 0;
        __syncthreads();
        int base = 0;
        for (int64_t id0 = 0; id0 < V; id0 += bs) {
          const int64_t id = id0 + tid;
          bool neg = false;
          if (id < V) {
            const bool allowed = !has_mask || ((__ldg(mrow + (id >> 5)) >> (id & 31)) & 1u);
            if (!allowed) {
              neg = true;
            } else {
              float x = load_logit(rowbase, DT, id);
              if (cap != 0.0f) x = softcap(x, cap, inv_cap);
              neg = x == -INFINITY;
            }
          }
          const unsigned bal = __ballot_sync(kFullMask, neg);
          if ((tid & 31) == 0) Z.red_i[tid >> 5] = __popc(bal);
          __syncthreads();
          int before = base;
          for (int w = 0; w < (tid >> 5); ++w) before += Z.red_i[w];
          before += __popc(bal & ((1u << (tid & 31)) - 1u));
          if (neg && before == want) Z.sres[2] = static_cast<int>(id);
          int sum = 0;
          for (int w = 0; w < (bs >> 5); ++w) sum += Z.red_i[w];
          __syncthreads();
          base += sum;
          if (base > want) break;
        }
        __syncthreads();
        tok = static_cast<uint32_t>(Z.sres[2]);
      }
    }
    __syncthreads();
  }

  // ---- outputs ----
  const unsigned fl = Z.flags;
  const bool err = (fl & GS_FLAG_ERRORS) != 0;
  if (tid == 0) {
    A.ids[row] = err ? -1 : static_cast<int32_t>(tok);
    if (A.flags) A.flags[row] = fl;
    if (A.cand_count) A.cand_count[row] = err ? 0 : L;
    if (A.logprob) {
      double lp = NAN;
      if (!err) {
        float x = load_logit(rowbase, DT, tok);
        if (cap != 0.0f) x = softcap(x, cap, inv_cap);
        lp = __dsub_rn(__dsub_rn(static_cast<double>(x), static_cast<double>(Z.raw_m)), log(Z.raw_s));
      }
      A.logprob[row] = lp;
    }
  }
  if (A.cand_ids) {
    // the first min(L, cand_cap) candidates in order, when they fit one gather
    int m = err ? 0 : (L < A.cand_cap ? L : A.cand_cap);
    if (m > n_fin) m = n_fin;
    int nw = 0;
    if (m > 0) {
      int cand = kNB;
      for (int b = tid; b < kNB; b += bs)
        if (static_cast<int>(bcnt[b]) <= m - 1 && m - 1 < static_cast<int>(bcnt[b + 1])) cand = b;
      for (int o = 16; o > 0; o >>= 1) cand = min(cand, __shfl_xor_sync(kFullMask, cand, o));
      __syncthreads();
      if ((tid & 31) == 0) Z.red_i[tid >> 5] = cand;
      __syncthreads();
      int b = kNB;
      for (int w = 0; w < (bs >> 5); ++w) b = min(b, Z.red_i[w]);
      __syncthreads();
      if (static_cast<int>(bcnt[b + 1]) <= GCAP) {
        gather(0, b);
        nw = m;
      }
    }
    for (int i = tid; i < A.cand_cap; i += bs) {
      A.cand_ids[static_cast<int64_t>(row) * A.cand_cap + i] = i < nw ? static_cast<int32_t>(G[i].id) : -1;
      if (A.cand_probs) A.cand_probs[static_cast<int64_t>(row) * A.cand_cap + i] = i < nw ? gp[i] : 0.0;
    }
  }
}

cudaError_t launch_large(const FinalizeArgs& a, int dtype, int rows, size_t smem, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  if (dtype == GS_DTYPE_F32) {
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(large_kernel<GS_DTYPE_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
      attr = true;
    }
    large_kernel<GS_DTYPE_F32><<<rows, kLargeThreads, smem, st>>>(a);
  } else {
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(large_kernel<GS_DTYPE_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
      attr = true;
    }
    large_kernel<GS_DTYPE_BF16><<<rows, kLargeThreads, smem, st>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace gs
