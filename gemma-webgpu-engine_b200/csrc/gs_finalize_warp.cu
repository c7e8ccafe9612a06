// Kernel 2, warp form: the per-row merge with one warp per row, for rows whose topK is at
// most 128 and whose history stride is at most 512 (the common decode settings).  The
// merge is a chain of dependent steps over few entries; one warp per row runs it without
// block barriers and keeps many rows in flight per SM.  It computes what finalize_kernel
// (gs_finalize.cu) computes, in the same IEEE double operations; only the order in which
// the full-vocabulary normaliser's terms are added differs (a few ulp, far inside the
// 1e-6 parity bar), and the cumulative sums of the filters and the draw use the same
// 4-items-per-lane prefix sums as the block version, so their decisions match it.
//
//   0. unit partials (lanes over the row's units)
//   1. penalised ids: a shared-memory hash counts each history id's occurrences (or adds
//      the counts of gs_batch.history_count) and keeps its first position; the entry of a
//      distinct, allowed id is scored exactly (src/runtime/sampling.ts:26-30) in the slot
//      of that first position
//   2. the units' candidate packs stream through a 256-entry buffer (threshold test,
//      radix-select compaction) down to the row's k best; a row of one unit (its packs
//      prefetched into registers) sorts them there first, largest first
//   3. maximum M, the penalised ids' normaliser terms (fixed slot order), then the entries
//      that can reach the top k (key >= the k-th streamed candidate's) are compacted in
//      place and sorted (logit/T desc, lower id first: src/runtime/sampling.ts:33-35) --
//      unless they are a one-unit row's sorted packs with no penalised entry among them
//   4. top-k, masked-id filler, probabilities, min-p, typical-p, top-p, seeded draw
//      (src/runtime/sampling.ts:44-64,82-90), log-probability, outputs
#include "gs_device.cuh"
#include "gs_block.cuh"
#include "gs_filter.cuh"
#include "gs_warp_filter.cuh"
#include "gs_internal.cuh"
#include "../../include/gsampler.h"

namespace gs {

namespace {

constexpr int kWWarps = 4;      // rows per CTA
constexpr int kWPack = 256;     // candidate buffer (packs)
constexpr int kWMaxK = kWFilterMax;
constexpr int kWMaxHist = 512;
constexpr int kWMaxUnits = 128;  // units per row (their counts stay in registers)
constexpr int kWHistPer = 8;     // history positions per lane per round of loads
constexpr int kWPackPer = 8;     // candidate packs per lane per round of loads
constexpr uint32_t kNone = 0xffffffffu;

__device__ __forceinline__ bool w_mask_allows(const uint32_t* mrow, uint32_t id) {
  return (__ldg(mrow + (id >> 5)) >> (id & 31)) & 1u;
}

__device__ __forceinline__ uint32_t w_hash(uint32_t v, int lg) { return (v * 2654435761u) >> (32 - lg); }

// In-place bitonic sort of e[0, n2) (power of two) into ent_before order by one warp.
__device__ void warp_sort_ent(Ent* e, int n2, int lane) {
  for (int k = 2; k <= n2; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = lane; i < n2; i += 32) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const Ent a = e[i], b = e[ixj];
          const bool up = (i & k) == 0;
          if (up ? ent_before(b, a) : ent_before(a, b)) {
            e[i] = b;
            e[ixj] = a;
          }
        }
      }
      __syncwarp();
    }
}

struct WGeom {
  int hcap, hlg, ecap, kc2;
  int bytes;  // per warp
};

WGeom warp_geom(int64_t history_stride, int kmax) {
  WGeom g{};
  g.kc2 = 1;
  while (g.kc2 < kmax) g.kc2 <<= 1;
  const int hs = static_cast<int>(history_stride);
  g.hcap = 0;
  g.hlg = 0;
  if (hs > 0) {
    g.hcap = 64;
    g.hlg = 6;
    while (g.hcap < 2 * hs) {
      g.hcap <<= 1;
      ++g.hlg;
    }
  }
  g.ecap = 32;
  while (g.ecap < hs + g.kc2) g.ecap <<= 1;
  const int hash_b = 12 * g.hcap;
  const int pack_b = 8 * kWPack + 4 * 256 + 4 * (kWMaxUnits + 1);
  const int work_b = g.kc2 * (4 + 8 + 8 + 8 + 4 + 4 + 1) + 64;
  int r = hash_b > pack_b ? hash_b : pack_b;
  r = r > work_b ? r : work_b;
  g.bytes = (16 * g.ecap + r + 15) & ~15;
  return g;
}

template <int DT>
__global__ void __launch_bounds__(kWWarps * 32) finalize_warp_kernel(const __grid_constant__ FinalizeArgs A, int rows,
                                                                     int hcap, int hlg, int ecap, int kc2, int wbytes) {
  extern __shared__ __align__(16) unsigned char dsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWWarps + warp;
  if (row >= rows) return;  // whole warp
  const RowPlan* pp = A.plans ? A.plans + row : &A.plan0;
  const int mode = pp->mode;
  if (mode == kModeLarge) return;
  const bool greedy = mode == kModeGreedy;
  const double T = pp->temperature;
  const int S = A.splits;
  const unsigned lane_lt = (1u << lane) - 1u;

  unsigned char* wb = dsm + static_cast<size_t>(warp) * wbytes;
  Ent* ent = reinterpret_cast<Ent*>(wb);
  unsigned char* R = wb + 16 * ecap;  // hash, then pack buffer, then filter work (aliased)

  const int32_t state = A.mask_state ? A.mask_state[row] : -1;
  const bool has_mask = A.mask_table != nullptr && state >= 0 && state < A.mask_states;
  const uint32_t* mrow = has_mask ? A.mask_table + static_cast<int64_t>(state) * A.mask_words : nullptr;
  const unsigned char* rowbase =
      static_cast<const unsigned char*>(A.logits) + static_cast<int64_t>(row) * A.row_stride * (DT == GS_DTYPE_F32 ? 4 : 2);
  const UnitStat* ust = A.stats + static_cast<int64_t>(row) * S;

  // ---- 0. unit partials (S <= 128: lane l holds units l, l+32, l+64, l+96) ----
  unsigned fl = 0;
  int na = 0, nc = 0;
  float rm = -INFINITY;
  int ucnt[kWMaxUnits / 32];
#pragma unroll
  for (int q = 0; q < kWMaxUnits / 32; ++q) {
    const int u = q * 32 + lane;
    ucnt[q] = 0;
    if (u < S) {
      const UnitStat& st = ust[u];
      fl |= st.flags;
      na += st.n_allowed;
      ucnt[q] = st.n_cand;
      rm = fmaxf(rm, st.raw_m);
    }
    nc += ucnt[q];
  }
  fl = __reduce_or_sync(kFullMask, fl);
  na = static_cast<int>(__reduce_add_sync(kFullMask, static_cast<unsigned>(na)));
  nc = static_cast<int>(__reduce_add_sync(kFullMask, static_cast<unsigned>(nc)));
  rm = warp_max(rm);
  double rs = 0.0;
  if (A.want_raw) {
    for (int u = lane; u < S; u += 32) {
      const UnitStat& st = ust[u];
      if (st.raw_m > -INFINITY) rs = __dadd_rn(rs, __dmul_rn(st.raw_s, exp(static_cast<double>(st.raw_m) - static_cast<double>(rm))));
    }
    rs = warp_sum(rs);
  }
  if (has_mask && na == 0) fl |= GS_FLAG_ERR_DEADEND;
  if (greedy) fl |= GS_FLAG_GREEDY;

  // Loads that depend on nothing below are issued here, so that their latencies overlap
  // instead of adding up: the history ids (up to 32·kWHistPer of them stay in registers
  // for both history passes) and, for a row of one unit, its candidate packs.
  int hl = 0;
  {
    int64_t h64 = A.history_len ? A.history_len[row] : 0;
    if (h64 > A.history_stride) h64 = A.history_stride;
    if (h64 < 0) h64 = 0;
    hl = static_cast<int>(h64);
  }
  const int32_t* hrow = A.history + static_cast<int64_t>(row) * A.history_stride;
  const bool hreg = hl <= 32 * kWHistPer;
  const int32_t* hcrow = A.history_count ? A.history_count + static_cast<int64_t>(row) * A.history_stride : nullptr;
  uint32_t hv[kWHistPer], hcv[kWHistPer];  // ids and the occurrences each stands for
#pragma unroll
  for (int q = 0; q < kWHistPer; ++q) {
    const int i = q * 32 + lane;
    hv[q] = hreg && i < hl ? static_cast<uint32_t>(hrow[i]) : kNone;
    hcv[q] = hcrow && hreg && i < hl ? static_cast<uint32_t>(max(hcrow[i], 1)) : 1u;
  }
  const bool pre_packs = S == 1 && nc <= 32 * kWPackPer;
  const bool packs_sorted = pre_packs && nc <= 128;  // (sorted in registers in phase 2)
  unsigned long long pre[kWPackPer];
#pragma unroll
  for (int q = 0; q < kWPackPer; ++q) {
    const int pidx = q * 32 + lane;
    pre[q] = pre_packs && pidx < nc ? A.cands[static_cast<int64_t>(row) * A.kcap + pidx] : 0ull;
  }

  // ---- 1. penalised ids ----
  if (fl & GS_FLAG_ERRORS) hl = 0;
  if (!(fl & GS_FLAG_ERRORS)) {
    if (hl > 0) {
      uint32_t* hk = reinterpret_cast<uint32_t*>(R);
      uint32_t* hp = hk + hcap;
      uint32_t* hc = hp + hcap;
      for (int i = lane; i < hcap; i += 32) {
        hk[i] = kNone;
        hp[i] = kNone;
        hc[i] = 0u;
      }
      __syncwarp();
      const int32_t* h = hrow;
      // (registers: the mask words of the ids are requested before the hash is built)
      uint32_t mwv[kWHistPer];
#pragma unroll
      for (int q = 0; q < kWHistPer; ++q)
        mwv[q] = hreg && has_mask && hv[q] < static_cast<uint64_t>(A.vocab) ? __ldg(mrow + (hv[q] >> 5)) : ~0u;
      auto insert = [&](uint32_t v, int i, uint32_t c) {
        uint32_t slot = w_hash(v, hlg);
        for (;;) {  // at most hl distinct ids in 2·hl+ slots: a free slot exists
          const uint32_t prev = atomicCAS(&hk[slot], kNone, v);
          if (prev == kNone || prev == v) break;
          slot = (slot + 1) & (hcap - 1);
        }
        atomicMin(&hp[slot], static_cast<uint32_t>(i));
        atomicAdd(&hc[slot], c);
      };
      if (hreg) {
#pragma unroll
        for (int q = 0; q < kWHistPer; ++q)
          if (hv[q] < static_cast<uint64_t>(A.vocab)) insert(hv[q], q * 32 + lane, hcv[q]);  // (negative ids are >= 2^31)
      } else {
        for (int i = lane; i < hl; i += 32) {
          const uint32_t v = static_cast<uint32_t>(h[i]);
          if (v < static_cast<uint64_t>(A.vocab)) insert(v, i, hcrow ? static_cast<uint32_t>(max(hcrow[i], 1)) : 1u);
        }
      }
      __syncwarp();
      const double rp = pp->repetition_penalty, pres = pp->presence_penalty, freq = pp->frequency_penalty;
      bool nonfinite = false;
      // positions holding an id's first occurrence (shared memory only), then their mask
      // words and logits loaded together: kWHistPer positions per lane per round
      for (int i0 = 0; i0 < hl; i0 += 32 * kWHistPer) {
        uint32_t v[kWHistPer], cnt[kWHistPer];
        bool first[kWHistPer];
#pragma unroll
        for (int q = 0; q < kWHistPer; ++q) {
          const int i = i0 + q * 32 + lane;
          first[q] = false;
          v[q] = kNone;
          cnt[q] = 0;
          if (i < hl) {
            v[q] = hreg ? hv[q] : static_cast<uint32_t>(h[i]);
            if (v[q] < static_cast<uint64_t>(A.vocab)) {
              uint32_t slot = w_hash(v[q], hlg);
              while (hk[slot] != v[q]) slot = (slot + 1) & (hcap - 1);
              first[q] = hp[slot] == static_cast<uint32_t>(i);
              cnt[q] = hc[slot];
            }
          }
        }
        bool allow[kWHistPer];
#pragma unroll
        for (int q = 0; q < kWHistPer; ++q)
          allow[q] = first[q] && !(has_mask && !(hreg ? (mwv[q] >> (v[q] & 31)) & 1u : w_mask_allows(mrow, v[q])));
        float x[kWHistPer];
#pragma unroll
        for (int q = 0; q < kWHistPer; ++q) x[q] = allow[q] ? load_logit(rowbase, DT, v[q]) : 0.0f;
#pragma unroll
        for (int q = 0; q < kWHistPer; ++q) {
          const int i = i0 + q * 32 + lane;
          if (i >= hl) continue;
          Ent e{-INFINITY, kNone, kNone};
          if (allow[q]) {  // entry at the id's first position; masked ids are -inf either way
            float xc = x[q];
            if (A.softcap != 0.0f) xc = softcap(xc, A.softcap, A.inv_softcap);
            if (!(xc < INFINITY)) nonfinite = true;  // NaN or +inf
            const double xp = penalise(static_cast<double>(xc), static_cast<double>(cnt[q]), rp, pres, freq);
            e = Ent{greedy ? xp : __ddiv_rn(xp, T), v[q], 1u};
          }
          ent[i] = e;
        }
      }
      if (__any_sync(kFullMask, nonfinite)) fl |= GS_FLAG_ERR_NONFINITE;
      __syncwarp();
    }
  }

  // ---- 2. the units' candidates: the row's k best ----
  const int k = greedy ? 1 : pp->k_eff;
  int n_all = hl;
  unsigned long long kth = 0;  // k-th best streamed pack (0: fewer than k)
  if (!(fl & GS_FLAG_ERRORS)) {
    unsigned long long* pb = reinterpret_cast<unsigned long long*>(R);
    unsigned* wh = reinterpret_cast<unsigned*>(pb + kWPack);
    int cnt = 0;
    unsigned long long tau = 0;
    const int kcap = A.kcap;
    // exclusive prefix of the units' candidate counts (unit u's packs are entries
    // [off_u, off_u + n_u) of the row's list), kept in shared memory for the lookups
    int* uo_s = reinterpret_cast<int*>(wh + 256);
    {
      int run = 0;
#pragma unroll
      for (int q = 0; q < kWMaxUnits / 32; ++q) {
        int incl = ucnt[q];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t = __shfl_up_sync(kFullMask, incl, o);
          if (lane >= o) incl += t;
        }
        const int u = q * 32 + lane;
        if (u < S) uo_s[u] = run + incl - ucnt[q];
        run += __shfl_sync(kFullMask, incl, 31);
      }
      if (lane == 0) uo_s[S] = run;  // == nc
      __syncwarp();
    }
    if (packs_sorted) {
      // a one-unit row's packs (at most 128, in registers): sorted here, largest first, so
      // that the entries below are in the reference's order unless a penalised one joins
      unsigned long long v[4] = {pre[0], pre[1], pre[2], pre[3]};
      int n2 = 2;
      while (n2 < nc) n2 <<= 1;
      warp_sort_desc_regs(v, n2, lane);
#pragma unroll
      for (int q = 0; q < 4; ++q) pre[q] = v[q];
    }
    for (int p0 = 0; p0 < nc; p0 += 32 * kWPackPer) {  // warp-uniform
      unsigned long long pk[kWPackPer];
#pragma unroll
      for (int q = 0; q < kWPackPer; ++q) {
        const int pidx = p0 + q * 32 + lane;
        pk[q] = 0ull;
        if (pidx < nc) {
          // the unit holding list entry pidx: the last u with off_u <= pidx (never an
          // empty unit: an empty unit shares its offset with the next one)
          int lo = 0, hi = S;
          while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (uo_s[mid] <= pidx) {
              lo = mid;
            } else {
              hi = mid;
            }
          }
          pk[q] = pre_packs ? pre[q] : A.cands[(static_cast<int64_t>(row) * S + lo) * kcap + (pidx - uo_s[lo])];
        }
      }
#pragma unroll
      for (int q = 0; q < kWPackPer; ++q) {
        bool pend = pk[q] != 0ull && pk[q] > tau;
        while (__any_sync(kFullMask, pend)) {
          const bool keep = pend && pk[q] > tau;
          const unsigned kb = __ballot_sync(kFullMask, keep);
          const int nk = __popc(kb);
          const int rank = __popc(kb & lane_lt);
          const int space = kWPack - cnt;
          if (keep && rank < space) pb[cnt + rank] = pk[q];
          pend = keep && rank >= space;
          cnt += nk < space ? nk : space;
          if (nk > space || cnt > kWPack - 32) {  // full: keep the k best
            __syncwarp();
            const unsigned long long t = warp_select_packs(pb, cnt, k, wh, lane);
            tau = t > tau ? t : tau;
            cnt = k;
          }
        }
      }
    }
    __syncwarp();
    if (cnt > k) {
      const unsigned long long t = warp_select_packs(pb, cnt, k, wh, lane);
      tau = t > tau ? t : tau;
      cnt = k;
    }
    __syncwarp();
    unsigned long long mn = ~0ull;
    for (int i = lane; i < cnt; i += 32) {
      const unsigned long long v = pb[i];
      mn = v < mn ? v : mn;
      const float x = pack_value(v);
      ent[hl + i] = Ent{greedy ? static_cast<double>(x) : __ddiv_rn(static_cast<double>(x), T), pack_id(v), 0u};
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(kFullMask, mn, o);
      mn = t < mn ? t : mn;
    }
    if (nc >= k && cnt >= k) kth = mn;
    n_all = hl + cnt;
    __syncwarp();
  }

  // ---- 3. maximum, the penalised ids' normaliser terms, the entries that can reach the top k ----
  double M = -INFINITY, pen_part = 0.0;
  int ns = 0;
  if (!(fl & GS_FLAG_ERRORS)) {
    double mx = -INFINITY;
    for (int i = lane; i < n_all; i += 32)
      if (ent[i].kind != kNone) mx = fmax(mx, ent[i].key);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(kFullMask, mx, o));
    M = mx;
    if (!greedy && M > -INFINITY) {
      for (int i = lane; i < hl; i += 32)
        if (ent[i].kind == 1u) pen_part = __dadd_rn(pen_part, exp(__dsub_rn(ent[i].key, M)));
      pen_part = warp_sum(pen_part);
    }
    double thr = -INFINITY;
    if (kth != 0ull) {
      const double x = static_cast<double>(pack_value(kth));
      thr = greedy ? x : __ddiv_rn(x, T);
    }
    int pen_kept = 0;  // penalised entries among them
    for (int i0 = 0; i0 < n_all; i0 += 32) {  // in place, order-preserving
      const int i = i0 + lane;
      Ent e{-INFINITY, kNone, kNone};
      if (i < n_all) e = ent[i];
      const bool keep = i < n_all && e.kind != kNone && e.key >= thr;
      const unsigned b = __ballot_sync(kFullMask, keep);
      pen_kept += __popc(__ballot_sync(kFullMask, keep && e.kind == 1u));
      __syncwarp();
      if (keep) ent[ns + __popc(b & lane_lt)] = e;
      ns += __popc(b);
      __syncwarp();
    }
    // A row of one unit holds its streamed entries in the reference's order already (its
    // packs sorted in phase 2 and kept in list order: at most k of them, no selection);
    // only penalised entries among them need the sort.
    if (!(packs_sorted && pen_kept == 0)) {
      const int n2 = pow2_ceil(ns > 0 ? ns : 1);
      for (int i = ns + lane; i < n2; i += 32) ent[i] = Ent{-INFINITY, kNone, kNone};
      __syncwarp();
      warp_sort_ent(ent, n2, lane);
    }
  }

  // ---- 4. top-k, filters, draw ----
  WWork w;
  {
    unsigned char* p = R;
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
  uint32_t tok = kNone;
  int n_final = 0;
  if (!(fl & GS_FLAG_ERRORS)) {
    if (greedy) {
      // argmax over the whole vocabulary: all -inf -> id 0 (sampling.ts:92-96)
      tok = (ns == 0 || ent[0].key == -INFINITY) ? 0u : ent[0].id;
      if (lane == 0) {
        w.cid[0] = tok;
        w.cp[0] = 1.0;
      }
      n_final = 1;
    } else {
      const int K = pp->top_k;
      int nC = ns < K ? ns : K;
      if (has_mask && ns < K && na < A.vocab) {
        // Fewer allowed ids than topK: the remaining slots are -inf ids (masked ones and
        // -inf logits) in ascending id order, exactly as the stable sort leaves them.
        int* mids = w.pos;
        const int nwords = static_cast<int>((A.vocab + 31) >> 5);
        int fill = 0;
        for (int w0 = 0; w0 < nwords && fill < K; w0 += 32) {  // warp-uniform
          const int wi = w0 + lane;
          uint32_t zero = 0;
          if (wi < nwords) {
            zero = ~__ldg(mrow + wi);
            if (wi == nwords - 1 && (A.vocab & 31)) zero &= (1u << (A.vocab & 31)) - 1u;
          }
          const int c = __popc(zero);
          int incl = c;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(kFullMask, incl, o);
            if (lane >= o) incl += u;
          }
          int base = fill + incl - c;
          for (uint32_t z = zero; z; z &= z - 1) {
            if (base < K) mids[base] = wi * 32 + __ffs(z) - 1;
            ++base;
          }
          fill += __shfl_sync(kFullMask, incl, 31);
        }
        __syncwarp();
        const int n_masked = fill < K ? fill : K;
        // merge the -inf tail of ent with the masked ids by id (serial, short)
        int j0 = 0;
        while (j0 < ns && ent[j0].key > -INFINITY) ++j0;
        Ent* tail = reinterpret_cast<Ent*>(w.cum);  // cum and skey: 16·kc2 bytes
        int t = 0;
        if (lane == 0) {
          int a = j0, b = 0, o = j0;
          while (o < K && (a < ns || b < n_masked)) {
            if (b >= n_masked || (a < ns && ent[a].id < static_cast<uint32_t>(mids[b]))) {
              tail[t++] = ent[a++];
            } else {
              tail[t++] = Ent{-INFINITY, static_cast<uint32_t>(mids[b++]), 2u};
            }
            ++o;
          }
          for (int i = 0; i < t; ++i) ent[j0 + i] = tail[i];
        }
        t = __shfl_sync(kFullMask, t, 0);
        __syncwarp();
        nC = j0 + t;
      }
      if (M == -INFINITY) {
        fl |= GS_FLAG_ERR_NONFINITE;  // every logit -inf: outside the domain
      } else {
        // full-vocabulary normaliser: streamed units + every penalised id
        double part = 0.0;
        for (int u = lane; u < S; u += 32) {
          const UnitStat& st = ust[u];
          if (st.m > -INFINITY) part = __dadd_rn(part, __dmul_rn(st.s, exp(__dsub_rn(__ddiv_rn(static_cast<double>(st.m), T), M))));
        }
        const double total = __dadd_rn(warp_sum(part), pen_part);
        for (int i = lane; i < nC; i += 32) {
          w.cid[i] = ent[i].id;
          w.cp[i] = __ddiv_rn(exp(__dsub_rn(ent[i].key, M)), total);
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

  // ---- outputs ----
  const bool err = (fl & GS_FLAG_ERRORS) != 0;
  if (lane == 0) {
    A.ids[row] = err ? -1 : static_cast<int32_t>(tok);
    if (A.flags) A.flags[row] = fl;
    if (A.cand_count) A.cand_count[row] = err ? 0 : n_final;
    if (A.logprob) {
      double lp = NAN;
      if (!err) {
        float x = load_logit(rowbase, DT, tok);
        if (A.softcap != 0.0f) x = softcap(x, A.softcap, A.inv_softcap);
        lp = __dsub_rn(__dsub_rn(static_cast<double>(x), static_cast<double>(rm)), log(rs));
      }
      A.logprob[row] = lp;
    }
  }
  if (A.cand_ids) {
    // final candidates in draw order; unused slots are -1 / 0 so outputs are fully defined
    const int nw = err ? 0 : (n_final < A.cand_cap ? n_final : A.cand_cap);
    for (int i = lane; i < A.cand_cap; i += 32) {
      A.cand_ids[static_cast<int64_t>(row) * A.cand_cap + i] = i < nw ? static_cast<int32_t>(w.cid[i]) : -1;
      if (A.cand_probs) A.cand_probs[static_cast<int64_t>(row) * A.cand_cap + i] = i < nw ? w.cp[i] : 0.0;
    }
  }
}

}  // namespace

bool finalize_warp_eligible(const FinalizeArgs& a, int kmax, size_t* smem) {
  if (a.shard_mode != 0 || kmax > kWMaxK || a.splits > kWMaxUnits) return false;
  const int64_t hs = a.history ? a.history_stride : 0;
  if (hs > kWMaxHist) return false;
  const WGeom g = warp_geom(hs, kmax);
  *smem = static_cast<size_t>(kWWarps) * g.bytes;
  return *smem <= 200 * 1024;
}

cudaError_t launch_finalize_warp(const FinalizeArgs& a, int dtype, int rows, int kmax, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  const int64_t hs = a.history ? a.history_stride : 0;
  const WGeom g = warp_geom(hs, kmax);
  const size_t smem = static_cast<size_t>(kWWarps) * g.bytes;
  const int grid = (rows + kWWarps - 1) / kWWarps;
  if (dtype == GS_DTYPE_F32) {
    const cudaError_t e = cudaFuncSetAttribute(finalize_warp_kernel<GS_DTYPE_F32>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    finalize_warp_kernel<GS_DTYPE_F32><<<grid, kWWarps * 32, smem, st>>>(a, rows, g.hcap, g.hlg, g.ecap, g.kc2, g.bytes);
  } else {
    const cudaError_t e = cudaFuncSetAttribute(finalize_warp_kernel<GS_DTYPE_BF16>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    finalize_warp_kernel<GS_DTYPE_BF16><<<grid, kWWarps * 32, smem, st>>>(a, rows, g.hcap, g.hlg, g.ecap, g.kc2, g.bytes);
  }
  return cudaGetLastError();
}

}  // namespace gs
