// Kernel 3: the histogram path, for rows whose candidate list is not bounded by a small
// topK (topK == 0 or topK > GS_MAX_TOP_K with V > GS_MAX_TOP_K).
//
// The reference keeps the whole sorted vocabulary as candidates (src/runtime/sampling.ts:44)
// and then cuts prefixes of it: min-p (:45-48, a prefix because p falls along the order),
// top-p (:56, cumulativeCut :82-90) and the draw (:58-64).  Every one of these is a
// position in the sorted order where a running count or a running probability crosses a
// value.  Instead of sorting 262144 entries, the path finds the crossings from a
// histogram and sorts only the few bins that hold them.  Four launches follow the
// streaming pass (which has produced each unit's live maximum and sum):
//   hist     a cluster of 8 CTAs per row, each streaming an eighth of the row into a
//            4096-bin histogram over logit/T distance below the row's live maximum
//            (monotone in the sort key, so a bin holds a contiguous range of the
//            reference's order): per bin the count of live values and the sum of
//            q = round((1 - e^-delta)·2^qbits), delta the value's key distance below the
//            bin's top, so that the bin's mass is e^(top - M)·(count - sum q·2^-qbits)
//            with 32-bit shared-memory atomics only.  The eight histograms are summed
//            through distributed shared memory;
//   select   one CTA per row: the penalised ids (distinct history ids counted in a
//            shared-memory hash table, scored exactly in double), the row maximum M, the
//            full-vocabulary normaliser, the binned masses and their prefix sums, and the
//            bins that can hold each crossing (min-p, topK, top-p, the draw, the head of
//            the candidate list);
//   gather   many CTAs per row append the live ids of the selected bins to a row list;
//   resolve  one CTA per row places the list bin by bin, sorts each bin exactly
//            (logit/T descending, lower id first) and resolves the crossings with exact
//            double probabilities, walking from the binned prefix at each bin's start.
// Sums are integer (fixed point) or taken in a fixed order, so the result is
// bit-reproducible.  Decisions within 1e-6 of a boundary are flagged.
#include <cooperative_groups.h>

#include <climits>

#include "gs_device.cuh"
#include "gs_block.cuh"
#include "gs_internal.cuh"
#include "../../include/gsampler.h"

namespace cg = cooperative_groups;

namespace gs {

namespace {

constexpr int kNB = 4096;              // histogram bins
constexpr double kRangeKeys = 40.0;    // bins span at most 40 units of logit/T below the maximum
constexpr double kMinRangeKeys = 1e-3; // ... and at least this many (all live values equal)
constexpr int kCluster = 8;            // histogram CTAs per row (one cluster)
constexpr int kHistThreads = 512;
constexpr int kHistSub = 32768;        // ids per live-bitmap pass of a histogram CTA
#ifndef GS_HIST_MIN_BLOCKS
#define GS_HIST_MIN_BLOCKS 3
#endif
constexpr int kHistMinBlocks = GS_HIST_MIN_BLOCKS;  // resident histogram CTAs per SM
constexpr int kHistQueue = 8192;       // live values a histogram CTA keeps in shared memory
constexpr int kSelectThreads = 1024;
constexpr int kGatherThreads = 256;
constexpr int kGatherIds = 16384;      // ids per gather CTA
constexpr int kResolveThreads = 1024;
constexpr int kGCap = 8192;            // entries of the selected bins per row
constexpr int kWarpSortMax = 1024;     // larger bins are sorted by the whole CTA
constexpr double kBoundary = 1e-6;
constexpr double kSelMargin = 4e-6;    // relative slack when bins are picked from binned masses
constexpr double kTypMargin = 1e-5;    // relative slack of the typical-p bounds (binned moments)
constexpr int kMaxRanges = 12;         // bin ranges the select kernel marks per row
constexpr int kSortSmem = 2048;        // typical-p: annulus entries sorted in shared memory
constexpr float kMaxDelta = 0.0105f;   // bin width (40/4096 key units) plus slack
constexpr size_t kSelUnion = (static_cast<size_t>(kNB + 1) * 12 + 15) / 16 * 16;  // select: start of its union
static_assert(kNB / kCluster == kHistThreads, "one reduced bin per thread and cluster rank (512-thread CTAs)");
static_assert(kNB == 4 * kSelectThreads && kNB == 4 * kResolveThreads, "four bins per thread");

// Per-row header shared by the four kernels (256-byte slot).
struct LargeRow {
  unsigned flags;
  int32_t n_allowed;
  int32_t n_slots;   // penalised-entry slots (the row's history length)
  int32_t n_fin;     // finite candidates: live values and penalised entries
  int32_t g_count;   // entries the gather kernel appended
  int32_t g_need;    // entries (live and penalised) of the selected bins
  int32_t mp_lo;     // min-p bins [mp_lo, mp_hi], -1 without min-p
  int32_t mp_hi;
  float gat_lo;      // raw logits below this lie below every selected bin
  float Mx;          // maximum over live values (allowed and not penalised)
  float bscale;      // bins per logit unit below Mx (the histogram kernel sets the row's bins)
  float bwidth;      // logit units per bin
  float Mn;          // minimum over live values
  float raw_m;
  double raw_s;
  double M;          // maximum key (logit/T) over live values and penalised entries
  double total;      // full-vocabulary normaliser relative to M
  double uniform;    // the draw's uniform
  double rng_next;   // the PRNG state after the draw
  // typical-p (select): bounds of the surprise centre H - ln(total) (key units) and of
  // the surprise level at the cut, and the bins [aL0, aL1], [aR0, aR1] (-1: none) that
  // can hold the cut's two ends
  double cc_lo, cc_hi, s_lo, s_hi;
  int32_t typ;  // kTypNone, kTypCut, kTypAll
  int32_t aL0, aL1, aR0, aR1;
  int32_t iB0, iB1;  // bins between the two ends (every entry's surprise below s_lo), -1: none
  // typical pre-pass (resolve kernel, phase 0): the run [t_r0, t_lend), the running
  // probability before it, and the bins of its second gather (W.sel2)
  int64_t t_r0, t_lend;
  double t_c0;
  int32_t g_need2;  // entries of the second gather's bins
  float gat_lo2;    // as gat_lo, for the second gather
};
constexpr int kTypNone = 0;  // no typical-p cut (or one equal to a top-p cut)
constexpr int kTypCut = 1;   // the cut lies in the annulus bins
constexpr int kTypAll = 2;   // the typical set is every candidate
static_assert(sizeof(LargeRow) <= 256, "header fits its slot");

// Per-row workspace: header | the histogram CTAs' row statistics | selected-bin bitmaps
// (first and second gather) | count prefix | mass prefix | first-moment prefix | penalised
// entries | gathered entries.
constexpr size_t kOffStats = 256;
constexpr size_t kOffSel = kOffStats + kCluster * sizeof(UnitStat);
constexpr size_t kOffSel2 = kOffSel + kNB / 8;
constexpr size_t kOffCpre = kOffSel2 + kNB / 8;
constexpr size_t kOffPpre = (kOffCpre + (kNB + 1) * 4 + 15) / 16 * 16;
constexpr size_t kOffM1 = (kOffPpre + (kNB + 1) * 8 + 15) / 16 * 16;
constexpr size_t kOffPen = (kOffM1 + (kNB + 1) * 8 + 15) / 16 * 16;

struct RowWs {
  LargeRow* hdr;
  UnitStat* hstat; // [kCluster] live maximum / sum, raw maximum / sum, allowed count, flags
  uint32_t* sel;   // [kNB / 32]
  uint32_t* sel2;  // [kNB / 32] bins of the second gather (typical-p rows)
  uint32_t* cpre;  // [kNB + 1] entries before bin b (the hist kernel leaves counts here)
  double* ppre;    // [kNB + 1] probability before bin b (the hist kernel leaves q sums here)
  double* m1pre;   // [kNB + 1] sum of e^(key - M)·(M - key) before bin b, typical-p rows (the
                   // hist kernel leaves its fixed-point within-bin sums here)
  Ent* pen;        // [n_slots] penalised entries (id 0xffffffff: empty slot)
  uint2* gath;     // [kGCap] {float bits of the soft-capped logit, id}
};

__device__ __forceinline__ RowWs row_ws(const FinalizeArgs& A, int row) {
  unsigned char* b = A.lws + static_cast<size_t>(row) * A.lrow_bytes;
  RowWs w;
  w.hdr = reinterpret_cast<LargeRow*>(b);
  w.hstat = reinterpret_cast<UnitStat*>(b + kOffStats);
  w.sel = reinterpret_cast<uint32_t*>(b + kOffSel);
  w.sel2 = reinterpret_cast<uint32_t*>(b + kOffSel2);
  w.cpre = reinterpret_cast<uint32_t*>(b + kOffCpre);
  w.ppre = reinterpret_cast<double*>(b + kOffPpre);
  w.m1pre = reinterpret_cast<double*>(b + kOffM1);
  w.pen = reinterpret_cast<Ent*>(b + kOffPen);
  w.gath = reinterpret_cast<uint2*>(b + kOffPen + static_cast<size_t>(A.lslots) * sizeof(Ent));
  return w;
}

__device__ __forceinline__ int bin_of(float x, float Mx, float scale) {
  const float d = Mx - x;
  if (!(d > 0.0f)) return 0;
  const float b = d * scale;
  return b >= static_cast<float>(kNB - 1) ? kNB - 1 : static_cast<int>(b);
}

// The row's bins: they span the live keys from the maximum Mx down to the minimum Mn (two
// bins of slack for the float binning, so the deepest bin stays empty), or 40 key units
// when the live keys spread wider (the deepest bin then gathers everything below, counted
// with zero mass: e^-40 each), so that a flat row (high temperature, small spread) still
// spreads its ids over the bins.
__device__ __forceinline__ void bin_geometry(double T, float Mx, float Mn, float* scale, float* width) {
  double r = kRangeKeys;
  if (Mx > -INFINITY && Mn > -INFINITY && Mx < INFINITY && Mx >= Mn) {
    const double fit = (static_cast<double>(Mx) - static_cast<double>(Mn)) / T * kNB / (kNB - 2);
    if (fit < r) r = fit > kMinRangeKeys ? fit : kMinRangeKeys;
  }
  *scale = static_cast<float>(static_cast<double>(kNB) / (r * T));
  *width = static_cast<float>(r * T / kNB);
}

// Ids of a histogram CTA: an eighth of the row, a multiple of 128.
__host__ __device__ inline int64_t hist_chunk(int64_t V) {
  const int64_t c = (V + kCluster - 1) / kCluster;
  return (c + 127) / 128 * 128;
}

// Bits of q (see the file comment): a histogram CTA sums at most hist_chunk(V) values of
// q <= kMaxDelta · 2^qbits in 32 bits.
__host__ __device__ inline int q_bits(int64_t V) {
  const int64_t hc = hist_chunk(V);
  int lg = 0;
  while ((1ll << lg) < hc) ++lg;
  return lg <= 15 ? 22 : 37 - lg;
}

__device__ __forceinline__ uint32_t hash_id(uint32_t v) { return v * 2654435761u; }

__device__ __forceinline__ double block_max_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(kFullMask, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double m = -INFINITY;
  for (int w = 0; w < nw; ++w) m = fmax(m, red[w]);
  __syncthreads();
  return m;
}

// Exclusive prefix sum of v over the block's threads (in thread order); *total: the sum.
__device__ __forceinline__ int block_excl_scan_i(int v, int* red, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFullMask, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) red[warp] = x;
  __syncthreads();
  int before = 0, tot = 0;
  for (int w = 0; w < nw; ++w) {
    const int t = red[w];
    if (w < warp) before += t;
    tot += t;
  }
  __syncthreads();
  *total = tot;
  return before + x - v;
}

__device__ __forceinline__ int block_min_i(int v, int* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(kFullMask, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int m = INT_MAX;
  for (int w = 0; w < nw; ++w) m = min(m, red[w]);
  __syncthreads();
  return m;
}

// Live bits of ids [lo, lo + n) of a row: allowed by the mask and not in the history
// (and, when `n_allowed` is given, this thread's count of allowed ids added to it).
__device__ __forceinline__ void build_live(uint32_t* live, const uint32_t* mrow, int64_t lo, int n, const int32_t* hrow,
                                           int64_t hl, int t, int nt, int* n_allowed = nullptr) {
  const int words = (n + 31) >> 5;
  for (int w = t; w < words; w += nt) {
    uint32_t m = mrow ? __ldg(mrow + (lo >> 5) + w) : 0xffffffffu;
    if (w == words - 1 && (n & 31)) m &= (1u << (n & 31)) - 1u;
    live[w] = m;
    if (n_allowed) *n_allowed += __popc(m);
  }
  __syncthreads();
  for (int64_t j = t; j < hl; j += nt) {
    const int64_t off = static_cast<int64_t>(hrow[j]) - lo;
    if (off >= 0 && off < n) atomicAnd(&live[off >> 5], ~(1u << (off & 31)));
  }
  __syncthreads();
}

// A raw-logit bound r such that every raw value v < r has softcap(v) < x (the soft cap
// is monotone over all float32 inputs), checked with the routine itself; -inf when no
// useful bound exists.  Lets a pass skip the soft cap of values that cannot matter.
__device__ float raw_below(float x, float cap, float inv_cap) {
  if (cap == 0.0f) return x;
  const double t = static_cast<double>(x) / static_cast<double>(cap);
  if (!(t > -1.0) || !(t < 0.999999)) return -INFINITY;
  float r = static_cast<float>(static_cast<double>(cap) * atanh(t));
  for (int i = 0; i < 16; ++i) {
    if (softcap(r, cap, inv_cap) < x) return r;
    r -= fmaxf(fabsf(r) * 9.765625e-4f, 9.765625e-4f);
  }
  return -INFINITY;
}

// In-place sort of e[0, n) into ent_before order by threads t of nt: a bitonic network
// whose every comparator puts the earlier entry at the lower index, so that entries
// past n behave as padding that sorts last and their comparators can be skipped.
template <bool kBlock>
__device__ void seg_sort(Ent* e, int n, int t, int nt) {
  if (n < 2) return;
  int lg = 0;
  while ((1 << lg) < n) ++lg;
  const int half_n2 = 1 << (lg - 1);
  for (int lk = 1; lk <= lg; ++lk) {
    for (int lj = lk - 1; lj >= 0; --lj) {
      // lj == lk - 1: the flip stage (partner i ^ (2^lk - 1)); below it the half-cleaners
      for (int q = t; q < half_n2; q += nt) {
        const int i = ((q >> lj) << (lj + 1)) | (q & ((1 << lj) - 1));
        const int p = lj == lk - 1 ? (i ^ ((1 << lk) - 1)) : (i + (1 << lj));
        if (p < n) {
          const Ent a = e[i], b = e[p];
          if (ent_before(b, a)) {
            e[i] = b;
            e[p] = a;
          }
        }
      }
      if (kBlock) __syncthreads();
      else __syncwarp();
    }
  }
}

}  // namespace

// resolve: entries | exact probabilities | bin starts | typical-p sort keys
static size_t large_resolve_smem_bytes() {
  return static_cast<size_t>(kGCap) * (sizeof(Ent) + 8) + (kNB + 4) * 4 + static_cast<size_t>(kSortSmem) * 8;
}

size_t large_row_bytes(int64_t slots) {
  const size_t gath = kOffPen + static_cast<size_t>(slots) * sizeof(Ent);
  return (gath + static_cast<size_t>(kGCap) * 8 + 255) / 256 * 256;
}

size_t large_select_smem_bytes(int64_t history_stride) {
  int64_t h2 = 64;
  while (h2 < 2 * history_stride) h2 <<= 1;
  const size_t hash = static_cast<size_t>(h2) * 12;
  const size_t pen_bins = static_cast<size_t>(kNB) * 20;  // fixed-point masses, counts and first moments of penalised entries
  return kSelUnion + (hash > pen_bins ? hash : pen_bins);
}

// ============================================================================ hist
// One cluster of kCluster CTAs per row, each owning hist_chunk(V) ids of the row.  The
// kernel takes the row statistics too (the streaming pass skips these rows):
//   phase 0: the maximum of the live (allowed, unpenalised) raw values; the soft cap is
//            monotone, so the capped maximum is the cap of the raw one (a raw -inf caps
//            to -cap, a finite value).  A chunk with at most kHistQueue live ids copies
//            their raw values into shared memory (the queue) on the way; a denser chunk
//            is read again in phase 1 (from L2).  The cluster combines the eight CTAs'
//            maxima through distributed shared memory.
//   phase 1: per live value its bin's count and q, and the sum of e^((x - Mx)/T) (and,
//            for log-probabilities, of e^(x - raw max) over every id).
// Rank r then sums bins [r·512, (r+1)·512) of the cluster's histograms into the row's
// workspace (counts over the count prefix array, q sums over the mass prefix array; the
// select kernel rewrites both with the prefix sums), and each CTA writes its statistics.
// RAW: the log-probability is wanted (phase 0 visits every id, and there is no queue).
// MOM: some row of the batch has typical-p; those rows also sum, per bin, the first moment
// r = round(dl·e^-dl·2^qbits) of their values (dl: the value's key distance below its
// bin's top), kept in a second dynamic shared-memory array after the queue.
// TPB: threads per CTA.  512 (three CTAs per SM) with the queue, for batches with a
// constraint table (sparse chunks); 256 (four per SM, no queue, 64 registers) otherwise, so
// that a batch of up to 74 rows' 8-CTA clusters fits in one wave.
template <int DT, bool RAW, bool MOM, int TPB>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(TPB, TPB == kHistThreads ? kHistMinBlocks : kHistMinBlocks + 1)
    large_hist_kernel(const __grid_constant__ FinalizeArgs A) {
  constexpr bool kQueue = TPB == kHistThreads;
  static_assert((kNB / kCluster) % TPB == 0, "whole bins per thread in the cluster reduction");
  __shared__ unsigned long long cq[kNB];  // per bin: count << 32 | sum of q
  __shared__ uint32_t live[kHistSub / 32];
  __shared__ float red_f[32];
  __shared__ int red_i[32];
  __shared__ double red_d[32];
  __shared__ float s_max[5];  // this CTA's raw maxima of the live / all values, any live / any value, live minimum
  extern __shared__ float queue[];  // [kHistQueue] live raw values of a sparse chunk
  cg::cluster_group cl = cg::this_cluster();
  const int rank = static_cast<int>(cl.block_rank());
  const int row = blockIdx.x / kCluster;
  const int tid = threadIdx.x, bs = blockDim.x;
  const RowPlan* pp = A.plans ? A.plans + row : &A.plan0;
  if (pp->mode != kModeLarge) return;  // the whole cluster (one row)
  const RowWs W = row_ws(A, row);
  const double T = pp->temperature;
  const float invT = static_cast<float>(1.0 / T);
  uint32_t* rsum_bins = reinterpret_cast<uint32_t*>(queue + (kQueue ? kHistQueue : 0));  // [kNB] (MOM launches)
  const bool mom = MOM && pp->typical_p < 1;  // (the whole cluster: one row)
  const float a2_hi = pp->a2_hi, a2_lo = pp->a2_lo;
  const float qmul = static_cast<float>(ldexp(1.0, q_bits(A.vocab)));
  const int64_t V = A.vocab;
  const int64_t hc = hist_chunk(V);
  const int64_t lo = rank * hc;
  const int n = static_cast<int>(V - lo < 0 ? 0 : (V - lo < hc ? V - lo : hc));
  const int32_t state = A.mask_state ? A.mask_state[row] : -1;
  const bool has_mask = A.mask_table != nullptr && state >= 0 && state < A.mask_states;
  const uint32_t* mrow = has_mask ? A.mask_table + static_cast<int64_t>(state) * A.mask_words : nullptr;
  constexpr int ESZ = DT == GS_DTYPE_F32 ? 4 : 2;
  constexpr int VE = 16 / ESZ;
  constexpr uint32_t kVecBits = (1u << VE) - 1u;
  const unsigned char* rowbase = static_cast<const unsigned char*>(A.logits) + static_cast<int64_t>(row) * A.row_stride * ESZ;
  const float cap = A.softcap, inv_cap = A.inv_softcap;
  // a raw value x is an error (NaN, or +inf without a soft cap) when !(x <= lim)
  const float lim = cap != 0.0f ? INFINITY : 3.40282347e38f;  // (the largest finite float)
  int64_t hl = A.history_len ? A.history_len[row] : 0;
  if (hl > A.history_stride) hl = A.history_stride;
  if (hl < 0) hl = 0;
  const int32_t* hrow = A.history + static_cast<int64_t>(row) * A.history_stride;
  const bool one_pass_bits = n <= kHistSub;  // the live bits stay valid for phase 1

  // ---- phase 0: maxima, allowed count, non-finite values (and the queue) ----
  float lmax = -INFINITY, rmax = -INFINITY, lmin = INFINITY;
  int nallow = 0, bad = 0, any_l = 0, any_v = 0;
  int qn = -1;  // queued values; -1: phase 1 reads the chunk again
  for (int s0 = 0; s0 < n; s0 += kHistSub) {
    const int sn = n - s0 < kHistSub ? n - s0 : kHistSub;
    const unsigned char* base = rowbase + (lo + s0) * ESZ;
    __syncthreads();
    build_live(live, mrow, lo + s0, sn, hrow, hl, tid, bs, &nallow);
    if (!RAW && one_pass_bits && kQueue) {
      // each thread takes a run of live words; their values land at its scan offset
      const int words = (sn + 31) >> 5;
      const int wpt = (words + bs - 1) / bs;
      const int w_lo = min(tid * wpt, words), w_hi = min(w_lo + wpt, words);
      int c = 0;
      for (int w = w_lo; w < w_hi; ++w) c += __popc(live[w]);
      int total = 0;
      int off = block_excl_scan_i(c, red_i, &total);
      if (total <= kHistQueue) {  // (block-uniform)
        qn = total;
        for (int w = w_lo; w < w_hi; ++w) {
          uint32_t bits = live[w];
          while (bits) {  // eight loads in flight
            float v[8];
            int k = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if (bits) {
                const int b = __ffs(bits) - 1;
                bits &= bits - 1u;
                v[j] = load_logit(base, DT, w * 32 + b);
                k = j + 1;
              }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (j < k) queue[off + j] = v[j];
            off += k;
          }
        }
        break;  // (one sub-chunk)
      }
    }
    int done = 0;
    if ((reinterpret_cast<uintptr_t>(base) & 15) == 0) {
      const int nv = sn / VE;
      const uint4* v4 = reinterpret_cast<const uint4*>(base);
      for (int v0 = tid; v0 < nv; v0 += 4 * bs) {  // four vectors per thread in flight
        uint4 r[4];
        uint32_t lb[4];
        bool in[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int vi = v0 + u * bs;
          in[u] = vi < nv;
          lb[u] = in[u] ? (live[(vi * VE) >> 5] >> ((vi * VE) & 31)) & kVecBits : 0u;
          if (RAW ? in[u] : lb[u] != 0u) r[u] = ld_stream_u4(v4 + vi);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (!(RAW ? in[u] : lb[u] != 0u)) continue;
          any_l |= lb[u] != 0u;
          any_v = 1;
          const uint32_t w[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
          for (int i = 0; i < VE; ++i) {
            const float x = DT == GS_DTYPE_F32 ? __uint_as_float(w[i]) : ((i & 1) ? bf16_hi(w[i >> 1]) : bf16_lo(w[i >> 1]));
            const bool l = (lb[u] >> i) & 1u;
            lmax = fmaxf(lmax, l ? x : -INFINITY);
            lmin = fminf(lmin, l ? x : INFINITY);
            if (RAW) {
              rmax = fmaxf(rmax, x);
              bad |= !(x <= lim);
            } else {
              bad |= l && !(x <= lim);
            }
          }
        }
      }
      done = nv * VE;
    }
    for (int i = done + tid; i < sn; i += bs) {
      const bool l = (live[i >> 5] >> (i & 31)) & 1u;
      if (!(RAW || l)) continue;
      const float x = load_logit(base, DT, i);
      any_l |= l;
      any_v = 1;
      if (l) {
        lmax = fmaxf(lmax, x);
        lmin = fminf(lmin, x);
      }
      if (RAW) rmax = fmaxf(rmax, x);
      if (RAW || l) bad |= !(x <= lim);
    }
  }
  if (qn >= 0) {
    __syncthreads();
    for (int i = tid; i < qn; i += bs) {
      const float x = queue[i];
      lmax = fmaxf(lmax, x);
      lmin = fminf(lmin, x);
      bad |= !(x <= lim);
    }
    any_l = qn > 0;
  }
  lmax = block_max_f(lmax, red_f);
  lmin = -block_max_f(-lmin, red_f);
  if (RAW) rmax = block_max_f(rmax, red_f);
  nallow = block_sum_i(nallow, red_i);
  bad = __syncthreads_or(bad);
  any_l = __syncthreads_or(any_l);
  any_v = __syncthreads_or(any_v);
  if (tid == 0) {
    s_max[0] = lmax;
    s_max[1] = rmax;
    s_max[2] = static_cast<float>(any_l);
    s_max[3] = static_cast<float>(any_v);
    s_max[4] = lmin;
  }
  for (int b = tid; b < kNB; b += bs) {
    cq[b] = 0ull;
    if (mom) rsum_bins[b] = 0;
  }
  cl.sync();
  float Mraw = -INFINITY, Rraw = -INFINITY, Nraw = INFINITY;
  bool row_l = false, row_v = false;
#pragma unroll
  for (int r = 0; r < kCluster; ++r) {
    const float* pm = cl.map_shared_rank(s_max, r);
    Mraw = fmaxf(Mraw, pm[0]);
    Rraw = fmaxf(Rraw, pm[1]);
    row_l |= pm[2] != 0.0f;
    row_v |= pm[3] != 0.0f;
    Nraw = fminf(Nraw, pm[4]);
  }
  const float Mx = cap != 0.0f ? (row_l ? softcap(Mraw, cap, inv_cap) : -INFINITY) : Mraw;
  const float Rm = cap != 0.0f ? (row_v ? softcap(Rraw, cap, inv_cap) : -INFINITY) : Rraw;
  const float Mn = cap != 0.0f ? (row_l ? softcap(Nraw, cap, inv_cap) : INFINITY) : Nraw;
  float scale, width;
  bin_geometry(T, Mx, Mn, &scale, &width);
  if (rank == 0 && tid == 0) {
    W.hdr->bscale = scale;
    W.hdr->bwidth = width;
    W.hdr->Mn = Mn;
  }

  // ---- phase 1: histogram and sums ----
  // Capped values, two at once (packed f32x2 arithmetic).
  auto cap2 = [&](float r0, float r1) {
    float2 x = make_float2(r0, r1);
    if (cap != 0.0f) {
      float2 z;
      x = softcap2_poly(x, cap, inv_cap, &z);
      if (!(z.x < kSoftcapPolyZ)) x.x = softcap(r0, cap, inv_cap);  // |x| >= c (and NaN)
      if (!(z.y < kSoftcapPolyZ)) x.y = softcap(r1, cap, inv_cap);
    }
    return x;
  };
  // Two capped values; l0 / l1: the value is live.  Per live value: e^((x - Mx)/T) (as
  // 2^(d·a2), a2 split in two products) into `acc`, its bin's count, and q (the deepest
  // bin's mass, below e^-40 of the top, is taken as 0).
  const float2 c_width = make_float2(width, width), c_invT = make_float2(invT, invT);
  auto hist2 = [&](float2 x, bool l0, bool l1, float& acc) {
    l0 = l0 && x.x > -INFINITY;  // -inf (no soft cap): not a finite candidate
    l1 = l1 && x.y > -INFINITY;
    const float d0 = fmaxf(Mx - x.x, 0.0f), d1 = fmaxf(Mx - x.y, 0.0f);
    const float e0 = ex2_approx(fmaf(-d0, a2_lo, -d0 * a2_hi)), e1 = ex2_approx(fmaf(-d1, a2_lo, -d1 * a2_hi));
    acc += (l0 ? e0 : 0.0f) + (l1 ? e1 : 0.0f);
    const int b0 = static_cast<int>(fminf(d0 * scale, static_cast<float>(kNB - 1)));
    const int b1 = static_cast<int>(fminf(d1 * scale, static_cast<float>(kNB - 1)));
    // 1 - e^-dl by its Taylor series (dl <= 0.0105: the truncation is below 1e-12)
    float2 dl = __fmul2_rn(__ffma2_rn(make_float2(-static_cast<float>(b0), -static_cast<float>(b1)), c_width,
                                      make_float2(d0, d1)), c_invT);
    dl.x = fminf(fmaxf(dl.x, 0.0f), kMaxDelta);
    dl.y = fminf(fmaxf(dl.y, 0.0f), kMaxDelta);
    float2 h = __ffma2_rn(dl, make_float2(-1.0f / 24.0f, -1.0f / 24.0f), make_float2(1.0f / 6.0f, 1.0f / 6.0f));
    h = __ffma2_rn(dl, h, make_float2(-0.5f, -0.5f));
    h = __ffma2_rn(dl, h, make_float2(1.0f, 1.0f));
    const float2 om = __fmul2_rn(__fmul2_rn(dl, h), make_float2(qmul, qmul));
    const uint32_t q0 = b0 < kNB - 1 ? __float2uint_rn(om.x) : 0u;
    const uint32_t q1 = b1 < kNB - 1 ? __float2uint_rn(om.y) : 0u;
    // (a CTA's sum of q stays below 2^32: no carry into the count)
    if (l0) atomicAdd(&cq[b0], (1ull << 32) | q0);
    if (l1) atomicAdd(&cq[b1], (1ull << 32) | q1);
    if (mom) {
      // dl·e^-dl = dl - dl·(1 - e^-dl)
      const float2 rm = __fmul2_rn(__ffma2_rn(make_float2(-dl.x, -dl.y), __fmul2_rn(dl, h), dl), make_float2(qmul, qmul));
      const uint32_t r0 = b0 < kNB - 1 ? __float2uint_rn(rm.x) : 0u;
      const uint32_t r1 = b1 < kNB - 1 ? __float2uint_rn(rm.y) : 0u;
      if (l0 && r0) atomicAdd(&rsum_bins[b0], r0);
      if (l1 && r1) atomicAdd(&rsum_bins[b1], r1);
    }
  };
  // (a thread adds at most 64 terms of at most 1 in float per sub-chunk, as the streaming
  // pass does per tile; the sub-chunk sums add in double)
  double ssum = 0.0, rsum = 0.0;
  if (qn >= 0) {
    float sacc = 0.0f;
    for (int i = 2 * tid; i < qn; i += 2 * bs) {
      const bool has1 = i + 1 < qn;
      hist2(cap2(queue[i], has1 ? queue[i + 1] : 0.0f), true, has1, sacc);
    }
    ssum = static_cast<double>(sacc);
  } else {
    for (int s0 = 0; s0 < n; s0 += kHistSub) {
      const int sn = n - s0 < kHistSub ? n - s0 : kHistSub;
      const unsigned char* base = rowbase + (lo + s0) * ESZ;
      if (!one_pass_bits) {
        __syncthreads();
        build_live(live, mrow, lo + s0, sn, hrow, hl, tid, bs);
      }
      float sacc = 0.0f, racc = 0.0f;
      // per pair of values: capped, raw sum (every id), histogram (live ids)
      auto pair = [&](float r0, float r1, bool v1, uint32_t lbits) {
        const float2 x = cap2(r0, r1);
        if (RAW) {
          const float g0 = x.x - Rm, g1 = x.y - Rm;
          racc += ex2_approx(fmaf(g0, kL2eLo, g0 * kL2eHi)) + (v1 ? ex2_approx(fmaf(g1, kL2eLo, g1 * kL2eHi)) : 0.0f);
        }
        if (lbits & 3u) hist2(x, lbits & 1u, (lbits >> 1) & 1u, sacc);
      };
      int done = 0;
      if ((reinterpret_cast<uintptr_t>(base) & 15) == 0) {
        const int nv = sn / VE;
        const uint4* v4 = reinterpret_cast<const uint4*>(base);
        for (int v0 = tid; v0 < nv; v0 += 4 * bs) {
          uint4 r[4];
          uint32_t lb[4];
          bool in[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int vi = v0 + u * bs;
            in[u] = vi < nv;
            lb[u] = in[u] ? (live[(vi * VE) >> 5] >> ((vi * VE) & 31)) & kVecBits : 0u;
            if (RAW ? in[u] : lb[u] != 0u) r[u] = ld_stream_u4(v4 + vi);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (!(RAW ? in[u] : lb[u] != 0u)) continue;
            const uint32_t w[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
            for (int i = 0; i < VE; i += 2) {
              const float a0 = DT == GS_DTYPE_F32 ? __uint_as_float(w[i & 3]) : bf16_lo(w[i >> 1]);
              const float a1 = DT == GS_DTYPE_F32 ? __uint_as_float(w[(i + 1) & 3]) : bf16_hi(w[i >> 1]);
              pair(a0, a1, true, lb[u] >> i);
            }
          }
        }
        done = nv * VE;
      }
      for (int i = done + tid; i < sn; i += bs) {
        const uint32_t l = (live[i >> 5] >> (i & 31)) & 1u;
        if (RAW || l) pair(load_logit(base, DT, i), 0.0f, false, l);
      }
      ssum += static_cast<double>(sacc);
      rsum += static_cast<double>(racc);
    }
  }
  ssum = block_sum_d(ssum, red_d);
  if (RAW) rsum = block_sum_d(rsum, red_d);
  if (tid == 0) {
    UnitStat u{};
    u.m = Mx;
    u.raw_m = Rm;
    u.s = Mx > -INFINITY ? ssum : 0.0;
    u.raw_s = Rm > -INFINITY ? rsum : 0.0;
    u.n_allowed = nallow;
    u.n_cand = 0;
    u.flags = (bad || ssum != ssum) ? GS_FLAG_ERR_NONFINITE : 0u;
    if (A.mask_table != nullptr && state >= A.mask_states) u.flags |= GS_FLAG_ERR_INVALID;
    W.hstat[rank] = u;
  }
  cl.sync();
  {
    for (int b = rank * (kNB / kCluster) + tid; b < (rank + 1) * (kNB / kCluster); b += TPB) {
      uint32_t c = 0;
      unsigned long long q = 0;
#pragma unroll
      for (int r = 0; r < kCluster; ++r) {
        const unsigned long long v = cl.map_shared_rank(cq, r)[b];
        c += static_cast<uint32_t>(v >> 32);
        q += v & 0xffffffffull;
      }
      W.cpre[b] = c;
      reinterpret_cast<unsigned long long*>(W.ppre)[b] = q;
      if (mom) {
        unsigned long long r1 = 0;
#pragma unroll
        for (int r = 0; r < kCluster; ++r) r1 += cl.map_shared_rank(rsum_bins, r)[b];
        reinterpret_cast<unsigned long long*>(W.m1pre)[b] = r1;
      }
    }
  }
  cl.sync();  // every CTA keeps its shared memory until its peers have read it
}

// Exclusive prefix sum, in place, of a[0, kNB) over kSelectThreads threads (four
// consecutive bins per thread, a fixed order); a[kNB] gets the total.
__device__ void bins_excl_scan_d(double* a, double* red) {
  constexpr int kPer = kNB / kSelectThreads;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  double m[kPer];
  double tm = 0.0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    m[i] = a[tid * kPer + i];
    tm = __dadd_rn(tm, m[i]);
  }
  double im = tm;
  for (int o = 1; o < 32; o <<= 1) {
    const double u = __shfl_up_sync(kFullMask, im, o);
    if (lane >= o) im = __dadd_rn(u, im);
  }
  if (lane == 31) red[warp] = im;
  __syncthreads();
  double bm = 0.0;
  for (int w = 0; w < warp; ++w) bm = __dadd_rn(bm, red[w]);
  double lm = __shfl_up_sync(kFullMask, im, 1);
  if (lane == 0) lm = 0.0;
  bm = __dadd_rn(bm, lm);
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    a[tid * kPer + i] = bm;
    bm = __dadd_rn(bm, m[i]);
  }
  if (tid == kSelectThreads - 1) a[kNB] = bm;
  __syncthreads();
}

// ============================================================================ select
// One CTA per row: the row's statistics, its penalised entries, the binned masses and
// their prefix sums, and the bins that can hold a crossing.
template <int DT>
__global__ void __launch_bounds__(kSelectThreads) large_select_kernel(const __grid_constant__ FinalizeArgs A) {
  extern __shared__ __align__(16) unsigned char dsm[];
  double* md = reinterpret_cast<double*>(dsm);                // [kNB + 1] masses, then their prefix
  uint32_t* cnt = reinterpret_cast<uint32_t*>(md + kNB + 1);  // [kNB + 1] counts, then their prefix
  unsigned char* un = dsm + kSelUnion;                        // history hash, then penalised bins
  __shared__ double red_d[32];
  __shared__ float red_f[32];
  __shared__ int red_i[32];
  __shared__ unsigned s_flags;
  __shared__ int s_rng[2][kMaxRanges];
  __shared__ int s_nr, s_cb0, s_cb;
  const int row = blockIdx.x, tid = threadIdx.x, bs = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5;
  const RowPlan* pp = A.plans ? A.plans + row : &A.plan0;
  if (pp->mode != kModeLarge) return;
  const RowWs W = row_ws(A, row);
  const double T = pp->temperature;
  const int S = kCluster;              // the histogram CTAs' row statistics
  const UnitStat* ustats = W.hstat;
  const int64_t V = A.vocab;
  const int32_t state = A.mask_state ? A.mask_state[row] : -1;
  const bool has_mask = A.mask_table != nullptr && state >= 0 && state < A.mask_states;
  const uint32_t* mrow = has_mask ? A.mask_table + static_cast<int64_t>(state) * A.mask_words : nullptr;
  const unsigned char* rowbase =
      static_cast<const unsigned char*>(A.logits) + static_cast<int64_t>(row) * A.row_stride * (DT == GS_DTYPE_F32 ? 4 : 2);
  const float cap = A.softcap, inv_cap = A.inv_softcap;
  if (tid == 0) s_flags = GS_FLAG_LARGE_PATH;
  __syncthreads();

  // ---- row statistics (the histogram kernel's CTAs) ----
  unsigned fl = 0;
  int na = 0;
  float mx = -INFINITY, rm = -INFINITY;
  for (int u = tid; u < S; u += bs) {
    const UnitStat& st = ustats[u];
    fl |= st.flags;
    na += st.n_allowed;
    mx = fmaxf(mx, st.m);
    rm = fmaxf(rm, st.raw_m);
  }
  if (fl) atomicOr(&s_flags, fl);
  na = block_sum_i(na, red_i);
  mx = block_max_f(mx, red_f);
  rm = block_max_f(rm, red_f);
  double rs = 0.0;
  if (A.want_raw) {
    for (int u = tid; u < S; u += bs) {
      const UnitStat& st = ustats[u];
      if (st.raw_m > -INFINITY)
        rs = __dadd_rn(rs, __dmul_rn(st.raw_s, exp(static_cast<double>(st.raw_m) - static_cast<double>(rm))));
    }
    rs = block_sum_d(rs, red_d);
  }

  // ---- distinct history ids with their counts and first positions (hash table) ----
  int64_t hl = A.history_len ? A.history_len[row] : 0;
  if (hl > A.history_stride) hl = A.history_stride;
  if (hl < 0) hl = 0;
  const int32_t* hrow = A.history + static_cast<int64_t>(row) * A.history_stride;
  int h2 = 64;
  while (h2 < 2 * hl) h2 <<= 1;
  uint32_t* hkey = reinterpret_cast<uint32_t*>(un);
  int* hcnt = reinterpret_cast<int*>(hkey + h2);
  int* hfirst = hcnt + h2;
  for (int i = tid; i < h2; i += bs) {
    hkey[i] = 0xffffffffu;
    hcnt[i] = 0;
    hfirst[i] = INT_MAX;
  }
  __syncthreads();
  auto find_slot = [&](uint32_t v, bool insert) -> int {
    uint32_t s = hash_id(v) & static_cast<uint32_t>(h2 - 1);
    for (;;) {  // the table is at most half full
      const uint32_t k = insert ? atomicCAS(&hkey[s], 0xffffffffu, v) : hkey[s];
      if (k == 0xffffffffu || k == v) return static_cast<int>(s);
      s = (s + 1) & static_cast<uint32_t>(h2 - 1);
    }
  };
  const int32_t* hcrow = A.history_count ? A.history_count + static_cast<int64_t>(row) * A.history_stride : nullptr;
  for (int64_t j = tid; j < hl; j += bs) {
    const int32_t v = hrow[j];
    if (v < 0 || v >= V) continue;
    const int s = find_slot(static_cast<uint32_t>(v), true);
    atomicAdd(&hcnt[s], hcrow ? max(hcrow[j], 1) : 1);
    atomicMin(&hfirst[s], static_cast<int>(j));
  }
  __syncthreads();

  // ---- penalised entries: slot j holds the id first seen at history position j ----
  const double rp = pp->repetition_penalty, pres = pp->presence_penalty, freq = pp->frequency_penalty;
  double pmax = -INFINITY, pmin = INFINITY;
  for (int64_t j = tid; j < hl; j += bs) {
    Ent e{-INFINITY, 0xffffffffu, 0u};
    const int32_t v = hrow[j];
    if (v >= 0 && v < V) {
      const int s = find_slot(static_cast<uint32_t>(v), false);
      if (hfirst[s] == j && (!has_mask || ((__ldg(mrow + (v >> 5)) >> (v & 31)) & 1u))) {
        float x = load_logit(rowbase, DT, v);
        if (cap != 0.0f) x = softcap(x, cap, inv_cap);
        if (!(x < INFINITY)) atomicOr(&s_flags, GS_FLAG_ERR_NONFINITE);
        // src/runtime/sampling.ts:21-30: divide positive / multiply negative logits by the
        // repetition penalty, then subtract presence + count · frequency
        double xp = static_cast<double>(x);
        xp = xp < 0 ? __dmul_rn(xp, rp) : __ddiv_rn(xp, rp);
        xp = __dsub_rn(xp, __dadd_rn(pres, __dmul_rn(static_cast<double>(hcnt[s]), freq)));
        // kind holds the float32 rounding of the penalised logit, used only for binning
        e = Ent{__ddiv_rn(xp, T), static_cast<uint32_t>(v), __float_as_uint(static_cast<float>(xp))};
        pmax = fmax(pmax, e.key);
        pmin = fmin(pmin, e.key);
      }
    }
    W.pen[j] = e;
  }
  pmax = block_max_d(pmax, red_d);
  pmin = -block_max_d(-pmin, red_d);
  const double mxk = mx > -INFINITY ? __ddiv_rn(static_cast<double>(mx), T) : -INFINITY;
  const double M = fmax(mxk, pmax);

  // ---- full-vocabulary normaliser relative to M (fixed summation order) ----
  double part = 0.0;
  if (M > -INFINITY) {
    for (int u = tid; u < S; u += bs) {
      const UnitStat& st = ustats[u];
      if (st.m > -INFINITY)
        part = __dadd_rn(part, __dmul_rn(st.s, exp(__dsub_rn(__ddiv_rn(static_cast<double>(st.m), T), M))));
    }
    for (int64_t j = tid; j < hl; j += bs) {
      const Ent e = W.pen[j];
      if (e.id != 0xffffffffu && e.key > -INFINITY) part = __dadd_rn(part, exp(__dsub_rn(e.key, M)));
    }
  }
  const double total = block_sum_d(part, red_d);
  if (tid == 0) {
    unsigned f = s_flags;
    if (has_mask && na == 0) f |= GS_FLAG_ERR_DEADEND;
    if (!(M > -INFINITY)) f |= GS_FLAG_ERR_NONFINITE;
    double u = 0.0, st_next = 0.0;
    if (!(f & GS_FLAG_ERRORS)) {
      if (A.uniforms) {
        u = A.uniforms[row];
      } else {
        st_next = A.rng_state[row];
        u = seeded_next(&st_next);
      }
    }
    LargeRow* H = W.hdr;
    H->flags = f;
    H->n_allowed = na;
    H->n_slots = static_cast<int32_t>(hl);
    H->n_fin = 0;
    H->g_count = 0;
    H->g_need = 0;
    H->mp_lo = -1;
    H->mp_hi = -1;
    H->typ = kTypNone;
    H->g_need2 = 0;
    H->Mx = mx;
    H->raw_m = rm;
    H->raw_s = rs;
    H->M = M;
    H->total = total;
    H->uniform = u;
    H->rng_next = st_next;
    s_flags = f;
  }
  __syncthreads();
  if (s_flags & GS_FLAG_ERRORS) return;

  // ---- binned masses relative to M: live values from the histogram, then the
  //      penalised entries (fixed point, so that their sums are order-independent) ----
  const float Mx = mx, scale = W.hdr->bscale, width = W.hdr->bwidth;
  const double qunit = ldexp(1.0, -q_bits(V));
  const double inv_total = 1.0 / total, invT = 1.0 / T;  // (binned values: products suffice)
  unsigned long long* pfix = reinterpret_cast<unsigned long long*>(un);  // (the hash table is done)
  unsigned long long* pm1 = pfix + kNB;                                // penalised first moments
  uint32_t* pcnt = reinterpret_cast<uint32_t*>(pm1 + kNB);
  const bool typ = pp->typical_p < 1;
  for (int b = tid; b < kNB; b += bs) {
    const uint32_t c = W.cpre[b];
    const unsigned long long q = reinterpret_cast<const unsigned long long*>(W.ppre)[b];
    double m = 0.0, m1v = 0.0;
    if (c && b < kNB - 1) {
      const double top = __dsub_rn(
          __dmul_rn(__dsub_rn(static_cast<double>(Mx), static_cast<double>(b) * static_cast<double>(width)), invT), M);
      const double et = exp(top), se = __dsub_rn(static_cast<double>(c), static_cast<double>(q) * qunit);
      m = __dmul_rn(et, se);
      // first moment, sum of e^(key - M)·(M - key) = e^top·((-top)·sum e^-dl + sum dl·e^-dl)
      if (typ)
        m1v = __dmul_rn(et, __dadd_rn(__dmul_rn(-top, se),
                                      static_cast<double>(reinterpret_cast<const unsigned long long*>(W.m1pre)[b]) * qunit));
    }
    if (typ) W.m1pre[b] = m1v;  // (the same thread read the histogram's sum)
    cnt[b] = c;
    md[b] = m;
    pfix[b] = 0;
    pm1[b] = 0;
    pcnt[b] = 0;
  }
  __syncthreads();
  for (int64_t j = tid; j < hl; j += bs) {
    const Ent e = W.pen[j];
    if (e.id == 0xffffffffu || !(e.key > -INFINITY)) continue;
    const int b = bin_of(__uint_as_float(e.kind), Mx, scale);
    atomicAdd(&pcnt[b], 1u);
    const double ex = exp(__dsub_rn(e.key, M));
    atomicAdd(&pfix[b], static_cast<unsigned long long>(__dmul_rn(ex, 17592186044416.0) + 0.5));
    if (typ) atomicAdd(&pm1[b], static_cast<unsigned long long>(__dmul_rn(__dmul_rn(ex, __dsub_rn(M, e.key)), 17592186044416.0) + 0.5));
  }
  __syncthreads();
  // exclusive prefix over the bins, 4 consecutive bins per thread (fixed order)
  {
    constexpr int kPer = kNB / kSelectThreads;
    double m[kPer];
    uint32_t c[kPer];
    double tm = 0.0;
    uint32_t tc = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int b = tid * kPer + i;
      m[i] = __dadd_rn(md[b], static_cast<double>(pfix[b]) * 5.684341886080802e-14);  // 2^-44
      c[i] = cnt[b] + pcnt[b];
      tm = __dadd_rn(tm, m[i]);
      tc += c[i];
    }
    double im = tm;
    uint32_t ic = tc;
    for (int o = 1; o < 32; o <<= 1) {
      const double um = __shfl_up_sync(kFullMask, im, o);
      const uint32_t uc = __shfl_up_sync(kFullMask, ic, o);
      if (lane >= o) {
        im = __dadd_rn(um, im);
        ic += uc;
      }
    }
    if (lane == 31) {
      red_d[warp] = im;
      red_i[warp] = static_cast<int>(ic);
    }
    __syncthreads();
    double bm = 0.0;
    uint32_t bc = 0;
    for (int w = 0; w < warp; ++w) {
      bm = __dadd_rn(bm, red_d[w]);
      bc += static_cast<uint32_t>(red_i[w]);
    }
    double lm = __shfl_up_sync(kFullMask, im, 1);  // the lanes before this one
    uint32_t lc = __shfl_up_sync(kFullMask, ic, 1);
    if (lane == 0) {
      lm = 0.0;
      lc = 0;
    }
    bm = __dadd_rn(bm, lm);
    bc += lc;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int b = tid * kPer + i;
      md[b] = bm;
      cnt[b] = bc;
      bm = __dadd_rn(bm, m[i]);
      bc += c[i];
    }
    if (tid == bs - 1) {
      md[kNB] = bm;
      cnt[kNB] = bc;
    }
    __syncthreads();
  }
  for (int b = tid; b <= kNB; b += bs) {
    W.cpre[b] = cnt[b];
    W.ppre[b] = __dmul_rn(md[b], inv_total);  // (bin choice and walk bases: binned values)
  }
  double* m1 = reinterpret_cast<double*>(pfix);  // (pfix was read by the mass prefix)
  if (typ) {
    // first moments per bin: the live values' (above) and the penalised entries' (fixed
    // point); their prefix over the bins into W.m1pre
    for (int b = tid; b < kNB; b += bs) m1[b] = __dadd_rn(W.m1pre[b], static_cast<double>(pm1[b]) * 5.684341886080802e-14);
    __syncthreads();
    bins_excl_scan_d(m1, red_d);
    for (int b = tid; b <= kNB; b += bs) W.m1pre[b] = m1[b];
  }

  // ---- bins that can hold a crossing (thread 0) ----
  // Bins that must be gathered: the min-p threshold's neighbourhood, the bin where the
  // binned running mass reaches topP, the bins of the ranks L1 - 1 can take when no
  // top-p crossing is certain below L1, and the bins the draw's cursor can reach.  Bins
  // within the slack of those edges (where the exact running sum could fall on either
  // side) are added while the list stays within the gather capacity.
  if (tid == 0) {
    auto P = [&](int b) { return __dmul_rn(md[b], inv_total); };
    auto bstart = [&](double t) {  // first bin b with P(b + 1) >= t, kNB if none
      int l = 0, h = kNB;
      while (l < h) {
        const int m = (l + h) >> 1;
        if (P(m + 1) >= t) h = m;
        else l = m + 1;
      }
      return l;
    };
    auto bin_of_rank = [&](int64_t r) {  // the bin holding rank r (0 <= r < n_fin)
      int l = 0, h = kNB - 1;
      while (l < h) {
        const int m = (l + h) >> 1;
        if (static_cast<int64_t>(cnt[m + 1]) > r) h = m;
        else l = m + 1;
      }
      return l;
    };
    const int64_t n_fin = cnt[kNB];
    unsigned xflags = 0;
    int nr = 0;
    int64_t used = 0;
    auto rc = [&](int a, int b) -> int64_t { return a <= b ? static_cast<int64_t>(cnt[b + 1]) - cnt[a] : 0; };
    auto fits = [&](int a, int b) { return used + rc(a, b) <= kGCap; };
    auto add = [&](int a, int b) {
      if (nr < kMaxRanges && a <= b) {
        s_rng[0][nr] = a;
        s_rng[1][nr] = b;
        ++nr;
        used += rc(a, b);
      }
    };
    const int last_bin = n_fin > 0 ? bin_of_rank(n_fin - 1) : 0;
    const int64_t K = pp->top_k;
    const int64_t klim = (K > 0 && K < V) ? K : V;
    int64_t L1_lo = klim, L1_hi = klim;
    int mp_lo = -1, mp_hi = -1;
    if (pp->min_p > 0) {
      // p_i >= p_0·minP with p_0 = 1/total: key >= M + ln(minP)
      const float xth = static_cast<float>(T * (M + log(pp->min_p)));
      const int bt = bin_of(xth, Mx, scale);
      mp_lo = bt > 0 ? bt - 1 : 0;
      mp_hi = bt < kNB - 1 ? bt + 1 : kNB - 1;
      add(mp_lo, mp_hi);
      if (L1_lo > cnt[mp_lo]) L1_lo = cnt[mp_lo];
      if (L1_hi > cnt[mp_hi + 1]) L1_hi = cnt[mp_hi + 1];
    }
    // typical-p: the reference's entropy is NaN when a candidate has probability 0 (an id
    // whose key is -inf among [0, L1)); its surprise sort then keeps the order and the
    // typical cut is a running-sum cut like top-p, so the two merge into one threshold
    int typ_mode = kTypNone;
    double tpe = pp->top_p;
    if (typ && n_fin > 0) {
      if (!(pp->min_p > 0) && klim > n_fin) {
        tpe = fmin(tpe, pp->typical_p);
      } else if (fmin(static_cast<double>(W.hdr->Mn) / T, pmin) - M < -700.0 &&
                 bin_of_rank((L1_hi < n_fin ? L1_hi : n_fin) - 1) == kNB - 1) {
        xflags |= GS_FLAG_ERR_UNSUPPORTED;  // a candidate's probability may underflow to 0
      } else {
        typ_mode = kTypCut;
      }
    }
    int cb0 = 0, cb = -1;
    if (typ_mode == kTypCut) {
      // ---- typical-p (sampling.ts:49-55) over the candidates [0, L1) ----
      // With p = e^(key - M)/total, -ln p = delta + ln total (delta = M - key), so the
      // surprise |-ln p - H| is |delta - cc| with cc = H - ln total = sum_C p·delta -
      // ln total·(1 - P_C): a run of consecutive ranks around the rank where delta
      // crosses cc.  From the binned masses and moments: bounds [c0, c1] of cc, bounds
      // [s_lo, s_hi] of the surprise level where the running sum (in surprise order)
      // reaches typicalP, and the bins that can hold the run's two ends (gathered now).
      const double lnZ = log(total);
      auto cc_at = [&](int b) {  // cc for the candidates before bin b
        return __dsub_rn(__ddiv_rn(m1[b], total), __dmul_rn(lnZ, __dsub_rn(P(kNB), P(b))));
      };
      const int bl = L1_lo >= n_fin ? kNB : bin_of_rank(L1_lo);          // every bin before bl is in C
      const int bh = L1_hi >= n_fin ? last_bin : bin_of_rank(L1_hi - 1);  // no bin after bh is
      double c0 = cc_at(bl), c1 = cc_at(bh + 1);
      c0 -= kTypMargin * (1.0 + fabs(c0));
      c1 += kTypMargin * (1.0 + fabs(c1));
      const double wk = 1.0 / (static_cast<double>(scale) * T);          // key units per bin
      const double offK = __dsub_rn(M, __ddiv_rn(static_cast<double>(Mx), T));  // delta at bin 0's top
      // bin of key distance x; an entry of bin b has delta in [offK + (b-1)·wk, offK + (b+2)·wk)
      // (one bin of slack for the float binning; bin 0 from delta 0, the deepest bin unbounded)
      auto dfl = [&](double x) {
        return static_cast<int>(fmin(fmax(floor((x - offK) / wk), -8.0), static_cast<double>(kNB + 8)));
      };
      auto fullmass = [&](double s) {  // bins certainly in C with every delta in (c1 - s, c0 + s)
        const double lo = c1 - s, hi = c0 + s;
        if (!(hi > lo)) return 0.0;
        const int a = lo < 0 ? 0 : max(1, dfl(lo) + 2);
        const int b = min(min(dfl(hi) - 2, kNB - 2), bl - 1);
        return b >= a ? P(b + 1) - P(a) : 0.0;
      };
      auto touchmass = [&](double s) {  // bins possibly in C that can hold a delta in [c0 - s, c1 + s]
        const int a = max(0, dfl(c0 - s) - 2);
        const int b = min(min(dfl(c1 + s) + 2, kNB - 1), bh);
        return b >= a ? P(b + 1) - P(a) : 0.0;
      };
      const double tq = pp->typical_p;
      if (P(bh + 1) < tq * (1.0 - kTypMargin)) {
        typ_mode = kTypAll;  // the running sum cannot reach typicalP: every candidate stays
      } else {
        const double smax = fmax(c1, offK + (bh + 2) * wk - c0) + 4 * wk;
        double s_hi = smax, s_lo = 0.0;
        if (fullmass(smax) >= tq * (1.0 + kTypMargin)) {
          double a = 0.0, b = smax;
          for (int it = 0; it < 48; ++it) {
            const double m = 0.5 * (a + b);
            if (fullmass(m) >= tq * (1.0 + kTypMargin)) b = m;
            else a = m;
          }
          s_hi = b;
        }
        if (touchmass(0.0) < tq * (1.0 - kTypMargin)) {
          double a = 0.0, b = s_hi;
          for (int it = 0; it < 48; ++it) {
            const double m = 0.5 * (a + b);
            if (touchmass(m) < tq * (1.0 - kTypMargin)) a = m;
            else b = m;
          }
          s_lo = a;
        }
        // the run's ends: deltas in [c0 - s_hi, c1 - s_lo] (left) and [c0 + s_lo, c1 + s_hi]
        // (right); every entry between them has surprise < s_lo
        int aL0 = -1, aL1 = -1, aR0 = -1, aR1 = -1, iB0 = -1, iB1 = -1;
        if (c1 - s_lo >= 0) {
          aL0 = c0 - s_hi < 0 ? 0 : max(0, dfl(c0 - s_hi) - 1);
          aL1 = min(bh, max(0, dfl(c1 - s_lo) + 1));
          if (aL0 > aL1) aL0 = aL1 = -1;
        }
        aR0 = max(0, dfl(c0 + s_lo) - 1);
        aR1 = min(bh, dfl(c1 + s_hi) + 1);
        if (aR0 > aR1) aR0 = aR1 = -1;
        if (aL0 >= 0 && aR0 >= 0 && aR0 <= aL1 + 1) {  // the two ends share bins
          aL1 = max(aL1, aR1);
          aR0 = aR1 = -1;
        } else {
          iB0 = aL0 >= 0 ? aL1 + 1 : 0;
          iB1 = aR0 >= 0 ? aR0 - 1 : bh;
          if (iB0 > iB1) iB0 = iB1 = -1;
        }
        if (aL0 < 0 && aR0 < 0) aR0 = aR1 = -1;
        add(aL0, aL1);
        add(aR0, aR1);
        if (klim < n_fin && klim <= L1_hi) add(bin_of_rank(klim - 1), bin_of_rank(klim));  // C's exact end
        // (the bins of the top-p crossing, the draw and the candidate list follow once the
        // run is exact: the typical pre-pass of the resolve kernel and a second gather)
        LargeRow* Hw = W.hdr;
        Hw->cc_lo = c0;
        Hw->cc_hi = c1;
        Hw->s_lo = s_lo;
        Hw->s_hi = s_hi;
        Hw->aL0 = aL0;
        Hw->aL1 = aL1;
        Hw->aR0 = aR0;
        Hw->aR1 = aR1;
        Hw->iB0 = iB0;
        Hw->iB1 = iB1;
      }
    }
    if (typ_mode != kTypCut) {
    double ct_lo = INFINITY, ct_hi = -INFINITY;
    bool tp_sure = false;
    int tp_hi = -1;
    if (tpe < 1 && n_fin > 0) {
      const double t = tpe;
      const int b0 = bstart(t);
      if (b0 < kNB && cnt[b0] < L1_hi) {
        tp_hi = b0;
        for (int ext = 0; ext < 4 && t >= P(tp_hi + 1) - kSelMargin * t; ++ext) {
          if (static_cast<int64_t>(cnt[tp_hi + 1]) >= n_fin) break;
          const int nb = bin_of_rank(cnt[tp_hi + 1]);
          if (cnt[nb] >= L1_hi || !fits(b0, nb)) break;
          tp_hi = nb;
        }
        add(b0, tp_hi);
        ct_lo = P(b0);
        ct_hi = P(tp_hi + 1);
        tp_sure = cnt[tp_hi + 1] <= L1_lo && t < P(tp_hi + 1) - kSelMargin * t;
      }
    }
    if (!tp_sure && n_fin > 0) {
      // L = L1: C(L) is the running sum through rank L1 - 1; from n_fin on it is the
      // binned total of every finite candidate
      if (L1_hi >= n_fin) {
        ct_lo = fmin(ct_lo, P(kNB));
        ct_hi = fmax(ct_hi, P(kNB));
      }
      const int64_t r_hi = (L1_hi < n_fin ? L1_hi : n_fin - 1) - 1;
      if (L1_lo >= 1 && L1_lo - 1 <= r_hi) {
        const int rl = bin_of_rank(L1_lo - 1), rh = bin_of_rank(r_hi);
        add(rl, rh);
        ct_lo = fmin(ct_lo, P(rl));
        ct_hi = fmax(ct_hi, P(rh + 1));
      }
    }
    // the draw: cursor = uniform · C(L) with C(L) in [ct_lo, ct_hi]
    if (ct_lo <= ct_hi && n_fin > 0) {
      const double u = W.hdr->uniform;
      auto clampb = [&](int b) { return b > last_bin ? last_bin : b; };
      const int e0 = clampb(bstart(u * ct_lo)), e1 = clampb(bstart(u * ct_hi));
      add(e0, e1);
      const int m0 = clampb(bstart(u * ct_lo * (1 - kSelMargin)));
      const int m1 = clampb(bstart(u * ct_hi * (1 + kSelMargin)));
      if (m0 < e0 && fits(m0, e0 - 1)) add(m0, e0 - 1);
      if (m1 > e1 && fits(e1 + 1, m1)) add(e1 + 1, m1);
    }
    // head of the candidate list (kept when it fits beside the bins above)
    if (A.cand_ids && A.cand_cap > 0 && n_fin > 0) {
      int64_t l_hi = L1_hi;
      if (tp_hi >= 0 && static_cast<int64_t>(cnt[tp_hi + 1]) > l_hi) l_hi = cnt[tp_hi + 1];
      if (tp_sure) l_hi = cnt[tp_hi + 1];
      int64_t m = A.cand_cap;
      if (m > n_fin) m = n_fin;
      if (m > l_hi) m = l_hi;
      if (m > 0) cb = bin_of_rank(m - 1);
    }
    }
    W.hdr->typ = typ_mode;
    s_nr = nr;
    s_cb0 = cb0;
    s_cb = cb;
    if (xflags) {
      s_flags |= xflags;
      W.hdr->flags = s_flags;
    }
    W.hdr->mp_lo = mp_lo;
    W.hdr->mp_hi = mp_hi;
    W.hdr->n_fin = static_cast<int32_t>(n_fin);
  }
  __syncthreads();
  // bitmap of the selected bins and its entry count; the candidate range goes in last,
  // and only when the total stays within the gather capacity
  const int nr = s_nr;
  // the bits of bins [a, b] within word w
  auto word_bits = [](int w, int a, int b) -> uint32_t {
    const int lo = a > w * 32 ? a : w * 32, hi = b < w * 32 + 31 ? b : w * 32 + 31;
    if (lo > hi) return 0u;
    return static_cast<uint32_t>(((1ull << (hi - lo + 1)) - 1ull) << (lo - w * 32));
  };
  auto mark = [&](bool with_cand) {
    int cntsel = 0;
    for (int w = tid; w < kNB / 32; w += bs) {
      uint32_t m = 0;
      for (int r = 0; r < nr; ++r) m |= word_bits(w, s_rng[0][r], s_rng[1][r]);
      if (with_cand && s_cb >= 0) m |= word_bits(w, s_cb0, s_cb);
      W.sel[w] = m;
      W.sel2[w] = 0u;
      for (uint32_t t = m; t; t &= t - 1u) {
        const int bin = w * 32 + __ffs(t) - 1;
        cntsel += static_cast<int>(cnt[bin + 1] - cnt[bin]);
      }
    }
    return block_sum_i(cntsel, red_i);
  };
  int need = mark(true);
  bool with_cand = true;
  if (need > kGCap && s_cb >= 0) {
    need = mark(false);
    with_cand = false;
  }
  if (tid == 0) {
    // the deepest selected bin bounds what the gather pass must soft-cap and bin (one bin
    // of slack for the binning's rounding)
    int bhi = with_cand ? s_cb : -1;
    for (int r = 0; r < nr; ++r) bhi = s_rng[1][r] > bhi ? s_rng[1][r] : bhi;
    W.hdr->gat_lo = bhi >= 0 && bhi < kNB - 2 ? raw_below(Mx - static_cast<float>(bhi + 2) * width, cap, inv_cap)
                                              : -INFINITY;
    W.hdr->g_need = need;
    if (need > kGCap) W.hdr->flags = s_flags | GS_FLAG_ERR_UNSUPPORTED;  // crossing bins beyond the gather capacity
  }
}

// ============================================================================ gather
// second: the typical pre-pass's bins (W.sel2), appended after the first gather's entries.
template <int DT>
__global__ void __launch_bounds__(kGatherThreads) large_gather_kernel(const __grid_constant__ FinalizeArgs A, int parts,
                                                                      int second) {
  constexpr int kParkVals = DT == GS_DTYPE_F32 ? 16 : 32;  // values a thread holds per step
  __shared__ uint32_t sel[kNB / 32];
  __shared__ uint32_t live[kGatherIds / 32];
  __shared__ float park[kParkVals][kGatherThreads];
  const int row = blockIdx.x / parts, part = blockIdx.x % parts;
  const int tid = threadIdx.x, bs = blockDim.x, lane = tid & 31;
  const RowPlan* pp = A.plans ? A.plans + row : &A.plan0;
  if (pp->mode != kModeLarge) return;
  const RowWs W = row_ws(A, row);
  LargeRow* Hp = W.hdr;
  if ((Hp->flags & GS_FLAG_ERRORS) || (second ? Hp->g_need2 : Hp->g_need) == 0) return;
  const int64_t V = A.vocab;
  const int64_t lo = static_cast<int64_t>(part) * kGatherIds;
  if (lo >= V) return;
  const int n = static_cast<int>(V - lo < kGatherIds ? V - lo : kGatherIds);
  const float Mx = Hp->Mx, scale = Hp->bscale, glo = second ? Hp->gat_lo2 : Hp->gat_lo;
  const int32_t state = A.mask_state ? A.mask_state[row] : -1;
  const bool has_mask = A.mask_table != nullptr && state >= 0 && state < A.mask_states;
  const uint32_t* mrow = has_mask ? A.mask_table + static_cast<int64_t>(state) * A.mask_words : nullptr;
  constexpr int ESZ = DT == GS_DTYPE_F32 ? 4 : 2;
  constexpr int VE = 16 / ESZ;
  const unsigned char* base =
      static_cast<const unsigned char*>(A.logits) + (static_cast<int64_t>(row) * A.row_stride + lo) * ESZ;
  const float cap = A.softcap, inv_cap = A.inv_softcap;
  int64_t hl = A.history_len ? A.history_len[row] : 0;
  if (hl > A.history_stride) hl = A.history_stride;
  if (hl < 0) hl = 0;
  const int32_t* hrow = A.history + static_cast<int64_t>(row) * A.history_stride;
  const uint32_t* wsel = second ? W.sel2 : W.sel;
  for (int w = tid; w < kNB / 32; w += bs) sel[w] = wsel[w];
  build_live(live, mrow, lo, n, hrow, hl, tid, bs);
  const unsigned lane_lt = (1u << lane) - 1u;
  auto wanted = [&](float x) {
    if (!(x > -INFINITY)) return false;
    const int b = bin_of(x, Mx, scale);
    return ((sel[b >> 5] >> (b & 31)) & 1u) != 0;
  };
  // Appends (x, id) for the lanes whose `take` is set (the whole warp calls).
  auto append = [&](bool take, float x, uint32_t id) {
    const unsigned bal = __ballot_sync(kFullMask, take);
    if (!bal) return;
    const int leader = __ffs(bal) - 1;
    int at = 0;
    if (lane == leader) at = atomicAdd(&Hp->g_count, __popc(bal));
    at = __shfl_sync(kFullMask, at, leader) + __popc(bal & lane_lt);
    if (take && at < kGCap) W.gath[at] = make_uint2(__float_as_uint(x), id);
  };
  int done = 0;
  if ((reinterpret_cast<uintptr_t>(base) & 15) == 0) {
    const int nv = n / VE;
    const uint4* v4 = reinterpret_cast<const uint4*>(base);
    for (int v0 = 0; v0 < nv; v0 += 4 * bs) {  // trip count uniform over the CTA
      // Four vectors per thread in flight.  The values that can reach a selected bin
      // (live, raw >= glo: a few percent) are parked in shared memory and then taken one
      // per lane per round, so that the warp soft-caps and bins only those.
      uint32_t pm = 0;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int vi = v0 + u * bs + tid;
        const uint32_t bits = vi < nv ? (live[(vi * VE) >> 5] >> ((vi * VE) & 31)) & ((1u << VE) - 1u) : 0u;
        uint4 r = make_uint4(0u, 0u, 0u, 0u);
        if (bits) r = ld_stream_u4(v4 + vi);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < VE; ++i) {
          const float x = DT == GS_DTYPE_F32 ? __uint_as_float(w[i & 3]) : ((i & 1) ? bf16_hi(w[i >> 1]) : bf16_lo(w[i >> 1]));
          park[u * VE + i][tid] = x;
          if (((bits >> i) & 1u) && x >= glo) pm |= 1u << (u * VE + i);
        }
      }
      while (__any_sync(kFullMask, pm != 0)) {
        const bool has = pm != 0;
        const int k = has ? __ffs(pm) - 1 : 0;
        pm &= pm - 1u;
        float x = 0.0f;
        bool take = false;
        if (has) {
          x = park[k][tid];
          if (cap != 0.0f) x = softcap(x, cap, inv_cap);
          take = wanted(x);
        }
        append(take, x, static_cast<uint32_t>(lo + (v0 + (k / VE) * bs + tid) * VE + (k % VE)));
      }
    }
    done = nv * VE;
  }
  for (int i0 = done; i0 < n; i0 += bs) {  // (trip count uniform over the CTA)
    const int i = i0 + tid;
    bool take = false;
    float x = 0.0f;
    if (i < n && ((live[i >> 5] >> (i & 31)) & 1u)) {
      x = load_logit(base, DT, i);
      if (x >= glo) {
        if (cap != 0.0f) x = softcap(x, cap, inv_cap);
        take = wanted(x);
      }
    }
    append(take, x, static_cast<uint32_t>(lo + i));
  }
}

// ============================================================================ resolve
// PH 0: the typical pre-pass (typical-p rows with an annulus cut only): the exact run and
// the bins of its second gather.  PH 1: the crossings, the draw and the outputs.
template <int DT, int PH>
__global__ void __launch_bounds__(kResolveThreads) large_resolve_kernel(const __grid_constant__ FinalizeArgs A) {
  extern __shared__ __align__(16) unsigned char dsm[];
  Ent* E = reinterpret_cast<Ent*>(dsm);               // [kGCap] selected bins, bin by bin
  double* gp = reinterpret_cast<double*>(E + kGCap);  // [kGCap] exact probabilities
  int* seg = reinterpret_cast<int*>(gp + kGCap);      // [kNB + 1] start of each bin in E
  unsigned long long* tsort = reinterpret_cast<unsigned long long*>(seg + kNB + 4);  // [kSortSmem] typical-p
  __shared__ uint32_t sel[kNB / 32];
  __shared__ double red_d[32];
  __shared__ int s_ti[4];
  __shared__ uint32_t nesel[kNB / 32];  // selected and non-empty
  __shared__ unsigned s_flags;
  __shared__ int red_i[32];
  __shared__ int s_nl;
  __shared__ long long s_res[2];
  __shared__ double s_resd[3];
  const int row = blockIdx.x, tid = threadIdx.x, bs = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nwarps = bs >> 5;
  const RowPlan* pp = A.plans ? A.plans + row : &A.plan0;
  if (pp->mode != kModeLarge) return;
  const RowWs W = row_ws(A, row);
  const LargeRow H = *W.hdr;
  if (PH == 0 && (H.typ != kTypCut || (H.flags & GS_FLAG_ERRORS))) return;
  const double T = pp->temperature, M = H.M, total = H.total;
  const float Mx = H.Mx, scale = H.bscale;
  const int64_t V = A.vocab;
  const int32_t state = A.mask_state ? A.mask_state[row] : -1;
  const bool has_mask = A.mask_table != nullptr && state >= 0 && state < A.mask_states;
  const uint32_t* mrow = has_mask ? A.mask_table + static_cast<int64_t>(state) * A.mask_words : nullptr;
  const unsigned char* rowbase =
      static_cast<const unsigned char*>(A.logits) + static_cast<int64_t>(row) * A.row_stride * (DT == GS_DTYPE_F32 ? 4 : 2);
  const float cap = A.softcap, inv_cap = A.inv_softcap;
  if (tid == 0) s_flags = H.flags;
  __syncthreads();
  const uint32_t* C = W.cpre;
  const double* P = W.ppre;
  auto selected = [&](int b) { return ((sel[b >> 5] >> (b & 31)) & 1u) != 0; };

  uint32_t tok = 0xffffffffu;
  int64_t L = 0, R0 = 0;  // the final candidates: ranks [R0, L)
  const int64_t n_fin = H.n_fin;
  if (!(H.flags & GS_FLAG_ERRORS)) {
    // ---- place the selected bins' entries: bin b occupies E[seg[b], seg[b + 1]) ----
    for (int w = tid; w < kNB / 32; w += bs) sel[w] = PH == 0 ? W.sel[w] : (W.sel[w] | W.sel2[w]);
    __syncthreads();
    {
      constexpr int kPer = kNB / kResolveThreads;
      int c[kPer];
      int tcount = 0;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int b = tid * kPer + i;
        c[i] = selected(b) ? static_cast<int>(C[b + 1] - C[b]) : 0;
        tcount += c[i];
      }
      int inc = tcount;
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(kFullMask, inc, o);
        if (lane >= o) inc += u;
      }
      if (lane == 31) red_i[warp] = inc;
      __syncthreads();
      int bsum = inc - tcount;
      for (int w = 0; w < warp; ++w) bsum += red_i[w];
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        seg[tid * kPer + i] = bsum;
        bsum += c[i];
      }
      if (tid == bs - 1) seg[kNB] = bsum;
      __syncthreads();
    }
    const int n_tot = seg[kNB];
    for (int w = tid; w < kNB / 32; w += bs) {
      uint32_t m = 0;
      for (int i = 0; i < 32; ++i)
        if (seg[w * 32 + i + 1] > seg[w * 32 + i]) m |= 1u << i;
      nesel[w] = m;
    }
    int* cur = reinterpret_cast<int*>(gp);  // fill counters during placement
    for (int b = tid; b < kNB; b += bs) cur[b] = 0;
    __syncthreads();
    int bad = n_tot > kGCap ? 1 : 0;
    if (!bad) {
      const int gn = H.g_count < kGCap ? H.g_count : kGCap;
      for (int i = tid; i < gn; i += bs) {
        const uint2 g = W.gath[i];
        const float x = __uint_as_float(g.x);
        const int b = bin_of(x, Mx, scale);
        const int pos = selected(b) ? seg[b] + atomicAdd(&cur[b], 1) : INT_MAX;
        if (pos < seg[b + 1]) E[pos] = Ent{__ddiv_rn(static_cast<double>(x), T), g.y, 0u};
        else bad = 1;
      }
      for (int j = tid; j < H.n_slots; j += bs) {
        const Ent e = W.pen[j];
        if (e.id == 0xffffffffu || !(e.key > -INFINITY)) continue;
        const int b = bin_of(__uint_as_float(e.kind), Mx, scale);
        if (!selected(b)) continue;
        const int pos = seg[b] + atomicAdd(&cur[b], 1);
        if (pos < seg[b + 1]) E[pos] = Ent{e.key, e.id, 1u};
        else bad = 1;
      }
    }
    __syncthreads();
    if (!bad)
      for (int b = tid; b < kNB; b += bs)
        if (cur[b] != seg[b + 1] - seg[b]) bad = 1;
    if (__syncthreads_or(bad)) {
      if (tid == 0) s_flags |= GS_FLAG_ERR_UNSUPPORTED;  // list overflowed (more than kGCap entries)
    } else {
      // list of the selected bins with more than one entry, then one warp per bin sorts it
      int* lst = cur;
      if (tid == 0) s_nl = 0;
      __syncthreads();
      for (int b = tid; b < kNB; b += bs)
        if (seg[b + 1] - seg[b] > 1) lst[atomicAdd(&s_nl, 1)] = b;
      __syncthreads();
      const int nl = s_nl;
      for (int q = warp; q < nl; q += nwarps) {
        const int b = lst[q];
        const int off = seg[b], nb = seg[b + 1] - off;
        if (nb <= kWarpSortMax) seg_sort<false>(E + off, nb, lane, 32);
      }
      __syncthreads();
      for (int q = 0; q < nl; ++q) {
        const int b = lst[q];
        const int off = seg[b], nb = seg[b + 1] - off;
        if (nb > kWarpSortMax) seg_sort<true>(E + off, nb, tid, bs);
      }
      __syncthreads();
      for (int i = tid; i < n_tot; i += bs) gp[i] = __ddiv_rn(exp(__dsub_rn(E[i].key, M)), total);
      __syncthreads();
    }
  }

  // first bin b with P(b + 1) >= t (kNB if none), all threads
  auto bstart = [&](double t) {
    int c = kNB;
    for (int b = tid; b < kNB; b += bs)
      if (P[b + 1] >= t) c = min(c, b);
    return block_min_i(c, red_i);
  };
  // the bin holding rank r, all threads
  auto bin_of_rank = [&](int64_t r) {
    int c = kNB - 1;
    for (int b = tid; b < kNB; b += bs)
      if (static_cast<int64_t>(C[b + 1]) > r) c = min(c, b);
    return block_min_i(c, red_i);
  };
  // First rank j < limit whose running probability reaches `target` (-1 if none),
  // walking the selected bins from the binned prefix at each bin's start (the
  // reference's running sums, sampling.ts:58-64 and :82-90).  s_resd[0..1] get the
  // running sums through j and j - 1.
  auto locate = [&](double target, int64_t limit) -> int64_t {
    int b = bstart(target);
    if (warp == 0) {  // one warp: a scan of 32 probabilities per step
      long long found = -1;
      double c_at = 0.0, c_prev = 0.0;
      int tries = 0;
      bool fail = false;
      while (b < kNB) {
        if (static_cast<int64_t>(C[b]) >= limit) break;
        const int nb = static_cast<int>(C[b + 1] - C[b]);
        if (nb > 0) {
          if (++tries > 4 || !selected(b)) {
            fail = true;
            break;
          }
          const int off = seg[b];
          const int64_t room = limit - static_cast<int64_t>(C[b]);
          const int nl = nb < room ? nb : static_cast<int>(room);
          double c = P[b];
          for (int i0 = 0; i0 < nl; i0 += 32) {
            const int i = i0 + lane;
            double v = i < nl ? gp[off + i] : 0.0;
            for (int o = 1; o < 32; o <<= 1) {
              const double t = __shfl_up_sync(kFullMask, v, o);
              if (lane >= o) v = __dadd_rn(t, v);
            }
            const double cl = __dadd_rn(c, v);
            const unsigned hit = __ballot_sync(kFullMask, i < nl && cl >= target);
            if (hit) {
              const int f = __ffs(hit) - 1;
              found = static_cast<long long>(C[b]) + i0 + f;
              c_at = __shfl_sync(kFullMask, cl, f);
              const double pv = __shfl_sync(kFullMask, cl, f > 0 ? f - 1 : 0);
              c_prev = f > 0 ? pv : c;
              break;
            }
            c = __shfl_sync(kFullMask, cl, 31);
          }
          if (found >= 0) break;
        }
        // next bin: the next selected non-empty one, unless an unselected non-empty bin
        // comes first
        if (static_cast<int64_t>(C[b + 1]) >= n_fin) break;
        int nbn = kNB;
        for (int w = (b + 1) >> 5; w < kNB / 32; ++w) {
          uint32_t m = nesel[w];
          if (w == ((b + 1) >> 5)) m &= ~((1u << ((b + 1) & 31)) - 1u);
          if (m) {
            nbn = w * 32 + __ffs(m) - 1;
            break;
          }
        }
        if (nbn >= kNB || C[nbn] != C[b + 1]) {
          // the walk would enter a bin that was not gathered
          if (static_cast<int64_t>(C[b + 1]) < limit) fail = true;
          break;
        }
        b = nbn;
      }
      if (lane == 0) {
        if (fail) s_flags |= GS_FLAG_BOUNDARY_DRAW;
        s_res[0] = found;
        s_resd[0] = c_at;
        s_resd[1] = c_prev;
      }
    }
    __syncthreads();
    const int64_t r = s_res[0];
    __syncthreads();
    return r;
  };

  // Sums over the gathered entries of bin b with ranks in [C[b], r): of p (returned) and of
  // p·(M - key) (*m1).  All threads.
  auto bin_part = [&](int b, int64_t r, double* m1) -> double {
    const int off = seg[b], n = static_cast<int>(r - C[b]);
    double sp = 0.0, sq = 0.0;
    for (int i = tid; i < n; i += bs) {
      sp = __dadd_rn(sp, gp[off + i]);
      sq = __dadd_rn(sq, __dmul_rn(gp[off + i], __dsub_rn(M, E[off + i].key)));
    }
    sp = block_sum_d(sp, red_d);
    if (m1) *m1 = block_sum_d(sq, red_d);
    return sp;
  };
  // Running probability before rank r, -1 when r's bin was not gathered.  All threads.
  auto prefix_at = [&](int64_t r) -> double {
    if (r >= n_fin) return P[kNB];
    const int b = bin_of_rank(r);
    if (r == static_cast<int64_t>(C[b])) return P[b];
    if (!selected(b)) return -1.0;
    return __dadd_rn(P[b], bin_part(b, r, nullptr));
  };
  // typical-p (sampling.ts:49-55) over the candidates [0, L1): the entropy H from the
  // binned first moments and the exact entries of L1's bin, the surprise |delta - cc| of
  // every entry of the two end ranges (cc = H - ln total).  Entries below the select
  // kernel's bound s_lo are kept whatever the order, entries above s_hi never are; those
  // between are sorted by surprise with the rank as the tie break (the reference's stable
  // sort), and the running sum continues from the mass of everything below s_lo until it
  // reaches typicalP.  The set is the ranks [*r0, *lend); *c0 is the running probability
  // before *r0.  A result outside the select kernel's bounds is reported as unsupported.
  // All threads.
  auto typical_cut = [&](int64_t L1, int64_t* r0, int64_t* lend, double* c0) {
    const double tq = pp->typical_p;
    const double lnZ = log(total);
    const double* Q = W.m1pre;
    auto fail = [&]() {
      if (tid == 0) s_flags |= GS_FLAG_ERR_UNSUPPORTED;
    };
    double pc, qc, out;  // P_C, sum_C p·delta, 1 - P_C
    if (L1 < n_fin) {
      const int b1 = bin_of_rank(L1);
      if (L1 == static_cast<int64_t>(C[b1])) {
        pc = P[b1];
        qc = __ddiv_rn(Q[b1], total);
        out = __dsub_rn(P[kNB], P[b1]);
      } else {
        if (!selected(b1)) return fail();
        double q1 = 0.0;
        const double p1 = bin_part(b1, L1, &q1);
        const double pb = bin_part(b1, C[b1 + 1], nullptr);
        pc = __dadd_rn(P[b1], p1);
        qc = __dadd_rn(__ddiv_rn(Q[b1], total), q1);
        out = __dadd_rn(__dsub_rn(P[kNB], P[b1 + 1]), __dsub_rn(pb, p1));
      }
    } else {
      pc = P[kNB];
      qc = __ddiv_rn(Q[kNB], total);
      out = 0.0;
    }
    const double cc = __dsub_rn(qc, __dmul_rn(lnZ, out));
    if (!(cc >= H.cc_lo && cc <= H.cc_hi)) return fail();
    // the end ranges must have been gathered
    int bad = 0;
    for (int b = tid; b < kNB; b += bs) {
      const bool in_end = (H.aL0 >= 0 && b >= H.aL0 && b <= H.aL1) || (H.aR0 >= 0 && b >= H.aR0 && b <= H.aR1);
      if (in_end && !selected(b) && C[b + 1] > C[b]) bad = 1;
    }
    if (__syncthreads_or(bad)) return fail();
    auto range_n = [&](int a0, int a1) -> int {  // entries of bins [a0, a1] with rank < L1
      if (a0 < 0) return 0;
      const int64_t e = static_cast<int64_t>(C[a1 + 1]) < L1 ? static_cast<int64_t>(C[a1 + 1]) : L1;
      return e > static_cast<int64_t>(C[a0]) ? static_cast<int>(e - C[a0]) : 0;
    };
    const int nL = range_n(H.aL0, H.aL1), nR = range_n(H.aR0, H.aR1), nA = nL + nR;
    const int eL = H.aL0 >= 0 ? seg[H.aL0] : 0, eR = H.aR0 >= 0 ? seg[H.aR0] : 0;
    int64_t iL = 0, iR = 0;  // inner ranks (surprise below s_lo)
    double mbase = 0.0;
    if (H.iB0 >= 0) {
      iL = C[H.iB0];
      iR = static_cast<int64_t>(C[H.iB1 + 1]) < L1 ? static_cast<int64_t>(C[H.iB1 + 1]) : L1;
      if (iR > iL) mbase = __dsub_rn(iR == static_cast<int64_t>(C[H.iB1 + 1]) ? P[H.iB1 + 1] : pc, P[H.iB0]);
      else iR = iL;
    }
    auto surprise = [&](int e) { return fabs(__dsub_rn(__dsub_rn(M, E[e].key), cc)); };
    // split the end ranges' entries at s_lo and s_hi; the band's sort keys: the surprise's
    // bits above the low 13 (a tie break 2^-39 relative) and the entry's position, which
    // follows the rank
    if (tid == 0) s_ti[1] = 0;
    __syncthreads();
    double mb = 0.0, s_below = -1.0;
    int n_below = 0, n_above = 0, emin = INT_MAX, emax = -1;  // (positions are >= 0)
    for (int i = tid; i < nA; i += bs) {
      const int e = i < nL ? eL + i : eR + (i - nL);
      const double sv = surprise(e);
      if (sv < H.s_lo) {
        mb = __dadd_rn(mb, gp[e]);
        s_below = fmax(s_below, sv);
        ++n_below;
        emin = min(emin, e);
        emax = max(emax, e);
      } else if (sv <= H.s_hi) {
        const int at = atomicAdd(&s_ti[1], 1);
        if (at < kSortSmem)
          tsort[at] = (static_cast<unsigned long long>(__double_as_longlong(sv)) & ~0x1fffull) |
                      static_cast<unsigned long long>(e);
      } else {
        ++n_above;
      }
    }
    mbase = __dadd_rn(mbase, block_sum_d(mb, red_d));
    s_below = block_max_d(s_below, red_d);
    n_below = block_sum_i(n_below, red_i);
    n_above = block_sum_i(n_above, red_i);
    const int nB = s_ti[1];
    if (nB > kSortSmem || mbase >= tq) return fail();
    const int n2 = pow2_ceil(nB > 0 ? nB : 1);
    for (int i = nB + tid; i < n2; i += bs) tsort[i] = ~0ull;
    __syncthreads();
    bitonic_sort_u64(tsort, n2);
    if (warp == 0) {
      double c = mbase, c_at = 0.0, c_prev = 0.0;
      int found = -1;
      for (int i0 = 0; i0 < nB; i0 += 32) {
        const int i = i0 + lane;
        double v = i < nB ? gp[static_cast<int>(tsort[i] & 0x1fffull)] : 0.0;
        for (int o = 1; o < 32; o <<= 1) {
          const double t = __shfl_up_sync(kFullMask, v, o);
          if (lane >= o) v = __dadd_rn(t, v);
        }
        const double cl = __dadd_rn(c, v);
        const unsigned hit = __ballot_sync(kFullMask, i < nB && cl >= tq);
        if (hit) {
          const int f = __ffs(hit) - 1;
          found = i0 + f;
          c_at = __shfl_sync(kFullMask, cl, f);
          const double pv = __shfl_sync(kFullMask, cl, f > 0 ? f - 1 : 0);
          c_prev = f > 0 ? pv : c;
          break;
        }
        c = __shfl_sync(kFullMask, cl, 31);
      }
      if (lane == 0) {
        s_ti[0] = found;
        s_resd[0] = c_at;
        s_resd[1] = c_prev;
      }
    }
    __syncthreads();
    const int found = s_ti[0];
    const int kept = found >= 0 ? found + 1 : nB;
    if (found >= 0) {
      if (tid == 0) {
        // near ties at the cut: the running sum, and the surprise against the neighbours
        // in the order (the next band entry or an entry above s_hi; the last entry below s_lo)
        const double sx = surprise(static_cast<int>(tsort[found] & 0x1fffull));
        const double tol = kBoundary * fmax(sx, 1.0);
        double m = fmin(fabs(s_resd[0] - tq), fabs(s_resd[1] - tq));
        bool near = m <= kBoundary * tq || (n_below > 0 && sx - s_below <= tol);
        if (found + 1 < nB) near = near || surprise(static_cast<int>(tsort[found + 1] & 0x1fffull)) - sx <= tol;
        else near = near || H.s_hi - sx <= tol;
        if (near) s_flags |= GS_FLAG_BOUNDARY_TYPICAL;
      }
    } else if (n_above > 0) {
      return fail();  // the running sum stays below typicalP through s_hi
    }
    // the run: the inner ranks, the entries below s_lo and the kept band entries
    for (int i = tid; i < kept; i += bs) {
      const int e = static_cast<int>(tsort[i] & 0x1fffull);
      emin = min(emin, e);
      emax = max(emax, e);
    }
    emin = block_min_i(emin, red_i);
    emax = -block_min_i(-emax, red_i);
    auto rank_of = [&](int e) -> int64_t {
      return (H.aR0 >= 0 && e >= eR) ? static_cast<int64_t>(C[H.aR0]) + (e - eR) : static_cast<int64_t>(C[H.aL0]) + (e - eL);
    };
    int64_t rl = INT64_MAX, rr = -1;
    if (iR > iL) {
      rl = iL;
      rr = iR - 1;
    }
    if (n_below + kept > 0) {
      const int64_t a = rank_of(emin), b = rank_of(emax);
      rl = rl < a ? rl : a;
      rr = rr > b ? rr : b;
    }
    if (rr < rl || rr - rl + 1 != (iR - iL) + n_below + kept) return fail();
    if (found < 0 && !(rl == 0 && rr + 1 == L1)) return fail();  // every candidate stays: all of [0, L1)
    const double pl = prefix_at(rl);
    if (pl < 0) return fail();
    *r0 = rl;
    *lend = rr + 1;
    *c0 = pl;
  };
  // Typical pre-pass: with the run [r0, lend) exact, the bins of the top-p crossing, the
  // draw, the run's last rank and the head of the candidate list that the first gather
  // did not take become W.sel2, for the second gather.  All threads.
  auto typical_bins = [&](int64_t r0, int64_t lend, double c0) {
    const double cend = prefix_at(lend);
    if (cend < 0) {
      if (tid == 0) s_flags |= GS_FLAG_ERR_UNSUPPORTED;
      return;
    }
    int ra[4], rb[4];
    int nr = 0;
    auto addr = [&](int a, int b) {
      if (nr < 4 && a <= b) {
        ra[nr] = a;
        rb[nr] = b;
        ++nr;
      }
    };
    const int blast = bin_of_rank(lend - 1);
    addr(blast, blast);
    double e_lo = cend, e_hi = cend;  // C(L): the running sum through the last candidate
    if (pp->top_p < 1) {
      const double t = __dadd_rn(c0, pp->top_p);
      if (t * (1 - kSelMargin) <= cend) {
        const int b0 = min(bstart(t * (1 - kSelMargin)), blast), b1 = min(bstart(t * (1 + kSelMargin)), blast);
        addr(b0, b1);
        e_lo = fmin(cend, P[b0]);
        e_hi = fmin(cend, P[b1 + 1]);
      }
    }
    const double u = H.uniform;
    const double y_lo = c0 + u * (e_lo - c0), y_hi = c0 + u * (e_hi - c0);
    addr(min(bstart(y_lo * (1 - kSelMargin)), blast), min(bstart(y_hi * (1 + kSelMargin)), blast));
    int cb0 = -1, cb1 = -1;
    if (A.cand_ids && A.cand_cap > 0) {
      cb0 = bin_of_rank(r0);
      cb1 = bin_of_rank((lend - r0 < A.cand_cap ? lend : r0 + A.cand_cap) - 1);
    }
    auto build = [&](bool with_cand) -> int {
      int c = 0;
      for (int w = tid; w < kNB / 32; w += bs) {
        uint32_t m = 0;
        for (int i = 0; i < 32; ++i) {
          const int b = w * 32 + i;
          bool in = with_cand && b >= cb0 && b <= cb1;
          for (int r = 0; r < nr; ++r) in = in || (b >= ra[r] && b <= rb[r]);
          if (in && !((sel[w] >> i) & 1u) && C[b + 1] > C[b]) {
            m |= 1u << i;
            c += static_cast<int>(C[b + 1] - C[b]);
          }
        }
        W.sel2[w] = m;
      }
      return block_sum_i(c, red_i);
    };
    bool wc = cb0 >= 0;
    int need = build(wc);
    if (H.g_need + need > kGCap && wc) {
      wc = false;
      need = build(false);
    }
    if (tid == 0) {
      int bhi = wc ? cb1 : -1;
      for (int r = 0; r < nr; ++r) bhi = rb[r] > bhi ? rb[r] : bhi;
      LargeRow* Hw = W.hdr;
      Hw->t_r0 = r0;
      Hw->t_lend = lend;
      Hw->t_c0 = c0;
      Hw->g_need2 = need;
      Hw->gat_lo2 = bhi >= 0 && bhi < kNB - 2 ? raw_below(Mx - static_cast<float>(bhi + 2) * H.bwidth, cap, inv_cap)
                                            : -INFINITY;
      if (H.g_need + need > kGCap) s_flags |= GS_FLAG_ERR_UNSUPPORTED;  // beyond the gather capacity
    }
  };

  __syncthreads();
  if (!(s_flags & GS_FLAG_ERRORS)) {
    const int64_t K = pp->top_k;
    int64_t L1 = (K > 0 && K < V) ? K : V;
    // ---- min-p (sampling.ts:45-48): p_i >= p_0·minP, with p_0 = 1/total ----
    if (pp->min_p > 0) {
      const double theta = __dmul_rn(__ddiv_rn(1.0, total), pp->min_p);
      int kept = 0, near = 0;
      for (int b = H.mp_lo; b <= H.mp_hi; ++b) {
        const int off = seg[b], nb = seg[b + 1] - off;
        for (int i = tid; i < nb; i += bs) {
          kept += gp[off + i] >= theta ? 1 : 0;
          if (fabs(gp[off + i] - theta) <= kBoundary * theta) near = 1;
        }
      }
      kept = block_sum_i(kept, red_i);
      if (__syncthreads_or(near) && tid == 0) s_flags |= GS_FLAG_BOUNDARY_MIN_P;
      const int64_t Lm = static_cast<int64_t>(C[H.mp_lo]) + kept;
      L1 = L1 < Lm ? L1 : Lm;
    }
    // ---- typical-p (sampling.ts:49-55): the typical set is ranks [R0, Lend) ----
    int64_t Lend = L1;
    double C0 = 0.0;  // running probability before rank R0
    // (no annulus cut: either none, or the entropy is NaN and the cut is a running-sum cut)
    const double tpe = (pp->typical_p < 1 && H.typ == kTypNone) ? fmin(pp->top_p, pp->typical_p) : pp->top_p;
    if (PH == 0) {
      typical_cut(L1, &R0, &Lend, &C0);
      __syncthreads();
      if (!(s_flags & GS_FLAG_ERRORS)) typical_bins(R0, Lend, C0);
    } else if (H.typ == kTypCut) {
      R0 = H.t_r0;
      Lend = H.t_lend;
      C0 = H.t_c0;
    }
    __syncthreads();
    if (PH == 1) {
    // ---- top-p (sampling.ts:56) over [R0, Lend) ----
    L = Lend;
    if (tpe < 1 && !(s_flags & GS_FLAG_ERRORS)) {
      const double t = __dadd_rn(C0, tpe);
      const int64_t j = locate(t, Lend);
      if (j >= 0) {
        L = j + 1;
        if (tid == 0) {
          const double m = fmin(fabs(s_resd[0] - t), j > R0 ? fabs(s_resd[1] - t) : INFINITY);
          if (m <= kBoundary * tpe) s_flags |= GS_FLAG_BOUNDARY_TOP_P;
        }
      }
    }
    __syncthreads();
    // ---- candidate total C(L) and the last candidate ----
    double CT;
    uint32_t last_id = 0xffffffffu;
    bool last_known = true;
    if (L < n_fin) {
      const int b = bin_of_rank(L - 1);
      if (warp == 0) {
        if (!selected(b)) {
          if (lane == 0) {
            s_flags |= GS_FLAG_ERR_UNSUPPORTED;
            s_resd[2] = 0.0;
            s_res[1] = 0xffffffffll;
          }
        } else {
          const int i = static_cast<int>(L - 1 - C[b]), off = seg[b];
          double v = 0.0;
          for (int q = lane; q <= i; q += 32) v = __dadd_rn(v, gp[off + q]);
          v = warp_sum(v);
          if (lane == 0) {
            s_resd[2] = __dadd_rn(P[b], v);
            s_res[1] = E[off + i].id;
          }
        }
      }
      __syncthreads();
      CT = __dsub_rn(s_resd[2], C0);
      last_id = static_cast<uint32_t>(s_res[1]);
      __syncthreads();
    } else {
      // every finite candidate: the binned total (within the boundary tolerance of the
      // exact running sum); the -inf group adds nothing
      CT = __dsub_rn(P[kNB], C0);
      if (L == n_fin) {
        // the last finite candidate, needed only if the draw falls through
        last_known = false;
        if (n_fin > 0) {
          const int b = bin_of_rank(n_fin - 1);
          if (selected(b)) {
            last_id = E[seg[b + 1] - 1].id;
            last_known = true;
          }
        }
      }
    }
    // ---- draw (sampling.ts:58-64) ----
    if (!(s_flags & GS_FLAG_ERRORS)) {
      const double cursor = __dmul_rn(H.uniform, CT);
      const double target = __dadd_rn(C0, cursor);
      const int64_t lim = L < n_fin ? L : n_fin;
      const int64_t j = locate(target, lim);
      if (j >= 0) {
        const int b = bin_of_rank(j);
        tok = E[seg[b] + static_cast<int>(j - C[b])].id;
        if (tid == 0) {
          const double m = fmin(fabs(s_resd[0] - target), j > R0 ? fabs(s_resd[1] - target) : INFINITY);
          if (m <= kBoundary * CT) s_flags |= GS_FLAG_BOUNDARY_DRAW;
        }
      } else {
        if (tid == 0) s_flags |= GS_FLAG_FELL_THROUGH;
        if (!last_known) {
          if (tid == 0) s_flags |= GS_FLAG_ERR_UNSUPPORTED;  // the last candidate's bin was not gathered
        } else if (last_id != 0xffffffffu) {
          tok = last_id;
        } else {
          // the (L - 1 - n_fin)-th id, in ascending order, of the ids whose key is -inf
          const int64_t want = L - 1 - n_fin;
          if (tid == 0) s_res[1] = 0;
          __syncthreads();
          int64_t base = 0;
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
            if (lane == 0) red_i[warp] = __popc(bal);
            __syncthreads();
            int64_t before = base;
            for (int w = 0; w < warp; ++w) before += red_i[w];
            before += __popc(bal & ((1u << lane) - 1u));
            if (neg && before == want) s_res[1] = id;
            int sum = 0;
            for (int w = 0; w < nwarps; ++w) sum += red_i[w];
            __syncthreads();
            base += sum;
            if (base > want) break;
          }
          __syncthreads();
          tok = static_cast<uint32_t>(s_res[1]);
        }
      }
    }
    }
    __syncthreads();
  }
  if (PH == 0) {
    if (tid == 0) W.hdr->flags = s_flags;
    return;
  }

  // ---- outputs ----
  const unsigned fl = s_flags;
  const bool err = (fl & GS_FLAG_ERRORS) != 0;
  if (tid == 0) {
    A.ids[row] = err ? -1 : static_cast<int32_t>(tok);
    if (A.flags) A.flags[row] = fl;
    if (A.cand_count) A.cand_count[row] = err ? 0 : static_cast<int32_t>(L - R0);
    if (!err && !A.uniforms && A.rng_state) A.rng_state[row] = H.rng_next;
    if (A.logprob) {
      double lp = NAN;
      if (!err) {
        float x = load_logit(rowbase, DT, tok);
        if (cap != 0.0f) x = softcap(x, cap, inv_cap);
        lp = __dsub_rn(__dsub_rn(static_cast<double>(x), static_cast<double>(H.raw_m)), log(H.raw_s));
      }
      A.logprob[row] = lp;
    }
  }
  if (A.cand_ids) {
    // the first min(L - R0, cand_cap) candidates in order, when their bins were gathered
    int64_t m = err ? 0 : (L - R0 < A.cand_cap ? L - R0 : A.cand_cap);
    if (m > n_fin - R0) m = n_fin - R0;
    int nw = 0, e0 = 0;
    if (m > 0) {
      const int b0 = bin_of_rank(R0), b1 = bin_of_rank(R0 + m - 1);
      if (seg[b1 + 1] - seg[b0] == static_cast<int>(C[b1 + 1] - C[b0])) {  // bins b0..b1 all gathered
        nw = static_cast<int>(m);
        e0 = seg[b0] + static_cast<int>(R0 - C[b0]);
      }
    }
    for (int i = tid; i < A.cand_cap; i += bs) {
      A.cand_ids[static_cast<int64_t>(row) * A.cand_cap + i] = i < nw ? static_cast<int32_t>(E[e0 + i].id) : -1;
      if (A.cand_probs) A.cand_probs[static_cast<int64_t>(row) * A.cand_cap + i] = i < nw ? gp[e0 + i] : 0.0;
    }
  }
}

namespace {

template <class Kern>
void set_smem(Kern k, size_t bytes) {
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
}

template <int DT>
cudaError_t launch_large_t(const FinalizeArgs& a, int rows, size_t select_smem, cudaStream_t st) {
  const size_t res_smem = large_resolve_smem_bytes();
  static std::atomic<uint64_t> attr{0};  // (set on each device's first call)
  if (device_todo(attr)) {
    set_smem(large_select_kernel<DT>, large_select_smem_bytes(GS_MAX_HISTORY));
    set_smem(large_resolve_kernel<DT, 0>, res_smem);
    set_smem(large_resolve_kernel<DT, 1>, res_smem);
    const size_t q = static_cast<size_t>(kHistQueue) * sizeof(float), qm = q + static_cast<size_t>(kNB) * 4;
    const size_t m = static_cast<size_t>(kNB) * 4;
    set_smem(large_hist_kernel<DT, false, false, kHistThreads>, q);
    set_smem(large_hist_kernel<DT, true, false, kHistThreads>, q);
    set_smem(large_hist_kernel<DT, false, true, kHistThreads>, qm);
    set_smem(large_hist_kernel<DT, true, true, kHistThreads>, qm);
    set_smem(large_hist_kernel<DT, false, false, kHistThreads / 2>, 0);
    set_smem(large_hist_kernel<DT, true, false, kHistThreads / 2>, 0);
    set_smem(large_hist_kernel<DT, false, true, kHistThreads / 2>, m);
    set_smem(large_hist_kernel<DT, true, true, kHistThreads / 2>, m);
    mark_device_done(attr);
  }
  const int grid = rows * kCluster;
  if (a.mask_table) {  // sparse chunks: 512-thread CTAs with the queue
    const size_t hq = static_cast<size_t>(kHistQueue) * sizeof(float) + (a.lmoments ? static_cast<size_t>(kNB) * 4 : 0);
    if (a.lmoments) {
      if (a.want_raw) large_hist_kernel<DT, true, true, kHistThreads><<<grid, kHistThreads, hq, st>>>(a);
      else large_hist_kernel<DT, false, true, kHistThreads><<<grid, kHistThreads, hq, st>>>(a);
    } else if (a.want_raw) {
      large_hist_kernel<DT, true, false, kHistThreads><<<grid, kHistThreads, hq, st>>>(a);
    } else {
      large_hist_kernel<DT, false, false, kHistThreads><<<grid, kHistThreads, hq, st>>>(a);
    }
  } else {
    constexpr int T2 = kHistThreads / 2;
    const size_t hm = a.lmoments ? static_cast<size_t>(kNB) * 4 : 0;
    if (a.lmoments) {
      if (a.want_raw) large_hist_kernel<DT, true, true, T2><<<grid, T2, hm, st>>>(a);
      else large_hist_kernel<DT, false, true, T2><<<grid, T2, hm, st>>>(a);
    } else if (a.want_raw) {
      large_hist_kernel<DT, true, false, T2><<<grid, T2, hm, st>>>(a);
    } else {
      large_hist_kernel<DT, false, false, T2><<<grid, T2, hm, st>>>(a);
    }
  }
  large_select_kernel<DT><<<rows, kSelectThreads, select_smem, st>>>(a);
  const int parts = static_cast<int>((a.vocab + kGatherIds - 1) / kGatherIds);
  large_gather_kernel<DT><<<rows * parts, kGatherThreads, 0, st>>>(a, parts, 0);
  if (a.lmoments) {  // typical-p rows: the exact run, then the bins that depend on it
    large_resolve_kernel<DT, 0><<<rows, kResolveThreads, res_smem, st>>>(a);
    large_gather_kernel<DT><<<rows * parts, kGatherThreads, 0, st>>>(a, parts, 1);
  }
  large_resolve_kernel<DT, 1><<<rows, kResolveThreads, res_smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_large(const FinalizeArgs& a, int dtype, int rows, size_t select_smem, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  return dtype == GS_DTYPE_F32 ? launch_large_t<GS_DTYPE_F32>(a, rows, select_smem, st)
                               : launch_large_t<GS_DTYPE_BF16>(a, rows, select_smem, st);
}

}  // namespace gs
