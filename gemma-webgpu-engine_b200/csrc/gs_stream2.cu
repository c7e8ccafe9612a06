// Kernel 1, warp-pipelined form: the streaming pass for rows whose topK is at most
// pipe_max_k() (and greedy / histogram-path rows), on 16-byte aligned rows.
//
// Every warp owns whole units (a row's chunk of the vocabulary) and never waits for
// another warp.  A unit is processed in one of two modes, chosen identically by the
// warp's producer and consumer from the unit's first 1024 constraint-mask bits:
//
//  * ring mode (unmasked rows, and masked rows allowing more than 1/8 of those ids):
//    the warp keeps a private ring of kStages shared-memory stages, each holding one
//    tile of logits (2 KB: 512 f32 / 1024 bf16 ids, one TMA bulk copy, no multicast)
//    and the tile's mask words.  A stage is refilled with the warp's next ring tile as
//    soon as it has been consumed.  Per tile the warp clears the penalty-history ids (a
//    sorted per-unit list) from the staged mask words and runs straight-line passes over
//    the lane's 4 vectors: soft cap (packed f32x2 polynomial; values outside its range
//    redone afterwards), dead ids set to -inf, tile maximum, candidate test, then (after
//    one warp-wide maximum, so the running sum is rescaled at most once per tile by the
//    whole warp) the sum of e^(x/T).
//  * gather mode (masked rows allowing few ids): the warp reads the unit's mask words,
//    clears the penalised ids, lists the live offsets (lane l scans word l of each group
//    of 32) and loads only those logits, four independent loads per lane in flight, so
//    disallowed logits are never read.
//
// Top-k candidates go to a per-warp buffer at ballot-ranked positions; the unit's first
// ring tile sets a threshold by a binary search on its values, and when the buffer fills
// up a radix select keeps the k best and raises the threshold.  A requested
// log-probability (the raw sum over every id) forces ring mode and is one more pass over
// each staged tile.  The unit outputs are those of stream_kernel (gs_stream.cu).
#include <type_traits>

#include "gs_device.cuh"
#include "gs_block.cuh"
#include "gs_internal.cuh"
#include "../../include/gsampler.h"

namespace gs {

namespace {

constexpr int kWarps = 16;
constexpr int kThreads3 = kWarps * 32;
constexpr int kStages = 4;
constexpr int kTileBytes = 2048;               // logits per stage
constexpr int kMaskBytes = 128;                // mask words per stage (<= 1024 ids)
constexpr int kStageBytes = kTileBytes + kMaskBytes;
constexpr int kPenCap = 256;                   // sorted penalised ids per unit (else scan mode)
constexpr int kWarpCand = 256;                 // per-warp candidate buffer
constexpr int kListCap = 128;                  // gather mode: live offsets per batch
constexpr int kGatherIds = kTileBytes * 8;     // gather mode: ids per stage (2 KB of mask words)
constexpr int kWarpBytes = kStages * kStageBytes + kPenCap * 4 + kWarpCand * 8 + 256 * 4 + kListCap * 4;
constexpr int kPipeMaxK = 112;

static_assert(kWarpBytes % 128 == 0, "per-warp shared slices keep 128-byte alignment");
static_assert((kStages & (kStages - 1)) == 0, "stage index wraps by mask");

// Out-of-line soft cap for the rare values outside the polynomial range.
__device__ __noinline__ float softcap_slow(float x, float cap, float inv_cap) { return softcap(x, cap, inv_cap); }

// Ascending bitonic sort of n2 (power of two, <= kPenCap) 32-bit values by one warp.
__device__ __noinline__ void warp_sort_u32(uint32_t* v, int n2, int lane) {
  for (int k = 2; k <= n2; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = lane; i < n2; i += 32) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint32_t a = v[i], b = v[ixj];
          if (((i & k) == 0) ? a > b : a < b) {
            v[i] = b;
            v[ixj] = a;
          }
        }
      }
      __syncwarp();
    }
}

template <int DT>
struct Ld;
template <>
struct Ld<GS_DTYPE_F32> {
  static constexpr int kVec = 4;
  static __device__ __forceinline__ void vec(const unsigned char* p, float (&x)[4]) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    x[0] = v.x;
    x[1] = v.y;
    x[2] = v.z;
    x[3] = v.w;
  }
  static __device__ __forceinline__ float one(const unsigned char* p) { return *reinterpret_cast<const float*>(p); }
  static __device__ __forceinline__ float global(const unsigned char* row, int64_t o) {
    return __ldg(reinterpret_cast<const float*>(row) + o);
  }
};
template <>
struct Ld<GS_DTYPE_BF16> {
  static constexpr int kVec = 8;
  static __device__ __forceinline__ void vec(const unsigned char* p, float (&x)[8]) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    x[0] = bf16_lo(v.x);
    x[1] = bf16_hi(v.x);
    x[2] = bf16_lo(v.y);
    x[3] = bf16_hi(v.y);
    x[4] = bf16_lo(v.z);
    x[5] = bf16_hi(v.z);
    x[6] = bf16_lo(v.w);
    x[7] = bf16_hi(v.w);
  }
  static __device__ __forceinline__ float one(const unsigned char* p) {
    return __uint_as_float(static_cast<uint32_t>(*reinterpret_cast<const unsigned short*>(p)) << 16);
  }
  static __device__ __forceinline__ float global(const unsigned char* row, int64_t o) {
    return __uint_as_float(static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short*>(row) + o)) << 16);
  }
};

struct Geom {
  int row;
  int n;        // ids in the unit
  int ntiles;
  int32_t state;
  int64_t lo;   // first local id of the unit
  bool masked;
};

__device__ __forceinline__ Geom geom(const StreamArgs& A, int unit, int te) {
  Geom g;
  g.row = unit / A.splits;
  const int part = unit - g.row * A.splits;
  g.lo = static_cast<int64_t>(part) * A.chunk;
  const int64_t hi = g.lo + A.chunk < A.vocab ? g.lo + A.chunk : A.vocab;
  g.n = static_cast<int>(hi > g.lo ? hi - g.lo : 0);
  g.ntiles = (g.n + te - 1) / te;
  g.state = A.mask_state ? A.mask_state[g.row] : -1;
  g.masked = A.mask_table != nullptr && g.state >= 0 && g.state < A.mask_states;
  return g;
}

// The first unit from u on (in steps of `step`) whose row is not on the histogram path
// (those rows' statistics come from the histogram kernel).
__device__ __forceinline__ int next_unit(const StreamArgs& A, int u, int n_units, int step) {
  for (; u < n_units; u += step) {
    const int row = u / A.splits;
    if ((A.plans ? A.plans[row].mode : A.plan0.mode) != kModeLarge) break;
  }
  return u;
}

// Gather mode for a unit: a masked unit (without a requested log-probability) whose
// first min(n, 1024) ids include at most 1/8 allowed ones.  Called by the whole warp;
// producer and consumer evaluate it on the same words, so they always agree.
__device__ __forceinline__ bool gather_mode(const StreamArgs& A, const Geom& g, int lane) {
  if (!g.masked || A.want_raw) return false;
  const int span = g.n < 1024 ? g.n : 1024;
  const int nw = (span + 31) >> 5;
  uint32_t w = 0;
  if (lane < nw) {
    w = __ldg(A.mask_table + static_cast<int64_t>(g.state) * A.mask_words + (g.lo >> 5) + lane);
    if (lane == nw - 1 && (span & 31)) w &= (1u << (span & 31)) - 1u;
  }
  const int c = static_cast<int>(__reduce_add_sync(kFullMask, static_cast<unsigned>(__popc(w))));
  return c * 8 <= span;
}

}  // namespace

int pipe_max_k() { return kPipeMaxK; }
int64_t pipe_max_chunk() { return 1ll << 30; }

size_t stream2_smem_bytes(int64_t) { return static_cast<size_t>(kWarps) * kWarpBytes; }

template <int DT>
__global__ void __launch_bounds__(kThreads3, 1) stream2_kernel(const __grid_constant__ StreamArgs A, int n_units) {
  using LD = Ld<DT>;
  constexpr int VE = LD::kVec;                 // ids per 16-byte vector
  constexpr int ESZ = DT == GS_DTYPE_F32 ? 4 : 2;
  constexpr int TE = kTileBytes / ESZ;         // ids per tile
  constexpr int NSUB = TE / 512;               // sub-tiles of 512 ids per tile
  constexpr int VPS = 512 / VE / 32;           // vectors per lane per sub-tile
  constexpr uint32_t kFull = (1u << VE) - 1u;
  constexpr int kPer = kListCap / 32;          // gather mode: values per lane per batch
  static_assert(VPS * VE == 16 && NSUB <= 2, "candidate bits of a lane fit one word");
  static_assert(TE / 32 <= 32 && TE / 32 * 4 <= kMaskBytes, "mask words of a tile: one per lane");
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ unsigned long long bars_s[kWarps][kStages];
  __shared__ unsigned char smode[kWarps][kStages];  // 1: the stage holds a gather-mode mask tile

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;  // warps per CTA (kWarps, fewer for small batches)
  const int total_warps = gridDim.x * nwarps;
  const int first_unit = blockIdx.x * nwarps + warp;
  if (first_unit >= n_units) return;  // whole warp; the kernel has no block-wide barrier
  unsigned char* ring = dsm + warp * kWarpBytes;
  uint32_t* pen = reinterpret_cast<uint32_t*>(ring + kStages * kStageBytes);
  unsigned long long* wbuf = reinterpret_cast<unsigned long long*>(pen + kPenCap);
  unsigned* whist = reinterpret_cast<unsigned*>(wbuf + kWarpCand);
  uint32_t* loffs = reinterpret_cast<uint32_t*>(whist + 256);
  uint64_t* bars = reinterpret_cast<uint64_t*>(&bars_s[warp][0]);
  const unsigned char* logits = static_cast<const unsigned char*>(A.logits);
  const float cap = A.softcap, inv_cap = A.inv_softcap;
  const bool want_raw = A.want_raw != 0;
  const unsigned lane_lt = (1u << lane) - 1u;

  if (lane == 0)
    for (int s = 0; s < kStages; ++s) mbar_init(bars + s, 1);
  __syncwarp();

  // ---- producer: a cursor over the warp's stages, one refill per consumed stage ----
  // A ring-mode unit is a sequence of logit tiles; a gather-mode unit is a sequence of
  // mask tiles (its constraint words, kGatherIds ids per stage).  The stage's mode byte
  // tells the consumer which (every unit has at least one stage).
  int c_unit = next_unit(A, first_unit, n_units, total_warps), c_tile = 0, c_ntiles = 0;
  bool c_gather = false;
  Geom cg;
  auto enter_unit = [&]() {
    c_tile = 0;
    if (c_unit < n_units) {
      cg = geom(A, c_unit, TE);
      c_gather = gather_mode(A, cg, lane);
      c_ntiles = c_gather ? (cg.n + kGatherIds - 1) / kGatherIds : cg.ntiles;
    }
  };
  enter_unit();
  uint32_t c_word = 0xffffffffu;  // ring tiles of masked units: this lane's mask word, loaded ahead
  auto load_word = [&]() {
    c_word = 0xffffffffu;
    if (c_unit < n_units && cg.masked && !c_gather) {
      const int t0 = c_tile * TE;
      const int cnt = cg.n - t0 < TE ? cg.n - t0 : TE;
      if (lane < ((cnt + 31) >> 5))
        c_word = __ldg(A.mask_table + static_cast<int64_t>(cg.state) * A.mask_words + ((cg.lo + t0) >> 5) + lane);
    }
  };
  load_word();
  uint32_t issued = 0;
  auto produce = [&]() {
    if (c_unit >= n_units) return;  // warp-uniform
    const int s = static_cast<int>(issued & (kStages - 1));
    unsigned char* st = ring + s * kStageBytes;
    if (c_gather) {
      if (lane == 0) {
        const int nwords = (cg.n + 31) >> 5;
        const int w0 = c_tile * (kGatherIds / 32);
        const int wn = nwords - w0 < kGatherIds / 32 ? nwords - w0 : kGatherIds / 32;
        // (rounding up to 16 bytes stays inside the mask row: mask_words % 4 == 0)
        const uint32_t bytes = (static_cast<uint32_t>(wn) * 4u + 15u) & ~15u;
        const uint32_t* src = A.mask_table + static_cast<int64_t>(cg.state) * A.mask_words + (cg.lo >> 5) + w0;
        smode[warp][s] = 1;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(bars + s, bytes);
        bulk_g2s(st, src, bytes, bars + s);
      }
    } else {
      uint32_t* smw = reinterpret_cast<uint32_t*>(st + kTileBytes);
      const int t0 = c_tile * TE;
      const int cnt = cg.n - t0 < TE ? cg.n - t0 : TE;
      const int words = (cnt + 31) >> 5;
      uint32_t w = c_word;
      if (lane == words - 1 && (cnt & 31)) w &= (1u << (cnt & 31)) - 1u;
      if (lane < words) smw[lane] = w;
      if (lane == 0) {
        const unsigned char* src = logits + (static_cast<int64_t>(cg.row) * A.row_stride + cg.lo + t0) * ESZ;
        const uint32_t bytes = static_cast<uint32_t>(cnt / VE) * 16u;  // whole 16-byte vectors
        smode[warp][s] = 0;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(bars + s, bytes);
        if (bytes) bulk_g2s(st, src, bytes, bars + s);
      }
    }
    ++issued;
    if (++c_tile >= c_ntiles) {
      c_unit = next_unit(A, c_unit + total_warps, n_units, total_warps);
      enter_unit();
    }
    load_word();
  };
#pragma unroll 1
  for (int i = 0; i < kStages; ++i) produce();

  // ---- consumer ----
  int cs = 0;        // stage of the next ring tile
  uint32_t cph = 0;  // its mbarrier phase parity
  for (int unit = next_unit(A, first_unit, n_units, total_warps); unit < n_units;
       unit = next_unit(A, unit + total_warps, n_units, total_warps)) {
    const Geom g = geom(A, unit, TE);
    const int row = g.row;
    const RowPlan* pp = A.plans ? A.plans + row : &A.plan0;
    const int k_eff = pp->k_eff;
    const bool do_sum = pp->mode != kModeGreedy;
    const double a2 = pp->a2;
    const float a2_hi = pp->a2_hi, a2_lo = pp->a2_lo;
    // Terms are taken against the running reference m_t while no value exceeds it by more
    // than dlim (then a term is at most 2^2 and its exponent keeps full float accuracy);
    // the warp-wide maximum and the rescale run only when some lane crosses that limit,
    // and the unit's true maximum is settled once, at its end.
    const float dlim = do_sum ? static_cast<float>(2.0 / a2) : 0.0f;
    const unsigned char* rowp = logits + (static_cast<int64_t>(row) * A.row_stride + g.lo) * ESZ;
    uint32_t uflags = (A.mask_table != nullptr && g.state >= A.mask_states) ? GS_FLAG_ERR_INVALID : 0u;
    const uint32_t id_base = static_cast<uint32_t>(A.vocab_offset + g.lo);

    // penalised ids of the unit, as sorted offsets (or, above kPenCap, scanned per tile)
    int64_t hl = A.history_len ? A.history_len[row] : 0;
    if (hl > A.history_stride) hl = A.history_stride;
    if (hl < 0) hl = 0;
    const int32_t* hrow = A.history + static_cast<int64_t>(row) * A.history_stride;
    int pen_n = 0;
    for (int64_t j0 = 0; j0 < hl; j0 += 128) {  // four loads per lane in flight
      int32_t hv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int64_t j = j0 + q * 32 + lane;
        hv[q] = j < hl ? hrow[j] : 0;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int64_t j = j0 + q * 32 + lane;
        int64_t off = -1;
        if (j < hl) off = static_cast<int64_t>(hv[q]) - A.vocab_offset - g.lo;
        const bool in = off >= 0 && off < g.n;
        const unsigned b = __ballot_sync(kFullMask, in);
        const int at = pen_n + __popc(b & lane_lt);
        if (in && at < kPenCap) pen[at] = static_cast<uint32_t>(off);
        pen_n += __popc(b);
      }
    }
    const bool pen_scan = pen_n > kPenCap;
    if (!pen_scan && pen_n > 1) {
      int n2 = 2;
      while (n2 < pen_n) n2 <<= 1;
      for (int i = pen_n + lane; i < n2; i += 32) pen[i] = 0xffffffffu;
      __syncwarp();
      warp_sort_u32(pen, n2, lane);
    }
    __syncwarp();
    int pen_cur = 0;

    float m_t = -INFINITY, rm_t = -INFINITY;  // warp-uniform running maxima (m_t: the sum's reference)
    float lmx = -INFINITY;                    // this lane's maximum of the live values
    double s_t = 0.0, rs_t = 0.0;             // per-lane sums relative to m_t / rm_t
    uint32_t bad = 0;
    int na = 0;
    int wcnt = 0;                             // warp-uniform candidate count
    unsigned long long wtau = 0;              // packs <= wtau cannot be among the unit's k best
    unsigned long long bp = 0;                // k = 1: the lane's best pack ...
    float bx = -INFINITY;                     // ... and its value
    int wcap = 4 * k_eff + 64;
    wcap = wcap > kWarpCand - 32 ? kWarpCand - 32 : wcap;

    unsigned long long* rtau = A.row_tau ? A.row_tau + row : nullptr;
    auto publish = [&](unsigned long long b) {  // raise the row's shared bound
      if (rtau && lane == 0) atomicMax(rtau, b);
    };
    auto compact = [&]() {
      __syncwarp();
      const unsigned long long kth = warp_select_packs(wbuf, wcnt, k_eff, whist, lane);
      wtau = kth > wtau ? kth : wtau;
      wcnt = k_eff;
      publish(kth);
    };
    // One pack per lane into the candidate buffer (called by the whole warp).  Returns
    // true when this lane's pack is settled (stored, below the threshold, or none);
    // false when the buffer was full and it must be offered again.
    auto offer = [&](bool has, unsigned long long pk) -> bool {
      const bool keep = has && pk > wtau;
      const unsigned kb = __ballot_sync(kFullMask, keep);
      const int nk = __popc(kb);
      const int rank = __popc(kb & lane_lt);
      const int space = kWarpCand - wcnt;
      if (keep && rank < space) wbuf[wcnt + rank] = pk;
      wcnt += nk < space ? nk : space;
      const bool done = !keep || rank < space;
      if (nk > space) compact();
      return done;
    };
    auto tau_value = [&]() { return wtau ? key32_value(static_cast<uint32_t>(wtau >> 32)) : -INFINITY; };
    auto rescale = [&](float mt) {  // warp-uniform
      if (mt > m_t) {
        if (m_t > -INFINITY) s_t = __dmul_rn(s_t, exp2(__dmul_rn(static_cast<double>(m_t) - static_cast<double>(mt), a2)));
        m_t = mt;
      }
    };
    auto rescale_raw = [&](float rt) {  // warp-uniform
      if (rt > rm_t) {
        if (rm_t > -INFINITY) rs_t = __dmul_rn(rs_t, exp(static_cast<double>(rm_t) - static_cast<double>(rt)));
        rm_t = rt;
      }
    };

    // ================================ ring mode ================================
    // Full tile, as NSUB sub-tiles of 512 ids, each straight-line over the lane's VPS
    // vectors.  Returns the candidate bits (bit sub*16 + j*VE + i: live value at or above
    // the running threshold).
    auto dense_tile = [&](auto masked_tag, const unsigned char* st, const uint32_t* smw, int t, int t0) -> uint32_t {
      constexpr bool MASKED = decltype(masked_tag)::value;
      uint32_t cm = 0;
#pragma unroll 1
      for (int sub = 0; sub < NSUB; ++sub) {
        float x[VPS][VE];
#pragma unroll
        for (int j = 0; j < VPS; ++j) LD::vec(st + ((sub * VPS + j) * 32 + lane) * 16, x[j]);
        if (cap != 0.0f) {
          float zm = 0.0f;
#pragma unroll
          for (int j = 0; j < VPS; ++j)
#pragma unroll
            for (int i = 0; i < VE; i += 2) {
              float2 z;
              const float2 c = softcap2_poly(make_float2(x[j][i], x[j][i + 1]), cap, inv_cap, &z);
              x[j][i] = c.x;
              x[j][i + 1] = c.y;
              zm = fmaxf(zm, fmaxf(z.x, z.y));  // (NaN inputs stay NaN through the polynomial)
            }
          if (!(zm < kSoftcapPolyZ)) {
            // rare: values outside the polynomial range take the full routine
#pragma unroll
            for (int j = 0; j < VPS; ++j) {
              float r[VE];
              LD::vec(st + ((sub * VPS + j) * 32 + lane) * 16, r);
#pragma unroll
              for (int i = 0; i < VE; ++i) {
                const float y = __fmul_rn(r[i], inv_cap);
                if (!(__fmul_rn(y, y) < kSoftcapPolyZ)) x[j][i] = softcap_slow(r[i], cap, inv_cap);
              }
            }
          }
        }
        uint32_t bu[VPS];
#pragma unroll
        for (int j = 0; j < VPS; ++j) {
          if constexpr (MASKED) {
            const int e = ((sub * VPS + j) * 32 + lane) * VE;
            bu[j] = (smw[e >> 5] >> (e & 31)) & kFull;
#pragma unroll
            for (int i = 0; i < VE; ++i)
              if (!((bu[j] >> i) & 1u)) x[j][i] = -INFINITY;
          } else {
            bu[j] = kFull;
          }
        }
        float vmx[VPS];
        float tmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < VPS; ++j) {
          float v = x[j][0];
#pragma unroll
          for (int i = 1; i < VE; ++i) v = fmaxf(v, x[j][i]);
          vmx[j] = v;
          tmax = fmaxf(tmax, v);
        }
        if (k_eff == 1) {
          if (tmax > bx || (bp == 0ull && tmax == tmax)) {
            // first live position of the lane's maximum (ids ascend with (j, i))
            int fj = -1, fi = 0;
#pragma unroll
            for (int j = VPS - 1; j >= 0; --j)
#pragma unroll
              for (int i = VE - 1; i >= 0; --i)
                if (((bu[j] >> i) & 1u) && x[j][i] == tmax) {
                  fj = j;
                  fi = i;
                }
            if (fj >= 0) {
              bx = tmax;
              bp = make_pack(tmax, id_base + static_cast<uint32_t>(t0 + ((sub * VPS + fj) * 32 + lane) * VE + fi));
            }
          }
        } else if (k_eff > 1) {
          if (t == 0 && sub == 0) {
            // Threshold from the unit's first 512 ids: the largest key K found by a
            // binary search such that at least k live values there are >= value(K).
            // Those values belong to the unit, so its k-th largest is >= value(K).
            int nlv = 512;
            if constexpr (MASKED) {
              int c = 0;
#pragma unroll
              for (int j = 0; j < VPS; ++j) c += __popc(bu[j]);
              nlv = static_cast<int>(__reduce_add_sync(kFullMask, static_cast<unsigned>(c)));
            }
            if (nlv >= k_eff) {
              const uint32_t kneg = key32(-INFINITY);
              uint32_t klo = kneg, khi = key32(warp_max(tmax)) + 1u;
#pragma unroll 1
              for (int it = 0; it < 14 && khi - klo > 1u; ++it) {
                const uint32_t mid = klo + ((khi - klo) >> 1);
                const float v = key32_value(mid);  // > -inf: dead (-inf) and NaN values never count
                int c = 0;
#pragma unroll
                for (int j = 0; j < VPS; ++j)
#pragma unroll
                  for (int i = 0; i < VE; ++i) c += x[j][i] >= v ? 1 : 0;
                c = static_cast<int>(__reduce_add_sync(kFullMask, static_cast<unsigned>(c)));
                if (c >= k_eff) {
                  klo = mid;
                } else {
                  khi = mid;
                }
              }
              if (klo != kneg) {
                // pack > t0b  <=>  key >= klo
                const unsigned long long t0b = (static_cast<unsigned long long>(klo) << 32) - 1ull;
                wtau = t0b > wtau ? t0b : wtau;
                publish(t0b);
              }
            }
          }
          const float tau_x = tau_value();
          bool any = false;
#pragma unroll
          for (int j = 0; j < VPS; ++j) any |= vmx[j] >= tau_x;
          if (any) {
#pragma unroll
            for (int j = 0; j < VPS; ++j)
              if (vmx[j] >= tau_x) {
#pragma unroll
                for (int i = 0; i < VE; ++i)
                  if (((bu[j] >> i) & 1u) && x[j][i] >= tau_x) cm |= 1u << (sub * 16 + j * VE + i);
              }
          }
        }
        if (do_sum) {
          lmx = fmaxf(lmx, tmax);
          if (__any_sync(kFullMask, tmax > m_t + dlim)) rescale(warp_max(tmax));
          if (m_t > -INFINITY) {
            // NaN and +inf reach the sum (as NaN); dead ids are -inf and add 0
            float2 acc0 = make_float2(0.0f, 0.0f), acc1 = make_float2(0.0f, 0.0f);
            const float2 nm = make_float2(-m_t, -m_t);
            const float2 ah = make_float2(a2_hi, a2_hi), al = make_float2(a2_lo, a2_lo);
#pragma unroll
            for (int j = 0; j < VPS; ++j)
#pragma unroll
              for (int i = 0; i < VE; i += 2) {
                const float2 d = __fadd2_rn(make_float2(x[j][i], x[j][i + 1]), nm);
                const float2 tt = __ffma2_rn(d, al, __fmul2_rn(d, ah));
                const float2 e = make_float2(ex2_approx(tt.x), ex2_approx(tt.y));
                if ((j * VE + i) & 2) {
                  acc1 = __fadd2_rn(acc1, e);
                } else {
                  acc0 = __fadd2_rn(acc0, e);
                }
              }
            s_t += static_cast<double>((acc0.x + acc0.y) + (acc1.x + acc1.y));
          }
        }
        if (!do_sum || !(m_t > -INFINITY)) {
          // no sum to carry a NaN: look for one explicitly
#pragma unroll
          for (int j = 0; j < VPS; ++j)
#pragma unroll
            for (int i = 0; i < VE; ++i)
              if (x[j][i] != x[j][i]) bad = 1u;  // (dead ids are -inf)
        }
      }
      return cm;
    };

    // Partial tile (the row's last, shorter than a tile): element by element from HBM.
    auto scalar_tile = [&](const uint32_t* smw, int t0, int cnt) {
      float lmax = -INFINITY, rmax = -INFINITY;
      for (int i = lane; i < cnt; i += 32) {
        float x = LD::global(rowp, t0 + i);
        if (cap != 0.0f) x = softcap(x, cap, inv_cap);
        if ((smw[i >> 5] >> (i & 31)) & 1u) {
          if (x != x) bad = 1u;
          lmax = fmaxf(lmax, x);
        }
        rmax = fmaxf(rmax, x);
      }
      if (do_sum) {
        lmx = fmaxf(lmx, lmax);
        rescale(warp_max(lmax));
      }
      if (want_raw) rescale_raw(warp_max(rmax));
      float acc = 0.0f, racc = 0.0f;
      for (int i0 = 0; i0 < cnt; i0 += 32) {  // warp-uniform
        const int i = i0 + lane;
        const bool valid = i < cnt;
        float x = -INFINITY;
        bool live = false;
        if (valid) {
          x = LD::global(rowp, t0 + i);
          if (cap != 0.0f) x = softcap(x, cap, inv_cap);
          live = ((smw[i >> 5] >> (i & 31)) & 1u) != 0u;
        }
        if (want_raw && valid && rm_t > -INFINITY) {
          const float d = x - rm_t;
          racc += ex2_approx(fmaf(d, kL2eLo, d * kL2eHi));
        }
        const uint32_t id = id_base + static_cast<uint32_t>(t0 + i);
        if (live && do_sum && m_t > -INFINITY) {
          const float d = x - m_t;
          acc += ex2_approx(fmaf(d, a2_lo, d * a2_hi));
        }
        if (k_eff == 1) {
          if (live && x == x) {
            const unsigned long long pk = make_pack(x, id);
            if (pk > bp) {
              bp = pk;
              bx = x;
            }
          }
        } else if (k_eff > 1) {
          const float tau_x = tau_value();
          bool pend = live && x >= tau_x;
          const unsigned long long pk = pend ? make_pack(x, id) : 0ull;
          while (__any_sync(kFullMask, pend)) pend = !offer(pend, pk);
        }
      }
      s_t += static_cast<double>(acc);
      rs_t += static_cast<double>(racc);
    };

    // Raw sum over every id of a full staged tile (log-probability requested).
    auto raw_tile = [&](const unsigned char* st) {
      float rmax = -INFINITY;
#pragma unroll 4
      for (int c = 0; c < TE / 32; ++c) {
        float x = LD::one(st + (c * 32 + lane) * ESZ);
        if (cap != 0.0f) x = softcap(x, cap, inv_cap);
        rmax = fmaxf(rmax, x);
      }
      rescale_raw(warp_max(rmax));
      if (rm_t > -INFINITY) {
        float es = 0.0f;
#pragma unroll 4
        for (int c = 0; c < TE / 32; ++c) {
          float x = LD::one(st + (c * 32 + lane) * ESZ);
          if (cap != 0.0f) x = softcap(x, cap, inv_cap);
          const float d = x - rm_t;
          es += ex2_approx(fmaf(d, kL2eLo, d * kL2eHi));
        }
        rs_t += static_cast<double>(es);
      }
    };

    // ================================ gather mode ================================
    // Live offsets are listed in order (a warp scan gives each lane its ranks); a full
    // list's loads are issued at once (kPer per lane) and its values processed only when
    // the next list is full, so the loads are in flight while mask words are scanned.
    int nl = 0;               // offsets listed
    bool inflight = false;    // a launched batch awaits processing
    bool first_batch = true;  // the unit's first batch sets the top-k threshold
    float pv[kPer];           // its values (loads in flight) ...
    uint32_t po[kPer];        // ... and unit offsets (~0u: empty slot)
    auto launch = [&]() {
      __syncwarp();
#pragma unroll
      for (int q = 0; q < kPer; ++q) {
        const int i = q * 32 + lane;
        po[q] = i < nl ? loffs[i] : 0xffffffffu;
      }
      __syncwarp();  // the list may be refilled from here on
#pragma unroll
      for (int q = 0; q < kPer; ++q) pv[q] = po[q] != 0xffffffffu ? LD::global(rowp, po[q]) : 0.0f;
      inflight = true;
      nl = 0;
    };
    auto finish = [&]() {
      float xv[kPer];
      if (cap != 0.0f) {
        float zm = 0.0f;
#pragma unroll
        for (int q = 0; q < kPer; q += 2) {
          float2 z;
          const float2 c = softcap2_poly(make_float2(pv[q], pv[q + 1]), cap, inv_cap, &z);
          xv[q] = c.x;
          xv[q + 1] = c.y;
          zm = fmaxf(zm, fmaxf(z.x, z.y));
        }
        if (!(zm < kSoftcapPolyZ)) {
#pragma unroll
          for (int q = 0; q < kPer; ++q) {
            const float y = __fmul_rn(pv[q], inv_cap);
            if (!(__fmul_rn(y, y) < kSoftcapPolyZ)) xv[q] = softcap_slow(pv[q], cap, inv_cap);
          }
        }
      } else {
#pragma unroll
        for (int q = 0; q < kPer; ++q) xv[q] = pv[q];
      }
      float lmax = -INFINITY;
      int nvalid = 0;
#pragma unroll
      for (int q = 0; q < kPer; ++q) {
        if (po[q] == 0xffffffffu) {
          xv[q] = -INFINITY;
        } else {
          ++nvalid;
        }
        if (xv[q] != xv[q]) bad = 1u;
        lmax = fmaxf(lmax, xv[q]);
      }
      if (k_eff > 1 && first_batch) {
        // threshold from the unit's first batch (as for a dense unit's first 512 ids): the
        // largest key K with at least k of the batch's values >= value(K)
        first_batch = false;
        nvalid = static_cast<int>(__reduce_add_sync(kFullMask, static_cast<unsigned>(nvalid)));
        if (nvalid >= k_eff) {
          const uint32_t kneg = key32(-INFINITY);
          uint32_t klo = kneg, khi = key32(warp_max(lmax)) + 1u;
#pragma unroll 1
          for (int it = 0; it < 14 && khi - klo > 1u; ++it) {
            const uint32_t mid = klo + ((khi - klo) >> 1);
            const float v = key32_value(mid);  // > -inf: empty slots and NaN never count
            int c = 0;
#pragma unroll
            for (int q = 0; q < kPer; ++q) c += xv[q] >= v ? 1 : 0;
            c = static_cast<int>(__reduce_add_sync(kFullMask, static_cast<unsigned>(c)));
            if (c >= k_eff) {
              klo = mid;
            } else {
              khi = mid;
            }
          }
          if (klo != kneg) {
            const unsigned long long t0b = (static_cast<unsigned long long>(klo) << 32) - 1ull;
            wtau = t0b > wtau ? t0b : wtau;
          }
        }
      }
      if (do_sum) {
        lmx = fmaxf(lmx, lmax);
        if (__any_sync(kFullMask, lmax > m_t + dlim)) rescale(warp_max(lmax));
        if (m_t > -INFINITY) {
          float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
          for (int q = 0; q < kPer; ++q) {
            const float d = xv[q] - m_t;  // (empty slots are -inf and add 0)
            const float e = ex2_approx(fmaf(d, a2_lo, d * a2_hi));
            if (q & 1) {
              acc1 += e;
            } else {
              acc0 += e;
            }
          }
          s_t += static_cast<double>(acc0 + acc1);
        }
      }
      if (k_eff == 1) {
#pragma unroll
        for (int q = 0; q < kPer; ++q)
          if (po[q] != 0xffffffffu && xv[q] == xv[q]) {
            const unsigned long long pk = make_pack(xv[q], id_base + po[q]);
            if (pk > bp) {
              bp = pk;
              bx = xv[q];
            }
          }
      } else if (k_eff > 1) {
        const float tau0 = tau_value();
        bool any = false;
#pragma unroll
        for (int q = 0; q < kPer; ++q) any |= xv[q] >= tau0;
        if (__any_sync(kFullMask, any)) {
#pragma unroll
          for (int q = 0; q < kPer; ++q) {
            const float tau_x = tau_value();
            bool pend = po[q] != 0xffffffffu && xv[q] >= tau_x;
            const unsigned long long pk = pend ? make_pack(xv[q], id_base + po[q]) : 0ull;
            while (__any_sync(kFullMask, pend)) pend = !offer(pend, pk);
          }
        }
      }
      inflight = false;
    };
    // Appends the live offsets of word wi (this lane's w) in id order, launching full lists.
    auto list_word = [&](uint32_t w, int wi) {
      const int c = __popc(w);
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(kFullMask, incl, o);
        if (lane >= o) incl += t;
      }
      const int total = __shfl_sync(kFullMask, incl, 31);
      int r = incl - c;  // rank of this lane's next offset within the 32 words
      int done = 0;
      while (done < total) {  // warp-uniform
        const int room = kListCap - nl;
        const int hi = done + room;
        uint32_t* dst = loffs + (nl - done);
        while (w != 0u && r < hi) {
          dst[r] = static_cast<uint32_t>(wi * 32 + __ffs(w) - 1);
          w &= w - 1u;
          ++r;
        }
        const int take = total - done < room ? total - done : room;
        nl += take;
        done += take;
        if (nl == kListCap) {
          if (inflight) finish();
          launch();
        }
      }
    };
    auto gather_unit = [&]() {
      const int nwords = (g.n + 31) >> 5;
      const int ntl = (g.n + kGatherIds - 1) / kGatherIds;
      for (int t = 0; t < ntl; ++t) {
        if (!mbar_wait(bars + cs, cph, kWaitNs)) {
          uflags |= GS_FLAG_ERR_TIMEOUT;
          mbar_wait(bars + cs, cph, kWaitNs);
        }
        const uint32_t* mw = reinterpret_cast<const uint32_t*>(ring + cs * kStageBytes);
        const int w0 = t * (kGatherIds / 32);
        const int ngr = (nwords - w0 + 31) >> 5 < kGatherIds / 1024 ? (nwords - w0 + 31) >> 5 : kGatherIds / 1024;
        for (int q = 0; q < ngr; ++q) {
          const int wl = q * 32 + lane;  // word within the stage
          const int wi = w0 + wl;        // word within the unit
          uint32_t w = wi < nwords ? mw[wl] : 0u;
          if (wi == nwords - 1 && (g.n & 31)) w &= (1u << (g.n & 31)) - 1u;
          na += __popc(w);
          // clear the penalised ids of these 32 words
          if (pen_scan) {
            for (int64_t j = 0; j < hl; ++j) {
              const int64_t off = static_cast<int64_t>(hrow[j]) - A.vocab_offset - g.lo;
              if ((off >> 5) == wi) w &= ~(1u << (off & 31));
            }
          } else {
            const uint32_t gend = static_cast<uint32_t>(w0 + (q + 1) * 32) * 32u;
            while (pen_cur < pen_n && pen[pen_cur] < gend) {  // warp-uniform
              const uint32_t off = pen[pen_cur];
              if (static_cast<int>(off >> 5) == wi) w &= ~(1u << (off & 31));
              ++pen_cur;
            }
          }
          list_word(w, wi);
        }
        // release the stage
        __syncwarp();
        cs = (cs + 1) & (kStages - 1);
        if (cs == 0) cph ^= 1u;
        produce();
      }
      if (inflight) finish();
      if (nl > 0) {
        launch();
        finish();
      }
    };

    __syncwarp();
    if (smode[warp][cs]) {
      gather_unit();
    } else {
      // the row's shared bound, read one tile ahead (its load overlaps the tile's work)
      unsigned long long rt_next = rtau && k_eff > 1 ? *reinterpret_cast<volatile unsigned long long*>(rtau) : 0ull;
      for (int t = 0; t < g.ntiles; ++t) {
        if (rtau && k_eff > 1) {
          wtau = rt_next > wtau ? rt_next : wtau;
          rt_next = *reinterpret_cast<volatile unsigned long long*>(rtau);
        }
        if (!mbar_wait(bars + cs, cph, kWaitNs)) {
          uflags |= GS_FLAG_ERR_TIMEOUT;
          mbar_wait(bars + cs, cph, kWaitNs);
        }
        const unsigned char* st = ring + cs * kStageBytes;
        uint32_t* smw = reinterpret_cast<uint32_t*>(ring + cs * kStageBytes + kTileBytes);
        const int t0 = t * TE;
        const int cnt = g.n - t0 < TE ? g.n - t0 : TE;
        const int words = (cnt + 31) >> 5;
        if (g.masked && lane < words) na += __popc(smw[lane]);
        // clear the penalised ids: their exact scores are computed by the merge kernel
        bool pen_hit = false;
        if (pen_scan) {
          for (int64_t j = lane; j < hl; j += 32) {
            const int64_t off = static_cast<int64_t>(hrow[j]) - A.vocab_offset - g.lo - t0;
            if (off >= 0 && off < cnt) atomicAnd(&smw[off >> 5], ~(1u << (off & 31)));
          }
          pen_hit = true;
        } else if (pen_cur < pen_n && pen[pen_cur] < static_cast<uint32_t>(t0 + cnt)) {
          pen_hit = true;
          while (pen_cur < pen_n) {
            const int i = pen_cur + lane;
            const uint32_t off = i < pen_n ? pen[i] : 0xffffffffu;
            const bool in = off < static_cast<uint32_t>(t0 + cnt);
            if (in) atomicAnd(&smw[(off - t0) >> 5], ~(1u << ((off - t0) & 31)));
            const unsigned b = __ballot_sync(kFullMask, in);
            pen_cur += __popc(b);
            if (b != kFullMask) break;
          }
        }
        __syncwarp();

        uint32_t cm = 0;
        if (cnt == TE) {
          bool full = !g.masked && !pen_hit;
          if (g.masked) {
            const uint32_t lw = lane < words ? smw[lane] : 0u;
            full = __reduce_add_sync(kFullMask, static_cast<unsigned>(__popc(lw))) == static_cast<unsigned>(TE);
          }
          // one instantiation for every tile (its mask bits are all set when `full`): the
          // loop body stays small enough for the instruction cache
          (void)full;
          cm = dense_tile(std::true_type{}, st, smw, t, t0);
          if (want_raw) raw_tile(st);
        } else {
          scalar_tile(smw, t0, cnt);
        }
        // candidates found by the dense pass: one per lane per round
        while (__any_sync(kFullMask, cm != 0u)) {
          const bool has = cm != 0u;
          unsigned long long pk = 0;
          if (has) {
            const int b = __ffs(cm) - 1;
            const int r = b & 15;
            const int e = (((b >> 4) * VPS + r / VE) * 32 + lane) * VE + (r % VE);
            float x = LD::one(st + e * ESZ);
            if (cap != 0.0f) x = softcap(x, cap, inv_cap);
            pk = make_pack(x, id_base + static_cast<uint32_t>(t0 + e));
          }
          if (offer(has, pk) && has) cm &= cm - 1u;
        }
        if (k_eff > 1 && wcnt > wcap) compact();

        // ---- release the stage: refill it with the warp's next ring tile ----
        __syncwarp();
        cs = (cs + 1) & (kStages - 1);
        if (cs == 0) cph ^= 1u;
        produce();
      }
      if (!g.masked) na = g.n;
    }

    // ---- unit outputs ----
    __syncwarp();
    UnitStat* out = A.stats + unit;
    int ncand = 0;
    if (k_eff > 1) {
      if (wcnt > k_eff) compact();
      ncand = wcnt;
      unsigned long long* dst = A.cands + static_cast<int64_t>(unit) * A.kcap;
      for (int i = lane; i < wcnt; i += 32) dst[i] = wbuf[i];
    } else if (k_eff == 1) {
      unsigned long long b = bp;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long q = __shfl_xor_sync(kFullMask, b, o);
        b = q > b ? q : b;
      }
      ncand = b != 0ull ? 1 : 0;
      if (lane == 0 && b != 0ull) A.cands[static_cast<int64_t>(unit) * A.kcap] = b;
    }
    if (do_sum) rescale(warp_max(lmx));  // the unit's true maximum (s_t rescaled onto it)
    const double c = warp_sum(s_t);
    const double rc = warp_sum(rs_t);
    na = g.masked ? warp_sum_i(na) : na;
    const bool wbad = __any_sync(kFullMask, bad != 0u);
    const uint32_t ufl = __reduce_or_sync(kFullMask, uflags);
    if (lane == 0) {
      uint32_t fl = ufl;
      if (wbad || c != c || rc != rc || m_t == INFINITY) fl |= GS_FLAG_ERR_NONFINITE;
      out->m = m_t;
      out->s = m_t > -INFINITY ? c : 0.0;
      out->raw_m = rm_t;
      out->raw_s = rm_t > -INFINITY ? rc : 0.0;
      out->n_allowed = na;
      out->n_cand = ncand;
      out->flags = fl;
    }
    __syncwarp();
  }
}

bool stream2_eligible(const StreamArgs& a, int dtype, int rows) {
  const int esz = dtype == GS_DTYPE_F32 ? 4 : 2;
  (void)rows;
  if (reinterpret_cast<uintptr_t>(a.logits) & 15) return false;
  if ((a.row_stride * esz) & 15) return false;
  if (a.chunk % 1024) return false;
  if (a.mask_table && ((reinterpret_cast<uintptr_t>(a.mask_table) & 15) || (a.mask_words & 3))) return false;
  return true;
}

cudaError_t launch_stream2(const StreamArgs& a, int dtype, int rows, size_t smem, cudaStream_t st, int num_sms) {
  const int units = rows * a.splits;
  if (units == 0) return cudaSuccess;
  // Batches with fewer units than the GPU's warp slots spread them over every SM (fewer
  // warps per CTA, so that each warp gets a larger share of its SM's issue slots).
  int wpc = kWarps;
  if (units < num_sms * kWarps) wpc = (units + num_sms - 1) / num_sms;
  int grid = (units + wpc - 1) / wpc;
  if (grid > num_sms) grid = num_sms;
  smem = static_cast<size_t>(wpc) * kWarpBytes;
  // (the attribute is set to the exact size: the per-block limit also counts static smem)
  if (dtype == GS_DTYPE_F32) {
    cudaError_t e = cudaFuncSetAttribute(stream2_kernel<GS_DTYPE_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    stream2_kernel<GS_DTYPE_F32><<<grid, wpc * 32, smem, st>>>(a, units);
  } else {
    cudaError_t e = cudaFuncSetAttribute(stream2_kernel<GS_DTYPE_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    stream2_kernel<GS_DTYPE_BF16><<<grid, wpc * 32, smem, st>>>(a, units);
  }
  return cudaGetLastError();
}

}  // namespace gs
