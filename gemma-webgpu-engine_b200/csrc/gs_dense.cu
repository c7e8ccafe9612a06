// Kernel 1, dense form: the streaming pass for unconstrained rows (no constraint table)
// with topK <= dense_max_k() or greedy, no requested log-probability, 16-byte aligned rows.
//
// Same ownership and outputs as stream2_kernel (gs_stream2.cu): every warp owns whole
// units (a row's chunk of the vocabulary) and writes each unit's statistics and top-k
// packs for the merge.  The logits stream through a per-warp ring of kDStages 2 KB
// shared-memory stages filled by per-lane 16-byte asynchronous copies (cp.async, L2 only):
// every lane copies and later reads only its own vectors, so a stage needs no barrier and
// four tiles per warp (128 KB per SM) are in flight while one is worked on.  The
// per-element work is cut to what every id of an unconstrained row needs:
//   * the soft cap by the packed f32x2 polynomial, its range check folded into one packed
//     sum of the squares per sub-tile (a sum that is not below 1 means a value at or past
//     the cap, an infinity or a NaN: only then are the sub-tile's values checked one by
//     one and the out-of-range ones redone by the full routine);
//   * the lane's maximum of its 16 values (the candidate test, the sum's running
//     reference and the unit's maximum all derive from it);
//   * the sum of 2^((x - m)·log2e/T) in packed arithmetic.
// Penalised ids are few (at most the history length per row): their tiles are known from
// the unit's sorted list (a warp-uniform test per tile), and only there do the lanes
// holding one set it to -inf (dead).  Top-k candidates are not extracted where they are
// read: a lane whose maximum reaches the running threshold queues its 16 capped values
// (with their tile, lane and dead bits) in a 16-chunk per-warp queue, and a full queue is
// tested against the threshold of that moment one chunk per lane, the survivors offered
// to the candidate buffer; the buffer is cut back to the k best (radix select) once it
// holds 2k + 32 packs, which raises the threshold.  The per-id cost of a sub-tile with a
// candidate is then a ballot and four 16-byte stores instead of a per-element extraction.
#include "gs_device.cuh"
#include "gs_block.cuh"
#include "gs_internal.cuh"
#include "../../include/gsampler.h"

namespace gs {

namespace {

constexpr int kDWarps = 16;
constexpr int kDThreads = kDWarps * 32;
constexpr int kDTileBytes = 2048;             // ids per tile: 512 f32 / 1024 bf16 (4 vectors per lane)
constexpr int kDStages = 5;                   // per-warp ring: four tiles in flight ahead of the one read
constexpr int kDPenCap = 256;                 // sorted penalised offsets per unit (else scanned per tile)
constexpr int kDWarpCand = 160;               // per-warp candidate buffer
constexpr int kDPend = 16;                    // queued lane chunks (16 capped values, a tag, dead bits)
constexpr int kDWarpBytes = kDStages * kDTileBytes + kDPenCap * 4 + kDWarpCand * 8 + kDPend * (64 + 8);
constexpr int kDMaxK = 112;

static_assert(kDWarpBytes % 128 == 0, "per-warp slices keep 128-byte alignment");

__device__ __noinline__ float dense_softcap_slow(float x, float cap, float inv_cap) { return softcap(x, cap, inv_cap); }

// Ascending bitonic sort of n2 (a power of two, <= kDPenCap) 32-bit values by one warp.
__device__ __noinline__ void dense_sort_u32(uint32_t* v, int n2, int lane) {
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
struct DLd;
template <>
struct DLd<GS_DTYPE_F32> {
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
struct DLd<GS_DTYPE_BF16> {
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

// The first unit from u on (in steps of `step`) whose row is not on the histogram path.
__device__ __forceinline__ int dense_next_unit(const StreamArgs& A, int u, int n_units, int step) {
  for (; u < n_units; u += step) {
    const int row = u / A.splits;
    if ((A.plans ? A.plans[row].mode : A.plan0.mode) != kModeLarge) break;
  }
  return u;
}

}  // namespace

int dense_max_k() { return kDMaxK; }

template <int DT>
__global__ void __launch_bounds__(kDThreads, 1) dense_kernel(const __grid_constant__ StreamArgs A, int n_units) {
  using LD = DLd<DT>;
  constexpr int VE = LD::kVec;                 // ids per 16-byte vector
  constexpr int ESZ = DT == GS_DTYPE_F32 ? 4 : 2;
  constexpr int TE = kDTileBytes / ESZ;        // ids per tile
  constexpr int VPT = TE / VE / 32;            // vectors per lane per tile (4)
  constexpr int NSUB = TE / 512;               // sub-tiles of 512 ids per tile
  constexpr int VPS = 512 / VE / 32;           // vectors per lane per sub-tile
  static_assert(VPS * VE == 16 && NSUB <= 2 && VPT == 4, "a lane's bits of a tile fit one word");
  extern __shared__ __align__(128) unsigned char dsm[];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int total_warps = gridDim.x * nwarps;
  const int first_unit = blockIdx.x * nwarps + warp;
  if (first_unit >= n_units) return;  // whole warp; the kernel has no block-wide barrier
  unsigned char* ring = dsm + warp * kDWarpBytes;
  uint32_t* pen = reinterpret_cast<uint32_t*>(ring + kDStages * kDTileBytes);
  unsigned long long* wbuf = reinterpret_cast<unsigned long long*>(pen + kDPenCap);
  float* pendf = reinterpret_cast<float*>(wbuf + kDWarpCand);
  uint32_t* ptag = reinterpret_cast<uint32_t*>(pendf + kDPend * 16);
  uint32_t* pdead = ptag + kDPend;
  const unsigned char* logits = static_cast<const unsigned char*>(A.logits);
  const float cap = A.softcap, inv_cap = A.inv_softcap;
  const unsigned lane_lt = (1u << lane) - 1u;
  const uint32_t ring0 = smem_addr(ring) + static_cast<uint32_t>(lane) * 16u;  // this lane's slot of stage 0
  const uint32_t ring_end = ring0 + kDStages * kDTileBytes;

  for (int unit = dense_next_unit(A, first_unit, n_units, total_warps); unit < n_units;
       unit = dense_next_unit(A, unit + total_warps, n_units, total_warps)) {
    const int row = unit / A.splits;
    const int64_t glo = static_cast<int64_t>(unit - row * A.splits) * A.chunk;
    const int64_t ghi = glo + A.chunk < A.vocab ? glo + A.chunk : A.vocab;
    const int gn = static_cast<int>(ghi > glo ? ghi - glo : 0);
    const int nfull = gn / TE;  // full tiles; a shorter last tile is read element by element
    const unsigned char* rowp = logits + (static_cast<int64_t>(row) * A.row_stride + glo) * ESZ;

    // Tiles go into the ring in order: this lane's four vectors of the next tile into the
    // next stage (one commit group per tile, empty past the last full tile, so that the
    // group count stays in step).
    const unsigned char* src = rowp + lane * 16;
    uint32_t wr = ring0;
    int issued = 0;
    auto issue = [&]() {
      if (issued < nfull) {
#pragma unroll
        for (int q = 0; q < VPT; ++q)
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(wr + q * 512u), "l"(src + q * 512) : "memory");
        src += kDTileBytes;
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
      ++issued;
      wr += kDTileBytes;
      if (wr == ring_end) wr = ring0;
    };
    // the unit's first tiles are in flight while its penalty list is built
#pragma unroll
    for (int t = 0; t < kDStages - 1; ++t) issue();

    const RowPlan* pp = A.plans ? A.plans + row : &A.plan0;
    const int k_eff = pp->k_eff;
    const bool do_sum = pp->mode != kModeGreedy;
    const float a2_hi = pp->a2_hi, a2_lo = pp->a2_lo;
    const double a2 = pp->a2;
    // the sum's terms are taken against a running reference m_t while no value exceeds it
    // by more than dlim (a term stays below 2^2); the unit's maximum is settled at its end
    const float dlim = do_sum ? static_cast<float>(2.0 / a2) : 0.0f;
    const uint32_t id_base = static_cast<uint32_t>(A.vocab_offset + glo);

    // penalised ids of the unit as sorted offsets (above kDPenCap: scanned per tile)
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
        if (j < hl) off = static_cast<int64_t>(hv[q]) - A.vocab_offset - glo;
        const bool in = off >= 0 && off < gn;
        const unsigned b = __ballot_sync(kFullMask, in);
        const int at = pen_n + __popc(b & lane_lt);
        if (in && at < kDPenCap) pen[at] = static_cast<uint32_t>(off);
        pen_n += __popc(b);
      }
    }
    const bool pen_scan = pen_n > kDPenCap;
    if (!pen_scan && pen_n > 1) {
      int n2 = 2;
      while (n2 < pen_n) n2 <<= 1;
      for (int i = pen_n + lane; i < n2; i += 32) pen[i] = 0xffffffffu;
      __syncwarp();
      dense_sort_u32(pen, n2, lane);
    }
    __syncwarp();
    int pen_cur = 0;
    // the next tile holding a penalised id (warp-uniform; every tile when scanning)
    int dead_t = pen_scan ? 0 : (pen_n > 0 ? static_cast<int>(pen[0] / TE) : INT_MAX);

    float m_t = -INFINITY;                    // warp-uniform running reference of the sum
    float m_lim = -INFINITY;                  // m_t + dlim
    float lmx = -INFINITY;                    // this lane's maximum of the live values
    double s_t = 0.0;                         // this lane's sum relative to m_t
    uint32_t bad = 0;
    int wcnt = 0;                             // warp-uniform candidate count
    int pend_n = 0;                           // warp-uniform pending chunk count
    unsigned long long wtau = 0;              // packs <= wtau cannot be among the unit's k best
    float tau_x = -INFINITY;                  // the value of wtau's key (the candidate test)
    unsigned long long bp = 0;                // k = 1: the lane's best pack ...
    float bx = -INFINITY;                     // ... and its value
    int wcap = 2 * k_eff + 32;
    wcap = wcap > kDWarpCand - 32 ? kDWarpCand - 32 : wcap;
    unsigned long long* rtau = A.row_tau ? A.row_tau + row : nullptr;

    auto set_tau = [&](unsigned long long v) {  // warp-uniform
      if (v > wtau) {
        wtau = v;
        tau_x = key32_value(static_cast<uint32_t>(wtau >> 32));
      }
    };
    // the k best of the buffer (radix select; `hist` is 1 KB of this warp's shared memory
    // that nothing else uses at the time)
    auto compact = [&](unsigned* hist) {
      __syncwarp();
      const unsigned long long kth = warp_select_packs(wbuf, wcnt, k_eff, hist, lane);
      set_tau(kth);
      wcnt = k_eff;
      if (rtau && lane == 0) atomicMax(rtau, kth);
      __syncwarp();
    };
    // One pack per lane into the candidate buffer (the whole warp calls).  True when this
    // lane's pack is settled (stored, below the threshold, or none); false when the buffer
    // was full and it must be offered again.
    auto offer = [&](bool has, unsigned long long pk, unsigned* hist) -> bool {
      const bool keep = has && pk > wtau;
      const unsigned kb = __ballot_sync(kFullMask, keep);
      const int nk = __popc(kb);
      const int rank = __popc(kb & lane_lt);
      const int space = kDWarpCand - wcnt;
      if (keep && rank < space) wbuf[wcnt + rank] = pk;
      wcnt += nk < space ? nk : space;
      const bool done = !keep || rank < space;
      if (nk > space) compact(hist);
      return done;
    };
    // The pending chunks (a lane's 16 capped values whose maximum reached the threshold
    // when they were read) against the current threshold: one chunk per lane, its values
    // at or above it offered to the buffer.  Tag: tile << 8 | sub-tile << 5 | lane; the
    // chunk's penalised positions (-inf there, but not candidates) beside it.
    auto flush = [&](unsigned* hist) {
      __syncwarp();
      uint32_t sb = 0u, tag = 0u;
      if (lane < pend_n) {
        const float4* cv = reinterpret_cast<const float4*>(pendf + lane * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = cv[q];
          sb |= (v.x >= tau_x ? 1u : 0u) << (q * 4);
          sb |= (v.y >= tau_x ? 1u : 0u) << (q * 4 + 1);
          sb |= (v.z >= tau_x ? 1u : 0u) << (q * 4 + 2);
          sb |= (v.w >= tau_x ? 1u : 0u) << (q * 4 + 3);
        }
        tag = ptag[lane];
        sb &= ~pdead[lane];
      }
      const int ct = static_cast<int>(tag >> 8), cs = static_cast<int>((tag >> 5) & 7u), cl = static_cast<int>(tag & 31u);
      while (__any_sync(kFullMask, sb != 0u)) {
        const bool has = sb != 0u;
        unsigned long long pk = 0ull;
        if (has) {
          const int e = __ffs(sb) - 1;
          const int off = ct * TE + ((cs * VPS + e / VE) * 32 + cl) * VE + e % VE;
          pk = make_pack(pendf[lane * 16 + e], id_base + static_cast<uint32_t>(off));
        }
        if (offer(has, pk, hist) && has) sb &= sb - 1u;
      }
      pend_n = 0;
      __syncwarp();
    };
    auto rescale = [&](float mt) {  // warp-uniform
      if (mt > m_t) {
        if (m_t > -INFINITY) s_t = __dmul_rn(s_t, exp2(__dmul_rn(static_cast<double>(m_t) - static_cast<double>(mt), a2)));
        m_t = mt;
        m_lim = m_t + dlim;
      }
    };

    // Dead bits of tile t (penalised ids): bit sub*16 + j*VE + i of the owning lane.  The
    // sorted list is walked by the whole warp (its next entry is the same for every lane).
    auto dead_bits = [&](int t0, int cnt) -> uint32_t {
      uint32_t dead = 0u;
      auto mark = [&](int e) {  // element e of the tile
        const int vi = e / VE;
        if ((vi & 31) == lane) dead |= 1u << ((vi >> 5) / VPS * 16 + ((vi >> 5) % VPS) * VE + e % VE);
      };
      if (pen_scan) {
        for (int64_t j = 0; j < hl; ++j) {
          const int64_t off = static_cast<int64_t>(hrow[j]) - A.vocab_offset - glo - t0;
          if (off >= 0 && off < cnt) mark(static_cast<int>(off));
        }
      } else {
        while (pen_cur < pen_n) {
          const uint32_t off = pen[pen_cur];
          if (off >= static_cast<uint32_t>(t0 + cnt)) break;
          mark(static_cast<int>(off) - t0);
          ++pen_cur;
        }
      }
      return dead;
    };

    // ---- the unit's full tiles: kDStages - 1 in flight while one is worked on ----
    unsigned long long rt_next = rtau && k_eff > 1 ? *reinterpret_cast<volatile unsigned long long*>(rtau) : 0ull;
    uint32_t rd = ring0;
    unsigned char* const ring_lane = ring + lane * 16;
    for (int t = 0; t < nfull; ++t) {
      issue();  // (into the stage read at t - 1)
      asm volatile("cp.async.wait_group %0;" ::"n"(kDStages - 1) : "memory");
      unsigned char* st = ring_lane + (rd - ring0);    // this lane's slot of the stage read now
      unsigned* sthist = reinterpret_cast<unsigned*>(ring + (rd - ring0));  // the stage as scratch (1 KB)
      if (rtau && k_eff > 1) {  // the row's shared bound, read one tile ahead
        set_tau(rt_next);
        rt_next = *reinterpret_cast<volatile unsigned long long*>(rtau);
      }
      uint32_t dead = 0u;
      const bool dead_tile = t == dead_t;  // (warp-uniform)
      if (dead_tile) {
        dead = dead_bits(t * TE, TE);
        dead_t = pen_scan ? t + 1 : (pen_cur < pen_n ? static_cast<int>(pen[pen_cur] / TE) : INT_MAX);
      }
      uint4 raw[VPT];  // this lane's vectors of the tile
#pragma unroll
      for (int j = 0; j < VPT; ++j) raw[j] = *reinterpret_cast<const uint4*>(st + j * 512);
#pragma unroll
      for (int sub = 0; sub < NSUB; ++sub) {
        const uint32_t dsub = (dead >> (sub * 16)) & 0xffffu;
        float x[VPS][VE];
#pragma unroll
        for (int j = 0; j < VPS; ++j) LD::vec(reinterpret_cast<const unsigned char*>(&raw[sub * VPS + j]), x[j]);
        bool rbad = false;  // a value outside the polynomial's range, an infinity or a NaN
        if (cap != 0.0f) {
          float2 za = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int j = 0; j < VPS; ++j)
#pragma unroll
            for (int i = 0; i < VE; i += 2) {
              float2 z;
              const float2 c = softcap2_poly(make_float2(x[j][i], x[j][i + 1]), cap, inv_cap, &z);
              x[j][i] = c.x;
              x[j][i + 1] = c.y;
              za = __fadd2_rn(za, z);  // (every z >= 0: a sum below 1 bounds each one)
            }
          rbad = !(za.x + za.y < kSoftcapPolyZ);
        } else {
          float2 xa = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int j = 0; j < VPS; ++j)
#pragma unroll
            for (int i = 0; i < VE; i += 2) xa = __fadd2_rn(xa, make_float2(x[j][i], x[j][i + 1]));
          rbad = !(fabsf(xa.x + xa.y) < INFINITY);  // a NaN or an infinity (or a huge sum)
        }
        if (__any_sync(kFullMask, rbad)) {
          // out-of-range values -> the full routine, NaN -> error
#pragma unroll
          for (int j = 0; j < VPS; ++j) {
            float r[VE];
            if constexpr (DT == GS_DTYPE_F32) {
              LD::vec(st + j * 512, r);  // (f32: the stage still holds the raw tile)
            } else {
              LD::vec(reinterpret_cast<const unsigned char*>(&raw[sub * VPS + j]), r);
            }
#pragma unroll
            for (int i = 0; i < VE; ++i) {
              if (cap != 0.0f) {
                const float y = __fmul_rn(r[i], inv_cap);
                if (!(__fmul_rn(y, y) < kSoftcapPolyZ)) x[j][i] = dense_softcap_slow(r[i], cap, inv_cap);
              }
              if (x[j][i] != x[j][i] && !((dsub >> (j * VE + i)) & 1u)) bad |= 1u;
            }
          }
        }
        if (dead_tile && __any_sync(kFullMask, dsub != 0u)) {
          // penalised ids -> -inf (the vectors holding one)
#pragma unroll
          for (int j = 0; j < VPS; ++j)
            if ((dsub >> (j * VE)) & ((1u << VE) - 1u)) {
#pragma unroll
              for (int i = 0; i < VE; ++i)
                if ((dsub >> (j * VE + i)) & 1u) x[j][i] = -INFINITY;
            }
        }
        float tmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < VPS; ++j) {
          float m = x[j][0];
#pragma unroll
          for (int i = 1; i < VE; ++i) m = fmaxf(m, x[j][i]);
          tmax = fmaxf(tmax, m);
        }
        if (k_eff == 1) {
          if (tmax > bx || (bp == 0ull && tmax == tmax)) {
            // first live position of the lane's maximum (ids ascend with (j, i))
            int fj = -1, fi = 0;
#pragma unroll
            for (int j = VPS - 1; j >= 0; --j)
#pragma unroll
              for (int i = VE - 1; i >= 0; --i)
                if (!((dsub >> (j * VE + i)) & 1u) && x[j][i] == tmax) {
                  fj = j;
                  fi = i;
                }
            if (fj >= 0) {
              bx = tmax;
              bp = make_pack(tmax, id_base + static_cast<uint32_t>(t * TE + ((sub * VPS + fj) * 32 + lane) * VE + fi));
            }
          }
        } else if (k_eff > 1) {
          if (t == 0 && sub == 0) {
            // threshold from the unit's first 512 ids: the largest key K found by a binary
            // search such that at least k live values there are >= value(K)
            int c = 0;
#pragma unroll
            for (int j = 0; j < VPS; ++j)
#pragma unroll
              for (int i = 0; i < VE; ++i) c += x[j][i] > -INFINITY ? 1 : 0;
            const int nlv = static_cast<int>(__reduce_add_sync(kFullMask, static_cast<unsigned>(c)));
            if (nlv >= k_eff) {
              const uint32_t kneg = key32(-INFINITY);
              uint32_t klo = kneg, khi = key32(warp_max(tmax)) + 1u;
#pragma unroll 1
              for (int it = 0; it < 14 && khi - klo > 1u; ++it) {
                const uint32_t mid = klo + ((khi - klo) >> 1);
                const float tv = key32_value(mid);  // > -inf: dead (-inf) and NaN values never count
                int cc = 0;
#pragma unroll
                for (int j = 0; j < VPS; ++j)
#pragma unroll
                  for (int i = 0; i < VE; ++i) cc += x[j][i] >= tv ? 1 : 0;
                cc = static_cast<int>(__reduce_add_sync(kFullMask, static_cast<unsigned>(cc)));
                if (cc >= k_eff) {
                  klo = mid;
                } else {
                  khi = mid;
                }
              }
              if (klo != kneg) {
                const unsigned long long t0b = (static_cast<unsigned long long>(klo) << 32) - 1ull;  // key >= klo
                set_tau(t0b);
                if (rtau && lane == 0) atomicMax(rtau, t0b);
              }
            }
          }
          // lanes whose maximum reaches the threshold queue their 16 values
          unsigned bq = __ballot_sync(kFullMask, tmax >= tau_x);
          while (bq) {
            if (pend_n == kDPend) flush(sthist);
            const int room = kDPend - pend_n;
            const int rank = __popc(bq & lane_lt);
            const bool go = ((bq >> lane) & 1u) && rank < room;
            if (go) {
              const int c = pend_n + rank;
              float4* pv = reinterpret_cast<float4*>(pendf + c * 16);
#pragma unroll
              for (int j = 0; j < VPS; ++j)
#pragma unroll
                for (int i = 0; i < VE; i += 4) pv[(j * VE + i) / 4] = make_float4(x[j][i], x[j][i + 1], x[j][i + 2], x[j][i + 3]);
              ptag[c] = static_cast<uint32_t>(t) << 8 | static_cast<uint32_t>(sub) << 5 | static_cast<uint32_t>(lane);
              pdead[c] = dsub;
            }
            const int nb = __popc(bq);
            pend_n += nb < room ? nb : room;
            bq &= ~__ballot_sync(kFullMask, go);
          }
        }
        if (do_sum) {
          lmx = fmaxf(lmx, tmax);
          if (__any_sync(kFullMask, tmax > m_lim)) rescale(warp_max(tmax));
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
        } else {
          // no sum to carry a NaN: look for one explicitly
#pragma unroll
          for (int j = 0; j < VPS; ++j)
#pragma unroll
            for (int i = 0; i < VE; ++i)
              if (x[j][i] != x[j][i]) bad |= 1u;
        }
      }
      if (k_eff > 1 && wcnt > wcap) compact(sthist);
      __syncwarp();  // (the stage is refilled by the next issue)
      rd += kDTileBytes;
      if (rd == ring_end) rd = ring0;
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // (empty groups past the last tile)
    __syncwarp();
    unsigned* rhist = reinterpret_cast<unsigned*>(ring);  // the ring is idle from here on
    if (k_eff > 1 && pend_n > 0) flush(rhist);

    // Partial tile (the row's last, shorter than a tile): element by element from HBM.
    if (gn > nfull * TE) {
      const int t0 = nfull * TE, cnt = gn - nfull * TE;
      const uint32_t dead_unused = dead_bits(t0, cnt);  // (advances the penalty cursor)
      (void)dead_unused;
      auto live_at = [&](int64_t off) {
        bool live = true;
        if (pen_scan) {
          for (int64_t j = 0; j < hl; ++j) live &= static_cast<int64_t>(hrow[j]) - A.vocab_offset - glo != off;
        } else {
          for (int p = 0; p < pen_n; ++p) live &= pen[p] != static_cast<uint32_t>(off);
        }
        return live;
      };
      float tmx = -INFINITY;
      for (int i = lane; i < cnt; i += 32) {
        if (!live_at(t0 + i)) continue;
        float x = LD::global(rowp, t0 + i);
        if (cap != 0.0f) x = softcap(x, cap, inv_cap);
        if (x != x) bad |= 1u;
        tmx = fmaxf(tmx, x);
      }
      if (do_sum) {
        lmx = fmaxf(lmx, tmx);
        rescale(warp_max(tmx));
      }
      float acc = 0.0f;
      for (int i0 = 0; i0 < cnt; i0 += 32) {  // warp-uniform trip count
        const int i = i0 + lane;
        const bool live = i < cnt && live_at(t0 + i);
        float x = -INFINITY;
        if (live) {
          x = LD::global(rowp, t0 + i);
          if (cap != 0.0f) x = softcap(x, cap, inv_cap);
          if (do_sum && m_t > -INFINITY) {
            const float d = x - m_t;
            acc += ex2_approx(fmaf(d, a2_lo, d * a2_hi));
          }
        }
        const uint32_t id = id_base + static_cast<uint32_t>(t0 + i);
        if (k_eff == 1) {
          if (live && x == x) {
            const unsigned long long pk = make_pack(x, id);
            if (pk > bp) {
              bp = pk;
              bx = x;
            }
          }
        } else if (k_eff > 1) {
          bool pend = live && x >= tau_x;
          const unsigned long long pk = pend ? make_pack(x, id) : 0ull;
          while (__any_sync(kFullMask, pend)) pend = !offer(pend, pk, rhist);
        }
      }
      s_t += static_cast<double>(acc);
    }

    // ---- unit outputs ----
    __syncwarp();
    UnitStat* out = A.stats + unit;
    int ncand = 0;
    if (k_eff > 1) {
      if (wcnt > k_eff) compact(rhist);
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
    const uint32_t wbad = __reduce_or_sync(kFullMask, bad);
    if (lane == 0) {
      uint32_t fl = 0u;
      if (wbad || c != c || m_t == INFINITY) fl |= GS_FLAG_ERR_NONFINITE;
      out->m = m_t;
      out->s = m_t > -INFINITY ? c : 0.0;
      out->raw_m = -INFINITY;
      out->raw_s = 0.0;
      out->n_allowed = gn;
      out->n_cand = ncand;
      out->flags = fl;
    }
    __syncwarp();
  }
}

// The dense kernel serves a batch when no row can be constrained or wants the raw sums.
bool dense_eligible(const StreamArgs& a, int dtype) {
  const int esz = dtype == GS_DTYPE_F32 ? 4 : 2;
  if (a.mask_table != nullptr || a.want_raw || a.kmax > kDMaxK) return false;
  if (reinterpret_cast<uintptr_t>(a.logits) & 15) return false;
  if ((a.row_stride * esz) & 15) return false;
  if (a.chunk % 1024) return false;
  return true;
}

cudaError_t launch_dense(const StreamArgs& a, int dtype, int rows, cudaStream_t st, int num_sms) {
  const int units = rows * a.splits;
  if (units == 0) return cudaSuccess;
  // batches with fewer units than the GPU's warp slots spread them over every SM
  int wpc = kDWarps;
  if (units < num_sms * kDWarps) wpc = (units + num_sms - 1) / num_sms;
  int grid = (units + wpc - 1) / wpc;
  if (grid > num_sms) grid = num_sms;
  const size_t smem = static_cast<size_t>(wpc) * kDWarpBytes;
  if (dtype == GS_DTYPE_F32) {
    cudaError_t e = cudaFuncSetAttribute(dense_kernel<GS_DTYPE_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dense_kernel<GS_DTYPE_F32><<<grid, wpc * 32, smem, st>>>(a, units);
  } else {
    cudaError_t e = cudaFuncSetAttribute(dense_kernel<GS_DTYPE_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dense_kernel<GS_DTYPE_BF16><<<grid, wpc * 32, smem, st>>>(a, units);
  }
  return cudaGetLastError();
}

}  // namespace gs
