// Block-level building blocks for the per-row kernels (sorts, scans, reductions).
#pragma once
#include "gs_device.cuh"

namespace gs {

// One candidate of a row: exact double sort key (logit/T, or the logit itself for
// temperature 0), token id, and whether it came from the penalty history.
struct Ent {
  double key;
  uint32_t id;
  uint32_t kind;  // 0 = streamed, 1 = penalised, 2 = masked fill, 0xffffffff = padding
};

// Reference order (src/runtime/sampling.ts:33-35): larger key first, lower id first.
__device__ __forceinline__ bool ent_before(const Ent& a, const Ent& b) {
  return a.key > b.key || (a.key == b.key && a.id < b.id);
}

// In-place bitonic sort of e[0, n2) (n2 a power of two) into ent_before order.
__device__ inline void bitonic_sort_ent(Ent* e, int n2) {
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n2; i += blockDim.x) {
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
      __syncthreads();
    }
  }
}

// Ascending bitonic sort of (key, payload) pairs by (key, payload).
__device__ inline void bitonic_sort_kv(unsigned long long* key, uint32_t* val, int n2) {
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n2; i += blockDim.x) {
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
      __syncthreads();
    }
  }
}

// Descending bitonic sort of n2 (a power of two, <= 128) packs held in registers, element
// q·32 + lane in v[q] (padding 0 sorts last): exchanges across lanes by shuffles, across a
// lane's registers by compile-time swaps.
static __device__ __forceinline__ void warp_sort_desc_regs(unsigned long long (&v)[4], int n2, int lane) {
  auto cx = [&](unsigned long long& a, unsigned long long& b, bool desc) {  // a: the lower index
    const bool sw = desc ? a < b : a > b;
    const unsigned long long t = a;
    a = sw ? b : a;
    b = sw ? t : b;
  };
  for (int k = 2; k <= n2; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j == 64) {
        cx(v[0], v[2], (lane & k) == 0);
        cx(v[1], v[3], ((32 + lane) & k) == 0);
      } else if (j == 32) {
        cx(v[0], v[1], (lane & k) == 0);
        if (n2 > 64) cx(v[2], v[3], ((64 + lane) & k) == 0);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (q * 32 < n2) {
            const unsigned long long p = __shfl_xor_sync(kFullMask, v[q], j);
            const int i = q * 32 + lane;
            const bool desc = (i & k) == 0, lo = (i & j) == 0;
            v[q] = desc == lo ? (v[q] > p ? v[q] : p) : (v[q] < p ? v[q] : p);
          }
        }
      }
    }
}

// Ascending block-wide sort of n2 (a power of two) 64-bit values, in shared or global
// memory (the block's own rows: __syncthreads orders both).
__device__ inline void bitonic_sort_u64(unsigned long long* v, int n2) {
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n2; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = v[i], b = v[ixj];
          const bool up = (i & k) == 0;
          if (up ? a > b : a < b) {
            v[i] = b;
            v[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Ascending sort of plain 32-bit values.
__device__ inline void bitonic_sort_u32(uint32_t* v, int n2) {
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n2; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint32_t a = v[i], b = v[ixj];
          const bool up = (i & k) == 0;
          if (up ? a > b : a < b) {
            v[i] = b;
            v[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Penalised value of one history id (src/runtime/sampling.ts:28-29), in double.
__device__ __forceinline__ double penalise(double x, double count, double rp, double pres, double freq) {
  double v = x < 0 ? __dmul_rn(x, rp) : __ddiv_rn(x, rp);
  return __dsub_rn(v, __dadd_rn(pres, __dmul_rn(count, freq)));
}

__device__ __forceinline__ int pow2_ceil(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

// Block-wide sum in a fixed order (deterministic).  `red` holds >= 32 doubles.
__device__ inline double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double s = 0.0;
  for (int w = 0; w < nw; ++w) s = __dadd_rn(s, red[w]);
  __syncthreads();
  return s;
}

// Block-wide maximum (fmaxf: NaN inputs are ignored).  `red` holds >= 32 floats.
__device__ inline float block_max_f(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = -INFINITY;
  for (int w = 0; w < nw; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  return m;
}

__device__ inline int block_sum_i(int v, int* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum_i(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int s = 0;
  for (int w = 0; w < nw; ++w) s += red[w];
  __syncthreads();
  return s;
}

// Inclusive prefix sums out[i] = in[0] + ... + in[i] for i < n (n <= 4·blockDim),
// each thread owning 4 consecutive items.  `red` holds >= 32 doubles.
__device__ inline void block_inclusive_scan_d(const double* in, double* out, int n, double* red) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = blockDim.x >> 5;
  double v[4];
  double run = 0.0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = 4 * t + j;
    run = __dadd_rn(run, i < n ? in[i] : 0.0);
    v[j] = run;
  }
  double incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double u = __shfl_up_sync(kFullMask, incl, o);
    if (lane >= o) incl = __dadd_rn(incl, u);
  }
  __syncthreads();
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  double wbase = 0.0;
  for (int w = 0; w < warp; ++w) wbase = __dadd_rn(wbase, red[w]);
  (void)nw;
  double excl = __shfl_up_sync(kFullMask, incl, 1);
  if (lane == 0) excl = 0.0;
  const double base = __dadd_rn(wbase, excl);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = 4 * t + j;
    if (i < n) out[i] = __dadd_rn(base, v[j]);
  }
  __syncthreads();
}

// Exclusive prefix count of flags (n <= 4·blockDim); returns the total.
__device__ inline int block_exclusive_count(const unsigned char* flag, int* pos, int n, int* red) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = blockDim.x >> 5;
  int c[4];
  int run = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = 4 * t + j;
    c[j] = run;
    run += (i < n && flag[i]) ? 1 : 0;
  }
  int incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(kFullMask, incl, o);
    if (lane >= o) incl += u;
  }
  __syncthreads();
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  int wbase = 0, total = 0;
  for (int w = 0; w < nw; ++w) {
    if (w < warp) wbase += red[w];
    total += red[w];
  }
  const int base = wbase + incl - run;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = 4 * t + j;
    if (i < n) pos[i] = base + c[j];
  }
  __syncthreads();
  return total;
}

// Threshold of the k largest non-zero values of buf[0, n) (zero slots are empty; at
// least k non-zero values): on return, the kept values are those with
// (v & mask) >= prefix.  MSB-first radix select with 8-bit digits, starting at the
// highest bit in which the non-zero values differ (the common high bits would put every
// value in one histogram bin), stopping as soon as the bin holding the k-th value is
// kept whole.  `hist` holds 256 counters; the s_* scalars are shared.
__device__ inline void select_threshold(const unsigned long long* buf, int n, int k, unsigned int* hist,
                                 int* s_digit, int* s_above, int* s_binc, unsigned long long& prefix,
                                 unsigned long long& mask) {
  __shared__ unsigned long long s_ref, s_dif;
  if (threadIdx.x == 0) {
    s_ref = 0;
    s_dif = 0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    if (buf[i] != 0ull) {
      atomicMax(&s_ref, buf[i]);
      break;
    }
  __syncthreads();
  const unsigned long long ref = s_ref;
  unsigned long long dif = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    if (buf[i] != 0ull) dif |= buf[i] ^ ref;
  dif |= __shfl_xor_sync(kFullMask, dif, 16);
  dif |= __shfl_xor_sync(kFullMask, dif, 8);
  dif |= __shfl_xor_sync(kFullMask, dif, 4);
  dif |= __shfl_xor_sync(kFullMask, dif, 2);
  dif |= __shfl_xor_sync(kFullMask, dif, 1);
  if ((threadIdx.x & 31) == 0 && dif) atomicOr(&s_dif, dif);
  __syncthreads();
  dif = s_dif;
  if (dif == 0ull) {  // one distinct non-zero value
    prefix = ref;
    mask = ~0ull;
    return;
  }
  const int hb = 63 - __clzll(static_cast<long long>(dif));
  mask = hb == 63 ? 0ull : (~0ull << (hb + 1));
  prefix = ref & mask;
  int shift = hb >= 7 ? hb - 7 : 0;
  int need = k;
  for (;;) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const unsigned long long v = buf[i];
      if (v != 0ull && (v & mask) == prefix) atomicAdd(&hist[(v >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      unsigned c[8];
      unsigned tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[255 - 8 * lane - j];
        tot += c[j];
      }
      unsigned incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_up_sync(kFullMask, incl, o);
        if (lane >= o) incl += t;
      }
      const unsigned excl = incl - tot;
      if (excl < static_cast<unsigned>(need) && static_cast<unsigned>(need) <= incl) {
        unsigned acc = excl;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (acc + c[j] >= static_cast<unsigned>(need)) {
            *s_digit = 255 - 8 * lane - j;
            *s_above = static_cast<int>(acc);
            *s_binc = static_cast<int>(c[j]);
            break;
          }
          acc += c[j];
        }
      }
    }
    __syncthreads();
    const int d = *s_digit, above = *s_above, binc = *s_binc;
    need -= above;
    // (with shift clamped to 0 the digit overlaps bits already in the prefix; the
    // counted values agree with it there, so the OR is consistent)
    prefix |= static_cast<unsigned long long>(d) << shift;
    mask |= 0xffull << shift;
    __syncthreads();
    if (binc == need || shift == 0) break;
    shift = shift >= 8 ? shift - 8 : 0;
  }
}

// Keeps the k largest of buf[0, n) (distinct values, k < n) at the front of buf, in
// order, and returns the smallest kept value (the k-th largest).  MSB-first radix select
// with 8-bit digits over a per-warp 256-bin histogram, starting at the highest bit in
// which the values differ (so the first digit already spreads them over the bins).
// Out of line (rare in the streaming pass); one copy per translation unit.
static __device__ __noinline__ unsigned long long warp_select_packs(unsigned long long* buf, int n, int k, unsigned* hist, int lane) {
  const unsigned long long ref = buf[0];
  unsigned long long dif = 0;
  for (int i = lane; i < n; i += 32) dif |= buf[i] ^ ref;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dif |= __shfl_xor_sync(kFullMask, dif, o);
  unsigned long long prefix, mask;
  if (dif == 0ull) {
    // all equal (not reached for distinct packs): keep the first k
    prefix = ref;
    mask = ~0ull;
  } else {
    const int hb = 63 - __clzll(static_cast<long long>(dif));
    mask = hb == 63 ? 0ull : (~0ull << (hb + 1));
    prefix = ref & mask;
    int shift = hb >= 7 ? hb - 7 : 0;
    int need = k;
    for (;;) {
#pragma unroll
      for (int j = 0; j < 8; ++j) hist[lane * 8 + j] = 0u;
      __syncwarp();
      for (int i = lane; i < n; i += 32) {
        const unsigned long long v = buf[i];
        if ((v & mask) == prefix) atomicAdd(&hist[(v >> shift) & 255u], 1u);
      }
      __syncwarp();
      // lane l owns digits 255-8l .. 248-8l (descending)
      unsigned c[8];
      unsigned tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[255 - 8 * lane - j];
        tot += c[j];
      }
      unsigned incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_up_sync(kFullMask, incl, o);
        if (lane >= o) incl += t;
      }
      const unsigned excl = incl - tot;
      int digit = -1, above = 0, binc = 0;
      if (excl < static_cast<unsigned>(need) && static_cast<unsigned>(need) <= incl) {
        unsigned acc = excl;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (digit < 0 && acc + c[j] >= static_cast<unsigned>(need)) {
            digit = 255 - 8 * lane - j;
            above = static_cast<int>(acc);
            binc = static_cast<int>(c[j]);
          }
          acc += c[j];
        }
      }
      const unsigned owner = __ballot_sync(kFullMask, digit >= 0);
      const int src = __ffs(owner) - 1;
      digit = __shfl_sync(kFullMask, digit, src);
      above = __shfl_sync(kFullMask, above, src);
      binc = __shfl_sync(kFullMask, binc, src);
      need -= above;
      // (when shift was clamped to 0 the digit overlaps bits already in the prefix; the
      // counted values agree with the prefix there, so the OR is consistent)
      prefix |= static_cast<unsigned long long>(digit) << shift;
      mask |= 0xffull << shift;
      __syncwarp();
      if (binc == need || shift == 0) break;
      shift = shift >= 8 ? shift - 8 : 0;
    }
  }
  // order-preserving compaction of the kept values to the front
  unsigned long long kth = ~0ull;
  int base = 0;
  for (int i0 = 0; i0 < n && base < k; i0 += 32) {
    const int i = i0 + lane;
    const unsigned long long v = i < n ? buf[i] : 0ull;
    const bool keep0 = i < n && (v & mask) >= prefix;
    const unsigned b0 = __ballot_sync(kFullMask, keep0);
    const int rank = __popc(b0 & ((1u << lane) - 1u));
    const bool keep = keep0 && base + rank < k;
    __syncwarp();
    if (keep) {
      buf[base + rank] = v;
      kth = v < kth ? v : kth;
    }
    base += __popc(b0);
    __syncwarp();
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(kFullMask, kth, o);
    kth = t < kth ? t : kth;
  }
  return kth;
}

}  // namespace gs
