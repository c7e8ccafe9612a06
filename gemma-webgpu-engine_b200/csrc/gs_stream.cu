// Kernel 1: the fused streaming pass.
//
// One CTA handles one unit = (row, vocabulary chunk).  It reads the chunk of logits once
// with 128-bit coalesced loads and, per element: applies the soft cap, drops ids the
// row's constraint state forbids (the per-state bitmask, staged into shared memory with
// a TMA bulk copy) and ids that appear in the row's penalty history (their exact double
// values are computed by kernel 2), keeps an online max / sum-exp of e^(x/T), and
// offers the element to a shared-memory top-k candidate buffer guarded by a threshold.
//
// Reference semantics it serves (aribornstein/gemma-webgpu-engine):
//   src/runtime/sampling.ts:20      f32 -> f64 widening (exact; candidates keep the f32)
//   src/runtime/sampling.ts:26-30   penalties: history ids are excluded here, done in kernel 2
//   src/runtime/sampling.ts:33-35   sort by logit/T desc, lower id first: pack = key32(x)<<32 | ~id
//   src/runtime/sampling.ts:36-41   full-vocabulary sum of exp(x/T - max): per-unit (m, s)
//   src/runtime/constraints.ts:159-173 masked ids are -inf: excluded from the stream
#include "gs_device.cuh"
#include "gs_block.cuh"
#include "gs_internal.cuh"
#include "../../include/gsampler.h"

#include <cfloat>

namespace gs {

struct StreamShared {
  unsigned long long bar;
  unsigned long long tau;
  int count;
  int overflow;
  unsigned int flags;
  int n_allowed;
  unsigned int hist[256];
  int sel_digit;
  int sel_above;
  int sel_binc;
  float red_f[32];
  float red_f2[32];
  double red_d[32];
  double red_d2[32];
};

template <int DT>
struct Vec;
template <>
struct Vec<GS_DTYPE_F32> {
  static constexpr int kElems = 4;
  using T = float4;
  static __device__ __forceinline__ T load(const void* base, int64_t vi) {
    return ld_stream_f4(static_cast<const float4*>(base) + vi);
  }
  static __device__ __forceinline__ float get(const T& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
  }
};
template <>
struct Vec<GS_DTYPE_BF16> {
  static constexpr int kElems = 8;
  using T = uint4;
  static __device__ __forceinline__ T load(const void* base, int64_t vi) {
    return ld_stream_u4(static_cast<const uint4*>(base) + vi);
  }
  static __device__ __forceinline__ float get(const T& v, int i) {
    const uint32_t w = (i >> 1) == 0 ? v.x : (i >> 1) == 1 ? v.y : (i >> 1) == 2 ? v.z : v.w;
    return (i & 1) ? bf16_hi(w) : bf16_lo(w);
  }
};

struct ThreadAcc {
  float m;
  double s;
  float rm;
  double rs;
  uint32_t bad;
};

// log2(e) split as hi (rounded toward zero) + lo, for 2^((x - m)·log2 e) = e^(x - m).
constexpr float kLog2eHi = 1.44269502162933349609375f;
constexpr float kLog2eLo = 1.925963033500011e-08f;

__device__ __forceinline__ float apply_cap(float x, float cap, float inv_cap) {
  return cap != 0.0f ? softcap(x, cap, inv_cap) : x;
}

template <int N>
__device__ __forceinline__ void raw_update(const float (&x)[N], ThreadAcc& acc) {
  float vmax = -INFINITY;
#pragma unroll
  for (int i = 0; i < N; ++i) vmax = fmaxf(vmax, x[i]);
  if (vmax > acc.rm) {
    if (acc.rm > -INFINITY) acc.rs = __dmul_rn(acc.rs, exp(static_cast<double>(acc.rm) - static_cast<double>(vmax)));
    acc.rm = vmax;
  }
  if (acc.rm > -INFINITY) {
    float e = 0.0f;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const float d = x[i] - acc.rm;
      e += ex2_approx(fmaf(d, kLog2eLo, d * kLog2eHi));
    }
    acc.rs += static_cast<double>(e);
  }
}

template <int DT>
__global__ void __launch_bounds__(kStreamThreads, 2) stream_kernel(const __grid_constant__ StreamArgs A) {
  using VT = Vec<DT>;
  constexpr int VE = VT::kElems;
  constexpr int U = 4;  // 16-byte loads in flight per thread per iteration
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ StreamShared S;

  const int tid = threadIdx.x;
  const int bs = blockDim.x;
  const int unit = blockIdx.x;
  const int row = unit / A.splits;
  const int part = unit - row * A.splits;
  const RowPlan* pp = A.plans ? A.plans + row : &A.plan0;
  const int mode = pp->mode;
  if (mode == kModeLarge) return;  // the histogram kernel takes this row's statistics
  const int k_eff = pp->k_eff;
  const double a2 = pp->a2;
  const float a2_hi = pp->a2_hi;
  const float a2_lo = pp->a2_lo;
  const bool do_sum = mode != kModeGreedy;
  const float cap = A.softcap, inv_cap = A.inv_softcap;
  const bool want_raw = A.want_raw != 0;

  const int64_t lo = static_cast<int64_t>(part) * A.chunk;
  const int64_t hi = lo + A.chunk < A.vocab ? lo + A.chunk : A.vocab;
  const int64_t n = hi > lo ? hi - lo : 0;
  const int nwords = static_cast<int>((n + 31) >> 5);
  const int nwords_pad = (static_cast<int>((A.chunk + 31) >> 5) + 3) & ~3;
  uint32_t* live = reinterpret_cast<uint32_t*>(dsm);
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(dsm + static_cast<size_t>(nwords_pad) * 4);
  const int KC = A.kc;

  if (tid == 0) {
    S.tau = 0;
    S.count = 0;
    S.overflow = 0;
    S.flags = 0;
    S.n_allowed = 0;
  }

  // ---- allowed-token bitmask of the row's constraint state (TMA bulk copy) ----------
  const int32_t state = A.mask_state ? A.mask_state[row] : -1;
  bool masked = A.mask_table != nullptr && state >= 0;
  if (masked && state >= A.mask_states) {
    masked = false;
    if (tid == 0) S.flags |= GS_FLAG_ERR_INVALID;
  }
  if (masked) {
    const uint32_t* src = A.mask_table + static_cast<int64_t>(state) * A.mask_words + (lo >> 5);
    const int nb = nwords & ~3;
    const bool tma = nb > 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
    if (tma) {
      if (tid == 0) mbar_init(reinterpret_cast<uint64_t*>(&S.bar), 1);
      __syncthreads();
      if (tid == 0) {
        mbar_expect_tx(reinterpret_cast<uint64_t*>(&S.bar), static_cast<uint32_t>(nb) * 4u);
        bulk_g2s(live, src, static_cast<uint32_t>(nb) * 4u, reinterpret_cast<uint64_t*>(&S.bar));
      }
      for (int w = nb + tid; w < nwords; w += bs) live[w] = __ldg(src + w);
      if (!mbar_wait(reinterpret_cast<uint64_t*>(&S.bar), 0, kWaitNs)) {
        atomicOr(&S.flags, GS_FLAG_ERR_TIMEOUT);
        mbar_wait(reinterpret_cast<uint64_t*>(&S.bar), 0, kWaitNs);  // let the copy land
      }
    } else {
      for (int w = tid; w < nwords; w += bs) live[w] = __ldg(src + w);
    }
  } else {
    for (int w = tid; w < nwords; w += bs) live[w] = 0xffffffffu;
  }
  __syncthreads();
  if (tid == 0 && nwords > 0 && (n & 31) != 0) live[nwords - 1] &= (1u << (n & 31)) - 1u;
  __syncthreads();
  {
    int na = 0;
    for (int w = tid; w < nwords; w += bs) na += __popc(live[w]);
    na = warp_sum_i(na);
    if ((tid & 31) == 0 && na) atomicAdd(&S.n_allowed, na);
  }
  __syncthreads();
  // ---- penalty history: those ids leave the stream (kernel 2 scores them in f64) ----
  {
    int64_t hl = A.history_len ? A.history_len[row] : 0;
    if (hl > A.history_stride) hl = A.history_stride;
    const int32_t* h = A.history + static_cast<int64_t>(row) * A.history_stride;
    for (int64_t j = tid; j < hl; j += bs) {
      const int64_t id = static_cast<int64_t>(h[j]) - A.vocab_offset - lo;
      if (id >= 0 && id < n) atomicAnd(&live[id >> 5], ~(1u << (id & 31)));
    }
  }
  __syncthreads();

  // ---- the stream ---------------------------------------------------------------
  const unsigned char* rowbase =
      static_cast<const unsigned char*>(A.logits) + (static_cast<int64_t>(row) * A.row_stride + lo) * (DT == GS_DTYPE_F32 ? 4 : 2);
  const bool vec_ok = (reinterpret_cast<uintptr_t>(rowbase) & 15) == 0;
  const int64_t nvec = vec_ok ? n / VE : 0;
  const uint32_t id_base = static_cast<uint32_t>(A.vocab_offset + lo);

  ThreadAcc acc{-INFINITY, 0.0, -INFINITY, 0.0, 0u};
  unsigned long long tau = 0;
  uint32_t tau_hi = 0;

  // Offers x (local offset off) to the candidate buffer; returns false when it must be
  // retried after a compaction.
  auto offer = [&](float x, int64_t off) -> bool {
    const unsigned long long pk = make_pack(x, id_base + static_cast<uint32_t>(off));
    if (pk <= tau) return true;
    const int pos = atomicAdd(&S.count, 1);
    if (pos < KC) {
      cand[pos] = pk;
      return true;
    }
    S.overflow = 1;
    return false;
  };

  // Processes N consecutive elements starting at local offset off; bit i of *pend is set
  // for elements that could not be inserted yet.
  auto process = [&](const float (&xin)[VE], int nvalid, int64_t off, uint32_t& pend) {
    const uint32_t word = live[off >> 5];
    uint32_t bits = (word >> (off & 31)) & ((1u << VE) - 1u);
    if (nvalid < VE) bits &= (1u << nvalid) - 1u;
    if (!want_raw && bits == 0) return;
    float x[VE];
#pragma unroll
    for (int i = 0; i < VE; ++i) x[i] = apply_cap(xin[i], cap, inv_cap);
    if (want_raw) {
      float xr[VE];
#pragma unroll
      for (int i = 0; i < VE; ++i) xr[i] = i < nvalid ? x[i] : -INFINITY;
      raw_update<VE>(xr, acc);
    }
    if (bits == 0) return;
    float vmax = -INFINITY;
    float xl[VE];
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      const bool l = (bits >> i) & 1u;
      xl[i] = l ? x[i] : -INFINITY;
      vmax = fmaxf(vmax, xl[i]);
      if (l && !(x[i] < INFINITY)) acc.bad |= 1u;  // NaN or +inf
    }
    if (do_sum) {
      if (vmax > acc.m) {
        if (acc.m > -INFINITY)
          acc.s = __dmul_rn(acc.s, exp2(__dmul_rn(static_cast<double>(acc.m) - static_cast<double>(vmax), a2)));
        acc.m = vmax;
      }
      if (acc.m > -INFINITY) {
        float e = 0.0f;
#pragma unroll
        for (int i = 0; i < VE; ++i) {
          const float d = xl[i] - acc.m;
          e += ex2_approx(fmaf(d, a2_lo, d * a2_hi));
        }
        acc.s += static_cast<double>(e);
      }
    }
    if (k_eff > 0 && key32(vmax) >= tau_hi) {
#pragma unroll
      for (int i = 0; i < VE; ++i)
        if ((bits >> i) & 1u)
          if (!offer(x[i], off + i)) pend |= 1u << i;
    }
  };

  // Compacts the candidate buffer to the k_eff best (radix select), raising tau.
  auto compact = [&]() {
    __syncthreads();
    const int cnt = S.count < KC ? S.count : KC;
    if (cnt > k_eff) {
      unsigned long long prefix, mask;
      select_threshold(cand, cnt, k_eff, S.hist, &S.sel_digit, &S.sel_above, &S.sel_binc, prefix, mask);
      unsigned long long mine[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int idx = tid + r * bs;
        mine[r] = idx < cnt ? cand[idx] : 0ull;
      }
      __syncthreads();
      if (tid == 0) {
        S.count = 0;
        S.tau = ~0ull;
      }
      __syncthreads();
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int idx = tid + r * bs;
        if (idx < cnt && (mine[r] & mask) >= prefix) {
          const int pos = atomicAdd(&S.count, 1);
          cand[pos] = mine[r];
          atomicMin(&S.tau, mine[r]);
        }
      }
    } else if (tid == 0) {
      S.count = cnt;
    }
    __syncthreads();
    if (tid == 0) S.overflow = 0;
    __syncthreads();
    tau = S.tau;
    tau_hi = static_cast<uint32_t>(tau >> 32);
  };

  for (int64_t base = 0; base < nvec; base += static_cast<int64_t>(bs) * U) {
    typename VT::T v[U];
    uint32_t pend[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t vi = base + static_cast<int64_t>(u) * bs + tid;
      pend[u] = 0;
      if (vi < nvec) v[u] = VT::load(rowbase, vi);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t vi = base + static_cast<int64_t>(u) * bs + tid;
      if (vi < nvec) {
        float xin[VE];
#pragma unroll
        for (int i = 0; i < VE; ++i) xin[i] = VT::get(v[u], i);
        process(xin, VE, vi * VE, pend[u]);
      }
    }
    if (k_eff > 0) {
      __syncthreads();
      while (S.overflow) {
        compact();
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (pend[u]) {
            const int64_t vi = base + static_cast<int64_t>(u) * bs + tid;
            uint32_t still = 0;
#pragma unroll
            for (int i = 0; i < VE; ++i)
              if ((pend[u] >> i) & 1u)
                if (!offer(apply_cap(VT::get(v[u], i), cap, inv_cap), vi * VE + i)) still |= 1u << i;
            pend[u] = still;
          }
        }
        __syncthreads();
      }
      tau = S.tau;
      tau_hi = static_cast<uint32_t>(tau >> 32);
    }
  }
  // Scalar remainder (and whole rows whose base is not 16-byte aligned).
  const float* rowf = reinterpret_cast<const float*>(rowbase);
  const unsigned short* rowh = reinterpret_cast<const unsigned short*>(rowbase);
  for (int64_t base = nvec * VE; base < n; base += static_cast<int64_t>(bs) * VE) {
    const int64_t off0 = base + static_cast<int64_t>(tid) * VE;
    float xin[VE];
    int nvalid = 0;
    uint32_t pend = 0;
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      const int64_t o = off0 + i;
      if (o < n) {
        xin[i] = DT == GS_DTYPE_F32 ? __ldg(rowf + o) : __uint_as_float(static_cast<uint32_t>(__ldg(rowh + o)) << 16);
        nvalid = i + 1;
      } else {
        xin[i] = -INFINITY;
      }
    }
    // off0 is a multiple of VE (<= 8), so the VE bits never straddle a mask word.
    if (nvalid > 0) process(xin, nvalid, off0, pend);
    if (k_eff > 0) {
      __syncthreads();
      while (S.overflow) {
        compact();
        uint32_t still = 0;
#pragma unroll
        for (int i = 0; i < VE; ++i)
          if ((pend >> i) & 1u)
            if (!offer(apply_cap(xin[i], cap, inv_cap), off0 + i)) still |= 1u << i;
        pend = still;
        __syncthreads();
      }
      tau = S.tau;
      tau_hi = static_cast<uint32_t>(tau >> 32);
    }
  }

  // ---- unit outputs ----------------------------------------------------------------
  UnitStat* out = A.stats + unit;
  if (k_eff > 0) {
    compact();
    const int nc = S.count < k_eff ? S.count : k_eff;
    unsigned long long* dst = A.cands + static_cast<int64_t>(unit) * A.kcap;
    for (int i = tid; i < nc; i += bs) dst[i] = cand[i];
    if (tid == 0) out->n_cand = nc;
  } else if (tid == 0) {
    out->n_cand = 0;
  }
  const int warp = tid >> 5, lane = tid & 31, nwarps = bs >> 5;
  // block max of m and raw m
  float wm = warp_max(acc.m), wrm = warp_max(acc.rm);
  if (lane == 0) {
    S.red_f[warp] = wm;
    S.red_f2[warp] = wrm;
  }
  __syncthreads();
  float M = -INFINITY, RM = -INFINITY;
  for (int w = 0; w < nwarps; ++w) {
    M = fmaxf(M, S.red_f[w]);
    RM = fmaxf(RM, S.red_f2[w]);
  }
  double c = acc.m > -INFINITY ? __dmul_rn(acc.s, exp2(__dmul_rn(static_cast<double>(acc.m) - static_cast<double>(M), a2))) : 0.0;
  double rc = acc.rm > -INFINITY ? __dmul_rn(acc.rs, exp(static_cast<double>(acc.rm) - static_cast<double>(RM))) : 0.0;
  c = warp_sum(c);
  rc = warp_sum(rc);
  const unsigned bad = __any_sync(kFullMask, acc.bad != 0) ? 1u : 0u;
  if (lane == 0) {
    S.red_d[warp] = c;
    S.red_d2[warp] = rc;
    if (bad) atomicOr(&S.flags, GS_FLAG_ERR_NONFINITE);
  }
  __syncthreads();
  if (tid == 0) {
    double s = 0.0, rs = 0.0;
    for (int w = 0; w < nwarps; ++w) {
      s = __dadd_rn(s, S.red_d[w]);
      rs = __dadd_rn(rs, S.red_d2[w]);
    }
    unsigned fl = S.flags;
    if (s != s || rs != rs || M == INFINITY) fl |= GS_FLAG_ERR_NONFINITE;
    out->m = M;
    out->s = s;
    out->raw_m = RM;
    out->raw_s = rs;
    out->n_allowed = S.n_allowed;
    out->flags = fl;
  }
}

size_t stream_smem_bytes(int64_t chunk, int kc) {
  const size_t nwords_pad = (static_cast<size_t>((chunk + 31) >> 5) + 3) & ~static_cast<size_t>(3);
  return nwords_pad * 4 + static_cast<size_t>(kc) * 8;
}

bool stream2_eligible(const StreamArgs& a, int dtype, int rows);
int pipe_max_k();
size_t stream2_smem_bytes(int64_t chunk);
cudaError_t launch_stream2(const StreamArgs& a, int dtype, int rows, size_t smem, cudaStream_t st, int num_sms);

int sm_count() {
  static int counts[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!counts[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = n > 0 ? n : 148;
  }
  return counts[dev];
}
bool dense_eligible(const StreamArgs& a, int dtype);
cudaError_t launch_dense(const StreamArgs& a, int dtype, int rows, cudaStream_t st, int num_sms);

cudaError_t launch_stream(const StreamArgs& a, int dtype, int rows, size_t smem, cudaStream_t st) {
  const int units = rows * a.splits;
  if (units == 0) return cudaSuccess;
  // unconstrained batches without raw sums: the dense kernel; other aligned small-topK
  // batches: the warp-pipelined kernel; the general kernel otherwise
  if (a.kmax <= pipe_max_k() && dense_eligible(a, dtype)) return launch_dense(a, dtype, rows, st, sm_count());
  if (a.kmax <= pipe_max_k() && stream2_eligible(a, dtype, rows))
    return launch_stream2(a, dtype, rows, stream2_smem_bytes(a.chunk), st, sm_count());
  if (dtype == GS_DTYPE_F32) {
    static std::atomic<uint64_t> attr{0};  // (set on each device's first call)
    if (device_todo(attr)) {
      cudaFuncSetAttribute(stream_kernel<GS_DTYPE_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      mark_device_done(attr);
    }
    stream_kernel<GS_DTYPE_F32><<<units, kStreamThreads, smem, st>>>(a);
  } else {
    static std::atomic<uint64_t> attr{0};  // (set on each device's first call)
    if (device_todo(attr)) {
      cudaFuncSetAttribute(stream_kernel<GS_DTYPE_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      mark_device_done(attr);
    }
    stream_kernel<GS_DTYPE_BF16><<<units, kStreamThreads, smem, st>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace gs
