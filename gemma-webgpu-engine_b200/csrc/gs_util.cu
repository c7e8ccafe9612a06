// Small kernels behind the auxiliary C-ABI entry points.
#include "gs_device.cuh"
#include "gs_block.cuh"
#include "gs_internal.cuh"
#include "../../include/gsampler.h"

namespace gs {

// tokenLogProbability (src/runtime/sampling.ts:67-80): x[tok] - max - log(sum exp(x - max))
// over the (soft-capped) raw logits of each row.  One CTA per row.
__global__ void __launch_bounds__(512) logprob_kernel(const void* logits, int dtype, int64_t vocab, int64_t stride,
                                                      float cap, float inv_cap, const int32_t* tokens, double* out) {
  __shared__ double red[32];
  __shared__ float redf[32];
  const int row = blockIdx.x;
  const unsigned char* base = static_cast<const unsigned char*>(logits) + static_cast<int64_t>(row) * stride * (dtype == GS_DTYPE_F32 ? 4 : 2);
  float m = -INFINITY;
  for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) {
    float x = load_logit(base, dtype, i);
    if (cap != 0.0f) x = softcap(x, cap, inv_cap);
    m = fmaxf(m, x);
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) redf[threadIdx.x >> 5] = m;
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < (blockDim.x >> 5); ++w) M = fmaxf(M, redf[w]);
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) {
    float x = load_logit(base, dtype, i);
    if (cap != 0.0f) x = softcap(x, cap, inv_cap);
    s = __dadd_rn(s, exp(static_cast<double>(x) - static_cast<double>(M)));
  }
  s = block_sum_d(s, red);
  if (threadIdx.x == 0) {
    float x = load_logit(base, dtype, tokens[row]);
    if (cap != 0.0f) x = softcap(x, cap, inv_cap);
    out[row] = __dsub_rn(__dsub_rn(static_cast<double>(x), static_cast<double>(M)), log(s));
  }
}

cudaError_t launch_logprob(const void* logits, int dtype, int rows, int64_t vocab, int64_t stride, float softcap_v,
                           float inv_softcap, const int32_t* tokens, double* out, int32_t* /*bad*/, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  logprob_kernel<<<rows, 512, 0, st>>>(logits, dtype, vocab, stride, softcap_v, inv_softcap, tokens, out);
  return cudaGetLastError();
}

// maskConstraintLogits (src/runtime/constraints.ts:159-173).
__global__ void fill_neg_inf(float* out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = -INFINITY;
}
__global__ void copy_ids(const float* raw, int64_t vocab, const int32_t* ids, int64_t n, float* out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t t = ids[i];
    if (t >= 0 && t < vocab) out[t] = raw[t];
  }
}

cudaError_t launch_mask_logits(const float* raw, int64_t vocab, const int32_t* legal, int64_t nl, const int32_t* term,
                               int64_t nt, float* out, cudaStream_t st) {
  if (vocab > 0) fill_neg_inf<<<296, 256, 0, st>>>(out, vocab);
  if (nl > 0) copy_ids<<<148, 256, 0, st>>>(raw, vocab, legal, nl, out);
  if (nt > 0) copy_ids<<<148, 256, 0, st>>>(raw, vocab, term, nt, out);
  return cudaGetLastError();
}

__global__ void set_bits(int64_t vocab, const int32_t* ids, int64_t n, uint32_t* row) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t t = ids[i];
    if (t >= 0 && t < vocab) atomicOr(row + (t >> 5), 1u << (t & 31));
  }
}

cudaError_t launch_build_mask_row(int64_t vocab, const int32_t* legal, int64_t nl, const int32_t* term, int64_t nt,
                                  uint32_t* row, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(row, 0, static_cast<size_t>((vocab + 31) >> 5) * 4, st);
  if (e != cudaSuccess) return e;
  if (nl > 0) set_bits<<<148, 256, 0, st>>>(vocab, legal, nl, row);
  if (nt > 0) set_bits<<<148, 256, 0, st>>>(vocab, term, nt, row);
  return cudaGetLastError();
}

// maskReasoningLogits (src/runtime/gemma-session.ts:1331-1345) as two bitmask rows: row 0
// allows the ids with token bytes, row 1 also the end-of-channel id.  One thread per id,
// one warp ballot per word.
__global__ void reasoning_rows_kernel(int64_t vocab, const uint8_t* has_bytes, int32_t end_id, uint32_t* rows,
                                      int64_t words) {
  const int64_t n = words * 32;
  for (int64_t i0 = blockIdx.x * static_cast<int64_t>(blockDim.x); i0 < n; i0 += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = i0 + threadIdx.x;  // (trip count uniform over the warp: n is a multiple of 32)
    const bool b = i < vocab && has_bytes[i] != 0;
    const uint32_t w = __ballot_sync(kFullMask, b);
    if ((threadIdx.x & 31) == 0) {
      const int64_t wi = i >> 5;
      uint32_t w1 = w;
      if (end_id >= 0 && end_id < vocab && (end_id >> 5) == wi) w1 |= 1u << (end_id & 31);
      rows[wi] = w;
      rows[words + wi] = w1;
    }
  }
}

cudaError_t launch_reasoning_rows(int64_t vocab, const uint8_t* has_bytes, int32_t end_id, uint32_t* rows,
                                  int64_t words, cudaStream_t st) {
  if (words > 0) reasoning_rows_kernel<<<148 * 4, 256, 0, st>>>(vocab, has_bytes, end_id, rows, words);
  return cudaGetLastError();
}

__global__ void softcap_kernel(const float* in, float* out, int64_t n, float cap, float inv_cap) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = softcap(in[i], cap, inv_cap);
}

cudaError_t launch_softcap(const float* in, float* out, int64_t n, float cap, float inv_cap, cudaStream_t st) {
  if (n > 0) softcap_kernel<<<148 * 8, 256, 0, st>>>(in, out, n, cap, inv_cap);
  return cudaGetLastError();
}

// Order-independent digest of softcap over float bit patterns [lo, hi): sum of a 64-bit
// mix of (input bits, output bits), NaN outputs canonicalised.
__global__ void softcap_digest_kernel(uint64_t lo, uint64_t hi, float cap, float inv_cap, unsigned long long* acc) {
  unsigned long long s = 0;
  for (uint64_t u = lo + blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; u < hi;
       u += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t xb = static_cast<uint32_t>(u);
    const float y = softcap(__uint_as_float(xb), cap, inv_cap);
    uint32_t yb = __float_as_uint(y);
    if (y != y) yb = 0x7fc00000u;
    uint64_t h = (static_cast<uint64_t>(xb) << 32) | yb;
    h ^= h >> 33;
    h *= 0xff51afd7ed558ccdULL;
    h ^= h >> 33;
    h *= 0xc4ceb9fe1a85ec53ULL;
    h ^= h >> 33;
    s += h;
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFullMask, s, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(acc, s);
}

cudaError_t launch_softcap_digest(uint64_t lo, uint64_t hi, float cap, float inv_cap, unsigned long long* acc,
                                  cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(acc, 0, sizeof(unsigned long long), st);
  if (e != cudaSuccess) return e;
  if (hi > lo) softcap_digest_kernel<<<148 * 16, 256, 0, st>>>(lo, hi, cap, inv_cap, acc);
  return cudaGetLastError();
}

}  // namespace gs
