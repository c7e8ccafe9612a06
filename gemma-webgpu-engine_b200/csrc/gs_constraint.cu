// Constraint bitmask builder: the per-state rows of the [S, mask_words] table that the
// sampler ANDs into the logits, built from a compiled DFA and the vocabulary's token
// bytes for every requested constraint state at once.
//
// Reference: CompiledGenerationConstraint.legalTokenIds (src/runtime/constraints.ts:56-92)
// walks a token-byte trie (src/runtime/token-byte-trie.ts:16-40) from the current state,
// moving byte by byte with transitionByte (:222-247; UTF-8 sequences are buffered as
// pending bytes and decoded to one code point) and keeping a token when every state
// reached after each of its bytes is viable (:254-267: the node can still reach a final
// node, or for pending bytes some completion leads to such a node).  selectConstrainedToken
// (src/runtime/gemma-session.ts:1315-1323) then adds the extra legal ids, removes the
// termination ids, and allows them again only when the state is accepting.
//
// Here every (state, token) pair is independent: one thread walks one token's bytes from
// one state, 32 consecutive tokens make one table word (a warp ballot), and a second
// kernel applies the extra / termination ids per state and flags rows that allow
// nothing (the reference's "tokenization dead end", gemma-session.ts:1324-1326).
#include <cstring>
#include <algorithm>
#include <string>
#include <vector>

#include "gs_device.cuh"
#include "gs_internal.cuh"
#include "gs_plan.cuh"
#include "../../include/gsampler.h"

struct gs_constraint {
  int device = 0;
  int32_t nodes = 0;
  int64_t vocab = 0;
  int64_t n_ranges = 0;
  // device copies
  int32_t* range_off = nullptr;   // [nodes + 1]
  uint32_t* range_lo = nullptr;   // [n_ranges]
  uint32_t* range_hi = nullptr;
  int32_t* range_target = nullptr;
  uint8_t* node_flags = nullptr;  // [nodes] bit 0 final, bit 1 viable
  uint32_t* tok_off = nullptr;    // [vocab + 1]
  uint8_t* tok_bytes = nullptr;
  int32_t* ascii = nullptr;       // [nodes][128] target of each ASCII character, -1: none
  uint4* tok16 = nullptr;         // [vocab] the first 16 bytes of each token
  uint16_t* tok_len = nullptr;    // [vocab] byte lengths (capped at 65535)
  // per-call staging (grown on demand)
  unsigned char* stage = nullptr;
  size_t stage_bytes = 0;
  std::string err;
};

namespace gs {
namespace {

constexpr int kWalkThreads = 256;
constexpr int kStatesPerBlock = 16;  // states one walk thread visits with its token's bytes in registers
constexpr int kPostThreads = 256;
constexpr int kMaxTokenBytes = 1 << 16;  // a longer token is rejected at set-up

struct DfaDev {
  const int32_t* ascii;  // [nodes][128]
  const int32_t* off;
  const uint32_t* lo;
  const uint32_t* hi;
  const int32_t* target;
  const uint8_t* flags;
  int32_t nodes;
};

struct StateDev {
  int32_t node;
  uint32_t pending;  // up to 3 pending bytes, first in the low byte
  int32_t plen;
  int32_t pad;
};

__device__ __forceinline__ bool node_viable(const DfaDev& D, int n) { return (D.flags[n] >> 1) & 1u; }

// Target of node n on code point c (transitionCharacter, constraints.ts:249-252): the
// range holding c, by binary search over the node's sorted ranges; -1 if none.
__device__ __forceinline__ int step_char(const DfaDev& D, int n, uint32_t c) {
  int l = D.off[n], h = D.off[n + 1];
  while (l < h) {
    const int m = (l + h) >> 1;
    if (D.hi[m] < c) l = m + 1;
    else h = m;
  }
  return (l < D.off[n + 1] && D.lo[l] <= c) ? D.target[l] : -1;
}

// Byte i of a packed pending sequence (first byte in the low byte).
__device__ __forceinline__ uint32_t pbyte(uint32_t p, int i) { return (p >> (8 * i)) & 0xffu; }

__device__ __forceinline__ uint32_t decode_cp(uint32_t b, int len) {
  uint32_t cp = pbyte(b, 0) & (len == 2 ? 0x1fu : len == 3 ? 0x0fu : 0x07u);
  for (int i = 1; i < len; ++i) cp = (cp << 6) | (pbyte(b, i) & 0x3fu);
  return cp;
}

// isViableConstraintState (constraints.ts:254-267) for a state with pending bytes: some
// out-range of the node whose target is viable meets the pending bytes' completion range
// (pendingUtf8CompletionRange, :269-292).
__device__ bool pending_viable(const DfaDev& D, int n, uint32_t p, int plen) {
  const uint32_t lead = pbyte(p, 0);
  const int len = lead <= 0xdf ? 2 : lead <= 0xef ? 3 : 4;
  if (plen == 0 || plen >= len) return false;
  const uint32_t second_min = lead == 0xe0 ? 0xa0 : lead == 0xf0 ? 0x90 : 0x80;
  const uint32_t second_max = lead == 0xed ? 0x9f : lead == 0xf4 ? 0x8f : 0xbf;
  if (plen > 1 && (pbyte(p, 1) < second_min || pbyte(p, 1) > second_max)) return false;
  for (int i = 2; i < plen; ++i)
    if (pbyte(p, i) < 0x80 || pbyte(p, i) > 0xbf) return false;
  uint32_t mn = p, mx = p;
  for (int i = plen; i < len; ++i) {
    mn |= (i == 1 ? second_min : 0x80u) << (8 * i);
    mx |= (i == 1 ? second_max : 0xbfu) << (8 * i);
  }
  const uint32_t cmin = decode_cp(mn, len), cmax = decode_cp(mx, len);
  // first range with hi >= cmin, then every range starting at or below cmax
  int l = D.off[n], h = D.off[n + 1];
  while (l < h) {
    const int m = (l + h) >> 1;
    if (D.hi[m] < cmin) l = m + 1;
    else h = m;
  }
  for (int r = l; r < D.off[n + 1] && D.lo[r] <= cmax; ++r)
    if (node_viable(D, D.target[r])) return true;
  return false;
}

// One byte through transitionByte (constraints.ts:222-247).  Returns false for null.
__device__ bool step_byte(const DfaDev& D, int& n, uint32_t& p, int& plen, uint32_t b) {
  if (plen == 0) {
    if (b <= 0x7f) {
      n = D.ascii[n * 128 + static_cast<int>(b)];
      return n >= 0;
    }
    if ((b >= 0xc2 && b <= 0xdf) || (b >= 0xe0 && b <= 0xef) || (b >= 0xf0 && b <= 0xf4)) {
      p = b;
      plen = 1;
      return true;
    }
    return false;
  }
  if (b < 0x80 || b > 0xbf) return false;
  p |= b << (8 * plen);
  ++plen;
  const uint32_t b0 = pbyte(p, 0), b1 = pbyte(p, 1);
  const int expected = b0 <= 0xdf ? 2 : b0 <= 0xef ? 3 : 4;
  if (plen < expected) return true;
  if ((b0 == 0xe0 && b1 < 0xa0) || (b0 == 0xed && b1 > 0x9f) || (b0 == 0xf0 && b1 < 0x90) || (b0 == 0xf4 && b1 > 0x8f))
    return false;
  const uint32_t cp = decode_cp(p, plen);
  p = 0;
  plen = 0;
  n = step_char(D, n, cp);
  return n >= 0;
}

// Table words of kStatesPerBlock states for 256 consecutive tokens.  Each thread holds
// its token's first 16 bytes in registers and walks them from each of the block's states
// in turn, one byte per loop iteration: when a walk ends (a dead or non-viable state, or
// the token's last byte) the lane records the result and starts the next state at once,
// so that the lanes of a warp stay busy until all of them have walked every state.  Warp
// ballots then make each state's word (bit i set: token 32·w + i is legal).
__global__ void __launch_bounds__(kWalkThreads) walk_kernel(DfaDev D, const uint4* __restrict__ tok16,
                                                            const uint16_t* __restrict__ tok_len,
                                                            const uint32_t* __restrict__ tok_off,
                                                            const uint8_t* __restrict__ tok_bytes, int64_t vocab,
                                                            const StateDev* __restrict__ states, int n_states,
                                                            uint32_t* table, int64_t mask_words) {
  __shared__ StateDev sst[kStatesPerBlock];
  const int64_t v = static_cast<int64_t>(blockIdx.x) * kWalkThreads + threadIdx.x;
  const int s0 = blockIdx.y * kStatesPerBlock;
  const int nk = n_states - s0 < kStatesPerBlock ? n_states - s0 : kStatesPerBlock;
  if (threadIdx.x < nk) sst[threadIdx.x] = states[s0 + threadIdx.x];
  __syncthreads();
  int len = 0;
  uint4 t = make_uint4(0u, 0u, 0u, 0u);
  uint32_t a = 0;
  if (v < vocab) {
    len = tok_len[v];
    if (len <= 16) t = tok16[v];
    else a = tok_off[v];
    if (len == 0xffff) len = static_cast<int>(tok_off[v + 1] - a);  // (lengths above 65534)
  }
  uint32_t res = 0;  // bit k: the token is legal from state s0 + k
  if (len > 0) {     // (an empty token is never in the trie)
    int k = 0, i = 0;
    StateDev st = sst[0];
    int n = st.node, plen = st.plen;
    uint32_t p = st.pending;
    while (k < nk) {
      uint32_t b;
      if (len <= 16) {
        const uint32_t wv = i < 4 ? t.x : i < 8 ? t.y : i < 12 ? t.z : t.w;
        b = (wv >> (8 * (i & 3))) & 0xffu;
      } else {
        b = tok_bytes[a + i];
      }
      bool ok = step_byte(D, n, p, plen, b);
      if (ok) ok = plen == 0 ? node_viable(D, n) : pending_viable(D, n, p, plen);
      const bool last = ++i == len;
      if (!ok || last) {
        res |= static_cast<uint32_t>(ok) << k;
        if (++k < nk) {
          st = sst[k];
          n = st.node;
          plen = st.plen;
          p = st.pending;
          i = 0;
        }
      }
    }
  }
  const int64_t word = v >> 5;
  for (int k = 0; k < nk; ++k) {
    const unsigned bits = __ballot_sync(kFullMask, (res >> k) & 1u);
    if ((threadIdx.x & 31) == 0 && word < mask_words) table[static_cast<int64_t>(s0 + k) * mask_words + word] = bits;
  }
}

// Per state: extra legal ids in, termination ids out (back in when the state accepts),
// padding words cleared, and dead_end[s] = 1 when nothing is left.
__global__ void __launch_bounds__(kPostThreads) post_kernel(const StateDev* __restrict__ states,
                                                            const uint8_t* __restrict__ flags, int64_t vocab,
                                                            const int32_t* __restrict__ extra, int64_t n_extra,
                                                            const int32_t* __restrict__ term, int64_t n_term,
                                                            uint32_t* table, int64_t mask_words, int32_t* dead_end) {
  const int s = blockIdx.x;
  uint32_t* row = table + static_cast<int64_t>(s) * mask_words;
  const StateDev st = states[s];
  const bool accepting = st.plen == 0 && (flags[st.node] & 1u);
  const int64_t used = (vocab + 31) >> 5;
  for (int64_t w = used + threadIdx.x; w < mask_words; w += blockDim.x) row[w] = 0u;
  for (int64_t i = threadIdx.x; i < n_extra; i += blockDim.x) {
    const int32_t v = extra[i];
    if (v >= 0 && v < vocab) atomicOr(&row[v >> 5], 1u << (v & 31));
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < n_term; i += blockDim.x) {
    const int32_t v = term[i];
    if (v >= 0 && v < vocab) atomicAnd(&row[v >> 5], ~(1u << (v & 31)));
  }
  __syncthreads();
  if (accepting)
    for (int64_t i = threadIdx.x; i < n_term; i += blockDim.x) {
      const int32_t v = term[i];
      if (v >= 0 && v < vocab) atomicOr(&row[v >> 5], 1u << (v & 31));
    }
  __syncthreads();
  int any = 0;
  for (int64_t w = threadIdx.x; w < used; w += blockDim.x) any |= row[w] != 0u;
  any = __syncthreads_or(any);
  if (threadIdx.x == 0 && dead_end) dead_end[s] = any ? 0 : 1;
}

template <class T>
cudaError_t upload(T** dst, const T* src, size_t n) {
  *dst = nullptr;
  if (n == 0) n = 1;
  cudaError_t e = cudaMalloc(dst, n * sizeof(T));
  if (e == cudaSuccess && src) e = cudaMemcpy(*dst, src, n * sizeof(T), cudaMemcpyHostToDevice);
  return e;
}

gs_status cfail(gs_constraint* c, gs_status s, const std::string& m) {
  if (c) c->err = m;
  return s;
}

void release(gs_constraint* c) {
  cudaFree(c->range_off);
  cudaFree(c->range_lo);
  cudaFree(c->range_hi);
  cudaFree(c->range_target);
  cudaFree(c->node_flags);
  cudaFree(c->tok_off);
  cudaFree(c->tok_bytes);
  cudaFree(c->ascii);
  cudaFree(c->tok16);
  cudaFree(c->tok_len);
  cudaFree(c->stage);
}

}  // namespace
}  // namespace gs

using namespace gs;

extern "C" {

gs_status gs_constraint_create(gs_ctx* ctx, const gs_dfa_desc* dfa, const gs_vocab_bytes_desc* vb,
                               gs_constraint** out) {
  if (!out) return GS_EINVAL;
  *out = nullptr;
  if (!ctx || !dfa || !vb) return GS_EINVAL;
  auto* c = new gs_constraint();
  c->device = ctx_device(ctx);
  const int32_t N = dfa->nodes;
  if (N <= 0 || !dfa->range_offsets || !dfa->final) {
    ctx_set_error(ctx, "a DFA needs nodes > 0, range_offsets and final");
    delete c;
    return GS_EINVAL;
  }
  const int64_t R = dfa->range_offsets[N];
  std::string why;
  if (dfa->range_offsets[0] != 0 || R < 0) why = "range_offsets must start at 0 and not decrease";
  for (int32_t n = 0; n < N && why.empty(); ++n) {
    if (dfa->range_offsets[n + 1] < dfa->range_offsets[n]) why = "range_offsets must not decrease";
    for (int64_t r = dfa->range_offsets[n]; r < dfa->range_offsets[n + 1] && why.empty(); ++r) {
      if (dfa->range_lo[r] > dfa->range_hi[r] || dfa->range_hi[r] > 0x10FFFFu) why = "ranges must satisfy lo <= hi <= 0x10FFFF";
      else if (r > dfa->range_offsets[n] && dfa->range_lo[r] <= dfa->range_hi[r - 1]) why = "a node's ranges must be sorted and disjoint";
      else if (dfa->range_target[r] < 0 || dfa->range_target[r] >= N) why = "range target out of range";
    }
  }
  const int64_t V = vb->vocab;
  if (why.empty() && (V <= 0 || V >= (1ll << 31) || !vb->offsets || (!vb->bytes && vb->offsets[V] > 0)))
    why = "vocabulary needs 0 < vocab < 2^31, offsets and bytes";
  if (why.empty()) {
    if (vb->offsets[0] != 0 || vb->offsets[V] >= (1ll << 32)) why = "token byte offsets must start at 0 and total below 2^32";
    for (int64_t v = 0; v < V && why.empty(); ++v)
      if (vb->offsets[v + 1] < vb->offsets[v] || vb->offsets[v + 1] - vb->offsets[v] > kMaxTokenBytes)
        why = "token byte offsets must not decrease (and a token holds at most 65536 bytes)";
  }
  if (!why.empty()) {
    ctx_set_error(ctx, why.c_str());
    delete c;
    return GS_EINVAL;
  }
  // viable nodes: the finals and every node that reaches one (constraints.ts:294-314)
  std::vector<uint8_t> flags(static_cast<size_t>(N), 0);
  std::vector<int64_t> rcount(static_cast<size_t>(N) + 1, 0);
  for (int64_t r = 0; r < R; ++r) ++rcount[static_cast<size_t>(dfa->range_target[r]) + 1];
  for (int32_t n = 0; n < N; ++n) rcount[n + 1] += rcount[n];
  std::vector<int32_t> pred(static_cast<size_t>(R));
  {
    std::vector<int64_t> fill(rcount.begin(), rcount.end() - 1);
    for (int32_t n = 0; n < N; ++n)
      for (int64_t r = dfa->range_offsets[n]; r < dfa->range_offsets[n + 1]; ++r)
        pred[static_cast<size_t>(fill[dfa->range_target[r]]++)] = n;
  }
  std::vector<int32_t> stack;
  for (int32_t n = 0; n < N; ++n)
    if (dfa->final[n]) {
      flags[n] = 3;
      stack.push_back(n);
    }
  while (!stack.empty()) {
    const int32_t t = stack.back();
    stack.pop_back();
    for (int64_t i = rcount[t]; i < rcount[t + 1]; ++i) {
      const int32_t p = pred[static_cast<size_t>(i)];
      if (!(flags[p] & 2)) {
        flags[p] |= 2;
        stack.push_back(p);
      }
    }
  }
  std::vector<uint32_t> toff(static_cast<size_t>(V) + 1);
  for (int64_t v = 0; v <= V; ++v) toff[v] = static_cast<uint32_t>(vb->offsets[v]);
  // dense ASCII transitions and the tokens' first 16 bytes (one vector load per token)
  std::vector<int32_t> ascii(static_cast<size_t>(N) * 128, -1);
  for (int32_t n = 0; n < N; ++n)
    for (int64_t r = dfa->range_offsets[n]; r < dfa->range_offsets[n + 1]; ++r)
      for (uint32_t ch = dfa->range_lo[r]; ch <= dfa->range_hi[r] && ch < 128; ++ch)
        ascii[static_cast<size_t>(n) * 128 + ch] = dfa->range_target[r];
  std::vector<uint4> t16(static_cast<size_t>(V), make_uint4(0u, 0u, 0u, 0u));
  std::vector<uint16_t> tlen(static_cast<size_t>(V));
  for (int64_t v = 0; v < V; ++v) {
    const int64_t len = vb->offsets[v + 1] - vb->offsets[v];
    tlen[v] = static_cast<uint16_t>(len < 0xffff ? len : 0xffff);
    if (len <= 16) std::memcpy(&t16[v], vb->bytes + vb->offsets[v], static_cast<size_t>(len));
  }
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != c->device) cudaSetDevice(c->device);
  cudaError_t e = upload(&c->range_off, dfa->range_offsets, static_cast<size_t>(N) + 1);
  if (e == cudaSuccess) e = upload(&c->range_lo, dfa->range_lo, static_cast<size_t>(R));
  if (e == cudaSuccess) e = upload(&c->range_hi, dfa->range_hi, static_cast<size_t>(R));
  if (e == cudaSuccess) e = upload(&c->range_target, dfa->range_target, static_cast<size_t>(R));
  if (e == cudaSuccess) e = upload(&c->node_flags, flags.data(), flags.size());
  if (e == cudaSuccess) e = upload(&c->tok_off, toff.data(), toff.size());
  if (e == cudaSuccess) e = upload(&c->tok_bytes, vb->bytes, static_cast<size_t>(toff[V]));
  if (e == cudaSuccess) e = upload(&c->ascii, ascii.data(), ascii.size());
  if (e == cudaSuccess) e = upload(&c->tok16, t16.data(), t16.size());
  if (e == cudaSuccess) e = upload(&c->tok_len, tlen.data(), tlen.size());
  if (prev >= 0 && prev != c->device) cudaSetDevice(prev);
  if (e != cudaSuccess) {
    ctx_set_error(ctx, (std::string("constraint upload: ") + cudaGetErrorString(e)).c_str());
    release(c);
    delete c;
    return GS_ENOMEM;
  }
  c->nodes = N;
  c->vocab = V;
  c->n_ranges = R;
  *out = c;
  return GS_OK;
}

gs_status gs_constraint_destroy(gs_constraint* c) {
  if (!c) return GS_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != c->device) cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  release(c);
  if (prev >= 0 && prev != c->device) cudaSetDevice(prev);
  delete c;
  return GS_OK;
}

const char* gs_constraint_last_error(const gs_constraint* c) { return c ? c->err.c_str() : ""; }

gs_status gs_constraint_build_masks(gs_constraint* c, int32_t n_states, const int32_t* node, const uint8_t* pending_len,
                                    const uint8_t* pending_bytes, const int32_t* termination, int64_t n_termination,
                                    const int32_t* extra_legal, int64_t n_extra, uint32_t* table, int64_t mask_words,
                                    int32_t* dead_end, void* stream) {
  if (!c) return GS_EINVAL;
  if (n_states < 0 || (n_states > 0 && (!node || !table))) return cfail(c, GS_EINVAL, "states and table are required");
  if (n_states > 65535) return cfail(c, GS_EUNSUPPORTED, "at most 65535 states per call");
  if (mask_words < (c->vocab + 31) / 32) return cfail(c, GS_EINVAL, "mask_words must be >= ceil(vocab/32)");
  if (n_termination < 0 || n_extra < 0 || (n_termination && !termination) || (n_extra && !extra_legal))
    return cfail(c, GS_EINVAL, "termination / extra id lists");
  if (n_states == 0) return GS_OK;
  std::vector<StateDev> st(static_cast<size_t>(n_states));
  for (int32_t s = 0; s < n_states; ++s) {
    const int plen = pending_len ? pending_len[s] : 0;
    if (node[s] < 0 || node[s] >= c->nodes) return cfail(c, GS_EINVAL, "state node out of range");
    if (plen < 0 || plen > 3) return cfail(c, GS_EINVAL, "pending UTF-8 bytes: at most 3");
    if (plen > 0) {
      // a pending sequence starts with a lead byte and is shorter than the sequence it leads
      const uint8_t lead = pending_bytes[3 * s];
      const bool ok = (lead >= 0xc2 && lead <= 0xdf) || (lead >= 0xe0 && lead <= 0xef) || (lead >= 0xf0 && lead <= 0xf4);
      const int expected = lead <= 0xdf ? 2 : lead <= 0xef ? 3 : 4;
      if (!ok || plen >= expected) return cfail(c, GS_EINVAL, "pending UTF-8 bytes must be an incomplete sequence");
    }
    uint32_t p = 0;
    for (int i = 0; i < plen; ++i) p |= static_cast<uint32_t>(pending_bytes[3 * s + i]) << (8 * i);
    st[s] = StateDev{node[s], p, plen, 0};
  }
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != c->device) cudaSetDevice(c->device);
  auto restore = [&]() {
    if (prev >= 0 && prev != c->device) cudaSetDevice(prev);
  };
  cudaStream_t sm = static_cast<cudaStream_t>(stream);
  // staging: states | termination | extra (one upload)
  const size_t b_st = align_up(st.size() * sizeof(StateDev), 256);
  const size_t b_term = align_up(static_cast<size_t>(n_termination) * 4, 256);
  const size_t b_extra = align_up(static_cast<size_t>(n_extra) * 4, 256);
  const size_t need = b_st + b_term + b_extra;
  if (need > c->stage_bytes) {
    cudaStreamSynchronize(sm);
    cudaFree(c->stage);
    c->stage = nullptr;
    c->stage_bytes = 0;
    cudaError_t e = cudaMalloc(&c->stage, need);
    if (e != cudaSuccess) {
      restore();
      return cfail(c, GS_ENOMEM, std::string("staging: ") + cudaGetErrorString(e));
    }
    c->stage_bytes = need;
  }
  std::vector<unsigned char> host(need);
  std::memcpy(host.data(), st.data(), st.size() * sizeof(StateDev));
  if (n_termination) std::memcpy(host.data() + b_st, termination, static_cast<size_t>(n_termination) * 4);
  if (n_extra) std::memcpy(host.data() + b_st + b_term, extra_legal, static_cast<size_t>(n_extra) * 4);
  // (a synchronous copy from pageable memory: the staging is free once it returns)
  cudaError_t e = cudaMemcpyAsync(c->stage, host.data(), need, cudaMemcpyHostToDevice, sm);
  if (e == cudaSuccess) e = cudaStreamSynchronize(sm);
  if (e != cudaSuccess) {
    restore();
    return cfail(c, GS_ECUDA, std::string("state upload: ") + cudaGetErrorString(e));
  }
  const StateDev* dst = reinterpret_cast<const StateDev*>(c->stage);
  const int32_t* dterm = reinterpret_cast<const int32_t*>(c->stage + b_st);
  const int32_t* dextra = reinterpret_cast<const int32_t*>(c->stage + b_st + b_term);
  DfaDev D{c->ascii, c->range_off, c->range_lo, c->range_hi, c->range_target, c->node_flags, c->nodes};
  dim3 grid(static_cast<unsigned>((c->vocab + kWalkThreads - 1) / kWalkThreads),
            static_cast<unsigned>((n_states + kStatesPerBlock - 1) / kStatesPerBlock));
  walk_kernel<<<grid, kWalkThreads, 0, sm>>>(D, c->tok16, c->tok_len, c->tok_off, c->tok_bytes, c->vocab, dst,
                                             n_states, table, mask_words);
  post_kernel<<<n_states, kPostThreads, 0, sm>>>(dst, c->node_flags, c->vocab, dextra, n_extra, dterm, n_termination,
                                                  table, mask_words, dead_end);
  e = cudaGetLastError();
  restore();
  if (e != cudaSuccess) return cfail(c, GS_ECUDA, std::string("mask builder launch: ") + cudaGetErrorString(e));
  return GS_OK;
}

}  // extern "C"
