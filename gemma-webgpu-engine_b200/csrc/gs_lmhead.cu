// int2 LM head on the 5th-generation tensor cores: the logits the sampler consumes,
// computed from the final activations and the model's packed 2-bit output weights.
//
// Reference: src/webgpu/decode-lm-head.ts.  Packed weights are V rows of hidden/16 u32
// words; code j of word w (bits 2j..2j+1) multiplies activation element 16w + j and the
// weight is (code - 2)·rowScale (createGemmaLmHeadShader, :176-256):
//   logit = srq(rowScale · fma(Σ_j (code_j / 255)·a_j, 255, -(2·sumA)), outputScale)
// with srq(x, s) = s == 0 ? x : clamp(round(x / s), -128, 127)·s (:196-199).  The
// activations come from decode-ple-proj-norm-codes.ts:251-258, already on the srq grid of
// the model's final input scale (a = q·inScale, q an int8 code), with sumA their sum.
//
// Here the dot product is exact: with inScale != 0 the activations are read as their
// int8 codes q = clamp(rint(a / inScale), -128, 127), the weights as int8 (code - 2), and
// tcgen05.mma kind::i8 accumulates Σ (code - 2)·q in s32 in tensor memory; Σ code·q is that
// plus 2·Σq, and t = fma(inScale, Σ code·q, -2·sumA) rounds once.  (inScale == 0 keeps the
// activations in float32: a CUDA-core kernel sums code·a in double, element by element.)
// The reference's f32 evaluation differs from this exact value by its own rounding.
//
// Device layout of the weights (repacked once at creation): tile-major, 128 vocab rows
// per tile, the hidden axis cut in 128-code chunks: [tile][chunk][128 rows][8 words] —
// every (tile, chunk) block is 4 KB, one bulk copy.  The activation codes are written per
// call as the smem image the MMA reads: [pass][chunk][64 rows][128 bytes], 128-byte
// swizzled, with the 16 codes of each packed word in the order the expansion produces.
//
// Kernel (one CTA per SM, persistent over vocab tiles; grid.y: passes of N batch rows):
//   warp 1      producer: the pass's activation image (once), then every (tile, chunk)
//               packed block into a ring of 24-40 stages (cp.async.bulk, mbarrier tx
//               counts): the weight bytes in flight from HBM
//   warps 8-15  expanders, two groups of four warps: packed 2-bit codes -> int8
//               (code - 2), one vocab row per thread written straight to its TMEM lane
//               (tcgen05.st): the weight operand never touches shared memory, whose
//               bandwidth the 4x inflated codes would otherwise saturate
//   warp 0      MMA issuer (one elected lane): 4 × tcgen05.mma (K = 32, A from TMEM,
//               B = the activation image from shared memory) per chunk into a
//               128 × N s32 accumulator (N = 16 or 64 batch columns), two accumulators in
//               TMEM (tile i+1 runs while the epilogue drains tile i); also allocates /
//               frees the TMEM columns
//   warps 4-7   epilogue: tcgen05.ld of their 32 TMEM lanes (one vocab row per thread,
//               the batch columns in 16-column loads), then logit = srq(scale · t),
//               stored coalesced
// Every wait is bounded (1 s); a timeout sets the handle's error flag and ends the
// CTA's loops without touching further stages.
#include <cstring>
#include <string>
#include <vector>

#include "gs_block.cuh"
#include "gs_device.cuh"
#include "gs_internal.cuh"
#include "gs_plan.cuh"
#include "../../include/gsampler.h"

struct gs_lm_head {
  gs_ctx* ctx = nullptr;  // the sampler context the handle was created on (gs_lm_head_sample)
  int device = 0;
  int64_t vocab = 0;
  int32_t hidden = 0;
  int32_t chunks = 0;   // hidden / 128
  int64_t tiles = 0;    // ceil(vocab / 128)
  float in_scale = 0.0f;
  float out_scale = 0.0f;
  uint32_t* packed = nullptr;  // [tiles][chunks][128][8]
  float* scales = nullptr;     // [tiles * 128] (0 past vocab)
  // per-call activation image (grown on demand): [passes][chunks][64][128] | Σq [passes * 64]
  unsigned char* img = nullptr;
  size_t img_bytes = 0;
  int32_t* flag = nullptr;  // device error flag (bit 0: a wait timed out); flag[1]: records kernel's finished-block count
  // gs_lm_head_sample's logits (grown on demand): rows × vocab float32
  float* scratch = nullptr;
  size_t scratch_bytes = 0;
  // fused gs_lm_head_sample: per (shard, row) records the vocabulary-sharded merge reads
  unsigned char* records = nullptr;
  size_t records_bytes = 0;
  int64_t fused_calls = 0;
  int32_t route = GS_LM_ROUTE_AUTO;
  int num_sms = 0;
  std::string err;
};

namespace gs {
namespace {

constexpr int kLmRows = 128;                    // vocab rows per tile (TMEM lanes)
constexpr int kLmKC = 128;                      // codes per chunk (one 128-byte swizzle row)
constexpr int kLmMaxChunks = 12;                // hidden <= 1536
constexpr int kGroups = 2;                      // expander groups (4 warps, one row each): chunk g -> g % 2
constexpr int kAStages = 4;                     // weight operand stages in TMEM (32 columns each)
// TMEM columns: two accumulators [0, 2N), then the operand stages
constexpr int kMmaRound = 1;                    // chunks the MMA issuer takes per round
#ifndef GS_LM_GEMV_ROWS
#define GS_LM_GEMV_ROWS 4
#endif
constexpr int kGemvRows = GS_LM_GEMV_ROWS;      // batches up to this many rows take the dp4a GEMV
constexpr int kPBytes = kLmRows * kLmKC / 4;    // 4 KB of packed codes per (tile, chunk)
constexpr int kExpanders = 256;                 // threads expanding packed codes (warps 4-11)
constexpr int kGroupThreads = kExpanders / kGroups;  // 128: one per vocab row of the tile
// Warp roles.  The MMA issuer and the producer take the lowest warp ids: the schedulers
// favour older warps, and the expanders keep their sub-partitions busy in bursts.
constexpr int kMmaWarp = 0, kProducerWarp = 1;  // (warps 2-3 idle)
constexpr int kEpiWarp0 = 4;                    // warps 4-7: TMEM lane quadrants 0-3
constexpr int kExpWarp0 = 8;                    // warps 8-15: two groups of four quadrants
constexpr int kLmThreads = (kExpWarp0 * 32) + kExpanders;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kImgRows = 64;                    // rows per pass of the activation image in HBM
constexpr int kIssue = 8;                       // producer lanes issuing packed-block copies at once

// Shared-memory plan of the kernel for N batch columns (16 or 64): the pass's activation
// image, then as many packed-block stages as fit (the bytes in flight from HBM per SM),
// then the barriers.  The expanded weight operand lives in TMEM, not here.
template <int N>
struct LmPlan {
  static constexpr int kQChunk = N * kLmKC;                    // activation codes per chunk
  static constexpr int kOffQ = 0;
  static constexpr int kOffP = kOffQ + kLmMaxChunks * kQChunk;
  static constexpr int kPStages = ((kSmemLimit - kOffP - 1024 - 1024) / kPBytes > 40 ? 40
                                   : (kSmemLimit - kOffP - 1024 - 1024) / kPBytes) / kIssue * kIssue;
  static constexpr int kOffBar = kOffP + kPStages * kPBytes;
  static constexpr int kSmem = kOffBar + 1024 + 1024;          // barriers + alignment slack
  static constexpr int kAColBase = 2 * N < 128 ? 128 : 2 * N;   // first operand-stage column
  static constexpr int kTmemCols = kAColBase + kAStages * 32 <= 256 ? 256 : 512;
  // Instruction descriptor of tcgen05.mma kind::i8: D s32 (bits 4-5 = 2), A and B signed
  // 8-bit (bits 7-9 = 1, 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
  static constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
                                     (static_cast<uint32_t>(kLmRows >> 4) << 24);
  static_assert(kOffP % 1024 == 0 && 2 * N <= kAColBase, "aligned stages; accumulators below the operands");
  static_assert(kAColBase + kAStages * 32 <= kTmemCols && kTmemCols <= 512, "TMEM columns");
  static_assert(kSmem <= kSmemLimit, "shared memory");
  static_assert(kPStages >= kIssue && kPStages % kIssue == 0, "whole producer rounds per ring");
  static_assert((1 + 2 * kPStages + 2 * kAStages + 5) * 8 + 8 <= 1024, "barriers fit their 1 KB");
};

// Shared-memory matrix descriptor of a K-major operand in the 128-byte swizzle layout:
// rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset), start address
// >> 4 in bits 0-13, leading byte offset 1 (unused by this layout), version 1 (bit 46),
// layout SWIZZLE_128B (2 << 61).  The K = 32 steps inside a row add 32 bytes to the start
// (the swizzle applies to the absolute address bits, the groups being 1024-aligned).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (static_cast<uint64_t>(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

// Bounded wait that first tests the phase without blocking (mbarrier.test_wait): the
// pipeline's consumers usually find their phase complete already.
__device__ __forceinline__ bool lm_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0 || mbar_wait(bar, parity, kWaitNs);
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// D (TMEM) += A (TMEM: lane m = row m, 4 int8 of K per 32-bit column) × B^T (smem desc).
__device__ __forceinline__ void tc_mma_i8_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// One lane of the (converged) warp.
__device__ __forceinline__ bool elect_one() {
  uint32_t p = 0;
  asm volatile("{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\tselp.b32 %0, 1, 0, P;\n\t}" : "=r"(p));
  return p != 0;
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 16 consecutive s32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int32_t* r) {
  uint32_t v[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) r[i] = static_cast<int32_t>(v[i]);
}

// srq(x, s) of decode-lm-head.ts:196-199 (round half to even, IEEE division).
__device__ __forceinline__ float srq(float x, float s) {
  if (s == 0.0f) return x;
  float r = rintf(__fdiv_rn(x, s));
  r = fminf(fmaxf(r, -128.0f), 127.0f);
  return __fmul_rn(r, s);
}

struct LmArgs {
  const uint32_t* packed;
  const float* scales;
  const unsigned char* img;  // activation codes, [passes][chunks][64][128]
  const int32_t* qsum;       // [passes * 64] Σ q per batch row
  int32_t pass_rows;         // batch rows per pass (the kernel's N)
  const float* act_sum;      // [rows]
  float* logits;
  int64_t ld;
  int64_t vocab;
  int64_t tiles;
  int32_t chunks;
  int32_t rows;
  float in_scale;
  float out_scale;
  int32_t* flag;
};

// Activation codes of one batch row (block b of rows padded to whole passes) in the MMA's
// smem image: chunk c, 16-byte slot w (swizzled by the row within its 8-row group), byte
// 4P + k = code of element 16w + 4k + P (the order the expansion writes weight codes).
__global__ void __launch_bounds__(256) lm_quant_kernel(const float* __restrict__ act, int64_t ld_act, int rows,
                                                       int hidden, float in_scale, unsigned char* __restrict__ img,
                                                       int32_t* __restrict__ qsum) {
  __shared__ int red[8];
  const int b = blockIdx.x;
  const int p = b / kImgRows, r = b % kImgRows;
  const int chunks = hidden / kLmKC;
  int s = 0;
  constexpr int kPer = kLmMaxChunks * kLmKC / 256;  // image bytes per thread (loads issued together)
  float x[kPer];
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int j = threadIdx.x + 256 * u;  // j: byte position in the image row
    const int e = (j & ~15) + 4 * (j & 3) + ((j & 15) >> 2);
    x[u] = (b < rows && j < hidden) ? __ldg(act + static_cast<int64_t>(b) * ld_act + e) : 0.0f;
  }
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int j = threadIdx.x + 256 * u;
    if (j >= hidden) break;
    const int c = j / kLmKC, w = (j % kLmKC) >> 4, pos = j & 15;
    const int q = static_cast<int>(fminf(fmaxf(rintf(__fdiv_rn(x[u], in_scale)), -128.0f), 127.0f));
    s += q;
    img[(static_cast<size_t>(p) * chunks + c) * (kImgRows * kLmKC) + r * kLmKC + ((w ^ (r & 7)) << 4) + pos] =
        static_cast<unsigned char>(static_cast<int8_t>(q));
  }
  s = warp_sum_i(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int i = 0; i < (blockDim.x >> 5); ++i) t += red[i];
    qsum[b] = t;
  }
}

template <int N>
__global__ void __launch_bounds__(kLmThreads, 1) lm_mma_kernel(const __grid_constant__ LmArgs A) {
  using P = LmPlan<N>;
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte aligned base (the swizzled operand groups need it)
  const uint32_t raw = smem_addr(smem_raw);
  unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + P::kOffBar);
  uint64_t* qfull = bars;                      // [1]
  uint64_t* pfull = bars + 1;                  // [kPStages]
  uint64_t* pfree = pfull + P::kPStages;       // [kPStages]
  uint64_t* afull = pfree + P::kPStages;       // [kAStages]
  uint64_t* afree = afull + kAStages;          // [kAStages]
  uint64_t* accfull = afree + kAStages;        // [2]
  uint64_t* accfree = accfull + 2;             // [2]
  uint64_t* mdone = accfree + 2;               // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pass = blockIdx.y;
  const int C = A.chunks;
  const int64_t my_tiles = A.tiles > blockIdx.x ? (A.tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

  if (threadIdx.x == 0) {
    mbar_init(qfull, 1);
    for (int s = 0; s < P::kPStages; ++s) {
      mbar_init(pfull + s, 1);
      mbar_init(pfree + s, kGroupThreads);
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(afull + s, kGroupThreads);  // (the 128 rows of a chunk)
      mbar_init(afree + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(accfull + s, 1);
      mbar_init(accfree + s, 128);
    }
    mbar_init(mdone, 1);
    *abort_flag = 0;
  }
  if (warp == kMmaWarp) {  // TMEM columns for the two accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(P::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto give_up = [&]() {
    *abort_flag = 1;
    atomicOr(A.flag, 1);
  };

  if (warp == kProducerWarp) {
    // ---------------- producer ----------------
    // Lanes 0..kIssue-1 each copy one of kIssue consecutive chunks per round (the copies
    // of one instruction go out together).
    if (lane == 0) {
      // the pass's N image rows of every chunk (the HBM image holds kImgRows rows per
      // chunk block: N = 128 takes two consecutive image passes)
      mbar_expect_tx(qfull, static_cast<uint32_t>(C * P::kQChunk));
      constexpr int kBlocks = N > kImgRows ? N / kImgRows : 1;
      constexpr int kBlockBytes = (N > kImgRows ? kImgRows : N) * kLmKC;
      for (int c = 0; c < C; ++c)
        for (int k = 0; k < kBlocks; ++k)
          bulk_g2s(sm + P::kOffQ + c * P::kQChunk + k * kBlockBytes,
                   A.img + (static_cast<size_t>(pass * kBlocks + k) * C + c) * (kImgRows * kLmKC), kBlockBytes, qfull);
    }
    __syncwarp();
    const int64_t total = my_tiles * C;
    for (int64_t g0 = 0; g0 < total && !*abort_flag; g0 += kIssue) {
      const int64_t g = g0 + lane;
      bool ok = true;
      if (lane < kIssue && g < total) {
        const int s = static_cast<int>(g % P::kPStages);  // (kIssue consecutive chunks: distinct stages)
        const int64_t k = g / P::kPStages;
        if (k > 0) ok = lm_wait(pfree + s, static_cast<uint32_t>((k - 1) & 1));
        if (ok) {
          const int64_t t = blockIdx.x + (g / C) * gridDim.x;
          const int c = static_cast<int>(g % C);
          mbar_expect_tx(pfull + s, kPBytes);
          bulk_g2s(sm + P::kOffP + s * kPBytes, A.packed + (static_cast<size_t>(t) * C + c) * (kPBytes / 4), kPBytes,
                   pfull + s);
        }
      }
      if (!__all_sync(kFullMask, ok)) {
        give_up();
        break;
      }
    }
  } else if (warp >= kExpWarp0) {
    // ---------------- expanders ----------------
    // Group k (four warps, one vocab row of the tile per thread: the TMEM lane its warp
    // may write) expands chunks k, k + 2, ... into operand stage g % 4: the row's 8 packed
    // words -> 32 columns of int8 (code - 2), column 4w + P holding the codes of elements
    // 16w + 4k + P in byte k (the order of the activation image).
    const int et = threadIdx.x - kExpWarp0 * 32;  // 0 .. kExpanders - 1
    const int grp = et / kGroupThreads, row = et % kGroupThreads;  // row = 32·(warp % 4) + lane
    const int64_t total = my_tiles * C;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(row & ~31) << 16);
    for (int64_t g = grp; g < total && !*abort_flag; g += kGroups) {
      const int s = static_cast<int>(g % P::kPStages), a = static_cast<int>(g % kAStages);
      const int64_t kp = g / P::kPStages, ka = g / kAStages;
      const bool ok = lm_wait(pfull + s, static_cast<uint32_t>(kp & 1)) &&
                      (ka == 0 || lm_wait(afree + a, static_cast<uint32_t>((ka - 1) & 1)));
      if (!__all_sync(kFullMask, ok)) {  // (the warp leaves together; TMEM stores are warp-collective)
        give_up();
        break;
      }
      const uint4* src = reinterpret_cast<const uint4*>(sm + P::kOffP + s * kPBytes) + row * 2;
      const uint4 p0 = src[0], p1 = src[1];
      mbar_arrive(pfree + s);  // (the row's packed words are in registers)
      const uint32_t x[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
      uint32_t o[32];
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        // byte k of word P = code 4k + P, mapped 0..3 -> -2..1: ((v + 0x7E) ^ 0x80) per byte
#pragma unroll
        for (int q = 0; q < 4; ++q) o[4 * w + q] = (((x[w] >> (2 * q)) & 0x03030303u) + 0x7E7E7E7Eu) ^ 0x80808080u;
      }
      tmem_st32(lane_base + static_cast<uint32_t>(P::kAColBase + 32 * a), o);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(afull + a);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    // The whole warp runs the loop (its descriptors stay warp-uniform); one elected lane
    // issues the MMAs and the commits that track them.
    const bool leader = elect_one();
    bool ok = __all_sync(kFullMask, lm_wait(qfull, 0));
    if (!ok) give_up();
    int64_t g = 0;
    const uint64_t qd0 = sw128_desc(smem_addr(sm + P::kOffQ));
    for (int64_t i = 0; ok && i < my_tiles && !*abort_flag; ++i) {
      const int j = static_cast<int>(i & 1);
      const int64_t kacc = i >> 1;
      if (kacc > 0 && !__all_sync(kFullMask, lm_wait(accfree + j, static_cast<uint32_t>((kacc - 1) & 1)))) {
        give_up();
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem + static_cast<uint32_t>(j * N);
      // chunks in rounds of kMmaRound: one wait per chunk, then all their MMAs (a round
      // trip through the barriers costs about as much as the MMAs of several chunks)
      for (int c = 0; c < C; c += kMmaRound) {
        const int nc = C - c < kMmaRound ? C - c : kMmaRound;
        bool okw = true;
        for (int u = 0; u < nc; ++u)
          okw = okw && lm_wait(afull + static_cast<int>((g + u) % kAStages), static_cast<uint32_t>(((g + u) / kAStages) & 1));
        if (!__all_sync(kFullMask, okw)) {
          give_up();
          ok = false;
          break;
        }
        tc_fence_after();
        if (leader) {
          for (int u = 0; u < nc; ++u) {
            const int a = static_cast<int>((g + u) % kAStages);
            // K = 32 steps: 8 TMEM columns of A, 32 bytes (2 descriptor units) of B
            const uint32_t at = tmem + static_cast<uint32_t>(P::kAColBase + 32 * a);
            const uint64_t bd = qd0 + static_cast<uint64_t>(((c + u) * P::kQChunk) >> 4);
#pragma unroll
            for (int k = 0; k < kLmKC / 32; ++k)
              tc_mma_i8_ts(d, at + 8 * k, bd + 2 * k, P::kIdesc, ((c + u) | k) != 0 ? 1u : 0u);
            tc_commit(afree + a);  // the stage is free once these MMAs have read it
          }
        }
        __syncwarp();
        g += nc;
      }
      if (!ok) break;
      if (leader) tc_commit(accfull + j);
      __syncwarp();
    }
    // every MMA this warp issued has completed before the columns are freed
    if (leader) tc_commit(mdone);
    __syncwarp();
    if (!__all_sync(kFullMask, lm_wait(mdone, 0))) give_up();
  } else if (warp >= kEpiWarp0) {
    // ---------------- epilogue (warps 4-7: TMEM lanes 32·(warp - 4) ..) ----------------
    const int quad = warp - kEpiWarp0;
    const int n_here = A.rows - pass * N < N ? A.rows - pass * N : N;
    const int groups = (n_here + 15) >> 4;  // 16-column TMEM loads needed (block-uniform)
    for (int64_t i = 0; i < my_tiles && !*abort_flag; ++i) {
      const int64_t t = blockIdx.x + i * gridDim.x;
      const int j = static_cast<int>(i & 1);
      // (warp-uniform: the TMEM loads below are warp-collective)
      if (!__all_sync(kFullMask, lm_wait(accfull + j, static_cast<uint32_t>((i >> 1) & 1)))) {
        give_up();
        break;
      }
      tc_fence_after();
      const int64_t v = t * kLmRows + 32 * quad + lane;
      const bool in = v < A.vocab;
      const float scale = in ? A.scales[v] : 0.0f;
      const uint32_t ta = tmem + (static_cast<uint32_t>(32 * quad) << 16) + static_cast<uint32_t>(j * N);
      for (int q = 0; q < groups; ++q) {
        int32_t acc[16];
        tmem_ld16(ta + 16 * q, acc);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (q == groups - 1) {
          tc_fence_before();
          mbar_arrive(accfree + j);  // the accumulator's columns are in registers
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int n = 16 * q + u;
          if (n >= n_here) break;  // (uniform)
          const int b = pass * N + n;
          const int32_t scq = acc[u] + 2 * A.qsum[b];  // Σ code·q, exact
          const float tt = __fmaf_rn(A.in_scale, static_cast<float>(scq), -(2.0f * A.act_sum[b]));
          if (in) A.logits[static_cast<int64_t>(b) * A.ld + v] = srq(__fmul_rn(scale, tt), A.out_scale);
        }
      }
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P::kTmemCols) : "memory");
  }
}

// Few batch rows (a GEMV): the tensor-core MMA streams a whole 128 × 32 expanded weight
// tile per instruction, so with a handful of columns it is bound by operand traffic;
// here the packed words come straight from HBM and dp4a accumulates Σ code·q (unsigned
// codes × signed activation codes, exact in int32).  Warp w of a tile's block reads the
// 1 KB of its 32 rows per chunk in two fully coalesced 512-byte loads: lane l holds half
// (l & 1) of rows l >> 1 and 16 + (l >> 1), and the halves meet in a shuffle at the end.
// Each (persistent) block quantises the activations itself into shared memory first:
// word 4w + P of a row holds the codes of elements 16w + 4k + P in byte k (the order
// the code extraction below produces), rows past `rows` zero; they are read four words
// at a time.
// Activation codes of rows [0, rows) into qw[b·kLmMaxChunks·32 + j] (zero for rows >= rows):
// word j = 4w + P packs the int8 codes of elements 16w + 4k + P, k = 0..3 (the order that
// lines up with the 2-bit codes of a packed weight word w).
template <int NB>
__device__ __forceinline__ void lm_quant_act(uint32_t* qw, const LmArgs& A, const float* __restrict__ act, int64_t ld_act,
                                             int rows) {
  const int C = A.chunks;
  for (int i = threadIdx.x; i < NB * C * 32; i += blockDim.x) {
    const int b = i / (C * 32), j = i % (C * 32);  // j = 4w + P
    uint32_t word = 0;
    if (b < rows) {
      const float* ar = act + static_cast<int64_t>(b) * ld_act + 16 * (j >> 2) + (j & 3);
      float x[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) x[k] = __ldg(ar + 4 * k);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float r = fminf(fmaxf(rintf(__fdiv_rn(x[k], A.in_scale)), -128.0f), 127.0f);
        word |= (static_cast<uint32_t>(static_cast<int32_t>(r)) & 0xffu) << (8 * k);
      }
    }
    qw[b * kLmMaxChunks * 32 + j] = word;
  }
}

// Integer dot products of one warp: rows 32·quad + (lane >> 1) (h = 0) and 16 more (h = 1)
// of tile t, half the row's words per lane; the lane pair's sum follows the shuffle.
template <int NB>
__device__ __forceinline__ void lm_tile_dots(const LmArgs& A, const uint32_t* qw, int64_t t, int quad, int lane,
                                             int32_t (&acc)[2][NB]) {
  const int C = A.chunks;
  const int half = lane & 1;
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[h][b] = 0;
  // this warp's 32 rows of chunk c: 1 KB at ((t·C + c)·128 + 32·quad)·32 bytes
  const uint4* wbase = reinterpret_cast<const uint4*>(A.packed) + (static_cast<size_t>(t) * C * kLmRows + 32 * quad) * 2;
  for (int c0 = 0; c0 < C; c0 += 4) {  // four chunks' loads in flight
    uint4 x[4][2];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (c0 + u < C) {
        const uint4* p = wbase + static_cast<size_t>(c0 + u) * kLmRows * 2;
        x[u][0] = ld_stream_u4(p + lane);       // rows lane >> 1, half lane & 1
        x[u][1] = ld_stream_u4(p + 32 + lane);  // rows 16 + (lane >> 1)
      }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (c0 + u >= C) break;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t wv[4] = {x[u][h].x, x[u][h].y, x[u][h].z, x[u][h].w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {  // packed word 4·half + w of the row's chunk
          const uint32_t c0w = wv[w] & 0x03030303u, c1w = (wv[w] >> 2) & 0x03030303u;
          const uint32_t c2w = (wv[w] >> 4) & 0x03030303u, c3w = (wv[w] >> 6) & 0x03030303u;
          const int qi = (c0 + u) * 32 + 4 * (4 * half + w);
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            const uint4 q = *reinterpret_cast<const uint4*>(&qw[b * kLmMaxChunks * 32 + qi]);  // words P = 0..3
            int32_t d = acc[h][b];
            asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(d) : "r"(c0w), "r"(q.x));
            asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(d) : "r"(c1w), "r"(q.y));
            asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(d) : "r"(c2w), "r"(q.z));
            asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(d) : "r"(c3w), "r"(q.w));
            acc[h][b] = d;
          }
        }
      }
    }
  }
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[h][b] += __shfl_xor_sync(kFullMask, acc[h][b], 1);
}

template <int NB>
__global__ void __launch_bounds__(128) lm_gemv_kernel(const __grid_constant__ LmArgs A, const float* __restrict__ act,
                                                      int64_t ld_act) {
  __shared__ __align__(16) uint32_t qw[NB * kLmMaxChunks * 32];  // [row][4·(16-code word) + P]
  const int rows = A.rows < NB ? A.rows : NB;
  lm_quant_act<NB>(qw, A, act, ld_act, rows);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane & 1;
  for (int64_t t = blockIdx.x; t < A.tiles; t += gridDim.x) {
  int32_t acc[2][NB];
  lm_tile_dots<NB>(A, qw, t, warp, lane, acc);
  // lane pair (2k, 2k+1) holds rows k and 16 + k: the even lane writes the first, the odd the second
  const int64_t v = t * kLmRows + 32 * warp + (lane >> 1) + 16 * half;
  if (v < A.vocab) {
    const float scale = A.scales[v];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b < rows) {
        const float tt = __fmaf_rn(A.in_scale, static_cast<float>(half ? acc[1][b] : acc[0][b]), -(2.0f * A.act_sum[b]));
        A.logits[static_cast<int64_t>(b) * A.ld + v] = srq(__fmul_rn(scale, tt), A.out_scale);
      }
    }
  }
  }
}

// ---------------------------------------------------------------- fused sampling
// gs_lm_head_sample for a few rows without a penalty history: the logits never leave the
// SM.  Block g computes the logits of vocabulary ids [g·R, (g+1)·R) (R = tiles per shard ·
// 128) for every row with the GEMV's dot products into shared memory, soft-caps them, and
// writes, per row, the record a vocabulary shard writes in gs_shard_partials: the live
// (allowed) maximum m and sum Σ 2^((x - m)·log2(e)/T), the maximum and sum of e^(x - max)
// over every id (log-probability), the allowed count, error flags, and the shard's k best
// candidate packs (key32(x) and ~id, as the streaming pass packs them; chosen exactly).
// The merge of vocabulary-sharded calls then treats the blocks as shards; no logits are
// stored.
constexpr int kRecMaxK = 64;     // topK the fused path serves (the merge's pack buffer)
// Rows of one fused call (the kernel's NB).  Measured against gs_lm_head_logits +
// gs_sample (p50 per call, V = 262144, topK 40): 60 vs 76 us at one row, 67 vs 81 at two,
// 95 vs 96 at three, 101 vs 98 at four (the dot products of more rows are issue-bound in
// one 1024-thread block per SM, where the GEMV spreads them over nine 128-thread blocks).
constexpr int kRecMaxRows = 2;
constexpr int kRecCandCap = 512; // packs at or above the per-row bound, ranked by counting
constexpr int kRecMaxHistory = 4096;  // penalty-history stride the fused route serves (its sort buffer)

struct RecArgs {
  LmArgs L;
  const float* act;
  int64_t ld_act;
  RowPlan plan[kRecMaxRows];
  float cap, inv_cap;
  const uint32_t* mask_table;
  int64_t mask_states, mask_words;
  const int32_t* mask_state;
  unsigned char* records;  // [shard][row] of rec_bytes
  int64_t rec_bytes;
  int32_t tps;             // tiles per shard
  int32_t want_raw;        // log-probabilities requested (a NaN raw sum is then an error)
  int32_t kcap;            // packs per record
  unsigned* done;          // blocks finished (the last one combines; it resets the count)
  unsigned char* combined; // [row] of rec_bytes: every shard's record of the row in one (null: no combining)
  const int32_t* history;  // [row][history_stride] penalty history (null: none)
  const int32_t* history_len;
  int64_t history_stride;
  int32_t hcap;            // penalised slots per record (history_stride; 0 without history)
  int32_t hsort;           // sort buffer entries (power of two >= hcap)
  int64_t hist_off;        // byte offset of the sort buffer and penalised-id bits in shared memory
};

inline int pow2_ceil_host(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

// shared memory of the records kernel: activation words | logits [NB][R] | packs [NB][R]
// (the last block reuses it for every shard's packs of a row and the shards' maxima),
// then, with a penalty history, its sort buffer and the penalised ids' bits [NB][R / 32]
__host__ __device__ inline size_t rec_base_bytes(int nb, int tps, int shards, int kcap) {
  const size_t own = static_cast<size_t>(nb) * kLmMaxChunks * 32 * 4 + static_cast<size_t>(nb) * tps * kLmRows * 12;
  const size_t comb = static_cast<size_t>(shards) * (kcap + 1) * 8;
  return ((own > comb ? own : comb) + 15) & ~static_cast<size_t>(15);
}
__host__ __device__ inline size_t rec_smem_bytes(int nb, int tps, int shards, int kcap, int hsort) {
  return rec_base_bytes(nb, tps, shards, kcap) + (hsort > 0 ? static_cast<size_t>(hsort) * 4 + static_cast<size_t>(nb) * tps * 16 : 0);
}

template <int NB, int THREADS>
__global__ void __launch_bounds__(THREADS) lm_records_kernel(const __grid_constant__ RecArgs R) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ float red_f[2][NB][32];
  __shared__ double red_d[2][NB][32];
  __shared__ int red_i[2][NB][32];
  __shared__ float fin_lm[NB], fin_rm[NB];
  __shared__ double fin_s[NB], fin_rs[NB];
  __shared__ int fin_na[NB], fin_bad[NB];
  __shared__ unsigned sel_hist[256];
  __shared__ int sel_digit, sel_above, sel_binc, n_out, n_cl, s_last, n_tot, s_hl;
  __shared__ unsigned pen_fl[NB];
  __shared__ unsigned long long top2[2 * (THREADS / 32)], cl[kRecCandCap], s_tau;
  const LmArgs& A = R.L;
  const int rows = A.rows < NB ? A.rows : NB;
  const int tps = R.tps;
  const int rlen = tps * kLmRows;
  uint32_t* qw = reinterpret_cast<uint32_t*>(dsm);                      // [NB][kLmMaxChunks * 32]
  float* lg = reinterpret_cast<float*>(dsm + static_cast<size_t>(NB) * kLmMaxChunks * 32 * 4);  // [NB][rlen]
  unsigned long long* buf = reinterpret_cast<unsigned long long*>(lg + static_cast<size_t>(NB) * rlen);  // [NB][rlen]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, half = lane & 1;
  const int64_t t_first = static_cast<int64_t>(blockIdx.x) * tps;
  const int ntile = static_cast<int>(A.tiles - t_first < tps ? A.tiles - t_first : tps);
  const int64_t v_lo = t_first * kLmRows;
  const int nids = static_cast<int>(A.vocab - v_lo < static_cast<int64_t>(ntile) * kLmRows ? A.vocab - v_lo
                                                                                          : static_cast<int64_t>(ntile) * kLmRows);
  lm_quant_act<NB>(qw, A, R.act, R.ld_act, rows);
  __syncthreads();
  // ---- logits: warp w takes quadrant w & 3 of tiles w >> 2, w >> 2 + THREADS / 128, ... ----
  for (int tt = warp >> 2; tt < ntile; tt += THREADS / 128) {
    const int quad = warp & 3;
    int32_t acc[2][NB];
    lm_tile_dots<NB>(A, qw, t_first + tt, quad, lane, acc);
    const int li = tt * kLmRows + 32 * quad + (lane >> 1) + 16 * half;  // local id
    const int64_t v = v_lo + li;
    if (v < A.vocab) {
      const float scale = A.scales[v];
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b < rows) {
          const float tt2 = __fmaf_rn(A.in_scale, static_cast<float>(half ? acc[1][b] : acc[0][b]),
                                      -(2.0f * A.act_sum[b]));
          float xl = srq(__fmul_rn(scale, tt2), A.out_scale);
          if (R.cap != 0.0f) xl = softcap(xl, R.cap, R.inv_cap);
          lg[static_cast<size_t>(b) * rlen + li] = xl;
        }
      }
    }
  }
  __syncthreads();
  // ---- the rows' statistics: two block-wide passes over every row at once ----
  const int nw = THREADS / 32;
  const uint32_t* mrow[NB];
  bool invalid[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int32_t state = (b < rows && R.mask_state) ? R.mask_state[b] : -1;
    const bool masked = R.mask_table != nullptr && state >= 0;
    const bool has_mask = masked && state < R.mask_states;
    mrow[b] = has_mask ? R.mask_table + static_cast<int64_t>(state) * R.mask_words : nullptr;
    invalid[b] = masked && !has_mask;
  }
  auto allowed = [&](int b, int i) -> bool {
    if (!mrow[b]) return true;
    const int64_t v = v_lo + i;
    return (__ldg(mrow[b] + (v >> 5)) >> (v & 31)) & 1u;
  };
  // ---- penalty history: the ids of this block's range leave the live set; their exact
  // penalised scores go to the record's fixed slots (sorted history position), as
  // gs_shard_partials writes them ----
  uint32_t* hs = reinterpret_cast<uint32_t*>(dsm + R.hist_off);  // [hsort] sorted history of a row
  uint32_t* penb = hs + R.hsort;                                 // [NB][rlen / 32]
  const int pw = rlen / 32;
  if (tid < NB) pen_fl[tid] = 0u;
  if (R.history) {
    for (int i = tid; i < NB * pw; i += THREADS) penb[i] = 0u;
    for (int b = 0; b < rows; ++b) {
      int64_t hl = R.history_len ? R.history_len[b] : 0;
      if (hl > R.history_stride) hl = R.history_stride;
      if (hl < 0) hl = 0;
      const int h2 = pow2_ceil(hl > 0 ? static_cast<int>(hl) : 1);
      const int32_t* hrow = R.history + static_cast<int64_t>(b) * R.history_stride;
      __syncthreads();
      for (int i = tid; i < h2; i += THREADS) hs[i] = i < hl ? static_cast<uint32_t>(hrow[i]) : 0xffffffffu;
      if (tid == 0) s_hl = static_cast<int>(hl);
      __syncthreads();
      bitonic_sort_u32(hs, h2);
      const RowPlan& pl = R.plan[b];
      unsigned char* r = R.records + (static_cast<int64_t>(blockIdx.x) * A.rows + b) * R.rec_bytes + sizeof(UnitStat) +
                         8ll * R.kcap;
      double* pkey = reinterpret_cast<double*>(r);
      uint32_t* pid = reinterpret_cast<uint32_t*>(r + 8ll * R.hcap);
      float* praw = reinterpret_cast<float*>(r + 12ll * R.hcap);
      for (int i = tid; i < R.hcap; i += THREADS) {
        double key = -INFINITY;
        uint32_t id = 0xffffffffu;
        float x = 0.0f;
        if (i < hl) {
          const uint32_t v = hs[i];  // negative ids sort past every vocabulary id
          const int64_t lv = static_cast<int64_t>(v) - v_lo;
          if (static_cast<int64_t>(v) < A.vocab && lv >= 0 && lv < nids && !(i > 0 && hs[i - 1] == v)) {
            atomicOr(&penb[b * pw + static_cast<int>(lv >> 5)], 1u << (lv & 31));
            if (allowed(b, static_cast<int>(lv))) {  // masked: -inf either way
              int cnt = 1;
              while (i + cnt < hl && hs[i + cnt] == v) ++cnt;
              x = lg[static_cast<size_t>(b) * rlen + lv];
              if (!(x < INFINITY)) atomicOr(&pen_fl[b], GS_FLAG_ERR_NONFINITE);  // NaN or +inf
              const double xp = penalise(static_cast<double>(x), static_cast<double>(cnt), pl.repetition_penalty,
                                         pl.presence_penalty, pl.frequency_penalty);
              key = pl.mode == kModeGreedy ? xp : __ddiv_rn(xp, pl.temperature);
              id = v;
            }
          }
        }
        pkey[i] = key;
        pid[i] = id;
        praw[i] = x;
      }
    }
  }
  __syncthreads();
  auto live = [&](int b, int i) -> bool {  // allowed and not penalised
    return allowed(b, i) && !(R.history && ((penb[b * pw + (i >> 5)] >> (i & 31)) & 1u));
  };
  {
    float lmax[NB], rmax[NB];
    int na[NB], bad[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      lmax[b] = -INFINITY;
      rmax[b] = -INFINITY;
      na[b] = 0;
      bad[b] = 0;
    }
    for (int i = tid; i < nids; i += THREADS) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b >= rows) break;
        const float xi = lg[static_cast<size_t>(b) * rlen + i];
        if (allowed(b, i)) {
          ++na[b];
          if (live(b, i)) {
            lmax[b] = fmaxf(lmax[b], xi);
            bad[b] |= xi != xi;
          }
        }
        rmax[b] = fmaxf(rmax[b], xi);
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        lmax[b] = fmaxf(lmax[b], __shfl_xor_sync(kFullMask, lmax[b], o));
        rmax[b] = fmaxf(rmax[b], __shfl_xor_sync(kFullMask, rmax[b], o));
        na[b] += __shfl_xor_sync(kFullMask, na[b], o);
        bad[b] |= __shfl_xor_sync(kFullMask, bad[b], o);
      }
      if (lane == 0) {
        red_f[0][b][warp] = lmax[b];
        red_f[1][b][warp] = rmax[b];
        red_i[0][b][warp] = na[b];
        red_i[1][b][warp] = bad[b];
      }
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        float m0 = lane < nw ? red_f[0][b][lane] : -INFINITY, r0 = lane < nw ? red_f[1][b][lane] : -INFINITY;
        int n0 = lane < nw ? red_i[0][b][lane] : 0, d0 = lane < nw ? red_i[1][b][lane] : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          m0 = fmaxf(m0, __shfl_xor_sync(kFullMask, m0, o));
          r0 = fmaxf(r0, __shfl_xor_sync(kFullMask, r0, o));
          n0 += __shfl_xor_sync(kFullMask, n0, o);
          d0 |= __shfl_xor_sync(kFullMask, d0, o);
        }
        if (lane == 0) {
          fin_lm[b] = m0;
          fin_rm[b] = r0;
          fin_na[b] = n0;
          fin_bad[b] = d0;
        }
      }
    }
    __syncthreads();
  }
  {
    float sp[NB], rp[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      sp[b] = 0.0f;
      rp[b] = 0.0f;
    }
    for (int i = tid; i < rlen; i += THREADS) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b >= rows) break;
        const RowPlan& pl = R.plan[b];
        const float m = pl.mode != kModeGreedy ? fin_lm[b] : -INFINITY;  // greedy: no normaliser (as the stream pass)
        const float rm = fin_rm[b];
        unsigned long long pk = 0ull;
        if (i < nids) {
          const float xi = lg[static_cast<size_t>(b) * rlen + i];
          if (live(b, i)) {
            if (m > -INFINITY) {
              const float d = xi - m;
              sp[b] += ex2_approx(fmaf(d, pl.a2_lo, d * pl.a2_hi));
            }
            if (xi == xi) pk = make_pack(xi, static_cast<uint32_t>(v_lo + i));
          }
          if (rm > -INFINITY) {
            const float g = xi - rm;
            rp[b] += ex2_approx(fmaf(g, kL2eLo, g * kL2eHi));
          }
        }
        buf[static_cast<size_t>(b) * rlen + i] = pk;
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      double s0 = sp[b], r0 = rp[b];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        s0 += __shfl_xor_sync(kFullMask, s0, o);
        r0 += __shfl_xor_sync(kFullMask, r0, o);
      }
      if (lane == 0) {
        red_d[0][b][warp] = s0;
        red_d[1][b][warp] = r0;
      }
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        double s0 = lane < nw ? red_d[0][b][lane] : 0.0, r0 = lane < nw ? red_d[1][b][lane] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          s0 += __shfl_xor_sync(kFullMask, s0, o);
          r0 += __shfl_xor_sync(kFullMask, r0, o);
        }
        if (lane == 0) {
          fin_s[b] = s0;
          fin_rs[b] = r0;
        }
      }
    }
    __syncthreads();
  }
  // ---- per row: the shard's k best packs, then the record's statistics ----
  for (int b = 0; b < rows; ++b) {
    const RowPlan& pl = R.plan[b];
    const unsigned long long* pb = buf + static_cast<size_t>(b) * rlen;
    unsigned char* rec = R.records + (static_cast<int64_t>(blockIdx.x) * A.rows + b) * R.rec_bytes;
    unsigned long long* packs = reinterpret_cast<unsigned long long*>(rec + sizeof(UnitStat));
    const int k = pl.k_eff > 0 ? pl.k_eff : 1;
    if (tid == 0) {
      n_out = 0;
      n_cl = 0;
    }
    __syncthreads();
    bool done = false;
    if (fin_na[b] > k && 2 * nw >= k) {
      // A lower bound on the k-th largest pack: the k-th largest of the warps' top-2 packs
      // (k distinct packs are at or above it).  The packs at or above it (usually a few
      // times k) go to a short list, ranked by counting: three block barriers in all.
      unsigned long long t1 = 0ull, t2 = 0ull;
      for (int i = tid; i < nids; i += THREADS) {
        const unsigned long long v = pb[i];
        if (v > t1) {
          t2 = t1;
          t1 = v;
        } else if (v > t2) {
          t2 = v;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {  // disjoint lane sets at every step: (top, second) of the union
        const unsigned long long u1 = __shfl_xor_sync(kFullMask, t1, o), u2 = __shfl_xor_sync(kFullMask, t2, o);
        const unsigned long long lo = t1 < u1 ? t1 : u1, s2 = t2 > u2 ? t2 : u2;
        t1 = t1 > u1 ? t1 : u1;
        t2 = lo > s2 ? lo : s2;
      }
      if (lane == 0) {
        top2[2 * warp] = t1;
        top2[2 * warp + 1] = t2;
      }
      __syncthreads();
      if (warp == 0) {
        unsigned long long tau = 0ull;
        for (int j = lane; j < 2 * nw; j += 32) {
          const unsigned long long v = top2[j];
          int above = 0;
#pragma unroll 4
          for (int q = 0; q < 2 * nw; ++q) above += top2[q] > v;
          if (v != 0ull && above == k - 1) tau = v;  // distinct non-zero packs: one has rank k
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const unsigned long long u = __shfl_xor_sync(kFullMask, tau, o);
          tau = u > tau ? u : tau;
        }
        if (lane == 0) s_tau = tau;
      }
      __syncthreads();
      const unsigned long long tau = s_tau;
      if (tau != 0ull) {
        for (int i = tid; i < nids; i += THREADS) {
          const unsigned long long v = pb[i];
          if (v >= tau) {
            const int slot = atomicAdd(&n_cl, 1);
            if (slot < kRecCandCap) cl[slot] = v;
          }
        }
        __syncthreads();
        const int nc = n_cl;
        if (nc <= kRecCandCap && nc >= k) {  // rank of each listed pack by counting (distinct packs)
          for (int j = tid; j < nc; j += THREADS) {
            const unsigned long long v = cl[j];
            int above = 0;
#pragma unroll 4
            for (int q = 0; q < nc; ++q) above += cl[q] > v;
            if (above < k) packs[above] = v;
          }
          if (tid == 0) n_out = k;
          done = true;
        }
      }
    }
    if (done) {
    } else if (fin_na[b] > k) {
      unsigned long long prefix, mask;
      select_threshold(pb, nids, k, sel_hist, &sel_digit, &sel_above, &sel_binc, prefix, mask);
      for (int i = tid; i < nids; i += THREADS) {
        const unsigned long long v = pb[i];
        if (v != 0ull && (v & mask) >= prefix) packs[atomicAdd(&n_out, 1)] = v;
      }
    } else {
      for (int i = tid; i < nids; i += THREADS)
        if (pb[i] != 0ull) packs[atomicAdd(&n_out, 1)] = pb[i];
    }
    __syncthreads();
    if (tid == 0) {
      const float m = pl.mode != kModeGreedy ? fin_lm[b] : -INFINITY;
      const float rm = fin_rm[b];
      const double ssum = fin_s[b], rsum = fin_rs[b];
      UnitStat u{};
      u.m = m;
      u.raw_m = rm;
      u.s = m > -INFINITY ? ssum : 0.0;
      u.raw_s = rm > -INFINITY ? rsum : 0.0;
      u.n_allowed = fin_na[b];
      u.n_cand = n_out;
      const bool nonfinite = fin_bad[b] || ssum != ssum || (R.want_raw && rsum != rsum) || m == INFINITY;
      u.flags = (nonfinite ? GS_FLAG_ERR_NONFINITE : 0u) | (invalid[b] ? GS_FLAG_ERR_INVALID : 0u) | pen_fl[b];
      u.pad = 1;  // raw sums recorded
      *reinterpret_cast<UnitStat*>(rec) = u;
    }
  }

  // ---- the last block to finish combines every shard's record of a row into one (the
  // merge then reads one record per row: its top-k select runs here, over the shards'
  // packs above a bound, instead of over all 147 x k packs in one CTA).  One block does
  // it row after row (~12 us a row against ~13 us saved in the merge per call), so the
  // host asks for it at one row only. ----
  if (!R.combined) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(R.done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int S = gridDim.x;
  const int kc = R.kcap;
  unsigned long long* gp = reinterpret_cast<unsigned long long*>(dsm);  // [S][kc] packs
  unsigned long long* smax = gp + static_cast<size_t>(S) * kc;           // [S] each shard's best pack
  auto rec_at = [&](int u, int b) -> const unsigned char* {
    return R.records + (static_cast<int64_t>(u) * A.rows + b) * R.rec_bytes;
  };
  for (int b = 0; b < rows; ++b) {
    const RowPlan& pl = R.plan[b];
    const int k = pl.k_eff > 0 ? pl.k_eff : 1;
    // statistics: maxima, counts and flags, then the sums rescaled to the maxima (the
    // combination gs_shard_partials applies to its units)
    float um = -INFINITY, rmx = -INFINITY;
    int na = 0;
    unsigned fl = 0;
    for (int u = tid; u < S; u += THREADS) {
      const UnitStat* st = reinterpret_cast<const UnitStat*>(rec_at(u, b));
      um = fmaxf(um, __ldcg(&st->m));
      rmx = fmaxf(rmx, __ldcg(&st->raw_m));
      na += __ldcg(&st->n_allowed);
      fl |= __ldcg(reinterpret_cast<const unsigned*>(&st->flags));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      um = fmaxf(um, __shfl_xor_sync(kFullMask, um, o));
      rmx = fmaxf(rmx, __shfl_xor_sync(kFullMask, rmx, o));
      na += __shfl_xor_sync(kFullMask, na, o);
      fl |= __shfl_xor_sync(kFullMask, fl, o);
    }
    if (lane == 0) {
      red_f[0][0][warp] = um;
      red_f[1][0][warp] = rmx;
      red_i[0][0][warp] = na;
      red_i[1][0][warp] = static_cast<int>(fl);
    }
    __syncthreads();
    if (warp == 0) {
      float m0 = lane < nw ? red_f[0][0][lane] : -INFINITY, r0 = lane < nw ? red_f[1][0][lane] : -INFINITY;
      int n0 = lane < nw ? red_i[0][0][lane] : 0;
      unsigned f0 = lane < nw ? static_cast<unsigned>(red_i[1][0][lane]) : 0u;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        m0 = fmaxf(m0, __shfl_xor_sync(kFullMask, m0, o));
        r0 = fmaxf(r0, __shfl_xor_sync(kFullMask, r0, o));
        n0 += __shfl_xor_sync(kFullMask, n0, o);
        f0 |= __shfl_xor_sync(kFullMask, f0, o);
      }
      if (lane == 0) {
        fin_lm[0] = m0;
        fin_rm[0] = r0;
        fin_na[0] = n0;
        fin_bad[0] = static_cast<int>(f0);
      }
    }
    __syncthreads();
    const float M = fin_lm[0], RM = fin_rm[0];
    double sm = 0.0, rs = 0.0;
    for (int u = tid; u < S; u += THREADS) {
      const UnitStat* st = reinterpret_cast<const UnitStat*>(rec_at(u, b));
      const float mu = __ldcg(&st->m), ru = __ldcg(&st->raw_m);
      if (mu > -INFINITY)
        sm = __dadd_rn(sm, __dmul_rn(__ldcg(&st->s), exp2(__dmul_rn(static_cast<double>(mu) - static_cast<double>(M), pl.a2))));
      if (ru > -INFINITY)
        rs = __dadd_rn(rs, __dmul_rn(__ldcg(&st->raw_s), exp(static_cast<double>(ru) - static_cast<double>(RM))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sm += __shfl_xor_sync(kFullMask, sm, o);
      rs += __shfl_xor_sync(kFullMask, rs, o);
    }
    if (lane == 0) {
      red_d[0][0][warp] = sm;
      red_d[1][0][warp] = rs;
    }
    // every shard's packs (0: empty slot), then each shard's best
    for (int i = tid; i < S * kc; i += THREADS) {
      const int u = i / kc, j = i - u * kc;
      const unsigned char* r = rec_at(u, b);
      const int nc = __ldcg(&reinterpret_cast<const UnitStat*>(r)->n_cand);
      gp[i] = j < nc ? __ldcg(reinterpret_cast<const unsigned long long*>(r + sizeof(UnitStat)) + j) : 0ull;
    }
    if (tid == 0) {
      n_out = 0;
      n_cl = 0;
      n_tot = 0;
      s_tau = 0ull;
    }
    __syncthreads();
    if (warp == 0) {
      double s0 = lane < nw ? red_d[0][0][lane] : 0.0, r0 = lane < nw ? red_d[1][0][lane] : 0.0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        s0 += __shfl_xor_sync(kFullMask, s0, o);
        r0 += __shfl_xor_sync(kFullMask, r0, o);
      }
      if (lane == 0) {
        fin_s[0] = s0;
        fin_rs[0] = r0;
      }
    }
    int npk = 0;
    for (int u = tid; u < S; u += THREADS) {
      unsigned long long mx = 0ull;
      for (int j = 0; j < kc; ++j) mx = gp[u * kc + j] > mx ? gp[u * kc + j] : mx;
      smax[u] = mx;
    }
    for (int i = tid; i < S * kc; i += THREADS) npk += gp[i] != 0ull;
    if (npk) atomicAdd(&n_tot, npk);
    __syncthreads();
    const int total = n_tot;
    unsigned char* out = R.combined + static_cast<int64_t>(b) * R.rec_bytes;
    unsigned long long* opk = reinterpret_cast<unsigned long long*>(out + sizeof(UnitStat));
    bool done = false;
    if (total <= k) {
      for (int i = tid; i < S * kc; i += THREADS)
        if (gp[i] != 0ull) opk[atomicAdd(&n_out, 1)] = gp[i];
      done = true;
    } else if (k <= S) {
      // bound: the k-th largest of the shards' best packs (k distinct packs at or above
      // it; none when fewer than k shards hold packs)
      for (int u = tid; u < S; u += THREADS) {
        const unsigned long long v = smax[u];
        int above = 0;
#pragma unroll 4
        for (int q = 0; q < S; ++q) above += smax[q] > v;
        if (v != 0ull && above == k - 1) s_tau = v;
      }
      __syncthreads();
      const unsigned long long tau = s_tau;
      if (tau != 0ull) {
        for (int i = tid; i < S * kc; i += THREADS) {
          const unsigned long long v = gp[i];
          if (v >= tau) {
            const int slot = atomicAdd(&n_cl, 1);
            if (slot < kRecCandCap) cl[slot] = v;
          }
        }
        __syncthreads();
        const int nc = n_cl;
        if (nc <= kRecCandCap && nc >= k) {
          for (int j = tid; j < nc; j += THREADS) {
            const unsigned long long v = cl[j];
            int above = 0;
#pragma unroll 4
            for (int q = 0; q < nc; ++q) above += cl[q] > v;
            if (above < k) opk[above] = v;
          }
          if (tid == 0) n_out = k;
          done = true;
        }
      }
    }
    if (!done) {
      unsigned long long prefix, mask;
      select_threshold(gp, S * kc, k, sel_hist, &sel_digit, &sel_above, &sel_binc, prefix, mask);
      for (int i = tid; i < S * kc; i += THREADS) {
        const unsigned long long v = gp[i];
        if (v != 0ull && (v & mask) >= prefix) opk[atomicAdd(&n_out, 1)] = v;
      }
    }
    __syncthreads();
    if (tid == 0) {
      UnitStat u{};
      u.m = M;
      u.raw_m = RM;
      u.s = M > -INFINITY ? fin_s[0] : 0.0;
      u.raw_s = RM > -INFINITY ? fin_rs[0] : 0.0;
      u.n_allowed = fin_na[0];
      u.n_cand = n_out;
      u.flags = static_cast<unsigned>(fin_bad[0]);
      u.pad = 1;
      *reinterpret_cast<UnitStat*>(out) = u;
    }
    if (R.history && rows == 1) {
      // penalised slots: slot i (sorted history position) from the shard that holds its id
      // (the sort buffer still holds this row's sorted history)
      const int hl = s_hl;
      unsigned char* orr = out + sizeof(UnitStat) + 8ll * R.kcap;
      for (int i = tid; i < R.hcap; i += THREADS) {
        double key = -INFINITY;
        uint32_t id = 0xffffffffu;
        float x = 0.0f;
        if (i < hl) {
          const uint32_t v = hs[i];
          if (static_cast<int64_t>(v) < A.vocab && !(i > 0 && hs[i - 1] == v)) {
            const int u = static_cast<int>(v / static_cast<uint32_t>(R.tps * kLmRows));
            const unsigned char* ur = rec_at(u, b) + sizeof(UnitStat) + 8ll * R.kcap;
            key = __ldcg(reinterpret_cast<const double*>(ur) + i);
            id = __ldcg(reinterpret_cast<const unsigned*>(ur + 8ll * R.hcap) + i);
            x = __ldcg(reinterpret_cast<const float*>(ur + 12ll * R.hcap) + i);
          }
        }
        reinterpret_cast<double*>(orr)[i] = key;
        reinterpret_cast<uint32_t*>(orr + 8ll * R.hcap)[i] = id;
        reinterpret_cast<float*>(orr + 12ll * R.hcap)[i] = x;
      }
    }
    __syncthreads();
  }
  if (tid == 0) *R.done = 0u;  // ready for the next call (stream order)
}

// Unquantised activations (inScale == 0): one thread per vocab row and batch row, Σ code·a
// in double element by element (every product exact), t = (float)(Σ - 2·sumA).
__global__ void __launch_bounds__(128) lm_f64_kernel(const __grid_constant__ LmArgs A, const float* __restrict__ act,
                                                     int64_t ld_act, int hidden) {
  const int64_t v = static_cast<int64_t>(blockIdx.x) * 128 + threadIdx.x;
  const int b = blockIdx.y;
  if (v >= A.vocab || b >= A.rows) return;
  const int64_t t = v / kLmRows;
  const int r = static_cast<int>(v % kLmRows);
  const float* a = act + static_cast<int64_t>(b) * ld_act;
  double s = 0.0;
  for (int c = 0; c < A.chunks; ++c) {
    const uint32_t* wrow = A.packed + ((static_cast<size_t>(t) * A.chunks + c) * kLmRows + r) * 8;
    for (int w = 0; w < 8; ++w) {
      const uint32_t x = wrow[w];
      const float* aw = a + c * kLmKC + w * 16;
#pragma unroll
      for (int jj = 0; jj < 16; ++jj)
        s = __dadd_rn(s, __dmul_rn(static_cast<double>((x >> (2 * jj)) & 3u), static_cast<double>(__ldg(aw + jj))));
    }
  }
  const float tt = static_cast<float>(__dsub_rn(s, 2.0 * static_cast<double>(A.act_sum[b])));
  A.logits[static_cast<int64_t>(b) * A.ld + v] = srq(__fmul_rn(A.scales[v], tt), A.out_scale);
}

gs_status lfail(gs_lm_head* h, gs_status s, const std::string& m) {
  h->err = m;
  return s;
}

void release(gs_lm_head* h) {
  cudaFree(h->packed);
  cudaFree(h->scales);
  cudaFree(h->img);
  cudaFree(h->flag);
  cudaFree(h->scratch);
  h->scratch = nullptr;
  h->scratch_bytes = 0;
  cudaFree(h->records);
  h->records = nullptr;
  h->records_bytes = 0;
  h->packed = nullptr;
  h->scales = nullptr;
  h->img = nullptr;
  h->flag = nullptr;
}

}  // namespace
}  // namespace gs

using namespace gs;

extern "C" {

gs_status gs_lm_head_create(gs_ctx* ctx, const gs_lm_head_desc* d, gs_lm_head** out) {
  if (!out) return GS_EINVAL;
  *out = nullptr;
  if (!ctx || !d) return GS_EINVAL;
  if (d->vocab <= 0 || d->vocab >= (1ll << 31) || !d->packed || !d->row_scales) {
    ctx_set_error(ctx, "LM head: vocab in (0, 2^31), packed weights and row scales are required");
    return GS_EINVAL;
  }
  if (d->hidden <= 0 || d->hidden % kLmKC != 0 || d->hidden > kLmKC * kLmMaxChunks) {
    ctx_set_error(ctx, "LM head: hidden must be a multiple of 128, at most 1536");
    return GS_EINVAL;
  }
  if (!(d->input_scale >= 0.0f) || !(d->output_scale >= 0.0f) || d->input_scale == INFINITY ||
      d->output_scale == INFINITY) {
    ctx_set_error(ctx, "LM head: input / output scales must be finite and >= 0");
    return GS_EINVAL;
  }
  auto* h = new gs_lm_head();
  h->ctx = ctx;
  h->device = ctx_device(ctx);
  h->vocab = d->vocab;
  h->hidden = d->hidden;
  h->chunks = d->hidden / kLmKC;
  h->tiles = (d->vocab + kLmRows - 1) / kLmRows;
  h->in_scale = d->input_scale;
  h->out_scale = d->output_scale;
  const int words = d->hidden / 16;
  // tile-major repack (decode-lm-head.ts keeps row-major words; rows past vocab hold code 2,
  // weight 0, and scale 0)
  std::vector<uint32_t> tp(static_cast<size_t>(h->tiles) * h->chunks * kLmRows * 8, 0xAAAAAAAAu);
  for (int64_t v = 0; v < d->vocab; ++v) {
    const int64_t t = v / kLmRows;
    const int r = static_cast<int>(v % kLmRows);
    for (int c = 0; c < h->chunks; ++c)
      std::memcpy(&tp[((static_cast<size_t>(t) * h->chunks + c) * kLmRows + r) * 8],
                  d->packed + static_cast<size_t>(v) * words + c * 8, 32);
  }
  std::vector<float> sc(static_cast<size_t>(h->tiles) * kLmRows, 0.0f);
  std::memcpy(sc.data(), d->row_scales, static_cast<size_t>(d->vocab) * sizeof(float));
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != h->device) cudaSetDevice(h->device);
  cudaError_t e = cudaMalloc(&h->packed, tp.size() * 4);
  if (e == cudaSuccess) e = cudaMemcpy(h->packed, tp.data(), tp.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&h->scales, sc.size() * 4);
  if (e == cudaSuccess) e = cudaMemcpy(h->scales, sc.data(), sc.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&h->flag, 8);
  if (e == cudaSuccess) e = cudaMemset(h->flag, 0, 8);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, h->device);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(lm_mma_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, LmPlan<16>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(lm_mma_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, LmPlan<64>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(lm_mma_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, LmPlan<128>::kSmem);
  if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
  if (e != cudaSuccess) {
    ctx_set_error(ctx, (std::string("LM head upload: ") + cudaGetErrorString(e)).c_str());
    release(h);
    delete h;
    return GS_ENOMEM;
  }
  *out = h;
  return GS_OK;
}

gs_status gs_lm_head_destroy(gs_lm_head* h) {
  if (!h) return GS_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != h->device) cudaSetDevice(h->device);
  cudaDeviceSynchronize();
  release(h);
  if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
  delete h;
  return GS_OK;
}

const char* gs_lm_head_last_error(const gs_lm_head* h) { return h ? h->err.c_str() : ""; }

gs_status gs_lm_head_logits(gs_lm_head* h, const float* activation, int64_t ld_activation, const float* activation_sum,
                            int32_t rows, float* logits, int64_t ld_logits, void* stream) {
  if (!h) return GS_EINVAL;
  if (rows < 0 || (rows > 0 && (!activation || !activation_sum || !logits)))
    return lfail(h, GS_EINVAL, "activation, activation_sum and logits are required");
  if (ld_activation < h->hidden || ld_logits < h->vocab)
    return lfail(h, GS_EINVAL, "ld_activation >= hidden and ld_logits >= vocab are required");
  if (rows > 65535) return lfail(h, GS_EUNSUPPORTED, "at most 65535 rows per call");
  if (rows == 0) return GS_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != h->device) cudaSetDevice(h->device);
  auto restore = [&]() {
    if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
  };
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LmArgs a{};
  a.packed = h->packed;
  a.scales = h->scales;
  a.act_sum = activation_sum;
  a.logits = logits;
  a.ld = ld_logits;
  a.vocab = h->vocab;
  a.tiles = h->tiles;
  a.chunks = h->chunks;
  a.rows = rows;
  a.in_scale = h->in_scale;
  a.out_scale = h->out_scale;
  a.flag = h->flag;
  cudaError_t e = cudaSuccess;
  if (h->in_scale == 0.0f) {
    dim3 grid(static_cast<unsigned>(h->tiles), static_cast<unsigned>(rows));
    lm_f64_kernel<<<grid, 128, 0, st>>>(a, activation, ld_activation, h->hidden);
    e = cudaGetLastError();
  } else {
    // N of the tensor-core kernel: the accumulator width, rows per pass
    const int n_mma = rows <= 16 ? 16 : rows <= 64 ? 64 : 128;
    const int passes = (rows + n_mma - 1) / n_mma * (n_mma > kImgRows ? n_mma / kImgRows : 1);  // image passes
    const size_t img = static_cast<size_t>(passes) * h->chunks * (kImgRows * kLmKC);
    const size_t need = img + static_cast<size_t>(passes) * kImgRows * 4;
    if (need > h->img_bytes) {  // (grown on demand; the first call of a larger batch allocates)
      cudaStreamSynchronize(st);
      cudaFree(h->img);
      h->img = nullptr;
      h->img_bytes = 0;
      e = cudaMalloc(&h->img, need);
      if (e != cudaSuccess) {
        restore();
        return lfail(h, GS_ENOMEM, std::string("activation image: ") + cudaGetErrorString(e));
      }
      h->img_bytes = need;
    }
    a.img = h->img;
    a.qsum = reinterpret_cast<const int32_t*>(h->img + img);
    if (rows > kGemvRows)
      lm_quant_kernel<<<passes * kImgRows, 256, 0, st>>>(activation, ld_activation, rows, h->hidden, h->in_scale,
                                                         h->img, reinterpret_cast<int32_t*>(h->img + img));
    const int gx = static_cast<int>(h->tiles < h->num_sms ? h->tiles : h->num_sms);
    // (up to kGemvRows rows: the dp4a GEMV; a few more: a 16-column accumulator, a smaller
    // activation image and a deeper packed-block ring; otherwise passes of 64 rows, the
    // image's pass size)
    if (rows <= kGemvRows) {
      // persistent: as many blocks as stay resident (whole waves), each looping over tiles
      auto gemv = [&](auto kern) {
        int per_sm = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 128, 0);
        const int64_t g = static_cast<int64_t>(per_sm > 0 ? per_sm : 1) * h->num_sms;
        kern<<<static_cast<unsigned>(g < h->tiles ? g : h->tiles), 128, 0, st>>>(a, activation, ld_activation);
      };
      if (rows <= 1) gemv(lm_gemv_kernel<1>);
      else if (rows <= 2) gemv(lm_gemv_kernel<2>);
      else if (rows <= 4) gemv(lm_gemv_kernel<4>);
      else if (rows <= 8) gemv(lm_gemv_kernel<8>);
      else gemv(lm_gemv_kernel<16>);
      static_assert(kGemvRows <= 16, "GEMV instantiations cover up to 16 rows");
    } else if (n_mma == 16) {
      a.pass_rows = 16;
      lm_mma_kernel<16><<<dim3(gx, 1), kLmThreads, LmPlan<16>::kSmem, st>>>(a);
    } else if (n_mma == 64) {
      a.pass_rows = 64;
      lm_mma_kernel<64><<<dim3(gx, passes), kLmThreads, LmPlan<64>::kSmem, st>>>(a);
    } else {
      a.pass_rows = 128;
      lm_mma_kernel<128><<<dim3(gx, passes / 2), kLmThreads, LmPlan<128>::kSmem, st>>>(a);
    }
    e = cudaGetLastError();
  }
  restore();
  if (e != cudaSuccess) return lfail(h, GS_ECUDA, std::string("LM head launch: ") + cudaGetErrorString(e));
  return GS_OK;
}

gs_status gs_lm_head_sample(gs_lm_head* h, const float* activation, int64_t ld_activation, const float* activation_sum,
                            const gs_batch* batch, const gs_outputs* out, void* stream) {
  if (!h || !batch) return GS_EINVAL;
  if (batch->logits) return lfail(h, GS_EINVAL, "gs_lm_head_sample computes the logits: batch->logits must be NULL");
  if (batch->vocab != 0 && batch->vocab != h->vocab) return lfail(h, GS_EINVAL, "batch->vocab must be 0 or the head's vocab");
  const int32_t rows = batch->rows;
  if (rows < 0 || rows > 65535) return lfail(h, GS_EINVAL, "rows must be in [0, 65535]");
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != h->device) cudaSetDevice(h->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Fused: up to kRecMaxRows rows of int8-grid activations (a penalty history at one row),
  // every row 1 <= topK <= kRecMaxK or greedy: the LM head writes shard records, the merge
  // samples them.
  bool fused = rows >= 1 && rows <= kRecMaxRows && h->in_scale != 0.0f && batch->params &&
               (batch->params_count == 1 || batch->params_count == rows) &&
               // a penalty history at one row only: the records are then combined into one, and the
               // merge plans its penalised slots as gs_sample does for one row (147 shards' slots
               // would not fit its shared memory)
               (!batch->history || (rows == 1 && batch->history_stride >= 1 && batch->history_stride <= kRecMaxHistory)) &&
               // (history counts: the two-step route, whose kernels read them)
               !(batch->history && batch->history_count);
  int kcap = 1;
  RecArgs ra{};
  if (fused) {
    for (int i = 0; i < rows && fused; ++i) {
      // (a row whose params fail validation leaves the fused route before it is planned;
      // the other route's batch check then reports the error)
      const gs_params& pr = batch->params[batch->params_count == 1 ? 0 : i];
      if (!valid_params(pr, nullptr)) {
        fused = false;
        break;
      }
      const RowPlan pl = make_plan(pr, h->vocab);
      if (pl.mode == kModeLarge || pl.k_eff > kRecMaxK) fused = false;
      ra.plan[i] = pl;
      kcap = pl.k_eff > kcap ? pl.k_eff : kcap;
    }
  }
  if (fused && h->route == GS_LM_ROUTE_TWO_STEP) fused = false;
  if (fused && h->route == GS_LM_ROUTE_AUTO) {
    // the two-step route is faster wherever its gs_sample takes the single-launch decode
    // step (one launch after the GEMV against the records kernel plus a 147-record merge)
    gs_batch b2 = *batch;
    b2.logits = nullptr;  // (the scratch it would sample: 256-byte aligned)
    b2.dtype = GS_DTYPE_F32;
    b2.vocab = h->vocab;
    b2.row_stride = h->vocab;
    if (step_eligible(&b2, kcap, false, rows)) fused = false;
  }
  const int tps = static_cast<int>((h->tiles + h->num_sms - 1) / h->num_sms);
  const int shards = static_cast<int>((h->tiles + tps - 1) / tps);
  const int nb = rows <= 1 ? 1 : 2;
  const int hcap = batch->history ? static_cast<int>(batch->history_stride) : 0;
  const int hsort = batch->history ? pow2_ceil_host(hcap) : 0;
  if (fused && rec_smem_bytes(nb, tps, shards, kcap, hsort) > 200 * 1024) fused = false;
  if (fused) {
    // the argument checks of gs_lm_head_logits, then the merge's batch checks, before any launch
    if (!activation || !activation_sum || ld_activation < h->hidden) {
      if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
      return lfail(h, GS_EINVAL, !activation || !activation_sum ? "activation, activation_sum and logits are required"
                                                                 : "ld_activation >= hidden and ld_logits >= vocab are required");
    }
    gs_batch b = *batch;
    b.logits = nullptr;
    b.dtype = GS_DTYPE_F32;
    b.vocab = h->vocab;
    b.row_stride = h->vocab;
    std::string err;
    const gs_status cs = check_batch(&b, out, &err, kCheckNoLogits);
    if (cs != GS_OK) {
      if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
      return lfail(h, cs, "sampling: " + err);
    }
    const int64_t rec_bytes = shard_record_bytes(kcap, hcap);
    const size_t rneed = static_cast<size_t>(shards + 1) * rows * rec_bytes;  // the shards' records, then the rows' combined
    if (rneed > h->records_bytes) {  // (grown on demand; the first call of a larger batch allocates)
      cudaStreamSynchronize(st);
      cudaFree(h->records);
      h->records = nullptr;
      h->records_bytes = 0;
      cudaError_t e = cudaMalloc(&h->records, rneed);
      if (e != cudaSuccess) {
        if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
        return lfail(h, GS_ENOMEM, std::string("shard records: ") + cudaGetErrorString(e));
      }
      h->records_bytes = rneed;
    }
    ra.L.packed = h->packed;
    ra.L.scales = h->scales;
    ra.L.act_sum = activation_sum;
    ra.L.vocab = h->vocab;
    ra.L.tiles = h->tiles;
    ra.L.chunks = h->chunks;
    ra.L.rows = rows;
    ra.L.in_scale = h->in_scale;
    ra.L.out_scale = h->out_scale;
    ra.L.flag = h->flag;
    ra.act = activation;
    ra.ld_act = ld_activation;
    ra.cap = batch->softcap;
    ra.inv_cap = batch->softcap != 0.0f ? static_cast<float>(1.0 / static_cast<double>(batch->softcap)) : 0.0f;
    ra.mask_table = batch->mask_table;
    ra.mask_states = batch->mask_states;
    ra.mask_words = batch->mask_words;
    ra.mask_state = batch->mask_table ? batch->mask_state : nullptr;
    ra.records = h->records;
    ra.rec_bytes = rec_bytes;
    ra.tps = tps;
    ra.want_raw = out->logprob != nullptr;
    ra.kcap = kcap;
    ra.done = reinterpret_cast<unsigned*>(h->flag + 1);
    ra.history = batch->history;
    ra.history_len = batch->history ? batch->history_len : nullptr;
    ra.history_stride = batch->history ? batch->history_stride : 0;
    ra.hcap = hcap;
    ra.hsort = hsort;
    ra.hist_off = static_cast<int64_t>(rec_base_bytes(nb, tps, shards, kcap));
    ra.combined = rows == 1 ? h->records + static_cast<size_t>(shards) * rows * rec_bytes : nullptr;
    const size_t smem = rec_smem_bytes(nb, tps, shards, kcap, hsort);
    cudaError_t e = cudaSuccess;
    auto go = [&](auto kern) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e == cudaSuccess) {
        kern<<<shards, 1024, smem, st>>>(ra);
        e = cudaGetLastError();
      }
    };
    if (nb == 1) go(lm_records_kernel<1, 1024>);
    else go(lm_records_kernel<2, 1024>);
    if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
    if (e != cudaSuccess) return lfail(h, GS_ECUDA, std::string("LM head records launch: ") + cudaGetErrorString(e));
    gs_status s = ra.combined ? gs_shard_merge(h->ctx, &b, 1, ra.combined, out, stream)
                              : gs_shard_merge(h->ctx, &b, shards, h->records, out, stream);
    if (s != GS_OK) h->err = std::string("sampling: ") + gs_last_error(h->ctx);
    else ++h->fused_calls;
    return s;
  }
  const size_t need = static_cast<size_t>(rows) * static_cast<size_t>(h->vocab) * sizeof(float);
  if (need > h->scratch_bytes) {  // (grown on demand; the first call of a larger batch allocates)
    cudaStreamSynchronize(st);
    cudaFree(h->scratch);
    h->scratch = nullptr;
    h->scratch_bytes = 0;
    cudaError_t e = cudaMalloc(&h->scratch, need > 0 ? need : 4);
    if (e != cudaSuccess) {
      if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
      return lfail(h, GS_ENOMEM, std::string("logits scratch: ") + cudaGetErrorString(e));
    }
    h->scratch_bytes = need;
  }
  if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
  gs_status s = gs_lm_head_logits(h, activation, ld_activation, activation_sum, rows, h->scratch, h->vocab, stream);
  if (s != GS_OK) return s;
  gs_batch b = *batch;
  b.logits = h->scratch;
  b.dtype = GS_DTYPE_F32;
  b.vocab = h->vocab;
  b.row_stride = h->vocab;
  s = gs_sample(h->ctx, &b, out, stream);
  if (s != GS_OK) h->err = std::string("sampling: ") + gs_last_error(h->ctx);
  return s;
}

int64_t gs_lm_head_fused_calls(const gs_lm_head* h) { return h ? h->fused_calls : -1; }

gs_status gs_lm_head_set_route(gs_lm_head* h, int32_t route) {
  if (!h) return GS_EINVAL;
  if (route != GS_LM_ROUTE_AUTO && route != GS_LM_ROUTE_FUSED && route != GS_LM_ROUTE_TWO_STEP)
    return lfail(h, GS_EINVAL, "route must be GS_LM_ROUTE_AUTO, GS_LM_ROUTE_FUSED or GS_LM_ROUTE_TWO_STEP");
  h->route = route;
  return GS_OK;
}

gs_status gs_lm_head_check(gs_lm_head* h, int32_t* timed_out) {
  if (!h || !timed_out) return GS_EINVAL;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != h->device) cudaSetDevice(h->device);
  int32_t f = 0;
  cudaError_t e = cudaMemcpy(&f, h->flag, 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && f) e = cudaMemset(h->flag, 0, 4);
  if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
  if (e != cudaSuccess) return lfail(h, GS_ECUDA, std::string("LM head flag: ") + cudaGetErrorString(e));
  *timed_out = f;
  return f ? GS_ETIMEOUT : GS_OK;
}

}  // extern "C"
