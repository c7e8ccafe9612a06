/*
 * gsampler — B200 (sm_100a) decode-sampling path, C ABI.
 *
 * Drop-in for the full-logit sampling path of aribornstein/gemma-webgpu-engine's
 * session.generate(): the reference runs it on the JS main thread over a 1 MiB
 * Float32Array read back per token; here the logits stay in device memory and only the
 * sampled ids (and optional log-probabilities) come back.
 *
 * Each entry point names the reference interface it replaces (file:line in the
 * reference repository).  All pointers are plain device pointers unless a comment says
 * "host"; sizes are element counts.  No entry point aborts: failures return a status
 * and gs_last_error() gives the text.
 */
#ifndef GSAMPLER_H_
#define GSAMPLER_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum gs_status {
  GS_OK = 0,
  GS_EINVAL = 1,        /* bad argument (reference: throw new Error(...)) */
  GS_EDEADEND = 2,      /* a constrained row admits no token
                           ("Generation constraint reached a tokenization dead end",
                           src/runtime/gemma-session.ts:1324-1326) */
  GS_ECUDA = 3,         /* a CUDA runtime call failed */
  GS_ENCCL = 4,         /* the vocabulary-sharded exchange failed (gs_nccl_last_error) */
  GS_ETIMEOUT = 5,      /* a bounded device wait ran out */
  GS_ENOMEM = 6,        /* device allocation failed */
  GS_EUNSUPPORTED = 7,  /* request outside the implemented envelope (see gs_last_error) */
  GS_EEMPTY = 8,        /* "Cannot sample empty logits" (src/runtime/sampling.ts:19) */
  GS_ENONFINITE = 9     /* a logit was NaN or +inf (outside the reference's domain) */
} gs_status;

enum { GS_DTYPE_F32 = 0, GS_DTYPE_BF16 = 1 };

/* Per-row flags written to gs_outputs.flags. */
enum {
  GS_FLAG_BOUNDARY_TOP_P = 1u << 0,   /* top-p cumulative within 1e-6 (relative) of topP */
  GS_FLAG_BOUNDARY_DRAW = 1u << 1,    /* draw cursor within 1e-6 of a CDF step */
  GS_FLAG_BOUNDARY_MIN_P = 1u << 2,   /* a probability within 1e-6 of the min-p threshold */
  GS_FLAG_BOUNDARY_TYPICAL = 1u << 3, /* typical-p cut or surprise order within 1e-6 */
  GS_FLAG_FELL_THROUGH = 1u << 4,     /* draw loop ended without cursor <= 0 (sampling.ts:64) */
  GS_FLAG_GREEDY = 1u << 5,           /* temperature 0: argmax, no draw consumed */
  GS_FLAG_LARGE_PATH = 1u << 6,       /* topK == 0 or topK > GS_MAX_TOP_K: histogram path */
  GS_FLAG_ERR_DEADEND = 1u << 8,
  GS_FLAG_ERR_NONFINITE = 1u << 9,
  GS_FLAG_ERR_INVALID = 1u << 10,     /* bad mask state / history id bookkeeping */
  GS_FLAG_ERR_UNSUPPORTED = 1u << 11, /* see GS_EUNSUPPORTED */
  GS_FLAG_ERR_TIMEOUT = 1u << 12,
  GS_FLAG_ERRORS = 0xff00u
};

#define GS_MAX_TOP_K 1024     /* topK above this (or 0) runs the histogram path */
#define GS_MAX_HISTORY 4096   /* history entries per row after the repetition window is
                                 applied; with gs_batch.history_count an entry stands for
                                 any number of occurrences, so the window itself is not
                                 bounded by this */

/*
 * DecodingConfig fields that sampleToken reads (src/runtime/decoding.ts:1-14).  The
 * window (repetitionWindow) is applied by the caller when it fills gs_batch.history,
 * exactly as `history.slice(-config.repetitionWindow)` (src/runtime/sampling.ts:22-24).
 * Validation (src/runtime/decoding.ts:31-59) is re-checked: GS_EINVAL on violation.
 */
typedef struct gs_params {
  double temperature;
  double top_p;
  double min_p;
  double typical_p;
  double repetition_penalty;
  double presence_penalty;
  double frequency_penalty;
  int32_t top_k;
  int32_t reserved;
} gs_params;

typedef struct gs_batch {
  const void* logits;         /* [rows, row_stride] raw model logits (f32 or bf16) */
  int32_t dtype;              /* GS_DTYPE_F32 / GS_DTYPE_BF16 */
  int32_t rows;
  int64_t vocab;              /* V (262144 for Gemma) */
  int64_t row_stride;         /* elements between rows, >= vocab */
  float softcap;              /* c·tanh(x/c) applied to the logits first; 0 = off */
  int32_t params_count;       /* 1 = params[0] for every row, else == rows */
  const gs_params* params;    /* HOST pointer */
  const int32_t* history;     /* [rows, history_stride] windowed token history, or NULL */
  const int32_t* history_len; /* [rows] entries used per row, or NULL (no history) */
  int64_t history_stride;     /* <= GS_MAX_HISTORY */
  const uint32_t* mask_table; /* [mask_states, mask_words] allowed-token bitmasks, or NULL */
  int64_t mask_states;
  int64_t mask_words;         /* words per state row, >= ceil(vocab / 32) */
  const int32_t* mask_state;  /* [rows] row -> state; < 0 = unconstrained; or NULL */
  double* rng_state;          /* [rows] SeededRandom states (the JS number), in/out */
  const double* uniforms;     /* [rows] pre-drawn random() values; overrides rng_state */
  /* [rows, history_stride] occurrences each history entry stands for, or NULL (each entry
   * is one occurrence).  The penalties depend only on each id's count in the window
   * (src/runtime/sampling.ts:21-30), so a window longer than GS_MAX_HISTORY can be passed
   * as its distinct ids (in order of first occurrence) with their counts.  Values below 1
   * count as 1; the occurrences of one id, summed over its entries, must stay below 2^31.
   * No reference counterpart: the reference counts a JS array each call. */
  const int32_t* history_count;
} gs_batch;

typedef struct gs_outputs {
  int32_t* ids;               /* [rows] sampled token ids (-1 on a row error) */
  double* logprob;            /* [rows] tokenLogProbability(raw logits, id), or NULL */
  uint32_t* flags;            /* [rows] GS_FLAG_* bits, or NULL */
  int32_t* cand_ids;          /* [rows, cand_cap] final candidates in draw order, or NULL */
  double* cand_probs;         /* [rows, cand_cap] their probabilities, or NULL */
  int32_t* cand_count;        /* [rows] number of final candidates, or NULL */
  int32_t cand_cap;
} gs_outputs;

typedef struct gs_ctx gs_ctx;

/* Creates a context bound to `device`; workspace grows on demand and is never freed
 * per call (the reference allocates no GPU memory per token, README.md:241-242). */
gs_status gs_create(int device, gs_ctx** out);
gs_status gs_destroy(gs_ctx* ctx);
/* Pre-sizes the workspace so that later gs_sample calls with at most these sizes
 * allocate nothing (and can be captured in a CUDA graph).  max_top_k 0 (or above
 * GS_MAX_TOP_K) also reserves the per-row workspace of the histogram path. */
gs_status gs_reserve(gs_ctx* ctx, int32_t rows, int64_t vocab, int32_t max_top_k, int64_t history_stride);
/* Message of the last failure on `ctx` (NULL: this thread's last gs_sample_noalloc failure). */
const char* gs_last_error(const gs_ctx* ctx);

/*
 * Samples one token per row: replaces sampleToken(rawLogits, history, config, random)
 * (src/runtime/sampling.ts:18-65) as called by GemmaGenerationSession.generate
 * (src/runtime/gemma-session.ts:686, 705, 1328), including the constraint mask of
 * selectConstrainedToken/maskConstraintLogits (src/runtime/gemma-session.ts:1305-1329,
 * src/runtime/constraints.ts:159-173) as a per-state bitmask, and the greedy GPU
 * argmax route (src/webgpu/decode-greedy.ts:171-249) for temperature 0.  With
 * out->logprob it also returns tokenLogProbability (src/runtime/sampling.ts:67-80).
 * Asynchronous on `stream` (a cudaStream_t; NULL = default stream).  Row errors are
 * reported through out->flags; the call itself fails only on argument or CUDA errors.
 */
gs_status gs_sample(gs_ctx* ctx, const gs_batch* batch, const gs_outputs* out, void* stream);

/*
 * Same as gs_sample with the pointers of `batch` and `out` in HOST memory, except
 * batch->mask_table, which stays a device pointer (a compiled constraint's table is
 * uploaded once and kept resident).  Copies the inputs to the device, samples, copies
 * the outputs (and the advanced rng_state) back and synchronizes.  Returns the first
 * row error as a status (GS_EDEADEND, GS_ENONFINITE, ...), i.e. the error the reference
 * would throw.  This is the call a synchronous sampleToken replacement makes.
 */
gs_status gs_sample_host(gs_ctx* ctx, const gs_batch* batch, const gs_outputs* out, void* stream);

/* tokenLogProbability (src/runtime/sampling.ts:67-80) for one token per row over the
 * (soft-capped) raw device logits.  `tokens` and `out` are HOST pointers; the call is
 * synchronous.  GS_EINVAL ("Token t is outside logits length n") when a token is
 * outside [0, vocab). */
gs_status gs_token_log_probability(gs_ctx* ctx, const void* logits, int32_t dtype, int32_t rows,
                                   int64_t vocab, int64_t row_stride, float softcap,
                                   const int32_t* tokens, double* out, void* stream);

/* maskConstraintLogits (src/runtime/constraints.ts:159-173): out = -inf except at legal
 * and termination ids in [0, vocab). */
gs_status gs_mask_constraint_logits(gs_ctx* ctx, const float* raw_logits, int64_t vocab,
                                    const int32_t* legal, int64_t n_legal,
                                    const int32_t* termination, int64_t n_termination,
                                    float* out, void* stream);

/* Builds one allowed-token bitmask row (ceil(vocab/32) words) from the legal and
 * termination id lists that selectConstrainedToken passes to maskConstraintLogits
 * (src/runtime/gemma-session.ts:1315-1327). */
gs_status gs_build_mask_row(gs_ctx* ctx, int64_t vocab, const int32_t* legal, int64_t n_legal,
                            const int32_t* termination, int64_t n_termination, uint32_t* row_out,
                            void* stream);

/* maskReasoningLogits (src/runtime/gemma-session.ts:1331-1345) as two rows of an
 * allowed-token bitmask table (rows_out: device [2, mask_words] uint32).  Row 0 allows
 * the ids whose tokenizer.tokenBytes(id) is not null (has_bytes: device [vocab] uint8,
 * nonzero = has bytes); row 1 allows the same ids plus end_channel_id
 * (GEMMA_END_CHANNEL_TOKEN_ID = 101, src/runtime/gemma-tokenizer.ts:19; ignored outside
 * [0, vocab)), which generate() re-allows once GEMMA_REQUIRED_REASONING_TOKENS = 16
 * reasoning tokens were sampled (src/runtime/gemma-session.ts:124,676-687).  Bits past
 * the vocabulary are zero.  A required-reasoning step then samples with
 * mask_state = (reasoning tokens >= 16) ? 1 : 0 over this table, exactly as the
 * reference samples the masked copy of the logits. */
gs_status gs_build_reasoning_mask_rows(gs_ctx* ctx, int64_t vocab, const uint8_t* has_bytes, int32_t end_channel_id,
                                       uint32_t* rows_out, int64_t mask_words, void* stream);

/* ---- Constraint bitmask builder: the [S, mask_words] table from a compiled DFA ----
 * Replaces CompiledGenerationConstraint.legalTokenIds (src/runtime/constraints.ts:56-92,
 * transitionByte :222-247, isViableConstraintState :254-292, findViableStates :294-314)
 * over the token-byte trie (src/runtime/token-byte-trie.ts:16-40), and the legal-set rule
 * of selectConstrainedToken (src/runtime/gemma-session.ts:1315-1326): row s allows the
 * tokens legal from constraint state s, plus `extra_legal`, minus `termination`, plus
 * `termination` when the state accepts; dead_end[s] = 1 when the row allows nothing.
 * The DFA works on Unicode code points: node n's transitions are the ranges
 * [range_offsets[n], range_offsets[n+1]) of (range_lo, range_hi, range_target), sorted
 * and disjoint, range_hi inclusive.  A constraint state is a node plus the pending bytes
 * of an incomplete UTF-8 sequence (0-3 bytes). */
typedef struct gs_dfa_desc {
  int32_t nodes;
  const int32_t* range_offsets; /* [nodes + 1], host memory */
  const uint32_t* range_lo;
  const uint32_t* range_hi;
  const int32_t* range_target;
  const uint8_t* final;         /* [nodes]: 1 = accepting */
} gs_dfa_desc;

typedef struct gs_vocab_bytes_desc {
  int64_t vocab;
  const int64_t* offsets;       /* [vocab + 1], host: token v is bytes[offsets[v], offsets[v+1]) */
  const uint8_t* bytes;         /* an empty token is never legal (not in the trie) */
} gs_vocab_bytes_desc;

typedef struct gs_constraint gs_constraint;

/* Uploads a DFA and a vocabulary to the context's device (set-up; allocates). */
gs_status gs_constraint_create(gs_ctx* ctx, const gs_dfa_desc* dfa, const gs_vocab_bytes_desc* vocab,
                               gs_constraint** out);
gs_status gs_constraint_destroy(gs_constraint* c);
const char* gs_constraint_last_error(const gs_constraint* c);
/* Builds rows [0, n_states) of `table` (device, [n_states, mask_words] uint32) for the
 * states (node[s], pending_len[s], pending_bytes[3s..3s+2]); node, pending and the id
 * lists are host memory, dead_end device memory (or NULL).  At most 65535 states. */
gs_status gs_constraint_build_masks(gs_constraint* c, int32_t n_states, const int32_t* node,
                                    const uint8_t* pending_len, const uint8_t* pending_bytes,
                                    const int32_t* termination, int64_t n_termination,
                                    const int32_t* extra_legal, int64_t n_extra, uint32_t* table,
                                    int64_t mask_words, int32_t* dead_end, void* stream);

/* ---- int2 LM head: the logits the sampler consumes ----
 * Replaces the Gemma int2 LM head pass (src/webgpu/decode-lm-head.ts:
 * createGemmaLmHeadResources :95-166, encodeGemmaLmHead :168-176, the shader :178-256):
 *   logit[b][v] = srq(row_scales[v] · (Σ_j code_j(v)·a[b][j] - 2·activation_sum[b]),
 *                     output_scale)
 * with code_j(v) = (packed[v][j/16] >> 2(j%16)) & 3 (weight code_j - 2) and
 * srq(x, s) = s == 0 ? x : clamp(round_half_even(x / s), -128, 127)·s.  The dot product
 * is exact: with input_scale != 0 the activations are read as their int8 srq codes
 * clamp(rint(a / input_scale), -128, 127) (the grid the producing pass writes them on,
 * decode-ple-proj-norm-codes.ts:251-258) and Σ code·q is an integer; the bracket is then
 * fma(input_scale, Σ code·q, -2·sumA) in float32.  With input_scale == 0 the activations
 * stay float32 and the sum is taken in double in element order.  The reference's f32
 * evaluation differs from these by its own rounding only. */
typedef struct gs_lm_head_desc {
  int64_t vocab;              /* output features (rows of the packed matrix), < 2^31 */
  int32_t hidden;             /* activation length: a multiple of 128, at most 1536 */
  const uint32_t* packed;     /* host [vocab][hidden/16] u32, decode-lm-head.ts's row-major layout */
  const float* row_scales;    /* host [vocab] */
  float input_scale;          /* srq step of the activations (0: unquantised float32) */
  float output_scale;         /* srq step of the logits (0: none) */
} gs_lm_head_desc;

typedef struct gs_lm_head gs_lm_head;

/* Uploads (and repacks) the weights to the context's device (set-up; allocates). */
gs_status gs_lm_head_create(gs_ctx* ctx, const gs_lm_head_desc* desc, gs_lm_head** out);
gs_status gs_lm_head_destroy(gs_lm_head* h);
const char* gs_lm_head_last_error(const gs_lm_head* h);
/* logits[b * ld_logits + v] for b < rows (device buffers: activation [rows][ld_activation]
 * float32, activation_sum [rows], logits).  The first call with more rows than before
 * grows the handle's activation staging (allocates).  Asynchronous on `stream`. */
gs_status gs_lm_head_logits(gs_lm_head* h, const float* activation, int64_t ld_activation,
                            const float* activation_sum, int32_t rows, float* logits, int64_t ld_logits,
                            void* stream);
/* Reads and clears the device-side error flag (synchronising): GS_ETIMEOUT when a bounded
 * wait inside the kernel ran out (its logits are then unspecified). */
gs_status gs_lm_head_check(gs_lm_head* h, int32_t* timed_out);
/* Activations -> tokens in one call on `stream` (the reference's decode step from the
 * LM head pass to sampleToken, decode-model.ts:135-139 then sampling.ts:18), sampled as by
 * gs_sample on the context the head was created on.  batch->logits must be NULL,
 * batch->vocab 0 or the head's vocab; dtype and row_stride are set here.
 * Route (gs_lm_head_set_route): GS_LM_ROUTE_AUTO (the default) takes the fused route
 * only where it measured faster than the two-step route, i.e. for batches the two-step
 * route cannot serve with the single-launch decode step (a penalty history longer than
 * 512 ids at one row); GS_LM_ROUTE_FUSED takes it wherever it applies;
 * GS_LM_ROUTE_TWO_STEP never.
 * Fused route (1 or 2 rows, input_scale != 0, a penalty history only at one row with a
 * history_stride of at most 4096, every row greedy or 1 <= topK <= 64): the logits stay on chip; each block of vocabulary ids writes the
 * record of a vocabulary shard (its statistics and top-k candidates, as
 * gs_shard_partials) to a handle-owned buffer (at one row the kernel's last block then
 * combines them into one record) and gs_shard_merge samples them.  Candidate
 * ids and order are those of gs_lm_head_logits + gs_sample; probabilities agree to
 * float64 summation order (normaliser partials per block instead of per streamed unit).
 * Other batches: the logits go to a handle-owned scratch (rows × vocab float32) and
 * gs_sample runs on it, identical to gs_lm_head_logits followed by gs_sample.  Either
 * buffer grows on the first call that needs more (allocates).  The buffers and the
 * records kernel's block counter belong to the handle: one call in flight per handle. */
gs_status gs_lm_head_sample(gs_lm_head* h, const float* activation, int64_t ld_activation,
                            const float* activation_sum, const gs_batch* batch, const gs_outputs* out,
                            void* stream);
/* Number of gs_lm_head_sample calls on `h` that took the fused route (diagnostics; no
 * reference counterpart).  -1 for a NULL handle. */
int64_t gs_lm_head_fused_calls(const gs_lm_head* h);
/* Route of gs_lm_head_sample on `h` (no reference counterpart: the reference always
 * reads the logits back and samples them on the host).  GS_EINVAL for a NULL handle or
 * an unknown route. */
#define GS_LM_ROUTE_AUTO 0
#define GS_LM_ROUTE_FUSED 1
#define GS_LM_ROUTE_TWO_STEP 2
gs_status gs_lm_head_set_route(gs_lm_head* h, int32_t route);

/* Elementwise soft cap, the same routine the sampling pass applies (no reference
 * counterpart: the reference never applies its declared cap). */
gs_status gs_softcap(gs_ctx* ctx, const float* in, float* out, int64_t n, float cap, void* stream);

/* Self-check: order-independent 64-bit digest of gs_softcap over the float bit patterns
 * [lo, hi), for exhaustive comparison with an independent host implementation. */
gs_status gs_softcap_digest(gs_ctx* ctx, uint64_t lo, uint64_t hi, float cap, uint64_t* digest_host);

/*
 * Allocation-free sampling.  No counterpart in the reference: its sampler runs on the JS
 * main thread and never holds device memory.  Some callers of this library cannot
 * allocate device memory: a serving runtime whose memory pool already owns the device,
 * a real-time decode loop that cannot take the device-wide synchronisation cudaMalloc /
 * cudaFree imply, or an embedding that only lends its own input and output buffers.
 * gs_sample_noalloc runs the same kernels as gs_sample without a context and without
 * allocating: its per-call scratch (per-row plans, the streaming units' partial sums and
 * candidates: about 2.1 MiB for 4096 rows at topK 50, 1.1 MiB for 8 rows at topK 1024)
 * lives in one fixed device array of GS_NOALLOC_SCRATCH_BYTES (8 MiB) that every GPU
 * which loads the library keeps until the process exits.  Larger requests fail with
 * GS_EUNSUPPORTED.  It runs on the current device and looks up the array's device
 * address there on every call (a host-side lookup, so a device whose primary context was
 * reset is served at the array's new address); the first call on a device also loads
 * the library's module there, so make it before any stream capture.  All calls share the
 * array (the previous call's contents stay in it; nothing needs clearing, every call
 * writes what it reads), so calls whose kernels overlap on the GPU race.  Per-row params
 * (params_count > 1) are uploaded from batch->params with cudaMemcpyAsync: from pageable
 * host memory that copy is staged and can block the calling thread, so a caller that
 * needs a fully asynchronous call passes a pinned host array or a single params entry.
 * After a failure, gs_last_error(NULL) returns this thread's message.
 */
#define GS_NOALLOC_SCRATCH_BYTES (8u << 20)
gs_status gs_sample_noalloc(const gs_batch* batch, const gs_outputs* out, void* stream);

/*
 * Kernel timing (the counterpart of measureGpuDispatches, src/webgpu/gpu-timestamp.ts:1-56,
 * which brackets dispatches with timestamp queries).  While enabled, every gs_sample
 * records CUDA events on its stream around the streaming pass and around the merge;
 * gs_profile_read waits for them, returns the summed milliseconds and launch counts
 * since the last read and clears the record.
 */
gs_status gs_profile_enable(gs_ctx* ctx, int32_t enable);
gs_status gs_profile_read(gs_ctx* ctx, double* stream_ms, int64_t* stream_launches, double* merge_ms,
                          int64_t* merge_launches);

/*
 * Vocabulary-sharded mode: no reference counterpart (the reference samples one row on
 * one device, src/runtime/sampling.ts:18).  For small batches whose rows are split by
 * vocabulary over several GPUs (one process per GPU; shard g holds ids
 * [vocab_offset, vocab_offset + shard->vocab) of every row, vocab_offset a multiple of
 * 4096):
 *   1. gs_shard_partials streams the local shard and writes one fixed-size record per
 *      row into `records` (device, rows x gs_shard_record_bytes): the shard's maximum
 *      and sum of e^(x/T) over live ids, its top-k candidates (global ids) and the exact
 *      penalised scores of the history ids it holds.  History ids are global; the mask
 *      table covers the whole vocabulary (mask_words >= ceil(vocab_total/32)).
 *      want_logprob != 0 also records the raw sums a merge with outputs.logprob needs
 *      (otherwise that merge writes NaN log-probabilities).
 *   2. the caller all-gathers the records (one collective, e.g. ncclAllGather) into
 *      [shards][rows] order;
 *   3. gs_shard_merge merges them and samples exactly as gs_sample would on the whole
 *      rows (`full`: rows, params, the full mask table and states, rng_state or
 *      uniforms, history / history_stride for the record layout only, vocab =
 *      vocab_total; logits may be NULL), identically on every rank.
 * Requires 1 <= topK <= GS_MAX_TOP_K or temperature 0 (GS_EUNSUPPORTED otherwise).
 * gs_shard_record_bytes returns the record size for a batch's params (-1 on bad input);
 * every rank must pass the same params and history_stride.
 */
int64_t gs_shard_record_bytes(const gs_params* params, int32_t params_count, int64_t vocab_total,
                              int64_t history_stride);
gs_status gs_shard_partials(gs_ctx* ctx, const gs_batch* shard, int64_t vocab_offset, int64_t vocab_total,
                            int32_t want_logprob, void* records, void* stream);
gs_status gs_shard_merge(gs_ctx* ctx, const gs_batch* full, int32_t shards, const void* gathered_records,
                         const gs_outputs* out, void* stream);

/*
 * The same vocabulary-sharded step with the exchange done here, over NCCL (no reference
 * counterpart: the reference samples on one device; this is what an addon without a host
 * framework binds).  NCCL is loaded at run time: the copy the process has already loaded,
 * else libnccl.so.2, or the library named by the environment variable GS_NCCL_LIBRARY.
 *   gs_nccl_unique_id   one rank makes the communicator's id (host); the caller sends its
 *                       128 bytes to the other ranks by any means;
 *   gs_nccl_create      every rank joins with the same id, its rank and the device it
 *                       samples on (< 0: the calling thread's current device); the
 *                       communicator is non-blocking and set-up waits at most timeout_ms
 *                       (<= 0: no limit) for the other ranks, else GS_ETIMEOUT;
 *   gs_shard_sample     gs_shard_partials of the local shard into communicator-owned
 *                       records, one ncclAllGather of them, gs_shard_merge, all on
 *                       `stream` (arguments as for gs_shard_partials; every rank passes
 *                       the same params, states and history_stride and gets the same
 *                       ids).  The record buffers grow on the first call of a larger
 *                       batch (allocates).  With timeout_ms > 0 the call also waits
 *                       (host) until the step has completed on the stream, at most
 *                       timeout_ms; a rank that never joins the exchange then ends it
 *                       with GS_ETIMEOUT instead of a wait without end.
 * After GS_ETIMEOUT or GS_ENCCL the communicator has been aborted: destroy it and create
 * a new one.  gs_nccl_last_error(NULL) gives this thread's last message.
 */
typedef struct gs_nccl_id {
  char internal[128];
} gs_nccl_id;
typedef struct gs_nccl gs_nccl;
gs_status gs_nccl_unique_id(gs_nccl_id* id);
gs_status gs_nccl_create(int device, const gs_nccl_id* id, int32_t nranks, int32_t rank, int32_t timeout_ms,
                         gs_nccl** out);
gs_status gs_nccl_destroy(gs_nccl* comm);
const char* gs_nccl_last_error(const gs_nccl* comm);
gs_status gs_shard_sample(gs_ctx* ctx, gs_nccl* comm, const gs_batch* shard, int64_t vocab_offset,
                          int64_t vocab_total, const gs_outputs* out, int32_t timeout_ms, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* GSAMPLER_H_ */
