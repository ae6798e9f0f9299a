/*
 * sonic_b200.h -- C ABI of the B200 (sm_100a) fused sampling / speculative-verification
 * hot path.
 *
 * Every entry point takes one argument struct of raw pointers, element strides and dtype
 * tags, plus an opaque CUDA stream handle (`cudaStream_t` passed as `void*`, NULL = legacy
 * default stream). Nothing in this header depends on PyTorch or on CUDA headers, so any FFI
 * (ctypes, cgo, JNI, N-API) can bind it. No entry point allocates device memory: the caller
 * passes a device workspace of at least the size the matching `*_workspace_size` query
 * returns; the workspace must be zero-filled once before first use, and every successful
 * call leaves its counters at zero again, so the same workspace serves any number of calls
 * (calls that overlap on the GPU must use distinct workspaces).
 *
 * Calls are asynchronous (kernel launches on `stream`, no host synchronisation, no
 * allocation), so they can be captured in a CUDA graph. Status codes never throw across
 * the ABI; `sonic_last_error()` returns the calling thread's last message.
 *
 * Reference interfaces replaced (tachyontrails/sonic-sampler, paths under src/sonic_sampler/):
 *   sonic_fused_singular   <- interface/functional/singular.py:75-322 (fused_singular:
 *                             ops/prologue.py:272 bitpacked_reduction_kernel +
 *                             ops/singular.py:154 cumulative_selection_kernel)
 *   sonic_fused_multistep  <- interface/functional/multistep.py:175-461 (fused_multistep:
 *                             ops/prologue.py:272 + ops/multistep.py:76
 *                             cumulative_unpack_kernel + ops/verify.py:244
 *                             chain_speculative_verification_kernel)
 *   sonic_bounded_topk     <- interface/topk.py:98-161 (UnshardedBoundedTopK.__call__:
 *                             ops/topk/bitpack.py:99 + ops/topk/unpack.py:312)
 *   sonic_indexed_copy     <- ops/copy.py:21-127 (indexed_copy, noise staging)
 *   sonic_populate_slots   <- core/buffer.py:1026-1052, 1098-1352 (SamplingBuffers
 *                             step_grammar / transfer / update / allocate, host population)
 */
#ifndef SONIC_B200_H
#define SONIC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SONIC_B200_ABI_VERSION 4

/* Candidate-set width of the two-stage top-k (reference ops/base.py:24, MAX_K). */
#define SONIC_MAX_K 128
/* Largest speculation lookahead gamma accepted by sonic_fused_multistep / drafting. */
#define SONIC_MAX_LOOKAHEAD 15

typedef int32_t sonic_status;
enum {
  SONIC_OK = 0,
  SONIC_ERR_INVALID_ARGUMENT = 1, /* bad shape, stride, dtype, null pointer or flag */
  SONIC_ERR_UNSUPPORTED = 2,      /* valid request this build does not implement */
  SONIC_ERR_WORKSPACE = 3,        /* workspace missing or smaller than required */
  SONIC_ERR_CUDA = 4              /* a CUDA runtime call failed (message has details) */
};

enum {
  SONIC_DTYPE_BF16 = 0,
  SONIC_DTYPE_F32 = 1,
  SONIC_DTYPE_I32 = 2,
  SONIC_DTYPE_I64 = 3
};

/* Call flags (bit set in the `flags` field of each argument struct). */
enum {
  SONIC_FLAG_PDL = 1u << 0,            /* launch with programmatic dependent launch */
  SONIC_FLAG_PREFILL = 1u << 1,        /* decode-count update writes 1 instead of +1 */
  SONIC_FLAG_UPDATE_COUNTS = 1u << 2,  /* update decode counts with the selected tokens */
  SONIC_FLAG_LOGPROBS = 1u << 3,       /* write selected (and top-Z) logprobs */
  SONIC_FLAG_PROBABILITIES = 1u << 4,  /* singular: write candidate probabilities */
  SONIC_FLAG_PHILOX = 1u << 5,         /* counter-based Philox noise instead of the noise buffers */
  /* Diagnostics, for tests of the error path: every CTA of a ring-streaming kernel first waits
   * on a barrier that nothing completes, with a short limit, and then takes the same path as a
   * real bounded-wait timeout (no outputs written, SONIC_DEVICE_ERR_WAIT in the error word). */
  SONIC_FLAG_DEBUG_STALL_RING = 1u << 15
};

/* Bits of a workspace's device error word (sonic_workspace_error). */
enum {
  /* A bounded wait for a bulk copy into shared memory gave up. The rows (singular, top-k) or
   * requests (multistep) of the affected CTAs wrote none of their outputs; the staged noise
   * rows of sonic_indexed_copy that timed out were not stored. */
  SONIC_DEVICE_ERR_WAIT = 1u << 0
};

/*
 * Per-request sampling parameters: the device-resident fields of the reference's
 * SamplingBuffers (core/buffer.py:784-817, core/flags.py:435-521). All are indexed by the
 * request slot (after slot indirection). Any pointer may be NULL when no row's indicator
 * needs it (the reference passes None the same way).
 */
typedef struct SonicSamplingParams {
  const uint16_t* indicators;     /* u16 [slots]: Indicator bit field (core/flags.py:58-95) */
  const void* slot_mapping;       /* [requests] i32 or i64, or NULL (identity) */
  int32_t slot_dtype;             /* SONIC_DTYPE_I32 / SONIC_DTYPE_I64 */
  int32_t num_slots;              /* rows of the per-slot buffers (bounds checks only) */
  const uint32_t* grammar;        /* u32 bit mask words, row (slot*timesteps+step) */
  int64_t grammar_stride;         /* words between consecutive grammar rows */
  const int32_t* context_counts;  /* i32 [slots, counts_stride] */
  int32_t* decode_counts;         /* i32 [slots, counts_stride] (updated in place) */
  int64_t counts_stride;          /* elements between count rows */
  const uint16_t* repetition;     /* bf16 [slots] multiplicative penalty */
  const uint16_t* frequency;      /* bf16 [slots] */
  const uint16_t* presence;       /* bf16 [slots] */
  const uint16_t* bias;           /* bf16 [slots, bias_stride] */
  int64_t bias_stride;            /* elements between bias rows */
  const uint16_t* temperature;    /* bf16 [slots] */
  const int32_t* top_k;           /* i32 [slots] */
  const uint16_t* top_p;          /* bf16 [slots] */
  const uint16_t* min_p;          /* bf16 [slots] */
  const int32_t* top_logprobs;    /* i32 [slots] number of top-Z logprobs requested */
} SonicSamplingParams;

/*
 * One-token selection per row (autoregressive decode or drafting step).
 * Replaces reference interface/functional/singular.py:75 fused_singular.
 */
typedef struct SonicSingularArgs {
  int32_t rows;              /* R logits rows */
  int32_t vocab_size;        /* columns sampled (local vocab) */
  int32_t block_n;           /* reference tile width: fixes the greedy tie rule */
  int32_t lookahead;         /* gamma: drafted-token columns counted (drafting, t > 0) */
  int32_t shard_offset;      /* added to columns before aux-buffer lookups */
  int32_t max_top_logprobs;  /* Z capacity of the top-logprob outputs */
  int32_t target_vocab;      /* row length of `probabilities` (bounds checks only) */
  uint32_t flags;            /* SONIC_FLAG_* */

  const void* logits;        /* [R, logits_stride] bf16 */
  int32_t logits_dtype;      /* SONIC_DTYPE_BF16 */
  int64_t logits_stride;

  SonicSamplingParams params;

  const void* d2t;           /* [vocab] draft->target id table (i32/i64) or NULL */
  int32_t d2t_dtype;
  const int32_t* drafted_tokens; /* [slots, drafted_stride] drafted ids or NULL */
  int64_t drafted_stride;

  const uint16_t* gumbel;    /* bf16 log(Exp(1)) noise, [slots, gumbel_stride] */
  int64_t gumbel_stride;
  uint64_t philox_seed;      /* SONIC_FLAG_PHILOX: key of the counter-based noise */
  uint64_t philox_offset;    /* SONIC_FLAG_PHILOX: per-call counter offset */

  int32_t* tokens;           /* out i32 [R] at tokens[r*tokens_stride] */
  int64_t tokens_stride;
  void* logprobs;            /* out [R] at logprobs[r*logprobs_stride] or NULL */
  int64_t logprobs_stride;
  int32_t logprobs_dtype;    /* SONIC_DTYPE_BF16 (reference) or SONIC_DTYPE_F32 */
  void* top_logprob_values;  /* out [R, top_stride] (logprobs_dtype) or NULL */
  int32_t* top_logprob_tokens;  /* out i32 [R, top_stride] or NULL */
  int64_t top_stride;
  void* probabilities;       /* out [slots, probabilities_stride] bf16/f32 or NULL */
  int32_t probabilities_dtype;
  int64_t probabilities_stride;

  void* workspace;           /* device scratch, zero-filled before first use */
  size_t workspace_bytes;
} SonicSingularArgs;

/*
 * Multi-step target verification of gamma drafted tokens per request.
 * Replaces reference interface/functional/multistep.py:175 fused_multistep.
 */
typedef struct SonicMultistepArgs {
  int32_t batch_size;        /* B requests */
  int32_t lookahead;         /* gamma (maximum, for varlen) */
  int32_t vocab_size;
  int32_t block_n;           /* reference tile width: fixes the greedy tie rule */
  int32_t shard_offset;
  int32_t max_top_logprobs;
  uint32_t flags;            /* SONIC_FLAG_PDL / _UPDATE_COUNTS / _LOGPROBS */
  int32_t total_rows;        /* L = B*(gamma+1), or cu_seqlens[B] for varlen */

  const void* logits;        /* [L, logits_stride] bf16 */
  int32_t logits_dtype;
  int64_t logits_stride;
  const int32_t* cu_seqlens; /* [B+1] row offsets (varlen) or NULL */

  SonicSamplingParams params;

  const int32_t* drafted_tokens; /* flat [L]: request b's draft ids at margin_b + s */
  const void* draft_probs;   /* q: [slots, draft_stride] rows, step stride draft_step_stride */
  int32_t draft_dtype;       /* SONIC_DTYPE_F32 / SONIC_DTYPE_BF16 */
  int64_t draft_stride;
  int64_t draft_step_stride;
  const uint16_t* uniform;   /* bf16 [slots, uniform_stride] acceptance draws */
  int64_t uniform_stride;
  const uint16_t* gumbel;    /* bf16 [slots, gumbel_stride], step stride gumbel_step_stride */
  int64_t gumbel_stride;
  int64_t gumbel_step_stride;

  float* values;             /* out f32 [L, 128] candidate probabilities or NULL */
  int32_t* indices;          /* out i32 [L, 128] candidate ids or NULL */
  int32_t* tokens;           /* out i32 flat [L]: tokens[margin_b + accepted_b] = token */
  int32_t* offsets;          /* out i32 [B] accepted counts */
  void* logprobs;            /* out flat [L] or NULL */
  int32_t logprobs_dtype;    /* SONIC_DTYPE_BF16 (reference) or SONIC_DTYPE_F32 */
  void* top_logprob_values;  /* out [L, top_stride] (logprobs_dtype) or NULL */
  int32_t* top_logprob_tokens;  /* out i32 [L, top_stride] or NULL */
  int64_t top_stride;

  void* workspace;
  size_t workspace_bytes;

  /* SONIC_FLAG_PHILOX (an addition of this library; the reference always reads buffers):
   * `uniform` and `gumbel` are not read. Step s of the call draws with counter offset
   * philox_offset + s under key philox_seed: the rejection step's log(Exp(1)) noise of token
   * t from counter (t, slot, offset + s), in fp32; the acceptance uniform from counter
   * (0xffffffff, slot, offset + s), rounded to bf16. Use distinct offsets for distinct calls,
   * and for the drafting calls whose noise must differ (on-policy rejection sampling). */
  uint64_t philox_seed;
  uint64_t philox_offset;
} SonicMultistepArgs;

/*
 * Bounded top-k (k a power of two <= 128) over each row, values descending, ties by the
 * lowest column. Row r's k results land at values[r*k + i] / indices[r*k + i] (the
 * reference's flat layout, interface/topk.py:117-159 with ops/topk/unpack.py:374-377).
 * Replaces reference interface/topk.py:98 UnshardedBoundedTopK.__call__.
 */
typedef struct SonicTopKArgs {
  int32_t rows;
  int32_t vocab_size;
  int32_t k;
  int32_t block_n;           /* accepted for interface parity; no effect on results */
  uint32_t flags;            /* SONIC_FLAG_PDL */
  const void* logits;        /* [rows, logits_stride] bf16 or f32 */
  int32_t logits_dtype;
  int64_t logits_stride;
  void* values;              /* out: bf16 (bf16 logits) or f32 (f32 logits) */
  int32_t values_dtype;
  void* indices;             /* out: i32 or i64 */
  int32_t indices_dtype;
  void* workspace;
  size_t workspace_bytes;
} SonicTopKArgs;

/* Device workspace (bytes) a call with these arguments needs. Only shape fields are read. */
size_t sonic_fused_singular_workspace_size(const SonicSingularArgs* args);
size_t sonic_fused_multistep_workspace_size(const SonicMultistepArgs* args);
size_t sonic_bounded_topk_workspace_size(const SonicTopKArgs* args);

sonic_status sonic_fused_singular(const SonicSingularArgs* args, void* stream);
sonic_status sonic_fused_multistep(const SonicMultistepArgs* args, void* stream);
sonic_status sonic_bounded_topk(const SonicTopKArgs* args, void* stream);

/* Vocab-sharded singular sampling in three steps, for a vocabulary split over `world` ranks
 * (rank r holds the logits columns [r * shard, r * shard + local), args->shard_offset = r * shard).
 * The reference's own sharded path is unfinished (interface/functional/singular.py:145-149
 * writes every shard at column 0; ops/singular.py:61-66 decodes greedy indices wrongly); these
 * entry points replace it.
 *   1. sonic_shard_candidates: streams this rank's shard exactly as sonic_fused_singular does
 *      and writes, per row, the shard's 128 best candidates as sorted 64-bit keys with GLOBAL
 *      columns to keys[rows][128] (greedy rows too). No selection, no output but `keys`.
 *   2. the caller all-gathers keys over the ranks into gathered[world][rows][128] (one
 *      ncclAllGather / torch.distributed.all_gather_into_tensor).
 *   3. sonic_merge_candidates: merges the world lists of every row and runs selection, logprobs
 *      and count updates exactly as sonic_fused_singular; args->vocab_size is the full
 *      vocabulary and the noise covers it, so every rank computes the same tokens. Greedy rows
 *      take the largest value with the lowest global column. */
sonic_status sonic_shard_candidates(const SonicSingularArgs* args, uint64_t* keys, void* stream);
sonic_status sonic_merge_candidates(const SonicSingularArgs* args, const uint64_t* gathered, int32_t world,
                                    void* stream);

/* sonic_fused_singular for callers that cannot allocate device memory (an engine whose KV
 * cache already holds all free HBM, a cgo / JNI binding without the framework's allocator,
 * a loop that cannot afford cudaMalloc's possible device synchronisation). No counterpart
 * in the reference: it is an addition of this library.
 *
 * args->workspace and args->workspace_bytes are ignored; the scratch is a fixed 4 MiB device
 * array inside this library, held by every GPU that loads it until the process exits.
 * Calls whose sonic_fused_singular_workspace_size() exceeds 4 MiB fail with
 * SONIC_ERR_WORKSPACE. The first call on a device looks up the array's device address (with
 * that device current); make that first call before any stream capture. Each call clears
 * the array's tickets with cudaMemsetAsync on `stream` and allocates nothing; the array's
 * error word is left for sonic_workspace_error(NULL, ...) to read. All calls
 * share the one array: calls that may overlap on the GPU (other streams, other host threads
 * on the same device) race and must be serialised by the caller. */
sonic_status sonic_fused_singular_static(const SonicSingularArgs* args, void* stream);

/* Reads the device error word (SONIC_DEVICE_ERR_* bits, 0 when clean) that the kernels of
 * earlier calls left in `workspace` (the buffer passed as args->workspace to
 * sonic_fused_singular, sonic_fused_multistep, sonic_bounded_topk or sonic_shard_candidates)
 * into *error_out, then clears it. With workspace == NULL it reads the library's own word on the
 * current device, which sonic_fused_singular_static and sonic_indexed_copy write. The word
 * stays set across calls until read. Synchronises `stream`: do not call it while the stream
 * is being captured. No counterpart in the reference, which has no device-side error path. */
sonic_status sonic_workspace_error(void* workspace, uint32_t* error_out, void* stream);

/* Noise staging: for each i < count, row r = indices[i] (i32 or i64, index_dtype); unless
 * indicator[r] has the greedy bit (0x40), copy `cols` elements of `elem_bytes` bytes from
 * source + r * stride to target + r * stride (elements; the same row stride for both).
 * Indices outside [0, rows) are skipped. Runs on `stream`, allocates nothing, never
 * synchronises. Replaces ops/copy.py:21-127 (`indexed_copy`, `indexed_copy_kernel`), called
 * by `GumbelNoise.stage_weights` (core/buffer.py:151-157) to move the draft noise of the
 * stochastic slots into the target noise after verification. */
sonic_status sonic_indexed_copy(const void* source, void* target, int64_t rows, int64_t stride, int64_t cols,
                                int32_t elem_bytes, const void* indices, int32_t index_dtype, int32_t count,
                                const uint16_t* indicator, void* stream);

/* Parts of the slot buffers sonic_populate_slots writes (SonicPopulateArgs.parts). */
enum {
  SONIC_POPULATE_SCALARS = 0x1,      /* temperature, top_p, min_p, top_k, top_logprobs, the three
                                        repetition penalties and the target/draft indicators */
  SONIC_POPULATE_HISTOGRAM = 0x2,    /* context counts = histogram of the slot's prompt tokens,
                                        decode counts = 0 (admission) */
  SONIC_POPULATE_DENSE_COUNTS = 0x4, /* context and decode counts copied from dense rows */
  SONIC_POPULATE_BIAS = 0x8,         /* bias row = 0, then the slot's (token, value) entries */
  SONIC_POPULATE_GRAMMAR = 0x10      /* grammar words of the slots that carry a bitmask */
};

/* One batched population of request slots (sonic_populate_slots). Every input array is device
 * memory (normally one staged blob copied from pinned host memory with one cudaMemcpyAsync);
 * the destinations are the slot buffers the sampler reads (layout as SonicSamplingParams:
 * bf16 scalars, i32 counts [num_slots][counts_stride], bf16 bias [num_slots][bias_stride],
 * u32 grammar words). Slot i of the call is buffer row positions[i]. */
typedef struct SonicPopulateArgs {
  int32_t count;        /* slots in this call */
  int32_t num_slots;    /* rows of the slot buffers; positions outside [0, num_slots) are skipped */
  int64_t vocab_size;   /* V: columns of the count and bias rows */
  uint32_t parts;       /* SONIC_POPULATE_* */
  int32_t timesteps;    /* T: grammar steps of a slot */
  int32_t grammar_step; /* >= 0: the bitmask goes to that step only (admission: 0);
                           -1: to every step (one row broadcast, or T rows) */
  int32_t _pad0;

  const int32_t* positions;    /* [count] slot ids, distinct */
  /* SONIC_POPULATE_SCALARS */
  const uint16_t* values_bf16; /* [count][6] temperature, top_p, min_p, multiplicative,
                                  frequency, presence (bf16 bits) */
  const int32_t* values_i32;   /* [count][2] top_k, top_logprobs */
  const uint16_t* indicators;  /* [count][2] target, draft */
  /* SONIC_POPULATE_HISTOGRAM: tokens of slot i are tokens[token_offsets[i] .. token_offsets[i+1]);
     ids outside [0, V) are not counted */
  const int64_t* token_offsets;
  const int32_t* tokens;
  /* SONIC_POPULATE_DENSE_COUNTS: rows i of [count][V] */
  const int32_t* dense_context;
  const int32_t* dense_decode;
  /* SONIC_POPULATE_BIAS: entries of slot i are [bias_offsets[i], bias_offsets[i+1]) of
     bias_tokens / bias_values (bf16 bits); tokens distinct within a slot; NULL offsets = no
     entries (rows zeroed) */
  const int64_t* bias_offsets;
  const int32_t* bias_tokens;
  const uint16_t* bias_values;
  /* SONIC_POPULATE_GRAMMAR: slot i's bitmask starts at row grammar_rows[i] (-1: none) of
     grammar_words [rows][ceil(V / 32)] and has grammar_steps[i] rows (1, or T when
     grammar_step is -1) */
  const int32_t* grammar_rows;
  const int32_t* grammar_steps;
  const uint32_t* grammar_words;

  /* destinations */
  uint16_t* temperature;
  uint16_t* top_p;
  uint16_t* min_p;
  int32_t* top_k;
  int32_t* top_logprobs;
  uint16_t* multiplicative;
  uint16_t* frequency;
  uint16_t* presence;
  uint16_t* flags_target; /* element s: slot s's target indicator */
  uint16_t* flags_draft;
  int32_t* context_counts;
  int32_t* decode_counts;
  int64_t counts_stride;
  uint16_t* bias;
  int64_t bias_stride;
  uint32_t* grammar;
  int64_t grammar_slot_stride; /* words */
  int64_t grammar_step_stride; /* words */
} SonicPopulateArgs;

/* Batched slot population: the device side of SamplingBuffers.allocate / update /
 * step_grammar (core/buffer.py:1026-1052, 1098-1352). The reference issues a dozen
 * `copy_` calls a slot through pinned memory (PinnedRelay.populate + transfer,
 * RepetitionPenalties.populate + transfer, TokenCounts.allocate / update, Flags.update,
 * step_grammar) and histograms the prompt on the host into a dense pinned row; this call
 * writes the same values for every slot of the batch in one kernel launch from sparse
 * inputs (prompt tokens, bias entries). Noise refresh stays with the caller's generator.
 * Runs on `stream`, allocates nothing, never synchronises. */
sonic_status sonic_populate_slots(const SonicPopulateArgs* args, void* stream);

/* ABI version (SONIC_B200_ABI_VERSION) the library was built with. */
int32_t sonic_abi_version(void);
/* Message of the calling thread's last failed call ("" when none). */
const char* sonic_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* SONIC_B200_H */
