/*
 * needle_cuda.h -- C-ABI of libneedle_cuda.so, the B200 (sm_100a) decode engine for Needle 2.
 *
 * The engine plugs in as a third needle.js backend: a TypeScript `CudaBackend implements
 * InferenceBackend` (packages/needle.js/src/backends/backend.ts:83-110) whose
 * createResidentSession() returns a `ResidentExecutionSession` (backend.ts:66-80) binds these
 * functions through bun:ffi.  Plain C types only: no exceptions, no C++ or torch types.
 *
 * Conventions
 *  - Every function returns a needle_status; the message of the last failure on the calling
 *    thread is available from needle_cuda_last_error().
 *  - Statuses 1..10 are NeedleErrorCode (packages/needle.js/src/errors.ts:1-11) in order, so the
 *    adapter rethrows `new NeedleError(CODES[status - 1], needle_cuda_last_error())`.
 *  - One context per GPU and one host thread per context.  Host pointers are borrowed for the
 *    duration of the call only.  The context owns all device memory it allocates.
 *  - Arithmetic follows the reference CPU backend: in NEEDLE_NUMERICS_EXACT every expression is
 *    evaluated in binary64 in the reference's order and rounded to binary32 where the reference
 *    stores into a Float32Array, so tokens and int8 KV codes match the CPU backend.
 */
#ifndef NEEDLE_CUDA_H
#define NEEDLE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum needle_status {
  NEEDLE_OK = 0,
  NEEDLE_INVALID_CACT = 1,
  NEEDLE_UNSUPPORTED_CACT = 2,
  NEEDLE_WEIGHTS_NOT_FOUND = 3,
  NEEDLE_WEIGHTS_INTEGRITY = 4,
  NEEDLE_WEBGPU_UNAVAILABLE = 5,
  NEEDLE_BACKEND_UNAVAILABLE = 6, /* also: CUDA errors, bad context, unsupported geometry */
  NEEDLE_CONTEXT_OVERFLOW = 7,
  NEEDLE_INVALID_TOOL_SCHEMA = 8,
  NEEDLE_GRAMMAR_DEAD_END = 9,
  NEEDLE_GENERATION_ABORTED = 10
} needle_status;

enum {
  NEEDLE_NUMERICS_EXACT = 0, /* binary64 in reference order: bit-faithful to the CPU backend */
  NEEDLE_NUMERICS_FAST = 1,  /* the projections (Q|K|V|gate, output, engram K|V, vocabulary) as
                                tcgen05 tensor-core GEMMs over the step's items, fp16 head/tail
                                split with fp32 accumulation (binary32-level accuracy), and the
                                layer's norm sums as block reductions; attention in binary32 (online
                                softmax over the int8 cache, CUDA cores); the K/V append, routing
                                and selection as in exact numerics; int8 KV cache only.  Same greedy
                                ids as the CPU backend, logits within 1e-3 */
  NEEDLE_NUMERICS_FAST_ATTENTION = 2, /* NEEDLE_NUMERICS_FAST with attention on the int8-MMA kernel
                                (integer-digit tensor-core products): logits within 3e-3 */
  NEEDLE_KV_INT8 = 0,        /* RuntimeOptions.kvCache "int8" (runtime.ts:30-32) */
  NEEDLE_KV_FLOAT32 = 1      /* RuntimeOptions.kvCache "float32": keys / values stored as given */
};

typedef struct needle_opts {
  uint32_t struct_size; /* sizeof(needle_opts) */
  int32_t device;       /* CUDA device ordinal */
  int32_t max_seqs;     /* sequence slots (concurrent sequences) */
  int32_t max_len;      /* largest maximumLength a slot accepts (<= geometry max sequence) */
  int32_t max_sink;     /* largest sinkLength a slot accepts */
  int32_t kv_mode;      /* NEEDLE_KV_INT8 or NEEDLE_KV_FLOAT32, for every slot of the context */
  int32_t numerics;     /* NEEDLE_NUMERICS_EXACT, _FAST or _FAST_ATTENTION */
  int32_t micro_batches; /* device-scheduled steps run as this many micro-batches on their own
                            streams (1..8; 0 = the default, 4), so latency-bound kernels of one
                            overlap the others' */
  int32_t sched_chunk;   /* device-scheduled steps: up to this many prompt positions of a slot that
                            is still reading its prompt go into one step, as a chunk of items (2..64;
                            0 or 1 = one position per slot and step, the default).  A chunk never
                            reaches past the slot's KV window (prompt positions beyond it go one
                            per step) and holds no selecting position; the results are the same */
  int32_t sched_items;   /* with sched_chunk >= 2: the items one step may hold -- a device-scheduled
                            step, spread over the micro-batches with whole chunks, or a host step
                            (needle_cuda_step, _begin) with prompt chunks (>= max_seqs; 0 = 2 x
                            max_seqs); without it a step holds max(max_seqs, 64) items */
  int32_t reserved[6];
} needle_opts;

typedef struct needle_ctx needle_ctx;

/* Geometry of the opened archive (CactGeometry, packages/needle.js/src/model/cact.ts:15-35). */
typedef struct needle_geometry {
  int32_t vocabulary_size, model_dimension, heads, kv_heads, layers, head_dimension,
      maximum_sequence_length, hadamard_dimension, mhc_lanes, engram_slots,
      engram_sub_dimension, engram_tables, engram_taps, engram_dilation, kv_window, kv_bits;
  int32_t engram_order_count, engram_orders[4], engram_site_count, engram_sites[4];
  float rope_theta;
  int32_t num_tensors;
  int32_t kv_capacity; /* KV slots per sequence allocated by this context */
} needle_geometry;

/* One sequence's work in a batched step (NeedleRuntime.step / stepSelected, runtime.ts:257-583).  A
 * slot appears once per step, or as a prompt chunk: consecutive items of the slot with their tokens
 * (no NEEDLE_TOKEN_PENDING), none selecting, for positions p, p + 1, ... -- the same result as that
 * many one-token steps (runtime.ts:227-243), provided the chunk does not reach past the slot's KV
 * window (INVALID_CACT otherwise) and no slot of the context collects confidence. */
typedef struct needle_step_item {
  int32_t seq;            /* slot in [0, max_seqs) prepared with needle_cuda_seq_reset */
  int32_t token;          /* token consumed at the slot's current position;
                             NEEDLE_TOKEN_PENDING takes the slot's last selected id */
  int32_t select;         /* 1: select a token after this step (argmax / masked argmax) */
  int32_t allowed_count;  /* -1: unmasked; >0: mask = allowed_ids[allowed_offset, +count);
                             NEEDLE_ALLOWED_MASK: mask = slot allowed_offset of the device mask
                             pool (needle_cuda_mask_pool / needle_cuda_masks_put) */
  uint32_t allowed_offset;
} needle_step_item;

#define NEEDLE_TOKEN_PENDING (-1)
#define NEEDLE_ALLOWED_MASK (-2)

/* SelectedToken (backend.ts:41-44). */
typedef struct needle_selected {
  int32_t id;
  int32_t reserved;
  double log_probability;
} needle_selected;

/* Last failure message of the calling thread ("" if none). */
const char* needle_cuda_last_error(void);

/* Fills *opts with defaults (device 0, 1 slot, max_len 2048, max_sink 160, int8, exact). */
int needle_cuda_default_opts(needle_opts* opts);

/* Parses a `.cact` archive (parseCact, cact.ts:189-562), checks the geometry this engine
 * supports (the same gate as supportsResidentExecution, packages/needle.js/src/resident/
 * compatibility.ts:4-40, except that kvWindow 0 is accepted), and uploads the weights to
 * `opts->device`.  Replaces CpuBackend construction (packages/needle.js/src/backends/cpu.ts:
 * 120-124) / createTypeGPUBackend. */
int needle_cuda_open(const uint8_t* cact, size_t n, const needle_opts* opts, needle_ctx** out);

/* InferenceBackend.dispose (backend.ts:109).  Frees every device allocation. */
int needle_cuda_close(needle_ctx* ctx);

int needle_cuda_geometry(const needle_ctx* ctx, needle_geometry* out);

/* ResidentExecutionSession.reset / NeedleRuntime.reset (backend.ts:67, runtime.ts:150-225):
 * position 0, empty history, sink = min(max(sink, 0), maximum_length).  Fails with
 * CONTEXT_OVERFLOW when maximum_length is outside (0, geometry max] or above opts.max_len, and
 * with BACKEND_UNAVAILABLE (the reference's "no resident execution") when sink + window exceeds
 * the context's KV capacity. */
int needle_cuda_seq_reset(needle_ctx* ctx, int32_t seq, int32_t maximum_length, int32_t sink_length);

/* needle_cuda_seq_reset with RuntimeOptions.collectConfidence (runtime.ts:36, 171-180): when
 * collect_confidence is 1 and the archive has a confidence probe head, the slot keeps the online
 * probe pool (OnlineProbePool, runtime.ts:48-105) over the scaled embedding and every layer's
 * hidden state.  needle_cuda_seq_reset(ctx, s, m, k) is needle_cuda_seq_reset_ex(ctx, s, m, k, 0). */
int needle_cuda_seq_reset_ex(needle_ctx* ctx, int32_t seq, int32_t maximum_length, int32_t sink_length,
                             int32_t collect_confidence);

/* NeedleRuntime.confidence (runtime.ts:634-645): sigmoid of the confidence head over the pooled
 * probes, or NaN through *value when the slot does not collect or the archive has no head. */
int needle_cuda_confidence(const needle_ctx* ctx, int32_t seq, double* value);

/* Position (tokens consumed) of a slot. */
int needle_cuda_seq_position(const needle_ctx* ctx, int32_t seq, int32_t* position);

/* One ragged batched decode step over n items (distinct slots, or a slot's prompt chunk).  For
 * every item the slot's token runs through all layers at the slot's position, its K/V are appended
 * to the int8 cache, and the position advances (runtime.ts:280-583).  Items with select=1 write
 * out_selected[i] (selectToken, runtime.ts:880-899).  out_logits (n * vocabulary floats, row i for
 * item i) may be NULL; when given, every item's logits are written (step with wantLogits).  The
 * call is synchronous: results are in host memory on return.  A step of 64 items or more without
 * out_logits runs as needle_opts.micro_batches micro-batches on their own streams, and from the
 * second such step on as a replay of a CUDA graph the engine captures on its own stream; results
 * are the same as one batch's. */
int needle_cuda_step(needle_ctx* ctx, const needle_step_item* items, int32_t n,
                     const uint32_t* allowed_ids, size_t allowed_total,
                     needle_selected* out_selected, float* out_logits);

/* needle_cuda_step in two halves, for constrained decoding, where the allowed ids of a step depend
 * only on tokens already chosen and can be computed on the host while the step's layers run.
 * needle_cuda_step_begin checks the items and enqueues every layer and the vocabulary projection,
 * then returns without waiting; needle_cuda_step_end takes the same items (same slots and tokens in
 * the same order; a select may be cleared, e.g. for a grammar dead end, but not set) with their
 * allowed lists, selects, waits and advances the slots, exactly as needle_cuda_step with those items
 * would have.  No other call may use the context in between (BACKEND_UNAVAILABLE), except
 * needle_cuda_masks_put.  If step_end fails, the step is dropped: the slots keep their positions.
 * Logits are not returned. */
int needle_cuda_step_begin(needle_ctx* ctx, const needle_step_item* items, int32_t n);
int needle_cuda_step_end(needle_ctx* ctx, const needle_step_item* items, int32_t n, const uint32_t* allowed_ids,
                         size_t allowed_total, needle_selected* out_selected);

/* Device-resident allowed-id masks.  An item with allowed_count = NEEDLE_ALLOWED_MASK selects among
 * the ids set in slot allowed_offset of the context's mask pool (bit id % 32 of word id / 32,
 * ceil(vocab / 32) words per slot), with the same result as the ascending id list of those ids: the
 * best logit, ties to the lowest id.  The masks cross PCIe once per new grammar state instead of as
 * an id list at every step (a needle_mask_cache keeps them per state, include/needle_grammar.h).
 * needle_cuda_mask_pool (re)allocates a pool of `capacity` empty slots.  needle_cuda_masks_put
 * copies the masks of the `n` listed slots from `table` (a host table indexed by slot, [capacity]
 * [words], as needle_mask_cache_table gives) into the pool, ordered before every later step on the
 * context (it may run between needle_cuda_step_begin and needle_cuda_step_end).  An item naming a
 * slot whose last put was empty, or never put, fails as an empty allowed set. */
int needle_cuda_mask_pool(needle_ctx* ctx, int32_t capacity);
int needle_cuda_masks_put(needle_ctx* ctx, const int32_t* slots, int32_t n, const uint32_t* table);

/* ---- ResidentExecutionSession (packages/needle.js/src/backends/backend.ts:66-80) ----
 * The per-token calls NeedleRuntime.step makes on a resident session (runtime.ts:305-372), with
 * the arguments it passes them, so an adapter serves an unmodified runtime:
 *   prepareResidentEngrams({indices, valid, position})  -> kept by the adapter (returns true)
 *   beginResidentToken(x)                               -> kept by the adapter (returns true)
 *   forwardResidentToken({position})                    -> needle_cuda_resident_forward
 *   finishResidentToken(wantLogits)                     -> needle_cuda_resident_finish
 *   finishResidentTokenForSelection()                   -> nothing (the vocabulary projection ran)
 *   selectResidentToken(allowed?)                       -> needle_cuda_resident_select
 * needle_cuda_resident_forward enqueues every layer and the vocabulary projection for slot `seq`
 * from the runtime's lanes (x: mhc_lanes * model_dimension floats, the scaled embedding row in each
 * lane, runtime.ts:305-313) and its engram lookup (engram_tables table indices and valid flags from
 * #engramLookup, runtime.ts:788-818; NULL / 0 for an archive without engram sites), then returns
 * without waiting.  `position` and `engram_position` must equal the slot's position.  The token
 * then ends with exactly one of needle_cuda_resident_finish (logits, vocabulary floats, written
 * when non-NULL; nothing is selected) or needle_cuda_resident_select (allowed ids; n_allowed -1 for
 * the whole vocabulary), which wait and advance the slot; no other call may use the context in
 * between.  If the end fails, the token is dropped and the slot keeps its position.  A slot stepped
 * this way keeps no token history: its engram lookups always come from the caller. */
int needle_cuda_resident_forward(needle_ctx* ctx, int32_t seq, int32_t position, const float* lanes,
                                 const uint32_t* engram_indices, const uint32_t* engram_valid,
                                 int32_t engram_tables, int32_t engram_position);
int needle_cuda_resident_finish(needle_ctx* ctx, int32_t seq, float* logits);
int needle_cuda_resident_select(needle_ctx* ctx, int32_t seq, const uint32_t* allowed_ids, int32_t n_allowed,
                                needle_selected* out_selected);

/* NeedleRuntime.prefill (runtime.ts:227-243) for one slot: the n tokens, logits of the last one
 * written to out_logits (vocabulary floats) when non-NULL.  The result is that of n one-token
 * steps; the tokens go through the layers in chunks of up to 64, one item per token (K/V of the
 * whole chunk appended before its items attend), except for a slot that collects confidence, for
 * positions whose chunk would wrap the KV window, and for the last token when its logits are
 * wanted. */
int needle_cuda_prefill(needle_ctx* ctx, int32_t seq, const int32_t* ids, int32_t n, float* out_logits);

/* Copies one layer of a slot's int8 KV cache (layout of runtime.ts:666-677): codes
 * [kv_heads][kv_allocation][head_dim], scales [kv_heads][kv_allocation], where kv_allocation is the
 * slot's min(maximum_length, sink + window) (runtime.ts:166-170).  Any pointer may be NULL.  Slots
 * of a loaded device-scheduler queue are read as the scheduler left them. */
int needle_cuda_read_kv(const needle_ctx* ctx, int32_t seq, int32_t layer, int8_t* key_codes,
                        int8_t* value_codes, float* key_scales, float* value_scales,
                        int32_t* kv_allocation);

/* Copies one layer of a slot's float32 KV cache (contexts opened with NEEDLE_KV_FLOAT32): keys and
 * values [kv_heads][kv_allocation][head_dim].  Either pointer may be NULL.  needle_cuda_read_kv
 * fails with INVALID_CACT on such a context, and this call on an int8 one. */
int needle_cuda_read_kv_f32(const needle_ctx* ctx, int32_t seq, int32_t layer, float* keys, float* values,
                            int32_t* kv_allocation);

/* Reads a slot's mHC lane state x (lanes * model_dimension floats) after its last step. */
int needle_cuda_read_lanes(const needle_ctx* ctx, int32_t seq, float* lanes);

/* InferenceBackend.matvec (backend.ts:89-93; CpuBackend.matvec cpu.ts:12-16): rows
 * [row_start, row_start + row_count) of archive tensor `tensor` (a CQ matrix) times `batch` input
 * vectors x (batch * input_size floats) into y (batch * row_count floats). */
int needle_cuda_matvec(needle_ctx* ctx, int32_t tensor, int32_t row_start, int32_t row_count,
                       const float* x, int32_t batch, float* y);

/* InferenceBackend.row (backend.ts:107; dequantizeCqRow, cq.ts:243-295). */
int needle_cuda_row(needle_ctx* ctx, int32_t tensor, int32_t row, float* out);

/* ---- Device-pointer operators (isolated kernels; the caller owns every buffer). ---- */

/* A Cactus-Quant matrix resident in device memory (CqMatrix, cact.ts:61-75). */
typedef struct needle_cq_matrix {
  const uint8_t* packed;  /* rows * row_bytes, 16-byte aligned */
  const uint16_t* norms;  /* rows * (input_padded / group) fp16, 4-byte aligned */
  int32_t rows;
  int32_t input_size;
  int32_t group_size;     /* 128 */
  int32_t bits;           /* 2, 3, 4 or 5 (ternary record marker) */
} needle_cq_matrix;

/* cqMatvec (cq.ts:233-240) on device buffers: x is batch * input_size floats (row stride
 * input_size), y is batch * rows floats.  `codebook` is 28 HOST floats (CQ2|CQ3|CQ4, the archive's
 * shared codebook).  Runs on `stream` (a cudaStream_t; NULL = legacy default stream) without
 * synchronising.  The prepared (Hadamard-rotated) activations go to a scratch buffer that the
 * library owns, one per device, grown with cudaMalloc when a call needs more. */
int needle_cuda_cq_matvec_dev(const needle_cq_matrix* m, const float* codebook, const float* x,
                              int32_t batch, float* y, void* stream);

/* The same matvec in fast numerics (record widths 2, 4 and ternary): results agree with cqMatvec
 * within binary32 rounding, not bit for bit.  Up to 15 items (5 for matrices of 4M weights and
 * more) it runs the table GEMV (binary32 per-group byte tables, weights streamed once per 8 items);
 * above, the tensor-core GEMM (fp16 head/tail split, fp32 accumulation, up to 128 items per pass).
 * Same arguments and scratch as needle_cuda_cq_matvec_dev; 3-bit matrices return
 * UNSUPPORTED_CACT. */
int needle_cuda_cq_matvec_dev_fast(const needle_cq_matrix* m, const float* codebook, const float* x,
                                   int32_t batch, float* y, void* stream);

/* Capacity, in floats, of the fixed scratch array used by needle_cuda_cq_matvec_dev_noalloc:
 * batch * input_padded must not exceed it (4 MiB of device memory per GPU). */
#define NEEDLE_NOALLOC_MAX_FLOATS (1 << 20)

/* Same result as needle_cuda_cq_matvec_dev, but the call allocates no device memory.
 * No counterpart in the reference: it exists for callers that cannot call cudaMalloc -- a host
 * that hands all device memory to its own pool at start-up, or a latency-critical serving loop
 * that must not take cudaMalloc's implicit device-wide synchronisation.  The rotated activations
 * go to a statically sized array inside the library (NEEDLE_NOALLOC_MAX_FLOATS floats, reserved
 * on every GPU that loads the library until the process exits); larger batch * input_padded is
 * rejected with BACKEND_UNAVAILABLE.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress), so make that first call before any stream capture.  All calls
 * share the one array and each call overwrites every element it reads, so no clearing is needed;
 * calls whose executions overlap on the GPU (different streams, or host threads) race on it and
 * must be serialised by the caller. */
int needle_cuda_cq_matvec_dev_noalloc(const needle_cq_matrix* m, const float* codebook,
                                      const float* x, int32_t batch, float* y, void* stream);

/* Decode attention over an int8 cache with kvWindow = 0 semantics (runtime.ts:719-786) for a
 * ragged batch, on device buffers:
 *   q        [batch][heads * head_dim] floats
 *   codes    [batch][kv_heads][capacity][head_dim] int8 (key_codes, value_codes)
 *   scales   [batch][kv_heads][capacity] floats
 *   counts   [batch] int32 visible positions (1..capacity)
 *   out      [batch][heads * head_dim] floats
 * heads = 8, kv_heads = 4, head_dim = 64 (the Needle 2 geometry). */
int needle_cuda_attention_dev(const float* q, const int8_t* key_codes, const float* key_scales,
                              const int8_t* value_codes, const float* value_scales,
                              const int32_t* counts, int32_t batch, int32_t capacity, float* out,
                              void* stream);

/* The same attention in fast numerics: binary32 arithmetic, online softmax, positions split
 * across CTAs and merged by max-rescaled sums (flash decoding).  Same arguments and layout as
 * needle_cuda_attention_dev; results agree with the reference within binary32 rounding (not bit
 * for bit).  capacity is unbounded.  Split partials go to a library-owned scratch buffer per
 * device, grown with cudaMalloc when a call needs more. */
int needle_cuda_attention_dev_fast(const float* q, const int8_t* key_codes, const float* key_scales,
                                   const int8_t* value_codes, const float* value_scales,
                                   const int32_t* counts, int32_t batch, int32_t capacity,
                                   float* out, void* stream);

/* ---- Bounded device waits ----
 * The kernels that wait on asynchronous copies or barriers -- the fast attention, the table matvec and
 * the tensor-core matvec -- give up after 2 s instead of spinning forever.  The outputs of that call
 * are then NaN, and the kernel records its kind in the device's wait-status word (pinned host memory:
 * readable without synchronising).  The next needle_cuda_cq_matvec_dev_fast or
 * needle_cuda_attention_dev_fast call on that device returns BACKEND_UNAVAILABLE, naming the kernels,
 * and clears the word.  (The reference's GPU path is WebGPU, whose device loss the browser reports;
 * these statuses play that part.) */
#define NEEDLE_WAIT_ATTENTION 1u   /* k_attention_fast_mma */
#define NEEDLE_WAIT_TABLE_GEMV 2u  /* k_cq_gemv_table */
#define NEEDLE_WAIT_TENSOR_GEMM 4u /* k_cq_gemm_tc */
#define NEEDLE_WAIT_SELFTEST 8u    /* needle_cuda_wait_selftest */

/* The wait-status bits of `device` (NEEDLE_WAIT_*) through *kinds; clear = 1 resets them. */
int needle_cuda_wait_status(int32_t device, uint32_t* kinds, int32_t clear);

/* Diagnostic of the path above: one GPU thread of the current device waits, up to limit_ns
 * (at most 1 s), on a device flag that nothing sets, gives up, records NEEDLE_WAIT_SELFTEST and
 * returns -- what every waiting kernel does when its wait runs out, without a stalled copy. */
int needle_cuda_wait_selftest(uint64_t limit_ns, void* stream);

/* ---- Benchmark / device-resident scheduling ---- */

/* Returns the context's CUDA stream (a cudaStream_t) so callers can time on it. */
void* needle_cuda_stream(const needle_ctx* ctx);

/* Device-resident ragged decode (continuous batching without host round trips).  Loads a queue
 * of sequences: prompt ids (concatenated, prompt_offsets has n_seqs + 1 entries) and the number
 * of greedy tokens each generates; slots [0, min(n_slots, n_seqs)) admit the first sequences.
 * Each needle_cuda_sched_step then runs one batched step over every busy slot: a slot consumes
 * its next prompt token or, after the prompt, its last greedily selected token; a slot whose
 * sequence has selected its last token admits the next queued sequence. */
int needle_cuda_sched_load(needle_ctx* ctx, int32_t n_slots, const int32_t* prompt_offsets,
                           const int32_t* prompt_ids, const int32_t* gen_steps, int32_t n_seqs);
/* Enqueues `steps` device-resident steps on the context stream without synchronising. */
int needle_cuda_sched_step(needle_ctx* ctx, int32_t steps);
/* Synchronises and reports progress: tokens processed (steps taken, prompt and generated tokens
 * alike), tokens generated (greedy selections), sequences finished, and for every queued
 * sequence its last selected token (n_seqs entries, -1 while unfinished; may be NULL). */
int needle_cuda_sched_status(needle_ctx* ctx, int64_t* tokens_processed, int64_t* tokens_generated,
                             int32_t* seqs_finished, int32_t* last_ids);

/* Every token the device scheduler has selected, by sequence: sequence s's greedy ids occupy
 * entries [G(s), G(s) + gen_steps[s]) with G(s) = gen_steps[0] + ... + gen_steps[s - 1], in the
 * order they were selected; entries not yet generated are -1.  Copies min(n, total) entries
 * (synchronising first) and reports the total through *total (either pointer may be NULL).  The
 * per-sequence id stream of NeedleModel.generate's greedy loop (packages/needle.js/src/model/
 * model.ts:116-137), for checking a scheduled run against one-sequence decodes. */
int needle_cuda_sched_ids(needle_ctx* ctx, int32_t* ids, size_t n, size_t* total);

/* State of one scheduler slot: the queued sequence it holds or last held (-1 if it never admitted
 * one), the tokens that sequence has consumed, and whether it is still running.  With
 * needle_cuda_read_kv on the same slot, this reads a scheduled sequence's int8 KV cache. */
int needle_cuda_sched_slot(needle_ctx* ctx, int32_t slot, int32_t* seq_id, int32_t* position, int32_t* busy);

/* Number of CUDA kernels this context has launched so far (for launch accounting). */
int needle_cuda_kernel_launches(const needle_ctx* ctx, int64_t* count);

/* Overrun check (no counterpart; the reference has no sanitizer, and compute-sanitizer is not
 * available where this runs): every device buffer of the context's model, slot state and step
 * scratch is followed by 256 guard bytes of a fixed pattern; this synchronises the device and
 * reports through *damaged how many guards no longer hold it (0: no kernel wrote past the end of
 * those buffers).  With the environment variable NEEDLE_NVTX set (not "0") when the context is
 * opened, every step and kernel class is also an NVTX range, for profilers that filter by range. */
int needle_cuda_check_guards(const needle_ctx* ctx, int32_t* damaged);

/* Per-kernel-class timing with CUDA events on the context stream (off by default).  enable=1
 * starts accumulating, enable=0 stops.  read fills up to n entries of (name, total ms, launches)
 * and returns the number of classes through *count. */
int needle_cuda_profile(needle_ctx* ctx, int32_t enable);
int needle_cuda_profile_read(needle_ctx* ctx, int32_t n, const char** names, double* total_ms,
                             int64_t* launches, int32_t* count);

#ifdef __cplusplus
}
#endif
#endif /* NEEDLE_CUDA_H */
