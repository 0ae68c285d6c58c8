/*
 * needle_ref -- CPU ORACLE for the Needle 2 decode path.  TEST INFRASTRUCTURE ONLY.
 *
 * A C++ restatement of the needle.js pure-TypeScript CPU backend, written to reproduce
 * JavaScript numeric semantics: every arithmetic expression is evaluated in binary64 and a
 * value is rounded to binary32 only where the TypeScript stores it into a Float32Array.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg / reference arm
 * may load this library; the CUDA engine never links or calls it.
 *
 * Parity status: pinned at the unit level against the reference's own fixtures
 * (packages/needle.js/tests/cq.test.ts, fp16.test.ts, cact.test.ts), restated in
 * tests/test_oracle_fixtures.py.  The reference publishes no model-level golden vectors
 * for synthetic weights, so model-level outputs of this oracle are the oracle of record.
 *
 * Status codes equal the needle_cuda status codes (include/needle_cuda.h), which map
 * 1:1 onto NeedleErrorCode (packages/needle.js/src/errors.ts:1-11).
 */
#ifndef NEEDLE_REF_H
#define NEEDLE_REF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ref_model ref_model;
typedef struct ref_runtime ref_runtime;

const char* ref_last_error(void);

/* fp16 codec: packages/needle.js/src/model/fp16.ts:5-74 */
double ref_float16_to_number(uint32_t h);
uint32_t ref_number_to_float16(double v);

/* FWHT in place on float32: packages/needle.js/src/backends/cq.ts:8-27 */
int ref_fwht(float* values, int32_t length);

/* A free-standing CQ matrix (pointers borrowed; cb2/cb3/cb4 are 4/8/16 floats). */
typedef struct ref_cq_desc {
  int32_t rows, input_size, group_size, bits; /* bits: 2, 3, 4 or 5 (ternary marker) */
  const uint8_t* packed;                      /* rows * row_bytes */
  const uint8_t* norms;                       /* rows * groups fp16, little endian */
  const float* cb2;
  const float* cb3;
  const float* cb4;
} ref_cq_desc;

/* cqMatvec (cq.ts:233-240 = prepareCqActivation cq.ts:30-46 + cqMatvecPrepared cq.ts:107-231) */
int ref_cq_matvec_desc(const ref_cq_desc* m, const float* x, int32_t row_start, int32_t row_count,
                       float* y);
/* prepareCqActivation only (cq.ts:30-46); out has input_size_padded floats. */
int ref_cq_prepare_desc(const ref_cq_desc* m, const float* x, float* out);
/* dequantizeCqRow (cq.ts:243-295) */
int ref_cq_row_desc(const ref_cq_desc* m, int32_t row, float* out);

/* Archive: parseCact (packages/needle.js/src/model/cact.ts:189-562).  Bytes are copied. */
int ref_model_open(const uint8_t* bytes, size_t n, ref_model** out);
void ref_model_close(ref_model* m);
/* Geometry as 32 int32 slots: the header's u32 fields 3..28 at indices 3..28, tensor count at
 * 1, codebook length at 2; rope theta returned separately. */
int ref_model_geometry(const ref_model* m, int32_t* fields32, float* rope_theta);
int ref_model_num_tensors(const ref_model* m);
/* Record of tensor i: dtype, rank, shape[4], group, bits; byte offset/length. */
int ref_model_record(const ref_model* m, int32_t index, int32_t* info8, uint64_t* offset,
                     uint64_t* length);
/* matvec / row on tensor i of the archive (a CQ tensor). */
int ref_model_matvec(const ref_model* m, int32_t tensor, const float* x, int32_t row_start,
                     int32_t row_count, float* y);
int ref_model_row(const ref_model* m, int32_t tensor, int32_t row, float* out);

/* NeedleRuntime (packages/needle.js/src/model/runtime.ts:108-878).  kv_mode 0 = int8, 1 = f32. */
int ref_runtime_new(const ref_model* m, int32_t kv_mode, int32_t collect_confidence,
                    ref_runtime** out);
void ref_runtime_free(ref_runtime* rt);
int ref_runtime_reset(ref_runtime* rt, int32_t maximum_length, int32_t sink_length);
int ref_runtime_position(const ref_runtime* rt);
int ref_runtime_kv_allocation(const ref_runtime* rt);
/* step (runtime.ts:280-583).  logits may be NULL (wantLogits false). */
int ref_runtime_step(ref_runtime* rt, int32_t token, float* logits);
/* stepSelected (runtime.ts:257-278) with selectToken (runtime.ts:880-899).
 * allowed == NULL selects over the full vocabulary (argmax). */
int ref_runtime_step_selected(ref_runtime* rt, int32_t token, const uint32_t* allowed,
                              int32_t n_allowed, int32_t* id, double* log_probability);
/* Copies one layer of the int8 cache: codes [kv_heads][alloc][head_dim], scales
 * [kv_heads][alloc].  Any pointer may be NULL. */
int ref_runtime_read_kv(const ref_runtime* rt, int32_t layer, int8_t* key_codes,
                        int8_t* value_codes, float* key_scales, float* value_scales);
/* Copies one layer of the float32 cache (kv_mode 1): keys / values [kv_heads][alloc][head_dim]. */
int ref_runtime_read_kv_f32(const ref_runtime* rt, int32_t layer, float* keys, float* values);
/* Lane state x: lanes * model_dimension floats. */
int ref_runtime_read_lanes(const ref_runtime* rt, float* lanes);
/* Confidence (runtime.ts:634-645); returns NaN through *value when unavailable. */
int ref_runtime_confidence(const ref_runtime* rt, double* value);

/* Greedy generation in the shape of NeedleModel.generate (packages/needle.js/src/model/model.ts:
 * 88-153) without tokenizer or EOS stop: reset(prompt + steps, sink), prefill(prompt), then
 * `steps` argmax tokens with a step() between consecutive ones.  logits (steps * vocab) and
 * log_probabilities may be NULL. */
int ref_generate_greedy(const ref_model* m, const int32_t* prompt, int32_t n_prompt,
                        int32_t steps, int32_t sink, int32_t* out_ids,
                        double* out_log_probabilities, float* out_logits);

/* Ragged CPU decode baseline: independent sequences spread over n_threads host threads; each
 * sequence runs prompt + greedy steps exactly as ref_generate_greedy.  Returns the number of
 * step() calls made (tokens processed) through *tokens_processed and, when out_seconds is not
 * NULL, each sequence's own compute time on its thread. */
int ref_decode_many(const ref_model* m, int32_t n_seqs, const int32_t* prompt_offsets,
                    const int32_t* prompt_ids, const int32_t* gen_steps, int32_t n_threads,
                    int32_t* out_last_ids, int64_t* tokens_processed, double* out_seconds);

/* Continuous batching on the host, the CPU counterpart of needle_cuda_sched_*: n_slots slots
 * admit queued sequences (prompt ids concatenated, prompt_offsets has n_seqs + 1 entries;
 * gen_steps greedy tokens each) in queue order into the lowest idle slot; every ref_sched_step
 * runs one step for every busy slot -- its next prompt token or its last greedy token -- spread
 * over n_threads host threads.  A sequence retires after selecting its last token. */
typedef struct ref_sched ref_sched;
int ref_sched_new(const ref_model* m, int32_t n_slots, const int32_t* prompt_offsets,
                  const int32_t* prompt_ids, const int32_t* gen_steps, int32_t n_seqs,
                  int32_t n_threads, ref_sched** out);
int ref_sched_step(ref_sched* s, int32_t steps);
int ref_sched_status(const ref_sched* s, int64_t* tokens_processed, int64_t* tokens_generated,
                     int32_t* seqs_finished, int32_t* last_ids);
void ref_sched_free(ref_sched* s);

/* Decode attention over an int8 cache with kvWindow = 0 semantics (runtime.ts:719-786):
 * visible positions 0..count-1.  q: heads*hd; caches [kv_heads][count][hd]; scales
 * [kv_heads][count]; out heads*hd. */
int ref_attention_int8(int32_t heads, int32_t kv_heads, int32_t head_dim, int32_t count,
                       const float* q, const int8_t* key_codes, const float* key_scales,
                       const int8_t* value_codes, const float* value_scales, float* out);

/* #storeKV quantisation of one head vector (runtime.ts:697-714). */
int ref_quantize_kv_head(const float* x, int32_t head_dim, int8_t* codes, float* scale);

#ifdef __cplusplus
}
#endif
#endif
