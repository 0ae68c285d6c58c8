/* needle_grammar.h -- host-side constrained tool-call grammar of the CUDA backend (plain C ABI).
 *
 * The constrained tool-call loop of needle.js (packages/needle.js/src/tools/agent.ts:157-210)
 * keeps a byte grammar of the tool-call JSON, asks it which vocabulary pieces may come next, lets
 * the device pick the best allowed token (needle_cuda_step with an allowed-id list: the fused mask +
 * argmax) and feeds the chosen piece back.  These entry points replace, for that loop:
 *
 *   needle_grammar_tools    new ToolCallGrammar(normalizeTools(tools), maxCalls)
 *                           (packages/needle.js/src/tools/grammar.ts:666-670, schema.ts:196-204)
 *   needle_grammar_schema   new JsonSchemaGrammar(schema)               (grammar.ts:263-266)
 *   needle_grammar_clone    grammar.clone()                              (grammar.ts:288-294, 681-697)
 *   needle_grammar_feed     grammar.feed(bytes)                          (grammar.ts:296-299, 699-702)
 *   needle_grammar_complete grammar.complete                             (grammar.ts:268-278, 672-674)
 *   needle_grammar_result   JSON.stringify(grammar.value) / (grammar.calls)
 *   needle_vocab_open       the pieces the loop may emit: tokenizer.pieceBytes(id) of the Normal and
 *                           Byte pieces (tokenizer.ts:257-282; agent.ts:168-170), empty for others
 *   needle_grammar_allowed  the loop's candidate scan (agent.ts:165-176): every id whose piece the
 *                           grammar accepts, ascending, with the 64 KiB output limit
 *
 * Status codes are those of needle_cuda.h (NEEDLE_INVALID_TOOL_SCHEMA for schema and argument
 * errors), with the message in needle_cuda_last_error().  A grammar is not thread-safe; distinct
 * grammars may be used from distinct threads.
 */
#ifndef NEEDLE_GRAMMAR_H
#define NEEDLE_GRAMMAR_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct needle_grammar needle_grammar;
typedef struct needle_vocab needle_vocab;

/* A tool-call grammar over `tools_json`, a JSON array of tools ({"name", "description"?,
 * "parameters"?} or OpenAI {"type": "function", "function": {...}}), normalised as normalizeTools
 * does; at most `maximum_calls` calls (at least 1). */
int needle_grammar_tools(const char* tools_json, int32_t maximum_calls, needle_grammar** out);
/* A JSON-value grammar for one JSON Schema. */
int needle_grammar_schema(const char* schema_json, needle_grammar** out);
int needle_grammar_clone(const needle_grammar* grammar, needle_grammar** out);
void needle_grammar_free(needle_grammar* grammar);
/* Feeds `n` bytes; *accepted = 0 as soon as one is rejected (the grammar is then spent, as in the
 * reference: keep a clone to retry). */
int needle_grammar_feed(needle_grammar* grammar, const uint8_t* bytes, int32_t n, int32_t* accepted);
int needle_grammar_complete(const needle_grammar* grammar, int32_t* complete);
/* The value (schema grammar; empty before it is complete) or the calls so far as a JSON array of
 * {"name", "arguments"} (tool-call grammar), NUL-terminated into buf[capacity]; *length is the
 * full length. */
int needle_grammar_result(const needle_grammar* grammar, char* buf, int32_t capacity, int32_t* length);

/* The vocabulary's piece bytes: piece `id` is bytes[offsets[id] .. offsets[id + 1]); pieces that
 * may not be emitted (control, unknown, user-defined) have no bytes. */
int needle_vocab_open(const uint8_t* bytes, const int32_t* offsets, int32_t count, needle_vocab** out);
void needle_vocab_free(needle_vocab* vocab);
/* The ids that may come next, ascending, given `output_bytes` already emitted; *count is the number
 * of ids (NEEDLE_INVALID_TOOL_SCHEMA when it exceeds `capacity`). */
int needle_grammar_allowed(const needle_grammar* grammar, const needle_vocab* vocab, int64_t output_bytes,
                           uint32_t* ids, int32_t capacity, int32_t* count);
/* The same for `n` grammars on up to `threads` host threads: grammar k's ids go to
 * ids[k * capacity_each ..], their number to counts[k]; a null grammar yields no ids. */
int needle_grammar_allowed_batch(const needle_grammar* const* grammars, const int64_t* output_bytes, int32_t n,
                                 const needle_vocab* vocab, int32_t threads, uint32_t* ids,
                                 int32_t capacity_each, int32_t* counts);

/* Allowed-token masks per grammar state.  Many sequences of a batch sit in the same grammar state
 * (inside the free content of an argument string, after the same key, at the same separator), and
 * one sequence revisits states; the scan above (agent.ts:165-176) depends only on that state and on
 * the room left under the 64 KiB limit, so its result is kept, as a bit mask over the vocabulary,
 * under a key of both.  The reference rescans the vocabulary at every step and has no counterpart;
 * a mask holds exactly the ids needle_grammar_allowed returns for the same grammar (bit id % 32 of
 * word id / 32).  The masks live in a table of `capacity` slots, reused least recently used first;
 * the slot numbers are meant to index a copy of the table on the device (needle_cuda_masks_put),
 * so a step's items can name a mask instead of carrying an id list.
 *
 * A cache serves the clones of one template grammar (it keeps a clone of it) and one vocabulary
 * (which must outlive it).  Not thread-safe. */
typedef struct needle_mask_cache needle_mask_cache;
int needle_mask_cache_open(const needle_grammar* template_grammar, const needle_vocab* vocab, int32_t capacity,
                           needle_mask_cache** out);
void needle_mask_cache_free(needle_mask_cache* cache);
/* The host table: capacity x words uint32, words = ceil(vocabulary size / 32); valid until the
 * cache is freed. */
int needle_mask_cache_table(const needle_mask_cache* cache, const uint32_t** table, int32_t* words);
/* For `n` grammars (clones of the template; null entries give slot -1 and count 0): slots[k] is the
 * table slot of grammar k's mask and counts[k] its number of ids (0: no token can continue).  States
 * not in the table are scanned on up to `threads` host threads into slots taken least recently used
 * first; those slots are listed in filled[0 .. *n_filled) (at most n entries; their contents
 * changed).  No slot that one call uses is evicted by the same call, so `capacity` must be at least
 * the number of distinct states in one call (NEEDLE_INVALID_TOOL_SCHEMA otherwise). */
int needle_mask_cache_lookup(needle_mask_cache* cache, const needle_grammar* const* grammars,
                             const int64_t* output_bytes, int32_t n, int32_t threads, int32_t* slots,
                             int32_t* counts, int32_t* filled, int32_t* n_filled);
int needle_mask_cache_stats(const needle_mask_cache* cache, int64_t* hits, int64_t* misses, int64_t* evictions);

#ifdef __cplusplus
}
#endif

#endif /* NEEDLE_GRAMMAR_H */
