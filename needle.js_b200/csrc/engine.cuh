// engine.cuh -- device-side data layout of the decode engine and the launchers of its fused
// per-sequence kernels (layer.cu).
#pragma once

#include <string>

#include "cq.cuh"

namespace needle {

constexpr int kMaxProbes = 32;  // confidence probes an archive may carry
constexpr int kMaxMicro = 8;    // micro-batches of a device-scheduled step

// A Cactus-Quant matrix in device memory (CqMatrix, packages/needle.js/src/model/cact.ts:61-75).
struct CqMat {
  const uint8_t* packed = nullptr;
  const uint16_t* norms = nullptr;
  int32_t rows = 0, input_size = 0, in_pad = 0, bits = 0, row_bytes = 0;
};

// Read-only model parameters (device pointers).  Per-layer dense vectors are packed [L][n].
struct ModelView {
  CqMat embedding, phi_pre, phi_post, phi_res;
  CqMat engram_tables[kMaxSites];
  int32_t layers, vocab, kv_window, max_seq;
  int32_t n_sites, sites[kMaxSites];
  int32_t n_orders, orders[4], max_order;
  int32_t n_tables, engram_slots, engram_sub, taps;
  const float *norm_input, *query_norm, *key_norm, *post_norm, *pre_had_norm;  // [L][512|64]
  const float *d1, *d2, *d3;                                                    // [L][512]
  const float* attn_gate;                                                       // [L]
  const float *a_pre, *a_post, *a_res, *b_pre, *b_post, *b_res;
  const float* taps_w;      // [sites][taps][512]
  const float* final_norm;  // [512]
  const double *rope_cos, *rope_sin;  // [max_seq][32], computed on the host in binary64
  Codebook cb;
  // Confidence probe head (cact.ts probe-head manifest code 2), or probe_count 0.
  const float* probes;      // [probe_count][512]
  const float* probe_proj;  // [probe_out][probe_count * 512]
  const float* probe_bias;  // [probe_out]
  int32_t probe_count, probe_out;
  int32_t fast;             // NEEDLE_NUMERICS_FAST: block-reduced sums in k_layer
};

// Per-slot sequence state (NeedleRuntime fields, runtime.ts:113-133), device-authoritative.
struct SeqState {
  int32_t position;    // tokens consumed
  int32_t sink;        // sinkLength
  int32_t max_len;     // maximumLength
  int32_t kv_alloc;    // min(maximumLength, sink + window) or maximumLength (runtime.ts:166-170)
  int32_t pending;     // last selected token
  int32_t hist[3];     // previous tokens, most recent first (engram n-grams, runtime.ts:788-818)
  // device scheduler
  int32_t busy, seq_id, prompt_off, prompt_len, gen_target, gen_done;
  int32_t collect;     // collectConfidence: feed the probe pool
};

// Slot-indexed device state.
struct SlotView {
  int32_t capacity;     // KV positions per (slot, layer, kv head)
  int32_t layers;
  float* x;             // [S][4][512] mHC lanes
  float* ring;          // [S][sites][10][512] engram value ring
  int32_t kv_f32;       // 1: float32 cache (kf / vf), 0: int8 cache (kcodes / vcodes)
  int8_t* kcodes;       // [S][L][4][capacity][64]
  int8_t* vcodes;
  float* kf;            // [S][L][4][capacity][64] (float32 mode)
  float* vf;
  float* kscale;        // [S][L][4][capacity] (1 in float32 mode)
  float* vscale;
  SeqState* seq;        // [S]
  // OnlineProbePool per slot (allocated when the archive has a confidence head)
  double* pool_max;     // [S][probes]
  double* pool_den;     // [S][probes]
  double* pool_w;       // [S][probes][512]
};

// One resolved item of a step (internal order: selecting items first).
struct DevItem {
  int32_t slot;
  int32_t token;            // >= 0, or NEEDLE_TOKEN_PENDING (-1) until k_embed resolves it
  int32_t select;
  int32_t allowed_count;    // -1 unmasked, >0 ids at allowed_offset, kAllowedMask: pool slot
  uint32_t allowed_offset;
  int32_t position;         // filled by k_embed
  int32_t out_index;        // caller's index
  int32_t flags;            // kItemLanes | kItemEngrams: inputs given by a resident session
  // A prefill chunk: chunk_len (>= 2) consecutive positions of one slot as consecutive items, this
  // one at chunk_index; 0 for an item of its own.  The chunk's items get their positions and tokens
  // from the item, their lanes per item (StepView::lanes), read the engram taps and token history
  // of the chunk's earlier items, append K/V before any of them attends (StepView::chunk), and the
  // slot advances once, at the chunk's last item.
  int32_t chunk_index;
  int32_t chunk_len;
};

// DevItem::flags.  A resident-session item (needle_cuda_resident_forward) brings the lanes that
// NeedleRuntime built from the embedding row (StepView::lanes, row = item) and the engram lookup it
// hashed from its token history (StepView::engram_in), instead of a token.
constexpr int32_t kItemLanes = 1;
constexpr int32_t kItemEngrams = 2;

// DevItem::allowed_count of an item whose allowed ids are a bit mask of the mask pool
// (StepView::masks, slot allowed_offset): NEEDLE_ALLOWED_MASK.
constexpr int32_t kAllowedMask = -2;

// Step scratch, indexed by internal item index.
struct StepView {
  DevItem* items;
  const int32_t* n_items;   // device count (all items)
  const int32_t* n_select;  // device count of selecting items (a prefix of items)
  const uint32_t* allowed;  // allowed ids
  const uint32_t* masks;    // [pool slots][mask_words] allowed-id bit masks (bit id % 32 of word id / 32)
  int32_t mask_words;
  float* prep_engram;       // [B][sites][512]
  float* engram_kv;         // [B][sites][2][512]  (K projection, V projection)
  float* engram_val;        // [B][sites][512]      convolved values
  float* update;            // [B][512]
  float* block;             // [B][512]
  float* prep_a;            // [B][512]  prepared attention input
  float* qkvg;              // [B][1536] q | k | v | gate
  float* prep_o;            // [B][512]  prepared output-projection input
  float* proj;              // [B][512]
  float* route;             // [B][20]   hPost[4] | routing[16]
  float* prep_f;            // [B][512]  prepared vocabulary input
  float* logits;            // [B][vocab]
  int32_t* out_id;          // [B]
  double* out_logprob;      // [B]
  // A prefill chunk: items 0..n-1 are the positions p0, p0 + 1, ... of one slot, in order, none
  // selecting.  Their lanes are per item (`lanes`) instead of per slot, K/V are appended for the
  // whole chunk before any item attends, and the slot's state (position, token history, engram
  // ring) advances once, after the chunk.
  // fast numerics: what the append pass (k_attention part 1) leaves for the fast attention kernel
  float* qrope;             // [B][512] normalised, rotated queries
  float* attn_out;          // [B][512] attention output (before the gate)
  int32_t* attn_count;      // [B] visible cache slots: slots 0 .. count-1 in the ring layout
  int64_t* attn_row;        // [B] cache row of (item, layer, KV head 0)
  int32_t chunk;            // the step may hold chunk items (DevItem::chunk_len): K/V append first
  float* lanes;             // [B][4][512] (chunk items; kItemLanes items)
  const uint32_t* engram_in;  // [B][2][kMaxTables]: table indices, then valid flags (kItemEngrams)
};

// Device scheduler queue (needle_cuda_sched_*).
struct SchedView {
  const int32_t* prompt_offsets;  // [n_seqs + 1]
  const int32_t* prompt_ids;
  const int32_t* gen_steps;       // [n_seqs]
  int32_t n_seqs;
  int32_t n_slots;
  int32_t* next_seq;              // queue head
  int32_t* finished;              // finished count
  int64_t* processed;             // tokens processed
  int64_t* generated;             // tokens selected (generated)
  int32_t* last_ids;              // [n_seqs]
  const int64_t* gen_offsets;     // [n_seqs]: start of each sequence's run in gen_ids
  int32_t* gen_ids;               // [sum of gen_steps]: every selected id, by sequence, in order
};

cudaError_t launch_embed(const ModelView& m, const SlotView& sv, const StepView& st, int n_host,
                         cudaStream_t s);
cudaError_t launch_layer(const ModelView& m, const SlotView& sv, const StepView& st, int layer,
                         int n_host, cudaStream_t s);
// Sinkhorn routing of the layer's items (reads and writes StepView::route[4..19]).
cudaError_t launch_route(const StepView& st, int n_host, cudaStream_t s);
// Steps that may hold chunk items (StepView::chunk) launch it twice: part 3 appends the chunk
// items' K/V, part 4 attends (and appends for the other items); otherwise part 0 does both per item.
cudaError_t launch_attention(const ModelView& m, const SlotView& sv, const StepView& st, int layer,
                             int n_host, cudaStream_t s, int part = 0);
cudaError_t launch_finish(const ModelView& m, const SlotView& sv, const StepView& st, int n_host,
                          const SchedView* sched, cudaStream_t s);
// Copies staged masks into the mask pool: mask k of `staged` ([n][words]) to slot slots[k].
cudaError_t launch_mask_scatter(const uint32_t* staged, const int32_t* slots, int n, int words, uint32_t* pool,
                                cudaStream_t s);
// Device scheduler: builds the step's item list and the counts [all, selecting, then (all,
// selecting) of each of `parts` micro-batches], micro-batch k being items [k * part, (k + 1) * part).
cudaError_t launch_sched(const SlotView& sv, const StepView& st, const SchedView& q, int32_t* counts, int part,
                         int parts, cudaStream_t s);
// The same with prompt chunks: micro-batch k holds slots [k * slots_per_part, ...) and item rows
// [k * items_per_part, ...); a prefilling slot takes up to chunk_max prompt positions (n_slots <= 1024).
cudaError_t launch_sched_chunked(const SlotView& sv, const StepView& st, const SchedView& q, int32_t* counts,
                                 int slots_per_part, int items_per_part, int parts, int chunk_max, int window,
                                 cudaStream_t s);
cudaError_t launch_sched_admit(const SlotView& sv, const SchedView& q, int window, cudaStream_t s);
cudaError_t launch_attention_dev(const float* q, const int8_t* kc, const float* ks, const int8_t* vc,
                                 const float* vs, const int32_t* counts, int32_t batch,
                                 int32_t capacity, float* out, cudaStream_t s);
size_t attention_smem_bytes(int32_t capacity, bool ring);
// Fast-numerics attention (attn_fast.cu): scratch holds the split partials.
size_t attention_fast_scratch_bytes(int32_t batch, int32_t capacity);
// row_base (optional, per item): the cache row of (item, KV head 0), head h at + h * capacity, in
// a cache of cache_rows rows of 64 codes (the engine's [slot][layer][head][capacity] blocks);
// without it item b's rows are b * kv_heads * capacity onwards.  `tensor`: the int8-MMA kernel
// where the cache allows it (false: the binary32 CUDA-core kernel).
cudaError_t launch_attention_fast(const float* q, const int8_t* kc, const float* ks, const int8_t* vc,
                                  const float* vs, const int32_t* counts, int32_t batch, int32_t capacity,
                                  float* out, void* scratch, cudaStream_t s, const int64_t* row_base = nullptr,
                                  int64_t cache_rows = 0, bool tensor = true);
// Fast numerics, after launch_attention (part 1) and launch_attention_fast: attention output times
// sigmoid(gate) and the output projection's prepared input, per (item, KV head).
cudaError_t launch_attention_gate(const StepView& st, int n_host, cudaStream_t s);
// Online probe pool (OnlineProbePool.add, runtime.ts:60-90) of the step's collecting items: source 0
// is the scaled embedding (lane 0 after k_embed), source 1 the mean of the lanes (after a layer).
cudaError_t launch_probe_add(const ModelView& m, const SlotView& sv, const StepView& st, int source, int n_host,
                             cudaStream_t s);
// Resets one slot's pool (maximum -inf, denominator 0, weighted 0).
cudaError_t launch_pool_reset(const ModelView& m, const SlotView& sv, int slot, cudaStream_t s);
// confidence() of one slot: sigmoid(denseMatvec(projection, pooled, bias)[0]) into *out (device).
cudaError_t launch_confidence(const ModelView& m, const SlotView& sv, int slot, double* out, cudaStream_t s);
// Records the message returned by needle_cuda_last_error() on this thread (engine.cu).
void set_last_error(const char* msg);
inline void set_last_error(const std::string& msg) { set_last_error(msg.c_str()); }
// Sets the dynamic shared-memory limits of the step kernels on the current device.
cudaError_t configure_step_kernels(int32_t capacity);

}  // namespace needle
