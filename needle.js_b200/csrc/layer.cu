// layer.cu -- fused per-sequence kernels of one decode step (exact numerics).
//
// Each kernel runs one CTA per sequence item (attention: one per item and KV head) and restates a
// contiguous stretch of NeedleRuntime.step (packages/needle.js/src/model/runtime.ts:280-583)
// between two quantised matvecs:
//
//   k_embed     embedding row x sqrt(512) into four lanes; engram n-gram hashes and table-row
//               gathers, prepared for the engram key/value projections (runtime.ts:305-324,
//               788-843)
//   k_layer     [layer > 0]  output-side of layer-1: post-norm, sigmoid(attention gate) residual,
//               Hadamard MLP, delta (runtime.ts:585-611), mHC post routing nextX (509-542)
//               [layer < L]  input-side of layer: rmsUnit lanes, phi matvecs, h_pre, update
//               input, engram injection, input RMSNorm, prepared Q/K/V/gate input (385-441);
//               h_post and the 20-step Sinkhorn routing for the output side
//               [layer == L] final lane mean, RMSNorm, prepared vocabulary input (570-577)
//   k_attention per-head Q/K RMSNorm, RoPE, int8 KV store, attention over the visible window,
//               sigmoid gate, prepared output-projection input (471-504, 679-786)
//   k_finish    selectToken / argmax + logSoftmaxAt (880-899), position advance, scheduler
//               bookkeeping
//
// Every binary64 expression keeps the reference's operand order; sums the reference runs as a
// loop are run by one thread in loop order.  Values the reference stores in a Float32Array are
// rounded with f32().
#include "engine.cuh"

namespace needle {

namespace {

constexpr int kThreads = 512;
constexpr uint32_t kEngramSeed = 0x9e3779b9u;   // runtime.ts:22
constexpr uint32_t kEngramPrime = 0x01000193u;  // runtime.ts:23

__device__ __forceinline__ double silu_d(double v) { return v * sigmoid_d(v); }  // math.ts:12-14

// roundTiesToEven, runtime.ts:901-907.
__device__ __forceinline__ int round_ties_even(double value) {
  const double lower = floor(value);
  const double fraction = value - lower;
  if (fraction < 0.5) return (int)lower;
  if (fraction > 0.5) return (int)lower + 1;
  return (((long long)lower) & 1) == 0 ? (int)lower : (int)lower + 1;
}



// One thread's sequential sum of squares -> 1 / sqrt(s / n + 1e-6) (rmsNorm / rmsUnit).
__device__ __forceinline__ double inverse_rms(const float* v, int n) {
  const double s = sum_squares_seq(v, n);
  return 1.0 / sqrt(s / (double)n + 1e-6);
}

// ------------------------------------------------------------------ k_embed

__global__ void __launch_bounds__(kThreads) k_embed(const ModelView m, const SlotView sv, const StepView st) {
  __shared__ float v[kDim];
  __shared__ uint32_t eidx[kMaxTables];
  __shared__ int evalid[kMaxTables];
  __shared__ int s_token, s_pos;
  const int b = blockIdx.x;
  if (b >= *st.n_items) return;
  const int tid = threadIdx.x;
  DevItem it = st.items[b];
  SeqState* q = sv.seq + it.slot;
  if (tid == 0) {
    // a chunk item's token and position are given (p0 + chunk_index); otherwise the slot's
    const int p = it.chunk_len ? it.position : q->position;
    const int token = it.token >= 0 ? it.token : q->pending;
    s_token = token;
    s_pos = p;
    st.items[b].token = token;
    st.items[b].position = p;
  }
  __syncthreads();
  const int token = s_token, p = s_pos;

  // #engramLookup (runtime.ts:788-818): history = [..., hist[1], hist[0], token].  In a chunk the
  // tokens before this item's come from the earlier items, then from the slot's history.  A
  // resident-session item brings the lookup NeedleRuntime computed (prepareResidentEngrams).
  if (it.flags & kItemEngrams) {
    if (tid < m.n_tables && m.n_sites > 0) {
      eidx[tid] = st.engram_in[(int64_t)b * 2 * kMaxTables + tid] % (uint32_t)m.engram_slots;
      evalid[tid] = st.engram_in[(int64_t)b * 2 * kMaxTables + kMaxTables + tid] != 0u;
    }
  } else if (tid < m.n_tables && m.n_sites > 0) {
    const int heads_per_order = m.n_tables / m.n_orders;
    const int oi = tid / heads_per_order, head = tid - oi * heads_per_order;
    const int order = m.orders[oi];
    uint32_t hash = kEngramSeed * (uint32_t)(oi * heads_per_order + head + 1);
    for (int off = 0; off < order; off++) {
      uint32_t tok;
      if (off > p) tok = 0u;
      else if (off == 0) tok = (uint32_t)token;
      else if (it.chunk_len && off <= it.chunk_index) tok = (uint32_t)st.items[b - off].token;
      else tok = (uint32_t)q->hist[it.chunk_len ? off - it.chunk_index - 1 : off - 1];
      hash = (hash ^ tok) * kEngramPrime;
    }
    hash = hash ^ (hash >> 15);
    eidx[tid] = hash % (uint32_t)m.engram_slots;
    evalid[tid] = (order - 1) <= p;
  }
  __syncthreads();
  if (tid == 0 && !it.chunk_len && !(it.flags & kItemEngrams)) {  // a chunk's history advances in k_finish
    q->hist[2] = q->hist[1];
    q->hist[1] = q->hist[0];
    q->hist[0] = token;
  }

  // Embedding: dequantizeCqRow(embedding, token) * sqrt(512), broadcast to the lanes (305-313).
  // A resident-session item's lanes are beginResidentToken's (built by the runtime the same way).
  if (it.flags & kItemLanes) {
    float* x = sv.x + (int64_t)it.slot * kLaneWidth;
    for (int c = tid; c < kLaneWidth; c += kThreads) x[c] = st.lanes[(int64_t)b * kLaneWidth + c];
    __syncthreads();
  } else {
    const CqMat& E = m.embedding;
    const int c = tid;
    const int g = c / kGroup;
    const uint8_t* rowp = E.packed + (int64_t)token * E.row_bytes;
    const double nrm = norm16(E.norms, (int64_t)token * (E.in_pad / kGroup) + g);
    v[c] = f32(cq_level(m.cb.v, E.bits, cq_index(rowp, E.bits, c)) * nrm);
    __syncthreads();
    fwht_smem(v, kGroup, kDim / kGroup);
    const double inverse_root = 1.0 / sqrt((double)kGroup);
    const float e = f32((double)v[c] * inverse_root);
    const float scaled = f32((double)e * sqrt((double)kDim));
    float* x = it.chunk_len ? st.lanes + (int64_t)b * kLaneWidth : sv.x + (int64_t)it.slot * kLaneWidth;
#pragma unroll
    for (int lane = 0; lane < kLanes; lane++) x[lane * kDim + c] = scaled;
    __syncthreads();
  }

  // Engram gathers (#engramStep, runtime.ts:825-841): concatenated table rows, then the
  // prepareCqActivation of the key/value projections.
  for (int si = 0; si < m.n_sites; si++) {
    const CqMat& T = m.engram_tables[si];
    const int c = tid;
    const int t = c / m.engram_sub, col = c - t * m.engram_sub;
    float val = 0.0f;
    if (evalid[t]) {
      const int64_t row = (int64_t)t * m.engram_slots + eidx[t];
      const uint8_t* rowp = T.packed + row * T.row_bytes;
      const int g = col / kGroup;
      const double nrm = norm16(T.norms, row * (T.in_pad / kGroup) + g);
      val = f32(cq_level(m.cb.v, T.bits, cq_index(rowp, T.bits, col)) * nrm);
    }
    v[c] = val;
    __syncthreads();
    const double inverse_root = 1.0 / sqrt((double)kGroup);
    fwht_smem(v, kGroup, kDim / kGroup);  // dequantizeCqRow's FWHT of each 128-wide table row
    v[c] = f32((double)v[c] * inverse_root);
    __syncthreads();
    fwht_smem(v, kGroup, kDim / kGroup);  // prepareCqActivation of the 512-wide concatenation
    st.prep_engram[((int64_t)b * m.n_sites + si) * kDim + c] = f32((double)v[c] * inverse_root);
    __syncthreads();
  }
}

// ------------------------------------------------------------------ k_layer

struct LayerSmem {
  float xl[kLaneWidth];     // lanes x
  double sq[kLaneWidth];    // terms of a sequential binary64 sum (squares / products)
  double sq2[kDim];         // terms of a second, concurrent sum
  double xd[kLaneWidth];    // prepared phi input in binary64
  float fw[kDim];           // FWHT exchange buffer
  double dots[24 * 16];     // phi (row, group) dots
  double lut[3][16];
  float phi[24];
  float hpre[kLanes], hpost[kLanes], routing[16];
  double red[4];
  double sk[16];            // routing logits (Float64Array of the Float32Array, math.ts:64)
  double part[kThreads / 32];  // block reductions (fast numerics)
};

__device__ void engram_mix(const ModelView& m, const SlotView& sv, const StepView& st, int b,
                           const DevItem& it) {
  const int slot = it.slot, p = it.position;
  // #engramStep ring write and causal tap convolution (runtime.ts:854-873).  The engram position
  // equals the token position: both start at 0 on reset and advance once per step.
  const int c = threadIdx.x;
  const int depth = (m.taps - 1) * m.max_order + 1;
  // In a chunk the ring is not written here (k_finish writes it after the chunk): a tap inside the
  // chunk reads that item's value, a tap before it the ring.
  for (int si = 0; si < m.n_sites; si++) {
    const float now = st.engram_kv[(((int64_t)b * m.n_sites + si) * 2 + 1) * kDim + c];
    float* ring = sv.ring + ((int64_t)slot * m.n_sites + si) * depth * kDim;
    if (!it.chunk_len) ring[(p % depth) * kDim + c] = now;
    float mixed = 0.0f;
    for (int tap = 0; tap < m.taps; tap++) {
      const int back = tap * m.max_order, prev = p - back;
      if (prev < 0) continue;
      float value;
      if (tap == 0) value = now;
      else if (it.chunk_len && back <= it.chunk_index)
        value = st.engram_kv[((((int64_t)(b - back)) * m.n_sites + si) * 2 + 1) * kDim + c];
      else value = ring[(prev % depth) * kDim + c];
      mixed = f32((double)mixed + (double)m.taps_w[((int64_t)si * m.taps + tap) * kDim + c] * (double)value);
    }
    st.engram_val[((int64_t)b * m.n_sites + si) * kDim + c] = mixed;
  }
}

// 20 log-space Sinkhorn iterations on a 4x4 matrix (sinkhorn, math.ts:63-92), run by one full
// warp (lanes 0-3 do the row / column passes); lanes 0-15 then write exp(values) as binary32.
__device__ void sinkhorn4(double* v, float* out, int lane) {
  for (int it = 0; it < 20; it++) {
    if (lane < 4) {
      const int o = lane * 4;
      double mx = v[o];
      for (int c = 1; c < 4; c++) mx = fmax(mx, v[o + c]);
      double sum = 0.0;
      for (int c = 0; c < 4; c++) sum = sum + exp(v[o + c] - mx);
      const double log_sum = log(sum) + mx;
      for (int c = 0; c < 4; c++) v[o + c] = v[o + c] - log_sum;
    }
    __syncwarp();
    if (lane < 4) {
      double mx = v[lane];
      for (int r = 1; r < 4; r++) mx = fmax(mx, v[r * 4 + lane]);
      double sum = 0.0;
      for (int r = 0; r < 4; r++) sum = sum + exp(v[r * 4 + lane] - mx);
      const double log_sum = log(sum) + mx;
      for (int r = 0; r < 4; r++) v[r * 4 + lane] = v[r * 4 + lane] - log_sum;
    }
    __syncwarp();
  }
  if (lane < 16) out[lane] = f32(exp(v[lane]));
}

// Exact dot of one 128-group of a CQ row with binary64 inputs, in the reference's chunk order
// (cq.ts:132-230).  `grp` is the group's 16-byte-aligned packed bytes; `lut` holds the matrix's
// levels as binary64 (ternary: crumbs [0, c, 0, -c]).
template <int BITS>
__device__ double group_dot_t(const uint8_t* __restrict__ grp, const double* lut, const double* xg) {
  constexpr int kWords = (BITS == 4 ? 64 : BITS == 3 ? 48 : 32) / 4;
  uint32_t w[kWords + 1];
#pragma unroll
  for (int q = 0; q < kWords / 4; q++) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(grp) + q);
    w[4 * q] = u.x;
    w[4 * q + 1] = u.y;
    w[4 * q + 2] = u.z;
    w[4 * q + 3] = u.w;
  }
  w[kWords] = 0;
  double dot = 0.0;
  if constexpr (BITS == 2 || BITS == kTernaryBits) {
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const uint32_t byte = (w[i >> 2] >> ((i & 3) * 8)) & 0xffu;
      const double a0 = lut[byte & 3], a1 = lut[(byte >> 2) & 3];
      const double a2 = lut[(byte >> 4) & 3], a3 = lut[(byte >> 6) & 3];
      const double2 x01 = *reinterpret_cast<const double2*>(xg + 4 * i);
      const double2 x23 = *reinterpret_cast<const double2*>(xg + 4 * i + 2);
      double s = a0 * x01.x;
      if constexpr (BITS == 2) {
        s = fma(a1, x01.y, s);
        s = fma(a2, x23.x, s);
        s = fma(a3, x23.y, s);
      } else {
        s = s + a1 * x01.y;
        s = s + a2 * x23.x;
        s = s + a3 * x23.y;
      }
      dot = dot + s;
    }
  } else if constexpr (BITS == 4) {
#pragma unroll
    for (int i = 0; i < 64; i++) {
      const uint32_t byte = (w[i >> 2] >> ((i & 3) * 8)) & 0xffu;
      const double2 x01 = *reinterpret_cast<const double2*>(xg + 2 * i);
      double s = lut[byte & 15] * x01.x;
      s = fma(lut[byte >> 4], x01.y, s);
      dot = dot + s;
    }
  } else {
#pragma unroll
    for (int c = 0; c < kGroup; c++) {
      const int bit = c * 3, wi = bit >> 5, sh = bit & 31;
      uint32_t v = w[wi] >> sh;
      if (sh > 29) v |= w[wi + 1] << (32 - sh);
      dot = fma(lut[v & 7], xg[c], dot);
    }
  }
  return dot;
}

__device__ __forceinline__ double group_dot_exact(const uint8_t* grp, int bits, const double* lut,
                                                  const double* xg) {
  switch (bits) {
    case 2: return group_dot_t<2>(grp, lut, xg);
    case 3: return group_dot_t<3>(grp, lut, xg);
    case 4: return group_dot_t<4>(grp, lut, xg);
    default: return group_dot_t<kTernaryBits>(grp, lut, xg);
  }
}

__device__ __forceinline__ double lut_level(const float* cb28, int bits, int t) {
  if (bits == kTernaryBits) {
    const double coefficient = kTernaryCentroid / sqrt((double)kGroup);
    return (t == 1) ? coefficient : (t == 3) ? -coefficient : 0.0;
  }
  return t < (1 << bits) ? (double)cb28[(bits == 2 ? 0 : bits == 3 ? 4 : 12) + t] : 0.0;
}

// 1 / sqrt(sum / n + 1e-6) of rmsNorm / rmsUnit (math.ts:22-27), the sum being the sequential
// binary64 sum of the staged terms.
__device__ __forceinline__ double inverse_rms_of(const double* terms, int n) {
  return 1.0 / sqrt(sum_seq(terms, n) / (double)n + 1e-6);
}

// Fast numerics: the same sums as binary64 tree reductions over the whole block (every thread
// calls it; `part` is kThreads / 32 doubles of shared scratch).  They differ from the sequential
// sums only in the last bits of a binary64 value (~1e-16 relative).
__device__ __forceinline__ double block_sum(const double* terms, int n, double* part) {
  const int tid = threadIdx.x;
  double v = 0.0;
  for (int i = tid; i < n; i += kThreads) v += terms[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((tid & 31) == 0) part[tid >> 5] = v;
  __syncthreads();
  double t = 0.0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; w++) t += part[w];
  return t;
}

// One binary64 sum of a k_layer phase: the reference's sequential sum by thread 0 (exact
// numerics; result valid in thread 0) or a block reduction (fast; result valid in every thread).
template <bool Fast>
__device__ __forceinline__ double phase_sum(const double* terms, int n, double* part) {
  if constexpr (Fast) return block_sum(terms, n, part);
  else return threadIdx.x == 0 ? sum_seq(terms, n) : 0.0;
}

// Three CTAs per SM (40 registers a thread, a few spilled): with many items per step the CTAs of
// every micro-batch stay resident together (measured: 76.2 k against 72.4 k processed tokens/s at
// two CTAs per SM, 72.6 k at four).
template <bool Fast>
__global__ void __launch_bounds__(kThreads, 3) k_layer(const ModelView m, const SlotView sv, const StepView st,
                                                     int layer) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  LayerSmem& S = *reinterpret_cast<LayerSmem*>(smem_raw);
  const int b = blockIdx.x;
  if (b >= *st.n_items) return;
  const int tid = threadIdx.x;
  const DevItem it = st.items[b];
  const int slot = it.slot;
  float* xg = it.chunk_len ? st.lanes + (int64_t)b * kLaneWidth : sv.x + (int64_t)slot * kLaneWidth;
  {
    float v[kLaneWidth / kThreads];  // all loads in flight before the first store
#pragma unroll
    for (int k = 0; k < kLaneWidth / kThreads; k++) v[k] = xg[tid + k * kThreads];
#pragma unroll
    for (int k = 0; k < kLaneWidth / kThreads; k++) S.xl[tid + k * kThreads] = v[k];
  }
  if (layer == 0 && m.n_sites > 0) engram_mix(m, sv, st, b, it);

  const double inv_root_128 = 1.0 / sqrt((double)kGroup);
  const int c = tid;

  if (layer > 0) {
    // ---------------- output side of layer l = layer - 1
    const int l = layer - 1;
    const float upd = st.update[(int64_t)b * kDim + c];
    const float blk = st.block[(int64_t)b * kDim + c];
    const float projected = st.proj[(int64_t)b * kDim + c];
    if (tid < 20) {
      const float r = st.route[(int64_t)b * 20 + tid];
      if (tid < 4) S.hpost[tid] = r;
      else S.routing[tid - 4] = r;
    }
    S.sq[c] = (double)projected * (double)projected;
    __syncthreads();
    {
      const double sum_ = phase_sum<Fast>(S.sq, kDim, S.part);
      if (tid == 0) S.red[0] = 1.0 / sqrt(sum_ / (double)kDim + 1e-6);
    }
    __syncthreads();
    // #attentionDelta (runtime.ts:585-611)
    const float normalized =
        f32((1.0 + (double)m.post_norm[(int64_t)l * kDim + c]) * (double)projected * S.red[0]);
    const double attention_scale = sigmoid_d((double)m.attn_gate[l]);
    const float after = f32((double)blk + attention_scale * (double)normalized);
    S.sq[c] = (double)after * (double)after;
    __syncthreads();
    {
      const double sum_ = phase_sum<Fast>(S.sq, kDim, S.part);
      if (tid == 0) S.red[1] = 1.0 / sqrt(sum_ / (double)kDim + 1e-6);
    }
    __syncthreads();
    const float pre = f32((1.0 + (double)m.pre_had_norm[(int64_t)l * kDim + c]) * (double)after * S.red[1]);
    // hadamardMlp (math.ts:117-138)
    const double inv_root_h = 1.0 / sqrt((double)kHadamard);
    float v = f32((double)pre * (double)m.d1[(int64_t)l * kHadamard + c]);
    v = fwht_reg(v, S.fw, kHadamard, kThreads);
    v = f32(silu_d((double)v * inv_root_h * (double)m.d2[(int64_t)l * kHadamard + c]));
    v = fwht_reg(v, S.fw, kHadamard, kThreads);
    const float mlp = f32((double)v * inv_root_h * (double)m.d3[(int64_t)l * kHadamard + c]);
    const float delta = f32((double)after + (double)mlp - (double)upd);
    // nextX (runtime.ts:530-541); thread c owns column c of every lane.
    float nx[kLanes];
#pragma unroll
    for (int lane = 0; lane < kLanes; lane++) {
      double sum = 0.0;
#pragma unroll
      for (int src = 0; src < kLanes; src++)
        sum = fma((double)S.routing[lane * kLanes + src], (double)S.xl[src * kDim + c], sum);
      nx[lane] = f32(sum + (double)S.hpost[lane] * (double)delta);
    }
#pragma unroll
    for (int lane = 0; lane < kLanes; lane++) {
      S.xl[lane * kDim + c] = nx[lane];
      xg[lane * kDim + c] = nx[lane];
    }
  }
  __syncthreads();

  if (layer == m.layers) {
    // a chunk's last item leaves its lanes in the slot (what a one-token step leaves there)
    if (it.chunk_len && it.chunk_index == it.chunk_len - 1) {
#pragma unroll
      for (int lane = 0; lane < kLanes; lane++) sv.x[(int64_t)slot * kLaneWidth + lane * kDim + c] = S.xl[lane * kDim + c];
    }
    // ---------------- final: lane mean, RMSNorm, prepared vocabulary input (runtime.ts:570-577)
    double sum = 0.0;
#pragma unroll
    for (int lane = 0; lane < kLanes; lane++) sum = sum + (double)S.xl[lane * kDim + c];
    const float mean = f32(sum / (double)kLanes);
    S.sq[c] = (double)mean * (double)mean;
    __syncthreads();
    {
      const double sum_ = phase_sum<Fast>(S.sq, kDim, S.part);
      if (tid == 0) S.red[0] = 1.0 / sqrt(sum_ / (double)kDim + 1e-6);
    }
    __syncthreads();
    float f = f32((1.0 + (double)m.final_norm[c]) * (double)mean * S.red[0]);
    f = fwht_reg(f, S.fw, kGroup, kThreads);
    st.prep_f[(int64_t)b * kDim + c] = f32((double)f * inv_root_128);
    return;
  }

  // ---------------- input side of layer l
  const int l = layer;
  // rmsUnit(x) over the 2048 lane values (runtime.ts:385)
#pragma unroll
  for (int k = 0; k < kLanes; k++) {
    const double xv = (double)S.xl[c + k * kDim];
    S.sq[c + k * kDim] = xv * xv;
  }
  if (tid >= 32 && tid < 80) {
    const int t = tid - 32, which = t >> 4, lev = t & 15;
    const int bits = which == 0 ? m.phi_pre.bits : which == 1 ? m.phi_post.bits : m.phi_res.bits;
    S.lut[which][lev] = lut_level(m.cb.v, bits, lev);
  }
  __syncthreads();
  {
      const double sum_ = phase_sum<Fast>(S.sq, kLaneWidth, S.part);
      if (tid == 0) S.red[2] = 1.0 / sqrt(sum_ / (double)kLaneWidth + 1e-6);
    }
  __syncthreads();
  // prepareCqActivation of the phi input: FWHT of each 128-group, * 1/sqrt(128)
#pragma unroll
  for (int k = 0; k < kLanes; k++) {
    float nl = f32((double)S.xl[c + k * kDim] * S.red[2]);
    nl = fwht_reg(nl, S.fw, kGroup, kThreads);
    S.xd[c + k * kDim] = (double)f32((double)nl * inv_root_128);
  }
  __syncthreads();

  // phi matvecs (matvecBatch, runtime.ts:386-402): rows 4l..4l+3 of phi_pre / phi_post and
  // 16l..16l+15 of phi_res; 24 rows x 16 groups, one (row, group) per thread.
  // Thread t takes row t % 24 and group t / 24, so a warp reads the binary64 inputs of at most
  // two groups (broadcasts) instead of sixteen (a 16-way bank conflict at the 1 KB group stride).
  constexpr int kPhiGroups = kLaneWidth / kGroup;
  if (tid < 24 * kPhiGroups) {
    const int rr = tid % 24, g = tid / 24;
    const CqMat& M = rr < 4 ? m.phi_pre : rr < 8 ? m.phi_post : m.phi_res;
    const int64_t row = rr < 4 ? (int64_t)l * 4 + rr : rr < 8 ? (int64_t)l * 4 + rr - 4 : (int64_t)l * 16 + rr - 8;
    const int gbytes = M.bits == 4 ? 64 : M.bits == 3 ? 48 : 32;
    S.dots[rr * kPhiGroups + g] = group_dot_exact(M.packed + row * M.row_bytes + g * gbytes, M.bits,
                                                  S.lut[rr < 4 ? 0 : rr < 8 ? 1 : 2], S.xd + g * kGroup);
  }
  __syncthreads();
  if (tid < 24) {
    const int rr = tid;
    const CqMat& M = rr < 4 ? m.phi_pre : rr < 8 ? m.phi_post : m.phi_res;
    const int64_t row = rr < 4 ? (int64_t)l * 4 + rr : rr < 8 ? (int64_t)l * 4 + rr - 4 : (int64_t)l * 16 + rr - 8;
    double nrm[kPhiGroups];
#pragma unroll
    for (int g = 0; g < kPhiGroups; g++) nrm[g] = norm16(M.norms, row * kPhiGroups + g);
    double total = 0.0;
#pragma unroll
    for (int g = 0; g < kPhiGroups; g++) total = total + nrm[g] * S.dots[rr * kPhiGroups + g];
    S.phi[rr] = f32(total);
  }
  __syncthreads();
  const int own = l % kLanes;
  if (tid < 4) {
    // h_pre (runtime.ts:404-413)
    const double offset = tid == own ? 4.0 : -4.0;
    S.hpre[tid] = f32(sigmoid_d((double)m.a_pre[l] * (double)S.phi[tid] +
                                (double)m.b_pre[(int64_t)l * 4 + tid] + offset));
  } else if (tid < 8) {
    // h_post (runtime.ts:512-522)
    const int lane = tid - 4;
    const double offset = lane == own ? 0.0 : -4.0;
    S.hpost[lane] = f32(2.0 * sigmoid_d((double)m.a_post[l] * (double)S.phi[tid] +
                                        (double)m.b_post[(int64_t)l * 4 + lane] + offset));
  } else if (tid < 24) {
    // routing logits (runtime.ts:523-528), Float32Array then Float64Array(logits)
    const int i = tid - 8;
    S.sk[i] = (double)f32((double)m.a_res[l] * (double)S.phi[tid] + (double)m.b_res[(int64_t)l * 16 + i]);
  }
  __syncthreads();

  // updateInput (runtime.ts:414-420)
  double sum = 0.0;
#pragma unroll
  for (int lane = 0; lane < kLanes; lane++) sum = fma((double)S.hpre[lane], (double)S.xl[lane * kDim + c], sum);
  const float upd = f32(sum);
  float blk = upd;
  int site = -1;
  for (int k = 0; k < m.n_sites; k++)
    if (m.sites[k] == l) site = k;
  if (site >= 0) {
    // engram injection (runtime.ts:423-438): rmsUnit of both vectors, then their dot product
    const float key = st.engram_kv[(((int64_t)b * m.n_sites + site) * 2) * kDim + c];
    S.sq[c] = (double)upd * (double)upd;
    S.sq2[c] = (double)key * (double)key;
    __syncthreads();
    if constexpr (Fast) {
      const double a_ = block_sum(S.sq, kDim, S.part);
      const double b_ = block_sum(S.sq2, kDim, S.part);
      if (tid == 0) {
        S.red[0] = 1.0 / sqrt(a_ / (double)kDim + 1e-6);
        S.red[1] = 1.0 / sqrt(b_ / (double)kDim + 1e-6);
      }
    } else {
      if (tid == 0) S.red[0] = inverse_rms_of(S.sq, kDim);
      if (tid == 32) S.red[1] = inverse_rms_of(S.sq2, kDim);
    }
    __syncthreads();
    const float ni = f32((double)upd * S.red[0]);
    const float nk = f32((double)key * S.red[1]);
    S.sq[c] = (double)ni * (double)nk;
    __syncthreads();
    {
      const double dot_ = phase_sum<Fast>(S.sq, kDim, S.part);
      if (tid == 0) S.red[3] = sigmoid_d(dot_ / sqrt((double)kDim));
    }
    __syncthreads();
    const float value = st.engram_val[((int64_t)b * m.n_sites + site) * kDim + c];
    blk = f32((double)upd + S.red[3] * (double)value);
  }
  st.update[(int64_t)b * kDim + c] = upd;
  st.block[(int64_t)b * kDim + c] = blk;
  S.sq[c] = (double)blk * (double)blk;
  __syncthreads();
  {
      const double sum_ = phase_sum<Fast>(S.sq, kDim, S.part);
      if (tid == 0) S.red[0] = 1.0 / sqrt(sum_ / (double)kDim + 1e-6);
    }
  __syncthreads();
  // rmsNorm(blockInput, normInput) then prepareCqActivation for Q/K/V/gate (runtime.ts:441, 465)
  float a = f32((1.0 + (double)m.norm_input[(int64_t)l * kDim + c]) * (double)blk * S.red[0]);
  a = fwht_reg(a, S.fw, kGroup, kThreads);
  st.prep_a[(int64_t)b * kDim + c] = f32((double)a * inv_root_128);
  // h_post and the routing logits; k_route turns the logits into the Sinkhorn routing matrix
  // while the attention half of the layer runs.
  if (tid < 4) st.route[(int64_t)b * 20 + tid] = S.hpost[tid];
  else if (tid < 20) st.route[(int64_t)b * 20 + tid] = (float)S.sk[tid - 4];
}

// Sinkhorn routing of one item (runtime.ts:523-529): one warp per item, in place on route[4..19].
__global__ void __launch_bounds__(32) k_route(const StepView st) {
  __shared__ double v[16];
  __shared__ float out[16];
  const int b = blockIdx.x;
  if (b >= *st.n_items) return;
  const int lane = threadIdx.x;
  float* r = st.route + (int64_t)b * 20 + 4;
  if (lane < 16) v[lane] = (double)r[lane];
  __syncwarp();
  sinkhorn4(v, out, lane);
  __syncwarp();
  if (lane < 16) r[lane] = out[lane];
}

// ------------------------------------------------------------------ k_attention

constexpr int kAttnThreads = 128;

// Cache addressing of the engine (ring = window/sink slots) or of the isolated operator
// (contiguous positions 0..count-1).
struct CacheRef {
  const int8_t* kc;
  const int8_t* vc;
  const float* ks;
  const float* vs;
};

// Attention of query heads 2h, 2h+1 over one KV head (the #attention loops of runtime.ts:732-784
// for one kvHead).  q: smem [2][64] (binary32 values widened to binary64); e: smem binary64 [2][count]; tile: smem staging
// area (kAttnTile value rows + scales + weights); slot_of(t) maps the t-th visible position to its
// cache row.  Leaves the gated outputs in out[2][64] (smem).
constexpr int kAttnTile = 256;
constexpr int kAttnSc = 1, kAttnMix = 1, kAttnMc = 0;  // attend_pair variant of the engine (measured best)
constexpr size_t kAttnTileBytes = kAttnTile * (kHeadDim + 2 * 8);  // codes, 2 x weight*scale

// softmaxInPlace (math.ts:46-60) of both heads' binary32 scores e[2][count]: max (order-free),
// exp in parallel, sequential total; leaves red[4 + h] = 1 / total (0 for an empty row).
__device__ __forceinline__ void softmax_pair(double* e, int count, double* red) {
  const int tid = threadIdx.x;
  {
    const int hh = tid >> 6, lane64 = tid & 63;
    double mx = -INFINITY;
    for (int t = lane64; t < count; t += 64) mx = fmax(mx, e[hh * count + t]);
    for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = fmax(red[hh * 2], red[hh * 2 + 1]);
    __syncthreads();
    for (int t = lane64; t < count; t += 64) e[hh * count + t] = exp(e[hh * count + t] - mx);
    __syncthreads();
    if (lane64 == 0) {  // sequential total; the values are read eight at a time ahead of the adds
      const double* eh = e + hh * count;
      double total = 0.0;
      int t = 0;
      for (; t + 8 <= count; t += 8) {
        double v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = eh[t + k];
#pragma unroll
        for (int k = 0; k < 8; k++) total = total + v[k];
      }
      for (; t < count; t++) total = total + eh[t];
      red[4 + hh] = total > 0.0 ? 1.0 / total : 0.0;
    }
    __syncthreads();
  }
}

// Widened int8 code: through the FP64 add pipe (Mc 0, int_to_double_exact) or the conversion unit.
template <int Mc>
__device__ __forceinline__ double code_d(int c) {
  if constexpr (Mc == 0) return int_to_double_exact(c);
  else return (double)c;
}
// round32 of one value-mix step: on the FP64 add pipe (R 0) or through the conversion unit (R 1).
template <int R>
__device__ __forceinline__ double round32_r(double v) {
  if constexpr (R == 0) return round32_add(v);
  else return round32_cvt(v);
}

// 16-byte asynchronous global -> shared copy (L2 only); completes at cp_async_wait.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Attention variants (all bit-identical): Sc = key-code widening (0 add pipe, 1 conversion unit);
// Mix = value-mix layout (0: one chain per thread, conversion rounding; 1: threads 0-63 run both
// heads' chains of one element, head 0 rounding on the add pipe and head 1 by conversion; 2: both on
// the add pipe; 3: both by conversion); Mc = value-code widening.  The engine's choice (kAttnSc,
// kAttnMix, kAttnMc) balances the FP64 pipe against the conversion unit: it measured fastest of the
// eight combinations at 256 items with full windows (1.15 against 1.26 ms per step for 0, 0, 0).
template <int Sc, int Mix, int Mc, class SlotOf>
__device__ void attend_pair(const CacheRef& C, int count, SlotOf slot_of, const double* q2, double* e,
                            unsigned char* tile, const float* gate, float* out, double* red) {
  const int tid = threadIdx.x;
  int8_t* vt = reinterpret_cast<int8_t*>(tile);                                 // [tile][64] value codes
  double2* wvt = reinterpret_cast<double2*>(tile + kAttnTile * kHeadDim);       // [tile] (head 0, head 1)
  // The first tile of value rows is fetched asynchronously while the scores and the softmax run.
  const int n0 = min(kAttnTile, count);
  for (int k = tid; k < n0 * 4; k += kAttnThreads)
    cp_async16(vt + (k >> 2) * kHeadDim + (k & 3) * 16, C.vc + (int64_t)slot_of(k >> 2) * kHeadDim + (k & 3) * 16);
  // scores[t] = f32((sum_i q_i * code_i * keyScale) / 8)  (runtime.ts:736-757), two positions per
  // thread at a time (four independent sums).  q * code * keyScale: q * code is exact in binary64 and
  // so is code * keyScale, so (q * code) * keyScale and q * (code * keyScale) are both the one rounding
  // of the same real product; the second form shares code * keyScale between the two heads.
  const double inverse_root = 1.0 / sqrt((double)kHeadDim);
  for (int t0 = tid; t0 < count; t0 += 2 * kAttnThreads) {
    const int t1 = t0 + kAttnThreads;
    const bool two = t1 < count;
    const int s0 = slot_of(t0), s1 = two ? slot_of(t1) : s0;
    const double ks0 = (double)C.ks[s0], ks1 = (double)C.ks[s1];
    const uint4* k0 = reinterpret_cast<const uint4*>(C.kc + (int64_t)s0 * kHeadDim);
    const uint4* k1 = reinterpret_cast<const uint4*>(C.kc + (int64_t)s1 * kHeadDim);
    uint4 u0[4], u1[4];
#pragma unroll
    for (int w4 = 0; w4 < 4; w4++) {
      u0[w4] = __ldg(k0 + w4);
      u1[w4] = __ldg(k1 + w4);
    }
    double a0 = 0.0, a1 = 0.0, b0 = 0.0, b1 = 0.0;
#pragma unroll
    for (int w4 = 0; w4 < 4; w4++) {
      const uint32_t wa[4] = {u0[w4].x, u0[w4].y, u0[w4].z, u0[w4].w};
      const uint32_t wb[4] = {u1[w4].x, u1[w4].y, u1[w4].z, u1[w4].w};
#pragma unroll
      for (int k = 0; k < 16; k++) {
        const int i = w4 * 16 + k;
        const double2 qq = reinterpret_cast<const double2*>(q2)[i];
        const double ca = code_d<Sc>((int)(int8_t)((wa[k >> 2] >> ((k & 3) * 8)) & 0xff)) * ks0;
        const double cb = code_d<Sc>((int)(int8_t)((wb[k >> 2] >> ((k & 3) * 8)) & 0xff)) * ks1;
        a0 = a0 + qq.x * ca;
        a1 = a1 + qq.y * ca;
        b0 = b0 + qq.x * cb;
        b1 = b1 + qq.y * cb;
      }
    }
    e[t0] = round32_cvt(a0 * inverse_root);
    e[count + t0] = round32_cvt(a1 * inverse_root);
    if (two) {
      e[t1] = round32_cvt(b0 * inverse_root);
      e[count + t1] = round32_cvt(b1 * inverse_root);
    }
  }
  __syncthreads();
  softmax_pair(e, count, red);
  // output[i] += weight * code * valueScale, sequentially in t with binary32 storage (760-782).
  // weight * code * valueScale == code * (weight * valueScale): weight (binary32) * valueScale
  // (binary32) is exact in binary64, and weight * code is exact too, so both orders are one
  // rounding of the same real product.
  const int i = tid & 63;
  double o0 = 0.0, o1 = 0.0;  // binary32 values, kept widened (rounded after every step)
  for (int t0 = 0; t0 < count; t0 += kAttnTile) {
    const int n = min(kAttnTile, count - t0);
    if (t0 > 0) {
      for (int k = tid; k < n * 4; k += kAttnThreads)
        cp_async16(vt + (k >> 2) * kHeadDim + (k & 3) * 16,
                   C.vc + (int64_t)slot_of(t0 + (k >> 2)) * kHeadDim + (k & 3) * 16);
    }
    for (int t = tid; t < n; t += kAttnThreads) {
      const double vs = (double)C.vs[slot_of(t0 + t)];
      const double w0 = round32_cvt(round32_cvt(e[t0 + t]) * red[4]);
      const double w1 = round32_cvt(round32_cvt(e[count + t0 + t]) * red[5]);
      wvt[t] = make_double2(w0 * vs, w1 * vs);
    }
    cp_async_wait_all();
    __syncthreads();
    if constexpr (Mix == 0) {
      const int hh = tid >> 6;
      double o = hh ? o1 : o0;
#pragma unroll 8
      for (int t = 0; t < n; t++) {
        const double2 w = wvt[t];
        o = round32_cvt(o + code_d<Mc>(vt[t * kHeadDim + i]) * (hh ? w.y : w.x));
      }
      if (hh) o1 = o; else o0 = o;
    } else if (tid < 64) {
      constexpr int R0 = Mix == 3 ? 1 : 0, R1 = Mix == 2 ? 0 : 1;
#pragma unroll 8
      for (int t = 0; t < n; t++) {
        const double c = code_d<Mc>(vt[t * kHeadDim + i]);
        const double2 w = wvt[t];
        o0 = round32_r<R0>(o0 + c * w.x);
        o1 = round32_r<R1>(o1 + c * w.y);
      }
    }
    __syncthreads();
  }
  // attentionOutput * sigmoid(gate) (runtime.ts:503-504)
  if constexpr (Mix == 0) {
    const int hh = tid >> 6;
    const double o = hh ? o1 : o0;
    out[hh * kHeadDim + i] = gate ? f32(o * sigmoid_d((double)gate[hh * kHeadDim + i])) : (float)o;
  } else if (tid < 64) {
    out[i] = gate ? f32(o0 * sigmoid_d((double)gate[i])) : (float)o0;
    out[kHeadDim + i] = gate ? f32(o1 * sigmoid_d((double)gate[kHeadDim + i])) : (float)o1;
  }
  __syncthreads();
}

// attend_pair over the float32 cache (runtime.ts:744-748, 768-772): keys and values are read as
// stored, and query * key and weight * value are exact binary64 products, so each accumulation is
// one fused multiply-add.  The weights are formed once per position in e (binary32 values), and
// the value chain reads the cache directly (the two heads share each row).  q is [i][head].
template <class SlotOf>
__device__ void attend_pair_f32(const float* kf, const float* vf, int count, SlotOf slot_of, const double* q,
                                double* e, const float* gate, float* out, double* red) {
  const int tid = threadIdx.x;
  const double inverse_root = 1.0 / sqrt((double)kHeadDim);
  for (int t = tid; t < count; t += kAttnThreads) {
    const float4* kr = reinterpret_cast<const float4*>(kf + (int64_t)slot_of(t) * kHeadDim);
    double d0 = 0.0, d1 = 0.0;
#pragma unroll 4
    for (int w4 = 0; w4 < kHeadDim / 4; w4++) {
      const float4 k4 = __ldg(kr + w4);
      const float kk[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
      for (int c = 0; c < 4; c++) {
        d0 = fma(q[(4 * w4 + c) * 2], (double)kk[c], d0);
        d1 = fma(q[(4 * w4 + c) * 2 + 1], (double)kk[c], d1);
      }
    }
    e[t] = round32_cvt(d0 * inverse_root);
    e[count + t] = round32_cvt(d1 * inverse_root);
  }
  __syncthreads();
  softmax_pair(e, count, red);
  for (int k = tid; k < 2 * count; k += kAttnThreads) e[k] = round32_cvt(round32_cvt(e[k]) * red[4 + k / count]);
  __syncthreads();
  const int hh = tid >> 6, i = tid & 63;
  const double* w = e + hh * count;
  double o = 0.0;  // a binary32 value, kept widened
#pragma unroll 4
  for (int t = 0; t < count; t++) o = round32_cvt(fma(w[t], (double)__ldg(vf + (int64_t)slot_of(t) * kHeadDim + i), o));
  out[hh * kHeadDim + i] = gate ? f32(o * sigmoid_d((double)gate[hh * kHeadDim + i])) : (float)o;
  __syncthreads();
}

// part 0: append this item's K/V, then attend; part 1: append only (fast numerics attends with
// the fast attention kernel); part 2: attend only; part 3: append the chunk items only; part 4: the chunk items
// attend, every other item appends and attends.  A step that holds chunk items runs parts 3 and 4:
// every item of a chunk appends before any of them attends.
template <int Sc, int Mix, int Mc>
__global__ void __launch_bounds__(kAttnThreads) k_attention(const ModelView m, const SlotView sv,
                                                           const StepView st, int l, int part) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float qv[2 * kHeadDim], kv[kHeadDim], vv[kHeadDim], gt[2 * kHeadDim], outv[2 * kHeadDim];
  __shared__ double red[8];
  __shared__ double amax[8];
  const int b = blockIdx.x, h = blockIdx.y;
  if (b >= *st.n_items) return;
  const int tid = threadIdx.x;
  const DevItem it = st.items[b];
  const bool chunk_item = it.chunk_len > 0;
  if (part == 3 && !chunk_item) return;
  const bool append = part == 0 || part == 1 || part == 3 || (part == 4 && !chunk_item);
  const bool attend = part == 0 || part == 2 || part == 4;
  const int slot = it.slot, p = it.position;
  const SeqState seq = sv.seq[slot];
  const float* qkvg = st.qkvg + (int64_t)b * 1536;
  qv[tid] = qkvg[2 * h * kHeadDim + tid];
  gt[tid] = qkvg[1024 + 2 * h * kHeadDim + tid];
  if (tid < kHeadDim) {
    kv[tid] = qkvg[512 + h * kHeadDim + tid];
    vv[tid] = qkvg[768 + h * kHeadDim + tid];
  }
  __syncthreads();
  // #rmsNormSlice on the two query heads and the key head (runtime.ts:471-486, 647-657)
  if (tid == 0) red[0] = inverse_rms(qv, kHeadDim);
  if (tid == 32) red[1] = inverse_rms(qv + kHeadDim, kHeadDim);
  if (tid == 64) red[2] = inverse_rms(kv, kHeadDim);
  __syncthreads();
  {
    const int i = tid & 63;
    qv[tid] = f32((1.0 + (double)m.query_norm[(int64_t)l * kHeadDim + i]) * (double)qv[tid] * red[tid >> 6]);
    if (tid < kHeadDim) kv[tid] = f32((1.0 + (double)m.key_norm[(int64_t)l * kHeadDim + tid]) * (double)kv[tid] * red[2]);
  }
  __syncthreads();
  // applyRope (math.ts:94-115) with host-computed binary64 cos/sin of position * theta^(-2d/64)
  if (tid < 96) {
    const int which = tid >> 5, d = tid & 31;
    float* vec = which < 2 ? qv + which * kHeadDim : kv;
    const double cs = m.rope_cos[(int64_t)p * 32 + d], sn = m.rope_sin[(int64_t)p * 32 + d];
    const double first = vec[d], second = vec[d + 32];
    vec[d] = f32(first * cs - second * sn);
    vec[d + 32] = f32(second * cs + first * sn);
  }
  __syncthreads();
  // #storeKV (runtime.ts:679-717): abs-max (order-free), scale = max / 127, codes = RNE(x / scale).
  const int window = m.kv_window;
  const int sink = seq.sink;
  auto kv_slot = [&](int pos) {
    if (window == 0) return pos;
    if (pos < sink) return pos;
    return sink + (pos - sink) % window;
  };
  const int64_t head_base = (((int64_t)slot * sv.layers + l) * kKvHeads + h) * sv.capacity;
  if (append) {
    double mk = 0.0, mv = 0.0;
    if (tid < kHeadDim) {
      mk = fabs((double)kv[tid]);
      mv = fabs((double)vv[tid]);
    }
    for (int o = 16; o > 0; o >>= 1) {
      mk = fmax(mk, __shfl_xor_sync(0xffffffffu, mk, o));
      mv = fmax(mv, __shfl_xor_sync(0xffffffffu, mv, o));
    }
    if ((tid & 31) == 0) {
      amax[tid >> 5] = mk;
      amax[4 + (tid >> 5)] = mv;
    }
    __syncthreads();
    const double key_scale = fmax(1e-12, fmax(amax[0], amax[1])) / 127.0;
    const double value_scale = fmax(1e-12, fmax(amax[4], amax[5])) / 127.0;
    const int sl = kv_slot(p);
    if (sv.kv_f32) {  // float32 cache: values as given, scales 1 (runtime.ts:686-693)
      if (tid < kHeadDim) {
        sv.kf[(head_base + sl) * kHeadDim + tid] = kv[tid];
        sv.vf[(head_base + sl) * kHeadDim + tid] = vv[tid];
      }
      if (tid == 0) {
        sv.kscale[head_base + sl] = 1.0f;
        sv.vscale[head_base + sl] = 1.0f;
      }
    } else {
      if (tid < kHeadDim) {
        sv.kcodes[(head_base + sl) * kHeadDim + tid] = (int8_t)round_ties_even((double)kv[tid] / key_scale);
        sv.vcodes[(head_base + sl) * kHeadDim + tid] = (int8_t)round_ties_even((double)vv[tid] / value_scale);
      }
      if (tid == 0) {
        sv.kscale[head_base + sl] = f32(key_scale);
        sv.vscale[head_base + sl] = f32(value_scale);
      }
    }
    __syncthreads();
  }
  if (!attend) {
    // fast numerics attends with the fast attention kernel next (binary32 or int8-MMA): leave it the
    // rotated queries, the visible count (slots 0 .. count-1 of the ring hold exactly the visible
    // positions) and the cache row
    if (part == 1 && st.qrope) {
      st.qrope[(int64_t)b * kDim + 2 * h * kHeadDim + tid] = qv[tid];
      if (h == 0 && tid == 0) {
        const int prefix = min(sink, p + 1);
        const int recent_low = window > 0 ? max(prefix, p + 1 - window) : prefix;
        st.attn_count[b] = prefix + (p - recent_low + 1);
        st.attn_row[b] = head_base;  // KV head 0 of this item's (slot, layer)
      }
    }
    return;
  }
  // Visible positions (runtime.ts:723-728): [0, prefix) U [recentLow, p].
  const int prefix = min(sink, p + 1);
  const int recent_low = window > 0 ? max(prefix, p + 1 - window) : prefix;
  const int count = prefix + (p - recent_low + 1);
  unsigned char* tile = smem_raw;
  double* e = reinterpret_cast<double*>(smem_raw + kAttnTileBytes);
  auto slot_of = [&](int t) { return kv_slot(t < prefix ? t : recent_low + (t - prefix)); };
  __shared__ __align__(16) double qd[2 * kHeadDim];  // [i][head]
  qd[(tid & 63) * 2 + (tid >> 6)] = (double)qv[tid];
  __syncthreads();
  if (sv.kv_f32) {
    attend_pair_f32(sv.kf + head_base * kHeadDim, sv.vf + head_base * kHeadDim, count, slot_of, qd, e, gt, outv,
                    red);
  } else {
    CacheRef C{sv.kcodes + head_base * kHeadDim, sv.vcodes + head_base * kHeadDim, sv.kscale + head_base,
               sv.vscale + head_base};
    attend_pair<Sc, Mix, Mc>(C, count, slot_of, qd, e, tile, gt, outv, red);
  }
  // prepareCqActivation of the output projection: heads 2h, 2h+1 are exactly input group h.
  fwht_smem(outv, kGroup, 1);
  st.prep_o[(int64_t)b * kDim + h * kGroup + tid] = f32((double)outv[tid] * (1.0 / sqrt((double)kGroup)));
}

// Fast numerics: attentionOutput * sigmoid(gate) (runtime.ts:503-504) of the fast attention's output,
// and the output projection's prepared input (heads 2h, 2h+1 are input group h).
__global__ void __launch_bounds__(kAttnThreads) k_attention_gate(const StepView st) {
  __shared__ float outv[2 * kHeadDim];
  const int b = blockIdx.x, h = blockIdx.y;
  if (b >= *st.n_items) return;
  const int tid = threadIdx.x;
  const float o = st.attn_out[(int64_t)b * kDim + 2 * h * kHeadDim + tid];
  const float g = st.qkvg[(int64_t)b * 1536 + 1024 + 2 * h * kHeadDim + tid];
  outv[tid] = f32((double)o * sigmoid_d((double)g));
  __syncthreads();
  fwht_smem(outv, kGroup, 1);
  st.prep_o[(int64_t)b * kDim + h * kGroup + tid] = f32((double)outv[tid] * (1.0 / sqrt((double)kGroup)));
}

// Isolated decode attention (needle_cuda_attention_dev): kvWindow = 0, positions 0..count-1,
// query already normalised and rotated, no gate.
__global__ void __launch_bounds__(kAttnThreads) k_attention_dev(const float* __restrict__ q,
                                                               const int8_t* kc, const float* ks,
                                                               const int8_t* vc, const float* vs,
                                                               const int32_t* counts, int32_t capacity,
                                                               float* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ __align__(16) double qd[2 * kHeadDim];  // [i][head]
  __shared__ float outv[2 * kHeadDim];
  __shared__ double red[8];
  const int b = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x;
  qd[(tid & 63) * 2 + (tid >> 6)] = (double)q[(int64_t)b * kHeads * kHeadDim + 2 * h * kHeadDim + tid];
  __syncthreads();
  const int count = min(max(counts[b], 0), capacity);
  const int64_t head_base = ((int64_t)b * kKvHeads + h) * capacity;
  CacheRef C{kc + head_base * kHeadDim, vc + head_base * kHeadDim, ks + head_base, vs + head_base};
  unsigned char* tile = smem_raw;
  double* e = reinterpret_cast<double*>(smem_raw + kAttnTileBytes);
  auto slot_of = [](int t) { return t; };
  attend_pair<kAttnSc, kAttnMix, kAttnMc>(C, count, slot_of, qd, e, tile, nullptr, outv, red);
  out[(int64_t)b * kHeads * kHeadDim + 2 * h * kHeadDim + tid] = outv[tid];
}

// ------------------------------------------------------------------ k_finish

constexpr int kFinishThreads = 256;

__device__ __forceinline__ bool better(float v, int k, float bv, int bk) {
  // strictly greater wins; equal values keep the earlier candidate (runtime.ts:889-896)
  return v > bv || (v == bv && k < bk);
}

__global__ void __launch_bounds__(kFinishThreads) k_finish(const ModelView m, const SlotView sv,
                                                         const StepView st, const SchedView q,
                                                         int has_sched) {
  __shared__ float sv_[kFinishThreads / 32];
  __shared__ int sk_[kFinishThreads / 32];
  __shared__ double sd_[kFinishThreads / 32];
  __shared__ int s_id;
  __shared__ double s_max;
  const int b = blockIdx.x;
  if (b >= *st.n_items) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const DevItem it = st.items[b];
  SeqState* seq = sv.seq + it.slot;
  const bool selecting = b < *st.n_select && it.select;
  int chosen = -1;
  if (selecting) {
    const float* lg = st.logits + (int64_t)b * m.vocab;
    // masked argmax / argmax (selectToken, runtime.ts:880-899; argmax, math.ts:140-151).  An id list
    // is ascending, so its earliest best entry is its lowest best id, as with a bit mask over ids.
    const bool masked = it.allowed_count >= 0;
    const uint32_t* mask =
        it.allowed_count == kAllowedMask ? st.masks + (int64_t)it.allowed_offset * st.mask_words : nullptr;
    const int n = masked ? it.allowed_count : m.vocab;
    float bv = -INFINITY;
    int bk = 0x7fffffff;
    for (int k = tid; k < n; k += kFinishThreads) {
      if (mask && !((mask[k >> 5] >> (k & 31)) & 1u)) continue;
      const int id = masked ? (int)st.allowed[it.allowed_offset + k] : k;
      const float v = lg[id];
      if (bk == 0x7fffffff || v > bv) {  // ascending k: strict > keeps the earliest
        bv = v;
        bk = k;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int ok = __shfl_xor_sync(0xffffffffu, bk, o);
      if (ok != 0x7fffffff && (bk == 0x7fffffff || better(ov, ok, bv, bk))) {
        bv = ov;
        bk = ok;
      }
    }
    if (lane == 0) {
      sv_[warp] = bv;
      sk_[warp] = bk;
    }
    __syncthreads();
    if (tid == 0) {
      float v0 = sv_[0];
      int k0 = sk_[0];
      for (int w = 1; w < kFinishThreads / 32; w++)
        if (sk_[w] != 0x7fffffff && (k0 == 0x7fffffff || better(sv_[w], sk_[w], v0, k0))) {
          v0 = sv_[w];
          k0 = sk_[w];
        }
      if (k0 == 0x7fffffff) k0 = 0;  // an empty mask: the host refuses those before the step
      s_id = masked ? (int)st.allowed[it.allowed_offset + k0] : k0;
    }
    // logSoftmaxAt (math.ts:153-160): max, then sum of exp(logit - max) as a binary64 tree sum.
    double mx = -INFINITY;
    for (int k = tid; k < m.vocab; k += kFinishThreads) mx = fmax(mx, (double)lg[k]);
    for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) sd_[warp] = mx;
    __syncthreads();
    if (tid == 0) {
      double v = sd_[0];
      for (int w = 1; w < kFinishThreads / 32; w++) v = fmax(v, sd_[w]);
      s_max = v;
    }
    __syncthreads();
    double sum = 0.0;
    for (int k = tid; k < m.vocab; k += kFinishThreads) sum += exp((double)lg[k] - s_max);
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) sd_[warp] = sum;
    __syncthreads();
    if (tid == 0) {
      double total = 0.0;
      for (int w = 0; w < kFinishThreads / 32; w++) total += sd_[w];
      chosen = s_id;
      st.out_id[b] = chosen;
      st.out_logprob[b] = (double)lg[chosen] - s_max - log(total);
      seq->pending = chosen;
    }
  }
  if (it.chunk_len) {
    // a prefill chunk: the engram values of its last ring-depth items enter the ring now that every
    // item has read its taps (k_layer, layer 0), and the slot advances once, past the last item,
    // with the chunk's last three tokens as its history
    const int n = it.chunk_len, ci = it.chunk_index;
    if (m.n_sites > 0) {
      const int depth = (m.taps - 1) * m.max_order + 1;
      if (ci >= n - depth) {
        for (int si = 0; si < m.n_sites; si++) {
          float* ring = sv.ring + ((int64_t)it.slot * m.n_sites + si) * depth * kDim;
          for (int c = tid; c < kDim; c += kFinishThreads)
            ring[(it.position % depth) * kDim + c] = st.engram_kv[(((int64_t)b * m.n_sites + si) * 2 + 1) * kDim + c];
        }
      }
    }
    if (tid == 0 && ci == n - 1) {
      int h[3];
#pragma unroll
      for (int k = 0; k < 3; k++) h[k] = k <= ci ? st.items[b - k].token : seq->hist[k - ci - 1];
      seq->hist[0] = h[0];
      seq->hist[1] = h[1];
      seq->hist[2] = h[2];
      seq->position = it.position + 1;
      if (has_sched) atomicAdd(reinterpret_cast<unsigned long long*>(q.processed), (unsigned long long)n);
    }
    return;
  }
  if (tid == 0) {
    seq->position = it.position + 1;
    if (has_sched) {
      atomicAdd(reinterpret_cast<unsigned long long*>(q.processed), 1ull);
      if (selecting) {
        atomicAdd(reinterpret_cast<unsigned long long*>(q.generated), 1ull);
        q.gen_ids[q.gen_offsets[seq->seq_id] + seq->gen_done] = chosen;
        const int done = seq->gen_done + 1;
        seq->gen_done = done;
        if (done >= seq->gen_target) {
          q.last_ids[seq->seq_id] = chosen;
          atomicAdd(q.finished, 1);
          seq->busy = 0;
        }
      }
    }
  }
}

// ------------------------------------------------------------------ confidence probe pool

// OnlineProbePool.add (runtime.ts:60-90) for the step's collecting items, one CTA of kDim threads
// per item.  cell: the scaled embedding (source 0: lane 0 right after k_embed, which holds it) or
// the mean of the lanes (source 1: f32(sum of lanes / lanes), runtime.ts:551-560).  score_p =
// (sum_i cell_i * probe_pi) / sqrt(d) sequentially in i (exact products: fused); then the pool's
// online softmax update in binary64 with separate roundings, as the reference writes it.
__global__ void __launch_bounds__(kDim) k_probe_add(const ModelView m, const SlotView sv, const StepView st,
                                                    int source) {
  __shared__ double cell[kDim];
  __shared__ double score[kMaxProbes];
  const int b = blockIdx.x;
  if (b >= *st.n_items) return;
  const int slot = st.items[b].slot;
  if (!sv.seq[slot].collect) return;
  const int tid = threadIdx.x, P = m.probe_count;
  const float* x = sv.x + (int64_t)slot * kLaneWidth;
  if (source == 0) {
    cell[tid] = (double)x[tid];
  } else {
    double sum = 0.0;
#pragma unroll
    for (int lane = 0; lane < kLanes; lane++) sum = sum + (double)x[lane * kDim + tid];
    cell[tid] = round32_cvt(sum / (double)kLanes);
  }
  __syncthreads();
  if (tid < P) {
    const float* pr = m.probes + (int64_t)tid * kDim;
    double sc = 0.0;
    for (int i = 0; i < kDim; i++) sc = fma(cell[i], (double)__ldg(pr + i), sc);
    score[tid] = sc * (1.0 / sqrt((double)kDim));
  }
  __syncthreads();
  double* mx = sv.pool_max + (int64_t)slot * P;
  double* den = sv.pool_den + (int64_t)slot * P;
  double* w = sv.pool_w + (int64_t)slot * P * kDim;
  for (int p = 0; p < P; p++) {
    const double sc = score[p], prev = mx[p];
    double* wp = w + (int64_t)p * kDim + tid;
    if (sc <= prev) {
      const double weight = exp(sc - prev);
      *wp = *wp + weight * cell[tid];
      if (tid == 0) den[p] = den[p] + weight;
    } else {
      const double old = isfinite(prev) ? exp(prev - sc) : 0.0;
      *wp = *wp * old + cell[tid];
      if (tid == 0) den[p] = den[p] * old + 1.0;
    }
  }
  __syncthreads();  // every thread has read the old maxima
  if (tid < P && score[tid] > mx[tid]) mx[tid] = score[tid];
}

// Pool of one slot back to its constructor state (runtime.ts:52-58).
__global__ void k_pool_reset(const ModelView m, const SlotView sv, int slot) {
  const int P = m.probe_count;
  for (int k = threadIdx.x; k < P * kDim; k += blockDim.x) sv.pool_w[(int64_t)slot * P * kDim + k] = 0.0;
  if (threadIdx.x < P) {
    sv.pool_max[(int64_t)slot * P + threadIdx.x] = -INFINITY;
    sv.pool_den[(int64_t)slot * P + threadIdx.x] = 0.0;
  }
}

// confidence (runtime.ts:634-645): pooled = f32(weighted / max(denominator, 1e-30)) (runtime.ts:
// 92-104), denseMatvec of the projection with bias (cq.ts:297-318: binary64 sum from the bias,
// exact products, sequential over the columns), sigmoid of output 0.
__global__ void __launch_bounds__(kDim) k_confidence(const ModelView m, const SlotView sv, int slot, double* out) {
  extern __shared__ float pooled[];  // [P * kDim]
  const int tid = threadIdx.x, P = m.probe_count;
  for (int p = 0; p < P; p++) {
    const double den = fmax(sv.pool_den[(int64_t)slot * P + p], 1e-30);
    pooled[p * kDim + tid] = f32(sv.pool_w[((int64_t)slot * P + p) * kDim + tid] / den);
  }
  __syncthreads();
  if (tid == 0) {
    const int n = P * kDim;
    double sum = (double)m.probe_bias[0];
    for (int c = 0; c < n; c++) sum = fma((double)__ldg(m.probe_proj + c), (double)pooled[c], sum);
    *out = sigmoid_d((double)f32(sum));
  }
}

// ------------------------------------------------------------------ device scheduler

// Admission: every idle slot takes the next queued sequence (reset as runtime.ts:150-225 with
// sink 0 and maximumLength = prompt + generated tokens).
__global__ void k_sched_admit(const SlotView sv, const SchedView q, int window) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= q.n_slots) return;
  SeqState* seq = sv.seq + s;
  if (seq->busy) return;
  const int id = atomicAdd(q.next_seq, 1);
  if (id >= q.n_seqs) return;
  const int off = q.prompt_offsets[id];
  const int len = q.prompt_offsets[id + 1] - off;
  const int gen = q.gen_steps[id];
  const int max_len = len + gen;
  seq->position = 0;
  seq->sink = 0;
  seq->max_len = max_len;
  seq->kv_alloc = window > 0 ? min(max_len, window) : max_len;
  seq->pending = 0;
  seq->hist[0] = seq->hist[1] = seq->hist[2] = 0;
  seq->seq_id = id;
  seq->prompt_off = off;
  seq->prompt_len = len;
  seq->gen_target = gen;
  seq->gen_done = 0;
  seq->collect = 0;
  seq->busy = 1;
}

// Builds the step's item list from the busy slots: selecting items (the last prompt token and
// every decode step) first, then prefill items.  One CTA.
// counts: [0] items, [1] selecting items, then for micro-batch k (items [k * part, (k + 1) *
// part)) its items at [2 + 2k] and its selecting items (a prefix of its items) at [3 + 2k].
__global__ void __launch_bounds__(1024) k_sched(const SlotView sv, const StepView st, const SchedView q,
                                              int32_t* counts, int part, int parts) {
  __shared__ int s_sel;
  const int tid = threadIdx.x;
  if (tid == 0) s_sel = 0;
  __syncthreads();
  // pass 1: count selecting items
  for (int s = tid; s < q.n_slots; s += blockDim.x) {
    const SeqState& seq = sv.seq[s];
    if (seq.busy && seq.position >= seq.prompt_len - 1) atomicAdd(&s_sel, 1);
  }
  __syncthreads();
  const int n_sel = s_sel;
  __shared__ int c_sel, c_pre;
  if (tid == 0) {
    c_sel = 0;
    c_pre = 0;
  }
  __syncthreads();
  for (int s = tid; s < q.n_slots; s += blockDim.x) {
    const SeqState& seq = sv.seq[s];
    if (!seq.busy) continue;
    const bool sel = seq.position >= seq.prompt_len - 1;
    const int idx = sel ? atomicAdd(&c_sel, 1) : n_sel + atomicAdd(&c_pre, 1);
    DevItem it;
    it.slot = s;
    it.token = seq.position < seq.prompt_len ? q.prompt_ids[seq.prompt_off + seq.position] : -1;
    it.select = sel ? 1 : 0;
    it.allowed_count = -1;
    it.allowed_offset = 0;
    it.position = seq.position;
    it.out_index = idx;
    it.flags = 0;
    it.chunk_index = 0;
    it.chunk_len = 0;
    st.items[idx] = it;
  }
  __syncthreads();
  if (tid == 0) {
    const int n = c_sel + c_pre;
    counts[0] = n;
    counts[1] = c_sel;
    for (int k = 0; k < parts; k++) {
      counts[2 + 2 * k] = min(max(n - k * part, 0), part);
      counts[3 + 2 * k] = min(max(c_sel - k * part, 0), part);
    }
  }
}

// Exclusive prefix sum of `v` over the block (a multiple of 32 threads, at most 1024); *total gets
// the block's sum.  Every thread of the block calls it.
__device__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[w] = x;
  __syncthreads();
  if (w == 0) {
    int t = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < nw) warp_sums[lane] = t;
  }
  __syncthreads();
  const int before = (w > 0 ? warp_sums[w - 1] : 0) + x - v;
  *total = warp_sums[nw - 1];
  __syncthreads();
  return before;
}

// The step's items with prompt chunks (needle_opts.sched_chunk).  Micro-batch k owns slots
// [k * slots_per_part, ...) and item rows [k * items_per_part, ...): its selecting items first
// (the last prompt position and every decode step), then its prefilling slots' items.  Each busy
// slot gets one item; a prefilling slot may take up to chunk_max consecutive prompt positions as a
// chunk -- never its last prompt position (that one selects) nor past its KV window (sink 0 here:
// positions beyond `window` would overwrite ring entries an earlier item of the chunk still reads)
// -- while the micro-batch's rows last, in slot order.  One CTA, one thread per slot (n_slots <= 1024).
__global__ void __launch_bounds__(1024) k_sched_chunked(const SlotView sv, const StepView st, const SchedView q,
                                                      int32_t* counts, int slots_per_part, int items_per_part,
                                                      int parts, int chunk_max, int window) {
  __shared__ int warp_sums[32];
  __shared__ int first_sel[kMaxMicro + 1], first_extra[kMaxMicro + 1], first_rows[kMaxMicro + 1];
  __shared__ int n_sel[kMaxMicro], n_pre[kMaxMicro], n_rows[kMaxMicro];
  const int s = threadIdx.x;
  const bool live = s < q.n_slots;
  const int part = live ? s / slots_per_part : 0;
  if (s < kMaxMicro) {
    n_sel[s] = 0;
    n_pre[s] = 0;
    n_rows[s] = 0;
  }
  __syncthreads();
  SeqState seq{};
  if (live) seq = sv.seq[s];
  const bool busy = live && seq.busy;
  const bool sel = busy && seq.position >= seq.prompt_len - 1;
  const bool pre = busy && !sel;
  int want = 1;
  if (pre) {
    want = min(chunk_max, seq.prompt_len - 1 - seq.position);
    if (window > 0) want = min(want, window - seq.position);
    want = max(want, 1);
  }
  if (sel) atomicAdd(&n_sel[part], 1);
  if (pre) atomicAdd(&n_pre[part], 1);
  int total;
  const int sel_before = block_exclusive_scan(sel ? 1 : 0, warp_sums, &total);
  const int extra_before = block_exclusive_scan(pre ? want - 1 : 0, warp_sums, &total);
  // the scans' values at each micro-batch's first slot
  if (live && s % slots_per_part == 0) {
    first_sel[part] = sel_before;
    first_extra[part] = extra_before;
  }
  __syncthreads();
  const int budget = items_per_part - n_sel[part] - n_pre[part];
  const int extra_in_part = extra_before - first_extra[part];
  const int grant = pre ? max(0, min(want - 1, budget - extra_in_part)) : 0;
  const int rows = pre ? 1 + grant : 0;
  const int rows_before = block_exclusive_scan(rows, warp_sums, &total);
  if (live && s % slots_per_part == 0) first_rows[part] = rows_before;
  if (pre) atomicAdd(&n_rows[part], rows);
  __syncthreads();
  const int base = part * items_per_part;
  if (sel) {
    const int idx = base + sel_before - first_sel[part];
    DevItem it;
    it.slot = s;
    it.token = seq.position < seq.prompt_len ? q.prompt_ids[seq.prompt_off + seq.position] : -1;
    it.select = 1;
    it.allowed_count = -1;
    it.allowed_offset = 0;
    it.position = seq.position;
    it.out_index = idx;
    it.flags = 0;
    it.chunk_index = 0;
    it.chunk_len = 0;
    st.items[idx] = it;
  } else if (pre) {
    const int first = base + n_sel[part] + rows_before - first_rows[part];
    for (int j = 0; j < rows; j++) {
      DevItem it;
      it.slot = s;
      it.token = q.prompt_ids[seq.prompt_off + seq.position + j];
      it.select = 0;
      it.allowed_count = -1;
      it.allowed_offset = 0;
      it.position = seq.position + j;
      it.out_index = first + j;
      it.flags = 0;
      it.chunk_index = rows > 1 ? j : 0;
      it.chunk_len = rows > 1 ? rows : 0;
      st.items[first + j] = it;
    }
  }
  if (s == 0) {
    int all = 0, all_sel = 0;
    for (int k = 0; k < parts; k++) {
      counts[2 + 2 * k] = n_sel[k] + n_rows[k];
      counts[3 + 2 * k] = n_sel[k];
      all += n_sel[k] + n_rows[k];
      all_sel += n_sel[k];
    }
    counts[0] = all;
    counts[1] = all_sel;
  }
}

}  // namespace

// ------------------------------------------------------------------ launchers

// The dynamic shared-memory limit is an attribute of the function on the device, shared by every
// context in the process, so it is raised to the device's opt-in maximum rather than to one
// context's need (a smaller later context must not lower it under a larger one).
static cudaError_t raise_smem_limit(const void* fn) {
  int device = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  cudaFuncAttributes attr{};
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, fn);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)attr.sharedSizeBytes);
  return e;
}

cudaError_t launch_embed(const ModelView& m, const SlotView& sv, const StepView& st, int n_host,
                         cudaStream_t s) {
  if (n_host <= 0) return cudaSuccess;
  k_embed<<<n_host, kThreads, 0, s>>>(m, sv, st);
  return cudaGetLastError();
}

cudaError_t launch_layer(const ModelView& m, const SlotView& sv, const StepView& st, int layer,
                         int n_host, cudaStream_t s) {
  if (n_host <= 0) return cudaSuccess;
  const size_t smem = sizeof(LayerSmem);
  if (m.fast)
    k_layer<true><<<n_host, kThreads, smem, s>>>(m, sv, st, layer);
  else
    k_layer<false><<<n_host, kThreads, smem, s>>>(m, sv, st, layer);
  return cudaGetLastError();
}

size_t attention_smem_bytes(int32_t capacity, bool) {
  return kAttnTileBytes + sizeof(double) * 2 * (size_t)capacity;
}

cudaError_t launch_attention(const ModelView& m, const SlotView& sv, const StepView& st, int layer,
                             int n_host, cudaStream_t s, int part) {
  if (n_host <= 0) return cudaSuccess;
  const size_t smem = attention_smem_bytes(sv.capacity, true);
  k_attention<kAttnSc, kAttnMix, kAttnMc><<<dim3(n_host, kKvHeads), kAttnThreads, smem, s>>>(m, sv, st, layer, part);
  return cudaGetLastError();
}

cudaError_t launch_attention_dev(const float* q, const int8_t* kc, const float* ks, const int8_t* vc,
                                 const float* vs, const int32_t* counts, int32_t batch,
                                 int32_t capacity, float* out, cudaStream_t s) {
  if (batch <= 0) return cudaSuccess;
  const size_t smem = attention_smem_bytes(capacity, false);
  cudaError_t e = raise_smem_limit(reinterpret_cast<const void*>(k_attention_dev));
  if (e != cudaSuccess) return e;
  k_attention_dev<<<dim3(batch, kKvHeads), kAttnThreads, smem, s>>>(q, kc, ks, vc, vs, counts, capacity, out);
  return cudaGetLastError();
}

cudaError_t launch_attention_gate(const StepView& st, int n_host, cudaStream_t s) {
  if (n_host <= 0) return cudaSuccess;
  k_attention_gate<<<dim3(n_host, kKvHeads), kAttnThreads, 0, s>>>(st);
  return cudaGetLastError();
}

cudaError_t launch_route(const StepView& st, int n_host, cudaStream_t s) {
  if (n_host <= 0) return cudaSuccess;
  k_route<<<n_host, 32, 0, s>>>(st);
  return cudaGetLastError();
}

cudaError_t configure_step_kernels(int32_t capacity) {
  if (sizeof(LayerSmem) > 200 * 1024 || attention_smem_bytes(capacity, true) > 200 * 1024)
    return cudaErrorInvalidValue;
  cudaError_t e = raise_smem_limit(reinterpret_cast<const void*>(k_layer<false>));
  if (e != cudaSuccess) return e;
  e = raise_smem_limit(reinterpret_cast<const void*>(k_layer<true>));
  if (e != cudaSuccess) return e;
  e = raise_smem_limit(reinterpret_cast<const void*>(k_attention<kAttnSc, kAttnMix, kAttnMc>));
  if (e != cudaSuccess) return e;
  return raise_smem_limit(reinterpret_cast<const void*>(k_attention_dev));
}

cudaError_t launch_finish(const ModelView& m, const SlotView& sv, const StepView& st, int n_host,
                          const SchedView* sched, cudaStream_t s) {
  if (n_host <= 0) return cudaSuccess;
  SchedView q{};
  if (sched) q = *sched;
  k_finish<<<n_host, kFinishThreads, 0, s>>>(m, sv, st, q, sched ? 1 : 0);
  return cudaGetLastError();
}

// One block per staged mask: a coalesced copy of its words into its pool slot.
__global__ void k_mask_scatter(const uint32_t* __restrict__ staged, const int32_t* __restrict__ slots, int words,
                               uint32_t* __restrict__ pool) {
  const uint32_t* src = staged + (int64_t)blockIdx.x * words;
  uint32_t* dst = pool + (int64_t)slots[blockIdx.x] * words;
  for (int k = threadIdx.x; k < words; k += blockDim.x) dst[k] = src[k];
}

cudaError_t launch_mask_scatter(const uint32_t* staged, const int32_t* slots, int n, int words, uint32_t* pool,
                                cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  k_mask_scatter<<<n, 256, 0, s>>>(staged, slots, words, pool);
  return cudaGetLastError();
}

cudaError_t launch_probe_add(const ModelView& m, const SlotView& sv, const StepView& st, int source, int n_host,
                             cudaStream_t s) {
  if (n_host <= 0 || m.probe_count <= 0) return cudaSuccess;
  k_probe_add<<<n_host, kDim, 0, s>>>(m, sv, st, source);
  return cudaGetLastError();
}

cudaError_t launch_pool_reset(const ModelView& m, const SlotView& sv, int slot, cudaStream_t s) {
  if (m.probe_count <= 0) return cudaSuccess;
  k_pool_reset<<<1, 256, 0, s>>>(m, sv, slot);
  return cudaGetLastError();
}

cudaError_t launch_confidence(const ModelView& m, const SlotView& sv, int slot, double* out, cudaStream_t s) {
  if (m.probe_count <= 0) return cudaSuccess;
  k_confidence<<<1, kDim, sizeof(float) * m.probe_count * kDim, s>>>(m, sv, slot, out);
  return cudaGetLastError();
}

cudaError_t launch_sched_admit(const SlotView& sv, const SchedView& q, int window, cudaStream_t s) {
  k_sched_admit<<<(q.n_slots + 255) / 256, 256, 0, s>>>(sv, q, window);
  return cudaGetLastError();
}

cudaError_t launch_sched(const SlotView& sv, const StepView& st, const SchedView& q, int32_t* counts, int part,
                         int parts, cudaStream_t s) {
  if (parts < 1 || parts > kMaxMicro) return cudaErrorInvalidValue;
  k_sched<<<1, 1024, 0, s>>>(sv, st, q, counts, part, parts);
  return cudaGetLastError();
}

cudaError_t launch_sched_chunked(const SlotView& sv, const StepView& st, const SchedView& q, int32_t* counts,
                                 int slots_per_part, int items_per_part, int parts, int chunk_max, int window,
                                 cudaStream_t s) {
  if (q.n_slots > 1024 || parts > kMaxMicro) return cudaErrorInvalidValue;
  k_sched_chunked<<<1, 1024, 0, s>>>(sv, st, q, counts, slots_per_part, items_per_part, parts, chunk_max, window);
  return cudaGetLastError();
}

}  // namespace needle
