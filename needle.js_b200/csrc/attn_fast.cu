// attn_fast.cu -- fast-numerics decode attention over the int8 KV cache (binary32, online softmax,
// split over positions).  It computes the same function as #attention (packages/needle.js/src/
// model/runtime.ts:719-786) but in binary32 with a different summation order, so it matches the
// reference within a tolerance rather than bit for bit; the exact kernel is attend_pair in
// layer.cu.
//
// Decomposition (flash-decoding): one CTA per (item, KV head, split of kSplit positions); each
// warp streams its own 32-position slice of every 128-position tile.  Four lanes share a
// position (16 head dimensions each), so one 16-byte load per lane brings a K or V row in with
// full coalescing, both query heads of the KV head (GQA x2) reuse it, and the K.q partial dots
// reduce with two shuffles.  int8 codes become binary32 exactly through a byte permute into the
// bit pattern of 2^23 + (code + 128) followed by one subtraction.  Each warp keeps a running max,
// denominator and value accumulator per query head (online softmax); warps and then splits are
// merged with the usual max-rescaled sums.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "engine.cuh"

namespace needle {

namespace {

constexpr int kFastThreads = 128;
// Positions per work unit (item, KV head, split).  Measured at batch 64, L = 8192: 1024 -> 42.6 us,
// 2048 -> 37.7 us, 4096 -> 38.9 us, 512 -> 52.5 us: each unit pays a query setup and a merge of the
// consumer warps, so units should be long, but not so long that the last ones leave SMs idle.
constexpr int kSplit = 2048;
constexpr int kTilePos = 128;    // positions per tile (32 per warp)
constexpr float kLog2e = 1.4426950408889634f;

// Partial result of one (item, KV head, split): per query head m, l and acc[64].
struct Partial {
  float m[2], l[2];
  float acc[2][kHeadDim];
};

// 16 int8 codes (one uint4) -> 16 exact binary32 values.
__device__ __forceinline__ void codes16(const uint4 u, float* out) {
  const uint32_t w[4] = {u.x ^ 0x80808080u, u.y ^ 0x80808080u, u.z ^ 0x80808080u, u.w ^ 0x80808080u};
#pragma unroll
  for (int k = 0; k < 4; k++) {
#pragma unroll
    for (int b = 0; b < 4; b++) {
      // bytes: [biased code, 0, 0, 0x4B] -> 8388608 + (code + 128)
      const uint32_t bits = __byte_perm(w[k], 0x4B000000u, 0x7440 + b);
      out[4 * k + b] = __uint_as_float(bits) - 8388736.0f;
    }
  }
}

__global__ void __launch_bounds__(kFastThreads) k_attention_fast(
    const float* __restrict__ q, const int8_t* __restrict__ kc, const float* __restrict__ ks,
    const int8_t* __restrict__ vc, const float* __restrict__ vs, const int32_t* __restrict__ counts,
    int32_t capacity, int32_t splits, Partial* __restrict__ partials, const int64_t* __restrict__ row_base) {
  __shared__ Partial warp_part[kFastThreads / 32];
  const int b = blockIdx.x, h = blockIdx.y, split = blockIdx.z;
  const int count = min(max(counts[b], 0), capacity);
  const int t_begin = split * kSplit;
  Partial* out = partials + ((int64_t)b * kKvHeads + h) * splits + split;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (t_begin >= count) {
    if (tid < 2) {
      out->m[tid] = -INFINITY;
      out->l[tid] = 0.0f;
    }
    return;
  }
  const int t_end = min(count, t_begin + kSplit);
  const int part = lane & 3;    // dims [16 part, 16 part + 16)
  const int pgrp = lane >> 2;   // position within an 8-position group
  // query of both heads for this lane's dims, pre-scaled by log2(e) / sqrt(64)
  float qr[2][16];
  const float* qb = q + (int64_t)b * kHeads * kHeadDim + 2 * h * kHeadDim + part * 16;
#pragma unroll
  for (int hh = 0; hh < 2; hh++)
#pragma unroll
    for (int d = 0; d < 16; d++) qr[hh][d] = qb[hh * kHeadDim + d] * (0.125f * kLog2e);

  const int64_t head_row = (row_base ? row_base[b] : (int64_t)b * kKvHeads * capacity) + (int64_t)h * capacity;
  const uint4* krows = reinterpret_cast<const uint4*>(kc + head_row * kHeadDim);
  const uint4* vrows = reinterpret_cast<const uint4*>(vc + head_row * kHeadDim);
  const float* ksc = ks + head_row;
  const float* vsc = vs + head_row;

  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
  float acc[2][16];
#pragma unroll
  for (int hh = 0; hh < 2; hh++)
#pragma unroll
    for (int d = 0; d < 16; d++) acc[hh][d] = 0.0f;

  // Each warp walks 8 positions per iteration: tile base + warp slice + 8 * it + pgrp.
  for (int t0 = t_begin + warp * 32; t0 < t_end; t0 += kTilePos) {
    uint4 kreg[4], vreg[4];
    float ksv[4], vsv[4];
#pragma unroll
    for (int it = 0; it < 4; it++) {
      const int t = t0 + it * 8 + pgrp;
      const bool ok = t < t_end;
      kreg[it] = ok ? __ldg(krows + (int64_t)t * 4 + part) : make_uint4(0, 0, 0, 0);
      vreg[it] = ok ? __ldg(vrows + (int64_t)t * 4 + part) : make_uint4(0, 0, 0, 0);
      ksv[it] = ok ? __ldg(ksc + t) : 0.0f;
      vsv[it] = ok ? __ldg(vsc + t) : 0.0f;
    }
#pragma unroll
    for (int it = 0; it < 4; it++) {
      const int t = t0 + it * 8 + pgrp;
      const bool ok = t < t_end;
      float kf[16];
      codes16(kreg[it], kf);
      float s[2];
#pragma unroll
      for (int hh = 0; hh < 2; hh++) {
        float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
        for (int d = 0; d < 16; d += 2) {
          d0 = fmaf(qr[hh][d], kf[d], d0);
          d1 = fmaf(qr[hh][d + 1], kf[d + 1], d1);
        }
        float dot = d0 + d1;
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        s[hh] = ok ? dot * ksv[it] : -INFINITY;  // log2-domain score
      }
      float vf[16];
      codes16(vreg[it], vf);
#pragma unroll
      for (int hh = 0; hh < 2; hh++) {
        float mx = s[hh];
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m[hh], mx);
        const float scale = exp2f(m[hh] - m_new);  // 0 on the first tile (m = -inf)
        const float p = ok ? exp2f(s[hh] - m_new) : 0.0f;
        float psum = p;
        psum += __shfl_xor_sync(0xffffffffu, psum, 4);
        psum += __shfl_xor_sync(0xffffffffu, psum, 8);
        psum += __shfl_xor_sync(0xffffffffu, psum, 16);  // the 8 positions, once each
        l[hh] = l[hh] * scale + psum;
        m[hh] = m_new;
        const float pv = p * vsv[it];
#pragma unroll
        for (int d = 0; d < 16; d++) acc[hh][d] = fmaf(pv, vf[d], acc[hh][d] * scale);
      }
    }
  }
  // Sum the eight position groups' accumulators (same m for the whole warp).
#pragma unroll
  for (int hh = 0; hh < 2; hh++)
#pragma unroll
    for (int d = 0; d < 16; d++) {
      float a = acc[hh][d];
      a += __shfl_xor_sync(0xffffffffu, a, 4);
      a += __shfl_xor_sync(0xffffffffu, a, 8);
      a += __shfl_xor_sync(0xffffffffu, a, 16);
      acc[hh][d] = a;
    }
  Partial& wp = warp_part[warp];
  if (lane < 4) {
#pragma unroll
    for (int hh = 0; hh < 2; hh++)
#pragma unroll
      for (int d = 0; d < 16; d++) wp.acc[hh][part * 16 + d] = acc[hh][d];
  }
  if (lane == 0) {
    wp.m[0] = m[0];
    wp.m[1] = m[1];
    wp.l[0] = l[0];
    wp.l[1] = l[1];
  }
  __syncthreads();
  // Merge the four warps: thread (hh, d) over 128 threads.
  {
    const int hh = tid >> 6, d = tid & 63;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; w++) M = fmaxf(M, warp_part[w].m[hh]);
    float L = 0.0f, A = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; w++) {
      const float f = warp_part[w].m[hh] == -INFINITY ? 0.0f : exp2f(warp_part[w].m[hh] - M);
      L += warp_part[w].l[hh] * f;
      A += warp_part[w].acc[hh][d] * f;
    }
    out->acc[hh][d] = A;
    if (d == 0) {
      out->m[hh] = M;
      out->l[hh] = L;
    }
  }
}

// Merges the splits of every (item, KV head): out = sum_s 2^(m_s - M) acc_s / sum_s 2^(m_s - M) l_s,
// in one pass with a running maximum (the loads of all splits are independent, so they overlap).
__global__ void __launch_bounds__(kFastThreads) k_attention_fast_combine(const Partial* __restrict__ partials,
                                                                         int32_t splits, float* __restrict__ out,
                                                                         const int32_t* __restrict__ status) {
  const int b = blockIdx.x, h = blockIdx.y;
  if (status && *status) {  // a bounded wait ran out: report NaN rather than a partial sum
    out[(int64_t)b * kHeads * kHeadDim + h * 2 * kHeadDim + threadIdx.x] = NAN;
    return;
  }
  const int hh = threadIdx.x >> 6, d = threadIdx.x & 63;
  const Partial* p = partials + ((int64_t)b * kKvHeads + h) * splits;
  float M = -INFINITY, L = 0.0f, A = 0.0f;
#pragma unroll 8
  for (int s = 0; s < splits; s++) {
    const float ms = __ldcg(&p[s].m[hh]), ls = __ldcg(&p[s].l[hh]), as = __ldcg(&p[s].acc[hh][d]);
    if (ms == -INFINITY) continue;
    const float Mn = fmaxf(M, ms);
    const float fo = exp2f(M - Mn), fs = exp2f(ms - Mn);  // M = -inf on the first live split: fo = 0
    L = L * fo + ls * fs;
    A = A * fo + as * fs;
    M = Mn;
  }
  out[(int64_t)b * kHeads * kHeadDim + (2 * h + hh) * kHeadDim + d] = L > 0.0f ? A / L : 0.0f;
}

// ------------------------------------------------------------------ tensor-core variant
//
// Same function, with the two contractions of every 32-position slice on the integer tensor cores
// (mma.sync m16n8k32 s8 x s8 -> s32), so that a position costs a few instructions instead of a few
// hundred.  Both operands must be int8; the K and V codes are, and the binary32 sides are split into
// exact integer digits:
//   * q of each head is scaled to Q = rint(q * 2^20 / max|q|) (|Q| <= 2^20) and written as three
//     balanced base-128 digits D0 + 128 D1 + 16384 D2 (each in [-64, 64]).  Rows (digit, head) of
//     the A operand hold the digits, the B operand is K^T straight from shared memory (ldmatrix),
//     and the three digit sums -- exact int32 -- are combined in binary32 with their powers of 128.
//     The relative error of the score is about 2^-21.
//   * the softmax weights w = p * vs of a 32-position slice are scaled to W = rint(w * (2^21 - 1) /
//     max w) and split into three base-128 digits in [0, 127]; rows (digit, head) of the A operand
//     hold them, the B operand is V with positions as the contraction index (ldmatrix .trans plus a
//     byte permute), and the int32 results are folded into binary32 accumulators per slice.
// Because the score MMA produces S^T (rows = digit/head, columns = positions), each lane ends up
// holding the scores of exactly the positions it must supply as A operand of the value MMA, so the
// softmax needs shuffles only for its reductions.
//
// K/V tiles of 256 positions (32 per consumer warp) come in through the tensor-copy engine (cp.async.bulk.tensor, 64-byte
// swizzle so that ldmatrix reads are free of bank conflicts) and the scales through bulk copies,
// into a 3-stage ring filled by one producer warp; every mbarrier wait is bounded in time.
constexpr int kMmaStages = 3;
constexpr int kMmaTile = 256;
constexpr int kMmaConsumers = 8;
constexpr int kMmaThreads = (kMmaConsumers + 1) * 32;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // an mbarrier wait gives up after 2 s

// One ring stage: a 256-position tile of one work item (item, split) plus its header; the first
// tile of an item also carries the item's two query heads.
struct MmaHeader {
  int32_t item;   // work item (b * 4 + h) * splits + split, or -1: no more work
  int32_t tile;   // tile index within the item
  int32_t n;      // valid positions in the tile
  int32_t last;   // last tile of the item
};
struct MmaStage {
  int8_t k[kMmaTile * kHeadDim];  // 64-byte rows, 16-byte chunks swizzled by (row >> 1) & 3
  int8_t v[kMmaTile * kHeadDim];
  float ks[kMmaTile];
  float vs[kMmaTile];
  float q[2 * kHeadDim];
  MmaHeader hdr;
  uint8_t pad[1024 - 2 * kHeadDim * 4 - sizeof(MmaHeader)];
};
static_assert(sizeof(MmaStage) % 1024 == 0, "stages stay 1024-byte aligned");

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits for the phase with the given parity; false once kWaitLimitNs has passed without it.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  for (;;) {
    for (int i = 0; i < 32; i++)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - start > kWaitLimitNs) return false;
  }
}
// Global -> shared bulk copy (no multicast) whose completion is counted on `bar`.
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Tiled 2D tensor copy (no multicast) of the box at (x, y) into shared memory, counted on `bar`.
__device__ __forceinline__ void tensor_copy_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t r[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t r[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
// d = A (16x32 s8, rows 8-15 zero) x B (32x8 s8) + c.  a0 / a2: row g, k 4q.. and 16 + 4q..
__device__ __forceinline__ void mma_s8(int32_t d[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1,
                                       const int32_t c[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %11, %12, %13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]));
}
// Byte offset of 16-byte chunk c of tile row r under the 64-byte swizzle.
__device__ __forceinline__ uint32_t swz64(int r, int c) {
  return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Persistent: every CTA takes work items from a counter until none is left.  The producer warp
// streams the tiles of consecutive items through the ring without draining it between items; the
// consumers follow the stage headers, set up a new item on its first tile and write the item's
// partial after its last.
__global__ void __launch_bounds__(kMmaThreads) k_attention_fast_mma(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const float* __restrict__ q,
    const float* __restrict__ ks, const float* __restrict__ vs, const int32_t* __restrict__ counts,
    int32_t capacity, int32_t splits, int32_t n_items, Partial* __restrict__ partials, int32_t* __restrict__ status,
    int32_t* __restrict__ work, int32_t* __restrict__ done, uint32_t* __restrict__ wait_words,
    const int64_t* __restrict__ row_base) {
  extern __shared__ unsigned char smem_raw[];
  MmaStage* stage = reinterpret_cast<MmaStage*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kMmaStages], empty[kMmaStages];
  __shared__ Partial warp_part[kMmaConsumers];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kMmaStages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kMmaConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kMmaConsumers) {
    // ---------------- producer: one elected lane claims items and issues the copies
    if (lane == 0) {
      int seq = 0;  // tiles issued by this CTA (ring position and phase)
      bool ok = true;
      auto next_stage = [&](int& sidx) -> bool {
        sidx = seq % kMmaStages;
        if (seq >= kMmaStages && !mbar_wait(&empty[sidx], ((seq / kMmaStages) - 1) & 1)) {
          { atomicExch(status, 1); report_wait_timeout(wait_words, kWaitAttention); }
          return false;
        }
        return true;
      };
      for (;;) {
        const int item = atomicAdd(work, 1);
        if (item >= n_items) break;
        const int split = item % splits, bh = item / splits, b = bh / kKvHeads;
        const int count = min(max(counts[b], 0), capacity);
        const int t_begin = split * kSplit;
        if (t_begin >= count) {  // nothing visible in this split
          partials[item].m[0] = partials[item].m[1] = -INFINITY;
          partials[item].l[0] = partials[item].l[1] = 0.0f;
          continue;
        }
        const int t_end = min(count, t_begin + kSplit);
        const int ntiles = (t_end - t_begin + kMmaTile - 1) / kMmaTile;
        const int64_t head_row =
            (row_base ? row_base[b] : (int64_t)b * kKvHeads * capacity) + (int64_t)(bh % kKvHeads) * capacity;
        for (int ti = 0; ti < ntiles && ok; ti++, seq++) {
          int sidx;
          if (!(ok = next_stage(sidx))) break;
          MmaStage& st = stage[sidx];
          const int t0 = t_begin + ti * kMmaTile;
          const int n = min(kMmaTile, t_end - t0);
          const int n4 = (n + 3) & ~3;  // scale copies in whole 16-byte units (capacity % 4 == 0)
          st.hdr.item = item;
          st.hdr.tile = ti;
          st.hdr.n = n;
          st.hdr.last = ti == ntiles - 1;
          mbar_expect_tx(&full[sidx], 2u * kMmaTile * kHeadDim + 2u * n4 * 4 + (ti == 0 ? 2u * kHeadDim * 4 : 0u));
          tensor_copy_2d(st.k, &kmap, 0, (int)(head_row + t0), &full[sidx]);
          tensor_copy_2d(st.v, &vmap, 0, (int)(head_row + t0), &full[sidx]);
          bulk_copy(st.ks, ks + head_row + t0, n4 * 4, &full[sidx]);
          bulk_copy(st.vs, vs + head_row + t0, n4 * 4, &full[sidx]);
          if (ti == 0)
            bulk_copy(st.q, q + (int64_t)b * kHeads * kHeadDim + 2 * (bh % kKvHeads) * kHeadDim, 2 * kHeadDim * 4,
                      &full[sidx]);
        }
        if (!ok) break;
      }
      // sentinel stage: no more work
      int sidx;
      if (ok && next_stage(sidx)) {
        stage[sidx].hdr.item = -1;
        mbar_arrive(&full[sidx]);
        seq++;
      }
      // The CTA must not retire with copies still landing in its shared memory: wait (bounded)
      // for the last tile issued into each stage.
      for (int i = max(0, seq - kMmaStages); i < seq; i++)
        if (!mbar_wait(&full[i % kMmaStages], (i / kMmaStages) & 1)) { atomicExch(status, 1); report_wait_timeout(wait_words, kWaitAttention); }
      // The last CTA to stop claiming work resets the counters for the next call (no CTA claims
      // any more once its claim failed, so nothing races with the reset).
      __threadfence();
      if (atomicAdd(done, 1) == (int)(gridDim.x - 1)) {
        *work = 0;
        *done = 0;
        __threadfence();
      }
    }
    return;
  }

  // ---------------- consumers: warp w takes positions [32 w, 32 w + 32) of every tile
  const int g = lane >> 2, qd = lane & 3;
  const int hh = g & 1, dig = g >> 1;  // A-operand row (digit, head); digit 3 = the zero rows 6, 7
  const float dweight = dig == 0 ? 1.0f : dig == 1 ? 128.0f : dig == 2 ? 16384.0f : 0.0f;
  const uint32_t wshift = 7u * (uint32_t)min(dig, 2), wmask = dig < 3 ? 127u : 0u;
  const int32_t zero4[4] = {0, 0, 0, 0};
  const int pw = warp * 32;
  uint32_t qa[2][2] = {{0u, 0u}, {0u, 0u}};  // [k-slice][a0, a2]: this row's digits of q
  float cmul = 0.0f;                          // digit weight * max|q| / 2^20 / 8 * log2(e)
  float m = -INFINITY, l = 0.0f;              // this lane's head
  float acc[8][2];                            // value rows (digit, head): n-tile 2 bb + parity, column 2 qd + e
  for (int seq = 0;; seq++) {
    const int sidx = seq % kMmaStages;
    // Every consumer warp waits on the same stages in the same order, so a bounded wait that runs out
    // runs out for all of them before any item barrier below.
    if (!mbar_wait(&full[sidx], (seq / kMmaStages) & 1)) {
      { atomicExch(status, 1); report_wait_timeout(wait_words, kWaitAttention); }
      break;
    }
    const MmaStage& st = stage[sidx];
    const MmaHeader hdr = st.hdr;
    if (hdr.item < 0) break;
    if (hdr.tile == 0) {  // new item: q digits of this lane's row, reset the running state
      float qmax[2];
#pragma unroll
      for (int x = 0; x < 2; x++) {
        float mx = fmaxf(fabsf(st.q[x * kHeadDim + lane]), fabsf(st.q[x * kHeadDim + 32 + lane]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        qmax[x] = mx;
      }
      const float qm = hh ? qmax[1] : qmax[0];
      const float qinv = qm > 0.0f ? 1048576.0f / qm : 0.0f;
#pragma unroll
      for (int kk = 0; kk < 2; kk++)
#pragma unroll
        for (int half = 0; half < 2; half++) {
          uint32_t word = 0;
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const int d = 32 * kk + 16 * half + 4 * qd + i;
            const int Q = __float2int_rn(st.q[hh * kHeadDim + d] * qinv);
            const int D0 = ((Q + 64) & 127) - 64;
            const int Q1 = (Q - D0) >> 7;
            const int D1 = ((Q1 + 64) & 127) - 64;
            const int D2 = (Q1 - D1) >> 7;
            const int digit = dig == 0 ? D0 : dig == 1 ? D1 : dig == 2 ? D2 : 0;
            word |= (uint32_t)(digit & 0xff) << (8 * i);
          }
          qa[kk][half] = word;
        }
      cmul = dweight * qm * (1.0f / 1048576.0f) * (0.125f * kLog2e);
      m = -INFINITY;
      l = 0.0f;
#pragma unroll
      for (int nt = 0; nt < 8; nt++) acc[nt][0] = acc[nt][1] = 0.0f;
    }
    const int n = hdr.n;
    const bool full_tile = n == kMmaTile;
    const uint32_t kbase = smem_u32(st.k), vbase = smem_u32(st.v);
    // scores S^T: 4 column tiles of 8 positions; lane holds positions pw + 8 j + 2 qd + e
    float sc[4][2];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int r = pw + 8 * j + (lane & 7);
      uint32_t kb[4];
      ldsm_x4(kbase + swz64(r, lane >> 3), kb);
      int32_t d0[4], d1[4];
      mma_s8(d0, qa[0][0], qa[0][1], kb[0], kb[1], zero4);
      mma_s8(d1, qa[1][0], qa[1][1], kb[2], kb[3], d0);
      const float2 k2 = *reinterpret_cast<const float2*>(&st.ks[pw + 8 * j + 2 * qd]);
#pragma unroll
      for (int e = 0; e < 2; e++) {
        float v = (float)d1[e] * cmul;
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        sc[j][e] = v * (e ? k2.y : k2.x);
      }
    }
    if (!full_tile) {
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int e = 0; e < 2; e++)
          if (pw + 8 * j + 2 * qd + e >= n) sc[j][e] = -INFINITY;
    }
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; j++) mt = fmaxf(mt, fmaxf(sc[j][0], sc[j][1]));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
    const float m_new = fmaxf(m, mt);
    const float scale = m_new == -INFINITY ? 1.0f : ex2_approx(m - m_new);  // 0 on the first live slice
    const float m_use = m_new == -INFINITY ? 0.0f : m_new;
    float w[4][2], psum = 0.0f, wmax = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 v2 = *reinterpret_cast<const float2*>(&st.vs[pw + 8 * j + 2 * qd]);
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const float p = ex2_approx(sc[j][e] - m_use);  // masked: 2^-inf = 0
        psum += p;
        w[j][e] = p * (e ? v2.y : v2.x);
        wmax = fmaxf(wmax, w[j][e]);
      }
    }
    if (!full_tile) {  // scales past the tile end are not copied: drop their (unspecified) products
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int e = 0; e < 2; e++)
          if (pw + 8 * j + 2 * qd + e >= n) w[j][e] = 0.0f;
      wmax = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; j++) wmax = fmaxf(wmax, fmaxf(w[j][0], w[j][1]));
    }
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    psum += __shfl_xor_sync(0xffffffffu, psum, 2);
    wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, 1));
    wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, 2));
    l = l * scale + psum;
    m = m_new;
    // W = rint(w * 2^(20 - e)) < 2^21 with wmax in [2^e, 2^(e+1)): the power of two comes from the
    // exponent bits, the rounding from adding 2^23; this lane's digit is bits [7 dig, 7 dig + 7).
    const int wexp = (int)((__float_as_uint(wmax) >> 23) & 255u);  // biased exponent of wmax
    const bool wlive = wexp > 20;  // below 2^-106 the slice's weights are dropped
    const float wscale = wlive ? __uint_as_float((uint32_t)(127 + 20 + 127 - wexp) << 23) : 0.0f;
    const float wunit = wlive ? __uint_as_float((uint32_t)(wexp - 20) << 23) : 0.0f;
    uint32_t pa[2] = {0u, 0u};  // A bytes k = 4 qd + i <-> (j, e) = (0,0), (0,1), (1,0), (1,1); j + 2 above
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const uint32_t bits = __float_as_uint(fmaf(w[j][e], wscale, 8388608.0f));
        const uint32_t digit = (bits >> wshift) & wmask;
        pa[j >> 1] |= digit << (8 * (2 * (j & 1) + e));
      }
    const bool rescale = !__all_sync(0xffffffffu, scale == 1.0f);
    // values: per 16-dimension block, 4 matrices of 8 positions transposed, then even / odd dims
#pragma unroll
    for (int bb = 0; bb < 4; bb++) {
      const int r = pw + 8 * (lane >> 3) + (lane & 7);
      uint32_t X[4];
      ldsm_x4_trans(vbase + swz64(r, bb), X);
#pragma unroll
      for (int par = 0; par < 2; par++) {
        const uint32_t sel = par ? 0x7531u : 0x6420u;
        int32_t d[4];
        mma_s8(d, pa[0], pa[1], __byte_perm(X[0], X[1], sel), __byte_perm(X[2], X[3], sel), zero4);
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const float prev = rescale ? acc[2 * bb + par][e] * scale : acc[2 * bb + par][e];
          acc[2 * bb + par][e] = fmaf((float)d[e], wunit, prev);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[sidx]);
    if (hdr.last) {
      // digit rows -> heads: sum_dig 128^dig * row, over lanes 8 dig + 4 hh + qd
      Partial& wp = warp_part[warp];
#pragma unroll
      for (int nt = 0; nt < 8; nt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          float v = acc[nt][e] * dweight;
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 16);
          if (g < 2) wp.acc[hh][16 * (nt >> 1) + 4 * qd + 2 * e + (nt & 1)] = v;
        }
      if (g < 2 && qd == 0) {
        wp.m[hh] = m;
        wp.l[hh] = l;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kMmaConsumers * 32) : "memory");
      if (tid < 128) {
        const int x = tid >> 6, d = tid & 63;
        float M = -INFINITY;
#pragma unroll
        for (int w2 = 0; w2 < kMmaConsumers; w2++) M = fmaxf(M, warp_part[w2].m[x]);
        float L = 0.0f, A = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < kMmaConsumers; w2++) {
          const float f = warp_part[w2].m[x] == -INFINITY ? 0.0f : exp2f(warp_part[w2].m[x] - M);
          L += warp_part[w2].l[x] * f;
          A += warp_part[w2].acc[x][d] * f;
        }
        Partial* out = partials + hdr.item;
        out->acc[x][d] = A;
        if (d == 0) {
          out->m[x] = M;
          out->l[x] = L;
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kMmaConsumers * 32) : "memory");  // warp_part reusable
    }
  }
}

// 2D map of an int8 code array viewed as rows of 64 bytes: boxes of 128 rows, 64-byte swizzle.
// The encoder comes from the driver through the runtime's entry-point query.
bool encode_rows_map(CUtensorMap* map, const int8_t* base, int64_t rows) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult found{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &found) == cudaSuccess &&
        found == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!encode) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kHeadDim};
  const cuuint32_t box[2] = {(cuuint32_t)kHeadDim, (cuuint32_t)kMmaTile};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(base), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t attention_fast_scratch_bytes(int32_t batch, int32_t capacity) {
  const int splits = (capacity + kSplit - 1) / kSplit;
  return 16 + sizeof(Partial) * (size_t)batch * kKvHeads * splits;  // status and counters, partials
}

cudaError_t launch_attention_fast(const float* q, const int8_t* kc, const float* ks, const int8_t* vc,
                                  const float* vs, const int32_t* counts, int32_t batch, int32_t capacity,
                                  float* out, void* scratch, cudaStream_t s, const int64_t* row_base,
                                  int64_t cache_rows, bool tensor) {
  if (batch <= 0) return cudaSuccess;
  const int splits = (capacity + kSplit - 1) / kSplit;
  int32_t* status = static_cast<int32_t*>(scratch);
  Partial* parts = reinterpret_cast<Partial*>(static_cast<char*>(scratch) + 16);
  // status (sticky: once a bounded wait has run out the operator reports NaN), work counter and
  // done counter live at the start of the scratch, zeroed when it was allocated; the persistent
  // kernel leaves the counters at zero.
  cudaError_t e = cudaSuccess;
  // The tensor and bulk copies need 16-byte aligned sources and sizes: rows are 64 bytes, and the
  // scale copies are whole 16-byte units when capacity is a multiple of 4.
  const int64_t rows_total = row_base ? cache_rows : (int64_t)batch * kKvHeads * capacity;
  const bool aligned = capacity % 4 == 0 && rows_total < (1ll << 31) &&
                       ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc) |
                         reinterpret_cast<uintptr_t>(ks) | reinterpret_cast<uintptr_t>(vs) |
                         reinterpret_cast<uintptr_t>(q)) & 15) == 0;
  CUtensorMap kmap, vmap;
  const bool mma = tensor && aligned && encode_rows_map(&kmap, kc, rows_total) &&
                   encode_rows_map(&vmap, vc, rows_total);
  if (mma) {
    const size_t smem = sizeof(MmaStage) * kMmaStages + 1024;  // + alignment slack
    static std::atomic<uint64_t> configured{0};
    static int per_sm[64] = {0};
    int device = 0, sms = 0;
    e = cudaGetDevice(&device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return e;
    if (!(configured.load() & (1ull << (device & 63)))) {
      e = cudaFuncSetAttribute(k_attention_fast_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      int nb = 1;
      if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k_attention_fast_mma, kMmaThreads, smem);
      if (e != cudaSuccess) return e;
      per_sm[device & 63] = nb > 0 ? nb : 1;
      configured.fetch_or(1ull << (device & 63));
    }
    const int n_items = batch * kKvHeads * splits;
    const int grid = std::max(1, std::min(n_items, sms * per_sm[device & 63]));
    k_attention_fast_mma<<<grid, kMmaThreads, smem, s>>>(kmap, vmap, q, ks, vs, counts, capacity, splits, n_items,
                                                         parts, status, status + 1, status + 2,
                                                         wait_status_words(device), row_base);
  } else {
    k_attention_fast<<<dim3(batch, kKvHeads, splits), kFastThreads, 0, s>>>(q, kc, ks, vc, vs, counts, capacity,
                                                                           splits, parts, row_base);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_attention_fast_combine<<<dim3(batch, kKvHeads), kFastThreads, 0, s>>>(parts, splits, out, status);
  return cudaGetLastError();
}

}  // namespace needle
