// cq_gemm_tc.cu -- batched fast-numerics Cactus-Quant matvec on the 5th-generation tensor cores
// (tcgen05.mma, weight operand and accumulator in tensor memory).  cqMatvec
// (packages/needle.js/src/backends/cq.ts:233-240) for a batch of B vectors, in binary32 accuracy:
//
//   y[b][r] = sum_g norm16[r][g] * sum_{k in g} level(code[r][k]) * x'[b][k]
//
// is a GEMM with A = the dequantised weights (rows x inputs; each element is level * norm of its
// group, folded in while decoding) and B = the prepared activations x' (B x inputs).  The tensor
// cores multiply fp16; to keep binary32-level accuracy each operand is split into an fp16 head and
// an fp16 tail (v = hi + lo up to 2^-22 |v|) and the four products A_hi B_hi + A_hi B_lo +
// A_lo B_hi + A_lo B_lo are accumulated in fp32.
// fp16 rather than bf16 (8-bit significands, 2^-16 per operand) because the decode step amplifies
// the projections' relative error about 500-fold over 27 layers: with bf16 heads and tails the
// logits drifted 3e-3 from the reference, with fp16 ones they stay well inside 1e-3.  The weights
// are scaled by 2^10 (exactly; undone in the epilogue) so that the tails of small level * norm
// values stay clear of fp16's subnormal range; activations (prepared, O(1)) are split unscaled.
// For N <= 64 two MMAs per K-step do it: A_hi x [B_hi; B_lo] (N' = 2N: columns [0, N) get A_hi B_hi
// and [N, 2N) A_hi B_lo) and A_lo x [B_hi; B_lo] into the same columns, and the epilogue adds the two
// column blocks; above, four MMAs of N columns accumulate into [0, N).
//
// Kernels.  k_cq_prep_f16 writes x' of every (group, item) as fp16 head and tail rows already in
// the shared-memory layout the MMA reads (K-major, 128-byte swizzle; per group and 64-column half
// the N head rows then the N tail rows), so the GEMM fetches a group's activations with one bulk
// copy.  k_cq_gemm_tc: one CTA per (128-row tile, range of groups) and SM; the groups are split
// across CTAs (split-K) when there are fewer row tiles than SMs, and k_splitk_sum adds the splits'
// partial results in a fixed order.
//
// k_cq_gemm_tc is warp-specialised around a ring of 3 group slots (A operand in tensor memory,
// activations in shared memory):
//   * decode warps 0-11, three teams of four (team t takes groups t, t + 3, ... into slot t, so that
//     each slot is used in one team's program order; warp w serves tensor-memory lanes
//     32 (w % 4) ..+31, one tile row per thread).  Per group a thread turns its
//     row's norm into a 16-entry table of split values (level * norm as fp16 head | tail), decodes
//     the row's 128 weights with one table read each and writes the head and tail words into tensor
//     memory (tcgen05.st); its packed bytes were loaded two of its groups earlier.
//   * warp 12 (one elected lane) issues a group's 8 K-steps x 2 (or 3) MMAs and commits them to the slot's
//     "empty" barrier, which frees the slot for the decoders and the producer.
//   * warp 13 (one thread) bulk-copies the groups' activation tiles into the ring.
// Every mbarrier wait gives up after 2 s and marks the tile failed (its outputs become NaN).  The
// epilogue reads the accumulator with tcgen05.ld (decode warps, one row per lane).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "cq.cuh"

namespace needle {

namespace {

constexpr int kTcTeams = 3;                 // decode teams of 4 warps (one per tensor-memory lane quarter)
constexpr int kTcDecodeWarps = 4 * kTcTeams;
constexpr int kTcDecodeThreads = kTcDecodeWarps * 32;
constexpr int kTcMmaWarp = kTcDecodeWarps, kTcCopyWarp = kTcDecodeWarps + 1;
constexpr int kTcThreads = kTcDecodeThreads + 64;
constexpr int kTcM = 128;                   // rows per tile (MMA M)
constexpr int kTcMaxN = 128;                // items per pass (MMA N, multiple of 16)
constexpr int kTcMaxSlots = 3;
constexpr uint32_t kTcCols = 512;           // tensor memory: accumulator, then the A slots (128 columns)
constexpr int kTcPrefetch = 2;              // groups of packed bytes in flight per decode thread
constexpr uint64_t kTcWaitNs = 2000000000ull;  // an mbarrier wait gives up after 2 s
constexpr size_t kTcTableBytes = 16 * kTcDecodeThreads * 4;  // per-thread split tables [code][thread]
// Smallest dynamic shared memory per CTA: more than half an SM's, so that no two CTAs share an SM
// (each holds all 512 tensor-memory columns).
constexpr size_t kTcMinSmem = 120 * 1024;

// Ring slots (one per decode team); accumulator columns [0, 128) then 3 A slots of 128 columns.
constexpr int kTcSlotsUsed = 3;
constexpr uint32_t kTcAccCols = 128;

// Byte offset of 16-bit element (row, k) (k < 64) in a K-major, 128-byte-swizzled tile.
__host__ __device__ __forceinline__ uint32_t sw128(int row, int k) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + (((k >> 3) ^ (row & 7)) << 4) + (k & 7) * 2);
}

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart,
// descriptor version 1.  The K offset inside the swizzle atom advances the start address.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t a) {
  return (uint64_t)((a >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
         ((uint64_t)2 << 61);
}

// Instruction descriptor: fp16 x fp16 -> fp32 (A and B type fields 0 = f16, both), A and B
// K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t f16_idesc(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcM >> 4) << 24);
}

constexpr float kTcWeightScale = 1024.0f;  // 2^10: A = level * norm * 2^10, undone in the epilogue

// D (tensor memory) (+)= A (tensor memory, 128 lanes x 8 columns = 16 fp16 per row) x B^T (shared);
// issued by one thread.
__device__ __forceinline__ void mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Arrive on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
               : "memory");
}

// True in one lane of the (converged) warp.
__device__ __forceinline__ bool elect_one() {
  uint32_t e;
  asm volatile("{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n" : "=r"(e));
  return e != 0;
}

__device__ __forceinline__ void bar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void bar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}

__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = saddr(bar);
  uint64_t start = 0;
  for (int it = 0;; it++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    uint64_t now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    if (it == 0) start = now;
    else if (now - start > kTcWaitNs) return false;
  }
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(saddr(bar))
               : "memory");
}

// 16 consecutive 32-bit tensor-memory columns of this thread's lane <- v[0..15].
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// v[0..7] <- 8 consecutive 32-bit tensor-memory columns of this thread's lane.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// fp16 head and tail of two binary32 values, as half2 words (first value in the low half).  The
// head is fp16(v); v - head is exact in binary32 and its fp16 rounding is the tail.
__device__ __forceinline__ void split2(float v0, float v1, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(v0, v1);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  const float r0 = __fsub_rn(v0, __low2float(h));
  const float r1 = __fsub_rn(v1, __high2float(h));
  const __half2 l = __floats2half2_rn(r0, r1);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// x' of (group g, item n) as fp16 head and tail, in the GEMM's activation layout
// [group][half (2)][2N rows: N head rows, N tail rows][128 bytes], rows swizzled as the MMA's
// K-major 128-byte layout.  One warp per (group, item); items nb <= n < N are zeros.
// `prepared` inputs are x' already (padded to whole groups); otherwise each group is prepared here.
// Items form tiles of N (the GEMM's item tiles), tile t at act + t * groups * 2 * 2N * 128; items
// past `batch` in the last tile are zeros.  One warp per (item slot, group).
__global__ void __launch_bounds__(256) k_cq_prep_f16(const float* __restrict__ x, int32_t x_stride, int32_t input_size,
                                                      int32_t groups, int32_t batch, int32_t N, int32_t tiles,
                                                      int32_t prepared, uint8_t* __restrict__ act_all) {
  const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (w >= groups * N * tiles) return;
  const int item = w / groups, g = w - item * groups;
  const int t = item / N, n = item - t * N;
  uint8_t* act = act_all + (size_t)t * groups * 2 * (2 * N) * 128;
  float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (item < batch) {
    x += (int64_t)item * x_stride;
    if (prepared) {
      const float4 p4 = __ldg(reinterpret_cast<const float4*>(x + g * kGroup + 4 * lane));
      v[0] = p4.x;
      v[1] = p4.y;
      v[2] = p4.z;
      v[3] = p4.w;
    } else {
      prepare_group_warp(x, input_size, g, v);
    }
  }
  uint32_t hi[2], lo[2];
  split2(v[0], v[1], hi[0], lo[0]);
  split2(v[2], v[3], hi[1], lo[1]);
  const int c = 4 * lane, half = c >> 6, k = c & 63;
  uint8_t* tile = act + ((size_t)g * 2 + half) * (size_t)(2 * N) * 128;
  *reinterpret_cast<uint2*>(tile + sw128(n, k)) = make_uint2(hi[0], hi[1]);
  *reinterpret_cast<uint2*>(tile + sw128(N + n, k)) = make_uint2(lo[0], lo[1]);
}

template <int BITS>
__global__ void __launch_bounds__(kTcThreads, 1) k_cq_gemm_tc(
    const uint8_t* __restrict__ packed, const uint16_t* __restrict__ norms, int32_t rows, int32_t groups,
    int32_t row_bytes, const uint8_t* __restrict__ act_all, int32_t N, int32_t batch, int32_t groups_per_split,
    float* __restrict__ out, int32_t out_stride, int64_t split_stride, Codebook cb, uint32_t* __restrict__ wait_words) {
  constexpr int kCodes = BITS == 4 ? 16 : BITS == 3 ? 8 : 4;
  constexpr int kGroupWords = BITS == 4 ? 16 : BITS == 3 ? 12 : 8;  // packed 32-bit words of one row's group
  constexpr int kPairsPerWord = BITS == 4 ? 4 : 8;  // column pairs (two codes) per packed word (2, 4 bits)
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t a_full[kTcMaxSlots];  // 4 decode-warp arrivals
  __shared__ __align__(8) uint64_t b_full[kTcMaxSlots];  // producer arrival + copied bytes
  __shared__ __align__(8) uint64_t empty[kTcMaxSlots];   // MMA commit: slot read
  __shared__ __align__(8) uint64_t acc_full;             // MMA commit: accumulator final
  __shared__ uint32_t tmem_base;
  __shared__ float lut[16];
  __shared__ int s_failed;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mt = blockIdx.x, split = blockIdx.y, zt = blockIdx.z;  // row tile, K split, item tile
  const int nb = min(N, batch - zt * N);                              // items of this tile
  const uint8_t* act = act_all + (size_t)zt * groups * 2 * (2 * N) * 128;
  const int g_begin = split * groups_per_split, g_end = min(groups, g_begin + groups_per_split);
  const int ng = g_end - g_begin;
  const int nslots = kTcSlotsUsed;
  const uint32_t acc_cols = kTcAccCols;
  const bool doubled = N <= 64;  // A_hi x [B_hi; B_lo] as one MMA of 2N columns
  const uint32_t half_bytes = (uint32_t)(2 * N) * 128;  // activation tile of one 64-column half
  const uint32_t group_bytes = 2 * half_bytes;
  // shared memory: activation ring [slot][half][head rows | tail rows] (1024-aligned), split tables
  const uint32_t b_sm = (saddr(smem_raw) + 1023u) & ~1023u;
  uint32_t* table = reinterpret_cast<uint32_t*>(smem_raw + (b_sm - saddr(smem_raw)) + (size_t)nslots * group_bytes);

  if (tid < 16) {
    float v = 0.0f;
    if constexpr (BITS == 4) {
#pragma unroll
      for (int k = 0; k < 16; k++) v = tid == k ? cb.v[12 + k] : v;
    } else if constexpr (BITS == 3) {
#pragma unroll
      for (int k = 0; k < 8; k++) v = tid == k ? cb.v[4 + k] : v;
    } else if constexpr (BITS == 2) {
#pragma unroll
      for (int k = 0; k < 4; k++) v = tid == k ? cb.v[k] : v;
    } else {
      // ternary crumbs 0..3 are the trits 0, +c, 0, -c (cq_index / cq_level)
      const float c = f32(kTernaryCentroid * (1.0 / sqrt((double)kGroup)));
      v = tid == 1 ? c : tid == 3 ? -c : 0.0f;
    }
    lut[tid] = v;
  }
  if (tid == 0) {
    for (int i = 0; i < kTcMaxSlots; i++) {
      bar_init(&a_full[i], 4);
      bar_init(&b_full[i], 1);
      bar_init(&empty[i], 1);
    }
    bar_init(&acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_failed = 0;
  }
  if (warp == kTcMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&tmem_base)),
                 "r"(kTcCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;

  if (warp == kTcCopyWarp) {
    // ---- producer: activations of group g_begin + gi into slot gi % nslots
    if (lane == 0) {
      bool failed = false;
      int issued = 0;
      for (int gi = 0; gi < ng; gi++) {
        const int sl = gi % nslots;
        if (gi >= nslots && !bar_wait(&empty[sl], (uint32_t)((gi / nslots - 1) & 1))) {
          failed = true;
          break;
        }
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(&b_full[sl])),
                     "r"(group_bytes)
                     : "memory");
        bulk_load(b_sm + sl * group_bytes, act + (size_t)(g_begin + gi) * group_bytes, group_bytes, &b_full[sl]);
        issued = gi + 1;
      }
      if (failed) {
        atomicExch(&s_failed, 1);
        // copies may still be landing: wait for the last one of each slot (bounded) before retiring
        for (int gi = max(0, issued - nslots); gi < issued; gi++)
          bar_wait(&b_full[gi % nslots], (uint32_t)((gi / nslots) & 1));
      }
    }
    __syncwarp();
  } else if (warp == kTcMmaWarp) {
    // ---- MMA issue: the whole warp waits (converged); the elected lane issues a group's MMAs back to
    // back from precomputed operands, so that the warp spends few issue slots next to the decoders
    const uint32_t idesc2 = f16_idesc(2 * N), idesc1 = f16_idesc(N);
    const bool leader = elect_one();
    const uint64_t half_units = half_bytes >> 4;  // descriptor start-address units of one half
    bool failed = false;
    for (int gi = 0; gi < ng; gi++) {
      const int sl = gi % nslots;
      const uint32_t par = (uint32_t)((gi / nslots) & 1);
      // the leader polls (many polling lanes would only add shared-memory traffic)
      const bool ok = !leader || (bar_wait(&b_full[sl], par) && bar_wait(&a_full[sl], par));
      if (!__all_sync(0xffffffffu, ok)) {
        failed = true;
        break;
      }
      if (leader) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_hi = tmem + acc_cols + sl * 128, a_lo = a_hi + 64;
        const uint64_t d0 = sw128_desc(b_sm + sl * group_bytes), d1 = d0 + half_units;
        // K-step kk: 8 A columns; activation half kk / 4 at 32 bytes (2 descriptor units) per step
#pragma unroll
        for (int kk = 0; kk < kGroup / 16; kk++) {
          const uint64_t bd = (kk < 4 ? d0 : d1) + (uint64_t)((kk & 3) * 2);
          const uint32_t first = (gi > 0 || kk > 0) ? 1u : 0u;
          if (doubled) {
            mma_ts(tmem, a_hi + kk * 8, bd, idesc2, first);  // [hh | hl] in columns [0, 2N)
            mma_ts(tmem, a_lo + kk * 8, bd, idesc2, 1u);     // += [lh | ll]
          } else {
            mma_ts(tmem, a_hi + kk * 8, bd, idesc1, first);                    // hh
            mma_ts(tmem, a_hi + kk * 8, bd + (uint64_t)(N * 8), idesc1, 1u);  // += hl (tail rows N..2N-1)
            mma_ts(tmem, a_lo + kk * 8, bd, idesc1, 1u);                       // += lh
            mma_ts(tmem, a_lo + kk * 8, bd + (uint64_t)(N * 8), idesc1, 1u);  // += ll
          }
        }
        mma_commit(&empty[sl]);
      }
      __syncwarp();
    }
    if (failed && lane == 0) atomicExch(&s_failed, 1);
    if (leader) mma_commit(&acc_full);  // arrives once every MMA issued above has completed
    __syncwarp();
  } else {
    // ---- decode: team t takes groups t, t + teams, ...; thread = one tile row
    const int team = warp >> 2, quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int grow = mt * kTcM + row;
    const bool row_ok = grow < rows;
    const uint8_t* rowp = packed + (int64_t)(row_ok ? grow : 0) * row_bytes;
    const uint16_t* nrow = norms + (int64_t)(row_ok ? grow : 0) * groups;
    uint32_t* tab = table + tid;  // entry c of this thread's table at tab[c * kTcDecodeThreads]
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    // one team per ring slot, so that the uses of a slot, and the phases of its barriers, follow one
    // team's program order
    const int teams = nslots;
    const int n_mine = team < teams && ng > team ? (ng - team + teams - 1) / teams : 0;
    uint32_t wr[kTcPrefetch][kGroupWords];
    float nr[kTcPrefetch];
    auto load_group = [&](int d, int j) {
      const int g = g_begin + team + teams * j;
      const uint4* src = reinterpret_cast<const uint4*>(rowp + (int64_t)g * (kGroupWords * 4));
#pragma unroll
      for (int q = 0; q < kGroupWords / 4; q++) {
        const uint4 u = row_ok ? __ldg(src + q) : make_uint4(0, 0, 0, 0);
        wr[d][4 * q] = u.x;
        wr[d][4 * q + 1] = u.y;
        wr[d][4 * q + 2] = u.z;
        wr[d][4 * q + 3] = u.w;
      }
      nr[d] = row_ok ? __half2float(__ushort_as_half(__ldg(nrow + g))) : 0.0f;
    };
#pragma unroll
    for (int d = 0; d < kTcPrefetch; d++)
      if (d < n_mine) load_group(d, d);
    bool failed = false;
    for (int j0 = 0; j0 < n_mine && !failed; j0 += kTcPrefetch) {
#pragma unroll
      for (int d = 0; d < kTcPrefetch; d++) {
        const int j = j0 + d;
        if (j >= n_mine || failed) break;
        const int sl = team;  // group team + teams * j
        // split table of this row's group: level * norm * 2^10 as fp16 head | tail, two codes at a time
#pragma unroll
        for (int c = 0; c < kCodes; c += 2) {
          uint32_t h2, l2;
          split2(__fmul_rn(__fmul_rn(lut[c], nr[d]), kTcWeightScale),
                 __fmul_rn(__fmul_rn(lut[c + 1], nr[d]), kTcWeightScale), h2, l2);
          tab[c * kTcDecodeThreads] = __byte_perm(h2, l2, 0x5410);
          tab[(c + 1) * kTcDecodeThreads] = __byte_perm(h2, l2, 0x7632);
        }
        // pairs 16q .. 16q + 15 (columns 32q .. 32q + 31) of the group as head and tail words; the
        // low and high codes of each packed byte are first split into separate byte lanes
        auto decode16 = [&](int q, uint32_t* hi, uint32_t* lo) {
          if constexpr (BITS == 3) {
            // 3-bit bitstream: pairs 16q .. 16q + 15 are the 96 bits of words 3q .. 3q + 2, pair j the
            // 6-bit field at bit 6j (low code first)
            const uint32_t* w3 = &wr[d][3 * q];
#pragma unroll
            for (int j = 0; j < 16; j++) {
              const int bit = 6 * j, wi = bit >> 5, sh = bit & 31;
              const uint32_t field = wi < 2 ? __funnelshift_r(w3[wi], w3[wi + 1], sh) : (w3[2] >> sh);
              const uint32_t t0 = tab[(field & 7u) * kTcDecodeThreads], t1 = tab[((field >> 3) & 7u) * kTcDecodeThreads];
              hi[j] = __byte_perm(t0, t1, 0x5410);
              lo[j] = __byte_perm(t0, t1, 0x7632);
            }
          } else {
#pragma unroll
            for (int wi = 0; wi < 16 / kPairsPerWord; wi++) {
              const uint32_t w = wr[d][q * (16 / kPairsPerWord) + wi];
#pragma unroll
              for (int i = 0; i < kPairsPerWord; i++) {
                uint32_t c0, c1;
                if constexpr (BITS == 4) {
                  const uint32_t t = w & 0x0F0F0F0Fu, u = (w >> 4) & 0x0F0F0F0Fu;
                  c0 = __byte_perm(t, 0, 0x4440 | i);
                  c1 = __byte_perm(u, 0, 0x4440 | i);
                } else {
                  const uint32_t t = w & 0x33333333u, u = (w >> 2) & 0x33333333u;
                  c0 = (t >> (4 * i)) & 3u;
                  c1 = (u >> (4 * i)) & 3u;
                }
                const uint32_t t0 = tab[c0 * kTcDecodeThreads], t1 = tab[c1 * kTcDecodeThreads];
                hi[wi * kPairsPerWord + i] = __byte_perm(t0, t1, 0x5410);
                lo[wi * kPairsPerWord + i] = __byte_perm(t0, t1, 0x7632);
              }
            }
          }
        };
        const uint32_t col = lane_addr + acc_cols + sl * 128;
        uint32_t hi[16], lo[16];
        decode16(0, hi, lo);
        // lane 0 waits for the MMAs that last read this slot; the outcome is made warp-uniform
        // (tcgen05.st is a warp instruction)
        if (j > 0 && lane == 0) failed = !bar_wait(&empty[sl], (uint32_t)((j - 1) & 1));
        failed = __any_sync(0xffffffffu, failed);
        if (failed) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        tmem_st16(col, hi);
        tmem_st16(col + 64, lo);
#pragma unroll
        for (int q = 1; q < 4; q++) {
          decode16(q, hi, lo);
          tmem_st16(col + 16 * q, hi);
          tmem_st16(col + 64 + 16 * q, lo);
        }
        if (j + kTcPrefetch < n_mine) load_group(d, j + kTcPrefetch);  // wr[d] fully used
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) bar_arrive(&a_full[sl]);
      }
    }
    if (failed) atomicExch(&s_failed, 1);
    // epilogue: wait for the last MMA; this warp's 32 rows x every third 8-column chunk (y = columns
    // [0, N), plus [N, 2N) when the head x tail products went there)
    const bool acc_ok = __all_sync(0xffffffffu, lane != 0 || bar_wait(&acc_full, 0));
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const bool bad = !acc_ok || *(volatile int*)&s_failed != 0;
    if (bad && lane == 0) report_wait_timeout(wait_words, kWaitTensorGemm);
    float* o = out + (int64_t)split * split_stride + (int64_t)zt * N * out_stride;
    for (int c0 = team * 8; c0 < N; c0 += kTcTeams * 8) {
      uint32_t v[8], w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      tmem_ld8(lane_addr + (uint32_t)c0, v);
      if (doubled) tmem_ld8(lane_addr + (uint32_t)(N + c0), w);
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < 8; j++)
          if (c0 + j < nb)
            o[(int64_t)(c0 + j) * out_stride + grow] =
                bad ? NAN : __fmul_rn(__fadd_rn(__uint_as_float(v[j]), __uint_as_float(w[j])), 1.0f / kTcWeightScale);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == kTcMmaWarp) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
  }
}

// y[n][r] = sum over splits s, in order, of part[s][n][r].
__global__ void k_splitk_sum(const float* __restrict__ part, int32_t splits, int64_t split_stride, int32_t rows,
                             int32_t nb, float* __restrict__ y, int32_t y_stride) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)rows * nb) return;
  const int n = (int)(i / rows), r = (int)(i - (int64_t)n * rows);
  float v = __ldg(part + i);
  for (int s = 1; s < splits; s++) v = __fadd_rn(v, __ldg(part + (int64_t)s * split_stride + i));
  y[(int64_t)n * y_stride + r] = v;
}

struct TcPlan {
  int m_tiles, groups, per, used;  // row tiles, groups, groups per split, splits
  int N, z;                        // items per tile (MMA N) and item tiles
};

// Rows of at most kTcGroupSplitMax groups (the engine's 512-input projections) accumulate each
// group separately -- one group per CTA, split-K -- and k_splitk_sum adds the groups' partials with
// IEEE binary32 adds in a fixed order: the tensor pipe's fp32 accumulation over a whole 512-input row
// (32 MMAs into one accumulator) measured 1.9e-6 relative error against 1.2e-7 per group, and the
// decode step amplifies that difference past the 1e-3 logits bar.  The item tile (16, 32, 64, 128)
// is then the smallest that keeps the grid within one CTA per SM.  Longer rows take all items in
// one tile (up to 128; a second tile would decode every weight again) and split K over the SMs.
constexpr int kTcGroupSplitMax = 8;

TcPlan plan_for(int32_t rows, int32_t in_pad, int32_t batch, int sms) {
  TcPlan p;
  p.m_tiles = (rows + kTcM - 1) / kTcM;
  p.groups = in_pad / kGroup;
  int splits;
  if (p.groups <= kTcGroupSplitMax) {
    const int64_t per_tile = (int64_t)p.m_tiles * p.groups;
    p.N = kTcMaxN;
    for (int n = 16; n <= kTcMaxN; n *= 2)
      if (per_tile * ((batch + n - 1) / n) <= sms) {
        p.N = n;
        break;
      }
    splits = p.groups;
  } else {
    p.N = kTcMaxN;
    splits = std::max(1, std::min(p.groups, sms / p.m_tiles));
  }
  p.N = std::min(p.N, std::max(16, (batch + 15) / 16 * 16));
  p.z = (batch + p.N - 1) / p.N;
  p.per = (p.groups + splits - 1) / splits;
  p.used = (p.groups + p.per - 1) / p.per;
  return p;
}

}  // namespace

int cq_gemm_tc_splits(int32_t rows, int32_t input_size, int32_t batch, int32_t sms) {
  return plan_for(rows, (input_size + kGroup - 1) / kGroup * kGroup, batch, sms).used;
}

bool cq_gemm_tc_supported(int32_t bits) { return bits == 2 || bits == 3 || bits == 4 || bits == kTernaryBits; }

// From 16 items the GEMM beats the table GEMV (one weight pass per 8 items) on every shape; for
// matrices of 4M weights and more already from 6 items (measured on the config-2 shapes).
bool cq_gemm_tc_preferred(int32_t rows, int32_t input_size, int32_t batch) {
  const int64_t in_pad = (input_size + kGroup - 1) / kGroup * kGroup;
  return batch >= kTcMinBatch || (batch >= 6 && (int64_t)rows * in_pad >= (int64_t(1) << 22));
}

size_t cq_gemm_tc_scratch_bytes(int32_t rows, int32_t input_size, int32_t batch, int32_t sms) {
  const int in_pad = (input_size + kGroup - 1) / kGroup * kGroup;
  const TcPlan p = plan_for(rows, in_pad, batch, sms);
  const size_t act = (size_t)p.z * p.groups * 2 * (2 * p.N) * 128;
  const size_t part = p.used > 1 ? (size_t)p.used * batch * rows * 4 : 0;
  return act + part;
}

cudaError_t launch_cq_gemm_tc(const uint8_t* packed, const uint16_t* norms, int32_t rows, int32_t input_size,
                              int32_t bits, const float* x, int32_t x_stride, int32_t prepared, int32_t batch, float* y,
                              int32_t y_stride, const Codebook& cb, void* scratch, int32_t sms, cudaStream_t s) {
  if (batch <= 0 || rows <= 0) return cudaSuccess;
  const int in_pad = (input_size + kGroup - 1) / kGroup * kGroup;
  const int pb = bits == kTernaryBits ? 2 : bits;
  const int row_bytes = in_pad * pb / 8;
  const TcPlan p = plan_for(rows, in_pad, batch, sms);
  const int N = p.N;
  uint8_t* act = static_cast<uint8_t*>(scratch);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  uint32_t* wait_words = wait_status_words(dev);
  const int64_t warps = (int64_t)p.groups * N * p.z;
  k_cq_prep_f16<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(x, x_stride, input_size, p.groups, batch, N, p.z, prepared,
                                                           act);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t act_bytes = (size_t)p.z * p.groups * 2 * (2 * N) * 128;
  float* part = reinterpret_cast<float*>(act + act_bytes);
  const int64_t split_stride = (int64_t)batch * rows;  // partials [split][item][row]
  const size_t smem = std::max(kTcMinSmem, (size_t)kTcSlotsUsed * 2 * (2 * N) * 128 + kTcTableBytes + 1024);
  auto launch = [&](auto kernel) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return;
    float* o = p.used > 1 ? part : y;
    kernel<<<dim3(p.m_tiles, p.used, p.z), kTcThreads, smem, s>>>(packed, norms, rows, p.groups, row_bytes, act, N, batch,
                                                                 p.per, o, p.used > 1 ? rows : y_stride, split_stride, cb,
                                                                 wait_words);
    e = cudaGetLastError();
  };
  if (bits == 4) launch(k_cq_gemm_tc<4>);
  else if (bits == 3) launch(k_cq_gemm_tc<3>);
  else if (bits == 2) launch(k_cq_gemm_tc<2>);
  else if (bits == kTernaryBits) launch(k_cq_gemm_tc<kTernaryBits>);
  else return cudaErrorInvalidValue;
  if (e != cudaSuccess) return e;
  if (p.used > 1) {
    const int64_t n = (int64_t)rows * batch;
    k_splitk_sum<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, p.used, split_stride, rows, batch, y, y_stride);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace needle
