// cq_fast.cu -- fast-numerics Cactus-Quant matvec (binary32, table lookups).  Computes
// cqMatvec (packages/needle.js/src/backends/cq.ts:233-240 = prepareCqActivation + cqMatvecPrepared,
// cq.ts:30-46 and 107-231) in binary32 with its own summation order, so results match the
// reference within binary32 rounding instead of bit for bit.  Record widths 4, 2 and ternary.
//
// Why tables.  At batch 1 the matvec streams each weight byte once, so HBM sets the floor
// (~5 us for 8192x8192 CQ4); a straightforward decode spends one codebook lookup plus one FMA per
// weight, and the lookups alone (one shared-memory access each) cap the SM below the rate HBM
// delivers.  The reference already works a byte at a time: for a 128-column group its inner step
// adds lut[byte] . x[pair or quad] (cq.ts:146-152, 170-175, 192-197).  With x fixed per call that
// whole term depends on the byte alone, so each CTA builds, for one group, the table
//     T[b][j] = sum_i level(code_i(b)) * x'[j * codes_per_byte + i]      (b < 256)
// (64 KB: 64 pairs for CQ4, 32 quads for CQ2 / ternary), and a byte of weights then costs one
// table read and one add -- half or a quarter of a lookup per weight.
//
// Work: the (group, block of 32 rows) pairs in group-major order, a contiguous range per CTA, so a
// CTA rebuilds its table only where its range crosses a group.  Each warp keeps its next block of
// weights in flight in registers (the first one is issued before the table is built).  The group's activation slice is
// prepared in the CTA (zero padding, FWHT in binary32 butterflies, scale by 1/sqrt(128) in
// binary64 -- the same values k_cq_prepare produces), so a call is one launch.
//
// Lookup phase: one lane per row, streaming the row's 64 (CQ4) or 32 (CQ2) bytes of the group as
// 16-byte loads (fully used sectors).  Table rows are 64 floats apart, so the bank of T[b][j] is
// j mod 32 whatever b is; lanes walk their chunks and bytes from lane-specific starting points,
// which makes the 32 lanes of every step read 32 different j -- no bank conflicts for any weights.
//
// Reduction: each block writes the group dot per (group, row) to scratch, and k_cq_fast_reduce sums
// norm * dot over the groups of every row in a fixed order; the result does not depend on
// scheduling.  (Fusing it behind a grid barrier in a cooperative launch measured slower: the
// cooperative launch costs more than the second kernel.)
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "cq.cuh"

namespace needle {

namespace {

constexpr int kTabThreads = 256;                 // 8 warps, two CTAs per SM
constexpr int kTabStride = 64;                   // floats per table byte-row
constexpr int kTabFloats = 256 * kTabStride;     // 64 KB
constexpr int kRing = 3;                         // 32-row weight blocks per warp in its copy ring
constexpr int kSlotBytes = 2048;                 // one block: 32 rows x 64 bytes (CQ4) or 32 bytes
constexpr int kRingBytes = kRing * kSlotBytes * (kTabThreads / 32);  // 48 KB per CTA
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // a copy wait gives up after 2 s
// A table build (inputs, FWHT, 64 KB of stores, barriers) costs about as much time as this many
// 32-row blocks of lookups (measured: CTAs with a second table ran ~2 us = ~18 blocks longer).
constexpr int kTableCost = 18;

template <int BITS>
struct TabGeom {
  static constexpr int codes_per_byte = BITS == 4 ? 2 : 4;
  static constexpr int group_bytes = kGroup / codes_per_byte;    // 64 or 32
  static constexpr int chunks = group_bytes / 16;                // 16-byte chunks per group row: 4 or 2
};

template <int BITS>
__device__ __forceinline__ void build_table(const float v[4], const float* __restrict__ lut, float* __restrict__ T) {
  const int t = threadIdx.x;
  static_assert(kTabThreads == 256, "table build assumes 256 threads");
  if constexpr (BITS == 4) {
    const int j = t & 63, lo_blk = t >> 6;  // pair j; low nibbles 4 lo_blk .. 4 lo_blk + 3
    // x'[2j] and x'[2j+1] live in lane j / 2 (elements 0, 1 or 2, 3)
    const int src = j >> 1;
    const float e0 = __shfl_sync(0xffffffffu, v[0], src), e1 = __shfl_sync(0xffffffffu, v[1], src);
    const float e2 = __shfl_sync(0xffffffffu, v[2], src), e3 = __shfl_sync(0xffffffffu, v[3], src);
    const float x0 = (j & 1) ? e2 : e0, x1 = (j & 1) ? e3 : e1;
    float p0[4], p1[16];
#pragma unroll
    for (int k = 0; k < 4; k++) p0[k] = lut[4 * lo_blk + k] * x0;
#pragma unroll
    for (int h = 0; h < 16; h++) p1[h] = lut[h] * x1;
    float* base = T + (4 * lo_blk) * kTabStride + j;
#pragma unroll
    for (int h = 0; h < 16; h++)
#pragma unroll
      for (int k = 0; k < 4; k++) base[(h * 16 + k) * kTabStride] = p0[k] + p1[h];
  } else {
    const int j = t & 31, hb = t >> 5;  // quad j = this lane; bytes 32 hb .. 32 hb + 31
    const float x0 = v[0], x1 = v[1], x2 = v[2], x3 = v[3];
    float p0[4], p1[4];
#pragma unroll
    for (int c = 0; c < 4; c++) {
      p0[c] = lut[c] * x0;
      p1[c] = lut[c] * x1;
    }
    const float s3 = lut[hb >> 1] * x3;                     // code of bits 6-7 = hb >> 1
    const float s23a = lut[(2 * hb) & 3] * x2 + s3;         // bits 4-5 for k < 16
    const float s23b = lut[(2 * hb + 1) & 3] * x2 + s3;     // and for k >= 16
    float* base = T + (32 * hb) * kTabStride + j;
#pragma unroll
    for (int k = 0; k < 32; k++) base[k * kTabStride] = (p0[k & 3] + p1[(k >> 2) & 3]) + (k < 16 ? s23a : s23b);
  }
}

// Rotates the 16 bytes of c so that byte s of the result is byte (s + rot) & 15 of c
// (selects and funnel shifts, no branches).
__device__ __forceinline__ void rotate16(const uint4 c, int rot, uint32_t o[4]) {
  const bool r1 = rot & 4, r2 = rot & 8;
  const uint32_t b0 = r1 ? c.y : c.x, b1 = r1 ? c.z : c.y, b2 = r1 ? c.w : c.z, b3 = r1 ? c.x : c.w;
  const uint32_t a0 = r2 ? b2 : b0, a1 = r2 ? b3 : b1, a2 = r2 ? b0 : b2, a3 = r2 ? b1 : b3;
  const uint32_t sh = 8u * (rot & 3);
  o[0] = __funnelshift_r(a0, a1, sh);
  o[1] = __funnelshift_r(a1, a2, sh);
  o[2] = __funnelshift_r(a2, a3, sh);
  o[3] = __funnelshift_r(a3, a0, sh);
}

// Sum of T over the 16 bytes of a rotated chunk.  pk packs the 16 byte-row offsets of the steps,
// three per word (the fourth byte is zero); one byte permute per step builds byte * 256 + offset.
__device__ __forceinline__ float lookup16(const char* __restrict__ Tc, const uint32_t o[4], const uint32_t pk[6]) {
  // two packed binary32 pairs (add.rn.f32x2) accumulate steps s and s + 1
  unsigned long long acc[2] = {0ull, 0ull};
#pragma unroll
  for (int s = 0; s < 16; s += 2) {
    float v[2];
#pragma unroll
    for (int e = 0; e < 2; e++) {
      const int st = s + e;
      // bytes of the offset: [offset of step st, weight byte st, 0, 0]
      const uint32_t sel = 0x7700u | ((uint32_t)(st & 3) << 4) | (4u + (uint32_t)(st % 3));
      const uint32_t at = __byte_perm(o[st >> 2], pk[st / 3], sel);
      v[e] = *reinterpret_cast<const float*>(Tc + at);
    }
    unsigned long long pair;
    asm("mov.b64 %0, {%1, %2};" : "=l"(pair) : "f"(v[0]), "f"(v[1]));
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(acc[(s >> 1) & 1]) : "l"(acc[(s >> 1) & 1]), "l"(pair));
  }
  unsigned long long t;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(t) : "l"(acc[0]), "l"(acc[1]));
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(t));
  return lo + hi;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
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
// Waits for the phase with the given parity; false once kWaitLimitNs has passed without it.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t start;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(start));
  for (;;) {
    for (int i = 0; i < 32; i++)
      if (mbar_try_wait(bar, parity)) return true;
    uint64_t now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    if (now - start > kWaitLimitNs) return false;
  }
}

template <int BITS>
__global__ void __launch_bounds__(kTabThreads, 2) k_cq_gemv_table(
    const __grid_constant__ CUtensorMap wmap, int32_t rows, int32_t input_size, int32_t in_pad,
    const float* __restrict__ x, int32_t x_stride, Codebook cb, float* __restrict__ partials,
    uint32_t* __restrict__ wait_words) {
  using G = TabGeom<BITS>;
  constexpr int NCH = G::chunks;
  constexpr int kWarps = kTabThreads / 32;
  constexpr uint32_t kBlockBytes = 32u * G::group_bytes;
  // Dynamic shared memory: the warps' weight rings (512-byte aligned, as the swizzled copies need),
  // then the table.
  extern __shared__ __align__(16) unsigned char dyn_smem[];
  __shared__ float lut[16];
  __shared__ __align__(8) uint64_t full[kWarps][kRing];
  float* T = reinterpret_cast<float*>(dyn_smem + ((((smem_u32(dyn_smem) + 511u) & ~511u) - smem_u32(dyn_smem)) +
                                                  kRingBytes));  // kTabFloats
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int item = blockIdx.y;
  const int groups = in_pad / kGroup;
  const int nblk = (rows + 31) / 32;  // 32-row blocks per group
  // Contiguous block ranges of equal cost: every group of many blocks is counted as kTableCost
  // blocks longer (its table build), so a CTA whose range crosses into another group gets that many
  // fewer blocks.  (Groups of few blocks are split evenly: there every CTA builds one table.)
  const int64_t tcost = nblk >= 128 ? kTableCost : 0;
  const int64_t per_group = nblk + tcost, cost = (int64_t)groups * per_group;
  auto block_at = [&](int64_t p) {
    const int64_t gq = p / per_group;
    return gq * nblk + max((int64_t)0, p - gq * per_group - tcost);
  };
  const int64_t b_begin = block_at(cost * blockIdx.x / gridDim.x), b_end = block_at(cost * (blockIdx.x + 1) / gridDim.x);
  x += (int64_t)item * x_stride;
  float* part = partials + (int64_t)item * groups * rows;
  if (tid < 16) {
    float v = 0.0f;
    if constexpr (BITS == 4) {
#pragma unroll
      for (int k = 0; k < 16; k++) v = tid == k ? cb.v[12 + k] : v;  // static indices: cb stays in param space
    } else if constexpr (BITS == 2) {
#pragma unroll
      for (int k = 0; k < 4; k++) v = tid == k ? cb.v[k] : v;
    } else {
      const float c = f32(kTernaryCentroid / sqrt((double)kGroup));
      v = tid == 1 ? c : tid == 3 ? -c : 0.0f;
    }
    lut[tid] = v;
  }

  if (lane == 0) {
    for (int r = 0; r < kRing; r++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[warp][r])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // Per-warp ring of 32-row weight blocks filled by the tensor-copy engine (box: the group's bytes
  // of 32 rows; rows past the matrix read as zeros).  Lane i reads row i: 16-byte chunk c sits at
  // slot c ^ ((i >> 1) & 3) (64-byte swizzle, CQ4) or c ^ ((i >> 2) & 1) (32-byte swizzle, CQ2 /
  // ternary), so the chunk reads of eight consecutive lanes hit eight distinct bank groups.
  const uint32_t ring0 = (smem_u32(dyn_smem) + 511u) & ~511u;
  const uint32_t ring_base = ring0 + (uint32_t)warp * kRing * kSlotBytes;
  const uint32_t row_off = (uint32_t)lane * G::group_bytes;
  const int swz = BITS == 4 ? (lane >> 1) & 3 : (lane >> 2) & 1;
  // Blocks this warp has issued / consumed, in the same order: block n uses ring slot n % kRing and
  // completes that slot's phase (n / kRing) & 1.
  int issued = 0, uses = 0;
  bool failed = false;

  // Lane geometry (constant for the kernel).  Lane i owns row i of a 32-row block: its NCH 16-byte
  // chunks of the group, walked in the order (i + p) mod NCH, each starting at byte rot = i / 2.
  // The bank of T[b][j] is j mod 32 = 16 (chunk & 1) + position; at every step the lanes of either
  // chunk parity hold the 16 distinct rotations, so the 32 lanes read 32 distinct banks.
  const int rot = lane >> 1;
  uint32_t pk[NCH][6];  // packed byte-row offsets (three per word) of every phase and step
#pragma unroll
  for (int ph = 0; ph < NCH; ph++)
#pragma unroll
    for (int m = 0; m < 6; m++) {
      uint32_t w = 0;
#pragma unroll
      for (int e = 0; e < 3; e++) {
        const int st = 3 * m + e;
        if (st < 16) w |= (uint32_t)(16 * ((lane + ph) % NCH) + ((st + rot) & 15)) * 4u << (8 * e);
      }
      pk[ph][m] = w;
    }
  const char* Tc = reinterpret_cast<const char*>(T);

  // The CTA's blocks [b_begin, b_end) in group-major order, one segment per group.
  for (int64_t seg = b_begin; seg < b_end;) {
    const int g = (int)(seg / nblk);
    const int64_t seg_end = min(b_end, (int64_t)(g + 1) * nblk);
    const int rb0 = (int)(seg - (int64_t)g * nblk), nseg = (int)(seg_end - seg);
    // lane 0 copies the warp's j-th block of the segment (block warp + j * kWarps) into the next
    // ring slot; that slot's previous block has been read by every lane (the __syncwarp before)
    auto issue = [&](int j) {
      const int k = warp + j * kWarps;
      if (k >= nseg || failed) return;
      const int slot = issued % kRing;
      issued++;
      if (lane != 0) return;
      const uint32_t bar = smem_u32(&full[warp][slot]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kBlockBytes) : "memory");
      asm volatile(
          "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
              ring_base + (uint32_t)slot * kSlotBytes),
          "l"(reinterpret_cast<uint64_t>(&wmap)), "r"(g * G::group_bytes), "r"((rb0 + k) * 32), "r"(bar)
          : "memory");
    };
#pragma unroll
    for (int j = 0; j < kRing - 1; j++) issue(j);  // in flight during the table build
    float xv[4];
    prepare_group_warp(x, input_size, g, xv);
    __syncthreads();  // every warp is done with the previous table (and lut / barriers are set)
    build_table<BITS>(xv, lut, T);
    __syncthreads();
    for (int j = 0; warp + j * kWarps < nseg; j++) {
      __syncwarp();
      issue(j + kRing - 1);
      const int slot = uses % kRing;
      // A copy that has not landed within kWaitLimitNs stops this warp's copies; its remaining
      // rows get NaN partials, so the row totals report the failure instead of stale values.
      if (!failed) failed = !__all_sync(0xffffffffu, mbar_wait(&full[warp][slot], (uint32_t)((uses / kRing) & 1)));
      float sum = NAN;
      if (!failed) {
        uses++;
        const uint32_t src = ring_base + (uint32_t)slot * kSlotBytes + row_off;
        sum = 0.0f;
#pragma unroll
        for (int ph = 0; ph < NCH; ph++) {
          const int c = (lane + ph) % NCH;
          uint4 v;
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                       : "r"(src + 16u * (uint32_t)(c ^ swz))
                       : "memory");
          uint32_t o[4];
          rotate16(v, rot, o);
          sum += lookup16(Tc, o, pk[ph]);
        }
      }
      const int row = (rb0 + warp + j * kWarps) * 32 + lane;
      if (row < rows) part[(int64_t)g * rows + row] = sum;
    }
    seg = seg_end;
  }
  if (failed && lane == 0) {
    report_wait_timeout(wait_words, kWaitTableGemv);
    // Copies still landing in this warp's ring must finish before the CTA retires: wait (bounded)
    // for the blocks issued and not consumed.
    for (int n = uses; n < issued; n++) mbar_wait(&full[warp][n % kRing], (uint32_t)((n / kRing) & 1));
  }
}

// Row totals: y[row] = sum_g norm16[row][g] * partials[g][row].  16 rows per CTA, 16 threads per row
// each summing every 16th group (so a 64-group row costs each thread four independent loads), the
// 16 partial sums combined in a fixed order: the result does not depend on scheduling.
constexpr int kReduceRows = 16;
constexpr int kReduceThreads = 256;
__global__ void __launch_bounds__(kReduceThreads) k_cq_fast_reduce(const float* __restrict__ partials,
                                                                   const uint16_t* __restrict__ norms, int32_t rows,
                                                                   int32_t groups, float* __restrict__ y,
                                                                   int32_t y_stride) {
  constexpr int kSub = kReduceThreads / kReduceRows;
  __shared__ float red[kSub][kReduceRows];
  const int tid = threadIdx.x, item = blockIdx.y;
  const int rl = tid % kReduceRows, sub = tid / kReduceRows;
  const int r = blockIdx.x * kReduceRows + rl;
  const float* part = partials + (int64_t)item * groups * rows;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (r < rows) {
    const uint16_t* nr = norms + (int64_t)r * groups;
    for (int gg = sub; gg < groups; gg += 4 * kSub) {
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int gk = gg + k * kSub;
        if (gk < groups)
          acc[k] += __half2float(__ushort_as_half(__ldg(nr + gk))) * __ldcg(part + (int64_t)gk * rows + r);
      }
    }
  }
  red[sub][rl] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  __syncthreads();
  if (sub == 0 && r < rows) {
    float v = red[0][rl];
#pragma unroll
    for (int k = 1; k < kSub; k++) v += red[k][rl];
    y[(int64_t)item * y_stride + r] = v;
  }
}

// 2D map of a packed CQ matrix [rows][row_bytes] with boxes of one group's bytes x 32 rows, 64-byte
// (CQ4) or 32-byte (CQ2 / ternary) swizzle.  The encoder comes from the driver through the
// runtime's entry-point query.
bool encode_weight_map(CUtensorMap* map, const uint8_t* packed, int64_t rows, int64_t row_bytes, int group_bytes) {
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
  const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)group_bytes, 32u};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(packed), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, group_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BITS>
cudaError_t launch_table(const uint8_t* packed, const uint16_t* norms, int32_t rows, int32_t input_size,
                         int32_t in_pad, const float* x, int32_t batch, float* y, const Codebook& cb,
                         float* partials, cudaStream_t s) {
  using G = TabGeom<BITS>;
  static std::atomic<uint64_t> configured{0};
  static int per_sm[64] = {0};
  int device = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return e;
  const size_t smem = sizeof(float) * kTabFloats + kRingBytes + 512;  // + ring alignment slack
  const uint64_t bit = 1ull << (device & 63);
  if (!(configured.load() & bit)) {
    e = cudaFuncSetAttribute(k_cq_gemv_table<BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int n = 1;
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_cq_gemv_table<BITS>, kTabThreads, smem);
    if (e != cudaSuccess) return e;
    per_sm[device & 63] = std::max(1, n);
    configured.fetch_or(bit);
  }
  const int groups = in_pad / kGroup;
  const int64_t total = (int64_t)groups * ((rows + 31) / 32);
  const int pb = BITS == kTernaryBits ? 2 : BITS;
  const int row_bytes = in_pad * pb / 8;
  CUtensorMap wmap;
  if (!encode_weight_map(&wmap, packed, rows, row_bytes, G::group_bytes)) return cudaErrorInvalidValue;
  for (int b0 = 0; b0 < batch; b0 += kFastMaxItems) {
    const int nb = std::min(kFastMaxItems, batch - b0);
    const int slots = sms * per_sm[device & 63];
    // one wave of CTAs over the items of the pass; at least one CTA per group (one table build
    // each) and, beyond that, at least one block per warp
    const int64_t want = std::max<int64_t>(groups, (total + kTabThreads / 32 - 1) / (kTabThreads / 32));
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>({total, want, (int64_t)std::max(1, slots / nb)}));
    const float* xb = x + (int64_t)b0 * input_size;
    float* yb = y + (int64_t)b0 * rows;
    k_cq_gemv_table<BITS><<<dim3(grid, nb), kTabThreads, smem, s>>>(wmap, rows, input_size, in_pad, xb,
                                                                     input_size, cb, partials,
                                                                     wait_status_words(device));
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    k_cq_fast_reduce<<<dim3((rows + kReduceRows - 1) / kReduceRows, nb), kReduceThreads, 0, s>>>(
        partials, norms, rows, groups, yb, rows);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

bool cq_gemv_fast_supported(int32_t bits) { return bits == 2 || bits == 4 || bits == kTernaryBits; }

size_t cq_gemv_fast_partial_floats(int32_t rows, int32_t in_pad) {
  return (size_t)kFastMaxItems * (in_pad / kGroup) * rows;
}

cudaError_t launch_cq_gemv_fast(const uint8_t* packed, const uint16_t* norms, int32_t rows, int32_t input_size,
                                int32_t bits, const float* x, int32_t batch, float* y, const Codebook& cb,
                                float* partials, cudaStream_t s) {
  if (batch <= 0 || rows <= 0) return cudaSuccess;
  const int in_pad = (input_size + kGroup - 1) / kGroup * kGroup;
  if (bits == 4) return launch_table<4>(packed, norms, rows, input_size, in_pad, x, batch, y, cb, partials, s);
  if (bits == 2) return launch_table<2>(packed, norms, rows, input_size, in_pad, x, batch, y, cb, partials, s);
  if (bits == kTernaryBits)
    return launch_table<kTernaryBits>(packed, norms, rows, input_size, in_pad, x, batch, y, cb, partials, s);
  return cudaErrorInvalidValue;
}

}  // namespace needle
