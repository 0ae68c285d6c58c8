// cq_fast.cu -- fast-numerics Cactus-Quant matvec (binary32 FMA, warp reductions).  Computes
// cqMatvec (packages/needle.js/src/backends/cq.ts:233-240) like the exact kernel in cq.cu, but in
// binary32 with a tree summation order, so results match the reference within binary32 rounding
// instead of bit for bit.
//
// Decomposition.  Weights are streamed once from HBM with fully coalesced 16-byte loads: a warp
// owns a row, lane l reads the l-th, (l+32)-th, ... 16-byte chunk of it.  The rotated activation
// (prepared per 128-group by k_cq_prepare) of up to kFastItems items sits in shared memory as
// binary32, the 16 codebook levels in a 64-byte shared table (lanes with different indices hit
// different banks).  Each chunk lies inside one 128-column group, so its partial dot is scaled
// by that group's fp16 norm before it joins the lane's row sum; a butterfly shuffle finishes the
// row.  A persistent grid walks rows; x is staged once per CTA in column tiles.
#include <cuda_runtime.h>

#include <algorithm>

#include "cq.cuh"

namespace needle {

namespace {

constexpr int kFastThreads = 256;  // 8 warps
constexpr int kFastItems = 4;      // items per launch pass
constexpr int kTileCols = 8192;    // columns of x staged per pass (kFastItems x 32 KB)

template <int BITS>
struct FastChunk {
  // columns covered by one 16-byte chunk
  static constexpr int cols = BITS == 4 ? 32 : BITS == 3 ? 0 : 64;
};

// Levels of 16 codes packed in `w` (CQ4: 8 per word, 2 words -> 16 levels).
template <int BITS>
__device__ __forceinline__ float level_of(uint32_t word, int k, const float* lut) {
  if constexpr (BITS == 4) return lut[(word >> (4 * k)) & 15];
  else return lut[(word >> (2 * k)) & 3];
}

template <int BITS>
__global__ void __launch_bounds__(kFastThreads) k_cq_gemv_fast(const uint8_t* __restrict__ packed,
                                                               const uint16_t* __restrict__ norms, int32_t rows,
                                                               int32_t in_pad, int32_t row_bytes,
                                                               const float* __restrict__ xp, int32_t nb,
                                                               float* __restrict__ y, Codebook cb) {
  extern __shared__ __align__(16) float xs[];  // [kFastItems][tile]
  __shared__ float lut[16];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < 16) {
    float v = 0.0f;
    if (BITS == kTernaryBits) {
      const float coefficient = (float)(kTernaryCentroid / sqrt((double)kGroup));
      v = (tid == 1) ? coefficient : (tid == 3) ? -coefficient : 0.0f;
    } else if (tid < (1 << BITS)) {
      v = cb.v[(BITS == 2 ? 0 : 12) + tid];
    }
    lut[tid] = v;
  }
  constexpr int kCols = FastChunk<BITS>::cols;  // columns per 16-byte chunk
  const int groups = in_pad / kGroup;
  const int warps_total = gridDim.x * (kFastThreads / 32);
  for (int c0 = 0; c0 < in_pad; c0 += kTileCols) {
    const int tile = min(kTileCols, in_pad - c0);
    __syncthreads();
    for (int i = tid; i < nb * tile; i += kFastThreads) {
      const int b = i / tile, c = i - b * tile;
      xs[b * kTileCols + c] = xp[(int64_t)b * in_pad + c0 + c];
    }
    __syncthreads();
    const int chunks = tile / kCols;          // 16-byte chunks of this tile in a row
    for (int row = blockIdx.x * (kFastThreads / 32) + warp; row < rows; row += warps_total) {
      const uint4* src = reinterpret_cast<const uint4*>(packed + (int64_t)row * row_bytes + c0 / kCols * 16);
      float acc[kFastItems] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 4
      for (int ch = lane; ch < chunks; ch += 32) {
        const uint4 u = __ldg(src + ch);
        const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
        const int col = ch * kCols;  // within the tile
        const float nrm = __half2float(__ushort_as_half(__ldg(norms + (int64_t)row * groups + (c0 + col) / kGroup)));
        float part[kFastItems] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          constexpr int per_word = BITS == 4 ? 8 : 16;
#pragma unroll
          for (int k = 0; k < per_word; k++) {
            const float a = level_of<BITS>(wv[q], k, lut);
            const int c = col + q * per_word + k;
#pragma unroll
            for (int b = 0; b < kFastItems; b++)
              if (b < nb) part[b] = fmaf(a, xs[b * kTileCols + c], part[b]);
          }
        }
#pragma unroll
        for (int b = 0; b < kFastItems; b++) acc[b] = fmaf(nrm, part[b], acc[b]);
      }
#pragma unroll
      for (int b = 0; b < kFastItems; b++) {
        float v = acc[b];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[b] = v;
      }
      if (lane == 0) {
        for (int b = 0; b < nb; b++) {
          float* dst = y + (int64_t)b * rows + row;
          *dst = c0 == 0 ? acc[b] : *dst + acc[b];
        }
      }
    }
  }
}

}  // namespace

bool cq_gemv_fast_supported(int32_t bits) { return bits == 2 || bits == 4 || bits == kTernaryBits; }

cudaError_t launch_cq_gemv_fast(const uint8_t* packed, const uint16_t* norms, int32_t rows, int32_t in_pad,
                                int32_t bits, const float* xp, int32_t batch, float* y, const Codebook& cb,
                                cudaStream_t s) {
  if (batch <= 0 || rows <= 0) return cudaSuccess;
  const int pb = bits == kTernaryBits ? 2 : bits;
  const int row_bytes = in_pad * pb / 8;
  int device = 0, sms = 0;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  for (int b0 = 0; b0 < batch; b0 += kFastItems) {
    const int nb = std::min(kFastItems, batch - b0);
    // x of nb items: shared memory sized to the pass, so batch-1 calls keep many CTAs per SM
    const size_t smem = sizeof(float) * kTileCols * nb;
    const float* xb = xp + (int64_t)b0 * in_pad;
    float* yb = y + (int64_t)b0 * rows;
    cudaError_t e = cudaSuccess;
    int per_sm = 1;
    auto run = [&](auto kernel) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(sizeof(float) * kTileCols * kFastItems));
      if (e != cudaSuccess) return;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kFastThreads, smem);
      const int grid = std::max(1, std::min((rows + 7) / 8, sms * std::max(1, per_sm)));
      kernel<<<grid, kFastThreads, smem, s>>>(packed, norms, rows, in_pad, row_bytes, xb, nb, yb, cb);
      e = cudaGetLastError();
    };
    if (bits == 4) run(k_cq_gemv_fast<4>);
    else if (bits == 2) run(k_cq_gemv_fast<2>);
    else if (bits == kTernaryBits) run(k_cq_gemv_fast<kTernaryBits>);
    else return cudaErrorInvalidValue;
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace needle
