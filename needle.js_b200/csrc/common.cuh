// common.cuh -- shared definitions of the needle_cuda engine (sm_100a).
//
// Numerics.  The reference CPU backend evaluates every expression in binary64 (a JS `number`)
// and rounds to binary32 only when it stores into a Float32Array.  The engine's exact kernels do
// the same, operation for operation.  The library is compiled with --fmad=false, so a * b + c is
// never contracted; where a fused multiply-add is used on purpose (fma()), the product is exact in
// binary64 (binary32 x binary32, or binary32 x int8), so fma(a, b, c) == round(round(a*b) + c).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace needle {

// Needle 2 geometry this engine is specialised for (packages/needle.js/src/resident/
// compatibility.ts:8-16 gates the reference's resident WebGPU engine on the same values).
constexpr int kDim = 512;        // model dimension
constexpr int kHeadDim = 64;     // attention head dimension
constexpr int kHeads = 8;        // query heads
constexpr int kKvHeads = 4;      // key/value heads (GQA x2)
constexpr int kLanes = 4;        // mHC lanes
constexpr int kLaneWidth = kLanes * kDim;
constexpr int kGroup = 128;      // Cactus-Quant group size
constexpr int kHadamard = 512;   // Hadamard MLP dimension
constexpr int kMaxSites = 4;     // engram sites (cact.ts:211-217)
constexpr int kMaxTables = 8;    // engram tables supported
constexpr int kEngramDepth = 10; // (taps - 1) * max order + 1 for taps 4, orders {2,3}
constexpr int kTernaryBits = 5;  // record-width marker of ternary matrices (cq.ts:5)
constexpr double kTernaryCentroid = 1.2240064;  // cq.ts:6

// Exact binary64 -> binary32 store (a Float32Array assignment).
__device__ __forceinline__ float f32(double v) { return __double2float_rn(v); }

// fp16 norm widened exactly (float16ToNumber, packages/needle.js/src/model/fp16.ts:5-32).
__device__ __forceinline__ double norm16(const uint16_t* norms, int64_t index) {
  return (double)__half2float(__ushort_as_half(__ldg(norms + index)));
}

// sigmoid (packages/needle.js/src/model/math.ts:3-10) in binary64.
__device__ __forceinline__ double sigmoid_d(double v) {
  if (v >= 0.0) {
    const double e = exp(-v);
    return 1.0 / (1.0 + e);
  }
  const double e = exp(v);
  return e / (1.0 + e);
}

// In-place fast Walsh-Hadamard transform over `groups` consecutive blocks of `len` floats in
// shared memory (fastWalshHadamard, packages/needle.js/src/backends/cq.ts:8-27).  Each butterfly
// is a binary32 add/sub, which equals the reference's binary64 add rounded to binary32 (double
// rounding is innocuous for + and - because 53 >= 2 * 24 + 2).  Every butterfly of a stage is
// independent, so the order in which threads run them does not change any value.
// Must be called by all threads of the block.
__device__ __forceinline__ void fwht_smem(float* v, int len, int groups) {
  const int pairs = (len >> 1) * groups;
  for (int stride = 1; stride < len; stride <<= 1) {
    for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
      const int g = p / (len >> 1);
      const int q = p - g * (len >> 1);
      const int base = (q / stride) * (stride << 1);
      const int inner = q % stride;
      const int l = g * len + base + inner;
      const int r = l + stride;
      const float a = v[l], b = v[r];
      v[l] = __fadd_rn(a, b);
      v[r] = __fsub_rn(a, b);
    }
    __syncthreads();
  }
}

// Sequential binary64 sum of squares (the `sumSquares += value * value` loops of rmsNorm /
// rmsUnit, math.ts:16-44) run by one thread.  value*value is exact in binary64, so each step is
// fma(v, v, s) == round(s + v*v).
__device__ __forceinline__ double sum_squares_seq(const float* v, int n) {
  double s = 0.0;
#pragma unroll 8
  for (int i = 0; i < n; i++) {
    const double x = (double)v[i];
    s = fma(x, x, s);
  }
  return s;
}

}  // namespace needle
