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

// In-place FWHTs of consecutive blocks of `len` values (power of two, >= 32), one value per thread:
// threads [0, active) hold the values (active a multiple of len).  Strides below 32 run in
// registers with warp shuffles, larger strides through shared memory `v` (>= active floats).
// Same butterflies, same binary32 results as fwht_smem.  Every thread of the block calls it.
__device__ __forceinline__ float fwht_reg(float mine, float* v, int len, int active) {
  const int t = threadIdx.x;
  const int lane = t & 31;
#pragma unroll
  for (int stride = 1; stride < 32; stride <<= 1) {
    const float other = __shfl_xor_sync(0xffffffffu, mine, stride);
    mine = (lane & stride) ? __fsub_rn(other, mine) : __fadd_rn(mine, other);
  }
  for (int stride = 32; stride < len; stride <<= 1) {
    if (t < active) v[t] = mine;
    __syncthreads();
    if (t < active) {
      const float other = v[t ^ stride];
      mine = (t & stride) ? __fsub_rn(other, mine) : __fadd_rn(mine, other);
    }
    __syncthreads();
  }
  return mine;
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

// Sequential binary64 sum of n precomputed terms, in index order (one thread).  The terms are
// staged in shared memory by the whole block first, so the dependent chain is one add per term;
// the next eight terms are loaded while the current eight are added.
__device__ __forceinline__ double sum_seq(const double* terms, int n) {
  double s = 0.0;
  int i = 0;
  if (n >= 8) {
    double2 a = *reinterpret_cast<const double2*>(terms);
    double2 b = *reinterpret_cast<const double2*>(terms + 2);
    double2 c = *reinterpret_cast<const double2*>(terms + 4);
    double2 d = *reinterpret_cast<const double2*>(terms + 6);
#pragma unroll 1
    for (; i + 16 <= n; i += 8) {
      const double2 na = *reinterpret_cast<const double2*>(terms + i + 8);
      const double2 nb = *reinterpret_cast<const double2*>(terms + i + 10);
      const double2 nc = *reinterpret_cast<const double2*>(terms + i + 12);
      const double2 nd = *reinterpret_cast<const double2*>(terms + i + 14);
      s = s + a.x;
      s = s + a.y;
      s = s + b.x;
      s = s + b.y;
      s = s + c.x;
      s = s + c.y;
      s = s + d.x;
      s = s + d.y;
      a = na;
      b = nb;
      c = nc;
      d = nd;
    }
    s = s + a.x;
    s = s + a.y;
    s = s + b.x;
    s = s + b.y;
    s = s + c.x;
    s = s + c.y;
    s = s + d.x;
    s = s + d.y;
    i += 8;
  }
  for (; i < n; i++) s = s + terms[i];
  return s;
}

// Exact binary64 value of a small integer (|v| < 2^31) through the FP64 add pipe instead of the
// conversion unit: the bit pattern 0x4338000000000000 + v is the double 2^52 + 2^51 + v.
__device__ __forceinline__ double int_to_double_exact(int v) {
  return __longlong_as_double(0x4338000000000000LL + (long long)v) - 6755399441055744.0;
}

// v rounded to binary32 (ties to even) and widened back: the value of (double)f32(v).
__device__ __forceinline__ double round32_cvt(double v) { return (double)__double2float_rn(v); }

// The same value without the conversion unit (which issues a quarter as many operations per clock
// as the FP64 add pipe).  With 2^e <= |v| < 2^(e+1) and e clamped to >= -126 (the binary32
// subnormal spacing below), c = 1.5 * 2^(e+29) is an even number of binary32 ulps of v and one
// binary64 ulp of v + c is one binary32 ulp of v, so v + c rounds v to binary32 precision with
// ties to even and subtracting c is exact.  Requires |v| < 2^127 (no binary32 overflow).
__device__ __forceinline__ double round32_add(double v) {
  const int hi = __double2hiint(v);
  const int ch = max(hi & 0x7ff00000, 897 << 20) + ((29 << 20) | 0x00080000);
  const double c = __hiloint2double(ch, 0);
  return (v + c) - c;
}

// Bounded device waits that ran out.  Every kernel that waits on a copy or a barrier gives up
// after a time limit; it then records its kind in the library's wait-status words of the device
// (mapped pinned host memory, so the host reads them without synchronising) and its outputs of
// that call are NaN.  The next operator call on the device reports BACKEND_UNAVAILABLE.
enum WaitKind { kWaitAttention = 0, kWaitTableGemv = 1, kWaitTensorGemm = 2, kWaitSelftest = 3, kWaitKinds = 4 };

__device__ __forceinline__ void report_wait_timeout(uint32_t* words, int kind) {
  if (words) *reinterpret_cast<volatile uint32_t*>(words + kind) = 1u;
}

// The wait-status words of a device (kWaitKinds of them), allocated on first use; nullptr if the
// pinned mapping cannot be made.
uint32_t* wait_status_words(int device);

}  // namespace needle
