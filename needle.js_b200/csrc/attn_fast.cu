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
#include <cuda_runtime.h>

#include "engine.cuh"

namespace needle {

namespace {

constexpr int kFastThreads = 128;
constexpr int kSplit = 1024;     // positions per CTA
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
    int32_t capacity, int32_t splits, Partial* __restrict__ partials) {
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

  const int64_t head_row = ((int64_t)b * kKvHeads + h) * capacity;
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

// Merges the splits of every (item, KV head): out = sum_s 2^(m_s - M) acc_s / sum_s 2^(m_s - M) l_s.
__global__ void __launch_bounds__(kFastThreads) k_attention_fast_combine(const Partial* __restrict__ partials,
                                                                         int32_t splits, float* __restrict__ out) {
  const int b = blockIdx.x, h = blockIdx.y;
  const int hh = threadIdx.x >> 6, d = threadIdx.x & 63;
  const Partial* p = partials + ((int64_t)b * kKvHeads + h) * splits;
  float M = -INFINITY;
  for (int s = 0; s < splits; s++) M = fmaxf(M, p[s].m[hh]);
  float L = 0.0f, A = 0.0f;
  for (int s = 0; s < splits; s++) {
    if (p[s].m[hh] == -INFINITY) continue;
    const float f = exp2f(p[s].m[hh] - M);
    L += p[s].l[hh] * f;
    A += p[s].acc[hh][d] * f;
  }
  out[(int64_t)b * kHeads * kHeadDim + (2 * h + hh) * kHeadDim + d] = L > 0.0f ? A / L : 0.0f;
}

}  // namespace

size_t attention_fast_scratch_bytes(int32_t batch, int32_t capacity) {
  const int splits = (capacity + kSplit - 1) / kSplit;
  return sizeof(Partial) * (size_t)batch * kKvHeads * splits;
}

cudaError_t launch_attention_fast(const float* q, const int8_t* kc, const float* ks, const int8_t* vc,
                                  const float* vs, const int32_t* counts, int32_t batch, int32_t capacity,
                                  float* out, void* scratch, cudaStream_t s) {
  if (batch <= 0) return cudaSuccess;
  const int splits = (capacity + kSplit - 1) / kSplit;
  Partial* parts = static_cast<Partial*>(scratch);
  k_attention_fast<<<dim3(batch, kKvHeads, splits), kFastThreads, 0, s>>>(q, kc, ks, vc, vs, counts, capacity,
                                                                         splits, parts);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_attention_fast_combine<<<dim3(batch, kKvHeads), kFastThreads, 0, s>>>(parts, splits, out);
  return cudaGetLastError();
}

}  // namespace needle
