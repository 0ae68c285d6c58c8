// cq.cu -- Cactus-Quant kernels (exact numerics).
//
//   k_cq_prepare  prepareCqActivation (packages/needle.js/src/backends/cq.ts:30-46)
//   k_cq_gemv     cqMatvecPrepared   (cq.ts:107-231), batched over items and several matrices
//   k_cq_rows     dequantizeCqRow    (cq.ts:243-295)
//
// GEMV decomposition.  The reference accumulates each (row, 128-group) dot product sequentially
// in binary64 -- four (2-bit, ternary), two (4-bit) or one (3-bit) column(s) per inner step --
// and then sums norm * dot over the groups of the row in order.  One thread owns one
// (row, group) dot for a tile of BT items, so the weights are decoded once and reused BT times;
// a warp covers 32 consecutive rows of the same group, so every x operand it reads from shared
// memory is a broadcast.  Groups are consumed in chunks of four (512 inputs), each chunk's dots
// are folded into the per-(row, item) totals in group order, which keeps the reference's
// summation order for any input length.
#include "cq.cuh"

namespace needle {

namespace {

constexpr int kRowsPerTile = 32;
constexpr int kGroupsPerChunk = 4;
constexpr int kGemvThreads = kRowsPerTile * kGroupsPerChunk;  // 128
constexpr int kBT = 8;                                        // items per CTA

__device__ __forceinline__ int item_count(int n_host, const int32_t* n_dev) {
  return n_dev ? *n_dev : n_host;
}

// ------------------------------------------------------------------ prepare

// One CTA per (item, 128-group): copy with zero padding, FWHT, multiply by 1/sqrt(128) in binary64.
__global__ void k_cq_prepare(const float* __restrict__ x, int32_t x_stride, int32_t input_size,
                             int32_t in_pad, float* __restrict__ out, int32_t out_stride,
                             int32_t n_host, const int32_t* n_dev) {
  __shared__ float v[kGroup];
  const int item = blockIdx.y;
  if (item >= item_count(n_host, n_dev)) return;
  const int g = blockIdx.x;
  const float* xi = x + (int64_t)item * x_stride;
  for (int c = threadIdx.x; c < kGroup; c += blockDim.x) {
    const int col = g * kGroup + c;
    v[c] = col < input_size ? xi[col] : 0.0f;
  }
  __syncthreads();
  fwht_smem(v, kGroup, 1);
  const double inverse_root = 1.0 / sqrt((double)kGroup);
  float* o = out + (int64_t)item * out_stride + g * kGroup;
  for (int c = threadIdx.x; c < kGroup; c += blockDim.x) o[c] = f32((double)v[c] * inverse_root);
}

// ------------------------------------------------------------------ GEMV

template <int BITS>
struct GroupBytes {
  static constexpr int value = BITS == 4 ? 64 : BITS == 3 ? 48 : 32;  // 128 columns
};

// Dot products of one (row, group) against kBT items; xs holds [kBT][512] binary64 inputs of the
// current chunk, `xg` points at this warp's group inside item 0.
template <int BITS>
__device__ __forceinline__ void group_dots(const uint32_t* __restrict__ w, const double* lut,
                                           const double* __restrict__ xg, int nb, double* dot) {
#pragma unroll
  for (int b = 0; b < kBT; b++) dot[b] = 0.0;
  if constexpr (BITS == 2 || BITS == kTernaryBits) {
    // 32 bytes: 4 columns per byte, low crumb first.  Fully unrolled so that every word index
    // is a compile-time constant (the weights stay in registers).
#pragma unroll
    for (int byte_i = 0; byte_i < 32; byte_i++) {
      const uint32_t byte = (w[byte_i >> 2] >> ((byte_i & 3) * 8)) & 0xffu;
      const double a0 = lut[byte & 3], a1 = lut[(byte >> 2) & 3];
      const double a2 = lut[(byte >> 4) & 3], a3 = lut[(byte >> 6) & 3];
      const int c = byte_i * 4;
#pragma unroll
      for (int b = 0; b < kBT; b++) {
        if (b < nb) {
          const double2 x01 = *reinterpret_cast<const double2*>(xg + b * 512 + c);
          const double2 x23 = *reinterpret_cast<const double2*>(xg + b * 512 + c + 2);
          double s;
          if constexpr (BITS == 2) {
            // codebook levels are binary32: every product is exact, so fma == add(product)
            s = a0 * x01.x;
            s = fma(a1, x01.y, s);
            s = fma(a2, x23.x, s);
            s = fma(a3, x23.y, s);
          } else {
            // ternary levels are binary64 (1.2240064 / sqrt(g)): round every product
            s = a0 * x01.x;
            s = s + a1 * x01.y;
            s = s + a2 * x23.x;
            s = s + a3 * x23.y;
          }
          dot[b] = dot[b] + s;
        }
      }
    }
  } else if constexpr (BITS == 4) {
#pragma unroll
    for (int byte_i = 0; byte_i < 64; byte_i++) {
      const uint32_t byte = (w[byte_i >> 2] >> ((byte_i & 3) * 8)) & 0xffu;
      const double a0 = lut[byte & 15], a1 = lut[byte >> 4];
      const int c = byte_i * 2;
#pragma unroll
      for (int b = 0; b < kBT; b++) {
        if (b < nb) {
          const double2 x01 = *reinterpret_cast<const double2*>(xg + b * 512 + c);
          double s = a0 * x01.x;
          s = fma(a1, x01.y, s);
          dot[b] = dot[b] + s;
        }
      }
    }
  } else {  // 3-bit: one column per step, dot = round(dot + level * x) with an exact product
#pragma unroll
    for (int c = 0; c < kGroup; c++) {
      const int bit = c * 3;
      const int wi = bit >> 5, sh = bit & 31;
      uint32_t v = w[wi] >> sh;
      if (sh > 29) v |= w[wi + 1] << (32 - sh);
      const double a = lut[v & 7];
#pragma unroll
      for (int b = 0; b < kBT; b++)
        if (b < nb) dot[b] = fma(a, xg[b * 512 + c], dot[b]);
    }
  }
}

template <int BITS>
__global__ void __launch_bounds__(kGemvThreads)
k_cq_gemv(const CqJobs jobs, const Codebook cb, int32_t n_host, const int32_t* n_dev) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  double* xs = reinterpret_cast<double*>(smem_raw);        // [kBT][512]
  double* dsm = xs + kBT * 512;                            // [kBT][4][32]
  double* lut = dsm + kBT * kGroupsPerChunk * kRowsPerTile;  // [16]

  const int n = item_count(n_host, n_dev);
  const int b0 = blockIdx.y * kBT;
  if (b0 >= n) return;
  const int nb = min(kBT, n - b0);

  // Locate this tile's job.
  int j = 0;
#pragma unroll 1
  for (int k = 1; k < jobs.count; k++)
    if ((int)blockIdx.x >= jobs.job[k].tile_begin) j = k;
  const CqJob& job = jobs.job[j];
  const int tile = blockIdx.x - job.tile_begin;
  const int lane = threadIdx.x & 31;
  const int gc = threadIdx.x >> 5;  // group within the chunk
  const int r_local = tile * kRowsPerTile + lane;
  const bool row_ok = r_local < job.rows;
  const int64_t row = (int64_t)job.row_start + r_local;
  const int groups = job.in_pad / kGroup;

  if (threadIdx.x < 16) {
    double v = 0.0;
    if (BITS == kTernaryBits) {
      const double coefficient = kTernaryCentroid / sqrt((double)kGroup);
      const int t = threadIdx.x;
      v = (t == 1) ? coefficient : (t == 3) ? -coefficient : 0.0;  // crumbs [0, c, 0, -c]
    } else if (threadIdx.x < (1 << BITS)) {
      v = (double)cb.v[(BITS == 2 ? 0 : BITS == 3 ? 4 : 12) + threadIdx.x];
    }
    lut[threadIdx.x] = v;
  }

  // Totals owned by this thread: pairs (row lane, item) = threadIdx.x + k * 128.
  constexpr int kPairs = kRowsPerTile * kBT / kGemvThreads;  // 2
  double total[kPairs];
#pragma unroll
  for (int k = 0; k < kPairs; k++) total[k] = 0.0;

  for (int g0 = 0; g0 < groups; g0 += kGroupsPerChunk) {
    const int gn = min(kGroupsPerChunk, groups - g0);
    __syncthreads();  // previous chunk's xs / dsm fully consumed
    // Stage the chunk's inputs as binary64 (exact widening).
    for (int idx = threadIdx.x; idx < nb * gn * kGroup; idx += kGemvThreads) {
      const int b = idx / (gn * kGroup);
      const int c = idx - b * gn * kGroup;
      xs[b * 512 + c] = (double)job.x[(int64_t)(b0 + b) * job.x_stride + g0 * kGroup + c];
    }
    __syncthreads();
    double dot[kBT];
    if (gc < gn && row_ok) {
      constexpr int kWords = GroupBytes<BITS>::value / 4;
      uint32_t w[kWords + 1];
      const uint4* src = reinterpret_cast<const uint4*>(job.packed + row * job.row_bytes +
                                                        (int64_t)(g0 + gc) * GroupBytes<BITS>::value);
#pragma unroll
      for (int q = 0; q < kWords / 4; q++) {
        const uint4 u = __ldg(src + q);
        w[4 * q] = u.x;
        w[4 * q + 1] = u.y;
        w[4 * q + 2] = u.z;
        w[4 * q + 3] = u.w;
      }
      w[kWords] = 0;
      group_dots<BITS>(w, lut, xs + gc * kGroup, nb, dot);
    } else {
#pragma unroll
      for (int b = 0; b < kBT; b++) dot[b] = 0.0;
    }
#pragma unroll
    for (int b = 0; b < kBT; b++) dsm[(b * kGroupsPerChunk + gc) * kRowsPerTile + lane] = dot[b];
    __syncthreads();
    // total += norm * dot, group by group in order (cq.ts:151).
#pragma unroll
    for (int k = 0; k < kPairs; k++) {
      const int pair = threadIdx.x + k * kGemvThreads;
      const int rl = pair & 31, b = pair >> 5;
      const int64_t prow = (int64_t)job.row_start + tile * kRowsPerTile + rl;
      if (b < nb && tile * kRowsPerTile + rl < job.rows) {
        double t = total[k];
        for (int q = 0; q < gn; q++) {
          const double nrm = norm16(job.norms, prow * groups + g0 + q);
          t = t + nrm * dsm[(b * kGroupsPerChunk + q) * kRowsPerTile + rl];
        }
        total[k] = t;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kPairs; k++) {
    const int pair = threadIdx.x + k * kGemvThreads;
    const int rl = pair & 31, b = pair >> 5;
    const int r = tile * kRowsPerTile + rl;
    if (b < nb && r < job.rows) job.y[(int64_t)(b0 + b) * job.y_stride + r] = f32(total[k]);
  }
}

// ------------------------------------------------------------------ rows

// One CTA per (requested row, group).
__global__ void k_cq_rows(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ norms,
                          int32_t bits, int32_t row_bytes, int32_t in_pad, int32_t input_size,
                          const int32_t* __restrict__ rows, float* __restrict__ out,
                          int32_t out_stride, const Codebook cb) {
  __shared__ float v[kGroup];
  const int k = blockIdx.y, g = blockIdx.x;
  const int64_t row = rows[k];
  const int groups = in_pad / kGroup;
  const double nrm = norm16(norms, row * groups + g);
  const uint8_t* rowp = packed + row * row_bytes;
  for (int c = threadIdx.x; c < kGroup; c += blockDim.x) {
    const int index = cq_index(rowp, bits, g * kGroup + c);
    v[c] = f32(cq_level(cb.v, bits, index) * nrm);
  }
  __syncthreads();
  fwht_smem(v, kGroup, 1);
  const double inverse_root = 1.0 / sqrt((double)kGroup);
  for (int c = threadIdx.x; c < kGroup; c += blockDim.x) {
    const int col = g * kGroup + c;
    if (col < input_size) out[(int64_t)k * out_stride + col] = f32((double)v[c] * inverse_root);
  }
}

}  // namespace

cudaError_t launch_cq_prepare(const float* x, int32_t x_stride, int32_t input_size, int32_t in_pad,
                              float* out, int32_t out_stride, int32_t n_host, const int32_t* n_dev,
                              cudaStream_t s) {
  if (n_host <= 0) return cudaSuccess;
  dim3 grid(in_pad / kGroup, n_host);
  k_cq_prepare<<<grid, 64, 0, s>>>(x, x_stride, input_size, in_pad, out, out_stride, n_host, n_dev);
  return cudaGetLastError();
}

static size_t gemv_smem() {
  return sizeof(double) * (kBT * 512 + kBT * kGroupsPerChunk * kRowsPerTile + 16);
}

cudaError_t launch_cq_gemv(const CqJobs& jobs, const Codebook& cb, int32_t n_host,
                           const int32_t* n_dev, cudaStream_t s) {
  if (n_host <= 0 || jobs.count <= 0) return cudaSuccess;
  const int bits = jobs.job[0].bits;
  for (int k = 1; k < jobs.count; k++)
    if (jobs.job[k].bits != bits) return cudaErrorInvalidValue;
  dim3 grid(jobs.total_tiles, (n_host + kBT - 1) / kBT);
  const size_t smem = gemv_smem();
  switch (bits) {
    case 2: k_cq_gemv<2><<<grid, kGemvThreads, smem, s>>>(jobs, cb, n_host, n_dev); break;
    case 3: k_cq_gemv<3><<<grid, kGemvThreads, smem, s>>>(jobs, cb, n_host, n_dev); break;
    case 4: k_cq_gemv<4><<<grid, kGemvThreads, smem, s>>>(jobs, cb, n_host, n_dev); break;
    case 5: k_cq_gemv<5><<<grid, kGemvThreads, smem, s>>>(jobs, cb, n_host, n_dev); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_cq_rows(const uint8_t* packed, const uint16_t* norms, int32_t bits,
                           int32_t row_bytes, int32_t in_pad, int32_t input_size,
                           const int32_t* rows, int32_t n_rows, float* out, int32_t out_stride,
                           const Codebook& cb, cudaStream_t s) {
  if (n_rows <= 0) return cudaSuccess;
  dim3 grid(in_pad / kGroup, n_rows);
  k_cq_rows<<<grid, 64, 0, s>>>(packed, norms, bits, row_bytes, in_pad, input_size, rows, out,
                                out_stride, cb);
  return cudaGetLastError();
}

}  // namespace needle
