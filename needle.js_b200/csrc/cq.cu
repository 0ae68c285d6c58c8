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
#include <algorithm>
#include <atomic>

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

constexpr int kRowsPerThread = 2;

// Dot products of kRowsPerThread rows (same group) against kBT items.  xg points at this warp's
// group inside item 0 of the staged [kBT][512] binary64 inputs; every x operand is loaded once
// and used for both rows.
template <int BITS>
__device__ __forceinline__ void group_dots(const uint32_t (&w)[kRowsPerThread][GroupBytes<BITS>::value / 4 + 1],
                                           const double* lut, const double* __restrict__ xg, int nb,
                                           double (&dot)[kRowsPerThread][kBT]) {
#pragma unroll
  for (int r = 0; r < kRowsPerThread; r++)
#pragma unroll
    for (int b = 0; b < kBT; b++) dot[r][b] = 0.0;
  if constexpr (BITS == 2 || BITS == kTernaryBits) {
    // 32 bytes per row: 4 columns per byte, low crumb first.  Fully unrolled so every word index
    // is a compile-time constant and the weights stay in registers.
#pragma unroll
    for (int byte_i = 0; byte_i < 32; byte_i++) {
      double a[kRowsPerThread][4];
#pragma unroll
      for (int r = 0; r < kRowsPerThread; r++) {
        const uint32_t byte = (w[r][byte_i >> 2] >> ((byte_i & 3) * 8)) & 0xffu;
        a[r][0] = lut[byte & 3];
        a[r][1] = lut[(byte >> 2) & 3];
        a[r][2] = lut[(byte >> 4) & 3];
        a[r][3] = lut[(byte >> 6) & 3];
      }
      const int c = byte_i * 4;
#pragma unroll
      for (int b = 0; b < kBT; b++) {
        if (b < nb) {
          const double2 x01 = *reinterpret_cast<const double2*>(xg + b * 512 + c);
          const double2 x23 = *reinterpret_cast<const double2*>(xg + b * 512 + c + 2);
#pragma unroll
          for (int r = 0; r < kRowsPerThread; r++) {
            double s;
            if constexpr (BITS == 2) {
              // codebook levels are binary32: every product is exact, so fma == add(product)
              s = a[r][0] * x01.x;
              s = fma(a[r][1], x01.y, s);
              s = fma(a[r][2], x23.x, s);
              s = fma(a[r][3], x23.y, s);
            } else {
              // ternary levels are binary64 (1.2240064 / sqrt(g)): round every product
              s = a[r][0] * x01.x;
              s = s + a[r][1] * x01.y;
              s = s + a[r][2] * x23.x;
              s = s + a[r][3] * x23.y;
            }
            dot[r][b] = dot[r][b] + s;
          }
        }
      }
    }
  } else if constexpr (BITS == 4) {
#pragma unroll
    for (int byte_i = 0; byte_i < 64; byte_i++) {
      double a[kRowsPerThread][2];
#pragma unroll
      for (int r = 0; r < kRowsPerThread; r++) {
        const uint32_t byte = (w[r][byte_i >> 2] >> ((byte_i & 3) * 8)) & 0xffu;
        a[r][0] = lut[byte & 15];
        a[r][1] = lut[byte >> 4];
      }
      const int c = byte_i * 2;
#pragma unroll
      for (int b = 0; b < kBT; b++) {
        if (b < nb) {
          const double2 x01 = *reinterpret_cast<const double2*>(xg + b * 512 + c);
#pragma unroll
          for (int r = 0; r < kRowsPerThread; r++) {
            double s = a[r][0] * x01.x;
            s = fma(a[r][1], x01.y, s);
            dot[r][b] = dot[r][b] + s;
          }
        }
      }
    }
  } else {  // 3-bit: dot = round(dot + level * x) per column, exact products; two columns a step
#pragma unroll
    for (int c = 0; c < kGroup; c += 2) {
      double a[kRowsPerThread][2];
#pragma unroll
      for (int r = 0; r < kRowsPerThread; r++)
#pragma unroll
        for (int k = 0; k < 2; k++) {
          const int bit = (c + k) * 3;
          const int wi = bit >> 5, sh = bit & 31;
          uint32_t v = w[r][wi] >> sh;
          if (sh > 29) v |= w[r][wi + 1] << (32 - sh);
          a[r][k] = lut[v & 7];
        }
#pragma unroll
      for (int b = 0; b < kBT; b++)
        if (b < nb) {
          const double2 x = *reinterpret_cast<const double2*>(xg + b * 512 + c);
#pragma unroll
          for (int r = 0; r < kRowsPerThread; r++) {
            dot[r][b] = fma(a[r][0], x.x, dot[r][b]);
            dot[r][b] = fma(a[r][1], x.y, dot[r][b]);
          }
        }
    }
  }
}

template <int BITS>
__global__ void __launch_bounds__(kGemvThreads)
k_cq_gemv(const CqJobs jobs, const Codebook cb, int32_t n_host, const int32_t* n_dev) {
  constexpr int kTileRows = kRowsPerTile * kRowsPerThread;  // 64
  extern __shared__ __align__(16) unsigned char smem_raw[];
  double* xs = reinterpret_cast<double*>(smem_raw);          // [kBT][512]
  double* dsm = xs + kBT * 512;                              // [kBT][4][64]
  double* lut = dsm + kBT * kGroupsPerChunk * kTileRows;     // [16]

  const int n = item_count(n_host, n_dev);
  const int item_tiles = (n + kBT - 1) / kBT;
  const int units = jobs.total_tiles * item_tiles;
  const int lane = threadIdx.x & 31;
  const int gc = threadIdx.x >> 5;  // group within the chunk
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

  // Persistent loop over (row tile, item tile) units; consecutive units share an item tile.
#pragma unroll 1
  for (int unit = blockIdx.x; unit < units; unit += gridDim.x) {
    const int gtile = unit % jobs.total_tiles;
    const int b0 = (unit / jobs.total_tiles) * kBT;
    const int nb = min(kBT, n - b0);
    int j = 0;
#pragma unroll 1
    for (int k = 1; k < jobs.count; k++)
      if (gtile >= jobs.job[k].tile_begin) j = k;
    const CqJob& job = jobs.job[j];
    const int tile = gtile - job.tile_begin;
    const int groups = job.in_pad / kGroup;

    // Totals owned by this thread: pairs (tile row, item) = threadIdx.x + k * 128.
    constexpr int kPairs = kTileRows * kBT / kGemvThreads;  // 4
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
      double dot[kRowsPerThread][kBT];
      constexpr int kWords = GroupBytes<BITS>::value / 4;
      uint32_t w[kRowsPerThread][kWords + 1];
      bool any = false;
#pragma unroll
      for (int r = 0; r < kRowsPerThread; r++) {
        const int r_local = tile * kTileRows + r * 32 + lane;
        const bool ok = gc < gn && r_local < job.rows;
        any |= ok;
        const uint4* src = reinterpret_cast<const uint4*>(
            job.packed + ((int64_t)job.row_start + r_local) * job.row_bytes + (int64_t)(g0 + gc) * GroupBytes<BITS>::value);
#pragma unroll
        for (int q = 0; q < kWords / 4; q++) {
          const uint4 u = ok ? __ldg(src + q) : make_uint4(0, 0, 0, 0);
          w[r][4 * q] = u.x;
          w[r][4 * q + 1] = u.y;
          w[r][4 * q + 2] = u.z;
          w[r][4 * q + 3] = u.w;
        }
        w[r][kWords] = 0;
      }
      if (any) {
        group_dots<BITS>(w, lut, xs + gc * kGroup, nb, dot);
      } else {
#pragma unroll
        for (int r = 0; r < kRowsPerThread; r++)
#pragma unroll
          for (int b = 0; b < kBT; b++) dot[r][b] = 0.0;
      }
#pragma unroll
      for (int r = 0; r < kRowsPerThread; r++)
#pragma unroll
        for (int b = 0; b < kBT; b++) dsm[(b * kGroupsPerChunk + gc) * kTileRows + r * 32 + lane] = dot[r][b];
      __syncthreads();
      // total += norm * dot, group by group in order (cq.ts:151).
#pragma unroll
      for (int k = 0; k < kPairs; k++) {
        const int pair = threadIdx.x + k * kGemvThreads;
        const int rl = pair % kTileRows, b = pair / kTileRows;
        const int64_t prow = (int64_t)job.row_start + tile * kTileRows + rl;
        if (b < nb && tile * kTileRows + rl < job.rows) {
          double t = total[k];
          for (int q = 0; q < gn; q++) {
            const double nrm = norm16(job.norms, prow * groups + g0 + q);
            t = t + nrm * dsm[(b * kGroupsPerChunk + q) * kTileRows + rl];
          }
          total[k] = t;
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kPairs; k++) {
      const int pair = threadIdx.x + k * kGemvThreads;
      const int rl = pair % kTileRows, b = pair / kTileRows;
      const int r = tile * kTileRows + rl;
      if (b < nb && r < job.rows) job.y[(int64_t)(b0 + b) * job.y_stride + r] = f32(total[k]);
    }
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
  return sizeof(double) * (kBT * 512 + kBT * kGroupsPerChunk * kRowsPerTile * kRowsPerThread + 16);
}

// Opts the GEMV instantiations into more than 48 KB of dynamic shared memory, once per device.
static cudaError_t configure_gemv() {
  static std::atomic<uint64_t> done{0};
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (device & 63);
  if (done.load() & bit) return cudaSuccess;
  const int smem = (int)gemv_smem();
  if ((e = cudaFuncSetAttribute(k_cq_gemv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(k_cq_gemv<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(k_cq_gemv<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(k_cq_gemv<5>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
  done.fetch_or(bit);
  return cudaSuccess;
}

// CTAs of k_cq_gemv that fit on the device at once (the persistent grid size).
static int gemv_resident_ctas() {
  static std::atomic<int> cached[64];
  int device = 0;
  cudaGetDevice(&device);
  int v = cached[device & 63].load();
  if (v > 0) return v;
  int per_sm = 0, sms = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_cq_gemv<2>, kGemvThreads, gemv_smem());
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  v = std::max(1, per_sm) * std::max(1, sms);
  cached[device & 63].store(v);
  return v;
}

cudaError_t launch_cq_gemv(const CqJobs& jobs, const Codebook& cb, int32_t n_host,
                           const int32_t* n_dev, cudaStream_t s) {
  if (n_host <= 0 || jobs.count <= 0) return cudaSuccess;
  cudaError_t ce = configure_gemv();
  if (ce != cudaSuccess) return ce;
  const int bits = jobs.job[0].bits;
  for (int k = 1; k < jobs.count; k++)
    if (jobs.job[k].bits != bits) return cudaErrorInvalidValue;
  const int units = jobs.total_tiles * ((n_host + kBT - 1) / kBT);
  dim3 grid(std::min(units, gemv_resident_ctas()));
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


// ------------------------------------------------------------------ split-group GEMV (small batch)
//
// For few items and long rows a (row tile, item tile) unit is too coarse to fill the GPU: the
// 8192 x 8192 stress matrix at batch 1 has 128 units for 148 SMs.  Here each unit is one
// (64-row tile, 4-group chunk): its per-(row, group) dots go to scratch, and k_cq_group_totals then
// forms every row's total over its groups in order -- the same operations, in the same order, as
// the single-pass kernel.
namespace {

template <int BITS>
__global__ void __launch_bounds__(kGemvThreads)
k_cq_group_dots(const CqJob job, const Codebook cb, int32_t n, double* __restrict__ dots) {
  constexpr int kTileRows = kRowsPerTile * kRowsPerThread;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  double* xs = reinterpret_cast<double*>(smem_raw);  // [kBT][512]
  double* lut = xs + kBT * 512;                      // [16]
  const int lane = threadIdx.x & 31, gc = threadIdx.x >> 5;
  const int groups = job.in_pad / kGroup;
  const int chunks = (groups + kGroupsPerChunk - 1) / kGroupsPerChunk;
  const int tiles = (job.rows + kTileRows - 1) / kTileRows;
  const int units = tiles * chunks;
  if (threadIdx.x < 16) {
    double v = 0.0;
    if (BITS == kTernaryBits) {
      const double coefficient = kTernaryCentroid / sqrt((double)kGroup);
      const int t = threadIdx.x;
      v = (t == 1) ? coefficient : (t == 3) ? -coefficient : 0.0;
    } else if (threadIdx.x < (1 << BITS)) {
      v = (double)cb.v[(BITS == 2 ? 0 : BITS == 3 ? 4 : 12) + threadIdx.x];
    }
    lut[threadIdx.x] = v;
  }
#pragma unroll 1
  for (int unit = blockIdx.x; unit < units; unit += gridDim.x) {
    const int chunk = unit % chunks, tile = unit / chunks;  // neighbouring CTAs share rows
    const int g0 = chunk * kGroupsPerChunk;
    const int gn = min(kGroupsPerChunk, groups - g0);
    const int nb = n;  // n <= kBT
    __syncthreads();
    for (int idx = threadIdx.x; idx < nb * gn * kGroup; idx += kGemvThreads) {
      const int b = idx / (gn * kGroup);
      const int c = idx - b * gn * kGroup;
      xs[b * 512 + c] = (double)job.x[(int64_t)b * job.x_stride + g0 * kGroup + c];
    }
    __syncthreads();
    if (gc >= gn) continue;
    constexpr int kWords = GroupBytes<BITS>::value / 4;
    uint32_t w[kRowsPerThread][kWords + 1];
#pragma unroll
    for (int r = 0; r < kRowsPerThread; r++) {
      const int r_local = tile * kTileRows + r * 32 + lane;
      const bool ok = r_local < job.rows;
      const uint4* src = reinterpret_cast<const uint4*>(job.packed + ((int64_t)job.row_start + r_local) * job.row_bytes +
                                                        (int64_t)(g0 + gc) * GroupBytes<BITS>::value);
#pragma unroll
      for (int q = 0; q < kWords / 4; q++) {
        const uint4 u = ok ? __ldg(src + q) : make_uint4(0, 0, 0, 0);
        w[r][4 * q] = u.x;
        w[r][4 * q + 1] = u.y;
        w[r][4 * q + 2] = u.z;
        w[r][4 * q + 3] = u.w;
      }
      w[r][kWords] = 0;
    }
    double dot[kRowsPerThread][kBT];
    group_dots<BITS>(w, lut, xs + gc * kGroup, nb, dot);
#pragma unroll
    for (int r = 0; r < kRowsPerThread; r++) {
      const int r_local = tile * kTileRows + r * 32 + lane;
      if (r_local >= job.rows) continue;
#pragma unroll
      for (int b = 0; b < kBT; b++)
        if (b < nb) dots[((int64_t)b * job.rows + r_local) * groups + g0 + gc] = dot[r][b];
    }
  }
}

// total = sum_g norm[g] * dot[g] in group order (cq.ts:137-153), one thread per (row, item).
__global__ void k_cq_group_totals(const CqJob job, int32_t n, const double* __restrict__ dots) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)n * job.rows) return;
  const int b = int(idx / job.rows), r = int(idx - (int64_t)b * job.rows);
  const int groups = job.in_pad / kGroup;
  const double* d = dots + ((int64_t)b * job.rows + r) * groups;
  const int64_t row = (int64_t)job.row_start + r;
  double total = 0.0;
  for (int g = 0; g < groups; g++) total = total + norm16(job.norms, row * groups + g) * d[g];
  job.y[(int64_t)b * job.y_stride + r] = f32(total);
}

template <int BITS>
cudaError_t split_launch(const CqJob& job, const Codebook& cb, int32_t n, double* scratch, cudaStream_t s) {
  constexpr int kTileRows = kRowsPerTile * kRowsPerThread;
  const size_t smem = sizeof(double) * (kBT * 512 + 16);
  const int groups = job.in_pad / kGroup;
  const int units = ((job.rows + kTileRows - 1) / kTileRows) * ((groups + kGroupsPerChunk - 1) / kGroupsPerChunk);
  int per_sm = 0, sms = 0, device = 0;
  cudaGetDevice(&device);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_cq_group_dots<BITS>, kGemvThreads, smem);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int grid = std::min(units, std::max(1, per_sm) * std::max(1, sms));
  k_cq_group_dots<BITS><<<grid, kGemvThreads, smem, s>>>(job, cb, n, scratch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t threads = (int64_t)n * job.rows;
  k_cq_group_totals<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(job, n, scratch);
  return cudaGetLastError();
}

}  // namespace

size_t cq_gemv_split_scratch_bytes(const CqJob& job, int32_t n) {
  return sizeof(double) * (size_t)n * job.rows * (job.in_pad / kGroup);
}

bool cq_gemv_prefers_split(const CqJob& job, int32_t n) {
  return n >= 1 && n <= kBT && job.in_pad / kGroup >= 16;
}

cudaError_t launch_cq_gemv_split(const CqJob& job, const Codebook& cb, int32_t n, double* scratch, cudaStream_t s) {
  if (n <= 0 || job.rows <= 0) return cudaSuccess;
  if (n > kBT) return cudaErrorInvalidValue;
  switch (job.bits) {
    case 2: return split_launch<2>(job, cb, n, scratch, s);
    case 3: return split_launch<3>(job, cb, n, scratch, s);
    case 4: return split_launch<4>(job, cb, n, scratch, s);
    case 5: return split_launch<5>(job, cb, n, scratch, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace needle
