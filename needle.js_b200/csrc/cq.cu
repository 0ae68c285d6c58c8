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

constexpr int kRowsPerThread = 2;                         // the split-group kernel's tile
constexpr int kTileRows = kRowsPerTile * kRowsPerThread;  // 64

// A (32 R-row, 4-group) weight tile staged in shared memory, [group][row][stride]; the stride is the
// group's bytes + 4, an odd number of words, so the 32 rows a warp reads sit on distinct banks.
template <int BITS, int R = kRowsPerThread>
struct Stage {
  static constexpr int kBytes = GroupBytes<BITS>::value;
  static constexpr int kStride = kBytes + 4;
  static constexpr int kRows = kRowsPerTile * R;
  static constexpr int kSize = kGroupsPerChunk * kRows * kStride;
};

// Both staging loops issue eight global loads before the first shared-memory store: a store
// waits for its load, so one word at a time would pay a full L2 round trip per word.
constexpr int kStageBatch = 8;

template <int BITS, int R = kRowsPerThread>
__device__ __forceinline__ void stage_weights(uint8_t* wt, const CqJob& job, int tile, int g0, int gn) {
  using St = Stage<BITS, R>;
  constexpr int kWords = St::kBytes / 4;
  constexpr int kTileRows = St::kRows;
  const int total = gn * kTileRows * kWords;
  for (int base = threadIdx.x; base < total; base += kStageBatch * kGemvThreads) {
    uint32_t v[kStageBatch];
#pragma unroll
    for (int k = 0; k < kStageBatch; k++) {
      const int idx = base + k * kGemvThreads;
      const int gq = idx / (kTileRows * kWords);
      const int rem = idx - gq * kTileRows * kWords;
      const int row = rem / kWords, w = rem - row * kWords;
      const int r_local = tile * kTileRows + row;
      v[k] = 0;
      if (idx < total && r_local < job.rows)
        v[k] = __ldg(reinterpret_cast<const uint32_t*>(job.packed + ((int64_t)job.row_start + r_local) * job.row_bytes +
                                                       (int64_t)(g0 + gq) * St::kBytes) + w);
    }
#pragma unroll
    for (int k = 0; k < kStageBatch; k++) {
      const int idx = base + k * kGemvThreads;
      if (idx < total) {
        const int gq = idx / (kTileRows * kWords);
        const int rem = idx - gq * kTileRows * kWords;
        const int row = rem / kWords, w = rem - row * kWords;
        *reinterpret_cast<uint32_t*>(wt + (gq * kTileRows + row) * St::kStride + 4 * w) = v[k];
      }
    }
  }
}

// Dot products of R rows of one group against BT items, the chains interleaved across the
// R x BT (row, item) pairs so that independent binary64 operations issue back to back.  Each
// chain is the reference's: per byte the 4 (2-bit, ternary) or 2 (4-bit) column products summed
// left to right, then added to the group's dot; 3-bit rows add one product per column.
// Row r's staged group is at wrow0 + r * rstride, `xg` points at the group's columns of item 0 of
// the [BT][512] binary64 inputs.
template <int BITS, int R = kRowsPerThread, int BT = kBT>
__device__ __forceinline__ void group_dots(const uint8_t* wrow0, int rstride, const double* lut,
                                           const double* __restrict__ xg, int nb, double (&dot)[R][BT]) {
  constexpr int kRowsPerThread = R;
  constexpr int kBT = BT;
#pragma unroll
  for (int r = 0; r < kRowsPerThread; r++)
#pragma unroll
    for (int b = 0; b < kBT; b++) dot[r][b] = 0.0;
  const uint8_t* wrow[kRowsPerThread];
#pragma unroll
  for (int r = 0; r < kRowsPerThread; r++) wrow[r] = wrow0 + r * rstride;
  if constexpr (BITS == 2 || BITS == kTernaryBits || BITS == 4) {
    constexpr int kCols = BITS == 4 ? 2 : 4;  // columns per byte
#pragma unroll 1
    for (int wi = 0; wi < GroupBytes<BITS>::value / 4; wi++) {
      uint32_t word[kRowsPerThread];
#pragma unroll
      for (int r = 0; r < kRowsPerThread; r++) word[r] = *reinterpret_cast<const uint32_t*>(wrow[r] + 4 * wi);
#pragma unroll
      for (int byte_i = 0; byte_i < 4; byte_i++) {
        const int c = (wi * 4 + byte_i) * kCols;
        double a[kRowsPerThread][kCols];
#pragma unroll
        for (int r = 0; r < kRowsPerThread; r++) {
          const uint32_t byte = (word[r] >> (8 * byte_i)) & 0xffu;
#pragma unroll
          for (int k = 0; k < kCols; k++)
            a[r][k] = BITS == 4 ? lut[(byte >> (4 * k)) & 15] : lut[(byte >> (2 * k)) & 3];
        }
        double x[kBT][kCols];
#pragma unroll
        for (int b = 0; b < kBT; b++) {
          if (b < nb) {
#pragma unroll
            for (int k = 0; k < kCols; k += 2) {
              const double2 v = *reinterpret_cast<const double2*>(xg + b * 512 + c + k);
              x[b][k] = v.x;
              x[b][k + 1] = v.y;
            }
          } else {
#pragma unroll
            for (int k = 0; k < kCols; k++) x[b][k] = 0.0;
          }
        }
        double sacc[kRowsPerThread][kBT];
#pragma unroll
        for (int r = 0; r < kRowsPerThread; r++)
#pragma unroll
          for (int b = 0; b < kBT; b++) sacc[r][b] = a[r][0] * x[b][0];
#pragma unroll
        for (int k = 1; k < kCols; k++)
#pragma unroll
          for (int r = 0; r < kRowsPerThread; r++)
#pragma unroll
            for (int b = 0; b < kBT; b++) {
              if constexpr (BITS == kTernaryBits)
                sacc[r][b] = sacc[r][b] + a[r][k] * x[b][k];  // binary64 levels: rounded product
              else
                sacc[r][b] = fma(a[r][k], x[b][k], sacc[r][b]);  // binary32 levels: exact product
            }
#pragma unroll
        for (int r = 0; r < kRowsPerThread; r++)
#pragma unroll
          for (int b = 0; b < kBT; b++) dot[r][b] = dot[r][b] + sacc[r][b];
      }
    }
  } else {
    // 3-bit: 32 columns (three words, 96 bits) per outer step, one exact-product fma per column.
#pragma unroll 1
    for (int q = 0; q < 4; q++) {
      uint32_t w[kRowsPerThread][3];
#pragma unroll
      for (int r = 0; r < kRowsPerThread; r++)
#pragma unroll
        for (int k = 0; k < 3; k++) w[r][k] = *reinterpret_cast<const uint32_t*>(wrow[r] + 12 * q + 4 * k);
#pragma unroll
      for (int c2 = 0; c2 < 32; c2 += 2) {
        double a[kRowsPerThread][2];
#pragma unroll
        for (int r = 0; r < kRowsPerThread; r++)
#pragma unroll
          for (int k = 0; k < 2; k++) {
            const int bit = (c2 + k) * 3, wi = bit >> 5, sh = bit & 31;
            uint32_t v = w[r][wi] >> sh;
            if (sh > 29) v |= w[r][wi + 1] << (32 - sh);
            a[r][k] = lut[v & 7];
          }
#pragma unroll
        for (int b = 0; b < kBT; b++) {
          if (b < nb) {
            const double2 v = *reinterpret_cast<const double2*>(xg + b * 512 + 32 * q + c2);
#pragma unroll
            for (int r = 0; r < kRowsPerThread; r++) {
              dot[r][b] = fma(a[r][0], v.x, dot[r][b]);
              dot[r][b] = fma(a[r][1], v.y, dot[r][b]);
            }
          }
        }
      }
    }
  }
}

__device__ __forceinline__ void fill_gemv_lut(double* lut, const Codebook& cb, int bits) {
  if (threadIdx.x < 16) {
    double v = 0.0;
    if (bits == kTernaryBits) {
      const double coefficient = kTernaryCentroid / sqrt((double)kGroup);
      const int t = threadIdx.x;
      v = (t == 1) ? coefficient : (t == 3) ? -coefficient : 0.0;  // crumbs [0, c, 0, -c]
    } else if ((int)threadIdx.x < (1 << bits)) {
      v = (double)cb.v[(bits == 2 ? 0 : bits == 3 ? 4 : 12) + threadIdx.x];
    }
    lut[threadIdx.x] = v;
  }
}

// Stages the chunk's inputs of items [b0, b0 + nb) as binary64 (exact widening), [item][512].
__device__ __forceinline__ void stage_inputs(double* xs, const CqJob& job, int b0, int nb, int g0, int gn) {
  const int total = nb * gn * kGroup;
  for (int base = threadIdx.x; base < total; base += kStageBatch * kGemvThreads) {
    float v[kStageBatch];
#pragma unroll
    for (int k = 0; k < kStageBatch; k++) {
      const int idx = base + k * kGemvThreads;
      const int b = idx / (gn * kGroup);
      const int c = idx - b * gn * kGroup;
      v[k] = idx < total ? job.x[(int64_t)(b0 + b) * job.x_stride + g0 * kGroup + c] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < kStageBatch; k++) {
      const int idx = base + k * kGemvThreads;
      if (idx < total) {
        const int b = idx / (gn * kGroup);
        xs[b * 512 + (idx - b * gn * kGroup)] = (double)v[k];
      }
    }
  }
}

// Units of (32 R-row tile, BT-item tile); jobs' tile_begin counts tiles of 32 R rows.
template <int BITS, int R, int BT>
__global__ void __launch_bounds__(kGemvThreads)
k_cq_gemv(const CqJobs jobs, const Codebook cb, int32_t n_host, const int32_t* n_dev) {
  using St = Stage<BITS, R>;
  constexpr int kRowsPerThread = R;
  constexpr int kBT = BT;
  constexpr int kTileRows = St::kRows;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  double* xs = reinterpret_cast<double*>(smem_raw);                   // [BT][512]
  double* dsm = xs + kBT * 512;                                       // [BT][4][32 R]
  double* lut = dsm + kBT * kGroupsPerChunk * kTileRows;              // [16]
  uint8_t* wt = reinterpret_cast<uint8_t*>(lut + 16);                 // Stage<BITS, R>
  const int n = item_count(n_host, n_dev);
  const int item_tiles = (n + kBT - 1) / kBT;
  const int units = jobs.total_tiles * item_tiles;
  const int lane = threadIdx.x & 31;
  const int gc = threadIdx.x >> 5;  // group within the chunk
  fill_gemv_lut(lut, cb, BITS);

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
      __syncthreads();  // previous chunk's xs / dsm / wt fully consumed
      stage_inputs(xs, job, b0, nb, g0, gn);
      stage_weights<BITS, R>(wt, job, tile, g0, gn);
      __syncthreads();
      double dot[kRowsPerThread][kBT];
      if (gc < gn) {
        const uint8_t* w0 = wt + (gc * kTileRows + lane) * St::kStride;
        group_dots<BITS, R, BT>(w0, 32 * St::kStride, lut, xs + gc * kGroup, nb, dot);
#pragma unroll
        for (int r = 0; r < kRowsPerThread; r++)
#pragma unroll
          for (int b = 0; b < kBT; b++) dsm[(b * kGroupsPerChunk + gc) * kTileRows + r * 32 + lane] = dot[r][b];
      }
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

template <int R, int BT>
static size_t gemv_smem() {
  return sizeof(double) * (BT * 512 + BT * kGroupsPerChunk * kRowsPerTile * R + 16) + Stage<4, R>::kSize;
}

// Per (R, BT) variant: opts the four record widths into their dynamic shared memory (once per
// device) and returns the CTAs that fit on the device at once (the persistent grid size).
template <int R, int BT>
static cudaError_t configure_gemv(int* resident) {
  static std::atomic<uint64_t> done{0};
  static std::atomic<int> cached[64];
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (device & 63);
  const int smem = (int)gemv_smem<R, BT>();
  if (!(done.load() & bit)) {
    if ((e = cudaFuncSetAttribute(k_cq_gemv<2, R, BT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(k_cq_gemv<3, R, BT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(k_cq_gemv<4, R, BT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(k_cq_gemv<5, R, BT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
    int per_sm = 0, sms = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_cq_gemv<2, R, BT>, kGemvThreads, smem);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cached[device & 63].store(std::max(1, per_sm) * std::max(1, sms));
    done.fetch_or(bit);
  }
  *resident = cached[device & 63].load();
  return cudaSuccess;
}

template <int R, int BT>
static cudaError_t launch_gemv_variant(CqJobs J, const Codebook& cb, int32_t n_host, const int32_t* n_dev,
                                       cudaStream_t s) {
  int resident = 0;
  cudaError_t e = configure_gemv<R, BT>(&resident);
  if (e != cudaSuccess) return e;
  constexpr int rows_per_tile = kRowsPerTile * R;
  J.total_tiles = 0;  // tiles of this variant's height
  for (int k = 0; k < J.count; k++) {
    J.job[k].tile_begin = J.total_tiles;
    J.total_tiles += (J.job[k].rows + rows_per_tile - 1) / rows_per_tile;
  }
  const int units = J.total_tiles * ((n_host + BT - 1) / BT);
  dim3 grid(std::min(units, resident));
  const size_t smem = gemv_smem<R, BT>();
  switch (J.job[0].bits) {
    case 2: k_cq_gemv<2, R, BT><<<grid, kGemvThreads, smem, s>>>(J, cb, n_host, n_dev); break;
    case 3: k_cq_gemv<3, R, BT><<<grid, kGemvThreads, smem, s>>>(J, cb, n_host, n_dev); break;
    case 4: k_cq_gemv<4, R, BT><<<grid, kGemvThreads, smem, s>>>(J, cb, n_host, n_dev); break;
    case 5: k_cq_gemv<5, R, BT><<<grid, kGemvThreads, smem, s>>>(J, cb, n_host, n_dev); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// Tile shape of the batched exact GEMV: two rows per thread (64-row tiles) and four items per
// tile measured best at 64-256 items (against 1 x 4, 1 x 8 and 2 x 8).
cudaError_t launch_cq_gemv(const CqJobs& jobs, const Codebook& cb, int32_t n_host,
                           const int32_t* n_dev, cudaStream_t s) {
  if (n_host <= 0 || jobs.count <= 0) return cudaSuccess;
  const int bits = jobs.job[0].bits;
  for (int k = 1; k < jobs.count; k++)
    if (jobs.job[k].bits != bits) return cudaErrorInvalidValue;
  return launch_gemv_variant<2, 4>(jobs, cb, n_host, n_dev, s);
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
  extern __shared__ __align__(16) unsigned char smem_raw[];
  double* xs = reinterpret_cast<double*>(smem_raw);  // [kBT][512]
  double* lut = xs + kBT * 512;                      // [16]
  uint8_t* wt = reinterpret_cast<uint8_t*>(lut + 16);
  const int lane = threadIdx.x & 31, gc = threadIdx.x >> 5;
  const int groups = job.in_pad / kGroup;
  const int chunks = (groups + kGroupsPerChunk - 1) / kGroupsPerChunk;
  const int tiles = (job.rows + kTileRows - 1) / kTileRows;
  const int units = tiles * chunks;
  fill_gemv_lut(lut, cb, BITS);
#pragma unroll 1
  for (int unit = blockIdx.x; unit < units; unit += gridDim.x) {
    const int chunk = unit % chunks, tile = unit / chunks;  // neighbouring CTAs share rows
    const int g0 = chunk * kGroupsPerChunk;
    const int gn = min(kGroupsPerChunk, groups - g0);
    __syncthreads();
    stage_inputs(xs, job, 0, n, g0, gn);
    stage_weights<BITS>(wt, job, tile, g0, gn);
    __syncthreads();
    if (gc >= gn) continue;
    double dot[kRowsPerThread][kBT];
    const uint8_t* w0 = wt + (gc * kTileRows + lane) * Stage<BITS>::kStride;
    group_dots<BITS>(w0, 32 * Stage<BITS>::kStride, lut, xs + gc * kGroup, n, dot);
#pragma unroll
    for (int r = 0; r < kRowsPerThread; r++) {
      const int r_local = tile * kTileRows + r * 32 + lane;
      if (r_local >= job.rows) continue;
#pragma unroll
      for (int b = 0; b < kBT; b++)
        if (b < n) dots[((int64_t)b * job.rows + r_local) * groups + g0 + gc] = dot[r][b];
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
  const size_t smem = sizeof(double) * (kBT * 512 + 16) + Stage<BITS>::kSize;
  static std::atomic<uint64_t> configured{0};  // per device: > 48 KB dynamic shared memory opt-in
  {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(configured.load() & bit)) {
      e = cudaFuncSetAttribute(k_cq_group_dots<BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      configured.fetch_or(bit);
    }
  }
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
