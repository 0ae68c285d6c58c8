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

// ------------------------------------------------------------------ byte-table GEMV (2-bit, many items)
//
// For a 2-bit row the reference's inner step is a whole byte: the four column products of the
// byte's crumbs, summed left to right, then added to the group's dot (cq.ts:137-153).  That byte
// term depends only on the byte's value and on the item's four inputs of that column quad, so for
// one (item, group) a table
//     T[b][j] = fma(l(c3), x[4j+3], fma(l(c2), x[4j+2], fma(l(c1), x[4j+1], l(c0) * x[4j])))
// (b = c3 c2 c1 c0 in crumbs, 256 x 32 binary64 = 64 KB) holds every term the rows can need, built
// with exactly the operations the per-byte chain performs, and a row's group dot becomes 32 table
// reads and 32 adds in byte order -- the same values in the same order, a quarter of the binary64
// operations and a third of the instructions.  The table is shared by every row of the launch's
// jobs, which must therefore read one input (the Q, K, V and gate projections of a layer do).
//
// A CTA owns one item and a part of the rows; thread t streams rows t, t + 256, ... of its part.
// All lanes of a warp would read column j of the table at once, with random bytes b -- a 16-way bank
// conflict.  So lane l runs d = l mod 16 bytes behind lane l - d: at step i it reads column
// (i - d) mod 32, and the 16 lanes of each half-warp read 16 different columns (conflict-free).
// During the block of 32 steps that starts row k, a lane spends its first d steps on the last d
// bytes of row k - 1 and the rest on the first 32 - d bytes of row k: a 32-byte window at offset
// 32 - d of the two rows' bytes, rotated into registers once per block.
namespace {

constexpr int kTableThreads = 256;
constexpr int kTableMaxPasses = 6;  // rows per thread and part: parts have at most 1536 rows
constexpr int kTableMinItems = 64;  // below this the tile kernel (more CTAs per item) is faster
constexpr int kTableBytes = 256 * 32 * 8;

// Row `rr` of the launch (jobs in order; tile_begin holds each job's first row here): its job and
// matrix row.
__device__ __forceinline__ const CqJob& table_row(const CqJobs& J, int rr, int& prow, int& local) {
  int j = 0;
#pragma unroll 1
  for (int k = 1; k < J.count; k++)
    if (rr >= J.job[k].tile_begin) j = k;
  local = rr - J.job[j].tile_begin;
  prow = J.job[j].row_start + local;
  return J.job[j];
}

// T[b][j] for one item's group.  Thread (j = t mod 32, h = t / 32) holds the group's inputs
// 4j .. 4j + 3 in xq and writes the 32 bytes whose top three bits are h; the partial sums of the
// two low crumbs are shared by them.
__device__ __forceinline__ void build_byte_table(double* __restrict__ T, const float xq[4], const double lut[4]) {
  const int t = threadIdx.x, j = t & 31, hb = t >> 5;
  const double x0 = (double)xq[0], x1 = (double)xq[1], x2 = (double)xq[2], x3 = (double)xq[3];
  double s01[16];  // [c1 * 4 + c0]
#pragma unroll
  for (int c0 = 0; c0 < 4; c0++) {
    const double p0 = lut[c0] * x0;
#pragma unroll
    for (int c1 = 0; c1 < 4; c1++) s01[c1 * 4 + c0] = fma(lut[c1], x1, p0);
  }
  auto level = [&](int c) { return c == 0 ? lut[0] : c == 1 ? lut[1] : c == 2 ? lut[2] : lut[3]; };
  const double a3 = level(hb >> 1);
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const double a2 = level(((hb & 1) << 1) | h);
#pragma unroll
    for (int k = 0; k < 16; k++) {
      const double s = fma(a2, x2, s01[k]);
      T[(((hb << 5) | (h << 4) | k) << 5) + j] = fma(a3, x3, s);
    }
  }
}

// Row `rr` of the launch, group g: its 32 bytes and its raw fp16 norm.  Row-major matrices keep a
// row's groups together (row_bytes apart per row); group-major ones ([group][row][32 bytes], row_bytes
// = the stride between groups) keep a group's rows together, so the 32 rows a warp reads are 1 KB.
template <bool kGroupMajor>
__device__ __forceinline__ void load_table_row(const CqJobs& J, int rr, int g, int groups, uint4& n0, uint4& n1,
                                               uint16_t& nn) {
  int prow, local;
  const CqJob& jb = table_row(J, rr, prow, local);
  const int64_t at = kGroupMajor ? (int64_t)g * jb.row_bytes + (int64_t)prow * (kGroup / 4)
                                 : (int64_t)prow * jb.row_bytes + g * (kGroup / 4);
  const uint4* p = reinterpret_cast<const uint4*>(jb.packed + at);
  n0 = __ldg(p);
  n1 = __ldg(p + 1);
  nn = __ldg(jb.norms + (int64_t)prow * groups + g);
}

// w = bytes [e, e + 32) of prev || cur (e in 17..32).
__device__ __forceinline__ void table_window(const uint32_t prev[8], const uint32_t cur[8], int e, uint32_t w[8]) {
  uint32_t s[13];  // words 4 .. 16 of prev || cur || 0
#pragma unroll
  for (int i = 0; i < 13; i++) s[i] = i < 4 ? prev[4 + i] : i < 12 ? cur[i - 4] : 0u;
  const int r = (e >> 2) - 4;  // 0 .. 4
  const uint32_t sh = 8u * uint32_t(e & 3);
#pragma unroll
  for (int i = 0; i < 9; i++) s[i] = (r & 4) ? s[i + 4] : s[i];
#pragma unroll
  for (int i = 0; i < 11; i++) s[i] = (r & 2) ? s[i + 2] : s[i];
#pragma unroll
  for (int i = 0; i < 9; i++) s[i] = (r & 1) ? s[i + 1] : s[i];
#pragma unroll
  for (int m = 0; m < 8; m++) w[m] = __funnelshift_r(s[m], s[m + 1], sh);
}

template <bool kGroupMajor>
__global__ void __launch_bounds__(kTableThreads, 3)
k_cq_gemv2_table(const CqJobs J, const Codebook cb, int32_t n_host, const int32_t* n_dev, int32_t parts,
                 int32_t part_rows) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  double* T = reinterpret_cast<double*>(smem_raw);  // [256][32]
  const char* Tb = reinterpret_cast<const char*>(smem_raw);
  const int n = item_count(n_host, n_dev);
  const int item = blockIdx.x / parts, part = blockIdx.x - item * parts;
  if (item >= n) return;  // the whole CTA, before any barrier
  const int t = threadIdx.x, lane = t & 31;
  const int r0 = part * part_rows, r1 = min(J.total_tiles, r0 + part_rows);
  const int passes = (r1 - r0 + kTableThreads - 1) / kTableThreads;  // <= kTableMaxPasses
  const CqJob& f = J.job[0];
  const int groups = f.in_pad / kGroup;
  const float* xi = f.x + (int64_t)item * f.x_stride;
  double lut[4];
#pragma unroll
  for (int c = 0; c < 4; c++) lut[c] = (double)cb.v[c];
  const int d = lane & 15, e = 32 - d;
  const uint32_t jd8 = uint32_t((32 - d) & 31) * 8u;  // byte offset of column (i - d) mod 32, at i = 0
  double tot[kTableMaxPasses];
#pragma unroll
  for (int k = 0; k < kTableMaxPasses; k++) tot[k] = 0.0;

  // Every global read is issued a block (a row's bytes and norm) or a group (the table's inputs,
  // the group's first row) before its use: the lookups hide their latency.
  const int jq = t & 31;
  float xq[4];
#pragma unroll
  for (int c = 0; c < 4; c++) xq[c] = xi[4 * jq + c];
  uint4 n0 = make_uint4(0u, 0u, 0u, 0u), n1 = n0;
  uint16_t nn = 0;  // raw fp16 norm of the row in n0 / n1
  if (r0 + t < r1) load_table_row<kGroupMajor>(J, r0 + t, 0, groups, n0, n1, nn);

#pragma unroll 1
  for (int g = 0; g < groups; g++) {
    if (g > 0) __syncthreads();  // every lookup of the previous group is done
    build_byte_table(T, xq, lut);
    __syncthreads();
    if (g + 1 < groups) {
#pragma unroll
      for (int c = 0; c < 4; c++) xq[c] = xi[(g + 1) * kGroup + 4 * jq + c];
    }
    uint32_t prev[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    uint16_t norm_prev = 0;
    double acc_prev = 0.0, acc_cur = 0.0;
#pragma unroll
    for (int k = 0; k <= kTableMaxPasses; k++) {
      if (k > passes) break;
      const uint32_t cur[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
      const uint16_t norm_cur = nn;
      n0 = make_uint4(0u, 0u, 0u, 0u);
      n1 = n0;
      nn = 0;
      const int rn = r0 + t + (k + 1) * kTableThreads;  // next row of this thread
      if (k + 1 < passes) {
        if (rn < r1) load_table_row<kGroupMajor>(J, rn, g, groups, n0, n1, nn);
      } else if (k == passes && g + 1 < groups && r0 + t < r1) {
        load_table_row<kGroupMajor>(J, r0 + t, g + 1, groups, n0, n1, nn);  // the next group's first row
      }
      uint32_t w[8];
      table_window(prev, cur, e, w);
      acc_cur = 0.0;
      if (k < passes) {
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const uint32_t b8 = __byte_perm(w[i >> 2], 0u, 0x4404u | (uint32_t(i & 3) << 4));  // byte << 8
          const uint32_t off = b8 | ((jd8 + 8u * uint32_t(i)) & 255u);
          const double v = *reinterpret_cast<const double*>(Tb + off);
          if (i < 16 && i < d)
            acc_prev = acc_prev + v;  // the last d bytes of row k - 1
          else
            acc_cur = acc_cur + v;
        }
      } else {  // drain: the last d bytes of the final row
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const uint32_t b8 = __byte_perm(w[i >> 2], 0u, 0x4404u | (uint32_t(i & 3) << 4));
          const uint32_t off = b8 | ((jd8 + 8u * uint32_t(i)) & 255u);
          const double v = *reinterpret_cast<const double*>(Tb + off);
          if (i < d) acc_prev = acc_prev + v;
        }
      }
      if (k >= 1 && r0 + t + (k - 1) * kTableThreads < r1) {
        // row k - 1 is complete: fold its group dot into the total (cq.ts:151)
        const double nrm = (double)__half2float(__ushort_as_half(norm_prev));
        tot[k - 1] = tot[k - 1] + nrm * acc_prev;
      }
      acc_prev = acc_cur;
      norm_prev = norm_cur;
#pragma unroll
      for (int m = 0; m < 8; m++) prev[m] = cur[m];
    }
  }
#pragma unroll
  for (int k = 0; k < kTableMaxPasses; k++) {
    const int rr = r0 + t + k * kTableThreads;
    if (k < passes && rr < r1) {
      int prow, local;
      const CqJob& jb = table_row(J, rr, prow, local);
      jb.y[(int64_t)item * jb.y_stride + local] = f32(tot[k]);
    }
  }
}

// The byte-table kernel applies to launches of 2-bit jobs that share one input, with 16-byte
// aligned rows, from kTableMinItems items.
bool table_gemv_applies(const CqJobs& J, int32_t n_host) {
  if (n_host < kTableMinItems || J.count <= 0) return false;
  const CqJob& f = J.job[0];
  if (f.in_pad <= 0 || f.in_pad % kGroup) return false;
  for (int k = 0; k < J.count; k++) {
    const CqJob& j = J.job[k];
    if (j.bits != 2 || j.x != f.x || j.x_stride != f.x_stride || j.in_pad != f.in_pad) return false;
    if (j.row_bytes % 16 || reinterpret_cast<uintptr_t>(j.packed) % 16 || j.row_bytes < f.in_pad / 4) return false;
  }
  return true;
}

template <bool kGroupMajor>
cudaError_t launch_gemv_table(CqJobs J, const Codebook& cb, int32_t n_host, const int32_t* n_dev, cudaStream_t s) {
  static std::atomic<uint64_t> configured{0};  // per device: 64 KB dynamic shared memory opt-in
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    e = cudaFuncSetAttribute(k_cq_gemv2_table<kGroupMajor>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTableBytes);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit);
  }
  int rows = 0;
  for (int k = 0; k < J.count; k++) {
    J.job[k].tile_begin = rows;  // first row of the job in the launch
    rows += J.job[k].rows;
  }
  J.total_tiles = rows;  // rows of the launch
  if (rows <= 0) return cudaSuccess;
  constexpr int kPartMax = kTableThreads * kTableMaxPasses;
  // Two parts per item below two CTAs per SM's worth of items (more CTAs to spread), as long as a
  // part keeps three rows per thread; more parts only where the rows need them.
  int parts = (rows + kPartMax - 1) / kPartMax;
  if (n_host < 296 && rows >= 2 * 3 * kTableThreads) parts = std::max(parts, 2);
  const int part_rows = (rows + parts - 1) / parts;
  const int64_t grid = (int64_t)n_host * parts;
  if (grid > 0x7fffffff) return cudaErrorInvalidValue;
  k_cq_gemv2_table<kGroupMajor>
      <<<(unsigned)grid, kTableThreads, kTableBytes, s>>>(J, cb, n_host, n_dev, parts, part_rows);
  return cudaGetLastError();
}

}  // namespace

// Tile shape of the batched exact GEMV: two rows per thread (64-row tiles) and four items per
// tile measured best at 64-256 items (against 1 x 4, 1 x 8 and 2 x 8).  2-bit launches of many
// items that share one input take the byte-table kernel instead (the same operations in the same
// order, so the same bits).
cudaError_t launch_cq_gemv(const CqJobs& jobs, const Codebook& cb, int32_t n_host,
                           const int32_t* n_dev, cudaStream_t s) {
  if (n_host <= 0 || jobs.count <= 0) return cudaSuccess;
  const int bits = jobs.job[0].bits;
  for (int k = 1; k < jobs.count; k++)
    if (jobs.job[k].bits != bits) return cudaErrorInvalidValue;
  if (table_gemv_applies(jobs, n_host)) return launch_gemv_table<false>(jobs, cb, n_host, n_dev, s);
  return launch_gemv_variant<2, 4>(jobs, cb, n_host, n_dev, s);
}

bool cq_gemv2_group_major_preferred(int32_t n_host) { return n_host >= kTableMinItems; }

cudaError_t launch_cq_gemv2_group_major(const CqJob& job, const Codebook& cb, int32_t n_host, const int32_t* n_dev,
                                        cudaStream_t s) {
  if (n_host <= 0 || job.rows <= 0) return cudaSuccess;
  if (job.bits != 2 || job.in_pad <= 0 || job.in_pad % kGroup || job.row_bytes % 16 ||
      job.row_bytes < job.rows * (kGroup / 4) || reinterpret_cast<uintptr_t>(job.packed) % 16)
    return cudaErrorInvalidValue;
  CqJobs J{};
  J.job[0] = job;
  J.count = 1;
  return launch_gemv_table<true>(J, cb, n_host, n_dev, s);
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
