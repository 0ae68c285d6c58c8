// cq.cuh -- Cactus-Quant matrix kernels: activation prepare (per-group FWHT), batched
// multi-matrix GEMV, and row dequantisation.
#pragma once

#include "common.cuh"

namespace needle {

// Rows of one GEMV tile (a CTA): tiles of consecutive rows are the unit of CqJob::tile_begin.
constexpr int kGemvTileRows = 64;

// One matrix-times-batch job of a GEMV launch.  Rows [row_start, row_start + rows) of the matrix
// multiply the prepared inputs x[i * x_stride ...] of every item i; row r of the job lands in
// y[i * y_stride + r].
struct CqJob {
  const uint8_t* packed;   // row 0 of the matrix
  const uint16_t* norms;   // fp16 norms of row 0
  int32_t row_start;
  int32_t rows;
  int32_t in_pad;          // padded input length (multiple of 128)
  int32_t bits;            // 2, 3, 4 or 5 (ternary)
  int32_t row_bytes;
  int32_t tile_begin;      // first kGemvTileRows-row tile of this job in the launch
  const float* x;
  int32_t x_stride;
  int32_t y_stride;
  float* y;
};

constexpr int kMaxJobs = 8;
struct CqJobs {
  CqJob job[kMaxJobs];
  int32_t count;
  int32_t total_tiles;
};

// Codebook (28 binary32 levels: CQ2 | CQ3 | CQ4) shared by every matrix of an archive.
struct Codebook {
  float v[28];
};

// Host launchers (cq.cu).  `n_dev` (device int, may be null) overrides `n_host` as item count so
// that graphs and the device scheduler can size the batch on the device.
cudaError_t launch_cq_prepare(const float* x, int32_t x_stride, int32_t input_size, int32_t in_pad,
                              float* out, int32_t out_stride, int32_t n_host, const int32_t* n_dev,
                              cudaStream_t s);
cudaError_t launch_cq_gemv(const CqJobs& jobs, const Codebook& cb, int32_t n_host,
                           const int32_t* n_dev, cudaStream_t s);
// Exact 2-bit GEMV of one group-major matrix ([group][row][32 bytes]; job.row_bytes = the byte
// stride between groups, at least rows * 32): the byte-table kernel with contiguous row loads.  The
// engine keeps its Q|K|V|gate projections in this layout too; preferred from the item count on.
bool cq_gemv2_group_major_preferred(int32_t n_host);
cudaError_t launch_cq_gemv2_group_major(const CqJob& job, const Codebook& cb, int32_t n_host, const int32_t* n_dev,
                                        cudaStream_t s);
// Small-batch path for long rows (cq.cu): per-(row, group) dots of (row tile, group chunk) units
// into `scratch` (cq_gemv_split_scratch_bytes), then ordered per-row totals.
bool cq_gemv_prefers_split(const CqJob& job, int32_t n);
size_t cq_gemv_split_scratch_bytes(const CqJob& job, int32_t n);
cudaError_t launch_cq_gemv_split(const CqJob& job, const Codebook& cb, int32_t n, double* scratch, cudaStream_t s);
// Fast-numerics matvec (cq_fast.cu): binary32 table lookups, record widths 2, 4 and ternary; takes
// the raw activation x [batch][input_size] (it prepares each group itself).  Scratch: per-group
// partial sums (cq_gemv_fast_partial_floats); up to kFastMaxItems items per pass of two launches.
constexpr int kFastMaxItems = 8;
bool cq_gemv_fast_supported(int32_t bits);
size_t cq_gemv_fast_partial_floats(int32_t rows, int32_t in_pad);
cudaError_t launch_cq_gemv_fast(const uint8_t* packed, const uint16_t* norms, int32_t rows, int32_t input_size,
                                int32_t bits, const float* x, int32_t batch, float* y, const Codebook& cb,
                                float* partials, cudaStream_t s);
// Batched fast-numerics matvec on the tensor cores (cq_gemm_tc.cu): fp16 head/tail split GEMM,
// record widths 2, 3, 4 and ternary.  Scratch (cq_gemm_tc_scratch_bytes, 256-byte aligned): the
// split activations and split-K partials; items are tiled over CTAs (tiles of 16-128).
constexpr int kTcMinBatch = 16;
bool cq_gemm_tc_supported(int32_t bits);
// Split-K factor of the GEMM for a matrix (1: no partials and no split-K sum kernel).
int cq_gemm_tc_splits(int32_t rows, int32_t input_size, int32_t batch, int32_t sms);
bool cq_gemm_tc_preferred(int32_t rows, int32_t input_size, int32_t batch);
size_t cq_gemm_tc_scratch_bytes(int32_t rows, int32_t input_size, int32_t batch, int32_t sms);
// x: rows of x_stride floats, raw (prepared = 0: each group is prepared here) or already prepared
// (x', input padded to whole groups); y: rows of y_stride floats.  Record widths 2, 3, 4, ternary.
cudaError_t launch_cq_gemm_tc(const uint8_t* packed, const uint16_t* norms, int32_t rows, int32_t input_size,
                              int32_t bits, const float* x, int32_t x_stride, int32_t prepared, int32_t batch, float* y,
                              int32_t y_stride, const Codebook& cb, void* scratch, int32_t sms, cudaStream_t s);
cudaError_t launch_cq_rows(const uint8_t* packed, const uint16_t* norms, int32_t bits,
                           int32_t row_bytes, int32_t in_pad, int32_t input_size,
                           const int32_t* rows, int32_t n_rows, float* out, int32_t out_stride,
                           const Codebook& cb, cudaStream_t s);

// Device helpers shared with the fused per-sequence kernels ---------------------------------

// Index of column `col` (within its row) of a packed CQ row (the bit layouts of
// packages/needle.js/src/backends/cq.ts:270-284); ternary crumbs map to trit indices 3->0, 0->1,
// 1->2, 2->3.
__device__ __forceinline__ int cq_index(const uint8_t* rowp, int bits, int col) {
  if (bits == 2 || bits == kTernaryBits) {
    const int byte = rowp[col >> 2];
    const int crumb = (byte >> ((col & 3) * 2)) & 3;
    return bits == kTernaryBits ? (crumb == 3 ? 0 : crumb + 1) : crumb;
  }
  if (bits == 4) return (rowp[col >> 1] >> ((col & 1) * 4)) & 15;
  // 3-bit bitstream: an index straddles two bytes only when its shift exceeds 5, and then the
  // second byte lies inside the same row; otherwise the neighbour byte is masked off anyway.
  const int bit = col * 3;
  const int shift = bit & 7;
  uint32_t word = rowp[bit >> 3];
  if (shift > 5) word |= (uint32_t)rowp[(bit >> 3) + 1] << 8;
  return (int)((word >> shift) & 7);
}

// Level of a dequantised index: the archive codebook, or for ternary rows the binary32 array
// [-c/sqrt(g), 0, c/sqrt(g)] (cq.ts:259-262); index 3 of a ternary row reads past that array and
// yields 0 (`codebook[index] ?? 0`).
__device__ __forceinline__ double cq_level(const float* cb28, int bits, int index) {
  if (bits == kTernaryBits) {
    const double inv = 1.0 / sqrt((double)kGroup);
    if (index == 0) return (double)f32(-kTernaryCentroid * inv);
    if (index == 2) return (double)f32(kTernaryCentroid * inv);
    return 0.0;
  }
  const int base = bits == 2 ? 0 : bits == 3 ? 4 : 12;
  return (double)cb28[base + index];
}

// x' of one group: zero padding, FWHT (binary32 butterflies, strides 1, 2, 4, ...), times
// 1/sqrt(128) in binary64 rounded to binary32 (prepareCqActivation, cq.ts:30-46).  Every warp
// computes it (four values per lane: lane l holds x'[4l .. 4l+3]), so no barrier is needed.
__device__ __forceinline__ void prepare_group_warp(const float* __restrict__ x, int input_size, int g, float v[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int col = g * kGroup + 4 * lane + k;
    v[k] = col < input_size ? __ldg(x + col) : 0.0f;
  }
  // strides 1 and 2 inside the lane
  {
    const float a0 = __fadd_rn(v[0], v[1]), a1 = __fsub_rn(v[0], v[1]);
    const float a2 = __fadd_rn(v[2], v[3]), a3 = __fsub_rn(v[2], v[3]);
    v[0] = __fadd_rn(a0, a2);
    v[2] = __fsub_rn(a0, a2);
    v[1] = __fadd_rn(a1, a3);
    v[3] = __fsub_rn(a1, a3);
  }
  // strides 4 .. 64 across lanes
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float other = __shfl_xor_sync(0xffffffffu, v[k], m);
      v[k] = (lane & m) ? __fsub_rn(other, v[k]) : __fadd_rn(v[k], other);
    }
  }
  const double inverse_root = 1.0 / sqrt((double)kGroup);
#pragma unroll
  for (int k = 0; k < 4; k++) v[k] = f32((double)v[k] * inverse_root);
}

}  // namespace needle
