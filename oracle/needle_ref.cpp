// needle_ref.cpp -- CPU ORACLE (test infrastructure only; see needle_ref.h).
//
// Restates the needle.js TypeScript CPU decode path with JavaScript numeric semantics:
//  * every JS `number` expression is evaluated in double;
//  * a value becomes float only where the TypeScript stores it into a Float32Array;
//  * Math.exp/log/sqrt/pow/cos/sin are the C library's double functions;
//  * Math.imul / `>>> 0` are uint32 wrap-around arithmetic.
// Compiled with -ffp-contract=off so no multiply-add is fused behind our back.
// Each function cites the reference file:line it follows (paths inside packages/needle.js).

#include "needle_ref.h"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

enum Code : int {
  OK = 0,
  INVALID_CACT = 1,
  UNSUPPORTED_CACT = 2,
  BACKEND_UNAVAILABLE = 6,
  CONTEXT_OVERFLOW = 7,
};

struct RefError {
  int code;
  std::string msg;
};

thread_local std::string g_last_error;

[[noreturn]] void fail(int code, const std::string& msg) { throw RefError{code, msg}; }
inline void invariant(bool cond, int code, const std::string& msg) {
  if (!cond) fail(code, msg);
}

template <class F>
int guard(F&& f) {
  try {
    f();
    return OK;
  } catch (const RefError& e) {
    g_last_error = e.msg;
    return e.code;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return BACKEND_UNAVAILABLE;
  }
}

constexpr double kNegInf = -std::numeric_limits<double>::infinity();

// ---------------------------------------------------------------- fp16 (src/model/fp16.ts)

// float16ToNumber, fp16.ts:5-32: widen binary16 to binary32 bits.
float f16_to_f32(uint32_t value) {
  uint32_t h = value & 0xffffu;
  uint32_t sign = (h & 0x8000u) << 16;
  int32_t exponent = (h >> 10) & 0x1f;
  uint32_t mantissa = h & 0x03ffu;
  uint32_t bits;
  if (exponent == 0) {
    if (mantissa == 0) {
      bits = sign;
    } else {
      exponent = 127 - 15 + 1;
      while ((mantissa & 0x0400u) == 0) {
        mantissa <<= 1;
        exponent--;
      }
      mantissa &= 0x03ffu;
      bits = sign | (uint32_t(exponent) << 23) | (mantissa << 13);
    }
  } else if (exponent == 0x1f) {
    bits = sign | 0x7f800000u | (mantissa << 13);
  } else {
    bits = sign | (uint32_t(exponent - 15 + 127) << 23) | (mantissa << 13);
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

// numberToFloat16, fp16.ts:35-74 (the value is first stored into a Float32Array).
uint32_t f32_to_f16(double value) {
  float f = float(value);
  uint32_t bits;
  std::memcpy(&bits, &f, 4);
  uint32_t sign = (bits >> 16) & 0x8000u;
  int32_t exponent = (bits >> 23) & 0xff;
  uint32_t mantissa = bits & 0x7fffffu;
  if (exponent == 0xff) return mantissa == 0 ? (sign | 0x7c00u) : (sign | 0x7e00u);
  int32_t halfExponent = exponent - 127 + 15;
  if (halfExponent >= 0x1f) return sign | 0x7c00u;
  if (halfExponent <= 0) {
    if (halfExponent < -10) return sign;
    uint32_t normalized = mantissa | 0x800000u;
    int32_t shift = 14 - halfExponent;
    uint32_t halfMantissa = normalized >> shift;
    uint32_t remainder = normalized & ((1u << shift) - 1);
    uint32_t halfway = 1u << (shift - 1);
    if (remainder > halfway || (remainder == halfway && (halfMantissa & 1) != 0)) halfMantissa++;
    return sign | halfMantissa;
  }
  uint32_t halfMantissa = mantissa >> 13;
  uint32_t remainder = mantissa & 0x1fffu;
  int32_t outExponent = halfExponent;
  if (remainder > 0x1000u || (remainder == 0x1000u && (halfMantissa & 1) != 0)) {
    halfMantissa++;
    if (halfMantissa == 0x0400u) {
      halfMantissa = 0;
      outExponent++;
      if (outExponent >= 0x1f) return sign | 0x7c00u;
    }
  }
  return sign | (uint32_t(outExponent) << 10) | halfMantissa;
}

inline uint32_t rd_u32(const uint8_t* p) {
  return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
}
inline uint64_t rd_u64(const uint8_t* p) { return uint64_t(rd_u32(p)) | (uint64_t(rd_u32(p + 4)) << 32); }
inline float rd_f32(const uint8_t* p) {
  uint32_t b = rd_u32(p);
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

// ---------------------------------------------------------------- CQ kernels (src/backends/cq.ts)

constexpr int kTernaryBits = 5;           // cq.ts:5
constexpr double kTernaryCentroid = 1.2240064;  // cq.ts:6

struct CqMatrix {
  int32_t outputSize = 0, inputSize = 0, inputSizePadded = 0, groupSize = 0, bits = 0;
  int64_t rowByteLength = 0;
  const uint8_t* packed = nullptr;
  const uint8_t* norms = nullptr;  // little-endian fp16
  const float* cb2 = nullptr;      // 4 entries
  const float* cb3 = nullptr;      // 8 entries
  const float* cb4 = nullptr;      // 16 entries
};

// fastWalshHadamard, cq.ts:8-27.  left/right are float32 values; `left + right` is evaluated in
// double and stored back into the Float32Array.
void fwht(float* values, int64_t offset, int64_t length) {
  invariant(length > 0 && (length & (length - 1)) == 0, UNSUPPORTED_CACT,
            "Walsh-Hadamard length " + std::to_string(length) + " is not a power of two");
  for (int64_t stride = 1; stride < length; stride <<= 1) {
    int64_t block = stride << 1;
    for (int64_t base = 0; base < length; base += block) {
      for (int64_t inner = 0; inner < stride; inner++) {
        int64_t l = offset + base + inner, r = l + stride;
        double left = values[l], right = values[r];
        values[l] = float(left + right);
        values[r] = float(left - right);
      }
    }
  }
}

// prepareCqActivation, cq.ts:30-46.
std::vector<float> prepare(const CqMatrix& m, const float* input, int64_t inputLength) {
  invariant(inputLength == m.inputSize, INVALID_CACT,
            "Matrix expects " + std::to_string(m.inputSize) + " inputs, received " +
                std::to_string(inputLength));
  std::vector<float> prepared(m.inputSizePadded, 0.0f);
  std::copy(input, input + inputLength, prepared.begin());
  const double inverseRoot = 1.0 / std::sqrt(double(m.groupSize));
  for (int64_t offset = 0; offset < m.inputSizePadded; offset += m.groupSize) {
    fwht(prepared.data(), offset, m.groupSize);
    for (int64_t i = 0; i < m.groupSize; i++)
      prepared[offset + i] = float(double(prepared[offset + i]) * inverseRoot);
  }
  return prepared;
}

// normAt, cq.ts:102-104.
inline double normAt(const CqMatrix& m, int64_t row, int64_t group, int64_t groupsPerRow) {
  const uint8_t* p = m.norms + (row * groupsPerRow + group) * 2;
  return f16_to_f32(uint32_t(p[0]) | (uint32_t(p[1]) << 8));
}

// cqMatvecPrepared, cq.ts:107-231.
std::vector<float> matvecPrepared(const CqMatrix& m, const std::vector<float>& prepared,
                                  int64_t rowStart, int64_t rowCount) {
  invariant(int64_t(prepared.size()) == m.inputSizePadded, INVALID_CACT,
            "Prepared activation has the wrong padded length");
  invariant(rowStart >= 0 && rowCount >= 0 && rowStart + rowCount <= m.outputSize, INVALID_CACT,
            "Invalid matrix row range " + std::to_string(rowStart) + ":" +
                std::to_string(rowStart + rowCount));
  std::vector<float> output(rowCount);
  const int64_t g = m.groupSize;
  const int64_t groupsPerRow = m.inputSizePadded / g;
  const uint8_t* packed = m.packed;
  const float* x = prepared.data();

  if (m.bits == 2) {
    invariant(m.cb2 && m.cb4, INVALID_CACT, "CQ2/CQ4 codebooks are missing");
    float lut2[256 * 4];  // cq.ts:88-96
    for (int b = 0; b < 256; b++)
      for (int c = 0; c < 4; c++) lut2[b * 4 + c] = m.cb2[(b >> (c * 2)) & 3];
    for (int64_t lr = 0; lr < rowCount; lr++) {
      const int64_t row = rowStart + lr, rowOffset = row * m.rowByteLength;
      double total = 0;
      for (int64_t group = 0; group < groupsPerRow; group++) {
        const int64_t io = group * g, po = rowOffset + group * g / 4;
        double dot = 0;
        for (int64_t col = 0; col < g; col += 4) {
          const int lookup = packed[po + (col >> 2)] * 4;
          dot += double(lut2[lookup]) * double(x[io + col]) +
                 double(lut2[lookup + 1]) * double(x[io + col + 1]) +
                 double(lut2[lookup + 2]) * double(x[io + col + 2]) +
                 double(lut2[lookup + 3]) * double(x[io + col + 3]);
        }
        total += normAt(m, row, group, groupsPerRow) * dot;
      }
      output[lr] = float(total);
    }
    return output;
  }

  if (m.bits == 4) {
    invariant(m.cb2 && m.cb4, INVALID_CACT, "CQ2/CQ4 codebooks are missing");
    float lut4[256 * 2];
    for (int b = 0; b < 256; b++) {
      lut4[b * 2] = m.cb4[b & 15];
      lut4[b * 2 + 1] = m.cb4[(b >> 4) & 15];
    }
    for (int64_t lr = 0; lr < rowCount; lr++) {
      const int64_t row = rowStart + lr, rowOffset = row * m.rowByteLength;
      double total = 0;
      for (int64_t group = 0; group < groupsPerRow; group++) {
        const int64_t io = group * g, po = rowOffset + group * g / 2;
        double dot = 0;
        for (int64_t col = 0; col < g; col += 2) {
          const int lookup = packed[po + (col >> 1)] * 2;
          dot += double(lut4[lookup]) * double(x[io + col]) +
                 double(lut4[lookup + 1]) * double(x[io + col + 1]);
        }
        total += normAt(m, row, group, groupsPerRow) * dot;
      }
      output[lr] = float(total);
    }
    return output;
  }

  if (m.bits == kTernaryBits) {
    const double coefficient = kTernaryCentroid / std::sqrt(double(g));
    const double crumbs[4] = {0.0, coefficient, 0.0, -coefficient};
    for (int64_t lr = 0; lr < rowCount; lr++) {
      const int64_t row = rowStart + lr, rowOffset = row * m.rowByteLength;
      double total = 0;
      for (int64_t group = 0; group < groupsPerRow; group++) {
        const int64_t io = group * g, po = rowOffset + group * g / 4;
        double dot = 0;
        for (int64_t col = 0; col < g; col += 4) {
          const int byte = packed[po + (col >> 2)];
          dot += crumbs[byte & 3] * double(x[io + col]) +
                 crumbs[(byte >> 2) & 3] * double(x[io + col + 1]) +
                 crumbs[(byte >> 4) & 3] * double(x[io + col + 2]) +
                 crumbs[(byte >> 6) & 3] * double(x[io + col + 3]);
        }
        total += normAt(m, row, group, groupsPerRow) * dot;
      }
      output[lr] = float(total);
    }
    return output;
  }

  // Three-bit rows: an uninterrupted little-endian bitstream (cq.ts:208-230).
  invariant(m.cb3 != nullptr, INVALID_CACT, "CQ3 codebook is missing");
  for (int64_t lr = 0; lr < rowCount; lr++) {
    const int64_t row = rowStart + lr, rowOffset = row * m.rowByteLength;
    double total = 0;
    for (int64_t group = 0; group < groupsPerRow; group++) {
      const int64_t io = group * g;
      double dot = 0;
      for (int64_t col = 0; col < g; col++) {
        const int64_t bitPosition = (group * g + col) * 3;
        const int64_t bytePosition = rowOffset + (bitPosition >> 3);
        const int shift = int(bitPosition & 7);
        // `packed[bytePosition + 1] ?? 0`: the last byte of the buffer reads a zero neighbour.
        const uint32_t hi = (bytePosition + 1 < m.outputSize * m.rowByteLength)
                                ? packed[bytePosition + 1] : 0u;
        const uint32_t word = uint32_t(packed[bytePosition]) | (hi << 8);
        dot += double(m.cb3[(word >> shift) & 7]) * double(x[io + col]);
      }
      total += normAt(m, row, group, groupsPerRow) * dot;
    }
    output[lr] = float(total);
  }
  return output;
}

std::vector<float> cqMatvec(const CqMatrix& m, const float* input, int64_t inputLength,
                            int64_t rowStart, int64_t rowCount) {
  return matvecPrepared(m, prepare(m, input, inputLength), rowStart, rowCount);
}

// dequantizeCqRow, cq.ts:243-295.
void dequantizeRow(const CqMatrix& m, int64_t row, float* result) {
  invariant(row >= 0 && row < m.outputSize, INVALID_CACT,
            "Matrix row " + std::to_string(row) + " is out of range");
  const int64_t g = m.groupSize;
  const int64_t groupsPerRow = m.inputSizePadded / g;
  std::vector<float> temporary(g);
  const double inverseRoot = 1.0 / std::sqrt(double(g));
  const int64_t rowOffset = row * m.rowByteLength;
  float ternary[3] = {float(-kTernaryCentroid * inverseRoot), 0.0f,
                      float(kTernaryCentroid * inverseRoot)};
  const float* codebook = m.bits == 5 ? ternary : m.bits == 2 ? m.cb2 : m.bits == 3 ? m.cb3 : m.cb4;
  const int codebookLength = m.bits == 5 ? 3 : m.bits == 2 ? 4 : m.bits == 3 ? 8 : 16;
  invariant(codebook != nullptr, INVALID_CACT, "Codebook W" + std::to_string(m.bits) + " is missing");
  const int64_t packedTotal = m.outputSize * m.rowByteLength;
  for (int64_t group = 0; group < groupsPerRow; group++) {
    const double norm = normAt(m, row, group, groupsPerRow);
    for (int64_t col = 0; col < g; col++) {
      const int64_t ac = group * g + col;
      int index;
      if (m.bits == 2 || m.bits == 5) {
        const int byte = m.packed[rowOffset + (ac >> 2)];
        const int crumb = (byte >> ((ac & 3) * 2)) & 3;
        index = m.bits == 5 ? (crumb == 3 ? 0 : crumb + 1) : crumb;
      } else if (m.bits == 4) {
        const int byte = m.packed[rowOffset + (ac >> 1)];
        index = (byte >> ((ac & 1) * 4)) & 15;
      } else {
        const int64_t bitPosition = ac * 3;
        const int64_t bytePosition = rowOffset + (bitPosition >> 3);
        const int shift = int(bitPosition & 7);
        const uint32_t hi = bytePosition + 1 < packedTotal ? m.packed[bytePosition + 1] : 0u;
        const uint32_t word = uint32_t(m.packed[bytePosition]) | (hi << 8);
        index = (word >> shift) & 7;
      }
      // `codebook[index] ?? 0`: ternary crumb 2 maps to index 3, past the 3-entry codebook.
      const double level = index < codebookLength ? double(codebook[index]) : 0.0;
      temporary[col] = float(level * norm);
    }
    fwht(temporary.data(), 0, g);
    const int64_t outputOffset = group * g;
    const int64_t count = std::min<int64_t>(g, m.inputSize - outputOffset);
    for (int64_t col = 0; col < count; col++)
      result[outputOffset + col] = float(double(temporary[col]) * inverseRoot);
  }
}

// denseMatvec, cq.ts:297-318.
std::vector<float> denseMatvec(const std::vector<float>& matrix, int64_t outputSize,
                               const std::vector<float>& input, const std::vector<float>* bias) {
  invariant(int64_t(matrix.size()) == outputSize * int64_t(input.size()), INVALID_CACT,
            "Dense matrix shape does not match the vector");
  std::vector<float> result(outputSize);
  for (int64_t row = 0; row < outputSize; row++) {
    double sum = bias && row < int64_t(bias->size()) ? double((*bias)[row]) : 0.0;
    const int64_t offset = row * int64_t(input.size());
    for (size_t c = 0; c < input.size(); c++) sum += double(matrix[offset + c]) * double(input[c]);
    result[row] = float(sum);
  }
  return result;
}

// ---------------------------------------------------------------- math (src/model/math.ts)

// sigmoid, math.ts:3-10.
inline double sigmoid(double value) {
  if (value >= 0) {
    const double e = std::exp(-value);
    return 1 / (1 + e);
  }
  const double e = std::exp(value);
  return e / (1 + e);
}
inline double silu(double value) { return value * sigmoid(value); }  // math.ts:12-14

// rmsNorm, math.ts:16-32.
std::vector<float> rmsNorm(const std::vector<float>& input, const std::vector<float>& scale,
                           double epsilon = 1e-6) {
  double sumSquares = 0;
  for (float v : input) sumSquares += double(v) * double(v);
  const double inverse = 1 / std::sqrt(sumSquares / double(input.size()) + epsilon);
  std::vector<float> output(input.size());
  for (size_t i = 0; i < input.size(); i++) {
    const double s = i < scale.size() ? double(scale[i]) : 0.0;
    output[i] = float((1 + s) * double(input[i]) * inverse);
  }
  return output;
}

// rmsUnit, math.ts:34-44.
std::vector<float> rmsUnit(const std::vector<float>& input, double epsilon = 1e-6) {
  double sumSquares = 0;
  for (float v : input) sumSquares += double(v) * double(v);
  const double inverse = 1 / std::sqrt(sumSquares / double(input.size()) + epsilon);
  std::vector<float> output(input.size());
  for (size_t i = 0; i < input.size(); i++) output[i] = float(double(input[i]) * inverse);
  return output;
}

// softmaxInPlace, math.ts:46-60.
void softmaxInPlace(float* values, int64_t length) {
  if (length == 0) return;
  double maximum = values[0];
  for (int64_t i = 1; i < length; i++) maximum = std::max(maximum, double(values[i]));
  double total = 0;
  for (int64_t i = 0; i < length; i++) {
    const double value = std::exp(double(values[i]) - maximum);
    values[i] = float(value);
    total += value;
  }
  const double inverse = total > 0 ? 1 / total : 0;
  for (int64_t i = 0; i < length; i++) values[i] = float(double(values[i]) * inverse);
}

// sinkhorn, math.ts:63-92 (log-space, Float64Array working copy).
void sinkhorn(float* logits, int size, int iterations = 20) {
  std::vector<double> v(logits, logits + size * size);
  for (int it = 0; it < iterations; it++) {
    for (int row = 0; row < size; row++) {
      const int o = row * size;
      double maximum = v[o];
      for (int c = 1; c < size; c++) maximum = std::max(maximum, v[o + c]);
      double sum = 0;
      for (int c = 0; c < size; c++) sum += std::exp(v[o + c] - maximum);
      const double logSum = std::log(sum) + maximum;
      for (int c = 0; c < size; c++) v[o + c] = v[o + c] - logSum;
    }
    for (int col = 0; col < size; col++) {
      double maximum = v[col];
      for (int r = 1; r < size; r++) maximum = std::max(maximum, v[r * size + col]);
      double sum = 0;
      for (int r = 0; r < size; r++) sum += std::exp(v[r * size + col] - maximum);
      const double logSum = std::log(sum) + maximum;
      for (int r = 0; r < size; r++) v[r * size + col] = v[r * size + col] - logSum;
    }
  }
  for (int i = 0; i < size * size; i++) logits[i] = float(std::exp(v[i]));
}

// applyRope, math.ts:94-115.  `theta ** e` is Math.pow.
void applyRope(float* vector, int headCount, int headDimension, int64_t position, double theta) {
  const int half = headDimension >> 1;
  for (int head = 0; head < headCount; head++) {
    const int offset = head * headDimension;
    for (int d = 0; d < half; d++) {
      const double frequency = std::pow(theta, -(2.0 * d) / double(headDimension));
      const double angle = double(position) * frequency;
      const double cosine = std::cos(angle), sine = std::sin(angle);
      const double first = vector[offset + d], second = vector[offset + d + half];
      vector[offset + d] = float(first * cosine - second * sine);
      vector[offset + d + half] = float(second * cosine + first * sine);
    }
  }
}

// hadamardMlp, math.ts:117-138.
std::vector<float> hadamardMlp(const std::vector<float>& input, const std::vector<float>& d1,
                               const std::vector<float>& d2, const std::vector<float>& d3,
                               int hadamardDimension) {
  std::vector<float> values(hadamardDimension, 0.0f);
  for (size_t i = 0; i < input.size(); i++) values[i] = float(double(input[i]) * double(d1[i]));
  const double inverseRoot = 1 / std::sqrt(double(hadamardDimension));
  fwht(values.data(), 0, hadamardDimension);
  for (int i = 0; i < hadamardDimension; i++)
    values[i] = float(silu(double(values[i]) * inverseRoot * double(d2[i])));
  fwht(values.data(), 0, hadamardDimension);
  std::vector<float> output(input.size());
  for (size_t i = 0; i < output.size(); i++)
    output[i] = float(double(values[i]) * inverseRoot * double(d3[i]));
  return output;
}

// argmax, math.ts:140-151 (strict >, so the lowest index wins ties).
int argmaxF(const float* values, int64_t n) {
  int best = 0;
  double bestValue = n > 0 ? double(values[0]) : kNegInf;
  for (int64_t i = 1; i < n; i++) {
    const double v = values[i];
    if (v > bestValue) {
      bestValue = v;
      best = int(i);
    }
  }
  return best;
}

// logSoftmaxAt, math.ts:153-160.
double logSoftmaxAt(const float* logits, int64_t n, int64_t token) {
  double maximum = n > 0 ? double(logits[0]) : kNegInf;
  for (int64_t i = 1; i < n; i++) maximum = std::max(maximum, double(logits[i]));
  double sum = 0;
  for (int64_t i = 0; i < n; i++) sum += std::exp(double(logits[i]) - maximum);
  const double at = token >= 0 && token < n ? double(logits[token]) : kNegInf;
  return at - maximum - std::log(sum);
}

// roundTiesToEven, runtime.ts:901-907.
inline double roundTiesToEven(double value) {
  const double lower = std::floor(value);
  const double fraction = value - lower;
  if (fraction < 0.5) return lower;
  if (fraction > 0.5) return lower + 1;
  return (int64_t(lower) & 1) == 0 ? lower : lower + 1;
}

// ---------------------------------------------------------------- archive (src/model/cact.ts)

constexpr uint32_t kCactTag = 0x05e12a83u;  // cact.ts:4
constexpr size_t kHeaderBytes = 120;        // cact.ts:5
constexpr size_t kRecordBytes = 44;         // cact.ts:6

struct Geometry {
  int32_t kvWindow, kvBits, vocabularySize, modelDimension, numberOfHeads, numberOfKVHeads,
      numberOfLayers, headDimension, maximumSequenceLength, hadamardDimension, mhcLanes,
      engramSlots, engramSubDimension, numberOfEngramTables, engramConvolutionTaps,
      engramConvolutionDilation;
  std::vector<int32_t> engramOrders, engramLayers;
  float ropeTheta;
  uint32_t fields[29];
};

struct Record {
  int dtype, rank;
  int64_t shape[4];
  uint64_t offset, byteLength;
  uint32_t groupSize, bits;
};

struct Tensor {
  enum Kind { Dense, Raw, Cq } kind;
  std::vector<float> data;  // dense
  CqMatrix cq;              // cq
  const Record* record;
};

struct Layer {
  std::vector<float> normInput, queryNorm, keyNorm, postAttentionNorm, preHadamardNorm,
      hadamardD1, hadamardD2, hadamardD3;
  CqMatrix queryProjection, keyProjection, valueProjection, gateProjection, outputProjection;
  double attentionGate;
};

struct EngramSite {
  CqMatrix tables, keyProjection, valueProjection;
  std::vector<float> taps;
};

struct ProbeHead {
  std::vector<float> probes, projection, bias;
  int64_t probeCount, outputSize;
};

}  // namespace

struct ref_model {
  std::vector<uint8_t> bytes;
  Geometry geometry;
  std::vector<float> codebook, cb2, cb3, cb4;
  std::vector<Record> records;
  std::vector<Tensor> tensors;
  CqMatrix embedding;
  std::vector<Layer> layers;
  std::vector<float> mhcAPre, mhcAPost, mhcAResidual, mhcBPre, mhcBPost, mhcBResidual;
  CqMatrix mhcPhiPre, mhcPhiPost, mhcPhiResidual;
  std::vector<EngramSite> engrams;
  std::vector<float> finalNorm;
  bool hasConfidence = false;
  ProbeHead confidence;
};

namespace {

void assertRange(size_t total, uint64_t offset, uint64_t length, const std::string& label) {
  invariant(offset <= total && length <= total - offset, INVALID_CACT,
            label + " points outside the " + std::to_string(total) + "-byte archive (offset " +
                std::to_string(offset) + ", length " + std::to_string(length) + ")");
}

// parseCact, cact.ts:189-562.
void parse(ref_model& M) {
  const std::vector<uint8_t>& bytes = M.bytes;
  assertRange(bytes.size(), 0, kHeaderBytes, "CACT header");
  const uint8_t* b = bytes.data();
  auto u32 = [&](int i) { return rd_u32(b + i * 4); };
  const uint32_t tag = u32(0);
  if (tag != kCactTag) {
    char buf[96];
    std::snprintf(buf, sizeof buf, "Invalid .cact tag 0x%x (expected 0x%x)", tag, kCactTag);
    fail(INVALID_CACT, buf);
  }
  const uint32_t numberOfTensors = u32(1), codebookLength = u32(2);
  invariant(numberOfTensors > 0, INVALID_CACT, "The .cact archive has no tensors");
  invariant(codebookLength >= 28, UNSUPPORTED_CACT,
            "Needle 2 requires the CQ2/CQ3/CQ4 codebook (28 entries); archive has " +
                std::to_string(codebookLength));
  const uint32_t numberOfOrders = u32(19), numberOfSites = u32(24);
  invariant(numberOfOrders <= 4 && numberOfSites <= 4, UNSUPPORTED_CACT,
            "The current .cact format supports at most four engram orders and sites");
  Geometry& G = M.geometry;
  for (int i = 0; i < 29; i++) G.fields[i] = u32(i);
  for (uint32_t i = 0; i < numberOfOrders; i++) G.engramOrders.push_back(int32_t(u32(20 + i)));
  for (uint32_t i = 0; i < numberOfSites; i++) G.engramLayers.push_back(int32_t(u32(25 + i)));
  G.kvWindow = u32(3);
  G.kvBits = u32(4);
  G.vocabularySize = u32(5);
  G.modelDimension = u32(6);
  G.numberOfHeads = u32(7);
  G.numberOfKVHeads = u32(8);
  G.numberOfLayers = u32(9);
  G.headDimension = u32(10);
  G.maximumSequenceLength = u32(11);
  G.hadamardDimension = u32(12);
  G.mhcLanes = u32(13);
  G.engramSlots = u32(14);
  G.engramSubDimension = u32(15);
  G.numberOfEngramTables = u32(16);
  G.engramConvolutionTaps = u32(17);
  G.engramConvolutionDilation = u32(18);
  G.ropeTheta = rd_f32(b + 29 * 4);
  invariant(G.modelDimension > 0 && G.vocabularySize > 0, INVALID_CACT,
            "Model geometry contains a zero-sized vocabulary or hidden dimension");
  invariant(G.numberOfHeads > 0 && G.numberOfKVHeads > 0 &&
                G.numberOfHeads % G.numberOfKVHeads == 0,
            UNSUPPORTED_CACT, "Attention heads must be a positive multiple of KV heads");
  invariant(int64_t(G.numberOfHeads) * G.headDimension > 0, INVALID_CACT,
            "Invalid attention dimensions");
  invariant((G.hadamardDimension & (G.hadamardDimension - 1)) == 0, UNSUPPORTED_CACT,
            "Hadamard dimension must be a power of two");

  const size_t codebookOffset = kHeaderBytes;
  assertRange(bytes.size(), codebookOffset, uint64_t(codebookLength) * 4, "CQ codebook");
  M.codebook.resize(codebookLength);
  for (uint32_t i = 0; i < codebookLength; i++) M.codebook[i] = rd_f32(b + codebookOffset + i * 4);
  M.cb2.assign(M.codebook.begin(), M.codebook.begin() + 4);
  M.cb3.assign(M.codebook.begin() + 4, M.codebook.begin() + 12);
  M.cb4.assign(M.codebook.begin() + 12, M.codebook.begin() + 28);

  const size_t directoryOffset = codebookOffset + size_t(codebookLength) * 4;
  assertRange(bytes.size(), directoryOffset, uint64_t(numberOfTensors) * kRecordBytes,
              "Tensor directory");
  M.records.resize(numberOfTensors);
  for (uint32_t i = 0; i < numberOfTensors; i++) {
    const uint8_t* r = b + directoryOffset + size_t(i) * kRecordBytes;
    Record& rec = M.records[i];
    rec.dtype = r[0];
    rec.rank = r[1];
    invariant(rec.rank <= 4, UNSUPPORTED_CACT,
              "Tensor " + std::to_string(i) + " has " + std::to_string(rec.rank) +
                  " dimensions; the format supports four");
    for (int d = 0; d < 4; d++) rec.shape[d] = d < rec.rank ? int64_t(rd_u32(r + 4 + d * 4)) : 0;
    rec.offset = rd_u64(r + 20);
    rec.byteLength = rd_u64(r + 28);
    const uint64_t safe = (uint64_t(1) << 53) - 1;
    invariant(rec.offset <= safe && rec.byteLength <= safe, UNSUPPORTED_CACT,
              "Tensor " + std::to_string(i) + " offset does not fit safely in JavaScript");
    assertRange(bytes.size(), rec.offset, rec.byteLength, "Tensor " + std::to_string(i));
    rec.groupSize = rd_u32(r + 36);
    rec.bits = rd_u32(r + 40);
  }

  M.tensors.resize(numberOfTensors);
  for (uint32_t i = 0; i < numberOfTensors; i++) {
    const Record& rec = M.records[i];
    Tensor& t = M.tensors[i];
    t.record = &rec;
    int64_t count = 1;
    for (int d = 0; d < rec.rank; d++) count *= rec.shape[d];
    if (rec.dtype == 1) {
      invariant(rec.byteLength == uint64_t(count) * 2, INVALID_CACT,
                "FP16 tensor " + std::to_string(i) + " has an inconsistent byte length");
      t.kind = Tensor::Dense;
      t.data.resize(count);
      for (int64_t k = 0; k < count; k++) {
        const uint8_t* p = b + rec.offset + k * 2;
        t.data[k] = f16_to_f32(uint32_t(p[0]) | (uint32_t(p[1]) << 8));
      }
    } else if (rec.dtype == 2) {
      invariant(rec.byteLength == uint64_t(count) * 4, INVALID_CACT,
                "FP32 tensor " + std::to_string(i) + " has an inconsistent byte length");
      t.kind = Tensor::Dense;
      t.data.resize(count);
      for (int64_t k = 0; k < count; k++) t.data[k] = rd_f32(b + rec.offset + k * 4);
    } else if (rec.dtype == 4) {
      t.kind = Tensor::Raw;
    } else if (rec.dtype == 3) {
      invariant(rec.rank == 2, INVALID_CACT, "CQ tensor " + std::to_string(i) + " is not a matrix");
      invariant(rec.groupSize > 0 && (rec.groupSize & (rec.groupSize - 1)) == 0, UNSUPPORTED_CACT,
                "CQ tensor " + std::to_string(i) + " has non-power-of-two group " +
                    std::to_string(rec.groupSize));
      invariant(rec.bits == 2 || rec.bits == 3 || rec.bits == 4 || rec.bits == 5,
                UNSUPPORTED_CACT,
                "CQ tensor " + std::to_string(i) + " uses unsupported record width " +
                    std::to_string(rec.bits));
      CqMatrix& m = t.cq;
      m.outputSize = int32_t(rec.shape[0]);
      m.inputSize = int32_t(rec.shape[1]);
      m.groupSize = int32_t(rec.groupSize);
      m.inputSizePadded = int32_t((rec.shape[1] + rec.groupSize - 1) / rec.groupSize * rec.groupSize);
      m.bits = int32_t(rec.bits);
      const int64_t packedBits = rec.bits == 5 ? 2 : rec.bits;
      invariant((int64_t(m.inputSizePadded) * packedBits) % 8 == 0, INVALID_CACT,
                "CQ tensor " + std::to_string(i) + " has a fractional packed row size");
      m.rowByteLength = int64_t(m.inputSizePadded) * packedBits / 8;
      const uint64_t packedByteLength = uint64_t(m.outputSize) * m.rowByteLength;
      const uint64_t normCount = uint64_t(m.outputSize) * (m.inputSizePadded / m.groupSize);
      invariant(rec.byteLength == packedByteLength + normCount * 2, INVALID_CACT,
                "CQ tensor " + std::to_string(i) + " has an inconsistent packed/norm length");
      m.packed = b + rec.offset;
      m.norms = b + rec.offset + packedByteLength;
      m.cb2 = M.cb2.data();
      m.cb3 = M.cb3.data();
      m.cb4 = M.cb4.data();
      t.kind = Tensor::Cq;
    } else {
      static const char* names[] = {"0", "FP16", "FP32", "CQ", "RAW"};
      fail(UNSUPPORTED_CACT, "Tensor " + std::to_string(i) + " uses unknown dtype " +
                                 (rec.dtype <= 4 ? std::string(names[rec.dtype])
                                                 : std::to_string(rec.dtype)));
    }
  }

  size_t cursor = 0;
  auto take = [&](const std::string& name) -> Tensor& {
    invariant(cursor < M.tensors.size(), INVALID_CACT, "Archive ended before " + name);
    return M.tensors[cursor++];
  };
  auto dense = [&](const std::string& name) -> std::vector<float> {
    Tensor& t = take(name);
    invariant(t.kind == Tensor::Dense, INVALID_CACT, name + " must be an FP16/FP32 tensor");
    return t.data;
  };
  auto cq = [&](const std::string& name) -> CqMatrix {
    Tensor& t = take(name);
    invariant(t.kind == Tensor::Cq, INVALID_CACT, name + " must be a Cactus-Quant matrix");
    return t.cq;
  };

  M.embedding = cq("embedding");
  invariant(M.embedding.outputSize == G.vocabularySize && M.embedding.inputSize == G.modelDimension,
            INVALID_CACT, "Embedding shape does not match model geometry");
  for (int l = 0; l < G.numberOfLayers; l++) {
    const std::string p = "layer " + std::to_string(l);
    Layer L;
    L.normInput = dense(p + " input norm");
    L.queryProjection = cq(p + " query projection");
    L.keyProjection = cq(p + " key projection");
    L.valueProjection = cq(p + " value projection");
    L.queryNorm = dense(p + " query norm");
    L.keyNorm = dense(p + " key norm");
    L.gateProjection = cq(p + " gate projection");
    L.outputProjection = cq(p + " output projection");
    L.postAttentionNorm = dense(p + " post-attention norm");
    std::vector<float> gate = dense(p + " attention gate");
    L.attentionGate = gate.empty() ? 0.0 : double(gate[0]);
    L.preHadamardNorm = dense(p + " pre-Hadamard norm");
    L.hadamardD1 = dense(p + " Hadamard d1");
    L.hadamardD2 = dense(p + " Hadamard d2");
    L.hadamardD3 = dense(p + " Hadamard d3");
    M.layers.push_back(std::move(L));
  }
  M.mhcAPre = dense("mHC a_pre");
  M.mhcAPost = dense("mHC a_post");
  M.mhcAResidual = dense("mHC a_res");
  M.mhcBPre = dense("mHC b_pre");
  M.mhcBPost = dense("mHC b_post");
  M.mhcBResidual = dense("mHC b_res");
  M.mhcPhiPre = cq("mHC phi_pre");
  M.mhcPhiPost = cq("mHC phi_post");
  M.mhcPhiResidual = cq("mHC phi_res");
  for (size_t s = 0; s < G.engramLayers.size(); s++) {
    const std::string p = "engram " + std::to_string(s);
    EngramSite E;
    E.tables = cq(p + " tables");
    E.keyProjection = cq(p + " key projection");
    E.valueProjection = cq(p + " value projection");
    E.taps = dense(p + " taps");
    M.engrams.push_back(std::move(E));
  }
  M.finalNorm = dense("final norm");

  if (cursor < M.tensors.size() && M.tensors[cursor].kind == Tensor::Dense) {
    std::vector<float> manifest = M.tensors[cursor].data;
    cursor++;
    for (float raw : manifest) {
      const double code = std::floor(double(raw) + 0.5);  // Math.round
      invariant(code == 1 || code == 2, UNSUPPORTED_CACT,
                "Unknown probe-head manifest code " + std::to_string(int64_t(code)));
      const std::string name = code == 1 ? "contrastive" : "confidence";
      Tensor& probesT = take(name + " probes");
      Tensor& projT = take(name + " projection");
      Tensor& biasT = take(name + " bias");
      invariant(probesT.kind == Tensor::Dense, INVALID_CACT, name + " probes must be an FP16/FP32 tensor");
      invariant(projT.kind == Tensor::Dense, INVALID_CACT, name + " projection must be an FP16/FP32 tensor");
      invariant(biasT.kind == Tensor::Dense, INVALID_CACT, name + " bias must be an FP16/FP32 tensor");
      ProbeHead H;
      H.probes = probesT.data;
      H.projection = projT.data;
      H.bias = biasT.data;
      H.probeCount = probesT.record->rank > 0 ? probesT.record->shape[0] : 0;
      H.outputSize = projT.record->rank > 0 ? projT.record->shape[0] : int64_t(H.bias.size());
      invariant(H.probeCount > 0 && int64_t(H.probes.size()) == H.probeCount * G.modelDimension,
                INVALID_CACT, name + " probe shape is inconsistent");
      invariant(int64_t(H.projection.size()) == H.outputSize * H.probeCount * G.modelDimension,
                INVALID_CACT, name + " projection shape is inconsistent");
      if (code == 2) {
        M.confidence = std::move(H);
        M.hasConfidence = true;
      }
    }
  }
  bool tokenizer = false;
  while (cursor < M.tensors.size()) {
    Tensor& t = take("trailing tensor");
    if (t.kind == Tensor::Raw) {
      invariant(!tokenizer, INVALID_CACT, "Archive contains more than one RAW tokenizer tensor");
      tokenizer = true;
    } else {
      fail(UNSUPPORTED_CACT, "Unexpected trailing tensor " + std::to_string(cursor - 1));
    }
  }
  invariant(tokenizer, INVALID_CACT, "Archive does not contain its RAW SentencePiece tokenizer");
}

// ---------------------------------------------------------------- runtime (src/model/runtime.ts)

constexpr uint32_t kEngramSeed = 0x9e3779b9u;   // runtime.ts:22
constexpr uint32_t kEngramPrime = 0x01000193u;  // runtime.ts:23

// OnlineProbePool, runtime.ts:48-105.
struct ProbePool {
  const ProbeHead* head;
  int64_t dimension;
  std::vector<double> maximum, denominator, weighted;
  ProbePool(const ProbeHead* h, int64_t d)
      : head(h), dimension(d), maximum(h->probeCount, kNegInf), denominator(h->probeCount, 0.0),
        weighted(h->probeCount * d, 0.0) {}
  void add(const std::vector<float>& cell) {
    const double scale = 1 / std::sqrt(double(dimension));
    for (int64_t p = 0; p < head->probeCount; p++) {
      double score = 0;
      const int64_t po = p * dimension;
      for (int64_t i = 0; i < dimension; i++) score += double(cell[i]) * double(head->probes[po + i]);
      score *= scale;
      const double prev = maximum[p];
      if (score <= prev) {
        const double w = std::exp(score - prev);
        denominator[p] = denominator[p] + w;
        for (int64_t i = 0; i < dimension; i++) weighted[po + i] = weighted[po + i] + w * double(cell[i]);
      } else {
        const double oldWeight = std::isfinite(prev) ? std::exp(prev - score) : 0;
        denominator[p] = denominator[p] * oldWeight + 1;
        for (int64_t i = 0; i < dimension; i++)
          weighted[po + i] = weighted[po + i] * oldWeight + double(cell[i]);
        maximum[p] = score;
      }
    }
  }
  std::vector<float> output() const {
    std::vector<float> pooled(head->probeCount * dimension);
    for (int64_t p = 0; p < head->probeCount; p++) {
      const double den = std::max(denominator[p], 1e-30);
      for (int64_t i = 0; i < dimension; i++)
        pooled[p * dimension + i] = float(weighted[p * dimension + i] / den);
    }
    return denseMatvec(head->projection, head->outputSize, pooled, &head->bias);
  }
};

}  // namespace

// NeedleRuntime, runtime.ts:108-878 (host loop path, no resident session).
struct ref_runtime {
  const ref_model* M;
  int kvMode;  // 0 int8, 1 float32
  bool collectConfidence;
  int64_t maximumLength = 0, sinkLength = 0, kvAllocation = 0, position = 0;
  std::vector<int32_t> history;
  std::vector<int8_t> keyInt8, valueInt8;
  std::vector<float> keyFloat, valueFloat, keyScale, valueScale;
  std::vector<float> engramRing;
  std::vector<uint8_t> engramValid;
  int64_t engramDepth = 0, engramPosition = 0;
  std::unique_ptr<ProbePool> pool;
  std::vector<float> x;

  const Geometry& G() const { return M->geometry; }

  // reset, runtime.ts:150-225.
  void reset(int64_t maxLen, int64_t sink) {
    const Geometry& g = G();
    invariant(maxLen > 0 && maxLen <= g.maximumSequenceLength, CONTEXT_OVERFLOW,
              "Runtime length " + std::to_string(maxLen) + " is outside model limit " +
                  std::to_string(g.maximumSequenceLength));
    maximumLength = maxLen;
    sinkLength = std::min(std::max<int64_t>(sink, 0), maxLen);
    position = 0;
    history.clear();
    kvAllocation = g.kvWindow > 0 ? std::min<int64_t>(maxLen, sinkLength + g.kvWindow) : maxLen;
    const int64_t kvElements = int64_t(g.numberOfLayers) * g.numberOfKVHeads * kvAllocation * g.headDimension;
    const int64_t scaleElements = int64_t(g.numberOfLayers) * g.numberOfKVHeads * kvAllocation;
    if (kvMode == 1) {
      keyFloat.assign(kvElements, 0.0f);
      valueFloat.assign(kvElements, 0.0f);
      keyInt8.clear();
      valueInt8.clear();
    } else {
      keyInt8.assign(kvElements, 0);
      valueInt8.assign(kvElements, 0);
      keyFloat.clear();
      valueFloat.clear();
    }
    keyScale.assign(scaleElements, 0.0f);
    valueScale.assign(scaleElements, 0.0f);
    int32_t maximumOrder = 1;
    for (int32_t o : g.engramOrders) maximumOrder = std::max(maximumOrder, o);
    engramDepth = int64_t(g.engramConvolutionTaps - 1) * maximumOrder + 1;
    engramRing.assign(g.engramLayers.size() * engramDepth * g.modelDimension, 0.0f);
    engramValid.assign(g.engramLayers.size() * engramDepth, 0);
    engramPosition = 0;
    pool.reset();
    if (collectConfidence && M->hasConfidence)
      pool = std::make_unique<ProbePool>(&M->confidence, g.modelDimension);
  }

  // #kvSlot / #cacheBase / #scaleIndex, runtime.ts:659-677.
  int64_t kvSlot(int64_t pos) const {
    const int64_t window = G().kvWindow;
    if (window == 0) return pos;
    if (pos < sinkLength) return pos;
    return sinkLength + (pos - sinkLength) % window;
  }
  int64_t cacheBase(int64_t layer, int64_t head, int64_t slot) const {
    return ((layer * G().numberOfKVHeads + head) * kvAllocation + slot) * G().headDimension;
  }
  int64_t scaleIndex(int64_t layer, int64_t head, int64_t slot) const {
    return (layer * G().numberOfKVHeads + head) * kvAllocation + slot;
  }

  // #rmsNormSlice, runtime.ts:647-657.
  static void rmsNormSlice(float* values, int64_t length, const std::vector<float>& scale) {
    double sumSquares = 0;
    for (int64_t i = 0; i < length; i++) sumSquares += double(values[i]) * double(values[i]);
    const double inverse = 1 / std::sqrt(sumSquares / double(length) + 1e-6);
    for (int64_t i = 0; i < length; i++)
      values[i] = float((1 + double(scale[i])) * double(values[i]) * inverse);
  }

  // #storeKV, runtime.ts:679-717.
  void storeKV(int64_t layer, int64_t pos, const std::vector<float>& key, const std::vector<float>& value) {
    const Geometry& g = G();
    const int64_t slot = kvSlot(pos);
    const int hd = g.headDimension;
    for (int head = 0; head < g.numberOfKVHeads; head++) {
      const int64_t vo = int64_t(head) * hd, co = cacheBase(layer, head, slot), so = scaleIndex(layer, head, slot);
      if (kvMode == 1) {
        for (int i = 0; i < hd; i++) {
          keyFloat[co + i] = key[vo + i];
          valueFloat[co + i] = value[vo + i];
        }
        keyScale[so] = 1;
        valueScale[so] = 1;
      } else {
        double keyMaximum = 1e-12, valueMaximum = 1e-12;
        for (int i = 0; i < hd; i++) {
          keyMaximum = std::max(keyMaximum, std::fabs(double(key[vo + i])));
          valueMaximum = std::max(valueMaximum, std::fabs(double(value[vo + i])));
        }
        const double ks = keyMaximum / 127, vs = valueMaximum / 127;
        keyScale[so] = float(ks);
        valueScale[so] = float(vs);
        for (int i = 0; i < hd; i++) {
          keyInt8[co + i] = int8_t(roundTiesToEven(double(key[vo + i]) / ks));
          valueInt8[co + i] = int8_t(roundTiesToEven(double(value[vo + i]) / vs));
        }
      }
    }
  }

  // #attention, runtime.ts:719-786.
  std::vector<float> attention(int64_t layer, int64_t pos, const std::vector<float>& query) const {
    const Geometry& g = G();
    const int reps = g.numberOfHeads / g.numberOfKVHeads, hd = g.headDimension;
    std::vector<float> output(int64_t(g.numberOfHeads) * hd, 0.0f);
    const int64_t prefixCount = std::min(sinkLength, pos + 1);
    const int64_t recentLow = g.kvWindow > 0 ? std::max(prefixCount, pos + 1 - g.kvWindow) : prefixCount;
    std::vector<int64_t> logical;
    for (int64_t i = 0; i < prefixCount; i++) logical.push_back(i);
    for (int64_t i = recentLow; i <= pos; i++) logical.push_back(i);
    const int64_t count = int64_t(logical.size());
    std::vector<float> scores(count);
    const double inverseRoot = 1 / std::sqrt(double(hd));
    for (int kvHead = 0; kvHead < g.numberOfKVHeads; kvHead++) {
      for (int rep = 0; rep < reps; rep++) {
        const int qh = kvHead * reps + rep;
        const int64_t qo = int64_t(qh) * hd;
        for (int64_t t = 0; t < count; t++) {
          const int64_t slot = kvSlot(logical[t]);
          const int64_t co = cacheBase(layer, kvHead, slot), so = scaleIndex(layer, kvHead, slot);
          const double ks = keyScale[so];
          double dot = 0;
          if (kvMode == 1) {
            for (int i = 0; i < hd; i++) dot += double(query[qo + i]) * double(keyFloat[co + i]);
          } else {
            for (int i = 0; i < hd; i++) dot += double(query[qo + i]) * double(keyInt8[co + i]) * ks;
          }
          scores[t] = float(dot * inverseRoot);
        }
        softmaxInPlace(scores.data(), count);
        const int64_t oo = int64_t(qh) * hd;
        for (int64_t t = 0; t < count; t++) {
          const int64_t slot = kvSlot(logical[t]);
          const int64_t co = cacheBase(layer, kvHead, slot), so = scaleIndex(layer, kvHead, slot);
          const double w = scores[t];
          if (kvMode == 1) {
            for (int i = 0; i < hd; i++)
              output[oo + i] = float(double(output[oo + i]) + w * double(valueFloat[co + i]));
          } else {
            const double vs = valueScale[so];
            for (int i = 0; i < hd; i++)
              output[oo + i] = float(double(output[oo + i]) + w * double(valueInt8[co + i]) * vs);
          }
        }
      }
    }
    return output;
  }

  // #engramLookup, runtime.ts:788-818.
  bool engramLookup(std::vector<uint32_t>& indices, std::vector<uint32_t>& valid) const {
    const Geometry& g = G();
    if (g.engramLayers.empty()) return false;
    invariant(!g.engramOrders.empty() && g.numberOfEngramTables % int(g.engramOrders.size()) == 0,
              INVALID_CACT, "Engram table count is not divisible by order count");
    const int headsPerOrder = g.numberOfEngramTables / int(g.engramOrders.size());
    indices.assign(g.numberOfEngramTables, 0);
    valid.assign(g.numberOfEngramTables, 0);
    int table = 0;
    for (int oi = 0; oi < int(g.engramOrders.size()); oi++) {
      const int order = g.engramOrders[oi];
      for (int head = 0; head < headsPerOrder; head++) {
        uint32_t hash = kEngramSeed * uint32_t(oi * headsPerOrder + head + 1);
        bool isValid = true;
        for (int offset = 0; offset < order; offset++) {
          const int64_t hi = int64_t(history.size()) - 1 - offset;
          const uint32_t token = hi >= 0 ? uint32_t(history[hi]) : 0u;
          hash = (hash ^ token) * kEngramPrime;
          if (offset == order - 1) isValid = hi >= 0;
        }
        hash = hash ^ (hash >> 15);
        indices[table] = hash % uint32_t(g.engramSlots);
        valid[table] = isValid ? 1 : 0;
        table++;
      }
    }
    return true;
  }

  // #engramStep, runtime.ts:820-877.
  void engramStep(bool have, const std::vector<uint32_t>& indices, const std::vector<uint32_t>& valid,
                  std::vector<std::vector<float>>& keys, std::vector<std::vector<float>>& values) {
    const Geometry& g = G();
    keys.clear();
    values.clear();
    if (!have) return;
    const int D = g.modelDimension;
    std::vector<std::vector<float>> projected;
    for (size_t s = 0; s < M->engrams.size(); s++) {
      const EngramSite& site = M->engrams[s];
      std::vector<float> concatenated(int64_t(g.numberOfEngramTables) * g.engramSubDimension, 0.0f);
      for (int t = 0; t < g.numberOfEngramTables; t++) {
        if (valid[t]) {
          const int64_t row = int64_t(t) * g.engramSlots + indices[t];
          std::vector<float> r(site.tables.inputSize);
          dequantizeRow(site.tables, row, r.data());
          std::copy(r.begin(), r.end(), concatenated.begin() + int64_t(t) * g.engramSubDimension);
        }
      }
      projected.push_back(cqMatvec(site.keyProjection, concatenated.data(), concatenated.size(), 0,
                                   site.keyProjection.outputSize));
      projected.push_back(cqMatvec(site.valueProjection, concatenated.data(), concatenated.size(), 0,
                                   site.valueProjection.outputSize));
    }
    int32_t maximumOrder = 0;
    for (int32_t o : g.engramOrders) maximumOrder = std::max(maximumOrder, o);
    for (size_t s = 0; s < M->engrams.size(); s++) {
      const EngramSite& site = M->engrams[s];
      keys.push_back(projected[s * 2]);
      const std::vector<float>& valueNow = projected[s * 2 + 1];
      const int64_t slot = engramPosition % engramDepth;
      const int64_t ringOffset = (int64_t(s) * engramDepth + slot) * D;
      std::copy(valueNow.begin(), valueNow.end(), engramRing.begin() + ringOffset);
      engramValid[s * engramDepth + slot] = 1;
      std::vector<float> mixed(D, 0.0f);
      for (int tap = 0; tap < g.engramConvolutionTaps; tap++) {
        const int64_t prev = engramPosition - int64_t(tap) * maximumOrder;
        if (prev < 0) continue;
        const int64_t prevSlot = prev % engramDepth;
        if (!engramValid[s * engramDepth + prevSlot]) continue;
        const int64_t po = (int64_t(s) * engramDepth + prevSlot) * D;
        const int64_t to = int64_t(tap) * D;
        for (int i = 0; i < D; i++)
          mixed[i] = float(double(mixed[i]) + double(site.taps[to + i]) * double(engramRing[po + i]));
      }
      values.push_back(std::move(mixed));
    }
    engramPosition++;
  }

  // #attentionDelta, runtime.ts:585-611.
  std::vector<float> attentionDelta(const std::vector<float>& projected, const std::vector<float>& blockInput,
                                    const std::vector<float>& updateInput, const Layer& L) const {
    const int D = G().modelDimension;
    std::vector<float> normalized = rmsNorm(projected, L.postAttentionNorm);
    const double attentionScale = sigmoid(L.attentionGate);
    std::vector<float> after(D);
    for (int i = 0; i < D; i++) after[i] = float(double(blockInput[i]) + attentionScale * double(normalized[i]));
    std::vector<float> pre = rmsNorm(after, L.preHadamardNorm);
    std::vector<float> mlp = hadamardMlp(pre, L.hadamardD1, L.hadamardD2, L.hadamardD3, G().hadamardDimension);
    std::vector<float> delta(D);
    for (int i = 0; i < D; i++)
      delta[i] = float(double(after[i]) + double(mlp[i]) - double(updateInput[i]));
    return delta;
  }

  // step, runtime.ts:280-583 (host-loop path).  Returns logits when wantLogits.
  void step(int32_t token, bool wantLogits, std::vector<float>* logitsOut) {
    const Geometry& g = G();
    invariant(maximumLength > 0, INVALID_CACT, "Call runtime.reset() before decoding");
    invariant(position < maximumLength, CONTEXT_OVERFLOW,
              "Position " + std::to_string(position) + " reached runtime limit " + std::to_string(maximumLength));
    invariant(token >= 0 && token < g.vocabularySize, INVALID_CACT,
              "Token " + std::to_string(token) + " is outside the vocabulary");
    const int64_t pos = position;
    history.push_back(token);
    const int D = g.modelDimension, lanes = g.mhcLanes;
    std::vector<float> embedding(M->embedding.inputSize);
    dequantizeRow(M->embedding, token, embedding.data());
    std::vector<float> scaled(D);
    const double embeddingScale = std::sqrt(double(D));
    for (int i = 0; i < D; i++) scaled[i] = float(double(embedding[i]) * embeddingScale);
    if (pool) pool->add(scaled);

    x.assign(int64_t(lanes) * D, 0.0f);
    for (int lane = 0; lane < lanes; lane++) std::copy(scaled.begin(), scaled.end(), x.begin() + int64_t(lane) * D);
    std::vector<uint32_t> indices, valid;
    const bool have = engramLookup(indices, valid);
    std::vector<std::vector<float>> engramKeys, engramValues;
    engramStep(have, indices, valid, engramKeys, engramValues);
    const int attentionWidth = g.numberOfHeads * g.headDimension;

    for (int li = 0; li < g.numberOfLayers; li++) {
      const Layer& L = M->layers[li];
      std::vector<float> nl = rmsUnit(x);
      // matvecBatch over phi slices (runtime.ts:386-402): one prepared activation per input.
      std::vector<float> prepPhi = prepare(M->mhcPhiPre, nl.data(), nl.size());
      std::vector<float> phiPre = matvecPrepared(M->mhcPhiPre, prepPhi, int64_t(li) * lanes, lanes);
      std::vector<float> phiPost = matvecPrepared(M->mhcPhiPost, prepPhi, int64_t(li) * lanes, lanes);
      std::vector<float> phiRes =
          matvecPrepared(M->mhcPhiResidual, prepPhi, int64_t(li) * lanes * lanes, int64_t(lanes) * lanes);

      std::vector<float> hPre(lanes);
      const int ownLane = li % lanes;
      for (int lane = 0; lane < lanes; lane++) {
        const double offset = lane == ownLane ? 4 : -4;
        hPre[lane] = float(sigmoid(double(M->mhcAPre[li]) * double(phiPre[lane]) +
                                   double(M->mhcBPre[int64_t(li) * lanes + lane]) + offset));
      }
      std::vector<float> updateInput(D);
      for (int c = 0; c < D; c++) {
        double sum = 0;
        for (int lane = 0; lane < lanes; lane++) sum += double(hPre[lane]) * double(x[int64_t(lane) * D + c]);
        updateInput[c] = float(sum);
      }
      std::vector<float> blockInput = updateInput;
      int site = -1;
      for (size_t s = 0; s < g.engramLayers.size(); s++)
        if (g.engramLayers[s] == li) {
          site = int(s);
          break;
        }
      if (site >= 0 && size_t(site) < engramKeys.size()) {
        const std::vector<float>& key = engramKeys[site];
        const std::vector<float>& value = engramValues[site];
        std::vector<float> ni = rmsUnit(updateInput), nk = rmsUnit(key);
        double dot = 0;
        for (int i = 0; i < D; i++) dot += double(ni[i]) * double(nk[i]);
        const double alpha = sigmoid(dot / std::sqrt(double(D)));
        for (int i = 0; i < D; i++) blockInput[i] = float(double(updateInput[i]) + alpha * double(value[i]));
      }
      std::vector<float> attentionInput = rmsNorm(blockInput, L.normInput);
      // matvecBatch Q/K/V/gate (runtime.ts:465-470): the shared input is prepared once.
      std::vector<float> prepA = prepare(L.queryProjection, attentionInput.data(), attentionInput.size());
      std::vector<float> query = matvecPrepared(L.queryProjection, prepA, 0, L.queryProjection.outputSize);
      std::vector<float> key = matvecPrepared(L.keyProjection, prepA, 0, L.keyProjection.outputSize);
      std::vector<float> value = matvecPrepared(L.valueProjection, prepA, 0, L.valueProjection.outputSize);
      std::vector<float> gate = matvecPrepared(L.gateProjection, prepA, 0, L.gateProjection.outputSize);
      for (int h = 0; h < g.numberOfHeads; h++)
        rmsNormSlice(query.data() + int64_t(h) * g.headDimension, g.headDimension, L.queryNorm);
      for (int h = 0; h < g.numberOfKVHeads; h++)
        rmsNormSlice(key.data() + int64_t(h) * g.headDimension, g.headDimension, L.keyNorm);
      applyRope(query.data(), g.numberOfHeads, g.headDimension, pos, g.ropeTheta);
      applyRope(key.data(), g.numberOfKVHeads, g.headDimension, pos, g.ropeTheta);
      storeKV(li, pos, key, value);
      std::vector<float> attn = attention(li, pos, query);
      for (int i = 0; i < attentionWidth; i++) attn[i] = float(double(attn[i]) * sigmoid(double(gate[i])));
      std::vector<float> projected = cqMatvec(L.outputProjection, attn.data(), attn.size(), 0,
                                              L.outputProjection.outputSize);
      std::vector<float> delta = attentionDelta(projected, blockInput, updateInput, L);

      std::vector<float> hPost(lanes);
      for (int lane = 0; lane < lanes; lane++) {
        const double offset = lane == ownLane ? 0 : -4;
        hPost[lane] = float(2 * sigmoid(double(M->mhcAPost[li]) * double(phiPost[lane]) +
                                        double(M->mhcBPost[int64_t(li) * lanes + lane]) + offset));
      }
      std::vector<float> routing(int64_t(lanes) * lanes);
      for (int i = 0; i < lanes * lanes; i++)
        routing[i] = float(double(M->mhcAResidual[li]) * double(phiRes[i]) +
                           double(M->mhcBResidual[int64_t(li) * lanes * lanes + i]));
      sinkhorn(routing.data(), lanes);
      std::vector<float> nextX(x.size());
      for (int lane = 0; lane < lanes; lane++) {
        for (int c = 0; c < D; c++) {
          double sum = 0;
          for (int src = 0; src < lanes; src++)
            sum += double(routing[lane * lanes + src]) * double(x[int64_t(src) * D + c]);
          nextX[int64_t(lane) * D + c] = float(sum + double(hPost[lane]) * double(delta[c]));
        }
      }
      x.swap(nextX);
      if (pool) {
        std::vector<float> hidden(D);
        for (int c = 0; c < D; c++) {
          double sum = 0;
          for (int lane = 0; lane < lanes; lane++) sum += double(x[int64_t(lane) * D + c]);
          hidden[c] = float(sum / lanes);
        }
        pool->add(hidden);
      }
    }
    position++;
    if (!wantLogits) return;
    std::vector<float> mean(D);
    for (int c = 0; c < D; c++) {
      double sum = 0;
      for (int lane = 0; lane < lanes; lane++) sum += double(x[int64_t(lane) * D + c]);
      mean[c] = float(sum / lanes);
    }
    std::vector<float> fin = rmsNorm(mean, M->finalNorm);
    *logitsOut = cqMatvec(M->embedding, fin.data(), fin.size(), 0, M->embedding.outputSize);
  }
};

namespace {

// selectToken, runtime.ts:880-899.
void selectToken(const std::vector<float>& logits, const uint32_t* allowed, int32_t n, int32_t* id,
                 double* logProbability) {
  const int64_t V = int64_t(logits.size());
  if (!allowed) {
    const int best = argmaxF(logits.data(), V);
    *id = best;
    *logProbability = logSoftmaxAt(logits.data(), V, best);
    return;
  }
  invariant(n > 0, INVALID_CACT, "Allowed token set is empty");
  uint32_t best = allowed[0];
  invariant(best < uint64_t(V), INVALID_CACT, "Token " + std::to_string(best) + " is outside logits");
  double bestValue = logits[best];
  for (int32_t i = 1; i < n; i++) {
    const uint32_t c = allowed[i];
    invariant(c < uint64_t(V), INVALID_CACT, "Token " + std::to_string(c) + " is outside logits");
    const double v = logits[c];
    if (v > bestValue) {
      bestValue = v;
      best = c;
    }
  }
  *id = int32_t(best);
  *logProbability = logSoftmaxAt(logits.data(), V, best);
}

CqMatrix fromDesc(const ref_cq_desc* d) {
  invariant(d && d->rows >= 0 && d->input_size > 0 && d->group_size > 0 &&
                (d->group_size & (d->group_size - 1)) == 0,
            INVALID_CACT, "Invalid CQ descriptor");
  invariant(d->bits == 2 || d->bits == 3 || d->bits == 4 || d->bits == 5, UNSUPPORTED_CACT,
            "Unsupported CQ record width " + std::to_string(d->bits));
  CqMatrix m;
  m.outputSize = d->rows;
  m.inputSize = d->input_size;
  m.groupSize = d->group_size;
  m.inputSizePadded = (d->input_size + d->group_size - 1) / d->group_size * d->group_size;
  m.bits = d->bits;
  m.rowByteLength = int64_t(m.inputSizePadded) * (d->bits == 5 ? 2 : d->bits) / 8;
  m.packed = d->packed;
  m.norms = d->norms;
  m.cb2 = d->cb2;
  m.cb3 = d->cb3;
  m.cb4 = d->cb4;
  return m;
}

const CqMatrix& modelCq(const ref_model* m, int32_t tensor) {
  invariant(m && tensor >= 0 && size_t(tensor) < m->tensors.size(), INVALID_CACT,
            "Tensor " + std::to_string(tensor) + " is out of range");
  invariant(m->tensors[tensor].kind == Tensor::Cq, INVALID_CACT,
            "Tensor " + std::to_string(tensor) + " must be a Cactus-Quant matrix");
  return m->tensors[tensor].cq;
}

}  // namespace

// ---------------------------------------------------------------- C API

extern "C" {

const char* ref_last_error(void) { return g_last_error.c_str(); }

double ref_float16_to_number(uint32_t h) { return double(f16_to_f32(h)); }
uint32_t ref_number_to_float16(double v) { return f32_to_f16(v); }

int ref_fwht(float* values, int32_t length) {
  return guard([&] { fwht(values, 0, length); });
}

int ref_cq_matvec_desc(const ref_cq_desc* d, const float* x, int32_t row_start, int32_t row_count,
                       float* y) {
  return guard([&] {
    CqMatrix m = fromDesc(d);
    std::vector<float> out = cqMatvec(m, x, m.inputSize, row_start, row_count);
    std::copy(out.begin(), out.end(), y);
  });
}

int ref_cq_prepare_desc(const ref_cq_desc* d, const float* x, float* out) {
  return guard([&] {
    CqMatrix m = fromDesc(d);
    std::vector<float> p = prepare(m, x, m.inputSize);
    std::copy(p.begin(), p.end(), out);
  });
}

int ref_cq_row_desc(const ref_cq_desc* d, int32_t row, float* out) {
  return guard([&] {
    CqMatrix m = fromDesc(d);
    dequantizeRow(m, row, out);
  });
}

int ref_model_open(const uint8_t* bytes, size_t n, ref_model** out) {
  return guard([&] {
    auto m = std::make_unique<ref_model>();
    m->bytes.assign(bytes, bytes + n);
    parse(*m);
    *out = m.release();
  });
}

void ref_model_close(ref_model* m) { delete m; }

int ref_model_geometry(const ref_model* m, int32_t* fields32, float* rope_theta) {
  return guard([&] {
    for (int i = 0; i < 29; i++) fields32[i] = int32_t(m->geometry.fields[i]);
    for (int i = 29; i < 32; i++) fields32[i] = 0;
    if (rope_theta) *rope_theta = m->geometry.ropeTheta;
  });
}

int ref_model_num_tensors(const ref_model* m) { return int(m->tensors.size()); }

int ref_model_record(const ref_model* m, int32_t index, int32_t* info8, uint64_t* offset,
                     uint64_t* length) {
  return guard([&] {
    invariant(index >= 0 && size_t(index) < m->records.size(), INVALID_CACT, "Record out of range");
    const Record& r = m->records[index];
    info8[0] = r.dtype;
    info8[1] = r.rank;
    for (int d = 0; d < 4; d++) info8[2 + d] = int32_t(r.shape[d]);
    info8[6] = int32_t(r.groupSize);
    info8[7] = int32_t(r.bits);
    if (offset) *offset = r.offset;
    if (length) *length = r.byteLength;
  });
}

int ref_model_matvec(const ref_model* m, int32_t tensor, const float* x, int32_t row_start,
                     int32_t row_count, float* y) {
  return guard([&] {
    const CqMatrix& c = modelCq(m, tensor);
    std::vector<float> out = cqMatvec(c, x, c.inputSize, row_start, row_count);
    std::copy(out.begin(), out.end(), y);
  });
}

int ref_model_row(const ref_model* m, int32_t tensor, int32_t row, float* out) {
  return guard([&] { dequantizeRow(modelCq(m, tensor), row, out); });
}

int ref_runtime_new(const ref_model* m, int32_t kv_mode, int32_t collect_confidence, ref_runtime** out) {
  return guard([&] {
    invariant(kv_mode == 0 || kv_mode == 1, INVALID_CACT, "kv_mode must be 0 (int8) or 1 (float32)");
    auto rt = std::make_unique<ref_runtime>();
    rt->M = m;
    rt->kvMode = kv_mode;
    rt->collectConfidence = collect_confidence != 0;
    *out = rt.release();
  });
}

void ref_runtime_free(ref_runtime* rt) { delete rt; }

int ref_runtime_reset(ref_runtime* rt, int32_t maximum_length, int32_t sink_length) {
  return guard([&] { rt->reset(maximum_length, sink_length); });
}

int ref_runtime_position(const ref_runtime* rt) { return int(rt->position); }
int ref_runtime_kv_allocation(const ref_runtime* rt) { return int(rt->kvAllocation); }

int ref_runtime_step(ref_runtime* rt, int32_t token, float* logits) {
  return guard([&] {
    std::vector<float> out;
    rt->step(token, logits != nullptr, &out);
    if (logits) std::copy(out.begin(), out.end(), logits);
  });
}

int ref_runtime_step_selected(ref_runtime* rt, int32_t token, const uint32_t* allowed,
                              int32_t n_allowed, int32_t* id, double* log_probability) {
  return guard([&] {
    std::vector<float> logits;
    rt->step(token, true, &logits);
    selectToken(logits, allowed, n_allowed, id, log_probability);
  });
}

int ref_runtime_read_kv(const ref_runtime* rt, int32_t layer, int8_t* key_codes, int8_t* value_codes,
                        float* key_scales, float* value_scales) {
  return guard([&] {
    const Geometry& g = rt->G();
    invariant(layer >= 0 && layer < g.numberOfLayers, INVALID_CACT, "Layer out of range");
    invariant(rt->kvMode == 0 && rt->maximumLength > 0, INVALID_CACT, "Int8 KV cache is not allocated");
    const int64_t per = int64_t(g.numberOfKVHeads) * rt->kvAllocation;
    const int64_t codes = per * g.headDimension;
    if (key_codes) std::copy_n(rt->keyInt8.data() + layer * codes, codes, key_codes);
    if (value_codes) std::copy_n(rt->valueInt8.data() + layer * codes, codes, value_codes);
    if (key_scales) std::copy_n(rt->keyScale.data() + layer * per, per, key_scales);
    if (value_scales) std::copy_n(rt->valueScale.data() + layer * per, per, value_scales);
  });
}

int ref_runtime_read_kv_f32(const ref_runtime* rt, int32_t layer, float* keys, float* values) {
  return guard([&] {
    const Geometry& g = rt->G();
    invariant(layer >= 0 && layer < g.numberOfLayers, INVALID_CACT, "Layer out of range");
    invariant(rt->kvMode == 1 && rt->maximumLength > 0, INVALID_CACT, "Float32 KV cache is not allocated");
    const int64_t n = int64_t(g.numberOfKVHeads) * rt->kvAllocation * g.headDimension;
    if (keys) std::copy_n(rt->keyFloat.data() + layer * n, n, keys);
    if (values) std::copy_n(rt->valueFloat.data() + layer * n, n, values);
  });
}

int ref_runtime_read_lanes(const ref_runtime* rt, float* lanes) {
  return guard([&] {
    const Geometry& g = rt->G();
    const int64_t n = int64_t(g.mhcLanes) * g.modelDimension;
    if (int64_t(rt->x.size()) == n) std::copy(rt->x.begin(), rt->x.end(), lanes);
    else std::fill_n(lanes, n, 0.0f);
  });
}

int ref_runtime_confidence(const ref_runtime* rt, double* value) {
  return guard([&] {
    *value = std::numeric_limits<double>::quiet_NaN();
    if (!rt->pool) return;
    std::vector<float> out = rt->pool->output();
    if (!out.empty()) *value = sigmoid(double(out[0]));
  });
}

int ref_generate_greedy(const ref_model* m, const int32_t* prompt, int32_t n_prompt, int32_t steps,
                        int32_t sink, int32_t* out_ids, double* out_log_probabilities, float* out_logits) {
  return guard([&] {
    invariant(n_prompt > 0, INVALID_CACT, "Cannot prefill an empty token sequence");
    ref_runtime rt;
    rt.M = m;
    rt.kvMode = 0;
    rt.collectConfidence = false;
    const int64_t V = m->geometry.vocabularySize;
    rt.reset(int64_t(n_prompt) + steps, sink);
    std::vector<float> logits;
    for (int32_t i = 0; i < n_prompt; i++) rt.step(prompt[i], i == n_prompt - 1, &logits);
    for (int32_t s = 0; s < steps; s++) {
      const int token = argmaxF(logits.data(), V);
      out_ids[s] = token;
      if (out_log_probabilities) out_log_probabilities[s] = logSoftmaxAt(logits.data(), V, token);
      if (out_logits) std::copy(logits.begin(), logits.end(), out_logits + int64_t(s) * V);
      if (s + 1 < steps) rt.step(token, true, &logits);
    }
  });
}

int ref_decode_many(const ref_model* m, int32_t n_seqs, const int32_t* prompt_offsets,
                    const int32_t* prompt_ids, const int32_t* gen_steps, int32_t n_threads,
                    int32_t* out_last_ids, int64_t* tokens_processed, double* out_seconds) {
  return guard([&] {
    invariant(n_threads > 0, INVALID_CACT, "n_threads must be positive");
    std::atomic<int32_t> next{0};
    std::atomic<int64_t> processed{0};
    std::vector<std::string> errors(n_threads);
    auto worker = [&](int tid) {
      try {
        ref_runtime rt;
        rt.M = m;
        rt.kvMode = 0;
        rt.collectConfidence = false;
        const int64_t V = m->geometry.vocabularySize;
        std::vector<float> logits;
        for (;;) {
          const int32_t s = next.fetch_add(1);
          if (s >= n_seqs) break;
          const int32_t p0 = prompt_offsets[s], n = prompt_offsets[s + 1] - p0, steps = gen_steps[s];
          const auto t0 = std::chrono::steady_clock::now();
          rt.reset(int64_t(n) + steps, 0);
          int64_t local = 0;
          for (int32_t i = 0; i < n; i++, local++) rt.step(prompt_ids[p0 + i], i == n - 1, &logits);
          int token = 0;
          for (int32_t k = 0; k < steps; k++) {
            token = argmaxF(logits.data(), V);
            if (k + 1 < steps) {
              rt.step(token, true, &logits);
              local++;
            }
          }
          if (out_last_ids) out_last_ids[s] = token;
          if (out_seconds)
            out_seconds[s] = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
          processed += local;
        }
      } catch (const RefError& e) {
        errors[tid] = e.msg;
      }
    };
    std::vector<std::thread> pool;
    for (int t = 0; t < n_threads; t++) pool.emplace_back(worker, t);
    for (auto& th : pool) th.join();
    for (auto& e : errors) invariant(e.empty(), BACKEND_UNAVAILABLE, e);
    *tokens_processed = processed.load();
  });
}

}  // extern "C"

struct ref_sched {
  const ref_model* M;
  std::vector<int32_t> offsets, ids, gen;
  int32_t n_seqs = 0, next = 0, finished = 0, n_threads = 1;
  int64_t processed = 0, generated = 0;
  std::vector<int32_t> last;
  struct Slot {
    std::unique_ptr<ref_runtime> rt;
    bool busy = false;
    int32_t seq = -1, pos = 0, len = 0, target = 0, done = 0, pending = 0;
    std::vector<float> logits;
  };
  std::vector<Slot> slots;

  void admit() {
    for (auto& sl : slots) {
      if (sl.busy || next >= n_seqs) continue;
      const int32_t id = next++;
      sl.seq = id;
      sl.len = offsets[id + 1] - offsets[id];
      sl.target = gen[id];
      sl.pos = 0;
      sl.done = 0;
      sl.busy = true;
      sl.rt->reset(int64_t(sl.len) + sl.target, 0);
    }
  }
  // One token for one busy slot (the device scheduler's item for that slot).
  void run(Slot& sl) {
    const bool select = sl.pos >= sl.len - 1;
    const int32_t token = sl.pos < sl.len ? ids[offsets[sl.seq] + sl.pos] : sl.pending;
    sl.rt->step(token, select, &sl.logits);
    sl.pos++;
    if (select) sl.pending = argmaxF(sl.logits.data(), int64_t(sl.logits.size()));
  }
};

extern "C" {

int ref_sched_new(const ref_model* m, int32_t n_slots, const int32_t* prompt_offsets, const int32_t* prompt_ids,
                  const int32_t* gen_steps, int32_t n_seqs, int32_t n_threads, ref_sched** out) {
  return guard([&] {
    invariant(n_slots > 0 && n_threads > 0 && n_seqs >= 0, INVALID_CACT, "bad scheduler arguments");
    auto s = std::make_unique<ref_sched>();
    s->M = m;
    s->offsets.assign(prompt_offsets, prompt_offsets + n_seqs + 1);
    s->ids.assign(prompt_ids, prompt_ids + (n_seqs ? prompt_offsets[n_seqs] : 0));
    s->gen.assign(gen_steps, gen_steps + n_seqs);
    s->n_seqs = n_seqs;
    s->n_threads = n_threads;
    s->last.assign(std::max(n_seqs, 1), -1);
    s->slots.resize(n_slots);
    for (auto& sl : s->slots) {
      sl.rt = std::make_unique<ref_runtime>();
      sl.rt->M = m;
      sl.rt->kvMode = 0;
      sl.rt->collectConfidence = false;
    }
    s->admit();
    *out = s.release();
  });
}

int ref_sched_step(ref_sched* s, int32_t steps) {
  return guard([&] {
    for (int32_t k = 0; k < steps; k++) {
      std::vector<ref_sched::Slot*> busy;
      for (auto& sl : s->slots)
        if (sl.busy) busy.push_back(&sl);
      if (busy.empty()) break;
      std::vector<std::string> errors(s->n_threads);
      std::atomic<size_t> cursor{0};
      auto worker = [&](int tid) {
        try {
          for (;;) {
            const size_t i = cursor.fetch_add(1);
            if (i >= busy.size()) break;
            s->run(*busy[i]);
          }
        } catch (const RefError& e) {
          errors[tid] = e.msg;
        }
      };
      std::vector<std::thread> pool;
      const int nt = std::min<int>(s->n_threads, int(busy.size()));
      for (int t = 1; t < nt; t++) pool.emplace_back(worker, t);
      worker(0);
      for (auto& th : pool) th.join();
      for (auto& e : errors) invariant(e.empty(), BACKEND_UNAVAILABLE, e);
      for (auto* sl : busy) {
        s->processed++;
        if (sl->pos - 1 >= sl->len - 1) {
          s->generated++;
          sl->done++;
          if (sl->done >= sl->target) {
            s->last[sl->seq] = sl->pending;
            s->finished++;
            sl->busy = false;
          }
        }
      }
      s->admit();
    }
  });
}

int ref_sched_status(const ref_sched* s, int64_t* tokens_processed, int64_t* tokens_generated, int32_t* seqs_finished,
                     int32_t* last_ids) {
  return guard([&] {
    if (tokens_processed) *tokens_processed = s->processed;
    if (tokens_generated) *tokens_generated = s->generated;
    if (seqs_finished) *seqs_finished = s->finished;
    if (last_ids) std::copy(s->last.begin(), s->last.begin() + s->n_seqs, last_ids);
  });
}

void ref_sched_free(ref_sched* s) { delete s; }

int ref_attention_int8(int32_t heads, int32_t kv_heads, int32_t head_dim, int32_t count,
                       const float* q, const int8_t* key_codes, const float* key_scales,
                       const int8_t* value_codes, const float* value_scales, float* out) {
  return guard([&] {
    invariant(heads > 0 && kv_heads > 0 && heads % kv_heads == 0 && head_dim > 0 && count >= 0,
              INVALID_CACT, "Invalid attention shape");
    const int reps = heads / kv_heads;
    std::vector<float> scores(count);
    const double inverseRoot = 1 / std::sqrt(double(head_dim));
    std::fill_n(out, int64_t(heads) * head_dim, 0.0f);
    for (int kh = 0; kh < kv_heads; kh++) {
      for (int rep = 0; rep < reps; rep++) {
        const int qh = kh * reps + rep;
        const float* qq = q + int64_t(qh) * head_dim;
        for (int t = 0; t < count; t++) {
          const int8_t* k = key_codes + (int64_t(kh) * count + t) * head_dim;
          const double ks = key_scales[int64_t(kh) * count + t];
          double dot = 0;
          for (int i = 0; i < head_dim; i++) dot += double(qq[i]) * double(k[i]) * ks;
          scores[t] = float(dot * inverseRoot);
        }
        softmaxInPlace(scores.data(), count);
        float* o = out + int64_t(qh) * head_dim;
        for (int t = 0; t < count; t++) {
          const int8_t* v = value_codes + (int64_t(kh) * count + t) * head_dim;
          const double vs = value_scales[int64_t(kh) * count + t];
          const double w = scores[t];
          for (int i = 0; i < head_dim; i++) o[i] = float(double(o[i]) + w * double(v[i]) * vs);
        }
      }
    }
  });
}

int ref_quantize_kv_head(const float* x, int32_t head_dim, int8_t* codes, float* scale) {
  return guard([&] {
    double maximum = 1e-12;
    for (int i = 0; i < head_dim; i++) maximum = std::max(maximum, std::fabs(double(x[i])));
    const double s = maximum / 127;
    *scale = float(s);
    for (int i = 0; i < head_dim; i++) codes[i] = int8_t(roundTiesToEven(double(x[i]) / s));
  });
}

}  // extern "C"
