// ops.cu -- stateless device-pointer operators of the C-ABI (isolated matvec and attention).
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/needle_cuda.h"
#include "engine.cuh"

using namespace needle;

namespace {

// Library-owned scratch for prepared activations, one growable buffer per device.
struct DeviceScratch {
  float* ptr = nullptr;
  size_t floats = 0;
};
std::mutex g_scratch_mu;
std::vector<DeviceScratch> g_scratch;

cudaError_t scratch_for(int device, size_t floats, float** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (int(g_scratch.size()) <= device) g_scratch.resize(device + 1);
  DeviceScratch& s = g_scratch[device];
  if (s.floats < floats) {
    if (s.ptr) {
      cudaError_t e = cudaDeviceSynchronize();
      if (e != cudaSuccess) return e;
      cudaFree(s.ptr);
      s.ptr = nullptr;
      s.floats = 0;
    }
    cudaError_t e = cudaMalloc(&s.ptr, floats * sizeof(float));
    if (e != cudaSuccess) return e;
    s.floats = floats;
  }
  *out = s.ptr;
  return cudaSuccess;
}

// Library-owned scratch for the split partials of the fast attention, one buffer per device.
std::vector<DeviceScratch> g_attn_scratch;

cudaError_t attn_scratch_for(int device, size_t bytes, void** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (int(g_attn_scratch.size()) <= device) g_attn_scratch.resize(device + 1);
  DeviceScratch& s = g_attn_scratch[device];
  const size_t floats = (bytes + 3) / 4;
  if (s.floats < floats) {
    if (s.ptr) {
      cudaError_t e = cudaDeviceSynchronize();
      if (e != cudaSuccess) return e;
      cudaFree(s.ptr);
      s.ptr = nullptr;
      s.floats = 0;
    }
    cudaError_t e = cudaMalloc(&s.ptr, floats * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(s.ptr, 0, 16);  // status and work counters start at zero
    if (e != cudaSuccess) return e;
    s.floats = floats;
  }
  *out = s.ptr;
  return cudaSuccess;
}

int op_fail(int code, const std::string& msg) {
  set_last_error(msg);
  return code;
}

// Wait-status words of every device: one pinned, mapped host allocation (kWaitKinds words per
// device), made on the first call that needs it.
constexpr int kStatusDevices = 64;
std::mutex g_status_mu;
uint32_t* g_status_host = nullptr;
bool g_status_failed = false;

const char* kWaitKindNames[kWaitKinds] = {"fast attention", "table matvec", "tensor-core matvec", "wait self-test"};

// Reports (and clears) the bounded waits of earlier calls on `device` that ran out.
int check_wait_status(int device) {
  uint32_t* w = wait_status_words(device);
  if (!w) return NEEDLE_OK;
  std::string names;
  for (int k = 0; k < kWaitKinds; k++) {
    volatile uint32_t* v = w + k;
    if (*v) {
      names += (names.empty() ? "" : ", ") + std::string(kWaitKindNames[k]);
      *v = 0;
    }
  }
  if (names.empty()) return NEEDLE_OK;
  return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "a bounded device wait ran out on device " + std::to_string(device) +
                                                 " (" + names + "); that call's outputs are NaN");
}

__device__ int g_never_set;  // nothing writes it: the self-test's wait always runs out

__global__ void k_wait_selftest(uint64_t limit_ns, uint32_t* words) {
  if (threadIdx.x != 0) return;
  uint64_t start, now;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(start));
  for (;;) {
    if (*reinterpret_cast<volatile int*>(&g_never_set) != 0) return;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    if (now - start > limit_ns) {
      report_wait_timeout(words, kWaitSelftest);
      return;
    }
    __nanosleep(1000);
  }
}

}  // namespace

uint32_t* needle::wait_status_words(int device) {
  if (device < 0 || device >= kStatusDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (!g_status_host && !g_status_failed) {
    void* p = nullptr;
    if (cudaHostAlloc(&p, sizeof(uint32_t) * kWaitKinds * kStatusDevices, cudaHostAllocMapped | cudaHostAllocPortable) ==
        cudaSuccess) {
      std::memset(p, 0, sizeof(uint32_t) * kWaitKinds * kStatusDevices);
      g_status_host = static_cast<uint32_t*>(p);
    } else {
      cudaGetLastError();
      g_status_failed = true;
    }
  }
  return g_status_host ? g_status_host + kWaitKinds * device : nullptr;
}

extern "C" int needle_cuda_wait_status(int32_t device, uint32_t* kinds, int32_t clear) {
  if (!kinds) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "null argument");
  uint32_t* w = wait_status_words(device);
  if (!w) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "no wait-status words for device " + std::to_string(device));
  uint32_t mask = 0;
  for (int k = 0; k < kWaitKinds; k++) {
    volatile uint32_t* v = w + k;
    if (*v) mask |= 1u << k;
    if (clear) *v = 0;
  }
  *kinds = mask;
  return NEEDLE_OK;
}

extern "C" int needle_cuda_wait_selftest(uint64_t limit_ns, void* stream) {
  if (limit_ns > 1000000000ull) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "self-test wait limit above 1 s");
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, cudaGetErrorString(e));
  uint32_t* w = wait_status_words(device);
  if (!w) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "no wait-status words");
  k_wait_selftest<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, w);
  e = cudaGetLastError();
  if (e != cudaSuccess) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, cudaGetErrorString(e));
  return NEEDLE_OK;
}

extern "C" int needle_cuda_cq_matvec_dev(const needle_cq_matrix* m, const float* codebook, const float* x,
                                         int32_t batch, float* y, void* stream) {
  if (!m || !codebook || (batch > 0 && (!x || !y)))
    return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "null argument");
  if (m->group_size != kGroup) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "CQ group size 128 only");
  if (!(m->bits == 2 || m->bits == 3 || m->bits == 4 || m->bits == 5))
    return op_fail(NEEDLE_UNSUPPORTED_CACT, "unsupported CQ record width");
  if (m->rows < 0 || m->input_size <= 0 || batch < 0) return op_fail(NEEDLE_INVALID_CACT, "bad matrix shape");
  if ((reinterpret_cast<uintptr_t>(m->packed) & 15) != 0)
    return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "packed rows must be 16-byte aligned");
  if (batch == 0 || m->rows == 0) return NEEDLE_OK;
  const int in_pad = (m->input_size + kGroup - 1) / kGroup * kGroup;
  const int pb = m->bits == 5 ? 2 : m->bits;
  const int row_bytes = in_pad * pb / 8;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Codebook cb{};
  for (int i = 0; i < 28; i++) cb.v[i] = codebook[i];
  int device = 0;
  cudaGetDevice(&device);
  // Scratch: prepared activations, then (small batches of long rows) the per-group dots.
  CqJob probe{};
  probe.rows = m->rows;
  probe.in_pad = in_pad;
  const bool split = cq_gemv_prefers_split(probe, batch);
  const size_t x_floats = (size_t(batch) * in_pad + 1) & ~size_t(1);  // keep the dots 8-byte aligned
  const size_t dot_floats = split ? cq_gemv_split_scratch_bytes(probe, batch) / 4 : 0;
  float* xp = nullptr;
  cudaError_t e = scratch_for(device, x_floats + dot_floats, &xp);
  if (e != cudaSuccess) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, cudaGetErrorString(e));
  e = launch_cq_prepare(x, m->input_size, m->input_size, in_pad, xp, in_pad, batch, nullptr, s);
  if (e != cudaSuccess) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, cudaGetErrorString(e));
  CqJobs J{};
  CqJob& j = J.job[0];
  j.packed = m->packed;
  j.norms = m->norms;
  j.row_start = 0;
  j.rows = m->rows;
  j.in_pad = in_pad;
  j.bits = m->bits;
  j.row_bytes = row_bytes;
  j.tile_begin = 0;
  j.x = xp;
  j.x_stride = in_pad;
  j.y = y;
  j.y_stride = m->rows;
  J.count = 1;
  J.total_tiles = (m->rows + kGemvTileRows - 1) / kGemvTileRows;
  e = split ? launch_cq_gemv_split(j, cb, batch, reinterpret_cast<double*>(xp + x_floats), s)
            : launch_cq_gemv(J, cb, batch, nullptr, s);
  if (e != cudaSuccess) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, cudaGetErrorString(e));
  return NEEDLE_OK;
}

// ---- no-allocation variant of needle_cuda_cq_matvec_dev
//
// For callers that cannot call cudaMalloc (all device memory handed to their own pool, or a
// serving loop that may not pay cudaMalloc's device-wide synchronisation): the rotated
// activations live in this fixed array instead of a growable buffer.  Host code cannot use the
// array's name as a device address, so the address is looked up once per device with
// cudaGetSymbolAddress while that device is current.
static __device__ __align__(256) float g_noalloc_prepared[NEEDLE_NOALLOC_MAX_FLOATS];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_addr[kNoAllocMaxDevices] = {};

cudaError_t noalloc_scratch(int device, float** out) {
  if (device < 0 || device >= kNoAllocMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_prepared);
    if (e != cudaSuccess) return e;
    g_noalloc_addr[device] = static_cast<float*>(p);
  }
  *out = g_noalloc_addr[device];
  return cudaSuccess;
}
}  // namespace

extern "C" int needle_cuda_cq_matvec_dev_noalloc(const needle_cq_matrix* m, const float* codebook, const float* x,
                                                 int32_t batch, float* y, void* stream) {
  if (!m || !codebook || (batch > 0 && (!x || !y)))
    return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "null argument");
  if (m->group_size != kGroup) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "CQ group size 128 only");
  if (!(m->bits == 2 || m->bits == 3 || m->bits == 4 || m->bits == 5))
    return op_fail(NEEDLE_UNSUPPORTED_CACT, "unsupported CQ record width");
  if (m->rows < 0 || m->input_size <= 0 || batch < 0) return op_fail(NEEDLE_INVALID_CACT, "bad matrix shape");
  if ((reinterpret_cast<uintptr_t>(m->packed) & 15) != 0)
    return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "packed rows must be 16-byte aligned");
  const int64_t in_pad = (int64_t(m->input_size) + kGroup - 1) / kGroup * kGroup;
  if (int64_t(batch) * in_pad > NEEDLE_NOALLOC_MAX_FLOATS)
    return op_fail(NEEDLE_BACKEND_UNAVAILABLE,
                   "batch * padded input (" + std::to_string(int64_t(batch) * in_pad) +
                       " floats) exceeds the no-allocation scratch of " + std::to_string(NEEDLE_NOALLOC_MAX_FLOATS) +
                       " floats");
  if (batch == 0 || m->rows == 0) return NEEDLE_OK;
  const int pb = m->bits == 5 ? 2 : m->bits;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Codebook cb{};
  for (int i = 0; i < 28; i++) cb.v[i] = codebook[i];
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  float* xp = nullptr;
  if (e == cudaSuccess) e = noalloc_scratch(device, &xp);
  if (e != cudaSuccess) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, cudaGetErrorString(e));
  e = launch_cq_prepare(x, m->input_size, m->input_size, int32_t(in_pad), xp, int32_t(in_pad), batch, nullptr, s);
  if (e != cudaSuccess) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, cudaGetErrorString(e));
  CqJobs J{};
  CqJob& j = J.job[0];
  j.packed = m->packed;
  j.norms = m->norms;
  j.row_start = 0;
  j.rows = m->rows;
  j.in_pad = int32_t(in_pad);
  j.bits = m->bits;
  j.row_bytes = int32_t(in_pad * pb / 8);
  j.tile_begin = 0;
  j.x = xp;
  j.x_stride = int32_t(in_pad);
  j.y = y;
  j.y_stride = m->rows;
  J.count = 1;
  J.total_tiles = (m->rows + kGemvTileRows - 1) / kGemvTileRows;
  e = launch_cq_gemv(J, cb, batch, nullptr, s);
  if (e != cudaSuccess) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, cudaGetErrorString(e));
  return NEEDLE_OK;
}

extern "C" int needle_cuda_attention_dev(const float* q, const int8_t* key_codes, const float* key_scales,
                                         const int8_t* value_codes, const float* value_scales, const int32_t* counts,
                                         int32_t batch, int32_t capacity, float* out, void* stream) {
  if (batch < 0 || capacity <= 0) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "bad batch / capacity");
  if (batch == 0) return NEEDLE_OK;
  if (!q || !key_codes || !key_scales || !value_codes || !value_scales || !counts || !out)
    return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "null argument");
  if (attention_smem_bytes(capacity, false) > 200 * 1024)
    return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "capacity too large for the exact attention kernel");
  cudaError_t e = launch_attention_dev(q, key_codes, key_scales, value_codes, value_scales, counts, batch, capacity,
                                       out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, cudaGetErrorString(e));
  return NEEDLE_OK;
}

extern "C" int needle_cuda_attention_dev_fast(const float* q, const int8_t* key_codes, const float* key_scales,
                                              const int8_t* value_codes, const float* value_scales,
                                              const int32_t* counts, int32_t batch, int32_t capacity, float* out,
                                              void* stream) {
  if (batch < 0 || capacity <= 0) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "bad batch / capacity");
  if (batch == 0) return NEEDLE_OK;
  if (!q || !key_codes || !key_scales || !value_codes || !value_scales || !counts || !out)
    return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "null argument");
  if ((reinterpret_cast<uintptr_t>(key_codes) & 15) != 0 || (reinterpret_cast<uintptr_t>(value_codes) & 15) != 0)
    return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "key/value codes must be 16-byte aligned");
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e == cudaSuccess && check_wait_status(device) != NEEDLE_OK) return NEEDLE_BACKEND_UNAVAILABLE;
  void* scratch = nullptr;
  if (e == cudaSuccess) e = attn_scratch_for(device, attention_fast_scratch_bytes(batch, capacity), &scratch);
  if (e == cudaSuccess)
    e = launch_attention_fast(q, key_codes, key_scales, value_codes, value_scales, counts, batch, capacity, out,
                              scratch, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, cudaGetErrorString(e));
  return NEEDLE_OK;
}

extern "C" int needle_cuda_cq_matvec_dev_fast(const needle_cq_matrix* m, const float* codebook, const float* x,
                                              int32_t batch, float* y, void* stream) {
  if (!m || !codebook || (batch > 0 && (!x || !y)))
    return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "null argument");
  if (m->group_size != kGroup) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "CQ group size 128 only");
  if (!cq_gemv_fast_supported(m->bits) && !cq_gemm_tc_supported(m->bits))
    return op_fail(NEEDLE_UNSUPPORTED_CACT, "unsupported CQ record width");
  if (m->rows < 0 || m->input_size <= 0 || batch < 0) return op_fail(NEEDLE_INVALID_CACT, "bad matrix shape");
  if ((reinterpret_cast<uintptr_t>(m->packed) & 15) != 0)
    return op_fail(NEEDLE_BACKEND_UNAVAILABLE, "packed rows must be 16-byte aligned");
  if (batch == 0 || m->rows == 0) return NEEDLE_OK;
  const int in_pad = (m->input_size + kGroup - 1) / kGroup * kGroup;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Codebook cb{};
  for (int i = 0; i < 28; i++) cb.v[i] = codebook[i];
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e == cudaSuccess && check_wait_status(device) != NEEDLE_OK) return NEEDLE_BACKEND_UNAVAILABLE;
  if (cq_gemm_tc_supported(m->bits) &&
      (cq_gemm_tc_preferred(m->rows, m->input_size, batch) || !cq_gemv_fast_supported(m->bits))) {
    // a real dense contraction: tensor-core GEMM
    int sms = 0;
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    float* scratch = nullptr;
    const size_t bytes = cq_gemm_tc_scratch_bytes(m->rows, m->input_size, batch, sms);
    if (e == cudaSuccess) e = scratch_for(device, (bytes + 3) / 4, &scratch);
    if (e == cudaSuccess)
      e = launch_cq_gemm_tc(m->packed, m->norms, m->rows, m->input_size, m->bits, x, m->input_size, 0, batch, y,
                            m->rows, cb, scratch, sms, s);
    if (e != cudaSuccess) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, cudaGetErrorString(e));
    return NEEDLE_OK;
  }
  float* partials = nullptr;
  const size_t floats = cq_gemv_fast_partial_floats(m->rows, in_pad);
  if (e == cudaSuccess) e = scratch_for(device, floats, &partials);
  if (e == cudaSuccess)
    e = launch_cq_gemv_fast(m->packed, m->norms, m->rows, m->input_size, m->bits, x, batch, y, cb, partials, s);
  if (e != cudaSuccess) return op_fail(NEEDLE_BACKEND_UNAVAILABLE, cudaGetErrorString(e));
  return NEEDLE_OK;
}
