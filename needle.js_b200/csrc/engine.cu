// engine.cu -- host side of libneedle_cuda.so: `.cact` parsing, weight upload, per-slot state,
// batched step orchestration, device scheduler, and the C-ABI of include/needle_cuda.h.
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/needle_cuda.h"
#include "engine.cuh"

using namespace needle;

namespace {

thread_local std::string g_error;

struct Failure {
  int code;
  std::string msg;
};

[[noreturn]] void fail(int code, const std::string& msg) { throw Failure{code, msg}; }
inline void require(bool ok, int code, const std::string& msg) {
  if (!ok) fail(code, msg);
}
inline void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    fail(NEEDLE_BACKEND_UNAVAILABLE, std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
}

template <class F>
int guarded(F&& f) {
  try {
    f();
    return NEEDLE_OK;
  } catch (const Failure& e) {
    g_error = e.msg;
    return e.code;
  } catch (const std::bad_alloc&) {
    g_error = "host allocation failed";
    return NEEDLE_BACKEND_UNAVAILABLE;
  } catch (const std::exception& e) {
    g_error = e.what();
    return NEEDLE_BACKEND_UNAVAILABLE;
  }
}

// ------------------------------------------------------------------ archive view (host)

inline uint32_t u32le(const uint8_t* p) {
  return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
}
inline uint64_t u64le(const uint8_t* p) { return uint64_t(u32le(p)) | (uint64_t(u32le(p + 4)) << 32); }
inline float f32le(const uint8_t* p) {
  uint32_t b = u32le(p);
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

float half_to_float(uint16_t h) {  // exact binary16 -> binary32 widening
  const uint32_t sign = uint32_t(h & 0x8000u) << 16;
  int32_t exponent = (h >> 10) & 0x1f;
  uint32_t mantissa = h & 0x3ffu, bits;
  if (exponent == 0) {
    if (mantissa == 0) {
      bits = sign;
    } else {
      exponent = 127 - 15 + 1;
      while ((mantissa & 0x400u) == 0) {
        mantissa <<= 1;
        exponent--;
      }
      bits = sign | (uint32_t(exponent) << 23) | ((mantissa & 0x3ffu) << 13);
    }
  } else if (exponent == 0x1f) {
    bits = sign | 0x7f800000u | (mantissa << 13);
  } else {
    bits = sign | (uint32_t(exponent - 15 + 127) << 23) | (mantissa << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

struct Record {
  int dtype = 0, rank = 0;
  int64_t shape[4] = {0, 0, 0, 0};
  uint64_t offset = 0, length = 0;
  uint32_t group = 0, bits = 0;
  // CQ derived
  int64_t rows = 0, input = 0, in_pad = 0, row_bytes = 0, packed_bytes = 0;
};

struct Archive {
  const uint8_t* b = nullptr;
  size_t n = 0;
  uint32_t hdr[30];
  float rope_theta = 0;
  std::vector<float> codebook;
  std::vector<Record> rec;

  std::vector<float> dense(int i) const {
    const Record& r = rec[i];
    int64_t count = 1;
    for (int d = 0; d < r.rank; d++) count *= r.shape[d];
    std::vector<float> out(count);
    for (int64_t k = 0; k < count; k++) {
      const uint8_t* p = b + r.offset + (r.dtype == 1 ? k * 2 : k * 4);
      out[k] = r.dtype == 1 ? half_to_float(uint16_t(p[0] | (p[1] << 8))) : f32le(p);
    }
    return out;
  }
};

// Parses and validates the archive like parseCact (packages/needle.js/src/model/cact.ts:189-401).
void parse_archive(const uint8_t* b, size_t n, Archive& A) {
  auto in_range = [&](uint64_t off, uint64_t len) { return off <= n && len <= n - off; };
  require(in_range(0, 120), NEEDLE_INVALID_CACT,
          "CACT header points outside the " + std::to_string(n) + "-byte archive");
  A.b = b;
  A.n = n;
  for (int i = 0; i < 29; i++) A.hdr[i] = u32le(b + i * 4);
  A.rope_theta = f32le(b + 29 * 4);
  require(A.hdr[0] == 0x05e12a83u, NEEDLE_INVALID_CACT, "Invalid .cact tag");
  const uint32_t tensors = A.hdr[1], cb_len = A.hdr[2];
  require(tensors > 0, NEEDLE_INVALID_CACT, "The .cact archive has no tensors");
  require(cb_len >= 28, NEEDLE_UNSUPPORTED_CACT,
          "Needle 2 requires the CQ2/CQ3/CQ4 codebook (28 entries); archive has " + std::to_string(cb_len));
  require(A.hdr[19] <= 4 && A.hdr[24] <= 4, NEEDLE_UNSUPPORTED_CACT,
          "The current .cact format supports at most four engram orders and sites");
  require(A.hdr[6] > 0 && A.hdr[5] > 0, NEEDLE_INVALID_CACT,
          "Model geometry contains a zero-sized vocabulary or hidden dimension");
  require(A.hdr[7] > 0 && A.hdr[8] > 0 && A.hdr[7] % A.hdr[8] == 0, NEEDLE_UNSUPPORTED_CACT,
          "Attention heads must be a positive multiple of KV heads");
  require((A.hdr[12] & (A.hdr[12] - 1)) == 0, NEEDLE_UNSUPPORTED_CACT, "Hadamard dimension must be a power of two");
  require(in_range(120, uint64_t(cb_len) * 4), NEEDLE_INVALID_CACT, "CQ codebook points outside the archive");
  A.codebook.resize(cb_len);
  for (uint32_t i = 0; i < cb_len; i++) A.codebook[i] = f32le(b + 120 + i * 4);
  const uint64_t dir = 120 + uint64_t(cb_len) * 4;
  require(in_range(dir, uint64_t(tensors) * 44), NEEDLE_INVALID_CACT, "Tensor directory points outside the archive");
  A.rec.resize(tensors);
  for (uint32_t i = 0; i < tensors; i++) {
    const uint8_t* r = b + dir + uint64_t(i) * 44;
    Record& R = A.rec[i];
    R.dtype = r[0];
    R.rank = r[1];
    require(R.rank <= 4, NEEDLE_UNSUPPORTED_CACT, "Tensor " + std::to_string(i) + " has more than four dimensions");
    for (int d = 0; d < R.rank; d++) R.shape[d] = u32le(r + 4 + d * 4);
    R.offset = u64le(r + 20);
    R.length = u64le(r + 28);
    R.group = u32le(r + 36);
    R.bits = u32le(r + 40);
    require(in_range(R.offset, R.length), NEEDLE_INVALID_CACT,
            "Tensor " + std::to_string(i) + " points outside the archive");
    int64_t count = 1;
    for (int d = 0; d < R.rank; d++) count *= R.shape[d];
    if (R.dtype == 1) {
      require(R.length == uint64_t(count) * 2, NEEDLE_INVALID_CACT,
              "FP16 tensor " + std::to_string(i) + " has an inconsistent byte length");
    } else if (R.dtype == 2) {
      require(R.length == uint64_t(count) * 4, NEEDLE_INVALID_CACT,
              "FP32 tensor " + std::to_string(i) + " has an inconsistent byte length");
    } else if (R.dtype == 3) {
      require(R.rank == 2, NEEDLE_INVALID_CACT, "CQ tensor " + std::to_string(i) + " is not a matrix");
      require(R.group > 0 && (R.group & (R.group - 1)) == 0, NEEDLE_UNSUPPORTED_CACT,
              "CQ tensor " + std::to_string(i) + " has non-power-of-two group");
      require(R.bits == 2 || R.bits == 3 || R.bits == 4 || R.bits == 5, NEEDLE_UNSUPPORTED_CACT,
              "CQ tensor " + std::to_string(i) + " uses unsupported record width " + std::to_string(R.bits));
      R.rows = R.shape[0];
      R.input = R.shape[1];
      R.in_pad = (R.input + R.group - 1) / R.group * R.group;
      const int64_t pb = R.bits == 5 ? 2 : R.bits;
      require((R.in_pad * pb) % 8 == 0, NEEDLE_INVALID_CACT, "CQ tensor has a fractional packed row size");
      R.row_bytes = R.in_pad * pb / 8;
      R.packed_bytes = R.rows * R.row_bytes;
      const uint64_t norms = uint64_t(R.rows) * (R.in_pad / R.group);
      require(R.length == uint64_t(R.packed_bytes) + norms * 2, NEEDLE_INVALID_CACT,
              "CQ tensor " + std::to_string(i) + " has an inconsistent packed/norm length");
    } else if (R.dtype != 4) {
      fail(NEEDLE_UNSUPPORTED_CACT, "Tensor " + std::to_string(i) + " uses unknown dtype " + std::to_string(R.dtype));
    }
  }
}

// Canonical tensor order (cact.ts:403-536): embedding, 14 per layer, 9 mHC, 4 per engram site,
// final norm, optional probe heads, RAW tokenizer.
struct Roles {
  int embedding = -1;
  struct L {
    int norm_input, q, k, v, qn, kn, gate, o, post, attn_gate, pre_had, d1, d2, d3;
  };
  std::vector<L> layers;
  int a_pre, a_post, a_res, b_pre, b_post, b_res, phi_pre, phi_post, phi_res;
  struct E {
    int tables, k, v, taps;
  };
  std::vector<E> sites;
  int final_norm;
  // confidence probe head (manifest code 2): probes, projection, bias; -1 when absent
  int conf_probes = -1, conf_proj = -1, conf_bias = -1;
  int64_t conf_count = 0, conf_out = 0;
};

Roles assign_roles(const Archive& A) {
  Roles R;
  size_t cur = 0;
  auto take = [&](int want, const std::string& name) {
    require(cur < A.rec.size(), NEEDLE_INVALID_CACT, "Archive ended before " + name);
    const int i = int(cur++);
    if (want == 3) require(A.rec[i].dtype == 3, NEEDLE_INVALID_CACT, name + " must be a Cactus-Quant matrix");
    if (want == 1) require(A.rec[i].dtype == 1 || A.rec[i].dtype == 2, NEEDLE_INVALID_CACT, name + " must be an FP16/FP32 tensor");
    return i;
  };
  R.embedding = take(3, "embedding");
  const int L = int(A.hdr[9]);
  for (int l = 0; l < L; l++) {
    const std::string p = "layer " + std::to_string(l);
    Roles::L x;
    x.norm_input = take(1, p + " input norm");
    x.q = take(3, p + " query projection");
    x.k = take(3, p + " key projection");
    x.v = take(3, p + " value projection");
    x.qn = take(1, p + " query norm");
    x.kn = take(1, p + " key norm");
    x.gate = take(3, p + " gate projection");
    x.o = take(3, p + " output projection");
    x.post = take(1, p + " post-attention norm");
    x.attn_gate = take(1, p + " attention gate");
    x.pre_had = take(1, p + " pre-Hadamard norm");
    x.d1 = take(1, p + " Hadamard d1");
    x.d2 = take(1, p + " Hadamard d2");
    x.d3 = take(1, p + " Hadamard d3");
    R.layers.push_back(x);
  }
  R.a_pre = take(1, "mHC a_pre");
  R.a_post = take(1, "mHC a_post");
  R.a_res = take(1, "mHC a_res");
  R.b_pre = take(1, "mHC b_pre");
  R.b_post = take(1, "mHC b_post");
  R.b_res = take(1, "mHC b_res");
  R.phi_pre = take(3, "mHC phi_pre");
  R.phi_post = take(3, "mHC phi_post");
  R.phi_res = take(3, "mHC phi_res");
  for (uint32_t s = 0; s < A.hdr[24]; s++) {
    const std::string p = "engram " + std::to_string(s);
    Roles::E e;
    e.tables = take(3, p + " tables");
    e.k = take(3, p + " key projection");
    e.v = take(3, p + " value projection");
    e.taps = take(1, p + " taps");
    R.sites.push_back(e);
  }
  R.final_norm = take(1, "final norm");
  // Optional probe-head manifest (cact.ts:537-556): a dense list of codes, 1 contrastive, 2
  // confidence, each followed by its probes, projection and bias.
  const int64_t D = A.hdr[6];
  if (cur < A.rec.size() && (A.rec[cur].dtype == 1 || A.rec[cur].dtype == 2)) {
    const std::vector<float> manifest = A.dense(int(cur++));
    for (float raw : manifest) {
      const double code = std::floor(double(raw) + 0.5);  // Math.round
      require(code == 1 || code == 2, NEEDLE_UNSUPPORTED_CACT,
              "Unknown probe-head manifest code " + std::to_string(int64_t(code)));
      const std::string name = code == 1 ? "contrastive" : "confidence";
      const int probes = take(1, name + " probes"), proj = take(1, name + " projection"),
                bias = take(1, name + " bias");
      auto count_of = [&](int i) {
        int64_t c = 1;
        for (int d = 0; d < A.rec[i].rank; d++) c *= A.rec[i].shape[d];
        return c;
      };
      const int64_t n_probes = A.rec[probes].rank > 0 ? A.rec[probes].shape[0] : 0;
      const int64_t n_out = A.rec[proj].rank > 0 ? A.rec[proj].shape[0] : count_of(bias);
      require(n_probes > 0 && count_of(probes) == n_probes * D, NEEDLE_INVALID_CACT,
              name + " probe shape is inconsistent");
      require(count_of(proj) == n_out * n_probes * D, NEEDLE_INVALID_CACT, name + " projection shape is inconsistent");
      if (code == 2) {
        R.conf_probes = probes;
        R.conf_proj = proj;
        R.conf_bias = bias;
        R.conf_count = n_probes;
        R.conf_out = n_out;
      }
    }
  }
  bool tokenizer = false;
  while (cur < A.rec.size()) {
    const int i = int(cur++);
    if (A.rec[i].dtype == 4) {
      require(!tokenizer, NEEDLE_INVALID_CACT, "Archive contains more than one RAW tokenizer tensor");
      tokenizer = true;
    } else {
      fail(NEEDLE_UNSUPPORTED_CACT, "Unexpected trailing tensor " + std::to_string(i));
    }
  }
  require(tokenizer, NEEDLE_INVALID_CACT, "Archive does not contain its RAW SentencePiece tokenizer");
  return R;
}

struct SlotHost {
  bool ready = false, collect = false;
  int32_t max_len = 0, sink = 0, kv_alloc = 0, position = 0;
};

// Prompt tokens of one slot processed together by needle_cuda_prefill (StepView::chunk); the step
// buffers hold at least this many items.
constexpr int kPrefillChunk = 64;

struct ProfEntry {
  int cls;
  cudaEvent_t a, b;
};

const char* kProfNames[] = {"embed", "gemv_engram", "layer", "gemv_qkvg", "attention", "gemv_o",
                            "gemv_vocab", "finish", "sched", "copy", "route"};
constexpr int kProfClasses = 11;
enum { P_EMBED, P_GEMV_ENGRAM, P_LAYER, P_GEMV_QKVG, P_ATTN, P_GEMV_O, P_GEMV_VOCAB, P_FINISH, P_SCHED, P_COPY,
       P_ROUTE };

}  // namespace

void needle::set_last_error(const char* msg) { g_error = msg ? msg : ""; }

struct needle_ctx {
  needle_opts opts{};
  int device = 0;
  cudaStream_t stream = nullptr;
  cudaStream_t side = nullptr;             // routing (Sinkhorn) overlapped with attention
  cudaEvent_t fork_ev[2] = {nullptr, nullptr}, join_ev[2] = {nullptr, nullptr};
  // Micro-batches 1.. of the device-scheduled step (each with its own main and routing streams;
  // micro-batch 0 runs on stream / side).
  cudaStream_t mb_main[kMaxMicro] = {}, mb_side[kMaxMicro] = {};
  cudaEvent_t mb_fork[kMaxMicro][2] = {}, mb_join[kMaxMicro][2] = {}, mb_done[kMaxMicro] = {};
  cudaEvent_t split_ev = nullptr;
  int micro = 4;  // micro-batches of a device-scheduled step (needle_opts.micro_batches)
  int sched_chunk = 0;  // prompt positions per slot and scheduled step (needle_opts.sched_chunk; 0: one)
  int sched_items = 0;  // items a scheduled step with chunks may hold (needle_opts.sched_items)
  int step_capacity = 0;  // items one step's buffers hold
  // The device-scheduled step captured as a CUDA graph after one eager step.
  cudaGraphExec_t sched_graph = nullptr;
  int64_t graph_launches = 0;
  int sched_eager_steps = 0;
  bool sched_inflight = false;  // scheduled steps enqueued since the stream was last drained
  // host steps as micro-batches (needle_cuda_step): the captured step and its shape
  cudaGraphExec_t host_graph = nullptr;        // whole step
  cudaGraphExec_t host_graph_begin = nullptr;  // needle_cuda_step_begin's part (no selection)
  cudaGraphExec_t single_graph = nullptr;      // a one-item step (batch-1 decode)
  int64_t host_graph_launches = 0, host_begin_launches = 0, single_launches = 0;
  int single_eager_steps = 0;
  int host_eager_steps = 0, host_m = 0, host_cap = 0;
  std::vector<uint8_t> bytes;  // archive copy (host)
  Archive A;
  Roles roles;
  std::vector<void*> allocs;
  std::vector<CqMat> cq;  // per archive tensor (CQ tensors only)
  ModelView mv{};
  SlotView sv{};
  StepView stv{};
  std::vector<CqMat> lq, lk, lv, lg, lo;
  std::vector<CqMat> ek, ev;
  // Fast numerics (NEEDLE_NUMERICS_FAST): Q|K|V|gate of each layer and K|V of each engram site as
  // one matrix each (one GEMM per shared input), and per micro-batch lane the GEMM's scratch.
  bool fast = false;
  bool fast_attention = false;  // NEEDLE_NUMERICS_FAST_ATTENTION: int8-MMA attention (else binary32)
  int sms = 0;
  std::vector<CqMat> lqkvg, ekv;
  // Exact numerics: Q|K|V|gate of each layer stacked group-major for the byte-table GEMV (empty when
  // the four are not all 2-bit rows of one input length).
  std::vector<CqMat> lqkvg_gm;
  void* gemm_scratch[kMaxMicro] = {};
  size_t gemm_scratch_bytes = 0;
  void* attn_scratch[kMaxMicro] = {};  // the fast attention's partials and counters, per lane
  int32_t* d_counts = nullptr;  // [0] n_items, [1] n_select
  std::vector<SlotHost> slots;
  // pinned staging
  DevItem* h_items = nullptr;
  int32_t* h_counts = nullptr;
  int32_t* h_ids = nullptr;
  double* h_logprob = nullptr;
  uint32_t* d_allowed = nullptr;
  size_t allowed_cap = 0;
  // allowed-id bit masks (needle_cuda_mask_pool / needle_cuda_masks_put)
  uint32_t* d_masks = nullptr;     // [mask_capacity][mask_words]
  int32_t mask_capacity = 0, mask_words = 0;
  std::vector<int32_t> mask_count;  // ids set in each slot's mask as last put (0: empty or never put)
  uint32_t* h_mask_stage = nullptr;  // pinned: max_seqs slot numbers, then max_seqs masks
  uint32_t* d_mask_stage = nullptr;
  cudaEvent_t mask_staged = nullptr;  // recorded after the last staging copy
  DevItem* h_items_end = nullptr;  // the items as needle_cuda_step_end re-uploads them
  SeqState* h_seq_stage = nullptr;  // pinned: each slot's state as needle_cuda_seq_reset uploads it
  float* h_lanes = nullptr;         // a resident-session item's lanes (pinned, kLaneWidth floats)
  uint32_t* h_engram = nullptr;     // and its engram lookup (pinned, 2 * kMaxTables)
  uint32_t* d_engram_in = nullptr;  // StepView::engram_in
  // a step begun by needle_cuda_step_begin and not yet ended
  struct PendingStep {
    bool active = false;
    int n = 0, n_sel = 0;
    std::vector<int> order;
    std::vector<needle_step_item> items;
    bool resident = false;  // begun by needle_cuda_resident_forward
    int mb = 0, cap = 0;    // begun as mb micro-batches of cap rows (0: one batch)
  } pending;
  // scheduler
  SchedView sched{};
  bool sched_loaded = false;
  int64_t sched_gen_total = 0;  // entries of sched.gen_ids
  std::vector<void*> sched_allocs;
  // matvec API scratch
  float* d_mv_x = nullptr;
  float* d_mv_xp = nullptr;
  float* d_mv_y = nullptr;
  size_t mv_cap = 0;
  int32_t* d_rows = nullptr;
  float* d_row_out = nullptr;
  // profiling
  bool profiling = false;
  bool nvtx = false;  // NEEDLE_NVTX set at open: an NVTX range around every step and kernel class
  int64_t launches = 0;  // kernels launched by this context
  int collecting = 0;    // slots that feed a confidence probe pool
  double* d_confidence = nullptr;
  std::vector<ProfEntry> prof_pending;
  std::vector<cudaEvent_t> event_pool;
  double prof_ms[kProfClasses] = {0};
  int64_t prof_n[kProfClasses] = {0};

  // Device buffers carry kGuardBytes of a known pattern after their last byte
  // (needle_cuda_check_guards reads them back: a kernel that wrote past a buffer is found).
  static constexpr size_t kGuardBytes = 256;
  static constexpr int kGuardByte = 0xA5;
  struct Guard {
    const uint8_t* at;
  };
  std::vector<Guard> guards;
  template <class T>
  T* dalloc(size_t count, bool zero = true) {
    void* p = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    cuda_check(cudaMalloc(&p, bytes + kGuardBytes), "cudaMalloc");
    allocs.push_back(p);
    if (zero) cuda_check(cudaMemset(p, 0, bytes), "cudaMemset");
    cuda_check(cudaMemset(static_cast<uint8_t*>(p) + bytes, kGuardByte, kGuardBytes), "cudaMemset");
    guards.push_back({static_cast<const uint8_t*>(p) + bytes});
    return static_cast<T*>(p);
  }

  cudaEvent_t get_event() {
    if (!event_pool.empty()) {
      cudaEvent_t e = event_pool.back();
      event_pool.pop_back();
      return e;
    }
    cudaEvent_t e;
    cuda_check(cudaEventCreate(&e), "cudaEventCreate");
    return e;
  }
  void prof_drain() {
    if (prof_pending.empty()) return;
    cuda_check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    for (auto& p : prof_pending) {
      float ms = 0;
      cuda_check(cudaEventElapsedTime(&ms, p.a, p.b), "cudaEventElapsedTime");
      prof_ms[p.cls] += ms;
      prof_n[p.cls] += 1;
      event_pool.push_back(p.a);
      event_pool.push_back(p.b);
    }
    prof_pending.clear();
  }
  // Runs `launch` (which enqueues on `s`) bracketed by events when profiling.
  template <class F>
  void timed(int cls, F&& launch, cudaStream_t s = nullptr) {
    if (!s) s = stream;
    if (cls != P_COPY) launches += cls == P_SCHED ? 2 : 1;
    struct Range {
      bool on;
      Range(bool o, const char* name) : on(o) {
        if (on) nvtxRangePushA(name);
      }
      ~Range() {
        if (on) nvtxRangePop();
      }
    } range(nvtx, kProfNames[cls]);
    if (!profiling) {
      cuda_check(launch(), kProfNames[cls]);
      return;
    }
    cudaEvent_t a = get_event(), b = get_event();
    cuda_check(cudaEventRecord(a, s), "cudaEventRecord");
    cuda_check(launch(), kProfNames[cls]);
    cuda_check(cudaEventRecord(b, s), "cudaEventRecord");
    prof_pending.push_back({cls, a, b});
    if (prof_pending.size() > 4096) prof_drain();
  }
};

namespace {

CqMat upload_cq(needle_ctx& C, int i) {
  const Record& R = C.A.rec[i];
  CqMat m;
  uint8_t* packed = C.dalloc<uint8_t>(size_t(R.packed_bytes) + 64);  // zero tail
  uint16_t* norms = C.dalloc<uint16_t>(size_t(R.length - R.packed_bytes) / 2 + 8, false);
  cuda_check(cudaMemcpy(packed, C.A.b + R.offset, R.packed_bytes, cudaMemcpyHostToDevice), "upload");
  cuda_check(cudaMemcpy(norms, C.A.b + R.offset + R.packed_bytes, R.length - R.packed_bytes,
                        cudaMemcpyHostToDevice), "upload");
  m.packed = packed;
  m.norms = norms;
  m.rows = int32_t(R.rows);
  m.input_size = int32_t(R.input);
  m.in_pad = int32_t(R.in_pad);
  m.bits = int32_t(R.bits);
  m.row_bytes = int32_t(R.row_bytes);
  return m;
}

// Matrices of equal record width and input length stacked row-wise into one (packed rows, then
// fp16 norms, as the archive lays out one matrix), copied on the device.
CqMat stack_rows(needle_ctx& C, std::initializer_list<CqMat> parts) {
  const CqMat& f = *parts.begin();
  int rows = 0;
  for (const CqMat& p : parts) {
    require(p.bits == f.bits && p.in_pad == f.in_pad && p.input_size == f.input_size, NEEDLE_UNSUPPORTED_CACT,
            "fast numerics needs the projections that share an input to share a record width");
    rows += p.rows;
  }
  const int groups = f.in_pad / kGroup;
  uint8_t* packed = C.dalloc<uint8_t>(size_t(rows) * f.row_bytes + 64);
  uint16_t* norms = C.dalloc<uint16_t>(size_t(rows) * groups + 8, false);
  size_t r0 = 0;
  for (const CqMat& p : parts) {
    cuda_check(cudaMemcpy(packed + r0 * f.row_bytes, p.packed, size_t(p.rows) * f.row_bytes, cudaMemcpyDeviceToDevice),
               "stack");
    cuda_check(cudaMemcpy(norms + r0 * groups, p.norms, size_t(p.rows) * groups * 2, cudaMemcpyDeviceToDevice), "stack");
    r0 += p.rows;
  }
  CqMat m = f;
  m.packed = packed;
  m.norms = norms;
  m.rows = rows;
  return m;
}

// 2-bit matrices of one input length stacked row-wise in group-major order: [group][row][32 bytes]
// (row_bytes of the result = the stride between groups), fp16 norms stacked row-major as usual.
// Returns an empty matrix (rows 0) when the parts do not qualify.
CqMat stack_group_major(needle_ctx& C, std::initializer_list<CqMat> parts) {
  const CqMat& f = *parts.begin();
  int rows = 0;
  for (const CqMat& p : parts) {
    if (p.bits != 2 || p.in_pad != f.in_pad || p.input_size != f.input_size || p.row_bytes != p.in_pad / 4)
      return CqMat{};
    rows += p.rows;
  }
  const int groups = f.in_pad / kGroup;
  constexpr int kRecord = kGroup / 4;  // bytes of one (row, group) record
  uint8_t* packed = C.dalloc<uint8_t>(size_t(groups) * rows * kRecord + 64);
  uint16_t* norms = C.dalloc<uint16_t>(size_t(rows) * groups + 8, false);
  size_t r0 = 0;
  for (const CqMat& p : parts) {
    for (int g = 0; g < groups; g++)
      cuda_check(cudaMemcpy2D(packed + (size_t(g) * rows + r0) * kRecord, kRecord, p.packed + size_t(g) * kRecord,
                              size_t(p.row_bytes), kRecord, size_t(p.rows), cudaMemcpyDeviceToDevice),
                 "group-major stack");
    cuda_check(cudaMemcpy(norms + r0 * groups, p.norms, size_t(p.rows) * groups * 2, cudaMemcpyDeviceToDevice), "stack");
    r0 += p.rows;
  }
  CqMat m = f;
  m.packed = packed;
  m.norms = norms;
  m.rows = rows;
  m.row_bytes = rows * kRecord;
  return m;
}

const float* upload_floats(needle_ctx& C, const std::vector<float>& v) {
  float* d = C.dalloc<float>(v.size(), false);
  cuda_check(cudaMemcpy(d, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice), "upload");
  return d;
}

std::vector<float> pack_layers(const needle_ctx& C, int Roles::L::*field, size_t expect) {
  std::vector<float> out;
  for (const auto& L : C.roles.layers) {
    std::vector<float> v = C.A.dense(L.*field);
    require(v.size() == expect, NEEDLE_UNSUPPORTED_CACT, "Unexpected dense tensor length");
    out.insert(out.end(), v.begin(), v.end());
  }
  return out;
}

void check_geometry(const needle_ctx& C) {
  const Archive& A = C.A;
  const uint32_t* h = A.hdr;
  auto gate = [&](bool ok, const std::string& what) {
    require(ok, NEEDLE_BACKEND_UNAVAILABLE, "CUDA backend does not support this geometry: " + what);
  };
  gate(h[6] == kDim && h[10] == kHeadDim && h[7] == kHeads && h[8] == kKvHeads && h[13] == kLanes &&
           h[12] == kHadamard,
       "needs d=512, head_dim=64, 8 query / 4 KV heads, 4 lanes, Hadamard 512");
  const Roles& R = C.roles;
  auto cqr = [&](int i) -> const Record& { return A.rec[i]; };
  for (const auto& L : R.layers) {
    gate(cqr(L.q).rows == 512 && cqr(L.q).input == 512 && cqr(L.k).rows == 256 && cqr(L.k).input == 512 &&
             cqr(L.v).rows == 256 && cqr(L.v).input == 512 && cqr(L.gate).rows == 512 &&
             cqr(L.gate).input == 512 && cqr(L.o).rows == 512 && cqr(L.o).input == 512,
         "projection shapes");
    for (int t : {L.q, L.k, L.v, L.gate, L.o}) gate(cqr(t).group == kGroup, "CQ group size 128");
  }
  gate(cqr(R.embedding).group == kGroup, "CQ group size 128");
  const int L = int(h[9]);
  gate(cqr(R.phi_pre).rows == int64_t(L) * 4 && cqr(R.phi_pre).input == kLaneWidth &&
           cqr(R.phi_post).rows == int64_t(L) * 4 && cqr(R.phi_post).input == kLaneWidth &&
           cqr(R.phi_res).rows == int64_t(L) * 16 && cqr(R.phi_res).input == kLaneWidth,
       "mHC phi shapes");
  for (int t : {R.phi_pre, R.phi_post, R.phi_res}) gate(cqr(t).group == kGroup, "CQ group size 128");
  if (!R.sites.empty()) {
    gate(h[16] >= 1 && h[16] <= kMaxTables && h[15] == kGroup && h[16] * h[15] == kDim,
         "engram tables x sub-dimension must be 512 with 128-wide rows");
    gate(h[19] >= 1 && h[16] % h[19] == 0, "engram table count divisible by order count");
    uint32_t mo = 1;
    for (uint32_t i = 0; i < h[19]; i++) {
      gate(h[20 + i] >= 1 && h[20 + i] <= 4, "engram orders in 1..4");
      mo = std::max(mo, h[20 + i]);
    }
    gate((h[17] - 1) * mo + 1 <= 64 && h[17] >= 1, "engram ring depth");
    for (const auto& e : R.sites) {
      gate(cqr(e.tables).input == kGroup && cqr(e.tables).group == kGroup &&
               cqr(e.tables).rows == int64_t(h[16]) * h[14],
           "engram table shape");
      gate(cqr(e.k).rows == 512 && cqr(e.k).input == 512 && cqr(e.v).rows == 512 && cqr(e.v).input == 512 &&
               cqr(e.k).group == kGroup && cqr(e.v).group == kGroup,
           "engram projection shape");
    }
    for (uint32_t s = 0; s < h[24]; s++) gate(h[25 + s] < uint32_t(L), "engram site layer");
  }
  gate(cqr(R.embedding).rows == h[5] && cqr(R.embedding).input == kDim, "embedding shape");
}

void build_model(needle_ctx& C) {
  Archive& A = C.A;
  const uint32_t* h = A.hdr;
  const int L = int(h[9]);
  C.cq.assign(A.rec.size(), CqMat{});
  for (size_t i = 0; i < A.rec.size(); i++)
    if (A.rec[i].dtype == 3) C.cq[i] = upload_cq(C, int(i));
  ModelView& m = C.mv;
  const Roles& R = C.roles;
  m.embedding = C.cq[R.embedding];
  m.phi_pre = C.cq[R.phi_pre];
  m.phi_post = C.cq[R.phi_post];
  m.phi_res = C.cq[R.phi_res];
  m.layers = L;
  m.vocab = int32_t(h[5]);
  m.kv_window = int32_t(h[3]);
  m.max_seq = int32_t(h[11]);
  m.n_sites = int32_t(R.sites.size());
  for (int s = 0; s < m.n_sites; s++) {
    m.sites[s] = int32_t(h[25 + s]);
    m.engram_tables[s] = C.cq[R.sites[s].tables];
    C.ek.push_back(C.cq[R.sites[s].k]);
    C.ev.push_back(C.cq[R.sites[s].v]);
  }
  m.n_orders = int32_t(h[19]);
  m.max_order = 1;
  for (int i = 0; i < m.n_orders; i++) {
    m.orders[i] = int32_t(h[20 + i]);
    m.max_order = std::max(m.max_order, m.orders[i]);
  }
  m.n_tables = int32_t(h[16]);
  m.engram_slots = int32_t(h[14]);
  m.engram_sub = int32_t(h[15]);
  m.taps = int32_t(h[17]);
  for (const auto& Lr : R.layers) {
    C.lq.push_back(C.cq[Lr.q]);
    C.lk.push_back(C.cq[Lr.k]);
    C.lv.push_back(C.cq[Lr.v]);
    C.lg.push_back(C.cq[Lr.gate]);
    C.lo.push_back(C.cq[Lr.o]);
  }
  m.fast = C.fast ? 1 : 0;
  if (C.fast) {
    for (int l = 0; l < L; l++) C.lqkvg.push_back(stack_rows(C, {C.lq[l], C.lk[l], C.lv[l], C.lg[l]}));
    for (int s = 0; s < m.n_sites; s++) C.ekv.push_back(stack_rows(C, {C.ek[s], C.ev[s]}));
  } else {
    for (int l = 0; l < L; l++) {
      CqMat gm = stack_group_major(C, {C.lq[l], C.lk[l], C.lv[l], C.lg[l]});
      if (gm.rows == 0) {
        C.lqkvg_gm.clear();
        break;
      }
      C.lqkvg_gm.push_back(gm);
    }
  }
  m.norm_input = upload_floats(C, pack_layers(C, &Roles::L::norm_input, kDim));
  m.query_norm = upload_floats(C, pack_layers(C, &Roles::L::qn, kHeadDim));
  m.key_norm = upload_floats(C, pack_layers(C, &Roles::L::kn, kHeadDim));
  m.post_norm = upload_floats(C, pack_layers(C, &Roles::L::post, kDim));
  m.pre_had_norm = upload_floats(C, pack_layers(C, &Roles::L::pre_had, kDim));
  m.d1 = upload_floats(C, pack_layers(C, &Roles::L::d1, kHadamard));
  m.d2 = upload_floats(C, pack_layers(C, &Roles::L::d2, kHadamard));
  m.d3 = upload_floats(C, pack_layers(C, &Roles::L::d3, kHadamard));
  {
    std::vector<float> g;
    for (const auto& Lr : R.layers) {
      std::vector<float> v = A.dense(Lr.attn_gate);
      g.push_back(v.empty() ? 0.0f : v[0]);
    }
    m.attn_gate = upload_floats(C, g);
  }
  auto dense_n = [&](int i, size_t n, const char* what) {
    std::vector<float> v = A.dense(i);
    require(v.size() >= n, NEEDLE_INVALID_CACT, std::string(what) + " is too short");
    return v;
  };
  m.a_pre = upload_floats(C, dense_n(R.a_pre, L, "mHC a_pre"));
  m.a_post = upload_floats(C, dense_n(R.a_post, L, "mHC a_post"));
  m.a_res = upload_floats(C, dense_n(R.a_res, L, "mHC a_res"));
  m.b_pre = upload_floats(C, dense_n(R.b_pre, size_t(L) * 4, "mHC b_pre"));
  m.b_post = upload_floats(C, dense_n(R.b_post, size_t(L) * 4, "mHC b_post"));
  m.b_res = upload_floats(C, dense_n(R.b_res, size_t(L) * 16, "mHC b_res"));
  {
    std::vector<float> taps;
    for (const auto& e : R.sites) {
      std::vector<float> v = dense_n(e.taps, size_t(m.taps) * kDim, "engram taps");
      taps.insert(taps.end(), v.begin(), v.begin() + size_t(m.taps) * kDim);
    }
    if (taps.empty()) taps.push_back(0.0f);
    m.taps_w = upload_floats(C, taps);
  }
  m.final_norm = upload_floats(C, dense_n(R.final_norm, kDim, "final norm"));
  if (R.conf_probes >= 0) {
    require(R.conf_count <= kMaxProbes, NEEDLE_UNSUPPORTED_CACT,
            "confidence head has more than " + std::to_string(kMaxProbes) + " probes");
    m.probes = upload_floats(C, A.dense(R.conf_probes));
    m.probe_proj = upload_floats(C, A.dense(R.conf_proj));
    std::vector<float> bias = A.dense(R.conf_bias);
    bias.resize(size_t(R.conf_out), 0.0f);  // rows past the bias length sum from 0 (cq.ts:307)
    m.probe_bias = upload_floats(C, bias);
    m.probe_count = int32_t(R.conf_count);
    m.probe_out = int32_t(R.conf_out);
  }
  // RoPE angles in binary64 exactly as applyRope (math.ts:104-108) evaluates them.
  {
    const double theta = double(A.rope_theta);
    std::vector<double> cs(size_t(m.max_seq) * 32), sn(size_t(m.max_seq) * 32);
    for (int p = 0; p < m.max_seq; p++)
      for (int d = 0; d < 32; d++) {
        const double frequency = std::pow(theta, -(2.0 * d) / double(kHeadDim));
        const double angle = double(p) * frequency;
        cs[size_t(p) * 32 + d] = std::cos(angle);
        sn[size_t(p) * 32 + d] = std::sin(angle);
      }
    double* dc = C.dalloc<double>(cs.size(), false);
    double* ds = C.dalloc<double>(sn.size(), false);
    cuda_check(cudaMemcpy(dc, cs.data(), cs.size() * 8, cudaMemcpyHostToDevice), "upload");
    cuda_check(cudaMemcpy(ds, sn.data(), sn.size() * 8, cudaMemcpyHostToDevice), "upload");
    m.rope_cos = dc;
    m.rope_sin = ds;
  }
  for (int i = 0; i < 28; i++) m.cb.v[i] = A.codebook[i];
}

void build_state(needle_ctx& C) {
  const needle_opts& o = C.opts;
  const ModelView& m = C.mv;
  const int S = o.max_seqs, L = m.layers;
  const int window = m.kv_window;
  const int capacity = window > 0 ? std::min(o.max_len, o.max_sink + window) : o.max_len;
  SlotView& sv = C.sv;
  sv.capacity = capacity;
  sv.layers = L;
  const int depth = (m.taps - 1) * m.max_order + 1;
  sv.x = C.dalloc<float>(size_t(S) * kLaneWidth);
  sv.ring = C.dalloc<float>(size_t(S) * std::max(1, m.n_sites) * depth * kDim);
  const size_t heads = size_t(S) * L * kKvHeads * capacity;
  sv.kv_f32 = o.kv_mode == NEEDLE_KV_FLOAT32 ? 1 : 0;
  if (sv.kv_f32) {
    sv.kf = C.dalloc<float>(heads * kHeadDim);
    sv.vf = C.dalloc<float>(heads * kHeadDim);
  } else {
    sv.kcodes = C.dalloc<int8_t>(heads * kHeadDim);
    sv.vcodes = C.dalloc<int8_t>(heads * kHeadDim);
  }
  sv.kscale = C.dalloc<float>(heads);
  sv.vscale = C.dalloc<float>(heads);
  sv.seq = C.dalloc<SeqState>(S);
  if (m.probe_count > 0) {
    sv.pool_max = C.dalloc<double>(size_t(S) * m.probe_count);
    sv.pool_den = C.dalloc<double>(size_t(S) * m.probe_count);
    sv.pool_w = C.dalloc<double>(size_t(S) * m.probe_count * kDim);
  }
  C.slots.assign(S, SlotHost{});
  StepView& st = C.stv;
  // scheduled steps with chunks use item rows up to ceil(sched_items / M) * M < sched_items + kMaxMicro
  const size_t B = size_t(std::max({S, kPrefillChunk, C.sched_items > 0 ? C.sched_items + kMaxMicro : 0}));
  C.step_capacity = int(B);
  st.items = C.dalloc<DevItem>(B);
  st.chunk = 0;
  st.lanes = C.dalloc<float>(B * kLaneWidth);
  C.d_engram_in = C.dalloc<uint32_t>(B * 2 * kMaxTables);
  st.engram_in = C.d_engram_in;
  C.d_counts = C.dalloc<int32_t>(2 + 2 * kMaxMicro);
  C.d_confidence = C.dalloc<double>(1);
  st.n_items = C.d_counts;
  st.n_select = C.d_counts + 1;
  const int ns = std::max(1, m.n_sites);
  st.prep_engram = C.dalloc<float>(B * ns * kDim);
  st.engram_kv = C.dalloc<float>(B * ns * 2 * kDim);
  st.engram_val = C.dalloc<float>(B * ns * kDim);
  st.update = C.dalloc<float>(B * kDim);
  st.block = C.dalloc<float>(B * kDim);
  st.prep_a = C.dalloc<float>(B * kDim);
  st.qkvg = C.dalloc<float>(B * 1536);
  st.prep_o = C.dalloc<float>(B * kDim);
  st.proj = C.dalloc<float>(B * kDim);
  st.route = C.dalloc<float>(B * 20);
  st.prep_f = C.dalloc<float>(B * kDim);
  st.logits = C.dalloc<float>(B * size_t(m.vocab));
  st.out_id = C.dalloc<int32_t>(B);
  st.out_logprob = C.dalloc<double>(B);
  C.allowed_cap = 1 << 16;
  C.d_allowed = C.dalloc<uint32_t>(C.allowed_cap);
  st.allowed = C.d_allowed;
  cuda_check(cudaMallocHost(&C.h_items, B * sizeof(DevItem)), "cudaMallocHost");
  cuda_check(cudaMallocHost(&C.h_items_end, B * sizeof(DevItem)), "cudaMallocHost");
  cuda_check(cudaMallocHost(&C.h_seq_stage, size_t(S) * sizeof(SeqState)), "cudaMallocHost");
  cuda_check(cudaMallocHost(&C.h_lanes, kLaneWidth * sizeof(float)), "cudaMallocHost");
  cuda_check(cudaMallocHost(&C.h_engram, 2 * kMaxTables * sizeof(uint32_t)), "cudaMallocHost");
  cuda_check(cudaMallocHost(&C.h_counts, (2 + 2 * kMaxMicro) * sizeof(int32_t)), "cudaMallocHost");
  cuda_check(cudaMallocHost(&C.h_ids, B * sizeof(int32_t)), "cudaMallocHost");
  cuda_check(cudaMallocHost(&C.h_logprob, B * sizeof(double)), "cudaMallocHost");
  cuda_check(configure_step_kernels(capacity), "cudaFuncSetAttribute");
  if (C.fast) {
    // the GEMM's tiling depends on the item count: size for every count a launch can have
    std::vector<const CqMat*> mats{&C.lqkvg[0], &C.lo[0], &m.embedding};
    if (!C.ekv.empty()) mats.push_back(&C.ekv[0]);
    size_t bytes = 0;
    for (const CqMat* M : mats)
      for (int n = 1; n <= int(B); n++) bytes = std::max(bytes, cq_gemm_tc_scratch_bytes(M->rows, M->input_size, n, C.sms));
    C.gemm_scratch_bytes = (bytes + 255) & ~size_t(255);
    for (int k = 0; k < kMaxMicro; k++) C.gemm_scratch[k] = C.dalloc<uint8_t>(C.gemm_scratch_bytes, false);
  }
  if (C.fast) {
    // fast attention: rotated queries, visible counts, cache rows, outputs; per lane its scratch
    // (status and work counters zeroed here, left at zero by every call)
    st.qrope = C.dalloc<float>(B * kDim);
    st.attn_out = C.dalloc<float>(B * kDim);
    st.attn_count = C.dalloc<int32_t>(B);
    st.attn_row = C.dalloc<int64_t>(B);
    for (int k = 0; k < kMaxMicro; k++)
      C.attn_scratch[k] = C.dalloc<uint8_t>(attention_fast_scratch_bytes(int32_t(B), capacity));
  }
}

// Builds the GEMV job list for matrices sharing one input (same bits per launch).
void add_job(CqJobs& J, const CqMat& M, int row_start, int rows, const float* x, int x_stride, float* y,
             int y_stride) {
  CqJob& j = J.job[J.count++];
  j.packed = M.packed;
  j.norms = M.norms;
  j.row_start = row_start;
  j.rows = rows;
  j.in_pad = M.in_pad;
  j.bits = M.bits;
  j.row_bytes = M.row_bytes;
  j.tile_begin = J.total_tiles;
  j.x = x;
  j.x_stride = x_stride;
  j.y = y;
  j.y_stride = y_stride;
  J.total_tiles += (rows + kGemvTileRows - 1) / kGemvTileRows;
}

struct JobSpec {
  CqMat M;
  int row_start, rows;
  const float* x;
  int x_stride;
  float* y;
  int y_stride;
};

// Launches the jobs grouped by record width (one GEMV launch per width present).  In fast numerics
// every job is a tensor-core GEMM over the lane's n_host item rows (rows past the device count hold
// stale inputs; their outputs are never read).
void run_gemv(needle_ctx& C, int cls, const std::vector<JobSpec>& specs, int n_host, const int32_t* n_dev,
              cudaStream_t strm = nullptr, int lane = 0) {
  if (!strm) strm = C.stream;
  if (C.fast) {
    for (const auto& sp : specs) {
      const CqMat& M = sp.M;
      const int splits = cq_gemm_tc_splits(sp.rows, M.input_size, n_host, C.sms);
      C.launches += (splits > 1 ? 3 : 2) - 1;  // prepare, GEMM, split-K sum; timed() counts one
      C.timed(cls, [&] {
        return launch_cq_gemm_tc(M.packed + int64_t(sp.row_start) * M.row_bytes,
                                 M.norms + int64_t(sp.row_start) * (M.in_pad / kGroup), sp.rows, M.input_size, M.bits,
                                 sp.x, sp.x_stride, 1, n_host, sp.y, sp.y_stride, C.mv.cb, C.gemm_scratch[lane], C.sms,
                                 strm);
      }, strm);
    }
    return;
  }
  for (int bits : {2, 3, 4, 5}) {
    CqJobs J{};
    for (const auto& s : specs)
      if (s.M.bits == bits) {
        require(J.count < kMaxJobs, NEEDLE_BACKEND_UNAVAILABLE, "too many GEMV jobs");
        add_job(J, s.M, s.row_start, s.rows, s.x, s.x_stride, s.y, s.y_stride);
      }
    if (J.count == 0) continue;
    C.timed(cls, [&] { return launch_cq_gemv(J, C.mv.cb, n_host, n_dev, strm); }, strm);
  }
}

// The streams one micro-batch of a step runs on: its main stream and the side stream of its
// Sinkhorn routing, with the events that fork and join them per layer.
struct Lane {
  cudaStream_t main, side;
  cudaEvent_t* fork;
  cudaEvent_t* join;
  int index;  // micro-batch lane (its own GEMM scratch in fast numerics)
};

// A view of the step scratch for the items [offset, ...) with their own device counts.
StepView half_view(const needle_ctx& C, int offset, const int32_t* n_items, const int32_t* n_select) {
  const StepView& st = C.stv;
  const int64_t o = offset, ns = C.mv.n_sites;
  StepView v = st;
  v.items = st.items + o;
  v.lanes = st.lanes + o * kLaneWidth;
  v.n_items = n_items;
  v.n_select = n_select;
  v.prep_engram = st.prep_engram + o * ns * kDim;
  v.engram_kv = st.engram_kv + o * ns * 2 * kDim;
  v.engram_val = st.engram_val + o * ns * kDim;
  v.update = st.update + o * kDim;
  v.block = st.block + o * kDim;
  v.prep_a = st.prep_a + o * kDim;
  v.qkvg = st.qkvg + o * 1536;
  v.prep_o = st.prep_o + o * kDim;
  v.proj = st.proj + o * kDim;
  v.route = st.route + o * 20;
  v.prep_f = st.prep_f + o * kDim;
  v.logits = st.logits + o * C.mv.vocab;
  v.out_id = st.out_id + o;
  v.out_logprob = st.out_logprob + o;
  if (st.qrope) {
    v.qrope = st.qrope + o * kDim;
    v.attn_out = st.attn_out + o * kDim;
    v.attn_count = st.attn_count + o;
    v.attn_row = st.attn_row + o;
  }
  return v;
}

// The kernel sequence of one batched step for up to n_host items of view `st` (device counts in
// st.n_items / st.n_select), on the lane's streams.
void enqueue_step(needle_ctx& C, const StepView& st, int n_host, bool any_select, const SchedView* sched,
                  const Lane& lane, bool finish = true) {
  const ModelView& m = C.mv;
  const SlotView& sv = C.sv;
  const int32_t* n_dev = st.n_items;
  cudaStream_t s0 = lane.main;
  const bool probes = !st.chunk && C.collecting > 0 && m.probe_count > 0;
  auto probe_add = [&](int source) {
    cuda_check(launch_probe_add(m, sv, st, source, n_host, s0), "probe pool");
    C.launches++;
  };
  C.timed(P_EMBED, [&] { return launch_embed(m, sv, st, n_host, s0); }, s0);
  if (probes) probe_add(0);
  if (m.n_sites > 0) {
    std::vector<JobSpec> jobs;
    for (int s = 0; s < m.n_sites; s++) {
      if (C.fast) {  // K and V rows of the site as one matrix: outputs [site][K | V]
        jobs.push_back({C.ekv[s], 0, 1024, st.prep_engram + s * kDim, m.n_sites * kDim,
                        st.engram_kv + (s * 2) * kDim, m.n_sites * 2 * kDim});
        continue;
      }
      jobs.push_back({C.ek[s], 0, 512, st.prep_engram + s * kDim, m.n_sites * kDim,
                      st.engram_kv + (s * 2) * kDim, m.n_sites * 2 * kDim});
      jobs.push_back({C.ev[s], 0, 512, st.prep_engram + s * kDim, m.n_sites * kDim,
                      st.engram_kv + (s * 2 + 1) * kDim, m.n_sites * 2 * kDim});
    }
    run_gemv(C, P_GEMV_ENGRAM, jobs, n_host, n_dev, s0, lane.index);
  }
  for (int l = 0; l <= m.layers; l++) {
    if (l > 0) cuda_check(cudaStreamWaitEvent(s0, lane.join[(l - 1) & 1], 0), "join");
    C.timed(P_LAYER, [&] { return launch_layer(m, sv, st, l, n_host, s0); }, s0);
    if (probes && l > 0) probe_add(1);  // lanes now hold the output of layer l - 1
    if (l == m.layers) break;
    // Sinkhorn routing of layer l on the side stream, joined before the next k_layer.
    cuda_check(cudaEventRecord(lane.fork[l & 1], s0), "fork");
    cuda_check(cudaStreamWaitEvent(lane.side, lane.fork[l & 1], 0), "fork");
    cuda_check(launch_route(st, n_host, lane.side), "route");
    C.launches++;
    cuda_check(cudaEventRecord(lane.join[l & 1], lane.side), "join");
    if (C.fast)
      run_gemv(C, P_GEMV_QKVG, {{C.lqkvg[l], 0, 1536, st.prep_a, kDim, st.qkvg, 1536}}, n_host, n_dev, s0,
               lane.index);
    else if (!C.lqkvg_gm.empty() && cq_gemv2_group_major_preferred(n_host)) {
      const CqMat& M = C.lqkvg_gm[l];
      CqJob j{};
      j.packed = M.packed;
      j.norms = M.norms;
      j.rows = M.rows;
      j.in_pad = M.in_pad;
      j.bits = M.bits;
      j.row_bytes = M.row_bytes;
      j.x = st.prep_a;
      j.x_stride = kDim;
      j.y = st.qkvg;
      j.y_stride = 1536;
      C.timed(P_GEMV_QKVG, [&] { return launch_cq_gemv2_group_major(j, C.mv.cb, n_host, n_dev, s0); }, s0);
    } else
      run_gemv(C, P_GEMV_QKVG,
               {{C.lq[l], 0, 512, st.prep_a, kDim, st.qkvg, 1536},
                {C.lk[l], 0, 256, st.prep_a, kDim, st.qkvg + 512, 1536},
                {C.lv[l], 0, 256, st.prep_a, kDim, st.qkvg + 768, 1536},
                {C.lg[l], 0, 512, st.prep_a, kDim, st.qkvg + 1024, 1536}},
               n_host, n_dev, s0);
    if (C.fast) {
      // append every item's K/V (and leave its rotated query, count and cache row), then attention
      // over the cache -- binary32 on the CUDA cores (NEEDLE_NUMERICS_FAST) or int8 MMAs
      // (NEEDLE_NUMERICS_FAST_ATTENTION) -- and the gate
      const int64_t cache_rows = int64_t(C.opts.max_seqs) * m.layers * kKvHeads * sv.capacity;
      C.launches += 3;  // + persistent attention, combine, gate (timed() counts the append)
      C.timed(P_ATTN, [&] {
        cudaError_t e = launch_attention(m, sv, st, l, n_host, s0, 1);
        if (e == cudaSuccess)
          e = launch_attention_fast(st.qrope, sv.kcodes, sv.kscale, sv.vcodes, sv.vscale, st.attn_count, n_host,
                                    sv.capacity, st.attn_out, C.attn_scratch[lane.index], s0, st.attn_row, cache_rows,
                                    C.fast_attention);
        if (e == cudaSuccess) e = launch_attention_gate(st, n_host, s0);
        return e;
      }, s0);
    } else if (st.chunk) {  // every chunk item's K/V before any of them attends (timed as one)
      C.launches++;  // timed() counts one of the two
      C.timed(P_ATTN, [&] {
        cudaError_t e = launch_attention(m, sv, st, l, n_host, s0, 3);
        return e == cudaSuccess ? launch_attention(m, sv, st, l, n_host, s0, 4) : e;
      }, s0);
    } else {
      C.timed(P_ATTN, [&] { return launch_attention(m, sv, st, l, n_host, s0); }, s0);
    }
    run_gemv(C, P_GEMV_O, {{C.lo[l], 0, 512, st.prep_o, kDim, st.proj, kDim}}, n_host, n_dev, s0, lane.index);
  }
  if (any_select)
    run_gemv(C, P_GEMV_VOCAB, {{m.embedding, 0, m.vocab, st.prep_f, kDim, st.logits, m.vocab}}, n_host,
             st.n_select, s0, lane.index);
  if (finish) C.timed(P_FINISH, [&] { return launch_finish(m, sv, st, n_host, sched, s0); }, s0);
}

Lane lane_a(needle_ctx& C) { return Lane{C.stream, C.side, C.fork_ev, C.join_ev, 0}; }
Lane lane_k(needle_ctx& C, int k) {
  return k == 0 ? lane_a(C) : Lane{C.mb_main[k], C.mb_side[k], C.mb_fork[k], C.mb_join[k], k};
}

// One device-scheduled step: admission and item list on the device, then the busy slots as
// `micro` micro-batches on their own stream pairs, so the latency-bound kernels of one (k_layer's
// sequential sums, attention's softmax and value chains) overlap the GEMVs and attention of the
// others (one batch when profiling, so per-kernel times stay unperturbed).
void enqueue_sched_step(needle_ctx& C) {
  const int S = C.sched.n_slots;
  const int M = C.profiling ? 1 : std::max(1, std::min(C.micro, S / 32));
  const int h = (S + M - 1) / M;
  // with prompt chunks, micro-batch k holds slots [k * h, (k + 1) * h) in item rows [k * hi, ...)
  const bool chunks = C.sched_chunk >= 2;
  const int hi = chunks ? (C.sched_items + M - 1) / M : h;
  C.timed(P_SCHED, [&] {
    cudaError_t e = launch_sched_admit(C.sv, C.sched, C.mv.kv_window, C.stream);
    if (e != cudaSuccess) return e;
    if (chunks)
      return launch_sched_chunked(C.sv, C.stv, C.sched, C.d_counts, h, hi, M, C.sched_chunk, C.mv.kv_window,
                                  C.stream);
    return launch_sched(C.sv, C.stv, C.sched, C.d_counts, h, M, C.stream);
  });
  auto view = [&](int off, const int32_t* n_items, const int32_t* n_select) {
    StepView v = half_view(C, off, n_items, n_select);
    v.chunk = chunks ? 1 : 0;
    return v;
  };
  if (M == 1) {
    enqueue_step(C, view(0, C.d_counts, C.d_counts + 1), hi, true, &C.sched, lane_a(C));
    return;
  }
  cuda_check(cudaEventRecord(C.split_ev, C.stream), "split");
  for (int k = 1; k < M; k++) cuda_check(cudaStreamWaitEvent(C.mb_main[k], C.split_ev, 0), "split");
  for (int k = 0; k < M; k++) {
    const int n = chunks ? hi : std::min(h, S - k * h);
    if (n <= 0 || k * h >= S) continue;
    enqueue_step(C, view(k * hi, C.d_counts + 2 + 2 * k, C.d_counts + 3 + 2 * k), n, true, &C.sched,
                 lane_k(C, k));
  }
  for (int k = 1; k < M; k++) {
    cuda_check(cudaEventRecord(C.mb_done[k], C.mb_main[k]), "merge");
    cuda_check(cudaStreamWaitEvent(C.stream, C.mb_done[k], 0), "merge");
  }
}

// Host steps of many items run as micro-batches, like device-scheduled steps: micro-batch k holds
// item rows [k * cap, (k + 1) * cap) with its own device counts, its selecting items first, and a
// slot's items (a prompt chunk) stay in one micro-batch.  Fills dst, order (item i's row) and
// h_counts; false when the items do not fit that shape.
bool stage_items_mb(needle_ctx& C, const needle_step_item* items, int32_t n, int M, int cap, std::vector<int>& order,
                    DevItem* dst) {
  std::vector<int> part(n);
  const int target = (n + M - 1) / M;
  int k = 0, fill = 0;
  for (int i = 0; i < n;) {
    int len = 1;
    while (i + len < n && items[i + len].seq == items[i].seq) len++;
    if (fill > 0 && (fill + len > cap || (fill >= target && k < M - 1))) {
      k++;
      fill = 0;
    }
    if (k >= M || len > cap) return false;
    for (int j = 0; j < len; j++) part[i + j] = k;
    fill += len;
    i += len;
  }
  std::vector<int> n_sel(M, 0), n_all(M, 0);
  for (int i = 0; i < n; i++) {
    n_all[part[i]]++;
    if (items[i].select) n_sel[part[i]]++;
  }
  std::vector<int> next_sel(M), next_rest(M);
  for (int q = 0; q < M; q++) {
    next_sel[q] = q * cap;
    next_rest[q] = q * cap + n_sel[q];
  }
  order.resize(n);
  int run_start = 0, run_len = 1;
  for (int i = 0; i < n; i++) {
    const needle_step_item& it = items[i];
    if (i == 0 || items[i - 1].seq != it.seq) {
      run_start = i;
      run_len = 1;
      while (i + run_len < n && items[i + run_len].seq == it.seq) run_len++;
    }
    const int row = it.select ? next_sel[part[i]]++ : next_rest[part[i]]++;
    order[i] = row;
    DevItem d{};
    d.slot = it.seq;
    d.token = it.token;
    d.select = it.select ? 1 : 0;
    d.allowed_count = it.select ? it.allowed_count : -1;
    d.allowed_offset = it.allowed_offset;
    d.position = C.slots[it.seq].position + (i - run_start);
    d.out_index = i;
    if (run_len > 1) {
      d.chunk_index = i - run_start;
      d.chunk_len = run_len;
    }
    dst[row] = d;
  }
  int sel_all = 0;
  for (int q = 0; q < M; q++) {
    C.h_counts[2 + 2 * q] = n_all[q];
    C.h_counts[3 + 2 * q] = n_sel[q];
    sel_all += n_sel[q];
  }
  C.h_counts[0] = n;
  C.h_counts[1] = sel_all;
  return true;
}

// The kernels of a micro-batched host step (every micro-batch sized `cap` rows; the device counts
// say how many each holds), forked from and joined back to the context stream; without selection
// when `finish` is false (needle_cuda_step_begin).
void enqueue_host_mb(needle_ctx& C, int M, int cap, bool finish = true) {
  cuda_check(cudaEventRecord(C.split_ev, C.stream), "split");
  for (int k = 1; k < M; k++) cuda_check(cudaStreamWaitEvent(C.mb_main[k], C.split_ev, 0), "split");
  for (int k = 0; k < M; k++) {
    StepView v = half_view(C, k * cap, C.d_counts + 2 + 2 * k, C.d_counts + 3 + 2 * k);
    v.chunk = 1;
    enqueue_step(C, v, cap, true, nullptr, lane_k(C, k), finish);
  }
  for (int k = 1; k < M; k++) {
    cuda_check(cudaEventRecord(C.mb_done[k], C.mb_main[k]), "merge");
    cuda_check(cudaStreamWaitEvent(C.stream, C.mb_done[k], 0), "merge");
  }
}

// Drops the captured host steps (their kernels hold buffer addresses that are about to change).
void drop_host_graph(needle_ctx& C) {
  if (!C.host_graph && !C.host_graph_begin && !C.single_graph) return;
  cudaStreamSynchronize(C.stream);
  if (C.host_graph) cudaGraphExecDestroy(C.host_graph);
  if (C.host_graph_begin) cudaGraphExecDestroy(C.host_graph_begin);
  if (C.single_graph) cudaGraphExecDestroy(C.single_graph);
  C.host_graph = C.host_graph_begin = C.single_graph = nullptr;
  C.host_eager_steps = 0;
  C.single_eager_steps = 0;
}

// A one-item host step (the batch-1 decode loop): its 140 kernels as one graph replay after the
// first eager run, so the GPU does not wait on launch gaps between the dependent kernels.
void run_single(needle_ctx& C) {
  auto enqueue = [&] { enqueue_step(C, C.stv, 1, true, nullptr, lane_a(C)); };
  if (C.single_eager_steps < 1) {
    enqueue();
    C.single_eager_steps++;
    return;
  }
  if (!C.single_graph) {
    cuda_check(cudaStreamBeginCapture(C.stream, cudaStreamCaptureModeThreadLocal), "capture");
    const int64_t l0 = C.launches;
    try {
      enqueue();
    } catch (...) {
      cudaGraph_t broken = nullptr;
      cudaStreamEndCapture(C.stream, &broken);
      if (broken) cudaGraphDestroy(broken);
      throw;
    }
    C.single_launches = C.launches - l0;
    C.launches = l0;
    cudaGraph_t g = nullptr;
    cuda_check(cudaStreamEndCapture(C.stream, &g), "capture");
    const cudaError_t e = cudaGraphInstantiate(&C.single_graph, g, 0);
    cudaGraphDestroy(g);
    cuda_check(e, "cudaGraphInstantiate");
  }
  cuda_check(cudaGraphLaunch(C.single_graph, C.stream), "cudaGraphLaunch");
  C.launches += C.single_launches;
}

// Runs a micro-batched host step's kernels: eagerly the first time, then as a replay of the step
// captured on the context stream (`graph` / `launches` hold the capture).
void run_host_mb(needle_ctx& C, int M, int cap, bool finish, cudaGraphExec_t& graph, int64_t& launches) {
  if (C.host_eager_steps < 1) {
    enqueue_host_mb(C, M, cap, finish);
    C.host_eager_steps++;
    return;
  }
  if (!graph) {
    cuda_check(cudaStreamBeginCapture(C.stream, cudaStreamCaptureModeThreadLocal), "capture");
    const int64_t l0 = C.launches;
    try {
      enqueue_host_mb(C, M, cap, finish);
    } catch (...) {
      cudaGraph_t broken = nullptr;
      cudaStreamEndCapture(C.stream, &broken);
      if (broken) cudaGraphDestroy(broken);
      throw;
    }
    launches = C.launches - l0;
    C.launches = l0;
    cudaGraph_t g = nullptr;
    cuda_check(cudaStreamEndCapture(C.stream, &g), "capture");
    const cudaError_t e = cudaGraphInstantiate(&graph, g, 0);
    cudaGraphDestroy(g);
    cuda_check(e, "cudaGraphInstantiate");
  }
  cuda_check(cudaGraphLaunch(graph, C.stream), "cudaGraphLaunch");
  C.launches += launches;
}

// Whether a host step of n items runs as micro-batches, and in what shape.
bool host_mb_shape(const needle_ctx& C, int32_t n, bool all_logits, int* M, int* cap) {
  if (all_logits || C.collecting != 0 || C.profiling || C.micro < 2 || n < 64) return false;
  *M = C.micro;
  *cap = C.step_capacity / C.micro;
  return true;
}

// Uploads a micro-batched step's item rows and per-micro-batch counts.
void upload_items_mb(needle_ctx& C, const DevItem* src, int M, int cap) {
  C.timed(P_COPY, [&] {
    cudaError_t e = cudaMemcpyAsync(C.stv.items, src, size_t(M) * cap * sizeof(DevItem), cudaMemcpyHostToDevice,
                                    C.stream);
    if (e != cudaSuccess) return e;
    return cudaMemcpyAsync(C.d_counts, C.h_counts, size_t(2 + 2 * M) * sizeof(int32_t), cudaMemcpyHostToDevice,
                           C.stream);
  });
}

// The context of every call except needle_cuda_step_end and needle_cuda_close: none may run while a
// step begun by needle_cuda_step_begin is waiting for its end.
needle_ctx* ctx_of(needle_ctx* c) {
  require(c != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "null needle context");
  require(!c->pending.active, NEEDLE_BACKEND_UNAVAILABLE,
          "needle_cuda_step_begin was called; needle_cuda_step_end must come first");
  cuda_check(cudaSetDevice(c->device), "cudaSetDevice");
  return c;
}

void destroy(needle_ctx* C) {
  if (!C) return;
  cudaSetDevice(C->device);
  if (C->stream) cudaStreamSynchronize(C->stream);
  for (auto& p : C->prof_pending) {
    cudaEventDestroy(p.a);
    cudaEventDestroy(p.b);
  }
  for (auto e : C->event_pool) cudaEventDestroy(e);
  for (void* p : C->sched_allocs) cudaFree(p);
  for (void* p : C->allocs) cudaFree(p);
  if (C->d_mv_x) cudaFree(C->d_mv_x);
  if (C->d_mv_xp) cudaFree(C->d_mv_xp);
  if (C->d_mv_y) cudaFree(C->d_mv_y);
  if (C->d_rows) cudaFree(C->d_rows);
  if (C->d_row_out) cudaFree(C->d_row_out);
  if (C->h_items) cudaFreeHost(C->h_items);
  if (C->h_items_end) cudaFreeHost(C->h_items_end);
  if (C->h_seq_stage) cudaFreeHost(C->h_seq_stage);
  if (C->h_lanes) cudaFreeHost(C->h_lanes);
  if (C->h_engram) cudaFreeHost(C->h_engram);
  if (C->h_counts) cudaFreeHost(C->h_counts);
  if (C->h_ids) cudaFreeHost(C->h_ids);
  if (C->h_logprob) cudaFreeHost(C->h_logprob);
  if (C->h_mask_stage) cudaFreeHost(C->h_mask_stage);
  if (C->d_masks) cudaFree(C->d_masks);
  if (C->d_mask_stage) cudaFree(C->d_mask_stage);
  if (C->mask_staged) cudaEventDestroy(C->mask_staged);
  for (int k = 0; k < 2; k++) {
    if (C->fork_ev[k]) cudaEventDestroy(C->fork_ev[k]);
    if (C->join_ev[k]) cudaEventDestroy(C->join_ev[k]);
  }
  if (C->sched_graph) cudaGraphExecDestroy(C->sched_graph);
  if (C->host_graph) cudaGraphExecDestroy(C->host_graph);
  if (C->host_graph_begin) cudaGraphExecDestroy(C->host_graph_begin);
  if (C->single_graph) cudaGraphExecDestroy(C->single_graph);
  if (C->split_ev) cudaEventDestroy(C->split_ev);
  for (int k = 1; k < kMaxMicro; k++) {
    for (int j = 0; j < 2; j++) {
      if (C->mb_fork[k][j]) cudaEventDestroy(C->mb_fork[k][j]);
      if (C->mb_join[k][j]) cudaEventDestroy(C->mb_join[k][j]);
    }
    if (C->mb_done[k]) cudaEventDestroy(C->mb_done[k]);
    if (C->mb_side[k]) cudaStreamDestroy(C->mb_side[k]);
    if (C->mb_main[k]) cudaStreamDestroy(C->mb_main[k]);
  }
  if (C->side) cudaStreamDestroy(C->side);
  if (C->stream) cudaStreamDestroy(C->stream);
  delete C;
}

// Grows the matvec API buffers.
void ensure_mv(needle_ctx& C, size_t floats) {
  if (floats <= C.mv_cap) return;
  for (float** p : {&C.d_mv_x, &C.d_mv_xp, &C.d_mv_y})
    if (*p) {
      cudaFree(*p);
      *p = nullptr;
    }
  cuda_check(cudaMalloc(&C.d_mv_x, floats * 4), "cudaMalloc");
  cuda_check(cudaMalloc(&C.d_mv_xp, floats * 4), "cudaMalloc");
  cuda_check(cudaMalloc(&C.d_mv_y, floats * 4), "cudaMalloc");
  C.mv_cap = floats;
}

}  // namespace

// ------------------------------------------------------------------ C-ABI

namespace {

// KV allocation of a slot: the host's record for slots reset through needle_cuda_seq_reset, the
// device's for slots the device scheduler admitted (after a synchronisation).
int slot_kv_alloc(needle_ctx& C, int seq) {
  const SlotHost& h = C.slots[seq];
  if (h.ready) return h.kv_alloc;
  require(C.sched_loaded, NEEDLE_INVALID_CACT, "KV cache was not allocated");
  SeqState st{};
  cuda_check(cudaStreamSynchronize(C.stream), "read_kv");
  cuda_check(cudaMemcpy(&st, C.sv.seq + seq, sizeof(st), cudaMemcpyDeviceToHost), "read_kv");
  require(st.kv_alloc > 0, NEEDLE_INVALID_CACT, "KV cache was not allocated");
  return st.kv_alloc;
}

// Checks one item's allowed list against the vocabulary (selectToken, runtime.ts:880-899), or its
// mask slot against the pool.
void check_allowed(const needle_ctx& C, const needle_step_item& it, const uint32_t* allowed_ids,
                   size_t allowed_total, int V) {
  if (it.allowed_count == NEEDLE_ALLOWED_MASK) {
    require(C.d_masks != nullptr && it.allowed_offset < uint32_t(C.mask_capacity), NEEDLE_INVALID_CACT,
            "allowed mask slot out of range");
    require(C.mask_count[it.allowed_offset] > 0, NEEDLE_INVALID_CACT, "Allowed token set is empty");
    return;
  }
  require(it.allowed_count >= -1, NEEDLE_INVALID_CACT, "allowed_count must be -1, NEEDLE_ALLOWED_MASK or a count");
  if (it.allowed_count < 0) return;
  require(it.allowed_count > 0, NEEDLE_INVALID_CACT, "Allowed token set is empty");
  require(allowed_ids != nullptr && uint64_t(it.allowed_offset) + uint64_t(it.allowed_count) <= allowed_total,
          NEEDLE_INVALID_CACT, "allowed ids out of range");
  const uint32_t* ids = allowed_ids + it.allowed_offset;
  for (int32_t k = 0; k < it.allowed_count; k++)
    if (ids[k] >= uint32_t(V)) fail(NEEDLE_INVALID_CACT, "Token " + std::to_string(ids[k]) + " is outside logits");
}

// Validates the items of a step (allowed lists too when `allowed` is set); returns the number that
// select.
// A slot's items in one step are one item, or a prompt chunk: consecutive items with given tokens,
// none selecting (positions p, p + 1, ...; the slot advances past all of them).  Returns the number
// of selecting items; *chunks is set when the step holds a chunk.
int check_items(needle_ctx& C, const needle_step_item* items, int32_t n, bool allowed, const uint32_t* allowed_ids,
                size_t allowed_total, bool have_selected, bool* chunks = nullptr) {
  require(n >= 0 && n <= C.step_capacity, NEEDLE_BACKEND_UNAVAILABLE, "item count out of range");
  require(n == 0 || items != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "null items");
  std::vector<char> seen(C.opts.max_seqs, 0);
  const int V = C.mv.vocab;
  int n_sel = 0;
  bool any_chunk = false;
  for (int i = 0; i < n; i++) {
    const needle_step_item& it = items[i];
    require(it.seq >= 0 && it.seq < C.opts.max_seqs, NEEDLE_BACKEND_UNAVAILABLE, "sequence slot out of range");
    const bool cont = i > 0 && items[i - 1].seq == it.seq;
    require(cont || !seen[it.seq], NEEDLE_BACKEND_UNAVAILABLE,
            "a slot appears twice in one step (a prompt chunk's items must be consecutive)");
    seen[it.seq] = 1;
    const SlotHost& h = C.slots[it.seq];
    require(h.ready, NEEDLE_INVALID_CACT, "Call runtime.reset() before decoding");
    if (cont || (i + 1 < n && items[i + 1].seq == it.seq)) {  // an item of a prompt chunk
      any_chunk = true;
      require(!it.select && it.token >= 0, NEEDLE_INVALID_CACT,
              "a prompt chunk's items carry their tokens and do not select");
      if (!cont) {
        int k = 1;
        while (i + k < n && items[i + k].seq == it.seq) k++;
        if (h.position + k > h.max_len)
          fail(NEEDLE_CONTEXT_OVERFLOW, "Position " + std::to_string(h.position + k) + " exceeds runtime limit " +
                                            std::to_string(h.max_len));
        require(C.mv.kv_window == 0 || h.position + k <= h.sink + C.mv.kv_window, NEEDLE_INVALID_CACT,
                "a prompt chunk may not reach past the KV window");
        require(C.collecting == 0, NEEDLE_INVALID_CACT,
                "prompt chunks are not taken while a slot collects confidence");
      }
    }
    // messages are built only on failure: this loop runs for every item of every step
    if (h.position >= h.max_len)
      fail(NEEDLE_CONTEXT_OVERFLOW,
           "Position " + std::to_string(h.position) + " reached runtime limit " + std::to_string(h.max_len));
    if (!(it.token == NEEDLE_TOKEN_PENDING || (it.token >= 0 && it.token < V)))
      fail(NEEDLE_INVALID_CACT, "Token " + std::to_string(it.token) + " is outside the vocabulary");
    if (it.select) {
      require(have_selected, NEEDLE_BACKEND_UNAVAILABLE, "selection requested without output");
      if (allowed) check_allowed(C, it, allowed_ids, allowed_total, V);
      n_sel++;
    }
  }
  if (chunks) *chunks = any_chunk;
  return n_sel;
}

// The device items in internal order (items that need logits first) into `dst`; order[i] is item
// i's row.
void stage_items(needle_ctx& C, const needle_step_item* items, int32_t n, int n_sel, bool all_logits,
                 std::vector<int>& order, DevItem* dst) {
  int pos_sel = 0, pos_rest = all_logits ? 0 : n_sel;
  order.resize(n);
  int run_start = 0, run_len = 1;  // the prompt chunk (or single item) item i belongs to
  for (int i = 0; i < n; i++) {
    const needle_step_item& it = items[i];
    if (i == 0 || items[i - 1].seq != it.seq) {
      run_start = i;
      run_len = 1;
      while (i + run_len < n && items[i + run_len].seq == it.seq) run_len++;
    }
    const bool first = all_logits || it.select;
    const int k = all_logits ? pos_sel++ : (first ? pos_sel++ : pos_rest++);  // chunks stay in order
    order[i] = k;
    DevItem d{};
    d.slot = it.seq;
    d.token = it.token;
    d.select = it.select ? 1 : 0;
    d.allowed_count = it.select ? it.allowed_count : -1;
    d.allowed_offset = it.allowed_offset;
    d.position = C.slots[it.seq].position + (i - run_start);
    d.out_index = i;
    if (run_len > 1) {
      d.chunk_index = i - run_start;
      d.chunk_len = run_len;
    }
    dst[k] = d;
  }
}

void upload_allowed(needle_ctx& C, const uint32_t* allowed_ids, size_t allowed_total) {
  if (allowed_total == 0 || !allowed_ids) return;
  if (allowed_total > C.allowed_cap) {
    drop_host_graph(C);
    uint32_t* p = nullptr;
    cuda_check(cudaMalloc(&p, allowed_total * 4), "cudaMalloc");
    C.allocs.push_back(p);
    C.d_allowed = p;
    C.allowed_cap = allowed_total;
    C.stv.allowed = p;
  }
  cuda_check(cudaMemcpyAsync(C.d_allowed, allowed_ids, allowed_total * 4, cudaMemcpyHostToDevice, C.stream),
             "allowed upload");
}

void upload_items(needle_ctx& C, const DevItem* src, int n, int rows) {
  C.h_counts[0] = n;
  C.h_counts[1] = rows;
  C.timed(P_COPY, [&] {
    cudaError_t e = cudaMemcpyAsync(C.stv.items, src, size_t(n) * sizeof(DevItem), cudaMemcpyHostToDevice, C.stream);
    if (e != cudaSuccess) return e;
    return cudaMemcpyAsync(C.d_counts, C.h_counts, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, C.stream);
  });
}

// Fails the call (BACKEND_UNAVAILABLE) when a bounded wait of a fast-numerics kernel ran out during
// the work just synchronised (its outputs are NaN); the wait status is cleared.
void check_device_waits(needle_ctx& C) {
  if (!C.fast) return;
  uint32_t* w = wait_status_words(C.device);
  if (!w) return;
  bool any = false;
  for (int k = 0; k < kWaitKinds; k++) {
    volatile uint32_t* v = w + k;
    if (*v) {
      any = true;
      *v = 0;
    }
  }
  require(!any, NEEDLE_BACKEND_UNAVAILABLE, "a bounded device wait ran out in a fast-numerics kernel (outputs are NaN)");
}

// Reads the selections (and logits) back, waits for the step and advances the slots.
void complete_step(needle_ctx& C, const needle_step_item* items, int32_t n, int rows, const std::vector<int>& order,
                   needle_selected* out_selected, float* out_logits) {
  const int V = C.mv.vocab;
  if (rows > 0) {
    cuda_check(cudaMemcpyAsync(C.h_ids, C.stv.out_id, size_t(rows) * 4, cudaMemcpyDeviceToHost, C.stream), "readback");
    cuda_check(cudaMemcpyAsync(C.h_logprob, C.stv.out_logprob, size_t(rows) * 8, cudaMemcpyDeviceToHost, C.stream),
               "readback");
  }
  if (out_logits) {
    for (int i = 0; i < n; i++)
      cuda_check(cudaMemcpyAsync(out_logits + size_t(i) * V, C.stv.logits + size_t(order[i]) * V, size_t(V) * 4,
                                 cudaMemcpyDeviceToHost, C.stream),
                 "logits readback");
  }
  cuda_check(cudaStreamSynchronize(C.stream), "step");
  check_device_waits(C);
  for (int i = 0; i < n; i++) {
    C.slots[items[i].seq].position++;
    if (items[i].select) {
      out_selected[i].id = C.h_ids[order[i]];
      out_selected[i].reserved = 0;
      out_selected[i].log_probability = C.h_logprob[order[i]];
    }
  }
}


// Second half of a begun step (needle_cuda_step_end, needle_cuda_resident_finish / _select): the
// same items with their allowed lists (a select may be cleared), selection, readback of the
// selections and of the logits rows when out_logits is given, and the slots advanced.  On any
// failure the begun work is drained and the step is dropped: the slots keep their positions, so
// their next step rewrites the K/V this one appended.
void end_step(needle_ctx& C, const needle_step_item* items, int32_t n, const uint32_t* allowed_ids,
              size_t allowed_total, needle_selected* out_selected, float* out_logits) {
  auto& P = C.pending;
  require(P.active, NEEDLE_BACKEND_UNAVAILABLE, "needle_cuda_step_end without needle_cuda_step_begin");
  cuda_check(cudaSetDevice(C.device), "cudaSetDevice");
  struct Drop {
    needle_ctx& C;
    bool armed = true;
    ~Drop() {
      if (!armed) return;
      cudaStreamSynchronize(C.stream);
      C.pending.active = false;
      C.pending.resident = false;
    }
  } drop{C};
  require(n == P.n && items != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "step_end items differ from step_begin's");
  const int V = C.mv.vocab;
  for (int i = 0; i < n; i++) {
    const needle_step_item& it = items[i];
    const needle_step_item& b = P.items[i];
    require(it.seq == b.seq && it.token == b.token && (!it.select || b.select), NEEDLE_BACKEND_UNAVAILABLE,
            "step_end items differ from step_begin's (only select may be cleared)");
    if (it.select) {
      require(out_selected != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "selection requested without output");
      check_allowed(C, it, allowed_ids, allowed_total, V);
    }
  }
  // the allowed fields (and cleared selects) go in with a second copy of the items, ordered after
  // the layers that read the first
  for (int i = 0; i < n; i++) {
    DevItem d = C.h_items[P.order[i]];
    d.select = items[i].select ? 1 : 0;
    d.allowed_count = items[i].select ? items[i].allowed_count : -1;
    d.allowed_offset = items[i].allowed_offset;
    C.h_items_end[P.order[i]] = d;
  }
  upload_allowed(C, allowed_ids, allowed_total);
  if (P.mb > 0) {  // micro-batched: every micro-batch's rows, then its selection
    C.timed(P_COPY, [&] {
      return cudaMemcpyAsync(C.stv.items, C.h_items_end, size_t(P.mb) * P.cap * sizeof(DevItem),
                             cudaMemcpyHostToDevice, C.stream);
    });
    for (int k = 0; k < P.mb; k++) {
      const StepView v = half_view(C, k * P.cap, C.d_counts + 2 + 2 * k, C.d_counts + 3 + 2 * k);
      C.timed(P_FINISH, [&] { return launch_finish(C.mv, C.sv, v, P.cap, nullptr, C.stream); }, C.stream);
    }
    complete_step(C, items, n, P.mb * P.cap, P.order, out_selected, out_logits);
  } else {
    C.timed(P_COPY, [&] {
      return cudaMemcpyAsync(C.stv.items, C.h_items_end, size_t(n) * sizeof(DevItem), cudaMemcpyHostToDevice,
                             C.stream);
    });
    C.timed(P_FINISH, [&] { return launch_finish(C.mv, C.sv, C.stv, n, nullptr, C.stream); }, C.stream);
    complete_step(C, items, n, P.n_sel, P.order, out_selected, out_logits);
  }
  drop.armed = false;
  P.active = false;
  P.resident = false;
}

}  // namespace

extern "C" {

const char* needle_cuda_last_error(void) { return g_error.c_str(); }

int needle_cuda_default_opts(needle_opts* o) {
  return guarded([&] {
    require(o != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "null options");
    std::memset(o, 0, sizeof(*o));
    o->struct_size = sizeof(needle_opts);
    o->device = 0;
    o->max_seqs = 1;
    o->max_len = 2048;
    o->max_sink = 160;
    o->kv_mode = NEEDLE_KV_INT8;
    o->numerics = NEEDLE_NUMERICS_EXACT;
  });
}

int needle_cuda_open(const uint8_t* cact, size_t n, const needle_opts* opts, needle_ctx** out) {
  needle_ctx* C = nullptr;
  const int rc = guarded([&] {
    require(out != nullptr && cact != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "null argument");
    *out = nullptr;
    C = new needle_ctx();
    if (opts) {
      require(opts->struct_size == sizeof(needle_opts), NEEDLE_BACKEND_UNAVAILABLE, "needle_opts size mismatch");
      C->opts = *opts;
    } else {
      needle_cuda_default_opts(&C->opts);
    }
    const needle_opts& o = C->opts;
    require(o.kv_mode == NEEDLE_KV_INT8 || o.kv_mode == NEEDLE_KV_FLOAT32, NEEDLE_BACKEND_UNAVAILABLE,
            "kv_mode must be NEEDLE_KV_INT8 or NEEDLE_KV_FLOAT32");
    require(o.numerics == NEEDLE_NUMERICS_EXACT || o.numerics == NEEDLE_NUMERICS_FAST ||
                o.numerics == NEEDLE_NUMERICS_FAST_ATTENTION,
            NEEDLE_BACKEND_UNAVAILABLE, "unknown numerics mode");
    require(o.numerics == NEEDLE_NUMERICS_EXACT || o.kv_mode == NEEDLE_KV_INT8, NEEDLE_BACKEND_UNAVAILABLE,
            "fast numerics runs on the int8 KV cache");
    require(o.max_seqs >= 1 && o.max_seqs <= 65536, NEEDLE_BACKEND_UNAVAILABLE, "max_seqs out of range");
    require(o.micro_batches >= 0 && o.micro_batches <= kMaxMicro, NEEDLE_BACKEND_UNAVAILABLE,
            "micro_batches out of range (0..8)");
    require(o.sched_chunk >= 0 && o.sched_chunk <= kPrefillChunk, NEEDLE_BACKEND_UNAVAILABLE,
            "sched_chunk out of range (0..64)");
    require(o.sched_items == 0 || (o.sched_items >= o.max_seqs && o.sched_items <= 8 * o.max_seqs + kPrefillChunk),
            NEEDLE_BACKEND_UNAVAILABLE, "sched_items out of range (max_seqs .. 8 x max_seqs + 64)");
    require(o.max_sink >= 0 && o.max_len >= 1, NEEDLE_BACKEND_UNAVAILABLE, "max_len / max_sink out of range");
    int devices = 0;
    cuda_check(cudaGetDeviceCount(&devices), "cudaGetDeviceCount");
    require(o.device >= 0 && o.device < devices, NEEDLE_BACKEND_UNAVAILABLE,
            "CUDA device " + std::to_string(o.device) + " is not available");
    C->device = o.device;
    cuda_check(cudaSetDevice(C->device), "cudaSetDevice");
    cudaDeviceProp prop;
    cuda_check(cudaGetDeviceProperties(&prop, C->device), "cudaGetDeviceProperties");
    require(prop.major == 10 && prop.minor == 0, NEEDLE_BACKEND_UNAVAILABLE,
            std::string("libneedle_cuda is built for sm_100a (B200); device is ") + prop.name);
    C->bytes.assign(cact, cact + n);
    parse_archive(C->bytes.data(), C->bytes.size(), C->A);
    C->roles = assign_roles(C->A);
    check_geometry(*C);
    require(int64_t(o.max_len) <= int64_t(C->A.hdr[11]), NEEDLE_CONTEXT_OVERFLOW,
            "max_len exceeds the model's maximum sequence length");
    cuda_check(cudaStreamCreateWithFlags(&C->stream, cudaStreamNonBlocking), "cudaStreamCreate");
    cuda_check(cudaStreamCreateWithFlags(&C->side, cudaStreamNonBlocking), "cudaStreamCreate");
    for (int k = 0; k < 2; k++) {
      cuda_check(cudaEventCreateWithFlags(&C->fork_ev[k], cudaEventDisableTiming), "cudaEventCreate");
      cuda_check(cudaEventCreateWithFlags(&C->join_ev[k], cudaEventDisableTiming), "cudaEventCreate");
    }
    for (int k = 1; k < kMaxMicro; k++) {
      cuda_check(cudaStreamCreateWithFlags(&C->mb_main[k], cudaStreamNonBlocking), "cudaStreamCreate");
      cuda_check(cudaStreamCreateWithFlags(&C->mb_side[k], cudaStreamNonBlocking), "cudaStreamCreate");
      for (int j = 0; j < 2; j++) {
        cuda_check(cudaEventCreateWithFlags(&C->mb_fork[k][j], cudaEventDisableTiming), "cudaEventCreate");
        cuda_check(cudaEventCreateWithFlags(&C->mb_join[k][j], cudaEventDisableTiming), "cudaEventCreate");
      }
      cuda_check(cudaEventCreateWithFlags(&C->mb_done[k], cudaEventDisableTiming), "cudaEventCreate");
    }
    cuda_check(cudaEventCreateWithFlags(&C->split_ev, cudaEventDisableTiming), "cudaEventCreate");
    if (o.micro_batches > 0) C->micro = std::min(kMaxMicro, int(o.micro_batches));
    if (const char* v = std::getenv("NEEDLE_NVTX")) C->nvtx = v[0] != 0 && v[0] != '0';
    if (o.sched_chunk >= 2) {
      C->sched_chunk = o.sched_chunk;
      C->sched_items = o.sched_items > 0 ? o.sched_items : 2 * o.max_seqs;
    }
    C->fast = o.numerics == NEEDLE_NUMERICS_FAST || o.numerics == NEEDLE_NUMERICS_FAST_ATTENTION;
    C->fast_attention = o.numerics == NEEDLE_NUMERICS_FAST_ATTENTION;
    cuda_check(cudaDeviceGetAttribute(&C->sms, cudaDevAttrMultiProcessorCount, C->device), "device attribute");
    build_model(*C);
    build_state(*C);
    cuda_check(cudaDeviceSynchronize(), "upload");
    *out = C;
  });
  if (rc != NEEDLE_OK && C) destroy(C);
  return rc;
}

int needle_cuda_close(needle_ctx* ctx) {
  return guarded([&] {
    require(ctx != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "null needle context");
    destroy(ctx);
  });
}

int needle_cuda_geometry(const needle_ctx* ctx, needle_geometry* g) {
  return guarded([&] {
    require(ctx && g, NEEDLE_BACKEND_UNAVAILABLE, "null argument");
    const uint32_t* h = ctx->A.hdr;
    std::memset(g, 0, sizeof(*g));
    g->kv_window = int32_t(h[3]);
    g->kv_bits = int32_t(h[4]);
    g->vocabulary_size = int32_t(h[5]);
    g->model_dimension = int32_t(h[6]);
    g->heads = int32_t(h[7]);
    g->kv_heads = int32_t(h[8]);
    g->layers = int32_t(h[9]);
    g->head_dimension = int32_t(h[10]);
    g->maximum_sequence_length = int32_t(h[11]);
    g->hadamard_dimension = int32_t(h[12]);
    g->mhc_lanes = int32_t(h[13]);
    g->engram_slots = int32_t(h[14]);
    g->engram_sub_dimension = int32_t(h[15]);
    g->engram_tables = int32_t(h[16]);
    g->engram_taps = int32_t(h[17]);
    g->engram_dilation = int32_t(h[18]);
    g->engram_order_count = int32_t(h[19]);
    for (int i = 0; i < 4; i++) g->engram_orders[i] = int32_t(h[20 + i]);
    g->engram_site_count = int32_t(h[24]);
    for (int i = 0; i < 4; i++) g->engram_sites[i] = int32_t(h[25 + i]);
    g->rope_theta = ctx->A.rope_theta;
    g->num_tensors = int32_t(ctx->A.rec.size());
    g->kv_capacity = ctx->sv.capacity;
  });
}

int needle_cuda_seq_reset(needle_ctx* ctx, int32_t seq, int32_t maximum_length, int32_t sink_length) {
  return needle_cuda_seq_reset_ex(ctx, seq, maximum_length, sink_length, 0);
}

int needle_cuda_seq_reset_ex(needle_ctx* ctx, int32_t seq, int32_t maximum_length, int32_t sink_length,
                             int32_t collect_confidence) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    require(seq >= 0 && seq < C.opts.max_seqs, NEEDLE_BACKEND_UNAVAILABLE, "sequence slot out of range");
    require(maximum_length > 0 && maximum_length <= C.mv.max_seq, NEEDLE_CONTEXT_OVERFLOW,
            "Runtime length " + std::to_string(maximum_length) + " is outside model limit " +
                std::to_string(C.mv.max_seq));
    require(maximum_length <= C.opts.max_len, NEEDLE_CONTEXT_OVERFLOW,
            "Runtime length exceeds the context's max_len");
    const int32_t sink = std::min(std::max(sink_length, 0), maximum_length);
    const int window = C.mv.kv_window;
    const int32_t kv_alloc = window > 0 ? std::min(maximum_length, sink + window) : maximum_length;
    require(kv_alloc <= C.sv.capacity, NEEDLE_BACKEND_UNAVAILABLE,
            "sink + window exceeds the context's KV capacity (raise max_sink / max_len)");
    const bool collect = collect_confidence != 0 && C.mv.probe_count > 0;
    // the slot's state goes in from pinned staging, ordered before every later step on the stream
    // (no wait here: a host loop resetting slots between steps keeps the GPU busy).  Host steps
    // end synchronised; scheduled steps may still be queued, and one of them could read this slot
    // between an earlier reset's copy and this one, so their work is drained first.
    if (C.sched_inflight) {
      cuda_check(cudaStreamSynchronize(C.stream), "reset");
      C.sched_inflight = false;
    }
    SeqState& st = C.h_seq_stage[seq];
    st = SeqState{};
    st.position = 0;
    st.sink = sink;
    st.max_len = maximum_length;
    st.kv_alloc = kv_alloc;
    st.collect = collect ? 1 : 0;
    cuda_check(cudaMemcpyAsync(C.sv.seq + seq, &st, sizeof(st), cudaMemcpyHostToDevice, C.stream), "reset");
    if (collect) cuda_check(launch_pool_reset(C.mv, C.sv, seq, C.stream), "pool reset");
    SlotHost& h = C.slots[seq];
    C.collecting += int(collect) - int(h.collect);
    h.collect = collect;
    h.ready = true;
    h.max_len = maximum_length;
    h.sink = sink;
    h.kv_alloc = kv_alloc;
    h.position = 0;
  });
}

int needle_cuda_seq_position(const needle_ctx* ctx, int32_t seq, int32_t* position) {
  return guarded([&] {
    require(ctx && position, NEEDLE_BACKEND_UNAVAILABLE, "null argument");
    require(seq >= 0 && seq < ctx->opts.max_seqs, NEEDLE_BACKEND_UNAVAILABLE, "sequence slot out of range");
    *position = ctx->slots[seq].position;
  });
}

int needle_cuda_step(needle_ctx* ctx, const needle_step_item* items, int32_t n, const uint32_t* allowed_ids,
                     size_t allowed_total, needle_selected* out_selected, float* out_logits) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    bool chunks = false;
    const int n_sel = check_items(C, items, n, true, allowed_ids, allowed_total, out_selected != nullptr, &chunks);
    if (n == 0) return;
    const bool all_logits = out_logits != nullptr;
    std::vector<int> order;
    // Many items: micro-batches on their own stream pairs, the step replayed as a CUDA graph after
    // its first (eager) run, as device-scheduled steps are.
    int M = 0, cap = 0;
    if (host_mb_shape(C, n, all_logits, &M, &cap) && stage_items_mb(C, items, n, M, cap, order, C.h_items)) {
      upload_allowed(C, allowed_ids, allowed_total);
      if (C.host_m != M || C.host_cap != cap) {
        drop_host_graph(C);
        C.host_m = M;
        C.host_cap = cap;
      }
      upload_items_mb(C, C.h_items, M, cap);
      run_host_mb(C, M, cap, true, C.host_graph, C.host_graph_launches);
      complete_step(C, items, n, M * cap, order, out_selected, nullptr);
      return;
    }
    stage_items(C, items, n, n_sel, all_logits, order, C.h_items);
    upload_allowed(C, allowed_ids, allowed_total);
    const int rows = all_logits ? n : n_sel;
    upload_items(C, C.h_items, n, rows);
    if (n == 1 && !all_logits && C.collecting == 0 && !C.profiling) {
      run_single(C);
      complete_step(C, items, n, rows, order, out_selected, out_logits);
      return;
    }
    StepView v = C.stv;
    v.chunk = chunks ? 1 : 0;
    enqueue_step(C, v, n, n_sel > 0 || all_logits, nullptr, lane_a(C));
    complete_step(C, items, n, rows, order, out_selected, out_logits);
  });
}

int needle_cuda_step_begin(needle_ctx* ctx, const needle_step_item* items, int32_t n) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    bool chunks = false;
    const int n_sel = check_items(C, items, n, false, nullptr, 0, true, &chunks);
    require(n > 0, NEEDLE_BACKEND_UNAVAILABLE, "a split step needs at least one item");
    auto& P = C.pending;
    int M = 0, cap = 0;
    P.mb = P.cap = 0;
    if (host_mb_shape(C, n, false, &M, &cap) && stage_items_mb(C, items, n, M, cap, P.order, C.h_items)) {
      if (C.host_m != M || C.host_cap != cap) {
        drop_host_graph(C);
        C.host_m = M;
        C.host_cap = cap;
      }
      upload_items_mb(C, C.h_items, M, cap);
      run_host_mb(C, M, cap, false, C.host_graph_begin, C.host_begin_launches);
      P.mb = M;
      P.cap = cap;
    } else {
      stage_items(C, items, n, n_sel, false, P.order, C.h_items);
      upload_items(C, C.h_items, n, n_sel);
      StepView v = C.stv;
      v.chunk = chunks ? 1 : 0;
      enqueue_step(C, v, n, n_sel > 0, nullptr, lane_a(C), /*finish=*/false);
    }
    P.items.assign(items, items + n);
    P.n = n;
    P.n_sel = n_sel;
    P.active = true;
  });
}

static_assert(kAllowedMask == NEEDLE_ALLOWED_MASK, "device and C-ABI mask markers differ");

int needle_cuda_mask_pool(needle_ctx* ctx, int32_t capacity) {
  return guarded([&] {
    require(ctx != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "null context");
    needle_ctx& C = *ctx;
    require(capacity > 0 && capacity <= (1 << 20), NEEDLE_BACKEND_UNAVAILABLE, "mask pool capacity out of range");
    require(!C.pending.active, NEEDLE_BACKEND_UNAVAILABLE, "a begun step is pending");
    cuda_check(cudaSetDevice(C.device), "cudaSetDevice");
    cuda_check(cudaStreamSynchronize(C.stream), "cudaStreamSynchronize");
    drop_host_graph(C);
    if (C.d_masks) cudaFree(C.d_masks);
    if (C.d_mask_stage) cudaFree(C.d_mask_stage);
    if (C.h_mask_stage) cudaFreeHost(C.h_mask_stage);
    C.d_masks = C.d_mask_stage = C.h_mask_stage = nullptr;
    C.mask_capacity = 0;
    const int words = (C.mv.vocab + 31) / 32;
    const size_t stage = size_t(C.opts.max_seqs) * (1 + words);
    cuda_check(cudaMalloc(&C.d_masks, size_t(capacity) * words * 4), "cudaMalloc");
    cuda_check(cudaMemsetAsync(C.d_masks, 0, size_t(capacity) * words * 4, C.stream), "cudaMemsetAsync");
    cuda_check(cudaMalloc(&C.d_mask_stage, stage * 4), "cudaMalloc");
    cuda_check(cudaHostAlloc(&C.h_mask_stage, stage * 4, cudaHostAllocDefault), "cudaHostAlloc");
    if (!C.mask_staged) cuda_check(cudaEventCreateWithFlags(&C.mask_staged, cudaEventDisableTiming), "cudaEventCreate");
    cuda_check(cudaEventRecord(C.mask_staged, C.stream), "cudaEventRecord");
    C.mask_capacity = capacity;
    C.mask_words = words;
    C.mask_count.assign(capacity, 0);
    C.stv.masks = C.d_masks;
    C.stv.mask_words = words;
  });
}

int needle_cuda_masks_put(needle_ctx* ctx, const int32_t* slots, int32_t n, const uint32_t* table) {
  return guarded([&] {
    require(ctx != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "null context");
    needle_ctx& C = *ctx;
    require(C.d_masks != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "no mask pool (needle_cuda_mask_pool)");
    require(n >= 0 && (n == 0 || (slots != nullptr && table != nullptr)), NEEDLE_BACKEND_UNAVAILABLE,
            "null argument");
    cuda_check(cudaSetDevice(C.device), "cudaSetDevice");
    const int words = C.mask_words, V = C.mv.vocab;
    const int per = C.opts.max_seqs;
    const uint32_t tail = (V & 31) ? ~((1u << (V & 31)) - 1u) : 0u;  // bits of ids >= V in the last word
    std::vector<int32_t> set(per);
    for (int32_t base = 0; base < n; base += per) {
      const int m = std::min<int32_t>(per, n - base);
      for (int k = 0; k < m; k++) {
        const int32_t s = slots[base + k];
        require(s >= 0 && s < C.mask_capacity, NEEDLE_BACKEND_UNAVAILABLE, "mask slot out of range");
        const uint32_t* w = table + size_t(s) * words;
        require(!(w[words - 1] & tail), NEEDLE_INVALID_CACT, "a mask sets an id outside the vocabulary");
        int c = 0;
        for (int j = 0; j < words; j++) c += __builtin_popcount(w[j]);
        set[k] = c;
      }
      // the staging buffer is free once the previous put's copy has run
      cuda_check(cudaEventSynchronize(C.mask_staged), "cudaEventSynchronize");
      for (int k = 0; k < m; k++) {
        const int32_t s = slots[base + k];
        C.h_mask_stage[k] = uint32_t(s);
        memcpy(C.h_mask_stage + per + size_t(k) * words, table + size_t(s) * words, size_t(words) * 4);
      }
      C.timed(P_COPY, [&] {
        cudaError_t e = cudaMemcpyAsync(C.d_mask_stage, C.h_mask_stage, size_t(m) * 4, cudaMemcpyHostToDevice,
                                        C.stream);
        if (e != cudaSuccess) return e;
        return cudaMemcpyAsync(C.d_mask_stage + per, C.h_mask_stage + per, size_t(m) * words * 4,
                               cudaMemcpyHostToDevice, C.stream);
      });
      cuda_check(cudaEventRecord(C.mask_staged, C.stream), "cudaEventRecord");
      C.timed(P_FINISH, [&] {
        return launch_mask_scatter(C.d_mask_stage + per, reinterpret_cast<const int32_t*>(C.d_mask_stage), m, words,
                                   C.d_masks, C.stream);
      });
      for (int k = 0; k < m; k++) C.mask_count[slots[base + k]] = set[k];
    }
  });
}

int needle_cuda_step_end(needle_ctx* ctx, const needle_step_item* items, int32_t n, const uint32_t* allowed_ids,
                         size_t allowed_total, needle_selected* out_selected) {
  return guarded([&] {
    require(ctx != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "null needle context");
    require(!ctx->pending.resident, NEEDLE_BACKEND_UNAVAILABLE,
            "a resident token is in flight; it ends with needle_cuda_resident_finish or _select");
    end_step(*ctx, items, n, allowed_ids, allowed_total, out_selected, nullptr);
  });
}

int needle_cuda_resident_forward(needle_ctx* ctx, int32_t seq, int32_t position, const float* lanes,
                                 const uint32_t* engram_indices, const uint32_t* engram_valid, int32_t engram_tables,
                                 int32_t engram_position) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    const ModelView& m = C.mv;
    require(seq >= 0 && seq < C.opts.max_seqs, NEEDLE_BACKEND_UNAVAILABLE, "sequence slot out of range");
    const SlotHost& h = C.slots[seq];
    require(h.ready, NEEDLE_INVALID_CACT, "Call runtime.reset() before decoding");
    if (h.position >= h.max_len)
      fail(NEEDLE_CONTEXT_OVERFLOW,
           "Position " + std::to_string(h.position) + " reached runtime limit " + std::to_string(h.max_len));
    require(position == h.position, NEEDLE_BACKEND_UNAVAILABLE,
            "resident token position " + std::to_string(position) + " differs from the session's " +
                std::to_string(h.position));
    require(lanes != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "beginResidentToken lanes are missing");
    int32_t flags = kItemLanes;
    if (m.n_sites > 0) {
      require(engram_indices != nullptr && engram_valid != nullptr && engram_tables == m.n_tables,
              NEEDLE_BACKEND_UNAVAILABLE, "prepareResidentEngrams lookup is missing or has the wrong table count");
      require(engram_position == position, NEEDLE_BACKEND_UNAVAILABLE,
              "engram position " + std::to_string(engram_position) + " differs from the token position");
      for (int t = 0; t < m.n_tables; t++) {
        require(engram_indices[t] < uint32_t(m.engram_slots), NEEDLE_INVALID_CACT, "engram index outside its table");
        C.h_engram[t] = engram_indices[t];
        C.h_engram[kMaxTables + t] = engram_valid[t] ? 1u : 0u;
      }
      flags |= kItemEngrams;
    }
    std::memcpy(C.h_lanes, lanes, kLaneWidth * sizeof(float));
    auto& P = C.pending;
    const needle_step_item item{seq, 0, 1, -1, 0};
    stage_items(C, &item, 1, 1, false, P.order, C.h_items);
    C.h_items[0].flags = flags;
    C.timed(P_COPY, [&] {
      cudaError_t e = cudaMemcpyAsync(C.stv.lanes, C.h_lanes, kLaneWidth * sizeof(float), cudaMemcpyHostToDevice,
                                      C.stream);
      if (e != cudaSuccess || !(flags & kItemEngrams)) return e;
      return cudaMemcpyAsync(C.d_engram_in, C.h_engram, 2 * kMaxTables * sizeof(uint32_t), cudaMemcpyHostToDevice,
                             C.stream);
    });
    upload_items(C, C.h_items, 1, 1);
    enqueue_step(C, C.stv, 1, true, nullptr, lane_a(C), /*finish=*/false);
    P.items.assign(&item, &item + 1);
    P.n = 1;
    P.n_sel = 1;
    P.mb = P.cap = 0;
    P.active = true;
    P.resident = true;
  });
}

namespace {
// The item a resident token began with, for its end (finish or select).
needle_ctx& resident_pending(needle_ctx* ctx, int32_t seq) {
  require(ctx != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "null needle context");
  require(ctx->pending.active && ctx->pending.resident && ctx->pending.items[0].seq == seq,
          NEEDLE_BACKEND_UNAVAILABLE, "no resident token of this slot is in flight");
  return *ctx;
}
}  // namespace

int needle_cuda_resident_finish(needle_ctx* ctx, int32_t seq, float* logits) {
  return guarded([&] {
    needle_ctx& C = resident_pending(ctx, seq);
    needle_step_item item = C.pending.items[0];
    item.select = 0;
    end_step(C, &item, 1, nullptr, 0, nullptr, logits);
  });
}

int needle_cuda_resident_select(needle_ctx* ctx, int32_t seq, const uint32_t* allowed_ids, int32_t n_allowed,
                                needle_selected* out_selected) {
  return guarded([&] {
    needle_ctx& C = resident_pending(ctx, seq);
    require(out_selected != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "selection requested without output");
    needle_step_item item = C.pending.items[0];
    item.allowed_count = n_allowed < 0 ? -1 : n_allowed;
    item.allowed_offset = 0;
    end_step(C, &item, 1, allowed_ids, n_allowed < 0 ? 0 : size_t(n_allowed), out_selected, nullptr);
  });
}

int needle_cuda_prefill(needle_ctx* ctx, int32_t seq, const int32_t* ids, int32_t n, float* out_logits) {
  return guarded([&] {
    require(ids != nullptr && n > 0, NEEDLE_INVALID_CACT, "Cannot prefill an empty token sequence");
    needle_ctx& C = *ctx_of(ctx);
    require(seq >= 0 && seq < C.opts.max_seqs, NEEDLE_BACKEND_UNAVAILABLE, "sequence slot out of range");
    const SlotHost& h = C.slots[seq];
    require(h.ready, NEEDLE_INVALID_CACT, "Call runtime.reset() before decoding");
    require(h.max_len - h.position >= n, NEEDLE_CONTEXT_OVERFLOW,
            "Prompt has " + std::to_string(n) + " tokens but runtime holds " + std::to_string(h.max_len));
    const int V = C.mv.vocab;
    for (int32_t i = 0; i < n; i++)
      if (ids[i] < 0 || ids[i] >= V) fail(NEEDLE_INVALID_CACT, "Token " + std::to_string(ids[i]) + " is outside the vocabulary");
    // Chunks of up to kPrefillChunk tokens, one item per token (the last token, when its logits
    // are wanted, is a step of its own).  A slot that feeds a confidence pool goes token by token
    // (the pool is updated in position order), and no chunk reaches past the KV ring: one of its
    // items would overwrite the slot of a position an earlier item still attends to.
    int32_t i = 0;
    const int32_t chunked_end = n - (out_logits ? 1 : 0);
    while (!C.slots[seq].collect && i < chunked_end) {
      SlotHost& hs = C.slots[seq];
      int k = std::min(kPrefillChunk, chunked_end - i);
      if (C.mv.kv_window > 0) k = std::min(k, hs.sink + C.mv.kv_window - hs.position);
      if (k < 2) break;
      for (int b = 0; b < k; b++) {
        DevItem d{};
        d.slot = seq;
        d.token = ids[i + b];
        d.select = 0;
        d.allowed_count = -1;
        d.position = hs.position + b;
        d.out_index = b;
        d.chunk_index = b;
        d.chunk_len = k;
        C.h_items[b] = d;
      }
      C.h_counts[0] = k;
      C.h_counts[1] = 0;
      C.timed(P_COPY, [&] {
        cudaError_t e = cudaMemcpyAsync(C.stv.items, C.h_items, size_t(k) * sizeof(DevItem), cudaMemcpyHostToDevice,
                                        C.stream);
        if (e != cudaSuccess) return e;
        return cudaMemcpyAsync(C.d_counts, C.h_counts, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, C.stream);
      });
      StepView cv = C.stv;
      cv.chunk = 1;
      enqueue_step(C, cv, k, false, nullptr, lane_a(C));
      cuda_check(cudaStreamSynchronize(C.stream), "prefill chunk");
      hs.position += k;
      i += k;
    }
    for (; i < n; i++) {
      needle_step_item it{seq, ids[i], 0, -1, 0};
      const bool last = i == n - 1 && out_logits != nullptr;
      const int rc = needle_cuda_step(ctx, &it, 1, nullptr, 0, nullptr, last ? out_logits : nullptr);
      if (rc != NEEDLE_OK) fail(rc, g_error);
    }
  });
}

int needle_cuda_read_kv(const needle_ctx* ctx, int32_t seq, int32_t layer, int8_t* key_codes, int8_t* value_codes,
                        float* key_scales, float* value_scales, int32_t* kv_allocation) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(const_cast<needle_ctx*>(ctx));
    require(seq >= 0 && seq < C.opts.max_seqs, NEEDLE_BACKEND_UNAVAILABLE, "sequence slot out of range");
    require(layer >= 0 && layer < C.mv.layers, NEEDLE_INVALID_CACT, "Layer out of range");
    require(!C.sv.kv_f32, NEEDLE_INVALID_CACT, "Int8 KV cache is not allocated");
    const int kv_alloc = slot_kv_alloc(C, seq);
    if (kv_allocation) *kv_allocation = kv_alloc;
    const int cap = C.sv.capacity;
    for (int head = 0; head < kKvHeads; head++) {
      const size_t base = ((size_t(seq) * C.mv.layers + layer) * kKvHeads + head) * cap;
      if (key_codes)
        cuda_check(cudaMemcpy(key_codes + size_t(head) * kv_alloc * kHeadDim, C.sv.kcodes + base * kHeadDim,
                              size_t(kv_alloc) * kHeadDim, cudaMemcpyDeviceToHost), "read_kv");
      if (value_codes)
        cuda_check(cudaMemcpy(value_codes + size_t(head) * kv_alloc * kHeadDim, C.sv.vcodes + base * kHeadDim,
                              size_t(kv_alloc) * kHeadDim, cudaMemcpyDeviceToHost), "read_kv");
      if (key_scales)
        cuda_check(cudaMemcpy(key_scales + size_t(head) * kv_alloc, C.sv.kscale + base, size_t(kv_alloc) * 4,
                              cudaMemcpyDeviceToHost), "read_kv");
      if (value_scales)
        cuda_check(cudaMemcpy(value_scales + size_t(head) * kv_alloc, C.sv.vscale + base, size_t(kv_alloc) * 4,
                              cudaMemcpyDeviceToHost), "read_kv");
    }
  });
}

int needle_cuda_read_kv_f32(const needle_ctx* ctx, int32_t seq, int32_t layer, float* keys, float* values,
                            int32_t* kv_allocation) {
  return guarded([&] {
    const needle_ctx& C = *ctx_of(const_cast<needle_ctx*>(ctx));
    require(seq >= 0 && seq < C.opts.max_seqs, NEEDLE_BACKEND_UNAVAILABLE, "sequence slot out of range");
    require(layer >= 0 && layer < C.mv.layers, NEEDLE_INVALID_CACT, "Layer out of range");
    const SlotHost& h = C.slots[seq];
    require(C.sv.kv_f32 && h.ready, NEEDLE_INVALID_CACT, "Float32 KV cache is not allocated");
    if (kv_allocation) *kv_allocation = h.kv_alloc;
    cuda_check(cudaStreamSynchronize(C.stream), "read_kv");
    for (int head = 0; head < kKvHeads; head++) {
      const int64_t base = ((int64_t(seq) * C.mv.layers + layer) * kKvHeads + head) * C.sv.capacity;
      const size_t n = size_t(h.kv_alloc) * kHeadDim;
      if (keys)
        cuda_check(cudaMemcpy(keys + size_t(head) * n, C.sv.kf + base * kHeadDim, n * 4, cudaMemcpyDeviceToHost),
                   "read_kv");
      if (values)
        cuda_check(cudaMemcpy(values + size_t(head) * n, C.sv.vf + base * kHeadDim, n * 4, cudaMemcpyDeviceToHost),
                   "read_kv");
    }
  });
}

int needle_cuda_confidence(const needle_ctx* ctx, int32_t seq, double* value) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(const_cast<needle_ctx*>(ctx));
    require(value != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "null argument");
    require(seq >= 0 && seq < C.opts.max_seqs, NEEDLE_BACKEND_UNAVAILABLE, "sequence slot out of range");
    *value = std::numeric_limits<double>::quiet_NaN();
    if (!C.slots[seq].collect || C.mv.probe_count == 0) return;
    double* d_out = C.d_confidence;
    cuda_check(launch_confidence(C.mv, C.sv, seq, d_out, C.stream), "confidence");
    C.launches++;
    cuda_check(cudaMemcpyAsync(value, d_out, sizeof(double), cudaMemcpyDeviceToHost, C.stream), "confidence");
    cuda_check(cudaStreamSynchronize(C.stream), "confidence");
  });
}

int needle_cuda_read_lanes(const needle_ctx* ctx, int32_t seq, float* lanes) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(const_cast<needle_ctx*>(ctx));
    require(seq >= 0 && seq < C.opts.max_seqs && lanes, NEEDLE_BACKEND_UNAVAILABLE, "bad argument");
    cuda_check(cudaMemcpy(lanes, C.sv.x + size_t(seq) * kLaneWidth, kLaneWidth * 4, cudaMemcpyDeviceToHost),
               "read_lanes");
  });
}

int needle_cuda_matvec(needle_ctx* ctx, int32_t tensor, int32_t row_start, int32_t row_count, const float* x,
                       int32_t batch, float* y) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    require(tensor >= 0 && size_t(tensor) < C.cq.size() && C.cq[tensor].packed, NEEDLE_INVALID_CACT,
            "Tensor " + std::to_string(tensor) + " must be a Cactus-Quant matrix");
    const CqMat& M = C.cq[tensor];
    require(row_start >= 0 && row_count >= 0 && int64_t(row_start) + row_count <= M.rows, NEEDLE_INVALID_CACT,
            "Invalid matrix row range " + std::to_string(row_start) + ":" + std::to_string(row_start + row_count));
    require(batch >= 0 && (batch == 0 || (x && y)), NEEDLE_BACKEND_UNAVAILABLE, "bad batch");
    require(C.A.rec[tensor].group == uint32_t(kGroup), NEEDLE_BACKEND_UNAVAILABLE, "CQ group size 128 only");
    if (batch == 0 || row_count == 0) return;
    const size_t need = std::max(size_t(batch) * M.in_pad, size_t(batch) * row_count);
    ensure_mv(C, need);
    cuda_check(cudaMemcpyAsync(C.d_mv_x, x, size_t(batch) * M.input_size * 4, cudaMemcpyHostToDevice, C.stream),
               "matvec upload");
    cuda_check(launch_cq_prepare(C.d_mv_x, M.input_size, M.input_size, M.in_pad, C.d_mv_xp, M.in_pad, batch, nullptr,
                                 C.stream),
               "prepare");
    run_gemv(C, P_GEMV_VOCAB, {{M, row_start, row_count, C.d_mv_xp, M.in_pad, C.d_mv_y, row_count}}, batch, nullptr);
    cuda_check(cudaMemcpyAsync(y, C.d_mv_y, size_t(batch) * row_count * 4, cudaMemcpyDeviceToHost, C.stream),
               "matvec readback");
    cuda_check(cudaStreamSynchronize(C.stream), "matvec");
  });
}

int needle_cuda_row(needle_ctx* ctx, int32_t tensor, int32_t row, float* out) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    require(tensor >= 0 && size_t(tensor) < C.cq.size() && C.cq[tensor].packed, NEEDLE_INVALID_CACT,
            "Tensor " + std::to_string(tensor) + " must be a Cactus-Quant matrix");
    const CqMat& M = C.cq[tensor];
    require(row >= 0 && row < M.rows, NEEDLE_INVALID_CACT, "Matrix row " + std::to_string(row) + " is out of range");
    require(out != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "null output");
    require(C.A.rec[tensor].group == uint32_t(kGroup), NEEDLE_BACKEND_UNAVAILABLE, "CQ group size 128 only");
    if (!C.d_rows) {
      cuda_check(cudaMalloc(&C.d_rows, 16), "cudaMalloc");
      cuda_check(cudaMalloc(&C.d_row_out, size_t(kLaneWidth) * 4 * 4), "cudaMalloc");
    }
    require(M.in_pad <= kLaneWidth * 4, NEEDLE_BACKEND_UNAVAILABLE, "row too wide");
    cuda_check(cudaMemcpyAsync(C.d_rows, &row, 4, cudaMemcpyHostToDevice, C.stream), "row upload");
    cuda_check(launch_cq_rows(M.packed, M.norms, M.bits, M.row_bytes, M.in_pad, M.input_size, C.d_rows, 1,
                              C.d_row_out, M.in_pad, C.mv.cb, C.stream),
               "row");
    cuda_check(cudaMemcpyAsync(out, C.d_row_out, size_t(M.input_size) * 4, cudaMemcpyDeviceToHost, C.stream),
               "row readback");
    cuda_check(cudaStreamSynchronize(C.stream), "row");
  });
}

void* needle_cuda_stream(const needle_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int needle_cuda_sched_load(needle_ctx* ctx, int32_t n_slots, const int32_t* prompt_offsets, const int32_t* prompt_ids,
                           const int32_t* gen_steps, int32_t n_seqs) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    require(n_slots >= 1 && n_slots <= C.opts.max_seqs, NEEDLE_BACKEND_UNAVAILABLE, "n_slots out of range");
    require(C.sched_chunk < 2 || n_slots <= 1024, NEEDLE_BACKEND_UNAVAILABLE,
            "prompt chunks (sched_chunk) schedule at most 1024 slots");
    require(n_seqs >= 0 && prompt_offsets && gen_steps && (n_seqs == 0 || prompt_ids), NEEDLE_BACKEND_UNAVAILABLE,
            "bad queue");
    const int window = C.mv.kv_window;
    for (int s = 0; s < n_seqs; s++) {
      const int len = prompt_offsets[s + 1] - prompt_offsets[s];
      require(len >= 1 && gen_steps[s] >= 1, NEEDLE_INVALID_CACT, "empty prompt or generation");
      const int max_len = len + gen_steps[s];
      require(max_len <= C.mv.max_seq && max_len <= C.opts.max_len, NEEDLE_CONTEXT_OVERFLOW,
              "sequence exceeds the maximum length");
      const int kv_alloc = window > 0 ? std::min(max_len, window) : max_len;
      require(kv_alloc <= C.sv.capacity, NEEDLE_BACKEND_UNAVAILABLE, "sequence exceeds the KV capacity");
    }
    for (int s = 0; s < n_seqs; s++)
      for (int32_t k = prompt_offsets[s]; k < prompt_offsets[s + 1]; k++)
        require(prompt_ids[k] >= 0 && prompt_ids[k] < C.mv.vocab, NEEDLE_INVALID_CACT, "prompt token outside vocabulary");
    cuda_check(cudaStreamSynchronize(C.stream), "sched_load");
    if (C.sched_graph) {
      cudaGraphExecDestroy(C.sched_graph);
      C.sched_graph = nullptr;
    }
    C.sched_eager_steps = 0;
    for (void* p : C.sched_allocs) cudaFree(p);
    C.sched_allocs.clear();
    auto alloc = [&](size_t bytes) {
      void* p = nullptr;
      cuda_check(cudaMalloc(&p, std::max<size_t>(bytes, 16)), "cudaMalloc");
      C.sched_allocs.push_back(p);
      return p;
    };
    const size_t total = size_t(prompt_offsets[n_seqs]);
    int32_t* d_off = static_cast<int32_t*>(alloc(size_t(n_seqs + 1) * 4));
    int32_t* d_ids = static_cast<int32_t*>(alloc(total * 4));
    int32_t* d_gen = static_cast<int32_t*>(alloc(size_t(n_seqs) * 4));
    int32_t* d_ctr = static_cast<int32_t*>(alloc(64));
    int32_t* d_last = static_cast<int32_t*>(alloc(size_t(std::max(n_seqs, 1)) * 4));
    std::vector<int64_t> gen_off(size_t(n_seqs) + 1, 0);
    for (int s = 0; s < n_seqs; s++) gen_off[s + 1] = gen_off[s] + gen_steps[s];
    int64_t* d_gen_off = static_cast<int64_t*>(alloc(gen_off.size() * 8));
    int32_t* d_gen_ids = static_cast<int32_t*>(alloc(size_t(std::max<int64_t>(gen_off[n_seqs], 1)) * 4));
    cuda_check(cudaMemcpy(d_gen_off, gen_off.data(), gen_off.size() * 8, cudaMemcpyHostToDevice), "sched upload");
    cuda_check(cudaMemset(d_gen_ids, 0xff, size_t(std::max<int64_t>(gen_off[n_seqs], 1)) * 4), "sched init");
    C.sched_gen_total = gen_off[n_seqs];
    cuda_check(cudaMemcpy(d_off, prompt_offsets, size_t(n_seqs + 1) * 4, cudaMemcpyHostToDevice), "sched upload");
    if (total) cuda_check(cudaMemcpy(d_ids, prompt_ids, total * 4, cudaMemcpyHostToDevice), "sched upload");
    cuda_check(cudaMemcpy(d_gen, gen_steps, size_t(n_seqs) * 4, cudaMemcpyHostToDevice), "sched upload");
    cuda_check(cudaMemset(d_ctr, 0, 64), "sched init");
    cuda_check(cudaMemset(d_last, 0xff, size_t(std::max(n_seqs, 1)) * 4), "sched init");
    // all slots idle
    cuda_check(cudaMemset(C.sv.seq, 0, size_t(C.opts.max_seqs) * sizeof(SeqState)), "sched init");
    for (auto& h : C.slots) h = SlotHost{};
    C.collecting = 0;
    SchedView& q = C.sched;
    q.prompt_offsets = d_off;
    q.prompt_ids = d_ids;
    q.gen_steps = d_gen;
    q.n_seqs = n_seqs;
    q.n_slots = n_slots;
    q.next_seq = d_ctr;
    q.finished = d_ctr + 1;
    q.processed = reinterpret_cast<int64_t*>(d_ctr + 2);
    q.generated = reinterpret_cast<int64_t*>(d_ctr + 4);
    q.last_ids = d_last;
    q.gen_offsets = d_gen_off;
    q.gen_ids = d_gen_ids;
    C.sched_loaded = true;
    cuda_check(launch_sched_admit(C.sv, q, window, C.stream), "admit");
    cuda_check(cudaStreamSynchronize(C.stream), "sched_load");
  });
}

int needle_cuda_sched_step(needle_ctx* ctx, int32_t steps) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    require(C.sched_loaded, NEEDLE_BACKEND_UNAVAILABLE, "no scheduler queue loaded");
    if (steps > 0) C.sched_inflight = true;
    for (int32_t k = 0; k < steps; k++) {
      if (C.profiling || C.sched_eager_steps < 1) {
        enqueue_sched_step(C);
        C.sched_eager_steps++;
        continue;
      }
      if (!C.sched_graph) {
        // Capture one step (kernels on both micro-batch lanes, joined on the main stream).
        cuda_check(cudaStreamBeginCapture(C.stream, cudaStreamCaptureModeThreadLocal), "capture");
        const int64_t l0 = C.launches;
        try {
          enqueue_sched_step(C);
        } catch (...) {
          cudaGraph_t broken = nullptr;
          cudaStreamEndCapture(C.stream, &broken);
          if (broken) cudaGraphDestroy(broken);
          throw;
        }
        C.graph_launches = C.launches - l0;
        C.launches = l0;
        cudaGraph_t g = nullptr;
        cuda_check(cudaStreamEndCapture(C.stream, &g), "capture");
        const cudaError_t e = cudaGraphInstantiate(&C.sched_graph, g, 0);
        cudaGraphDestroy(g);
        cuda_check(e, "cudaGraphInstantiate");
      }
      cuda_check(cudaGraphLaunch(C.sched_graph, C.stream), "cudaGraphLaunch");
      C.launches += C.graph_launches;
    }
  });
}

int needle_cuda_sched_status(needle_ctx* ctx, int64_t* tokens_processed, int64_t* tokens_generated,
                             int32_t* seqs_finished, int32_t* last_ids) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    require(C.sched_loaded, NEEDLE_BACKEND_UNAVAILABLE, "no scheduler queue loaded");
    cuda_check(cudaStreamSynchronize(C.stream), "sched_status");
    check_device_waits(C);
    int32_t ctr[6];
    cuda_check(cudaMemcpy(ctr, C.sched.next_seq, 24, cudaMemcpyDeviceToHost), "sched_status");
    int64_t processed = 0, generated = 0;
    std::memcpy(&processed, ctr + 2, 8);
    std::memcpy(&generated, ctr + 4, 8);
    if (tokens_processed) *tokens_processed = processed;
    if (tokens_generated) *tokens_generated = generated;
    if (seqs_finished) *seqs_finished = ctr[1];
    if (last_ids && C.sched.n_seqs > 0)
      cuda_check(cudaMemcpy(last_ids, C.sched.last_ids, size_t(C.sched.n_seqs) * 4, cudaMemcpyDeviceToHost),
                 "sched_status");
  });
}

int needle_cuda_sched_ids(needle_ctx* ctx, int32_t* ids, size_t n, size_t* total) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    require(C.sched_loaded, NEEDLE_BACKEND_UNAVAILABLE, "no scheduler queue loaded");
    if (total) *total = size_t(C.sched_gen_total);
    cuda_check(cudaStreamSynchronize(C.stream), "sched_ids");
    const size_t k = std::min(n, size_t(C.sched_gen_total));
    if (ids && k) cuda_check(cudaMemcpy(ids, C.sched.gen_ids, k * 4, cudaMemcpyDeviceToHost), "sched_ids");
  });
}

int needle_cuda_sched_slot(needle_ctx* ctx, int32_t slot, int32_t* seq_id, int32_t* position, int32_t* busy) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    require(C.sched_loaded, NEEDLE_BACKEND_UNAVAILABLE, "no scheduler queue loaded");
    require(slot >= 0 && slot < C.sched.n_slots, NEEDLE_BACKEND_UNAVAILABLE, "slot out of range");
    SeqState st{};
    cuda_check(cudaStreamSynchronize(C.stream), "sched_slot");
    cuda_check(cudaMemcpy(&st, C.sv.seq + slot, sizeof(st), cudaMemcpyDeviceToHost), "sched_slot");
    if (seq_id) *seq_id = st.kv_alloc > 0 ? st.seq_id : -1;
    if (position) *position = st.position;
    if (busy) *busy = st.busy;
  });
}

int needle_cuda_check_guards(const needle_ctx* ctx, int32_t* damaged) {
  return guarded([&] {
    require(ctx != nullptr && damaged != nullptr, NEEDLE_BACKEND_UNAVAILABLE, "null argument");
    needle_ctx& C = *ctx_of(const_cast<needle_ctx*>(ctx));
    cuda_check(cudaDeviceSynchronize(), "check_guards");
    std::vector<uint8_t> host(needle_ctx::kGuardBytes);
    int32_t bad = 0;
    for (const auto& g : C.guards) {
      cuda_check(cudaMemcpy(host.data(), g.at, host.size(), cudaMemcpyDeviceToHost), "check_guards");
      for (uint8_t b : host)
        if (b != needle_ctx::kGuardByte) {
          bad++;
          break;
        }
    }
    *damaged = bad;
  });
}

int needle_cuda_kernel_launches(const needle_ctx* ctx, int64_t* count) {
  return guarded([&] {
    require(ctx && count, NEEDLE_BACKEND_UNAVAILABLE, "null argument");
    *count = ctx->launches;
  });
}

int needle_cuda_profile(needle_ctx* ctx, int32_t enable) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    if (enable && !C.profiling) {
      C.prof_drain();
      for (int i = 0; i < kProfClasses; i++) {
        C.prof_ms[i] = 0;
        C.prof_n[i] = 0;
      }
    }
    C.profiling = enable != 0;
  });
}

int needle_cuda_profile_read(needle_ctx* ctx, int32_t n, const char** names, double* total_ms, int64_t* launches,
                             int32_t* count) {
  return guarded([&] {
    needle_ctx& C = *ctx_of(ctx);
    C.prof_drain();
    if (count) *count = kProfClasses;
    for (int i = 0; i < std::min<int32_t>(n, kProfClasses); i++) {
      if (names) names[i] = kProfNames[i];
      if (total_ms) total_ms[i] = C.prof_ms[i];
      if (launches) launches[i] = C.prof_n[i];
    }
  });
}

}  // extern "C"
