// capi.cu -- the C ABI of libedgexpu_cuda.so (declared in include/edgexpu_cuda.h).
//
// Owns the per-process device context: the CUDA stream, the weight registry (device address
// ranges of every uploaded or registered GGUF tensor), the activation/output scratch in HBM,
// pinned host staging for the synchronous host-buffer calls, and the device status word the
// kernels report timeouts through.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "../../include/edgexpu_cuda.h"
#include "capi_internal.h"
#include "common.cuh"
#include "launch.h"

namespace {

struct WeightRec {
  size_t capacity;
  uint32_t type;
  int n_out;
  int n_in;
  bool owned;
};

struct DevBuf {
  void* p = nullptr;
  size_t cap = 0;
};

struct HostBuf {
  void* p = nullptr;
  size_t cap = 0;
};

// A Q8_0 weight (rows [w, w + n_out) of width n_in) repacked for the tensor-core GEMM (gemm_q8_tc.cu).
struct Q8Pack {
  void* p = nullptr;
  int n_out = 0;
  int n_in = 0;
};

// A synchronous host-buffer call's three launches (pull, product, finish) recorded once per call
// shape and replayed as one CUDA graph.
struct ZcKey {
  int kind;  // 0: linear, 1: greedy logits
  uintptr_t weight;
  uint32_t type;
  int m, n_out, n_in;
  int has_bias;
  int order;
  bool operator<(const ZcKey& o) const {
    return std::tie(kind, weight, type, m, n_out, n_in, has_bias, order) <
           std::tie(o.kind, o.weight, o.type, o.m, o.n_out, o.n_in, o.has_bias, o.order);
  }
};
struct ZcGraph {
  cudaGraphExec_t exec = nullptr;  // null: recording was refused, the call launches directly
  uint64_t gen = 0;                // buffer generation the graph's pointers belong to
};
constexpr size_t ZC_MAX_GRAPHS = 4096;

struct Ctx {
  bool ready = false;
  std::map<uintptr_t, Q8Pack> q8packs;
  int device = -1;
  cudaStream_t stream = nullptr;
  ex::DeviceInfo info{};
  std::map<uintptr_t, WeightRec> weights;
  DevBuf x, xq, out, bias, wrow, samp, sstat, tcpart;
  HostBuf hx, hout, hbias;
  unsigned long long* d_key = nullptr;
  uint32_t* d_status = nullptr;
  unsigned long long* h_key = nullptr;
  uint32_t* h_status = nullptr;
  // Mapped pinned buffer of the synchronous host-buffer calls (zerocopy.cu): control words
  // [sequence, status] at 0, then the call's inputs and outputs at 256-byte aligned offsets.
  uint8_t* zc_h = nullptr;
  uint8_t* zc_d = nullptr;  // the same buffer's device address
  size_t zc_cap = 0;
  uint32_t zc_seq = 0;
  std::map<ZcKey, ZcGraph> zc_graphs;
  uint64_t buf_gen = 1;  // advances whenever a scratch or mapped buffer moves, or a weight is freed
};

Ctx g;
std::recursive_mutex g_mu;
// EDGEXPU_CUDA_ORDER_X86 (default) or EDGEXPU_CUDA_ORDER_RELAXED; process-wide, survives shutdown.
int g_order = EDGEXPU_CUDA_ORDER_X86;
bool exact_order() { return g_order == EDGEXPU_CUDA_ORDER_X86; }
char g_err[512] = "";

int fail(char* error, size_t error_size, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  if (error != nullptr && error_size > 0) snprintf(error, error_size, "%s", g_err);
  return 0;
}

#define EX_CUDA(call, error, error_size)                                                                   \
  do {                                                                                                     \
    cudaError_t e_ = (call);                                                                               \
    if (e_ != cudaSuccess) return fail(error, error_size, "%s: %s", #call, cudaGetErrorString(e_));       \
  } while (0)

// edgexpu_gguf_row_bytes (gguf_quant.c:468-480) for the quantized types of the path; 0 otherwise.
size_t row_bytes_of(uint32_t type, int n) {
  if (n <= 0) return 0;
  int qk = ex::QK_K, bb = 0;
  switch (type) {
    case ex::TYPE_Q8_0: qk = ex::QK8_0; bb = ex::Q8_0_BYTES; break;
    case ex::TYPE_Q4_0: qk = ex::QK8_0; bb = ex::Q4_0_BYTES; break;
    case ex::TYPE_Q5_0: qk = ex::QK8_0; bb = ex::Q5_0_BYTES; break;
    case ex::TYPE_Q4_K: bb = ex::Q4_K_BYTES; break;
    case ex::TYPE_Q5_K: bb = ex::Q5_K_BYTES; break;
    case ex::TYPE_Q6_K: bb = ex::Q6_K_BYTES; break;
    case ex::TYPE_F16: return static_cast<size_t>(n) * 2;
    case ex::TYPE_F32: return static_cast<size_t>(n) * 4;
    default: return 0;
  }
  return (n % qk) ? 0 : static_cast<size_t>(n / qk) * bb;
}

// F16/F32 weights: the reference's linear dots them against the fp32 activations directly
// (cpu_kernel.c:565-568, :633-643).
bool is_float_type(uint32_t type) { return type == ex::TYPE_F16 || type == ex::TYPE_F32; }

size_t act_row_bytes_of(uint32_t type, int n) {
  if (ex::acts_are_q8_0(type)) return static_cast<size_t>(n / ex::QK8_0) * ex::Q8_0_BYTES;
  return static_cast<size_t>(n / ex::QK_K) * ex::Q8_K_BYTES;
}

// NULL selects the CUDA default stream (the convention of every CUDA API, and the handle torch
// reports for its default stream); the library's own stream only serves the synchronous calls.
cudaStream_t pick(void* stream) { return static_cast<cudaStream_t>(stream); }

int need_ready(char* error, size_t error_size) {
  if (!g.ready) return fail(error, error_size, "edgexpu_cuda_init has not been called");
  cudaError_t e = cudaSetDevice(g.device);
  if (e != cudaSuccess) return fail(error, error_size, "cudaSetDevice: %s", cudaGetErrorString(e));
  return 1;
}

bool capturing(cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) return false;
  return cs != cudaStreamCaptureStatusNone;
}

int grow_dev(DevBuf& b, size_t need, cudaStream_t st, char* error, size_t error_size) {
  if (b.cap >= need) return 1;
  if (capturing(st)) return fail(error, error_size, "scratch must grow during stream capture; call edgexpu_cuda_reserve first");
  size_t cap = std::max<size_t>(need, 2 * b.cap);
  cap = (cap + 4095) & ~static_cast<size_t>(4095);
  EX_CUDA(cudaDeviceSynchronize(), error, error_size);
  if (b.p != nullptr) cudaFree(b.p);
  b.p = nullptr;
  b.cap = 0;
  ++g.buf_gen;
  EX_CUDA(cudaMalloc(&b.p, cap), error, error_size);
  b.cap = cap;
  return 1;
}

int grow_host(HostBuf& b, size_t need, char* error, size_t error_size) {
  if (b.cap >= need) return 1;
  size_t cap = std::max<size_t>(need, 2 * b.cap);
  cap = (cap + 4095) & ~static_cast<size_t>(4095);
  if (b.p != nullptr) {
    EX_CUDA(cudaDeviceSynchronize(), error, error_size);
    cudaFreeHost(b.p);
  }
  b.p = nullptr;
  b.cap = 0;
  EX_CUDA(cudaHostAlloc(&b.p, cap, cudaHostAllocDefault), error, error_size);
  b.cap = cap;
  return 1;
}

size_t al256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

int grow_zc(size_t need, char* error, size_t error_size) {
  if (g.zc_cap >= need) return 1;
  size_t cap = std::max<size_t>(need, 2 * g.zc_cap);
  cap = (cap + 65535) & ~static_cast<size_t>(65535);
  if (g.zc_h != nullptr) {
    EX_CUDA(cudaDeviceSynchronize(), error, error_size);
    cudaFreeHost(g.zc_h);
  }
  g.zc_h = g.zc_d = nullptr;
  g.zc_cap = 0;
  ++g.buf_gen;
  EX_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&g.zc_h), cap, cudaHostAllocMapped), error, error_size);
  EX_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&g.zc_d), g.zc_h, 0), error, error_size);
  std::memset(g.zc_h, 0, 256);
  g.zc_cap = cap;
  return 1;
}

int check_status(char* error, size_t error_size);

void zc_graphs_clear() {
  for (auto& kv : g.zc_graphs)
    if (kv.second.exec != nullptr) cudaGraphExecDestroy(kv.second.exec);
  g.zc_graphs.clear();
}

// The next call's sequence number, written into the mapped buffer at `off` (after the call's
// inputs, inside the range its pull kernel copies to the device).
uint32_t zc_stage_seq(size_t off) {
  if (++g.zc_seq == 0) g.zc_seq = 1;
  *reinterpret_cast<volatile uint32_t*>(g.zc_h + off) = g.zc_seq;
  std::atomic_thread_fence(std::memory_order_release);
  return g.zc_seq;
}

// Run a synchronous call's launches: `enqueue(error, error_size)` puts pull, product and finish on
// st.  The first call of a shape launches them directly (sizing any scratch) and then records them
// into a CUDA graph; later calls of that shape replay the graph, one launch instead of three.  A
// graph belongs to one buffer generation: once a buffer moved it is recorded again.
template <class F>
int zc_run(const ZcKey& key, cudaStream_t st, F&& enqueue, char* error, size_t error_size) {
  auto it = g.zc_graphs.find(key);
  if (it != g.zc_graphs.end() && it->second.gen == g.buf_gen) {
    if (it->second.exec == nullptr) return enqueue(error, error_size);
    EX_CUDA(cudaGraphLaunch(it->second.exec, st), error, error_size);
    return 1;
  }
  const uint64_t gen = g.buf_gen;
  if (!enqueue(error, error_size)) return 0;
  if (g.buf_gen != gen) return 1;  // a buffer moved during the call: record on a later one
  if (g.zc_graphs.size() >= ZC_MAX_GRAPHS) zc_graphs_clear();
  ZcGraph zg;
  zg.gen = gen;
  char saved[sizeof g_err];
  std::memcpy(saved, g_err, sizeof g_err);
  cudaGraph_t graph = nullptr;
  if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
    const int ok = enqueue(nullptr, 0);
    const cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (ok && e == cudaSuccess && graph != nullptr && cudaGraphInstantiate(&zg.exec, graph, 0) != cudaSuccess)
      zg.exec = nullptr;
    if (graph != nullptr) cudaGraphDestroy(graph);
  }
  (void)cudaGetLastError();  // a refused recording is not the call's error
  std::memcpy(g_err, saved, sizeof g_err);
  ZcGraph& slot = g.zc_graphs[key];
  if (slot.exec != nullptr) cudaGraphExecDestroy(slot.exec);
  slot = zg;
  return 1;
}

// Wait until the call's finish kernel has published sequence number `seq`.  The wait is bounded:
// the stream is polled for errors every ~1000 spins, and after 60 s the call fails.
int zc_wait(uint32_t seq, cudaStream_t st, char* error, size_t error_size) {
  volatile uint32_t* ctrl = reinterpret_cast<volatile uint32_t*>(g.zc_h);
  const auto t0 = std::chrono::steady_clock::now();
  for (unsigned it = 1;; ++it) {
    if (ctrl[0] == seq) break;
    if ((it & 1023) == 0) {
      const cudaError_t e = cudaStreamQuery(st);
      if (e != cudaSuccess && e != cudaErrorNotReady) return fail(error, error_size, "device work failed: %s", cudaGetErrorString(e));
      if (e == cudaSuccess && ctrl[0] != seq) return fail(error, error_size, "the call's completion word did not arrive");
      if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(60)) {
        return fail(error, error_size, "the call did not complete within 60 s");
      }
    }
  }
  std::atomic_thread_fence(std::memory_order_acquire);
  *g.h_status = ctrl[1];
  return check_status(error, error_size);
}

// Find the registered tensor holding rows [weight, weight + n_out rows) of width n_in.
int lookup(const uint8_t* weight, uint32_t type, int n_out, int n_in, char* error, size_t error_size) {
  const size_t rb = row_bytes_of(type, n_in);
  if (rb == 0)
    return fail(error, error_size,
                "unsupported weight type %u or n_in %d (Q8_0/Q5_0/Q4_0: n_in %% 32, Q4_K/Q5_K/Q6_K: n_in %% 256)", type,
                n_in);
  const uintptr_t w = reinterpret_cast<uintptr_t>(weight);
  auto it = g.weights.upper_bound(w);
  if (it == g.weights.begin()) return fail(error, error_size, "weight %p is not a registered device tensor", weight);
  --it;
  const WeightRec& rec = it->second;
  const uintptr_t base = it->first;
  if (w >= base + rec.capacity) return fail(error, error_size, "weight %p is not a registered device tensor", weight);
  if (rec.type != type) return fail(error, error_size, "weight %p was registered with type %u, called with %u", weight, rec.type, type);
  if (rec.n_in != n_in) return fail(error, error_size, "weight %p was registered with n_in %d, called with %d", weight, rec.n_in, n_in);
  if ((w - base) % rb != 0) return fail(error, error_size, "weight %p does not point at a row start", weight);
  const size_t row = (w - base) / rb;
  if (row + static_cast<size_t>(n_out) > static_cast<size_t>(rec.n_out))
    return fail(error, error_size, "rows [%zu, %zu) exceed the tensor's %d rows", row, row + n_out, rec.n_out);
  return 1;
}

// One row-stream launch per chunk of <= max_m activation rows.  act is either fp32 rows [m][n_in]
// (act_f32: the kernel quantizes them) or pre-quantized GGUF rows [m][act_row_bytes].
int run_rows_dev(float* out, const void* act, bool act_f32, const uint8_t* weight, uint32_t type, const float* bias,
                 int m, int n_out, int n_in, cudaStream_t st, char* error, size_t error_size) {
  const size_t qb = act_row_bytes_of(type, n_in);
  const size_t stride = act_f32 ? static_cast<size_t>(n_in) * 4 : qb;
  const ex::Fmt fmt = ex::fmt_q8(type);
  const int max_m = ex::rowstream_max_m(fmt, n_in, g.info);
  if (max_m <= 0) return fail(error, error_size, "n_in %d too large for the shared-memory activation tile", n_in);
  for (int t0 = 0; t0 < m; t0 += max_m) {
    ex::RowStreamArgs a{};
    a.fmt = fmt;
    a.mode = ex::RowOut::Store;
    a.w = weight;
    a.n_rows = n_out;
    a.row0 = 0;
    a.row_bytes = static_cast<int>(row_bytes_of(type, n_in));
    a.K = n_in;
    a.m = std::min(max_m, m - t0);
    a.act = static_cast<const uint8_t*>(act) + static_cast<size_t>(t0) * stride;
    a.act_row_bytes = static_cast<int>(qb);
    a.act_f32 = act_f32;
    a.bias = bias;
    a.out = out + static_cast<size_t>(t0) * n_out;
    a.out_stride = n_out;
    a.status = g.d_status;
    a.exact = exact_order();
    EX_CUDA(ex::launch_rowstream(a, g.info, st), error, error_size);
  }
  return 1;
}

// Q4_K batches of TC_SMALL_MIN_M rows and more run as a tensor-core GEMM (gemm_tc.cu; 16-token
// tiles below TC_MIN_M): always for the integer partials (bit-exact either way), for float outputs
// only in the relaxed order (its epilogue sums the super-blocks in its own order).
bool use_tc_partials(uint32_t type, int m, int n_in) {
  return type == ex::TYPE_Q4_K && m >= ex::TC_SMALL_MIN_M && n_in % ex::QK_K == 0;
}
bool use_tc(uint32_t type, int m, int n_in) { return !exact_order() && use_tc_partials(type, m, n_in); }
// Prefill-sized Q8_0 batches in the relaxed order run as the Q8_0 tensor-core GEMM.
bool use_tc_q8(uint32_t type, int m, int n_in) {
  return !exact_order() && type == ex::TYPE_Q8_0 && m >= ex::TC_MIN_M && n_in % ex::QK8_0 == 0;
}

// The repacked form of rows [weight, weight + n_out) (made on first use, kept until the tensor
// is freed).
const uint8_t* q8_pack_of(const uint8_t* weight, int n_out, int n_in, cudaStream_t st, char* error, size_t error_size) {
  const uintptr_t key = reinterpret_cast<uintptr_t>(weight);
  auto it = g.q8packs.find(key);
  if (it != g.q8packs.end() && it->second.n_out == n_out && it->second.n_in == n_in)
    return static_cast<const uint8_t*>(it->second.p);
  if (it != g.q8packs.end()) {
    cudaStreamSynchronize(st);
    cudaFree(it->second.p);
    g.q8packs.erase(it);
  }
  if (capturing(st)) {
    fail(error, error_size, "the Q8_0 GEMM's weight repack cannot be made during stream capture");
    return nullptr;
  }
  void* p = nullptr;
  if (cudaMalloc(&p, ex::q8_weight_pack_bytes(n_out, n_in)) != cudaSuccess) {
    fail(error, error_size, "cudaMalloc of a Q8_0 repack failed");
    return nullptr;
  }
  if (ex::launch_q8_repack_weight(weight, n_out, n_in, static_cast<uint8_t*>(p), st) != cudaSuccess) {
    cudaFree(p);
    fail(error, error_size, "Q8_0 repack launch failed");
    return nullptr;
  }
  g.q8packs[key] = Q8Pack{p, n_out, n_in};
  return static_cast<const uint8_t*>(p);
}

// Drop the repacks of rows inside [base, base + bytes).
void q8_unpack_range(uintptr_t base, size_t bytes) {
  for (auto it = g.q8packs.lower_bound(base); it != g.q8packs.end() && it->first < base + bytes;) {
    cudaFree(it->second.p);
    it = g.q8packs.erase(it);
  }
}

// out = x . W^T (+ bias) for a Q8_0 prefill batch on the tensor cores; x fp32 rows, or
// pre-quantized Q8_0 rows xq.
int tc_q8_linear(float* out, const float* x, const uint8_t* xq, const uint8_t* weight, const float* bias, int m,
                 int n_out, int n_in, cudaStream_t st, char* error, size_t error_size) {
  const uint8_t* wp = q8_pack_of(weight, n_out, n_in, st, error, error_size);
  if (wp == nullptr) return 0;
  if (!grow_dev(g.xq, ex::q8_act_pack_bytes(m, n_in) + 64, st, error, error_size)) return 0;
  uint8_t* ap = static_cast<uint8_t*>(g.xq.p);
  EX_CUDA(ex::launch_q8_pack_act(x, xq, m, n_in, ap, st), error, error_size);
  EX_CUDA(ex::launch_q8_gemm(wp, n_out, ap, m, n_in, bias, out, n_out, g.d_status, g.info, st), error, error_size);
  return 1;
}

// Pack m activation rows (fp32 x, or Q8_K rows xq) into the GEMM's tile layout in g.xq.
int tc_pack(const float* x, const uint8_t* xq, int m, int n_in, cudaStream_t st, char* error, size_t error_size) {
  if (!grow_dev(g.xq, ex::tc_act_bytes(m, n_in) + 64, st, error, error_size)) return 0;
  uint8_t* act = static_cast<uint8_t*>(g.xq.p);
  EX_CUDA(x != nullptr ? ex::launch_tc_pack_f32(x, m, n_in, act, st) : ex::launch_tc_pack_q8k(xq, m, n_in, act, st),
          error, error_size);
  return 1;
}

int tc_gemm(float* out, int32_t* partials, const uint8_t* weight, const float* bias, int m, int n_out, int n_in,
            cudaStream_t st, char* error, size_t error_size) {
  ex::TcGemmArgs a{};
  a.w = weight;
  a.n_rows = n_out;
  a.K = n_in;
  a.act = static_cast<const uint8_t*>(g.xq.p);
  a.m = m;
  a.bias = bias;
  a.out = out;
  a.out_stride = n_out;
  a.partials = partials;
  a.status = g.d_status;
  const size_t pb = partials == nullptr ? ex::tc_split_bytes(m, n_out, n_in, g.info) : 0;
  if (pb != 0 && !grow_dev(g.tcpart, pb, st, error, error_size)) return 0;
  a.part = pb != 0 ? static_cast<float*>(g.tcpart.p) : nullptr;
  EX_CUDA(ex::launch_tc_gemm(a, g.info, st), error, error_size);
  return 1;
}

int run_linear_dev(float* out, const float* x, const uint8_t* weight, uint32_t type, const float* bias, int m,
                   int n_out, int n_in, cudaStream_t st, char* error, size_t error_size) {
  if (out == nullptr || x == nullptr || weight == nullptr || m <= 0 || n_out <= 0 || n_in <= 0)
    return fail(error, error_size, "invalid arguments");
  if (!lookup(weight, type, n_out, n_in, error, error_size)) return 0;
  if (is_float_type(type)) {
    EX_CUDA(ex::launch_dot_f32(type, weight, row_bytes_of(type, n_in), n_out, n_in, x, m, bias, out, st), error,
            error_size);
    return 1;
  }
  if (use_tc(type, m, n_in))
    return tc_pack(x, nullptr, m, n_in, st, error, error_size) &&
           tc_gemm(out, nullptr, weight, bias, m, n_out, n_in, st, error, error_size);
  if (use_tc_q8(type, m, n_in)) return tc_q8_linear(out, x, nullptr, weight, bias, m, n_out, n_in, st, error, error_size);
  const ex::Fmt fmt = ex::fmt_q8(type);
  // cpu_kernel.c:577-631: every activation row is quantized once, then each weight row is dotted
  // against every quantized row.  Small batches quantize inside the GEMV launch itself.
  if (ex::rowstream_quantizes_itself(fmt, m))
    return run_rows_dev(out, x, true, weight, type, bias, m, n_out, n_in, st, error, error_size);
  const size_t qb = act_row_bytes_of(type, n_in);
  if (!grow_dev(g.xq, static_cast<size_t>(m) * qb + 64, st, error, error_size)) return 0;
  uint8_t* xq = static_cast<uint8_t*>(g.xq.p);
  EX_CUDA(ex::launch_quantize_for(type, x, m, n_in, xq, st), error, error_size);
  return run_rows_dev(out, xq, false, weight, type, bias, m, n_out, n_in, st, error, error_size);
}

int run_logits_dev(const uint8_t* weight, uint32_t type, const float* hidden, int n_embd, int vocab, const float* bias,
                   int64_t row0, unsigned long long* key, cudaStream_t st, char* error, size_t error_size) {
  if (weight == nullptr || hidden == nullptr || key == nullptr || n_embd <= 0 || vocab <= 0)
    return fail(error, error_size, "invalid arguments");
  if (row0 < 0 || row0 + vocab > 0xFFFFFFFFll) return fail(error, error_size, "row0 %lld out of range", (long long)row0);
  if (!lookup(weight, type, vocab, n_embd, error, error_size)) return 0;
  EX_CUDA(cudaMemsetAsync(key, 0, sizeof(unsigned long long), st), error, error_size);
  if (is_float_type(type)) {  // F16/F32 output weights: fp32 scores (dot_f16 / dot_f32_row), then the key
    if (!grow_dev(g.out, static_cast<size_t>(vocab) * 4, st, error, error_size)) return 0;
    float* scores = static_cast<float*>(g.out.p);
    EX_CUDA(ex::launch_dot_f32(type, weight, row_bytes_of(type, n_embd), vocab, n_embd, hidden, 1, bias, scores, st),
            error, error_size);
    EX_CUDA(ex::launch_argmax_key(scores, vocab, row0, key, st), error, error_size);
    return 1;
  }
  ex::RowStreamArgs a{};
  a.mode = ex::RowOut::Argmax;
  a.w = weight;
  a.n_rows = vocab;
  a.row0 = row0;
  a.row_bytes = static_cast<int>(row_bytes_of(type, n_embd));
  a.K = n_embd;
  a.m = 1;
  a.bias = bias;
  a.key = key;
  a.status = g.d_status;
  a.act = hidden;
  a.act_f32 = true;
  a.fmt = ex::logits_fmt(type);
  a.exact = exact_order();
  if (ex::acts_are_q8_0(type)) {
    // native.c:2317-2319: Q8_0-class logits weights (can_dot_q8) see a Q8_0-quantized hidden
    // state (the kernel quantizes it in its prologue).
    a.act_row_bytes = static_cast<int>(act_row_bytes_of(type, n_embd));
  } else {
    // logit_dot_row native.c:445-462 -> edgexpu_gguf_dot_quant gguf_quant.c:894-918: the K-quants
    // see the fp32 hidden state.
    a.act_row_bytes = n_embd * 4;
  }
  if (ex::rowstream_max_m(a.fmt, n_embd, g.info) < 1) return fail(error, error_size, "n_embd %d too large", n_embd);
  EX_CUDA(ex::launch_rowstream(a, g.info, st), error, error_size);
  return 1;
}

// Every logit score of the greedy/sampling path (native.c:500-514: dot + output bias) into
// scores[vocab]: the GEMV of run_logits_dev in Store mode.
int run_scores_dev(const uint8_t* weight, uint32_t type, const float* hidden, int n_embd, int vocab, const float* bias,
                   float* scores, cudaStream_t st, char* error, size_t error_size) {
  if (weight == nullptr || hidden == nullptr || scores == nullptr || n_embd <= 0 || vocab <= 0)
    return fail(error, error_size, "invalid arguments");
  if (!lookup(weight, type, vocab, n_embd, error, error_size)) return 0;
  if (is_float_type(type)) {
    EX_CUDA(ex::launch_dot_f32(type, weight, row_bytes_of(type, n_embd), vocab, n_embd, hidden, 1, bias, scores, st),
            error, error_size);
    return 1;
  }
  ex::RowStreamArgs a{};
  a.mode = ex::RowOut::Store;
  a.w = weight;
  a.n_rows = vocab;
  a.row_bytes = static_cast<int>(row_bytes_of(type, n_embd));
  a.K = n_embd;
  a.m = 1;
  a.bias = bias;
  a.out = scores;
  a.out_stride = vocab;
  a.status = g.d_status;
  a.act = hidden;
  a.act_f32 = true;
  a.fmt = ex::logits_fmt(type);
  a.exact = exact_order();
  a.act_row_bytes = ex::acts_are_q8_0(type) ? static_cast<int>(act_row_bytes_of(type, n_embd)) : n_embd * 4;
  if (ex::rowstream_max_m(a.fmt, n_embd, g.info) < 1) return fail(error, error_size, "n_embd %d too large", n_embd);
  EX_CUDA(ex::launch_rowstream(a, g.info, st), error, error_size);
  return 1;
}

// The reference's xorshift64 step and draw (cpu_kernel.c:780-785, :813 / :840).
double sample_draw(uint64_t* rng) {
  if (*rng == 0) *rng = 0x00ED6E50ULL;
  *rng ^= *rng << 13;
  *rng ^= *rng >> 7;
  *rng ^= *rng << 17;
  return static_cast<double>(*rng & 0xFFFFFFFu) / static_cast<double>(0x10000000u);
}

int sync_and_check(cudaStream_t st, char* error, size_t error_size);

// Softmax of io[n] (divided by temperature first when > 0) and the draw, on the device; the id
// into *out.  Synchronous.
int sample_dev(float* io, int n, float temperature, float top_p, uint64_t* rng, uint32_t* out, cudaStream_t st,
               char* error, size_t error_size) {
  const double u = sample_draw(rng);
  const size_t need = ex::sample_scratch_bytes(n);
  if (!grow_dev(g.samp, need, st, error, error_size) || !grow_dev(g.sstat, 64, st, error, error_size)) return 0;
  uint32_t* out_dev = static_cast<uint32_t*>(g.sstat.p);
  double* stats = reinterpret_cast<double*>(static_cast<uint8_t*>(g.sstat.p) + 32);
  EX_CUDA(ex::launch_sample(io, n, temperature, top_p, u, g.samp.p, g.samp.cap, out_dev, stats, st), error, error_size);
  EX_CUDA(cudaMemcpyAsync(g.h_key, out_dev, 4, cudaMemcpyDeviceToHost, st), error, error_size);
  if (!sync_and_check(st, error, error_size)) return 0;
  std::memcpy(out, g.h_key, 4);
  return 1;
}

int check_status(char* error, size_t error_size) {
  // Called after the stream was synchronised and the status word copied to h_status.
  if (*g.h_status != 0) {
    const uint32_t s = *g.h_status;
    *g.h_status = 0;
    cudaMemset(g.d_status, 0, sizeof(uint32_t));
    return fail(error, error_size, "device status 0x%x:%s%s%s%s%s", s,
                (s & ex::ST_TIMEOUT_FULL) ? " a consumer gave up waiting for a tile copy;" : "",
                (s & ex::ST_TIMEOUT_EMPTY) ? " the producer gave up waiting for a free stage;" : "",
                (s & ex::ST_TIMEOUT_DRAIN) ? " copies were still in flight at exit;" : "",
                (s & ex::ST_TIMEOUT_PEER) ? " a tensor-parallel peer did not deliver its partial in time;" : "",
                (s & ex::ST_BAD_INDEX) ? " a row id was outside the tensor;" : "");
  }
  return 1;
}

int sync_and_check(cudaStream_t st, char* error, size_t error_size) {
  EX_CUDA(cudaMemcpyAsync(g.h_status, g.d_status, sizeof(uint32_t), cudaMemcpyDeviceToHost, st), error, error_size);
  EX_CUDA(cudaStreamSynchronize(st), error, error_size);
  return check_status(error, error_size);
}

}  // namespace

extern "C" {

int edgexpu_cuda_abi_version(void) { return EDGEXPU_CUDA_ABI_VERSION; }

int edgexpu_cuda_set_float_order(int order) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (order != EDGEXPU_CUDA_ORDER_X86 && order != EDGEXPU_CUDA_ORDER_RELAXED)
    return fail(nullptr, 0, "set_float_order: unknown order %d", order);
  g_order = order;
  return 1;
}

int edgexpu_cuda_float_order(void) { return g_order; }

const char* edgexpu_cuda_last_error(void) { return g_err; }

int edgexpu_cuda_init(int device, char* error, size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (g.ready) {
    if (g.device == device) return 1;
    return fail(error, error_size, "already initialised on device %d", g.device);
  }
  int n = 0;
  EX_CUDA(cudaGetDeviceCount(&n), error, error_size);
  if (device < 0 || device >= n) return fail(error, error_size, "CUDA device %d not present (%d devices)", device, n);
  EX_CUDA(cudaSetDevice(device), error, error_size);
  int major = 0, minor = 0;
  EX_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device), error, error_size);
  EX_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device), error, error_size);
  if (major != 10 || minor != 0) return fail(error, error_size, "device %d is sm_%d%d; this build targets sm_100a (B200)", device, major, minor);
  EX_CUDA(cudaDeviceGetAttribute(&g.info.sm_count, cudaDevAttrMultiProcessorCount, device), error, error_size);
  EX_CUDA(cudaDeviceGetAttribute(&g.info.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device), error, error_size);
  EX_CUDA(cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking), error, error_size);
  EX_CUDA(cudaMalloc(reinterpret_cast<void**>(&g.d_key), 64), error, error_size);
  EX_CUDA(cudaMalloc(reinterpret_cast<void**>(&g.d_status), 64), error, error_size);
  EX_CUDA(cudaMemset(g.d_status, 0, 64), error, error_size);
  EX_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&g.h_key), 64, cudaHostAllocDefault), error, error_size);
  EX_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&g.h_status), 64, cudaHostAllocDefault), error, error_size);
  *g.h_status = 0;
  g.device = device;
  g.ready = true;
  return 1;
}

int edgexpu_cuda_shutdown(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!g.ready) return 1;
  cudaSetDevice(g.device);
  cudaDeviceSynchronize();
  ex::tp_release();
  zc_graphs_clear();
  for (auto& kv : g.weights)
    if (kv.second.owned) cudaFree(reinterpret_cast<void*>(kv.first));
  g.weights.clear();
  for (auto& kv : g.q8packs) cudaFree(kv.second.p);
  g.q8packs.clear();
  for (DevBuf* b : {&g.x, &g.xq, &g.out, &g.bias, &g.wrow, &g.samp, &g.sstat, &g.tcpart})
    if (b->p) cudaFree(b->p);
  for (HostBuf* b : {&g.hx, &g.hout, &g.hbias})
    if (b->p) cudaFreeHost(b->p);
  cudaFree(g.d_key);
  cudaFree(g.d_status);
  cudaFreeHost(g.h_key);
  cudaFreeHost(g.h_status);
  if (g.zc_h != nullptr) cudaFreeHost(g.zc_h);
  cudaStreamDestroy(g.stream);
  g = Ctx{};
  return 1;
}

int edgexpu_cuda_upload_weight(const uint8_t* host, size_t nbytes, uint32_t type, int n_out, int n_in,
                               const uint8_t** handle, char* error, size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(error, error_size)) return 0;
  const size_t rb = row_bytes_of(type, n_in);
  if (host == nullptr || handle == nullptr || n_out <= 0 || rb == 0) return fail(error, error_size, "invalid arguments");
  if (rb > (1u << 19)) return fail(error, error_size, "row of %zu bytes too large", rb);
  if (nbytes < rb * static_cast<size_t>(n_out)) return fail(error, error_size, "%zu bytes < %d rows x %zu", nbytes, n_out, rb);
  const size_t data = rb * static_cast<size_t>(n_out);
  const size_t cap = ((data + 255) & ~static_cast<size_t>(255)) + 256;  // padding for the aligned tail copy
  void* d = nullptr;
  EX_CUDA(cudaMalloc(&d, cap), error, error_size);
  cudaError_t e = cudaMemcpy(d, host, data, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(static_cast<uint8_t*>(d) + data, 0, cap - data);
  if (e != cudaSuccess) {
    cudaFree(d);
    return fail(error, error_size, "upload: %s", cudaGetErrorString(e));
  }
  g.weights[reinterpret_cast<uintptr_t>(d)] = WeightRec{cap, type, n_out, n_in, true};
  *handle = static_cast<const uint8_t*>(d);
  return 1;
}

int edgexpu_cuda_register_weight(const void* device_ptr, size_t capacity, uint32_t type, int n_out, int n_in,
                                 char* error, size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(error, error_size)) return 0;
  const size_t rb = row_bytes_of(type, n_in);
  if (device_ptr == nullptr || n_out <= 0 || rb == 0) return fail(error, error_size, "invalid arguments");
  if (rb > (1u << 19)) return fail(error, error_size, "row of %zu bytes too large", rb);
  if (reinterpret_cast<uintptr_t>(device_ptr) & 15u) return fail(error, error_size, "device_ptr must be 16-byte aligned");
  if (capacity < rb * static_cast<size_t>(n_out) + 16) return fail(error, error_size, "capacity must cover the rows plus 16 bytes");
  cudaPointerAttributes attr{};
  EX_CUDA(cudaPointerGetAttributes(&attr, device_ptr), error, error_size);
  if (attr.type != cudaMemoryTypeDevice || attr.device != g.device)
    return fail(error, error_size, "device_ptr is not device memory of device %d", g.device);
  g.weights[reinterpret_cast<uintptr_t>(device_ptr)] = WeightRec{capacity, type, n_out, n_in, false};
  return 1;
}

int edgexpu_cuda_free_weight(const void* handle) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto it = g.weights.find(reinterpret_cast<uintptr_t>(handle));
  if (it == g.weights.end()) return fail(nullptr, 0, "free_weight: %p is not a registered handle", handle);
  cudaDeviceSynchronize();
  zc_graphs_clear();  // recorded calls may name this tensor
  q8_unpack_range(it->first, it->second.capacity);
  if (it->second.owned) cudaFree(const_cast<void*>(handle));
  g.weights.erase(it);
  return 1;
}

static int quantize_host(uint32_t wtype, const float* x, int n, uint8_t* dst, char* error, size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(error, error_size)) return 0;
  const int blk = wtype == ex::TYPE_Q8_0 ? ex::QK8_0 : ex::QK_K;
  if (x == nullptr || dst == nullptr || n <= 0 || n % blk != 0) return fail(error, error_size, "invalid arguments");
  const size_t qb = act_row_bytes_of(wtype, n);
  cudaStream_t st = g.stream;
  if (!grow_host(g.hx, static_cast<size_t>(n) * 4, error, error_size) || !grow_dev(g.x, static_cast<size_t>(n) * 4, st, error, error_size) ||
      !grow_dev(g.xq, qb + 64, st, error, error_size) || !grow_host(g.hout, qb, error, error_size))
    return 0;
  std::memcpy(g.hx.p, x, static_cast<size_t>(n) * 4);
  EX_CUDA(cudaMemcpyAsync(g.x.p, g.hx.p, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, st), error, error_size);
  uint8_t* xq = static_cast<uint8_t*>(g.xq.p);
  EX_CUDA(wtype == ex::TYPE_Q8_0 ? ex::launch_quantize_q8_0(static_cast<float*>(g.x.p), 1, n, xq, st)
                                 : ex::launch_quantize_q8_k(static_cast<float*>(g.x.p), 1, n, xq, st),
          error, error_size);
  EX_CUDA(cudaMemcpyAsync(g.hout.p, xq, qb, cudaMemcpyDeviceToHost, st), error, error_size);
  EX_CUDA(cudaStreamSynchronize(st), error, error_size);
  std::memcpy(dst, g.hout.p, qb);
  return 1;
}

int edgexpu_cuda_quantize_q8_0(const float* x, int n, uint8_t* dst, char* error, size_t error_size) {
  return quantize_host(ex::TYPE_Q8_0, x, n, dst, error, error_size);
}

int edgexpu_cuda_quantize_q8_k(const float* x, int n, uint8_t* dst, char* error, size_t error_size) {
  return quantize_host(ex::TYPE_Q4_K, x, n, dst, error, error_size);
}

int edgexpu_cuda_linear_quant_batch(float* out, const float* x, const uint8_t* weight, uint32_t type, const float* bias,
                                    int m, int n_out, int n_in, char* error, size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(error, error_size)) return 0;
  if (out == nullptr || x == nullptr || weight == nullptr || m <= 0 || n_out <= 0 || n_in <= 0)
    return fail(error, error_size, "invalid arguments");
  if (!lookup(weight, type, n_out, n_in, error, error_size)) return 0;
  cudaStream_t st = g.stream;
  const size_t xb = static_cast<size_t>(m) * n_in * 4, ob = static_cast<size_t>(m) * n_out * 4;
  const size_t bb = bias != nullptr ? static_cast<size_t>(n_out) * 4 : 0;
  if (al256(xb) + bb <= ex::ZC_MAX_BYTES && ob <= ex::ZC_MAX_BYTES) {
    // Decode-sized call: inputs pulled from and outputs pushed to the mapped buffer by kernels;
    // the call's sequence number sits after the inputs.
    const size_t xoff = 256, soff = al256(al256(xb) + bb), ooff = xoff + soff + 256;
    if (!grow_zc(ooff + al256(ob), error, error_size) || !grow_dev(g.x, soff + 16 + 64, st, error, error_size) ||
        !grow_dev(g.out, ob, st, error, error_size))
      return 0;
    std::memcpy(g.zc_h + xoff, x, xb);
    if (bb) std::memcpy(g.zc_h + xoff + al256(xb), bias, bb);
    const uint32_t seq = zc_stage_seq(xoff + soff);
    float* xd = static_cast<float*>(g.x.p);
    float* od = static_cast<float*>(g.out.p);
    const uint32_t* seq_dev = reinterpret_cast<const uint32_t*>(static_cast<uint8_t*>(g.x.p) + soff);
    auto enqueue = [&](char* e, size_t es) -> int {
      EX_CUDA(ex::launch_zc_pull(reinterpret_cast<const float*>(g.zc_d + xoff), xd, static_cast<int>((soff + 16) / 4), st),
              e, es);
      if (!run_linear_dev(od, xd, weight, type, bb ? xd + al256(xb) / 4 : nullptr, m, n_out, n_in, st, e, es)) return 0;
      EX_CUDA(ex::launch_zc_finish(od, reinterpret_cast<float*>(g.zc_d + ooff), m * n_out, g.d_status,
                                   reinterpret_cast<uint32_t*>(g.zc_d), seq_dev, st),
              e, es);
      return 1;
    };
    const ZcKey key{0, reinterpret_cast<uintptr_t>(weight), type, m, n_out, n_in, bb != 0, g_order};
    if (!zc_run(key, st, enqueue, error, error_size) || !zc_wait(seq, st, error, error_size)) return 0;
    std::memcpy(out, g.zc_h + ooff, ob);
    return 1;
  }
  if (!grow_host(g.hx, xb, error, error_size) || !grow_dev(g.x, xb, st, error, error_size) ||
      !grow_host(g.hout, ob, error, error_size) || !grow_dev(g.out, ob, st, error, error_size))
    return 0;
  if (bb && (!grow_host(g.hbias, bb, error, error_size) || !grow_dev(g.bias, bb, st, error, error_size))) return 0;
  std::memcpy(g.hx.p, x, xb);
  EX_CUDA(cudaMemcpyAsync(g.x.p, g.hx.p, xb, cudaMemcpyHostToDevice, st), error, error_size);
  if (bb) {
    std::memcpy(g.hbias.p, bias, bb);
    EX_CUDA(cudaMemcpyAsync(g.bias.p, g.hbias.p, bb, cudaMemcpyHostToDevice, st), error, error_size);
  }
  if (!run_linear_dev(static_cast<float*>(g.out.p), static_cast<const float*>(g.x.p), weight, type,
                      bb ? static_cast<const float*>(g.bias.p) : nullptr, m, n_out, n_in, st, error, error_size))
    return 0;
  EX_CUDA(cudaMemcpyAsync(g.hout.p, g.out.p, ob, cudaMemcpyDeviceToHost, st), error, error_size);
  if (!sync_and_check(st, error, error_size)) return 0;
  std::memcpy(out, g.hout.p, ob);
  return 1;
}

int edgexpu_cuda_logits_argmax(const uint8_t* weight, uint32_t type, const float* hidden, int n_embd, int vocab,
                               const float* bias, uint32_t* token_id, float* best_score, char* error,
                               size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(error, error_size)) return 0;
  if (hidden == nullptr || token_id == nullptr || n_embd <= 0 || vocab <= 0) return fail(error, error_size, "invalid arguments");
  cudaStream_t st = g.stream;
  const size_t hb = static_cast<size_t>(n_embd) * 4, bb = bias != nullptr ? static_cast<size_t>(vocab) * 4 : 0;
  unsigned long long key = 0;
  if (al256(hb) + bb <= ex::ZC_MAX_BYTES) {  // through the mapped buffer (zerocopy.cu)
    const size_t xoff = 256, soff = al256(al256(hb) + bb), koff = xoff + soff + 256;
    if (!grow_zc(koff + 256, error, error_size) || !grow_dev(g.x, soff + 16 + 64, st, error, error_size)) return 0;
    std::memcpy(g.zc_h + xoff, hidden, hb);
    if (bb) std::memcpy(g.zc_h + xoff + al256(hb), bias, bb);
    const uint32_t seq = zc_stage_seq(xoff + soff);
    float* xd = static_cast<float*>(g.x.p);
    const uint32_t* seq_dev = reinterpret_cast<const uint32_t*>(static_cast<uint8_t*>(g.x.p) + soff);
    auto enqueue = [&](char* e, size_t es) -> int {
      EX_CUDA(ex::launch_zc_pull(reinterpret_cast<const float*>(g.zc_d + xoff), xd, static_cast<int>((soff + 16) / 4), st),
              e, es);
      if (!run_logits_dev(weight, type, xd, n_embd, vocab, bb ? xd + al256(hb) / 4 : nullptr, 0, g.d_key, st, e, es))
        return 0;
      EX_CUDA(ex::launch_zc_finish(reinterpret_cast<const float*>(g.d_key), reinterpret_cast<float*>(g.zc_d + koff), 2,
                                   g.d_status, reinterpret_cast<uint32_t*>(g.zc_d), seq_dev, st),
              e, es);
      return 1;
    };
    const ZcKey zk{1, reinterpret_cast<uintptr_t>(weight), type, 1, vocab, n_embd, bb != 0, g_order};
    if (!zc_run(zk, st, enqueue, error, error_size) || !zc_wait(seq, st, error, error_size)) return 0;
    std::memcpy(&key, g.zc_h + koff, 8);
  } else {
    if (!grow_host(g.hx, hb, error, error_size) || !grow_dev(g.x, hb, st, error, error_size)) return 0;
    if (bb && (!grow_host(g.hbias, bb, error, error_size) || !grow_dev(g.bias, bb, st, error, error_size))) return 0;
    std::memcpy(g.hx.p, hidden, hb);
    EX_CUDA(cudaMemcpyAsync(g.x.p, g.hx.p, hb, cudaMemcpyHostToDevice, st), error, error_size);
    if (bb) {
      std::memcpy(g.hbias.p, bias, bb);
      EX_CUDA(cudaMemcpyAsync(g.bias.p, g.hbias.p, bb, cudaMemcpyHostToDevice, st), error, error_size);
    }
    if (!run_logits_dev(weight, type, static_cast<const float*>(g.x.p), n_embd, vocab,
                        bb ? static_cast<const float*>(g.bias.p) : nullptr, 0, g.d_key, st, error, error_size))
      return 0;
    EX_CUDA(cudaMemcpyAsync(g.h_key, g.d_key, 8, cudaMemcpyDeviceToHost, st), error, error_size);
    if (!sync_and_check(st, error, error_size)) return 0;
    key = *g.h_key;
  }
  *token_id = edgexpu_cuda_argmax_key_id(key);
  if (best_score != nullptr) {
    uint32_t u = static_cast<uint32_t>(key >> 32);
    u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
    float s;
    std::memcpy(&s, &u, 4);
    *best_score = key == 0 ? -INFINITY : s;
  }
  return 1;
}

// Where the registered tensor holding `weight` starts, and its row count (0 if not registered).
static const uint8_t* tensor_of(const uint8_t* weight, long long* n_rows) {
  auto it = g.weights.upper_bound(reinterpret_cast<uintptr_t>(weight));
  if (it == g.weights.begin()) return nullptr;
  --it;
  if (reinterpret_cast<uintptr_t>(weight) >= it->first + it->second.capacity) return nullptr;
  *n_rows = it->second.n_out;
  return reinterpret_cast<const uint8_t*>(it->first);
}

int edgexpu_cuda_dequantize_rows_dev(float* out, const uint8_t* weight, uint32_t type, const int32_t* ids, int n_ids,
                                     int n_in, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(nullptr, 0)) return 0;
  if (out == nullptr || weight == nullptr || n_ids <= 0 || n_in <= 0) return fail(nullptr, 0, "dequantize_rows: invalid arguments");
  long long n_rows = 0;
  if (tensor_of(weight, &n_rows) != weight) return fail(nullptr, 0, "dequantize_rows: %p is not a registered tensor handle", weight);
  if (!lookup(weight, type, static_cast<int>(n_rows), n_in, nullptr, 0)) return 0;
  if (ids == nullptr && n_ids > n_rows) return fail(nullptr, 0, "dequantize_rows: %d rows exceed the tensor's %lld", n_ids, n_rows);
  EX_CUDA(ex::launch_dequant_rows(type, weight, row_bytes_of(type, n_in), n_rows, ids, n_ids, n_in, out, g.d_status,
                                  pick(stream)),
          nullptr, 0);
  return 1;
}

int edgexpu_cuda_dequantize_row(const uint8_t* weight, uint32_t type, int64_t row, int n_in, float* dst, char* error,
                                size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(error, error_size)) return 0;
  if (weight == nullptr || dst == nullptr || n_in <= 0) return fail(error, error_size, "dequantize_row: invalid arguments");
  long long n_rows = 0;
  if (tensor_of(weight, &n_rows) != weight) return fail(error, error_size, "dequantize_row: %p is not a registered tensor handle", weight);
  if (!lookup(weight, type, static_cast<int>(n_rows), n_in, error, error_size)) return 0;
  if (row < 0 || row >= n_rows) return fail(error, error_size, "dequantize_row: row %lld outside the tensor's %lld rows", (long long)row, n_rows);
  cudaStream_t st = g.stream;
  const size_t ob = static_cast<size_t>(n_in) * 4;
  if (!grow_dev(g.out, ob, st, error, error_size) || !grow_host(g.hout, ob, error, error_size)) return 0;
  const size_t rb = row_bytes_of(type, n_in);
  EX_CUDA(ex::launch_dequant_rows(type, weight + static_cast<size_t>(row) * rb, rb, 1, nullptr, 1, n_in,
                                  static_cast<float*>(g.out.p), g.d_status, st),
          error, error_size);
  EX_CUDA(cudaMemcpyAsync(g.hout.p, g.out.p, ob, cudaMemcpyDeviceToHost, st), error, error_size);
  if (!sync_and_check(st, error, error_size)) return 0;
  std::memcpy(dst, g.hout.p, ob);
  return 1;
}

int edgexpu_cuda_dot_quant(uint32_t type, const uint8_t* wrow, const void* x, int x_quantized, int n, float* result,
                           char* error, size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(error, error_size)) return 0;
  const size_t rb = row_bytes_of(type, n);
  ex::Fmt fmt;
  if (wrow == nullptr || x == nullptr || result == nullptr || rb == 0) return fail(error, error_size, "dot_quant: invalid arguments or type %u", type);
  if (x_quantized && !ex::fmt_of_type(type, &fmt)) return fail(error, error_size, "dot_quant: type %u has no quantized-activation dot", type);
  cudaStream_t st = g.stream;
  // The row: a row of a registered tensor is used in place; anything else is host memory (the
  // reference's mmap'd row) and is copied first.
  long long n_rows = 0;
  const uint8_t* w = wrow;
  if (tensor_of(wrow, &n_rows) == nullptr) {
    if (!grow_dev(g.wrow, rb + 256, st, error, error_size)) return 0;
    EX_CUDA(cudaMemcpyAsync(g.wrow.p, wrow, rb, cudaMemcpyHostToDevice, st), error, error_size);
    EX_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(g.wrow.p) + rb, 0, 256, st), error, error_size);
    w = static_cast<const uint8_t*>(g.wrow.p);
  } else if (!lookup(wrow, type, 1, n, error, error_size)) {
    return 0;
  }
  const size_t xb = x_quantized ? act_row_bytes_of(type, n) : static_cast<size_t>(n) * 4;
  if (!grow_host(g.hx, xb, error, error_size) || !grow_dev(g.x, xb + 64, st, error, error_size) ||
      !grow_dev(g.out, 64, st, error, error_size) || !grow_host(g.hout, 64, error, error_size))
    return 0;
  std::memcpy(g.hx.p, x, xb);
  EX_CUDA(cudaMemcpyAsync(g.x.p, g.hx.p, xb, cudaMemcpyHostToDevice, st), error, error_size);
  float* d_out = static_cast<float*>(g.out.p);
  if (x_quantized) {
    if (!run_rows_dev(d_out, g.x.p, false, w, type, nullptr, 1, 1, n, st, error, error_size)) return 0;
  } else {
    EX_CUDA(ex::launch_dot_f32(type, w, rb, 1, n, static_cast<const float*>(g.x.p), 1, nullptr, d_out, st), error,
            error_size);
  }
  EX_CUDA(cudaMemcpyAsync(g.hout.p, d_out, 4, cudaMemcpyDeviceToHost, st), error, error_size);
  if (!sync_and_check(st, error, error_size)) return 0;
  std::memcpy(result, g.hout.p, 4);
  return 1;
}

int edgexpu_cuda_quantize_dev(uint32_t weight_type, const float* x, int m, int n, uint8_t* dst, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(nullptr, 0)) return 0;
  ex::Fmt f;
  const int blk = !ex::fmt_of_type(weight_type, &f) ? 0 : (ex::acts_are_q8_0(weight_type) ? ex::QK8_0 : ex::QK_K);
  if (blk == 0 || x == nullptr || dst == nullptr || m <= 0 || n <= 0 || n % blk != 0) return fail(nullptr, 0, "invalid arguments");
  cudaStream_t st = pick(stream);
  EX_CUDA(ex::launch_quantize_for(weight_type, x, m, n, dst, st), nullptr, 0);
  return 1;
}

int edgexpu_cuda_linear_quant_batch_dev(float* out, const float* x, const uint8_t* weight, uint32_t type,
                                        const float* bias, int m, int n_out, int n_in, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(nullptr, 0)) return 0;
  return run_linear_dev(out, x, weight, type, bias, m, n_out, n_in, pick(stream), nullptr, 0);
}

int edgexpu_cuda_linear_quant_multi_dev(int n, float* const* outs, const uint8_t* const* weights, const int* n_outs,
                                        const float* const* biases, uint32_t type, const float* x, int m, int n_in,
                                        void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(nullptr, 0)) return 0;
  if (n < 1 || n > ex::MAX_SEGS || outs == nullptr || weights == nullptr || n_outs == nullptr || x == nullptr || m <= 0 ||
      n_in <= 0)
    return fail(nullptr, 0, "multi linear: invalid arguments (1..%d tensors)", ex::MAX_SEGS);
  for (int i = 0; i < n; ++i) {
    if (outs[i] == nullptr || n_outs[i] <= 0) return fail(nullptr, 0, "multi linear: invalid tensor %d", i);
    if (!lookup(weights[i], type, n_outs[i], n_in, nullptr, 0)) return 0;
  }
  cudaStream_t st = pick(stream);
  if (use_tc(type, m, n_in)) {  // one packing of the activations, one GEMM per tensor
    if (!tc_pack(x, nullptr, m, n_in, st, nullptr, 0)) return 0;
    for (int i = 0; i < n; ++i)
      if (!tc_gemm(outs[i], nullptr, weights[i], biases != nullptr ? biases[i] : nullptr, m, n_outs[i], n_in, st,
                   nullptr, 0))
        return 0;
    return 1;
  }
  if (use_tc_q8(type, m, n_in)) {  // one GEMM per tensor (each packs the activations)
    for (int i = 0; i < n; ++i)
      if (!tc_q8_linear(outs[i], x, nullptr, weights[i], biases != nullptr ? biases[i] : nullptr, m, n_outs[i], n_in, st,
                        nullptr, 0))
        return 0;
    return 1;
  }
  const ex::Fmt fmt = ex::fmt_q8(type);
  const size_t qb = act_row_bytes_of(type, n_in);
  const bool fused = ex::rowstream_quantizes_itself(fmt, m);
  const uint8_t* act = reinterpret_cast<const uint8_t*>(x);
  if (!fused) {
    if (!grow_dev(g.xq, static_cast<size_t>(m) * qb + 64, st, nullptr, 0)) return 0;
    EX_CUDA(ex::launch_quantize_for(type, x, m, n_in, static_cast<uint8_t*>(g.xq.p), st), nullptr, 0);
    act = static_cast<const uint8_t*>(g.xq.p);
  }
  const size_t stride = fused ? static_cast<size_t>(n_in) * 4 : qb;
  const int max_m = ex::rowstream_max_m(fmt, n_in, g.info);
  if (max_m <= 0) return fail(nullptr, 0, "n_in %d too large for the shared-memory activation tile", n_in);
  for (int t0 = 0; t0 < m; t0 += max_m) {
    ex::RowStreamArgs a{};
    a.fmt = fmt;
    a.mode = ex::RowOut::Store;
    a.row_bytes = static_cast<int>(row_bytes_of(type, n_in));
    a.K = n_in;
    a.m = std::min(max_m, m - t0);
    a.act = act + static_cast<size_t>(t0) * stride;
    a.act_row_bytes = static_cast<int>(qb);
    a.act_f32 = fused;
    a.status = g.d_status;
    a.n_seg = n;
    a.exact = exact_order();
    for (int i = 0; i < n; ++i)
      a.seg[i] = ex::RowSeg{weights[i], n_outs[i], biases != nullptr ? biases[i] : nullptr,
                            outs[i] + static_cast<size_t>(t0) * n_outs[i], 0};
    EX_CUDA(ex::launch_rowstream(a, g.info, st), nullptr, 0);
  }
  return 1;
}

int edgexpu_cuda_dot_quant_q8_dev(float* out, const uint8_t* xq, const uint8_t* weight, uint32_t type, const float* bias,
                                  int m, int n_out, int n_in, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(nullptr, 0)) return 0;
  if (out == nullptr || xq == nullptr || weight == nullptr || m <= 0 || n_out <= 0 || n_in <= 0)
    return fail(nullptr, 0, "invalid arguments");
  if (!lookup(weight, type, n_out, n_in, nullptr, 0)) return 0;
  if (use_tc(type, m, n_in))
    return tc_pack(nullptr, xq, m, n_in, pick(stream), nullptr, 0) &&
           tc_gemm(out, nullptr, weight, bias, m, n_out, n_in, pick(stream), nullptr, 0);
  if (use_tc_q8(type, m, n_in)) return tc_q8_linear(out, nullptr, xq, weight, bias, m, n_out, n_in, pick(stream), nullptr, 0);
  return run_rows_dev(out, xq, false, weight, type, bias, m, n_out, n_in, pick(stream), nullptr, 0);
}

int edgexpu_cuda_logits_argmax_dev(const uint8_t* weight, uint32_t type, const float* hidden, int n_embd, int vocab,
                                   const float* bias, int64_t row0, uint64_t* key, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(nullptr, 0)) return 0;
  return run_logits_dev(weight, type, hidden, n_embd, vocab, bias, row0, reinterpret_cast<unsigned long long*>(key),
                        pick(stream), nullptr, 0);
}

int edgexpu_cuda_block_partials_dev(int32_t* partials, const uint8_t* xq, const uint8_t* weight, uint32_t type, int m,
                                    int n_out, int n_in, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(nullptr, 0)) return 0;
  if (partials == nullptr || xq == nullptr || m <= 0) return fail(nullptr, 0, "invalid arguments");
  if (!lookup(weight, type, n_out, n_in, nullptr, 0)) return 0;
  if (use_tc_partials(type, m, n_in))
    return tc_pack(nullptr, xq, m, n_in, pick(stream), nullptr, 0) &&
           tc_gemm(nullptr, partials, weight, nullptr, m, n_out, n_in, pick(stream), nullptr, 0);
  ex::RowStreamArgs a{};
  a.fmt = ex::fmt_q8(type);
  a.mode = ex::RowOut::Partials;
  a.w = weight;
  a.n_rows = n_out;
  a.row_bytes = static_cast<int>(row_bytes_of(type, n_in));
  a.K = n_in;
  a.m = m;
  a.act = xq;
  a.act_row_bytes = static_cast<int>(act_row_bytes_of(type, n_in));
  a.partials = partials;
  a.status = g.d_status;
  if (ex::rowstream_max_m(a.fmt, n_in, g.info) < m) return fail(nullptr, 0, "m %d too large for one partials launch", m);
  EX_CUDA(ex::launch_rowstream(a, g.info, pick(stream)), nullptr, 0);
  return 1;
}

int edgexpu_cuda_reserve(int m, int n_in, char* error, size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(error, error_size)) return 0;
  if (m <= 0 || n_in <= 0) return fail(error, error_size, "invalid arguments");
  size_t need = static_cast<size_t>(m) * std::max(act_row_bytes_of(ex::TYPE_Q8_0, n_in), act_row_bytes_of(ex::TYPE_Q4_K, n_in)) + 64;
  if (use_tc_partials(ex::TYPE_Q4_K, m, n_in)) need = std::max(need, ex::tc_act_bytes(m, n_in) + 64);
  return grow_dev(g.xq, need, g.stream, error, error_size);
}

int edgexpu_cuda_stream_sync(void* stream, char* error, size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(error, error_size)) return 0;
  return sync_and_check(pick(stream), error, error_size);
}

}  // extern "C"

extern "C" int edgexpu_cuda_sample_softmax(float* logits, int n, float top_p, uint64_t* rng, uint32_t* out, char* error,
                                           size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(error, error_size)) return 0;
  if (logits == nullptr || rng == nullptr || out == nullptr || n <= 0) return fail(error, error_size, "sample_softmax: invalid arguments");
  cudaStream_t st = g.stream;
  const size_t b = static_cast<size_t>(n) * 4;
  if (!grow_dev(g.out, b, st, error, error_size) || !grow_host(g.hout, b, error, error_size)) return 0;
  std::memcpy(g.hout.p, logits, b);
  EX_CUDA(cudaMemcpyAsync(g.out.p, g.hout.p, b, cudaMemcpyHostToDevice, st), error, error_size);
  if (!sample_dev(static_cast<float*>(g.out.p), n, 0.0f, top_p, rng, out, st, error, error_size)) return 0;
  // the reference leaves the probabilities in `logits` (softmax in place)
  EX_CUDA(cudaMemcpyAsync(g.hout.p, g.out.p, b, cudaMemcpyDeviceToHost, st), error, error_size);
  EX_CUDA(cudaStreamSynchronize(st), error, error_size);
  std::memcpy(logits, g.hout.p, b);
  return 1;
}

extern "C" int edgexpu_cuda_logits_sample(const uint8_t* weight, uint32_t type, const float* hidden, int n_embd, int vocab,
                                          const float* bias, float temperature, float top_p, uint64_t* rng,
                                          uint32_t* token_id, char* error, size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!need_ready(error, error_size)) return 0;
  if (hidden == nullptr || rng == nullptr || token_id == nullptr || n_embd <= 0 || vocab <= 0 || !(temperature > 0.0f))
    return fail(error, error_size, "logits_sample: invalid arguments");
  cudaStream_t st = g.stream;
  const size_t hb = static_cast<size_t>(n_embd) * 4, bb = bias != nullptr ? static_cast<size_t>(vocab) * 4 : 0;
  if (!grow_host(g.hx, hb, error, error_size) || !grow_dev(g.x, hb, st, error, error_size) ||
      !grow_dev(g.out, static_cast<size_t>(vocab) * 4, st, error, error_size))
    return 0;
  if (bb && (!grow_host(g.hbias, bb, error, error_size) || !grow_dev(g.bias, bb, st, error, error_size))) return 0;
  std::memcpy(g.hx.p, hidden, hb);
  EX_CUDA(cudaMemcpyAsync(g.x.p, g.hx.p, hb, cudaMemcpyHostToDevice, st), error, error_size);
  if (bb) {
    std::memcpy(g.hbias.p, bias, bb);
    EX_CUDA(cudaMemcpyAsync(g.bias.p, g.hbias.p, bb, cudaMemcpyHostToDevice, st), error, error_size);
  }
  float* scores = static_cast<float*>(g.out.p);
  if (!run_scores_dev(weight, type, static_cast<const float*>(g.x.p), n_embd, vocab,
                      bb ? static_cast<const float*>(g.bias.p) : nullptr, scores, st, error, error_size))
    return 0;
  return sample_dev(scores, vocab, temperature, top_p, rng, token_id, st, error, error_size);
}

namespace ex {

std::recursive_mutex& api_mutex() { return g_mu; }
int api_ready(char* error, size_t error_size) { return need_ready(error, error_size); }
int api_lookup(const uint8_t* weight, uint32_t type, int n_out, int n_in, char* error, size_t error_size) {
  return lookup(weight, type, n_out, n_in, error, error_size);
}
int api_fail(char* error, size_t error_size, const char* fmt, ...) {
  char msg[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof msg, fmt, ap);
  va_end(ap);
  return fail(error, error_size, "%s", msg);
}
const DeviceInfo& api_device_info() { return g.info; }
int api_device() { return g.device; }
bool api_exact_order() { return exact_order(); }
cudaStream_t api_stream() { return g.stream; }
int api_logit_scores(const uint8_t* weight, uint32_t type, const float* hidden, int n_embd, int vocab, const float* bias,
                     float* scores, cudaStream_t st, char* error, size_t error_size) {
  return run_scores_dev(weight, type, hidden, n_embd, vocab, bias, scores, st, error, error_size);
}
int api_sample(float* io, int n, float temperature, float top_p, uint64_t* rng, uint32_t* out, cudaStream_t st,
               char* error, size_t error_size) {
  return sample_dev(io, n, temperature, top_p, rng, out, st, error, error_size);
}
uint32_t* api_status_word() { return g.d_status; }
size_t api_row_bytes(uint32_t type, int n) { return row_bytes_of(type, n); }
size_t api_act_row_bytes(uint32_t type, int n) { return act_row_bytes_of(type, n); }
void* api_act_scratch(size_t bytes, cudaStream_t st, char* error, size_t error_size) {
  return grow_dev(g.xq, bytes, st, error, error_size) ? g.xq.p : nullptr;
}

}  // namespace ex
