// noalloc.cu -- edgexpu_cuda_linear_quant_batch_noalloc: the batched quantized linear without any
// memory allocation in the call.
//
// Who needs it: callers that must not allocate device memory once they are running -- runtimes that
// fix their HBM budget when the model is loaded and refuse to grow afterwards (an admission rule like
// the reference's host-RAM budget, applied to HBM), and latency-critical decode loops where an
// allocation or free may synchronise the whole device.  The regular device entry point
// (edgexpu_cuda_linear_quant_batch_dev) may grow its scratch buffer with cudaMalloc when a larger
// batch arrives; this one never does.
//
// How: batches of up to two rows need no scratch at all -- the GEMV quantizes the fp32 rows in its
// own prologue, exactly as the regular path does.  Larger batches are quantized into a file-scope
// __device__ array of fixed size (NOALLOC_SCRATCH_BYTES, 1 MiB), present on every GPU that loads this
// library until the process exits.  Host code cannot pass the array's name to a kernel (on the host
// it is only a stand-in symbol), so the first call on each device, with that device current, asks the
// runtime for the array's device address with cudaGetSymbolAddress and caches it; that first call
// should therefore happen before any stream capture.  Every byte the GEMV reads is written earlier in
// the same call, so nothing needs clearing; but all calls share the one array, so calls whose GPU work
// overlaps (for instance on two streams at once) race on it and must be serialised by the caller.
// Speed: the same GEMV as the regular entry point for decode-sized batches; for Q4_K batches of 64
// rows and more in the relaxed float order the regular entry point runs the tensor-core GEMM, while
// this one streams the weight once per 8 rows, which is several times slower near the 1 MiB limit.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "../../include/edgexpu_cuda.h"
#include "capi_internal.h"
#include "common.cuh"
#include "launch.h"

namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = size_t{1} << 20;
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

uint8_t* g_scratch_addr[MAX_DEVICES];  // device address of g_noalloc_scratch, per device

}  // namespace

extern "C" int edgexpu_cuda_linear_quant_batch_noalloc(float* out, const float* x, const uint8_t* weight, uint32_t type,
                                                       const float* bias, int m, int n_out, int n_in, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(ex::api_mutex());
  if (!ex::api_ready(nullptr, 0)) return 0;
  if (out == nullptr || x == nullptr || weight == nullptr || m <= 0 || n_out <= 0 || n_in <= 0)
    return ex::api_fail(nullptr, 0, "noalloc linear: invalid arguments");
  if (!ex::api_lookup(weight, type, n_out, n_in, nullptr, 0)) return 0;
  const size_t qb = ex::api_act_row_bytes(type, n_in);
  const size_t need = static_cast<size_t>(m) * qb;
  if (need > NOALLOC_SCRATCH_BYTES)
    return ex::api_fail(nullptr, 0,
                        "noalloc linear: %d rows of %d inputs need %zu bytes of quantized activations, more than the "
                        "fixed %zu-byte scratch; split the batch",
                        m, n_in, need, NOALLOC_SCRATCH_BYTES);
  const int dev = ex::api_device();
  if (dev < 0 || dev >= MAX_DEVICES) return ex::api_fail(nullptr, 0, "noalloc linear: device %d out of range", dev);
  if (g_scratch_addr[dev] == nullptr) {  // once per device, with that device current (api_ready set it)
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return ex::api_fail(nullptr, 0, "noalloc linear: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_addr[dev] = static_cast<uint8_t*>(p);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const ex::Fmt fmt = ex::fmt_q8(type);
  const int max_m = ex::rowstream_max_m(fmt, n_in, ex::api_device_info());
  if (max_m <= 0) return ex::api_fail(nullptr, 0, "noalloc linear: n_in %d too large for the activation tile", n_in);
  // Up to two rows the GEMV quantizes fp32 x itself (as run_linear_dev does): no scratch at all.
  const bool fused = ex::rowstream_quantizes_itself(fmt, m);
  uint8_t* xq = g_scratch_addr[dev];
  cudaError_t e = cudaSuccess;
  if (!fused) {
    e = ex::launch_quantize_for(type, x, m, n_in, xq, st);
    if (e != cudaSuccess) return ex::api_fail(nullptr, 0, "noalloc linear: quantize launch: %s", cudaGetErrorString(e));
  }
  const size_t stride = fused ? static_cast<size_t>(n_in) * 4 : qb;
  const uint8_t* act = fused ? reinterpret_cast<const uint8_t*>(x) : xq;
  for (int t0 = 0; t0 < m; t0 += max_m) {
    ex::RowStreamArgs a{};
    a.fmt = fmt;
    a.mode = ex::RowOut::Store;
    a.w = weight;
    a.n_rows = n_out;
    a.row_bytes = static_cast<int>(ex::api_row_bytes(type, n_in));
    a.K = n_in;
    a.m = std::min(max_m, m - t0);
    a.act = act + static_cast<size_t>(t0) * stride;
    a.act_row_bytes = static_cast<int>(qb);
    a.act_f32 = fused;
    a.bias = bias;
    a.out = out + static_cast<size_t>(t0) * n_out;
    a.out_stride = n_out;
    a.status = ex::api_status_word();
    a.exact = ex::api_exact_order();
    e = ex::launch_rowstream(a, ex::api_device_info(), st);
    if (e != cudaSuccess) return ex::api_fail(nullptr, 0, "noalloc linear: GEMV launch: %s", cudaGetErrorString(e));
  }
  return 1;
}
