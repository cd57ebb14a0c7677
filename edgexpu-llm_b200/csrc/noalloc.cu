// noalloc.cu -- edgexpu_cuda_linear_quant_batch_noalloc: the batched quantized linear without any
// memory allocation in the call.
//
// Who needs it: callers that must not allocate device memory once they are running.  Examples
// are code being recorded into a CUDA graph (cudaMalloc/cudaFree are not stream operations and
// cannot be captured), runtimes that fix their HBM budget when the model is loaded and refuse to
// grow afterwards (an admission rule like the reference's host-RAM budget, applied to HBM), and
// latency-critical decode loops where an allocation or free may synchronise the whole device.
// The regular device entry point (edgexpu_cuda_linear_quant_batch_dev) may grow its scratch
// buffer with cudaMalloc when a larger batch arrives; this one never does.
//
// How: the quantized activation rows live in a file-scope __device__ array of fixed size
// (NOALLOC_SCRATCH_BYTES, 1 MiB), present on every GPU that loads this library until the process
// exits.  Host code cannot pass the array's name to a kernel (on the host it is only a stand-in
// symbol), so the first call on each device, with that device current, asks the runtime for the
// array's device address with cudaGetSymbolAddress and caches it; that first call should
// therefore happen before any stream capture.  Each call then quantizes x into the array (the
// same kernel and bytes as the regular path) and runs the row-stream GEMV on it.  Every byte the
// GEMV reads is written earlier in the same call, so nothing needs clearing; but all calls share
// the one array, so calls whose GPU work overlaps (for instance on two streams at once) race on it
// and must be serialised by the caller.
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
  uint8_t* xq = g_scratch_addr[dev];
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = ex::launch_quantize_for(type, x, m, n_in, xq, st);
  if (e != cudaSuccess) return ex::api_fail(nullptr, 0, "noalloc linear: quantize launch: %s", cudaGetErrorString(e));
  const ex::Fmt fmt = ex::fmt_q8(type);
  const int max_m = ex::rowstream_max_m(fmt, n_in, ex::api_device_info());
  if (max_m <= 0) return ex::api_fail(nullptr, 0, "noalloc linear: n_in %d too large for the activation tile", n_in);
  for (int t0 = 0; t0 < m; t0 += max_m) {
    ex::RowStreamArgs a{};
    a.fmt = fmt;
    a.mode = ex::RowOut::Store;
    a.w = weight;
    a.n_rows = n_out;
    a.row_bytes = static_cast<int>(ex::api_row_bytes(type, n_in));
    a.K = n_in;
    a.m = std::min(max_m, m - t0);
    a.act = xq + static_cast<size_t>(t0) * qb;
    a.act_row_bytes = static_cast<int>(qb);
    a.act_f32 = false;
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
