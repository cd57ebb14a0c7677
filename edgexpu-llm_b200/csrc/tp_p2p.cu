// tp_p2p.cu -- tensor-parallel linear whose all-reduce runs inside the GEMV over peer memory.
//
// With the weight sharded by input columns (o and down projections of a tensor-parallel layer),
// every rank computes a partial of the whole output and the partials must be summed.  Instead of
// a GEMV launch followed by a collective, the row-stream GEMV stores every partial output, tagged
// with the launch's epoch in the same 64-bit word, into every rank's exchange region (NVLink
// stores through CUDA IPC mappings: as each output is computed with up to 4 ranks, as coalesced
// per-CTA copies after the last tile with more); each CTA then waits for the tagged partials of
// its own rows in local memory and sums them in rank order (rowstream.cu, tp_finalize).  One
// launch per projection, no separate collective kernel, no fences, and the same additions in the
// same order on every rank.
//
// Set-up, once per process (one process per GPU): edgexpu_cuda_tp_init allocates the local region
// and exports its IPC handle; the caller exchanges the handles (e.g. torch.distributed
// all_gather_object) and passes all of them to edgexpu_cuda_tp_connect.  Calls are serialised on
// one stream per rank and every rank makes the same sequence of calls.  Peer memory is touched
// only by plain stores of this library's own kernels (no loads, no TMA, no multicast).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "../../include/edgexpu_cuda.h"
#include "capi_internal.h"
#include "common.cuh"
#include "launch.h"

namespace {

struct TpState {
  int world = 0, rank = 0;
  bool connected = false;
  uint8_t* local = nullptr;
  uint8_t* peer[ex::TP_MAX_WORLD] = {};
};
TpState t;

int tp_close() {
  for (int r = 0; r < ex::TP_MAX_WORLD; ++r) {
    if (t.peer[r] != nullptr && t.peer[r] != t.local) cudaIpcCloseMemHandle(t.peer[r]);
    t.peer[r] = nullptr;
  }
  if (t.local != nullptr) cudaFree(t.local);
  t = TpState{};
  return 1;
}

}  // namespace

namespace ex {
void tp_release() { tp_close(); }
}  // namespace ex

extern "C" {

int edgexpu_cuda_tp_init(int world, int rank, uint8_t* handle_out, char* error, size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(ex::api_mutex());
  if (!ex::api_ready(error, error_size)) return 0;
  if (world < 2 || world > ex::TP_MAX_WORLD || rank < 0 || rank >= world || handle_out == nullptr)
    return ex::api_fail(error, error_size, "tp_init: need 2 <= world <= %d, 0 <= rank < world", ex::TP_MAX_WORLD);
  tp_close();
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, ex::TP_REGION_BYTES);
  if (e == cudaSuccess) e = cudaMemset(p, 0, ex::TP_REGION_BYTES);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p != nullptr) cudaFree(p);
    return ex::api_fail(error, error_size, "tp_init: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == EDGEXPU_CUDA_TP_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  t.world = world;
  t.rank = rank;
  t.local = static_cast<uint8_t*>(p);
  return 1;
}

int edgexpu_cuda_tp_connect(const uint8_t* handles, char* error, size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(ex::api_mutex());
  if (!ex::api_ready(error, error_size)) return 0;
  if (t.local == nullptr || handles == nullptr) return ex::api_fail(error, error_size, "tp_connect: call tp_init first");
  for (int r = 0; r < t.world; ++r) {
    if (r == t.rank) {
      t.peer[r] = t.local;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles + static_cast<size_t>(r) * sizeof(h), sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      tp_close();
      return ex::api_fail(error, error_size, "tp_connect: rank %d: %s", r, cudaGetErrorString(e));
    }
    t.peer[r] = static_cast<uint8_t*>(p);
  }
  t.connected = true;
  return 1;
}

int edgexpu_cuda_tp_shutdown(void) {
  std::lock_guard<std::recursive_mutex> lk(ex::api_mutex());
  cudaDeviceSynchronize();
  return tp_close();
}

int edgexpu_cuda_linear_quant_batch_tp_dev(float* out, const float* x, const uint8_t* weight, uint32_t type,
                                           const float* bias, int m, int n_out, int n_in, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(ex::api_mutex());
  if (!ex::api_ready(nullptr, 0)) return 0;
  if (!t.connected) return ex::api_fail(nullptr, 0, "linear_tp: tensor-parallel group not connected");
  if (out == nullptr || x == nullptr || weight == nullptr || m <= 0 || n_out <= 0 || n_in <= 0)
    return ex::api_fail(nullptr, 0, "linear_tp: invalid arguments");
  if (!ex::api_lookup(weight, type, n_out, n_in, nullptr, 0)) return 0;
  if (type != ex::TYPE_Q8_0 && type != ex::TYPE_Q4_K)
    return ex::api_fail(nullptr, 0, "linear_tp: the in-kernel all-reduce is built for Q8_0 and Q4_K weights, not type %u",
                        type);
  const ex::Fmt fmt = ex::fmt_q8(type);
  const int max_m = ex::rowstream_max_m(fmt, n_in, ex::api_device_info());
  if (max_m <= 0) return ex::api_fail(nullptr, 0, "linear_tp: n_in %d too large for the activation tile", n_in);
  const int slot_m = static_cast<int>(ex::TP_SLOT_BYTES / 8 / static_cast<size_t>(n_out));  // rows one slot holds
  if (slot_m == 0)
    return ex::api_fail(nullptr, 0, "linear_tp: %d outputs exceed the exchange slot (%zu entries)", n_out,
                        ex::TP_SLOT_BYTES / 8);
  const int cap = max_m < slot_m ? max_m : slot_m;
  const int chunk = m < cap ? m : cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t qb = ex::api_act_row_bytes(type, n_in);
  const bool fused = ex::rowstream_quantizes_itself(fmt, chunk);
  const uint8_t* act = reinterpret_cast<const uint8_t*>(x);
  if (!fused) {  // quantize every row once (cpu_kernel.c:577-631), then stream
    void* xq = ex::api_act_scratch(static_cast<size_t>(m) * qb + 64, st, nullptr, 0);
    if (xq == nullptr) return 0;
    const cudaError_t e = ex::launch_quantize_for(type, x, m, n_in, static_cast<uint8_t*>(xq), st);
    if (e != cudaSuccess) return ex::api_fail(nullptr, 0, "linear_tp: %s", cudaGetErrorString(e));
    act = static_cast<const uint8_t*>(xq);
  }
  const size_t stride = fused ? static_cast<size_t>(n_in) * 4 : qb;
  for (int t0 = 0; t0 < m; t0 += chunk) {
    ex::RowStreamArgs a{};
    a.fmt = fmt;
    a.mode = ex::RowOut::StoreTp;
    a.w = weight;
    a.n_rows = n_out;
    a.row0 = 0;
    a.row_bytes = static_cast<int>(ex::api_row_bytes(type, n_in));
    a.K = n_in;
    a.m = m - t0 < chunk ? m - t0 : chunk;
    a.act = act + static_cast<size_t>(t0) * stride;
    a.act_row_bytes = static_cast<int>(qb);
    a.act_f32 = fused;
    a.bias = t.rank == 0 ? bias : nullptr;  // added once, by rank 0's partial
    a.out = out + static_cast<size_t>(t0) * n_out;
    a.out_stride = n_out;
    a.status = ex::api_status_word();
    a.tp.world = t.world;
    a.tp.rank = t.rank;
    for (int r = 0; r < t.world; ++r) a.tp.peer[r] = t.peer[r];
    const cudaError_t e = ex::launch_rowstream(a, ex::api_device_info(), st);
    if (e != cudaSuccess) return ex::api_fail(nullptr, 0, "linear_tp: %s", cudaGetErrorString(e));
  }
  return 1;
}

}  // extern "C"
