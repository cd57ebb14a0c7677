// exptab.cu -- builds the expf table of exptab.cuh: the host's expf at every float input in
// [-104, 88.8], computed by all host threads into pinned chunks that are copied to HBM while the
// next chunk is computed.  Reference-counted: freed when the last user releases it.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "capi_internal.h"
#include "exptab.cuh"

namespace ex {

namespace {

std::mutex g_mu;
int g_refs = 0;
float* g_neg = nullptr;
float* g_pos = nullptr;

constexpr size_t CHUNK = size_t(1) << 26;  // entries per pinned chunk (256 MB)

// dst[i] = expf(+-bits_to_float(first + i)) for i < n, on every host thread.
void fill(float* dst, uint32_t first, size_t n, bool negative) {
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 4;
  if (nt > 64) nt = 64;
  std::vector<std::thread> th;
  const size_t per = (n + nt - 1) / nt;
  for (unsigned t = 0; t < nt; ++t) {
    th.emplace_back([=]() {
      const size_t lo = t * per, hi = std::min(n, lo + per);
      for (size_t i = lo; i < hi; ++i) {
        uint32_t b = first + static_cast<uint32_t>(i);
        if (negative) b |= 0x80000000u;
        float x;
        std::memcpy(&x, &b, 4);
        dst[i] = expf(x);
      }
    });
  }
  for (auto& t : th) t.join();
}

int build(float* dev, size_t entries, bool negative, float* pin[2], cudaEvent_t ev[2], cudaStream_t st) {
  size_t done = 0;
  for (int k = 0; done < entries; k ^= 1) {
    const size_t n = std::min(CHUNK, entries - done);
    if (cudaEventSynchronize(ev[k]) != cudaSuccess) return 0;
    fill(pin[k], static_cast<uint32_t>(done), n, negative);
    if (cudaMemcpyAsync(dev + done, pin[k], n * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaEventRecord(ev[k], st) != cudaSuccess)
      return 0;
    done += n;
  }
  return 1;
}

}  // namespace

int exptab_acquire(ExpTab* out, char* error, size_t error_size) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_refs == 0) {
    const size_t nn = size_t(EXPTAB_NEG_MAX) + 1, np = size_t(EXPTAB_POS_MAX) + 1;
    if (cudaMalloc(&g_neg, nn * 4) != cudaSuccess || cudaMalloc(&g_pos, np * 4) != cudaSuccess) {
      cudaFree(g_neg);
      g_neg = nullptr;
      return api_fail(error, error_size, "exp table: cannot allocate %.1f GB of HBM", (nn + np) * 4 / 1e9);
    }
    float* pin[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    cudaStream_t st = nullptr;
    bool ok = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess;
    for (int k = 0; k < 2 && ok; ++k)
      ok = cudaHostAlloc(reinterpret_cast<void**>(&pin[k]), CHUNK * 4, cudaHostAllocDefault) == cudaSuccess &&
           cudaEventCreateWithFlags(&ev[k], cudaEventDisableTiming) == cudaSuccess;
    ok = ok && build(g_neg, nn, true, pin, ev, st) && build(g_pos, np, false, pin, ev, st) &&
         cudaStreamSynchronize(st) == cudaSuccess;
    for (int k = 0; k < 2; ++k) {
      if (ev[k] != nullptr) cudaEventDestroy(ev[k]);
      if (pin[k] != nullptr) cudaFreeHost(pin[k]);
    }
    if (st != nullptr) cudaStreamDestroy(st);
    if (!ok) {
      cudaFree(g_neg);
      cudaFree(g_pos);
      g_neg = g_pos = nullptr;
      return api_fail(error, error_size, "exp table: building it failed");
    }
  }
  ++g_refs;
  out->neg = g_neg;
  out->pos = g_pos;
  return 1;
}

void exptab_release() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_refs > 0 && --g_refs == 0) {
    cudaDeviceSynchronize();
    cudaFree(g_neg);
    cudaFree(g_pos);
    g_neg = g_pos = nullptr;
  }
}

}  // namespace ex
