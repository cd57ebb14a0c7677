// zerocopy.cu -- the two small kernels around a synchronous host-buffer call.
//
// A call such as edgexpu_cuda_linear_quant_batch moves a few KB each way (one activation row in,
// one output row out) around a few microseconds of GEMV.  Done with copy-engine transfers and a
// stream synchronisation, the two copies and the wait cost more than the kernel.  Instead the
// caller's rows go through one mapped, pinned host buffer:
//   * zc_pull_kernel reads the inputs (activations and bias, contiguous in the buffer) over the
//     bus into device scratch; it lets the GEMV launch behind it at once (programmatic dependent
//     launch), and the GEMV reads the scratch only after its dependency wait;
//   * zc_finish_kernel, launched after the GEMV and waiting for it, writes the outputs and the
//     device status word back into the buffer and then the call's sequence number; the host spins
//     on that number instead of synchronising the stream.  The number travels in with the inputs
//     (the host writes it after them, the pull kernel copies it), so the three launches take no
//     per-call argument and the host can replay them as one CUDA graph per call shape.
// Writers order their stores to host memory with a system-scope fence before the block barrier
// that precedes the sequence-number store, so a host that sees the number sees the data.
#include <cuda_runtime.h>

#include "common.cuh"
#include "launch.h"

namespace ex {

namespace {

__global__ void __launch_bounds__(256) zc_pull_kernel(const float* __restrict__ src, float* __restrict__ dst, int n) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int n4 = n >> 2;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) d4[i] = s4[i];
  if (blockIdx.x == 0 && threadIdx.x < n - (n4 << 2)) dst[(n4 << 2) + threadIdx.x] = src[(n4 << 2) + threadIdx.x];
}

__global__ void __launch_bounds__(ZC_FINISH_THREADS) zc_finish_kernel(const float* __restrict__ src, float* dst, int n,
                                                                      uint32_t* d_status, uint32_t* ctrl,
                                                                      const uint32_t* seq_dev) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the producing grid (and the pull before it) has completed
  const int n4 = n >> 2;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  for (int i = threadIdx.x; i < n4; i += blockDim.x) d4[i] = s4[i];
  for (int i = (n4 << 2) + threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile uint32_t* ds = d_status;
    const uint32_t s = *ds;
    if (s != 0) *ds = 0u;
    volatile uint32_t* c = ctrl;
    c[1] = s;
    __threadfence_system();
    c[0] = *seq_dev;
  }
}

}  // namespace

cudaError_t launch_zc_pull(const float* src, float* dst, int n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int grid = (n / 4 + 255) / 256;
  grid = grid < 1 ? 1 : (grid > ZC_PULL_MAX_CTAS ? ZC_PULL_MAX_CTAS : grid);
  zc_pull_kernel<<<grid, 256, 0, st>>>(src, dst, n);
  return cudaGetLastError();
}

cudaError_t launch_zc_finish(const float* src, float* dst, int n, uint32_t* d_status, uint32_t* ctrl,
                             const uint32_t* seq_dev, cudaStream_t st) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(ZC_FINISH_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, zc_finish_kernel, src, dst, n, d_status, ctrl, seq_dev);
}

}  // namespace ex
