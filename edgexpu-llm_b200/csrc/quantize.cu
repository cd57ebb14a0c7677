// quantize.cu -- standalone fp32 -> Q8_0 / Q8_K activation quantizers for sm_100a, writing the
// reference's GGUF block layout (gguf_dot_q8.c:269-412).  The arithmetic lives in quant.cuh and
// is shared with the GEMV prologue.
#include "common.cuh"
#include "launch.h"
#include "quant.cuh"

namespace ex {
namespace {

// One warp per 32-element block; lane i owns element i.
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const float* __restrict__ x, int n, long long n_blocks,
                                                            uint8_t* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  const int nb = n / QK8_0;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long blk = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; blk < n_blocks;
       blk += nwarps) {
    const long long t = blk / nb;
    const int b = static_cast<int>(blk - t * nb);
    uint32_t dbits;
    const int q = warp_q8_0(x[t * n + static_cast<long long>(b) * QK8_0 + lane], &dbits);
    uint8_t* o8 = dst + blk * Q8_0_BYTES;
    o8[2 + lane] = static_cast<uint8_t>(static_cast<int8_t>(q));
    if (lane == 0) *reinterpret_cast<unsigned short*>(o8) = static_cast<unsigned short>(dbits);
  }
}

// One warp per 256-element block; lane i owns elements 8i .. 8i+7.
__global__ void __launch_bounds__(256) quantize_q8_k_kernel(const float* __restrict__ x, int n, long long n_blocks,
                                                            uint8_t* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  const int nb = n / QK_K;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long blk = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; blk < n_blocks;
       blk += nwarps) {
    const long long t = blk / nb;
    const int b = static_cast<int>(blk - t * nb);
    const float4* src = reinterpret_cast<const float4*>(x + t * n + static_cast<long long>(b) * QK_K + lane * 8);
    const float4 v0 = src[0], v1 = src[1];
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    int q[8];
    int gsum;
    const float d = warp_q8_k(v, q, &gsum);
    uint8_t* o8 = dst + blk * Q8_K_BYTES;
    uint32_t* o32 = reinterpret_cast<uint32_t*>(o8);  // Q8_K blocks are 4-byte aligned (292 = 4*73)
    o32[1 + lane * 2] = pack4_i8(q[0], q[1], q[2], q[3]);
    o32[2 + lane * 2] = pack4_i8(q[4], q[5], q[6], q[7]);
    if ((lane & 1) == 0) *reinterpret_cast<int16_t*>(o8 + 4 + QK_K + (lane >> 1) * 2) = static_cast<int16_t>(gsum);
    if (lane == 0) o32[0] = __float_as_uint(d);
  }
}

int grid_for(long long n_blocks) {
  long long warps = n_blocks;
  long long blocks = (warps + 7) / 8;  // 8 warps per 256-thread block
  if (blocks > 148 * 16) blocks = 148 * 16;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

}  // namespace

cudaError_t launch_quantize_q8_0(const float* x, int m, int n, uint8_t* dst, cudaStream_t st) {
  const long long nblk = static_cast<long long>(m) * (n / QK8_0);
  if (nblk <= 0) return cudaSuccess;
  quantize_q8_0_kernel<<<grid_for(nblk), 256, 0, st>>>(x, n, nblk, dst);
  return cudaGetLastError();
}

cudaError_t launch_quantize_q8_k(const float* x, int m, int n, uint8_t* dst, cudaStream_t st) {
  const long long nblk = static_cast<long long>(m) * (n / QK_K);
  if (nblk <= 0) return cudaSuccess;
  quantize_q8_k_kernel<<<grid_for(nblk), 256, 0, st>>>(x, n, nblk, dst);
  return cudaGetLastError();
}

}  // namespace ex
