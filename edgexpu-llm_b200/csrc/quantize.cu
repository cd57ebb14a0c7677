// quantize.cu -- fp32 -> Q8_0 / Q8_K activation quantizers for sm_100a.
//
// Bit-exact with the reference's x86 Release build:
//   Q8_0: src/gguf_dot_q8.c:276-324 (AVX2 + F16C): d = amax/127 rounded to fp16 with
//         round-to-nearest-even, id = 127/amax, q = round-half-even(x*id) saturated to int8.
//   Q8_K: src/gguf_dot_q8.c:360-412: scale from the SIGNED first element of largest |x|,
//         iscale = -127/maxv, q = lrint(iscale*x) clamped to +-127, int16 bsums per 16,
//         d = 1/iscale; all-zero blocks are written as zeros.
// Divisions and products use the IEEE-rounded intrinsics (no fused multiply-add, no fast math),
// so every intermediate equals the CPU's single-precision result.
#include "common.cuh"
#include "launch.h"

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
    const float v = x[t * n + static_cast<long long>(b) * QK8_0 + lane];
    float a = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
    const float d = __fdiv_rn(a, 127.0f);
    const float id = a != 0.0f ? __fdiv_rn(127.0f, a) : 0.0f;
    const float r = rintf(__fmul_rn(v, id));
    int q;
    if (!(r >= -128.0f)) {
      q = -128;  // also NaN: the SIMD convert yields INT_MIN, which packs saturates to -128
    } else {
      q = r > 127.0f ? 127 : static_cast<int>(r);
    }
    uint8_t* o8 = dst + blk * Q8_0_BYTES;
    o8[2 + lane] = static_cast<uint8_t>(static_cast<int8_t>(q));
    if (lane == 0) *reinterpret_cast<unsigned short*>(o8) = __half_as_ushort(__float2half_rn(d));
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

    // First index of the largest |x| (strict '>' from 0, as gguf_dot_q8.c:377-383).
    float am = 0.0f;
    int ai = 0x7FFFFFFF;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float ax = fabsf(v[i]);
      if (ax > am) {
        am = ax;
        ai = lane * 8 + i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float oam = __shfl_xor_sync(0xFFFFFFFFu, am, o);
      const int oai = __shfl_xor_sync(0xFFFFFFFFu, ai, o);
      if (oam > am || (oam == am && oai < ai)) {
        am = oam;
        ai = oai;
      }
    }
    uint8_t* o8 = dst + blk * Q8_K_BYTES;
    uint32_t* o32 = reinterpret_cast<uint32_t*>(o8);  // Q8_K blocks are 4-byte aligned (292 = 4*73)
    if (am == 0.0f) {
      for (int w = lane; w < Q8_K_BYTES / 4; w += 32) o32[w] = 0u;
      continue;
    }
    float mine = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (lane * 8 + i == ai) mine = v[i];
    const float maxv = __shfl_sync(0xFFFFFFFFu, mine, ai >> 3);
    const float iscale = __fdiv_rn(-127.0f, maxv);
    int q[8];
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int qi = static_cast<int>(rintf(__fmul_rn(iscale, v[i])));
      qi = qi > 127 ? 127 : (qi < -127 ? -127 : qi);
      q[i] = qi;
      s += qi;
    }
    s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);  // the 16-element group of lanes (2g, 2g+1)
    uint32_t p0 = 0, p1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      p0 |= (static_cast<uint32_t>(q[i]) & 0xFFu) << (8 * i);
      p1 |= (static_cast<uint32_t>(q[4 + i]) & 0xFFu) << (8 * i);
    }
    o32[1 + lane * 2] = p0;
    o32[2 + lane * 2] = p1;
    if ((lane & 1) == 0) {
      *reinterpret_cast<int16_t*>(o8 + 4 + QK_K + (lane >> 1) * 2) = static_cast<int16_t>(s);
    }
    if (lane == 0) {
      const float d = __fdiv_rn(1.0f, iscale);
      o32[0] = __float_as_uint(d);
    }
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
