// quant.cuh -- warp-cooperative activation quantizers shared by the standalone quantize kernels
// and the prologue of the row-stream GEMV, so both produce the same bits.
//
// Bit-exact with the reference's x86 Release build:
//   Q8_0: src/gguf_dot_q8.c:276-324 (AVX2 + F16C): d = amax/127 rounded to fp16 with
//         round-to-nearest-even, id = 127/amax, q = round-half-even(x*id) saturated to int8.
//   Q8_K: src/gguf_dot_q8.c:360-412: scale from the SIGNED first element of largest |x|,
//         iscale = -127/maxv, q = lrint(iscale*x) clamped to +-127, int16 bsums per 16,
//         d = 1/iscale; all-zero blocks are written as zeros.
// Divisions and products use the IEEE-rounded intrinsics (no fused multiply-add, no fast math),
// so every intermediate equals the CPU's single-precision result.
#pragma once

#include "common.cuh"

namespace ex {

// Q8_0 block of 32: lane i holds x_i.  Returns q_i; *dbits gets the fp16 bits of d.
__device__ __forceinline__ int warp_q8_0(float v, uint32_t* dbits) {
  float a = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
  const float d = __fdiv_rn(a, 127.0f);
  const float id = a != 0.0f ? __fdiv_rn(127.0f, a) : 0.0f;
  const float r = rintf(__fmul_rn(v, id));
  *dbits = __half_as_ushort(__float2half_rn(d));
  if (!(r >= -128.0f)) return -128;  // also NaN: the SIMD convert gives INT_MIN, packs saturates to -128
  return r > 127.0f ? 127 : static_cast<int>(r);
}

// Q8_K block of 256: lane i holds elements 8i .. 8i+7 in v.  Fills q (clamped int8 values) and
// returns d (0 for an all-zero block, whose q are then all 0).  *gsum16 gets the sum of the
// 16-element group (lanes 2g, 2g+1) -- the reference's int16 bsum.
__device__ __forceinline__ float warp_q8_k(const float (&v)[8], int (&q)[8], int* gsum16) {
  const int lane = threadIdx.x & 31;
  float am = 0.0f;
  int ai = 0x7FFFFFFF;
#pragma unroll
  for (int i = 0; i < 8; ++i) {  // first index of the largest |x| (strict '>' from 0)
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
  if (am == 0.0f) {
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = 0;
    *gsum16 = 0;
    return 0.0f;
  }
  float mine = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (lane * 8 + i == ai) mine = v[i];
  const float maxv = __shfl_sync(0xFFFFFFFFu, mine, ai >> 3);
  const float iscale = __fdiv_rn(-127.0f, maxv);
  int s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int qi = static_cast<int>(rintf(__fmul_rn(iscale, v[i])));
    qi = qi > 127 ? 127 : (qi < -127 ? -127 : qi);
    q[i] = qi;
    s += qi;
  }
  *gsum16 = s + __shfl_xor_sync(0xFFFFFFFFu, s, 1);
  return __fdiv_rn(1.0f, iscale);
}

__device__ __forceinline__ uint32_t pack4_i8(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

}  // namespace ex
