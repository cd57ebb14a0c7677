// dequant.cu -- element-wise decoding of GGUF weight rows on the device, for the parts of the
// reference's quant API that are not the streamed matrix product:
//   * row dequantization to fp32 (edgexpu_gguf_dequantize_row, gguf_quant.c:428-466: the token
//     embedding gather of native.c:428-443), for a batch of row ids in one launch;
//   * the fp32-activation dot of any supported type (edgexpu_gguf_dot_quant, gguf_quant.c:894-918),
//     the linear of F16/F32 weights, which the reference routes to that dot
//     (cpu_kernel.c:565-568, :633-643), and the greedy logits of F16/F32 output weights
//     (logit_dot_row, native.c:445-462).
// One element is decoded with the reference's own float expression per type (gguf_quant.c:139-353),
// so a dequantized row is bit-identical to the reference's.  These calls are small next to the
// streamed projections; they read bytes one at a time and are not tuned for bandwidth.
#include "common.cuh"
#include "launch.h"

namespace ex {
namespace {

__device__ __forceinline__ float ld_fp16(const uint8_t* p) {
  return fp16_bits_to_float(static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8));
}

// 6-bit scale and min of sub-block j (0..7) from the 12 packed bytes (get_scale_min_k4,
// gguf_quant.c:212-220).
__device__ __forceinline__ void scale_min_k4(const uint8_t* q, int j, int& sc, int& mn) {
  if (j < 4) {
    sc = q[j] & 63;
    mn = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// Element e of a row of `type`, as the reference's dequantizer computes it.
__device__ float weight_elem(uint32_t type, const uint8_t* row, int e) {
  switch (type) {
    case TYPE_F32: {
      const uint8_t* p = row + 4 * e;
      return __uint_as_float(static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) |
                             (static_cast<uint32_t>(p[2]) << 16) | (static_cast<uint32_t>(p[3]) << 24));
    }
    case TYPE_F16:
      return ld_fp16(row + 2 * e);
    case TYPE_Q8_0: {  // d * (float)q (:139-155)
      const uint8_t* b = row + (e / QK8_0) * Q8_0_BYTES;
      return ld_fp16(b) * static_cast<float>(static_cast<int8_t>(b[2 + e % QK8_0]));
    }
    case TYPE_Q4_0: {  // ((float)nibble - 8.0f) * d (:193-210)
      const uint8_t* b = row + (e / QK8_0) * Q4_0_BYTES;
      const int j = e % QK8_0;
      const int q = j < 16 ? (b[2 + j] & 0xF) : (b[2 + j - 16] >> 4);
      return (static_cast<float>(q) - 8.0f) * ld_fp16(b);
    }
    case TYPE_Q5_0: {  // (float)(q - 16) * d (:157-181)
      const uint8_t* b = row + (e / QK8_0) * Q5_0_BYTES;
      const int j = e % QK8_0;
      const uint32_t qh = static_cast<uint32_t>(b[2]) | (static_cast<uint32_t>(b[3]) << 8) |
                          (static_cast<uint32_t>(b[4]) << 16) | (static_cast<uint32_t>(b[5]) << 24);
      const int nib = j < 16 ? (b[6 + j] & 0xF) : (b[6 + j - 16] >> 4);
      return static_cast<float>((nib | static_cast<int>(((qh >> j) & 1u) << 4)) - 16) * ld_fp16(b);
    }
    case TYPE_Q4_K:
    case TYPE_Q5_K: {  // d1 * (float)q - m1, d1 = d * sc, m1 = dmin * m (:223-266, :305-353)
      const bool q5 = type == TYPE_Q5_K;
      const uint8_t* b = row + (e / QK_K) * (q5 ? Q5_K_BYTES : Q4_K_BYTES);
      const int j = e % QK_K, g = j / 64, l = j % 64;
      int sc, mn;
      scale_min_k4(b + 4, j / 32, sc, mn);
      const uint8_t* ql = b + (q5 ? 48 : 16) + 32 * g;
      int q = l < 32 ? (ql[l] & 0xF) : (ql[l - 32] >> 4);
      if (q5) q += ((b[16 + (l & 31)] >> (2 * g + (l >= 32 ? 1 : 0))) & 1) << 4;
      const float d1 = ld_fp16(b) * static_cast<float>(sc), m1 = ld_fp16(b + 2) * static_cast<float>(mn);
      return d1 * static_cast<float>(q) - m1;
    }
    case TYPE_Q6_K: {  // d * (float)sc * (float)q (:269-303)
      const uint8_t* b = row + (e / QK_K) * Q6_K_BYTES;
      const int j = e % QK_K, n = j / 128, r = j % 128, qq = r / 32, l = r % 32;
      const uint8_t lo = (qq & 1) ? b[64 * n + l + 32] : b[64 * n + l];
      const int nib = (qq & 2) ? (lo >> 4) : (lo & 0xF);
      const int q = (nib | (((b[128 + 32 * n + l] >> (2 * qq)) & 3) << 4)) - 32;
      return ld_fp16(b + 208) * static_cast<float>(static_cast<int8_t>(b[192 + j / 16])) * static_cast<float>(q);
    }
    default:
      return __int_as_float(0x7FC00000);
  }
}

// out[i][e] = element e of row ids[i] (row i when ids is null).  An id outside [0, n_rows) gives a
// NaN row and sets ST_BAD_INDEX.
__global__ void __launch_bounds__(256) dequant_rows_kernel(uint32_t type, const uint8_t* __restrict__ w,
                                                           long long row_bytes, long long n_rows,
                                                           const int32_t* __restrict__ ids, int n_ids, int n,
                                                           float* __restrict__ out, uint32_t* status) {
  const long long total = static_cast<long long>(n_ids) * n;
  for (long long k = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; k < total;
       k += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(k / n), e = static_cast<int>(k - static_cast<long long>(i) * n);
    const long long r = ids != nullptr ? ids[i] : i;
    if (r < 0 || r >= n_rows) {
      out[k] = __int_as_float(0x7FC00000);
      if (e == 0) atomicOr(status, ST_BAD_INDEX);
      continue;
    }
    out[k] = weight_elem(type, w + r * row_bytes, e);
  }
}

// One warp per (token t, row o): out[t*n_out + o] = bias[o] + sum_e w_oe * x_te (fp32 activations).
__global__ void __launch_bounds__(256) dot_f32_kernel(uint32_t type, const uint8_t* __restrict__ w, long long row_bytes,
                                                      int n_out, int n, const float* __restrict__ x, int m,
                                                      const float* __restrict__ bias, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long pairs = static_cast<long long>(m) * n_out;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long p = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; p < pairs; p += nwarps) {
    const int t = static_cast<int>(p / n_out), o = static_cast<int>(p - static_cast<long long>(t) * n_out);
    const uint8_t* row = w + o * row_bytes;
    const float* xt = x + static_cast<long long>(t) * n;
    float acc = 0.0f;
    for (int e = lane; e < n; e += 32) acc = fmaf(weight_elem(type, row, e), xt[e], acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, off);
    if (lane == 0) out[p] = (bias != nullptr ? bias[o] : 0.0f) + acc;
  }
}

// Greedy key of scores[0, n): max over argmax_key(score_i, row0 + i) (the lowest id wins ties).
__global__ void __launch_bounds__(256) argmax_key_kernel(const float* __restrict__ scores, int n, long long row0,
                                                         unsigned long long* key) {
  unsigned long long best = 0ull;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned long long k = argmax_key(scores[i], static_cast<uint32_t>(row0 + i));
    best = k > best ? k : best;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, best, off);
    best = o > best ? o : best;
  }
  if ((threadIdx.x & 31) == 0 && best != 0ull) atomicMax(key, best);
}

int blocks_for(long long threads) {
  long long b = (threads + 255) / 256;
  if (b > 148 * 16) b = 148 * 16;
  return static_cast<int>(b < 1 ? 1 : b);
}

}  // namespace

cudaError_t launch_argmax_key(const float* scores, int n, long long row0, unsigned long long* key, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  argmax_key_kernel<<<blocks_for(n), 256, 0, st>>>(scores, n, row0, key);
  return cudaGetLastError();
}

cudaError_t launch_dequant_rows(uint32_t type, const uint8_t* w, size_t row_bytes, long long n_rows,
                                const int32_t* ids, int n_ids, int n, float* out, uint32_t* status, cudaStream_t st) {
  if (n_ids <= 0 || n <= 0) return cudaSuccess;
  dequant_rows_kernel<<<blocks_for(static_cast<long long>(n_ids) * n), 256, 0, st>>>(
      type, w, static_cast<long long>(row_bytes), n_rows, ids, n_ids, n, out, status);
  return cudaGetLastError();
}

cudaError_t launch_dot_f32(uint32_t type, const uint8_t* w, size_t row_bytes, int n_out, int n, const float* x, int m,
                           const float* bias, float* out, cudaStream_t st) {
  if (n_out <= 0 || m <= 0) return cudaSuccess;
  dot_f32_kernel<<<blocks_for(static_cast<long long>(n_out) * m * 32), 256, 0, st>>>(
      type, w, static_cast<long long>(row_bytes), n_out, n, x, m, bias, out);
  return cudaGetLastError();
}

}  // namespace ex
