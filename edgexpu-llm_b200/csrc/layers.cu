// layers.cu -- the non-matrix ops of a llama decoder layer on the device, restating the reference's
// CPU ops with their float operations:
//   RMSNorm          edgexpu_cpu_rmsnorm (src/cpu_kernel.c:220-242): ss = sum (double)x^2,
//                    mean = (float)(ss / n), scale = 1.0f / sqrtf(mean + eps), out = (x * scale) * w
//   residual add     edgexpu_cpu_add (cpu_kernel.c:200-208), fused into the norm that follows it
//   RoPE (norm)      edgexpu_cpu_rope_norm (cpu_kernel.c:707-737): adjacent pairs rotated by the
//                    cos/sin cache of rope_fill_cache (:659-669, computed on the host with the same
//                    libm calls), x0*c - x1*s and x0*s + x1*c without contraction (ISO C build)
//   attention        native.c:2545-2569: score_s = edgexpu_cpu_dot(q, k_s) * (1/sqrt(head_dim))
//                    (the AVX2 dot: 8 FMA lanes, then ((a0+a4)+(a1+a5))+((a2+a6)+(a3+a7))),
//                    edgexpu_cpu_softmax (:328-353), out = sum_s p_s v_s as the AVX2 saxpy's FMAs
//   SwiGLU           edgexpu_cpu_silu / _mul (:244-252, :210-218): g = (g / (1 + expf(-g))) * u
// exp is the host C library's expf, looked up in the table of exptab.cuh (the reference calls that
// expf).  The double sums run in a tree order rather than left to right; the float values they are
// rounded to are the same unless a sum lies within ~1e-16 (relative) of a float rounding boundary.
#include <cuda_runtime.h>

#include "common.cuh"
#include "exptab.cuh"
#include "launch.h"

namespace ex {

namespace {

constexpr int NORM_THREADS = 1024;
constexpr int ATTN_THREADS = 256;

__device__ __forceinline__ double cta_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    if (lane == 0) red[32] = v;
  }
  __syncthreads();
  const double r = red[32];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float cta_max_f(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    if (lane == 0) red[32] = v;
  }
  __syncthreads();
  const float r = red[32];
  __syncthreads();
  return r;
}

// One CTA.  hidden += add (when add != nullptr), then out = rmsnorm(hidden) * w.
__global__ void __launch_bounds__(NORM_THREADS) add_rmsnorm_kernel(float* hidden, const float* add, const float* w,
                                                                  float* out, int n, float eps) {
  __shared__ double red[33];
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float x = hidden[i];
    if (add != nullptr) {
      x = __fadd_rn(x, add[i]);
      hidden[i] = x;
    }
    ss += static_cast<double>(x) * static_cast<double>(x);
  }
  ss = cta_sum_d(ss, red);
  const float mean = static_cast<float>(ss / static_cast<double>(n));
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(hidden[i], scale), w[i]);
}

// Pairs (2j, 2j+1) of every q head rotated in place, of every k head rotated into the K cache
// slot; v copied into the V cache slot.  rope[2j] = cos, rope[2j+1] = sin of pair j at this position.
__global__ void rope_kv_kernel(float* q, const float* k, const float* v, const float* rope, int n_heads, int n_kv, int hd,
                               float* k_slot, float* v_slot) {
  const int half = hd / 2;
  const int nq = n_heads * half, nk = n_kv * half;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nq + nk; i += gridDim.x * blockDim.x) {
    const bool isq = i < nq;
    const int j = isq ? i : i - nq;
    const int head = j / half, pr = j - head * half;
    const float c = rope[2 * pr], s = rope[2 * pr + 1];
    const float* src = isq ? q : k;
    const int off = head * hd + 2 * pr;
    const float x0 = src[off], x1 = src[off + 1];
    const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    float* dst = isq ? q : k_slot;
    dst[off] = y0;
    dst[off + 1] = y1;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_kv * hd; i += gridDim.x * blockDim.x) v_slot[i] = v[i];
}

// One CTA per query head, for the query at position pos: scores over positions 0..pos of the
// head's KV group, softmax, and the weighted sum of the V rows.  Cache rows: [pos][n_kv][hd].
__global__ void __launch_bounds__(ATTN_THREADS) attention_kernel(const float* q, const float* kc, const float* vc, int pos,
                                                                int n_heads, int n_kv, int hd, float attn_scale,
                                                                float* out, ExpTab et) {
  extern __shared__ float sm[];
  float* qh = sm;        // [hd]
  float* p = sm + hd;    // [pos + 1]
  __shared__ double dred[33];
  __shared__ float fred[33];
  const int h = blockIdx.x, kvh = h / (n_heads / n_kv);
  for (int i = threadIdx.x; i < hd; i += blockDim.x) qh[i] = q[h * hd + i];
  __syncthreads();
  const int n8 = hd / 8 * 8;
  float m = -INFINITY;
  for (int s = threadIdx.x; s <= pos; s += blockDim.x) {
    const float* kr = kc + (static_cast<size_t>(s) * n_kv + kvh) * hd;
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int i = 0; i < n8; i += 8) {
#pragma unroll
      for (int l = 0; l < 8; ++l) a[l] = fmaf(qh[i + l], kr[i + l], a[l]);
    }
    float d = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[4]), __fadd_rn(a[1], a[5])),
                        __fadd_rn(__fadd_rn(a[2], a[6]), __fadd_rn(a[3], a[7])));
    for (int i = n8; i < hd; ++i) d = __fadd_rn(d, __fmul_rn(qh[i], kr[i]));
    const float sc = __fmul_rn(d, attn_scale);
    p[s] = sc;
    m = fmaxf(m, sc);
  }
  m = cta_max_f(m, fred);
  double sum = 0.0;
  for (int s = threadIdx.x; s <= pos; s += blockDim.x) {
    const float e = exp_lookup(et, __fsub_rn(p[s], m));
    p[s] = e;
    sum += static_cast<double>(e);
  }
  sum = cta_sum_d(sum, dred);
  if (sum > 0.0) {
    for (int s = threadIdx.x; s <= pos; s += blockDim.x) p[s] = static_cast<float>(static_cast<double>(p[s]) / sum);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.0f;
    const float* vr = vc + static_cast<size_t>(kvh) * hd + d;
    const size_t stride = static_cast<size_t>(n_kv) * hd;
    if (d < n8) {
      for (int s = 0; s <= pos; ++s) acc = fmaf(p[s], vr[s * stride], acc);
    } else {
      for (int s = 0; s <= pos; ++s) acc = __fadd_rn(acc, __fmul_rn(p[s], vr[s * stride]));
    }
    out[h * hd + d] = acc;
  }
}

__global__ void swiglu_kernel(float* g, const float* u, int n, ExpTab et) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float x = g[i];
    const float s = __fdiv_rn(x, __fadd_rn(1.0f, exp_lookup(et, -x)));
    g[i] = __fmul_rn(s, u[i]);
  }
}

}  // namespace

cudaError_t launch_add_rmsnorm(float* hidden, const float* add, const float* w, float* out, int n, float eps,
                               cudaStream_t st) {
  add_rmsnorm_kernel<<<1, NORM_THREADS, 0, st>>>(hidden, add, w, out, n, eps);
  return cudaGetLastError();
}

cudaError_t launch_rope_kv(float* q, const float* k, const float* v, const float* rope, int n_heads, int n_kv, int hd,
                           float* k_slot, float* v_slot, cudaStream_t st) {
  const int work = (n_heads + n_kv) * hd / 2;
  rope_kv_kernel<<<(work + 255) / 256, 256, 0, st>>>(q, k, v, rope, n_heads, n_kv, hd, k_slot, v_slot);
  return cudaGetLastError();
}

cudaError_t launch_attention(const float* q, const float* kc, const float* vc, int pos, int n_heads, int n_kv, int hd,
                             float attn_scale, float* out, const ExpTab& et, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(hd + pos + 1) * 4;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
  }
  attention_kernel<<<n_heads, ATTN_THREADS, smem, st>>>(q, kc, vc, pos, n_heads, n_kv, hd, attn_scale, out, et);
  return cudaGetLastError();
}

cudaError_t launch_swiglu(float* g, const float* u, int n, const ExpTab& et, cudaStream_t st) {
  swiglu_kernel<<<(n + 255) / 256 < 296 ? (n + 255) / 256 : 296, 256, 0, st>>>(g, u, n, et);
  return cudaGetLastError();
}

}  // namespace ex
