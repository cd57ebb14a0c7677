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

// Every kernel here is launched as a programmatic dependent of the kernel before it (the decode
// step is one chain of them): it lets its own dependent launch at once, so that kernel's CTAs are
// placed (and a following GEMV starts streaming its weights) while this one runs, and then waits
// until the previous grid has completed before touching memory.  Every block passes the wait
// before it can exit, so this grid's completion implies its predecessors'.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

constexpr int NORM_THREADS = 1024;
constexpr int NORM_PER_THREAD = NORM_MAX_N / NORM_THREADS;
constexpr int V_CHUNK = 64;  // V rows staged in shared memory at a time by the softmax/V kernel
constexpr int V_LD = V_CHUNK * 256 / 4 / 256;  // float4 loads per thread per chunk (head_dim <= 256, 256 threads)

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

// One CTA.  hidden += add (when add != nullptr), then out = rmsnorm(hidden) * w.  Thread t holds
// elements t, t + blockDim, ... (at most NORM_PER_THREAD) in registers for both passes; its
// partial sum of squares runs over them in that order.
__global__ void __launch_bounds__(NORM_THREADS) add_rmsnorm_kernel(float* hidden, const float* add, const float* w,
                                                                  float* out, int n, float eps) {
  pdl_enter();
  __shared__ double red[33];
  float xv[NORM_PER_THREAD], wv[NORM_PER_THREAD];
#pragma unroll
  for (int k = 0; k < NORM_PER_THREAD; ++k) {  // every load of the kernel issued up front
    const int i = threadIdx.x + k * NORM_THREADS;
    xv[k] = 0.0f;
    wv[k] = 0.0f;
    if (i < n) {
      xv[k] = hidden[i];
      wv[k] = w[i];
      if (add != nullptr) xv[k] = __fadd_rn(xv[k], add[i]);
    }
  }
  double ss = 0.0;
#pragma unroll
  for (int k = 0; k < NORM_PER_THREAD; ++k) {
    const int i = threadIdx.x + k * NORM_THREADS;
    if (i < n) {
      if (add != nullptr) hidden[i] = xv[k];
      ss += static_cast<double>(xv[k]) * static_cast<double>(xv[k]);
    }
  }
  ss = cta_sum_d(ss, red);
  const float mean = static_cast<float>(ss / static_cast<double>(n));
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
#pragma unroll
  for (int k = 0; k < NORM_PER_THREAD; ++k) {
    const int i = threadIdx.x + k * NORM_THREADS;
    if (i < n) out[i] = __fmul_rn(__fmul_rn(xv[k], scale), wv[k]);
  }
}

// RoPE and attention scores of the query at position pos = step[1] (rope_all[pos*hd + 2j] = cos,
// [.. + 2j+1] = sin of pair j): score[h][s] = dot(rot(q_h), K[s][h/rep]) * scale for s = 0..pos.
// Each block rotates its head's q pairs (x0*c - x1*s, x0*s + x1*c, unfused) into shared memory; a
// block that covers pos rotates k of its kv head the same way and uses it for s = pos, and the
// first head of each kv group writes that row and v into the caches (the softmax/V kernel reads
// them after this grid).  Eight lanes share a position: lane l runs the AVX2 dot's FMA lane l
// (elements l, l+8, ...), and the eight lanes are combined in that dot's order.
// grid = (n_heads, ceil(window/32)); blocks past pos return at once.  Cache layout per layer:
// [kv head][window][hd].
__global__ void __launch_bounds__(256) attn_scores_kernel(const float* q, const float* k, const float* v,
                                                          const float* rope_all, float* kc, float* vc, const int* step,
                                                          int window, int n_heads, int n_kv, int hd, float attn_scale,
                                                          float* scores, int ld) {
  pdl_enter();
  __shared__ float qr[256], kp[256];  // hd <= 256
  const int pos = step[1];
  if (static_cast<int>(blockIdx.y) * 32 > pos) return;
  const int h = blockIdx.x, rep = n_heads / n_kv, kvh = h / rep;
  const bool covers_pos = static_cast<int>(blockIdx.y) == pos / 32;
  const float* rope = rope_all + static_cast<size_t>(pos) * hd;
  for (int e = threadIdx.x; e < hd; e += blockDim.x) {
    const int j2 = e & ~1;
    const float c = rope[j2], sn = rope[j2 + 1];
    const float x0 = q[static_cast<size_t>(h) * hd + j2], x1 = q[static_cast<size_t>(h) * hd + j2 + 1];
    qr[e] = (e & 1) ? __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c)) : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
    if (covers_pos) {
      const float y0 = k[static_cast<size_t>(kvh) * hd + j2], y1 = k[static_cast<size_t>(kvh) * hd + j2 + 1];
      const float kr = (e & 1) ? __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, c)) : __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, sn));
      kp[e] = kr;
      if (h % rep == 0) {
        const size_t row = (static_cast<size_t>(kvh) * window + pos) * hd + e;
        kc[row] = kr;
        vc[row] = v[static_cast<size_t>(kvh) * hd + e];
      }
    }
  }
  __syncthreads();
  const int l = threadIdx.x & 7;
  const int s = blockIdx.y * 32 + (threadIdx.x >> 3);
  const int n8 = hd / 8 * 8;
  const bool live = s <= pos;
  const float* kr = s == pos ? kp : kc + (static_cast<size_t>(kvh) * window + (live ? s : 0)) * hd;
  float a = 0.0f;
  for (int i = l; i < n8; i += 8) a = fmaf(qr[i], kr[i], a);
  // ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)) within each group of eight lanes
  const float a4 = __shfl_down_sync(0xFFFFFFFFu, a, 4, 8);
  const float b = __fadd_rn(a, a4);              // lane l < 4: a_l + a_{l+4}
  const float b1 = __shfl_down_sync(0xFFFFFFFFu, b, 1, 8);
  const float c = __fadd_rn(b, b1);              // lane 0: b0 + b1, lane 2: b2 + b3
  const float c2 = __shfl_down_sync(0xFFFFFFFFu, c, 2, 8);
  if (l == 0 && live) {
    float d = __fadd_rn(c, c2);
    for (int i = n8; i < hd; ++i) d = __fadd_rn(d, __fmul_rn(qr[i], kr[i]));
    scores[static_cast<size_t>(h) * ld + s] = __fmul_rn(d, attn_scale);
  }
}

// Softmax of score[h][0..pos] and out[h][d] = sum_s p_s * V[s][h/rep][d] (the saxpy's FMAs in s
// order).  One CTA per head; the V rows come through shared memory V_CHUNK at a time, loaded by
// every thread, and one thread per output element d runs its FMA chain over them.
__global__ void __launch_bounds__(256) attn_softmax_v_kernel(const float* scores, int ld, const float* vc, const int* step,
                                                             int window, int n_heads, int n_kv, int hd, float* out,
                                                             ExpTab et) {
  pdl_enter();
  extern __shared__ float p[];  // [window], then V_CHUNK rows of hd at vs
  const int pos = step[1];
  float* vs = p + ((window + 3) & ~3);
  __shared__ double dred[33];
  __shared__ float fred[33];
  const int h = blockIdx.x, kvh = h / (n_heads / n_kv);
  const float* sc = scores + static_cast<size_t>(h) * ld;
  float m = -INFINITY;
  for (int s = threadIdx.x; s <= pos; s += blockDim.x) {
    const float v = sc[s];
    p[s] = v;
    m = fmaxf(m, v);
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
  const int n8 = hd / 8 * 8;
  // this head's V rows are contiguous: chunk c is V_CHUNK * hd floats at vbase + c * V_CHUNK * hd;
  // each thread holds up to V_LD float4 of the next chunk in registers while the current one is
  // used (hd % 4 == 0).
  const float4* vbase = reinterpret_cast<const float4*>(vc + static_cast<size_t>(kvh) * window * hd);
  float4* vs4 = reinterpret_cast<float4*>(vs);
  const int d = threadIdx.x;  // blockDim.x >= hd
  float acc = 0.0f;
  float4 nxt[V_LD];
  auto fetch = [&](int s0) {
    const int n4 = min(V_CHUNK, pos + 1 - s0) * hd / 4;
    const float4* src = vbase + static_cast<size_t>(s0) * hd / 4;
#pragma unroll
    for (int u = 0; u < V_LD; ++u) {
      const int i = threadIdx.x + u * static_cast<int>(blockDim.x);
      if (i < n4) nxt[u] = src[i];
    }
  };
  fetch(0);
  for (int s0 = 0; s0 <= pos; s0 += V_CHUNK) {
    const int n = min(V_CHUNK, pos + 1 - s0);
    __syncthreads();  // the previous chunk has been used (and p is complete on the first pass)
#pragma unroll
    for (int u = 0; u < V_LD; ++u) {
      const int i = threadIdx.x + u * static_cast<int>(blockDim.x);
      if (i < n * hd / 4) vs4[i] = nxt[u];
    }
    __syncthreads();
    if (s0 + V_CHUNK <= pos) fetch(s0 + V_CHUNK);
    if (d < n8) {
      for (int r = 0; r < n; ++r) acc = fmaf(p[s0 + r], vs[r * hd + d], acc);
    } else if (d < hd) {
      for (int r = 0; r < n; ++r) acc = __fadd_rn(acc, __fmul_rn(p[s0 + r], vs[r * hd + d]));
    }
  }
  if (d < hd) out[h * hd + d] = acc;
}

__global__ void swiglu_kernel(float* g, const float* u, int n, ExpTab et) {
  pdl_enter();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float x = g[i];
    const float s = __fdiv_rn(x, __fadd_rn(1.0f, exp_lookup(et, -x)));
    g[i] = __fmul_rn(s, u[i]);
  }
}

// The token id and position of the next forward step, for the kernels that read them.
__global__ void set_step_kernel(int* step, int token, int pos) {
  step[0] = token;
  step[1] = pos;
}

}  // namespace

cudaError_t launch_add_rmsnorm(float* hidden, const float* add, const float* w, float* out, int n, float eps,
                               cudaStream_t st) {
  if (n > NORM_THREADS * NORM_PER_THREAD) return cudaErrorInvalidValue;
  return launch_pdl(add_rmsnorm_kernel, dim3(1), dim3(NORM_THREADS), 0, st, hidden, add, w, out, n, eps);
}

cudaError_t launch_set_step(int* step, int token, int pos, cudaStream_t st) {
  set_step_kernel<<<1, 1, 0, st>>>(step, token, pos);
  return cudaGetLastError();
}

size_t attention_smem_bytes(int window, int hd) {
  return (static_cast<size_t>((window + 3) & ~3) + static_cast<size_t>(V_CHUNK) * hd) * 4;
}

cudaError_t launch_attention(const float* q, const float* k, const float* v, const float* rope, float* kc, float* vc,
                             const int* step, int window, int n_heads, int n_kv, int hd, float attn_scale, float* scores,
                             int ld, float* out, const ExpTab& et, cudaStream_t st) {
  if (window > ld || hd % 4 != 0 || hd > 256) return cudaErrorInvalidValue;
  cudaError_t e = launch_pdl(attn_scores_kernel, dim3(n_heads, (window + 31) / 32), dim3(256), 0, st, q, k, v, rope, kc, vc,
                             step, window, n_heads, n_kv, hd, attn_scale, scores, ld);
  if (e != cudaSuccess) return e;
  if (hd > 256) return cudaErrorInvalidValue;
  const size_t smem = attention_smem_bytes(window, hd);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  return launch_pdl(attn_softmax_v_kernel, dim3(n_heads), dim3(256), smem, st, scores, ld, vc, step, window, n_heads, n_kv,
                    hd, out, et);
}

cudaError_t prepare_attention(int window, int hd) {
  return cudaFuncSetAttribute(attn_softmax_v_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(attention_smem_bytes(window, hd)));
}

cudaError_t launch_swiglu(float* g, const float* u, int n, const ExpTab& et, cudaStream_t st) {
  return launch_pdl(swiglu_kernel, dim3((n + 255) / 256 < 296 ? (n + 255) / 256 : 296), dim3(256), 0, st, g, u, n, et);
}

}  // namespace ex
