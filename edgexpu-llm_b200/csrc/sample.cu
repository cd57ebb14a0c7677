// sample.cu -- temperature sampling over the logits on the device: the reference's
// edgexpu_cpu_sample_softmax (src/cpu_kernel.c:762-849) after the logits loop of
// sample_next_token (src/native.c:2322-2353).
//
//   softmax (cpu_kernel.c:328-353):  x_i = score_i / temperature; m = max x; e_i = expf(x_i - m);
//                                    s = sum e_i (double); p_i = (float)((double)e_i / s)
//   draw (cpu_kernel.c:780-785):     xorshift64 (13, 7, 17) of the caller's state, on the host;
//                                    u = (state & 0xFFFFFFF) / 2^28
//   top_p in (0, 1) (:787-830):      order by p descending, ties by id ascending; keep the shortest
//                                    prefix whose double sum reaches top_p; pick = u * (its sum);
//                                    the first kept id whose running sum reaches pick
//   otherwise (:832-847):            pick = u * sum p; the first id (ascending) whose running sum
//                                    reaches pick
// The sums run in double like the reference's, but in a fixed tree order rather than left to
// right, and e_i comes from a double-precision exp rounded to float (glibc's expf is within 0.502
// ulp, so the two agree except where the exact value sits next to a rounding boundary).  The
// chosen id can therefore differ from the reference's only when the pick lands within ~1e-7 of a
// running-sum boundary.  The descending sort is CUB's stable radix sort of the float keys with the
// ids as values (ties keep ascending ids).
#include <cuda_runtime.h>

#include <cub/device/device_radix_sort.cuh>

#include "common.cuh"
#include "launch.h"

namespace ex {

namespace {

constexpr int SM_THREADS = 1024;

__device__ __forceinline__ double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = lane < (blockDim.x >> 5) ? red[lane] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    if (lane == 0) red[32] = v;
  }
  __syncthreads();
  return red[32];
}

// One CTA: x_i = io_i / temperature (temperature > 0), softmax in place, sum of the result
// (the reference's `sum` of the untruncated branch) into *total.
__global__ void __launch_bounds__(SM_THREADS) softmax_kernel(float* io, int n, float temperature, double* stats) {
  __shared__ float fred[32];
  __shared__ double red[33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float x = temperature > 0.0f ? __fdiv_rn(io[i], temperature) : io[i];
    io[i] = x;
    m = fmaxf(m, x);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  if (lane == 0) fred[w] = m;
  __syncthreads();
  if (w == 0) {
    float v = lane < (blockDim.x >> 5) ? fred[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    if (lane == 0) fred[0] = v;
  }
  __syncthreads();
  m = fred[0];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float e = static_cast<float>(exp(static_cast<double>(__fsub_rn(io[i], m))));
    io[i] = e;
    s += static_cast<double>(e);
  }
  const double sum = block_sum_d(s, red);
  double t = 0.0;
  if (sum > 0.0) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float p = static_cast<float>(static_cast<double>(io[i]) / sum);
      io[i] = p;
      t += static_cast<double>(p);
    }
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) t += static_cast<double>(io[i]);
  }
  const double total = block_sum_d(t, red);
  if (threadIdx.x == 0) {
    stats[0] = sum;
    stats[1] = total;
  }
}

// One CTA over p[0 .. n) in order.  Thread t owns the contiguous chunk [t*per, (t+1)*per); the
// running sum at index i is (the sum of the earlier chunks) + (the chunk's terms up to i), all in
// double, in that fixed order.
struct Scan {
  const float* p;
  int n, lo, hi;
  double* pre;  // [blockDim.x] exclusive chunk prefixes
  int* first;
  double* val;

  __device__ void build() {
    double cs = 0.0;
    for (int i = lo; i < hi; ++i) cs += static_cast<double>(p[i]);
    pre[threadIdx.x] = cs;
    __syncthreads();
    if (threadIdx.x == 0) {
      double run = 0.0;
      for (int c = 0; c < static_cast<int>(blockDim.x); ++c) {
        const double v = pre[c];
        pre[c] = run;
        run += v;
      }
    }
    __syncthreads();
  }
  // First index < end whose running sum reaches target (end if none).
  __device__ int first_reach(int end, double target) {
    if (threadIdx.x == 0) *first = end;
    __syncthreads();
    double run = pre[threadIdx.x];
    for (int i = lo; i < min(hi, end); ++i) {
      run += static_cast<double>(p[i]);
      if (run >= target) {
        atomicMin(first, i);
        break;
      }
    }
    __syncthreads();
    const int f = *first;
    __syncthreads();
    return f;
  }
  // Running sum through index idx (0 <= idx < n).
  __device__ double through(int idx) {
    if (idx >= lo && idx < hi) {
      double run = pre[threadIdx.x];
      for (int i = lo; i <= idx; ++i) run += static_cast<double>(p[i]);
      *val = run;
    }
    __syncthreads();
    const double v = *val;
    __syncthreads();
    return v;
  }
};

// ids == nullptr: p in id order, no truncation (cpu_kernel.c:832-847).  Otherwise p sorted
// descending with its ids, truncated at top_p (cpu_kernel.c:787-830).  u = the draw in [0, 1).
__global__ void __launch_bounds__(SM_THREADS) prefix_pick_kernel(const float* p, const uint32_t* ids, int n, float top_p,
                                                                 double u, uint32_t* out, double* stats) {
  __shared__ double pre[SM_THREADS];
  __shared__ int first;
  __shared__ double val;
  const int per = (n + blockDim.x - 1) / blockDim.x;
  Scan sc{p, n, min(n, static_cast<int>(threadIdx.x) * per), min(n, static_cast<int>(threadIdx.x) * per + per), pre, &first,
          &val};
  sc.build();
  int limit = n;
  if (ids != nullptr) {
    const int f = sc.first_reach(n, static_cast<double>(top_p));
    limit = f < n ? f + 1 : n;
  }
  const double limit_sum = sc.through(limit - 1);
  if (!(limit_sum > 0.0)) {  // cpu_kernel.c:818-822 (the first kept id) and :836-839 (id 0)
    if (threadIdx.x == 0) {
      *out = ids != nullptr ? ids[0] : 0u;
      stats[2] = limit_sum;
      stats[3] = static_cast<double>(limit);
    }
    return;
  }
  const int f = sc.first_reach(limit, u * limit_sum);
  if (threadIdx.x == 0) {
    const int k = f < limit ? f : limit - 1;  // no crossing: the last candidate
    *out = ids != nullptr ? ids[k] : static_cast<uint32_t>(k);
    stats[2] = limit_sum;
    stats[3] = static_cast<double>(limit);
  }
}

__global__ void iota_kernel(uint32_t* ids, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) ids[i] = static_cast<uint32_t>(i);
}

}  // namespace

size_t sample_scratch_bytes(int n) {
  size_t sort_tmp = 0;
  cub::DeviceRadixSort::SortPairsDescending(nullptr, sort_tmp, static_cast<const float*>(nullptr),
                                            static_cast<float*>(nullptr), static_cast<const uint32_t*>(nullptr),
                                            static_cast<uint32_t*>(nullptr), n);
  // sorted keys, ids in and out, stats, sort temporaries
  return ((static_cast<size_t>(n) * 12 + 255) & ~static_cast<size_t>(255)) + 256 + sort_tmp + 256;
}

cudaError_t launch_sample(float* io, int n, float temperature, float top_p, double u, void* scratch, size_t scratch_bytes,
                          uint32_t* out_dev, double* stats_dev, cudaStream_t st) {
  softmax_kernel<<<1, SM_THREADS, 0, st>>>(io, n, temperature, stats_dev);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (top_p > 0.0f && top_p < 1.0f) {
    uint8_t* base = static_cast<uint8_t*>(scratch);
    float* keys_out = reinterpret_cast<float*>(base);
    uint32_t* ids_in = reinterpret_cast<uint32_t*>(base + static_cast<size_t>(n) * 4);
    uint32_t* ids_out = reinterpret_cast<uint32_t*>(base + static_cast<size_t>(n) * 8);
    const size_t used = ((static_cast<size_t>(n) * 12 + 255) & ~static_cast<size_t>(255)) + 256;
    size_t tmp = scratch_bytes - used;
    iota_kernel<<<(n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024, 256, 0, st>>>(ids_in, n);
    e = cub::DeviceRadixSort::SortPairsDescending(base + used, tmp, io, keys_out, ids_in, ids_out, n, 0, 32, st);
    if (e != cudaSuccess) return e;
    prefix_pick_kernel<<<1, SM_THREADS, 0, st>>>(keys_out, ids_out, n, top_p, u, out_dev, stats_dev);
  } else {
    prefix_pick_kernel<<<1, SM_THREADS, 0, st>>>(io, nullptr, n, top_p, u, out_dev, stats_dev);
  }
  return cudaGetLastError();
}

}  // namespace ex
