// rowstream.cu -- persistent weight-streaming GEMV for quantized GGUF rows on sm_100a.
//
// One kernel serves the reference's three hot dots (per output row o, per token t):
//   Q8_0 x Q8_0  out = bias + sum_b d_w*d_x*(sum_{j<32} qw*qx)          gguf_dot_q8.c:436-480
//   Q4_K x Q8_K  out = bias + sum_b d_x*d_w*sumi_b - d_x*dmin_w*summ_b     gguf_dot_q8.c:603-762
//   Q4_K x fp32  out = bias + sum_subblocks d*sc*sum(q*x) - dmin*m*sum(x)  gguf_quant.c:704-752
// and three epilogues: store rows (cpu_kernel.c:545-644), greedy argmax over rows
// (native.c:2355-2397), or per-block int32 partials (test hook for bit-exactness).
//
// Design (HBM-bound streaming):
//   * grid = one CTA per SM (persistent); CTA c takes tiles c, c+grid, ...; a tile is R whole
//     rows, i.e. one contiguous byte range of the row-major GGUF tensor.
//   * warp 0, lane 0 is the producer: it moves each tile into a ring of shared-memory stages
//     with a 1-D TMA bulk copy (cp.async.bulk, L2 evict-first hint) that completes on the
//     stage's "full" mbarrier.  Misaligned starts are rounded down to 16 bytes and the
//     in-stage offset is applied by the consumers.
//   * warps 1..8 are consumers: the quantized activations live in shared memory for the whole
//     kernel; each (row, block) work item is one thread; integer dots use dp4a; per-block
//     floats go to a small partials buffer and each row is summed in a fixed order
//     (deterministic results), then stored or folded into the argmax key.
//   * every mbarrier wait is bounded; a timeout sets a status bit, raises a CTA-wide abort
//     flag, and the producer still waits (bounded) for its in-flight copies before exiting.
#include <cstdio>

#include "common.cuh"
#include "launch.h"

namespace ex {
namespace {

constexpr int CONSUMER_WARPS = 8;
constexpr int CONSUMERS = CONSUMER_WARPS * 32;
constexpr int THREADS = CONSUMERS + 32;
constexpr int STAGE_TARGET = 16384;
constexpr int MAX_STAGES = 8;
constexpr int BAR_BYTES = 256;        // full[8], empty[8], abort flag
constexpr int ACT_BUDGET = 100 * 1024;
constexpr int STAGE_SLACK = 48;       // alignment round-down (<16) + over-read of the last block

struct Layout {
  int tile_rows;
  long long n_tiles;
  int stage_bytes;
  int n_stages;
  int act_off;
  int part_off;
  int part_stride;  // floats per partials buffer
  int stage_off;
  int smem_total;
};

__device__ __forceinline__ int blocks_per_row(Fmt f, int K) { return f == Fmt::Q8_0xQ8_0 ? K / QK8_0 : K / QK_K; }

// Bounded mbarrier wait that also gives up as soon as another thread raised the abort flag.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31u) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > WAIT_LIMIT_NS) return false;
    }
  }
}

// ---- activation prologue: quantized (or fp32) activations -> shared memory -------------------

__device__ void load_act(const RowStreamArgs& a, uint8_t* act, int ct) {
  const int K = a.K;
  if (a.fmt == Fmt::Q8_0xQ8_0) {
    const int nb = K / QK8_0;
    int8_t* xs = reinterpret_cast<int8_t*>(act);
    float* xd = reinterpret_cast<float*>(act + ((a.m * K + 15) & ~15));
    const uint8_t* src = static_cast<const uint8_t*>(a.act);
    const int total = a.m * nb * 17;  // 17 half-words per 34-byte block
    for (int i = ct; i < total; i += CONSUMERS) {
      const int t = i / (nb * 17);
      const int rem = i - t * nb * 17;
      const int b = rem / 17, hw = rem - b * 17;
      const uint16_t v = *reinterpret_cast<const uint16_t*>(src + static_cast<size_t>(t) * a.act_row_bytes +
                                                            b * Q8_0_BYTES + hw * 2);
      if (hw == 0) {
        xd[t * nb + b] = fp16_bits_to_float(v);
      } else {
        *reinterpret_cast<uint16_t*>(xs + t * K + b * QK8_0 + (hw - 1) * 2) = v;
      }
    }
  } else if (a.fmt == Fmt::Q4_KxQ8_K) {
    const int nb = K / QK_K;
    int8_t* xs = reinterpret_cast<int8_t*>(act);
    float* xd = reinterpret_cast<float*>(act + a.m * K);
    int* xbs = reinterpret_cast<int*>(act + a.m * K + ((a.m * nb * 4 + 15) & ~15));
    const uint8_t* src = static_cast<const uint8_t*>(a.act);
    const int total = a.m * nb * 73;  // 73 words per 292-byte block
    for (int i = ct; i < total; i += CONSUMERS) {
      const int t = i / (nb * 73);
      const int rem = i - t * nb * 73;
      const int b = rem / 73, wi = rem - b * 73;
      const uint32_t v = *reinterpret_cast<const uint32_t*>(src + static_cast<size_t>(t) * a.act_row_bytes +
                                                            b * Q8_K_BYTES + wi * 4);
      if (wi == 0) {
        xd[t * nb + b] = __uint_as_float(v);
      } else if (wi <= 64) {
        *reinterpret_cast<uint32_t*>(xs + t * K + b * QK_K + (wi - 1) * 4) = v;
      } else {
        const int lo = static_cast<int16_t>(v & 0xFFFFu), hi = static_cast<int16_t>(v >> 16);
        xbs[(t * nb + b) * 8 + (wi - 65)] = lo + hi;  // bsum of sub-block (wi-65): groups 2j, 2j+1
      }
    }
  } else {
    float* xf = reinterpret_cast<float*>(act);
    float* xsx = xf + a.m * K;
    const float* src = static_cast<const float*>(a.act);
    const int n4 = a.m * K / 4;
    for (int i = ct; i < n4; i += CONSUMERS) {
      reinterpret_cast<float4*>(xf)[i] = reinterpret_cast<const float4*>(src)[i];
    }
    const int nsub = a.m * K / 32;
    for (int i = ct; i < nsub; i += CONSUMERS) {
      const float4* p = reinterpret_cast<const float4*>(src + static_cast<size_t>(i) * 32);
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 v = p[j];
        s += v.x;
        s += v.y;
        s += v.z;
        s += v.w;
      }
      xsx[i] = s;
    }
  }
}

// ---- per-tile compute ------------------------------------------------------------------------

// Q8_0 weight block (34 B, only 2-byte aligned inside the stage) x Q8_0 activation block.
template <RowOut MODE>
__device__ __forceinline__ void tile_q8_0(const RowStreamArgs& a, const uint8_t* act, const uint8_t* tb, int nr,
                                          long long r0, float* pb, int part_stride, int ct) {
  const int K = a.K, nb = K / QK8_0, items = nr * nb;
  const int8_t* xs = reinterpret_cast<const int8_t*>(act);
  const float* xd = reinterpret_cast<const float*>(act + ((a.m * K + 15) & ~15));
  for (int item = ct; item < items; item += CONSUMERS) {
    const int r = item / nb, b = item - r * nb;
    const uint8_t* p = tb + static_cast<size_t>(r) * a.row_bytes + b * Q8_0_BYTES;
    const bool odd = (reinterpret_cast<uintptr_t>(p) & 2u) != 0;  // rows and blocks have even sizes
    const uint32_t* w = reinterpret_cast<const uint32_t*>(p - (odd ? 2 : 0));
    uint32_t wv[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) wv[i] = w[i];
    const uint32_t dbits = odd ? (wv[0] >> 16) : (wv[0] & 0xFFFFu);
    int q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = static_cast<int>(odd ? wv[i + 1] : __funnelshift_r(wv[i], wv[i + 1], 16));
    const float dw = fp16_bits_to_float(dbits);
    for (int t = 0; t < a.m; ++t) {
      const int4* xv = reinterpret_cast<const int4*>(xs + t * K + b * QK8_0);
      const int4 x0 = xv[0], x1 = xv[1];
      int ip = dp4a(q[0], x0.x, 0);
      ip = dp4a(q[1], x0.y, ip);
      ip = dp4a(q[2], x0.z, ip);
      ip = dp4a(q[3], x0.w, ip);
      ip = dp4a(q[4], x1.x, ip);
      ip = dp4a(q[5], x1.y, ip);
      ip = dp4a(q[6], x1.z, ip);
      ip = dp4a(q[7], x1.w, ip);
      if constexpr (MODE == RowOut::Partials) {
        a.partials[(static_cast<size_t>(t) * a.n_rows + r0 + r) * nb + b] = ip;
      } else {
        // gguf_dot_q8.c:475-476: d_w * d_x * (float)ip
        pb[t * part_stride + r * nb + b] = (dw * xd[t * nb + b]) * static_cast<float>(ip);
      }
    }
  }
}

// Unpack the four 6-bit (scale, min) pairs of sub-blocks 4h..4h+3 (get_scale_min_k4,
// gguf_quant.c:212-220) from the 12 scale bytes held as words s0, s1, s2.
__device__ __forceinline__ void q4k_scales_half(uint32_t s0, uint32_t s1, uint32_t s2, int h, uint32_t& sc4,
                                                uint32_t& mn4) {
  if (h == 0) {
    sc4 = s0 & 0x3F3F3F3Fu;
    mn4 = s1 & 0x3F3F3F3Fu;
  } else {
    sc4 = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
    mn4 = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
  }
}

// Q4_K weight x Q8_K activation.  A work item is half a super-block (4 sub-blocks, 64 quant
// bytes); the two halves of a super-block sit in adjacent lanes and are combined in int32
// before the float step, so every per-block int32 (sumi, summ) equals the reference's.
template <RowOut MODE>
__device__ __forceinline__ void tile_q4k_q8k(const RowStreamArgs& a, const uint8_t* act, const uint8_t* tb, int nr,
                                             long long r0, float* pb, int part_stride, int ct) {
  const int K = a.K, nb = K / QK_K, U = 2 * nb, items = nr * U;
  const int lane = ct & 31;
  const int8_t* xs = reinterpret_cast<const int8_t*>(act);
  const float* xd = reinterpret_cast<const float*>(act + a.m * K);
  const int* xbs = reinterpret_cast<const int*>(act + a.m * K + ((a.m * nb * 4 + 15) & ~15));
  for (int base = ct - lane; base < items; base += CONSUMERS) {
    const int item = base + lane;
    const bool live = item < items;
    int r = 0, sb = 0, h = 0;
    uint4 hdr = make_uint4(0, 0, 0, 0);
    uint32_t qw[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) qw[i] = 0;
    if (live) {
      r = item / U;
      const int u = item - r * U;
      sb = u >> 1;
      h = u & 1;
      const uint8_t* blk = tb + static_cast<size_t>(r) * a.row_bytes + sb * Q4_K_BYTES;
      hdr = *reinterpret_cast<const uint4*>(blk);
      const uint4* qp = reinterpret_cast<const uint4*>(blk + 16 + 64 * h);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = qp[i];
        qw[4 * i + 0] = v.x;
        qw[4 * i + 1] = v.y;
        qw[4 * i + 2] = v.z;
        qw[4 * i + 3] = v.w;
      }
    }
    uint32_t sc4, mn4;
    q4k_scales_half(hdr.y, hdr.z, hdr.w, h, sc4, mn4);
    const float dw = fp16_bits_to_float(hdr.x), dmw = fp16_bits_to_float(hdr.x >> 16);
    for (int t = 0; t < a.m; ++t) {
      int sumi = 0, summ = 0;
      if (live) {
        const int4* xv = reinterpret_cast<const int4*>(xs + t * K + sb * QK_K + 128 * h);
        int ip[4] = {0, 0, 0, 0};
#pragma unroll
        for (int g = 0; g < 2; ++g) {  // quant group 2h+g: low nibbles -> ip[2g], high -> ip[2g+1]
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int4 xl = xv[4 * g + c];      // elements 64g + 16c .. +16 (low-nibble sub-block)
            const int4 xh = xv[4 * g + 2 + c];  // elements 64g + 32 + 16c .. +16 (high-nibble sub-block)
            const uint32_t w0 = qw[8 * g + 4 * c + 0], w1 = qw[8 * g + 4 * c + 1];
            const uint32_t w2 = qw[8 * g + 4 * c + 2], w3 = qw[8 * g + 4 * c + 3];
            ip[2 * g] = dp4a(static_cast<int>(w0 & 0x0F0F0F0Fu), xl.x, ip[2 * g]);
            ip[2 * g] = dp4a(static_cast<int>(w1 & 0x0F0F0F0Fu), xl.y, ip[2 * g]);
            ip[2 * g] = dp4a(static_cast<int>(w2 & 0x0F0F0F0Fu), xl.z, ip[2 * g]);
            ip[2 * g] = dp4a(static_cast<int>(w3 & 0x0F0F0F0Fu), xl.w, ip[2 * g]);
            ip[2 * g + 1] = dp4a(static_cast<int>((w0 >> 4) & 0x0F0F0F0Fu), xh.x, ip[2 * g + 1]);
            ip[2 * g + 1] = dp4a(static_cast<int>((w1 >> 4) & 0x0F0F0F0Fu), xh.y, ip[2 * g + 1]);
            ip[2 * g + 1] = dp4a(static_cast<int>((w2 >> 4) & 0x0F0F0F0Fu), xh.z, ip[2 * g + 1]);
            ip[2 * g + 1] = dp4a(static_cast<int>((w3 >> 4) & 0x0F0F0F0Fu), xh.w, ip[2 * g + 1]);
          }
        }
        const int4 bs = *reinterpret_cast<const int4*>(xbs + (t * nb + sb) * 8 + 4 * h);
        sumi = static_cast<int>(sc4 & 0xFFu) * ip[0] + static_cast<int>((sc4 >> 8) & 0xFFu) * ip[1] +
               static_cast<int>((sc4 >> 16) & 0xFFu) * ip[2] + static_cast<int>(sc4 >> 24) * ip[3];
        summ = static_cast<int>(mn4 & 0xFFu) * bs.x + static_cast<int>((mn4 >> 8) & 0xFFu) * bs.y +
               static_cast<int>((mn4 >> 16) & 0xFFu) * bs.z + static_cast<int>(mn4 >> 24) * bs.w;
      }
      sumi += __shfl_xor_sync(0xFFFFFFFFu, sumi, 1);
      summ += __shfl_xor_sync(0xFFFFFFFFu, summ, 1);
      if (live && h == 0) {
        if constexpr (MODE == RowOut::Partials) {
          int32_t* pp = a.partials + ((static_cast<size_t>(t) * a.n_rows + r0 + r) * nb + sb) * 2;
          pp[0] = sumi;
          pp[1] = summ;
        } else {
          // gguf_dot_q8.c:619-620 and :640/:661: d = d_x*d_w, dmin = -d_x*dmin_w per super-block.
          const float dx = xd[t * nb + sb];
          pb[t * part_stride + r * nb + sb] = (dx * dw) * static_cast<float>(sumi) - (dx * dmw) * static_cast<float>(summ);
        }
      }
    }
  }
}

__device__ __forceinline__ float nib_f(uint32_t masked, int k) {
  // byte k of a word whose bytes are 0..15, as an exact float: 2^23 + v, minus 2^23.
  return __uint_as_float(__byte_perm(masked, 0x4B000000u, 0x7440u | static_cast<uint32_t>(k))) - 8388608.0f;
}

// Q4_K weight x fp32 activation (the reference's logits path for non-Q8_0 weights).
template <RowOut MODE>
__device__ __forceinline__ void tile_q4k_f32(const RowStreamArgs& a, const uint8_t* act, const uint8_t* tb, int nr,
                                             float* pb, int part_stride, int ct) {
  const int K = a.K, nb = K / QK_K, U = 2 * nb, items = nr * U;
  const int lane = ct & 31;
  const float* xf = reinterpret_cast<const float*>(act);
  const float* xsx = xf + a.m * K;
  for (int base = ct - lane; base < items; base += CONSUMERS) {
    const int item = base + lane;
    const bool live = item < items;
    int r = 0, sb = 0, h = 0;
    uint4 hdr = make_uint4(0, 0, 0, 0);
    uint32_t qw[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) qw[i] = 0;
    if (live) {
      r = item / U;
      const int u = item - r * U;
      sb = u >> 1;
      h = u & 1;
      const uint8_t* blk = tb + static_cast<size_t>(r) * a.row_bytes + sb * Q4_K_BYTES;
      hdr = *reinterpret_cast<const uint4*>(blk);
      const uint4* qp = reinterpret_cast<const uint4*>(blk + 16 + 64 * h);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = qp[i];
        qw[4 * i + 0] = v.x;
        qw[4 * i + 1] = v.y;
        qw[4 * i + 2] = v.z;
        qw[4 * i + 3] = v.w;
      }
    }
    uint32_t sc4, mn4;
    q4k_scales_half(hdr.y, hdr.z, hdr.w, h, sc4, mn4);
    const float dw = fp16_bits_to_float(hdr.x), dmw = fp16_bits_to_float(hdr.x >> 16);
    for (int t = 0; t < a.m; ++t) {
      float acc = 0.0f;
      if (live) {
        const float* xr = xf + t * K + sb * QK_K + 128 * h;
        const float* sx = xsx + t * (K / 32) + sb * 8 + 4 * h;
#pragma unroll
        for (int s = 0; s < 4; ++s) {  // sub-block 4h+s: group 2h+(s>>1), nibble half (s&1)
          float qx = 0.0f;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t mw = (qw[8 * (s >> 1) + i] >> (4 * (s & 1))) & 0x0F0F0F0Fu;
            const float4 xv = *reinterpret_cast<const float4*>(xr + 32 * s + 4 * i);
            qx = fmaf(nib_f(mw, 0), xv.x, qx);
            qx = fmaf(nib_f(mw, 1), xv.y, qx);
            qx = fmaf(nib_f(mw, 2), xv.z, qx);
            qx = fmaf(nib_f(mw, 3), xv.w, qx);
          }
          const float d1 = dw * static_cast<float>((sc4 >> (8 * s)) & 0xFFu);
          const float m1 = dmw * static_cast<float>((mn4 >> (8 * s)) & 0xFFu);
          acc += d1 * qx - m1 * sx[s];  // gguf_quant.c:744/746
        }
      }
      acc += __shfl_xor_sync(0xFFFFFFFFu, acc, 1);
      if (live && h == 0) pb[t * part_stride + r * nb + sb] = acc;
    }
  }
}

// ---- the kernel ---------------------------------------------------------------------------------

template <Fmt F, RowOut MODE>
__global__ void __launch_bounds__(THREADS, 1) rowstream_kernel(const RowStreamArgs a, const Layout L) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + MAX_STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 2 * MAX_STAGES * 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = L.n_stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CONSUMER_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane != 0) return;
    // ---------------- producer ----------------
    const uint64_t pol = l2_evict_first_policy();
    long long it = 0;
    for (long long tile = blockIdx.x; tile < L.n_tiles; tile += gridDim.x, ++it) {
      const int s = static_cast<int>(it % S);
      if (it >= S) {
        if (!wait_or_abort(&empty[s], static_cast<uint32_t>((it / S - 1) & 1), abort_flag)) {
          atomicOr(a.status, ST_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
      }
      const long long r0 = tile * L.tile_rows;
      const long long nr = min(static_cast<long long>(L.tile_rows), a.n_rows - r0);
      const uintptr_t start = reinterpret_cast<uintptr_t>(a.w) + static_cast<uintptr_t>(r0) * a.row_bytes;
      const uintptr_t al = start & ~static_cast<uintptr_t>(15);
      const uint32_t bytes = static_cast<uint32_t>((start - al + nr * a.row_bytes + 15) & ~15ull);
      mbar_arrive_expect_tx(&full[s], bytes);
      bulk_g2s(smem + L.stage_off + s * L.stage_bytes, reinterpret_cast<const void*>(al), bytes, &full[s], pol);
    }
    // Drain: the last copies issued into each stage must land before the CTA may exit.
    for (long long j = (it > S ? it - S : 0); j < it; ++j) {
      if (!mbar_wait(&full[j % S], static_cast<uint32_t>((j / S) & 1))) atomicOr(a.status, ST_TIMEOUT_DRAIN);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int ct = threadIdx.x - 32;
  const int cw = ct >> 5;
  uint8_t* act = smem + L.act_off;
  float* part = reinterpret_cast<float*>(smem + L.part_off);
  load_act(a, act, ct);
  named_bar_sync(1, CONSUMERS);

  const int nb = blocks_per_row(F, a.K);
  unsigned long long best = 0ull;
  bool dead = false;
  long long it = 0;
  for (long long tile = blockIdx.x; tile < L.n_tiles; tile += gridDim.x, ++it) {
    const int s = static_cast<int>(it % S);
    if (!dead && !wait_or_abort(&full[s], static_cast<uint32_t>((it / S) & 1), abort_flag)) {
      atomicOr(a.status, ST_TIMEOUT_FULL);
      *abort_flag = 1;
      dead = true;
    }
    const long long r0 = tile * L.tile_rows;
    const int nr = static_cast<int>(min(static_cast<long long>(L.tile_rows), a.n_rows - r0));
    float* pb = part + (it & 1) * L.part_stride;
    if (!dead) {
      const uintptr_t start = reinterpret_cast<uintptr_t>(a.w) + static_cast<uintptr_t>(r0) * a.row_bytes;
      const uint8_t* tb = smem + L.stage_off + s * L.stage_bytes + (start & 15u);
      if constexpr (F == Fmt::Q8_0xQ8_0) {
        tile_q8_0<MODE>(a, act, tb, nr, r0, pb, L.tile_rows * nb, ct);
      } else if constexpr (F == Fmt::Q4_KxQ8_K) {
        tile_q4k_q8k<MODE>(a, act, tb, nr, r0, pb, L.tile_rows * nb, ct);
      } else {
        tile_q4k_f32<MODE>(a, act, tb, nr, pb, L.tile_rows * nb, ct);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if constexpr (MODE != RowOut::Partials) {
      named_bar_sync(1, CONSUMERS);
      if (!dead) {
        for (int r = cw; r < nr; r += CONSUMER_WARPS) {
          for (int t = 0; t < a.m; ++t) {
            float v = 0.0f;
            for (int b = lane; b < nb; b += 32) v += pb[t * L.tile_rows * nb + r * nb + b];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
            if (lane == 0) {
              const long long row = r0 + r;
              const float y = (a.bias != nullptr ? a.bias[row] : 0.0f) + v;  // cpu_kernel.c:596-597
              if constexpr (MODE == RowOut::Store) {
                a.out[static_cast<size_t>(t) * a.out_stride + row] = y;
              } else {
                const unsigned long long k = argmax_key(y, static_cast<uint32_t>(a.row0 + row));
                best = k > best ? k : best;
              }
            }
          }
        }
      }
    }
  }
  if constexpr (MODE == RowOut::Argmax) {
    if (lane == 0 && best != 0ull) atomicMax(a.key, best);
  }
}

template <Fmt F, RowOut MODE>
cudaError_t launch_impl(const RowStreamArgs& a, const Layout& L, int grid, cudaStream_t st) {
  static int configured_smem = 0;  // per instantiation; the host API is single-threaded per process
  auto kern = rowstream_kernel<F, MODE>;
  if (L.smem_total > configured_smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem_total);
    if (e != cudaSuccess) return e;
    configured_smem = L.smem_total;
  }
  kern<<<grid, THREADS, L.smem_total, st>>>(a, L);
  return cudaGetLastError();
}

int act_bytes_per_row(Fmt f, int K) {
  switch (f) {
    case Fmt::Q8_0xQ8_0:
      return K + 4 * (K / QK8_0);
    case Fmt::Q4_KxQ8_K:
      return K + 4 * (K / QK_K) + 32 * (K / QK_K);
    default:
      return 4 * K + 4 * (K / 32);
  }
}

int act_bytes_total(Fmt f, int K, int m) {
  if (f == Fmt::Q8_0xQ8_0) return ((m * K + 15) & ~15) + m * (K / QK8_0) * 4;
  if (f == Fmt::Q4_KxQ8_K) return m * K + ((m * (K / QK_K) * 4 + 15) & ~15) + m * (K / QK_K) * 32;
  return 4 * m * K + 4 * m * (K / 32);
}

}  // namespace

int rowstream_max_m(Fmt fmt, int K, const DeviceInfo& dev) {
  (void)dev;
  const int per = act_bytes_per_row(fmt, K) + 64;
  return per > ACT_BUDGET ? 0 : ACT_BUDGET / per;
}

cudaError_t launch_rowstream(const RowStreamArgs& a, const DeviceInfo& dev, cudaStream_t st) {
  if (a.n_rows <= 0 || a.m <= 0) return cudaSuccess;
  const int nb = a.fmt == Fmt::Q8_0xQ8_0 ? a.K / QK8_0 : a.K / QK_K;
  Layout L{};
  L.stage_bytes = STAGE_TARGET;
  if (a.row_bytes + STAGE_SLACK > L.stage_bytes) L.stage_bytes = (a.row_bytes + STAGE_SLACK + 127) & ~127;
  const int r_cap = (L.stage_bytes - STAGE_SLACK) / a.row_bytes;
  long long r_want = (a.n_rows + 4LL * dev.sm_count - 1) / (4LL * dev.sm_count);
  if (r_want < 1) r_want = 1;
  L.tile_rows = static_cast<int>(r_want < r_cap ? r_want : r_cap);
  const int act = (act_bytes_total(a.fmt, a.K, a.m) + 127) & ~127;
  L.act_off = BAR_BYTES;
  L.part_off = L.act_off + act;
  int S = 0;
  for (;;) {  // shrink the tile until the partials buffer leaves room for >= 2 stages
    L.part_stride = a.m * L.tile_rows * nb;
    const int part = (2 * L.part_stride * 4 + 127) & ~127;
    L.stage_off = L.part_off + part;
    S = (dev.max_smem_optin - L.stage_off) / L.stage_bytes;
    if (S >= 2 || L.tile_rows == 1) break;
    L.tile_rows = (L.tile_rows + 1) / 2;
  }
  L.n_tiles = (a.n_rows + L.tile_rows - 1) / L.tile_rows;
  if (S > MAX_STAGES) S = MAX_STAGES;
  if (S < 2) return cudaErrorInvalidConfiguration;
  L.n_stages = S;
  L.smem_total = L.stage_off + S * L.stage_bytes;
  const int grid = static_cast<int>(L.n_tiles < dev.sm_count ? L.n_tiles : dev.sm_count);

#define EX_DISPATCH_MODE(FMT)                                                 \
  switch (a.mode) {                                                           \
    case RowOut::Store:                                                       \
      return launch_impl<FMT, RowOut::Store>(a, L, grid, st);                 \
    case RowOut::Argmax:                                                      \
      return launch_impl<FMT, RowOut::Argmax>(a, L, grid, st);                \
    default:                                                                  \
      return launch_impl<FMT, RowOut::Partials>(a, L, grid, st);              \
  }
  switch (a.fmt) {
    case Fmt::Q8_0xQ8_0:
      EX_DISPATCH_MODE(Fmt::Q8_0xQ8_0)
    case Fmt::Q4_KxQ8_K:
      EX_DISPATCH_MODE(Fmt::Q4_KxQ8_K)
    default:
      switch (a.mode) {
        case RowOut::Store:
          return launch_impl<Fmt::Q4_KxF32, RowOut::Store>(a, L, grid, st);
        case RowOut::Argmax:
          return launch_impl<Fmt::Q4_KxF32, RowOut::Argmax>(a, L, grid, st);
        default:
          return cudaErrorInvalidValue;
      }
  }
#undef EX_DISPATCH_MODE
}

}  // namespace ex
