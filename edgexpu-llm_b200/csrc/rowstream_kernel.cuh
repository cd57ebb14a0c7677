// rowstream_kernel.cuh -- persistent weight-streaming GEMV for quantized GGUF rows on sm_100a
// (the kernel template; rowstream.cu and rowstream_more.cu instantiate it).
//
// One kernel serves the reference's three hot dots (per output row o, per token t):
//   Q8_0 x Q8_0  out = bias + sum_b d_w*d_x*(sum_{j<32} qw*qx)          gguf_dot_q8.c:436-480
//   Q4_K x Q8_K  out = bias + sum_b d_x*d_w*sumi_b - d_x*dmin_w*summ_b     gguf_dot_q8.c:603-762
//   Q4_K x fp32  out = bias + sum_subblocks d*sc*sum(q*x) - dmin*m*sum(x)  gguf_quant.c:704-752
// and three epilogues: store rows (cpu_kernel.c:545-644), greedy argmax over rows
// (native.c:2355-2397), or per-block int32 partials (test hook for bit-exactness).
//
// Design (HBM-bound streaming, batch 1-16):
//   * grid = one CTA per SM (persistent); CTA c takes tiles c, c+grid, ...; a tile is R whole
//     rows, i.e. one contiguous byte range (up to 32 KB) of the row-major GGUF tensor.
//   * warp 0, lane 0 is the producer: it moves each tile into a ring of shared-memory stages
//     with a 1-D TMA bulk copy (cp.async.bulk, L2 evict-first hint) that completes on the
//     stage's "full" mbarrier.  Misaligned starts are rounded down to 16 bytes and the
//     in-stage offset is applied by the consumers.  The producer starts streaming weights at
//     once; only the consumers depend on the activations.
//   * warps 1..15 are consumers.  They first bring the activations into shared memory: for
//     small batches they quantize the fp32 rows themselves (Q8_0 / Q8_K, same arithmetic as the
//     standalone quantizer), otherwise they copy pre-quantized GGUF blocks.  The layout is
//     "unit-interleaved": 16-byte chunk j of work unit u of token t sits at (t*J + j)*U + u, so
//     the lanes of a warp, which hold consecutive units, read consecutive chunks.
//   * rows are dealt round-robin over the consumer warps along the CTA's tile sequence; a warp
//     computes a whole row (lane = work unit: a Q8_0 block or half a Q4_K super-block; integer
//     dots use dp4a), sums its lanes with a fixed shuffle tree (deterministic results), stores
//     the row or folds it into the argmax key, and releases a stage once done with its rows in
//     it.  No CTA-wide barrier sits in the loop, so warps overlap each other's latency.
//   * every mbarrier wait is bounded; a timeout sets a status bit, raises a CTA-wide abort
//     flag, and the producer still waits (bounded) for its in-flight copies before exiting.
#pragma once

#include "common.cuh"
#include "launch.h"
#include "quant.cuh"

namespace ex {

// Launch geometry, computed by launch_rowstream (rowstream.cu) and passed to every instantiation.
struct Layout {
  int tile_rows;
  long long n_tiles;
  int stage_bytes;
  int n_stages;
  int act_off;
  int stage_off;
  int smem_total;
  int row_stride;  // bytes between rows in a stage: row_bytes, or padded (each row its own copy)
  int part_off;    // sliced rows: per-(stage, row) slice partials and arrival counters
};

// Launches the formats of the other GGUF types (rowstream_more.cu).
cudaError_t launch_rowstream_more(const RowStreamArgs& a, const Layout& L, int grid, cudaStream_t st);

// Q4_K rows longer than one warp pass (K > 4096) at batch 1 in the relaxed order run sliced: each
// consumer warp keeps 16 units' activations in registers and computes that slice of two rows at
// a time (rowstream_kernel, SLICE).  At most 15 slices: K <= 30720.
inline bool rowstream_sliced(const RowStreamArgs& a) {
  const int U = a.K / 128;
  return a.fmt == Fmt::Q4_KxQ8_K && a.m == 1 && !a.exact && (a.mode == RowOut::Store || a.mode == RowOut::Argmax) &&
         U > 32 && (U + 15) / 16 <= 15;
}

namespace {

constexpr int CONSUMER_WARPS = 15;  // + 1 producer warp = 16 warps, 4 per SM sub-partition (128 registers each)
constexpr int CONSUMERS = CONSUMER_WARPS * 32;
constexpr int THREADS = CONSUMERS + 32;
#ifndef EX_RS_STAGE
#define EX_RS_STAGE 32768
#endif
constexpr int STAGE_TARGET = EX_RS_STAGE;
constexpr int MAX_STAGES = 16;
constexpr int BAR_BYTES = 1024;       // full[16], empty[16], abort flag, xin barrier; tile descriptors[16] at 512
constexpr int DESC_OFF = 512;
constexpr int ACT_BUDGET = 96 * 1024;
constexpr int STAGE_SLACK = 48;       // alignment round-down (<16) + over-read of the last block
constexpr int MAX_M = 16;             // activation rows (tokens) per launch; the host splits more
constexpr int PROLOGUE_QUANT_MAX_M = 2;
constexpr int PRO_BATCH = 4;          // activation blocks a consumer warp loads before quantizing them
constexpr int SLICE_UNITS = 16;       // sliced rows: units per slice (half a warp)
#ifndef EX_RS_PRE
#define EX_RS_PRE 2
#endif
constexpr int PRE_STAGES = EX_RS_PRE;  // weight copies the producer issues before the activations land
constexpr unsigned long long HOLD_LIMIT_NS = 20000;  // the hold is a scheduling aid: give up after 20 us

// ---- activation layout in shared memory ----------------------------------------------------------
//   Q8_0 x Q8_0 : unit = block (U = K/32): q chunks (t*2 + j)*U + u, then d[t*U + u]
//   Q4_K x Q8_K : unit = half super-block (U = K/128): q chunks (t*8 + j)*U + u, then bsum chunks
//                 [t*U + u] (4 ints: sub-blocks 4h..4h+3), then d[t*(U/2) + sb], then the int16
//                 bsums of the unit's 8 groups of 16 [t*U + u][8] (the Q6_K exact-order path reads them)
//   Q4_K x fp32 : unit = half super-block: x chunks (t*32 + j)*U + u, then sum chunks [t*U + u]
//                 (4 floats: sub-block sums)
__host__ __device__ __forceinline__ int units_per_row(Fmt f, int K) { return act_of(f) == Act::Q8_0 ? K / QK8_0 : K / 128; }

// Byte offset of the int16 bsums of the Q8_K layout (16-byte aligned: they are read as 64-bit words).
__host__ __device__ __forceinline__ int xb16_off(int m, int U) { return (m * U * 144 + m * (U / 2) * 4 + 15) & ~15; }

__host__ __device__ __forceinline__ int act_bytes_total(Fmt f, int K, int m) {
  const int U = units_per_row(f, K);
  if (act_of(f) == Act::Q8_0) return m * U * 32 + m * U * 4;
  if (act_of(f) == Act::Q8_K) return xb16_off(m, U) + m * U * 16;
  return m * U * 512 + m * U * 16;
}

__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
  // unsigned bytes of a times signed bytes of b, accumulated into c
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Wait (at most HOLD_LIMIT_NS; nothing depends on it for correctness) until every consumer warp
// reported its activation loads landed.
__device__ __forceinline__ void hold_for_activations(uint64_t* xin) {
  if (mbar_try_wait(xin, 0)) return;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait_sleep(xin, 0, 1000u))
    if (global_ns() - t0 > HOLD_LIMIT_NS) return;
}

// ---- activation prologue ---------------------------------------------------------------------------

// Lane 0 of every consumer warp arrives once on `xin` when the warp's first activation loads
// have landed (or, on paths without a separate load phase, when it is done): the producer holds
// back all but its first PRE_STAGES weight copies until then, so the activations -- on the
// critical path of every launch -- do not queue behind a full ring of weights into the SM.
__device__ void load_act(const RowStreamArgs& a, uint8_t* act, int ct, uint64_t* xin) {
  bool arrived = false;
  const int K = a.K, m = a.m, lane = ct & 31, cw = ct >> 5;
  const int U = units_per_row(a.fmt, K);
  const Act kind = act_of(a.fmt);
  if (kind == Act::Q8_0) {
    int4* xq = reinterpret_cast<int4*>(act);
    float* xd = reinterpret_cast<float*>(act + m * U * 32);
    if (a.act_f32) {  // quantize in place: one warp per block (quant.cuh), loads of a batch issued first
      const float* x = static_cast<const float*>(a.act);
      const int nblk = m * U;
      for (int base = cw; base < nblk; base += PRO_BATCH * CONSUMER_WARPS) {
        float v[PRO_BATCH];
#pragma unroll
        for (int k = 0; k < PRO_BATCH; ++k) {
          const int blk = base + k * CONSUMER_WARPS;
          if (blk < nblk) {
            const int t = blk / U, b = blk - t * U;
            v[k] = x[static_cast<size_t>(t) * K + b * QK8_0 + lane];
          }
        }
#pragma unroll
        for (int k = 0; k < PRO_BATCH; ++k) {
          const int blk = base + k * CONSUMER_WARPS;
          if (blk < nblk) {  // warp-uniform
            const int t = blk / U, b = blk - t * U;
            uint32_t dbits;
            const int q = warp_q8_0(v[k], &dbits);
            // lane i holds element i: gather 4 consecutive lanes into one word
            const int q1 = __shfl_down_sync(0xFFFFFFFFu, q, 1), q2 = __shfl_down_sync(0xFFFFFFFFu, q, 2),
                      q3 = __shfl_down_sync(0xFFFFFFFFu, q, 3);
            if ((lane & 3) == 0) {
              reinterpret_cast<uint32_t*>(xq + (t * 2 + (lane >> 4)) * U + b)[(lane >> 2) & 3] = pack4_i8(q, q1, q2, q3);
            }
            if (lane == 0) xd[t * U + b] = fp16_bits_to_float(dbits);
          }
        }
      }
    } else {  // pre-quantized GGUF Q8_0 rows: 17 half-words per 34-byte block
      const uint8_t* src = static_cast<const uint8_t*>(a.act);
      for (int i = ct; i < m * U * 17; i += CONSUMERS) {
        const int t = i / (U * 17), rem = i - t * U * 17, b = rem / 17, hw = rem - b * 17;
        const uint16_t v = *reinterpret_cast<const uint16_t*>(src + static_cast<size_t>(t) * a.act_row_bytes +
                                                              b * Q8_0_BYTES + hw * 2);
        if (hw == 0) {
          xd[t * U + b] = fp16_bits_to_float(v);
        } else {
          const int e = (hw - 1) * 2;  // element offset inside the block
          reinterpret_cast<uint16_t*>(xq + (t * 2 + (e >> 4)) * U + b)[(e & 15) >> 1] = v;
        }
      }
    }
  } else if (kind == Act::Q8_K) {
    const int nb = U / 2;
    int4* xq = reinterpret_cast<int4*>(act);
    int* xb = reinterpret_cast<int*>(act + m * U * 128);
    float* xd = reinterpret_cast<float*>(act + m * U * 128 + m * U * 16);
    int16_t* xb16 = reinterpret_cast<int16_t*>(act + xb16_off(m, U));
    if (a.act_f32) {  // quantize in place: one warp per 256-block (quant.cuh), loads of a batch issued first
      const float* x = static_cast<const float*>(a.act);
      const int nblk = m * nb;
      for (int base = cw; base < nblk; base += PRO_BATCH * CONSUMER_WARPS) {
        float4 ld[PRO_BATCH][2];
#pragma unroll
        for (int k = 0; k < PRO_BATCH; ++k) {
          const int blk = base + k * CONSUMER_WARPS;
          if (blk < nblk) {
            const int t = blk / nb, sb = blk - t * nb;
            const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * K + sb * QK_K + lane * 8);
            ld[k][0] = src[0];
            ld[k][1] = src[1];
          }
        }
        if (!arrived) {  // the vote issues once every lane's first load has landed; the arrive after it
          const int seen = __any_sync(0xFFFFFFFFu, ld[0][0].x != ld[0][0].x);
          uint64_t* bar = xin;
          asm volatile("" : "+l"(bar) : "r"(seen));  // keeps the arrive after the vote
          if (lane == 0) mbar_arrive(bar);
          arrived = true;
        }
#pragma unroll
        for (int k = 0; k < PRO_BATCH; ++k) {
          const int blk = base + k * CONSUMER_WARPS;
          if (blk < nblk) {  // warp-uniform
            const int t = blk / nb, sb = blk - t * nb;
            const float v[8] = {ld[k][0].x, ld[k][0].y, ld[k][0].z, ld[k][0].w,
                                ld[k][1].x, ld[k][1].y, ld[k][1].z, ld[k][1].w};
            int q[8], gsum;
            const float d = warp_q8_k(v, q, &gsum);
            // lane l holds elements 8l..8l+7: unit h = l/16, chunk j = (l%16)/2, half (l&1)
            const int u = 2 * sb + (lane >> 4), j = (lane & 15) >> 1;
            uint2* dst = reinterpret_cast<uint2*>(xq + (t * 8 + j) * U + u) + (lane & 1);
            *dst = make_uint2(pack4_i8(q[0], q[1], q[2], q[3]), pack4_i8(q[4], q[5], q[6], q[7]));
            // sub-block (32 elements) sums: lanes 4s .. 4s+3 (gsum already covers lane pairs)
            const int s32 = gsum + __shfl_down_sync(0xFFFFFFFFu, gsum, 2);
            if ((lane & 3) == 0) xb[(t * U + u) * 4 + ((lane >> 2) & 3)] = s32;
            if ((lane & 1) == 0) xb16[(t * U + u) * 8 + ((lane >> 1) & 7)] = static_cast<int16_t>(gsum);
            if (lane == 0) xd[t * nb + sb] = d;
          }
        }
      }
    } else {  // pre-quantized GGUF Q8_K rows: 73 words per 292-byte block
      const uint8_t* src = static_cast<const uint8_t*>(a.act);
      for (int i = ct; i < m * nb * 73; i += CONSUMERS) {
        const int t = i / (nb * 73), rem = i - t * nb * 73, sb = rem / 73, wi = rem - sb * 73;
        const uint32_t v = *reinterpret_cast<const uint32_t*>(src + static_cast<size_t>(t) * a.act_row_bytes +
                                                              sb * Q8_K_BYTES + wi * 4);
        if (wi == 0) {
          xd[t * nb + sb] = __uint_as_float(v);
        } else if (wi <= 64) {
          const int e = (wi - 1) * 4;  // element offset inside the super-block
          const int u = 2 * sb + (e >> 7), j = (e & 127) >> 4;
          reinterpret_cast<uint32_t*>(xq + (t * 8 + j) * U + u)[(e & 15) >> 2] = v;
        } else {
          const int s = wi - 65;  // sub-block s: bsum groups 2s, 2s+1
          const int lo = static_cast<int16_t>(v & 0xFFFFu), hi = static_cast<int16_t>(v >> 16);
          xb[(t * U + 2 * sb + (s >> 2)) * 4 + (s & 3)] = lo + hi;
          xb16[(t * U + 2 * sb + (s >> 2)) * 8 + (s & 3) * 2] = static_cast<int16_t>(lo);
          xb16[(t * U + 2 * sb + (s >> 2)) * 8 + (s & 3) * 2 + 1] = static_cast<int16_t>(hi);
        }
      }
    }
  } else {  // fp32 activations for the Q4_K logits path
    const float* x = static_cast<const float*>(a.act);
    float4* xf = reinterpret_cast<float4*>(act);
    float* xs = reinterpret_cast<float*>(act + m * U * 512);
    for (int i = ct; i < m * U * 32; i += CONSUMERS) {  // i = source float4 index
      const int t = i / (U * 32), rem = i - t * U * 32, u = rem >> 5, j = rem & 31;
      xf[(t * 32 + j) * U + u] = reinterpret_cast<const float4*>(x)[i];
    }
    for (int i = ct; i < m * U * 4; i += CONSUMERS) {
      // Sub-block sums in the order of the reference's x86 build (dot_u4_f32_32, gguf_quant.c:545-565:
      // lane l adds elements l, l+8, l+16, l+24; hsum256 then sums the 8 lanes), which the exact-order
      // logits use as they are.
      const float4* p = reinterpret_cast<const float4*>(x + static_cast<size_t>(i) * 32);
      float4 q[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) q[k] = p[k];
      const float e[32] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w,
                           q[2].x, q[2].y, q[2].z, q[2].w, q[3].x, q[3].y, q[3].z, q[3].w,
                           q[4].x, q[4].y, q[4].z, q[4].w, q[5].x, q[5].y, q[5].z, q[5].w,
                           q[6].x, q[6].y, q[6].z, q[6].w, q[7].x, q[7].y, q[7].z, q[7].w};
      float v[8];
#pragma unroll
      for (int l = 0; l < 8; ++l) v[l] = ((e[l] + e[l + 8]) + e[l + 16]) + e[l + 24];
      const float s = ((v[0] + v[4]) + (v[1] + v[5])) + ((v[2] + v[6]) + (v[3] + v[7]));
      const int t = i / (U * 4), rem = i - t * U * 4;
      xs[(t * U + (rem >> 2)) * 4 + (rem & 3)] = s;
    }
  }
  if (!arrived) {
    __syncwarp();
    if (lane == 0) mbar_arrive(xin);
  }
}

// ---- per-row compute: one warp per row, lane = work unit ------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// Activations of one lane's work unit held in registers for the whole kernel.  Used when a
// single token is streamed and a row fits in one warp pass (U <= 32: Q8_0 K <= 1024, Q4_K K <= 4096):
// the lane then owns the same unit in every row, so its activation chunks never change.
struct XRegs {
  int4 q[8];        // Q8_K: the unit's 8 chunks; Q8_0: q[0..1]
  uint32_t sl, sh;  // Q8_K: 32-element sums S_j of the unit's 4 sub-blocks as 7-bit digits, S = 128*sh + sl
  float d;          // activation scale of the unit's block
};

__device__ __forceinline__ void load_xregs(Fmt f, const RowStreamArgs& a, const uint8_t* act, int lane, XRegs& xr) {
  const int U = units_per_row(f, a.K);
  xr.sl = xr.sh = 0u;
  xr.d = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) xr.q[j] = make_int4(0, 0, 0, 0);
  if (lane >= U) return;
  const int4* xq = reinterpret_cast<const int4*>(act);
  if (act_of(f) == Act::Q8_0) {
    xr.q[0] = xq[lane];
    xr.q[1] = xq[U + lane];
    xr.d = reinterpret_cast<const float*>(act + U * 32)[lane];
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) xr.q[j] = xq[j * U + lane];
    const int4 b = reinterpret_cast<const int4*>(act + U * 128)[lane];  // |S_j| <= 32 * 127
    xr.sl = pack4_i8(b.x & 127, b.y & 127, b.z & 127, b.w & 127);
    xr.sh = pack4_i8(b.x >> 7, b.y >> 7, b.z >> 7, b.w >> 7);
    xr.d = reinterpret_cast<const float*>(act + U * 128 + U * 16)[lane >> 1];
  }
}

// Q8_0 weight row x Q8_0 activations.  Blocks are 34 B, so inside the stage they are only
// 2-byte aligned: read the 9 covering words and realign.
template <RowOut MODE, int MTOK, bool XREG>
__device__ __forceinline__ void row_q8_0(const RowStreamArgs& a, const uint8_t* act, const uint8_t* rowp,
                                         long long row, float (&acc)[MTOK], int lane, const XRegs& xr) {
  const int U = a.K / QK8_0;
  const int4* xq = reinterpret_cast<const int4*>(act);
  const float* xd = reinterpret_cast<const float*>(act + a.m * U * 32);
  for (int b = lane; b < U; b += 32) {
    const uint8_t* p = rowp + b * Q8_0_BYTES;
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
#pragma unroll
    for (int t = 0; t < MTOK; ++t) {
      if (MTOK == 1 || t < a.m) {
        const int4 x0 = XREG ? xr.q[0] : xq[(t * 2) * U + b], x1 = XREG ? xr.q[1] : xq[(t * 2 + 1) * U + b];
        int ip = dp4a(q[0], x0.x, 0);
        ip = dp4a(q[1], x0.y, ip);
        ip = dp4a(q[2], x0.z, ip);
        ip = dp4a(q[3], x0.w, ip);
        ip = dp4a(q[4], x1.x, ip);
        ip = dp4a(q[5], x1.y, ip);
        ip = dp4a(q[6], x1.z, ip);
        ip = dp4a(q[7], x1.w, ip);
        if constexpr (MODE == RowOut::Partials) {
          a.partials[(static_cast<size_t>(t) * a.n_rows + row) * U + b] = ip;
        } else {
          acc[t] += (dw * (XREG ? xr.d : xd[t * U + b])) * static_cast<float>(ip);  // gguf_dot_q8.c:475-476
        }
      }
    }
  }
}

// Load half h of super-block sb of a Q4_K row: header (d, dmin, scales) and 64 quant bytes.
__device__ __forceinline__ void q4k_load_half(const uint8_t* rowp, int sb, int h, uint4& hdr, uint32_t (&qw)[16]) {
  const uint8_t* blk = rowp + sb * Q4_K_BYTES;
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

// Q4_K weight row x Q8_K activations.  A lane takes half a super-block u = 2*sb + h (4
// sub-blocks, 64 quant bytes); the halves of one super-block sit in adjacent lanes and are
// combined in int32 before the float step, so every per-block (sumi, summ) equals the
// reference's int32 values.  High nibbles are used in place (byte & 0xF0 = 16*q) with an
// unsigned-by-signed dp4a and the exact sum is shifted down by 4 afterwards.
// Per-lane constants of the one-unit-per-lane Q4_K row (U == 32, activations in registers):
// where the lane's half super-block sits in a row, and masks that select the 6-bit scale/min
// layout of its half (get_scale_min_k4, gguf_quant.c:212-220) without a branch.
struct Q4kLane {
  int hdr_off, q_off;         // byte offsets of the super-block header and of the half's 64 quant bytes
  uint32_t m_lo, m_s2, m_hi;  // h = 0: (0x3F.., 0, 0); h = 1: (0, 0x0F.., 0x30..)
};

__device__ __forceinline__ Q4kLane q4k_lane(int lane) {
  const int sb = lane >> 1, h = lane & 1;
  Q4kLane c;
  c.hdr_off = sb * Q4_K_BYTES;
  c.q_off = sb * Q4_K_BYTES + 16 + 64 * h;
  c.m_lo = h ? 0u : 0x3F3F3F3Fu;
  c.m_s2 = h ? 0x0F0F0F0Fu : 0u;
  c.m_hi = h ? 0x30303030u : 0u;
  return c;
}

// One Q4_K row of K = 4096 (32 half super-blocks) against one token whose Q8_K activations are
// held in registers.  Each lane adds its own half super-block to acc:
//   acc += (d_x d_w) * sumi_half - (d_x dmin_w) * summ_half
// with sumi_half (|.| <= 945*127*128 < 2^24) and summ_half exact in int32 and in fp32; the
// reference adds the two halves in int32 first (gguf_dot_q8.c:711-759), which differs only in
// the fp32 rounding of the final sum.
__device__ __forceinline__ void row_q4k_full(const uint8_t* rowp, float& acc, const XRegs& xr, const Q4kLane& c) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(rowp + c.hdr_off);
  const uint4* qp = reinterpret_cast<const uint4*>(rowp + c.q_off);
  const uint4 w0 = qp[0], w1 = qp[1], w2 = qp[2], w3 = qp[3];
  const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
  const uint32_t sc4 = (s0 & c.m_lo) | (s2 & c.m_s2) | ((s0 >> 2) & c.m_hi);
  const uint32_t mn4 = (s1 & c.m_lo) | ((s2 >> 4) & c.m_s2) | ((s1 >> 2) & c.m_hi);
  // Sub-block 2g: low nibbles of group g's 32 bytes against chunks 4g, 4g+1; sub-block 2g+1: high
  // nibbles (16*q in place, unsigned x signed dp4a) against chunks 4g+2, 4g+3.
  const uint32_t g0[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const uint32_t g1[8] = {w2.x, w2.y, w2.z, w2.w, w3.x, w3.y, w3.z, w3.w};
  const int xw[8][4] = {{xr.q[0].x, xr.q[0].y, xr.q[0].z, xr.q[0].w}, {xr.q[1].x, xr.q[1].y, xr.q[1].z, xr.q[1].w},
                        {xr.q[2].x, xr.q[2].y, xr.q[2].z, xr.q[2].w}, {xr.q[3].x, xr.q[3].y, xr.q[3].z, xr.q[3].w},
                        {xr.q[4].x, xr.q[4].y, xr.q[4].z, xr.q[4].w}, {xr.q[5].x, xr.q[5].y, xr.q[5].z, xr.q[5].w},
                        {xr.q[6].x, xr.q[6].y, xr.q[6].z, xr.q[6].w}, {xr.q[7].x, xr.q[7].y, xr.q[7].z, xr.q[7].w}};
  int ip0 = 0, ip1 = 0, ip2 = 0, ip3 = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int c4 = k >> 2, wi = k & 3;
    ip0 = dp4a(static_cast<int>(g0[k] & 0x0F0F0F0Fu), xw[c4][wi], ip0);
    ip1 = dp4a_us(g0[k] & 0xF0F0F0F0u, xw[2 + c4][wi], ip1);
    ip2 = dp4a(static_cast<int>(g1[k] & 0x0F0F0F0Fu), xw[4 + c4][wi], ip2);
    ip3 = dp4a_us(g1[k] & 0xF0F0F0F0u, xw[6 + c4][wi], ip3);
  }
  // ip1, ip3 are 16x their sub-block sums; their scaled sum stays exact below 2^31 before the shift.
  const int sumi = static_cast<int>(sc4 & 0xFFu) * ip0 + static_cast<int>((sc4 >> 16) & 0xFFu) * ip2 +
                   ((static_cast<int>((sc4 >> 8) & 0xFFu) * ip1 + static_cast<int>(sc4 >> 24) * ip3) >> 4);
  const int summ = dp4a_us(mn4, xr.sl, dp4a_us(mn4, xr.sh, 0) * 128);
  const float dw = fp16_bits_to_float(hdr.x), dmw = fp16_bits_to_float(hdr.x >> 16);
  acc += (xr.d * dw) * static_cast<float>(sumi) - (xr.d * dmw) * static_cast<float>(summ);
}

template <RowOut MODE, int MTOK, bool XREG, bool FULL = false>
__device__ __forceinline__ void row_q4k_q8k(const RowStreamArgs& a, const uint8_t* act, const uint8_t* rowp,
                                            long long row, float (&acc)[MTOK], int lane, const XRegs& xr) {
  static_assert(!FULL || XREG, "FULL: one unit per lane, activations in registers");
  const int U = a.K / 128, nb = U / 2;
  const int4* xq = reinterpret_cast<const int4*>(act);
  const int4* xb = reinterpret_cast<const int4*>(act + a.m * U * 128);
  const float* xd = reinterpret_cast<const float*>(act + a.m * U * 128 + a.m * U * 16);
  for (int u0 = 0; u0 < U; u0 += 32) {
    const int u = u0 + lane;
    const bool live = FULL || u < U;
    const int sb = u >> 1, h = u & 1;
    uint4 hdr;
    uint32_t qw[16];
    if (FULL) {
      q4k_load_half(rowp, sb, h, hdr, qw);
    } else {
      hdr = make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int i = 0; i < 16; ++i) qw[i] = 0;
      if (live) q4k_load_half(rowp, sb, h, hdr, qw);
    }
    uint32_t sc4, mn4;
    q4k_scales_half(hdr.y, hdr.z, hdr.w, h, sc4, mn4);
    const float dw = fp16_bits_to_float(hdr.x), dmw = fp16_bits_to_float(hdr.x >> 16);
#pragma unroll
    for (int t = 0; t < MTOK; ++t) {
      if (MTOK == 1 || t < a.m) {  // warp-uniform
        int sumi = 0, summ = 0;
        if (live) {
          int ip[4] = {0, 0, 0, 0};
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // chunk j: group g = j/4; j%4 < 2 low nibbles, else high
            const int4 x = XREG ? xr.q[j] : xq[(t * 8 + j) * U + u];
            const int g = j >> 2, c = j & 1;
            const uint32_t* w = qw + 8 * g + 4 * c;
            if ((j & 2) == 0) {
              ip[2 * g] = dp4a(static_cast<int>(w[0] & 0x0F0F0F0Fu), x.x, ip[2 * g]);
              ip[2 * g] = dp4a(static_cast<int>(w[1] & 0x0F0F0F0Fu), x.y, ip[2 * g]);
              ip[2 * g] = dp4a(static_cast<int>(w[2] & 0x0F0F0F0Fu), x.z, ip[2 * g]);
              ip[2 * g] = dp4a(static_cast<int>(w[3] & 0x0F0F0F0Fu), x.w, ip[2 * g]);
            } else {
              ip[2 * g + 1] = dp4a_us(w[0] & 0xF0F0F0F0u, x.x, ip[2 * g + 1]);
              ip[2 * g + 1] = dp4a_us(w[1] & 0xF0F0F0F0u, x.y, ip[2 * g + 1]);
              ip[2 * g + 1] = dp4a_us(w[2] & 0xF0F0F0F0u, x.z, ip[2 * g + 1]);
              ip[2 * g + 1] = dp4a_us(w[3] & 0xF0F0F0F0u, x.w, ip[2 * g + 1]);
            }
          }
          ip[1] >>= 4;  // exact: the sums of 16*q*x are multiples of 16
          ip[3] >>= 4;
          sumi = static_cast<int>(sc4 & 0xFFu) * ip[0] + static_cast<int>((sc4 >> 8) & 0xFFu) * ip[1] +
                 static_cast<int>((sc4 >> 16) & 0xFFu) * ip[2] + static_cast<int>(sc4 >> 24) * ip[3];
          if constexpr (XREG) {  // sum_j m_j * (128*Sh_j + Sl_j), exact (m_j <= 63, Sl_j <= 127)
            summ = dp4a_us(mn4, xr.sl, dp4a_us(mn4, xr.sh, 0) * 128);
          } else {
            const int4 bs = xb[t * U + u];
            summ = static_cast<int>(mn4 & 0xFFu) * bs.x + static_cast<int>((mn4 >> 8) & 0xFFu) * bs.y +
                   static_cast<int>((mn4 >> 16) & 0xFFu) * bs.z + static_cast<int>(mn4 >> 24) * bs.w;
          }
        }
        sumi += __shfl_xor_sync(0xFFFFFFFFu, sumi, 1);
        summ += __shfl_xor_sync(0xFFFFFFFFu, summ, 1);
        if (live && h == 0) {
          if constexpr (MODE == RowOut::Partials) {
            int32_t* pp = a.partials + ((static_cast<size_t>(t) * a.n_rows + row) * nb + sb) * 2;
            pp[0] = sumi;
            pp[1] = summ;
          } else {
            // gguf_dot_q8.c:619-620, :640, :661: d = d_x*d_w and dmin = -d_x*dmin_w per super-block.
            const float dx = XREG ? xr.d : xd[t * nb + sb];
            acc[t] += (dx * dw) * static_cast<float>(sumi) - (dx * dmw) * static_cast<float>(summ);
          }
        }
      }
    }
  }
}

__device__ __forceinline__ float nib_f(uint32_t masked, int k) {
  // byte k of a word whose bytes are 0..15, as an exact float: (2^23 + v) - 2^23.
  return __uint_as_float(__byte_perm(masked, 0x4B000000u, 0x7440u | static_cast<uint32_t>(k))) - 8388608.0f;
}

// Q4_K weight row x fp32 activations (the reference's logits path for non-Q8_0 weights).
template <RowOut MODE, int MTOK>
__device__ __forceinline__ void row_q4k_f32(const RowStreamArgs& a, const uint8_t* act, const uint8_t* rowp,
                                            float (&acc)[MTOK], int lane) {
  const int U = a.K / 128;
  const float4* xf = reinterpret_cast<const float4*>(act);
  const float4* xs = reinterpret_cast<const float4*>(act + a.m * U * 512);
  for (int u0 = 0; u0 < U; u0 += 32) {
    const int u = u0 + lane;
    if (u >= U) break;
    const int sb = u >> 1, h = u & 1;
    uint4 hdr;
    uint32_t qw[16];
    q4k_load_half(rowp, sb, h, hdr, qw);
    uint32_t sc4, mn4;
    q4k_scales_half(hdr.y, hdr.z, hdr.w, h, sc4, mn4);
    const float dw = fp16_bits_to_float(hdr.x), dmw = fp16_bits_to_float(hdr.x >> 16);
#pragma unroll
    for (int t = 0; t < MTOK; ++t) {
      if (MTOK == 1 || t < a.m) {
        const float4 sx = xs[t * U + u];
        const float sxs[4] = {sx.x, sx.y, sx.z, sx.w};
        float c = 0.0f;
#pragma unroll
        for (int s = 0; s < 4; ++s) {  // sub-block 4h+s: group s>>1, nibble half (s&1)
          float qx = 0.0f;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t mw = (qw[8 * (s >> 1) + i] >> (4 * (s & 1))) & 0x0F0F0F0Fu;
            const float4 x4 = xf[(t * 32 + 8 * s + i) * U + u];
            qx = fmaf(nib_f(mw, 0), x4.x, qx);
            qx = fmaf(nib_f(mw, 1), x4.y, qx);
            qx = fmaf(nib_f(mw, 2), x4.z, qx);
            qx = fmaf(nib_f(mw, 3), x4.w, qx);
          }
          const float d1 = dw * static_cast<float>((sc4 >> (8 * s)) & 0xFFu);
          const float m1 = dmw * static_cast<float>((mn4 >> (8 * s)) & 0xFFu);
          c += d1 * qx - m1 * sxs[s];  // gguf_quant.c:744/746
        }
        acc[t] += c;
      }
    }
  }
}

// ---- the other GGUF types -------------------------------------------------------------------------
// The quants are rebuilt in registers as SIGNED bytes scaled by a power of two, so that one signed
// dp4a chain forms 2^s * (integer dot) exactly and an arithmetic shift recovers the reference's
// int32 value:
//   Q4_0: 16*(q - 8)  = (q << 4) ^ 0x80               (q: 4-bit nibble, offset 8)
//   Q5_0:  8*(q - 16) = ((q << 3) | (h << 7)) ^ 0x80   (h: fifth bit, offset 16)
//   Q6_K:  4*(q - 32) = ((q << 2) | (h2 << 6)) ^ 0x80  (h2: two high bits, offset 32)
// (x ^ 0x80 subtracts 128 from a byte holding 0..255 read as int8; every sum of 2^s-multiples is a
// 2^s-multiple, so the shift is exact.)  Q5_K keeps its unsigned 5-bit values and a separate mins
// term, like Q4_K.

// Bits j .. j+3 of `bits` as bit 7 of the four bytes of a word (byte k gets bit j + k).
__device__ __forceinline__ uint32_t spread4_msb(uint32_t bits, int j) {
  return ((((bits >> j) & 0xFu) * 0x00204081u) & 0x01010101u) << 7;
}

// The 32-bit word at even byte offset `off` of a 2-byte aligned block whose covering aligned words
// are wv[] (wv[0] starts at the block, or 2 bytes before it when `odd`).
template <int OFF, int NW>
__device__ __forceinline__ uint32_t word_at(const uint32_t (&wv)[NW], bool odd) {
  static_assert(OFF % 2 == 0, "even offsets only");
  if constexpr (OFF % 4 == 0) {
    return odd ? __funnelshift_r(wv[OFF / 4], wv[OFF / 4 + 1], 16) : wv[OFF / 4];
  } else {
    return odd ? wv[(OFF + 2) / 4] : __funnelshift_r(wv[OFF / 4], wv[OFF / 4 + 1], 16);
  }
}

// Q4_0 (18 B: fp16 d, 16 nibble bytes) and Q5_0 (22 B: fp16 d, 32 fifth bits, 16 nibble bytes)
// rows against Q8_0 activations: a lane takes a block (gguf_dot_q8.c:584-599, :529-548):
// acc += d_w * d_x * ip with ip = sum_j (q_j - offset) * x_j exact in int32.
template <Fmt F, RowOut MODE, int MTOK>
__device__ __forceinline__ void row_b32(const RowStreamArgs& a, const uint8_t* act, const uint8_t* rowp,
                                        long long row, float (&acc)[MTOK], int lane) {
  constexpr bool Q5 = F == Fmt::Q5_0xQ8_0;
  constexpr int BB = Q5 ? 22 : 18;
  constexpr int NW = Q5 ? 6 : 5;  // aligned words covering the block (2 bytes of over-read at most)
  constexpr int QS = Q5 ? 6 : 2;  // offset of the nibble bytes
  const int U = a.K / QK8_0;
  const int4* xq = reinterpret_cast<const int4*>(act);
  const float* xd = reinterpret_cast<const float*>(act + a.m * U * 32);
  for (int b = lane; b < U; b += 32) {
    const uint8_t* p = rowp + b * BB;
    const bool odd = (reinterpret_cast<uintptr_t>(p) & 2u) != 0;  // blocks have even sizes
    const uint32_t* w = reinterpret_cast<const uint32_t*>(p - (odd ? 2 : 0));
    uint32_t wv[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) wv[i] = w[i];
    const uint32_t dbits = odd ? (wv[0] >> 16) : (wv[0] & 0xFFFFu);
    const uint32_t qs[4] = {word_at<QS, NW>(wv, odd), word_at<QS + 4, NW>(wv, odd), word_at<QS + 8, NW>(wv, odd),
                            word_at<QS + 12, NW>(wv, odd)};
    int lo[4], hi[4];  // signed scaled quants of elements 4i.. (lo) and 16+4i.. (hi)
    if constexpr (Q5) {
      const uint32_t qh = word_at<2, NW>(wv, odd);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        lo[i] = static_cast<int>((((qs[i] << 3) & 0x78787878u) | spread4_msb(qh, 4 * i)) ^ 0x80808080u);
        hi[i] = static_cast<int>((((qs[i] >> 1) & 0x78787878u) | spread4_msb(qh, 16 + 4 * i)) ^ 0x80808080u);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        lo[i] = static_cast<int>(((qs[i] << 4) & 0xF0F0F0F0u) ^ 0x80808080u);
        hi[i] = static_cast<int>((qs[i] & 0xF0F0F0F0u) ^ 0x80808080u);
      }
    }
    const float dw = fp16_bits_to_float(dbits);
#pragma unroll
    for (int t = 0; t < MTOK; ++t) {
      if (MTOK == 1 || t < a.m) {
        const int4 x0 = xq[(t * 2) * U + b], x1 = xq[(t * 2 + 1) * U + b];
        int ip = dp4a(lo[0], x0.x, 0);
        ip = dp4a(lo[1], x0.y, ip);
        ip = dp4a(lo[2], x0.z, ip);
        ip = dp4a(lo[3], x0.w, ip);
        ip = dp4a(hi[0], x1.x, ip);
        ip = dp4a(hi[1], x1.y, ip);
        ip = dp4a(hi[2], x1.z, ip);
        ip = dp4a(hi[3], x1.w, ip);
        ip >>= Q5 ? 3 : 4;  // exact: a multiple of 8 (Q5_0) or 16 (Q4_0)
        if constexpr (MODE == RowOut::Partials) {
          a.partials[(static_cast<size_t>(t) * a.n_rows + row) * U + b] = ip;
        } else {
          acc[t] += (dw * xd[t * U + b]) * static_cast<float>(ip);
        }
      }
    }
  }
}

// Half h of a Q5_K super-block (176 B: fp16 d, fp16 dmin, 12 scale bytes, qh[32] @16, ql[128] @48):
// the 5-bit values of its four sub-blocks s (= 4h+s of the super-block) as 4 x 8 words.  Sub-block
// s takes the low (s even) or high (s odd) nibbles of ql group s/2 and bit 4h+s of qh[l]
// (gguf_dot_q8.c:847-860).
__device__ __forceinline__ void q5k_half_values(const uint8_t* blk, int h, uint32_t (&v)[4][8]) {
  const uint4* qhp = reinterpret_cast<const uint4*>(blk + 16);
  const uint4* qlp = reinterpret_cast<const uint4*>(blk + 48 + 64 * h);
  const uint4 h0 = qhp[0], h1 = qhp[1];
  const uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const uint4 l0 = qlp[2 * g], l1 = qlp[2 * g + 1];
    const uint32_t ql[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t bl = 4 * h + 2 * g, bh = bl + 1;
      v[2 * g][k] = (ql[k] & 0x0F0F0F0Fu) | (((qh[k] >> bl) & 0x01010101u) << 4);
      v[2 * g + 1][k] = ((ql[k] >> 4) & 0x0F0F0F0Fu) | (((qh[k] >> bh) & 0x01010101u) << 4);
    }
  }
}

// Q5_K row x Q8_K activations: as row_q4k_q8k with 5-bit values (gguf_dot_q8.c:764-895).
template <RowOut MODE, int MTOK>
__device__ __forceinline__ void row_q5k_q8k(const RowStreamArgs& a, const uint8_t* act, const uint8_t* rowp,
                                            long long row, float (&acc)[MTOK], int lane) {
  const int U = a.K / 128, nb = U / 2;
  const int4* xq = reinterpret_cast<const int4*>(act);
  const int4* xb = reinterpret_cast<const int4*>(act + a.m * U * 128);
  const float* xd = reinterpret_cast<const float*>(act + a.m * U * 128 + a.m * U * 16);
  for (int u0 = 0; u0 < U; u0 += 32) {
    const int u = u0 + lane;
    const bool live = u < U;
    const int sb = u >> 1, h = u & 1;
    uint4 hdr = make_uint4(0, 0, 0, 0);
    uint32_t v[4][8];
#pragma unroll
    for (int s = 0; s < 4; ++s)
#pragma unroll
      for (int k = 0; k < 8; ++k) v[s][k] = 0;
    if (live) {
      const uint8_t* blk = rowp + sb * Q5_K_BYTES;
      hdr = *reinterpret_cast<const uint4*>(blk);
      q5k_half_values(blk, h, v);
    }
    uint32_t sc4, mn4;
    q4k_scales_half(hdr.y, hdr.z, hdr.w, h, sc4, mn4);
    const float dw = fp16_bits_to_float(hdr.x), dmw = fp16_bits_to_float(hdr.x >> 16);
#pragma unroll
    for (int t = 0; t < MTOK; ++t) {
      if (MTOK == 1 || t < a.m) {  // warp-uniform
        int sumi = 0, summ = 0;
        if (live) {
          int ip[4] = {0, 0, 0, 0};
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // chunk j: group j/4, low nibbles if j%4 < 2, words 4*(j&1)..
            const int4 x = xq[(t * 8 + j) * U + u];
            const int s = 2 * (j >> 2) + ((j >> 1) & 1), c = j & 1;
            ip[s] = dp4a_us(v[s][4 * c + 0], x.x, ip[s]);
            ip[s] = dp4a_us(v[s][4 * c + 1], x.y, ip[s]);
            ip[s] = dp4a_us(v[s][4 * c + 2], x.z, ip[s]);
            ip[s] = dp4a_us(v[s][4 * c + 3], x.w, ip[s]);
          }
          sumi = static_cast<int>(sc4 & 0xFFu) * ip[0] + static_cast<int>((sc4 >> 8) & 0xFFu) * ip[1] +
                 static_cast<int>((sc4 >> 16) & 0xFFu) * ip[2] + static_cast<int>(sc4 >> 24) * ip[3];
          const int4 bs = xb[t * U + u];
          summ = static_cast<int>(mn4 & 0xFFu) * bs.x + static_cast<int>((mn4 >> 8) & 0xFFu) * bs.y +
                 static_cast<int>((mn4 >> 16) & 0xFFu) * bs.z + static_cast<int>(mn4 >> 24) * bs.w;
        }
        sumi += __shfl_xor_sync(0xFFFFFFFFu, sumi, 1);
        summ += __shfl_xor_sync(0xFFFFFFFFu, summ, 1);
        if (live && h == 0) {
          if constexpr (MODE == RowOut::Partials) {
            int32_t* pp = a.partials + ((static_cast<size_t>(t) * a.n_rows + row) * nb + sb) * 2;
            pp[0] = sumi;
            pp[1] = summ;
          } else {
            const float dx = xd[t * nb + sb];
            acc[t] += (dx * dw) * static_cast<float>(sumi) - (dx * dmw) * static_cast<float>(summ);
          }
        }
      }
    }
  }
}

// Half h of a Q6_K super-block (210 B: ql[128], qh[64] @128, int8 scales[16] @192, fp16 d @208;
// only 2-byte aligned): the unsigned 6-bit values of its 128 elements as 4 quarters x 8 words
// (quarter q: the low (q < 2) or high nibbles of ql[l] (q even) or ql[l+32] (q odd) and bits
// 2q..2q+1 of qh[l], gguf_dot_q8.c:972-982), its 8 scales (two words) and d.
__device__ __forceinline__ void q6k_half_load(const uint8_t* blk, int h, uint32_t (&ql)[16], uint32_t (&qh)[8],
                                              uint32_t (&sc)[2], uint32_t& dbits) {
  const bool odd = (reinterpret_cast<uintptr_t>(blk) & 2u) != 0;
  const uint32_t* w = reinterpret_cast<const uint32_t*>(blk - (odd ? 2 : 0));
  const uint32_t* wl = w + 16 * h;       // ql of the half: bytes 64h ..
  const uint32_t* wh = w + 32 + 8 * h;   // qh of the half: bytes 128 + 32h ..
  const uint32_t* ws = w + 48 + 2 * h;   // scales of the half: bytes 192 + 8h ..
  uint32_t prev = wl[0];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t next = wl[i + 1];
    ql[i] = odd ? __funnelshift_r(prev, next, 16) : prev;
    prev = next;
  }
  prev = wh[0];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t next = wh[i + 1];
    qh[i] = odd ? __funnelshift_r(prev, next, 16) : prev;
    prev = next;
  }
  const uint32_t s0 = ws[0], s1 = ws[1], s2 = ws[2];
  sc[0] = odd ? __funnelshift_r(s0, s1, 16) : s0;
  sc[1] = odd ? __funnelshift_r(s1, s2, 16) : s1;
  const uint32_t dw = w[52];
  dbits = odd ? (dw >> 16) : (dw & 0xFFFFu);
}

// Unsigned 6-bit values (one per byte) of word k of quarter q.
__device__ __forceinline__ uint32_t q6k_word(const uint32_t (&ql)[16], const uint32_t (&qh)[8], int q, int k) {
  const uint32_t src = ql[8 * (q & 1) + k];
  const uint32_t nib = (q & 2) ? ((src >> 4) & 0x0F0F0F0Fu) : (src & 0x0F0F0F0Fu);
  return nib | (((qh[k] >> (2 * q)) & 0x03030303u) << 4);
}

// Q6_K row x Q8_K activations (gguf_dot_q8.c:897-1002): per half super-block
// sumi = sum over 16-element groups j of sc_j * sum (q - 32) * x, the halves combined in int32,
// then acc += (d_x * d_w) * sumi.
template <RowOut MODE, int MTOK>
__device__ __forceinline__ void row_q6k_q8k(const RowStreamArgs& a, const uint8_t* act, const uint8_t* rowp,
                                            long long row, float (&acc)[MTOK], int lane) {
  const int U = a.K / 128, nb = U / 2;
  const int4* xq = reinterpret_cast<const int4*>(act);
  const float* xd = reinterpret_cast<const float*>(act + a.m * U * 128 + a.m * U * 16);
  for (int u0 = 0; u0 < U; u0 += 32) {
    const int u = u0 + lane;
    const bool live = u < U;
    const int sb = u >> 1, h = u & 1;
    int v[4][8];  // signed 4*(q - 32)
    uint32_t sc[2] = {0u, 0u}, dbits = 0u;
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int k = 0; k < 8; ++k) v[q][k] = 0;
    if (live) {
      uint32_t ql[16], qh[8];
      q6k_half_load(rowp + sb * Q6_K_BYTES, h, ql, qh, sc, dbits);
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < 8; ++k) v[q][k] = static_cast<int>((q6k_word(ql, qh, q, k) << 2) ^ 0x80808080u);
    }
    const float dw = fp16_bits_to_float(dbits);
#pragma unroll
    for (int t = 0; t < MTOK; ++t) {
      if (MTOK == 1 || t < a.m) {  // warp-uniform
        int sumi = 0;
        if (live) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // chunk j = 16 elements = quarter j/2, words 4*(j&1) ..
            const int4 x = xq[(t * 8 + j) * U + u];
            const int q = j >> 1, c = j & 1;
            int ip = dp4a(v[q][4 * c + 0], x.x, 0);
            ip = dp4a(v[q][4 * c + 1], x.y, ip);
            ip = dp4a(v[q][4 * c + 2], x.z, ip);
            ip = dp4a(v[q][4 * c + 3], x.w, ip);
            const int scj = static_cast<int>(static_cast<int8_t>(sc[j >> 2] >> (8 * (j & 3))));
            sumi += scj * (ip >> 2);  // exact: ip is a multiple of 4
          }
        }
        sumi += __shfl_xor_sync(0xFFFFFFFFu, sumi, 1);
        if (live && h == 0) {
          if constexpr (MODE == RowOut::Partials) {
            int32_t* pp = a.partials + ((static_cast<size_t>(t) * a.n_rows + row) * nb + sb) * 2;
            pp[0] = sumi;
            pp[1] = 0;
          } else {
            acc[t] += (xd[t * nb + sb] * dw) * static_cast<float>(sumi);
          }
        }
      }
    }
  }
}

// Q5_K / Q6_K rows x fp32 activations (the logits path of these types: gguf_quant.c:837-892 and
// :754-794).  Float per element; the reference's scalar loop sums in another order, within the
// tolerance bound.
template <Fmt F, RowOut MODE, int MTOK>
__device__ __forceinline__ void row_k56_f32(const RowStreamArgs& a, const uint8_t* act, const uint8_t* rowp,
                                            float (&acc)[MTOK], int lane) {
  constexpr bool Q6 = F == Fmt::Q6_KxF32;
  const int U = a.K / 128;
  const float4* xf = reinterpret_cast<const float4*>(act);
  const float4* xs = reinterpret_cast<const float4*>(act + a.m * U * 512);
  for (int u0 = 0; u0 < U; u0 += 32) {
    const int u = u0 + lane;
    if (u >= U) break;
    const int sb = u >> 1, h = u & 1;
    if constexpr (Q6) {
      uint32_t ql[16], qh[8], sc[2], dbits;
      q6k_half_load(rowp + sb * Q6_K_BYTES, h, ql, qh, sc, dbits);
      const float dw = fp16_bits_to_float(dbits);
#pragma unroll
      for (int t = 0; t < MTOK; ++t) {
        if (MTOK == 1 || t < a.m) {
          float c = 0.0f;
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // 16-element group j: quarter j/2, words 4*(j&1) ..
            float qx = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int k = 4 * (j & 1) + i;
              const uint32_t vw = q6k_word(ql, qh, j >> 1, k);
              const float4 x4 = xf[(t * 32 + 8 * (j >> 1) + k) * U + u];
              qx = fmaf(nib_f(vw, 0) - 32.0f, x4.x, qx);
              qx = fmaf(nib_f(vw, 1) - 32.0f, x4.y, qx);
              qx = fmaf(nib_f(vw, 2) - 32.0f, x4.z, qx);
              qx = fmaf(nib_f(vw, 3) - 32.0f, x4.w, qx);
            }
            const float scj = static_cast<float>(static_cast<int8_t>(sc[j >> 2] >> (8 * (j & 3))));
            c = fmaf(dw * scj, qx, c);
          }
          acc[t] += c;
        }
      }
    } else {
      const uint8_t* blk = rowp + sb * Q5_K_BYTES;
      const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
      uint32_t v[4][8];
      q5k_half_values(blk, h, v);
      uint32_t sc4, mn4;
      q4k_scales_half(hdr.y, hdr.z, hdr.w, h, sc4, mn4);
      const float dw = fp16_bits_to_float(hdr.x), dmw = fp16_bits_to_float(hdr.x >> 16);
#pragma unroll
      for (int t = 0; t < MTOK; ++t) {
        if (MTOK == 1 || t < a.m) {
          const float4 sx = xs[t * U + u];
          const float sxs[4] = {sx.x, sx.y, sx.z, sx.w};
          float c = 0.0f;
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            float qx = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 x4 = xf[(t * 32 + 8 * s + i) * U + u];
              qx = fmaf(nib_f(v[s][i], 0), x4.x, qx);
              qx = fmaf(nib_f(v[s][i], 1), x4.y, qx);
              qx = fmaf(nib_f(v[s][i], 2), x4.z, qx);
              qx = fmaf(nib_f(v[s][i], 3), x4.w, qx);
            }
            const float d1 = dw * static_cast<float>((sc4 >> (8 * s)) & 0xFFu);
            const float m1 = dmw * static_cast<float>((mn4 >> (8 * s)) & 0xFFu);
            c += d1 * qx - m1 * sxs[s];
          }
          acc[t] += c;
        }
      }
    }
  }
}

// ---- the x86 float order (exact mode) -------------------------------------------------------------
// The reference's x86 Release build (AVX2 + FMA) keeps 8 float accumulators per row: accumulator m
// adds, block after block, fma(d_block, (float)P_m, acc_m) where P_m is an exact int32 partial over
// bytes 4m..4m+3 of each 32-byte group of the block (gguf_dot_q8.c:436-1002, SIMD branches), and
// the 8 are summed by a fixed tree (hsum_float_8, :125-131).  Exact mode reproduces that order bit
// for bit: a warp takes EX_ROWS rows at a time; lane EX_LPR*r + c runs accumulators m = 2c and 2c+1
// of row r over the whole row in block order (their bytes are 8 consecutive bytes of each group, so
// weights and activations load as 64-bit words), and the 4 lanes of a row finish with the same
// tree through xor-shuffles.  Non-fused float steps of the reference (its C is compiled in ISO mode,
// without contraction) use the _rn intrinsics so that the compiler cannot fuse them.
constexpr int EX_LPR = 4;              // lanes per row
constexpr int EX_ROWS = 32 / EX_LPR;   // rows per warp pass

// A 32-bit word at a 2-byte aligned shared-memory address.
__device__ __forceinline__ uint32_t ld_u32_a2(const uint8_t* p) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(p) & ~static_cast<uintptr_t>(3));
  const uint32_t lo = w[0];
  if ((reinterpret_cast<uintptr_t>(p) & 2u) == 0) return lo;
  return __funnelshift_r(lo, w[1], 16);
}

__device__ __forceinline__ uint32_t ld_u16_a2(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

__device__ __forceinline__ int2 ld_i2(const int* p) { return *reinterpret_cast<const int2*>(p); }

// hsum_float_8 (gguf_dot_q8.c:125-131), ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)), of the row's 8
// accumulators held as (v0, v1) = (a_2c, a_2c+1) by lane c of the row.  Lanes c and c^2 hold m and
// m + 4; every lane of the row ends with the same bits (float addition is commutative).
__device__ __forceinline__ float hsum8_dot_pairs(float v0, float v1) {
  const float r0 = v0 + __shfl_xor_sync(0xFFFFFFFFu, v0, 2);  // c = 0: a0+a4, c = 1: a2+a6
  const float r1 = v1 + __shfl_xor_sync(0xFFFFFFFFu, v1, 2);  // c = 0: a1+a5, c = 1: a3+a7
  return (r0 + __shfl_xor_sync(0xFFFFFFFFu, r0, 1)) + (r1 + __shfl_xor_sync(0xFFFFFFFFu, r1, 1));
}

// hsum256 (gguf_quant.c:488-495), ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)), same holding.
__device__ __forceinline__ float hsum8_quant_pairs(float v0, float v1) {
  const float r0 = v0 + __shfl_xor_sync(0xFFFFFFFFu, v0, 2);
  const float r1 = v1 + __shfl_xor_sync(0xFFFFFFFFu, v1, 2);
  const float h = r0 + r1;  // c = 0: (a0+a4)+(a1+a5), c = 1: (a2+a6)+(a3+a7)
  return h + __shfl_xor_sync(0xFFFFFFFFu, h, 1);
}

// Q8_0 / Q4_0 / Q5_0 rows x Q8_0 activations (gguf_dot_q8.c:440-452, :486-503, :556-569): for every
// block, P_m = sum of the products of elements 4m..4m+3, d = d_w * d_x, acc_m = fma(d, (float)P_m, acc_m).
template <Fmt F, int MTOK>
__device__ __forceinline__ void exact_b32(const RowStreamArgs& a, const uint8_t* act, const uint8_t* rowp, int c,
                                          float (&y)[MTOK]) {
  constexpr int BB = F == Fmt::Q8_0xQ8_0 ? Q8_0_BYTES : (F == Fmt::Q4_0xQ8_0 ? Q4_0_BYTES : Q5_0_BYTES);
  constexpr int SH = F == Fmt::Q8_0xQ8_0 ? 0 : (F == Fmt::Q4_0xQ8_0 ? 4 : 3);
  const int U = a.K / QK8_0;
  const int* xq = reinterpret_cast<const int*>(act);
  const float* xd = reinterpret_cast<const float*>(act + a.m * U * 32);
  float a0[MTOK], a1[MTOK];
#pragma unroll
  for (int t = 0; t < MTOK; ++t) a0[t] = a1[t] = 0.0f;
#pragma unroll 2
  for (int b = 0; b < U; ++b) {
    const uint8_t* blk = rowp + b * BB;
    int w0, w1;  // elements 8c .. 8c+3 and 8c+4 .. 8c+7, as signed bytes scaled by 2^SH
    if constexpr (F == Fmt::Q8_0xQ8_0) {
      w0 = static_cast<int>(ld_u32_a2(blk + 2 + 8 * c));
      w1 = static_cast<int>(ld_u32_a2(blk + 6 + 8 * c));
    } else {
      const uint32_t q0 = ld_u32_a2(blk + (BB - 16) + 8 * (c & 1)), q1 = ld_u32_a2(blk + (BB - 16) + 8 * (c & 1) + 4);
      if constexpr (F == Fmt::Q4_0xQ8_0) {  // 16*(q - 8): low nibbles for elements < 16, high for >= 16
        w0 = static_cast<int>(((c < 2 ? (q0 << 4) : q0) & 0xF0F0F0F0u) ^ 0x80808080u);
        w1 = static_cast<int>(((c < 2 ? (q1 << 4) : q1) & 0xF0F0F0F0u) ^ 0x80808080u);
      } else {  // 8*(q - 16), the fifth bit of element e at bit e of qh
        const uint32_t qh = ld_u32_a2(blk + 2);
        w0 = static_cast<int>((((c < 2 ? (q0 << 3) : (q0 >> 1)) & 0x78787878u) | spread4_msb(qh, 8 * c)) ^ 0x80808080u);
        w1 = static_cast<int>((((c < 2 ? (q1 << 3) : (q1 >> 1)) & 0x78787878u) | spread4_msb(qh, 8 * c + 4)) ^ 0x80808080u);
      }
    }
    const float dw = fp16_bits_to_float(ld_u16_a2(blk));
#pragma unroll
    for (int t = 0; t < MTOK; ++t) {
      if (MTOK == 1 || t < a.m) {
        // words 2c, 2c+1 of the block's 8 activation words: chunk c/2, words 2(c%2), 2(c%2)+1
        const int2 xw = ld_i2(xq + ((t * 2 + (c >> 1)) * U + b) * 4 + 2 * (c & 1));
        const float d = __fmul_rn(dw, xd[t * U + b]);
        a0[t] = fmaf(d, static_cast<float>(dp4a(w0, xw.x, 0) >> SH), a0[t]);
        a1[t] = fmaf(d, static_cast<float>(dp4a(w1, xw.y, 0) >> SH), a1[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < MTOK; ++t) y[t] = hsum8_dot_pairs(a0[t], a1[t]);
}

// Q4_K / Q5_K / Q6_K rows x Q8_K activations (gguf_dot_q8.c:612-664, :772-830, :905-963).  P_m per
// super-block: Q4_K / Q5_K sum_j sc_2j * sum(elements 64j+4m..) + sc_2j+1 * sum(elements 64j+32+4m..);
// Q6_K sum over the eight 32-element groups g of sc[2g + (m >= 4)] * sum(elements 32g+4m..) minus
// 32 * (bsum_2m * sc_2m + bsum_2m+1 * sc_2m+1).  The Q4_K mins run in 4 more accumulators
// (fma(dmin, mn_2k*S_2k + mn_2k+1*S_2k+1)), summed as (m0+m2) + (m1+m3) and added after the tree;
// Q5_K adds dmin * (float)(all mins) to one scalar per super-block.
template <Fmt F, int MTOK>
__device__ __forceinline__ void exact_k(const RowStreamArgs& a, const uint8_t* act, const uint8_t* rowp, int c,
                                        float (&y)[MTOK]) {
  constexpr bool Q6 = F == Fmt::Q6_KxQ8_K, Q5 = F == Fmt::Q5_KxQ8_K;
  constexpr int BB = Q6 ? Q6_K_BYTES : (Q5 ? Q5_K_BYTES : Q4_K_BYTES);
  const int U = a.K / 128, nb = U / 2;
  const int* xq = reinterpret_cast<const int*>(act);
  const int* xb = reinterpret_cast<const int*>(act + a.m * U * 128);
  const float* xd = reinterpret_cast<const float*>(act + a.m * U * 128 + a.m * U * 16);
  const int16_t* xb16 = reinterpret_cast<const int16_t*>(act + xb16_off(a.m, U));
  float a0[MTOK], a1[MTOK], m0[MTOK], m1[MTOK];
#pragma unroll
  for (int t = 0; t < MTOK; ++t) a0[t] = a1[t] = m0[t] = m1[t] = 0.0f;
#pragma unroll 2
  for (int sb = 0; sb < nb; ++sb) {
    const uint8_t* blk = rowp + sb * BB;
    if constexpr (Q6) {
      // group g = 4j + k: unsigned 6-bit values of elements 128j + 32k + 8c .. +7 (two words)
      uint32_t v[8][2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint32_t h0 = ld_u32_a2(blk + 128 + 32 * j + 8 * c), h1 = ld_u32_a2(blk + 132 + 32 * j + 8 * c);
        const uint32_t l00 = ld_u32_a2(blk + 64 * j + 8 * c), l01 = ld_u32_a2(blk + 64 * j + 4 + 8 * c);
        const uint32_t l10 = ld_u32_a2(blk + 64 * j + 32 + 8 * c), l11 = ld_u32_a2(blk + 64 * j + 36 + 8 * c);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t s0 = (k & 1) ? l10 : l00, s1 = (k & 1) ? l11 : l01;
          const uint32_t n0 = (k & 2) ? ((s0 >> 4) & 0x0F0F0F0Fu) : (s0 & 0x0F0F0F0Fu);
          const uint32_t n1 = (k & 2) ? ((s1 >> 4) & 0x0F0F0F0Fu) : (s1 & 0x0F0F0F0Fu);
          v[4 * j + k][0] = n0 | (((h0 >> (2 * k)) & 0x03030303u) << 4);
          v[4 * j + k][1] = n1 | (((h1 >> (2 * k)) & 0x03030303u) << 4);
        }
      }
      // scales: group g uses sc[2g + (m >= 4)] (m = 2c, 2c+1 share it); the subtracted bsum terms use
      // sc_2m, sc_2m+1 = sc[4c .. 4c+3]
      const uint32_t s_lo = ld_u32_a2(blk + 192), s_hi = ld_u32_a2(blk + 196), s_lo2 = ld_u32_a2(blk + 200),
                     s_hi2 = ld_u32_a2(blk + 204);
      const uint32_t sw[4] = {s_lo, s_hi, s_lo2, s_hi2};
      int scg[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const int idx = 2 * g + (c >= 2 ? 1 : 0);
        scg[g] = static_cast<int8_t>(sw[idx >> 2] >> (8 * (idx & 3)));
      }
      const uint32_t own = c == 0 ? s_lo : (c == 1 ? s_hi : (c == 2 ? s_lo2 : s_hi2));  // sc[4c .. 4c+3]
      const float dw = fp16_bits_to_float(ld_u16_a2(blk + 208));
#pragma unroll
      for (int t = 0; t < MTOK; ++t) {
        if (MTOK == 1 || t < a.m) {
          int p0 = 0, p1 = 0;
#pragma unroll
          for (int g = 0; g < 8; ++g) {  // element 32g + 8c: unit 2sb + g/4, chunk 2(g%4) + c/2, words 2(c%2)..
            const int2 xw = ld_i2(xq + ((t * 8 + 2 * (g & 3) + (c >> 1)) * U + 2 * sb + (g >> 2)) * 4 + 2 * (c & 1));
            p0 += scg[g] * dp4a(static_cast<int>(v[g][0]), xw.x, 0);
            p1 += scg[g] * dp4a(static_cast<int>(v[g][1]), xw.y, 0);
          }
          // bsums 4c .. 4c+3: unit 2sb + c/2, groups 4(c%2) .. of that unit
          const int2 bsw = ld_i2(reinterpret_cast<const int*>(xb16 + (t * U + 2 * sb + (c >> 1)) * 8 + 4 * (c & 1)));
          const int b0 = static_cast<int16_t>(bsw.x & 0xFFFF), b1 = bsw.x >> 16;
          const int b2 = static_cast<int16_t>(bsw.y & 0xFFFF), b3 = bsw.y >> 16;
          p0 -= 32 * (b0 * static_cast<int8_t>(own) + b1 * static_cast<int8_t>(own >> 8));
          p1 -= 32 * (b2 * static_cast<int8_t>(own >> 16) + b3 * static_cast<int8_t>(own >> 24));
          const float d = __fmul_rn(xd[t * nb + sb], dw);
          a0[t] = fmaf(d, static_cast<float>(p0), a0[t]);
          a1[t] = fmaf(d, static_cast<float>(p1), a1[t]);
        }
      }
    } else {
      const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
      // elements 64j + 8c .. +7 (lo) and 64j + 32 + 8c .. (hi) of the lane's two accumulators
      uint32_t lo[4][2], hi[4][2];
      uint2 qh = make_uint2(0u, 0u);
      if constexpr (Q5) qh = *reinterpret_cast<const uint2*>(blk + 16 + 8 * c);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint2 q = *reinterpret_cast<const uint2*>(blk + (Q5 ? 48 : 16) + 32 * j + 8 * c);
        lo[j][0] = q.x & 0x0F0F0F0Fu;
        lo[j][1] = q.y & 0x0F0F0F0Fu;
        hi[j][0] = (q.x >> 4) & 0x0F0F0F0Fu;
        hi[j][1] = (q.y >> 4) & 0x0F0F0F0Fu;
        if constexpr (Q5) {
          lo[j][0] |= ((qh.x >> (2 * j)) & 0x01010101u) << 4;
          lo[j][1] |= ((qh.y >> (2 * j)) & 0x01010101u) << 4;
          hi[j][0] |= ((qh.x >> (2 * j + 1)) & 0x01010101u) << 4;
          hi[j][1] |= ((qh.y >> (2 * j + 1)) & 0x01010101u) << 4;
        }
      }
      uint32_t sc_lo, mn_lo, sc_hi, mn_hi;  // the eight 6-bit scales and mins (get_scale_min_k4)
      q4k_scales_half(hdr.y, hdr.z, hdr.w, 0, sc_lo, mn_lo);
      q4k_scales_half(hdr.y, hdr.z, hdr.w, 1, sc_hi, mn_hi);
      int sc[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sc[j] = static_cast<int>((sc_lo >> (8 * j)) & 0xFFu);
        sc[4 + j] = static_cast<int>((sc_hi >> (8 * j)) & 0xFFu);
      }
      // mins accumulators k = 2(c%2), 2(c%2)+1 use mins 4(c%2) .. 4(c%2)+3 and S of the same indices
      const uint32_t mw = (c & 1) ? mn_hi : mn_lo;
      const float dw = fp16_bits_to_float(hdr.x), dmw = fp16_bits_to_float(hdr.x >> 16);
#pragma unroll
      for (int t = 0; t < MTOK; ++t) {
        if (MTOK == 1 || t < a.m) {
          int p0 = 0, p1 = 0;
#pragma unroll
          for (int j = 0; j < 4; ++j) {  // element 64j + 8c (+32): unit 2sb + j/2, chunk 4(j%2) + c/2 (+2)
            const int* xr = xq + ((t * 8 + 4 * (j & 1) + (c >> 1)) * U + 2 * sb + (j >> 1)) * 4 + 2 * (c & 1);
            const int2 xl = ld_i2(xr), xh = ld_i2(xr + 8 * U);
            p0 += sc[2 * j] * dp4a(static_cast<int>(lo[j][0]), xl.x, 0) + sc[2 * j + 1] * dp4a(static_cast<int>(hi[j][0]), xh.x, 0);
            p1 += sc[2 * j] * dp4a(static_cast<int>(lo[j][1]), xl.y, 0) + sc[2 * j + 1] * dp4a(static_cast<int>(hi[j][1]), xh.y, 0);
          }
          const float xdt = xd[t * nb + sb];
          const float d = __fmul_rn(xdt, dw);
          a0[t] = fmaf(d, static_cast<float>(p0), a0[t]);
          a1[t] = fmaf(d, static_cast<float>(p1), a1[t]);
          const float dmin = __fmul_rn(-xdt, dmw);
          if constexpr (Q5) {
            const int4 s0 = *reinterpret_cast<const int4*>(xb + (t * U + 2 * sb) * 4);
            const int4 s1 = *reinterpret_cast<const int4*>(xb + (t * U + 2 * sb + 1) * 4);
            const int tot = static_cast<int>(mn_lo & 0xFFu) * s0.x + static_cast<int>((mn_lo >> 8) & 0xFFu) * s0.y +
                            static_cast<int>((mn_lo >> 16) & 0xFFu) * s0.z + static_cast<int>(mn_lo >> 24) * s0.w +
                            static_cast<int>(mn_hi & 0xFFu) * s1.x + static_cast<int>((mn_hi >> 8) & 0xFFu) * s1.y +
                            static_cast<int>((mn_hi >> 16) & 0xFFu) * s1.z + static_cast<int>(mn_hi >> 24) * s1.w;
            m0[t] = __fadd_rn(m0[t], __fmul_rn(dmin, static_cast<float>(tot)));
          } else {
            const int4 S = *reinterpret_cast<const int4*>(xb + (t * U + 2 * sb + (c & 1)) * 4);
            const int pr0 = static_cast<int>(mw & 0xFFu) * S.x + static_cast<int>((mw >> 8) & 0xFFu) * S.y;
            const int pr1 = static_cast<int>((mw >> 16) & 0xFFu) * S.z + static_cast<int>(mw >> 24) * S.w;
            m0[t] = fmaf(dmin, static_cast<float>(pr0), m0[t]);
            m1[t] = fmaf(dmin, static_cast<float>(pr1), m1[t]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < MTOK; ++t) {
    const float s8 = hsum8_dot_pairs(a0[t], a1[t]);
    if constexpr (Q6) {
      y[t] = s8;
    } else if constexpr (Q5) {
      y[t] = s8 + m0[t];
    } else {  // lane c%2 = 0 holds mins 0, 1, lane c%2 = 1 mins 2, 3: (m0 + m2) + (m1 + m3)
      const float mm = (m0[t] + __shfl_xor_sync(0xFFFFFFFFu, m0[t], 1)) + (m1[t] + __shfl_xor_sync(0xFFFFFFFFu, m1[t], 1));
      y[t] = s8 + mm;
    }
  }
}

// Q4_K / Q5_K / Q6_K rows x fp32 activations (the greedy-logits path) in the x86 order.
// Q4_K (gguf_quant.c:704-752 with the AVX2 dot_u4_f32_32 :545-565): per sub-block s, accumulator m runs
// fma(q, x) over elements 32s + 8i + m (i < 4) and hsum256 sums the 8; the x sums of the sub-block are
// the ones the activation prologue formed in the same order; acc = acc + ((d*sc)*qx - (dmin*mn)*sx).
// Q5_K and Q6_K have no SIMD branch there (gguf_quant.c:837-892, :754-794): one scalar sum over the
// row in the reference's element order, run by lane 0 of the row.
template <Fmt F, int MTOK>
__device__ __forceinline__ void exact_f32(const RowStreamArgs& a, const uint8_t* act, const uint8_t* rowp, int c,
                                          float (&y)[MTOK]) {
  const int U = a.K / 128, nb = U / 2;
  const float* xf = reinterpret_cast<const float*>(act);
  // element e of the row, token t: unit e/128, float4 chunk (e%128)/4, component e%4
  auto xat = [&](int t, int e) -> const float* { return xf + ((t * 32 + ((e & 127) >> 2)) * U + (e >> 7)) * 4 + (e & 3); };
  if constexpr (F == Fmt::Q4_KxF32) {
    const float* xs = reinterpret_cast<const float*>(act + a.m * U * 512);  // [t][K/32] sums, x86 order
    float acc[MTOK];
#pragma unroll
    for (int t = 0; t < MTOK; ++t) acc[t] = 0.0f;
    for (int sb = 0; sb < nb; ++sb) {
      const uint8_t* blk = rowp + sb * Q4_K_BYTES;
      const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
      const float d = fp16_bits_to_float(hdr.x), dmin = fp16_bits_to_float(hdr.x >> 16);
      uint32_t sc_lo, mn_lo, sc_hi, mn_hi;
      q4k_scales_half(hdr.y, hdr.z, hdr.w, 0, sc_lo, mn_lo);
      q4k_scales_half(hdr.y, hdr.z, hdr.w, 1, sc_hi, mn_hi);
#pragma unroll
      for (int g = 0; g < 4; ++g) {  // 32 bytes of group g: sub-block 2g (low nibbles), 2g+1 (high)
        uint32_t qb[4];  // bytes 8i + 2c, 8i + 2c + 1 for i < 4 (two per 16-bit load)
#pragma unroll
        for (int i = 0; i < 4; ++i) qb[i] = *reinterpret_cast<const uint16_t*>(blk + 16 + 32 * g + 8 * i + 2 * c);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int s = 2 * g + h;
          const uint32_t scw = s < 4 ? sc_lo : sc_hi, mnw = s < 4 ? mn_lo : mn_hi;
          const float d1 = __fmul_rn(d, static_cast<float>((scw >> (8 * (s & 3))) & 0xFFu));
          const float m1 = __fmul_rn(dmin, static_cast<float>((mnw >> (8 * (s & 3))) & 0xFFu));
#pragma unroll
          for (int t = 0; t < MTOK; ++t) {
            if (MTOK == 1 || t < a.m) {
              float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float2 xv = *reinterpret_cast<const float2*>(xat(t, sb * QK_K + 32 * s + 8 * i + 2 * c));
                const uint32_t nb2 = h ? (qb[i] >> 4) : qb[i];
                v0 = fmaf(static_cast<float>(nb2 & 0xFu), xv.x, v0);
                v1 = fmaf(static_cast<float>((nb2 >> 8) & 0xFu), xv.y, v1);
              }
              const float qx = hsum8_quant_pairs(v0, v1), sx = xs[t * (U * 4) + sb * 8 + s];
              acc[t] = __fadd_rn(acc[t], __fsub_rn(__fmul_rn(d1, qx), __fmul_rn(m1, sx)));
            }
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < MTOK; ++t) y[t] = acc[t];
  } else {
    // The scalar loops, in lane 0 of the row; the other lanes take the result by shuffle.
    float acc[MTOK];
#pragma unroll
    for (int t = 0; t < MTOK; ++t) acc[t] = 0.0f;
    if (c == 0) {
      for (int sb = 0; sb < nb; ++sb) {
        if constexpr (F == Fmt::Q5_KxF32) {  // gguf_quant.c:866-887: acc += (d1*q0 - m1)*x[l]; acc += (d2*q1 - m2)*x[l+32]
          const uint8_t* blk = rowp + sb * Q5_K_BYTES;
          const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
          const float d = fp16_bits_to_float(hdr.x), dmin = fp16_bits_to_float(hdr.x >> 16);
          uint32_t sc_lo, mn_lo, sc_hi, mn_hi;
          q4k_scales_half(hdr.y, hdr.z, hdr.w, 0, sc_lo, mn_lo);
          q4k_scales_half(hdr.y, hdr.z, hdr.w, 1, sc_hi, mn_hi);
          for (int g = 0; g < 4; ++g) {
            const uint32_t scw = g < 2 ? sc_lo : sc_hi, mnw = g < 2 ? mn_lo : mn_hi;
            const int sh = 16 * (g & 1);
            const float d1 = __fmul_rn(d, static_cast<float>((scw >> sh) & 0xFFu));
            const float m1 = __fmul_rn(dmin, static_cast<float>((mnw >> sh) & 0xFFu));
            const float d2 = __fmul_rn(d, static_cast<float>((scw >> (sh + 8)) & 0xFFu));
            const float m2 = __fmul_rn(dmin, static_cast<float>((mnw >> (sh + 8)) & 0xFFu));
            for (int l = 0; l < 32; ++l) {
              const int ql = blk[48 + 32 * g + l], qh = blk[16 + l];
              const float q0 = static_cast<float>((ql & 0xF) + (((qh >> (2 * g)) & 1) << 4));
              const float q1 = static_cast<float>((ql >> 4) + (((qh >> (2 * g + 1)) & 1) << 4));
#pragma unroll
              for (int t = 0; t < MTOK; ++t) {
                if (MTOK == 1 || t < a.m) {
                  const int e = sb * QK_K + 64 * g + l;
                  acc[t] = __fadd_rn(acc[t], __fmul_rn(__fsub_rn(__fmul_rn(d1, q0), m1), *xat(t, e)));
                  acc[t] = __fadd_rn(acc[t], __fmul_rn(__fsub_rn(__fmul_rn(d2, q1), m2), *xat(t, e + 32)));
                }
              }
            }
          }
        } else {  // Q6_K, gguf_quant.c:771-791: acc += d*sc*q*x for the four quarters of each l
          const uint8_t* blk = rowp + sb * Q6_K_BYTES;
          const float d = fp16_bits_to_float(ld_u16_a2(blk + 208));
          for (int h = 0; h < 2; ++h) {
            for (int l = 0; l < 32; ++l) {
              const int qh = blk[128 + 32 * h + l], l0 = blk[64 * h + l], l1 = blk[64 * h + 32 + l];
              const int qv[4] = {(l0 & 0xF) | ((qh & 3) << 4), (l1 & 0xF) | (((qh >> 2) & 3) << 4),
                                 (l0 >> 4) | (((qh >> 4) & 3) << 4), (l1 >> 4) | (((qh >> 6) & 3) << 4)};
#pragma unroll
              for (int qq = 0; qq < 4; ++qq) {
                const float sc = static_cast<float>(static_cast<int8_t>(blk[192 + 8 * h + l / 16 + 2 * qq]));
                const float wv = __fmul_rn(__fmul_rn(d, sc), static_cast<float>(qv[qq] - 32));
#pragma unroll
                for (int t = 0; t < MTOK; ++t) {
                  if (MTOK == 1 || t < a.m) {
                    acc[t] = __fadd_rn(acc[t], __fmul_rn(wv, *xat(t, sb * QK_K + 128 * h + 32 * qq + l)));
                  }
                }
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < MTOK; ++t) y[t] = __shfl_sync(0xFFFFFFFFu, acc[t], (threadIdx.x & 31) & ~(EX_LPR - 1));
  }
}

template <Fmt F, int MTOK>
__device__ __forceinline__ void exact_row(const RowStreamArgs& a, const uint8_t* act, const uint8_t* rowp, int c,
                                          float (&y)[MTOK]) {
  if constexpr (act_of(F) == Act::Q8_0) {
    exact_b32<F, MTOK>(a, act, rowp, c, y);
  } else if constexpr (act_of(F) == Act::Q8_K) {
    exact_k<F, MTOK>(a, act, rowp, c, y);
  } else {
    exact_f32<F, MTOK>(a, act, rowp, c, y);
  }
}

// ---- the kernel ---------------------------------------------------------------------------------

// Tile -> (segment, first row, rows, weight base, output, bias, output stride).
struct TileRef {
  const uint8_t* w;
  const float* bias;
  float* out;
  long long stride;
  long long r0;
  int nr;
};

// What consumers need of a stage's tile, written by the producer before it arms the stage's
// barrier (the barrier's release/acquire orders it), so consumer warps need not re-derive it.
struct __align__(16) TileDesc {
  float* out;
  const float* bias;
  int r0;        // first row of the tile within its tensor
  int nr;        // rows in the tile
  int stride;    // output row stride (elements)
  int misalign;  // start of the tile's first row inside the stage (the copy starts 16-byte aligned)
};
static_assert(sizeof(TileDesc) == 32, "two 16-byte words");

__device__ __forceinline__ TileRef tile_ref(const RowStreamArgs& a, const Layout& L, long long tile) {
  int s = 0;
#pragma unroll
  for (int i = 1; i < MAX_SEGS; ++i)
    if (i < a.n_seg && tile >= a.seg[i].tile0) s = i;
  const RowSeg& g = a.seg[s];
  TileRef t;
  t.w = g.w;
  t.bias = g.bias;
  t.out = g.out;
  t.stride = a.n_seg > 1 ? g.n_rows : a.out_stride;
  t.r0 = (tile - g.tile0) * L.tile_rows;
  t.nr = static_cast<int>(min(static_cast<long long>(L.tile_rows), g.n_rows - t.r0));
  return t;
}

// ---- tensor-parallel all-reduce over peer memory -------------------------------------------------
// Each partial output travels with its own flag: the consumer lane that computes output (t, row)
// writes the 64-bit word (float bits, tag = epoch + 1) to entry [parity][rank][t*n + row] of every
// rank's exchange region (CUDA IPC mappings over NVLink). Up to TP_DIRECT_WORLD ranks the lane
// stores to every peer as soon as it has the value (the stores overlap the remaining tiles); with
// more ranks the one-word-per-output NVLink writes cost more than they overlap (measured: 4096
// outputs x 7 peers added ~4 us per launch), so the lane writes only the local entry and after its
// last tile the CTA copies its entries to every peer with coalesced stores. An aligned 64-bit store
// is single-copy atomic, so a reader that sees the current tag also sees that store's value -- no
// fences, no separate flag. Each CTA then polls (bounded) the entries of its own rows in the local
// region until every rank's tag is current and sums them in rank order, so every rank gets the same
// bits. The row-to-CTA map is the same on every rank. Parity: a rank writes parity p again only in
// launch e + 2, which starts after its launch e + 1 read every peer's entries of e + 1, which the
// peers wrote only after finishing their launch e (and its reads).
__device__ __forceinline__ void st_relaxed_sys_u64(void* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const void* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ void tp_finalize(const RowStreamArgs& a, const Layout& L, uint32_t e, int ct) {
  const uint8_t* local = a.tp.peer[a.tp.rank];
  uint32_t* counter = reinterpret_cast<uint32_t*>(a.tp.peer[a.tp.rank] + TP_CTRL_OFF);
  const uint32_t f = e + 1u;
  const int n = static_cast<int>(a.seg[0].n_rows);
  const unsigned long long* slots =
      reinterpret_cast<const unsigned long long*>(local + static_cast<size_t>(e & 1u) * TP_MAX_WORLD * TP_SLOT_BYTES);
  const size_t per_rank = TP_SLOT_BYTES / 8;
  // Push (more than TP_DIRECT_WORLD ranks): this CTA's own entries, written by its consumer warps
  // before the barrier, go to every peer as warp-wide stores of consecutive rows -- a few large
  // NVLink writes instead of one 8-byte write per output and peer.
  const size_t own = static_cast<size_t>(a.tp.rank) * per_rank;
  if (a.tp.world > TP_DIRECT_WORLD) named_bar_sync(2, CONSUMERS);
  for (long long tile = a.tp.world > TP_DIRECT_WORLD ? blockIdx.x : L.n_tiles; tile < L.n_tiles; tile += gridDim.x) {
    const TileRef tr = tile_ref(a, L, tile);
    const int cnt = tr.nr * a.m;
    for (int i = ct; i < cnt; i += CONSUMERS) {
      const int t = i / tr.nr, row = static_cast<int>(tr.r0) + (i - t * tr.nr);
      const size_t idx = static_cast<size_t>(t) * n + row;
      const unsigned long long v = slots[own + idx];  // written by this CTA before the barrier
      const size_t off = reinterpret_cast<const uint8_t*>(slots + own + idx) - local;
      for (int r = 0; r < a.tp.world; ++r)
        if (r != a.tp.rank) st_relaxed_sys_u64(a.tp.peer[r] + off, v);
    }
  }
  const unsigned long long t0 = global_ns();
  bool ok = true;
  for (long long tile = blockIdx.x; tile < L.n_tiles; tile += gridDim.x) {
    const TileRef tr = tile_ref(a, L, tile);
    const int cnt = tr.nr * a.m;
    for (int i = ct; i < cnt; i += CONSUMERS) {
      const int t = i / tr.nr, row = static_cast<int>(tr.r0) + (i - t * tr.nr);
      const size_t idx = static_cast<size_t>(t) * n + row;
      // All ranks' entries in flight at once (one L2 round trip when they have arrived), then
      // re-poll only the stale ones.
      unsigned long long v[TP_MAX_WORLD];
#pragma unroll
      for (int r = 0; r < TP_MAX_WORLD; ++r)
        if (r < a.tp.world) v[r] = ld_relaxed_sys_u64(slots + r * per_rank + idx);
      float sum = 0.0f;
#pragma unroll
      for (int r = 0; r < TP_MAX_WORLD; ++r) {  // rank order: the same additions on every rank
        if (r >= a.tp.world) break;
        for (uint32_t k = 0; ok && static_cast<uint32_t>(v[r] >> 32) != f; ++k) {
          if ((k & 63u) == 63u && global_ns() - t0 > WAIT_LIMIT_NS) ok = false;
          v[r] = ld_relaxed_sys_u64(slots + r * per_rank + idx);
        }
        sum += __uint_as_float(static_cast<uint32_t>(v[r]));
      }
      a.seg[0].out[static_cast<size_t>(t) * a.out_stride + row] = sum;
    }
  }
  if (!ok) atomicOr(a.status, ST_TIMEOUT_PEER);
  // Advance the epoch once every CTA of this launch is done with it (it read it at its start).
  named_bar_sync(2, CONSUMERS);
  if (ct == 0) {
    __threadfence();
    if (atomicAdd(counter, 1u) == gridDim.x - 1) {
      counter[0] = 0u;
      counter[1] = e + 1u;  // the next launch reads it after its griddepcontrol.wait
    }
  }
}

template <Fmt F, RowOut MODE, int MTOK, bool XREG, bool EXACT, bool SLICE>
__global__ void __launch_bounds__(THREADS, 1) rowstream_kernel(const RowStreamArgs a, const Layout L) {
  static_assert(!SLICE || (F == Fmt::Q4_KxQ8_K && MTOK == 1 && !XREG && !EXACT &&
                           (MODE == RowOut::Store || MODE == RowOut::Argmax)), "sliced rows: Q4_K, batch 1");
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + MAX_STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 2 * MAX_STAGES * 8);
  uint64_t* xin = reinterpret_cast<uint64_t*>(smem + 2 * MAX_STAGES * 8 + 8);
  TileDesc* descs = reinterpret_cast<TileDesc*>(smem + DESC_OFF);
  static_assert(2 * MAX_STAGES * 8 + 16 <= DESC_OFF, "barriers fit below the descriptors");
  static_assert(DESC_OFF + MAX_STAGES * sizeof(TileDesc) <= BAR_BYTES, "tile descriptors fit the header");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = L.n_stages;

  // Tile slot r belongs to consumer warp (it*R + r) % CONSUMER_WARPS.  Every consumer warp waits
  // for every tile and releases it, owner or not: a warp that skipped tiles could otherwise reach
  // a stage's fill k before fill k - 1 completed, when the parity wait for k returns at once.
  const int R = L.tile_rows;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CONSUMER_WARPS);
    }
    mbar_init(xin, CONSUMER_WARPS);
    *abort_flag = 0;
    if constexpr (SLICE) {
      int* cnt = reinterpret_cast<int*>(smem + L.part_off + MAX_STAGES * R * SLICE_UNITS * 4);
      for (int i = 0; i < MAX_STAGES * R; ++i) cnt[i] = 0;
    }
    fence_mbar_init();
  }
  __syncthreads();
  // Dependent launches may start their weight prefetch as soon as every CTA of this grid runs;
  // they wait (griddepcontrol.wait) for this grid to finish before touching its outputs.
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane != 0) return;
    // ---------------- producer (weights only: never waits on the previous grid) ----------------
    const uint64_t pol = l2_evict_first_policy();
    long long it = 0;
    int s = 0;
    uint32_t ephase = 1;  // iteration it >= S waits for completion (it/S - 1) of empty[s]: parity (it/S - 1) & 1
    for (long long tile = blockIdx.x; tile < L.n_tiles; tile += gridDim.x, ++it) {
      if (it == PRE_STAGES) hold_for_activations(xin);
      if (it >= S) {
        if (!wait_or_abort(&empty[s], ephase, abort_flag)) {
          atomicOr(a.status, ST_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
      }
      const TileRef tr = tile_ref(a, L, tile);
      const uintptr_t start = reinterpret_cast<uintptr_t>(tr.w) + static_cast<uintptr_t>(tr.r0) * a.row_bytes;
      const uintptr_t al = start & ~static_cast<uintptr_t>(15);
      TileDesc& td = descs[s];
      td.out = tr.out;
      td.bias = tr.bias;
      td.r0 = static_cast<int>(tr.r0);
      td.nr = tr.nr;
      td.stride = static_cast<int>(tr.stride);
      td.misalign = static_cast<int>(start - al);
      uint8_t* dst = smem + L.stage_off + s * L.stage_bytes;
      if (L.row_stride != a.row_bytes) {  // padded rows (16-byte multiples, so start == al): one copy per row
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(tr.nr) * a.row_bytes);
        for (int i = 0; i < tr.nr; ++i)
          bulk_g2s(dst + i * L.row_stride, reinterpret_cast<const void*>(start + static_cast<uintptr_t>(i) * a.row_bytes),
                   a.row_bytes, &full[s], pol);
      } else {
        const uint32_t bytes = static_cast<uint32_t>((start - al + static_cast<long long>(tr.nr) * a.row_bytes + 15) & ~15ull);
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s(dst, reinterpret_cast<const void*>(al), bytes, &full[s], pol);
      }
      if (++s == S) {
        s = 0;
        ephase ^= 1u;
      }
    }
    // Drain: the last copies issued into each stage must land before the CTA may exit.
    for (long long j = (it > S ? it - S : 0); j < it; ++j) {
      if (!mbar_wait(&full[j % S], static_cast<uint32_t>((j / S) & 1))) atomicOr(a.status, ST_TIMEOUT_DRAIN);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int cw = warp - 1;
  uint8_t* act = smem + L.act_off;
  griddep_wait();  // the activations may be the previous grid's output
  constexpr bool TP = MODE == RowOut::StoreTp;
  const uint32_t tp_e = TP ? *reinterpret_cast<volatile const uint32_t*>(a.tp.peer[a.tp.rank] + TP_CTRL_OFF + 4) : 0u;
  const size_t tp_slot =
      TP ? (static_cast<size_t>(tp_e & 1u) * TP_MAX_WORLD + a.tp.rank) * TP_SLOT_BYTES : 0;  // [parity][rank]
  load_act(a, act, threadIdx.x - 32, xin);
  named_bar_sync(1, CONSUMERS);

  XRegs xr;
  if constexpr (XREG) load_xregs(F, a, act, lane, xr);
  const bool full_warp = units_per_row(F, a.K) == 32;  // every lane has a unit (XREG rows)
  const Q4kLane q4l = q4k_lane(lane);

  unsigned long long best = 0ull;
  bool dead = false;
  int s = 0;
  uint32_t fphase = 0;
  if constexpr (SLICE) {
    // Long Q4_K rows at batch 1 (U > 32 units): the row is cut into NSL slices of 16 units.  Warp cw
    // owns slice sl = cw % NSL for good, so the activations of its lane's unit stay in registers,
    // and takes the row pairs p = j, j + G, ... of every tile (j = cw / NSL): half-warp h computes
    // row 2p + h.  The slice partials of a row meet in shared memory; the warp that adds the
    // last one sums them in slice order (a fixed order: deterministic results) and stores.
    const int U = a.K / 128;
    const int NSL = (U + SLICE_UNITS - 1) / SLICE_UNITS;
    const int G = CONSUMER_WARPS / NSL;
    const int sl = cw % NSL, j = cw / NSL;
    const int h = lane >> 4;
    const int u = sl * SLICE_UNITS + (lane & (SLICE_UNITS - 1));
    const bool unit_live = u < U;
    const int ue = unit_live ? u : 0;  // dead lanes read a valid unit and contribute 0
    load_xregs(F, a, act, ue, xr);
    const Q4kLane ql = q4k_lane(ue);
    float* part = reinterpret_cast<float*>(smem + L.part_off);
    int* cnt = reinterpret_cast<int*>(smem + L.part_off + MAX_STAGES * R * SLICE_UNITS * 4);
    for (long long tile = blockIdx.x; tile < L.n_tiles; tile += gridDim.x) {
      if (!dead && !wait_or_abort(&full[s], fphase, abort_flag)) {
        atomicOr(a.status, ST_TIMEOUT_FULL);
        *abort_flag = 1;
        dead = true;
      }
      if (!dead && j < G) {
        const TileDesc tr = descs[s];
        const uint8_t* tb = smem + L.stage_off + s * L.stage_bytes + tr.misalign;
        const int pairs = (tr.nr + 1) >> 1;
        for (int p = j; p < pairs; p += G) {
          const int r = 2 * p + h;
          const bool valid = r < tr.nr;
          float v = 0.0f;
          row_q4k_full(tb + static_cast<size_t>(valid ? r : 0) * a.row_bytes, v, xr, ql);
          v = unit_live ? v : 0.0f;
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
          int last = 0;
          if ((lane & 15) == 0 && valid) {
            volatile float* pr = part + (s * R + r) * SLICE_UNITS;
            pr[sl] = v;
            __threadfence_block();
            last = atomicAdd(cnt + s * R + r, 1) == NSL - 1;
            if (last) {
              __threadfence_block();
              float y = pr[0];
              for (int q = 1; q < NSL; ++q) y += pr[q];
              cnt[s * R + r] = 0;
              const long long row = static_cast<long long>(tr.r0) + r;
              if constexpr (MODE == RowOut::Store) {
                tr.out[row] = (tr.bias != nullptr ? tr.bias[row] : 0.0f) + y;  // cpu_kernel.c:596-597
              } else {
                const float sc = tr.bias != nullptr ? tr.bias[row] + y : y;
                const unsigned long long k = argmax_key(sc, static_cast<uint32_t>(a.row0 + row));
                best = k > best ? k : best;
              }
            }
          }
        }
      }
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == S) {
        s = 0;
        fphase ^= 1u;
      }
    }
  } else if constexpr (EXACT) {
    // Exact mode: slot g of a tile is rows EX_ROWS*g .. EX_ROWS*g + EX_ROWS-1; slot g belongs to
    // consumer warp (it*G + g) % CONSUMER_WARPS.  Lane EX_LPR*r + c runs accumulators 2c, 2c+1 of row
    // EX_ROWS*g + r (the x86 float order).
    const int G = (R + EX_ROWS - 1) / EX_ROWS;
    const int stepg = G % CONSUMER_WARPS;
    const int c = lane & (EX_LPR - 1), rq = lane / EX_LPR;
    int firstg = cw;
    for (long long tile = blockIdx.x; tile < L.n_tiles; tile += gridDim.x) {
      if (!dead && !wait_or_abort(&full[s], fphase, abort_flag)) {
        atomicOr(a.status, ST_TIMEOUT_FULL);
        *abort_flag = 1;
        dead = true;
      }
      if (!dead && firstg < G) {
        const TileDesc tr = descs[s];
        const uint8_t* tb = smem + L.stage_off + s * L.stage_bytes + tr.misalign;
        const int groups = (tr.nr + EX_ROWS - 1) / EX_ROWS;
        for (int g = firstg; g < groups; g += CONSUMER_WARPS) {
          const int r = EX_ROWS * g + rq;
          const bool valid = r < tr.nr;
          const uint8_t* rowp = tb + static_cast<size_t>(valid ? r : EX_ROWS * g) * L.row_stride;
          float y[MTOK];
          exact_row<F, MTOK>(a, act, rowp, c, y);
          const long long row = static_cast<long long>(tr.r0) + r;
          if constexpr (MODE == RowOut::Store) {
            // cpu_kernel.c:594-597: out = b + dot with b = bias or 0.0f; lane c stores tokens c, c + EX_LPR, ...
#pragma unroll
            for (int t = 0; t < MTOK; ++t)
              if (valid && t < a.m && (t % EX_LPR) == c)
                tr.out[static_cast<size_t>(t) * tr.stride + row] = (tr.bias != nullptr ? tr.bias[row] : 0.0f) + y[t];
          } else if constexpr (MODE == RowOut::Argmax) {
            // native.c:500-514: score = dot, plus the output bias when there is one
            const float sc = tr.bias != nullptr ? y[0] + tr.bias[row] : y[0];
            if (valid && c == 0) {
              const unsigned long long k = argmax_key(sc, static_cast<uint32_t>(a.row0 + row));
              best = k > best ? k : best;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      firstg -= stepg;
      if (firstg < 0) firstg += CONSUMER_WARPS;
      if (++s == S) {
        s = 0;
        fphase ^= 1u;
      }
    }
  } else {
  const int step = R % CONSUMER_WARPS;
  int first = cw;  // first slot of this warp in the current tile: (cw - it*R) mod CONSUMER_WARPS
  for (long long tile = blockIdx.x; tile < L.n_tiles; tile += gridDim.x) {
    {
      if (!dead && !wait_or_abort(&full[s], fphase, abort_flag)) {
        atomicOr(a.status, ST_TIMEOUT_FULL);
        *abort_flag = 1;
        dead = true;
      }
      if (!dead && first < R) {  // this warp owns at least one slot of the tile
        const TileDesc tr = descs[s];
        const long long r0 = tr.r0;
        const uint8_t* tb = smem + L.stage_off + s * L.stage_bytes + tr.misalign;
        for (int r = first; r < tr.nr; r += CONSUMER_WARPS) {
          float acc[MTOK];
#pragma unroll
          for (int t = 0; t < MTOK; ++t) acc[t] = 0.0f;
          const uint8_t* rowp = tb + static_cast<size_t>(r) * a.row_bytes;
          if constexpr (F == Fmt::Q8_0xQ8_0) {
            row_q8_0<MODE, MTOK, XREG>(a, act, rowp, r0 + r, acc, lane, xr);
          } else if constexpr (F == Fmt::Q4_KxQ8_K) {
            if constexpr (XREG && MTOK == 1 && MODE != RowOut::Partials) {
              if (full_warp) {
                row_q4k_full(rowp, acc[0], xr, q4l);
              } else {
                row_q4k_q8k<MODE, MTOK, XREG>(a, act, rowp, r0 + r, acc, lane, xr);
              }
            } else if (XREG && full_warp) {
              row_q4k_q8k<MODE, MTOK, XREG, XREG>(a, act, rowp, r0 + r, acc, lane, xr);
            } else {
              row_q4k_q8k<MODE, MTOK, XREG>(a, act, rowp, r0 + r, acc, lane, xr);
            }
          } else if constexpr (F == Fmt::Q4_0xQ8_0 || F == Fmt::Q5_0xQ8_0) {
            row_b32<F, MODE, MTOK>(a, act, rowp, r0 + r, acc, lane);
          } else if constexpr (F == Fmt::Q5_KxQ8_K) {
            row_q5k_q8k<MODE, MTOK>(a, act, rowp, r0 + r, acc, lane);
          } else if constexpr (F == Fmt::Q6_KxQ8_K) {
            row_q6k_q8k<MODE, MTOK>(a, act, rowp, r0 + r, acc, lane);
          } else if constexpr (F == Fmt::Q5_KxF32 || F == Fmt::Q6_KxF32) {
            row_k56_f32<F, MODE, MTOK>(a, act, rowp, acc, lane);
          } else {
            row_q4k_f32<MODE, MTOK>(a, act, rowp, acc, lane);
          }
          if constexpr (MODE != RowOut::Partials) {
            const long long row = r0 + r;
            float mine = 0.0f;
#pragma unroll
            for (int t = 0; t < MTOK; ++t) {
              if (MTOK == 1 || t < a.m) {
                const float v = warp_sum(acc[t]);
                if (lane == t) mine = v;
              }
            }
            if (lane < a.m) {
              const float y = (tr.bias != nullptr ? tr.bias[row] : 0.0f) + mine;  // cpu_kernel.c:596-597
              if constexpr (TP) {  // (partial, tag) into entry [parity][rank][t*n + row]: every rank's, or ours
                const size_t off = tp_slot + (static_cast<size_t>(lane) * a.seg[0].n_rows + row) * 8;
                const unsigned long long v = (static_cast<unsigned long long>(tp_e + 1u) << 32) | __float_as_uint(y);
                if (a.tp.world <= TP_DIRECT_WORLD) {
                  for (int r = 0; r < a.tp.world; ++r) st_relaxed_sys_u64(a.tp.peer[r] + off, v);
                } else {  // tp_finalize pushes it
                  *reinterpret_cast<unsigned long long*>(a.tp.peer[a.tp.rank] + off) = v;
                }
              } else if constexpr (MODE == RowOut::Store) {
                tr.out[static_cast<size_t>(lane) * tr.stride + row] = y;  // stride: int, outputs < 2^31
              } else {
                const unsigned long long k = argmax_key(y, static_cast<uint32_t>(a.row0 + row));
                best = k > best ? k : best;
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    first -= step;
    if (first < 0) first += CONSUMER_WARPS;
    if (++s == S) {
      s = 0;
      fphase ^= 1u;
    }
  }
  }  // EXACT
  if constexpr (TP) tp_finalize(a, L, tp_e, threadIdx.x - 32);
  if constexpr (MODE == RowOut::Argmax) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0 && best != 0ull) atomicMax(a.key, best);
  }
}

template <Fmt F, RowOut MODE, int MTOK, bool XREG = false, bool EXACT = false, bool SLICE = false>
cudaError_t launch_impl(const RowStreamArgs& a, const Layout& L, int grid, cudaStream_t st) {
  static int configured_smem = 0;  // per instantiation; the host API serialises its callers
  auto kern = rowstream_kernel<F, MODE, MTOK, XREG, EXACT, SLICE>;
  if (L.smem_total > configured_smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem_total);
    if (e != cudaSuccess) return e;
    configured_smem = L.smem_total;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = L.smem_total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a, L);
}

// The x86-float-order variants (RowStreamArgs::exact): Store and Argmax epilogues.
template <Fmt F, RowOut MODE>
cudaError_t launch_exact(const RowStreamArgs& a, const Layout& L, int grid, cudaStream_t st) {
  if (a.m <= 1) return launch_impl<F, MODE, 1, false, true>(a, L, grid, st);
  if constexpr (MODE == RowOut::Store) {
    if (a.m <= 2) return launch_impl<F, MODE, 2, false, true>(a, L, grid, st);
    if (a.m <= 4) return launch_impl<F, MODE, 4, false, true>(a, L, grid, st);
    if (a.m <= 8) return launch_impl<F, MODE, 8, false, true>(a, L, grid, st);
    return launch_impl<F, MODE, 16, false, true>(a, L, grid, st);
  }
  return cudaErrorInvalidValue;
}

template <Fmt F, RowOut MODE>
cudaError_t launch_mtok(const RowStreamArgs& a, const Layout& L, int grid, cudaStream_t st) {
  if constexpr (MODE == RowOut::Store || MODE == RowOut::Argmax) {
    if (a.exact) return launch_exact<F, MODE>(a, L, grid, st);
  }
  if constexpr (F == Fmt::Q8_0xQ8_0 || F == Fmt::Q4_KxQ8_K) {  // activations held in registers
    if (a.m == 1 && units_per_row(F, a.K) <= 32) return launch_impl<F, MODE, 1, true>(a, L, grid, st);
  }
  if constexpr (F == Fmt::Q4_KxQ8_K && (MODE == RowOut::Store || MODE == RowOut::Argmax)) {
    if (rowstream_sliced(a)) return launch_impl<F, MODE, 1, false, false, true>(a, L, grid, st);
  }
  if (a.m <= 1) return launch_impl<F, MODE, 1>(a, L, grid, st);
  if (a.m <= 2) return launch_impl<F, MODE, 2>(a, L, grid, st);
  if (a.m <= 4) return launch_impl<F, MODE, 4>(a, L, grid, st);
  if (a.m <= 8) return launch_impl<F, MODE, 8>(a, L, grid, st);
  return launch_impl<F, MODE, 16>(a, L, grid, st);
}

}  // namespace

}  // namespace ex
