// gemm_q8_tc.cu -- Q8_0 weight x Q8_0 activation GEMM on the 5th-generation tensor cores for
// prefill-sized batches: the batched form of dot_q8_0_q8_0 (src/gguf_dot_q8.c:436-480) that
// edgexpu_cpu_linear_quant_batch (src/cpu_kernel.c:545-644) runs per row and token.
//
// Arithmetic.  out[t][r] = bias[r] + sum_b (d_w[r][b] * d_x[t][b]) * ip[t][r][b], where
// ip = sum of the 32 int8 products of block b.  Every ip comes out of one tcgen05.mma kind::i8
// with K = 32 into its own int32 accumulator (exact), and the epilogue converts it (|ip| <= 32 *
// 127 * 127 < 2^24, exact in fp32) and accumulates the scaled blocks in fp32 -- the relaxed float
// order, within 1e-5 * sum |w*x| of the reference.
//
// Operands.  The GGUF blocks interleave a 2-byte scale with 32 quants, which no tensor-core
// layout can read, so the weight is repacked once per tensor (cached by the host): its quants as a
// row-major int8 matrix [n_rows][K] and its scales as floats in tile order.  The activations are
// quantized to Q8_0 (bit-exact with edgexpu_gguf_quantize_q8_0) into the same two forms.  Both
// int8 matrices are loaded by 2-D TMA with the 128-byte swizzle into K-major tiles; K steps past
// the end read zeros (and their scales are 0).
//
// Tile: 128 weight rows x 64 tokens, K chunks of 128 (4 blocks, 4 MMAs of N = 64).  Tensor memory:
// two buffers of 4 accumulators x 64 columns (512 columns), so the epilogue of one chunk overlaps
// the MMAs of the next.  Warps: 0 producer (TMA A and B tiles, bulk copies of the chunk's weight
// and activation scales), 1 MMA issuer, 2..17 epilogue (4 per 32-lane quadrant, 16 tokens each).
// Every wait is bounded; a timeout sets a status bit and all roles fall through to teardown.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "common.cuh"
#include "launch.h"
#include "quant.cuh"

namespace ex {
namespace {

constexpr int Q8_BM = 128;                    // weight rows per tile (MMA M)
constexpr int Q8_BN = 64;                     // tokens per tile (MMA N)
constexpr int Q8_KC = 128;                    // K bytes per chunk (4 blocks)
constexpr int Q8_BPC = Q8_KC / QK8_0;         // blocks per chunk
constexpr int QA_TILE = Q8_BM * Q8_KC;        // 16 KB
constexpr int QB_TILE = Q8_BN * Q8_KC;        // 8 KB
constexpr int QS_BYTES = Q8_BM * Q8_BPC * 4;  // weight scales of a chunk: [128 rows][4]
constexpr int QX_BYTES = Q8_BN * Q8_BPC * 4;  // activation scales of a chunk: [64 tokens][4]
constexpr int Q8_STAGES = 6;
constexpr int Q8_EPI_WARPS = 16;
constexpr int Q8_EPI_TOK = Q8_BN / 4;         // tokens per epilogue warp
constexpr int Q8_THREADS = 32 * (2 + Q8_EPI_WARPS);
constexpr uint32_t Q8_ACC_COLS = Q8_BPC * Q8_BN;  // one buffer: 256 columns
constexpr uint32_t Q8_TMEM_COLS = 512;

// kind::i8: D int32, A and B signed int8, K-major, N = 64, M = 128.
constexpr uint32_t IDESC_Q8 = (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(Q8_BN >> 3) << 17) |
                              (uint32_t(Q8_BM >> 4) << 24);

struct Q8Layout {
  static constexpr int STAGE = QA_TILE + QB_TILE + QS_BYTES + QX_BYTES;  // 27 KB
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = QA_TILE;
  static constexpr int S_OFF = QA_TILE + QB_TILE;
  static constexpr int X_OFF = S_OFF + QS_BYTES;
  static constexpr int BAR_OFF = Q8_STAGES * STAGE;
  static constexpr int N_BARS = 2 * Q8_STAGES + 4 + 1;
  static constexpr int MISC_OFF = BAR_OFF + 8 * N_BARS;
  static constexpr int ALLOC = MISC_OFF + 16 + 1024;
};
static_assert(Q8Layout::STAGE % 1024 == 0, "stages keep the 1024-byte alignment of the swizzled tiles");
static_assert(Q8Layout::ALLOC > 116 * 1024, "one CTA per SM keeps the tensor-memory allocation uncontended");
static_assert(Q8Layout::ALLOC <= 227 * 1024, "shared memory per CTA");

struct Q8KernelArgs {
  int n_rows, K, m, n_rt, n_tt, nch;
  const float* ws;    // weight scales [n_rt][nch][128][4]
  const float* xs;    // activation scales [n_tt][nch][64][4]
  const float* bias;
  float* out;
  long long out_stride;
  uint32_t* status;
};

__device__ __forceinline__ void q8_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void q8_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] = A x B (the accumulator is overwritten: enable-input-d false)
__device__ __forceinline__ void mma_i8_fresh(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(IDESC_Q8)
      : "memory");
}

__device__ __forceinline__ void q8_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void q8_ld8(uint32_t addr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(addr)
               : "memory");
}

// K-major tile with the 128-byte swizzle (as written by a SWIZZLE_128B TMA box of 128-byte rows):
// 8-row atoms of 128 bytes, 1024 bytes apart; descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t q8_sw128_desc(uint32_t smem_addr) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void q8_tma_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ bool q8_spin(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > WAIT_LIMIT_NS) return false;
    }
  }
}

__device__ __forceinline__ bool q8_warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const bool ok = wait_or_abort(bar, parity, abort_flag);
  return __all_sync(0xFFFFFFFFu, ok);
}

// ---- repacking ------------------------------------------------------------------------------------

// One thread per (row, block): the 32 quants into qs[row][32b..], the scale into the tile-ordered
// scale array; blocks of a chunk past the end of K get scale 0.
__global__ void q8_repack_weight_kernel(const uint8_t* __restrict__ w, int n_rows, int nb, int nch, uint8_t* __restrict__ qs,
                                        float* __restrict__ ws) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int n_rt = (n_rows + Q8_BM - 1) / Q8_BM;
  if (i >= (long long)n_rt * Q8_BM * nch * Q8_BPC) return;
  const int b = (int)(i % (nch * Q8_BPC));
  const long long row = i / (nch * Q8_BPC);
  const int c = b / Q8_BPC, bj = b % Q8_BPC;
  float d = 0.0f;
  if (row < n_rows && b < nb) {
    const uint8_t* blk = w + (size_t)row * nb * Q8_0_BYTES + (size_t)b * Q8_0_BYTES;
    d = fp16_bits_to_float(static_cast<uint32_t>(blk[0]) | (static_cast<uint32_t>(blk[1]) << 8));
    uint8_t* dst = qs + (size_t)row * nb * QK8_0 + (size_t)b * QK8_0;
#pragma unroll
    for (int k = 0; k < QK8_0; ++k) dst[k] = blk[2 + k];
  }
  const long long rt = row / Q8_BM, r = row % Q8_BM;
  ws[((rt * nch + c) * Q8_BM + r) * Q8_BPC + bj] = d;
}

// One warp per (token, block): Q8_0-quantize 32 values (bit-exact with edgexpu_gguf_quantize_q8_0)
// or take a Q8_0 block as it is; quants into xq[t][32b..], the scale into the tile-ordered array.
template <bool FROM_F32>
__global__ void __launch_bounds__(256) q8_pack_act_kernel(const float* __restrict__ x, const uint8_t* __restrict__ xq_in,
                                                          int m, int K, int nch, int8_t* __restrict__ xq,
                                                          float* __restrict__ xs) {
  const int nb = K / QK8_0, lane = threadIdx.x & 31;
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int n_tt = (m + Q8_BN - 1) / Q8_BN;
  if (gw >= (long long)n_tt * Q8_BN * nch * Q8_BPC) return;
  const int t = (int)(gw / (nch * Q8_BPC)), b = (int)(gw % (nch * Q8_BPC));
  float d = 0.0f;
  if (t < m && b < nb) {
    int q;
    if constexpr (FROM_F32) {
      uint32_t dbits;
      q = warp_q8_0(x[(size_t)t * K + (size_t)b * QK8_0 + lane], &dbits);
      d = fp16_bits_to_float(dbits);
    } else {
      const uint8_t* blk = xq_in + ((size_t)t * nb + b) * Q8_0_BYTES;
      q = static_cast<int8_t>(blk[2 + lane]);
      d = fp16_bits_to_float(static_cast<uint32_t>(blk[0]) | (static_cast<uint32_t>(blk[1]) << 8));
    }
    xq[(size_t)t * K + (size_t)b * QK8_0 + lane] = static_cast<int8_t>(q);
  }
  if (lane == 0) {
    const int tt = t / Q8_BN, r = t % Q8_BN, c = b / Q8_BPC, bj = b % Q8_BPC;
    xs[(((size_t)tt * nch + c) * Q8_BN + r) * Q8_BPC + bj] = d;
  }
}

// ---- the GEMM ---------------------------------------------------------------------------------------

__global__ void __launch_bounds__(Q8_THREADS, 1)
    gemm_q8_tc_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                      const Q8KernelArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Q8Layout::BAR_OFF);
  uint64_t* full = bars;                     // the chunk's tiles and scales landed (tx bytes)
  uint64_t* empty = full + Q8_STAGES;        // the epilogue is done with the stage (16 warps)
  uint64_t* acc_full = empty + Q8_STAGES;    // the MMAs of an accumulator buffer completed
  uint64_t* acc_empty = acc_full + 2;        // the epilogue drained an accumulator buffer (16 warps)
  uint64_t* fin = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Q8Layout::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Q8Layout::MISC_OFF + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < Q8_STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], Q8_EPI_WARPS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], Q8_EPI_WARPS);
    }
    mbar_init(fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {  // a warp that has not diverged: the warp-collective allocation is converged
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(Q8_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  q8_fence_before();
  __syncthreads();
  q8_fence_after();
  const uint32_t tmem = *tmem_slot;
  const long long n_tiles = (long long)a.n_rt * a.n_tt;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      uint32_t s = 0, ph = 0;
      long long issued = 0;
      bool ok = true;
      for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        const int rt = (int)(tile / a.n_tt), tt = (int)(tile % a.n_tt);
        for (int c = 0; c < a.nch; ++c) {
          if (!wait_or_abort(&empty[s], ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * Q8Layout::STAGE;
          mbar_arrive_expect_tx(&full[s], QA_TILE + QB_TILE + QS_BYTES + QX_BYTES);
          q8_tma_2d(st + Q8Layout::A_OFF, &amap, c * Q8_KC, rt * Q8_BM, &full[s]);
          q8_tma_2d(st + Q8Layout::B_OFF, &bmap, c * Q8_KC, tt * Q8_BN, &full[s]);
          bulk_g2s(st + Q8Layout::S_OFF, a.ws + ((size_t)rt * a.nch + c) * Q8_BM * Q8_BPC, QS_BYTES, &full[s], pol);
          bulk_g2s(st + Q8Layout::X_OFF, a.xs + ((size_t)tt * a.nch + c) * Q8_BN * Q8_BPC, QX_BYTES, &full[s], pol);
          ++issued;
          if (++s == Q8_STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(a.status, ST_TIMEOUT_EMPTY);
      }
      bool drained = true;  // no copy may still be landing when the CTA exits
      for (long long n = issued - Q8_STAGES; n < issued; ++n)
        if (n >= 0 && !mbar_wait(&full[n % Q8_STAGES], (uint32_t)((n / Q8_STAGES) & 1))) drained = false;
      if (!drained) atomicOr(a.status, ST_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t s = 0, ph = 0, accb = 0;
      bool ok = true;
      for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        for (int c = 0; ok && c < a.nch; ++c) {
          const uint32_t ab = accb & 1u;
          if (!q8_spin(&acc_empty[ab], ((accb >> 1) & 1u) ^ 1u, abort_flag) || !q8_spin(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          q8_fence_after();
          const uint8_t* st = smem + s * Q8Layout::STAGE;
          const uint64_t ad = q8_sw128_desc(smem_u32(st + Q8Layout::A_OFF));
          const uint64_t bd = q8_sw128_desc(smem_u32(st + Q8Layout::B_OFF));
#pragma unroll
          for (int b = 0; b < Q8_BPC; ++b) {
            const uint64_t k = (uint64_t)((b * QK8_0) >> 4);
            mma_i8_fresh(tmem + ab * Q8_ACC_COLS + b * Q8_BN, ad + k, bd + k);
          }
          q8_commit(&acc_full[ab]);
          ++accb;
          if (++s == Q8_STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(a.status, ST_TIMEOUT_FULL);
      }
      q8_commit(fin);  // everything issued above completes before tensor memory is released
      if (!mbar_wait(fin, 0)) atomicOr(a.status, ST_TIMEOUT_DRAIN);
    }
  } else {
    // Epilogue: a warp reads the tensor-memory lanes of its own quadrant, warp % 4 (rows 32q + lane);
    // the four warps of each quadrant take tokens Q8_EPI_TOK * j ...
    const int q = warp & 3, j = (warp - 2) >> 2;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(Q8_EPI_TOK * j);
    uint32_t s = 0, ph = 0, accb = 0;
    bool ok = true;
    for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
      const int rt = (int)(tile / a.n_tt), tt = (int)(tile % a.n_tt);
      const int r = 32 * q + lane, n = rt * Q8_BM + r;
      float acc[Q8_EPI_TOK];
#pragma unroll
      for (int e = 0; e < Q8_EPI_TOK; ++e) acc[e] = 0.0f;
      for (int c = 0; c < a.nch; ++c) {
        const uint32_t ab = accb & 1u;
        if (!q8_warp_wait(&full[s], ph, abort_flag) || !q8_warp_wait(&acc_full[ab], (accb >> 1) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        q8_fence_after();
        const uint8_t* st = smem + s * Q8Layout::STAGE;
        const float4 dw4 = reinterpret_cast<const float4*>(st + Q8Layout::S_OFF)[r];
        const float dw[Q8_BPC] = {dw4.x, dw4.y, dw4.z, dw4.w};
        const float4* dx4 = reinterpret_cast<const float4*>(st + Q8Layout::X_OFF) + Q8_EPI_TOK * j;
#pragma unroll
        for (int b = 0; b < Q8_BPC; ++b) {
          uint32_t v0[8], v1[8];
          const uint32_t col = lane_base + ab * Q8_ACC_COLS + b * Q8_BN;
          __syncwarp();
          q8_ld8(col, v0);
          q8_ld8(col + 8, v1);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int e = 0; e < Q8_EPI_TOK; ++e) {
            const float4 dx = dx4[e];
            const float dxb = b == 0 ? dx.x : (b == 1 ? dx.y : (b == 2 ? dx.z : dx.w));
            const int ip = static_cast<int>(e < 8 ? v0[e] : v1[e - 8]);
            acc[e] = fmaf(dw[b] * dxb, static_cast<float>(ip), acc[e]);
          }
        }
        q8_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&acc_empty[ab]);
          mbar_arrive(&empty[s]);
        }
        ++accb;
        if (++s == Q8_STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (!ok) break;
      if (n < a.n_rows) {
        const float bv = a.bias != nullptr ? a.bias[n] : 0.0f;
#pragma unroll
        for (int e = 0; e < Q8_EPI_TOK; ++e) {
          const int t = tt * Q8_BN + Q8_EPI_TOK * j + e;
          if (t < a.m) a.out[(size_t)t * a.out_stride + n] = acc[e] + bv;
        }
      }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicOr(a.status, ST_TIMEOUT_FULL);
    }
  }

  q8_fence_before();
  __syncthreads();
  q8_fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Q8_TMEM_COLS) : "memory");
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn q8_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// An int8 matrix [rows][K] (row stride K bytes) as 128-byte x box_rows swizzled boxes.
bool q8_map(CUtensorMap* map, const void* base, int K, int rows, int box_rows) {
  EncodeTiledFn enc = q8_encode_tiled();
  if (enc == nullptr) return false;
  std::memset(map, 0, sizeof(*map));
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K};
  const cuuint32_t box[2] = {(cuuint32_t)Q8_KC, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t q8_weight_pack_bytes(int n_rows, int K) {
  const size_t n_rt = (size_t)(n_rows + Q8_BM - 1) / Q8_BM, nch = (size_t)(K / QK8_0 + Q8_BPC - 1) / Q8_BPC;
  return (((size_t)n_rows * K + 255) & ~(size_t)255) + n_rt * nch * QS_BYTES;
}

size_t q8_act_pack_bytes(int m, int K) {
  const size_t n_tt = (size_t)(m + Q8_BN - 1) / Q8_BN, nch = (size_t)(K / QK8_0 + Q8_BPC - 1) / Q8_BPC;
  return (((size_t)m * K + 255) & ~(size_t)255) + n_tt * nch * QX_BYTES;
}

cudaError_t launch_q8_repack_weight(const uint8_t* w, int n_rows, int K, uint8_t* pack, cudaStream_t st) {
  if (n_rows <= 0 || K <= 0 || K % QK8_0 != 0) return cudaErrorInvalidValue;
  const int nb = K / QK8_0, nch = (nb + Q8_BPC - 1) / Q8_BPC, n_rt = (n_rows + Q8_BM - 1) / Q8_BM;
  uint8_t* qs = pack;
  float* ws = reinterpret_cast<float*>(pack + (((size_t)n_rows * K + 255) & ~(size_t)255));
  const long long n = (long long)n_rt * Q8_BM * nch * Q8_BPC;
  q8_repack_weight_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, n_rows, nb, nch, qs, ws);
  return cudaGetLastError();
}

cudaError_t launch_q8_pack_act(const float* x, const uint8_t* xq, int m, int K, uint8_t* pack, cudaStream_t st) {
  if (m <= 0 || K <= 0 || K % QK8_0 != 0) return cudaErrorInvalidValue;
  const int nb = K / QK8_0, nch = (nb + Q8_BPC - 1) / Q8_BPC, n_tt = (m + Q8_BN - 1) / Q8_BN;
  int8_t* q = reinterpret_cast<int8_t*>(pack);
  float* xs = reinterpret_cast<float*>(pack + (((size_t)m * K + 255) & ~(size_t)255));
  const long long warps = (long long)n_tt * Q8_BN * nch * Q8_BPC;
  const unsigned grid = (unsigned)((warps + 7) / 8);
  if (x != nullptr)
    q8_pack_act_kernel<true><<<grid, 256, 0, st>>>(x, nullptr, m, K, nch, q, xs);
  else
    q8_pack_act_kernel<false><<<grid, 256, 0, st>>>(nullptr, xq, m, K, nch, q, xs);
  return cudaGetLastError();
}

cudaError_t launch_q8_gemm(const uint8_t* wpack, int n_rows, const uint8_t* apack, int m, int K, const float* bias,
                           float* out, long long out_stride, uint32_t* status, const DeviceInfo& dev, cudaStream_t st) {
  if (n_rows <= 0 || m <= 0 || K <= 0 || K % QK8_0 != 0 || K % 16 != 0) return cudaErrorInvalidValue;
  const int nb = K / QK8_0, nch = (nb + Q8_BPC - 1) / Q8_BPC;
  CUtensorMap amap, bmap;
  if (!q8_map(&amap, wpack, K, n_rows, Q8_BM) || !q8_map(&bmap, apack, K, m, Q8_BN)) return cudaErrorInvalidValue;
  Q8KernelArgs k;
  k.n_rows = n_rows;
  k.K = K;
  k.m = m;
  k.n_rt = (n_rows + Q8_BM - 1) / Q8_BM;
  k.n_tt = (m + Q8_BN - 1) / Q8_BN;
  k.nch = nch;
  k.ws = reinterpret_cast<const float*>(wpack + (((size_t)n_rows * K + 255) & ~(size_t)255));
  k.xs = reinterpret_cast<const float*>(apack + (((size_t)m * K + 255) & ~(size_t)255));
  k.bias = bias;
  k.out = out;
  k.out_stride = out_stride;
  k.status = status;
  static bool attr_set = false;
  if (!attr_set) {
    const cudaError_t e = cudaFuncSetAttribute(gemm_q8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Q8Layout::ALLOC);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const long long tiles = (long long)k.n_rt * k.n_tt;
  const int grid = (int)(tiles < dev.sm_count ? tiles : dev.sm_count);
  gemm_q8_tc_kernel<<<grid, Q8_THREADS, Q8Layout::ALLOC, st>>>(amap, bmap, k);
  return cudaGetLastError();
}

}  // namespace ex
