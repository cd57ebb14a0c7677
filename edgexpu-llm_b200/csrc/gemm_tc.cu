// gemm_tc.cu -- Q4_K weight x Q8_K activation GEMM on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, int32 accumulators in tensor memory) for prefill-sized batches: the
// batched form of dot_q4_k_q8_k (src/gguf_dot_q8.c:603-762) that
// edgexpu_cpu_linear_quant_batch (src/cpu_kernel.c:545-644) runs per row and token.
//
// Arithmetic.  Per super-block the reference computes, in int32,
//   sumi = sum_j sc_j * sum_{l<32} q4 * q8      summ = sum_j m_j * (bsum_2j + bsum_2j+1)
// and then acc += d_x*d_w*sumi - d_x*dmin_w*summ (gguf_dot_q8.c:711-759).
//  * sumi on the tensor cores.  The folded weight v = sc_j * q4 lies in [0, 945] (10 bits); it
//    is split into v = 256*h + l with l in [-128, 127] and h in [0, 4], and two int8
//    contractions over the super-block accumulate L = sum l*q8 and H = sum h*q8 in int32, so
//    sumi = L + 256*H exactly.
//  * summ on the CUDA cores.  It has only 8 terms per super-block: m_j (6-bit, unsigned) times
//    the 32-element activation sums S_j (13-bit, signed).  The packing kernel stores the S_j as
//    16-bit pairs, and four dp2a (two 16-bit x 8-bit products each) give summ exactly.
//
// Float conversion without I2F.  The L and H accumulators start at the bit pattern 0x4B400000
// (1.5 * 2^23 as a float) instead of 0; the MMA adds exact int32 products to it, and since
// |L| <= 128*127*256 < 2^22 (likewise H and summ), the float value of the bits is
// 1.5*2^23 + L exactly, so the epilogue converts with one FADD.
//
// Shapes.  A tcgen05.mma of M = 128, K = 32 takes about the same time for every N up to 256
// (measured on B200), so the tile is 128 weight rows x 128 tokens with N = 128 MMAs: 16 MMAs
// per super-block and tile.  Tensor-memory columns (of 512):
//   [0,128) L  [128,256) H    accumulator buffer 0
//   [256,384) L [384,512) H   accumulator buffer 1
// Two buffers let the epilogue drain super-block s while the MMAs of s+1 run.  Operands come
// from shared memory: A (the expanded weight, L and H parts) and B (activations) are K-major
// tiles with the 128-byte swizzle, one K-half (128 elements) per pipeline stage.
//
// Batches of 9..63 tokens use the same kernel with 16-token tiles (template parameter BN):
// N = 16 MMAs, 64 tensor-memory columns, one epilogue warp per quadrant (10 warps), and the
// super-blocks of each row tile split into K ranges over several CTAs, whose fp32 partial sums
// tc_split_reduce_kernel adds in range order.
//
// Warp roles (22 warps with 128-token tiles):
//   0      producer: 2-D TMA of the raw Q4_K super-block of 128 rows (tensor map, zero-filled
//          past the last row), bulk copies of activation tiles and per-token scale data
//   1      tensor-memory allocation and the single-thread MMA issuer
//   2..5   converters: one weight row per thread, nibbles and 6-bit scales -> L/H tiles
//   6..21  epilogue: 4 warps per 32-lane quadrant, 32 tokens each: drain accumulators (loads
//          of the next 8-token group in flight while the current one is computed), mins term,
//          scale, accumulate in fp32 registers, store
// The epilogue is the busiest role (about 12 operations per output and super-block), so it
// gets most of the warps; 4 warps per quadrant and 8-token load groups measured fastest with
// 128-token tiles.
// Every wait is bounded; a timeout sets a status bit, raises the CTA abort flag and all roles
// fall through to teardown (copies drained, MMAs committed, tensor memory freed).  The kernel
// needs a whole SM (about 196 / 140 KB of shared memory), so its tensor-memory allocation is
// never contended by another CTA.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "common.cuh"
#include "launch.h"
#include "quant.cuh"

namespace ex {
namespace {

constexpr int TC_BM = 128;                       // weight rows per tile (MMA M)
constexpr int KH_BYTES = 128;                    // K elements (int8 bytes) per stage
constexpr int A_TILE = TC_BM * KH_BYTES;         // 16 KB, one part (L or H) of a stage
constexpr int RAW_BYTES = TC_BM * Q4_K_BYTES;    // one super-block of 128 rows: 18432
constexpr int N_STAGES = 3;
constexpr int NR_STAGES = 2;
constexpr int NX_STAGES = 4;
constexpr int N_CONV_WARPS = 4;
#ifndef EX_TC_EPI_PER_Q
#define EX_TC_EPI_PER_Q 4
#endif
constexpr int EG = 8;                            // tokens per tensor-memory load group
constexpr int WARP_PROD = 0;
constexpr int WARP_MMA = 1;
constexpr int WARP_CONV0 = 2;
constexpr int WARP_EPI0 = WARP_CONV0 + N_CONV_WARPS;

constexpr uint32_t ACC_BIAS = 0x4B400000u;
constexpr float ACC_BIAS_F = 12582912.0f;

// Everything that depends on the token tile BN (MMA N): 128 for prefill batches, 16 for batches
// of 9..63 tokens (the decode batches of the configurations), where a 128-token tile would leave
// most of every MMA and of the epilogue idle.
template <int BN>
struct Cfg {
  static_assert(BN == 16 || BN == 128, "token tiles of 16 or 128");
  static constexpr int B_TILE = BN * KH_BYTES;               // 16 KB / 2 KB
  static constexpr int AUX_DX = BN * 4;                      // d of the tile's tokens
  static constexpr int AUX_BYTES = AUX_DX + BN * 16;         // + the eight 16-bit sub-block sums of each token
  static constexpr int EPI_PER_Q = BN == 128 ? EX_TC_EPI_PER_Q : 1;  // epilogue warps per 32-lane quadrant
  static constexpr int N_EPI_WARPS = 4 * EPI_PER_Q;
  static constexpr int EPI_TOK = BN / EPI_PER_Q;             // tokens per epilogue warp
  static constexpr int THREADS = 32 * (WARP_EPI0 + N_EPI_WARPS);
  static constexpr uint32_t ACC_COLS = 2 * BN;               // L and H of one buffer
  static constexpr uint32_t TMEM_COLS = BN == 128 ? 512 : 64; // two buffers, a power of two >= 32
  // kind::i8 instruction descriptor: D int32 (c_format 2 at bit 4), A and B signed int8
  // (formats 1 at bits 7 and 10), both K-major, N>>3 at bit 17, M>>4 at bit 24.
  static constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) |
                                    (uint32_t(TC_BM >> 4) << 24);
  // shared memory
  static constexpr int A_OFF = 0;                                  // [stage][L, H] 32 KB
  static constexpr int B_OFF = A_OFF + N_STAGES * 2 * A_TILE;      // [stage] B_TILE
  static constexpr int R_OFF = B_OFF + N_STAGES * B_TILE;          // [raw stage] 18 KB
  static constexpr int X_OFF = R_OFF + NR_STAGES * RAW_BYTES;      // [aux stage]
  static constexpr int BAR_OFF = X_OFF + NX_STAGES * AUX_BYTES;
  static constexpr int N_BARS = 3 * N_STAGES + 2 * NR_STAGES + 2 * NX_STAGES + 4 + 1;
  static constexpr int MISC_OFF = BAR_OFF + 8 * N_BARS;
  static constexpr int BYTES = MISC_OFF + 16;
  static constexpr int ALLOC = BYTES + 1024;  // base rounded up to 1024 for the swizzled tiles
  static_assert(ALLOC > 116 * 1024, "one CTA per SM keeps the tensor-memory allocation uncontended");
  static_assert(ALLOC <= 227 * 1024, "shared memory per CTA");
  static_assert(R_OFF % 1024 == 0 && B_TILE % 1024 == 0 && AUX_BYTES % 16 == 0 && BAR_OFF % 8 == 0, "alignment");
};

// Work item = (row tile, token tile, K range): with n_ks > 1 the super-blocks of a row tile are
// split over several CTAs (sb_per each), which write fp32 partial sums for tc_split_reduce_kernel.
struct TcKernelArgs {
  int n_rows, row_bytes, nb, m, n_tt, n_rt, n_ks, sb_per;
  const uint8_t* w;       // Q4_K rows (header of each super-block for the epilogue)
  const uint8_t* bt;      // activation tiles [n_tt][nb][2][B_TILE]
  const uint8_t* aux;     // [n_tt][nb][AUX_BYTES]: d[BN] floats, sums[BN][4] words of two int16
  const float* bias;
  float* out;
  long long out_stride;
  float* part;            // n_ks > 1: partial sums [n_ks][m][n_rows]
  int32_t* partials;      // non-null: write (sumi, summ) per (token, row, super-block) instead of out
  uint32_t* status;
};

// Row tile, token tile and super-block range of work item `tile` (128-token tiles are never split).
template <int BN>
__device__ __forceinline__ void tc_item(const TcKernelArgs& a, long long tile, int& rt, int& tt, int& ks, int& sb0,
                                        int& sb1) {
  if constexpr (BN == 128) {
    rt = (int)(tile / a.n_tt);
    tt = (int)(tile - (long long)rt * a.n_tt);
    ks = 0;
    sb0 = 0;
    sb1 = a.nb;
    return;
  }
  const long long per_rt = (long long)a.n_tt * a.n_ks;
  rt = (int)(tile / per_rt);
  const int rem = (int)(tile - (long long)rt * per_rt);
  tt = rem / a.n_ks;
  ks = rem - tt * a.n_ks;
  sb0 = ks * a.sb_per;
  sb1 = min(a.nb, sb0 + a.sb_per);
}

// ---- tcgen05 / TMA wrappers -------------------------------------------------------------------

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t addr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(addr), "r"(ncols) : "memory");
}

// D[tmem] += A[smem descriptor] x B[smem descriptor]
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, 1, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t addr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t addr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(addr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major tile with the 128-byte swizzle: 8-row atoms of
// 128 bytes, atoms 1024 bytes apart (stride byte offset), leading byte offset 16 (unused for
// this layout), descriptor version 1, layout type 2 (SWIZZLE_128B).  The tile base must be
// 1024-byte aligned; a K step inside the atom adds its byte offset to the start address.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Generic-proxy shared-memory writes become visible to the tensor cores (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Byte offset of 16-byte chunk c (K-bytes 16c..16c+15) of row r in a 128-byte-swizzled K-major tile.
__host__ __device__ __forceinline__ int sw128_chunk(int r, int c) {
  return (r >> 3) * 1024 + (r & 7) * 128 + (((c ^ r) & 7) << 4);
}

// ---- activation packing -------------------------------------------------------------------------
// One warp per (token, super-block): Q8_K-quantize 256 values (bit-exact with
// edgexpu_gguf_quantize_q8_k) or take them from a Q8_K row, scatter the int8 values into the two
// swizzled K-half tiles, and store d and the eight 32-element sums S_j = bsum_2j + bsum_2j+1 as
// int16 pairs (|S_j| <= 32 * 127).  Rows past m are written as zeros.
template <bool FROM_F32, int BN>
__global__ void __launch_bounds__(256) tc_pack_kernel(const float* __restrict__ x, const uint8_t* __restrict__ xq,
                                                      int m, int K, uint8_t* __restrict__ bt,
                                                      uint8_t* __restrict__ aux) {
  const int nb = K / QK_K;
  const int lane = threadIdx.x & 31;
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int n_tt = (m + BN - 1) / BN;
  if (gw >= (long long)n_tt * BN * nb) return;
  const int t = (int)(gw / nb), sb = (int)(gw % nb);
  const int tt = t / BN, r = t % BN;
  uint32_t w0 = 0, w1 = 0;
  float d = 0.0f;
  int s8 = 0;  // this lane's share of its 32-element sum
  if (t < m) {
    if constexpr (FROM_F32) {
      const float4* src = reinterpret_cast<const float4*>(x + (size_t)t * K + (size_t)sb * QK_K + lane * 8);
      const float4 a = src[0], b = src[1];
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      int q[8], gs;
      d = warp_q8_k(v, q, &gs);
      w0 = pack4_i8(q[0], q[1], q[2], q[3]);
      w1 = pack4_i8(q[4], q[5], q[6], q[7]);
#pragma unroll
      for (int i = 0; i < 8; ++i) s8 += q[i];
    } else {
      const uint8_t* blk = xq + ((size_t)t * nb + sb) * Q8_K_BYTES;
      const uint32_t* qw = reinterpret_cast<const uint32_t*>(blk + 4 + lane * 8);
      w0 = qw[0];
      w1 = qw[1];
      d = *reinterpret_cast<const float*>(blk);
      // the block's own int16 bsums, as the reference's summ reads them (gguf_dot_q8.c:745-750)
      if ((lane & 3) == 0) {
        const int16_t* bs = reinterpret_cast<const int16_t*>(blk + 260);
        s8 = (int)bs[lane >> 1] + (int)bs[(lane >> 1) + 1];
      }
    }
  }
  const int kh = lane >> 4, kb = (lane & 15) * 8;
  uint8_t* tile = bt + (((size_t)tt * nb + sb) * 2 + kh) * Cfg<BN>::B_TILE;
  *reinterpret_cast<uint2*>(tile + sw128_chunk(r, kb >> 4) + (kb & 15)) = make_uint2(w0, w1);
  // 32-element sums: lanes 4j..4j+3 hold sub-block j
  int s32 = s8 + __shfl_xor_sync(0xFFFFFFFFu, s8, 1);
  s32 += __shfl_xor_sync(0xFFFFFFFFu, s32, 2);
  // sums of a token: words [S0|S1][S2|S3][S4|S5][S6|S7], S_2w in the low half
  uint32_t dig[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t v = static_cast<uint32_t>(__shfl_sync(0xFFFFFFFFu, s32, 4 * j)) & 0xFFFFu;
    dig[j >> 1] |= v << (16 * (j & 1));
  }
  if (lane == 0) {
    uint8_t* xa = aux + ((size_t)tt * nb + sb) * Cfg<BN>::AUX_BYTES;
    reinterpret_cast<float*>(xa)[r] = d;
    *reinterpret_cast<uint4*>(xa + Cfg<BN>::AUX_DX + r * 16) = make_uint4(dig[0], dig[1], dig[2], dig[3]);
  }
}

// ---- the GEMM ---------------------------------------------------------------------------------------

// v = q4 * sc split into low bytes (v mod 256, as int8) and high parts ((v + 128) >> 8) for the
// four nibbles held in the low nibble of each byte of x.  Packed 16-bit lanes keep the
// products apart (945 + 128 < 65536).
__device__ __forceinline__ void expand4(uint32_t x, uint32_t sc, uint32_t& lo, uint32_t& hi) {
  const uint32_t a0 = __byte_perm(x, 0u, 0x4140);
  const uint32_t a1 = __byte_perm(x, 0u, 0x4342);
  const uint32_t v0 = a0 * sc + 0x00800080u;
  const uint32_t v1 = a1 * sc + 0x00800080u;
  hi = __byte_perm(v0, v1, 0x7531);
  lo = __byte_perm(v0, v1, 0x6420) ^ 0x80808080u;
}

// Bounded busy wait without the suspend hint, for the single-thread MMA issuer whose handoffs
// are on the critical path.
__device__ __forceinline__ bool spin_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
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

// Bounded wait whose outcome is the same for every lane of the warp (the tcgen05 ld/st that
// follow are warp-collective); returns converged.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const bool ok = wait_or_abort(bar, parity, abort_flag);
  return __all_sync(0xFFFFFFFFu, ok);
}

__device__ __forceinline__ void raise_abort(volatile int* abort_flag, uint32_t* status, uint32_t bit) {
  *abort_flag = 1;
  atomicOr(status, bit);
}

// PARTIALS: write the exact (sumi, summ) per block instead of the fp32 outputs (test hook).
template <bool PARTIALS, int BN>
__global__ void __launch_bounds__(Cfg<BN>::THREADS, 1)
    gemm_q4k_tc_kernel(const __grid_constant__ CUtensorMap wmap, const TcKernelArgs a) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ast = smem + C::A_OFF;
  uint8_t* bst = smem + C::B_OFF;
  uint8_t* rst = smem + C::R_OFF;
  uint8_t* xst = smem + C::X_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* a_full = bars;                // A tiles of a stage written (4 converter warps)
  uint64_t* b_full = a_full + N_STAGES;   // B tile of a stage landed (producer, tx bytes)
  uint64_t* empty = b_full + N_STAGES;    // the MMAs of a stage completed
  uint64_t* r_full = empty + N_STAGES;
  uint64_t* r_empty = r_full + NR_STAGES;
  uint64_t* x_full = r_empty + NR_STAGES;
  uint64_t* x_empty = x_full + NX_STAGES;
  uint64_t* acc_full = x_empty + NX_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* fin = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < N_STAGES; ++i) {
      mbar_init(&a_full[i], N_CONV_WARPS);
      mbar_init(&b_full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < NR_STAGES; ++i) {
      mbar_init(&r_full[i], 1);
      mbar_init(&r_empty[i], N_CONV_WARPS);
    }
    for (int i = 0; i < NX_STAGES; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], C::N_EPI_WARPS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], C::N_EPI_WARPS);
    }
    mbar_init(fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == WARP_MMA) {  // warp 1 has not diverged: the warp-collective allocation is converged
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int nb = a.nb, n_tt = a.n_tt;
  const long long n_tiles = (long long)a.n_rt * n_tt * (BN == 128 ? 1 : a.n_ks);

  if (warp == WARP_PROD) {
    if (lane == 0) {
      const uint64_t pol = l2_evict_last_policy();
      uint32_t s = 0, ph = 0, rs = 0, rph = 0, xs = 0, xph = 0;
      long long b_issued = 0, r_issued = 0, x_issued = 0;
      bool ok = true;
      for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        int rt, tt, ks, sb0, sb1;
        tc_item<BN>(a, tile, rt, tt, ks, sb0, sb1);
        for (int sb = sb0; ok && sb < sb1; ++sb) {
          if (!wait_or_abort(&r_empty[rs], rph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&r_full[rs], RAW_BYTES);
          tma_load_2d(rst + rs * RAW_BYTES, &wmap, sb * Q4_K_BYTES, rt * TC_BM, &r_full[rs]);
          ++r_issued;
          if (++rs == NR_STAGES) {
            rs = 0;
            rph ^= 1u;
          }
          if (!wait_or_abort(&x_empty[xs], xph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&x_full[xs], C::AUX_BYTES);
          bulk_g2s(xst + xs * C::AUX_BYTES, a.aux + ((size_t)tt * nb + sb) * C::AUX_BYTES, C::AUX_BYTES, &x_full[xs], pol);
          ++x_issued;
          if (++xs == NX_STAGES) {
            xs = 0;
            xph ^= 1u;
          }
          for (int kh = 0; kh < 2; ++kh) {
            if (!wait_or_abort(&empty[s], ph ^ 1u, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&b_full[s], C::B_TILE);
            bulk_g2s(bst + s * C::B_TILE, a.bt + (((size_t)tt * nb + sb) * 2 + kh) * C::B_TILE, C::B_TILE, &b_full[s], pol);
            ++b_issued;
            if (++s == N_STAGES) {
              s = 0;
              ph ^= 1u;
            }
          }
        }
      }
      if (!ok) raise_abort(abort_flag, a.status, ST_TIMEOUT_EMPTY);
      // No copy may still be landing in shared memory when the CTA exits.
      bool drained = true;
      for (long long n = b_issued - N_STAGES; n < b_issued; ++n)
        if (n >= 0 && !mbar_wait(&b_full[n % N_STAGES], (uint32_t)((n / N_STAGES) & 1))) drained = false;
      for (long long n = r_issued - NR_STAGES; n < r_issued; ++n)
        if (n >= 0 && !mbar_wait(&r_full[n % NR_STAGES], (uint32_t)((n / NR_STAGES) & 1))) drained = false;
      for (long long n = x_issued - NX_STAGES; n < x_issued; ++n)
        if (n >= 0 && !mbar_wait(&x_full[n % NX_STAGES], (uint32_t)((n / NX_STAGES) & 1))) drained = false;
      if (!drained) atomicOr(a.status, ST_TIMEOUT_DRAIN);
    }
  } else if (warp == WARP_MMA) {
    if (lane == 0) {
      uint32_t s = 0, ph = 0, accb = 0;
      bool ok = true;
      for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        int rt, tt, ks, sb0, sb1;
        tc_item<BN>(a, tile, rt, tt, ks, sb0, sb1);
        for (int sb = sb0; ok && sb < sb1; ++sb) {
          const uint32_t ab = accb & 1u;
          if (!spin_wait(&acc_empty[ab], (accb >> 1) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t d_l = tmem + ab * C::ACC_COLS, d_h = d_l + BN;
          for (int kh = 0; kh < 2; ++kh) {
            if (!spin_wait(&b_full[s], ph, abort_flag) || !spin_wait(&a_full[s], ph, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t al = sw128_desc(smem_u32(ast + s * 2 * A_TILE));
            const uint64_t ah = sw128_desc(smem_u32(ast + s * 2 * A_TILE + A_TILE));
            const uint64_t bd = sw128_desc(smem_u32(bst + s * C::B_TILE));
#pragma unroll
            for (int ks = 0; ks < KH_BYTES / 32; ++ks) {
              const uint64_t k = (uint64_t)((ks * 32) >> 4);
              mma_i8_ss(d_l, al + k, bd + k, C::IDESC);
              mma_i8_ss(d_h, ah + k, bd + k, C::IDESC);
            }
            tc_commit(&empty[s]);
            if (++s == N_STAGES) {
              s = 0;
              ph ^= 1u;
            }
          }
          if (!ok) break;
          tc_commit(&acc_full[ab]);
          ++accb;
        }
      }
      if (!ok) raise_abort(abort_flag, a.status, ST_TIMEOUT_FULL);
      // Everything issued above completes before tensor memory is released.
      tc_commit(fin);
      if (!mbar_wait(fin, 0)) atomicOr(a.status, ST_TIMEOUT_DRAIN);
    }
  } else if (warp < WARP_EPI0) {
    // Converters: thread = one weight row of the tile; per stage (K-half) 64 nibble bytes ->
    // 128 bytes of L and 128 bytes of H in the swizzled A tiles.
    const int r = 32 * (warp - WARP_CONV0) + lane;
    uint32_t s = 0, ph = 0, rs = 0, rph = 0;
    bool ok = true;
    for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
      int rt, tt, ks, sb0, sb1;
      tc_item<BN>(a, tile, rt, tt, ks, sb0, sb1);
      for (int sb = sb0; ok && sb < sb1; ++sb) {
        if (!warp_wait(&r_full[rs], rph, abort_flag)) {
          ok = false;
          break;
        }
        const uint8_t* raw = rst + rs * RAW_BYTES + r * Q4_K_BYTES;
        const uint4 hdr = *reinterpret_cast<const uint4*>(raw);
        for (int kh = 0; kh < 2; ++kh) {
          uint32_t sc4, mn4;
          q4k_scales_half(hdr.y, hdr.z, hdr.w, kh, sc4, mn4);
          const uint4* qp = reinterpret_cast<const uint4*>(raw + 16 + 64 * kh);
          if (!warp_wait(&empty[s], ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* al = ast + s * 2 * A_TILE;
          uint8_t* ah = al + A_TILE;
#pragma unroll
          for (int g = 0; g < 2; ++g) {  // nibble group: low nibbles = sub-block 2g, high = 2g + 1
            const uint4 n0 = qp[2 * g], n1 = qp[2 * g + 1];
            const uint32_t nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
            const uint32_t sc_lo = (sc4 >> (16 * g)) & 0xFFu, sc_hi = (sc4 >> (16 * g + 8)) & 0xFFu;
#pragma unroll
            for (int c = 0; c < 4; ++c) {  // K-bytes 64g + 16c .. +15: low nibbles (c < 2), then high
              uint32_t L[4], H[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint32_t w = nw[4 * (c & 1) + k];
                expand4(c < 2 ? (w & 0x0F0F0F0Fu) : ((w >> 4) & 0x0F0F0F0Fu), c < 2 ? sc_lo : sc_hi, L[k], H[k]);
              }
              *reinterpret_cast<uint4*>(al + sw128_chunk(r, 4 * g + c)) = make_uint4(L[0], L[1], L[2], L[3]);
              *reinterpret_cast<uint4*>(ah + sw128_chunk(r, 4 * g + c)) = make_uint4(H[0], H[1], H[2], H[3]);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[s]);
          if (++s == N_STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&r_empty[rs]);
        if (++rs == NR_STAGES) {
          rs = 0;
          rph ^= 1u;
        }
      }
    }
    if (!ok && lane == 0) raise_abort(abort_flag, a.status, ST_TIMEOUT_FULL);
  } else {
    // Epilogue: quadrant q (rows 32q + lane), token half j (tokens 64j..64j+63 of the tile).
    const int q = warp & 3, j = (warp - WARP_EPI0) >> 2;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(C::EPI_TOK * j);
    uint32_t bias8[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) bias8[k] = ACC_BIAS;
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int p = 0; p < 2; ++p)
#pragma unroll
        for (int h = 0; h < C::EPI_TOK / 8; ++h) tmem_st8(lane_base + b * C::ACC_COLS + p * BN + 8 * h, bias8);
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&acc_empty[0]);
      mbar_arrive(&acc_empty[1]);
    }
    uint32_t accb = 0, xs = 0, xph = 0;
    bool ok = true;
    for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
      int rt, tt, ks, sb0, sb1;
      tc_item<BN>(a, tile, rt, tt, ks, sb0, sb1);
      const int n = rt * TC_BM + 32 * q + lane;
      const bool valid = n < a.n_rows;
      const uint8_t* rowp = a.w + (size_t)(valid ? n : 0) * a.row_bytes;
      const int t0 = tt * BN + C::EPI_TOK * j;
      float acc[C::EPI_TOK];
#pragma unroll
      for (int e = 0; e < C::EPI_TOK; ++e) acc[e] = 0.0f;
      uint4 hdr = __ldg(reinterpret_cast<const uint4*>(rowp + sb0 * Q4_K_BYTES));
      for (int sb = sb0; sb < sb1; ++sb) {
        const float dw = fp16_bits_to_float(hdr.x), dmw = fp16_bits_to_float(hdr.x >> 16);
        uint32_t sc4, m03, m47;
        q4k_scales_half(hdr.y, hdr.z, hdr.w, 0, sc4, m03);
        q4k_scales_half(hdr.y, hdr.z, hdr.w, 1, sc4, m47);
        if (sb + 1 < sb1) hdr = __ldg(reinterpret_cast<const uint4*>(rowp + (sb + 1) * Q4_K_BYTES));
        const uint32_t ab = accb & 1u;
        if (!warp_wait(&x_full[xs], xph, abort_flag) || !warp_wait(&acc_full[ab], (accb >> 1) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float* dxs = reinterpret_cast<const float*>(xst + xs * C::AUX_BYTES) + C::EPI_TOK * j;
        const uint4* dgs = reinterpret_cast<const uint4*>(xst + xs * C::AUX_BYTES + C::AUX_DX) + C::EPI_TOK * j;
        const uint32_t col = lane_base + ab * C::ACC_COLS;
        // One group = EG tokens.  The loads of group h + 1 are issued right after the wait for
        // group h, so their latency overlaps the arithmetic of group h.
        uint32_t Lb[2][EG], Hb[2][EG];
        tmem_ld8(col, Lb[0]);
        tmem_ld8(col + BN, Hb[0]);
#pragma unroll
        for (int h = 0; h < C::EPI_TOK / EG; ++h) {
          const int c = h & 1;
          __syncwarp();  // tcgen05.ld/st are warp-collective; the partials stores below diverge
          tmem_wait_ld();
          tmem_st8(col + EG * h, bias8);
          tmem_st8(col + BN + EG * h, bias8);
          if (h + 1 < C::EPI_TOK / EG) {
            tmem_ld8(col + EG * (h + 1), Lb[c ^ 1]);
            tmem_ld8(col + BN + EG * (h + 1), Hb[c ^ 1]);
          }
#pragma unroll
          for (int e = 0; e < EG; ++e) {
            const uint32_t Le = Lb[c][e], He = Hb[c][e];
            const uint4 dg = dgs[EG * h + e];  // S0|S1, S2|S3, S4|S5, S6|S7
            // summ = sum_j m_j * S_j (m_j <= 63 reads the same as a signed byte), carried with the float bias
            int sm = __dp2a_lo(static_cast<int>(dg.x), static_cast<int>(m03), static_cast<int>(ACC_BIAS));
            sm = __dp2a_hi(static_cast<int>(dg.y), static_cast<int>(m03), sm);
            sm = __dp2a_lo(static_cast<int>(dg.z), static_cast<int>(m47), sm);
            sm = __dp2a_hi(static_cast<int>(dg.w), static_cast<int>(m47), sm);
            if constexpr (PARTIALS) {
              const int t = t0 + EG * h + e;
              if (valid && t < a.m) {
                const int sumi = (int)(Le - ACC_BIAS) + (int)((He - ACC_BIAS) << 8);
                *reinterpret_cast<int2*>(a.partials + (((size_t)t * a.n_rows + n) * nb + sb) * 2) =
                    make_int2(sumi, sm - (int)ACC_BIAS);
              }
            } else {
              const float fl = __uint_as_float(Le) - ACC_BIAS_F;
              const float fh = __uint_as_float(He) - ACC_BIAS_F;
              const float fm = __int_as_float(sm) - ACC_BIAS_F;
              const float fs = fmaf(256.0f, fh, fl);
              const float tv = fmaf(-dmw, fm, dw * fs);
              acc[EG * h + e] = fmaf(dxs[EG * h + e], tv, acc[EG * h + e]);
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&acc_empty[ab]);
          mbar_arrive(&x_empty[xs]);
        }
        ++accb;
        if (++xs == NX_STAGES) {
          xs = 0;
          xph ^= 1u;
        }
      }
      if (!ok) break;
      if (!PARTIALS && valid) {
        if (BN == 128 || a.n_ks == 1) {
          const float bv = a.bias != nullptr ? a.bias[n] : 0.0f;
#pragma unroll
          for (int e = 0; e < C::EPI_TOK; ++e) {
            const int t = t0 + e;
            if (t < a.m) a.out[(size_t)t * a.out_stride + n] = acc[e] + bv;
          }
        } else if constexpr (BN == 16) {  // this K range's sum, for tc_split_reduce_kernel
#pragma unroll
          for (int e = 0; e < C::EPI_TOK; ++e) {
            const int t = t0 + e;
            if (t < a.m) a.part[((size_t)ks * a.m + t) * a.n_rows + n] = acc[e];
          }
        }
      }
    }
    if (!ok && lane == 0) raise_abort(abort_flag, a.status, ST_TIMEOUT_FULL);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == WARP_MMA) {
    __syncwarp();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// out[t][n] = bias[n] + sum over the K ranges of part[ks][t][n], in K-range order (deterministic).
__global__ void tc_split_reduce_kernel(const float* __restrict__ part, int n_ks, int m, int n_rows,
                                       const float* __restrict__ bias, float* __restrict__ out, long long out_stride) {
  const long long total = (long long)m * n_rows;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / n_rows), n = (int)(i - (long long)t * n_rows);
    float acc = part[i];
    for (int k = 1; k < n_ks; ++k) acc += part[(size_t)k * total + i];
    out[(size_t)t * out_stride + n] = acc + (bias != nullptr ? bias[n] : 0.0f);
  }
}

// ---- host side --------------------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace

// Token tile of a batch of m tokens: 16 below the prefill threshold, else 128.
static int tc_bn(int m) { return m < TC_MIN_M ? 16 : 128; }

size_t tc_act_bytes(int m, int K) {
  const int bn = tc_bn(m);
  const size_t n_tt = (size_t)(m + bn - 1) / bn, nb = (size_t)K / QK_K;
  return bn == 16 ? n_tt * nb * (2 * Cfg<16>::B_TILE + Cfg<16>::AUX_BYTES)
                  : n_tt * nb * (2 * Cfg<128>::B_TILE + Cfg<128>::AUX_BYTES);
}

// K split of a launch: with 16-token tiles the row tiles alone leave most SMs idle, so the
// super-blocks of each row tile are split (at least 2 per range) until there are about two work
// items per SM.  128-token tiles are not split.
static void tc_split(int m, int n_rows, int K, const DeviceInfo& dev, int& n_ks, int& sb_per) {
  const int nb = K / QK_K, bn = tc_bn(m);
  const long long base = (long long)((n_rows + TC_BM - 1) / TC_BM) * ((m + bn - 1) / bn);
  n_ks = 1;
  if (bn == 16 && base < 2LL * dev.sm_count) {
    long long want = (2LL * dev.sm_count + base - 1) / base;
    if (want > nb / 2) want = nb / 2;
    n_ks = want < 1 ? 1 : (int)want;
  }
  sb_per = (nb + n_ks - 1) / n_ks;
  n_ks = (nb + sb_per - 1) / sb_per;
}

size_t tc_split_bytes(int m, int n_rows, int K, const DeviceInfo& dev) {
  int n_ks, sb_per;
  tc_split(m, n_rows, K, dev, n_ks, sb_per);
  return n_ks > 1 ? (size_t)n_ks * m * n_rows * sizeof(float) : 0;
}

template <int BN>
static cudaError_t launch_pack_bn(bool from_f32, const float* x, const uint8_t* xq, int m, int K, uint8_t* act,
                                  cudaStream_t st) {
  const int n_tt = (m + BN - 1) / BN, nb = K / QK_K;
  uint8_t* bt = act;
  uint8_t* aux = act + (size_t)n_tt * nb * 2 * Cfg<BN>::B_TILE;
  const long long warps = (long long)n_tt * BN * nb;
  const unsigned grid = (unsigned)((warps + 7) / 8);
  if (from_f32)
    tc_pack_kernel<true, BN><<<grid, 256, 0, st>>>(x, nullptr, m, K, bt, aux);
  else
    tc_pack_kernel<false, BN><<<grid, 256, 0, st>>>(nullptr, xq, m, K, bt, aux);
  return cudaGetLastError();
}

static cudaError_t launch_pack(bool from_f32, const float* x, const uint8_t* xq, int m, int K, uint8_t* act,
                               cudaStream_t st) {
  if (m <= 0 || K <= 0 || K % QK_K != 0) return cudaErrorInvalidValue;
  return tc_bn(m) == 16 ? launch_pack_bn<16>(from_f32, x, xq, m, K, act, st)
                        : launch_pack_bn<128>(from_f32, x, xq, m, K, act, st);
}

cudaError_t launch_tc_pack_f32(const float* x, int m, int K, uint8_t* act, cudaStream_t st) {
  return launch_pack(true, x, nullptr, m, K, act, st);
}

cudaError_t launch_tc_pack_q8k(const uint8_t* xq, int m, int K, uint8_t* act, cudaStream_t st) {
  return launch_pack(false, nullptr, xq, m, K, act, st);
}

template <int BN>
static cudaError_t launch_gemm_bn(const CUtensorMap& map, const TcKernelArgs& k, int grid, cudaStream_t st) {
  static bool attr_set = false;  // per instantiation; the host API serialises its callers
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(gemm_q4k_tc_kernel<false, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg<BN>::ALLOC);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_q4k_tc_kernel<true, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Cfg<BN>::ALLOC);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  if (k.partials != nullptr)
    gemm_q4k_tc_kernel<true, BN><<<grid, Cfg<BN>::THREADS, Cfg<BN>::ALLOC, st>>>(map, k);
  else
    gemm_q4k_tc_kernel<false, BN><<<grid, Cfg<BN>::THREADS, Cfg<BN>::ALLOC, st>>>(map, k);
  return cudaGetLastError();
}

cudaError_t launch_tc_gemm(const TcGemmArgs& g, const DeviceInfo& dev, cudaStream_t st) {
  if (g.n_rows <= 0 || g.m <= 0 || g.K <= 0 || g.K % QK_K != 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(g.w) & 15u) != 0) return cudaErrorMisalignedAddress;
  EncodeTiledFn enc = encode_tiled();
  if (enc == nullptr) return cudaErrorNotSupported;
  const int nb = g.K / QK_K, row_bytes = nb * Q4_K_BYTES, bn = tc_bn(g.m);
  // The weight as a 2-D byte array [n_rows][row_bytes]; one box = one super-block of 128 rows.
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)g.n_rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)Q4_K_BYTES, (cuuint32_t)TC_BM};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(g.w), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;

  TcKernelArgs k;
  k.n_rows = g.n_rows;
  k.row_bytes = row_bytes;
  k.nb = nb;
  k.m = g.m;
  k.n_tt = (g.m + bn - 1) / bn;
  k.n_rt = (g.n_rows + TC_BM - 1) / TC_BM;
  tc_split(g.m, g.n_rows, g.K, dev, k.n_ks, k.sb_per);
  // (the exact partials are written per super-block, so a split needs no partial sums there)
  if (g.partials == nullptr && k.n_ks > 1 && g.part == nullptr) return cudaErrorInvalidValue;
  k.w = g.w;
  k.bt = g.act;
  k.aux = g.act + (size_t)k.n_tt * nb * 2 * (bn == 16 ? Cfg<16>::B_TILE : Cfg<128>::B_TILE);
  k.bias = g.bias;
  k.out = g.out;
  k.out_stride = g.out_stride;
  k.part = g.part;
  k.partials = g.partials;
  k.status = g.status;

  const long long tiles = (long long)k.n_tt * k.n_rt * k.n_ks;
  const int grid = (int)(tiles < dev.sm_count ? tiles : dev.sm_count);
  cudaError_t e = bn == 16 ? launch_gemm_bn<16>(map, k, grid, st) : launch_gemm_bn<128>(map, k, grid, st);
  if (e != cudaSuccess || g.partials != nullptr || k.n_ks == 1) return e;
  const long long total = (long long)g.m * g.n_rows;
  const int rgrid = (int)((total + 255) / 256 < 4LL * dev.sm_count ? (total + 255) / 256 : 4LL * dev.sm_count);
  tc_split_reduce_kernel<<<rgrid, 256, 0, st>>>(g.part, k.n_ks, g.m, g.n_rows, g.bias, g.out, g.out_stride);
  return cudaGetLastError();
}

}  // namespace ex
