// gemm_tc.cu -- Q4_K weight x Q8_K activation GEMM on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, operand A and the accumulators in tensor memory) for prefill-sized
// batches: the batched form of dot_q4_k_q8_k (src/gguf_dot_q8.c:603-762) that
// edgexpu_cpu_linear_quant_batch (src/cpu_kernel.c:545-644) runs per row and token.
//
// Arithmetic.  Per super-block the reference computes, in int32,
//   sumi = sum_j sc_j * sum_{l<32} q4 * q8      summ = sum_j m_j * (bsum_2j + bsum_2j+1)
// and then acc += d_x*d_w*sumi - d_x*dmin_w*summ (gguf_dot_q8.c:711-759).  The folded weight
// v = sc_j * q4 lies in [0, 945] (10 bits), so it is split into v = 256*h + l with l in
// [-128, 127] and h in [0, 4], and three int8 contractions over the super-block run on the
// tensor cores into three int32 accumulators:
//   L = sum l*q8,   H = sum h*q8,   M = sum m_j*q8      =>  sumi = L + 256*H,  summ = M.
// All three are exact integer sums, so (sumi, summ) equal the reference's int32 values.
//
// Float conversion without I2F.  Every accumulator starts at the bit pattern 0x4B400000
// (1.5 * 2^23 as a float) instead of 0; the MMA adds exact int32 products to it, and since
// |L| <= 128*127*256 < 2^22 (likewise H, M), the float value of the bits is 1.5*2^23 + L
// exactly.  The epilogue therefore converts with one FADD per accumulator.
//
// Tile: 128 weight rows (tensor-memory lanes, MMA M) x 64 tokens (MMA N); K advances one
// Q4_K nibble group (64 elements) per A chunk.  Tensor-memory columns (of 512):
//   [0,192)   accumulator buffer 0: L [0,64) H [64,128) M [128,192)
//   [192,384) accumulator buffer 1
//   [384,432) A chunk buffer 0: L [0,16) H [16,32) M [32,48)  (4 int8 per column, K-major)
//   [448,496) A chunk buffer 1
// Two accumulator buffers let the epilogue drain super-block s while the MMAs of s+1 run.
//
// Warp roles (18 warps):
//   0      producer: 2-D TMA of the raw Q4_K super-block of 128 rows (tensor map, zero-filled
//          past the last row) and 1-D bulk copies of pre-swizzled activation tiles
//   1      tensor-memory allocation and the single-thread MMA issuer
//   2..9   converters: expand nibbles and 6-bit scales into the L/H/M int8 operand and store
//          it to tensor memory (2 warps per 32-lane quadrant, one per A buffer)
//   10..17 epilogue: drain accumulators, scale, accumulate in fp32 registers, store
// Every wait is bounded; a timeout sets a status bit, raises the CTA abort flag and all roles
// fall through to teardown (bulk copies drained, MMAs committed, tensor memory freed).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "common.cuh"
#include "launch.h"
#include "quant.cuh"

namespace ex {
namespace {

constexpr int TC_BM = 128;
constexpr int TC_BN = 64;
constexpr int B_TILE_BYTES = TC_BN * 128;   // 64 tokens x 128 K-bytes, 128-byte swizzle, K-major
constexpr int RAW_BYTES = TC_BM * Q4_K_BYTES;  // one super-block of 128 rows: 18432
constexpr int NB_STAGES = 8;
constexpr int NR_STAGES = 4;
constexpr int N_CONV_WARPS = 8;
constexpr int N_EPI_WARPS = 8;
constexpr int WARP_PROD = 0;
constexpr int WARP_MMA = 1;
constexpr int WARP_CONV0 = 2;
constexpr int WARP_EPI0 = WARP_CONV0 + N_CONV_WARPS;
constexpr int TC_THREADS = 32 * (WARP_EPI0 + N_EPI_WARPS);

constexpr uint32_t ACC_COLS = 3 * TC_BN;
constexpr uint32_t A_COL0 = 384;
constexpr uint32_t A_BUF_STRIDE = 64;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t ACC_BIAS = 0x4B400000u;
constexpr float ACC_BIAS_F = 12582912.0f;

// kind::i8 instruction descriptor: D int32 (c_format 2 at bit 4), A and B signed int8
// (formats 1 at bits 7 and 10), both K-major, N>>3 at bit 17, M>>4 at bit 24.
constexpr uint32_t IDESC_I8 = (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(TC_BN >> 3) << 17) |
                              (uint32_t(TC_BM >> 4) << 24);

struct SmemLayout {
  static constexpr int B_OFF = 0;
  static constexpr int R_OFF = B_OFF + NB_STAGES * B_TILE_BYTES;
  static constexpr int BAR_OFF = R_OFF + NR_STAGES * RAW_BYTES;
  static constexpr int N_BARS = 2 * NB_STAGES + 2 * NR_STAGES + 8 + 1;
  static constexpr int MISC_OFF = BAR_OFF + 8 * N_BARS;
  static constexpr int BYTES = MISC_OFF + 16;
  static constexpr int ALLOC = BYTES + 1024;  // base rounded up to 1024 for the swizzled tiles
};

struct TcKernelArgs {
  int n_rows, row_bytes, nb, m, n_tt, n_rt;
  const uint8_t* w;       // Q4_K rows (for d/dmin in the epilogue)
  const uint8_t* bt;      // activation tiles [n_tt][nb][2][8 KB]
  const float* dx;        // [n_tt][nb][64]
  const float* bias;
  float* out;
  long long out_stride;
  int32_t* partials;      // non-null: write (sumi, summ) per (token, row, super-block) instead of out
  uint32_t* status;
};

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

// D[tmem] (+)= A[tmem] x B[smem descriptor]
__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %3, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %4, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(acc), "r"(IDESC_I8)
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
__device__ __forceinline__ void tmem_st16(uint32_t addr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(addr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
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

// Byte of the packed activation tile holding K-byte kb (0..127) of token row r (0..63).
__host__ __device__ __forceinline__ int sw128_offset(int r, int kb) {
  return (r >> 3) * 1024 + (r & 7) * 128 + ((((kb >> 4) ^ (r & 7)) & 7) << 4) + (kb & 15);
}

// ---- activation packing -------------------------------------------------------------------------
// One warp per (token, super-block): Q8_K-quantize 256 values (bit-exact with
// edgexpu_gguf_quantize_q8_k) or copy them from a Q8_K row, and scatter the int8 values into
// the two swizzled K-half tiles; lane 0 stores d.  Rows past m are written as zeros.
template <bool FROM_F32>
__global__ void __launch_bounds__(256) tc_pack_kernel(const float* __restrict__ x, const uint8_t* __restrict__ xq,
                                                      int m, int K, uint8_t* __restrict__ bt, float* __restrict__ dx) {
  const int nb = K / QK_K;
  const int lane = threadIdx.x & 31;
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int n_tt = (m + TC_BN - 1) / TC_BN;
  if (gw >= (long long)n_tt * TC_BN * nb) return;
  const int t = (int)(gw / nb), sb = (int)(gw % nb);
  const int tt = t / TC_BN, r = t % TC_BN;
  uint32_t w0 = 0, w1 = 0;
  float d = 0.0f;
  if (t < m) {
    if constexpr (FROM_F32) {
      const float4* src = reinterpret_cast<const float4*>(x + (size_t)t * K + (size_t)sb * QK_K + lane * 8);
      const float4 a = src[0], b = src[1];
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      int q[8], gs;
      d = warp_q8_k(v, q, &gs);
      w0 = pack4_i8(q[0], q[1], q[2], q[3]);
      w1 = pack4_i8(q[4], q[5], q[6], q[7]);
    } else {
      const uint8_t* blk = xq + ((size_t)t * nb + sb) * Q8_K_BYTES;
      const uint32_t* qw = reinterpret_cast<const uint32_t*>(blk + 4 + lane * 8);
      w0 = qw[0];
      w1 = qw[1];
      d = *reinterpret_cast<const float*>(blk);
    }
  }
  const int kh = lane >> 4, kb = (lane & 15) * 8;
  uint8_t* tile = bt + (((size_t)tt * nb + sb) * 2 + kh) * B_TILE_BYTES;
  *reinterpret_cast<uint2*>(tile + sw128_offset(r, kb)) = make_uint2(w0, w1);
  if (lane == 0) dx[((size_t)tt * nb + sb) * TC_BN + r] = d;
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

__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_q4k_tc_kernel(const __grid_constant__ CUtensorMap wmap, const TcKernelArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bst = smem + SmemLayout::B_OFF;
  uint8_t* rst = smem + SmemLayout::R_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemLayout::BAR_OFF);
  uint64_t* b_full = bars;
  uint64_t* b_empty = b_full + NB_STAGES;
  uint64_t* r_full = b_empty + NB_STAGES;
  uint64_t* r_empty = r_full + NR_STAGES;
  uint64_t* a_full = r_empty + NR_STAGES;
  uint64_t* a_empty = a_full + 2;
  uint64_t* acc_full = a_empty + 2;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* fin = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SmemLayout::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + SmemLayout::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NB_STAGES; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < NR_STAGES; ++i) {
      mbar_init(&r_full[i], 1);
      mbar_init(&r_empty[i], N_CONV_WARPS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&a_full[i], 4);
      mbar_init(&a_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], N_EPI_WARPS);
    }
    mbar_init(fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int nb = a.nb, n_tt = a.n_tt;
  const long long n_tiles = (long long)a.n_rt * n_tt;

  if (warp == WARP_PROD) {
    if (lane == 0) {
      const uint64_t pol = l2_evict_last_policy();
      uint32_t bs = 0, bph = 0, rs = 0, rph = 0;
      long long b_issued = 0, r_issued = 0;
      bool ok = true;
      for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        const int rt = (int)(tile / n_tt), tt = (int)(tile % n_tt);
        const uint8_t* src = a.bt + (size_t)tt * nb * 2 * B_TILE_BYTES;
        for (int sb = 0; ok && sb < nb; ++sb) {
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
          for (int kh = 0; kh < 2; ++kh) {
            if (!wait_or_abort(&b_empty[bs], bph ^ 1u, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&b_full[bs], B_TILE_BYTES);
            bulk_g2s(bst + bs * B_TILE_BYTES, src + ((size_t)sb * 2 + kh) * B_TILE_BYTES, B_TILE_BYTES, &b_full[bs],
                     pol);
            ++b_issued;
            if (++bs == NB_STAGES) {
              bs = 0;
              bph ^= 1u;
            }
          }
        }
      }
      if (!ok) raise_abort(abort_flag, a.status, ST_TIMEOUT_EMPTY);
      // No copy may still be landing in shared memory when the CTA exits.
      bool drained = true;
      for (long long n = b_issued - NB_STAGES; n < b_issued; ++n)
        if (n >= 0 && !mbar_wait(&b_full[n % NB_STAGES], (uint32_t)((n / NB_STAGES) & 1))) drained = false;
      for (long long n = r_issued - NR_STAGES; n < r_issued; ++n)
        if (n >= 0 && !mbar_wait(&r_full[n % NR_STAGES], (uint32_t)((n / NR_STAGES) & 1))) drained = false;
      if (!drained) atomicOr(a.status, ST_TIMEOUT_DRAIN);
    }
  } else if (warp == WARP_MMA) {
    if (lane == 0) {
      uint32_t bs = 0, bph = 0, g = 0, accb = 0;
      bool ok = true;
      for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        for (int sb = 0; ok && sb < nb; ++sb) {
          const uint32_t ab = accb & 1u;
          if (!wait_or_abort(&acc_empty[ab], (accb >> 1) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_col = tmem + ab * ACC_COLS;
          for (int c = 0; c < 4; ++c) {
            if ((c & 1) == 0) {
              if (!wait_or_abort(&b_full[bs], bph, abort_flag)) {
                ok = false;
                break;
              }
            }
            const uint32_t ai = g & 1u;
            if (!wait_or_abort(&a_full[ai], (g >> 1) & 1u, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_col = tmem + A_COL0 + ai * A_BUF_STRIDE;
            const uint64_t bdesc = sw128_desc(smem_u32(bst + bs * B_TILE_BYTES));
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {
              const uint64_t bd = bdesc + (uint64_t)((((c & 1) * 2 + ks) * 32) >> 4);
#pragma unroll
              for (int p = 0; p < 3; ++p) mma_i8_ts(d_col + p * TC_BN, a_col + p * 16 + ks * 8, bd, 1u);
            }
            tc_commit(&a_empty[ai]);
            if (c & 1) {
              tc_commit(&b_empty[bs]);
              if (++bs == NB_STAGES) {
                bs = 0;
                bph ^= 1u;
              }
            }
            ++g;
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
    // Converters: quadrant q owns tensor-memory lanes (= tile rows) 32q..32q+31; set i fills
    // A buffer i, i.e. chunks c = i and i + 2 of every super-block.
    const int q = warp & 3, i = (warp - WARP_CONV0) >> 2;
    const int r = 32 * q + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + A_COL0 + (uint32_t)i * A_BUF_STRIDE;
    uint32_t rs = 0, rph = 0, uses = 0;
    bool ok = true;
    for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
      for (int sb = 0; ok && sb < nb; ++sb) {
        if (!warp_wait(&r_full[rs], rph, abort_flag)) {
          ok = false;
          break;
        }
        const uint8_t* raw = rst + rs * RAW_BYTES + r * Q4_K_BYTES;
        const uint4 hdr = *reinterpret_cast<const uint4*>(raw);
        for (int c = i; c < 4; c += 2) {
          const uint4 n0 = *reinterpret_cast<const uint4*>(raw + 16 + 32 * c);
          const uint4 n1 = *reinterpret_cast<const uint4*>(raw + 32 + 32 * c);
          uint32_t sc4, mn4;
          q4k_scales_half(hdr.y, hdr.z, hdr.w, c >> 1, sc4, mn4);
          const int sh = 16 * (c & 1);
          const uint32_t sc_lo = (sc4 >> sh) & 0xFFu, sc_hi = (sc4 >> (sh + 8)) & 0xFFu;
          const uint32_t m_lo = ((mn4 >> sh) & 0xFFu) * 0x01010101u, m_hi = ((mn4 >> (sh + 8)) & 0xFFu) * 0x01010101u;
          const uint32_t nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
          uint32_t L[16], H[16], M[16];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            expand4(nw[k] & 0x0F0F0F0Fu, sc_lo, L[k], H[k]);
            expand4((nw[k] >> 4) & 0x0F0F0F0Fu, sc_hi, L[8 + k], H[8 + k]);
            M[k] = m_lo;
            M[8 + k] = m_hi;
          }
          if (!warp_wait(&a_empty[i], (uses & 1u) ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          tmem_st16(lane_base + 0, L);
          tmem_st16(lane_base + 16, H);
          tmem_st16(lane_base + 32, M);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[i]);
          ++uses;
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
    // Epilogue: quadrant q (rows 32q + lane), token half j (tokens 32j..32j+31 of the tile).
    const int q = warp & 3, j = (warp - WARP_EPI0) >> 2;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(32 * j);
    {
      uint32_t bias8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) bias8[k] = ACC_BIAS;
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
          for (int h = 0; h < 4; ++h) tmem_st8(lane_base + b * ACC_COLS + p * TC_BN + 8 * h, bias8);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acc_empty[0]);
        mbar_arrive(&acc_empty[1]);
      }
    }
    uint32_t accb = 0;
    bool ok = true;
    for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
      const int rt = (int)(tile / n_tt), tt = (int)(tile % n_tt);
      const int n = rt * TC_BM + 32 * q + lane;
      const bool valid = n < a.n_rows;
      const uint8_t* rowp = a.w + (size_t)(valid ? n : 0) * a.row_bytes;
      const int t0 = tt * TC_BN + 32 * j;
      float acc[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) acc[e] = 0.0f;
      uint32_t ddm = __ldg(reinterpret_cast<const uint32_t*>(rowp));
      for (int sb = 0; sb < nb; ++sb) {
        const float dw = fp16_bits_to_float(ddm), dmw = fp16_bits_to_float(ddm >> 16);
        if (sb + 1 < nb) ddm = __ldg(reinterpret_cast<const uint32_t*>(rowp + (sb + 1) * Q4_K_BYTES));
        const float* dxp = a.dx + ((size_t)tt * nb + sb) * TC_BN + 32 * j;
        const uint32_t ab = accb & 1u;
        if (!warp_wait(&acc_full[ab], (accb >> 1) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t col = lane_base + ab * ACC_COLS;
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          uint32_t L[8], H[8], M[8];
          tmem_ld8(col + 8 * h, L);
          tmem_ld8(col + TC_BN + 8 * h, H);
          tmem_ld8(col + 2 * TC_BN + 8 * h, M);
          const float4 x0 = __ldg(reinterpret_cast<const float4*>(dxp + 8 * h));
          const float4 x1 = __ldg(reinterpret_cast<const float4*>(dxp + 8 * h + 4));
          const float dxv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
          tmem_wait_ld();
          {
            uint32_t bias8[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) bias8[k] = ACC_BIAS;
            tmem_st8(col + 8 * h, bias8);
            tmem_st8(col + TC_BN + 8 * h, bias8);
            tmem_st8(col + 2 * TC_BN + 8 * h, bias8);
          }
          if (a.partials != nullptr) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int t = t0 + 8 * h + e;
              if (valid && t < a.m) {
                const int sumi = (int)(L[e] - ACC_BIAS) + (int)((H[e] - ACC_BIAS) << 8);
                const int summ = (int)(M[e] - ACC_BIAS);
                *reinterpret_cast<int2*>(a.partials + (((size_t)t * a.n_rows + n) * nb + sb) * 2) =
                    make_int2(sumi, summ);
              }
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float fl = __uint_as_float(L[e]) - ACC_BIAS_F;
              const float fh = __uint_as_float(H[e]) - ACC_BIAS_F;
              const float fm = __uint_as_float(M[e]) - ACC_BIAS_F;
              const float fs = fmaf(256.0f, fh, fl);
              const float tv = fmaf(-dmw, fm, dw * fs);
              acc[8 * h + e] = fmaf(dxv[e], tv, acc[8 * h + e]);
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[ab]);
        ++accb;
      }
      if (!ok) break;
      if (a.partials == nullptr && valid) {
        const float bv = a.bias != nullptr ? a.bias[n] : 0.0f;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int t = t0 + e;
          if (t < a.m) a.out[(size_t)t * a.out_stride + n] = acc[e] + bv;
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
    tmem_dealloc(tmem, TMEM_COLS);
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

size_t tc_act_bytes(int m, int K) {
  const size_t n_tt = (size_t)(m + TC_BN - 1) / TC_BN, nb = (size_t)K / QK_K;
  return n_tt * nb * (2 * B_TILE_BYTES + TC_BN * sizeof(float));
}

static cudaError_t launch_pack(bool from_f32, const float* x, const uint8_t* xq, int m, int K, uint8_t* act,
                               cudaStream_t st) {
  if (m <= 0 || K <= 0 || K % QK_K != 0) return cudaErrorInvalidValue;
  const int n_tt = (m + TC_BN - 1) / TC_BN, nb = K / QK_K;
  uint8_t* bt = act;
  float* dx = reinterpret_cast<float*>(act + (size_t)n_tt * nb * 2 * B_TILE_BYTES);
  const long long warps = (long long)n_tt * TC_BN * nb;
  const unsigned grid = (unsigned)((warps + 7) / 8);
  if (from_f32)
    tc_pack_kernel<true><<<grid, 256, 0, st>>>(x, nullptr, m, K, bt, dx);
  else
    tc_pack_kernel<false><<<grid, 256, 0, st>>>(nullptr, xq, m, K, bt, dx);
  return cudaGetLastError();
}

cudaError_t launch_tc_pack_f32(const float* x, int m, int K, uint8_t* act, cudaStream_t st) {
  return launch_pack(true, x, nullptr, m, K, act, st);
}

cudaError_t launch_tc_pack_q8k(const uint8_t* xq, int m, int K, uint8_t* act, cudaStream_t st) {
  return launch_pack(false, nullptr, xq, m, K, act, st);
}

cudaError_t launch_tc_gemm(const TcGemmArgs& g, const DeviceInfo& dev, cudaStream_t st) {
  if (g.n_rows <= 0 || g.m <= 0 || g.K <= 0 || g.K % QK_K != 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(g.w) & 15u) != 0) return cudaErrorMisalignedAddress;
  EncodeTiledFn enc = encode_tiled();
  if (enc == nullptr) return cudaErrorNotSupported;
  const int nb = g.K / QK_K, row_bytes = nb * Q4_K_BYTES;
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
  k.n_tt = (g.m + TC_BN - 1) / TC_BN;
  k.n_rt = (g.n_rows + TC_BM - 1) / TC_BM;
  k.w = g.w;
  k.bt = g.act;
  k.dx = reinterpret_cast<const float*>(g.act + (size_t)k.n_tt * nb * 2 * B_TILE_BYTES);
  k.bias = g.bias;
  k.out = g.out;
  k.out_stride = g.out_stride;
  k.partials = g.partials;
  k.status = g.status;

  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(gemm_q4k_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SmemLayout::ALLOC);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const long long tiles = (long long)k.n_tt * k.n_rt;
  const int grid = (int)(tiles < dev.sm_count ? tiles : dev.sm_count);
  gemm_q4k_tc_kernel<<<grid, TC_THREADS, SmemLayout::ALLOC, st>>>(map, k);
  return cudaGetLastError();
}

}  // namespace ex
