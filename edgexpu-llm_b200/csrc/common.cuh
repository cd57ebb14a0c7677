// common.cuh -- block layouts and sm_100a device helpers shared by the edgexpu CUDA kernels.
//
// GGUF block layouts (the reference's src/gguf_dot_q8.c:18-26 and :90-110, src/gguf_quant.c:139-353):
//   Q8_0  34 B : fp16 d @0, int8 qs[32] @2
//   Q8_K  292 B: fp32 d @0, int8 qs[256] @4, int16 bsums[16] @260
//   Q4_K  144 B: fp16 d @0, fp16 dmin @2, 12 B packed 6-bit scales/mins @4, 128 B nibbles @16
//   Q4_0  18 B : fp16 d @0, 16 B nibbles @2 (element j low nibble, 16+j high; offset 8)
//   Q5_0  22 B : fp16 d @0, u32 fifth bits @2, 16 B nibbles @6 (offset 16)
//   Q5_K  176 B: fp16 d @0, fp16 dmin @2, 12 B scales/mins @4, qh[32] @16, ql[128] @48
//   Q6_K  210 B: ql[128] @0, qh[64] @128, int8 scales[16] @192, fp16 d @208 (offset 32)
// Weights stay in exactly this layout in HBM; nothing is repacked at upload.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace ex {

constexpr int QK8_0 = 32;
constexpr int QK_K = 256;
constexpr int Q8_0_BYTES = 34;
constexpr int Q8_K_BYTES = 292;
constexpr int Q4_K_BYTES = 144;
constexpr int Q4_0_BYTES = 18;   // fp16 d, 16 nibble bytes                         (gguf_dot_q8.c:23)
constexpr int Q5_0_BYTES = 22;   // fp16 d, 32 fifth bits, 16 nibble bytes          (gguf_dot_q8.c:22)
constexpr int Q5_K_BYTES = 176;  // fp16 d, fp16 dmin, 12 scale bytes, qh[32], ql[128] (gguf_dot_q8.c:25)
constexpr int Q6_K_BYTES = 210;  // ql[128], qh[64], int8 scales[16], fp16 d          (gguf_dot_q8.c:26)

// GGUF type ids, EDGEXPU_GGUF_TYPE_* in include/edgexpu/gguf_quant.h:17-24.
constexpr uint32_t TYPE_F32 = 0;
constexpr uint32_t TYPE_F16 = 1;
constexpr uint32_t TYPE_Q4_0 = 2;
constexpr uint32_t TYPE_Q5_0 = 6;
constexpr uint32_t TYPE_Q8_0 = 8;
constexpr uint32_t TYPE_Q4_K = 12;
constexpr uint32_t TYPE_Q5_K = 13;
constexpr uint32_t TYPE_Q6_K = 14;

// Bits of the device status word (host-mapped; kernels only ever OR into it).
constexpr uint32_t ST_TIMEOUT_FULL = 1u;   // a consumer gave up waiting for a tile copy
constexpr uint32_t ST_TIMEOUT_EMPTY = 2u;  // the producer gave up waiting for a free stage
constexpr uint32_t ST_TIMEOUT_DRAIN = 4u;  // copies still in flight at exit after the limit
constexpr uint32_t ST_TIMEOUT_PEER = 8u;   // a tensor-parallel peer did not deliver its partial in time
constexpr uint32_t ST_BAD_INDEX = 16u;     // a row id passed to a gather was outside the tensor

// Every mbarrier wait gives up after this long and reports through the status word.
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_try_wait, but a thread whose phase has not completed may sleep up to `hint_ns` (it
// wakes as soon as the phase completes), so waiting warps leave issue slots to working ones.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete; false after WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31u) == 0 && global_ns() - t0 > WAIT_LIMIT_NS) return false;
  }
}

// 1-D bulk copy global -> this CTA's shared memory, completing on an mbarrier (TMA engine, no
// tensor map, no multicast).  dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// L2 policy for data read exactly once (streamed weights): evict first.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ float fp16_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

// Bounded mbarrier wait that also gives up as soon as another thread raised the abort flag.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_sleep(bar, parity, 2000u)) return true;
    if ((i & 31u) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > WAIT_LIMIT_NS) return false;
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

// Greedy-argmax key: larger key = better.  The high word orders float scores, the low word
// prefers the LOWER token id on equal scores (the reference's tie rule, native.c:2380).
// NaN and -inf never win (the reference compares with strict '>' against -inf, :2373).
__device__ __forceinline__ unsigned long long argmax_key(float score, uint32_t id) {
  if (!(score > -INFINITY)) return 0ull;
  uint32_t u = score == 0.0f ? 0u : __float_as_uint(score);  // -0 and +0 compare equal there
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(u) << 32) | static_cast<unsigned long long>(0xFFFFFFFFu - id);
}

}  // namespace ex
