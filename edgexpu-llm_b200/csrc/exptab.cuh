// exptab.cuh -- expf with the host C library's results, for the device ops that must give the
// reference's bits.  The reference calls libm's expf in its softmax (src/cpu_kernel.c:344) and
// SiLU (:250); libm's expf is not correctly rounded in every case, so no device formula matches
// it everywhere.  Instead the host evaluates expf at every float where its value is neither 0
// nor +inf (x in [-104, 88.8]: about 2.24e9 inputs) and the device looks the result up, indexed
// by the input's bits (exptab.cu builds the table, 9 GB of HBM, once per process).
#pragma once

#include <cstdint>

namespace ex {

constexpr uint32_t EXPTAB_NEG_MAX = 0x42D00000u;  // |x| bits of -104.0f: expf is 0 below it
constexpr uint32_t EXPTAB_POS_MAX = 0x42B1999Au;  // bits of 88.8f: expf is +inf above it

struct ExpTab {
  const float* neg;  // [EXPTAB_NEG_MAX + 1]: expf(-x) for the |x| bits
  const float* pos;  // [EXPTAB_POS_MAX + 1]: expf(x)
};

__device__ __forceinline__ float exp_lookup(const ExpTab& t, float x) {
  const uint32_t b = __float_as_uint(x), a = b & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return x;  // NaN
  if (b >> 31) return a <= EXPTAB_NEG_MAX ? t.neg[a] : 0.0f;
  return a <= EXPTAB_POS_MAX ? t.pos[a] : __int_as_float(0x7F800000);
}

// The process-wide table (built on the first call; the host's expf); release when done.
int exptab_acquire(ExpTab* out, char* error, size_t error_size);
void exptab_release();

}  // namespace ex
