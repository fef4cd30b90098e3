// Division by a runtime-invariant divisor, usable from host and device code.
//
// Unsigned 32-bit n / d as one multiply-high, an add and a shift (Granlund & Montgomery,
// "Division by invariant integers using multiplication", PLDI 1994, round-up method):
//   l = ceil(log2 d),  m = floor(2^32 (2^l - d) / d) + 1,  n / d = (mulhi(n, m) + n) >> l
// exact for every 0 <= n < 2^32 and 1 <= d < 2^32. Kernels use it instead of the emulated
// 64-bit division in per-element index math.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define TB_HD __host__ __device__
#else
#define TB_HD
#endif

namespace tb {

struct FastDiv {
  uint32_t d, m, l;
  TB_HD FastDiv() : d(1), m(1), l(0) {}
  TB_HD explicit FastDiv(uint32_t div) : d(div), m(1), l(0) {
    while (l < 32 && (1ull << l) < div) ++l;
    m = (uint32_t)((((1ull << 32) * ((1ull << l) - div)) / div) + 1);
  }
  TB_HD inline uint32_t div(uint32_t n) const {
#if defined(__CUDA_ARCH__)
    const uint32_t hi = __umulhi(n, m);
#else
    const uint32_t hi = (uint32_t)(((uint64_t)n * m) >> 32);
#endif
    return (uint32_t)(((uint64_t)hi + n) >> l);
  }
  TB_HD inline void divmod(uint32_t n, uint32_t &q, uint32_t &r) const {
    q = div(n);
    r = n - q * d;
  }
};

}  // namespace tb
