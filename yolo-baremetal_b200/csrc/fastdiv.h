// Division of 32-bit unsigned values by a divisor fixed at launch, with one
// multiply-high, one subtract and two shifts instead of the ~20-instruction
// integer division sequence: the per-tile index arithmetic of the
// single-thread producers and the MMA issuer sits on their critical path.
// Granlund and Montgomery, "Division by invariant integers using
// multiplication" (1994): l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1,
// q = (t + ((x - t) >> 1)) >> (l - 1) with t = umulhi(m, x); exact for every
// x < 2^32 and d >= 1 (d = 1: m = 1 and both shifts 0).  Built on the host.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace yb {

struct FastDiv {
  uint32_t d = 1, m = 1, s1 = 0, s2 = 0;
  FastDiv() = default;
  __host__ __device__ explicit FastDiv(uint32_t div) : d(div ? div : 1) {
    uint32_t l = 0;
    while (l < 32 && (1ull << l) < d) ++l;
    m = static_cast<uint32_t>(((1ull << 32) * ((1ull << l) - d)) / d + 1);
    s1 = l > 0 ? 1u : 0u;
    s2 = l > 0 ? l - 1 : 0u;
  }
#ifdef __CUDACC__
  __device__ __forceinline__ uint32_t div(uint32_t x) const {
    const uint32_t t = __umulhi(m, x);
    return (t + ((x - t) >> s1)) >> s2;
  }
#endif
};

}  // namespace yb
