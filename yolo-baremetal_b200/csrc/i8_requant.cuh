// Requantisation of int32 tcgen05 accumulators to int8 (the kind::i8
// convolution epilogues: conv_i8.cu and the fused Bottleneck of
// bottleneck_i8.cu).  Integer rules as in i8k.h: y = rne((acc + bias) * M,
// shift), then the SiLU table or the clamp, plus the residual table term.
#pragma once
#include <cstdint>

#include "sm100.cuh"

namespace yb {
namespace {

// (p >> sh) rounded half to even, sh >= 1, without branches: with
// p = q*2^sh + r (q = floor), adding 2^(sh-1) - 1 + (q & 1) carries into q
// exactly when r > half, or r == half and q is odd.  |p| <= 2^62 here.
__device__ __forceinline__ long long rshift_rne(long long p, int sh) {
  return (p + ((1LL << (sh - 1)) - 1) + ((p >> sh) & 1)) >> sh;
}

// Requantises 16 channels of one pixel into 4 packed words: acc + bias,
// fixed-point multiply, round-half-even shift, then the SiLU table (LUT) or
// the clamp, plus the residual table term (RES).  FAST: one 64-bit
// multiply-add per channel, acc * M + D with D = bias * M + 2^(sh-1) - 1,
// whose high word shifted by sh - 32 is floor((p + 2^(sh-1) - 1) / 2^sh) for
// p = (acc + bias) * M: the round-half-even result except at an exact tie,
// where the low sh bits of the sum are all ones (so its low word is too) and
// an odd quotient must be raised by one; such a unit is redone exactly.
// Otherwise every intermediate is kept in 64 bits.
// Exact path: every intermediate in 64 bits (rare: shifts below 32, table
// terms too large for the fast path, or a unit with a tie).
// Warp-collective (it reloads the 16 accumulators from tensor memory at
// taddr): call with the whole warp.
template <bool LUT, bool RES>
__device__ __noinline__ uint4 requant16_exact(uint32_t taddr, const uint4 rw, const int4* qc, const int32_t* sb,
                                              const int8_t* slut, const int32_t* srtab, int res_mult,
                                              int res_shift) {
  uint32_t r[16];
  tc_ld_32x32b_x16(taddr, r);
  tc_wait_ld();
  uint32_t packed[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t rword = j == 0 ? rw.x : j == 1 ? rw.y : j == 2 ? rw.z : rw.w;
    uint32_t w = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = 4 * j + k;
      const int rve = static_cast<int>(static_cast<int8_t>((rword >> (8 * k)) & 0xFFu));
      const long long v = static_cast<long long>(static_cast<int32_t>(r[e])) + sb[e];
      long long y = rshift_rne(v * qc[e].x, qc[e].w + 32);
      if (LUT) y = slut[(y < -128 ? -128 : y > 127 ? 127 : y) + 128];
      if (RES) y += rshift_rne(static_cast<long long>(rve) * res_mult, res_shift);
      const int o = static_cast<int>(y < -127 ? -127 : y > 127 ? 127 : y);
      w |= (static_cast<uint32_t>(o) & 0xFFu) << (8 * k);
    }
    packed[j] = w;
  }
  return make_uint4(packed[0], packed[1], packed[2], packed[3]);
}

// Fast path (every shift >= 32): one 64-bit multiply-add per channel,
// acc * M + D with D = bias * M + 2^(sh-1) - 1, whose high word shifted by
// sh - 32 is floor((p + 2^(sh-1) - 1) / 2^sh) for p = (acc + bias) * M: the
// round-half-even result except at an exact tie, where the low sh bits of the
// sum are all ones (so its low word is too) and an odd quotient must be
// raised by one.  Returns whether a low word was all ones; the caller then
// redoes the unit on the exact path.
template <bool LUT, bool RES>
__device__ __forceinline__ bool requant16_fast(const uint32_t (&r)[16], const uint4 rw, const int4* qc,
                                               const int8_t* slut, const int32_t* srtab, uint32_t (&packed)[4]) {
  bool tie = false;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int o[4];
    const uint32_t rword = j == 0 ? rw.x : j == 1 ? rw.y : j == 2 ? rw.z : rw.w;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = 4 * j + k;
      const int4 q = qc[e];
      const long long d = (static_cast<long long>(q.z) << 32) | static_cast<unsigned>(q.y);
      const long long p = static_cast<long long>(static_cast<int32_t>(r[e])) * q.x + d;
      tie |= static_cast<unsigned>(p) == 0xFFFFFFFFu;
      int v = static_cast<int>(p >> 32) >> q.w;
      if (LUT) v = slut[min(max(v, -128), 127) + 128];
      if (RES) {
        // |table term| < 2^29: clamping v to +-2^30 first keeps the sum
        // exact wherever the result is not saturated.
        const int rve = static_cast<int>(static_cast<int8_t>((rword >> (8 * k)) & 0xFFu));
        v = min(max(v, -(1 << 30)), 1 << 30) + srtab[rve + 128];
      }
      // Table values already lie in [-127, 127].
      o[k] = (LUT && !RES) ? v : min(max(v, -127), 127);
    }
    packed[j] = __byte_perm(__byte_perm(o[0], o[1], 0x0040), __byte_perm(o[2], o[3], 0x0040), 0x5410);
  }
  return tie;
}

}  // namespace
}  // namespace yb
