// Device helpers for the split activation format (kernels.h): value = hi + lo
// with hi = bf16_rn(v), lo = bf16_rn(v - hi), both planes NHWC bf16.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>

namespace yb {

__device__ __forceinline__ float bf16_bits_to_f(uint32_t h) { return __uint_as_float(h << 16); }

__device__ __forceinline__ uint32_t f_to_bf16_bits(float v) {
  const __nv_bfloat16 b = __float2bfloat16_rn(v);
  return static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&b));
}

// v - hi is exact in fp32, so hi + lo reproduces v to ~16 significant bits.
__device__ __forceinline__ void split1(float v, uint32_t& hi, uint32_t& lo) {
  hi = f_to_bf16_bits(v);
  lo = f_to_bf16_bits(__fsub_rn(v, bf16_bits_to_f(hi)));
}

__device__ __forceinline__ float join1(uint16_t hi, uint16_t lo) {
  return bf16_bits_to_f(hi) + bf16_bits_to_f(lo);
}

// 8 consecutive channels: one 16-byte load per plane.
__device__ __forceinline__ void load8(const uint16_t* hi, long long plane, float (&v)[8]) {
  const uint4 h = __ldg(reinterpret_cast<const uint4*>(hi));
  const uint4 l = __ldg(reinterpret_cast<const uint4*>(hi + plane));
  const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
  const uint32_t lw[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 s = __fadd2_rn(make_float2(bf16_bits_to_f(hw[i] & 0xFFFFu), bf16_bits_to_f(hw[i] >> 16)),
                                make_float2(bf16_bits_to_f(lw[i] & 0xFFFFu), bf16_bits_to_f(lw[i] >> 16)));
    v[2 * i] = s.x;
    v[2 * i + 1] = s.y;
  }
}

// Plain (non-__ldg) variant for buffers written earlier by the same kernel.
__device__ __forceinline__ void load8_rw(const uint16_t* hi, long long plane, float (&v)[8]) {
  const uint4 h = *reinterpret_cast<const uint4*>(hi);
  const uint4 l = *reinterpret_cast<const uint4*>(hi + plane);
  const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
  const uint32_t lw[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 s = __fadd2_rn(make_float2(bf16_bits_to_f(hw[i] & 0xFFFFu), bf16_bits_to_f(hw[i] >> 16)),
                                make_float2(bf16_bits_to_f(lw[i] & 0xFFFFu), bf16_bits_to_f(lw[i] >> 16)));
    v[2 * i] = s.x;
    v[2 * i + 1] = s.y;
  }
}

// Splits two values at once: packed (v0 in the low half) hi and lo words.
// The remainders are exact (v - hi needs no rounding) and computed as one
// paired fused multiply-add with -1 (exact too), explicitly rounded so that
// the compiler never fuses them with the multiply that produced v0 / v1 (an
// FMA there would take the remainder of the unrounded product): the split of
// a value is then the same in every kernel, whatever code computed it.
__device__ __forceinline__ void split2(float v0, float v1, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  const float2 r = __ffma2_rn(make_float2(__uint_as_float(hi << 16), __uint_as_float(hi & 0xFFFF0000u)),
                              make_float2(-1.0f, -1.0f), make_float2(v0, v1));
  const __nv_bfloat162 l = __floats2bfloat162_rn(r.x, r.y);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Elementwise sums of N (even) values in pairs (one paired add per two).
template <int N>
__device__ __forceinline__ void add_pairs(float (&v)[N], const float* a, const float* b) {
#pragma unroll
  for (int e = 0; e < N; e += 2) {
    const float2 s = __fadd2_rn(make_float2(a[e], a[e + 1]), make_float2(b[e], b[e + 1]));
    v[e] = s.x;
    v[e + 1] = s.y;
  }
}

__device__ __forceinline__ void store8(uint16_t* hi, long long plane, const float (&v)[8]) {
  uint32_t hw[4], lw[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) split2(v[2 * i], v[2 * i + 1], hw[i], lw[i]);
  *reinterpret_cast<uint4*>(hi) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  *reinterpret_cast<uint4*>(hi + plane) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}

// SiLU without branches: x * 1 / (1 + 2^(-x log2 e)), with the hardware's
// approximate base-2 exponential and reciprocal in their flush-to-zero forms
// (no denormal handling; about 2^-22 relative error each).  For x below
// about -88 the exponential overflows to +inf and the result is -0 (the exact
// value is below 1e-36 in magnitude).  The multiplies are explicitly rounded
// and callers add to the result with __fadd_rn, so that SiLU + residual
// rounds the same way in every kernel.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_ftz(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float silu_fast(float x) {
  return __fmul_rn(x, rcp_ftz(__fadd_rn(1.0f, ex2_ftz(__fmul_rn(x, -1.4426950408889634f)))));
}
// The same for N (even) values, the multiplies and adds paired: equal to
// silu_fast on each value, bit for bit.
template <int N>
__device__ __forceinline__ void silu_fast_n(float (&v)[N]) {
#pragma unroll
  for (int e = 0; e < N; e += 2) {
    const float2 x = make_float2(v[e], v[e + 1]);
    const float2 t = __fmul2_rn(x, make_float2(-1.4426950408889634f, -1.4426950408889634f));
    const float2 d = __fadd2_rn(make_float2(1.0f, 1.0f), make_float2(ex2_ftz(t.x), ex2_ftz(t.y)));
    const float2 y = __fmul2_rn(x, make_float2(rcp_ftz(d.x), rcp_ftz(d.y)));
    v[e] = y.x;
    v[e + 1] = y.y;
  }
}

}  // namespace yb
