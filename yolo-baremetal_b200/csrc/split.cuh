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
    v[2 * i] = bf16_bits_to_f(hw[i] & 0xFFFFu) + bf16_bits_to_f(lw[i] & 0xFFFFu);
    v[2 * i + 1] = bf16_bits_to_f(hw[i] >> 16) + bf16_bits_to_f(lw[i] >> 16);
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
    v[2 * i] = bf16_bits_to_f(hw[i] & 0xFFFFu) + bf16_bits_to_f(lw[i] & 0xFFFFu);
    v[2 * i + 1] = bf16_bits_to_f(hw[i] >> 16) + bf16_bits_to_f(lw[i] >> 16);
  }
}

// Splits two values at once: packed (v0 in the low half) hi and lo words.
// The remainders use explicitly rounded subtractions so that the compiler
// never fuses them with the multiply that produced v0 / v1 (an FMA there
// would take the remainder of the unrounded product): the split of a value
// is then the same in every kernel, whatever code computed it.
__device__ __forceinline__ void split2(float v0, float v1, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  const float r0 = __fsub_rn(v0, __uint_as_float(hi << 16));
  const float r1 = __fsub_rn(v1, __uint_as_float(hi & 0xFFFF0000u));
  const __nv_bfloat162 l = __floats2bfloat162_rn(r0, r1);
  lo = *reinterpret_cast<const uint32_t*>(&l);
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
__device__ __forceinline__ float silu_fast(float x) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(__fmul_rn(x, -1.4426950408889634f)));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fadd_rn(1.0f, e)));
  return __fmul_rn(x, r);
}

}  // namespace yb
