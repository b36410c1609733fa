// Device-side weight preparation (see weight_prep.h).  The host path's
// arithmetic is restated with explicitly rounded intrinsics (no contraction
// into fused multiply-adds), so each device image equals the host image bit
// for bit: tests/test_gpu_weight_prep.py compares them.
#include <cstdint>

#include "sm100.cuh"
#include "weight_prep.h"

namespace yb {
namespace {

inline unsigned blocks_of(long long n, int t) { return static_cast<unsigned>((n + t - 1) / t); }

// One block per convolution (utils.c:81-106): the per-channel scale is
// recomputed by every thread that needs it, with the same operations.
__global__ void fold_bn_kernel(const FoldDesc* __restrict__ descs, float* __restrict__ arena) {
  const FoldDesc d = descs[blockIdx.x];
  const long long total = static_cast<long long>(d.oc) * d.per;
  for (long long i = threadIdx.x; i < total; i += blockDim.x) {
    const int o = static_cast<int>(i / d.per);
    const float scale = __fdiv_rn(arena[d.g + o], __fsqrt_rn(__fadd_rn(arena[d.var + o], 1e-5f)));
    arena[d.w + i] = __fmul_rn(arena[d.w + i], scale);
  }
  for (int o = threadIdx.x; o < d.oc; o += blockDim.x) {
    const float scale = __fdiv_rn(arena[d.g + o], __fsqrt_rn(__fadd_rn(arena[d.var + o], 1e-5f)));
    const float t = __fsub_rn(arena[d.b + o], arena[d.mu + o]);
    arena[d.b + o] = __fadd_rn(__fmul_rn(t, scale), arena[d.be + o]);
  }
}

// Round to nearest even bf16 bits, the host packer's integer rule.
__device__ __forceinline__ uint16_t bf16_bits(float f) {
  uint32_t u = __float_as_uint(f);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

// One thread per (N tile, K chunk, row, k) element of the packed image.
__global__ void pack_conv_kernel(const float* __restrict__ w, int co, int ci, int kh, int kw, int n_tile,
                                 int num_kc, long long total, uint8_t* __restrict__ dst) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int kk = static_cast<int>(i % 64);
  const int r = static_cast<int>((i / 64) % n_tile);
  const long long tc = i / (64LL * n_tile);  // nt * num_kc + kc
  const int kc = static_cast<int>(tc % num_kc);
  const int nt = static_cast<int>(tc / num_kc);
  const int n = nt * n_tile + r;
  const int K = kh * kw * ci;
  const int k = kc * 64 + kk;
  if (n >= co || k >= K) return;
  const int tap = k / ci;
  const int c = k - tap * ci;
  const int ky = tap / kw;
  const int kx = tap - ky * kw;
  const float v = w[((static_cast<long long>(n) * ci + c) * kh + ky) * kw + kx];
  const uint16_t h = bf16_bits(v);
  const uint16_t l = bf16_bits(__fsub_rn(v, __uint_as_float(static_cast<uint32_t>(h) << 16)));
  uint8_t* hi_plane = dst + tc * (static_cast<long long>(n_tile) * 256);
  const uint32_t off = sw128_offset(static_cast<uint32_t>(r), static_cast<uint32_t>(kk >> 3)) + (kk & 7) * 2;
  *reinterpret_cast<uint16_t*>(hi_plane + off) = h;
  *reinterpret_cast<uint16_t*>(hi_plane + static_cast<long long>(n_tile) * 128 + off) = l;
}

__global__ void taps_transpose_kernel(const float* __restrict__ w, int C, float* __restrict__ dst) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 9 * C) return;
  const int k = i / C, c = i - k * C;
  dst[i] = w[c * 9 + k];
}

}  // namespace

cudaError_t launch_fold_bn(const FoldDesc* d_desc, int n, float* arena, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  fold_bn_kernel<<<n, 256, 0, s>>>(d_desc, arena);
  return cudaGetLastError();
}

cudaError_t launch_pack_conv(const float* w, int co, int ci, int kh, int kw, int n_tile, uint8_t* dst, size_t bytes,
                             cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(dst, 0, bytes, s);
  if (e != cudaSuccess) return e;
  const int K = kh * kw * ci;
  const int num_kc = (K + 63) / 64;
  const int n_tiles = (co + n_tile - 1) / n_tile;
  const long long total = static_cast<long long>(n_tiles) * num_kc * n_tile * 64;
  pack_conv_kernel<<<blocks_of(total, 256), 256, 0, s>>>(w, co, ci, kh, kw, n_tile, num_kc, total, dst);
  return cudaGetLastError();
}

cudaError_t launch_taps_transpose(const float* w, int C, float* dst, cudaStream_t s) {
  taps_transpose_kernel<<<blocks_of(9LL * C, 256), 256, 0, s>>>(w, C, dst);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ INT8
namespace {

// ratio -> (M, sh), the host rule: frexp, M = rint(f * 2^31) in [2^30, 2^31).
__device__ bool multiplier_dev(double ratio, int32_t* m, int32_t* sh) {
  if (!(ratio > 0.0)) {
    *m = 0;
    *sh = 1;
    return true;
  }
  int e = 0;
  const double f = frexp(ratio, &e);
  long long mm = __double2ll_rn(__dmul_rn(f, 2147483648.0));
  if (mm == 2147483648LL) {
    mm = 1073741824LL;
    e += 1;
  }
  const int s = 31 - e;
  if (s < 1) return false;
  if (s > 62) {
    *m = 0;
    *sh = 1;
    return true;
  }
  *m = static_cast<int32_t>(mm);
  *sh = s;
  return true;
}

// One warp per output channel.
__global__ void quantize_i8_kernel(QuantArgs a) {
  const int o = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (o >= a.co) return;  // warp-uniform
  const int per = a.ci * a.kk;
  const float s_ref = a.per_out ? a.cs[o] : a.cs[0];
  const float* wr = a.w + static_cast<long long>(o) * per;
  auto we = [&](int idx) {
    const float c = a.per_out ? a.cs[o] : a.cs[idx / a.kk];
    return __double2float_rn(
        __ddiv_rn(__dmul_rn(static_cast<double>(wr[idx]), static_cast<double>(c)), static_cast<double>(s_ref)));
  };
  float m = 0.0f;
  for (int idx = lane; idx < per; idx += 32) m = fmaxf(m, fabsf(we(idx)));
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
  const float sw = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
  for (int idx = lane; idx < per; idx += 32) {
    const float v = rintf(__fdiv_rn(we(idx), sw));
    a.wq[static_cast<long long>(o) * per + idx] =
        static_cast<int8_t>(v < -127.0f ? -127 : v > 127.0f ? 127 : static_cast<int>(v));
  }
  if (lane == 0) {
    const double prod = __dmul_rn(static_cast<double>(s_ref), static_cast<double>(sw));
    long long bv = a.b ? __double2ll_rn(__ddiv_rn(static_cast<double>(a.b[o]), prod)) : 0;
    bv = bv < -2147483647LL ? -2147483647LL : bv > 2147483647LL ? 2147483647LL : bv;
    a.bq[o] = static_cast<int32_t>(bv);
    a.deq[o] = __double2float_rn(prod);
    int32_t mu = 0, sh = 1;
    if (a.s_t > 0.0 && !multiplier_dev(__ddiv_rn(prod, a.s_t), &mu, &sh)) atomicExch(a.bad, 1);
    a.mult[o] = mu;
    a.shift[o] = sh;
  }
}

__host__ __device__ constexpr int p2_tap_order(int pos) {
  return pos == 3 ? 4 : pos == 4 ? 3 : pos == 5 ? 7 : pos == 6 ? 5 : pos == 7 ? 6 : pos;
}

__global__ void pack_i8_kernel(const int8_t* __restrict__ wq, int co, int ci, int kh, int kw, I8Tiling t,
                               long long total, uint8_t* __restrict__ dst) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int kk = static_cast<int>(i % 128);
  const int r = static_cast<int>((i / 128) % t.n_tile);
  const long long tc = i / (128LL * t.n_tile);
  const int kc = static_cast<int>(tc % t.num_kc);
  const int nt = static_cast<int>(tc / t.num_kc);
  const int n = nt * t.n_tile + r;
  const int k = kc * 128 + kk;
  if (n >= co || k >= t.K) return;
  const int pos = k / t.ci_pad;
  const int tap = t.tap_perm ? p2_tap_order(pos) : pos;
  const int cc = k - pos * t.ci_pad;
  if (cc >= ci) return;
  const int ky = tap / kw, kx = tap - (tap / kw) * kw;
  const int8_t v = wq[((static_cast<long long>(n) * ci + cc) * kh + ky) * kw + kx];
  uint8_t* out = dst + tc * (128LL * t.n_tile);
  out[sw128_offset(static_cast<uint32_t>(r), static_cast<uint32_t>(kk >> 4)) + (kk & 15)] = static_cast<uint8_t>(v);
}

__device__ __forceinline__ uint32_t byte_of(int8_t v, int slot) {
  return (static_cast<uint32_t>(v) & 0xFFu) << (8 * slot);
}

__global__ void pack_dw_i8_kernel(const int8_t* __restrict__ wq, int C, uint32_t* __restrict__ wt) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 3 * C) return;
  const int ky = i / C, c = i - ky * C;
  const int8_t* q = wq + c * 9 + 3 * ky;
  wt[i] = byte_of(q[0], 0) | byte_of(q[1], 1) | byte_of(q[2], 2);
}

__global__ void pack_pe_i8_kernel(const int8_t* __restrict__ wq, int C, int8_t* __restrict__ wt) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 9 * C) return;
  const int k = i / C, c = i - k * C;
  wt[i] = wq[c * 9 + k];
}

__global__ void pack_stem_i8_kernel(const int8_t* __restrict__ wq, int co, uint32_t* __restrict__ wp) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 9 * co) return;
  const int t = i / co, o = i - t * co;
  wp[i] = byte_of(wq[(o * 3 + 0) * 9 + t], 0) | byte_of(wq[(o * 3 + 1) * 9 + t], 1) |
          byte_of(wq[(o * 3 + 2) * 9 + t], 2);
}

}  // namespace

cudaError_t launch_quantize_i8(const QuantArgs& a, cudaStream_t s) {
  if (a.co <= 0) return cudaSuccess;
  quantize_i8_kernel<<<blocks_of(32LL * a.co, 256), 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_pack_i8(const int8_t* wq, int co, int ci, int kh, int kw, const I8Tiling& t, uint8_t* dst,
                           size_t bytes, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(dst, 0, bytes, s);
  if (e != cudaSuccess) return e;
  const long long total = static_cast<long long>(t.n_tiles) * t.num_kc * t.n_tile * 128;
  pack_i8_kernel<<<blocks_of(total, 256), 256, 0, s>>>(wq, co, ci, kh, kw, t, total, dst);
  return cudaGetLastError();
}

cudaError_t launch_pack_dw_i8(const int8_t* wq, int C, uint32_t* wt, cudaStream_t s) {
  pack_dw_i8_kernel<<<blocks_of(3LL * C, 256), 256, 0, s>>>(wq, C, wt);
  return cudaGetLastError();
}

cudaError_t launch_pack_pe_i8(const int8_t* wq, int C, int8_t* wt, cudaStream_t s) {
  pack_pe_i8_kernel<<<blocks_of(9LL * C, 256), 256, 0, s>>>(wq, C, wt);
  return cudaGetLastError();
}

cudaError_t launch_pack_stem_i8(const int8_t* wq, int co, uint32_t* wp, cudaStream_t s) {
  pack_stem_i8_kernel<<<blocks_of(9LL * co, 256), 256, 0, s>>>(wq, co, wp);
  return cudaGetLastError();
}

}  // namespace yb
