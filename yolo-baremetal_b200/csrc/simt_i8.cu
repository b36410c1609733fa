// CUDA-core kernels of the INT8 forward: input quantisation (alone or fused
// into the first convolution), max pool, depthwise 3x3, upsample + concat.
// All activations are NHWC int8 views {ptr, cstride (per pixel), bstride (per
// image)}; every rule is the integer arithmetic declared in i8k.h, which the
// CPU INT8 oracle restates.
#include <atomic>
#include <climits>
#include <cstdint>

#include "pdl.cuh"
#include "i8k.h"

namespace yb {
namespace {

__device__ __forceinline__ long long rne(long long p, int sh) {
  return (p + ((1LL << (sh - 1)) - 1) + ((p >> sh) & 1)) >> sh;
}

inline unsigned blocks_for(long long n, int t) { return static_cast<unsigned>((n + t - 1) / t); }

// --------------------------------------------------------------- input
__global__ void quantize_input_kernel(const float* in, int B, int C, int H, int W, float s, I8View out) {
  pdl_wait();
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(B) * H * W;
  if (idx >= total) return;
  const int b = static_cast<int>(idx / (static_cast<long long>(H) * W));
  const long long p = idx - static_cast<long long>(b) * H * W;
  int8_t* o = out.p + b * out.bstride + p * out.cstride;
  for (int c = 0; c < C; ++c) {
    const float v = rintf(__fdiv_rn(in[(static_cast<long long>(b) * C + c) * H * W + p], s));
    o[c] = static_cast<int8_t>(v < -127.f ? -127 : v > 127.f ? 127 : static_cast<int>(v));
  }
}

// ------------------------------------------------------------ max pool
// k x k, stride 1, padding k / 2 excluded (the -128 sentinel is below every
// quantised value); 16 channels per thread.
__global__ void maxpool_i8_kernel(I8View in, I8View out, int B, int H, int W, int C, int k) {
  pdl_wait();
  const int C16 = C >> 4;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(B) * H * W * C16;
  if (idx >= total) return;
  const int c = static_cast<int>(idx % C16) * 16;
  const long long pix = idx / C16;
  const int b = static_cast<int>(pix / (static_cast<long long>(H) * W));
  const int p = static_cast<int>(pix - static_cast<long long>(b) * H * W);
  const int y = p / W, x = p - (p / W) * W, pad = k / 2;
  int m[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) m[e] = -128;
  for (int ky = 0; ky < k; ++ky) {
    const int iy = y - pad + ky;
    if (iy < 0 || iy >= H) continue;
    for (int kx = 0; kx < k; ++kx) {
      const int ix = x - pad + kx;
      if (ix < 0 || ix >= W) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(in.p + b * in.bstride +
                                                      static_cast<long long>(iy * W + ix) * in.cstride + c);
      const int8_t* vb = reinterpret_cast<const int8_t*>(&v);
#pragma unroll
      for (int e = 0; e < 16; ++e) m[e] = max(m[e], static_cast<int>(vb[e]));
    }
  }
  uint4 o;
  int8_t* ob = reinterpret_cast<int8_t*>(&o);
#pragma unroll
  for (int e = 0; e < 16; ++e) ob[e] = static_cast<int8_t>(m[e]);
  *reinterpret_cast<uint4*>(out.p + b * out.bstride + static_cast<long long>(p) * out.cstride + c) = o;
}

// ------------------------------------------------------- depthwise 3x3
// y = rne((bq + sum x*wq) * mult, shift), then the SiLU table (lut != null)
// or clamp to [-127, 127].  A thread computes 4 channels of R consecutive
// output rows of one column.  Each input row's three pixels x-1, x, x+1 (one
// word of 4 channels each) are transposed once into 4 per-channel words
// (byte kx = pixel x-1+kx) and serve the outputs above, at and below the row,
// each of which is then 3 dp4a per channel against the weights packed the
// same way on the host: wr[ky][c] byte kx = wq[c][ky][kx].  Pixels outside
// the image are zero words; all loads of a strip are in flight together.
// The sum fits int32 (|sum| <= 9 * 128 * 127);
// the requantisation is sum * M + (bq * M + 2^(sh-1) - 1) >> sh, redone in
// 64 bits for shifts below 32 or a possible tie (low word all ones).
__device__ __forceinline__ void transpose4(uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t (&y)[4]) {
  const uint32_t t0 = __byte_perm(a, b, 0x5140), t1 = __byte_perm(a, b, 0x7362);
  const uint32_t t2 = __byte_perm(c, d, 0x5140), t3 = __byte_perm(c, d, 0x7362);
  y[0] = __byte_perm(t0, t2, 0x5410);
  y[1] = __byte_perm(t0, t2, 0x7632);
  y[2] = __byte_perm(t1, t3, 0x5410);
  y[3] = __byte_perm(t1, t3, 0x7632);
}

template <int R>
__global__ void __launch_bounds__(256) dw3x3_i8_kernel(I8View in, I8View out, int B, int H, int W, int C,
                                                       const uint32_t* wr, const int32_t* bq, const int32_t* mult,
                                                       const int32_t* shift, const int8_t* lut) {
  __shared__ int8_t slut[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) slut[i] = lut ? lut[i] : 0;
  __syncthreads();
  // 32-bit indexing: the launcher checks that threads and per-image offsets fit.
  const int C4 = C >> 2;
  const int strips = (H + R - 1) / R;
  const int idx = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= B * strips * W * C4) return;
  const int c = (idx % C4) * 4;
  int r = idx / C4;
  const int x = r % W;
  r /= W;
  const int strip = r % strips;
  const int b = r / strips;
  uint32_t wk[3][4];
#pragma unroll
  for (int ky = 0; ky < 3; ++ky) {
    const uint4 w4 = __ldg(reinterpret_cast<const uint4*>(wr + ky * C + c));
    wk[ky][0] = w4.x;
    wk[ky][1] = w4.y;
    wk[ky][2] = w4.z;
    wk[ky][3] = w4.w;
  }
  int M[4], sx[4];
  long long D[4];
  bool fast = true;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int m = __ldg(mult + c + e);
    const int sh = m == 0 ? 32 : __ldg(shift + c + e);
    M[e] = m;
    sx[e] = sh - 32;
    fast = fast && sh >= 32;
    D[e] = static_cast<long long>(__ldg(bq + c + e)) * m + ((1LL << (sh - 1)) - 1);
  }
  pdl_wait();
  const bool cl = x > 0, cr = x < W - 1;
  const int y0 = strip * R;
  const int8_t* ib = in.p + b * in.bstride + c;
  // Every load of the strip is issued before the first sum (R + 2 rows x 3
  // pixels in flight per thread), then each row is transposed once.
  uint32_t raw[R + 2][3];
#pragma unroll
  for (int k = 0; k < R + 2; ++k) {
    const int iy = y0 - 1 + k;
    const bool ok = iy >= 0 && iy < H;
    const int8_t* rp = ib + (iy * W + x - 1) * static_cast<int>(in.cstride);
    raw[k][0] = ok && cl ? __ldg(reinterpret_cast<const uint32_t*>(rp)) : 0u;
    raw[k][1] = ok ? __ldg(reinterpret_cast<const uint32_t*>(rp + in.cstride)) : 0u;
    raw[k][2] = ok && cr ? __ldg(reinterpret_cast<const uint32_t*>(rp + 2 * in.cstride)) : 0u;
  }
  uint32_t v[R + 2][4];
#pragma unroll
  for (int k = 0; k < R + 2; ++k) transpose4(raw[k][0], raw[k][1], raw[k][2], 0u, v[k]);
  int8_t* ob = out.p + b * out.bstride + c;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int y = y0 + i;
    if (y >= H) break;
    int acc[4], o[4];
    bool exact = !fast;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc[e] = __dp4a(static_cast<int>(v[i][e]), static_cast<int>(wk[0][e]), 0);
      acc[e] = __dp4a(static_cast<int>(v[i + 1][e]), static_cast<int>(wk[1][e]), acc[e]);
      acc[e] = __dp4a(static_cast<int>(v[i + 2][e]), static_cast<int>(wk[2][e]), acc[e]);
      const long long pr = static_cast<long long>(acc[e]) * M[e] + D[e];
      exact = exact || static_cast<unsigned>(pr) == 0xFFFFFFFFu;
      o[e] = static_cast<int>(pr >> 32) >> (sx[e] & 31);
    }
    if (__builtin_expect(exact, 0)) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const long long yv = rne((static_cast<long long>(acc[e]) + __ldg(bq + c + e)) * M[e], sx[e] + 32);
        o[e] = static_cast<int>(yv < -128 ? -128 : yv > 127 ? 127 : yv);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int yv = min(max(o[e], -128), 127);
      o[e] = lut ? slut[yv + 128] : max(yv, -127);
    }
    *reinterpret_cast<uint32_t*>(ob + (y * W + x) * static_cast<int>(out.cstride)) =
        __byte_perm(__byte_perm(o[0], o[1], 0x0040), __byte_perm(o[2], o[3], 0x0040), 0x5410);
  }
}

// ---------------------------------------------------------- SPPF pools
// The three chained 5x5 stride-1 pools of SPPF in one launch: with
// out-of-image positions excluded they are the 5x5, 9x9 and 13x13 pools of
// the input.  One CTA per (image, 16 channels) holds the map in shared
// memory (one uint4 per pixel), takes row maxima over 5, 9 and 13 columns
// and then column maxima over 5, 9 and 13 rows, with byte-wise signed max.
__device__ __forceinline__ uint4 vmax16(uint4 a, uint4 b) {
  return make_uint4(__vmaxs4(a.x, b.x), __vmaxs4(a.y, b.y), __vmaxs4(a.z, b.z), __vmaxs4(a.w, b.w));
}

__global__ void __launch_bounds__(256) sppf_pool_i8_kernel(I8View in, I8View o1, I8View o2, I8View o3, int B, int H,
                                                           int W, int C) {
  extern __shared__ uint4 sppf8_smem[];  // [4][H*W]: input, row maxima over 5, 9, 13
  const int HW = H * W;
  uint4* sx = sppf8_smem;
  uint4* s5 = sx + HW;
  uint4* s9 = s5 + HW;
  uint4* s13 = s9 + HW;
  const int groups = C >> 4;
  const int b = blockIdx.x / groups, c = (blockIdx.x - b * groups) * 16;
  pdl_wait();
  for (int p = threadIdx.x; p < HW; p += blockDim.x)
    sx[p] = *reinterpret_cast<const uint4*>(in.p + b * in.bstride + static_cast<long long>(p) * in.cstride + c);
  __syncthreads();
  for (int p = threadIdx.x; p < HW; p += blockDim.x) {
    const int x = p - (p / W) * W;
    uint4 m5 = sx[p], m9 = m5, m13 = m5;
#pragma unroll
    for (int d = 1; d <= 6; ++d) {
      uint4 t = sx[p];
      if (x - d >= 0) t = vmax16(t, sx[p - d]);
      if (x + d < W) t = vmax16(t, sx[p + d]);
      m13 = vmax16(m13, t);
      if (d <= 4) m9 = vmax16(m9, t);
      if (d <= 2) m5 = vmax16(m5, t);
    }
    s5[p] = m5;
    s9[p] = m9;
    s13[p] = m13;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < HW; p += blockDim.x) {
    const int y = p / W;
    uint4 m5 = s5[p], m9 = s9[p], m13 = s13[p];
#pragma unroll
    for (int d = 1; d <= 6; ++d) {
      const bool up = y - d >= 0, dn = y + d < H;
      if (d <= 2) {
        if (up) m5 = vmax16(m5, s5[p - d * W]);
        if (dn) m5 = vmax16(m5, s5[p + d * W]);
      }
      if (d <= 4) {
        if (up) m9 = vmax16(m9, s9[p - d * W]);
        if (dn) m9 = vmax16(m9, s9[p + d * W]);
      }
      if (up) m13 = vmax16(m13, s13[p - d * W]);
      if (dn) m13 = vmax16(m13, s13[p + d * W]);
    }
    *reinterpret_cast<uint4*>(o1.p + b * o1.bstride + static_cast<long long>(p) * o1.cstride + c) = m5;
    *reinterpret_cast<uint4*>(o2.p + b * o2.bstride + static_cast<long long>(p) * o2.cstride + c) = m9;
    *reinterpret_cast<uint4*>(o3.p + b * o3.bstride + static_cast<long long>(p) * o3.cstride + c) = m13;
  }
}

// ------------------------------------------------- upsample and concat
// out[b, y, x, 0:c0] = src0[b, y >> lg0, x >> lg0, :]; out[..., c0:] = src1.
// 16 channels per thread (c0, c1 multiples of 16).
__global__ void concat_i8_kernel(I8View s0, int c0, int lg0, I8View s1, int c1, int B, int H, int W, I8View out) {
  pdl_wait();
  const int C16 = (c0 + c1) >> 4;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(B) * H * W * C16;
  if (idx >= total) return;
  const int c = static_cast<int>(idx % C16) * 16;
  const long long pix = idx / C16;
  const int b = static_cast<int>(pix / (static_cast<long long>(H) * W));
  const int p = static_cast<int>(pix - static_cast<long long>(b) * H * W);
  const int y = p / W, x = p - (p / W) * W;
  const int8_t* src;
  if (c < c0) {
    const int ws = W >> lg0;
    src = s0.p + b * s0.bstride + static_cast<long long>((y >> lg0) * ws + (x >> lg0)) * s0.cstride + c;
  } else {
    src = s1.p + b * s1.bstride + static_cast<long long>(p) * s1.cstride + (c - c0);
  }
  *reinterpret_cast<uint4*>(out.p + b * out.bstride + static_cast<long long>(p) * out.cstride + c) =
      *reinterpret_cast<const uint4*>(src);
}

// ---------------------------------------------------- NHWC -> NCHW dump
__global__ void nhwc_to_nchw_i8_kernel(I8View in, int C, int H, int W, int8_t* out) {
  pdl_wait();
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(C) * H * W;
  if (idx >= total) return;
  const int c = static_cast<int>(idx / (static_cast<long long>(H) * W));
  const long long p = idx - static_cast<long long>(c) * H * W;
  out[idx] = in.p[p * in.cstride + c];
}

}  // namespace

cudaError_t launch_quantize_input(const float* in, int B, int C, int H, int W, float s, I8View out, cudaStream_t st) {
  const long long total = static_cast<long long>(B) * H * W;
  return launch_pdl(quantize_input_kernel, dim3(blocks_for(total, 256)), dim3(256), 0, st, in, B, C, H, W, s, out);
}

cudaError_t launch_maxpool_i8(I8View in, I8View out, int B, int H, int W, int C, int k, cudaStream_t st) {
  if (C % 16 || in.cstride % 16 || out.cstride % 16) return cudaErrorInvalidValue;
  const long long total = static_cast<long long>(B) * H * W * (C / 16);
  return launch_pdl(maxpool_i8_kernel, dim3(blocks_for(total, 256)), dim3(256), 0, st, in, out, B, H, W, C, k);
}

int sppf_pool_i8_smem_bytes(int H, int W) { return 4 * H * W * 16; }

cudaError_t launch_sppf_pool_i8(I8View in, I8View o1, I8View o2, I8View o3, int B, int H, int W, int C,
                                cudaStream_t st) {
  const int smem = sppf_pool_i8_smem_bytes(H, W);
  if (C % 16 || B < 1 || H < 1 || W < 1 || smem > kSppfI8SmemMax) return cudaErrorInvalidValue;
  for (const I8View& v : {in, o1, o2, o3})
    if (v.cstride % 16 || v.bstride % 16 || reinterpret_cast<uintptr_t>(v.p) % 16) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_done{0};
  const cudaError_t e = smem_attr_once(sppf_pool_i8_kernel, kSppfI8SmemMax, attr_done);
  if (e != cudaSuccess) return e;
  return launch_pdl(sppf_pool_i8_kernel, dim3(static_cast<unsigned>(B * (C / 16))), dim3(256), smem, st, in, o1, o2, o3,
                    B, H, W, C);
}

cudaError_t launch_dw3x3_i8(I8View in, I8View out, int B, int H, int W, int C, const uint32_t* wr, const int32_t* bq,
                            const int32_t* mult, const int32_t* shift, const int8_t* lut, cudaStream_t st) {
  if (C % 16 || in.cstride % 16 || out.cstride % 16 || in.bstride % 16 || out.bstride % 16 ||
      reinterpret_cast<uintptr_t>(in.p) % 16 || reinterpret_cast<uintptr_t>(out.p) % 16 ||
      reinterpret_cast<uintptr_t>(wr) % 16)
    return cudaErrorInvalidValue;
  if (B <= 0 || H <= 0 || W <= 0) return cudaSuccess;
  // 32-bit thread indices and per-image byte offsets.
  if (static_cast<long long>(B) * ((H + 3) / 4) * W * (C / 4) + 256 > INT_MAX ||
      static_cast<long long>(H) * W * in.cstride > INT_MAX || static_cast<long long>(H) * W * out.cstride > INT_MAX)
    return cudaErrorInvalidValue;
  if (H >= 40) {
    const long long total = static_cast<long long>(B) * ((H + 7) / 8) * W * (C / 4);
    return launch_pdl(dw3x3_i8_kernel<8>, dim3(blocks_for(total, 256)), dim3(256), 0, st, in, out, B, H, W, C, wr, bq,
                      mult, shift, lut);
  }
  const long long total = static_cast<long long>(B) * ((H + 3) / 4) * W * (C / 4);
  return launch_pdl(dw3x3_i8_kernel<4>, dim3(blocks_for(total, 256)), dim3(256), 0, st, in, out, B, H, W, C, wr, bq,
                    mult, shift, lut);
}

cudaError_t launch_concat_i8(I8View s0, int c0, int lg0, I8View s1, int c1, int B, int H, int W, I8View out,
                             cudaStream_t st) {
  if ((c0 | c1) % 16 || s0.cstride % 16 || (c1 && s1.cstride % 16) || out.cstride % 16) return cudaErrorInvalidValue;
  const long long total = static_cast<long long>(B) * H * W * ((c0 + c1) / 16);
  return launch_pdl(concat_i8_kernel, dim3(blocks_for(total, 256)), dim3(256), 0, st, s0, c0, lg0, s1, c1, B, H, W, out);
}

cudaError_t launch_nhwc_to_nchw_i8(I8View in, int C, int H, int W, int8_t* out, cudaStream_t st) {
  const long long total = static_cast<long long>(C) * H * W;
  nhwc_to_nchw_i8_kernel<<<blocks_for(total, 256), 256, 0, st>>>(in, C, H, W, out);
  return cudaGetLastError();
}

}  // namespace yb
