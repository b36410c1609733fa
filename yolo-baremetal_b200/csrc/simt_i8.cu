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

// ------------------------------------------------------------------ stem
// Tiles of 8 output rows x 16 P columns (P = 64 / CO pixels per thread), as
// the fp32 stem: the fp32 input patch (3 channels x 17 rows x (32 P + 4)
// columns from input column 2 * ox0 - 4) arrives by 16-byte asynchronous
// copies, is quantised into one word per input pixel (channels 0..2 in
// bytes 0..2), and the next tile's copy lands while each output is computed
// as 9 dp4a of such words with the packed weights.  36 KB of shared memory:
// five or six CTAs per SM hide each other's latency.
template <int CO>
struct StemI8Tile {
  static constexpr int P = 64 / CO;
  static constexpr int TW = 16 * P, TH = 8;
  static constexpr int PR = 2 * TH + 1, PC = 2 * TW + 4;
  static constexpr int kBuf = 3 * PR * PC;  // floats per fp32 patch
  static constexpr int kSmem = (kBuf + PR * PC + 9 * CO) * 4 + CO * 16 + CO * 8 + 256;
};

template <int CO>
__device__ __forceinline__ void stem_i8_fetch(const StemI8Args& a, float* sx, int t, int tiles_x, int tiles_y) {
  using T = StemI8Tile<CO>;
  const int b = t / (tiles_x * tiles_y);
  const int rem = t - b * tiles_x * tiles_y;
  const int iy0 = (rem / tiles_x) * T::TH * 2 - 1, ix0 = (rem % tiles_x) * T::TW * 2 - 4;
  const long long plane = static_cast<long long>(a.H) * a.W;
  const float* inb = a.in + static_cast<long long>(b) * 3 * plane;
  if ((a.W & 3) == 0) {
    constexpr int Q = T::PC / 4;
    for (int i = threadIdx.x; i < 3 * T::PR * Q; i += 128) {
      const int row = i / Q;
      const int q = i - row * Q;
      const int c = row / T::PR;
      const int rr = row - c * T::PR;
      const int iy = iy0 + rr, ix = ix0 + 4 * q;
      const int nvalid = (iy >= 0 && iy < a.H && ix >= 0) ? min(4, a.W - ix) : 0;
      const float* src = nvalid > 0 ? inb + c * plane + static_cast<long long>(iy) * a.W + ix : inb;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(static_cast<uint32_t>(
                       __cvta_generic_to_shared(sx + (c * T::PR + rr) * T::PC + 4 * q))),
                   "l"(src), "r"(nvalid > 0 ? 4 * nvalid : 0)
                   : "memory");
    }
  } else {
    for (int i = threadIdx.x; i < 3 * T::PR * T::PC; i += 128) {
      const int c = i / (T::PR * T::PC);
      const int rr = (i / T::PC) % T::PR;
      const int cc = i % T::PC;
      const int iy = iy0 + rr, ix = ix0 + cc;
      const bool ok = iy >= 0 && iy < a.H && ix >= 0 && ix < a.W;
      const float* src = ok ? inb + c * plane + static_cast<long long>(iy) * a.W + ix : inb;
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(static_cast<uint32_t>(
                       __cvta_generic_to_shared(sx + (c * T::PR + rr) * T::PC + cc))),
                   "l"(src), "r"(ok ? 4 : 0)
                   : "memory");
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// clamp(rint(v / s), -127, 127) as a byte, v / s correctly rounded.  With
// r = fl(1 / s), y = fl(v * r) lies within 2^-15 of fl(v / s) for |y| <= 200,
// so when y is further than 2^-12 from a half-integer both round to the same
// integer, read from the mantissa of y + 1.5 * 2^23 (round half to even,
// like rintf).  Otherwise (near a rounding boundary, large, or NaN) the exact
// quotient is used.
__device__ __forceinline__ uint32_t quant_byte(float v, float s, float r) {
  const float y = __fmul_rn(v, r);
  const float m = __fadd_rn(y, 12582912.0f);
  const float d = __fsub_rn(y, __fsub_rn(m, 12582912.0f));
  int q;
  if (fabsf(y) <= 200.f && fabsf(d) < 0.49975586f) {
    q = __float_as_int(m) - 0x4B400000;
  } else {
    const float e = rintf(__fdiv_rn(v, s));
    q = static_cast<int>(e < -127.f ? -127.f : e > 127.f ? 127.f : e);
  }
  return static_cast<uint32_t>(min(max(q, -127), 127)) & 0xFFu;
}

template <int CO>
__global__ void __launch_bounds__(128) stem_i8_kernel(const StemI8Args a) {
  using T = StemI8Tile<CO>;
  constexpr int P = T::P;
  extern __shared__ __align__(16) float stem_i8_smem[];
  float* sxb = stem_i8_smem;
  uint32_t* sq = reinterpret_cast<uint32_t*>(stem_i8_smem + T::kBuf);  // [PR][PC] packed int8 pixels
  uint32_t* sw = sq + T::PR * T::PC;                                      // [9][CO]
  int4* sp = reinterpret_cast<int4*>(sw + 9 * CO);                        // {M, D lo, D hi, shift - 32}
  int2* sx2 = reinterpret_cast<int2*>(sp + CO);                           // {bias, shift}
  int8_t* slut = reinterpret_cast<int8_t*>(sx2 + CO);
  const int tid = threadIdx.x;
  for (int i = tid; i < 9 * CO; i += 128) sw[i] = a.w[i];
  for (int i = tid; i < CO; i += 128) {
    const int m = a.mult[i], b = a.bias[i];
    const int sh = m == 0 ? 32 : a.shift[i];
    const long long d = static_cast<long long>(b) * m + ((1LL << (sh - 1)) - 1);
    sp[i] = make_int4(m, static_cast<int>(static_cast<unsigned long long>(d) & 0xFFFFFFFFull),
                      static_cast<int>(d >> 32), sh - 32);
    sx2[i] = make_int2(b, sh);
  }
  for (int i = tid; i < 256; i += 128) slut[i] = a.lut[i];
  pdl_wait();
  const int tiles_x = (a.Wo + T::TW - 1) / T::TW, tiles_y = (a.Ho + T::TH - 1) / T::TH;
  const int total = a.B * tiles_x * tiles_y;
  const int r = tid >> 4, x0 = tid & 15;
  const float rcp = __frcp_rn(a.s_in);
  // One fp32 staging buffer: once a tile is quantised, the next tile's copy
  // goes into it and lands while this tile computes.
  if (static_cast<int>(blockIdx.x) < total) {
    stem_i8_fetch<CO>(a, sxb, blockIdx.x, tiles_x, tiles_y);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
  }
  __syncthreads();
  for (int t = blockIdx.x; t < total; t += gridDim.x) {
    const int tn = t + gridDim.x;
    for (int i = tid; i < T::PR * T::PC; i += 128)
      sq[i] = quant_byte(sxb[i], a.s_in, rcp) | (quant_byte(sxb[T::PR * T::PC + i], a.s_in, rcp) << 8) |
              (quant_byte(sxb[2 * T::PR * T::PC + i], a.s_in, rcp) << 16);
    __syncthreads();
    if (tn < total) stem_i8_fetch<CO>(a, sxb, tn, tiles_x, tiles_y);
    int acc[P][CO];
#pragma unroll
    for (int j = 0; j < P; ++j)
#pragma unroll
      for (int c = 0; c < CO; ++c) acc[j][c] = 0;
#pragma unroll
    for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        int xv[P];
#pragma unroll
        for (int j = 0; j < P; ++j) xv[j] = static_cast<int>(sq[(2 * r + ky) * T::PC + 2 * (x0 + 16 * j) + kx + 3]);
        const uint32_t* wr = sw + (ky * 3 + kx) * CO;
#pragma unroll
        for (int c = 0; c < CO; c += 4) {
          const uint4 w = *reinterpret_cast<const uint4*>(wr + c);
#pragma unroll
          for (int j = 0; j < P; ++j) {
            acc[j][c + 0] = __dp4a(xv[j], static_cast<int>(w.x), acc[j][c + 0]);
            acc[j][c + 1] = __dp4a(xv[j], static_cast<int>(w.y), acc[j][c + 1]);
            acc[j][c + 2] = __dp4a(xv[j], static_cast<int>(w.z), acc[j][c + 2]);
            acc[j][c + 3] = __dp4a(xv[j], static_cast<int>(w.w), acc[j][c + 3]);
          }
        }
      }
    }
    const int b = t / (tiles_x * tiles_y);
    const int rem = t - b * tiles_x * tiles_y;
    const int oy = (rem / tiles_x) * T::TH + r;
    // Requantise: acc * M + (bias * M + 2^(sh-1) - 1) >> sh for every
    // channel (branch-free), exact unless a shift is below 32 or a low word
    // is all ones (a possible tie); then the thread redoes its pixels in 64
    // bits.
    bool exact = false;
#pragma unroll
    for (int c = 0; c < CO; ++c) {
      const int4 q = sp[c];
      const long long d = (static_cast<long long>(q.z) << 32) | static_cast<unsigned>(q.y);
#pragma unroll
      for (int j = 0; j < P; ++j) {
        const long long pr = static_cast<long long>(acc[j][c]) * q.x + d;
        exact |= (q.w < 0) | (static_cast<unsigned>(pr) == 0xFFFFFFFFu);
        const int y = static_cast<int>(pr >> 32) >> (q.w & 31);
        acc[j][c] = slut[min(max(y, -128), 127) + 128];
      }
    }
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const int ox = (rem % tiles_x) * T::TW + x0 + 16 * j;
      if (oy >= a.Ho || ox >= a.Wo) continue;
      int8_t* o = a.out.p + static_cast<long long>(b) * a.out.bstride +
                  (static_cast<long long>(oy) * a.Wo + ox) * a.out.cstride;
#pragma unroll
      for (int c = 0; c < CO; c += 16) {
        uint32_t wv[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int* ov = &acc[j][c + 4 * g];
          wv[g] = __byte_perm(__byte_perm(ov[0], ov[1], 0x0040), __byte_perm(ov[2], ov[3], 0x0040), 0x5410);
        }
        *reinterpret_cast<uint4*>(o + c) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      }
    }
    if (exact) {
      // Rare: redo this thread's outputs in 64 bits and overwrite them.
      for (int j = 0; j < P; ++j) {
        const int ox = (rem % tiles_x) * T::TW + x0 + 16 * j;
        if (oy >= a.Ho || ox >= a.Wo) continue;
        int8_t* o = a.out.p + static_cast<long long>(b) * a.out.bstride +
                    (static_cast<long long>(oy) * a.Wo + ox) * a.out.cstride;
        for (int c = 0; c < CO; ++c) {
          int raw = 0;
          for (int tap = 0; tap < 9; ++tap)
            raw = __dp4a(static_cast<int>(sq[(2 * r + tap / 3) * T::PC + 2 * (x0 + 16 * j) + tap % 3 + 3]),
                         static_cast<int>(sw[tap * CO + c]), raw);
          const int2 bs = sx2[c];
          const long long y = rne((static_cast<long long>(raw) + bs.x) * sp[c].x, bs.y);
          o[c] = slut[(y < -128 ? -128 : y > 127 ? 127 : y) + 128];
        }
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // the next tile has landed; the patch is rewritten next iteration
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

cudaError_t init_stem_i8_attributes() {
  cudaError_t e = cudaFuncSetAttribute(stem_i8_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       StemI8Tile<16>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(stem_i8_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, StemI8Tile<32>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(stem_i8_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, StemI8Tile<64>::kSmem);
  return e;
}

cudaError_t launch_stem_i8(const StemI8Args& a, cudaStream_t st) {
  if ((a.Co != 16 && a.Co != 32 && a.Co != 64) || a.Ho != (a.H - 1) / 2 + 1 || a.Wo != (a.W - 1) / 2 + 1 ||
      a.out.cstride < a.Co || a.out.cstride % 16 || reinterpret_cast<uintptr_t>(a.out.p) % 16 || !a.lut ||
      !(a.s_in > 0.f))
    return cudaErrorInvalidValue;
  const int tw = 16 * (64 / a.Co);
  const long long tiles = static_cast<long long>(a.B) * ((a.Ho + 7) / 8) * ((a.Wo + tw - 1) / tw);
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidValue;
  if (tiles == 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned grid = static_cast<unsigned>(tiles < 6LL * sms ? tiles : 6LL * sms);
  if (a.Co == 16) return launch_pdl(stem_i8_kernel<16>, dim3(grid), dim3(128), StemI8Tile<16>::kSmem, st, a);
  if (a.Co == 32) return launch_pdl(stem_i8_kernel<32>, dim3(grid), dim3(128), StemI8Tile<32>::kSmem, st, a);
  return launch_pdl(stem_i8_kernel<64>, dim3(grid), dim3(128), StemI8Tile<64>::kSmem, st, a);
}

}  // namespace yb
