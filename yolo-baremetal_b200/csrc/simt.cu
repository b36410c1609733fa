// CUDA-core kernels of the YOLO26 path: the ops that are not contractions
// (depthwise, pooling, decode, layout) or too small to tile (the 3-channel stem
// convolution).  All are HBM- or latency-bound; they
// read and write split NHWC views (kernels.h) 8 channels (two 16-byte
// accesses) at a time.  Summation orders follow the reference loops so that
// results stay within a few ulps of it.
#include <atomic>
#include <cfloat>
#include <climits>
#include "pdl.cuh"
#include "kernels.h"
#include "split.cuh"

namespace yb {
namespace {

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

inline int blocks_for(long long n, int t) { return static_cast<int>((n + t - 1) / t); }

template <typename V>
__device__ __forceinline__ long long vaddr(const V& v, int b, long long p) {
  return static_cast<long long>(b) * v.bstride + p * v.cstride + v.coff;
}

// ------------------------------------------------------------------ stem conv
// Direct 3x3 stride-2 pad-1 convolution of the NCHW fp32 input (Ci <= 4),
// + bias + SiLU, into the split NHWC stage-0 buffer (layers.c:41-81 for the
// arithmetic, here with fused multiply-add).  Persistent CTAs of 128 threads
// walk tiles of 8 output rows x (16 * P) columns.  A tile's 17 x (32 P + 1)
// input patch (every channel) is fetched with 4-byte asynchronous copies
// into one of two shared buffers while the previous tile computes; thread
// (r, x) computes the P pixels x, x + 16, ... of row r for all CO channels,
// so a half-warp's stores cover 16 consecutive pixels.
template <int CO>
struct StemTile {
  static constexpr int P = 64 / CO;  // pixels per thread
  static constexpr int TW = 16 * P, TH = 8;
  // Patch columns start at input column 2 * ox0 - 4 (16-byte aligned when W
  // is a multiple of 4); the conv reads columns 3 .. 2 TW + 3 of it.
  static constexpr int PR = 2 * TH + 1, PC = 2 * TW + 4, PCS = PC;
  static constexpr int kBuf = 4 * PR * PCS;  // floats per patch buffer (Ci <= 4)
  static constexpr int kSmem = (2 * kBuf + 4 * 9 * CO + CO) * 4;
};

template <int CO>
__device__ __forceinline__ void stem_fetch(const StemArgs& a, float* sx, int t, int tiles_x, int tiles_y) {
  using T = StemTile<CO>;
  const int b = t / (tiles_x * tiles_y);
  const int rem = t - b * tiles_x * tiles_y;
  const int iy0 = (rem / tiles_x) * T::TH * 2 - 1, ix0 = (rem % tiles_x) * T::TW * 2 - 4;
  const long long plane = static_cast<long long>(a.H) * a.W;
  const float* inb = a.in + static_cast<long long>(b) * a.Ci * plane;
  if ((a.W & 3) == 0) {
    // 16-byte copies of 4 columns; partial or outside chunks zero-filled.
    constexpr int Q = T::PC / 4;
    for (int i = threadIdx.x; i < a.Ci * T::PR * Q; i += 128) {
      const int row = i / Q;
      const int q = i - row * Q;
      const int c = row / T::PR;
      const int rr = row - c * T::PR;
      const int iy = iy0 + rr, ix = ix0 + 4 * q;
      const int nvalid = (iy >= 0 && iy < a.H && ix >= 0) ? min(4, a.W - ix) : 0;
      const float* src = nvalid > 0 ? inb + c * plane + static_cast<long long>(iy) * a.W + ix : inb;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(static_cast<uint32_t>(
                       __cvta_generic_to_shared(sx + (c * T::PR + rr) * T::PCS + 4 * q))),
                   "l"(src), "r"(nvalid > 0 ? 4 * nvalid : 0)
                   : "memory");
    }
  } else {
    for (int i = threadIdx.x; i < a.Ci * T::PR * T::PC; i += 128) {
      const int c = i / (T::PR * T::PC);
      const int rr = (i / T::PC) % T::PR;
      const int cc = i % T::PC;
      const int iy = iy0 + rr, ix = ix0 + cc;
      const bool ok = iy >= 0 && iy < a.H && ix >= 0 && ix < a.W;
      const float* src = ok ? inb + c * plane + static_cast<long long>(iy) * a.W + ix : inb;
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(static_cast<uint32_t>(
                       __cvta_generic_to_shared(sx + (c * T::PR + rr) * T::PCS + cc))),
                   "l"(src), "r"(ok ? 4 : 0)
                   : "memory");
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Calibration statistics: one atomicMax per converged lane group.
__device__ __forceinline__ void amax_warp(unsigned* amax, float mpre, float mout) {
  const unsigned am = __activemask();
  const unsigned wp = __reduce_max_sync(am, __float_as_uint(mpre));
  const unsigned wo = __reduce_max_sync(am, __float_as_uint(mout));
  if ((threadIdx.x & 31) == static_cast<unsigned>(__ffs(am) - 1)) {
    atomicMax(amax, wp);
    atomicMax(amax + 1, wo);
  }
}

template <int CO>
__global__ void __launch_bounds__(128) stem_kernel(const StemArgs a) {
  using T = StemTile<CO>;
  constexpr int P = T::P;
  extern __shared__ __align__(16) float stem_smem[];
  float* sxb = stem_smem;                      // two patch buffers
  float* sw = stem_smem + 2 * T::kBuf;         // [ci*9 + tap][co]
  float* sb = sw + 4 * 9 * CO;
  const int tid = threadIdx.x;
  const int taps = a.Ci * 9;
  for (int i = tid; i < CO * taps; i += 128) sw[(i % taps) * CO + i / taps] = a.w[i];
  for (int i = tid; i < CO; i += 128) sb[i] = a.bias ? a.bias[i] : 0.f;
  pdl_wait();
  const int tiles_x = (a.Wo + T::TW - 1) / T::TW, tiles_y = (a.Ho + T::TH - 1) / T::TH;
  const int total = a.B * tiles_x * tiles_y;
  const int r = tid >> 4, x0 = tid & 15;
  float mpre = 0.0f, mout = 0.0f;  // calibration statistics (a.amax)
  int k = 0;
  if (static_cast<int>(blockIdx.x) < total) stem_fetch<CO>(a, sxb, blockIdx.x, tiles_x, tiles_y);
  for (int t = blockIdx.x; t < total; t += gridDim.x, ++k) {
    const int tn = t + gridDim.x;
    if (tn < total) stem_fetch<CO>(a, sxb + ((k + 1) & 1) * T::kBuf, tn, tiles_x, tiles_y);
    if (tn < total) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    const float* sx = sxb + (k & 1) * T::kBuf;
    float acc[P][CO];
#pragma unroll
    for (int j = 0; j < P; ++j)
#pragma unroll
      for (int c = 0; c < CO; ++c) acc[j][c] = sb[c];
    for (int ci = 0; ci < a.Ci; ++ci) {
#pragma unroll
      for (int ky = 0; ky < 3; ++ky) {
        const float* row = sx + (ci * T::PR + 2 * r + ky) * T::PCS;
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
          float xv[P];
#pragma unroll
          for (int j = 0; j < P; ++j) xv[j] = row[2 * (x0 + 16 * j) + kx + 3];
          const float* wr = sw + (ci * 9 + ky * 3 + kx) * CO;
#pragma unroll
          for (int c = 0; c < CO; c += 4) {
            const float4 w = *reinterpret_cast<const float4*>(wr + c);
#pragma unroll
            for (int j = 0; j < P; ++j) {
              acc[j][c + 0] = fmaf(xv[j], w.x, acc[j][c + 0]);
              acc[j][c + 1] = fmaf(xv[j], w.y, acc[j][c + 1]);
              acc[j][c + 2] = fmaf(xv[j], w.z, acc[j][c + 2]);
              acc[j][c + 3] = fmaf(xv[j], w.w, acc[j][c + 3]);
            }
          }
        }
      }
    }
    const int b = t / (tiles_x * tiles_y);
    const int rem = t - b * tiles_x * tiles_y;
    const int oy = (rem / tiles_x) * T::TH + r;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const int ox = (rem % tiles_x) * T::TW + x0 + 16 * j;
      if (oy >= a.Ho || ox >= a.Wo) continue;
      uint16_t* o = a.out.hi + vaddr(a.out, b, static_cast<long long>(oy) * a.Wo + ox);
#pragma unroll
      for (int c = 0; c < CO; c += 8) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = a.act == kActSiLU ? silu_fast(acc[j][c + e]) : acc[j][c + e];
        if (a.amax) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            mpre = fmaxf(mpre, fabsf(acc[j][c + e]));
            mout = fmaxf(mout, fabsf(v[e]));
          }
        }
        store8(o + c, a.out.plane, v);
      }
    }
    __syncthreads();  // this buffer is refilled by the next iteration's prefetch
  }
  if (a.amax) amax_warp(a.amax, mpre, mout);
}

// ------------------------------------------------------------- depthwise 3x3
// w is [9][C] (tap-major, transposed on the host).  A thread computes 2
// channels of R consecutive output rows of one column: the 3 x 3 window
// slides down the strip, so each input row (three pixels, hi and lo planes)
// is loaded once and serves three outputs; weights and bias stay in
// registers, and all loads of the strip are in flight together.
// Out-of-image taps are skipped, not added as zeros: the sum is the
// reference's (bias, then the taps in (ky, kx) order, every product and sum
// rounded on its own).
template <int R>
__global__ void __launch_bounds__(256, 2) dw3x3_kernel(const DwArgs a) {
  // 32-bit indexing: the launcher checks that threads and per-image offsets fit.
  const int C2 = a.C >> 1;
  const int strips = (a.H + R - 1) / R;
  const int idx = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= a.B * strips * a.W * C2) return;
  const int c = (idx % C2) * 2;
  int r = idx / C2;
  const int x = r % a.W;
  r /= a.W;
  const int strip = r % strips;
  const int b = r / strips;
  float wk[9][2], bias[2] = {0.f, 0.f};
#pragma unroll
  for (int t = 0; t < 9; ++t) {
    const float2 w2 = __ldg(reinterpret_cast<const float2*>(a.w + t * a.C + c));
    wk[t][0] = w2.x;
    wk[t][1] = w2.y;
  }
  if (a.bias) {
    const float2 b2 = __ldg(reinterpret_cast<const float2*>(a.bias + c));
    bias[0] = b2.x;
    bias[1] = b2.y;
  }
  pdl_wait();
  const bool cl = x > 0, cr = x < a.W - 1;
  const uint16_t* base = a.in.hi + vaddr(a.in, b, 0) + c;
  const int y0 = strip * R;
  // Every load of the strip (R + 2 rows x 3 pixels, both planes) is issued
  // before the first sum; each value is joined (hi + lo) once.
  uint32_t rh[R + 2][3], rl[R + 2][3];
#pragma unroll
  for (int k = 0; k < R + 2; ++k) {
    const int iy = y0 - 1 + k;
    const bool ok = iy >= 0 && iy < a.H;
    const uint16_t* p = base + (iy * a.W + x - 1) * a.in.cstride;
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      const bool in = ok && (kx == 0 ? cl : kx == 2 ? cr : true);
      rh[k][kx] = in ? __ldg(reinterpret_cast<const uint32_t*>(p + kx * a.in.cstride)) : 0u;
      rl[k][kx] = in ? __ldg(reinterpret_cast<const uint32_t*>(p + kx * a.in.cstride + a.in.plane)) : 0u;
    }
  }
  float v[R + 2][3][2];
#pragma unroll
  for (int k = 0; k < R + 2; ++k) {
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      v[k][kx][0] = bf16_bits_to_f(rh[k][kx] & 0xFFFFu) + bf16_bits_to_f(rl[k][kx] & 0xFFFFu);
      v[k][kx][1] = bf16_bits_to_f(rh[k][kx] >> 16) + bf16_bits_to_f(rl[k][kx] >> 16);
    }
  }
  float mpre = 0.0f, mout = 0.0f;
  uint16_t* ob = a.out.hi + vaddr(a.out, b, 0) + c;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int y = y0 + i;
    if (y >= a.H) break;
    const bool rok[3] = {y > 0, true, y < a.H - 1};
    float s[2] = {bias[0], bias[1]};
#pragma unroll
    for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        const bool ok = rok[ky] && (kx == 0 ? cl : kx == 2 ? cr : true);
        const float p0 = __fmul_rn(v[i + ky][kx][0], wk[ky * 3 + kx][0]);
        const float p1 = __fmul_rn(v[i + ky][kx][1], wk[ky * 3 + kx][1]);
        if (ok) {
          s[0] = __fadd_rn(s[0], p0);
          s[1] = __fadd_rn(s[1], p1);
        }
      }
    }
    if (a.amax) mpre = fmaxf(mpre, fmaxf(fabsf(s[0]), fabsf(s[1])));
    if (a.act == kActSiLU) {
      s[0] = silu_fast(s[0]);
      s[1] = silu_fast(s[1]);
    }
    uint32_t hw, lw;
    split2(s[0], s[1], hw, lw);
    uint16_t* o = ob + (y * a.W + x) * a.out.cstride;
    *reinterpret_cast<uint32_t*>(o) = hw;
    *reinterpret_cast<uint32_t*>(o + a.out.plane) = lw;
    if (a.amax) mout = fmaxf(mout, fmaxf(fabsf(s[0]), fabsf(s[1])));
  }
  if (a.amax) amax_warp(a.amax, mpre, mout);
}

// Four channels per thread (8-byte loads and stores per plane) over a strip
// of R output rows at one column, with a rolling window of three joined
// input rows: each input row of the strip is loaded and joined (hi + lo)
// once, the next row's loads are in flight while the current output row is
// summed, and every tap is one fused multiply-add (out-of-image taps read
// zeros).  About a third of the instructions per output of the two-channel
// form, which was issue-bound.
template <int R>
__global__ void __launch_bounds__(256, 2) dw3x3_c4_kernel(const DwArgs a) {
  // 32-bit indexing: the launcher checks that threads and per-image offsets fit.
  const int C4 = a.C >> 2;
  const int strips = (a.H + R - 1) / R;
  const int idx = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= a.B * strips * a.W * C4) return;
  const int c = (idx % C4) * 4;
  int r = idx / C4;
  const int x = r % a.W;
  r /= a.W;
  const int strip = r % strips;
  const int b = r / strips;
  float wk[9][4], bias[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int t = 0; t < 9; ++t) {
    const float4 w4 = __ldg(reinterpret_cast<const float4*>(a.w + t * a.C + c));
    wk[t][0] = w4.x;
    wk[t][1] = w4.y;
    wk[t][2] = w4.z;
    wk[t][3] = w4.w;
  }
  if (a.bias) {
    const float4 b4 = __ldg(reinterpret_cast<const float4*>(a.bias + c));
    bias[0] = b4.x;
    bias[1] = b4.y;
    bias[2] = b4.z;
    bias[3] = b4.w;
  }
  pdl_wait();
  const bool cl = x > 0, cr = x < a.W - 1;
  const uint16_t* base = a.in.hi + vaddr(a.in, b, 0) + c;
  const int y0 = strip * R;
  // Raw words of input row iy (pixels x - 1, x, x + 1; zeros outside).
  auto fetch = [&](int iy, uint2 (&h)[3], uint2 (&l)[3]) {
    const bool ok = iy >= 0 && iy < a.H;
    const uint16_t* p = base + (iy * a.W + x - 1) * a.in.cstride;
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      const bool in = ok && (kx == 0 ? cl : kx == 2 ? cr : true);
      h[kx] = in ? __ldg(reinterpret_cast<const uint2*>(p + kx * a.in.cstride)) : make_uint2(0u, 0u);
      l[kx] = in ? __ldg(reinterpret_cast<const uint2*>(p + kx * a.in.cstride + a.in.plane)) : make_uint2(0u, 0u);
    }
  };
  auto join = [&](const uint2 (&h)[3], const uint2 (&l)[3], float (&v)[3][4]) {
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      const float2 s0 =
          __fadd2_rn(make_float2(bf16_bits_to_f(h[kx].x & 0xFFFFu), __uint_as_float(h[kx].x & 0xFFFF0000u)),
                     make_float2(bf16_bits_to_f(l[kx].x & 0xFFFFu), __uint_as_float(l[kx].x & 0xFFFF0000u)));
      const float2 s1 =
          __fadd2_rn(make_float2(bf16_bits_to_f(h[kx].y & 0xFFFFu), __uint_as_float(h[kx].y & 0xFFFF0000u)),
                     make_float2(bf16_bits_to_f(l[kx].y & 0xFFFFu), __uint_as_float(l[kx].y & 0xFFFF0000u)));
      v[kx][0] = s0.x;
      v[kx][1] = s0.y;
      v[kx][2] = s1.x;
      v[kx][3] = s1.y;
    }
  };
  float win[3][3][4];  // input rows y - 1, y, y + 1 of output row y, slot (row - y0 + 1) % 3
  {
    uint2 h[3], l[3];
    fetch(y0 - 1, h, l);
    join(h, l, win[0]);
    fetch(y0, h, l);
    join(h, l, win[1]);
  }
  uint2 nh[3], nl[3];
  fetch(y0 + 1, nh, nl);
  float mpre = 0.0f, mout = 0.0f;
  uint16_t* ob = a.out.hi + vaddr(a.out, b, 0) + c;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int y = y0 + i;
    if (y >= a.H) break;
    join(nh, nl, win[(i + 2) % 3]);
    if (i + 1 < R) fetch(y + 2, nh, nl);
    float sum[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) sum[e] = bias[e];
#pragma unroll
    for (int ky = 0; ky < 3; ++ky)
#pragma unroll
      for (int kx = 0; kx < 3; ++kx)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const float* wv = win[(i + ky) % 3][kx];
          const float2 f = __ffma2_rn(make_float2(wv[e], wv[e + 1]),
                                      make_float2(wk[ky * 3 + kx][e], wk[ky * 3 + kx][e + 1]),
                                      make_float2(sum[e], sum[e + 1]));
          sum[e] = f.x;
          sum[e + 1] = f.y;
        }
    if (a.amax) mpre = fmaxf(mpre, fmaxf(fmaxf(fabsf(sum[0]), fabsf(sum[1])), fmaxf(fabsf(sum[2]), fabsf(sum[3]))));
    if (a.act == kActSiLU) silu_fast_n<4>(sum);
    uint32_t hw0, lw0, hw1, lw1;
    split2(sum[0], sum[1], hw0, lw0);
    split2(sum[2], sum[3], hw1, lw1);
    uint16_t* o = ob + (y * a.W + x) * a.out.cstride;
    *reinterpret_cast<uint2*>(o) = make_uint2(hw0, hw1);
    *reinterpret_cast<uint2*>(o + a.out.plane) = make_uint2(lw0, lw1);
    if (a.amax) mout = fmaxf(mout, fmaxf(fmaxf(fabsf(sum[0]), fabsf(sum[1])), fmaxf(fabsf(sum[2]), fabsf(sum[3]))));
  }
  if (a.amax) amax_warp(a.amax, mpre, mout);
}

// ------------------------------------------------------------- SPPF pools
// SPPF's three chained 5x5 stride-1 max pools (layers.c:230-265) in one
// launch.  With out-of-image positions excluded, pooling twice is the 9x9
// pool and three times the 13x13 pool (each in-image position of the larger
// window is reached through an in-image intermediate), and the joined
// (hi + lo) maxima are the same values.  One CTA per (image, 8 channels)
// loads the image into shared memory, takes the row maxima over 5, 9 and 13
// columns, then the column maxima over 5, 9 and 13 rows.
__global__ void __launch_bounds__(256) sppf_pool_kernel(SView in, SOut o1, SOut o2, SOut o3, int B, int H, int W,
                                                        int C) {
  extern __shared__ float4 sppf_smem[];  // [4][H*W][2]: input, row maxima over 5, 9, 13
  const int HW = H * W;
  float4* sx = sppf_smem;
  float4* s5 = sx + 2 * HW;
  float4* s9 = s5 + 2 * HW;
  float4* s13 = s9 + 2 * HW;
  const int groups = C >> 3;
  const int b = blockIdx.x / groups, c = (blockIdx.x - b * groups) * 8;
  pdl_wait();
  for (int p = threadIdx.x; p < HW; p += blockDim.x) {
    float v[8];
    load8_rw(in.hi + vaddr(in, b, p) + c, in.plane, v);
    sx[2 * p] = make_float4(v[0], v[1], v[2], v[3]);
    sx[2 * p + 1] = make_float4(v[4], v[5], v[6], v[7]);
  }
  __syncthreads();
  const auto mx4 = [](float4 a, float4 b) {
    return make_float4(fmaxf(a.x, b.x), fmaxf(a.y, b.y), fmaxf(a.z, b.z), fmaxf(a.w, b.w));
  };
  for (int p = threadIdx.x; p < HW; p += blockDim.x) {
    const int x = p - (p / W) * W;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float4 m5 = sx[2 * p + h], m9 = m5, m13 = m5;
#pragma unroll
      for (int d = 1; d <= 6; ++d) {
        float4 t = make_float4(-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX);
        if (x - d >= 0) t = sx[2 * (p - d) + h];
        if (x + d < W) t = mx4(t, sx[2 * (p + d) + h]);
        m13 = mx4(m13, t);
        if (d <= 4) m9 = mx4(m9, t);
        if (d <= 2) m5 = mx4(m5, t);
      }
      s5[2 * p + h] = m5;
      s9[2 * p + h] = m9;
      s13[2 * p + h] = m13;
    }
  }
  __syncthreads();
  for (int p = threadIdx.x; p < HW; p += blockDim.x) {
    const int y = p / W;
    float o[3][8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float4 m5 = s5[2 * p + h], m9 = s9[2 * p + h], m13 = s13[2 * p + h];
#pragma unroll
      for (int d = 1; d <= 6; ++d) {
        const bool up = y - d >= 0, dn = y + d < H;
        if (d <= 2) {
          if (up) m5 = mx4(m5, s5[2 * (p - d * W) + h]);
          if (dn) m5 = mx4(m5, s5[2 * (p + d * W) + h]);
        }
        if (d <= 4) {
          if (up) m9 = mx4(m9, s9[2 * (p - d * W) + h]);
          if (dn) m9 = mx4(m9, s9[2 * (p + d * W) + h]);
        }
        if (up) m13 = mx4(m13, s13[2 * (p - d * W) + h]);
        if (dn) m13 = mx4(m13, s13[2 * (p + d * W) + h]);
      }
      const float4 r[3] = {m5, m9, m13};
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        o[k][4 * h + 0] = r[k].x;
        o[k][4 * h + 1] = r[k].y;
        o[k][4 * h + 2] = r[k].z;
        o[k][4 * h + 3] = r[k].w;
      }
    }
    store8(o1.hi + vaddr(o1, b, p) + c, o1.plane, o[0]);
    store8(o2.hi + vaddr(o2, b, p) + c, o2.plane, o[1]);
    store8(o3.hi + vaddr(o3, b, p) + c, o3.plane, o[2]);
  }
}

// ------------------------------------------------------------- calibration
__global__ void absmax_split_kernel(SView v, int B, int H, int W, int C, unsigned* amax) {
  pdl_wait();
  const long long total = static_cast<long long>(B) * H * W * C;
  float m = 0.0f;
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % C);
    const long long pix = idx / C;
    const int b = static_cast<int>(pix / (static_cast<long long>(H) * W));
    const long long p = pix - static_cast<long long>(b) * H * W;
    const long long o = vaddr(v, b, p) + c;
    m = fmaxf(m, fabsf(join1(v.hi[o], v.hi[o + v.plane])));
  }
  amax_warp(amax, 0.0f, m);
}

__global__ void absmax_f32_kernel(const float* x, long long n, unsigned* amax) {
  pdl_wait();
  float m = 0.0f;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(x[i]));
  amax_warp(amax, 0.0f, m);
}

// ------------------------------------------------------------------ max pool
__global__ void maxpool_kernel(const PoolArgs a) {
  pdl_wait();
  const int C8 = a.C >> 3;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(a.B) * a.Ho * a.Wo * C8;
  if (idx >= total) return;
  const int c = static_cast<int>(idx % C8) * 8;
  const long long pix = idx / C8;
  const int b = static_cast<int>(pix / (a.Ho * a.Wo));
  const int p = static_cast<int>(pix - static_cast<long long>(b) * a.Ho * a.Wo);
  const int y = (p / a.Wo) * a.stride, x = (p - (p / a.Wo) * a.Wo) * a.stride;
  const int pad = a.k / 2;
  float m[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) m[e] = -FLT_MAX;
  const uint16_t* base = a.in.hi + vaddr(a.in, b, 0) + c;
  for (int ky = 0; ky < a.k; ++ky) {
    const int iy = y - pad + ky;
    if (iy < 0 || iy >= a.H) continue;
    for (int kx = 0; kx < a.k; ++kx) {
      const int ix = x - pad + kx;
      if (ix < 0 || ix >= a.W) continue;
      float v[8];
      load8_rw(base + static_cast<long long>(iy * a.W + ix) * a.in.cstride, a.in.plane, v);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (v[e] > m[e]) m[e] = v[e];
    }
  }
  store8(a.out.hi + vaddr(a.out, b, p) + c, a.out.plane, m);
}

// -------------------------------------------------------------------- decode
// Four threads per anchor: the anchor's nc logits are read as float4 by the
// four lanes in turn (a warp covers 8 consecutive anchors, 2.5 KB of
// contiguous logits for nc = 80), reduced to the maximum logit with two
// shuffles.  The maximum score is sigmoid(max logit): the reference takes the
// maximum of the per-class sigmoids, which sigmoid's monotonicity makes the
// same value up to the rounding of expf.  It only orders the anchors for the
// top-k, which recomputes the chosen scores per class.  Lane 0 of the four
// decodes the box.
__global__ void decode_kernel(const DecodeArgs a) {
  pdl_wait();
  const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long idx = t >> 2;
  const int sub = static_cast<int>(t & 3);
  const long long total = static_cast<long long>(a.B) * a.N;
  const bool ok = idx < total;
  float m = -FLT_MAX;
  if (ok && !a.max_ready) {
    const float* lg = a.logits + idx * a.nc;
    if ((a.nc & 3) == 0) {
      const int n4 = a.nc >> 2;
      for (int c4 = sub; c4 < n4; c4 += 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(lg) + c4);
        m = fmaxf(fmaxf(m, v.x), fmaxf(v.y, fmaxf(v.z, v.w)));
      }
    } else {
      for (int c = sub; c < a.nc; c += 4) m = fmaxf(m, __ldg(lg + c));
    }
  }
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  if (!ok || sub != 0) return;
  if (!a.max_ready) a.maxscore[idx] = sigmoid(m);
  const int j = static_cast<int>(idx % a.N);
  int s = 0;
  while (s + 1 < a.nscales && j >= a.base[s + 1]) ++s;
  const int local = j - a.base[s];
  const int gy = local / a.w[s], gx = local - (local / a.w[s]) * a.w[s];
  const float ax = static_cast<float>(gx) + 0.5f;
  const float ay = static_cast<float>(gy) + 0.5f;
  const float st = static_cast<float>(a.stride[s]);
  const float4 d = __ldg(reinterpret_cast<const float4*>(a.dist + idx * 4));
  float4 bx;
  bx.x = __fmul_rn(__fsub_rn(ax, d.x), st);
  bx.y = __fmul_rn(__fsub_rn(ay, d.y), st);
  bx.z = __fmul_rn(__fadd_rn(ax, d.z), st);
  bx.w = __fmul_rn(__fadd_rn(ay, d.w), st);
  *reinterpret_cast<float4*>(a.boxes + idx * 4) = bx;
}

// -------------------------------------------------------------------- layout
__global__ void nchw_to_split_kernel(const float* in, int B, int C, int H, int W, SOut out) {
  pdl_wait();
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(B) * C * H * W;
  if (idx >= total) return;
  const long long hw = static_cast<long long>(H) * W;
  const int c = static_cast<int>(idx % C);
  const long long pix = idx / C;
  const int b = static_cast<int>(pix / hw);
  const long long p = pix - b * hw;
  uint32_t hi, lo;
  split1(in[(static_cast<long long>(b) * C + c) * hw + p], hi, lo);
  const long long o = vaddr(out, b, p) + c;
  out.hi[o] = static_cast<uint16_t>(hi);
  out.hi[o + out.plane] = static_cast<uint16_t>(lo);
}

__global__ void split_to_nchw_kernel(SView in, int B, int C, int H, int W, float* out) {
  pdl_wait();
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(B) * C * H * W;
  if (idx >= total) return;
  const long long hw = static_cast<long long>(H) * W;
  const long long p = idx % hw;
  const long long bc = idx / hw;
  const int c = static_cast<int>(bc % C);
  const int b = static_cast<int>(bc / C);
  const long long o = vaddr(in, b, p) + c;
  out[idx] = join1(in.hi[o], in.hi[o + in.plane]);
}

__global__ void gather_concat_kernel(SView s0, int c0, int up0, SView s1, int c1, int B, int H, int W, SOut out) {
  pdl_wait();
  const int C = c0 + c1;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(B) * H * W * C;
  if (idx >= total) return;
  const int c = static_cast<int>(idx % C);
  const long long pix = idx / C;
  const int b = static_cast<int>(pix / (static_cast<long long>(H) * W));
  const int p = static_cast<int>(pix - static_cast<long long>(b) * H * W);
  const int y = p / W, x = p - (p / W) * W;
  long long i;
  const uint16_t* src;
  long long pl;
  if (c < c0) {
    const int w0 = W / up0;
    i = vaddr(s0, b, static_cast<long long>((y / up0) * w0 + (x / up0))) + c;
    src = s0.hi;
    pl = s0.plane;
  } else {
    i = vaddr(s1, b, p) + (c - c0);
    src = s1.hi;
    pl = s1.plane;
  }
  const long long o = vaddr(out, b, p) + c;
  out.hi[o] = src[i];
  out.hi[o + out.plane] = src[i + pl];
}

// Standalone layers.h element-wise and copy operations on plain fp32 NCHW
// tensors (the host tensors' own layout, all images): silu_forward
// (layers.c:10-21), pool2d_max_forward (layers.c:191-217) and
// upsample_nearest_forward (layers.c:23-39).  Pooling and upsampling copy
// values, so they are exact; SiLU is x / (1 + expf(-x)) in fp32.
__global__ void silu_f32_kernel(float* __restrict__ x, long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) x[i] = silu(x[i]);
}

__global__ void maxpool_nchw_kernel(const float* __restrict__ in, long long planes, int H, int W, int k, int stride,
                                    int Ho, int Wo, float* __restrict__ out) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= planes * Ho * Wo) return;
  const int ox = static_cast<int>(i % Wo);
  const int oy = static_cast<int>((i / Wo) % Ho);
  const long long pl = i / (static_cast<long long>(Wo) * Ho);
  const float* src = in + pl * H * W;
  const int pad = k / 2;
  float m = -FLT_MAX;
  for (int ky = 0; ky < k; ++ky) {
    const int iy = oy * stride - pad + ky;
    if (iy < 0 || iy >= H) continue;
    for (int kx = 0; kx < k; ++kx) {
      const int ix = ox * stride - pad + kx;
      if (ix < 0 || ix >= W) continue;
      const float v = src[static_cast<long long>(iy) * W + ix];
      if (v > m) m = v;
    }
  }
  out[i] = m;
}

__global__ void upsample_nchw_kernel(const float* __restrict__ in, long long planes, int H, int W, int scale,
                                     float* __restrict__ out) {
  const int Ho = H * scale, Wo = W * scale;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= planes * Ho * Wo) return;
  const int ox = static_cast<int>(i % Wo);
  const int oy = static_cast<int>((i / Wo) % Ho);
  const long long pl = i / (static_cast<long long>(Wo) * Ho);
  out[i] = in[(pl * H + oy / scale) * W + ox / scale];
}

}  // namespace

cudaError_t init_stem_kernel_attributes() {
  cudaError_t e = cudaFuncSetAttribute(stem_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, StemTile<16>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(stem_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, StemTile<32>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(stem_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, StemTile<64>::kSmem);
  return e;
}

cudaError_t launch_stem(const StemArgs& a, cudaStream_t s) {
  if (stem_tc_supported(a)) return launch_stem_tc(a, s);
  if (a.Ci < 1 || a.Ci > 4 || a.k != 3 || a.stride != 2 || a.pad != 1 || (a.Co != 16 && a.Co != 32 && a.Co != 64))
    return cudaErrorInvalidValue;
  if (a.Ho != (a.H - 1) / 2 + 1 || a.Wo != (a.W - 1) / 2 + 1) return cudaErrorInvalidValue;
  const int tw = 16 * (64 / a.Co);
  const long long tiles = static_cast<long long>(a.B) * ((a.Ho + 7) / 8) * ((a.Wo + tw - 1) / tw);
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned grid = static_cast<unsigned>(tiles < 3LL * sms ? tiles : 3LL * sms);
  if (a.Co == 16) return launch_pdl(stem_kernel<16>, dim3(grid), dim3(128), StemTile<16>::kSmem, s, a);
  if (a.Co == 32) return launch_pdl(stem_kernel<32>, dim3(grid), dim3(128), StemTile<32>::kSmem, s, a);
  return launch_pdl(stem_kernel<64>, dim3(grid), dim3(128), StemTile<64>::kSmem, s, a);
}

cudaError_t launch_absmax_split(SView v, int B, int H, int W, int C, unsigned* amax, cudaStream_t s) {
  // The statistic lands in amax[1] (amax[0] receives 0).
  const long long total = static_cast<long long>(B) * H * W * C;
  const long long blocks = (total + 255) / 256;
  return launch_pdl(absmax_split_kernel, dim3(static_cast<unsigned>(blocks < 1184 ? (blocks < 1 ? 1 : blocks) : 1184)),
                    dim3(256), 0, s, v, B, H, W, C, amax);
}

cudaError_t launch_absmax_f32(const float* x, long long n, unsigned* amax, cudaStream_t s) {
  const long long blocks = (n + 255) / 256;
  return launch_pdl(absmax_f32_kernel, dim3(static_cast<unsigned>(blocks < 1184 ? (blocks < 1 ? 1 : blocks) : 1184)),
                    dim3(256), 0, s, x, n, amax);
}

cudaError_t launch_dwconv3x3(const DwArgs& a, cudaStream_t s) {
  // 4-byte loads and stores of 2 channels per plane; float2 weight pairs.
  if (a.C % 2 || a.in.cstride % 2 || a.in.coff % 2 || a.in.bstride % 2 || a.in.plane % 2 || a.out.cstride % 2 ||
      a.out.coff % 2 || a.out.bstride % 2 || a.out.plane % 2 || reinterpret_cast<uintptr_t>(a.in.hi) % 4 ||
      reinterpret_cast<uintptr_t>(a.out.hi) % 4 || reinterpret_cast<uintptr_t>(a.w) % 8 ||
      reinterpret_cast<uintptr_t>(a.bias) % 8)
    return cudaErrorInvalidValue;
  if (a.B <= 0 || a.H <= 0 || a.W <= 0 || a.C <= 0) return cudaSuccess;
  // 32-bit thread indices and per-image element offsets.
  if (static_cast<long long>(a.B) * ((a.H + 3) / 4) * a.W * (a.C / 2) + 256 > INT_MAX ||
      static_cast<long long>(a.H) * a.W * a.in.cstride > INT_MAX ||
      static_cast<long long>(a.H) * a.W * a.out.cstride > INT_MAX)
    return cudaErrorInvalidValue;
  // Four channels per thread when every pixel's channel run and the weights
  // allow 8- and 16-byte vectors.
  if (a.C % 4 == 0 && a.in.cstride % 4 == 0 && a.in.coff % 4 == 0 && a.in.bstride % 4 == 0 && a.in.plane % 4 == 0 &&
      a.out.cstride % 4 == 0 && a.out.coff % 4 == 0 && a.out.bstride % 4 == 0 && a.out.plane % 4 == 0 &&
      reinterpret_cast<uintptr_t>(a.in.hi) % 8 == 0 && reinterpret_cast<uintptr_t>(a.out.hi) % 8 == 0 &&
      reinterpret_cast<uintptr_t>(a.w) % 16 == 0 && reinterpret_cast<uintptr_t>(a.bias) % 16 == 0) {
    if (a.H >= 40) {
      const long long total = static_cast<long long>(a.B) * ((a.H + 7) / 8) * a.W * (a.C / 4);
      return launch_pdl(dw3x3_c4_kernel<8>, dim3(blocks_for(total, 256)), dim3(256), 0, s, a);
    }
    const long long total = static_cast<long long>(a.B) * ((a.H + 3) / 4) * a.W * (a.C / 4);
    return launch_pdl(dw3x3_c4_kernel<4>, dim3(blocks_for(total, 256)), dim3(256), 0, s, a);
  }
  if (a.H >= 40) {
    const long long total = static_cast<long long>(a.B) * ((a.H + 7) / 8) * a.W * (a.C / 2);
    return launch_pdl(dw3x3_kernel<8>, dim3(blocks_for(total, 256)), dim3(256), 0, s, a);
  }
  const long long total = static_cast<long long>(a.B) * ((a.H + 3) / 4) * a.W * (a.C / 2);
  return launch_pdl(dw3x3_kernel<4>, dim3(blocks_for(total, 256)), dim3(256), 0, s, a);
}

int sppf_pool_smem_bytes(int H, int W) { return 4 * H * W * 32; }

cudaError_t launch_sppf_pool(SView in, SOut o1, SOut o2, SOut o3, int B, int H, int W, int C, cudaStream_t s) {
  const int smem = sppf_pool_smem_bytes(H, W);
  if (C % 8 || B < 1 || H < 1 || W < 1 || smem > kSppfSmemMax) return cudaErrorInvalidValue;
  for (const long long v : {static_cast<long long>(in.cstride), static_cast<long long>(in.coff), in.bstride, in.plane,
                            static_cast<long long>(o1.cstride), static_cast<long long>(o1.coff), o1.bstride, o1.plane,
                            static_cast<long long>(o2.cstride), static_cast<long long>(o2.coff), o2.bstride, o2.plane,
                            static_cast<long long>(o3.cstride), static_cast<long long>(o3.coff), o3.bstride, o3.plane})
    if (v % 8) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_done{0};
  const cudaError_t e = smem_attr_once(sppf_pool_kernel, kSppfSmemMax, attr_done);
  if (e != cudaSuccess) return e;
  return launch_pdl(sppf_pool_kernel, dim3(static_cast<unsigned>(B * (C / 8))), dim3(256), smem, s, in, o1, o2, o3, B, H,
                    W, C);
}

cudaError_t launch_maxpool(const PoolArgs& a, cudaStream_t s) {
  if (a.C % 8) return cudaErrorInvalidValue;
  PoolArgs b = a;
  if (b.Ho <= 0 || b.Wo <= 0) {
    b.Ho = a.H;
    b.Wo = a.W;
  }
  if (b.stride < 1) return cudaErrorInvalidValue;
  const long long total = static_cast<long long>(b.B) * b.Ho * b.Wo * (b.C / 8);
  return launch_pdl(maxpool_kernel, dim3(blocks_for(total, 256)), dim3(256), 0, s, b);
}

cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t s) {
  const long long total = static_cast<long long>(a.B) * a.N * 4;
  if (total == 0) return cudaSuccess;
  return launch_pdl(decode_kernel, dim3(blocks_for(total, 256)), dim3(256), 0, s, a);
}

cudaError_t launch_nchw_to_split(const float* in, int B, int C, int H, int W, SOut out, cudaStream_t s) {
  const long long total = static_cast<long long>(B) * C * H * W;
  nchw_to_split_kernel<<<blocks_for(total, 256), 256, 0, s>>>(in, B, C, H, W, out);
  return cudaGetLastError();
}

cudaError_t launch_split_to_nchw(SView in, int B, int C, int H, int W, float* out, cudaStream_t s) {
  const long long total = static_cast<long long>(B) * C * H * W;
  split_to_nchw_kernel<<<blocks_for(total, 256), 256, 0, s>>>(in, B, C, H, W, out);
  return cudaGetLastError();
}

cudaError_t launch_gather_concat(SView src0, int c0, int up0, SView src1, int c1, int B, int H, int W, SOut out,
                                 cudaStream_t s) {
  const long long total = static_cast<long long>(B) * H * W * (c0 + c1);
  gather_concat_kernel<<<blocks_for(total, 256), 256, 0, s>>>(src0, c0, up0, src1, c1, B, H, W, out);
  return cudaGetLastError();
}

cudaError_t launch_silu_f32(float* x, long long n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  silu_f32_kernel<<<blocks_for(n, 256), 256, 0, s>>>(x, n);
  return cudaGetLastError();
}

cudaError_t launch_maxpool_nchw(const float* in, long long planes, int H, int W, int k, int stride, int Ho, int Wo,
                                float* out, cudaStream_t s) {
  const long long total = planes * Ho * Wo;
  if (total <= 0) return cudaSuccess;
  maxpool_nchw_kernel<<<blocks_for(total, 256), 256, 0, s>>>(in, planes, H, W, k, stride, Ho, Wo, out);
  return cudaGetLastError();
}

cudaError_t launch_upsample_nchw(const float* in, long long planes, int H, int W, int scale, float* out,
                                 cudaStream_t s) {
  const long long total = planes * H * scale * W * scale;
  if (total <= 0) return cudaSuccess;
  upsample_nchw_kernel<<<blocks_for(total, 256), 256, 0, s>>>(in, planes, H, W, scale, out);
  return cudaGetLastError();
}

}  // namespace yb
