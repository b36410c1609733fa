// Image preprocessing on the device: uint8 HWC RGB images -> bilinear resize
// -> / 255 -> the fp32 NCHW network input, in one kernel (one thread per
// output pixel, three channels).  The two resize rules are the reference's:
//   YB_RESIZE_ALIGN_CORNERS  src/main.c:18-51 (resize_rgb_bilinear, the
//       image and camera paths): source coordinate dx * (sw - 1) / (dw - 1),
//       blend of the two rows' horizontal blends, (int)(v + 0.5f), clamp;
//   YB_RESIZE_HALF_PIXEL     tests/dump_model_stages.c:58-96 (after decoding):
//       source coordinate (x + 0.5) * iw / out_w - 0.5 truncated and clamped,
//       four-term weighted sum, truncation to uint8;
// then value / 255.0f (main.c:53-64).  Every product, sum and quotient is
// an explicitly rounded intrinsic in the reference's evaluation order, so the
// result is bit-identical to the reference's C (which is compiled without
// floating-point contraction).
#include <atomic>
#include <cstdint>

#include "kernels.h"
#include "pdl.cuh"
#include "yb_cuda.h"

namespace yb {
namespace {

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

__global__ void preprocess_kernel(const uint8_t* src, int B, int sh, int sw, int mode, float* dst, int H, int W) {
  pdl_wait();
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(B) * H * W;
  if (idx >= total) return;
  const int b = static_cast<int>(idx / (static_cast<long long>(H) * W));
  const int p = static_cast<int>(idx - static_cast<long long>(b) * H * W);
  const int y = p / W, x = p - (p / W) * W;
  const uint8_t* img = src + static_cast<long long>(b) * sh * sw * 3;
  float* out = dst + static_cast<long long>(b) * 3 * H * W + p;
  if (mode == YB_RESIZE_ALIGN_CORNERS) {
    const float sx = W == 1 ? 0.f : __fdiv_rn(__fmul_rn(static_cast<float>(x), static_cast<float>(sw - 1)),
                                              static_cast<float>(W - 1));
    const float sy = H == 1 ? 0.f : __fdiv_rn(__fmul_rn(static_cast<float>(y), static_cast<float>(sh - 1)),
                                              static_cast<float>(H - 1));
    const int x0 = static_cast<int>(floorf(sx)), y0 = static_cast<int>(floorf(sy));
    const int x1 = x0 + 1 < sw ? x0 + 1 : x0;
    const int y1 = y0 + 1 < sh ? y0 + 1 : y0;
    const float fx = __fsub_rn(sx, static_cast<float>(x0)), fy = __fsub_rn(sy, static_cast<float>(y0));
    const float gx = __fsub_rn(1.f, fx), gy = __fsub_rn(1.f, fy);
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const float a = img[(y0 * sw + x0) * 3 + c], bb = img[(y0 * sw + x1) * 3 + c];
      const float d = img[(y1 * sw + x0) * 3 + c], e = img[(y1 * sw + x1) * 3 + c];
      const float top = __fadd_rn(__fmul_rn(a, gx), __fmul_rn(bb, fx));
      const float bot = __fadd_rn(__fmul_rn(d, gx), __fmul_rn(e, fx));
      const float v = __fadd_rn(__fmul_rn(top, gy), __fmul_rn(bot, fy));
      const int iv = clampi(__float2int_rz(__fadd_rn(v, 0.5f)), 0, 255);
      out[static_cast<long long>(c) * H * W] = __fdiv_rn(static_cast<float>(iv), 255.0f);
    }
  } else {
    const float fx = __fsub_rn(__fdiv_rn(__fmul_rn(__fadd_rn(static_cast<float>(x), 0.5f), static_cast<float>(sw)),
                                         static_cast<float>(W)),
                               0.5f);
    const float fy = __fsub_rn(__fdiv_rn(__fmul_rn(__fadd_rn(static_cast<float>(y), 0.5f), static_cast<float>(sh)),
                                         static_cast<float>(H)),
                               0.5f);
    const int sx = clampi(__float2int_rz(fx), 0, sw - 1), sy = clampi(__float2int_rz(fy), 0, sh - 1);
    const int sx1 = sx + 1 < sw ? sx + 1 : sx;
    const int sy1 = sy + 1 < sh ? sy + 1 : sy;
    const float tx = __fsub_rn(fx, static_cast<float>(sx)), ty = __fsub_rn(fy, static_cast<float>(sy));
    const float ux = __fsub_rn(1.f, tx), uy = __fsub_rn(1.f, ty);
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const float a = img[(sy * sw + sx) * 3 + c], bb = img[(sy * sw + sx1) * 3 + c];
      const float d = img[(sy1 * sw + sx) * 3 + c], e = img[(sy1 * sw + sx1) * 3 + c];
      float v = __fmul_rn(__fmul_rn(a, ux), uy);
      v = __fadd_rn(v, __fmul_rn(__fmul_rn(bb, tx), uy));
      v = __fadd_rn(v, __fmul_rn(__fmul_rn(d, ux), ty));
      v = __fadd_rn(v, __fmul_rn(__fmul_rn(e, tx), ty));
      const int iv = v < 0.f ? 0 : v > 255.f ? 255 : __float2int_rz(v);
      out[static_cast<long long>(c) * H * W] = __fdiv_rn(static_cast<float>(iv), 255.0f);
    }
  }
}

// Table form of the same arithmetic: a CTA takes kPreRows output rows of one
// image.  The source columns and weights of every output column (x0, x1 and
// the two weights, which depend on x alone), those of its rows, and the 256
// possible values of v / 255 are computed once per CTA, with the same
// intrinsics, so each pixel is loads, the blend and a table lookup.
constexpr int kPreRows = 4;
constexpr int kPreMaxW = 4096;
struct PreAxis {
  int i0, i1;
  float f, g;  // weight of i1 and of i0
};

__device__ __forceinline__ PreAxis pre_axis(int x, int s, int d, int mode) {
  PreAxis r;
  if (mode == YB_RESIZE_ALIGN_CORNERS) {
    const float sx =
        d == 1 ? 0.f : __fdiv_rn(__fmul_rn(static_cast<float>(x), static_cast<float>(s - 1)), static_cast<float>(d - 1));
    r.i0 = static_cast<int>(floorf(sx));
    r.i1 = r.i0 + 1 < s ? r.i0 + 1 : r.i0;
    r.f = __fsub_rn(sx, static_cast<float>(r.i0));
  } else {
    const float fx = __fsub_rn(
        __fdiv_rn(__fmul_rn(__fadd_rn(static_cast<float>(x), 0.5f), static_cast<float>(s)), static_cast<float>(d)),
        0.5f);
    r.i0 = clampi(__float2int_rz(fx), 0, s - 1);
    r.i1 = r.i0 + 1 < s ? r.i0 + 1 : r.i0;
    r.f = __fsub_rn(fx, static_cast<float>(r.i0));
  }
  r.g = __fsub_rn(1.f, r.f);
  return r;
}

__global__ void __launch_bounds__(256) preprocess_rows_kernel(const uint8_t* src, int sh, int sw, int mode, float* dst,
                                                              int H, int W) {
  extern __shared__ PreAxis pre_xt[];  // W entries
  __shared__ PreAxis yt[kPreRows];
  __shared__ float lut[256];
  const int b = blockIdx.y, yb0 = blockIdx.x * kPreRows;
  for (int x = threadIdx.x; x < W; x += blockDim.x) pre_xt[x] = pre_axis(x, sw, W, mode);
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = __fdiv_rn(static_cast<float>(i), 255.0f);
  if (threadIdx.x < kPreRows) yt[threadIdx.x] = pre_axis(min(yb0 + static_cast<int>(threadIdx.x), H - 1), sh, H, mode);
  __syncthreads();
  pdl_wait();
  const uint8_t* img = src + static_cast<long long>(b) * sh * sw * 3;
  float* out = dst + static_cast<long long>(b) * 3 * H * W;
  const long long plane = static_cast<long long>(H) * W;
  for (int r = 0; r < kPreRows; ++r) {
    const int y = yb0 + r;
    if (y >= H) break;
    const PreAxis Y = yt[r];
    const uint8_t* row0 = img + static_cast<long long>(Y.i0) * sw * 3;
    const uint8_t* row1 = img + static_cast<long long>(Y.i1) * sw * 3;
    for (int x = threadIdx.x; x < W; x += blockDim.x) {
      const PreAxis X = pre_xt[x];
      float* o = out + static_cast<long long>(y) * W + x;
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const float a = row0[X.i0 * 3 + c], bb = row0[X.i1 * 3 + c];
        const float d = row1[X.i0 * 3 + c], e = row1[X.i1 * 3 + c];
        int iv;
        if (mode == YB_RESIZE_ALIGN_CORNERS) {
          const float top = __fadd_rn(__fmul_rn(a, X.g), __fmul_rn(bb, X.f));
          const float bot = __fadd_rn(__fmul_rn(d, X.g), __fmul_rn(e, X.f));
          const float v = __fadd_rn(__fmul_rn(top, Y.g), __fmul_rn(bot, Y.f));
          iv = clampi(__float2int_rz(__fadd_rn(v, 0.5f)), 0, 255);
        } else {
          float v = __fmul_rn(__fmul_rn(a, X.g), Y.g);
          v = __fadd_rn(v, __fmul_rn(__fmul_rn(bb, X.f), Y.g));
          v = __fadd_rn(v, __fmul_rn(__fmul_rn(d, X.g), Y.f));
          v = __fadd_rn(v, __fmul_rn(__fmul_rn(e, X.f), Y.f));
          iv = v < 0.f ? 0 : v > 255.f ? 255 : __float2int_rz(v);
        }
        o[c * plane] = lut[iv];
      }
    }
  }
}

}  // namespace

cudaError_t launch_preprocess(const uint8_t* src, int B, int sh, int sw, int mode, float* dst, int H, int W,
                              cudaStream_t s) {
  if (B < 0 || sh < 1 || sw < 1 || H < 1 || W < 1 || (mode != YB_RESIZE_ALIGN_CORNERS && mode != YB_RESIZE_HALF_PIXEL))
    return cudaErrorInvalidValue;
  const long long total = static_cast<long long>(B) * H * W;
  if (total == 0) return cudaSuccess;
  if (W <= kPreMaxW && B <= 65535) {
    const int smem = W * static_cast<int>(sizeof(PreAxis));
    if (smem > 48 * 1024) {
      static std::atomic<uint64_t> attr_done{0};
      const cudaError_t e = smem_attr_once(preprocess_rows_kernel, kPreMaxW * static_cast<int>(sizeof(PreAxis)), attr_done);
      if (e != cudaSuccess) return e;
    }
    return launch_pdl(preprocess_rows_kernel, dim3(static_cast<unsigned>((H + kPreRows - 1) / kPreRows), B), dim3(256),
                      smem, s, src, sh, sw, mode, dst, H, W);
  }
  return launch_pdl(preprocess_kernel, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0, s, src, B, sh,
                    sw, mode, dst, H, W);
}

}  // namespace yb
