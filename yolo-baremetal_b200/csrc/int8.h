// INT8 convolution internals shared by the layer API (conv_i8.cu) and the
// INT8 engine (engine_i8.cu).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include <cuda.h>
#include <cuda_runtime.h>

#include "fastdiv.h"

namespace yb {

// One launch of the kind::i8 convolution.  Input: NHWC int8 view given to
// launch_conv_i8 (channel stride, image stride; Ci channels read, the rest of
// each a_cpp-channel box zero).  Output element (pixel m, channel n) lives at
// out[m * out_cstride + out_coff + n]; the residual (res != null) is read the
// same way and added after requantisation as rshift_rne(r * res_mult,
// res_shift).  With out_f32 set the accumulator is dequantised instead:
// out_f32[b * f32_bstride + p * f32_cstride + n] = float(acc) * deq[n] for
// n < f32_co (pixel p of image b).
struct I8Args {
  int B = 0, H = 0, W = 0, Ci = 0, Co = 0, kh = 1, kw = 1, stride = 1, pad = 0, Ho = 0, Wo = 0;
  int K = 0, num_kc = 0, n_tile = 0, n_tiles = 0, m_tiles = 0, a_cpp = 0;
  // Patch mode (set by launch_conv_i8 for 3x3 convolutions of at most 64
  // input channels with one N tile; 1: stride 1, 2: stride 2): tiles of
  // 16 x 8 output pixels, m_tiles = B * tiles_y * tiles_x.
  int patch = 0, tiles_y = 0, tiles_x = 0;
  int tap_perm = 0;  // the weights hold the taps in the stride-2 patch order (16 channels)
  const uint8_t* wpack = nullptr;
  const int32_t* bias = nullptr;
  const int32_t* mult = nullptr;
  const int32_t* shift = nullptr;
  const int8_t* lut = nullptr;
  int8_t* out = nullptr;
  long long out_cstride = 0, out_coff = 0;
  const int8_t* res = nullptr;
  long long res_cstride = 0, res_coff = 0;
  int res_mult = 0, res_shift = 1;
  float* out_f32 = nullptr;
  long long f32_cstride = 0, f32_bstride = 0;  // element (b, p, n) at b*f32_bstride + p*f32_cstride + n
  int f32_co = 0;                              // channels stored (the rest of the tile is padding)
  const float* deq = nullptr;
  float* rowmax = nullptr;  // optional: sigmoid(max over the f32_co outputs) per pixel, one N tile
  long long rm_bstride = 0;
  int* err = nullptr;
  // Divisors of the per-tile index arithmetic, filled by launch_conv_i8:
  // stages, n_tiles, Ho*Wo, Wo, tiles_y*tiles_x and tiles_x.
  FastDiv fd_stages, fd_ntiles, fd_howo, fd_wo, fd_per, fd_tx;
  alignas(64) CUtensorMap tm;
};

// Fused INT8 Bottleneck (bottleneck_i8.cu): two 3x3 stride-1 pad-1
// convolutions C -> CM -> C ((C, CM) = (16, 16), (32, 32), (32, 16) or
// (16, 8)) with SiLU tables, conv2 adding the residual term of the block
// input; bit-identical to the two conv_i8_kernel launches.  w1 / w2 and the
// per-channel arrays are those the INT8 graph builds for the two
// convolutions (one N tile each).  in / out: NHWC int8 at their first
// channel; filled by i8_bottleneck_setup.
struct I8BottleneckArgs {
  int B = 0, H = 0, W = 0, C = 0, CM = 0;
  const int8_t* in = nullptr;
  long long in_cstride = 0, in_bstride = 0;
  int8_t* out = nullptr;
  long long out_cstride = 0, out_bstride = 0;
  const uint8_t* w1 = nullptr;
  const int32_t *b1 = nullptr, *m1 = nullptr, *s1 = nullptr;
  const int8_t* lut1 = nullptr;
  const uint8_t* w2 = nullptr;
  const int32_t *b2 = nullptr, *m2 = nullptr, *s2 = nullptr;
  const int8_t* lut2 = nullptr;
  int res_mult = 0, res_shift = 1;
  int* err = nullptr;
  int tiles_x = 0, tiles_y = 0, tiles = 0;
  FastDiv fd_per, fd_tx;
  alignas(64) CUtensorMap tm;
};
bool i8_bottleneck_supported(int C, int CM);
bool i8_bottleneck_setup(I8BottleneckArgs* a);
cudaError_t launch_i8_bottleneck(const I8BottleneckArgs& a, cudaStream_t s, int num_sms);
cudaError_t init_i8_bottleneck_attributes();

// K layout of a convolution: input channels padded to ci_pad (a multiple of
// 32; for 3x3 kernels 32, 64 or a multiple of 128), K = kh*kw*ci_pad ordered
// (ky, kx, ci) in 128-wide chunks; a_cpp channels per TMA copy.
struct I8Tiling {
  int ci_pad = 0, a_cpp = 0, K = 0, num_kc = 0, n_tile = 0, n_tiles = 0;
  int tap_perm = 0;  // 1: the stride-2 patch mode's K order of the taps (16 channels)
};
void i8_tiling(int co, int ci, int kh, int kw, I8Tiling* t);
// 3x3 stride-1 convolutions of at most 16 input channels in patch mode: K
// ordered (tap, channel) with 16 channels per tap, two taps per UMMA.
void i8_tiling_pair(int co, I8Tiling* t);
// The same for 3x3 stride-2 convolutions (stride-2 patch mode): the taps in
// the K order {0, 1, 2, 4, 3, 7, 5, 6, 8}.
void i8_tiling_pair_s2(int co, I8Tiling* t);
// wq [co][ci][kh][kw] -> per N tile and K chunk, n_tile 128-byte rows,
// 128B-swizzled (what the kernel's bulk copies load).
std::vector<uint8_t> i8_pack_weights(const int8_t* wq, int co, int ci, int kh, int kw, const I8Tiling& t);
// Entries of the per-channel bias / multiplier / shift arrays: n_tile * n_tiles.
int i8_bias_slots(const I8Tiling& t);
cudaError_t i8_init_kernel();
// Encodes the im2col map of the input view and launches.  a.Ci = channels
// read (<= the view's channels); m_tiles = ceil(B*Ho*Wo / 128).
cudaError_t launch_conv_i8(I8Args& a, const int8_t* x, long long x_cstride, long long x_bstride, cudaStream_t s,
                           int sms, std::string* why);

}  // namespace yb
