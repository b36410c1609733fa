// CUDA-core kernels of the INT8 forward (simt_i8.cu).  Integer rules (the
// CPU INT8 oracle restates them):
//   rne(p, sh)    = p >> sh rounded half to even (64-bit)
//   requantise    y = rne(acc * mult, shift); SiLU via a 256-entry table
//                 indexed by clamp(y, -128, 127) + 128; clamp to [-127, 127]
//   input         q = clamp(rint(x / s), -127, 127) in fp32
//   max pool      int8 max, padding excluded
//   attention     per head (kd 32, hd 64): S = q.k; t = min(255,
//                 rne((max S - S) * mt, sht)); p = E[t]; l = sum p,
//                 o = sum p v; out = div_rne(rne(o * mo, sho), l) + the
//                 positional depthwise term rne((pe_bq + sum v*pe_w) *
//                 pe_mult, pe_shift), clamped.  q.k and p.v run on the
//                 tensor cores (attn_i8.cu, kind::i8), p split as
//                 64 * (p >> 6) + (p & 63) so both factors fit int8.
#pragma once
#include <cstdint>

#include <cuda_runtime.h>

namespace yb {

// NHWC int8 view: element (b, pixel p, channel c) at p[b*bstride + p*cstride + c].
struct I8View {
  int8_t* p = nullptr;
  long long cstride = 0;
  long long bstride = 0;
};

struct I8AttnArgs {
  I8View qkv;  // [B, H*W, heads * (2*kd + hd)], per head q | k | v
  I8View out;  // [B, H*W, heads * hd]
  int B = 0, H = 0, W = 0, heads = 1, kd = 32, hd = 64, dim = 0;
  int mt = 0, sht = 1, mo = 0, sho = 1;
  const int32_t* E = nullptr;        // [256] softmax weight table
  const int8_t* pe_w = nullptr;      // [9][dim]
  const int32_t* pe_bq = nullptr;    // [dim]
  const int32_t* pe_mult = nullptr;  // [dim]
  const int32_t* pe_shift = nullptr;
  int* err = nullptr;  // kernel error word (bounded waits that gave up)
};

cudaError_t launch_quantize_input(const float* in, int B, int C, int H, int W, float s, I8View out, cudaStream_t st);

// The first convolution fused with the input quantisation: 3x3 stride 2
// pad 1 from the NCHW fp32 input [B, 3, H, W] (quantised with the input
// rule, padding 0) to int8 NHWC [B, Ho, Wo, Co], Co in {16, 32, 64}, with
// the convolution requantisation and SiLU table (stem_i8.cu, kind::i8).
// w: [9][Co] words, each the taps of input channels 0..2 of one output
// channel (byte 3 zero); bias / mult / shift / lut as for the kind::i8 conv.
struct StemI8Args {
  const float* in = nullptr;
  int B = 0, H = 0, W = 0, Ho = 0, Wo = 0, Co = 0;
  float s_in = 1.f;
  const uint32_t* w = nullptr;
  const int32_t* bias = nullptr;
  const int32_t* mult = nullptr;
  const int32_t* shift = nullptr;
  const int8_t* lut = nullptr;
  I8View out;
  int* err = nullptr;  // kernel error word (a bounded wait that gave up)
};
cudaError_t launch_stem_i8(const StemI8Args& a, cudaStream_t st);
cudaError_t init_stem_i8_attributes();
cudaError_t launch_maxpool_i8(I8View in, I8View out, int B, int H, int W, int C, int k, cudaStream_t st);
// SPPF's three chained 5x5 pools in one launch: o1, o2, o3 receive the 5x5,
// 9x9 and 13x13 max pools of `in` (padding excluded), C a multiple of 16; the
// map of 16 channels is held in shared memory (sppf_pool_i8_smem_bytes(H, W)
// <= kSppfI8SmemMax).
constexpr int kSppfI8SmemMax = 220 * 1024;
int sppf_pool_i8_smem_bytes(int H, int W);
cudaError_t launch_sppf_pool_i8(I8View in, I8View o1, I8View o2, I8View o3, int B, int H, int W, int C,
                                cudaStream_t st);
// Depthwise 3x3 pad 1; wr: [3][C] words of packed int8 taps, one per filter
// row (byte kx of wr[ky][c] = tap (ky, kx)), bq / mult / shift per channel,
// lut nullable.
cudaError_t launch_dw3x3_i8(I8View in, I8View out, int B, int H, int W, int C, const uint32_t* wr, const int32_t* bq,
                            const int32_t* mult, const int32_t* shift, const int8_t* lut, cudaStream_t st);
cudaError_t launch_concat_i8(I8View s0, int c0, int lg0, I8View s1, int c1, int B, int H, int W, I8View out,
                             cudaStream_t st);
cudaError_t launch_attention_i8(const I8AttnArgs& a, cudaStream_t st);
cudaError_t launch_nhwc_to_nchw_i8(I8View in, int C, int H, int W, int8_t* out, cudaStream_t st);

}  // namespace yb
