// Device-side weight preparation: the BatchNorm fold of the converter's raw
// records (utils.c:81-106, model.c:121-180 of phucb2/yolo-baremetal), the
// tcgen05 operand packing of the FP32 convolutions, and the INT8
// quantisation and packing, all as kernels over weights already in HBM.
// Every rule is the host path's rule written with explicitly rounded
// operations, so the device images are bit-identical to the host-packed ones.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "int8.h"

namespace yb {

// One convolution to fold: offsets (in floats) into the weight arena.
struct FoldDesc {
  long long w = 0, g = 0, be = 0, mu = 0, var = 0, b = 0;
  int oc = 0, per = 0;
};
// scale = gamma / sqrtf(var + 1e-5); w *= scale; b = (b - mean) * scale + beta.
cudaError_t launch_fold_bn(const FoldDesc* d_desc, int n, float* arena, cudaStream_t s);

// pack_conv_weights (conv_tc.cu) on the device: w [co][ci][kh][kw] fp32 ->
// per N tile and 64-wide K chunk, hi then lo bf16 planes, 128B-swizzled.
// dst must hold the packed size (pack_conv_weights(nullptr)) and is cleared.
cudaError_t launch_pack_conv(const float* w, int co, int ci, int kh, int kw, int n_tile, uint8_t* dst, size_t bytes,
                             cudaStream_t s);

// Depthwise / positional taps [C][9] -> tap-major [9][C] (fp32).
cudaError_t launch_taps_transpose(const float* w, int C, float* dst, cudaStream_t s);

// Per-output-channel INT8 quantisation of w [co][ci][kh*kw] (the rule of
// engine_i8.cu's quantize): input-channel scales cs[ci] with s_ref = cs[0],
// or with per_out, one scale cs[o] per output channel (depthwise layers,
// ci = 1).  Writes wq [co][ci*kk], bq, mult, shift, deq [co]; *bad is set
// when a requantisation ratio is out of range.  s_t <= 0: dequantised
// output (mult 0, shift 1).
struct QuantArgs {
  const float* w = nullptr;
  const float* b = nullptr;
  const float* cs = nullptr;
  int co = 0, ci = 0, kk = 0, per_out = 0;
  double s_t = 0.0;
  int8_t* wq = nullptr;
  int32_t *bq = nullptr, *mult = nullptr, *shift = nullptr;
  float* deq = nullptr;
  int* bad = nullptr;
};
cudaError_t launch_quantize_i8(const QuantArgs& a, cudaStream_t s);

// i8_pack_weights (conv_i8.cu) on the device: wq [co][ci][kh][kw] with co
// real rows (rows up to the tiling's are zero) -> dst (cleared here).
cudaError_t launch_pack_i8(const int8_t* wq, int co, int ci, int kh, int kw, const I8Tiling& t, uint8_t* dst,
                           size_t bytes, cudaStream_t s);

// INT8 depthwise layout: one word per filter row, wt[ky][c] byte kx.
cudaError_t launch_pack_dw_i8(const int8_t* wq, int C, uint32_t* wt, cudaStream_t s);
// INT8 positional (pe) taps: wt[k][c] = wq[c][k].
cudaError_t launch_pack_pe_i8(const int8_t* wq, int C, int8_t* wt, cudaStream_t s);
// INT8 first layer (3 input channels): wp[t][o] = bytes of channels 0..2.
cudaError_t launch_pack_stem_i8(const int8_t* wq, int co, uint32_t* wp, cudaStream_t s);

}  // namespace yb
