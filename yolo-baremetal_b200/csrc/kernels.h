// Host-visible descriptions of the device kernels of the YOLO26 sm_100a path
// and their launchers.
//
// Activation format.  Every activation is an NHWC tensor stored as two bf16
// planes in one allocation: hi = bf16_rn(v) and lo = bf16_rn(v - hi), so
// v = hi + lo carries ~16 significant bits (relative representation error
// <= 2^-17) in the same 4 bytes per element as fp32.  The tcgen05 convolution
// consumes the planes directly as its split-bf16 operands (hi*hi + hi*lo +
// lo*hi), so operand tiles are plain asynchronous copies; CUDA-core kernels
// read hi + lo as fp32 and write results split again.
//
// A tensor is addressed through a view {hi, plane, bstride, cstride, coff}:
// element (b, pixel p, channel c) is hi[b*bstride + p*cstride + coff + c] and
// its low part sits `plane` elements later.  Views let a kernel read or write
// a channel slice of a larger buffer, which is how every concat of the
// reference (layers.c:145-153, :185-186, :251-254, :493, model.c:547-550,
// :657-660) is folded away: producers write straight into their slice and
// consumers read the whole buffer.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "detection.h"
#include "fastdiv.h"

namespace yb {

struct SView {
  const uint16_t* hi = nullptr;
  long long plane = 0;    // elements from the hi plane to the lo plane
  long long bstride = 0;  // elements between images
  int cstride = 0;        // elements between pixels
  int coff = 0;           // first channel of the slice
};

struct SOut {
  uint16_t* hi = nullptr;
  long long plane = 0;
  long long bstride = 0;
  int cstride = 0;
  int coff = 0;
};

// Plain fp32 views (Detect head outputs, NCHW host-layout tensors).
struct FView {
  const float* ptr = nullptr;
  long long bstride = 0;
  int cstride = 0;
  int coff = 0;
};

struct FOut {
  float* ptr = nullptr;
  long long bstride = 0;
  int cstride = 0;
  int coff = 0;
  // Optional: the sigmoid of the largest of a pixel's Co outputs at
  // rowmax[b * rm_bstride + p] (pixel p of image b; one N tile only), the
  // Detect head's per-anchor best class score.
  float* rowmax = nullptr;
  long long rm_bstride = 0;
};

enum Act : int { kActNone = 0, kActSiLU = 1 };

// Implicit-GEMM convolution on tcgen05: M = B*Ho*Wo output pixels, N = Co,
// K = kh*kw*Ci ordered (ky, kx, ci).  Input channels [0, c_split) come from
// src0 and [c_split, Ci) from src1; a source with lg_up = 1 is a nearest x2
// upsample of a map half the logical size (the reference's upsample+concat,
// layers.c:23-39 and :219-228, read in place).  Epilogue: + bias, optional
// SiLU, optional + residual (after the activation, as in layers.c:103-106,
// :259-263, :422-450), stored split into `out`, or as fp32 into `out_f32`
// when out_f32.ptr is set.  Ci, c_split, view offsets and strides must be
// multiples of 8 (16-byte copies of bf16); Co a multiple of 8 for split
// output, of 4 for fp32 output.
struct ConvArgs {
  int B = 0, H = 0, W = 0;  // logical input size (after upsampling)
  int Ci = 0, Co = 0;
  int kh = 1, kw = 1, stride = 1, pad = 0;
  int Ho = 0, Wo = 0;
  int K = 0, num_kc = 0;  // K = kh*kw*Ci, num_kc = ceil(K / 64)
  int n_tile = 0, n_tiles = 0, m_tiles = 0;
  int c_split = 0;
  SView src0, src1;
  int lg_up0 = 0, lg_up1 = 0;
  const uint8_t* wpack = nullptr;  // packed split-bf16 weights (see pack_conv_weights)
  const float* bias = nullptr;     // [n_tile * n_tiles] (zero padded) or null
  int act = kActNone;
  SOut out;
  FOut out_f32;  // used instead of `out` when out_f32.ptr != nullptr
  SView res;     // res.hi == nullptr: no residual
  int* err = nullptr;
  // Calibration statistics (null in inference plans): amax[0] |= max
  // |pre-activation|, amax[1] |= max |output| over the SiLU output and the
  // residual sum, as float bits (atomicMax on non-negative floats).
  unsigned* amax = nullptr;
  // Activation operand source.  a_tma == 0: the producer warps gather it with
  // cp.async (any view, upsampled or two-source inputs).  a_tma == 1: one
  // thread loads it with TMA im2col copies through tm_hi / tm_lo (one
  // single-source, non-upsampled input; see conv_setup_tma), a_cpp channels
  // of one filter tap per copy (16, 32 or 64).
  int a_tma = 0;
  int a_cpp = 0;
  // a_tma == 2 (3x3 stride-1 convolutions, see conv_setup_patch): tiles of
  // 16 x 8 output pixels, tiles_y x tiles_x per image; the 18 x 10 input
  // patch of a tile is loaded once per 8-channel chunk and plane, and the
  // weights stay resident in shared memory.  a_tma == 3: the same for 3x3
  // stride-2 convolutions (33 x 17 patch as odd / even column boxes).
  int tiles_y = 0, tiles_x = 0;
  // Test hook of the bounded waits (0 in every plan): with debug_withhold the
  // producer warps arm no barrier and issue no copy, and every wait gives up
  // after wait_ns (0: the default bound), so the MMA issuer's first wait runs
  // out and the kernel records an error, drains and returns.
  int debug_withhold = 0;
  uint64_t wait_ns = 0;
  // Divisors of the per-tile index arithmetic, filled by launch_conv_tc:
  // stages, n_tiles, Ho*Wo, Wo, tiles_y*tiles_x and tiles_x.
  FastDiv fd_stages, fd_ntiles, fd_howo, fd_wo, fd_per, fd_tx;
  alignas(64) CUtensorMap tm_hi;
  alignas(64) CUtensorMap tm_lo;
};

// Switches `a` (fully set up for the cp.async path) to TMA im2col operand
// loads when its input allows it: one source (c_split == Ci), no upsampling,
// Ci a multiple of 16, and for kh*kw > 1 Ci in {16, 32} or a multiple of 64
// (each 64-wide K chunk then holds whole taps).  Leaves `a` unchanged
// otherwise or when the tensor maps cannot be encoded.
void conv_setup_tma(ConvArgs* a);

// Switches a 3x3, stride-1, pad-1 convolution with one non-upsampled source,
// Ci a multiple of 16, Co <= 256 and weights small enough to stay resident
// in shared memory to the patch mode (a_tma == 2); returns whether it did.
// Changes m_tiles to the 2-D tile count.
bool conv_setup_patch(ConvArgs* a);

// Bytes of one packed weight chunk: hi and lo planes of n_tile rows x 128 B.
inline size_t conv_chunk_bytes(int n_tile) { return static_cast<size_t>(n_tile) * 256; }

// Packs w[co][ci][kh][kw] (fp32) into the tcgen05 operand image used by the
// convolution kernel: for each N tile and each 64-wide K chunk, the hi plane
// (bf16 round-to-nearest of w) then the lo plane (bf16 of w - hi), each as
// n_tile rows of 128 bytes in the 128B-swizzled K-major layout.  Rows past Co
// and K past kh*kw*ci are zero.  Returns the byte size; dst may be null to
// query it.
size_t pack_conv_weights(const float* w, int co, int ci, int kh, int kw, int n_tile, uint8_t* dst);

// Chooses n_tile (multiple of 16, <= 256) and n_tiles for Co output channels.
void choose_n_tiling(int co, int* n_tile, int* n_tiles);

cudaError_t launch_conv_tc(const ConvArgs& a, cudaStream_t s, int num_sms);
// Must run once per device before the first launch_conv_tc (not under capture).
cudaError_t init_conv_kernel_attributes();

// Fused Bottleneck (bottleneck_tc.cu; layers.c:92-108 with shortcut):
// out = in + SiLU(conv2(SiLU(conv1(in)))), both convolutions 3x3 stride 1
// pad 1, conv1 C -> CM and conv2 CM -> C channels ((C, CM) = (16, 16),
// (32, 32), (32, 16) or (16, 8)), weights packed by pack_conv_weights in
// their full N tiling (choose_n_tiling).  Tiles of 16 x 8 output pixels,
// tiles_y x tiles_x per image; filled by bottleneck_setup.
struct BottleneckArgs {
  int B = 0, H = 0, W = 0, C = 0, CM = 0;
  SView in;  // channels [coff, coff + C) of the block input (also the residual)
  SOut out;
  const uint8_t* w1 = nullptr;
  const uint8_t* w2 = nullptr;
  const float* b1 = nullptr;  // [C] or null
  const float* b2 = nullptr;
  int* err = nullptr;         // kernel error word (bounded waits that gave up)
  int tiles_x = 0, tiles_y = 0, tiles = 0;
  FastDiv fd_per, fd_tx;
  alignas(64) CUtensorMap tm_hi;
  alignas(64) CUtensorMap tm_lo;
};
bool bottleneck_supported(int C, int CM);
// Encodes the input tensor maps and the tiling; false when the view cannot
// be read by the fused kernel (the caller then launches the two convolutions).
bool bottleneck_setup(BottleneckArgs* a);
cudaError_t launch_bottleneck(const BottleneckArgs& a, cudaStream_t s, int num_sms);
// Must run once per device before the first launch_bottleneck (not under capture).
cudaError_t init_bottleneck_kernel_attributes();

// ---------------------------------------------------------------- SIMT kernels
// First convolution, reading the NCHW host-layout fp32 input directly:
// 3x3 stride 2 pad 1, Ci <= 4, Co in {16, 32, 64}, + bias + SiLU.
struct StemArgs {
  const float* in = nullptr;  // [B, Ci, H, W]
  int B = 0, Ci = 0, H = 0, W = 0, Co = 0, Ho = 0, Wo = 0, stride = 2, pad = 1, k = 3;
  const float* w = nullptr;   // device copy of [Co][Ci][k][k]
  const float* bias = nullptr;
  int act = kActSiLU;
  SOut out;
  unsigned* amax = nullptr;  // calibration statistics, as in ConvArgs
  int* err = nullptr;        // kernel error word (tensor-core form: a bounded wait that gave up)
};
// Runs the tensor-core first layer (stem_tc.cu) when stem_tc_supported(a)
// (1-3 input channels, 16 or 32 outputs, SiLU, no statistics, 32-byte
// aligned output), else the CUDA-core kernel.
cudaError_t launch_stem(const StemArgs& a, cudaStream_t s);
bool stem_tc_supported(const StemArgs& a);
cudaError_t launch_stem_tc(const StemArgs& a, cudaStream_t s);
// Must run once per device before the first launch_stem (not under capture).
cudaError_t init_stem_kernel_attributes();

// Depthwise 3x3, pad 1, + bias, optional SiLU (layers.c:269-290 plus
// detect.c:219-228).  w: device [9][C] (tap-major).  C a multiple of 8.
struct DwArgs {
  SView in;
  int B = 0, H = 0, W = 0, C = 0;
  const float* w = nullptr;
  const float* bias = nullptr;
  int act = kActNone;
  SOut out;
  unsigned* amax = nullptr;  // calibration statistics, as in ConvArgs
};
cudaError_t launch_dwconv3x3(const DwArgs& a, cudaStream_t s);

// Calibration: *amax |= max |x| (float bits) over a split tensor view
// [B, H, W, C] (value = hi + lo) or a plain fp32 array of n elements.
cudaError_t launch_absmax_split(SView v, int B, int H, int W, int C, unsigned* amax, cudaStream_t s);
cudaError_t launch_absmax_f32(const float* x, long long n, unsigned* amax, cudaStream_t s);

// Max pool with padding k/2 excluded from the max (layers.c:191-217).
// Output size Ho x Wo (0 = same as the input, for stride 1).
struct PoolArgs {
  SView in;
  int B = 0, H = 0, W = 0, C = 0, k = 5, stride = 1, Ho = 0, Wo = 0;
  SOut out;
};
cudaError_t launch_maxpool(const PoolArgs& a, cudaStream_t s);
// SPPF's three chained 5x5 stride-1 pools in one launch: o1, o2, o3 receive
// the 5x5, 9x9 and 13x13 max pools of `in` (padding excluded), C channels
// (a multiple of 8).  The whole H x W map of 8 channels is held in shared
// memory: sppf_pool_smem_bytes(H, W) <= kSppfSmemMax.
constexpr int kSppfSmemMax = 220 * 1024;
int sppf_pool_smem_bytes(int H, int W);
cudaError_t launch_sppf_pool(SView in, SOut o1, SOut o2, SOut o3, int B, int H, int W, int C, cudaStream_t s);

// Multi-head attention of the PSA block (layers.c:310-405): per head h the
// qkv channels [h*(2kd+hd), +kd) are q, the next kd are k, the next hd are v;
// S = q.k * kd^-0.5, row softmax, out = P.v; then + depthwise 3x3 of v
// (pe conv, weight [9][heads*hd] tap-major + bias).  out channels h*hd + d.
struct AttnArgs {
  SView qkv;
  int B = 0, H = 0, W = 0, heads = 0, kd = 0, hd = 0;
  float scale = 1.f;
  const float* pe_w = nullptr;
  const float* pe_b = nullptr;
  SOut out;
  int* err = nullptr;  // kernel error word (bounded waits that gave up)
};
// Device preprocess (preprocess.cu): uint8 HWC RGB [B, sh, sw, 3] -> resize
// (mode: yb_resize_mode) -> / 255 -> fp32 NCHW [B, 3, H, W].
cudaError_t launch_preprocess(const uint8_t* src, int B, int sh, int sw, int mode, float* dst, int H, int W,
                              cudaStream_t s);

// Batched decode_detections (detections.cu): dets [B, rows, 6] -> per image
// the rows with score not <= threshold, in order, at most capacity.
cudaError_t launch_detections(const float* dets, int B, int rows, float threshold, int capacity, detection_t* out,
                              int* counts, cudaStream_t s);

// tcgen05 kernel (attn_tc.cu): kd = 32, hd = 64.
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s);

// Detect decode (detect.c:21-61, :407-418): from box distances dist
// [B, N, 4] (l, t, r, b in grid units) and class logits [B, N, nc], write
// xyxy pixel boxes [B, N, 4] and the per-anchor maximum class score
// max_c sigmoid(logit) [B, N].  Scales: anchors [0, n0) stride s0, ... .
struct DecodeArgs {
  const float* dist = nullptr;
  const float* logits = nullptr;
  float* boxes = nullptr;
  float* maxscore = nullptr;
  int max_ready = 0;  // maxscore already written (by the class convolutions' epilogues)
  int B = 0, N = 0, nc = 0;
  int nscales = 0;
  int base[4] = {0, 0, 0, 0};
  int w[4] = {0, 0, 0, 0};
  int stride[4] = {0, 0, 0, 0};
};
cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t s);

// Two-stage top-k of detect_postprocess_from_pred (detect.c:63-166), one CTA
// per image, total order (score desc, index asc) in both stages; writes
// dets [B, cap, 6] (rows >= k zero-filled).
// Class values are read as scores[b*s_bstride + anchor*s_rstride + c]
// (sigmoid applied first when apply_sigmoid), boxes as
// boxes[b*b_bstride + anchor*b_rstride + 0..3].  maxscore (nullable) holds
// the per-anchor maximum class score; when null it is recomputed.
struct TopkArgs {
  const float* maxscore = nullptr;
  const float* scores = nullptr;
  long long s_bstride = 0;
  int s_rstride = 0;
  int apply_sigmoid = 1;
  const float* boxes = nullptr;
  long long b_bstride = 0;
  int b_rstride = 4;
  float* dets = nullptr;  // [B, cap, 6]
  int B = 0, N = 0, nc = 0, max_det = 300, cap = 300;
};
cudaError_t launch_topk(const TopkArgs& a, cudaStream_t s);
// Sets the top-k kernel's shared-memory attribute on the current device (done
// once per device), which also loads its code there.
cudaError_t prepare_topk();
// Largest k supported by the top-k kernel.
constexpr int kTopkMax = 1024;

// Layout conversions for the host API and stage dumps.
// NCHW fp32 [B,C,H,W] -> split NHWC view (channels [0, C) of the view).
cudaError_t launch_nchw_to_split(const float* in, int B, int C, int H, int W, SOut out, cudaStream_t s);
// Split NHWC view -> NCHW fp32 [B,C,H,W] (value hi + lo).
cudaError_t launch_split_to_nchw(SView in, int B, int C, int H, int W, float* out, cudaStream_t s);
// out[B,H,W,c0+c1] = nearest-upsample(src0 by the integer factor up0) ++ src1
// along channels (stage dumps and the layer-level API).
cudaError_t launch_gather_concat(SView src0, int c0, int up0, SView src1, int c1, int B, int H, int W, SOut out,
                                 cudaStream_t s);
// In-place SiLU on a split view.
// Plain fp32 NCHW kernels behind the standalone layers.h entry points:
// in-place SiLU over n values; max pool (padding k/2 excluded) and nearest
// upsample of `planes` = N*C planes of H x W.
cudaError_t launch_silu_f32(float* x, long long n, cudaStream_t s);
cudaError_t launch_maxpool_nchw(const float* in, long long planes, int H, int W, int k, int stride, int Ho, int Wo,
                                float* out, cudaStream_t s);
cudaError_t launch_upsample_nchw(const float* in, long long planes, int H, int W, int scale, float* out,
                                 cudaStream_t s);

}  // namespace yb
