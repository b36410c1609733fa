// Device-resident FP32 convolution handle: one convolution of the YOLO26 graph
// (conv2d_forward + bias + optional SiLU, layers.c:41-90 of
// phucb2/yolo-baremetal) run on tensors that already live in HBM, with the
// kernel and operand mode the model graph would pick for the same shape:
//   * 3x3 stride-2 convolutions of <= 4 input channels (the first layer)
//     read an NCHW fp32 input with the stem kernel, as the graph does;
//   * every other shape runs the tcgen05 implicit GEMM on split NHWC
//     activations (hi plane, then lo plane), with the patch / TMA im2col /
//     gather modes and the narrow-N rule of the graph.
// It serves the isolated convolution sweep (timing) and its parity tests.
#include <climits>
#include <string>
#include <vector>

#include "kernels.h"
#include "runtime.h"
#include "status.h"
#include "yb_cuda.h"

namespace yb {
namespace {

inline int pad8(int c) { return (c + 7) & ~7; }

struct Fp32Conv {
  int device = 0, num_sms = 148;
  int co = 0, cop = 0, ci = 0, cip = 0, kh = 0, kw = 0, stride = 1, pad = 0, act = kActNone;
  bool stem = false;
  bool withhold_next = false;  // test hook armed by yb_conv_debug_withhold
  int K = 0, num_kc = 0, n_tile = 0, n_tiles = 0;
  uint8_t* wpack[3] = {nullptr, nullptr, nullptr};  // full tiling, 64-wide, 128-wide N tiles
  float* bias = nullptr;
  float* stem_w = nullptr;
  int* err = nullptr;
  std::vector<float> w;  // [cop][cip][kh][kw], kept to pack narrow tilings on demand
};

void free_conv(Fp32Conv* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  for (uint8_t* p : c->wpack)
    if (p) cudaFree(p);
  if (c->bias) cudaFree(c->bias);
  if (c->stem_w) cudaFree(c->stem_w);
  if (c->err) cudaFree(c->err);
  delete c;
}

cudaError_t upload_pack(Fp32Conv* c, int n_tile, uint8_t** dst) {
  const size_t bytes = pack_conv_weights(c->w.data(), c->cop, c->cip, c->kh, c->kw, n_tile, nullptr);
  std::vector<uint8_t> pk(bytes);
  pack_conv_weights(c->w.data(), c->cop, c->cip, c->kh, c->kw, n_tile, pk.data());
  cudaError_t e = cudaMalloc(dst, bytes);
  if (e == cudaSuccess) e = cudaMemcpy(*dst, pk.data(), bytes, cudaMemcpyHostToDevice);
  return e;
}

}  // namespace
}  // namespace yb

using namespace yb;

extern "C" status_t yb_conv_create(int device, const float* w, const float* b, int co, int ci, int kh, int kw,
                                   int stride, int pad, int act, void** conv) {
  if (!w || !conv) return ERROR_NULL_POINTER;
  *conv = nullptr;
  if (co < 1 || co > 1024 || ci < 1 || ci > 4096 || kh != kw || (kh != 1 && kh != 3) || stride < 1 || pad < 0 ||
      (act != 0 && act != 1)) {
    set_error("conv: co in [1, 1024], kernel 1x1 or 3x3, act 0 (none) or 1 (SiLU)");
    return ERROR_INVALID_DIMS;
  }
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  if ((e = init_conv_kernel_attributes()) != cudaSuccess) return cuda_status(e, "conv kernel attributes");
  auto* c = new Fp32Conv();
  c->device = device;
  cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  c->co = co;
  c->cop = pad8(co);
  c->ci = ci;
  c->kh = kh;
  c->kw = kw;
  c->stride = stride;
  c->pad = pad;
  c->act = act;
  c->stem = ci <= 4 && kh == 3 && stride == 2 && pad == 1 && (co == 16 || co == 32 || co == 64) && act == kActSiLU;
  e = cudaMalloc(&c->err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->err, 0, sizeof(int));
  std::vector<float> bp;
  if (c->stem) {
    const size_t n = static_cast<size_t>(co) * ci * 9;
    if (e == cudaSuccess) e = cudaMalloc(&c->stem_w, n * 4);
    if (e == cudaSuccess) e = cudaMemcpy(c->stem_w, w, n * 4, cudaMemcpyHostToDevice);
    bp.assign(static_cast<size_t>(co), 0.f);
  } else {
    c->cip = pad8(ci);
    c->w.assign(static_cast<size_t>(c->cop) * c->cip * kh * kw, 0.f);
    for (int o = 0; o < co; ++o)
      for (int i = 0; i < ci; ++i)
        for (int t = 0; t < kh * kw; ++t)
          c->w[(static_cast<size_t>(o) * c->cip + i) * kh * kw + t] = w[(static_cast<size_t>(o) * ci + i) * kh * kw + t];
    c->K = kh * kw * c->cip;
    c->num_kc = (c->K + 63) / 64;
    choose_n_tiling(c->cop, &c->n_tile, &c->n_tiles);
    if (e == cudaSuccess) e = upload_pack(c, c->n_tile, &c->wpack[0]);
    bp.assign(static_cast<size_t>(c->n_tile) * c->n_tiles, 0.f);
  }
  if (b)
    for (int o = 0; o < co; ++o) bp[o] = b[o];
  if (e == cudaSuccess) e = cudaMalloc(&c->bias, bp.size() * 4);
  if (e == cudaSuccess) e = cudaMemcpy(c->bias, bp.data(), bp.size() * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    free_conv(c);
    return cuda_status(e, "conv create");
  }
  *conv = c;
  return SUCCESS;
}

extern "C" int yb_conv_ci_pad(void* conv) {
  auto* c = static_cast<Fp32Conv*>(conv);
  return c && !c->stem ? c->cip : 0;
}

extern "C" status_t yb_conv_run(void* conv, const void* d_x, int B, int H, int W, void* d_y, void* stream) {
  auto* c = static_cast<Fp32Conv*>(conv);
  if (!c || !d_x || !d_y) return ERROR_NULL_POINTER;
  if (B < 1 || H < 1 || W < 1) return ERROR_INVALID_DIMS;
  const int Ho = (H + 2 * c->pad - c->kh) / c->stride + 1, Wo = (W + 2 * c->pad - c->kw) / c->stride + 1;
  if (Ho < 1 || Wo < 1) return ERROR_INVALID_DIMS;
  const long long M = static_cast<long long>(B) * Ho * Wo;
  if (M > INT_MAX - 256 || static_cast<long long>(B) * H * W * (c->stem ? c->ci : c->cip) > (1LL << 40))
    return ERROR_INVALID_DIMS;
  if (reinterpret_cast<uintptr_t>(d_x) % 16 || reinterpret_cast<uintptr_t>(d_y) % 16) {
    set_error("conv: buffers must be 16-byte aligned");
    return ERROR_INVALID_DIMS;
  }
  cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SOut out;
  out.hi = static_cast<uint16_t*>(d_y);
  out.plane = M * c->cop;
  out.bstride = static_cast<long long>(Ho) * Wo * c->cop;
  out.cstride = c->cop;
  if (c->stem) {
    StemArgs sa;
    sa.err = c->err;
    sa.in = static_cast<const float*>(d_x);
    sa.B = B;
    sa.Ci = c->ci;
    sa.H = H;
    sa.W = W;
    sa.Co = c->co;
    sa.Ho = Ho;
    sa.Wo = Wo;
    sa.k = c->kh;
    sa.w = c->stem_w;
    sa.bias = c->bias;
    sa.act = c->act;
    sa.out = out;
    return cuda_status(launch_stem(sa, s), "stem conv");
  }
  ConvArgs a;
  a.B = B;
  a.H = H;
  a.W = W;
  a.Ci = c->cip;
  a.Co = c->cop;
  a.kh = c->kh;
  a.kw = c->kw;
  a.stride = c->stride;
  a.pad = c->pad;
  a.Ho = Ho;
  a.Wo = Wo;
  a.K = c->K;
  a.num_kc = c->num_kc;
  a.n_tile = c->n_tile;
  a.n_tiles = c->n_tiles;
  a.m_tiles = static_cast<int>((M + 127) / 128);
  SView in;
  in.hi = static_cast<const uint16_t*>(d_x);
  in.plane = static_cast<long long>(B) * H * W * c->cip;
  in.bstride = static_cast<long long>(H) * W * c->cip;
  in.cstride = c->cip;
  a.src0 = in;
  a.src1 = in;
  a.c_split = c->cip;
  a.wpack = c->wpack[0];
  a.bias = c->bias;
  // The graph's rule: fewer than two waves of tiles take 64- or 128-wide N
  // tiles so that more SMs share the work.
  if (a.n_tiles * a.m_tiles < 2 * c->num_sms && c->cop >= 128) {
    const int nt = a.m_tiles * ((c->cop + 127) / 128) >= 2 * c->num_sms ? 128 : 64;
    uint8_t** slot = &c->wpack[nt == 64 ? 1 : 2];
    if (!*slot && (e = upload_pack(c, nt, slot)) != cudaSuccess) return cuda_status(e, "conv narrow packing");
    a.wpack = *slot;
    a.n_tile = nt;
    a.n_tiles = (c->cop + nt - 1) / nt;
  }
  a.act = c->act;
  a.out = out;
  a.err = c->err;
  conv_setup_tma(&a);
  if (c->withhold_next) {
    c->withhold_next = false;
    a.debug_withhold = 1;
    a.wait_ns = 1000000;  // 1 ms
  }
  return cuda_status(launch_conv_tc(a, s, c->num_sms), "conv");
}

extern "C" status_t yb_conv_debug_withhold(void* conv) {
  auto* c = static_cast<Fp32Conv*>(conv);
  if (!c) return ERROR_NULL_POINTER;
  if (c->stem) {
    set_error("conv: the first-layer kernel has no barrier waits to test");
    return ERROR_NOT_IMPLEMENTED;
  }
  c->withhold_next = true;
  return SUCCESS;
}

extern "C" status_t yb_conv_check(void* conv) {
  auto* c = static_cast<Fp32Conv*>(conv);
  if (!c) return ERROR_NULL_POINTER;
  cudaError_t e = cudaSetDevice(c->device);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  int k = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&k, c->err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "conv check");
  if (k) {
    cudaMemset(c->err, 0, sizeof(int));
    set_error("conv kernel reported error code " + std::to_string(k));
    return ERROR_DEVICE;
  }
  return SUCCESS;
}

extern "C" status_t yb_conv_destroy(void* conv) {
  if (!conv) return ERROR_NULL_POINTER;
  const status_t st = yb_conv_check(conv);
  free_conv(static_cast<Fp32Conv*>(conv));
  return st;
}
