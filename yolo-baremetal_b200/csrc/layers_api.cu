// Layer-level entry points of layers.h (reference: src/layers.c of
// phucb2/yolo-baremetal) and tensor_gemm (src/tensor.c:64-113), each running
// on the current CUDA device.  Host NCHW tensors are staged into HBM in the
// split NHWC format with the channel count padded to a multiple of 8 (zeros),
// all on one stream (allocation zero-fill, copies, kernels), weights are packed
// for the tcgen05 convolution per call, the block runs with the same kernels
// as the model graph, and the result is copied back.  These calls exist for
// drop-in completeness and per-block parity tests; the model path
// (model_forward / yb_cuda_forward) keeps everything in HBM.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <vector>

#include "kernels.h"
#include "layers.h"
#include "runtime.h"
#include "tensor.h"

namespace yb {
namespace {

inline int pad8(int c) { return (c + 7) & ~7; }

// Split device tensor [1, H, W, Cp] (hi plane then lo plane) with C logical
// channels; channels C..Cp-1 are zero.
struct DT {
  uint16_t* hi = nullptr;
  int H = 0, W = 0, C = 0, Cp = 0;
  long long plane() const { return static_cast<long long>(H) * W * Cp; }
  SView v(int coff = 0) const {
    SView t;
    t.hi = hi;
    t.plane = plane();
    t.bstride = plane();
    t.cstride = Cp;
    t.coff = coff;
    return t;
  }
  SOut o(int coff = 0) const {
    SOut t;
    t.hi = hi;
    t.plane = plane();
    t.bstride = plane();
    t.cstride = Cp;
    t.coff = coff;
    return t;
  }
};

struct PackedConv {
  uint8_t* wpack = nullptr;
  float* bias = nullptr;
  int co = 0, cop = 0, cip = 0, kh = 0, kw = 0, K = 0, num_kc = 0, n_tile = 0, n_tiles = 0;
};

class Kit {
 public:
  DevScope* sc = nullptr;
  cudaError_t err = cudaSuccess;
  status_t st = SUCCESS;

  Kit() {
    sc = current_scope();
    if (!sc) st = ERROR_DEVICE;
  }
  bool ok() const { return st == SUCCESS && err == cudaSuccess; }
  // Host -> device copy on the scope's stream, so it is ordered after the
  // stream's zero-fill of the destination (alloc) and before the kernels.
  cudaError_t h2d(void* dst, const void* src, size_t bytes) {
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, sc->stream);
  }

  float* alloc(size_t n) {
    if (!ok()) return nullptr;
    mem_.emplace_back(new DevMem());
    err = mem_.back()->alloc(n * 4);
    if (err != cudaSuccess) return nullptr;
    err = cudaMemsetAsync(mem_.back()->p, 0, n * 4, sc->stream);
    return mem_.back()->f();
  }
  DT tensor(int H, int W, int C) {
    DT d;
    d.H = H;
    d.W = W;
    d.C = C;
    d.Cp = pad8(C);
    // two bf16 planes: the same bytes as one fp32 tensor
    d.hi = reinterpret_cast<uint16_t*>(alloc(static_cast<size_t>(H) * W * d.Cp));
    return d;
  }
  // Image 0 of a host NCHW tensor.
  DT upload(const tensor_t* t) {
    DT d = tensor(t->dims[2], t->dims[3], t->dims[1]);
    if (!ok()) return d;
    const size_t n = static_cast<size_t>(t->dims[1]) * t->dims[2] * t->dims[3];
    float* tmp = alloc(n);
    if (!ok()) return d;
    err = cudaMemcpyAsync(tmp, t->data, n * 4, cudaMemcpyHostToDevice, sc->stream);
    if (ok()) err = launch_nchw_to_split(tmp, 1, d.C, d.H, d.W, d.o(), sc->stream);
    return d;
  }
  // Writes image 0 of `out` (NCHW host) from the first C channels of d.
  void download(const DT& d, tensor_t* out) {
    if (!ok()) return;
    const size_t n = static_cast<size_t>(d.C) * d.H * d.W;
    float* tmp = alloc(n);
    if (!ok()) return;
    err = launch_split_to_nchw(d.v(), 1, d.C, d.H, d.W, tmp, sc->stream);
    if (ok()) err = cudaMemcpyAsync(out->data, tmp, n * 4, cudaMemcpyDeviceToHost, sc->stream);
    if (ok()) err = cudaStreamSynchronize(sc->stream);
    if (ok()) {
      int kerr = 0;
      err = cudaMemcpy(&kerr, sc->d_err, sizeof(int), cudaMemcpyDeviceToHost);
      if (ok() && kerr) {
        cudaMemset(sc->d_err, 0, sizeof(int));
        set_error("device kernel reported error code " + std::to_string(kerr));
        st = ERROR_DEVICE;
      }
    }
  }
  // Packs w [co, ci, kh, kw] with input channels padded to cip.
  PackedConv pack(const tensor_t* w, const tensor_t* b, int cip) {
    PackedConv p;
    if (!ok()) return p;
    p.co = w->dims[0];
    p.cop = pad8(p.co);
    const int ci = w->dims[1];
    p.cip = cip;
    p.kh = w->dims[2];
    p.kw = w->dims[3];
    p.K = p.kh * p.kw * cip;
    p.num_kc = (p.K + 63) / 64;
    choose_n_tiling(p.cop, &p.n_tile, &p.n_tiles);
    std::vector<float> wp(static_cast<size_t>(p.cop) * cip * p.kh * p.kw, 0.f);
    for (int o = 0; o < p.co; ++o)
      for (int c = 0; c < ci; ++c)
        for (int k = 0; k < p.kh * p.kw; ++k)
          wp[(static_cast<size_t>(o) * cip + c) * p.kh * p.kw + k] = w->data[(static_cast<size_t>(o) * ci + c) * p.kh * p.kw + k];
    const size_t bytes = pack_conv_weights(wp.data(), p.cop, cip, p.kh, p.kw, p.n_tile, nullptr);
    std::vector<uint8_t> pk(bytes);
    pack_conv_weights(wp.data(), p.cop, cip, p.kh, p.kw, p.n_tile, pk.data());
    p.wpack = reinterpret_cast<uint8_t*>(alloc((bytes + 3) / 4));
    if (ok()) err = h2d(p.wpack, pk.data(), bytes);
    std::vector<float> bp(static_cast<size_t>(p.n_tile) * p.n_tiles, 0.f);
    if (b) std::copy(b->data, b->data + p.co, bp.begin());
    p.bias = alloc(bp.size());
    if (ok()) err = h2d(p.bias, bp.data(), bp.size() * 4);
    return p;
  }
  // Convolution of in (channels [coff, coff+cin) of x) into out slice.
  void conv(const PackedConv& p, const DT& x, int coff, int stride, int pad, int act, const DT& y, int ycoff,
            const DT* res = nullptr, int rcoff = 0) {
    if (!ok()) return;
    ConvArgs a;
    a.B = 1;
    a.H = x.H;
    a.W = x.W;
    a.Ci = p.cip;
    a.Co = p.cop;
    a.kh = p.kh;
    a.kw = p.kw;
    a.stride = stride;
    a.pad = pad;
    a.Ho = (x.H + 2 * pad - p.kh) / stride + 1;
    a.Wo = (x.W + 2 * pad - p.kw) / stride + 1;
    if (a.Ho != y.H || a.Wo != y.W) {
      st = ERROR_INVALID_DIMS;
      return;
    }
    a.K = p.K;
    a.num_kc = p.num_kc;
    a.n_tile = p.n_tile;
    a.n_tiles = p.n_tiles;
    a.m_tiles = (a.Ho * a.Wo + 127) / 128;
    a.c_split = p.cip;
    a.src0 = x.v(coff);
    a.src1 = a.src0;
    a.wpack = p.wpack;
    a.bias = p.bias;
    a.act = act;
    a.out = y.o(ycoff);
    if (res) a.res = res->v(rcoff);
    a.err = sc->d_err;
    conv_setup_tma(&a);
    err = launch_conv_tc(a, sc->stream, sc->num_sms);
  }
  void dw(const tensor_t* w, const tensor_t* b, const DT& x, int coff, int act, const DT& y, int ycoff) {
    if (!ok()) return;
    const int C = w->dims[0];
    const int Cp = pad8(C);
    std::vector<float> t(static_cast<size_t>(9) * Cp, 0.f), bb(Cp, 0.f);
    for (int c = 0; c < C; ++c)
      for (int k = 0; k < 9; ++k) t[static_cast<size_t>(k) * Cp + c] = w->data[static_cast<size_t>(c) * 9 + k];
    if (b) std::copy(b->data, b->data + C, bb.begin());
    float* dw = alloc(t.size());
    float* db = alloc(bb.size());
    if (!ok()) return;
    err = h2d(dw, t.data(), t.size() * 4);
    if (ok()) err = h2d(db, bb.data(), bb.size() * 4);
    DwArgs a;
    a.in = x.v(coff);
    a.B = 1;
    a.H = x.H;
    a.W = x.W;
    a.C = Cp;
    a.w = dw;
    a.bias = db;
    a.act = act;
    a.out = y.o(ycoff);
    if (ok()) err = launch_dwconv3x3(a, sc->stream);
  }
  void attention(const DT& qkv, int heads, int kd, int hd, const tensor_t* pe_w, const tensor_t* pe_b, const DT& out) {
    if (!ok()) return;
    const int C = heads * hd;
    std::vector<float> t(static_cast<size_t>(9) * C), bb(pe_b->data, pe_b->data + C);
    for (int c = 0; c < C; ++c)
      for (int k = 0; k < 9; ++k) t[static_cast<size_t>(k) * C + c] = pe_w->data[static_cast<size_t>(c) * 9 + k];
    float* dw = alloc(t.size());
    float* db = alloc(bb.size());
    if (!ok()) return;
    err = h2d(dw, t.data(), t.size() * 4);
    if (ok()) err = h2d(db, bb.data(), bb.size() * 4);
    AttnArgs a;
    a.qkv = qkv.v();
    a.B = 1;
    a.H = qkv.H;
    a.W = qkv.W;
    a.heads = heads;
    a.kd = kd;
    a.hd = hd;
    a.scale = std::pow(static_cast<float>(kd), -0.5f);
    a.pe_w = dw;
    a.pe_b = db;
    a.out = out.o();
    if (ok()) err = launch_attention(a, sc->stream);
  }
  void pool(const DT& x, int coff, int k, int stride, const DT& y, int ycoff, int C) {
    if (!ok()) return;
    PoolArgs a;
    a.in = x.v(coff);
    a.B = 1;
    a.H = x.H;
    a.W = x.W;
    a.C = pad8(C);
    a.k = k;
    a.stride = stride;
    a.Ho = y.H;
    a.Wo = y.W;
    a.out = y.o(ycoff);
    err = launch_maxpool(a, sc->stream);
  }
  status_t finish(const char* what) {
    if (st != SUCCESS) return st;
    return cuda_status(err, what);
  }

 private:
  std::vector<std::unique_ptr<DevMem>> mem_;
};

bool all_mult8(std::initializer_list<int> cs) {
  for (int c : cs)
    if (c % 8) return false;
  return true;
}

// PSABlock body shared by psablock_forward and c2psa_forward.
void psa_block(Kit& k, const DT& x, int xcoff, int c, const tensor_t* w, int heads, float attn_ratio, const DT& y,
               int ycoff, bool shortcut) {
  const int hd = c / heads;
  const int kd = static_cast<int>(static_cast<float>(hd) * attn_ratio);
  const PackedConv qkv = k.pack(&w[0], &w[1], c);
  const PackedConv proj = k.pack(&w[2], &w[3], c);
  const PackedConv f0 = k.pack(&w[6], &w[7], c);
  const PackedConv f1 = k.pack(&w[8], &w[9], f0.cop);
  if (!k.ok()) return;
  if (qkv.co != c + 2 * kd * heads || kd != 32 || hd != 64) {
    k.st = qkv.co != c + 2 * kd * heads ? ERROR_INVALID_DIMS : ERROR_NOT_IMPLEMENTED;
    set_error("attention shape: the device kernel takes key_dim 32 and head_dim 64");
    return;
  }
  DT q = k.tensor(x.H, x.W, qkv.co);
  k.conv(qkv, x, xcoff, 1, 0, kActNone, q, 0);
  DT ao = k.tensor(x.H, x.W, c);
  k.attention(q, heads, kd, hd, &w[4], &w[5], ao);
  DT x1 = k.tensor(x.H, x.W, c);
  k.conv(proj, ao, 0, 1, 0, kActNone, x1, 0, shortcut ? &x : nullptr, xcoff);
  DT f = k.tensor(x.H, x.W, f0.co);
  k.conv(f0, x1, 0, 1, 0, kActSiLU, f, 0);
  k.conv(f1, f, 0, 1, 0, kActNone, y, ycoff, shortcut ? &x1 : nullptr, 0);
}

}  // namespace
}  // namespace yb

using namespace yb;

extern "C" status_t conv_block_forward(tensor_t* output, const tensor_t* input, const tensor_t* weight,
                                       const tensor_t* bias, conv_params_t params, bool act) {
  if (!output || !input || !weight || !output->data || !input->data || !weight->data) return ERROR_NULL_POINTER;
  if (weight->dims[1] != input->dims[1] || output->dims[1] != weight->dims[0] || params.stride < 1)
    return ERROR_INVALID_DIMS;
  Kit k;
  DT x = k.upload(input);
  const PackedConv p = k.pack(weight, bias, x.Cp);
  DT y = k.tensor(output->dims[2], output->dims[3], weight->dims[0]);
  k.conv(p, x, 0, params.stride, params.padding, act ? kActSiLU : kActNone, y, 0);
  k.download(y, output);
  return k.finish("conv2d");
}

extern "C" status_t conv2d_forward(tensor_t* output, const tensor_t* input, const tensor_t* weight,
                                   const tensor_t* bias, conv_params_t params) {
  return conv_block_forward(output, input, weight, bias, params, false);
}

namespace {
// Runs `fn(d_in, d_out)` on device copies of a whole host fp32 tensor (n_in
// values in, n_out values out; out may alias in when in_place), then copies
// the result back: the element-wise and copy layers work on the reference's
// own NCHW layout, all images, with no split representation in between.
template <class F>
status_t nchw_call(const float* in, size_t n_in, float* out, size_t n_out, bool in_place, const char* what, F fn) {
  DevScope* sc = current_scope();
  if (!sc) return ERROR_DEVICE;
  DevMem din, dout;
  cudaError_t e = din.alloc(n_in * 4);
  if (e == cudaSuccess && !in_place) e = dout.alloc(n_out * 4);
  if (e != cudaSuccess) return cuda_status(e, what);
  float* d_out = in_place ? din.f() : dout.f();
  e = cudaMemcpyAsync(din.p, in, n_in * 4, cudaMemcpyHostToDevice, sc->stream);
  if (e == cudaSuccess) e = fn(din.f(), d_out, sc->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, d_out, n_out * 4, cudaMemcpyDeviceToHost, sc->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(sc->stream);
  return cuda_status(e, what);
}

size_t numel(const tensor_t* t) {
  return static_cast<size_t>(t->dims[0]) * t->dims[1] * t->dims[2] * t->dims[3];
}
}  // namespace

extern "C" status_t silu_forward(tensor_t* t) {
  if (!t || !t->data) return ERROR_NULL_POINTER;
  const size_t n = numel(t);
  if (n == 0) return SUCCESS;
  return nchw_call(t->data, n, t->data, n, true, "silu",
                   [n](float* x, float*, cudaStream_t s) { return launch_silu_f32(x, static_cast<long long>(n), s); });
}

extern "C" status_t pool2d_max_forward(tensor_t* output, const tensor_t* input, int kernel_size, int stride) {
  if (!output || !input || !output->data || !input->data) return ERROR_NULL_POINTER;
  if (kernel_size < 1 || stride < 1 || output->dims[1] != input->dims[1] || output->dims[0] != input->dims[0])
    return ERROR_INVALID_DIMS;
  const long long planes = static_cast<long long>(input->dims[0]) * input->dims[1];
  const int H = input->dims[2], W = input->dims[3], Ho = output->dims[2], Wo = output->dims[3];
  if (numel(output) == 0) return SUCCESS;
  return nchw_call(input->data, numel(input), output->data, numel(output), false, "max pool",
                   [=](float* x, float* y, cudaStream_t s) {
                     return launch_maxpool_nchw(x, planes, H, W, kernel_size, stride, Ho, Wo, y, s);
                   });
}

extern "C" status_t upsample_nearest_forward(tensor_t* output, const tensor_t* input, int scale) {
  if (!output || !input || !output->data || !input->data) return ERROR_NULL_POINTER;
  if (scale < 1 || output->dims[0] != input->dims[0] || output->dims[1] != input->dims[1] ||
      output->dims[2] != input->dims[2] * scale || output->dims[3] != input->dims[3] * scale)
    return ERROR_INVALID_DIMS;
  const long long planes = static_cast<long long>(input->dims[0]) * input->dims[1];
  const int H = input->dims[2], W = input->dims[3];
  if (numel(output) == 0) return SUCCESS;
  return nchw_call(input->data, numel(input), output->data, numel(output), false, "upsample",
                   [=](float* x, float* y, cudaStream_t s) { return launch_upsample_nchw(x, planes, H, W, scale, y, s); });
}

extern "C" status_t concat_forward(tensor_t* output, const tensor_t* input1, const tensor_t* input2, int dim) {
  if (dim != 1) return ERROR_NOT_IMPLEMENTED;
  if (!output || !input1 || !input2 || !output->data || !input1->data || !input2->data) return ERROR_NULL_POINTER;
  if (input1->dims[2] != input2->dims[2] || input1->dims[3] != input2->dims[3] ||
      output->dims[1] != input1->dims[1] + input2->dims[1])
    return ERROR_INVALID_DIMS;
  // Channel concat is a pure copy: each image's two NCHW blocks are moved
  // device-side into place.
  Kit k;
  const size_t n1 = static_cast<size_t>(input1->dims[1]) * input1->dims[2] * input1->dims[3];
  const size_t n2 = static_cast<size_t>(input2->dims[1]) * input2->dims[2] * input2->dims[3];
  const int B = input1->dims[0];
  float* d = k.alloc((n1 + n2) * B);
  for (int b = 0; b < B && k.ok(); ++b) {
    k.err = cudaMemcpyAsync(d + b * (n1 + n2), input1->data + b * n1, n1 * 4, cudaMemcpyHostToDevice, k.sc->stream);
    if (k.ok())
      k.err = cudaMemcpyAsync(d + b * (n1 + n2) + n1, input2->data + b * n2, n2 * 4, cudaMemcpyHostToDevice, k.sc->stream);
  }
  if (k.ok()) k.err = cudaMemcpyAsync(output->data, d, (n1 + n2) * B * 4, cudaMemcpyDeviceToHost, k.sc->stream);
  if (k.ok()) k.err = cudaStreamSynchronize(k.sc->stream);
  return k.finish("concat");
}

extern "C" status_t dwconv3x3_same_forward(tensor_t* out, const tensor_t* in, const tensor_t* w, const tensor_t* bias) {
  if (!out || !in || !w || !out->data || !in->data || !w->data) return ERROR_NULL_POINTER;
  if (w->dims[0] != in->dims[1] || w->dims[2] != 3 || w->dims[3] != 3) return ERROR_INVALID_DIMS;
  Kit k;
  DT x = k.upload(in);
  DT y = k.tensor(in->dims[2], in->dims[3], in->dims[1]);
  k.dw(w, bias, x, 0, kActNone, y, 0);
  k.download(y, out);
  return k.finish("depthwise conv");
}

extern "C" status_t bottleneck_forward(tensor_t* output, const tensor_t* input, const tensor_t* cv1_w,
                                       const tensor_t* cv1_b, const tensor_t* cv2_w, const tensor_t* cv2_b,
                                       bool shortcut, tensor_t* temp) {
  (void)temp;
  if (!output || !input || !cv1_w || !cv2_w) return ERROR_NULL_POINTER;
  if (!all_mult8({input->dims[1], cv1_w->dims[0], cv2_w->dims[0]})) return ERROR_INVALID_DIMS;
  Kit k;
  DT x = k.upload(input);
  const PackedConv p1 = k.pack(cv1_w, cv1_b, x.Cp);
  const PackedConv p2 = k.pack(cv2_w, cv2_b, p1.cop);
  DT t = k.tensor(x.H, x.W, p1.co);
  DT y = k.tensor(x.H, x.W, p2.co);
  k.conv(p1, x, 0, 1, (p1.kh - 1) / 2, kActSiLU, t, 0);
  k.conv(p2, t, 0, 1, (p2.kh - 1) / 2, kActSiLU, y, 0, shortcut ? &x : nullptr, 0);
  k.download(y, output);
  return k.finish("bottleneck");
}

extern "C" status_t c3k2_forward(tensor_t* output, const tensor_t* input, int n, bool shortcut,
                                 const tensor_t* cv1_w, const tensor_t* cv1_b, const tensor_t* cv2_w,
                                 const tensor_t* cv2_b, const tensor_t* bw, tensor_t* buffers) {
  (void)buffers;
  if (!output || !input || !cv1_w || !cv2_w || (n > 0 && !bw)) return ERROR_NULL_POINTER;
  const int ct = cv1_w->dims[0], ch = ct / 2;
  if (!all_mult8({input->dims[1], ct, ch, cv2_w->dims[0]}) || cv2_w->dims[1] != (2 + n) * ch) return ERROR_INVALID_DIMS;
  Kit k;
  DT x = k.upload(input);
  const PackedConv p1 = k.pack(cv1_w, cv1_b, x.Cp);
  DT cat = k.tensor(x.H, x.W, (2 + n) * ch);
  k.conv(p1, x, 0, 1, 0, kActSiLU, cat, 0);
  int prev = ch;
  for (int i = 0; i < n && k.ok(); ++i) {
    const PackedConv b1 = k.pack(&bw[4 * i + 0], &bw[4 * i + 1], ch);
    const PackedConv b2 = k.pack(&bw[4 * i + 2], &bw[4 * i + 3], b1.cop);
    if (!k.ok()) break;
    if (b2.co != ch || b1.co % 8) return ERROR_INVALID_DIMS;
    DT t = k.tensor(x.H, x.W, b1.co);
    k.conv(b1, cat, prev, 1, (b1.kh - 1) / 2, kActSiLU, t, 0);
    k.conv(b2, t, 0, 1, (b2.kh - 1) / 2, kActSiLU, cat, (2 + i) * ch, shortcut ? &cat : nullptr, prev);
    prev = (2 + i) * ch;
  }
  const PackedConv p2 = k.pack(cv2_w, cv2_b, cat.Cp);
  DT y = k.tensor(x.H, x.W, p2.co);
  k.conv(p2, cat, 0, 1, 0, kActSiLU, y, 0);
  k.download(y, output);
  return k.finish("c3k2");
}

extern "C" status_t c3_forward(tensor_t* output, const tensor_t* input, const tensor_t* cv1_w, const tensor_t* cv1_b,
                               const tensor_t* cv2_w, const tensor_t* cv2_b, const tensor_t* cv3_w,
                               const tensor_t* cv3_b, const tensor_t* bw, int n_bottles, bool shortcut,
                               tensor_t* buffers) {
  if (!output || !input || !cv1_w || !cv1_b || !cv2_w || !cv2_b || !cv3_w || !cv3_b || !bw || !buffers)
    return ERROR_NULL_POINTER;
  const int cm = cv1_w->dims[0], c2 = cv2_w->dims[0];
  if (!all_mult8({input->dims[1], cm, c2, cv3_w->dims[0]}) || cv3_w->dims[1] != cm + c2) return ERROR_INVALID_DIMS;
  Kit k;
  DT x = k.upload(input);
  const PackedConv p1 = k.pack(cv1_w, cv1_b, x.Cp);
  const PackedConv p2 = k.pack(cv2_w, cv2_b, x.Cp);
  DT cat = k.tensor(x.H, x.W, cm + c2);
  DT y0 = k.tensor(x.H, x.W, cm);
  k.conv(p1, x, 0, 1, 0, kActSiLU, y0, 0);
  k.conv(p2, x, 0, 1, 0, kActSiLU, cat, cm);
  DT cur = y0;
  for (int i = 0; i < n_bottles && k.ok(); ++i) {
    const PackedConv b1 = k.pack(&bw[4 * i + 0], &bw[4 * i + 1], cm);
    const PackedConv b2 = k.pack(&bw[4 * i + 2], &bw[4 * i + 3], b1.cop);
    if (!k.ok()) break;
    if (b2.co != cm || b1.co % 8) return ERROR_INVALID_DIMS;
    DT t = k.tensor(x.H, x.W, b1.co);
    k.conv(b1, cur, 0, 1, (b1.kh - 1) / 2, kActSiLU, t, 0);
    if (i == n_bottles - 1) {
      k.conv(b2, t, 0, 1, (b2.kh - 1) / 2, kActSiLU, cat, 0, shortcut ? &cur : nullptr, 0);
    } else {
      DT nxt = k.tensor(x.H, x.W, cm);
      k.conv(b2, t, 0, 1, (b2.kh - 1) / 2, kActSiLU, nxt, 0, shortcut ? &cur : nullptr, 0);
      cur = nxt;
    }
  }
  if (n_bottles == 0 && k.ok())
    k.err = launch_gather_concat(y0.v(), cm, 1, y0.v(), 0, 1, x.H, x.W, cat.o(0), k.sc->stream);
  const PackedConv p3 = k.pack(cv3_w, cv3_b, cat.Cp);
  DT y = k.tensor(x.H, x.W, p3.co);
  k.conv(p3, cat, 0, 1, 0, kActSiLU, y, 0);
  k.download(y, output);
  return k.finish("c3");
}

extern "C" status_t sppf_forward(tensor_t* output, const tensor_t* input, const tensor_t* cv1_w,
                                 const tensor_t* cv1_b, const tensor_t* cv2_w, const tensor_t* cv2_b,
                                 int kernel_size, int n_pool, bool shortcut, tensor_t* buffers) {
  if (!output || !input || !cv1_w || !cv1_b || !cv2_w || !cv2_b || !buffers) return ERROR_NULL_POINTER;
  if (n_pool < 1) return ERROR_INVALID_DIMS;
  const int c = cv1_w->dims[0];
  if (!all_mult8({input->dims[1], c, cv2_w->dims[0]}) || cv2_w->dims[1] != c * (n_pool + 1)) return ERROR_INVALID_DIMS;
  Kit k;
  DT x = k.upload(input);
  const PackedConv p1 = k.pack(cv1_w, cv1_b, x.Cp);
  DT cat = k.tensor(x.H, x.W, c * (n_pool + 1));
  k.conv(p1, x, 0, 1, 0, kActNone, cat, 0);
  for (int j = 0; j < n_pool; ++j) k.pool(cat, j * c, kernel_size, 1, cat, (j + 1) * c, c);
  const PackedConv p2 = k.pack(cv2_w, cv2_b, cat.Cp);
  DT y = k.tensor(x.H, x.W, p2.co);
  const bool res = shortcut && input->dims[1] == output->dims[1] && input->dims[2] == output->dims[2] &&
                   input->dims[3] == output->dims[3];
  k.conv(p2, cat, 0, 1, 0, kActSiLU, y, 0, res ? &x : nullptr, 0);
  k.download(y, output);
  return k.finish("sppf");
}

extern "C" status_t psablock_forward(tensor_t* output, const tensor_t* input, bool shortcut, const tensor_t* qkv_w,
                                     const tensor_t* qkv_b, const tensor_t* proj_w, const tensor_t* proj_b,
                                     const tensor_t* pe_w, const tensor_t* pe_b, const tensor_t* ffn0_w,
                                     const tensor_t* ffn0_b, const tensor_t* ffn1_w, const tensor_t* ffn1_b,
                                     int num_heads, float attn_ratio) {
  if (!output || !input || !qkv_w || !qkv_b || !proj_w || !proj_b || !pe_w || !pe_b || !ffn0_w || !ffn0_b ||
      !ffn1_w || !ffn1_b)
    return ERROR_NULL_POINTER;
  const int c = input->dims[1];
  if (num_heads < 1 || c % num_heads || !all_mult8({c, ffn0_w->dims[0]})) return ERROR_INVALID_DIMS;
  const tensor_t w[10] = {*qkv_w, *qkv_b, *proj_w, *proj_b, *pe_w, *pe_b, *ffn0_w, *ffn0_b, *ffn1_w, *ffn1_b};
  Kit k;
  DT x = k.upload(input);
  DT y = k.tensor(x.H, x.W, c);
  psa_block(k, x, 0, c, w, num_heads, attn_ratio, y, 0, shortcut);
  k.download(y, output);
  return k.finish("psablock");
}

extern "C" status_t c2psa_forward(tensor_t* output, const tensor_t* input, int n_blocks, float e, float attn_ratio,
                                  const tensor_t* cv1_w, const tensor_t* cv1_b, const tensor_t* cv2_w,
                                  const tensor_t* cv2_b, const tensor_t* psa_weights, tensor_t* buffers) {
  if (!output || !input || !cv1_w || !cv1_b || !cv2_w || !cv2_b || !psa_weights || !buffers) return ERROR_NULL_POINTER;
  const int c1 = input->dims[1];
  const int ch = static_cast<int>(static_cast<float>(c1) * e);
  if (ch < 1 || n_blocks < 1 || cv1_w->dims[0] != 2 * ch || !all_mult8({c1, ch})) return ERROR_INVALID_DIMS;
  int heads = ch / 64;
  if (heads < 1) heads = 1;
  Kit k;
  DT x = k.upload(input);
  const PackedConv p1 = k.pack(cv1_w, cv1_b, x.Cp);
  DT cat = k.tensor(x.H, x.W, 2 * ch);
  k.conv(p1, x, 0, 1, 0, kActSiLU, cat, 0);
  for (int bi = 0; bi < n_blocks && k.ok(); ++bi) psa_block(k, cat, ch, ch, psa_weights + bi * 10, heads, attn_ratio, cat, ch, true);
  const PackedConv p2 = k.pack(cv2_w, cv2_b, cat.Cp);
  DT y = k.tensor(x.H, x.W, p2.co);
  k.conv(p2, cat, 0, 1, 0, kActSiLU, y, 0);
  k.download(y, output);
  return k.finish("c2psa");
}

// C = alpha * A[MxK] * B[KxN] + beta * C, through the 1x1 convolution: the
// N columns of B are pixels with K channels, the M rows of A are output
// channels.  alpha/beta are applied on the host after the copy back.
extern "C" status_t tensor_gemm(float* C, const float* A, const float* B, int M, int N, int K, float alpha, float beta) {
  if (!C || !A || !B) return ERROR_NULL_POINTER;
  if (M < 1 || N < 1 || K < 1) return ERROR_INVALID_DIMS;
  tensor_t x, w, y;
  x.dims[0] = 1;
  x.dims[1] = K;
  x.dims[2] = 1;
  x.dims[3] = N;
  x.data = const_cast<float*>(B);
  x.is_owner = false;
  w.dims[0] = M;
  w.dims[1] = K;
  w.dims[2] = 1;
  w.dims[3] = 1;
  w.data = const_cast<float*>(A);
  w.is_owner = false;
  std::vector<float> prod(static_cast<size_t>(M) * N);
  y.dims[0] = 1;
  y.dims[1] = M;
  y.dims[2] = 1;
  y.dims[3] = N;
  y.data = prod.data();
  y.is_owner = false;
  conv_params_t p = {1, 0, 1};
  status_t st = conv_block_forward(&y, &x, &w, nullptr, p, false);
  if (st != SUCCESS) return st;
  for (size_t i = 0; i < prod.size(); ++i) {
    const float base = beta == 0.0f ? 0.0f : beta * C[i];
    C[i] = alpha * prod[i] + base;
  }
  return SUCCESS;
}
