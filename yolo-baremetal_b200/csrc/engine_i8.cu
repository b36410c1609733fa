// INT8 plan of the YOLO26 forward: the same graph as Engine::build
// (model.c:764-903, detect.c:253-454) with int8 NHWC activations, the kind::i8
// convolution (conv_i8.cu) and the int8 CUDA-core kernels (simt_i8.cu).
//
// Quantisation is done here, on the host, from the engine's BN-folded fp32
// weights and a scale table (tensor name -> per-tensor scale):
//  - a conv named P writes tensor "P" (after its residual) and, with SiLU,
//    requantises to "P:pre" before the activation table;
//  - every tensor keeps one scale per channel, so a concat keeps its parts'
//    scales and its consumer folds them into its weights (w * s_c / s_ref,
//    s_ref = the scale of input channel 0) before per-output-channel
//    quantisation (s_w = max|w| / 127, round half to even);
//  - requantisation ratios become a 31-bit multiplier and a shift (frexp).
// Output channel counts are padded to multiples of 16 with zero weights;
// consumers read only the real channels.
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "engine.h"
#include "weight_prep.h"
#include "i8k.h"
#include "int8.h"
#include "kernels.h"

namespace yb {
namespace {

inline int round16(int c) { return (c + 15) / 16 * 16; }

// int8 NHWC tensor or channel slice; scales shared with the parent tensor.
struct QT {
  int8_t* base = nullptr;
  long long cstride = 0, bstride = 0;
  int c0 = 0, C = 0, H = 0, W = 0;
  std::shared_ptr<std::vector<float>> cs;
  int8_t* ptr() const { return base + c0; }
  float scale(int i) const { return (*cs)[c0 + i]; }
  void set_scale(float s) const {
    for (int i = 0; i < C; ++i) (*cs)[c0 + i] = s;
  }
  QT sub(int a, int n) const {
    QT v = *this;
    v.c0 = c0 + a;
    v.C = n;
    return v;
  }
  I8View view() const {
    I8View v;
    v.p = ptr();
    v.cstride = cstride;
    v.bstride = bstride;
    return v;
  }
};

// ratio -> (M, sh): ratio = M * 2^-sh, M in [2^30, 2^31); 0 / tiny -> (0, 1).
bool multiplier(double ratio, int32_t* m, int32_t* sh) {
  if (!(ratio > 0.0)) {
    *m = 0;
    *sh = 1;
    return true;
  }
  int e = 0;
  const double f = std::frexp(ratio, &e);
  long long mm = std::llrint(f * 2147483648.0);
  if (mm == 2147483648LL) {
    mm = 1073741824LL;
    e += 1;
  }
  const int s = 31 - e;
  if (s < 1) return false;
  if (s > 62) {
    *m = 0;
    *sh = 1;
    return true;
  }
  *m = static_cast<int32_t>(mm);
  *sh = s;
  return true;
}

void silu_lut(int8_t* lut, double s_pre, double s_out) {
  for (int i = 0; i < 256; ++i) {
    const double x = static_cast<double>(i - 128) * s_pre;
    const double y = x / (1.0 + std::exp(-x));
    const long long q = std::llrint(y / s_out);
    lut[i] = static_cast<int8_t>(q < -127 ? -127 : q > 127 ? 127 : q);
  }
}

struct QWeights {
  std::vector<int8_t> wq;  // [co][ci][kh][kw]
  std::vector<int32_t> bq, mult, shift;
  std::vector<float> deq;
};

// Per-output-channel quantisation of w [co][ci][kh][kw] for an input whose
// channel c has scale cs[c]; requantisation target s_t (0: dequantised).
bool quantize(const HostTensor& w, const HostTensor* b, const float* cs, double s_t, QWeights* q) {
  const int co = w.dims[0], ci = w.dims[1], kk = w.dims[2] * w.dims[3];
  const int per = ci * kk;
  const float s_ref = cs[0];
  q->wq.assign(static_cast<size_t>(co) * per, 0);
  q->bq.assign(co, 0);
  q->mult.assign(co, 0);
  q->shift.assign(co, 1);
  q->deq.assign(co, 0.f);
  std::vector<float> we(per);
  for (int o = 0; o < co; ++o) {
    float m = 0.0f;
    for (int i = 0; i < ci; ++i)
      for (int k = 0; k < kk; ++k) {
        const int idx = i * kk + k;
        we[idx] = static_cast<float>(static_cast<double>(w.data[static_cast<size_t>(o) * per + idx]) *
                                     static_cast<double>(cs[i]) / static_cast<double>(s_ref));
        if (std::fabs(we[idx]) > m) m = std::fabs(we[idx]);
      }
    const float sw = m > 0.0f ? m / 127.0f : 1.0f;
    for (int idx = 0; idx < per; ++idx) {
      const float v = std::nearbyint(we[idx] / sw);
      q->wq[static_cast<size_t>(o) * per + idx] = static_cast<int8_t>(v < -127.0f ? -127 : v > 127.0f ? 127 : static_cast<int>(v));
    }
    long long bv = b ? std::llrint(static_cast<double>(b->data[o]) / (static_cast<double>(s_ref) * static_cast<double>(sw)))
                     : 0;
    bv = bv < -2147483647LL ? -2147483647LL : bv > 2147483647LL ? 2147483647LL : bv;
    q->bq[o] = static_cast<int32_t>(bv);
    q->deq[o] = static_cast<float>(static_cast<double>(s_ref) * static_cast<double>(sw));
    if (s_t > 0.0 && !multiplier(static_cast<double>(s_ref) * static_cast<double>(sw) / s_t, &q->mult[o], &q->shift[o]))
      return false;
  }
  return true;
}

}  // namespace

cudaError_t Engine::build_i8(Plan* p, std::string* why) {
  const int B = p->B, H = p->H, W = p->W;
  const int nc = nc_;
  cudaError_t e = i8_init_kernel();
  if (e != cudaSuccess) return e;
#define YB_TRY(x)                            \
  do {                                       \
    cudaError_t e_ = (x);                    \
    if (e_ != cudaSuccess) return e_;        \
  } while (0)
  auto fail = [&](const std::string& m) {
    *why = m;
    return cudaErrorInvalidValue;
  };
  auto scale = [&](const std::string& n, float* s) -> bool {
    auto it = i8_scales_.find(n);
    if (it == i8_scales_.end() || !(it->second > 0.0f)) {
      *why = "int8 scale missing or not positive: " + n;
      return false;
    }
    *s = it->second;
    return true;
  };
  auto dalloc = [&](size_t bytes, void** q) -> cudaError_t {
    cudaError_t r = cudaMalloc(q, bytes < 256 ? 256 : bytes);
    if (r == cudaSuccess) {
      p->allocs.push_back(*q);
      r = cudaMemset(*q, 0, bytes < 256 ? 256 : bytes);
    }
    return r;
  };
  auto upload = [&](const void* src, size_t bytes, void** dst) -> cudaError_t {
    cudaError_t r = dalloc(bytes, dst);
    if (r == cudaSuccess && bytes) r = cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice);
    return r;
  };
  auto tensor = [&](int C, int h, int w, QT* t) -> cudaError_t {
    t->C = C;
    t->H = h;
    t->W = w;
    t->c0 = 0;
    t->cstride = round16(C);
    t->bstride = static_cast<long long>(h) * w * t->cstride;
    t->cs = std::make_shared<std::vector<float>>(C, 0.f);
    void* q = nullptr;
    cudaError_t r = dalloc(static_cast<size_t>(B) * t->bstride, &q);
    t->base = static_cast<int8_t*>(q);
    return r;
  };
  // Device weight preparation: quantises w (device values) per output
  // channel with the same rule as quantize(), into plan-owned device arrays.
  struct QDev {
    int8_t* wq = nullptr;
    int32_t *bq = nullptr, *mult = nullptr, *shift = nullptr;
    float* deq = nullptr;
  };
  auto quantize_dev = [&](const HostTensor& w, const HostTensor* b, const float* cs, int ncs, bool per_out,
                          double s_t, QDev* q) -> cudaError_t {
    const int co = w.dims[0], kk = w.dims[2] * w.dims[3];
    const int per = static_cast<int>(w.count() / static_cast<size_t>(co));
    void *wq = nullptr, *bq = nullptr, *mu = nullptr, *sh = nullptr, *dq = nullptr, *dcs = nullptr, *bad = nullptr;
    YB_TRY(dalloc(static_cast<size_t>(co) * per, &wq));
    YB_TRY(dalloc(static_cast<size_t>(co) * 4, &bq));
    YB_TRY(dalloc(static_cast<size_t>(co) * 4, &mu));
    YB_TRY(dalloc(static_cast<size_t>(co) * 4, &sh));
    YB_TRY(dalloc(static_cast<size_t>(co) * 4, &dq));
    YB_TRY(upload(cs, static_cast<size_t>(ncs) * 4, &dcs));
    YB_TRY(dalloc(4, &bad));
    // dalloc clears on the legacy stream; this plan's stream does not wait
    // for it, so finish those before the kernel writes.
    YB_TRY(cudaDeviceSynchronize());
    QuantArgs qa;
    qa.w = w.dev;
    qa.b = b ? b->dev : nullptr;
    qa.cs = static_cast<const float*>(dcs);
    qa.co = co;
    qa.ci = per / kk;
    qa.kk = kk;
    qa.per_out = per_out ? 1 : 0;
    qa.s_t = s_t;
    qa.wq = static_cast<int8_t*>(wq);
    qa.bq = static_cast<int32_t*>(bq);
    qa.mult = static_cast<int32_t*>(mu);
    qa.shift = static_cast<int32_t*>(sh);
    qa.deq = static_cast<float*>(dq);
    qa.bad = static_cast<int*>(bad);
    YB_TRY(launch_quantize_i8(qa, stream_));
    int hbad = 0;
    YB_TRY(cudaMemcpyAsync(&hbad, bad, 4, cudaMemcpyDeviceToHost, stream_));
    YB_TRY(cudaStreamSynchronize(stream_));
    if (hbad) return cudaErrorInvalidValue;
    q->wq = qa.wq;
    q->bq = qa.bq;
    q->mult = qa.mult;
    q->shift = qa.shift;
    q->deq = qa.deq;
    return cudaSuccess;
  };
  // Copies n device int32 values into a new array of `slots` entries whose
  // remaining entries hold `fill`.
  auto padded_i32 = [&](const int32_t* src, int n, int slots, int32_t fill, void** dst) -> cudaError_t {
    std::vector<int32_t> h(static_cast<size_t>(slots), fill);
    YB_TRY(upload(h.data(), h.size() * 4, dst));
    return cudaMemcpy(*dst, src, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToDevice);
  };
  i8_images_.clear();
  const int sms = num_sms_;
  int step = 0;  // profile step (model_forward_profile_t index)
  auto add_op = [&](int kind, double flops, double bytes, std::function<cudaError_t(cudaStream_t)> fn) {
    Op op{step, std::move(fn)};
    op.kind = kind;
    op.flops = flops;
    op.bytes = bytes;
    p->ops.push_back(std::move(op));
  };
  struct F32Out {
    float* ptr = nullptr;
    long long cstride = 0, bstride = 0;
    float* rowmax = nullptr;  // sigmoid of each pixel's largest output
    long long rm_bstride = 0;
  };
  // Convolution named P (P.conv.* or, plain, P.*) from `in` into `out`
  // (or dequantised into f32 when f32.ptr).  With `cap` the launch
  // arguments are returned there instead of adding the launch.
  auto conv = [&](const std::string& P, bool plain, const QT& out, const QT& in, int stride, int pad, bool act,
                  const QT* res, F32Out f32 = F32Out(), I8Args* cap = nullptr) -> cudaError_t {
    const HostTensor* w = find(P + (plain ? ".weight" : ".conv.weight"));
    const HostTensor* b = find(P + (plain ? ".bias" : ".conv.bias"));
    if (!w || w->ndim != 4) return fail("int8: missing weight " + P);
    const int co = w->dims[0], ci = w->dims[1], k = w->dims[2];
    if (ci != in.C || w->dims[3] != k || (k != 1 && k != 3)) return fail("int8: conv shape " + P);
    if (!f32.ptr && co != out.C) return fail("int8: conv output width " + P);
    float s_out = 0.f, s_pre = 0.f;
    if (!f32.ptr && !scale(P, &s_out)) return cudaErrorInvalidValue;
    if (act && !scale(P + ":pre", &s_pre)) return cudaErrorInvalidValue;
    std::vector<float> cs(ci);
    for (int i = 0; i < ci; ++i) cs[i] = in.scale(i);
    const double s_t = f32.ptr ? 0.0 : act ? static_cast<double>(s_pre) : static_cast<double>(s_out);
    QWeights q;
    QDev qd;
    if (w->dev) {
      const cudaError_t r = quantize_dev(*w, b, cs.data(), ci, false, s_t, &qd);
      if (r == cudaErrorInvalidValue) return fail("int8: requantisation ratio out of range in " + P);
      YB_TRY(r);
    } else if (!quantize(*w, b, cs.data(), s_t, &q)) {
      return fail("int8: requantisation ratio out of range in " + P);
    }
    const int co_pad = round16(co);
    // Padded channels write zeros, so they must land in the tensor's own
    // channel padding, not in a neighbouring concat slice.
    if (!f32.ptr && co_pad != co && (out.c0 != 0 || out.cstride != co_pad))
      return fail("int8: padded output must own its tensor: " + P);
    I8Tiling t;
    if (k == 3 && stride == 1 && pad == 1 && ci <= 16 && co_pad <= 128 && !f32.ptr) i8_tiling_pair(co_pad, &t);
    else if (k == 3 && stride == 2 && pad == 1 && ci <= 16 && co_pad <= 128 && !f32.ptr) i8_tiling_pair_s2(co_pad, &t);
    else i8_tiling(co_pad, ci, k, k, &t);
    if (t.ci_pad != 16) {
      // Fewer than two waves of tiles: narrower N tiles (64 or 128 columns)
      // so that more SMs share the work.
      const int ho = (in.H + 2 * pad - k) / stride + 1, wo = (in.W + 2 * pad - k) / stride + 1;
      const long long mt = (static_cast<long long>(B) * ho * wo + 127) / 128;
      if (mt * t.n_tiles < 2LL * sms && co_pad >= 128 && !f32.ptr) {
        const int nt = mt * ((co_pad + 127) / 128) >= 2LL * sms ? 128 : 64;
        t.n_tile = nt;
        t.n_tiles = (co_pad + nt - 1) / nt;
      }
    }
    const int nq = i8_bias_slots(t);
    void *dw = nullptr, *db = nullptr, *dm = nullptr, *ds = nullptr, *dd = nullptr, *dl = nullptr;
    size_t pk_bytes = 0;
    if (w->dev) {
      pk_bytes = static_cast<size_t>(t.n_tiles) * t.num_kc * t.n_tile * 128;
      YB_TRY(dalloc(pk_bytes, &dw));
      YB_TRY(cudaDeviceSynchronize());
      YB_TRY(launch_pack_i8(qd.wq, co, ci, k, k, t, static_cast<uint8_t*>(dw), pk_bytes, stream_));
      YB_TRY(cudaStreamSynchronize(stream_));
      YB_TRY(padded_i32(qd.bq, co, nq, 0, &db));
      YB_TRY(padded_i32(qd.mult, co, nq, 0, &dm));
      YB_TRY(padded_i32(qd.shift, co, nq, 1, &ds));
      if (f32.ptr) {
        YB_TRY(dalloc(static_cast<size_t>(nq) * 4, &dd));
        YB_TRY(cudaMemcpy(dd, qd.deq, static_cast<size_t>(co) * 4, cudaMemcpyDeviceToDevice));
      }
    } else {
      std::vector<int8_t> wpad(static_cast<size_t>(co_pad) * ci * k * k, 0);
      std::copy(q.wq.begin(), q.wq.end(), wpad.begin());
      const std::vector<uint8_t> pk = i8_pack_weights(wpad.data(), co_pad, ci, k, k, t);
      std::vector<int32_t> hb(nq, 0), hm(nq, 0), hs(nq, 1);
      std::vector<float> hd(nq, 0.f);
      for (int i = 0; i < co; ++i) {
        hb[i] = q.bq[i];
        hm[i] = q.mult[i];
        hs[i] = q.shift[i];
        hd[i] = q.deq[i];
      }
      pk_bytes = pk.size();
      YB_TRY(upload(pk.data(), pk.size(), &dw));
      YB_TRY(upload(hb.data(), hb.size() * 4, &db));
      YB_TRY(upload(hm.data(), hm.size() * 4, &dm));
      YB_TRY(upload(hs.data(), hs.size() * 4, &ds));
      if (f32.ptr) YB_TRY(upload(hd.data(), hd.size() * 4, &dd));
    }
    i8_images_[P] = {static_cast<const uint8_t*>(dw), pk_bytes};
    if (act) {
      int8_t lut[256];
      silu_lut(lut, s_pre, s_out);
      YB_TRY(upload(lut, 256, &dl));
    }
    I8Args a;
    a.B = B;
    a.H = in.H;
    a.W = in.W;
    a.Ci = ci;
    a.Co = co_pad;
    a.kh = a.kw = k;
    a.stride = stride;
    a.pad = pad;
    a.Ho = (in.H + 2 * pad - k) / stride + 1;
    a.Wo = (in.W + 2 * pad - k) / stride + 1;
    if (!f32.ptr && (a.Ho != out.H || a.Wo != out.W)) return fail("int8: conv output size " + P);
    a.K = t.K;
    a.num_kc = t.num_kc;
    a.n_tile = t.n_tile;
    a.n_tiles = t.n_tiles;
    a.m_tiles = static_cast<int>((static_cast<long long>(B) * a.Ho * a.Wo + 127) / 128);
    a.a_cpp = t.a_cpp;
    a.tap_perm = t.tap_perm;
    a.wpack = static_cast<const uint8_t*>(dw);
    a.bias = static_cast<const int32_t*>(db);
    a.mult = static_cast<const int32_t*>(dm);
    a.shift = static_cast<const int32_t*>(ds);
    a.lut = static_cast<const int8_t*>(dl);
    if (f32.ptr) {
      a.out_f32 = f32.ptr;
      a.f32_cstride = f32.cstride;
      a.f32_bstride = f32.bstride;
      a.f32_co = co;
      a.deq = static_cast<const float*>(dd);
      a.rowmax = f32.rowmax;
      a.rm_bstride = f32.rm_bstride;
    } else {
      a.out = out.base;
      a.out_cstride = out.cstride;
      a.out_coff = out.c0;
    }
    if (res) {
      if (res->C != co || res->H != a.Ho || res->W != a.Wo) return fail("int8: residual shape " + P);
      a.res = res->base;
      a.res_cstride = res->cstride;
      a.res_coff = res->c0;
      if (!multiplier(static_cast<double>(res->scale(0)) / static_cast<double>(s_out), &a.res_mult, &a.res_shift))
        return fail("int8: residual ratio out of range in " + P);
    }
    a.err = d_err_;
    if (cap) {
      *cap = a;
      if (!f32.ptr) out.set_scale(s_out);
      return cudaSuccess;
    }
    const int8_t* x = in.ptr();
    const long long xc = in.cstride, xb = in.bstride;
    const double px = static_cast<double>(B) * a.Ho * a.Wo;
    add_op(kOpConv, 2.0 * px * co * ci * k * k,
           static_cast<double>(B) * in.H * in.W * ci + px * co * (f32.ptr ? 4.0 : 1.0) + 1.0 * co * ci * k * k,
           [a, x, xc, xb, sms](cudaStream_t st) mutable { return launch_conv_i8(a, x, xc, xb, st, sms, nullptr); });
    if (!f32.ptr) out.set_scale(s_out);
    return cudaSuccess;
  };
  // Depthwise 3x3 + SiLU named P (Detect class branch).
  auto dwconv = [&](const std::string& P, const QT& out, const QT& in) -> cudaError_t {
    const HostTensor* w = find(P + ".conv.weight");
    const HostTensor* b = find(P + ".conv.bias");
    const int C = in.C;
    if (!w || w->dims[0] != C || w->dims[2] != 3 || C % 16) return fail("int8: depthwise " + P);
    float s_out = 0.f, s_pre = 0.f;
    if (!scale(P, &s_out) || !scale(P + ":pre", &s_pre)) return cudaErrorInvalidValue;
    void *dw = nullptr, *db = nullptr, *dm = nullptr, *ds = nullptr, *dl = nullptr;
    if (w->dev) {
      std::vector<float> cs(C);
      for (int c = 0; c < C; ++c) cs[c] = in.scale(c);
      QDev qd;
      const cudaError_t r = quantize_dev(*w, b, cs.data(), C, true, s_pre, &qd);
      if (r == cudaErrorInvalidValue) return fail("int8: depthwise ratio " + P);
      YB_TRY(r);
      YB_TRY(dalloc(static_cast<size_t>(3) * C * 4, &dw));
      YB_TRY(cudaDeviceSynchronize());
      YB_TRY(launch_pack_dw_i8(qd.wq, C, static_cast<uint32_t*>(dw), stream_));
      YB_TRY(cudaStreamSynchronize(stream_));
      db = qd.bq;
      dm = qd.mult;
      ds = qd.shift;
    }
    std::vector<uint32_t> wt(static_cast<size_t>(3) * C, 0u);
    std::vector<int32_t> bq(C), mu(C), sh(C);
    for (int c = 0; c < C && !w->dev; ++c) {
      HostTensor wc;
      wc.dims[0] = 1;
      wc.dims[1] = 1;
      wc.dims[2] = 3;
      wc.dims[3] = 3;
      wc.ndim = 4;
      wc.data.assign(w->data.begin() + c * 9, w->data.begin() + c * 9 + 9);
      HostTensor bc;
      if (b) bc.data.assign(1, b->data[c]);
      const float sc = in.scale(c);
      QWeights q;
      if (!quantize(wc, b ? &bc : nullptr, &sc, s_pre, &q)) return fail("int8: depthwise ratio " + P);
      // One word per filter row: wt[ky][c] byte kx = tap (ky, kx).
      for (int k = 0; k < 9; ++k)
        wt[static_cast<size_t>(k / 3) * C + c] |= (static_cast<uint32_t>(q.wq[k]) & 0xFFu) << (8 * (k % 3));
      bq[c] = q.bq[0];
      mu[c] = q.mult[0];
      sh[c] = q.shift[0];
    }
    int8_t lut[256];
    silu_lut(lut, s_pre, s_out);
    if (!w->dev) {
      YB_TRY(upload(wt.data(), wt.size() * 4, &dw));
      YB_TRY(upload(bq.data(), bq.size() * 4, &db));
      YB_TRY(upload(mu.data(), mu.size() * 4, &dm));
      YB_TRY(upload(sh.data(), sh.size() * 4, &ds));
    }
    YB_TRY(upload(lut, 256, &dl));
    const I8View iv = in.view(), ovw = out.view();
    const int h = in.H, wd = in.W;
    add_op(kOpDw, 18.0 * B * h * wd * C, 2.0 * B * h * wd * C, [=](cudaStream_t st) {
      return launch_dw3x3_i8(iv, ovw, B, h, wd, C, static_cast<const uint32_t*>(dw), static_cast<const int32_t*>(db),
                             static_cast<const int32_t*>(dm), static_cast<const int32_t*>(ds),
                             static_cast<const int8_t*>(dl), st);
    });
    out.set_scale(s_out);
    return cudaSuccess;
  };
  auto wdim0 = [&](const std::string& n) -> int {
    const HostTensor* t = find(n);
    return t ? t->dims[0] : 0;
  };
  // Bottleneck (layers.c:92-108).  With 3x3 convolutions C -> CM -> C of
  // the shapes bottleneck_i8.cu fuses and a shortcut, one launch keeping the
  // int8 intermediate in shared memory (bit-identical) unless fusion is off.
  auto bottleneck = [&](const std::string& P, const QT& out, const QT& in, bool shortcut) -> cudaError_t {
    const HostTensor* w1 = find(P + ".cv1.conv.weight");
    const HostTensor* w2 = find(P + ".cv2.conv.weight");
    if (!w1 || !w2) return fail("int8: missing " + P);
    QT t;
    YB_TRY(tensor(w1->dims[0], in.H, in.W, &t));
    const int C = in.C, CM = w1->dims[0];
    if (fuse_ && shortcut && w1->ndim == 4 && w2->ndim == 4 && w1->dims[1] == C && w1->dims[2] == 3 &&
        w1->dims[3] == 3 && w2->dims[0] == C && w2->dims[1] == CM && w2->dims[2] == 3 && w2->dims[3] == 3 &&
        out.C == C && out.H == in.H && out.W == in.W && i8_bottleneck_supported(C, CM)) {
      I8Args a1, a2;
      YB_TRY(conv(P + ".cv1", false, t, in, 1, 1, true, nullptr, F32Out(), &a1));
      YB_TRY(conv(P + ".cv2", false, out, t, 1, 1, true, &in, F32Out(), &a2));
      I8BottleneckArgs f;
      f.B = B;
      f.H = in.H;
      f.W = in.W;
      f.C = C;
      f.CM = CM;
      f.in = in.ptr();
      f.in_cstride = in.cstride;
      f.in_bstride = in.bstride;
      f.out = out.ptr();
      f.out_cstride = out.cstride;
      f.out_bstride = out.bstride;
      f.w1 = a1.wpack;
      f.b1 = a1.bias;
      f.m1 = a1.mult;
      f.s1 = a1.shift;
      f.lut1 = a1.lut;
      f.w2 = a2.wpack;
      f.b2 = a2.bias;
      f.m2 = a2.mult;
      f.s2 = a2.shift;
      f.lut2 = a2.lut;
      f.res_mult = a2.res_mult;
      f.res_shift = a2.res_shift;
      f.err = d_err_;
      if (a1.n_tiles != 1 || a2.n_tiles != 1 || !i8_bottleneck_setup(&f)) return fail("int8: fused bottleneck " + P);
      const double px = static_cast<double>(B) * in.H * in.W;
      add_op(kOpConv, 2.0 * 2.0 * px * C * CM * 9.0, 2.0 * px * C + 18.0 * C * CM,
             [f, sms](cudaStream_t st) { return launch_i8_bottleneck(f, st, sms); });
      return cudaSuccess;
    }
    YB_TRY(conv(P + ".cv1", false, t, in, 1, (w1->dims[2] - 1) / 2, true, nullptr));
    return conv(P + ".cv2", false, out, t, 1, (w2->dims[2] - 1) / 2, true, shortcut ? &in : nullptr);
  };
  auto c3k2_plain = [&](const std::string& L, int n, bool shortcut, const QT& out, const QT& in) -> cudaError_t {
    const int ct = wdim0(L + ".cv1.conv.weight"), ch = ct / 2;
    if (!ct) return fail("int8: missing " + L);
    QT cat;
    YB_TRY(tensor((2 + n) * ch, in.H, in.W, &cat));
    YB_TRY(conv(L + ".cv1", false, cat.sub(0, ct), in, 1, 0, true, nullptr));
    for (int i = 0; i < n; ++i)
      YB_TRY(bottleneck(L + ".m." + std::to_string(i), cat.sub((2 + i) * ch, ch),
                        cat.sub(i == 0 ? ch : (1 + i) * ch, ch), shortcut));
    return conv(L + ".cv2", false, out, cat, 1, 0, true, nullptr);
  };
  auto c3 = [&](const std::string& P, const QT& out, const QT& in) -> cudaError_t {
    const int cm = wdim0(P + ".cv1.conv.weight"), c2 = wdim0(P + ".cv2.conv.weight");
    if (!cm || !c2) return fail("int8: missing " + P);
    QT cat, y, z;
    YB_TRY(tensor(cm + c2, in.H, in.W, &cat));
    YB_TRY(conv(P + ".cv2", false, cat.sub(cm, c2), in, 1, 0, true, nullptr));
    int nb = 0;
    while (find(P + ".m." + std::to_string(nb) + ".cv1.conv.weight")) ++nb;
    if (nb == 0) {
      YB_TRY(conv(P + ".cv1", false, cat.sub(0, cm), in, 1, 0, true, nullptr));
    } else {
      YB_TRY(tensor(cm, in.H, in.W, &y));
      YB_TRY(conv(P + ".cv1", false, y, in, 1, 0, true, nullptr));
      QT cur = y;
      for (int i = 0; i < nb; ++i) {
        QT nxt;
        if (i == nb - 1) {
          nxt = cat.sub(0, cm);
        } else {
          YB_TRY(tensor(cm, in.H, in.W, &z));
          nxt = z;
        }
        YB_TRY(bottleneck(P + ".m." + std::to_string(i), nxt, cur, true));
        cur = nxt;
      }
    }
    return conv(P + ".cv3", false, out, cat, 1, 0, true, nullptr);
  };
  auto c3k2_c3k = [&](const std::string& L, const QT& out, const QT& in) -> cudaError_t {
    const int ch = wdim0(L + ".cv1.conv.weight") / 2, c3o = wdim0(L + ".m.0.cv3.conv.weight");
    if (!ch || !c3o) return fail("int8: missing " + L);
    int n = 0;
    while (find(L + ".m." + std::to_string(n) + ".cv3.conv.weight")) ++n;
    QT cat;
    YB_TRY(tensor(2 * ch + n * c3o, in.H, in.W, &cat));
    YB_TRY(conv(L + ".cv1", false, cat.sub(0, 2 * ch), in, 1, 0, true, nullptr));
    for (int i = 0; i < n; ++i)
      YB_TRY(c3(L + ".m." + std::to_string(i), cat.sub(2 * ch + i * c3o, c3o),
                i == 0 ? cat.sub(ch, ch) : cat.sub(2 * ch + (i - 1) * c3o, c3o)));
    return conv(L + ".cv2", false, out, cat, 1, 0, true, nullptr);
  };
  auto sppf = [&](const std::string& L, const QT& out, const QT& in) -> cudaError_t {
    const int c = wdim0(L + ".cv1.conv.weight");
    if (!c || c % 16) return fail("int8: sppf " + L);
    QT cat;
    YB_TRY(tensor(4 * c, in.H, in.W, &cat));
    YB_TRY(conv(L + ".cv1", false, cat.sub(0, c), in, 1, 0, false, nullptr));
    const bool fused = sppf_pool_i8_smem_bytes(in.H, in.W) <= kSppfI8SmemMax;
    if (fused) {
      // The three pools in one launch (the 5x5, 9x9 and 13x13 pools of cv1).
      const I8View iv = cat.sub(0, c).view(), v1 = cat.sub(c, c).view(), v2 = cat.sub(2 * c, c).view(),
                   v3 = cat.sub(3 * c, c).view();
      const int h = in.H, wd = in.W;
      add_op(kOpPool, 0.0, 4.0 * B * h * wd * c,
             [=](cudaStream_t st) { return launch_sppf_pool_i8(iv, v1, v2, v3, B, h, wd, c, st); });
    }
    for (int j = 0; j < 3; ++j) {
      const QT src = cat.sub(j * c, c), dst = cat.sub((j + 1) * c, c);
      if (!fused) {
        const I8View iv = src.view(), ovw = dst.view();
        const int h = in.H, wd = in.W;
        add_op(kOpPool, 0.0, 2.0 * B * h * wd * c,
               [=](cudaStream_t st) { return launch_maxpool_i8(iv, ovw, B, h, wd, c, 5, st); });
      }
      for (int i = 0; i < c; ++i) (*cat.cs)[cat.c0 + (j + 1) * c + i] = src.scale(i);
    }
    return conv(L + ".cv2", false, out, cat, 1, 0, true, (in.C == out.C) ? &in : nullptr);
  };
  auto psablock = [&](const std::string& P, int heads, const QT& out, const QT& in) -> cudaError_t {
    const int dim = in.C, hd = dim / heads, kd = static_cast<int>(static_cast<float>(hd) * 0.5f);
    const int cq = wdim0(P + ".attn.qkv.conv.weight"), cf = wdim0(P + ".ffn.0.conv.weight");
    if (dim % heads || cq != dim + 2 * kd * heads || !cf) return fail("int8: psa " + P);
    QT qkv, ope, x1, f;
    YB_TRY(tensor(cq, in.H, in.W, &qkv));
    YB_TRY(conv(P + ".attn.qkv", false, qkv, in, 1, 0, false, nullptr));
    YB_TRY(tensor(dim, in.H, in.W, &ope));
    float s_ope = 0.f;
    if (!scale(P + ".attn.ope", &s_ope)) return cudaErrorInvalidValue;
    const double s_qkv = qkv.scale(0);
    I8AttnArgs aa;
    aa.qkv = qkv.view();
    aa.out = ope.view();
    aa.B = B;
    aa.H = in.H;
    aa.W = in.W;
    aa.heads = heads;
    aa.kd = kd;
    aa.hd = hd;
    aa.dim = dim;
    if (!multiplier(s_qkv * s_qkv / std::sqrt(static_cast<double>(kd)) * 16.0, &aa.mt, &aa.sht) ||
        !multiplier(s_qkv / static_cast<double>(s_ope), &aa.mo, &aa.sho))
      return fail("int8: attention ratio out of range in " + P);
    int32_t E[256];
    for (int t = 0; t < 256; ++t) E[t] = static_cast<int32_t>(std::llrint(4096.0 * std::exp(-static_cast<double>(t) / 16.0)));
    const HostTensor* pw = find(P + ".attn.pe.conv.weight");
    const HostTensor* pb = find(P + ".attn.pe.conv.bias");
    if (!pw || pw->dims[0] != dim) return fail("int8: missing pe " + P);
    std::vector<int8_t> wt(static_cast<size_t>(9) * dim);
    std::vector<int32_t> bq(dim), mu(dim), sh(dim);
    const float sv = static_cast<float>(s_qkv);
    void *dE = nullptr, *dw = nullptr, *db = nullptr, *dm = nullptr, *ds = nullptr;
    if (pw->dev) {
      QDev qd;
      const cudaError_t r = quantize_dev(*pw, pb, &sv, 1, false, static_cast<double>(s_ope), &qd);
      if (r == cudaErrorInvalidValue) return fail("int8: pe ratio " + P);
      YB_TRY(r);
      YB_TRY(dalloc(static_cast<size_t>(9) * dim, &dw));
      YB_TRY(cudaDeviceSynchronize());
      YB_TRY(launch_pack_pe_i8(qd.wq, dim, static_cast<int8_t*>(dw), stream_));
      YB_TRY(cudaStreamSynchronize(stream_));
      db = qd.bq;
      dm = qd.mult;
      ds = qd.shift;
    }
    for (int c = 0; c < dim && !pw->dev; ++c) {
      HostTensor wc;
      wc.dims[0] = wc.dims[1] = 1;
      wc.dims[2] = wc.dims[3] = 3;
      wc.ndim = 4;
      wc.data.assign(pw->data.begin() + c * 9, pw->data.begin() + c * 9 + 9);
      HostTensor bc;
      if (pb) bc.data.assign(1, pb->data[c]);
      QWeights q;
      if (!quantize(wc, pb ? &bc : nullptr, &sv, static_cast<double>(s_ope), &q)) return fail("int8: pe ratio " + P);
      for (int k = 0; k < 9; ++k) wt[static_cast<size_t>(k) * dim + c] = q.wq[k];
      bq[c] = q.bq[0];
      mu[c] = q.mult[0];
      sh[c] = q.shift[0];
    }
    YB_TRY(upload(E, sizeof E, &dE));
    if (!pw->dev) {
      YB_TRY(upload(wt.data(), wt.size(), &dw));
      YB_TRY(upload(bq.data(), bq.size() * 4, &db));
      YB_TRY(upload(mu.data(), mu.size() * 4, &dm));
      YB_TRY(upload(sh.data(), sh.size() * 4, &ds));
    }
    aa.E = static_cast<const int32_t*>(dE);
    aa.pe_w = static_cast<const int8_t*>(dw);
    aa.pe_bq = static_cast<const int32_t*>(db);
    aa.pe_mult = static_cast<const int32_t*>(dm);
    aa.pe_shift = static_cast<const int32_t*>(ds);
    aa.err = d_err_;
    const double N = static_cast<double>(in.H) * in.W;
    add_op(kOpAttn, 2.0 * B * heads * N * N * (kd + hd), static_cast<double>(B) * N * (cq + dim),
           [aa](cudaStream_t st) { return launch_attention_i8(aa, st); });
    ope.set_scale(s_ope);
    YB_TRY(tensor(dim, in.H, in.W, &x1));
    YB_TRY(conv(P + ".attn.proj", false, x1, ope, 1, 0, false, &in));
    YB_TRY(tensor(cf, in.H, in.W, &f));
    YB_TRY(conv(P + ".ffn.0", false, f, x1, 1, 0, true, nullptr));
    return conv(P + ".ffn.1", false, out, f, 1, 0, false, &x1);
  };
  auto heads_for = [](int ch) { return ch / 64 < 1 ? 1 : ch / 64; };
  auto c2psa = [&](const std::string& L, const QT& out, const QT& in) -> cudaError_t {
    const int ch = static_cast<int>(static_cast<float>(in.C) * 0.5f);
    QT cat, t;
    YB_TRY(tensor(2 * ch, in.H, in.W, &cat));
    YB_TRY(conv(L + ".cv1", false, cat, in, 1, 0, true, nullptr));
    YB_TRY(tensor(ch, in.H, in.W, &t));
    YB_TRY(psablock(L + ".m.0", heads_for(ch), t, cat.sub(ch, ch)));
    // The block's output replaces b in the concat (layers.c:489).
    const QT bdst = cat.sub(ch, ch);
    const I8View sv = t.view(), dv = bdst.view();
    const int h = in.H, wd = in.W;
    add_op(kOpPool, 0.0, 2.0 * B * h * wd * ch, [=](cudaStream_t st) {
      return launch_concat_i8(sv, ch, 0, I8View(), 0, B, h, wd, dv, st);
    });
    for (int i = 0; i < ch; ++i) (*cat.cs)[cat.c0 + ch + i] = t.scale(i);
    return conv(L + ".cv2", false, out, cat, 1, 0, true, nullptr);
  };
  auto c3k2_attn = [&](const std::string& L, const QT& out, const QT& in) -> cudaError_t {
    const int ch = wdim0(L + ".cv1.conv.weight") / 2;
    if (!ch) return fail("int8: missing " + L);
    QT cat, bo;
    YB_TRY(tensor(3 * ch, in.H, in.W, &cat));
    YB_TRY(conv(L + ".cv1", false, cat.sub(0, 2 * ch), in, 1, 0, true, nullptr));
    YB_TRY(tensor(ch, in.H, in.W, &bo));
    YB_TRY(bottleneck(L + ".m.0.0", bo, cat.sub(ch, ch), true));
    YB_TRY(psablock(L + ".m.0.1", heads_for(ch), cat.sub(2 * ch, ch), bo));
    return conv(L + ".cv2", false, out, cat, 1, 0, true, nullptr);
  };
  // 2x nearest upsample of a into channels [0, a.C) of cat (the rest of cat
  // was written by the layer that produced it).
  auto upsample_into = [&](const QT& a, const QT& cat) -> cudaError_t {
    if (cat.C < a.C || cat.c0 != 0) return fail("int8: upsample target");
    const I8View av = a.view(), ov = cat.view();
    const int ca = a.C, h = cat.H, wd = cat.W;
    add_op(kOpPool, 0.0, 2.0 * B * h * wd * ca,
           [=](cudaStream_t st) { return launch_concat_i8(av, ca, 1, I8View(), 0, B, h, wd, ov, st); });
    for (int i = 0; i < ca; ++i) (*cat.cs)[i] = a.scale(i);
    return cudaSuccess;
  };

  // ----------------------------------------------------------- the graph
  if (H % 32 || W % 32) return fail("int8: H and W must be multiples of 32");
  float s_in = 0.f;
  if (!scale("input", &s_in)) return cudaErrorInvalidValue;
  {
    void* q = nullptr;
    YB_TRY(dalloc(static_cast<size_t>(B) * 3 * H * W * 4, &q));
    p->d_in = static_cast<float*>(q);
  }
  // model.0 (3x3 stride 2 from the 3 input channels): one kernel quantises
  // the fp32 input and convolves (stem_i8); other first layers take the
  // quantised input through the general convolution.
  const HostTensor* w0 = find("model.0.conv.weight");
  const bool fused_stem = w0 && w0->ndim == 4 && w0->dims[1] == 3 && w0->dims[2] == 3 && w0->dims[3] == 3 &&
                          (w0->dims[0] == 16 || w0->dims[0] == 32 || w0->dims[0] == 64);
  QT xin;
  if (!fused_stem) {
    YB_TRY(tensor(3, H, W, &xin));
    const I8View ov = xin.view();
    float* din = p->d_in;
    add_op(kOpStem, 0.0, 7.0 * B * H * W,
           [=](cudaStream_t st) { return launch_quantize_input(din, B, 3, H, W, s_in, ov, st); });
    xin.set_scale(s_in);
  }
  QT b[23];
  // Downsampling conv model.i into b[i]: a new tensor, or `dst` (a slice of
  // a concat that the conv then fills directly).
  auto down = [&](int i, const QT& src, const QT* dst = nullptr) -> cudaError_t {
    const std::string P = "model." + std::to_string(i);
    const int co = wdim0(P + ".conv.weight");
    if (!co) return fail("int8: missing " + P);
    if (dst) {
      if (dst->C != co || dst->H != src.H / 2 || dst->W != src.W / 2) return fail("int8: concat slice of " + P);
      b[i] = *dst;
    } else {
      YB_TRY(tensor(co, src.H / 2, src.W / 2, &b[i]));
    }
    return conv(P, false, b[i], src, 2, 1, true, nullptr);
  };
  auto outw = [&](const std::string& L) { return wdim0(L + ".cv2.conv.weight"); };
  if (fused_stem) {
    const int co = w0->dims[0];
    float s_out = 0.f, s_pre = 0.f;
    if (!scale("model.0", &s_out) || !scale("model.0:pre", &s_pre)) return cudaErrorInvalidValue;
    const float cs[3] = {s_in, s_in, s_in};
    void *dw = nullptr, *db = nullptr, *dm = nullptr, *ds = nullptr, *dl = nullptr;
    if (w0->dev) {
      QDev qd;
      const cudaError_t r = quantize_dev(*w0, find("model.0.conv.bias"), cs, 3, false, static_cast<double>(s_pre), &qd);
      if (r == cudaErrorInvalidValue) return fail("int8: requantisation ratio out of range in model.0");
      YB_TRY(r);
      YB_TRY(dalloc(static_cast<size_t>(9) * co * 4, &dw));
      YB_TRY(cudaDeviceSynchronize());
      YB_TRY(launch_pack_stem_i8(qd.wq, co, static_cast<uint32_t*>(dw), stream_));
      YB_TRY(cudaStreamSynchronize(stream_));
      db = qd.bq;
      dm = qd.mult;
      ds = qd.shift;
    } else {
      QWeights q;
      if (!quantize(*w0, find("model.0.conv.bias"), cs, static_cast<double>(s_pre), &q))
        return fail("int8: requantisation ratio out of range in model.0");
      std::vector<uint32_t> wp(static_cast<size_t>(9) * co);
      for (int o = 0; o < co; ++o)
        for (int t = 0; t < 9; ++t) {
          uint32_t v = 0;
          for (int c = 0; c < 3; ++c)
            v |= (static_cast<uint32_t>(q.wq[(static_cast<size_t>(o) * 3 + c) * 9 + t]) & 0xFFu) << (8 * c);
          wp[static_cast<size_t>(t) * co + o] = v;
        }
      YB_TRY(upload(wp.data(), wp.size() * 4, &dw));
      YB_TRY(upload(q.bq.data(), q.bq.size() * 4, &db));
      YB_TRY(upload(q.mult.data(), q.mult.size() * 4, &dm));
      YB_TRY(upload(q.shift.data(), q.shift.size() * 4, &ds));
    }
    int8_t lut[256];
    silu_lut(lut, s_pre, s_out);
    YB_TRY(upload(lut, 256, &dl));
    YB_TRY(tensor(co, (H - 1) / 2 + 1, (W - 1) / 2 + 1, &b[0]));
    YB_TRY(init_stem_i8_attributes());
    StemI8Args sa;
    sa.in = p->d_in;
    sa.B = B;
    sa.H = H;
    sa.W = W;
    sa.Ho = b[0].H;
    sa.Wo = b[0].W;
    sa.Co = co;
    sa.s_in = s_in;
    sa.w = static_cast<const uint32_t*>(dw);
    sa.bias = static_cast<const int32_t*>(db);
    sa.mult = static_cast<const int32_t*>(dm);
    sa.shift = static_cast<const int32_t*>(ds);
    sa.lut = static_cast<const int8_t*>(dl);
    sa.out = b[0].view();
    sa.err = d_err_;
    const double po = static_cast<double>(B) * sa.Ho * sa.Wo;
    add_op(kOpStem, 2.0 * po * co * 27, 4.0 * B * 3 * H * W + po * co,
           [sa](cudaStream_t st) { return launch_stem_i8(sa, st); });
    b[0].set_scale(s_out);
  } else {
    YB_TRY(down(0, xin));
  }
  step = 1;
  YB_TRY(down(1, b[0]));
  step = 2;
  YB_TRY(tensor(outw("model.2"), b[1].H, b[1].W, &b[2]));
  YB_TRY(c3k2_plain("model.2", 1, true, b[2], b[1]));
  step = 3;
  YB_TRY(down(3, b[2]));
  step = 4;
  // model.4 and model.6 write their outputs straight into the right-hand
  // slices of the step-15 and step-12 concats (upsample(model.13) ++ model.4,
  // upsample(model.10) ++ model.6), which then copy only their upsampled
  // halves; the later layers read the slices as strided views.
  QT cat15, cat12;
  YB_TRY(tensor(outw("model.13") + outw("model.4"), b[3].H, b[3].W, &cat15));
  b[4] = cat15.sub(outw("model.13"), outw("model.4"));
  YB_TRY(c3k2_plain("model.4", 1, true, b[4], b[3]));
  step = 5;
  YB_TRY(down(5, b[4]));
  step = 6;
  YB_TRY(tensor(outw("model.10") + outw("model.6"), b[5].H, b[5].W, &cat12));
  b[6] = cat12.sub(outw("model.10"), outw("model.6"));
  YB_TRY(c3k2_c3k("model.6", b[6], b[5]));
  step = 7;
  YB_TRY(down(7, b[6]));
  step = 8;
  YB_TRY(tensor(outw("model.8"), b[7].H, b[7].W, &b[8]));
  YB_TRY(c3k2_c3k("model.8", b[8], b[7]));
  step = 9;
  YB_TRY(tensor(outw("model.9"), b[8].H, b[8].W, &b[9]));
  YB_TRY(sppf("model.9", b[9], b[8]));
  step = 10;
  // model.10 and model.20 fill the step-21 concat (model.20 ++ model.10)
  // directly, as model.13 and model.17 fill the step-18 one: no copies.
  const int c17 = wdim0("model.17.conv.weight"), c20 = wdim0("model.20.conv.weight");
  QT cat21, cat18;
  YB_TRY(tensor(c20 + outw("model.10"), b[9].H, b[9].W, &cat21));
  b[10] = cat21.sub(c20, outw("model.10"));
  YB_TRY(c2psa("model.10", b[10], b[9]));
  // steps 11-12: upsample(buf10) ++ buf6, one concat launch.
  step = 12;
  YB_TRY(upsample_into(b[10], cat12));
  b[12] = cat12;
  step = 13;
  YB_TRY(tensor(c17 + outw("model.13"), b[12].H, b[12].W, &cat18));
  b[13] = cat18.sub(c17, outw("model.13"));
  YB_TRY(c3k2_c3k("model.13", b[13], b[12]));
  step = 15;
  YB_TRY(upsample_into(b[13], cat15));
  b[15] = cat15;
  step = 16;
  YB_TRY(tensor(outw("model.16"), b[15].H, b[15].W, &b[16]));
  YB_TRY(c3k2_c3k("model.16", b[16], b[15]));
  const int after16 = static_cast<int>(p->ops.size()) - 1;
  step = 17;
  {
    const QT d17 = cat18.sub(0, c17);
    YB_TRY(down(17, b[16], &d17));
  }
  step = 18;
  b[18] = cat18;
  step = 19;
  YB_TRY(tensor(outw("model.19"), b[18].H, b[18].W, &b[19]));
  YB_TRY(c3k2_c3k("model.19", b[19], b[18]));
  const int after19 = static_cast<int>(p->ops.size()) - 1;
  step = 20;
  {
    const QT d20 = cat21.sub(0, c20);
    YB_TRY(down(20, b[19], &d20));
  }
  step = 21;
  b[21] = cat21;
  step = 22;
  YB_TRY(tensor(outw("model.22"), b[21].H, b[21].W, &b[22]));
  YB_TRY(c3k2_attn("model.22", b[22], b[21]));
  step = 23;
  // Stage tensors 01-23 for the int8 stage getter (11 and 14 are the
  // upsampled maps, read here from their concats' first channels).
  p->i8stage.assign(23, Plan::I8Stage());
  for (int i = 0; i < 23; ++i) {
    QT t = b[i];
    if (i == 11) t = b[12].sub(0, b[10].C);
    if (i == 14) t = b[15].sub(0, b[13].C);
    Plan::I8Stage& s = p->i8stage[i];
    s.p = t.ptr();
    s.cstride = t.cstride;
    s.bstride = t.bstride;
    s.C = t.C;
    s.H = t.H;
    s.W = t.W;
    s.cs.assign(t.cs->begin() + t.c0, t.cs->begin() + t.c0 + t.C);
  }

  // --------------------------------------------------------- Detect head
  const QT* feats[3] = {&b[16], &b[19], &b[22]};
  const int strides[3] = {8, 16, 32};
  int N = 0, base[3];
  for (int s = 0; s < 3; ++s) {
    base[s] = N;
    N += feats[s]->H * feats[s]->W;
  }
  p->n_anchors = N;
  {
    void* q = nullptr;
    YB_TRY(dalloc(static_cast<size_t>(B) * N * 4 * 4, &q));
    p->d_dist = static_cast<float*>(q);
    YB_TRY(dalloc(static_cast<size_t>(B) * N * nc * 4, &q));
    p->d_logits = static_cast<float*>(q);
    YB_TRY(dalloc(static_cast<size_t>(B) * N * 4 * 4, &q));
    p->d_boxes = static_cast<float*>(q);
    YB_TRY(dalloc(static_cast<size_t>(B) * N * 4, &q));
    p->d_maxscore = static_cast<float*>(q);
    YB_TRY(dalloc(static_cast<size_t>(B) * p->max_det * 6 * 4, &q));
    p->d_out = static_cast<float*>(q);
  }
  const std::string b2 = find("model.23.one2one_cv2.0.0.conv.weight") ? "model.23.one2one_cv2." : "model.23.cv2.";
  const std::string b3 = b2 == "model.23.one2one_cv2." ? "model.23.one2one_cv3." : "model.23.cv3.";
  for (int s = 0; s < 3; ++s) {
    const QT& f = *feats[s];
    const std::string si = std::to_string(s);
    const size_t first_op = p->ops.size();
    const int c2 = wdim0(b2 + si + ".0.conv.weight"), c3 = wdim0(b3 + si + ".0.1.conv.weight");
    if (!c2 || !c3) return fail("int8: missing detect weights");
    QT s1, s2, d0, p0, d1, p1;
    YB_TRY(tensor(c2, f.H, f.W, &s1));
    YB_TRY(conv(b2 + si + ".0", false, s1, f, 1, 1, true, nullptr));
    YB_TRY(tensor(c2, f.H, f.W, &s2));
    YB_TRY(conv(b2 + si + ".1", false, s2, s1, 1, 1, true, nullptr));
    F32Out dv;
    dv.ptr = p->d_dist + static_cast<size_t>(base[s]) * 4;
    dv.cstride = 4;
    dv.bstride = static_cast<long long>(N) * 4;
    YB_TRY(conv(b2 + si + ".2", true, QT(), s2, 1, 0, false, nullptr, dv));
    YB_TRY(tensor(f.C, f.H, f.W, &d0));
    YB_TRY(dwconv(b3 + si + ".0.0", d0, f));
    YB_TRY(tensor(c3, f.H, f.W, &p0));
    YB_TRY(conv(b3 + si + ".0.1", false, p0, d0, 1, 0, true, nullptr));
    YB_TRY(tensor(c3, f.H, f.W, &d1));
    YB_TRY(dwconv(b3 + si + ".1.0", d1, p0));
    YB_TRY(tensor(c3, f.H, f.W, &p1));
    YB_TRY(conv(b3 + si + ".1.1", false, p1, d1, 1, 0, true, nullptr));
    F32Out lv;
    lv.ptr = p->d_logits + static_cast<size_t>(base[s]) * nc;
    lv.cstride = nc;
    lv.bstride = static_cast<long long>(N) * nc;
    lv.rowmax = p->d_maxscore + base[s];
    lv.rm_bstride = N;
    YB_TRY(conv(b3 + si + ".2", true, QT(), p1, 1, 0, false, nullptr, lv));
    // The P3 and P4 heads read model.16 / model.19 only: side lanes 1 and 2,
    // beside the rest of the neck.
    if (s < 2) {
      for (size_t i = first_op; i < p->ops.size(); ++i) p->ops[i].lane = s + 1;
      p->fork_after[s + 1] = s == 0 ? after16 : after19;
    }
  }
  DecodeArgs de;
  de.dist = p->d_dist;
  de.logits = p->d_logits;
  de.boxes = p->d_boxes;
  de.maxscore = p->d_maxscore;
  de.B = B;
  de.N = N;
  de.nc = nc;
  de.nscales = 3;
  de.max_ready = 1;
  for (int s = 0; s < 3; ++s) {
    de.base[s] = base[s];
    de.w[s] = feats[s]->W;
    de.stride[s] = strides[s];
  }
  add_op(kOpDecode, 0.0, 4.0 * B * N * (4.0 + 4.0), [de](cudaStream_t st) { return launch_decode(de, st); });
  p->ops.back().join = true;
  TopkArgs ta;
  ta.maxscore = p->d_maxscore;
  ta.scores = p->d_logits;
  ta.s_bstride = static_cast<long long>(N) * nc;
  ta.s_rstride = nc;
  ta.apply_sigmoid = 1;
  ta.boxes = p->d_boxes;
  ta.b_bstride = static_cast<long long>(N) * 4;
  ta.b_rstride = 4;
  ta.dets = p->d_out;
  ta.B = B;
  ta.N = N;
  ta.nc = nc;
  ta.max_det = p->max_det;
  ta.cap = p->max_det;
  add_op(kOpTopk, 0.0, 4.0 * B * (N + static_cast<double>(p->max_det) * (nc + 4 + 6)),
         [ta](cudaStream_t st) { return launch_topk(ta, st); });
#undef YB_TRY
  return cudaSuccess;
}

}  // namespace yb
