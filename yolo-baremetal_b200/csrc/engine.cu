// Lowering of the YOLO26 graph to sm_100a kernel launches (see engine.h).
#include "engine.h"
#include "weight_prep.h"

#include <cmath>
#include <cstdio>
#include <cstring>

namespace yb {

namespace {

SView tv(const Buf& b, int coff = 0) {
  SView v;
  v.hi = b.hi;
  v.plane = b.plane;
  v.bstride = b.bstride;
  v.cstride = b.C;
  v.coff = coff;
  return v;
}
SOut ov(const Buf& b, int coff = 0) {
  SOut v;
  v.hi = b.hi;
  v.plane = b.plane;
  v.bstride = b.bstride;
  v.cstride = b.C;
  v.coff = coff;
  return v;
}
Src src_of(const Buf& b, int coff, int c) {
  Src s;
  s.v0 = tv(b, coff);
  s.c0 = c;
  s.H = b.H;
  s.W = b.W;
  return s;
}
Src src_cat(const Buf& a, int lg_a, const Buf& b, int H, int W) {
  Src s;
  s.v0 = tv(a);
  s.c0 = a.C;
  s.lg0 = lg_a;
  s.v1 = tv(b);
  s.c1 = b.C;
  s.H = H;
  s.W = W;
  return s;
}

bool ends_with(const std::string& s, const std::string& suf) {
  return s.size() >= suf.size() && s.compare(s.size() - suf.size(), suf.size(), suf) == 0;
}

}  // namespace

// ------------------------------------------------------------- weight files
bool read_weight_bin(const char* path, WeightMap* out, int* num_classes, std::string* why) {
  FILE* f = std::fopen(path, "rb");
  if (!f) {
    *why = std::string("cannot open ") + path;
    return false;
  }
  int32_t nc = 0, count = 0;
  if (std::fread(&nc, 4, 1, f) != 1 || std::fread(&count, 4, 1, f) != 1 || count < 0) {
    std::fclose(f);
    *why = "truncated header";
    return false;
  }
  for (int i = 0; i < count; ++i) {
    int32_t nl = 0;
    if (std::fread(&nl, 4, 1, f) != 1 || nl <= 0 || nl >= 128) {
      std::fclose(f);
      *why = "bad record name length";
      return false;
    }
    std::string name(static_cast<size_t>(nl), '\0');
    int32_t nd = 0;
    if (std::fread(&name[0], 1, nl, f) != static_cast<size_t>(nl) || std::fread(&nd, 4, 1, f) != 1 || nd < 0 ||
        nd > 4) {
      std::fclose(f);
      *why = "bad record header for " + name;
      return false;
    }
    HostTensor t;
    t.ndim = nd;
    size_t n = 1;
    for (int d = 0; d < nd; ++d) {
      int32_t v = 0;
      if (std::fread(&v, 4, 1, f) != 1 || v < 0) {
        std::fclose(f);
        *why = "bad dims for " + name;
        return false;
      }
      t.dims[d] = v;
      n *= static_cast<size_t>(v);
    }
    t.data.resize(n);
    if (n && std::fread(t.data.data(), 4, n, f) != n) {
      std::fclose(f);
      *why = "truncated data for " + name;
      return false;
    }
    (*out)[name] = std::move(t);
  }
  std::fclose(f);
  *num_classes = nc;
  return true;
}

// Folds every <p>.bn.{weight,bias,running_mean,running_var} into
// <p>.conv.weight / <p>.conv.bias (created as zeros when absent) and drops the
// BN records, with the reference's fp32 arithmetic (utils.c:81-106).
void fold_all_bn_map(WeightMap* w) {
  std::vector<std::string> convs;
  for (const auto& kv : *w)
    if (ends_with(kv.first, ".conv.weight")) convs.push_back(kv.first);
  for (const std::string& cname : convs) {
    const std::string p = cname.substr(0, cname.size() - std::strlen(".conv.weight"));
    auto g = w->find(p + ".bn.weight");
    auto be = w->find(p + ".bn.bias");
    auto mu = w->find(p + ".bn.running_mean");
    auto var = w->find(p + ".bn.running_var");
    if (g == w->end() || be == w->end() || mu == w->end() || var == w->end()) continue;
    HostTensor& cw = (*w)[cname];
    const int out_c = cw.dims[0];
    const size_t per = cw.data.size() / static_cast<size_t>(out_c);
    const std::string bname = p + ".conv.bias";
    if (w->find(bname) == w->end()) {
      HostTensor b;
      b.ndim = 4;
      b.dims[0] = 1;
      b.dims[1] = out_c;
      b.data.assign(static_cast<size_t>(out_c), 0.0f);
      (*w)[bname] = std::move(b);
    }
    HostTensor& cb = (*w)[bname];
    const float eps = 1e-5f;
    for (int i = 0; i < out_c; ++i) {
      const float gamma = g->second.data[i];
      const float beta = be->second.data[i];
      const float mean = mu->second.data[i];
      const float v = var->second.data[i];
      const float scale = gamma / std::sqrt(v + eps);
      for (size_t j = 0; j < per; ++j) cw.data[i * per + j] *= scale;
      const float b0 = cb.data[i];
      const float t = b0 - mean;
      const float t2 = t * scale;
      cb.data[i] = t2 + beta;
    }
    w->erase(p + ".bn.weight");
    w->erase(p + ".bn.bias");
    w->erase(p + ".bn.running_mean");
    w->erase(p + ".bn.running_var");
    w->erase(p + ".bn.num_batches_tracked");
  }
}

// ------------------------------------------------------------------- engine
Engine::Engine(int device) : device_(device) {
  cudaSetDevice(device);
  cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device);
  cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking);
  cudaMalloc(&d_err_, sizeof(int));
  cudaMemset(d_err_, 0, sizeof(int));
  init_conv_kernel_attributes();
}

Engine::~Engine() {
  cudaSetDevice(device_);
  for (auto& p : plans_) release_plan(p.get());
  for (void* q : weight_allocs_) cudaFree(q);
  if (d_err_) cudaFree(d_err_);
  if (stream_) cudaStreamDestroy(stream_);
}

void Engine::release_plan(Plan* p) {
  if (p->int8) i8_images_.clear();  // they may point into this plan's buffers
  if (p->graph) cudaGraphExecDestroy(p->graph);
  p->graph = nullptr;
  for (int L = 1; L < 3; ++L) {
    if (p->lane_s[L]) cudaStreamDestroy(p->lane_s[L]);
    if (p->ev_fork[L]) cudaEventDestroy(p->ev_fork[L]);
    if (p->ev_join[L]) cudaEventDestroy(p->ev_join[L]);
    p->lane_s[L] = nullptr;
    p->ev_fork[L] = p->ev_join[L] = nullptr;
  }
  for (void* q : p->allocs) cudaFree(q);
  p->allocs.clear();
}

cudaError_t Engine::dev_alloc(size_t bytes, void** p) {
  cudaError_t e = cudaMalloc(p, bytes < 256 ? 256 : bytes);
  if (e == cudaSuccess) weight_allocs_.push_back(*p);
  return e;
}

int Engine::take_kernel_error() {
  int v = 0;
  cudaSetDevice(device_);
  if (cudaMemcpy(&v, d_err_, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  if (v) cudaMemset(d_err_, 0, sizeof(int));
  return v;
}

const HostTensor* Engine::find(const std::string& name) const {
  auto it = hw_.find(name);
  return it == hw_.end() ? nullptr : &it->second;
}

namespace {
// Copies `n` floats of a weight tensor (host values or device values) into
// device memory at dst.
cudaError_t tensor_to_device(const HostTensor& t, float* dst, size_t n) {
  if (t.dev) return cudaMemcpy(dst, t.dev, n * 4, cudaMemcpyDeviceToDevice);
  return cudaMemcpy(dst, t.data.data(), n * 4, cudaMemcpyHostToDevice);
}
}  // namespace

void Engine::reset_weights() {
  cudaSetDevice(device_);
  for (auto& p : plans_) release_plan(p.get());
  plans_.clear();
  for (void* q : weight_allocs_) cudaFree(q);
  weight_allocs_.clear();
  convs_.clear();
  dws_.clear();
  i8_images_.clear();
  stem_ = DevStem();
  dev_arena_ = nullptr;
}

cudaError_t Engine::setup_stem() {
  const HostTensor* sw = find("model.0.conv.weight");
  const HostTensor* sb = find("model.0.conv.bias");
  // Any weight file loads, as in the reference (model.c:182-198); a missing
  // layer is reported when a forward needs it (plan build).
  if (!sw || !sb) return cudaSuccess;
  stem_.co = sw->dims[0];
  stem_.ci = sw->dims[1];
  stem_.k = sw->dims[2];
  cudaError_t e = dev_alloc(sw->count() * 4, reinterpret_cast<void**>(&stem_.w));
  if (e != cudaSuccess) return e;
  e = dev_alloc(sb->count() * 4, reinterpret_cast<void**>(&stem_.bias));
  if (e != cudaSuccess) return e;
  e = tensor_to_device(*sw, stem_.w, sw->count());
  if (e != cudaSuccess) return e;
  return tensor_to_device(*sb, stem_.bias, sb->count());
}

cudaError_t Engine::set_weights(WeightMap&& w, int num_classes, std::string* why) {
  (void)why;
  reset_weights();
  hw_ = std::move(w);
  nc_ = num_classes;
  return setup_stem();
}

cudaError_t Engine::set_weights_device(WeightMap&& raw, int num_classes, std::string* why) {
  reset_weights();
  hw_.clear();
  nc_ = num_classes;
  // Convolutions with BatchNorm records, and the zero biases the fold
  // creates where a convolution has none (fold_all_bn_map's rule).
  std::vector<std::string> folds;
  for (const auto& kv : raw) {
    if (!ends_with(kv.first, ".conv.weight")) continue;
    const std::string p = kv.first.substr(0, kv.first.size() - std::strlen(".conv.weight"));
    if (!raw.count(p + ".bn.weight") || !raw.count(p + ".bn.bias") || !raw.count(p + ".bn.running_mean") ||
        !raw.count(p + ".bn.running_var"))
      continue;
    folds.push_back(p);
  }
  for (const std::string& p : folds) {
    if (raw.count(p + ".conv.bias")) continue;
    HostTensor b;
    b.ndim = 4;
    b.dims[1] = raw[p + ".conv.weight"].dims[0];
    b.data.assign(static_cast<size_t>(b.dims[1]), 0.0f);
    raw[p + ".conv.bias"] = std::move(b);
  }
  // One arena, every tensor at a 64-byte aligned offset, filled by one copy.
  std::map<std::string, long long> off;
  long long total = 0;
  for (const auto& kv : raw) {
    off[kv.first] = total;
    total += (static_cast<long long>(kv.second.data.size()) + 15) / 16 * 16;
  }
  std::vector<float> stage(static_cast<size_t>(total > 0 ? total : 1), 0.0f);
  for (const auto& kv : raw) std::copy(kv.second.data.begin(), kv.second.data.end(), stage.begin() + off[kv.first]);
  cudaError_t e = dev_alloc(stage.size() * 4, reinterpret_cast<void**>(&dev_arena_));
  if (e != cudaSuccess) return e;
  e = cudaMemcpy(dev_arena_, stage.data(), stage.size() * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return e;
  std::vector<FoldDesc> fd;
  for (const std::string& p : folds) {
    FoldDesc d;
    const HostTensor& w = raw[p + ".conv.weight"];
    d.w = off[p + ".conv.weight"];
    d.b = off[p + ".conv.bias"];
    d.g = off[p + ".bn.weight"];
    d.be = off[p + ".bn.bias"];
    d.mu = off[p + ".bn.running_mean"];
    d.var = off[p + ".bn.running_var"];
    d.oc = w.dims[0];
    d.per = static_cast<int>(w.data.size() / static_cast<size_t>(d.oc));
    fd.push_back(d);
  }
  if (!fd.empty()) {
    FoldDesc* d_fd = nullptr;
    e = cudaMalloc(&d_fd, fd.size() * sizeof(FoldDesc));
    if (e == cudaSuccess) e = cudaMemcpy(d_fd, fd.data(), fd.size() * sizeof(FoldDesc), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = launch_fold_bn(d_fd, static_cast<int>(fd.size()), dev_arena_, stream_);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
    if (d_fd) cudaFree(d_fd);
    if (e != cudaSuccess) return e;
  }
  const char* sfx[5] = {".bn.weight", ".bn.bias", ".bn.running_mean", ".bn.running_var", ".bn.num_batches_tracked"};
  for (const std::string& p : folds)
    for (const char* x : sfx) raw.erase(p + x);
  for (auto& kv : raw) {
    HostTensor t;
    t.ndim = kv.second.ndim;
    for (int i = 0; i < 4; ++i) t.dims[i] = kv.second.dims[i];
    t.n = kv.second.data.size();
    t.dev = dev_arena_ + off[kv.first];
    hw_[kv.first] = std::move(t);
  }
  (void)why;
  return setup_stem();
}

cudaError_t Engine::conv_w(const std::string& prefix, bool plain, DevConv** out, std::string* why) {
  auto it = convs_.find(prefix);
  if (it != convs_.end()) {
    *out = &it->second;
    return cudaSuccess;
  }
  const std::string wn = prefix + (plain ? ".weight" : ".conv.weight");
  const std::string bn = prefix + (plain ? ".bias" : ".conv.bias");
  const HostTensor* w = find(wn);
  const HostTensor* b = find(bn);
  if (!w || !b) {
    *why = "missing weight " + (w ? bn : wn);
    return cudaErrorInvalidValue;
  }
  DevConv d;
  d.name = prefix;
  d.co = w->dims[0];
  d.ci = w->dims[1];
  d.kh = w->dims[2];
  d.kw = w->dims[3];
  if (d.ci % 8 || d.co % 4 || static_cast<int>(b->count()) != d.co) {
    *why = "unsupported conv shape at " + prefix;
    return cudaErrorInvalidValue;
  }
  d.K = d.kh * d.kw * d.ci;
  d.num_kc = (d.K + 63) / 64;
  choose_n_tiling(d.co, &d.n_tile, &d.n_tiles);
  const size_t bytes = pack_conv_weights(nullptr, d.co, d.ci, d.kh, d.kw, d.n_tile, nullptr);
  cudaError_t e = dev_alloc(bytes, reinterpret_cast<void**>(&d.wpack));
  if (e != cudaSuccess) return e;
  if (w->dev) {
    e = launch_pack_conv(w->dev, d.co, d.ci, d.kh, d.kw, d.n_tile, d.wpack, bytes, stream_);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
  } else {
    std::vector<uint8_t> pack(bytes);
    pack_conv_weights(w->data.data(), d.co, d.ci, d.kh, d.kw, d.n_tile, pack.data());
    e = cudaMemcpy(d.wpack, pack.data(), bytes, cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) return e;
  e = dev_alloc(static_cast<size_t>(d.n_tile) * d.n_tiles * 4, reinterpret_cast<void**>(&d.bias));
  if (e != cudaSuccess) return e;
  cudaMemset(d.bias, 0, static_cast<size_t>(d.n_tile) * d.n_tiles * 4);
  e = tensor_to_device(*b, d.bias, b->count());
  if (e != cudaSuccess) return e;
  auto ins = convs_.emplace(prefix, d);
  *out = &ins.first->second;
  return cudaSuccess;
}

cudaError_t Engine::conv_pair(const std::string& pa, const std::string& pb, DevConv** out, std::string* why) {
  const std::string key = pa + "|" + pb;
  auto it = convs_.find(key);
  if (it != convs_.end()) {
    *out = &it->second;
    return cudaSuccess;
  }
  const HostTensor* wa = find(pa + ".conv.weight");
  const HostTensor* ba = find(pa + ".conv.bias");
  const HostTensor* wb = find(pb + ".conv.weight");
  const HostTensor* bb = find(pb + ".conv.bias");
  if (!wa || !ba || !wb || !bb) {
    *why = "missing weights of " + key;
    return cudaErrorInvalidValue;
  }
  DevConv d;
  d.name = key;
  d.merged = true;
  d.co = wa->dims[0] + wb->dims[0];
  d.ci = wa->dims[1];
  d.kh = wa->dims[2];
  d.kw = wa->dims[3];
  if (wb->dims[1] != d.ci || wb->dims[2] != d.kh || wb->dims[3] != d.kw || d.ci % 8 || wa->dims[0] % 8 ||
      wb->dims[0] % 8 || static_cast<int>(ba->count()) != wa->dims[0] || static_cast<int>(bb->count()) != wb->dims[0]) {
    *why = "conv pair shapes at " + key;
    return cudaErrorInvalidValue;
  }
  d.K = d.kh * d.kw * d.ci;
  d.num_kc = (d.K + 63) / 64;
  choose_n_tiling(d.co, &d.n_tile, &d.n_tiles);
  // Both weight tensors side by side in a temporary device buffer, packed
  // there by the same kernel as the device preparation path.
  const size_t na = wa->count(), nb = wb->count();
  float* tmp = nullptr;
  cudaError_t e = cudaMalloc(&tmp, (na + nb) * 4);
  if (e != cudaSuccess) return e;
  e = tensor_to_device(*wa, tmp, na);
  if (e == cudaSuccess) e = tensor_to_device(*wb, tmp + na, nb);
  const size_t bytes = pack_conv_weights(nullptr, d.co, d.ci, d.kh, d.kw, d.n_tile, nullptr);
  if (e == cudaSuccess) e = dev_alloc(bytes, reinterpret_cast<void**>(&d.wpack));
  if (e == cudaSuccess) e = launch_pack_conv(tmp, d.co, d.ci, d.kh, d.kw, d.n_tile, d.wpack, bytes, stream_);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
  cudaFree(tmp);
  if (e != cudaSuccess) return e;
  e = dev_alloc(static_cast<size_t>(d.n_tile) * d.n_tiles * 4, reinterpret_cast<void**>(&d.bias));
  if (e != cudaSuccess) return e;
  cudaMemset(d.bias, 0, static_cast<size_t>(d.n_tile) * d.n_tiles * 4);
  e = tensor_to_device(*ba, d.bias, ba->count());
  if (e == cudaSuccess) e = tensor_to_device(*bb, d.bias + ba->count(), bb->count());
  if (e != cudaSuccess) return e;
  auto ins = convs_.emplace(key, d);
  *out = &ins.first->second;
  return cudaSuccess;
}

cudaError_t Engine::conv_narrow(DevConv* d, int n_tile, const uint8_t** wpack) {
  const int slot = n_tile == 64 ? 0 : 1;
  if (!d->wpack_n[slot]) {
    const std::string wn = d->name + (find(d->name + ".conv.weight") ? ".conv.weight" : ".weight");
    const HostTensor* w = find(wn);
    if (!w) return cudaErrorInvalidValue;
    const size_t bytes = pack_conv_weights(nullptr, d->co, d->ci, d->kh, d->kw, n_tile, nullptr);
    cudaError_t e = dev_alloc(bytes, reinterpret_cast<void**>(&d->wpack_n[slot]));
    if (e != cudaSuccess) return e;
    if (w->dev) {
      e = launch_pack_conv(w->dev, d->co, d->ci, d->kh, d->kw, n_tile, d->wpack_n[slot], bytes, stream_);
      if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
    } else {
      std::vector<uint8_t> pack(bytes);
      pack_conv_weights(w->data.data(), d->co, d->ci, d->kh, d->kw, n_tile, pack.data());
      e = cudaMemcpy(d->wpack_n[slot], pack.data(), bytes, cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) return e;
  }
  *wpack = d->wpack_n[slot];
  return cudaSuccess;
}

// ------------------------------------------------------ prepared-weight blob
namespace {
constexpr char kBlobMagic[8] = {'Y', 'B', '2', '6', 'P', 'R', 'E', 'P'};
constexpr int32_t kBlobVersion = 1;

// Convolution prefixes of a weight map, with whether they are plain (P.weight)
// rather than Conv+BN (P.conv.weight): every 4-D, non-depthwise weight.
std::vector<std::pair<std::string, bool>> conv_prefixes(const WeightMap& w) {
  std::vector<std::pair<std::string, bool>> out;
  for (const auto& kv : w) {
    const HostTensor& t = kv.second;
    if (t.ndim != 4 || t.dims[1] == 1) continue;
    if (ends_with(kv.first, ".conv.weight"))
      out.emplace_back(kv.first.substr(0, kv.first.size() - std::strlen(".conv.weight")), false);
    else if (ends_with(kv.first, ".weight") && !ends_with(kv.first, ".bn.weight"))
      out.emplace_back(kv.first.substr(0, kv.first.size() - std::strlen(".weight")), true);
  }
  return out;
}

bool put(FILE* f, const void* p, size_t n) { return std::fwrite(p, 1, n, f) == n; }
bool get(FILE* f, void* p, size_t n) { return std::fread(p, 1, n, f) == n; }

bool put_name(FILE* f, const std::string& s) {
  const int32_t n = static_cast<int32_t>(s.size());
  return put(f, &n, 4) && put(f, s.data(), s.size());
}
bool get_name(FILE* f, std::string* s) {
  int32_t n = 0;
  if (!get(f, &n, 4) || n < 0 || n > 4096) return false;
  s->resize(static_cast<size_t>(n));
  return get(f, &(*s)[0], static_cast<size_t>(n));
}
}  // namespace

cudaError_t Engine::save_blob(const std::string& path, std::string* why) {
  cudaSetDevice(device_);
  // Every convolution the graph can use, packed in its full N tiling.
  std::vector<std::pair<std::string, DevConv*>> images;
  for (const auto& pc : conv_prefixes(hw_)) {
    DevConv* d = nullptr;
    std::string w2;
    if (conv_w(pc.first, pc.second, &d, &w2) == cudaSuccess) images.emplace_back(pc.first, d);
  }
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) {
    *why = "cannot write " + path;
    return cudaErrorInvalidValue;
  }
  bool ok = put(f, kBlobMagic, 8) && put(f, &kBlobVersion, 4) && put(f, &nc_, 4);
  const int32_t nt = static_cast<int32_t>(hw_.size()), ni = static_cast<int32_t>(images.size());
  ok = ok && put(f, &nt, 4) && put(f, &ni, 4);
  std::vector<float> buf;
  cudaError_t e = cudaSuccess;
  for (const auto& kv : hw_) {
    if (!ok) break;
    const HostTensor& t = kv.second;
    const int64_t n = static_cast<int64_t>(t.count());
    buf.resize(static_cast<size_t>(n));
    if (t.dev) e = cudaMemcpy(buf.data(), t.dev, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost);
    else std::copy(t.data.begin(), t.data.end(), buf.begin());
    if (e != cudaSuccess) break;
    ok = put_name(f, kv.first) && put(f, &t.ndim, 4) && put(f, t.dims, 16) && put(f, &n, 8) &&
         put(f, buf.data(), static_cast<size_t>(n) * 4);
  }
  std::vector<uint8_t> img;
  for (const auto& im : images) {
    if (!ok || e != cudaSuccess) break;
    const DevConv& d = *im.second;
    const int64_t bytes = static_cast<int64_t>(pack_conv_weights(nullptr, d.co, d.ci, d.kh, d.kw, d.n_tile, nullptr));
    img.resize(static_cast<size_t>(bytes));
    e = cudaMemcpy(img.data(), d.wpack, static_cast<size_t>(bytes), cudaMemcpyDeviceToHost);
    const int32_t hdr[5] = {d.co, d.ci, d.kh, d.kw, d.n_tile};
    ok = e == cudaSuccess && put_name(f, im.first) && put(f, hdr, 20) && put(f, &bytes, 8) &&
         put(f, img.data(), img.size());
  }
  std::fclose(f);
  if (e != cudaSuccess) return e;
  if (!ok) {
    *why = "short write to " + path;
    return cudaErrorInvalidValue;
  }
  return cudaSuccess;
}

cudaError_t Engine::load_blob(const std::string& path, int* num_classes, std::string* why) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) {
    *why = "cannot open " + path;
    return cudaErrorInvalidValue;
  }
  char magic[8];
  int32_t ver = 0, nc = 0, nt = 0, ni = 0;
  bool ok = get(f, magic, 8) && std::memcmp(magic, kBlobMagic, 8) == 0 && get(f, &ver, 4) && ver == kBlobVersion &&
            get(f, &nc, 4) && get(f, &nt, 4) && get(f, &ni, 4) && nt >= 0 && ni >= 0;
  WeightMap raw;
  for (int i = 0; ok && i < nt; ++i) {
    std::string name;
    HostTensor t;
    int64_t n = 0;
    ok = get_name(f, &name) && get(f, &t.ndim, 4) && get(f, t.dims, 16) && get(f, &n, 8) && n >= 0 &&
         n < (int64_t{1} << 32);
    if (!ok) break;
    t.data.resize(static_cast<size_t>(n));
    ok = get(f, t.data.data(), static_cast<size_t>(n) * 4);
    raw[name] = std::move(t);
  }
  struct Img {
    std::string name;
    int32_t hdr[5];
    std::vector<uint8_t> bytes;
  };
  std::vector<Img> imgs(static_cast<size_t>(ok ? ni : 0));
  for (auto& im : imgs) {
    int64_t bytes = 0;
    ok = ok && get_name(f, &im.name) && get(f, im.hdr, 20) && get(f, &bytes, 8) && bytes > 0 &&
         bytes < (int64_t{1} << 31);
    if (!ok) break;
    im.bytes.resize(static_cast<size_t>(bytes));
    ok = get(f, im.bytes.data(), im.bytes.size());
  }
  std::fclose(f);
  if (!ok) {
    *why = "not a prepared-weight blob (or truncated): " + path;
    return cudaErrorInvalidValue;
  }
  // The folded tensors: one arena, one copy (no BatchNorm records remain, so
  // set_weights_device folds nothing).
  cudaError_t e = set_weights_device(std::move(raw), nc, why);
  if (e != cudaSuccess) return e;
  *num_classes = nc;
  for (const Img& im : imgs) {
    const bool plain = !find(im.name + ".conv.weight");
    const HostTensor* w = find(im.name + (plain ? ".weight" : ".conv.weight"));
    const HostTensor* b = find(im.name + (plain ? ".bias" : ".conv.bias"));
    DevConv d;
    d.name = im.name;
    d.co = im.hdr[0];
    d.ci = im.hdr[1];
    d.kh = im.hdr[2];
    d.kw = im.hdr[3];
    d.K = d.kh * d.kw * d.ci;
    d.num_kc = (d.K + 63) / 64;
    choose_n_tiling(d.co, &d.n_tile, &d.n_tiles);
    if (!w || !b || w->dims[0] != d.co || w->dims[1] != d.ci || d.n_tile != im.hdr[4] ||
        im.bytes.size() != pack_conv_weights(nullptr, d.co, d.ci, d.kh, d.kw, d.n_tile, nullptr)) {
      *why = "prepared-weight blob does not match its tensors at " + im.name;
      return cudaErrorInvalidValue;
    }
    e = dev_alloc(im.bytes.size(), reinterpret_cast<void**>(&d.wpack));
    if (e == cudaSuccess) e = cudaMemcpy(d.wpack, im.bytes.data(), im.bytes.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = dev_alloc(static_cast<size_t>(d.n_tile) * d.n_tiles * 4, reinterpret_cast<void**>(&d.bias));
    if (e == cudaSuccess) e = cudaMemset(d.bias, 0, static_cast<size_t>(d.n_tile) * d.n_tiles * 4);
    if (e == cudaSuccess) e = tensor_to_device(*b, d.bias, b->count());
    if (e != cudaSuccess) return e;
    convs_.emplace(im.name, d);
  }
  return cudaSuccess;
}

cudaError_t Engine::weight_image(const std::string& name, int kind, int n_tile, std::vector<uint8_t>* out,
                                 std::string* why) {
  cudaSetDevice(device_);
  const void* src = nullptr;
  size_t bytes = 0;
  bool on_device = true;
  if (kind == 0) {
    const HostTensor* t = find(name);
    if (!t) {
      *why = "no tensor " + name;
      return cudaErrorInvalidValue;
    }
    bytes = t->count() * 4;
    src = t->dev ? static_cast<const void*>(t->dev) : static_cast<const void*>(t->data.data());
    on_device = t->dev != nullptr;
  } else if (kind == 1) {
    const bool plain = !find(name + ".conv.weight");
    DevConv* d = nullptr;
    cudaError_t e = conv_w(name, plain, &d, why);
    if (e != cudaSuccess) return e;
    const uint8_t* p = d->wpack;
    int nt = d->n_tile;
    if (n_tile != 0 && n_tile != d->n_tile) {
      if (n_tile != 64 && n_tile != 128) {
        *why = "n_tile must be 0 (full tiling), 64 or 128";
        return cudaErrorInvalidValue;
      }
      if ((e = conv_narrow(d, n_tile, &p)) != cudaSuccess) return e;
      nt = n_tile;
    }
    src = p;
    bytes = pack_conv_weights(nullptr, d->co, d->ci, d->kh, d->kw, nt, nullptr);
  } else if (kind == 2) {
    auto it = i8_images_.find(name);
    if (it == i8_images_.end()) {
      *why = "no INT8 operand image of " + name + " (build an INT8 plan first)";
      return cudaErrorInvalidValue;
    }
    src = it->second.first;
    bytes = it->second.second;
  } else {
    *why = "kind must be 0, 1 or 2";
    return cudaErrorInvalidValue;
  }
  out->resize(bytes);
  if (!on_device) {
    std::memcpy(out->data(), src, bytes);
    return cudaSuccess;
  }
  return cudaMemcpy(out->data(), src, bytes, cudaMemcpyDeviceToHost);
}

cudaError_t Engine::dw_w(const std::string& prefix, DevDw** out, std::string* why) {
  auto it = dws_.find(prefix);
  if (it != dws_.end()) {
    *out = &it->second;
    return cudaSuccess;
  }
  const HostTensor* w = find(prefix + ".conv.weight");
  const HostTensor* b = find(prefix + ".conv.bias");
  if (!w || !b || w->dims[1] != 1 || w->dims[2] != 3 || w->dims[3] != 3 || w->dims[0] % 8) {
    *why = "missing or unsupported depthwise weight " + prefix;
    return cudaErrorInvalidValue;
  }
  DevDw d;
  d.c = w->dims[0];
  cudaError_t e = dev_alloc(static_cast<size_t>(9) * d.c * 4, reinterpret_cast<void**>(&d.w));
  if (e != cudaSuccess) return e;
  if (w->dev) {
    e = launch_taps_transpose(w->dev, d.c, d.w, stream_);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
  } else {
    std::vector<float> t(static_cast<size_t>(9) * d.c);
    for (int c = 0; c < d.c; ++c)
      for (int k = 0; k < 9; ++k) t[static_cast<size_t>(k) * d.c + c] = w->data[static_cast<size_t>(c) * 9 + k];
    e = cudaMemcpy(d.w, t.data(), t.size() * 4, cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) return e;
  e = dev_alloc(static_cast<size_t>(d.c) * 4, reinterpret_cast<void**>(&d.bias));
  if (e != cudaSuccess) return e;
  e = tensor_to_device(*b, d.bias, static_cast<size_t>(d.c));
  if (e != cudaSuccess) return e;
  auto ins = dws_.emplace(prefix, d);
  *out = &ins.first->second;
  return cudaSuccess;
}

#define YB_TRY(x)                          \
  do {                                     \
    cudaError_t e_ = (x);                  \
    if (e_ != cudaSuccess) return e_;      \
  } while (0)

cudaError_t Engine::build(Plan* p, std::string* why) {
  const int B = p->B;
  int step = 0;
  std::vector<Op>& ops = p->ops;

  auto alloc_buf = [&](int H, int W, int C, Buf* b) -> cudaError_t {
    b->H = H;
    b->W = W;
    b->C = C;
    b->bstride = static_cast<long long>(H) * W * C;
    b->plane = static_cast<long long>(B) * b->bstride;
    const size_t bytes = static_cast<size_t>(b->plane) * 2 * sizeof(uint16_t);
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, bytes);
    if (e != cudaSuccess) return e;
    p->allocs.push_back(q);
    p->arena_bytes += bytes;
    b->hi = static_cast<uint16_t*>(q);
    return cudaSuccess;
  };
  auto alloc_raw = [&](size_t bytes, float** q) -> cudaError_t {
    void* r = nullptr;
    cudaError_t e = cudaMalloc(&r, bytes);
    if (e != cudaSuccess) return e;
    p->allocs.push_back(r);
    p->arena_bytes += bytes;
    *q = static_cast<float*>(r);
    return cudaSuccess;
  };
  // Calibration plans: a pair of max-|x| words, [0] registered under `pre`
  // (when non-empty) and [1] under `out`.
  auto stat_slot = [&](const std::string& out, const std::string& pre) -> unsigned* {
    if (!p->calib || p->amax_used + 2 > p->amax_cap) return nullptr;
    const int k = p->amax_used;
    p->amax_used += 2;
    if (!pre.empty()) p->amax_names.emplace_back(pre, k);
    p->amax_names.emplace_back(out, k + 1);
    return p->d_amax + k;
  };
  if (p->calib) {
    p->amax_cap = 2048;
    YB_TRY(cudaMalloc(&p->d_amax, p->amax_cap * sizeof(unsigned)));
    p->allocs.push_back(p->d_amax);
    YB_TRY(cudaMemset(p->d_amax, 0, p->amax_cap * sizeof(unsigned)));
  }
  auto add_conv = [&](const DevConv* w, const Src& in, int stride, int pad, int act, SOut out, SView res,
                      FOut fout = FOut()) -> cudaError_t {
    if (in.c0 + in.c1 != w->ci || in.c0 % 8 || w->ci % 8) {
      *why = "conv input channels must match and be multiples of 8";
      return cudaErrorInvalidValue;
    }
    if (!fout.ptr && w->co % 8) {
      *why = "conv output channels must be a multiple of 8";
      return cudaErrorInvalidValue;
    }
    ConvArgs a;
    a.B = B;
    a.H = in.H;
    a.W = in.W;
    a.Ci = w->ci;
    a.Co = w->co;
    a.kh = w->kh;
    a.kw = w->kw;
    a.stride = stride;
    a.pad = pad;
    a.Ho = (in.H + 2 * pad - w->kh) / stride + 1;
    a.Wo = (in.W + 2 * pad - w->kw) / stride + 1;
    a.K = w->K;
    a.num_kc = w->num_kc;
    a.n_tile = w->n_tile;
    a.n_tiles = w->n_tiles;
    a.m_tiles = static_cast<int>((static_cast<long long>(B) * a.Ho * a.Wo + 127) / 128);
    a.src0 = in.v0;
    a.lg_up0 = in.lg0;
    if (in.c1) {
      a.c_split = in.c0;
      a.src1 = in.v1;
      a.lg_up1 = 0;
    } else {
      a.c_split = w->ci;
      a.src1 = in.v0;
      a.lg_up1 = in.lg0;
    }
    a.wpack = w->wpack;
    a.bias = w->bias;
    // Fewer than two waves of tiles: narrower N tiles (64 or 128 columns,
    // im2col operand mode) so that more SMs share the work.
    if (a.n_tiles * a.m_tiles < 2 * num_sms_ && w->co >= 128 && !fout.ptr && !w->merged) {
      const int nt = a.m_tiles * ((w->co + 127) / 128) >= 2 * num_sms_ ? 128 : 64;
      const uint8_t* wp = nullptr;
      YB_TRY(conv_narrow(const_cast<DevConv*>(w), nt, &wp));
      a.wpack = const_cast<uint8_t*>(wp);
      a.n_tile = nt;
      a.n_tiles = (w->co + nt - 1) / nt;
    }
    a.act = act;
    a.out = out;
    a.out_f32 = fout;
    a.res = res;
    a.err = d_err_;
    if (p->calib && !fout.ptr) a.amax = stat_slot(w->name, act == kActSiLU ? w->name + ":pre" : std::string());
    conv_setup_tma(&a);
    const int sms = num_sms_;
    Op op{step, [a, sms](cudaStream_t s) { return launch_conv_tc(a, s, sms); }};
    op.kind = kOpConv;
    const double pix_out = static_cast<double>(B) * a.Ho * a.Wo;
    op.flops = 2.0 * pix_out * a.Co * a.K;
    const double in0 = static_cast<double>(B) * (in.H >> in.lg0) * (in.W >> in.lg0) * in.c0;
    const double in1 = static_cast<double>(B) * in.H * in.W * in.c1;
    op.bytes = 4.0 * (in0 + in1 + static_cast<double>(a.Co) * (a.K + 1) + pix_out * a.Co * (res.hi ? 2 : 1));
    ops.push_back(op);
    return cudaSuccess;
  };
  auto add_op = [&](int kind, double flops, double bytes, std::function<cudaError_t(cudaStream_t)> fn) {
    Op op{step, std::move(fn)};
    op.kind = kind;
    op.flops = flops;
    op.bytes = bytes;
    ops.push_back(op);
  };
  auto conv = [&](const std::string& prefix, DevConv** w) { return conv_w(prefix, false, w, why); };
  auto exists = [&](const std::string& n) { return find(n) != nullptr; };

  auto downconv = [&](int li, const Buf& in, Buf* out) -> cudaError_t {
    DevConv* w;
    YB_TRY(conv("model." + std::to_string(li), &w));
    YB_TRY(alloc_buf((in.H + 2 - w->kh) / 2 + 1, (in.W + 2 - w->kw) / 2 + 1, w->co, out));
    return add_conv(w, src_of(in, 0, in.C), 2, (w->kh - 1) / 2, kActSiLU, ov(*out), SView());
  };
  // Bottleneck (layers.c:92-108): cv1+SiLU -> cv2+SiLU (+ input).  With
  // 3x3 convolutions C -> CM -> C ((C, CM) in bottleneck_supported) and a
  // shortcut, one fused launch (bottleneck_tc.cu, bit-identical to the pair
  // below) unless the plan gathers calibration statistics or fusion is
  // switched off.
  auto bottleneck = [&](const std::string& pre, const Src& in, SOut out, bool shortcut) -> cudaError_t {
    DevConv *w1, *w2;
    YB_TRY(conv(pre + ".cv1", &w1));
    YB_TRY(conv(pre + ".cv2", &w2));
    const int c = w1->ci, cm = w1->co;
    if (fuse_ && !p->calib && shortcut && !in.c1 && !in.lg0 && in.c0 == c && w1->kh == 3 && w1->kw == 3 &&
        w2->kh == 3 && w2->kw == 3 && w2->ci == cm && w2->co == c && bottleneck_supported(c, cm) &&
        w1->n_tiles == 1 && w1->n_tile == (cm + 15) / 16 * 16 && w2->n_tiles == 1 && w2->n_tile == c) {
      BottleneckArgs ba;
      ba.B = B;
      ba.H = in.H;
      ba.W = in.W;
      ba.C = c;
      ba.CM = cm;
      ba.in = in.v0;
      ba.out = out;
      ba.w1 = w1->wpack;
      ba.w2 = w2->wpack;
      ba.b1 = w1->bias;
      ba.b2 = w2->bias;
      ba.err = d_err_;
      if (bottleneck_setup(&ba)) {
        const double pix = static_cast<double>(B) * in.H * in.W;
        const int sms = num_sms_;
        add_op(kOpConv, 2.0 * 2.0 * pix * c * 9.0 * cm, 4.0 * (2.0 * pix * c + 2.0 * cm * (9.0 * c + 1.0)),
               [ba, sms](cudaStream_t s) { return launch_bottleneck(ba, s, sms); });
        return cudaSuccess;
      }
    }
    Buf t;
    YB_TRY(alloc_buf(in.H, in.W, w1->co, &t));
    YB_TRY(add_conv(w1, in, 1, (w1->kh - 1) / 2, kActSiLU, ov(t), SView()));
    return add_conv(w2, src_of(t, 0, t.C), 1, (w2->kh - 1) / 2, kActSiLU, out, shortcut ? in.v0 : SView());
  };
  // C3k2 without C3k (layers.c:110-154, model.c:208-283), shortcut bottlenecks.
  auto c3k2_plain = [&](int li, const Src& in, Buf* out) -> cudaError_t {
    const std::string L = "model." + std::to_string(li);
    DevConv *cv1, *cv2;
    YB_TRY(conv(L + ".cv1", &cv1));
    YB_TRY(conv(L + ".cv2", &cv2));
    const int c = cv1->co / 2;
    int n = 0;
    while (exists(L + ".m." + std::to_string(n) + ".cv1.conv.weight")) ++n;
    if (n < 1) {
      *why = L + ": no bottlenecks";
      return cudaErrorInvalidValue;
    }
    Buf cat;
    YB_TRY(alloc_buf(in.H, in.W, (2 + n) * c, &cat));
    YB_TRY(add_conv(cv1, in, 1, 0, kActSiLU, ov(cat, 0), SView()));
    int prev = c;
    for (int i = 0; i < n; ++i) {
      YB_TRY(bottleneck(L + ".m." + std::to_string(i), src_of(cat, prev, c), ov(cat, (2 + i) * c), true));
      prev = (2 + i) * c;
    }
    YB_TRY(alloc_buf(in.H, in.W, cv2->co, out));
    return add_conv(cv2, src_of(cat, 0, (2 + n) * c), 1, 0, kActSiLU, ov(*out), SView());
  };
  // C3k2 with an inner C3k (layers.c:156-189, model.c:415-557).
  auto c3k2_c3k = [&](int li, const Src& in, Buf* out) -> cudaError_t {
    const std::string L = "model." + std::to_string(li);
    DevConv *cv1, *cv2, *k1, *k2, *k3;
    YB_TRY(conv(L + ".cv1", &cv1));
    YB_TRY(conv(L + ".cv2", &cv2));
    YB_TRY(conv(L + ".m.0.cv1", &k1));
    YB_TRY(conv(L + ".m.0.cv2", &k2));
    YB_TRY(conv(L + ".m.0.cv3", &k3));
    const int c = cv1->co / 2;
    int nb = 0;
    while (exists(L + ".m.0.m." + std::to_string(nb) + ".cv1.conv.weight")) ++nb;
    if (nb < 1) {
      *why = L + ": no C3k bottlenecks";
      return cudaErrorInvalidValue;
    }
    Buf catO, y, catC;
    YB_TRY(alloc_buf(in.H, in.W, 2 * c + k3->co, &catO));
    YB_TRY(add_conv(cv1, in, 1, 0, kActSiLU, ov(catO, 0), SView()));
    const Src b = src_of(catO, c, c);
    const int cm = k1->co;
    YB_TRY(alloc_buf(in.H, in.W, cm + k2->co, &catC));
    Src cur;
    if (fuse_ && !p->calib && nb >= 2 && k1->ci == k2->ci && k1->kh == k2->kh && k1->kw == k2->kw) {
      // C3k's cv1 and cv2 read the same input: one launch writes both into
      // catC, cv1's half first.  The bottleneck chain reads that half, and
      // its last bottleneck (whose input is the previous one's output)
      // overwrites it with the chain's result.
      DevConv* k12;
      YB_TRY(conv_pair(L + ".m.0.cv1", L + ".m.0.cv2", &k12, why));
      YB_TRY(add_conv(k12, b, 1, 0, kActSiLU, ov(catC, 0), SView()));
      cur = src_of(catC, 0, cm);
    } else {
      YB_TRY(alloc_buf(in.H, in.W, cm, &y));
      YB_TRY(add_conv(k1, b, 1, 0, kActSiLU, ov(y), SView()));
      YB_TRY(add_conv(k2, b, 1, 0, kActSiLU, ov(catC, cm), SView()));
      cur = src_of(y, 0, cm);
    }
    for (int i = 0; i < nb; ++i) {
      const std::string pre = L + ".m.0.m." + std::to_string(i);
      if (i == nb - 1) {
        YB_TRY(bottleneck(pre, cur, ov(catC, 0), true));
      } else {
        Buf nxt;
        YB_TRY(alloc_buf(in.H, in.W, cm, &nxt));
        YB_TRY(bottleneck(pre, cur, ov(nxt), true));
        cur = src_of(nxt, 0, cm);
      }
    }
    YB_TRY(add_conv(k3, src_of(catC, 0, catC.C), 1, 0, kActSiLU, ov(catO, 2 * c), SView()));
    YB_TRY(alloc_buf(in.H, in.W, cv2->co, out));
    return add_conv(cv2, src_of(catO, 0, catO.C), 1, 0, kActSiLU, ov(*out), SView());
  };
  // SPPF k=5, 3 pools, shortcut (layers.c:230-265, model.c:285-320, :825).
  auto sppf = [&](int li, const Buf& in, Buf* out) -> cudaError_t {
    const std::string L = "model." + std::to_string(li);
    DevConv *cv1, *cv2;
    YB_TRY(conv(L + ".cv1", &cv1));
    YB_TRY(conv(L + ".cv2", &cv2));
    const int c = cv1->co;
    Buf cat;
    YB_TRY(alloc_buf(in.H, in.W, 4 * c, &cat));
    YB_TRY(add_conv(cv1, src_of(in, 0, in.C), 1, 0, kActNone, ov(cat, 0), SView()));
    if (c % 8 == 0 && sppf_pool_smem_bytes(in.H, in.W) <= kSppfSmemMax) {
      // The three pools in one launch (the 5x5, 9x9 and 13x13 pools of cv1).
      const SView src = tv(cat, 0);
      const SOut p1 = ov(cat, c), p2 = ov(cat, 2 * c), p3 = ov(cat, 3 * c);
      const int h = in.H, w = in.W;
      const double n = static_cast<double>(B) * h * w * c;
      add_op(kOpPool, 0.0, 8.0 * n, [=](cudaStream_t s) { return launch_sppf_pool(src, p1, p2, p3, B, h, w, c, s); });
    } else {
      for (int j = 0; j < 3; ++j) {
        PoolArgs pa;
        pa.in = tv(cat, j * c);
        pa.B = B;
        pa.H = in.H;
        pa.W = in.W;
        pa.C = c;
        pa.k = 5;
        pa.out = ov(cat, (j + 1) * c);
        const double n = static_cast<double>(B) * in.H * in.W * c;
        add_op(kOpPool, 0.0, 8.0 * n, [pa](cudaStream_t s) { return launch_maxpool(pa, s); });
      }
    }
    YB_TRY(alloc_buf(in.H, in.W, cv2->co, out));
    const bool res = in.C == cv2->co;
    return add_conv(cv2, src_of(cat, 0, cat.C), 1, 0, kActSiLU, ov(*out), res ? tv(in) : SView());
  };
  // PSABlock (layers.c:407-453) with attention (layers.c:310-405).
  auto psablock = [&](const std::string& pre, const Src& x, int c, SOut y, int heads) -> cudaError_t {
    DevConv *qkv, *proj, *f0, *f1;
    DevDw* pe;
    YB_TRY(conv(pre + ".attn.qkv", &qkv));
    YB_TRY(conv(pre + ".attn.proj", &proj));
    YB_TRY(conv(pre + ".ffn.0", &f0));
    YB_TRY(conv(pre + ".ffn.1", &f1));
    YB_TRY(dw_w(pre + ".attn.pe", &pe, why));
    if (c % heads) {
      *why = pre + ": channels not divisible by heads";
      return cudaErrorInvalidValue;
    }
    const int hd = c / heads;
    const int kd = static_cast<int>(static_cast<float>(hd) * 0.5f);
    if (qkv->co != c + 2 * kd * heads || pe->c != c) {
      *why = pre + ": qkv/pe width mismatch";
      return cudaErrorInvalidValue;
    }
    Buf q, ao, x1, f;
    YB_TRY(alloc_buf(x.H, x.W, qkv->co, &q));
    YB_TRY(add_conv(qkv, x, 1, 0, kActNone, ov(q), SView()));
    YB_TRY(alloc_buf(x.H, x.W, c, &ao));
    AttnArgs aa;
    aa.qkv = tv(q);
    aa.B = B;
    aa.H = x.H;
    aa.W = x.W;
    aa.heads = heads;
    aa.kd = kd;
    aa.hd = hd;
    aa.scale = std::pow(static_cast<float>(kd), -0.5f);
    aa.pe_w = pe->w;
    aa.pe_b = pe->bias;
    aa.out = ov(ao);
    aa.err = d_err_;
    if (p->calib) {
      // Attention output plus positional term: the INT8 plan's "<psa>.attn.ope".
      unsigned* st = stat_slot(pre + ".attn.ope", std::string());
      const SView av = tv(ao);
      const int h = x.H, w = x.W;
      add_op(kOpAttn, 0.0, 0.0, [aa](cudaStream_t s) { return launch_attention(aa, s); });
      add_op(kOpPool, 0.0, 0.0, [=](cudaStream_t s) { return launch_absmax_split(av, B, h, w, c, st, s); });
    } else {
      const double ntok = static_cast<double>(x.H) * x.W;
      const double fl = static_cast<double>(B) * heads * (2.0 * ntok * ntok * (kd + hd) + 18.0 * ntok * hd);
      const double by = 4.0 * B * ntok * (qkv->co + c) + 4.0 * 10.0 * c;
      add_op(kOpAttn, fl, by, [aa](cudaStream_t s) { return launch_attention(aa, s); });
    }
    YB_TRY(alloc_buf(x.H, x.W, c, &x1));
    YB_TRY(add_conv(proj, src_of(ao, 0, c), 1, 0, kActNone, ov(x1), x.v0));
    YB_TRY(alloc_buf(x.H, x.W, f0->co, &f));
    YB_TRY(add_conv(f0, src_of(x1, 0, c), 1, 0, kActSiLU, ov(f), SView()));
    return add_conv(f1, src_of(f, 0, f.C), 1, 0, kActNone, y, tv(x1));
  };
  // C2PSA (layers.c:455-496, model.c:322-412); blocks update the b half in place.
  auto c2psa = [&](int li, const Buf& in, Buf* out) -> cudaError_t {
    const std::string L = "model." + std::to_string(li);
    DevConv *cv1, *cv2;
    YB_TRY(conv(L + ".cv1", &cv1));
    YB_TRY(conv(L + ".cv2", &cv2));
    const int ch = static_cast<int>(static_cast<float>(in.C) * 0.5f);
    if (cv1->co != 2 * ch) {
      *why = L + ": cv1 width mismatch";
      return cudaErrorInvalidValue;
    }
    int heads = ch / 64;
    if (heads < 1) heads = 1;
    Buf cat;
    YB_TRY(alloc_buf(in.H, in.W, 2 * ch, &cat));
    YB_TRY(add_conv(cv1, src_of(in, 0, in.C), 1, 0, kActSiLU, ov(cat), SView()));
    int nb = 0;
    while (exists(L + ".m." + std::to_string(nb) + ".attn.qkv.conv.weight")) {
      YB_TRY(psablock(L + ".m." + std::to_string(nb), src_of(cat, ch, ch), ch, ov(cat, ch), heads));
      ++nb;
    }
    if (nb < 1) {
      *why = L + ": no PSA blocks";
      return cudaErrorInvalidValue;
    }
    YB_TRY(alloc_buf(in.H, in.W, cv2->co, out));
    return add_conv(cv2, src_of(cat, 0, cat.C), 1, 0, kActSiLU, ov(*out), SView());
  };
  // Head C3k2 with Bottleneck + PSABlock (model.c:560-665).
  auto c3k2_attn = [&](int li, const Src& in, Buf* out) -> cudaError_t {
    const std::string L = "model." + std::to_string(li);
    DevConv *cv1, *cv2;
    YB_TRY(conv(L + ".cv1", &cv1));
    YB_TRY(conv(L + ".cv2", &cv2));
    const int c = cv1->co / 2;
    Buf cat, bo;
    YB_TRY(alloc_buf(in.H, in.W, 3 * c, &cat));
    YB_TRY(add_conv(cv1, in, 1, 0, kActSiLU, ov(cat, 0), SView()));
    YB_TRY(alloc_buf(in.H, in.W, c, &bo));
    YB_TRY(bottleneck(L + ".m.0.0", src_of(cat, c, c), ov(bo), true));
    int heads = c / 64;
    if (heads < 1) heads = 1;
    YB_TRY(psablock(L + ".m.0.1", src_of(bo, 0, c), c, ov(cat, 2 * c), heads));
    YB_TRY(alloc_buf(in.H, in.W, cv2->co, out));
    return add_conv(cv2, src_of(cat, 0, cat.C), 1, 0, kActSiLU, ov(*out), SView());
  };

  Buf* S = p->stage;
  const int H = p->H, W = p->W;
  // step 0: stem (model.0), NCHW input read directly.
  step = 0;
  if (!stem_.w) {
    *why = "missing model.0.conv.weight/bias";
    return cudaErrorInvalidValue;
  }
  YB_TRY(alloc_raw(static_cast<size_t>(B) * 3 * H * W * 4, &p->d_in));
  {
    YB_TRY(alloc_buf((H + 2 - stem_.k) / 2 + 1, (W + 2 - stem_.k) / 2 + 1, stem_.co, &S[0]));
    StemArgs sa;
    sa.err = d_err_;
    sa.in = p->d_in;
    sa.B = B;
    sa.Ci = stem_.ci;
    sa.H = H;
    sa.W = W;
    sa.Co = stem_.co;
    sa.Ho = S[0].H;
    sa.Wo = S[0].W;
    sa.k = stem_.k;
    sa.w = stem_.w;
    sa.bias = stem_.bias;
    sa.act = kActSiLU;
    sa.out = ov(S[0]);
    if (p->calib) {
      unsigned* st = stat_slot("input", std::string());
      const float* din = p->d_in;
      const long long n = static_cast<long long>(B) * 3 * H * W;
      add_op(kOpPool, 0.0, 0.0, [=](cudaStream_t s) { return launch_absmax_f32(din, n, st, s); });
      sa.amax = stat_slot("model.0", "model.0:pre");
    }
    if (stem_.ci != 3 || stem_.k != 3) {
      *why = "unsupported stem";
      return cudaErrorInvalidValue;
    }
    const double po = static_cast<double>(B) * sa.Ho * sa.Wo;
    add_op(kOpStem, 2.0 * po * sa.Co * sa.Ci * 9, 4.0 * (static_cast<double>(B) * 3 * H * W + po * sa.Co),
           [sa](cudaStream_t s) { return launch_stem(sa, s); });
  }
  step = 1;
  YB_TRY(downconv(1, S[0], &S[1]));
  step = 2;
  YB_TRY(c3k2_plain(2, src_of(S[1], 0, S[1].C), &S[2]));
  step = 3;
  YB_TRY(downconv(3, S[2], &S[3]));
  step = 4;
  YB_TRY(c3k2_plain(4, src_of(S[3], 0, S[3].C), &S[4]));
  step = 5;
  YB_TRY(downconv(5, S[4], &S[5]));
  step = 6;
  YB_TRY(c3k2_c3k(6, src_of(S[5], 0, S[5].C), &S[6]));
  step = 7;
  YB_TRY(downconv(7, S[6], &S[7]));
  step = 8;
  YB_TRY(c3k2_c3k(8, src_of(S[7], 0, S[7].C), &S[8]));
  step = 9;
  YB_TRY(sppf(9, S[8], &S[9]));
  step = 10;
  YB_TRY(c2psa(10, S[9], &S[10]));
  // steps 11-12: upsample(buf10) ++ buf6, read in place by model.13's cv1.
  step = 13;
  YB_TRY(c3k2_c3k(13, src_cat(S[10], 1, S[6], S[6].H, S[6].W), &S[13]));
  // steps 14-15: upsample(buf13) ++ buf4.
  step = 16;
  YB_TRY(c3k2_c3k(16, src_cat(S[13], 1, S[4], S[4].H, S[4].W), &S[16]));
  const int after16 = static_cast<int>(ops.size()) - 1;
  step = 17;
  YB_TRY(downconv(17, S[16], &S[17]));
  // step 18: buf17 ++ buf13.
  step = 19;
  YB_TRY(c3k2_c3k(19, src_cat(S[17], 0, S[13], S[13].H, S[13].W), &S[19]));
  const int after19 = static_cast<int>(ops.size()) - 1;
  step = 20;
  YB_TRY(downconv(20, S[19], &S[20]));
  // step 21: buf20 ++ buf10.
  step = 22;
  YB_TRY(c3k2_attn(22, src_cat(S[20], 0, S[10], S[10].H, S[10].W), &S[22]));

  // step 23: Detect one2one (detect.c:253-454).
  step = 23;
  {
    const std::string d = "model." + std::to_string(23);
    const bool o2o = exists(d + ".one2one_cv2.0.0.conv.weight");
    const std::string b2 = d + (o2o ? ".one2one_cv2." : ".cv2.");
    const std::string b3 = d + (o2o ? ".one2one_cv3." : ".cv3.");
    const Buf* feats[3] = {&S[16], &S[19], &S[22]};
    const int strides[3] = {8, 16, 32};
    int N = 0, base[3];
    for (int s = 0; s < 3; ++s) {
      base[s] = N;
      N += feats[s]->H * feats[s]->W;
    }
    p->n_anchors = N;
    const int nc = nc_;
    if (nc < 1 || nc % 4) {
      *why = "num_classes must be a positive multiple of 4";
      return cudaErrorInvalidValue;
    }
    YB_TRY(alloc_raw(static_cast<size_t>(B) * N * 4 * 4, &p->d_dist));
    YB_TRY(alloc_raw(static_cast<size_t>(B) * N * nc * 4, &p->d_logits));
    YB_TRY(alloc_raw(static_cast<size_t>(B) * N * 4 * 4, &p->d_boxes));
    YB_TRY(alloc_raw(static_cast<size_t>(B) * N * 4, &p->d_maxscore));
    YB_TRY(alloc_raw(static_cast<size_t>(B) * p->max_det * 6 * 4, &p->d_out));
    for (int s = 0; s < 3; ++s) {
      const Buf& f = *feats[s];
      const std::string si = std::to_string(s);
      const size_t first_op = ops.size();
      DevConv *w0, *w1, *w2, *pw0, *pw1, *wf;
      DevDw *dw0, *dw1;
      YB_TRY(conv(b2 + si + ".0", &w0));
      YB_TRY(conv(b2 + si + ".1", &w1));
      YB_TRY(conv_w(b2 + si + ".2", true, &w2, why));
      YB_TRY(dw_w(b3 + si + ".0.0", &dw0, why));
      YB_TRY(conv(b3 + si + ".0.1", &pw0));
      YB_TRY(dw_w(b3 + si + ".1.0", &dw1, why));
      YB_TRY(conv(b3 + si + ".1.1", &pw1));
      YB_TRY(conv_w(b3 + si + ".2", true, &wf, why));
      if (w2->co != 4 || wf->co != nc) {
        *why = "detect head output widths";
        return cudaErrorInvalidValue;
      }
      // box branch (detect.c:168-191)
      Buf t1, t2;
      YB_TRY(alloc_buf(f.H, f.W, w0->co, &t1));
      YB_TRY(add_conv(w0, src_of(f, 0, f.C), 1, 1, kActSiLU, ov(t1), SView()));
      YB_TRY(alloc_buf(f.H, f.W, w1->co, &t2));
      YB_TRY(add_conv(w1, src_of(t1, 0, t1.C), 1, 1, kActSiLU, ov(t2), SView()));
      FOut dv;
      dv.ptr = p->d_dist + static_cast<size_t>(base[s]) * 4;
      dv.bstride = static_cast<long long>(N) * 4;
      dv.cstride = 4;
      YB_TRY(add_conv(w2, src_of(t2, 0, t2.C), 1, 0, kActNone, SOut(), SView(), dv));
      // class branch (detect.c:193-232)
      Buf d0, p0, d1, p1;
      YB_TRY(alloc_buf(f.H, f.W, f.C, &d0));
      DwArgs da;
      da.in = tv(f);
      da.B = B;
      da.H = f.H;
      da.W = f.W;
      da.C = f.C;
      da.w = dw0->w;
      da.bias = dw0->bias;
      da.act = kActSiLU;
      da.out = ov(d0);
      da.amax = stat_slot(b3 + si + ".0.0", b3 + si + ".0.0:pre");
      if (dw0->c != f.C) {
        *why = "detect dw width";
        return cudaErrorInvalidValue;
      }
      const double px = static_cast<double>(B) * f.H * f.W;
      add_op(kOpDw, 18.0 * px * f.C, 8.0 * px * f.C, [da](cudaStream_t st) { return launch_dwconv3x3(da, st); });
      YB_TRY(alloc_buf(f.H, f.W, pw0->co, &p0));
      YB_TRY(add_conv(pw0, src_of(d0, 0, d0.C), 1, 0, kActSiLU, ov(p0), SView()));
      YB_TRY(alloc_buf(f.H, f.W, p0.C, &d1));
      DwArgs db = da;
      db.in = tv(p0);
      db.C = p0.C;
      db.w = dw1->w;
      db.bias = dw1->bias;
      db.out = ov(d1);
      db.amax = stat_slot(b3 + si + ".1.0", b3 + si + ".1.0:pre");
      if (dw1->c != p0.C) {
        *why = "detect dw width";
        return cudaErrorInvalidValue;
      }
      add_op(kOpDw, 18.0 * px * p0.C, 8.0 * px * p0.C, [db](cudaStream_t st) { return launch_dwconv3x3(db, st); });
      YB_TRY(alloc_buf(f.H, f.W, pw1->co, &p1));
      YB_TRY(add_conv(pw1, src_of(d1, 0, d1.C), 1, 0, kActSiLU, ov(p1), SView()));
      FOut lv;
      lv.ptr = p->d_logits + static_cast<size_t>(base[s]) * nc;
      lv.bstride = static_cast<long long>(N) * nc;
      lv.cstride = nc;
      lv.rowmax = p->d_maxscore + base[s];
      lv.rm_bstride = N;
      YB_TRY(add_conv(wf, src_of(p1, 0, p1.C), 1, 0, kActNone, SOut(), SView(), lv));
      // The P3 and P4 heads read model.16 / model.19 only: side lanes 1 and
      // 2, beside the rest of the neck (inference plans).
      if (!p->calib && s < 2) {
        for (size_t i = first_op; i < ops.size(); ++i) ops[i].lane = s + 1;
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
    ops.back().join = true;
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
  }
  return cudaSuccess;
}

cudaError_t Engine::profile_ops(Plan* p, int reps, std::vector<double>* ms) {
  const size_t n = p->ops.size();
  ms->assign(n, 0.0);
  std::vector<cudaEvent_t> ev(2 * n, nullptr);
  cudaError_t e = cudaSuccess;
  for (auto& x : ev)
    if (e == cudaSuccess) e = cudaEventCreate(&x);
  for (int r = 0; r < reps && e == cudaSuccess; ++r) {
    for (size_t i = 0; i < n && e == cudaSuccess; ++i) {
      cudaEventRecord(ev[2 * i], stream_);
      e = p->ops[i].run(stream_);
      cudaEventRecord(ev[2 * i + 1], stream_);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
    for (size_t i = 0; i < n && e == cudaSuccess; ++i) {
      float t = 0.f;
      cudaEventElapsedTime(&t, ev[2 * i], ev[2 * i + 1]);
      (*ms)[i] += t / reps;
    }
  }
  for (auto& x : ev)
    if (x) cudaEventDestroy(x);
  return e;
}

void Engine::set_fusion(bool on) {
  if (on == fuse_) return;
  cudaSetDevice(device_);
  cudaStreamSynchronize(stream_);
  for (auto& q : plans_) release_plan(q.get());
  plans_.clear();
  fuse_ = on;
}

void Engine::set_int8_scales(std::map<std::string, float> s) {
  cudaSetDevice(device_);
  cudaStreamSynchronize(stream_);
  for (auto it = plans_.begin(); it != plans_.end();) {
    if ((*it)->int8) {
      release_plan(it->get());
      it = plans_.erase(it);
    } else {
      ++it;
    }
  }
  i8_scales_ = std::move(s);
}

cudaError_t Engine::get_plan(int B, int H, int W, int max_det, Plan** out, std::string* why, int slot) {
  for (auto& p : plans_) {
    if (p->B == B && p->H == H && p->W == W && p->max_det == max_det && p->slot == slot &&
        p->int8 == int8_mode()) {
      *out = p.get();
      return cudaSuccess;
    }
  }
  if (hw_.empty()) {
    *why = "no weights uploaded";
    return cudaErrorInvalidValue;
  }
  if (B < 1 || H < 32 || W < 32 || H % 32 || W % 32 || max_det < 1 || max_det > kTopkMax) {
    *why = "unsupported input shape (H, W must be multiples of 32; 1 <= max_det <= 1024)";
    return cudaErrorInvalidValue;
  }
  cudaSetDevice(device_);
  std::unique_ptr<Plan> p(new Plan());
  p->B = B;
  p->H = H;
  p->W = W;
  p->max_det = max_det;
  p->slot = slot;
  p->int8 = int8_mode();
  cudaError_t e = p->int8 ? build_i8(p.get(), why) : build(p.get(), why);
  for (int L = 1; L < 3 && e == cudaSuccess; ++L) {
    if (p->fork_after[L] < 0) continue;
    e = cudaStreamCreateWithFlags(&p->lane_s[L], cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->ev_fork[L], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->ev_join[L], cudaEventDisableTiming);
    if (e != cudaSuccess) *why = std::string("side streams: ") + cudaGetErrorString(e);
  }
  if (e != cudaSuccess) {
    release_plan(p.get());
    return e;
  }
  // One eager pass validates every launch before the graph is captured.
  cudaMemsetAsync(p->d_in, 0, static_cast<size_t>(B) * 3 * H * W * 4, stream_);
  e = run(p.get(), stream_, nullptr);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
  if (e != cudaSuccess) {
    *why = std::string("validation pass: ") + cudaGetErrorString(e);
    release_plan(p.get());
    return e;
  }
  const int kerr = take_kernel_error();
  if (kerr) {
    *why = "kernel error flag " + std::to_string(kerr) + " in validation pass";
    release_plan(p.get());
    return cudaErrorLaunchFailure;
  }
  cudaGraph_t g = nullptr;
  e = cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal);
  if (e == cudaSuccess) {
    e = run(p.get(), stream_, nullptr);  // no graph yet: the launches, side streams included
    cudaError_t e2 = cudaStreamEndCapture(stream_, &g);
    if (e == cudaSuccess) e = e2;
  }
  if (e == cudaSuccess) e = cudaGraphInstantiate(&p->graph, g, 0);
  if (g) cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    *why = std::string("graph capture: ") + cudaGetErrorString(e);
    release_plan(p.get());
    return e;
  }
  *out = p.get();
  plans_.push_back(std::move(p));
  return cudaSuccess;
}

cudaError_t Engine::calibrate(const float* images, int n, int H, int W, std::map<std::string, float>* table,
                              std::string* why) {
  if (hw_.empty()) {
    *why = "no weights uploaded";
    return cudaErrorInvalidValue;
  }
  if (n < 1 || H < 32 || W < 32 || H % 32 || W % 32) {
    *why = "calibration needs n >= 1 images with H, W multiples of 32";
    return cudaErrorInvalidValue;
  }
  cudaSetDevice(device_);
  Plan p;
  p.B = 1;
  p.H = H;
  p.W = W;
  p.calib = true;
  cudaError_t e = build(&p, why);
  if (e == cudaSuccess && p.amax_used > p.amax_cap) {
    *why = "calibration statistics table too small";
    e = cudaErrorInvalidValue;
  }
  const size_t img = static_cast<size_t>(3) * H * W;
  for (int i = 0; i < n && e == cudaSuccess; ++i) {
    e = cudaMemcpyAsync(p.d_in, images + i * img, img * 4, cudaMemcpyHostToDevice, stream_);
    if (e == cudaSuccess) e = run(&p, stream_, nullptr);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
  std::vector<unsigned> words(p.amax_cap);
  if (e == cudaSuccess)
    e = cudaMemcpy(words.data(), p.d_amax, words.size() * sizeof(unsigned), cudaMemcpyDeviceToHost);
  const int kerr = take_kernel_error();
  if (e == cudaSuccess && kerr) {
    *why = "kernel error flag " + std::to_string(kerr) + " during calibration";
    e = cudaErrorLaunchFailure;
  }
  if (e == cudaSuccess) {
    std::map<std::string, float> amax;
    for (const auto& nk : p.amax_names) {
      float v;
      std::memcpy(&v, &words[nk.second], sizeof v);
      auto it = amax.find(nk.first);
      if (it == amax.end()) amax[nk.first] = v;
      else if (v > it->second) it->second = v;
    }
    table->clear();
    for (const auto& kv : amax) (*table)[kv.first] = kv.second > 0.0f ? kv.second / 127.0f : 1.0f;
  }
  release_plan(&p);
  return e;
}

cudaError_t Engine::run(Plan* p, cudaStream_t s, cudaEvent_t* ev) {
  if (!ev && p->graph) return cudaGraphLaunch(p->graph, s);
  // Side lanes only without per-step events (those time every op in order).
  const bool lanes = !ev;
  bool started[3] = {true, false, false};
  auto join_lanes = [&]() -> cudaError_t {
    for (int L = 1; L < 3; ++L) {
      if (!started[L]) continue;
      cudaError_t e = cudaEventRecord(p->ev_join[L], p->lane_s[L]);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(s, p->ev_join[L], 0);
      if (e != cudaSuccess) return e;
      started[L] = false;
    }
    return cudaSuccess;
  };
  int cur = -1;
  for (size_t i = 0; i < p->ops.size(); ++i) {
    const Op& op = p->ops[i];
    if (ev && op.step != cur) {
      if (cur >= 0) cudaEventRecord(ev[2 * cur + 1], s);
      cur = op.step;
      cudaEventRecord(ev[2 * cur], s);
    }
    cudaStream_t st = s;
    if (lanes && op.join) {
      cudaError_t e = join_lanes();
      if (e != cudaSuccess) return e;
    }
    if (lanes && op.lane > 0 && p->lane_s[op.lane]) {
      st = p->lane_s[op.lane];
      if (!started[op.lane]) {
        cudaError_t e = cudaStreamWaitEvent(st, p->ev_fork[op.lane], 0);
        if (e != cudaSuccess) return e;
        started[op.lane] = true;
      }
    }
    cudaError_t e = op.run(st);
    if (e != cudaSuccess) return e;
    for (int L = 1; lanes && L < 3; ++L) {
      if (p->lane_s[L] && p->fork_after[L] == static_cast<int>(i)) {
        e = cudaEventRecord(p->ev_fork[L], s);
        if (e != cudaSuccess) return e;
      }
    }
  }
  if (ev && cur >= 0) cudaEventRecord(ev[2 * cur + 1], s);
  return lanes ? join_lanes() : cudaSuccess;
}

}  // namespace yb
