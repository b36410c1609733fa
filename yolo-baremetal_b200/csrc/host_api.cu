// Host entry points: the reference's model/tensor/utils/detect/detection API
// (phucb2/yolo-baremetal include/*.h) and the yb_cuda_* C-ABI shim, on top of
// the device engine.  Every status code follows status.h; CUDA failures are
// mapped by cuda_status() and described by yb_cuda_last_error().
#include <time.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "detect.h"
#include "detection.h"
#include "engine.h"
#include "i8k.h"
#include "model.h"
#include "runtime.h"
#include "tensor.h"
#include "utils.h"
#include "yb_cuda.h"

namespace yb {

namespace {
thread_local std::string g_err;
}

void set_error(const std::string& msg) { g_err = msg; }
const char* last_error() { return g_err.c_str(); }

status_t cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SUCCESS;
  set_error(std::string(what) + ": " + cudaGetErrorString(e));
  return e == cudaErrorMemoryAllocation ? ERROR_OUT_OF_MEMORY : ERROR_DEVICE;
}

DevScope* current_scope() {
  thread_local std::map<int, DevScope> scopes;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error(std::string("no CUDA device: ") + cudaGetErrorString(e));
    return nullptr;
  }
  auto it = scopes.find(dev);
  if (it != scopes.end()) return &it->second;
  DevScope s;
  s.device = dev;
  if ((e = cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaMalloc(&s.d_err, sizeof(int))) != cudaSuccess || (e = cudaMemset(s.d_err, 0, sizeof(int))) != cudaSuccess ||
      (e = init_conv_kernel_attributes()) != cudaSuccess) {
    set_error(std::string("device scope: ") + cudaGetErrorString(e));
    return nullptr;
  }
  cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev);
  return &scopes.emplace(dev, s).first->second;
}

// One device replica behind a void* context.
constexpr int kPipeSlotsMax = 4;  // stream / event arrays of a context

struct Ctx {
  std::unique_ptr<Engine> eng;
  Plan* last = nullptr;
  cudaEvent_t ev[2 * MODEL_FORWARD_PROFILE_STEPS] = {};
  cudaEvent_t h2d_done = nullptr;
  cudaEvent_t done = nullptr;
  float* h_stage = nullptr;  // pinned staging for detections of a sharded call
  size_t h_stage_bytes = 0;
  bool inflight = false;
  int stall_ms = 0;  // host-side fault injection for deadline tests
  // Pipelined host forwards: input copies run on copy_stream while the
  // previous sub-batch computes; one event pair per plan slot.
  cudaStream_t copy_stream = nullptr;
  cudaStream_t slot_stream[kPipeSlotsMax] = {};
  cudaEvent_t in_ready[kPipeSlotsMax] = {};
  cudaEvent_t slot_free[kPipeSlotsMax] = {};
  // Device staging of yb_cuda_forward_rgb8's 8-bit input (grown on demand).
  uint8_t* d_rgb = nullptr;
  size_t d_rgb_bytes = 0;
  // Scale table of the last yb_cuda_calibrate_int8, in name order.
  std::vector<std::pair<std::string, float>> calib;
  // Streaming forwards (yb_cuda_forward_submit / _wait): two slots, each a
  // plan (tag kStreamTag + slot) on its own stream, with its own 8-bit input
  // staging; ticket 0 marks a free slot.
  struct StreamSlot {
    cudaStream_t st = nullptr;
    cudaEvent_t h2d = nullptr, done = nullptr;
    long long ticket = 0;
    Plan* plan = nullptr;
    uint8_t* d_rgb = nullptr;
    size_t d_rgb_bytes = 0;
  };
  StreamSlot sslot[2];
  int sslot_next = 0;
  long long next_ticket = 1;
};
constexpr int kStreamTag = 8;

// Sub-batch of a pipelined host forward (yb_cuda_forward with B >= 2 chunks)
// and the number of plan slots (each with its own stream) it rotates over.
constexpr int kPipeChunk = 16;
constexpr int kPipeSlots = 3;
static_assert(kPipeSlots <= kPipeSlotsMax, "pipeline slots");

namespace {

Ctx* as_ctx(void* p) { return static_cast<Ctx*>(p); }

status_t ctx_ready(Ctx* c) {
  if (!c) return ERROR_NULL_POINTER;
  cudaError_t e = cudaSetDevice(c->eng->device());
  if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  if (c->inflight) {
    e = cudaEventSynchronize(c->done);
    if (e != cudaSuccess) return cuda_status(e, "previous call");
    c->inflight = false;
  }
  return SUCCESS;
}

status_t check_kernel_flag(Ctx* c) {
  const int k = c->eng->take_kernel_error();
  if (k) {
    set_error("device kernel reported error code " + std::to_string(k));
    return ERROR_DEVICE;
  }
  return SUCCESS;
}

// Waits for the streaming batch in slot S and frees the slot.
status_t finish_stream_slot(Ctx* c, Ctx::StreamSlot& S) {
  if (!S.ticket) return SUCCESS;
  const cudaError_t e = cudaEventSynchronize(S.done);
  S.ticket = 0;
  if (e != cudaSuccess) return cuda_status(e, "streaming forward");
  c->last = S.plan;
  return check_kernel_flag(c);
}

// Finishes every streaming batch in flight (before plans are replaced).
status_t drain_stream(Ctx* c) {
  status_t st = SUCCESS;
  for (auto& S : c->sslot) {
    const status_t s2 = finish_stream_slot(c, S);
    if (st == SUCCESS) st = s2;
  }
  return st;
}

status_t plan_for(Ctx* c, int B, int H, int W, int max_det, Plan** p, int slot = 0) {
  std::string why;
  cudaError_t e = c->eng->get_plan(B, H, W, max_det, p, &why, slot);
  if (e == cudaSuccess) return SUCCESS;
  if (e == cudaErrorInvalidValue) {
    set_error("plan: " + why);
    return why.rfind("missing", 0) == 0 ? ERROR_FILE_NOT_FOUND : ERROR_INVALID_DIMS;
  }
  const status_t st = cuda_status(e, "plan");
  set_error(std::string(last_error()) + (why.empty() ? "" : " (" + why + ")"));
  return st;
}

// Stage tensors of image 0 in the reference's order and names (model.c:782-887).
status_t dump_stages(Ctx* c, Plan* p, const float* in_nchw, yb_stage_cb cb, void* user) {
  cudaStream_t s = c->eng->stream();
  const Buf* S = p->stage;
  size_t maxe = static_cast<size_t>(3) * p->H * p->W;
  for (int i = 0; i < 23; ++i)
    if (S[i].hi) maxe = std::max(maxe, static_cast<size_t>(S[i].H) * S[i].W * S[i].C * 2);
  DevMem t0, t1;
  cudaError_t e = t0.alloc(maxe * 4);
  if (e == cudaSuccess) e = t1.alloc(maxe * 4);
  if (e != cudaSuccess) return cuda_status(e, "stage dump buffers");
  std::vector<float> host(maxe);
  auto tv = [](const Buf& b) {
    SView v;
    v.hi = b.hi;
    v.plane = b.plane;
    v.bstride = b.bstride;
    v.cstride = b.C;
    return v;
  };
  auto emit = [&](const char* name, SView v, int C, int H, int W) -> status_t {
    cudaError_t er = launch_split_to_nchw(v, 1, C, H, W, t1.f(), s);
    if (er == cudaSuccess) er = cudaMemcpyAsync(host.data(), t1.p, static_cast<size_t>(C) * H * W * 4, cudaMemcpyDeviceToHost, s);
    if (er == cudaSuccess) er = cudaStreamSynchronize(s);
    if (er != cudaSuccess) return cuda_status(er, name);
    cb(user, name, host.data(), 1, C, H, W);
    return SUCCESS;
  };
  auto emit_buf = [&](const char* name, int k) { return emit(name, tv(S[k]), S[k].C, S[k].H, S[k].W); };
  auto emit_cat = [&](const char* name, const Buf& a, int up, const Buf* b, int H, int W) -> status_t {
    SOut o;
    o.hi = static_cast<uint16_t*>(t0.p);
    o.cstride = a.C + (b ? b->C : 0);
    o.bstride = static_cast<long long>(H) * W * o.cstride;
    o.plane = o.bstride;
    SView bv = b ? tv(*b) : tv(a);
    cudaError_t er = launch_gather_concat(tv(a), a.C, up, bv, b ? b->C : 0, 1, H, W, o, s);
    if (er != cudaSuccess) return cuda_status(er, name);
    SView v;
    v.hi = o.hi;
    v.plane = o.plane;
    v.cstride = o.cstride;
    v.bstride = o.bstride;
    return emit(name, v, o.cstride, H, W);
  };
  status_t st;
  cb(user, "stage_00_input", in_nchw, 1, 3, p->H, p->W);
  static const char* direct[11] = {"stage_01_buf0", "stage_02_buf1", "stage_03_buf2", "stage_04_buf3",
                                   "stage_05_buf4", "stage_06_buf5", "stage_07_buf6", "stage_08_buf7",
                                   "stage_09_buf8", "stage_10_buf9", "stage_11_buf10"};
  for (int k = 0; k <= 10; ++k)
    if ((st = emit_buf(direct[k], k)) != SUCCESS) return st;
  if ((st = emit_cat("stage_12_buf11", S[10], 2, nullptr, S[6].H, S[6].W)) != SUCCESS) return st;
  if ((st = emit_cat("stage_13_buf12", S[10], 2, &S[6], S[6].H, S[6].W)) != SUCCESS) return st;
  if ((st = emit_buf("stage_14_buf13", 13)) != SUCCESS) return st;
  if ((st = emit_cat("stage_15_buf14", S[13], 2, nullptr, S[4].H, S[4].W)) != SUCCESS) return st;
  if ((st = emit_cat("stage_16_buf15", S[13], 2, &S[4], S[4].H, S[4].W)) != SUCCESS) return st;
  if ((st = emit_buf("stage_17_buf16", 16)) != SUCCESS) return st;
  if ((st = emit_buf("stage_18_buf17", 17)) != SUCCESS) return st;
  if ((st = emit_cat("stage_19_buf18", S[17], 1, &S[13], S[13].H, S[13].W)) != SUCCESS) return st;
  if ((st = emit_buf("stage_20_buf19", 19)) != SUCCESS) return st;
  if ((st = emit_buf("stage_21_buf20", 20)) != SUCCESS) return st;
  if ((st = emit_cat("stage_22_buf21", S[20], 1, &S[10], S[10].H, S[10].W)) != SUCCESS) return st;
  if ((st = emit_buf("stage_23_buf22", 22)) != SUCCESS) return st;
  std::vector<float> dets(static_cast<size_t>(p->max_det) * 6);
  e = cudaMemcpy(dets.data(), p->d_out, dets.size() * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "stage dump detections");
  cb(user, "stage_24_buf23", dets.data(), 1, p->max_det, 6, 1);
  cb(user, "stage_25_detect", dets.data(), 1, p->max_det, 6, 1);
  return SUCCESS;
}

// Stage tensor k of image `image` of an INT8 plan as NCHW int8 on the host.
status_t fetch_i8_stage(Ctx* c, Plan* p, int k, int image, int8_t* out) {
  const Plan::I8Stage& S = p->i8stage[k];
  cudaStream_t s = c->eng->stream();
  DevMem t;
  const size_t n = static_cast<size_t>(S.C) * S.H * S.W;
  cudaError_t e = t.alloc(n);
  I8View v;
  v.p = S.p + static_cast<long long>(image) * S.bstride;
  v.cstride = S.cstride;
  v.bstride = S.bstride;
  if (e == cudaSuccess) e = launch_nhwc_to_nchw_i8(v, S.C, S.H, S.W, static_cast<int8_t*>(t.p), s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, t.p, n, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return cuda_status(e, "int8 stage fetch");
}

// Stage tensors of image 0 of an INT8 forward, dequantised (q * scale of its
// channel), under the reference's stage names.
status_t dump_stages_i8(Ctx* c, Plan* p, const float* in_nchw, yb_stage_cb cb, void* user) {
  cb(user, "stage_00_input", in_nchw, 1, 3, p->H, p->W);
  std::vector<int8_t> q;
  std::vector<float> f;
  char name[32];
  for (int k = 0; k < 23; ++k) {
    const Plan::I8Stage& S = p->i8stage[k];
    const size_t hw = static_cast<size_t>(S.H) * S.W;
    q.resize(hw * S.C);
    f.resize(hw * S.C);
    const status_t st = fetch_i8_stage(c, p, k, 0, q.data());
    if (st != SUCCESS) return st;
    for (int ch = 0; ch < S.C; ++ch)
      for (size_t i = 0; i < hw; ++i) f[ch * hw + i] = static_cast<float>(q[ch * hw + i]) * S.cs[ch];
    snprintf(name, sizeof name, "stage_%02d_buf%d", k + 1, k);
    cb(user, name, f.data(), 1, S.C, S.H, S.W);
  }
  std::vector<float> dets(static_cast<size_t>(p->max_det) * 6);
  cudaError_t e = cudaMemcpy(dets.data(), p->d_out, dets.size() * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "stage dump detections");
  cb(user, "stage_24_buf23", dets.data(), 1, p->max_det, 6, 1);
  cb(user, "stage_25_detect", dets.data(), 1, p->max_det, 6, 1);
  return SUCCESS;
}

status_t set_int8(Ctx* c, const char* const* names, const float* scales, int n) {
  if (n < 0 || (n > 0 && (!names || !scales))) return n < 0 ? ERROR_INVALID_DIMS : ERROR_NULL_POINTER;
  std::map<std::string, float> t;
  for (int i = 0; i < n; ++i) {
    if (!names[i]) return ERROR_NULL_POINTER;
    if (!(scales[i] > 0.0f) || !std::isfinite(scales[i])) {
      set_error(std::string("int8 scale not positive and finite: ") + names[i]);
      return ERROR_INVALID_DIMS;
    }
    t[names[i]] = scales[i];
  }
  c->eng->set_int8_scales(std::move(t));
  c->last = nullptr;
  return SUCCESS;
}

void weights_from_model(const model_t* m, WeightMap* out) {
  for (int i = 0; i < m->num_weights; ++i) {
    const tensor_t& t = m->weights[i].tensor;
    HostTensor h;
    h.ndim = 4;
    size_t n = 1;
    for (int d = 0; d < 4; ++d) {
      h.dims[d] = t.dims[d];
      n *= static_cast<size_t>(t.dims[d]);
    }
    h.data.assign(t.data, t.data + n);
    (*out)[m->weights[i].name] = std::move(h);
  }
}

// Model side table: device replicas keyed by model_t*, so model_t keeps the
// reference's layout.
std::mutex g_models_mu;
std::map<const model_t*, Ctx*> g_models;

Ctx* model_ctx(const model_t* m) {
  std::lock_guard<std::mutex> lk(g_models_mu);
  auto it = g_models.find(m);
  return it == g_models.end() ? nullptr : it->second;
}

}  // namespace
}  // namespace yb

using namespace yb;

// ====================================================================== shim
extern "C" const char* yb_cuda_last_error(void) { return yb::last_error(); }

extern "C" status_t yb_cuda_init(int device, void** ctx) {
  if (!ctx) return ERROR_NULL_POINTER;
  *ctx = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceCount");
  if (device < 0 || device >= n) {
    set_error("device index out of range");
    return ERROR_INVALID_DIMS;
  }
  if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  status_t pst = noalloc_prepare_current_device();
  if (pst != SUCCESS) return pst;
  std::unique_ptr<Ctx> c(new Ctx());
  c->eng.reset(new Engine(device));
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_status(e, "engine init");
  for (auto& ev : c->ev)
    if ((e = cudaEventCreate(&ev)) != cudaSuccess) return cuda_status(e, "cudaEventCreate");
  if ((e = cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming)) != cudaSuccess ||
      (e = cudaEventCreateWithFlags(&c->h2d_done, cudaEventDisableTiming)) != cudaSuccess)
    return cuda_status(e, "cudaEventCreate");
  if ((e = cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking)) != cudaSuccess)
    return cuda_status(e, "cudaStreamCreate");
  for (int i = 0; i < kPipeSlots; ++i)
    if ((e = cudaEventCreateWithFlags(&c->in_ready[i], cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&c->slot_free[i], cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaStreamCreateWithFlags(&c->slot_stream[i], cudaStreamNonBlocking)) != cudaSuccess)
      return cuda_status(e, "cudaEventCreate");
  for (auto& S : c->sslot)
    if ((e = cudaEventCreateWithFlags(&S.h2d, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&S.done, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaStreamCreateWithFlags(&S.st, cudaStreamNonBlocking)) != cudaSuccess)
      return cuda_status(e, "cudaEventCreate");
  *ctx = c.release();
  return SUCCESS;
}

extern "C" status_t yb_cuda_destroy(void* ctx) {
  Ctx* c = as_ctx(ctx);
  if (!c) return ERROR_NULL_POINTER;
  cudaSetDevice(c->eng->device());
  if (c->inflight) cudaEventSynchronize(c->done);
  drain_stream(c);
  for (auto& S : c->sslot) {
    if (S.st) {
      cudaStreamSynchronize(S.st);
      cudaStreamDestroy(S.st);
    }
    if (S.h2d) cudaEventDestroy(S.h2d);
    if (S.done) cudaEventDestroy(S.done);
    if (S.d_rgb) cudaFree(S.d_rgb);
  }
  for (auto& ev : c->ev)
    if (ev) cudaEventDestroy(ev);
  if (c->done) cudaEventDestroy(c->done);
  if (c->h2d_done) cudaEventDestroy(c->h2d_done);
  for (int i = 0; i < kPipeSlots; ++i) {
    if (c->in_ready[i]) cudaEventDestroy(c->in_ready[i]);
    if (c->slot_free[i]) cudaEventDestroy(c->slot_free[i]);
    if (c->slot_stream[i]) {
      cudaStreamSynchronize(c->slot_stream[i]);
      cudaStreamDestroy(c->slot_stream[i]);
    }
  }
  if (c->copy_stream) {
    cudaStreamSynchronize(c->copy_stream);
    cudaStreamDestroy(c->copy_stream);
  }
  if (c->h_stage) cudaFreeHost(c->h_stage);
  if (c->d_rgb) cudaFree(c->d_rgb);
  c->eng.reset();
  delete c;
  return SUCCESS;
}

extern "C" status_t yb_cuda_upload_weights(void* ctx, const model_t* m, yb_precision p, const void* qparams) {
  Ctx* c = as_ctx(ctx);
  if (!c || !m) return ERROR_NULL_POINTER;
  if ((p != YB_PRECISION_FP32 && p != YB_PRECISION_INT8) || (p == YB_PRECISION_FP32 && qparams)) {
    set_error("precision must be YB_PRECISION_FP32 (qparams NULL) or YB_PRECISION_INT8");
    return ERROR_INVALID_DIMS;
  }
  if (p == YB_PRECISION_INT8 && !qparams) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  // Plans are replaced below: finish the streaming batches using them.
  if ((st = drain_stream(c)) != SUCCESS) return st;
  WeightMap w;
  weights_from_model(m, &w);
  std::string why;
  cudaError_t e = c->eng->set_weights(std::move(w), m->num_classes, &why);
  if (e == cudaErrorInvalidValue) {
    set_error(why);
    return ERROR_FILE_NOT_FOUND;
  }
  c->last = nullptr;
  st = cuda_status(e, "upload weights");
  if (st != SUCCESS) return st;
  if (p == YB_PRECISION_INT8) {
    const auto* q = static_cast<const yb_int8_scales*>(qparams);
    return set_int8(c, q->names, q->scales, q->n);
  }
  return set_int8(c, nullptr, nullptr, 0);
}

extern "C" status_t yb_cuda_set_int8(void* ctx, const char* const* names, const float* scales, int n) {
  Ctx* c = as_ctx(ctx);
  if (!c) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  // Plans are replaced below: finish the streaming batches using them.
  if ((st = drain_stream(c)) != SUCCESS) return st;
  return set_int8(c, names, scales, n);
}

extern "C" status_t yb_cuda_set_fusion(void* ctx, int enable) {
  Ctx* c = as_ctx(ctx);
  if (!c) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  if ((st = drain_stream(c)) != SUCCESS) return st;
  c->eng->set_fusion(enable != 0);
  c->last = nullptr;
  return SUCCESS;
}

extern "C" status_t yb_cuda_calibrate_int8(void* ctx, const float* images, int n, int H, int W, int apply,
                                           int* n_scales) {
  Ctx* c = as_ctx(ctx);
  if (!c || !images) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  // Plans are replaced below: finish the streaming batches using them.
  if ((st = drain_stream(c)) != SUCCESS) return st;
  std::map<std::string, float> table;
  std::string why;
  cudaError_t e = c->eng->calibrate(images, n, H, W, &table, &why);
  if (e == cudaErrorInvalidValue) {
    set_error("calibration: " + why);
    return ERROR_INVALID_DIMS;
  }
  if (e != cudaSuccess) {
    st = cuda_status(e, "calibration");
    if (!why.empty()) set_error(std::string(last_error()) + " (" + why + ")");
    return st;
  }
  c->calib.assign(table.begin(), table.end());
  if (n_scales) *n_scales = static_cast<int>(c->calib.size());
  if (apply) c->eng->set_int8_scales(std::move(table));
  if (apply) c->last = nullptr;
  return SUCCESS;
}

extern "C" status_t yb_cuda_int8_scale_entry(void* ctx, int i, char* name, int cap, float* scale) {
  Ctx* c = as_ctx(ctx);
  if (!c) return ERROR_NULL_POINTER;
  if (i < 0 || i >= static_cast<int>(c->calib.size())) return ERROR_INVALID_DIMS;
  const std::string& nm = c->calib[i].first;
  if (name) {
    if (cap < static_cast<int>(nm.size()) + 1) return ERROR_INVALID_DIMS;
    std::memcpy(name, nm.c_str(), nm.size() + 1);
  }
  if (scale) *scale = c->calib[i].second;
  return SUCCESS;
}

extern "C" status_t yb_cuda_get_int8_stage(void* ctx, int idx, int image, signed char* out_nchw, float* scales,
                                           int* c_out, int* h_out, int* w_out) {
  Ctx* c = as_ctx(ctx);
  if (!c) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  Plan* p = c->last;
  if (!p || !p->int8) {
    set_error("no int8 stage tensors kept: the last forward was not a non-pipelined INT8 forward");
    return ERROR_INVALID_DIMS;
  }
  if (idx < 0 || idx >= static_cast<int>(p->i8stage.size()) || image < 0 || image >= p->B) return ERROR_INVALID_DIMS;
  const Plan::I8Stage& S = p->i8stage[idx];
  if (c_out) *c_out = S.C;
  if (h_out) *h_out = S.H;
  if (w_out) *w_out = S.W;
  if (scales) std::copy(S.cs.begin(), S.cs.end(), scales);
  if (!out_nchw) return SUCCESS;
  cudaError_t e = cudaStreamSynchronize(c->eng->stream());
  if (e != cudaSuccess) return cuda_status(e, "int8 stage");
  return fetch_i8_stage(c, p, idx, image, reinterpret_cast<int8_t*>(out_nchw));
}

extern "C" status_t yb_cuda_load_bin(void* ctx, const char* path) {
  Ctx* c = as_ctx(ctx);
  if (!c || !path) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  // Plans are replaced below: finish the streaming batches using them.
  if ((st = drain_stream(c)) != SUCCESS) return st;
  WeightMap w;
  int nc = 0;
  std::string why;
  if (!read_weight_bin(path, &w, &nc, &why)) {
    set_error(why);
    return why.rfind("cannot open", 0) == 0 ? ERROR_FILE_NOT_FOUND : ERROR_INVALID_FORMAT;
  }
  fold_all_bn_map(&w);
  cudaError_t e = c->eng->set_weights(std::move(w), nc, &why);
  if (e == cudaErrorInvalidValue) {
    set_error(why);
    return ERROR_FILE_NOT_FOUND;
  }
  c->last = nullptr;
  return cuda_status(e, "upload weights");
}

extern "C" status_t yb_cuda_load_bin_device(void* ctx, const char* path) {
  Ctx* c = as_ctx(ctx);
  if (!c || !path) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  if ((st = drain_stream(c)) != SUCCESS) return st;
  WeightMap w;
  int nc = 0;
  std::string why;
  if (!read_weight_bin(path, &w, &nc, &why)) {
    set_error(why);
    return why.rfind("cannot open", 0) == 0 ? ERROR_FILE_NOT_FOUND : ERROR_INVALID_FORMAT;
  }
  cudaError_t e = c->eng->set_weights_device(std::move(w), nc, &why);
  c->last = nullptr;
  if (e == cudaErrorInvalidValue) {
    set_error(why);
    return ERROR_INVALID_FORMAT;
  }
  return cuda_status(e, "device weight preparation");
}

extern "C" status_t yb_cuda_save_prepared(void* ctx, const char* path) {
  Ctx* c = as_ctx(ctx);
  if (!c || !path) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  if ((st = drain_stream(c)) != SUCCESS) return st;
  std::string why;
  cudaError_t e = c->eng->save_blob(path, &why);
  if (e == cudaErrorInvalidValue) {
    set_error(why);
    return ERROR_FILE_NOT_FOUND;
  }
  return cuda_status(e, "save prepared weights");
}

extern "C" status_t yb_cuda_load_prepared(void* ctx, const char* path) {
  Ctx* c = as_ctx(ctx);
  if (!c || !path) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  if ((st = drain_stream(c)) != SUCCESS) return st;
  std::string why;
  int nc = 0;
  cudaError_t e = c->eng->load_blob(path, &nc, &why);
  c->last = nullptr;
  if (e == cudaErrorInvalidValue) {
    set_error(why);
    return why.rfind("cannot open", 0) == 0 ? ERROR_FILE_NOT_FOUND : ERROR_INVALID_FORMAT;
  }
  return cuda_status(e, "load prepared weights");
}

extern "C" status_t yb_cuda_weight_image(void* ctx, const char* name, int kind, int n_tile, void* out, size_t cap,
                                         size_t* bytes) {
  Ctx* c = as_ctx(ctx);
  if (!c || !name) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  std::vector<uint8_t> img;
  std::string why;
  cudaError_t e = c->eng->weight_image(name, kind, n_tile, &img, &why);
  if (e == cudaErrorInvalidValue) {
    set_error(why);
    return ERROR_FILE_NOT_FOUND;
  }
  if (e != cudaSuccess) return cuda_status(e, "weight image");
  if (bytes) *bytes = img.size();
  if (out) {
    if (cap < img.size()) {
      set_error("weight image: buffer too small");
      return ERROR_INVALID_DIMS;
    }
    std::memcpy(out, img.data(), img.size());
  }
  return SUCCESS;
}

extern "C" status_t yb_cuda_forward(void* ctx, const float* in_nchw, int B, int H, int W, float* out_dets,
                                    int max_det, yb_stage_cb dump, void* user, double* step_ms) {
  Ctx* c = as_ctx(ctx);
  if (!c || !in_nchw || !out_dets) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  Plan* p = nullptr;
  cudaStream_t s = c->eng->stream();
  if (!dump && !step_ms && B >= 2 * kPipeChunk && B % kPipeChunk == 0) {
    // Pipelined: sub-batches of kPipeChunk images rotate over kPipeSlots
    // plans, each with its own stream.  The input copies run back to back on
    // the copy stream; chunk i's graph starts when its copy lands and may
    // overlap the graphs of the chunks before it (small sub-batches leave
    // SMs idle in their late layers).  A slot's input is refilled only after
    // its previous graph and result copy ran.
    Plan* slots[kPipeSlots] = {};
    for (int k = 0; k < kPipeSlots; ++k)
      if ((st = plan_for(c, kPipeChunk, H, W, max_det, &slots[k], 1 + k)) != SUCCESS) return st;
    const size_t in_elems = static_cast<size_t>(kPipeChunk) * 3 * H * W;
    const size_t det_elems = static_cast<size_t>(kPipeChunk) * max_det * 6;
    const int n = B / kPipeChunk;
    auto prefetch = [&](int j) {
      const int k = j % kPipeSlots;
      cudaError_t r = j >= kPipeSlots ? cudaStreamWaitEvent(c->copy_stream, c->slot_free[k], 0) : cudaSuccess;
      if (r == cudaSuccess)
        r = cudaMemcpyAsync(slots[k]->d_in, in_nchw + j * in_elems, in_elems * 4, cudaMemcpyHostToDevice,
                            c->copy_stream);
      if (r == cudaSuccess) r = cudaEventRecord(c->in_ready[k], c->copy_stream);
      return r;
    };
    cudaError_t e = cudaSuccess;
    for (int j = 0; j < n && j < kPipeSlots && e == cudaSuccess; ++j) e = prefetch(j);
    for (int i = 0; i < n && e == cudaSuccess; ++i) {
      const int k = i % kPipeSlots;
      cudaStream_t ss = c->slot_stream[k];
      Plan* q = slots[k];
      e = cudaStreamWaitEvent(ss, c->in_ready[k], 0);
      if (e == cudaSuccess) e = c->eng->run(q, ss, nullptr);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(out_dets + i * det_elems, q->d_out, det_elems * 4, cudaMemcpyDeviceToHost, ss);
      if (e == cudaSuccess) e = cudaEventRecord(c->slot_free[k], ss);
      if (e == cudaSuccess && i + kPipeSlots < n) e = prefetch(i + kPipeSlots);
    }
    // Head tensors of a pipelined forward are spread over both slots and
    // partly overwritten; yb_cuda_get_head reports that none are kept.
    c->last = nullptr;
    for (int k = 0; k < kPipeSlots; ++k) {
      const cudaError_t e2 = cudaStreamSynchronize(c->slot_stream[k]);
      if (e == cudaSuccess) e = e2;
    }
    const cudaError_t e2 = cudaStreamSynchronize(c->copy_stream);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) return cuda_status(e, "pipelined forward");
    return check_kernel_flag(c);
  }
  if ((st = plan_for(c, B, H, W, max_det, &p)) != SUCCESS) return st;
  cudaError_t e = cudaMemcpyAsync(p->d_in, in_nchw, static_cast<size_t>(B) * 3 * H * W * 4, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return cuda_status(e, "input copy");
  if (step_ms) {
    for (int i = 0; i < 2 * MODEL_FORWARD_PROFILE_STEPS; ++i) cudaEventRecord(c->ev[i], s);
  }
  e = c->eng->run(p, s, step_ms ? c->ev : nullptr);
  if (e != cudaSuccess) return cuda_status(e, "forward launch");
  if (step_ms) cudaEventRecord(c->ev[2 * 24], s);
  e = cudaMemcpyAsync(out_dets, p->d_out, static_cast<size_t>(B) * max_det * 6 * 4, cudaMemcpyDeviceToHost, s);
  if (step_ms) cudaEventRecord(c->ev[2 * 24 + 1], s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e, "forward");
  if ((st = check_kernel_flag(c)) != SUCCESS) return st;
  c->last = p;
  if (step_ms) {
    bool has[MODEL_FORWARD_PROFILE_STEPS] = {};
    for (const Op& op : p->ops) has[op.step] = true;
    has[24] = true;
    for (int i = 0; i < MODEL_FORWARD_PROFILE_STEPS; ++i) {
      float ms = 0.f;
      if (has[i]) cudaEventElapsedTime(&ms, c->ev[2 * i], c->ev[2 * i + 1]);
      step_ms[i] = ms;
    }
  }
  if (dump) return p->int8 ? dump_stages_i8(c, p, in_nchw, dump, user) : dump_stages(c, p, in_nchw, dump, user);
  return SUCCESS;
}

extern "C" status_t yb_cuda_forward_rgb8(void* ctx, const unsigned char* rgb_hwc, int B, int src_h, int src_w,
                                         int resize, int H, int W, float* out_dets, int max_det) {
  Ctx* c = as_ctx(ctx);
  if (!c || !rgb_hwc || !out_dets) return ERROR_NULL_POINTER;
  if (B < 1 || src_h < 1 || src_w < 1 || (resize != YB_RESIZE_ALIGN_CORNERS && resize != YB_RESIZE_HALF_PIXEL))
    return ERROR_INVALID_DIMS;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  Plan* p = nullptr;
  if ((st = plan_for(c, B, H, W, max_det, &p)) != SUCCESS) return st;
  const size_t bytes = static_cast<size_t>(B) * src_h * src_w * 3;
  if (bytes > c->d_rgb_bytes) {
    if (c->d_rgb) cudaFree(c->d_rgb);
    c->d_rgb = nullptr;
    c->d_rgb_bytes = 0;
    cudaError_t e = cudaMalloc(&c->d_rgb, bytes);
    if (e != cudaSuccess) return cuda_status(e, "rgb staging");
    c->d_rgb_bytes = bytes;
  }
  cudaStream_t s = c->eng->stream();
  cudaError_t e = cudaMemcpyAsync(c->d_rgb, rgb_hwc, bytes, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = launch_preprocess(c->d_rgb, B, src_h, src_w, resize, p->d_in, H, W, s);
  if (e == cudaSuccess) e = c->eng->run(p, s, nullptr);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(out_dets, p->d_out, static_cast<size_t>(B) * max_det * 6 * 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e, "forward_rgb8");
  if ((st = check_kernel_flag(c)) != SUCCESS) return st;
  c->last = p;
  return SUCCESS;
}

extern "C" status_t yb_cuda_get_detections(void* ctx, float threshold, int capacity, detection_t* out, int* counts) {
  Ctx* c = as_ctx(ctx);
  if (!c || !out || !counts) return ERROR_NULL_POINTER;
  if (capacity < 0) return ERROR_INVALID_DIMS;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  Plan* p = c->last;
  if (!p) {
    set_error("no detections kept: no forward has run on this context, or the last one was pipelined");
    return ERROR_INVALID_DIMS;
  }
  cudaStream_t s = c->eng->stream();
  const size_t n_out = static_cast<size_t>(p->B) * capacity;
  DevMem d_out, d_cnt;
  cudaError_t e = d_out.alloc(n_out * sizeof(detection_t) + 16);
  if (e == cudaSuccess) e = d_cnt.alloc(static_cast<size_t>(p->B) * sizeof(int));
  if (e == cudaSuccess)
    e = launch_detections(p->d_out, p->B, p->max_det, threshold, capacity, static_cast<detection_t*>(d_out.p),
                          static_cast<int*>(d_cnt.p), s);
  if (e == cudaSuccess && n_out)
    e = cudaMemcpyAsync(out, d_out.p, n_out * sizeof(detection_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(counts, d_cnt.p, static_cast<size_t>(p->B) * sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return cuda_status(e, "get_detections");
}

extern "C" status_t yb_cuda_detections(const float* d_dets, int B, int rows, float threshold, int capacity,
                                       detection_t* d_out, int* d_counts, void* stream) {
  if (!d_dets || !d_out || !d_counts) return ERROR_NULL_POINTER;
  if (B < 0 || rows < 0 || capacity < 0) return ERROR_INVALID_DIMS;
  return cuda_status(launch_detections(d_dets, B, rows, threshold, capacity, d_out, d_counts,
                                       static_cast<cudaStream_t>(stream)),
                     "detections");
}

namespace {

// Queues one batch on the next streaming slot: input copy on the copy stream
// (back to back with other copies), then on the slot's stream the optional
// preprocess, the plan's graph and the detections' copy to the host.
status_t stream_submit(Ctx* c, const void* src, size_t src_bytes, bool rgb8, int B, int src_h, int src_w, int resize,
                       int H, int W, float* out_dets, int max_det, long long* ticket) {
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  const int k = c->sslot_next;
  Ctx::StreamSlot& S = c->sslot[k];
  // The slot's previous batch must be done before its input is overwritten.
  if ((st = finish_stream_slot(c, S)) != SUCCESS) return st;
  Plan* p = nullptr;
  if ((st = plan_for(c, B, H, W, max_det, &p, kStreamTag + k)) != SUCCESS) return st;
  cudaError_t e = cudaSuccess;
  void* dst = p->d_in;
  if (rgb8) {
    if (src_bytes > S.d_rgb_bytes) {
      if (S.d_rgb) cudaFree(S.d_rgb);
      S.d_rgb = nullptr;
      S.d_rgb_bytes = 0;
      if ((e = cudaMalloc(&S.d_rgb, src_bytes)) != cudaSuccess) return cuda_status(e, "rgb staging");
      S.d_rgb_bytes = src_bytes;
    }
    dst = S.d_rgb;
  }
  e = cudaMemcpyAsync(dst, src, src_bytes, cudaMemcpyHostToDevice, c->copy_stream);
  if (e == cudaSuccess) e = cudaEventRecord(S.h2d, c->copy_stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(S.st, S.h2d, 0);
  // The other slot's batch computes first: the forwards run back to back on
  // the GPU (two at once only compete for the SMs), while this batch's input
  // copy overlaps the other's compute.
  Ctx::StreamSlot& O = c->sslot[k ^ 1];
  if (e == cudaSuccess && O.ticket) e = cudaStreamWaitEvent(S.st, O.done, 0);
  if (e == cudaSuccess && rgb8) e = launch_preprocess(S.d_rgb, B, src_h, src_w, resize, p->d_in, H, W, S.st);
  if (e == cudaSuccess) e = c->eng->run(p, S.st, nullptr);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(out_dets, p->d_out, static_cast<size_t>(B) * max_det * 6 * 4, cudaMemcpyDeviceToHost, S.st);
  if (e == cudaSuccess) e = cudaEventRecord(S.done, S.st);
  if (e != cudaSuccess) return cuda_status(e, "streaming forward");
  S.plan = p;
  S.ticket = c->next_ticket++;
  c->sslot_next = k ^ 1;
  *ticket = S.ticket;
  return SUCCESS;
}

}  // namespace

extern "C" status_t yb_cuda_forward_submit(void* ctx, const float* in_nchw, int B, int H, int W, float* out_dets,
                                           int max_det, long long* ticket) {
  Ctx* c = as_ctx(ctx);
  if (!c || !in_nchw || !out_dets || !ticket) return ERROR_NULL_POINTER;
  if (B < 1) return ERROR_INVALID_DIMS;
  return stream_submit(c, in_nchw, static_cast<size_t>(B) * 3 * H * W * 4, false, B, 0, 0, 0, H, W, out_dets, max_det,
                       ticket);
}

extern "C" status_t yb_cuda_forward_rgb8_submit(void* ctx, const unsigned char* rgb_hwc, int B, int src_h, int src_w,
                                                int resize, int H, int W, float* out_dets, int max_det,
                                                long long* ticket) {
  Ctx* c = as_ctx(ctx);
  if (!c || !rgb_hwc || !out_dets || !ticket) return ERROR_NULL_POINTER;
  if (B < 1 || src_h < 1 || src_w < 1 || (resize != YB_RESIZE_ALIGN_CORNERS && resize != YB_RESIZE_HALF_PIXEL))
    return ERROR_INVALID_DIMS;
  return stream_submit(c, rgb_hwc, static_cast<size_t>(B) * src_h * src_w * 3, true, B, src_h, src_w, resize, H, W,
                       out_dets, max_det, ticket);
}

extern "C" status_t yb_cuda_forward_wait(void* ctx, long long ticket) {
  Ctx* c = as_ctx(ctx);
  if (!c) return ERROR_NULL_POINTER;
  cudaError_t e = cudaSetDevice(c->eng->device());
  if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  for (auto& S : c->sslot)
    if (S.ticket == ticket && ticket != 0) return finish_stream_slot(c, S);
  if (ticket > 0 && ticket < c->next_ticket) return SUCCESS;  // already finished
  set_error("unknown streaming ticket");
  return ERROR_INVALID_DIMS;
}

extern "C" status_t yb_cuda_preprocess_rgb8(const unsigned char* d_rgb, int B, int src_h, int src_w, int resize,
                                            float* d_nchw, int H, int W, void* stream) {
  if (!d_rgb || !d_nchw) return ERROR_NULL_POINTER;
  if (B < 0 || src_h < 1 || src_w < 1 || H < 1 || W < 1 ||
      (resize != YB_RESIZE_ALIGN_CORNERS && resize != YB_RESIZE_HALF_PIXEL))
    return ERROR_INVALID_DIMS;
  const cudaError_t e = launch_preprocess(d_rgb, B, src_h, src_w, resize, d_nchw, H, W, static_cast<cudaStream_t>(stream));
  return cuda_status(e, "preprocess_rgb8");
}

extern "C" status_t yb_cuda_plan_io(void* ctx, int B, int H, int W, int max_det, float** d_in, float** d_out) {
  Ctx* c = as_ctx(ctx);
  if (!c || !d_in || !d_out) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  Plan* p = nullptr;
  if ((st = plan_for(c, B, H, W, max_det, &p)) != SUCCESS) return st;
  *d_in = p->d_in;
  *d_out = p->d_out;
  return SUCCESS;
}

extern "C" status_t yb_cuda_forward_device(void* ctx, const float* d_in, int B, int H, int W, float* d_out,
                                           int max_det, void* stream) {
  Ctx* c = as_ctx(ctx);
  if (!c || !d_in || !d_out) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  Plan* p = nullptr;
  if ((st = plan_for(c, B, H, W, max_det, &p)) != SUCCESS) return st;
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->eng->stream();
  cudaError_t e = cudaSuccess;
  if (d_in != p->d_in)
    e = cudaMemcpyAsync(p->d_in, d_in, static_cast<size_t>(B) * 3 * H * W * 4, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess) e = c->eng->run(p, s, nullptr);
  if (e == cudaSuccess && d_out != p->d_out)
    e = cudaMemcpyAsync(d_out, p->d_out, static_cast<size_t>(B) * max_det * 6 * 4, cudaMemcpyDeviceToDevice, s);
  c->last = p;
  return cuda_status(e, "forward_device");
}

extern "C" status_t yb_cuda_get_head(void* ctx, float* logits, float* boxes, int* n_anchors, int* nc) {
  Ctx* c = as_ctx(ctx);
  if (!c) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  Plan* p = c->last;
  if (!p) {
    set_error("no head tensors kept: no forward has run on this context, or the last one was pipelined");
    return ERROR_INVALID_DIMS;
  }
  cudaError_t e = cudaStreamSynchronize(c->eng->stream());
  const size_t n = static_cast<size_t>(p->B) * p->n_anchors;
  if (e == cudaSuccess && logits)
    e = cudaMemcpy(logits, p->d_logits, n * c->eng->num_classes() * 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && boxes) e = cudaMemcpy(boxes, p->d_boxes, n * 4 * 4, cudaMemcpyDeviceToHost);
  if (n_anchors) *n_anchors = p->n_anchors;
  if (nc) *nc = c->eng->num_classes();
  return cuda_status(e, "get_head");
}

extern "C" status_t yb_cuda_profile_ops(void* ctx, int B, int H, int W, int max_det, int reps, yb_op_stat* stats,
                                        int cap, int* n_ops) {
  Ctx* c = as_ctx(ctx);
  if (!c || !n_ops) return ERROR_NULL_POINTER;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  Plan* p = nullptr;
  if ((st = plan_for(c, B, H, W, max_det, &p)) != SUCCESS) return st;
  *n_ops = static_cast<int>(p->ops.size());
  if (!stats) return SUCCESS;
  std::vector<double> ms;
  cudaError_t e = c->eng->profile_ops(p, reps < 1 ? 1 : reps, &ms);
  if (e != cudaSuccess) return cuda_status(e, "profile_ops");
  if ((st = check_kernel_flag(c)) != SUCCESS) return st;
  for (int i = 0; i < *n_ops && i < cap; ++i) {
    stats[i].kind = p->ops[i].kind;
    stats[i].step = p->ops[i].step;
    stats[i].ms = ms[i];
    stats[i].flops = p->ops[i].flops;
    stats[i].bytes = p->ops[i].bytes;
  }
  return SUCCESS;
}

extern "C" status_t yb_cuda_debug_inject_stall(void* ctx, int ms) {
  Ctx* c = as_ctx(ctx);
  if (!c) return ERROR_NULL_POINTER;
  c->stall_ms = ms;
  return SUCCESS;
}

namespace {

// One shard of yb_cuda_forward_sharded, run on its own host thread.
status_t run_shard(Ctx* c, const float* in, int B, int H, int W, float* out, int max_det,
                   std::chrono::steady_clock::time_point deadline, bool has_deadline, std::string* msg) {
  using clock = std::chrono::steady_clock;
  auto expired = [&] { return has_deadline && clock::now() >= deadline; };
  cudaError_t e = cudaSetDevice(c->eng->device());
  if (e != cudaSuccess) {
    *msg = cudaGetErrorString(e);
    return ERROR_DEVICE;
  }
  if (c->inflight) {
    while (cudaEventQuery(c->done) == cudaErrorNotReady) {
      if (expired()) {
        *msg = "previous call still running at the deadline";
        return ERROR_TIMEOUT;
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    c->inflight = false;
  }
  if (c->stall_ms > 0) std::this_thread::sleep_for(std::chrono::milliseconds(c->stall_ms));
  if (expired()) {
    *msg = "shard did not start before the deadline";
    return ERROR_TIMEOUT;
  }
  Plan* p = nullptr;
  status_t st = plan_for(c, B, H, W, max_det, &p);
  if (st != SUCCESS) {
    *msg = last_error();
    return st;
  }
  const size_t det_bytes = static_cast<size_t>(B) * max_det * 6 * 4;
  if (c->h_stage_bytes < det_bytes) {
    if (c->h_stage) cudaFreeHost(c->h_stage);
    c->h_stage = nullptr;
    c->h_stage_bytes = 0;
    if ((e = cudaMallocHost(&c->h_stage, det_bytes)) != cudaSuccess) {
      *msg = cudaGetErrorString(e);
      return ERROR_OUT_OF_MEMORY;
    }
    c->h_stage_bytes = det_bytes;
  }
  cudaStream_t s = c->eng->stream();
  e = cudaMemcpyAsync(p->d_in, in, static_cast<size_t>(B) * 3 * H * W * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaEventRecord(c->h2d_done, s);
  if (e == cudaSuccess) e = c->eng->run(p, s, nullptr);
  if (e == cudaSuccess) e = cudaMemcpyAsync(c->h_stage, p->d_out, det_bytes, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaEventRecord(c->done, s);
  if (e != cudaSuccess) {
    *msg = cudaGetErrorString(e);
    return ERROR_DEVICE;
  }
  c->inflight = true;
  c->last = p;
  while (true) {
    e = cudaEventQuery(c->done);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) {
      *msg = cudaGetErrorString(e);
      return ERROR_DEVICE;
    }
    if (expired()) {
      // The input may still be read by the copy engine: give that copy up to
      // a second to finish.  The copy is queued behind earlier work on this
      // context's stream, so it can outlast the wait; the caller must keep
      // the input valid until the next call on this context returns (the
      // header states this).
      const auto t0 = clock::now();
      while (cudaEventQuery(c->h2d_done) == cudaErrorNotReady && clock::now() - t0 < std::chrono::seconds(1))
        std::this_thread::sleep_for(std::chrono::microseconds(50));
      *msg = "shard on device " + std::to_string(c->eng->device()) + " missed the deadline";
      return ERROR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  c->inflight = false;
  const int k = c->eng->take_kernel_error();
  if (k) {
    *msg = "device kernel reported error code " + std::to_string(k);
    return ERROR_DEVICE;
  }
  std::memcpy(out, c->h_stage, det_bytes);
  return SUCCESS;
}

}  // namespace

extern "C" status_t yb_cuda_forward_sharded(void* const* ctxs, int G, const float* in_nchw, int B, int H, int W,
                                            float* out_dets, int max_det, int timeout_ms) {
  if (!ctxs || !in_nchw || !out_dets) return ERROR_NULL_POINTER;
  if (G < 1 || B < 1) return ERROR_INVALID_DIMS;
  for (int g = 0; g < G; ++g)
    if (!ctxs[g]) return ERROR_NULL_POINTER;
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : 0);
  std::vector<status_t> st(G, SUCCESS);
  std::vector<std::string> msg(G);
  std::vector<std::thread> th;
  const size_t img = static_cast<size_t>(3) * H * W;
  const size_t det = static_cast<size_t>(max_det) * 6;
  for (int g = 0; g < G; ++g) {
    const int b0 = static_cast<int>(static_cast<long long>(g) * B / G);
    const int b1 = static_cast<int>(static_cast<long long>(g + 1) * B / G);
    if (b1 == b0) continue;
    th.emplace_back([&, g, b0, b1] {
      st[g] = run_shard(as_ctx(ctxs[g]), in_nchw + b0 * img, b1 - b0, H, W, out_dets + b0 * det, max_det, deadline,
                        timeout_ms > 0, &msg[g]);
    });
  }
  for (auto& t : th) t.join();
  status_t result = SUCCESS;
  for (int g = 0; g < G; ++g) {
    if (st[g] != SUCCESS && (result == SUCCESS || st[g] == ERROR_TIMEOUT)) {
      result = st[g];
      set_error("shard " + std::to_string(g) + ": " + msg[g]);
    }
  }
  return result;
}

// ================================================================ tensor.h
extern "C" void* malloc_aligned(size_t size, size_t alignment) {
  void* p = nullptr;
  if (posix_memalign(&p, alignment, size ? size : alignment) != 0) return nullptr;
  return p;
}
extern "C" void free_aligned(void* ptr) { free(ptr); }

extern "C" status_t tensor_allocate(tensor_t* t, int n, int c, int h, int w) {
  if (!t) return ERROR_NULL_POINTER;
  t->dims[0] = n;
  t->dims[1] = c;
  t->dims[2] = h;
  t->dims[3] = w;
  t->stride[3] = 1;
  t->stride[2] = w;
  t->stride[1] = h * w;
  t->stride[0] = c * h * w;
  const size_t bytes = static_cast<size_t>(n) * c * h * w * sizeof(float);
  t->data = static_cast<float*>(malloc_aligned(bytes, 64));
  t->is_owner = t->data != nullptr;
  return t->data ? SUCCESS : ERROR_OUT_OF_MEMORY;
}

extern "C" status_t tensor_free(tensor_t* t) {
  if (!t) return ERROR_NULL_POINTER;
  if (t->is_owner && t->data) {
    free_aligned(t->data);
    t->data = nullptr;
  }
  return SUCCESS;
}

extern "C" status_t tensor_fill(tensor_t* t, float v) {
  if (!t || !t->data) return ERROR_NULL_POINTER;
  const size_t n = static_cast<size_t>(t->dims[0]) * t->dims[1] * t->dims[2] * t->dims[3];
  std::fill(t->data, t->data + n, v);
  return SUCCESS;
}

extern "C" status_t tensor_copy(tensor_t* dst, const tensor_t* src) {
  if (!dst || !src || !dst->data || !src->data) return ERROR_NULL_POINTER;
  for (int i = 0; i < 4; ++i)
    if (dst->dims[i] != src->dims[i]) return ERROR_INVALID_DIMS;
  const size_t n = static_cast<size_t>(src->dims[0]) * src->dims[1] * src->dims[2] * src->dims[3];
  std::memcpy(dst->data, src->data, n * sizeof(float));
  return SUCCESS;
}

// ================================================================= utils.h
extern "C" void timer_start(yb_timer_t* t) {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  t->start = static_cast<uint64_t>(ts.tv_sec) * 1000000000ull + static_cast<uint64_t>(ts.tv_nsec);
}
extern "C" void timer_stop(yb_timer_t* t) {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  t->end = static_cast<uint64_t>(ts.tv_sec) * 1000000000ull + static_cast<uint64_t>(ts.tv_nsec);
}
extern "C" double timer_elapsed_ms(const yb_timer_t* t) { return static_cast<double>(t->end - t->start) / 1e6; }

extern "C" status_t load_named_tensor(FILE* f, char* name, tensor_t* tensor) {
  if (!f || !name || !tensor) return ERROR_NULL_POINTER;
  int32_t nl = 0;
  if (std::fread(&nl, 4, 1, f) != 1) return ERROR_FILE_NOT_FOUND;
  if (nl < 0 || nl >= 128 || std::fread(name, 1, static_cast<size_t>(nl), f) != static_cast<size_t>(nl))
    return ERROR_INVALID_FORMAT;
  name[nl] = '\0';
  int32_t nd = 0;
  if (std::fread(&nd, 4, 1, f) != 1 || nd < 0 || nd > 4) return ERROR_INVALID_FORMAT;
  int dims[4] = {1, 1, 1, 1};
  for (int d = 0; d < nd; ++d)
    if (std::fread(&dims[d], 4, 1, f) != 1 || dims[d] < 0) return ERROR_INVALID_FORMAT;
  status_t st = tensor_allocate(tensor, dims[0], dims[1], dims[2], dims[3]);
  if (st != SUCCESS) return st;
  const size_t n = static_cast<size_t>(dims[0]) * dims[1] * dims[2] * dims[3];
  if (std::fread(tensor->data, sizeof(float), n, f) != n) {
    tensor_free(tensor);
    return ERROR_INVALID_FORMAT;
  }
  return SUCCESS;
}

extern "C" status_t save_named_tensor(FILE* f, const char* name, const tensor_t* t) {
  if (!f || !name || !t || !t->data) return ERROR_NULL_POINTER;
  const int32_t nl = static_cast<int32_t>(std::strlen(name));
  const int32_t nd = 4;
  if (std::fwrite(&nl, 4, 1, f) != 1 || std::fwrite(name, 1, static_cast<size_t>(nl), f) != static_cast<size_t>(nl) ||
      std::fwrite(&nd, 4, 1, f) != 1 || std::fwrite(t->dims, 4, 4, f) != 4)
    return ERROR_FILE_NOT_FOUND;
  const size_t n = static_cast<size_t>(t->dims[0]) * t->dims[1] * t->dims[2] * t->dims[3];
  if (std::fwrite(t->data, sizeof(float), n, f) != n) return ERROR_FILE_NOT_FOUND;
  return SUCCESS;
}

extern "C" void fold_bn(tensor_t* conv_w, tensor_t* conv_b, const tensor_t* bn_w, const tensor_t* bn_b,
                        const tensor_t* bn_rm, const tensor_t* bn_rv) {
  const int out_c = conv_w->dims[0];
  const size_t per = static_cast<size_t>(conv_w->dims[1]) * conv_w->dims[2] * conv_w->dims[3];
  const float eps = 1e-5f;
  for (int i = 0; i < out_c; ++i) {
    const float scale = bn_w->data[i] / std::sqrt(bn_rv->data[i] + eps);
    for (size_t j = 0; j < per; ++j) conv_w->data[i * per + j] *= scale;
    if (conv_b) {
      const float t = conv_b->data[i] - bn_rm->data[i];
      const float t2 = t * scale;
      conv_b->data[i] = t2 + bn_b->data[i];
    }
  }
}

// ============================================================= detection.h
extern "C" status_t decode_detections(detection_results_t* results, const tensor_t* head, float threshold) {
  if (!results || !head) return ERROR_NULL_POINTER;
  if (head->dims[0] < 1) return ERROR_INVALID_DIMS;
  const int rows = head->dims[1];
  const int feat = head->dims[2];
  const int w = head->dims[3];
  if (feat < 6 || w < 1) return ERROR_INVALID_DIMS;
  const int rs = feat * w;
  results->count = 0;
  for (int i = 0; i < rows; ++i) {
    const float* r = head->data + static_cast<size_t>(i) * rs;
    if (r[4] <= threshold) continue;
    if (results->count >= results->capacity) break;
    detection_t* d = &results->detections[results->count++];
    d->x1 = r[0];
    d->y1 = r[1];
    d->x2 = r[2];
    d->y2 = r[3];
    d->score = r[4];
    d->class_id = static_cast<int>(r[5]);
  }
  return SUCCESS;
}

// ================================================================ detect.h
extern "C" status_t detect_postprocess_from_pred(const float* pred, int N, int nc, int max_det, tensor_t* out) {
  if (!pred || !out || !out->data) return ERROR_NULL_POINTER;
  if (out->dims[0] != 1 || out->dims[2] < 6 || out->dims[3] < 1) return ERROR_INVALID_DIMS;
  if (N < 0 || nc < 1) return ERROR_INVALID_DIMS;
  const int cap = out->dims[1];
  int k = std::min(max_det, N);
  k = std::min(k, cap);
  const int rs = out->dims[2] * out->dims[3];
  std::vector<float> rows(static_cast<size_t>(cap) * 6, 0.f);
  if (k > 0) {
    if (k > kTopkMax) {
      set_error("min(max_det, N, output rows) = " + std::to_string(k) + " exceeds the device top-k limit of " +
                std::to_string(kTopkMax) + " (the reference has no limit)");
      return ERROR_INVALID_DIMS;
    }
    DevScope* sc = current_scope();
    if (!sc) return ERROR_DEVICE;
    DevMem dp, dd;
    cudaError_t e = dp.alloc(static_cast<size_t>(N) * (4 + nc) * 4);
    if (e == cudaSuccess) e = dd.alloc(static_cast<size_t>(k) * 6 * 4);
    if (e != cudaSuccess) return cuda_status(e, "postprocess buffers");
    e = cudaMemcpyAsync(dp.p, pred, static_cast<size_t>(N) * (4 + nc) * 4, cudaMemcpyHostToDevice, sc->stream);
    TopkArgs ta;
    ta.scores = dp.f() + 4;
    ta.s_bstride = 0;
    ta.s_rstride = 4 + nc;
    ta.apply_sigmoid = 0;
    ta.boxes = dp.f();
    ta.b_rstride = 4 + nc;
    ta.dets = dd.f();
    ta.B = 1;
    ta.N = N;
    ta.nc = nc;
    ta.max_det = k;
    ta.cap = k;
    if (e == cudaSuccess) e = launch_topk(ta, sc->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(rows.data(), dd.p, static_cast<size_t>(k) * 6 * 4, cudaMemcpyDeviceToHost, sc->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(sc->stream);
    if (e != cudaSuccess) return cuda_status(e, "postprocess");
  }
  for (int t = 0; t < cap; ++t) {
    float* r = out->data + static_cast<size_t>(t) * rs;
    for (int u = 0; u < 6; ++u) r[u] = rows[static_cast<size_t>(t) * 6 + u];
  }
  return SUCCESS;
}

// ================================================================= model.h
static const char* const k_step_names[MODEL_FORWARD_PROFILE_STEPS] = {
    "conv model.0 /2 + SiLU",
    "conv model.1 /2 + SiLU",
    "C3k2 model.2 (n=1)",
    "conv model.3 /2 + SiLU",
    "C3k2 model.4 (n=1)",
    "conv model.5 /2 + SiLU",
    "C3k2 inner model.6",
    "conv model.7 /2 + SiLU",
    "C3k2 inner model.8",
    "SPPF model.9",
    "C2PSA model.10",
    "upsample 2x \xe2\x86\x92 buf11",
    "concat(buf11, buf6) \xe2\x86\x92 buf12",
    "C3k2 inner model.13",
    "upsample 2x \xe2\x86\x92 buf14",
    "concat(buf14, buf4) \xe2\x86\x92 buf15",
    "C3k2 inner model.16 (P3)",
    "conv model.17 /2 + SiLU",
    "concat(buf17, buf13) \xe2\x86\x92 buf18",
    "C3k2 inner model.19 (P4)",
    "conv model.20 /2 + SiLU",
    "concat(buf20, buf10) \xe2\x86\x92 buf21",
    "C3k2 attn head model.22 (P5)",
    "Detect one2one \xe2\x86\x92 buf23",
    "tensor_copy buf23 \xe2\x86\x92 output",
};

extern "C" void model_forward_profile_reset(model_forward_profile_t* p) {
  if (!p) return;
  std::memset(p, 0, sizeof(*p));
}

extern "C" const char* model_forward_profile_step_name(int i) {
  if (i < 0 || i >= MODEL_FORWARD_PROFILE_STEPS) return "?";
  return k_step_names[i];
}

extern "C" void model_forward_profile_print_last(const model_forward_profile_t* p, FILE* fp, const char* title) {
  if (!p || !fp || p->runs == 0) return;
  std::fprintf(fp, "%s\n", title);
  std::fprintf(fp, "%-4s %-44s %12s %8s\n", "#", "step", "ms", "% fwd");
  double tot = 0;
  for (int i = 0; i < MODEL_FORWARD_PROFILE_STEPS; ++i) tot += p->ms_last[i];
  for (int i = 0; i < MODEL_FORWARD_PROFILE_STEPS; ++i)
    std::fprintf(fp, "%2d   %-44s %12.4f %7.2f%%\n", i + 1, k_step_names[i], p->ms_last[i],
                 tot > 0 ? 100.0 * p->ms_last[i] / tot : 0.0);
  std::fprintf(fp, "%-4s %-44s %12.4f\n", "", "total (timed steps)", tot);
}

extern "C" void model_forward_profile_print_aggregate(const model_forward_profile_t* p, FILE* fp) {
  if (!fp) return;
  if (!p || p->runs == 0) {
    std::fprintf(fp, "No model_forward profile (no successful runs).\n");
    return;
  }
  std::fprintf(fp, "\n=== model_forward per-step (avg over %u run(s)) ===\n", p->runs);
  std::fprintf(fp, "%-4s %-44s %12s %8s\n", "#", "step", "avg ms", "% fwd");
  double avg[MODEL_FORWARD_PROFILE_STEPS], tot = 0;
  int hot = 0;
  for (int i = 0; i < MODEL_FORWARD_PROFILE_STEPS; ++i) {
    avg[i] = p->ms_sum[i] / p->runs;
    tot += avg[i];
    if (avg[i] > avg[hot]) hot = i;
  }
  for (int i = 0; i < MODEL_FORWARD_PROFILE_STEPS; ++i)
    std::fprintf(fp, "%2d   %-44s %12.4f %7.2f%%\n", i + 1, k_step_names[i], avg[i], tot > 0 ? 100.0 * avg[i] / tot : 0.0);
  std::fprintf(fp, "%-4s %-44s %12.4f\n", "", "total (sum of steps)", tot);
  std::fprintf(fp, "\nHot step inside model_forward: #%d %s (~%.1f%% of forward).\n", hot + 1, k_step_names[hot],
               tot > 0 ? 100.0 * avg[hot] / tot : 0.0);
}

extern "C" status_t model_create(model_t* m, int input_w, int input_h) {
  if (!m) return ERROR_NULL_POINTER;
  m->input_w = input_w;
  m->input_h = input_h;
  m->weights = nullptr;
  m->num_weights = 0;
  m->num_classes = 80;
  m->num_buffers = 24;
  m->buffers = static_cast<tensor_t*>(std::calloc(24, sizeof(tensor_t)));
  if (!m->buffers) return ERROR_OUT_OF_MEMORY;
  return tensor_allocate(&m->buffers[23], 1, 300, 6, 1);
}

extern "C" status_t model_destroy(model_t* m) {
  if (!m) return ERROR_NULL_POINTER;
  Ctx* c = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_models_mu);
    auto it = g_models.find(m);
    if (it != g_models.end()) {
      c = it->second;
      g_models.erase(it);
    }
  }
  if (c) yb_cuda_destroy(c);
  for (int i = 0; i < m->num_weights; ++i) tensor_free(&m->weights[i].tensor);
  std::free(m->weights);
  m->weights = nullptr;
  m->num_weights = 0;
  if (m->buffers) {
    for (int i = 0; i < m->num_buffers; ++i) tensor_free(&m->buffers[i]);
    std::free(m->buffers);
    m->buffers = nullptr;
  }
  return SUCCESS;
}

extern "C" tensor_t* model_get_weight(model_t* m, const char* name) {
  if (!m || !name) return nullptr;
  for (int i = 0; i < m->num_weights; ++i)
    if (std::strcmp(m->weights[i].name, name) == 0) return &m->weights[i].tensor;
  return nullptr;
}

extern "C" status_t model_load_weights(model_t* m, const char* path) {
  if (!m || !path) return ERROR_NULL_POINTER;
  WeightMap w;
  int nc = 0;
  std::string why;
  int raw_count = 0;
  {
    FILE* f = std::fopen(path, "rb");
    if (!f) return ERROR_FILE_NOT_FOUND;
    int32_t hdr[2] = {0, 0};
    if (std::fread(hdr, 4, 2, f) == 2) raw_count = hdr[1];
    std::fclose(f);
  }
  if (!read_weight_bin(path, &w, &nc, &why)) {
    set_error(why);
    return ERROR_INVALID_FORMAT;
  }
  fold_all_bn_map(&w);
  for (int i = 0; i < m->num_weights; ++i) tensor_free(&m->weights[i].tensor);
  std::free(m->weights);
  m->weights = static_cast<named_tensor_t*>(std::calloc(w.size() ? w.size() : 1, sizeof(named_tensor_t)));
  if (!m->weights) return ERROR_OUT_OF_MEMORY;
  m->num_weights = 0;
  for (const auto& kv : w) {
    named_tensor_t& nt = m->weights[m->num_weights];
    std::strncpy(nt.name, kv.first.c_str(), sizeof(nt.name) - 1);
    const HostTensor& h = kv.second;
    status_t st = tensor_allocate(&nt.tensor, h.dims[0], h.dims[1], h.dims[2], h.dims[3]);
    if (st != SUCCESS) return st;
    std::memcpy(nt.tensor.data, h.data.data(), h.data.size() * 4);
    ++m->num_weights;
  }
  m->num_classes = nc;
  std::printf("Successfully loaded %d tensors (after BN fold, %d tensors in memory)\n", raw_count, m->num_weights);

  Ctx* c = model_ctx(m);
  if (!c) {
    int dev = 0;
    const char* env = std::getenv("YB_DEVICE");
    if (env && *env) dev = std::atoi(env);
    else if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    void* vc = nullptr;
    status_t st = yb_cuda_init(dev, &vc);
    if (st != SUCCESS) return st;
    c = as_ctx(vc);
    std::lock_guard<std::mutex> lk(g_models_mu);
    g_models[m] = c;
  }
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  cudaError_t e = c->eng->set_weights(std::move(w), nc, &why);
  if (e == cudaErrorInvalidValue) {
    set_error(why);
    return ERROR_FILE_NOT_FOUND;
  }
  return cuda_status(e, "upload weights");
}

namespace {
void stage_to_file(void* user, const char* name, const float* data, int n, int c, int h, int w) {
  FILE* f = static_cast<FILE*>(user);
  tensor_t t;
  t.data = const_cast<float*>(data);
  t.dims[0] = n;
  t.dims[1] = c;
  t.dims[2] = h;
  t.dims[3] = w;
  t.is_owner = false;
  save_named_tensor(f, name, &t);
}
}  // namespace

extern "C" status_t model_forward_ex(model_t* m, const tensor_t* input, tensor_t* output, FILE* stage_dump,
                                     model_forward_profile_t* profile) {
  if (!m || !input || !output || !input->data || !output->data) return ERROR_NULL_POINTER;
  Ctx* c = model_ctx(m);
  if (!c) {
    set_error("model has no weights loaded");
    return ERROR_FILE_NOT_FOUND;
  }
  const int B = input->dims[0], C = input->dims[1], H = input->dims[2], W = input->dims[3];
  if (B < 1 || C != 3 || H % 32 || W % 32 || H < 32 || W < 32) return ERROR_INVALID_DIMS;
  const int max_det = output->dims[1];
  if (output->dims[0] != B || output->dims[2] < 6 || output->dims[3] < 1 || max_det < 1) return ERROR_INVALID_DIMS;
  const int rs = output->dims[2] * output->dims[3];
  std::vector<float> tmp;
  float* dst = output->data;
  if (rs != 6) {
    tmp.resize(static_cast<size_t>(B) * max_det * 6);
    dst = tmp.data();
  }
  double ms[MODEL_FORWARD_PROFILE_STEPS] = {0};
  status_t st = yb_cuda_forward(c, input->data, B, H, W, dst, max_det, stage_dump ? stage_to_file : nullptr,
                                stage_dump, profile ? ms : nullptr);
  if (st != SUCCESS) return st;
  if (rs != 6) {
    for (int b = 0; b < B; ++b)
      for (int t = 0; t < max_det; ++t)
        for (int u = 0; u < 6; ++u)
          output->data[(static_cast<size_t>(b) * max_det + t) * rs + u] = tmp[(static_cast<size_t>(b) * max_det + t) * 6 + u];
  }
  tensor_t* b23 = m->buffers && m->num_buffers > 23 ? &m->buffers[23] : nullptr;
  if (b23 && b23->data && b23->dims[1] == max_det && b23->dims[2] * b23->dims[3] == rs)
    std::memcpy(b23->data, output->data, static_cast<size_t>(max_det) * rs * 4);
  if (profile) {
    for (int i = 0; i < MODEL_FORWARD_PROFILE_STEPS; ++i) {
      profile->ms_sum[i] += ms[i];
      profile->ms_last[i] = ms[i];
    }
    profile->runs++;
  }
  return SUCCESS;
}

extern "C" status_t model_forward(model_t* m, const tensor_t* input, tensor_t* output) {
  return model_forward_ex(m, input, output, nullptr, nullptr);
}

extern "C" status_t model_forward_batch(model_t* m, const tensor_t* input, tensor_t* output) {
  return model_forward_ex(m, input, output, nullptr, nullptr);
}

extern "C" status_t detect_forward_one2one(model_t* m, int detect_module_idx, const tensor_t* p3, const tensor_t* p4,
                                           const tensor_t* p5, tensor_t* out) {
  if (!m || !p3 || !p4 || !p5 || !out || !out->data) return ERROR_NULL_POINTER;
  if (detect_module_idx != YOLO26_DETECT_IDX) {
    set_error("the device graph wires the Detect head at model.23");
    return ERROR_NOT_IMPLEMENTED;
  }
  Ctx* c = model_ctx(m);
  if (!c) return ERROR_FILE_NOT_FOUND;
  status_t st = ctx_ready(c);
  if (st != SUCCESS) return st;
  const int H = p3->dims[2] * 8, W = p3->dims[3] * 8;
  const int max_det = out->dims[1];
  if (out->dims[0] != 1 || out->dims[2] < 6 || out->dims[3] < 1) return ERROR_INVALID_DIMS;
  Plan* p = nullptr;
  if ((st = plan_for(c, 1, H, W, max_det, &p)) != SUCCESS) return st;
  const tensor_t* f[3] = {p3, p4, p5};
  const Buf* dst[3] = {&p->stage[16], &p->stage[19], &p->stage[22]};
  cudaStream_t s = c->eng->stream();
  DevMem tmp;
  size_t maxe = 0;
  for (int i = 0; i < 3; ++i) {
    if (f[i]->dims[1] != dst[i]->C || f[i]->dims[2] != dst[i]->H || f[i]->dims[3] != dst[i]->W) return ERROR_INVALID_DIMS;
    maxe = std::max(maxe, static_cast<size_t>(dst[i]->C) * dst[i]->H * dst[i]->W);
  }
  cudaError_t e = tmp.alloc(maxe * 4);
  for (int i = 0; i < 3 && e == cudaSuccess; ++i) {
    const size_t n = static_cast<size_t>(dst[i]->C) * dst[i]->H * dst[i]->W;
    e = cudaMemcpyAsync(tmp.p, f[i]->data, n * 4, cudaMemcpyHostToDevice, s);
    SOut o;
    o.hi = dst[i]->hi;
    o.plane = dst[i]->plane;
    o.bstride = dst[i]->bstride;
    o.cstride = dst[i]->C;
    if (e == cudaSuccess) e = launch_nchw_to_split(tmp.f(), 1, dst[i]->C, dst[i]->H, dst[i]->W, o, s);
  }
  for (const Op& op : p->ops)
    if (e == cudaSuccess && op.step == 23) e = op.run(s);
  std::vector<float> rows(static_cast<size_t>(max_det) * 6);
  if (e == cudaSuccess) e = cudaMemcpyAsync(rows.data(), p->d_out, rows.size() * 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e, "detect head");
  if ((st = check_kernel_flag(c)) != SUCCESS) return st;
  c->last = p;
  const int rs = out->dims[2] * out->dims[3];
  for (int t = 0; t < max_det; ++t)
    for (int u = 0; u < 6; ++u) out->data[static_cast<size_t>(t) * rs + u] = rows[static_cast<size_t>(t) * 6 + u];
  return SUCCESS;
}
