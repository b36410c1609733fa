// Device replica of a YOLO26 model and its execution plans.
//
// The reference walks a fixed 24-step graph in model_forward_ex
// (model.c:764-903), allocating scratch per block.  Here the same graph is
// lowered once per input shape (B, H, W) into a flat list of kernel launches
// over a single HBM arena: every concat is a channel slice of a shared buffer,
// every upsample is an addressing mode of the consumer's loads, and the whole
// list is captured as one CUDA graph.  Widths come from the weight shapes, so
// any YOLO26 width (n, s, ...) runs unchanged.
#pragma once
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>
#include <cuda_runtime.h>
#include "kernels.h"

namespace yb {

struct HostTensor {
  int dims[4] = {1, 1, 1, 1};
  int ndim = 0;
  std::vector<float> data;  // host values (empty when the values live on the device)
  float* dev = nullptr;     // device values (device weight preparation), else null
  size_t n = 0;             // element count when `data` is empty
  size_t count() const { return dev ? n : data.size(); }
};
using WeightMap = std::map<std::string, HostTensor>;

struct DevConv {
  std::string name;  // weight prefix (the scale-table name of its output)
  uint8_t* wpack = nullptr;
  float* bias = nullptr;
  int co = 0, ci = 0, kh = 0, kw = 0;
  int n_tile = 0, n_tiles = 0, num_kc = 0, K = 0;
  // The same weights packed in narrower N tiles (64 and 128 columns), for
  // launches with too few M tiles to fill the SMs (packed on first use).
  uint8_t* wpack_n[2] = {nullptr, nullptr};
  // Two convolutions of one input stacked along the output channels
  // (conv_pair): packed only in the full tiling.
  bool merged = false;
};
struct DevDw {
  float* w = nullptr;  // [9][C]
  float* bias = nullptr;
  int c = 0;
};
struct DevStem {
  float* w = nullptr;  // [Co][Ci][3][3]
  float* bias = nullptr;
  int co = 0, ci = 0, k = 0;
};

// A full split NHWC activation tensor [B, H, W, C] in the arena: the hi plane
// followed by the lo plane (kernels.h).
struct Buf {
  uint16_t* hi = nullptr;
  int H = 0, W = 0, C = 0;
  long long bstride = 0;
  long long plane = 0;
};

// An input of a convolution: one tensor, or the channel concat of an
// (optionally nearest-upsampled) first source and a second source.
struct Src {
  SView v0;
  int c0 = 0;
  int lg0 = 0;
  SView v1;
  int c1 = 0;
  int H = 0, W = 0;
};

enum OpKind : int { kOpConv = 0, kOpStem = 1, kOpDw = 2, kOpPool = 3, kOpAttn = 4, kOpDecode = 5, kOpTopk = 6 };

struct Op {
  int step;  // profile step (model_forward_profile_t index)
  std::function<cudaError_t(cudaStream_t)> run;
  int kind = kOpConv;
  double flops = 0;  // algorithmic FLOPs of the launch (2 x MACs)
  double bytes = 0;  // algorithmic HBM bytes: inputs + weights read once, outputs written once
  int lane = 0;       // 0: the plan's stream; 1, 2: a side stream (see Plan::fork_after)
  bool join = false;  // every side stream's work completes before this op starts
};

struct Plan {
  int B = 0, H = 0, W = 0;
  int max_det = 300;
  int slot = 0;  // several plans of one shape can coexist (pipelined forwards)
  std::vector<Op> ops;
  std::vector<void*> allocs;
  float* d_in = nullptr;    // [B,3,H,W]
  float* d_out = nullptr;   // [B,max_det,6]
  float* d_dist = nullptr;  // [B,N,4]
  float* d_logits = nullptr;
  float* d_boxes = nullptr;
  float* d_maxscore = nullptr;
  int n_anchors = 0;
  Buf stage[23];  // model->buffers[0..22] equivalents (concat/upsample ones unset)
  cudaGraphExec_t graph = nullptr;
  size_t arena_bytes = 0;
  // Concurrent branches: the ops of side lane L (1, 2) run on lane_s[L] once
  // op fork_after[L] of the plan's stream has run (their only input), and
  // the next op marked `join` waits for them.  The Detect head of the P3
  // and P4 scales runs this way beside the rest of the neck.  Unused (null
  // streams) in calibration plans; per-op profiling runs every op in order
  // on one stream.
  int fork_after[3] = {-1, -1, -1};
  cudaStream_t lane_s[3] = {nullptr, nullptr, nullptr};
  cudaEvent_t ev_fork[3] = {nullptr, nullptr, nullptr};
  cudaEvent_t ev_join[3] = {nullptr, nullptr, nullptr};
  // INT8 plans: stage tensors 01-23 as NHWC int8 with per-channel scales.
  bool int8 = false;
  struct I8Stage {
    int8_t* p = nullptr;
    long long cstride = 0, bstride = 0;
    int C = 0, H = 0, W = 0;
    std::vector<float> cs;
  };
  std::vector<I8Stage> i8stage;
  // Calibration plans (FP32 with statistics): per named tensor the index of
  // its max-|x| word in d_amax (float bits, atomically raised by the kernels).
  bool calib = false;
  unsigned* d_amax = nullptr;
  int amax_used = 0, amax_cap = 0;
  std::vector<std::pair<std::string, int>> amax_names;
};

class Engine {
 public:
  explicit Engine(int device);
  ~Engine();
  Engine(const Engine&) = delete;
  Engine& operator=(const Engine&) = delete;

  // Takes BN-folded host weights (names as written by the converter).
  cudaError_t set_weights(WeightMap&& w, int num_classes, std::string* why);
  // Device weight preparation: takes the converter's raw (unfolded) records,
  // uploads them in one copy and folds BatchNorm on the device; every later
  // packing (FP32 operand images, INT8 quantisation and layouts) then runs
  // as kernels on the device values.  The host keeps only names and shapes.
  cudaError_t set_weights_device(WeightMap&& raw, int num_classes, std::string* why);
  bool device_prep() const { return dev_arena_ != nullptr; }
  // Prepared-weight blob: the folded weights and the packed FP32 operand
  // image (full N tiling) of every convolution, written from device memory;
  // load_blob restores both without folding or packing.
  cudaError_t save_blob(const std::string& path, std::string* why);
  cudaError_t load_blob(const std::string& path, int* num_classes, std::string* why);
  // Test access: kind 0 = the folded fp32 tensor `name`; kind 1 = the packed
  // FP32 operand image of convolution prefix `name` in n_tile-wide N tiles
  // (0: the full tiling); kind 2 = the packed INT8 operand image of
  // convolution `name` in the last-built INT8 plan.
  cudaError_t weight_image(const std::string& name, int kind, int n_tile, std::vector<uint8_t>* out,
                           std::string* why);
  bool has_weights() const { return !hw_.empty(); }

  // Plan for (B, H, W, max_det), built and captured on first use.  Plans with
  // different `slot` values have separate buffers and graphs.
  cudaError_t get_plan(int B, int H, int W, int max_det, Plan** out, std::string* why, int slot = 0);

  // Enqueues the forward of `p` on `s` (graph launch, or eager when
  // step_events != nullptr: then events[2*step], events[2*step+1] bracket
  // each profile step's launches).
  cudaError_t run(Plan* p, cudaStream_t s, cudaEvent_t* step_events);

  // Runs the plan's launches eagerly `reps` times with an event pair around
  // each launch; ms[i] receives launch i's mean device time.
  cudaError_t profile_ops(Plan* p, int reps, std::vector<double>* ms);

  // Reads and clears the kernel error word; returns its value.
  int take_kernel_error();

  // INT8 mode: a non-empty scale table (tensor name -> per-tensor scale)
  // makes get_plan build INT8 plans; an empty one returns to FP32.  INT8
  // plans built under the previous table are released.
  void set_int8_scales(std::map<std::string, float> s);
  bool int8_mode() const { return !i8_scales_.empty(); }

  // Fused block kernels (the Bottleneck pairs of the C3k2 / C3k blocks; on
  // by default).  Off, every convolution is its own launch; the results are
  // bit-identical either way.  Changing it releases every plan.
  void set_fusion(bool on);
  bool fusion() const { return fuse_; }

  // FP32 forwards of n images [n,3,H,W] (host) with statistics: the INT8
  // scale table max|x| / 127 (1 for an all-zero tensor) of every tensor the
  // INT8 plan names.  Uses its own batch-1 plan, released on return.
  cudaError_t calibrate(const float* images, int n, int H, int W, std::map<std::string, float>* table,
                        std::string* why);

  int device() const { return device_; }
  cudaStream_t stream() const { return stream_; }
  int num_classes() const { return nc_; }
  int num_sms() const { return num_sms_; }

 private:
  const HostTensor* find(const std::string& name) const;
  cudaError_t conv_w(const std::string& prefix, bool plain, DevConv** out, std::string* why);
  // The convolutions `a` and `b` (same input and kernel size) as one, output
  // channels [0, co_a) from a and [co_a, co_a + co_b) from b.
  cudaError_t conv_pair(const std::string& a, const std::string& b, DevConv** out, std::string* why);
  // Packing of `d` in N tiles of n_tile (64 or 128) columns, created on first use.
  cudaError_t conv_narrow(DevConv* d, int n_tile, const uint8_t** wpack);
  cudaError_t dw_w(const std::string& prefix, DevDw** out, std::string* why);
  cudaError_t dev_alloc(size_t bytes, void** p);
  void reset_weights();
  cudaError_t setup_stem();
  cudaError_t build(Plan* p, std::string* why);
  cudaError_t build_i8(Plan* p, std::string* why);
  void release_plan(Plan* p);

  int device_ = 0;
  int num_sms_ = 148;
  int nc_ = 80;
  cudaStream_t stream_ = nullptr;
  int* d_err_ = nullptr;
  WeightMap hw_;
  std::map<std::string, DevConv> convs_;
  std::map<std::string, DevDw> dws_;
  DevStem stem_;
  std::vector<void*> weight_allocs_;
  std::vector<std::unique_ptr<Plan>> plans_;
  std::map<std::string, float> i8_scales_;
  bool fuse_ = true;
  float* dev_arena_ = nullptr;  // folded weights (device preparation)
  // INT8 packed operand images of the last INT8 plan: prefix -> (ptr, bytes).
  std::map<std::string, std::pair<const uint8_t*, size_t>> i8_images_;
};

// Reads the converter's .bin layout (int32 nc, int32 count, records) and folds
// BatchNorm exactly like the reference (model.c:121-180, utils.c:81-106).
bool read_weight_bin(const char* path, WeightMap* out, int* num_classes, std::string* why);
void fold_all_bn_map(WeightMap* w);

}  // namespace yb
