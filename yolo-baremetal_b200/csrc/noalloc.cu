// Detect-head top-k that allocates nothing.
//
// The top-k of the Detect post-process (detect.c:63-166 of
// phucb2/yolo-baremetal) first ranks the anchors by their best class score.
// Inside a full forward those per-anchor maxima are scratch memory in the
// plan's arena.  This entry point takes the head tensors already on the device
// and keeps its scratch in one fixed-size array that is part of the library's
// device image, so a call makes no device (or, on success, host) allocation.
// It is meant for callers that cannot allocate: a serving process whose device
// memory is fully owned by its own pool allocator, or a per-frame loop that
// cannot afford the stall of cudaMalloc/cudaFree (cudaFree waits for all work
// on the device).
#include <atomic>
#include <cfloat>
#include <climits>
#include <mutex>
#include <string>

#include "kernels.h"
#include "runtime.h"
#include "status.h"
#include "yb_cuda.h"

namespace yb {
namespace {

// Capacity of the scratch array, in anchors (B * N): 4 MiB of floats, enough
// for 124 images of 640x640 (8400 anchors each).  Every GPU on which the
// library's device code has been loaded holds this array until the process
// exits.
constexpr long long kScratchAnchors = 1ll << 20;

static __device__ __align__(256) float g_anchor_max[kScratchAnchors];

constexpr int kMaxDevices = 64;
std::atomic<float*> g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

// maxscore[a] = max_c sigmoid(logits[a*nc + c]); one warp per anchor, lanes
// over classes (coalesced row reads).  Every element of maxscore[0, anchors)
// is written, so the array needs no clearing between calls.
__global__ void __launch_bounds__(256) anchor_max_kernel(const float* __restrict__ logits, long long anchors, int nc,
                                                         float* __restrict__ maxscore) {
  const long long a = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (a >= anchors) return;  // warp-uniform
  const float* row = logits + a * nc;
  float m = -FLT_MAX;
  for (int c = lane; c < nc; c += 32) {
    const float v = sigmoid(__ldg(row + c));
    if (v > m) m = v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, m, o);
    if (t > m) m = t;
  }
  if (lane == 0) maxscore[a] = m;
}

// Device address of the scratch array on the current device, looked up once
// per device (with that device current) and cached for the life of the
// process.  The cache does not survive cudaDeviceReset (which also ends every
// context of this library on that device).
status_t scratch_on_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("device ordinal beyond the supported 64");
    return ERROR_DEVICE;
  }
  float* p = g_scratch[dev].load(std::memory_order_acquire);
  if (!p) {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    p = g_scratch[dev].load(std::memory_order_relaxed);
    if (!p) {
      e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_anchor_max);
      if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(anchor scratch)");
      g_scratch[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return SUCCESS;
}

}  // namespace

// Loads everything the entry point touches on the current device: the scratch
// array's address (which brings the library's device image, and with it the
// array, onto the device under lazy module loading), the anchor-max kernel and
// the top-k kernel with its shared-memory attribute.  yb_cuda_init calls this,
// so a process that creates a context on a device before its pool allocator
// reserves the remaining memory has nothing left to load on the first call.
status_t noalloc_prepare_current_device() {
  float* p = nullptr;
  status_t st = scratch_on_current_device(&p);
  if (st != SUCCESS) return st;
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, anchor_max_kernel);
  if (e != cudaSuccess) return cuda_status(e, "anchor_max_kernel attributes");
  return cuda_status(prepare_topk(), "topk_kernel attributes");
}

}  // namespace yb

using namespace yb;

extern "C" status_t yb_cuda_detect_topk_noalloc(const float* d_logits, const float* d_boxes, int B, int N, int nc,
                                                int max_det, float* d_dets, void* stream) {
  if (!d_logits || !d_boxes || !d_dets) return ERROR_NULL_POINTER;
  if (B < 1 || N < 1 || nc < 1 || max_det < 1 || nc > (1 << 20)) {
    set_error("detect_topk_noalloc: B, N, nc and max_det must be >= 1 (nc <= 1048576)");
    return ERROR_INVALID_DIMS;
  }
  const int k = max_det < N ? max_det : N;
  if (k > kTopkMax) {
    set_error("detect_topk_noalloc: min(max_det, N) exceeds the top-k limit of 1024");
    return ERROR_INVALID_DIMS;
  }
  const long long anchors = static_cast<long long>(B) * N;
  if (anchors > kScratchAnchors) {
    set_error("detect_topk_noalloc: B*N exceeds the scratch capacity of 1048576 anchors");
    return ERROR_INVALID_DIMS;
  }
  float* maxscore = nullptr;
  status_t st = scratch_on_current_device(&maxscore);
  if (st != SUCCESS) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long blocks = (anchors * 32 + 255) / 256;
  anchor_max_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(d_logits, anchors, nc, maxscore);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "anchor_max_kernel");
  TopkArgs ta;
  ta.maxscore = maxscore;
  ta.scores = d_logits;
  ta.s_bstride = static_cast<long long>(N) * nc;
  ta.s_rstride = nc;
  ta.apply_sigmoid = 1;
  ta.boxes = d_boxes;
  ta.b_bstride = static_cast<long long>(N) * 4;
  ta.b_rstride = 4;
  ta.dets = d_dets;
  ta.B = B;
  ta.N = N;
  ta.nc = nc;
  ta.max_det = max_det;
  ta.cap = max_det;
  return cuda_status(launch_topk(ta, s), "topk_kernel");
}
