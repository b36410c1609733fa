// Detection lists on the device: decode_detections (detection.c:3-34) for a
// batch.  Per image, the rows of its [rows, 6] detections whose score is not
// <= threshold are kept in row order until `capacity` are kept, as
// detection_t {x1, y1, x2, y2, score, (int) class}.  One warp per image:
// each 32-row chunk is compacted with a ballot and a prefix popcount, so the
// kept rows keep their order.
#include <cstdint>

#include "detection.h"
#include "kernels.h"
#include "pdl.cuh"

namespace yb {
namespace {

__global__ void detections_kernel(const float* dets, int B, int rows, float threshold, int capacity,
                                  detection_t* out, int* counts) {
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= B) return;
  const float* d = dets + static_cast<long long>(warp) * rows * 6;
  detection_t* o = out + static_cast<long long>(warp) * capacity;
  int count = 0;
  for (int r0 = 0; r0 < rows && count < capacity; r0 += 32) {
    const int r = r0 + lane;
    const float* row = d + static_cast<long long>(r) * 6;
    const bool keep = r < rows && !(row[4] <= threshold);
    const unsigned m = __ballot_sync(0xffffffffu, keep);
    const int pos = count + __popc(m & ((1u << lane) - 1u));
    if (keep && pos < capacity) {
      detection_t t;
      t.x1 = row[0];
      t.y1 = row[1];
      t.x2 = row[2];
      t.y2 = row[3];
      t.score = row[4];
      t.class_id = static_cast<int>(row[5]);
      o[pos] = t;
    }
    count += __popc(m);
  }
  if (lane == 0) counts[warp] = count < capacity ? count : capacity;
}

}  // namespace

cudaError_t launch_detections(const float* dets, int B, int rows, float threshold, int capacity, detection_t* out,
                              int* counts, cudaStream_t s) {
  if (B < 0 || rows < 0 || capacity < 0) return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  const long long threads = static_cast<long long>(B) * 32;
  return launch_pdl(detections_kernel, dim3(static_cast<unsigned>((threads + 127) / 128)), dim3(128), 0, s, dets, B,
                    rows, threshold, capacity, out, counts);
}

}  // namespace yb
