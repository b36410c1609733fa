// Two-stage top-k of the Detect post-process, one CTA (1024 threads) per image.
//
// Reference: detect_postprocess_from_pred (detect.c:63-166).  Stage 1 ranks the
// N anchors by their maximum class score and keeps k = min(max_det, N, cap);
// stage 2 ranks the k*nc (anchor slot, class) scores of those anchors and keeps
// k again.  The reference sorts with qsort on the score alone; glibc's qsort is
// a stable merge sort, so equal scores keep ascending index order (anchor index
// in stage 1, slot*nc + class in stage 2).  Here that order is made explicit:
// (score desc, index asc) is a total order, selected with a 4-pass radix select
// on order-preserving float keys plus an index-ordered scan for ties at the
// threshold, then a bitonic sort of the k survivors in shared memory.
#include <cfloat>
#include "pdl.cuh"
#include "kernels.h"

namespace yb {
namespace {

constexpr int kT = 1024;

__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

// Monotone map float -> uint32 (larger float, larger key).
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct TopkSmem {
  int idx1[kTopkMax];
  int idx2[kTopkMax];
  unsigned long long sbuf[kTopkMax];
  int hist[256];
  int wtot[32];
  int scratch[8];
};

// Inclusive block scan of v over 1024 threads; *total receives the block sum.
__device__ int block_scan(int v, TopkSmem& sm, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  if (lane == 31) sm.wtot[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = sm.wtot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    sm.wtot[lane] = w;
  }
  __syncthreads();
  if (warp > 0) v += sm.wtot[warp - 1];
  *total = sm.wtot[31];
  __syncthreads();
  return v;
}

// Selects the k largest of get(0..n-1) under (value desc, index asc) and
// writes their indices, in that order, to out[0..k).
template <typename Get>
__device__ void select_topk(const Get& get, int n, int k, int* out, TopkSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (k <= 0) return;
  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kT) sm.hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += kT) {
      const uint32_t key = fkey(get(i));
      if ((key & mask) == prefix) atomicAdd(&sm.hist[(key >> shift) & 255u], 1);
    }
    __syncthreads();
    if (warp == 0) {
      // Bins in descending digit order: lane l owns digits 255-8l .. 248-8l.
      int cnt[8];
      int s = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        cnt[j] = sm.hist[255 - (lane * 8 + j)];
        s += cnt[j];
      }
      int incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const unsigned ballot = __ballot_sync(0xffffffffu, incl >= remaining);
      const int L = ballot ? __ffs(ballot) - 1 : 31;
      if (lane == L) {
        int cum = incl - s;
        int d = 255 - lane * 8 - 7;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (cum + cnt[j] >= remaining) {
            d = 255 - (lane * 8 + j);
            break;
          }
          cum += cnt[j];
        }
        sm.scratch[0] = d;
        sm.scratch[1] = cum;
      }
    }
    __syncthreads();
    const int d = sm.scratch[0];
    remaining -= sm.scratch[1];
    prefix |= static_cast<uint32_t>(d) << shift;
    mask |= 255u << shift;
    __syncthreads();
  }
  const uint32_t T = prefix;
  const int G = k - remaining;  // keys strictly above T
  if (tid == 0) sm.scratch[2] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += kT) {
    if (fkey(get(i)) > T) out[atomicAdd(&sm.scratch[2], 1)] = i;
  }
  __syncthreads();
  // Ties at T: the first `remaining` in ascending index order.
  int base = 0;
  for (int c0 = 0; c0 < n && base < remaining; c0 += kT) {
    const int i = c0 + tid;
    const int flag = (i < n && fkey(get(i)) == T) ? 1 : 0;
    int total;
    const int incl = block_scan(flag, sm, &total);
    const int excl = incl - flag;
    if (flag && base + excl < remaining) out[G + base + excl] = i;
    base += total;
  }
  __syncthreads();
  int P = 1;
  while (P < k) P <<= 1;
  for (int i = tid; i < P; i += kT) {
    unsigned long long v = 0ull;
    if (i < k) {
      const int j = out[i];
      v = (static_cast<unsigned long long>(fkey(get(j))) << 32) | static_cast<unsigned long long>(~static_cast<uint32_t>(j));
    }
    sm.sbuf[i] = v;
  }
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < (P >> 1); i += kT) {
        const int lo = 2 * stride * (i / stride) + (i % stride);
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const unsigned long long x = sm.sbuf[lo], y = sm.sbuf[hi];
        if ((x < y) == desc) {
          sm.sbuf[lo] = y;
          sm.sbuf[hi] = x;
        }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < k; i += kT) out[i] = static_cast<int>(~static_cast<uint32_t>(sm.sbuf[i] & 0xffffffffull));
  __syncthreads();
}

__global__ void __launch_bounds__(kT) topk_kernel(const TopkArgs a) {
  pdl_wait();
  __shared__ TopkSmem sm;
  const int b = blockIdx.x;
  int k = a.max_det < a.N ? a.max_det : a.N;
  if (k > a.cap) k = a.cap;
  const float* ms = a.maxscore ? a.maxscore + static_cast<long long>(b) * a.N : nullptr;
  const float* sc = a.scores + static_cast<long long>(b) * a.s_bstride;
  const int nc = a.nc;
  const int rs = a.s_rstride;
  const bool sig = a.apply_sigmoid != 0;
  auto value = [&](int anchor, int c) {
    const float v = __ldg(sc + static_cast<long long>(anchor) * rs + c);
    return sig ? sigmoid(v) : v;
  };
  auto get1 = [&](int i) {
    if (ms) return __ldg(ms + i);
    float m = -FLT_MAX;
    for (int c = 0; c < nc; ++c) {
      const float v = value(i, c);
      if (v > m) m = v;
    }
    return m;
  };
  select_topk(get1, a.N, k, sm.idx1, sm);
  auto get2 = [&](int f) {
    const int slot = f / nc;
    const int c = f - slot * nc;
    return value(sm.idx1[slot], c);
  };
  select_topk(get2, k * nc, k, sm.idx2, sm);
  float* out = a.dets + static_cast<long long>(b) * a.cap * 6;
  for (int t = threadIdx.x; t < a.cap; t += kT) {
    float* row = out + static_cast<long long>(t) * 6;
    if (t < k) {
      const int f = sm.idx2[t];
      const int slot = f / nc;
      const int c = f - slot * nc;
      const int anchor = sm.idx1[slot];
      const float* bx = a.boxes + static_cast<long long>(b) * a.b_bstride + static_cast<long long>(anchor) * a.b_rstride;
      row[0] = bx[0];
      row[1] = bx[1];
      row[2] = bx[2];
      row[3] = bx[3];
      row[4] = get2(f);
      row[5] = static_cast<float>(c);
    } else {
      row[0] = row[1] = row[2] = row[3] = row[4] = row[5] = 0.f;
    }
  }
}

}  // namespace

cudaError_t launch_topk(const TopkArgs& a, cudaStream_t s) {
  int k = a.max_det < a.N ? a.max_det : a.N;
  if (k > a.cap) k = a.cap;
  if (k > kTopkMax || a.B <= 0) return cudaErrorInvalidValue;
  return launch_pdl(topk_kernel, dim3(a.B), dim3(kT), 0, s, a);
}

}  // namespace yb
