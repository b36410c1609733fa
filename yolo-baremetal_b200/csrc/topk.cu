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
// threshold, then the k survivors are ordered by rank (each counts the
// survivors above it).  Stage-1 keys are computed once into shared memory (up
// to kCache of them; more are recomputed per pass).  Stage 2 only ranks the
// pairs that can still make the cut (see the kernel).
#include <atomic>
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
constexpr int kCache = 24576;  // cached keys per stage (dynamic shared memory)
constexpr int kCand = 4096;    // stage-2 candidates (dynamic shared memory, after the keys)

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

// Selects the k largest of key(0..n-1) (order-preserving uint32 keys) under
// (key desc, index asc), writes their indices, in that order, to out[0..k),
// and returns the k-th largest key.
template <typename Key>
__device__ uint32_t select_topk(const Key& key, int n, int k, int* out, TopkSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (k <= 0) return 0u;
  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kT) sm.hist[i] = 0;
    __syncthreads();
#pragma unroll 4
    for (int i = tid; i < n; i += kT) {
      const uint32_t kv = key(i);
      if ((kv & mask) == prefix) atomicAdd(&sm.hist[(kv >> shift) & 255u], 1);
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
    if (key(i) > T) out[atomicAdd(&sm.scratch[2], 1)] = i;
  }
  __syncthreads();
  // Ties at T: the first `remaining` in ascending index order.
  int base = 0;
  for (int c0 = 0; c0 < n && base < remaining; c0 += kT) {
    const int i = c0 + tid;
    const int flag = (i < n && key(i) == T) ? 1 : 0;
    int total;
    const int incl = block_scan(flag, sm, &total);
    const int excl = incl - flag;
    if (flag && base + excl < remaining) out[G + base + excl] = i;
    base += total;
  }
  __syncthreads();
  // Order the k survivors: (key, ~index) is unique, so each survivor's rank
  // is the number of survivors above it.
  for (int i = tid; i < k; i += kT) {
    const int j = out[i];
    sm.sbuf[i] = (static_cast<unsigned long long>(key(j)) << 32) | static_cast<unsigned long long>(~static_cast<uint32_t>(j));
  }
  __syncthreads();
  for (int i = tid; i < k; i += kT) {
    const unsigned long long v = sm.sbuf[i];
    int rank = 0;
    for (int j = 0; j < k; ++j) rank += sm.sbuf[j] > v ? 1 : 0;
    out[rank] = static_cast<int>(~static_cast<uint32_t>(v & 0xffffffffull));
  }
  __syncthreads();
  return T;
}

__global__ void __launch_bounds__(kT) topk_kernel(const TopkArgs a) {
  __shared__ TopkSmem sm;
  extern __shared__ __align__(16) uint32_t keys[];  // kCache keys, then kCand candidates
  pdl_wait();
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
  const bool cache1 = a.N <= kCache;
  if (cache1) {
#pragma unroll 4
    for (int i = threadIdx.x; i < a.N; i += kT) keys[i] = fkey(get1(i));
  }
  __syncthreads();
  const uint32_t T1 = select_topk([&](int i) { return cache1 ? keys[i] : fkey(get1(i)); }, a.N, k, sm.idx1, sm);
  auto get2 = [&](int f) {
    const int slot = f / nc;
    const int c = f - slot * nc;
    return value(sm.idx1[slot], c);
  };
  // Stage 2.  Every selected anchor's best pair scores its stage-1 key, so at
  // least k pairs score >= T1 (the k-th stage-1 key) and only those can be
  // kept: the candidates are the pairs within 16 ulps below T1 or above (a
  // superset, whatever the rounding of the max).  All k * nc keys are
  // computed once into shared memory; each warp then compacts the candidates
  // of its contiguous index range, in index order, into cand[] as
  // (key << 32 | ~index), unique values whose descending order is the
  // wanted one.  Up to kTopkMax candidates are ordered by rank, up to kCand
  // by the radix select over the candidates; more (or fewer than k, or
  // more than kCache pairs) take the radix select over all k * nc pairs.
  const int n2 = k * nc;
  const uint32_t tk = T1 > 16u ? T1 - 16u : 0u;
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(keys + kCache);
  const bool cache2 = n2 <= kCache;
  int m = -1;
  if (cache2) {
#pragma unroll 4
    for (int f = threadIdx.x; f < n2; f += kT) keys[f] = fkey(get2(f));
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int span = (n2 + 31) / 32, f0 = warp * span, f1 = min(n2, f0 + span);
    int cnt = 0;
    for (int f = f0 + lane; f - lane < f1; f += 32)
      cnt += __popc(__ballot_sync(0xffffffffu, f < f1 && keys[f] >= tk));
    if (lane == 0) sm.wtot[warp] = cnt;
    __syncthreads();
    if (warp == 0) {
      const int c = sm.wtot[lane];
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      sm.wtot[lane] = incl - c;  // exclusive offsets
      if (lane == 31) sm.scratch[3] = incl;
    }
    __syncthreads();
    m = sm.scratch[3];
    if (m >= k && m <= kCand) {
      int pos = sm.wtot[warp];
      for (int f = f0 + lane; f - lane < f1; f += 32) {
        const bool hit = f < f1 && keys[f] >= tk;
        const unsigned bal = __ballot_sync(0xffffffffu, hit);
        if (hit)
          cand[pos + __popc(bal & ((1u << lane) - 1u))] =
              (static_cast<unsigned long long>(keys[f]) << 32) | static_cast<unsigned long long>(~static_cast<uint32_t>(f));
        pos += __popc(bal);
      }
    }
    __syncthreads();
  }
  if (m >= k && m <= kTopkMax) {
    for (int i = threadIdx.x; i < m; i += kT) {
      const unsigned long long v = cand[i];
      int rank = 0;
      for (int j = 0; j < m; ++j) rank += cand[j] > v ? 1 : 0;
      if (rank < k) sm.idx2[rank] = static_cast<int>(~static_cast<uint32_t>(v & 0xffffffffull));
    }
    __syncthreads();
  } else if (m >= k && m <= kCand) {
    select_topk([&](int i) { return static_cast<uint32_t>(cand[i] >> 32); }, m, k, sm.idx2, sm);
    for (int t = threadIdx.x; t < k; t += kT)
      sm.idx2[t] = static_cast<int>(~static_cast<uint32_t>(cand[sm.idx2[t]] & 0xffffffffull));
    __syncthreads();
  } else {
    select_topk([&](int f) { return cache2 ? keys[f] : fkey(get2(f)); }, n2, k, sm.idx2, sm);
  }
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

namespace {
constexpr int kTopkSmem = kCache * 4 + kCand * 8;
std::atomic<uint64_t> g_topk_attr_done{0};
}  // namespace

cudaError_t prepare_topk() { return smem_attr_once(topk_kernel, kTopkSmem, g_topk_attr_done); }

cudaError_t launch_topk(const TopkArgs& a, cudaStream_t s) {
  int k = a.max_det < a.N ? a.max_det : a.N;
  if (k > a.cap) k = a.cap;
  if (k > kTopkMax || a.B <= 0) return cudaErrorInvalidValue;
  const cudaError_t e = prepare_topk();
  if (e != cudaSuccess) return e;
  return launch_pdl(topk_kernel, dim3(a.B), dim3(kT), kTopkSmem, s, a);
}

}  // namespace yb
