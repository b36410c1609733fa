// First convolution (3x3 stride 2 pad 1, 3 input channels, 16 or 32 output
// channels, + bias + SiLU) on the tensor cores: the model.0 conv_block of
// the reference (layers.c:41-90) reading the NCHW fp32 network input.
//
// Per tile of 128 output pixels (one output row, 128 columns) every thread
// builds the im2col row of its pixel -- the 27 inputs (c, ky, kx) split into
// bf16 hi and lo, 5 zero K values after them -- in a no-swizzle K-major
// shared-memory tile; one thread issues two K = 16 steps of two UMMAs
// against the stacked [W_hi; W_lo] weights (hi*hi + hi*lo + lo*hi + lo*lo,
// fp32 accumulation in TMEM), and every thread reads its pixel's
// accumulator row back, adds the bias, applies SiLU and stores the split
// NHWC output.  Persistent CTAs, several per SM, overlap each other's
// phases; each thread loads the next tile's inputs before the current
// tile's epilogue.  27 products per output channel on the tensor pipe
// replace 27 fused multiply-adds per channel on the CUDA cores.
#include "kernels.h"
#include "pdl.cuh"
#include "sm100.cuh"
#include "split.cuh"

namespace yb {
namespace {

constexpr int kThreads = 128;
constexpr int kTaps = 27;             // 3 channels x 3 x 3
constexpr uint32_t kAPlane = 128 * 64;  // 128 rows x 32 bf16 (K) = 8 KB
constexpr uint32_t kALbo = 128, kASbo = 512;

// Byte offset of 16-byte K chunk kc of row r in the no-swizzle K-major tile
// (core matrices of 8 rows x 16 bytes, LBO along K, SBO along the rows).
__device__ __forceinline__ uint32_t a_off(int r, int kc) {
  return static_cast<uint32_t>((r >> 3) * kASbo + kc * kALbo + (r & 7) * 16);
}

template <int CO>
__global__ void __launch_bounds__(kThreads, 4) stem_tc_kernel(const __grid_constant__ StemArgs a, int tiles_x,
                                                               int tiles) {
  constexpr int N = 2 * CO;                        // stacked [W_hi; W_lo] rows
  constexpr uint32_t kBLbo = static_cast<uint32_t>(N) * 16u;  // K-direction core-matrix stride of B
  constexpr uint32_t kCols = N <= 32 ? 32u : 64u;
  __shared__ __align__(1024) uint8_t sa[2 * kAPlane];
  __shared__ __align__(1024) uint8_t sbw[4 * kBLbo];
  __shared__ float sbias[CO];
  __shared__ uint64_t mbar;
  __shared__ uint32_t tslot;

  const int tid = threadIdx.x, warp = tid >> 5;
  // Weights: K index k = c * 9 + ky * 3 + kx (w's own order), rows n < CO the
  // hi parts, n >= CO the lo parts; K values past 27 are zero.
  for (int i = tid; i < N * 32; i += kThreads) {
    const int n = i >> 5, k = i & 31;
    const int co = n < CO ? n : n - CO;
    const float v = k < a.Ci * 9 ? a.w[co * a.Ci * 9 + k] : 0.0f;
    uint32_t hb, lb;
    split1(v, hb, lb);
    const uint32_t off = static_cast<uint32_t>((k >> 3) * kBLbo + (n >> 3) * 128 + (n & 7) * 16 + (k & 7) * 2);
    *reinterpret_cast<uint16_t*>(sbw + off) = static_cast<uint16_t>(n < CO ? hb : lb);
  }
  for (int i = tid; i < CO; i += kThreads) sbias[i] = a.bias ? a.bias[i] : 0.0f;
  if (tid == 0) {
    mbar_init(&mbar, 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tslot, kCols);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  if (tid == 0) pdl_trigger();
  pdl_wait();

  const uint32_t idesc = idesc_bf16_f32(128, N);
  const uint32_t sa_hi = smem_u32(sa), sa_lo = sa_hi + kAPlane, sb = smem_u32(sbw);
  const long long plane = static_cast<long long>(a.H) * a.W;
  // This thread's pixel of tile t: image b, output row oy, column ox.
  auto locate = [&](int t, int& b, int& oy, int& ox) {
    const int row = t / tiles_x;
    ox = (t - row * tiles_x) * 128 + tid;
    b = row / a.Ho;
    oy = row - b * a.Ho;
  };
  float x[kTaps];
  auto load = [&](int t) {
    int b, oy, ox;
    locate(t, b, oy, ox);
    const bool valid = ox < a.Wo;
    const float* img = a.in + static_cast<long long>(b) * a.Ci * plane;
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
      for (int ky = 0; ky < 3; ++ky)
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
          const int iy = 2 * oy - 1 + ky, ix = 2 * ox - 1 + kx;
          const bool in = valid && c < a.Ci && iy >= 0 && iy < a.H && ix >= 0 && ix < a.W;
          x[c * 9 + ky * 3 + kx] = in ? __ldg(img + c * plane + static_cast<long long>(iy) * a.W + ix) : 0.0f;
        }
  };
  int it = 0;
  if (static_cast<int>(blockIdx.x) < tiles) load(blockIdx.x);
  for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
    // im2col row of this thread's pixel, split into the hi and lo planes.
    uint32_t hw[16], lw[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float v0 = 2 * i < kTaps ? x[2 * i] : 0.0f;
      const float v1 = 2 * i + 1 < kTaps ? x[2 * i + 1] : 0.0f;
      split2(v0, v1, hw[i], lw[i]);
    }
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      const uint32_t o = a_off(tid, kc);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sa_hi + o), "r"(hw[4 * kc]), "r"(hw[4 * kc + 1]),
                   "r"(hw[4 * kc + 2]), "r"(hw[4 * kc + 3])
                   : "memory");
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sa_lo + o), "r"(lw[4 * kc]), "r"(lw[4 * kc + 1]),
                   "r"(lw[4 * kc + 2]), "r"(lw[4 * kc + 3])
                   : "memory");
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint64_t ah = kmajor_desc_noswizzle(sa_hi, kALbo, kASbo);
      const uint64_t al = kmajor_desc_noswizzle(sa_lo, kALbo, kASbo);
      const uint64_t bd = kmajor_desc_noswizzle(sb, kBLbo, 128);
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const uint64_t ao = static_cast<uint64_t>(2 * ks * kALbo) >> 4;
        const uint64_t bo = static_cast<uint64_t>(2 * ks * kBLbo) >> 4;
        tc_mma_bf16(tmem, ah + ao, bd + bo, idesc, ks != 0 ? 1u : 0u);
        tc_mma_bf16(tmem, al + ao, bd + bo, idesc, 1u);
      }
      tc_commit(&mbar);
    }
    // Next tile's inputs while the tensor cores run.
    int b, oy, ox;
    locate(t, b, oy, ox);
    const int tn = t + gridDim.x;
    if (tn < tiles) load(tn);
    volatile int never = 0;
    if (!mbar_wait(&mbar, static_cast<uint32_t>(it & 1), &never, kWaitNs)) {
      if (a.err) atomicCAS(a.err, 0, kErrWaitAccFull);
    }
    tc_fence_after();
    const uint32_t tb = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const bool valid = ox < a.Wo;
    uint16_t* o = a.out.hi + static_cast<long long>(b) * a.out.bstride +
                  (static_cast<long long>(oy) * a.Wo + ox) * a.out.cstride + a.out.coff;
#pragma unroll
    for (int u = 0; u < CO / 16; ++u) {
      uint32_t r[16], r2[16];
      tc_ld_32x32b_x16(tb + 16u * u, r);
      tc_ld_32x32b_x16(tb + CO + 16u * u, r2);
      tc_wait_ld();
      tc_ld_dep(r);
      tc_ld_dep(r2);
      float v[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = __uint_as_float(r[e]) + __uint_as_float(r2[e]) + sbias[16 * u + e];
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = silu_fast(v[e]);
      uint32_t h8[8], l8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) split2(v[2 * i], v[2 * i + 1], h8[i], l8[i]);
      if (valid) {
        st_global_v8(o + 16 * u, h8);
        st_global_v8(o + 16 * u + a.out.plane, l8);
      }
    }
    tc_fence_before();
    __syncthreads();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

}  // namespace

bool stem_tc_supported(const StemArgs& a) {
  return !a.amax && a.Ci >= 1 && a.Ci <= 3 && a.k == 3 && a.stride == 2 && a.pad == 1 &&
         (a.Co == 16 || a.Co == 32) && a.act == kActSiLU && a.out.cstride % 16 == 0 && a.out.coff % 16 == 0 &&
         a.out.bstride % 16 == 0 && a.out.plane % 16 == 0 && reinterpret_cast<uintptr_t>(a.out.hi) % 32 == 0 &&
         a.Ho == (a.H - 1) / 2 + 1 && a.Wo == (a.W - 1) / 2 + 1;
}

cudaError_t launch_stem_tc(const StemArgs& a, cudaStream_t s) {
  if (!stem_tc_supported(a)) return cudaErrorInvalidValue;
  const int tiles_x = (a.Wo + 127) / 128;
  const long long tiles = static_cast<long long>(a.B) * a.Ho * tiles_x;
  if (tiles <= 0) return cudaSuccess;
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long cap = 4LL * sms;
  const unsigned grid = static_cast<unsigned>(tiles < cap ? tiles : cap);
  if (a.Co == 16)
    return launch_pdl(stem_tc_kernel<16>, dim3(grid), dim3(kThreads), 0, s, a, tiles_x, static_cast<int>(tiles));
  return launch_pdl(stem_tc_kernel<32>, dim3(grid), dim3(kThreads), 0, s, a, tiles_x, static_cast<int>(tiles));
}

}  // namespace yb
