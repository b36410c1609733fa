// First convolution (3x3 stride 2 pad 1, 1-3 input channels, 16 or 32 output
// channels, + bias + SiLU) on the tensor cores: the model.0 conv_block of
// the reference (layers.c:41-90) reading the NCHW fp32 network input.
//
// Per tile of 128 output pixels (2 output rows x 64 columns):
//   * the tile's fp32 input patch (3 channels x 5 rows x 136 columns, from
//     column 2 ox0 - 4) arrives by 16-byte asynchronous copies into one of
//     two shared buffers while the previous tile computes; positions outside
//     the image arrive as zeros, which is the convolution's padding;
//   * every thread reads the 27 inputs (c, ky, kx) of its pixel from the
//     patch and writes them, split into bf16 hi and lo, as its row of a
//     no-swizzle K-major tile pair (K = 32, the last 5 zero);
//   * one thread issues two K = 16 steps of two UMMAs against the stacked
//     [W_hi; W_lo] weights (hi*hi + hi*lo + lo*hi + lo*lo, fp32
//     accumulation in tensor memory);
//   * every thread reads its pixel's accumulator row back, adds the bias,
//     applies SiLU and stores the split NHWC output (32 bytes per plane per
//     16 channels).
// The operand tiles and the accumulators are double-buffered and the
// epilogue of tile i runs after the UMMAs of tile i + 1 are issued, so each
// CTA's tensor-core round trip overlaps its own CUDA-core work; several CTAs
// per SM overlap the rest.
#include "fastdiv.h"
#include "kernels.h"
#include "pdl.cuh"
#include "sm100.cuh"
#include "split.cuh"

namespace yb {
namespace {

constexpr int kThreads = 128;
constexpr int kTW = 64;                       // output columns per tile (2 rows)
constexpr int kPR = 5, kPC = 2 * kTW + 8;     // patch rows, columns (from 2 ox0 - 4)
constexpr int kPatch = 3 * kPR * kPC;         // floats per patch
constexpr uint32_t kPatchBytes = kPatch * 4;  // 8,160
constexpr uint32_t kALbo = 128, kASbo = 512;  // core matrices 8 rows x 16 bytes; 4 along K
constexpr uint32_t kAPlane = 128 * 64;        // 128 rows x 32 bf16
template <int CO>
struct StemTcSmem {
  static constexpr int N = 2 * CO;                                     // stacked [W_hi; W_lo] rows
  static constexpr uint32_t kBLbo = static_cast<uint32_t>(N) * 16u;  // K-direction core-matrix stride of B
  static constexpr uint32_t kOffA = 0;                                 // 2 stages x (hi, lo)
  static constexpr uint32_t kOffB = 4 * kAPlane;
  static constexpr uint32_t kOffX = kOffB + 4 * kBLbo;
  static constexpr uint32_t kOffBias = kOffX + 2 * kPatchBytes;
  static constexpr uint32_t kBytes = kOffBias + 4 * CO + 16;
  static constexpr uint32_t kAccCols = static_cast<uint32_t>(N);      // one accumulator
  static constexpr uint32_t kCols = 2 * kAccCols;                       // two accumulators
};

// Byte offset of 16-byte K chunk kc of row r in the no-swizzle K-major tile.
__device__ __forceinline__ uint32_t a_off(int r, int kc) {
  return static_cast<uint32_t>((r >> 3) * kASbo + kc * kALbo + (r & 7) * 16);
}

// The fp32 input patch of tile t (image b, output rows 2 ty, 2 ty + 1,
// columns 64 tx ..) into sx: 16-byte copies when every row starts 16-byte
// aligned (W a multiple of 4, the input 16-byte aligned), else 4-byte
// copies; positions outside the image, and channels past Ci, arrive as
// zeros.
// This thread's 16-byte chunks of a patch (the same in every tile): chunk
// i = tid + 128 k is patch row i / 34 (channel, row) and column 4 (i % 34).
struct StemChunks {
  long long goff[4];  // channel plane offset + 4 q
  uint32_t sdst[4];   // shared address offset (bytes) in a patch buffer
  int rr[4], q4[4];   // patch row within the channel, first column
  bool live[4];       // chunk exists and its channel is below Ci
};

__device__ __forceinline__ StemChunks stem_chunks(const StemArgs& a) {
  StemChunks ch;
  const long long plane = static_cast<long long>(a.H) * a.W;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = static_cast<int>(threadIdx.x) + kThreads * k;
    const int row = i / (kPC / 4), q = i - row * (kPC / 4);
    const int c = row / kPR;
    ch.live[k] = i < 3 * kPR * (kPC / 4) && c < a.Ci;
    ch.rr[k] = row - c * kPR;
    ch.q4[k] = 4 * q;
    ch.goff[k] = c * plane;
    ch.sdst[k] = static_cast<uint32_t>((row * kPC + 4 * q) * 4);
  }
  return ch;
}

__device__ __forceinline__ void stem_tc_fetch(const StemArgs& a, const StemChunks& ch, float* sx, int t,
                                              const FastDiv& fd_per, const FastDiv& fd_tx) {
  const int b = static_cast<int>(fd_per.div(static_cast<uint32_t>(t)));
  const int rem = t - b * static_cast<int>(fd_per.d);
  const int ty = static_cast<int>(fd_tx.div(static_cast<uint32_t>(rem)));
  const int iy0 = 4 * ty - 1, ix0 = 2 * (rem - ty * static_cast<int>(fd_tx.d)) * kTW - 4;
  const long long plane = static_cast<long long>(a.H) * a.W;
  const float* inb = a.in + static_cast<long long>(b) * a.Ci * plane;
  if ((a.W & 3) == 0 && (reinterpret_cast<uintptr_t>(a.in) & 15) == 0) {
    const uint32_t sbase = smem_u32(sx);
    // Chunks 0..2 exist for every thread, chunk 3 for the first 126.
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (k == 3 && threadIdx.x >= 3 * kPR * (kPC / 4) - 3 * kThreads) break;
      const int iy = iy0 + ch.rr[k], ix = ix0 + ch.q4[k];
      const int nvalid = (ch.live[k] && iy >= 0 && iy < a.H && ix >= 0) ? min(4, a.W - ix) : 0;
      const float* src = nvalid > 0 ? inb + ch.goff[k] + static_cast<long long>(iy) * a.W + ix : a.in;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sbase + ch.sdst[k]), "l"(src),
                   "r"(nvalid > 0 ? 4 * nvalid : 0)
                   : "memory");
    }
  } else {
    for (int i = threadIdx.x; i < kPatch; i += kThreads) {
      const int row = i / kPC;
      const int cc = i - row * kPC;
      const int c = row / kPR;
      const int iy = iy0 + (row - c * kPR), ix = ix0 + cc;
      const bool ok = c < a.Ci && iy >= 0 && iy < a.H && ix >= 0 && ix < a.W;
      const float* src = ok ? inb + c * plane + static_cast<long long>(iy) * a.W + ix : a.in;
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(sx + i)), "l"(src), "r"(ok ? 4 : 0)
                   : "memory");
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int CO>
__global__ void __launch_bounds__(kThreads, 4) stem_tc_kernel(const __grid_constant__ StemArgs a, FastDiv fd_per,
                                                               FastDiv fd_tx) {
  using L = StemTcSmem<CO>;
  constexpr int N = L::N;
  extern __shared__ __align__(128) uint8_t smem[];
  float* sx = reinterpret_cast<float*>(smem + L::kOffX);
  float* sbias = reinterpret_cast<float*>(smem + L::kOffBias);
  __shared__ uint64_t mbar[2];
  __shared__ uint32_t tslot;

  const int tid = threadIdx.x, warp = tid >> 5;
  // Weights: K index k = c * 9 + ky * 3 + kx (w's own order), rows n < CO the
  // hi parts, n >= CO the lo parts; K values past Ci * 9 are zero.
  for (int i = tid; i < N * 32; i += kThreads) {
    const int n = i >> 5, k = i & 31;
    const int co = n < CO ? n : n - CO;
    const float v = k < a.Ci * 9 ? a.w[co * a.Ci * 9 + k] : 0.0f;
    uint32_t hb, lb;
    split1(v, hb, lb);
    const uint32_t off = static_cast<uint32_t>((k >> 3) * L::kBLbo + (n >> 3) * 128 + (n & 7) * 16 + (k & 7) * 2);
    *reinterpret_cast<uint16_t*>(smem + L::kOffB + off) = static_cast<uint16_t>(n < CO ? hb : lb);
  }
  for (int i = tid; i < CO; i += kThreads) sbias[i] = a.bias ? a.bias[i] : 0.0f;
  if (tid == 0) {
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tslot, L::kCols);
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
  const uint32_t sa0 = smem_u32(smem + L::kOffA), sb = smem_u32(smem + L::kOffB);
  const int tiles = a.B * static_cast<int>(fd_per.d);
  const int r = tid >> 6, cx = tid & 63;  // this thread's output pixel in the tile
  const StemChunks ch = stem_chunks(a);
  volatile int never = 0;
  // Epilogue of this CTA's j-th tile (accumulator j & 1).
  auto epilogue = [&](int j) {
    const int t = static_cast<int>(blockIdx.x) + j * static_cast<int>(gridDim.x);
    if (!mbar_wait(&mbar[j & 1], static_cast<uint32_t>((j >> 1) & 1), &never, kWaitNs)) {
      if (a.err) atomicCAS(a.err, 0, kErrWaitAccFull);
    }
    tc_fence_after();
    const int b = static_cast<int>(fd_per.div(static_cast<uint32_t>(t)));
    const int rem = t - b * static_cast<int>(fd_per.d);
    const int ty = static_cast<int>(fd_tx.div(static_cast<uint32_t>(rem)));
    const int oy = 2 * ty + r, ox = (rem - ty * static_cast<int>(fd_tx.d)) * kTW + cx;
    const uint32_t tb = tmem + (j & 1) * L::kAccCols + (static_cast<uint32_t>(warp * 32) << 16);
    const bool valid = oy < a.Ho && ox < a.Wo;
    uint16_t* o = a.out.hi + static_cast<long long>(b) * a.out.bstride +
                  (static_cast<long long>(oy) * a.Wo + ox) * a.out.cstride + a.out.coff;
#pragma unroll
    for (int u = 0; u < CO / 16; ++u) {
      uint32_t r1[16], r2[16];
      tc_ld_32x32b_x16(tb + 16u * u, r1);
      tc_ld_32x32b_x16(tb + CO + 16u * u, r2);
      tc_wait_ld();
      tc_ld_dep(r1);
      tc_ld_dep(r2);
      float v[16];
#pragma unroll
      for (int e4 = 0; e4 < 4; ++e4) {
        const float4 b4 = *reinterpret_cast<const float4*>(sbias + 16 * u + 4 * e4);
        const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int e = 4 * e4; e < 4 * e4 + 4; e += 2) {
          const float2 t = __fadd2_rn(make_float2(__uint_as_float(r1[e]), __uint_as_float(r1[e + 1])),
                                      make_float2(__uint_as_float(r2[e]), __uint_as_float(r2[e + 1])));
          const float2 u2 = __fadd2_rn(t, make_float2(bb[e - 4 * e4], bb[e + 1 - 4 * e4]));
          v[e] = u2.x;
          v[e + 1] = u2.y;
        }
      }
      silu_fast_n<16>(v);
      uint32_t h8[8], l8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) split2(v[2 * i], v[2 * i + 1], h8[i], l8[i]);
      if (valid) {
        st_global_v8(o + 16 * u, h8);
        st_global_v8(o + 16 * u + a.out.plane, l8);
      }
    }
    tc_fence_before();
  };
  int it = 0;
  if (static_cast<int>(blockIdx.x) < tiles) stem_tc_fetch(a, ch, sx, blockIdx.x, fd_per, fd_tx);
  for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
    const int tn = t + gridDim.x;
    // The next tile's patch goes into the other buffer, read by the last
    // iteration before its barrier below.
    if (tn < tiles) stem_tc_fetch(a, ch, sx + ((it + 1) & 1) * kPatch, tn, fd_per, fd_tx);
    if (tn < tiles) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // Im2col row of this thread's pixel, inputs (c, 2 r + ky, 2 cx + 3 + kx)
    // of the patch, split into operand stage it & 1 (whose previous UMMAs,
    // two tiles ago, completed before the last epilogue).
    const float* px = sx + (it & 1) * kPatch + (2 * r) * kPC + 2 * cx + 3;
    float x[28];
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
      for (int ky = 0; ky < 3; ++ky)
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) x[c * 9 + ky * 3 + kx] = px[(c * kPR + ky) * kPC + kx];
    x[27] = 0.0f;
    uint32_t hw[16], lw[16];
#pragma unroll
    for (int i = 0; i < 14; ++i) split2(x[2 * i], x[2 * i + 1], hw[i], lw[i]);
    hw[14] = hw[15] = lw[14] = lw[15] = 0u;
    const uint32_t ahi = sa0 + (it & 1) * 2 * kAPlane, alo = ahi + kAPlane;
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      const uint32_t o = a_off(tid, kc);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(ahi + o), "r"(hw[4 * kc]), "r"(hw[4 * kc + 1]),
                   "r"(hw[4 * kc + 2]), "r"(hw[4 * kc + 3])
                   : "memory");
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(alo + o), "r"(lw[4 * kc]), "r"(lw[4 * kc + 1]),
                   "r"(lw[4 * kc + 2]), "r"(lw[4 * kc + 3])
                   : "memory");
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint64_t ah = kmajor_desc_noswizzle(ahi, kALbo, kASbo);
      const uint64_t al = kmajor_desc_noswizzle(alo, kALbo, kASbo);
      const uint64_t bd = kmajor_desc_noswizzle(sb, L::kBLbo, 128);
      const uint32_t d = tmem + (it & 1) * L::kAccCols;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const uint64_t ao = static_cast<uint64_t>(2 * ks * kALbo) >> 4;
        const uint64_t bo = static_cast<uint64_t>(2 * ks * L::kBLbo) >> 4;
        tc_mma_bf16(d, ah + ao, bd + bo, idesc, ks != 0 ? 1u : 0u);
        tc_mma_bf16(d, al + ao, bd + bo, idesc, 1u);
      }
      tc_commit(&mbar[it & 1]);
    }
    if (it > 0) epilogue(it - 1);
  }
  if (it > 0) epilogue(it - 1);
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kCols);
  }
}

std::atomic<uint64_t> g_stem_tc_attr16{0}, g_stem_tc_attr32{0};

}  // namespace

bool stem_tc_supported(const StemArgs& a) {
  return !a.amax && a.Ci >= 1 && a.Ci <= 3 && a.k == 3 && a.stride == 2 && a.pad == 1 &&
         (a.Co == 16 || a.Co == 32) && a.act == kActSiLU && a.out.cstride % 16 == 0 && a.out.coff % 16 == 0 &&
         a.out.bstride % 16 == 0 && a.out.plane % 16 == 0 && reinterpret_cast<uintptr_t>(a.out.hi) % 32 == 0 &&
         a.Ho == (a.H - 1) / 2 + 1 && a.Wo == (a.W - 1) / 2 + 1;
}

cudaError_t launch_stem_tc(const StemArgs& a, cudaStream_t s) {
  if (!stem_tc_supported(a)) return cudaErrorInvalidValue;
  const int tiles_x = (a.Wo + kTW - 1) / kTW, tiles_y = (a.Ho + 1) / 2;
  const long long tiles = static_cast<long long>(a.B) * tiles_y * tiles_x;
  if (tiles <= 0) return cudaSuccess;
  if (tiles > 0x7fffffffLL - 4096) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long cap = 4LL * sms;
  const unsigned grid = static_cast<unsigned>(tiles < cap ? tiles : cap);
  const FastDiv fd_per(static_cast<uint32_t>(tiles_x * tiles_y)), fd_tx(static_cast<uint32_t>(tiles_x));
  if (a.Co == 16) {
    cudaError_t e = smem_attr_once(stem_tc_kernel<16>, StemTcSmem<16>::kBytes, g_stem_tc_attr16);
    if (e != cudaSuccess) return e;
    return launch_pdl(stem_tc_kernel<16>, dim3(grid), dim3(kThreads), StemTcSmem<16>::kBytes, s, a, fd_per, fd_tx);
  }
  cudaError_t e = smem_attr_once(stem_tc_kernel<32>, StemTcSmem<32>::kBytes, g_stem_tc_attr32);
  if (e != cudaSuccess) return e;
  return launch_pdl(stem_tc_kernel<32>, dim3(grid), dim3(kThreads), StemTcSmem<32>::kBytes, s, a, fd_per, fd_tx);
}

}  // namespace yb
