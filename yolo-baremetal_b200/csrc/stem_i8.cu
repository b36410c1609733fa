// First convolution of the INT8 forward on the tensor cores: the input
// quantisation q = clamp(rint(x / s), -127, 127) fused with model.0 (3x3
// stride 2 pad 1, 3 input channels, 16, 32 or 64 outputs) and its
// requantisation + SiLU table (the scheme in i8k.h), reading the NCHW fp32
// network input.
//
// Per tile of 8 x 16 output pixels: the fp32 input patch (3 channels x 17
// rows x 36 columns) arrives by 16-byte asynchronous copies, double-buffered
// so that the next tile's copy lands while this one is computed; every input
// of the patch is quantised once into one word per input pixel (channels
// 0..2 in bytes 0..2, as the packed weights); every thread gathers the nine
// tap words of its output pixel into the 36-byte im2col row, zero-padded to
// 64 bytes, of a no-swizzle K-major tile; one thread issues two K = 32
// kind::i8 UMMAs against the weights (int32 accumulation in tensor memory);
// every thread then requantises its pixel's accumulator row (the convolution
// epilogue's code, i8_requant.cuh) and stores 16 bytes per 16 channels.
// The A tile and the accumulator are double-buffered and the epilogue of
// tile i runs after the UMMAs of tile i + 1 are issued, so each CTA's
// tensor-core round trip overlaps its own quantisation and requantisation;
// several CTAs per SM overlap the rest.  The products are exact, so the
// result equals the dp4a form of the rule bit for bit.
#include "fastdiv.h"
#include "i8_requant.cuh"
#include "i8k.h"
#include "pdl.cuh"
#include "sm100.cuh"

namespace yb {
namespace {

constexpr int kThreads = 128;
constexpr int kTH = 8, kTW = 16;                    // output tile
constexpr int kPR = 2 * kTH + 1, kPC = 2 * kTW + 4;  // input patch: rows 2 oy0 - 1.., columns 2 ox0 - 4..
constexpr int kPatch = 3 * kPR * kPC;                // floats per fp32 patch
constexpr uint32_t kALbo = 128, kASbo = 512;         // A: 128 rows x 64 bytes of K, core matrices 8 x 16 bytes
constexpr uint32_t kATile = 128 * 64;

__device__ __forceinline__ uint32_t a_off(int r, int kc) {
  return static_cast<uint32_t>((r >> 3) * kASbo + kc * kALbo + (r & 7) * 16);
}

// clamp(rint(v / s), -127, 127) as a byte, v / s correctly rounded.  With
// r = fl(1 / s), y = fl(v * r) lies within 2^-15 of fl(v / s) for |y| <= 200,
// so when y is further than 2^-12 from a half-integer both round to the same
// integer, read from the mantissa of y + 1.5 * 2^23 (round half to even,
// like rintf).  Otherwise (near a rounding boundary, large, or NaN) the exact
// quotient is used.
__device__ __forceinline__ uint32_t quant_byte(float v, float s, float r) {
  const float y = __fmul_rn(v, r);
  const float m = __fadd_rn(y, 12582912.0f);
  const float d = __fsub_rn(y, __fsub_rn(m, 12582912.0f));
  int q;
  if (fabsf(y) <= 200.f && fabsf(d) < 0.49975586f) {
    q = __float_as_int(m) - 0x4B400000;
  } else {
    const float e = rintf(__fdiv_rn(v, s));
    q = static_cast<int>(e < -127.f ? -127.f : e > 127.f ? 127.f : e);
  }
  return static_cast<uint32_t>(min(max(q, -127), 127)) & 0xFFu;
}

// This thread's 16-byte chunks of a patch (the same in every tile): chunk
// i = tid + 128 k is patch row i / 9 (channel, row) and column 4 (i % 9).
struct StemI8Chunks {
  long long goff[4];  // channel plane offset
  uint32_t sdst[4];   // shared byte offset in a patch buffer
  int rr[4], q4[4];   // patch row within the channel, first column
};

__device__ __forceinline__ StemI8Chunks stem_i8_chunks(const StemI8Args& a) {
  StemI8Chunks ch;
  const long long plane = static_cast<long long>(a.H) * a.W;
  constexpr int Q = kPC / 4;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = static_cast<int>(threadIdx.x) + kThreads * k;
    const int row = i / Q, q = i - row * Q;
    const int c = row / kPR;
    ch.rr[k] = row - c * kPR;
    ch.q4[k] = 4 * q;
    ch.goff[k] = c * plane;
    ch.sdst[k] = static_cast<uint32_t>((row * kPC + 4 * q) * 4);
  }
  return ch;
}

// The fp32 input patch of tile t into sx: 16-byte copies when every row
// starts 16-byte aligned (W a multiple of 4, the input 16-byte aligned),
// else 4-byte copies; positions outside the image arrive as zeros.
__device__ __forceinline__ void stem_fetch(const StemI8Args& a, const StemI8Chunks& ch, float* sx, int t,
                                           const FastDiv& fd_per, const FastDiv& fd_tx) {
  const int b = static_cast<int>(fd_per.div(static_cast<uint32_t>(t)));
  const int rem = t - b * static_cast<int>(fd_per.d);
  const int ty = static_cast<int>(fd_tx.div(static_cast<uint32_t>(rem)));
  const int iy0 = ty * kTH * 2 - 1, ix0 = (rem - ty * static_cast<int>(fd_tx.d)) * kTW * 2 - 4;
  const long long plane = static_cast<long long>(a.H) * a.W;
  const float* inb = a.in + static_cast<long long>(b) * 3 * plane;
  if ((a.W & 3) == 0 && (reinterpret_cast<uintptr_t>(a.in) & 15) == 0) {
    constexpr int kChunks = 3 * kPR * (kPC / 4);  // 459: three per thread, a fourth for the first 75
    const uint32_t sbase = smem_u32(sx);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (k == 3 && static_cast<int>(threadIdx.x) >= kChunks - 3 * kThreads) break;
      const int iy = iy0 + ch.rr[k], ix = ix0 + ch.q4[k];
      const int nvalid = (iy >= 0 && iy < a.H && ix >= 0) ? min(4, a.W - ix) : 0;
      const float* src = nvalid > 0 ? inb + ch.goff[k] + static_cast<long long>(iy) * a.W + ix : a.in;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sbase + ch.sdst[k]), "l"(src),
                   "r"(nvalid > 0 ? 4 * nvalid : 0)
                   : "memory");
    }
  } else {
    for (int i = threadIdx.x; i < kPatch; i += kThreads) {
      const int c = i / (kPR * kPC);
      const int rr = (i / kPC) % kPR;
      const int cc = i % kPC;
      const int iy = iy0 + rr, ix = ix0 + cc;
      const bool ok = iy >= 0 && iy < a.H && ix >= 0 && ix < a.W;
      const float* src = ok ? inb + c * plane + static_cast<long long>(iy) * a.W + ix : inb;
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(sx + i)), "l"(src), "r"(ok ? 4 : 0)
                   : "memory");
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// CTAs per SM: shared memory allows six; the 64-channel form's two
// 64-column accumulators allow four in tensor memory.
__host__ __device__ constexpr int stem_i8_ctas(int co) { return co == 64 ? 4 : 6; }

template <int CO>
__global__ void __launch_bounds__(kThreads, stem_i8_ctas(CO)) stem_i8_tc_kernel(const __grid_constant__ StemI8Args a,
                                                                                 FastDiv fd_per, FastDiv fd_tx) {
  constexpr uint32_t kBLbo = static_cast<uint32_t>(CO) * 16u;  // K-direction core-matrix stride of B
  constexpr uint32_t kAcc = static_cast<uint32_t>(CO);          // columns per accumulator
  constexpr uint32_t kCols = 2 * CO < 32 ? 32u : static_cast<uint32_t>(2 * CO);
  __shared__ __align__(1024) uint8_t sa[2][kATile];
  __shared__ __align__(128) uint8_t sbw[4 * kBLbo];
  __shared__ __align__(16) float sx[2][kPatch];  // fp32 patches (double buffer)
  __shared__ uint32_t sqw[kPR * kPC];             // quantised patch, one word per input pixel
  __shared__ int4 sq[CO];  // {M, D low, D high, shift - 32}, D = bias * M + 2^(shift-1) - 1
  __shared__ int32_t sbias[CO];
  __shared__ int8_t slut[256];
  __shared__ uint64_t mbar[2];
  __shared__ uint32_t tslot;

  const int tid = threadIdx.x, warp = tid >> 5;
  // Weights: row n = output channel, K byte 4 tap + c = byte c of w[tap][n]
  // (byte 3 of every word is zero, and so is K past 36).
  for (int i = tid; i < CO * 16; i += kThreads) {
    const int n = i >> 4, kw = i & 15;
    const uint32_t word = kw < 9 ? a.w[kw * CO + n] : 0u;
    const int k = 4 * kw;
    const uint32_t off = static_cast<uint32_t>((k >> 4) * kBLbo + (n >> 3) * 128 + (n & 7) * 16 + (k & 15));
    *reinterpret_cast<uint32_t*>(sbw + off) = word;
  }
  int fast_ok = 1;
  for (int i = tid; i < CO; i += kThreads) {
    const int b = a.bias[i], m = a.mult[i];
    const int sh = m == 0 ? 32 : a.shift[i];
    if (sh < 32) fast_ok = 0;
    const long long d = static_cast<long long>(b) * m + ((1LL << (sh - 1)) - 1);
    sq[i] = make_int4(m, static_cast<int>(static_cast<unsigned long long>(d) & 0xFFFFFFFFull),
                      static_cast<int>(d >> 32), sh - 32);
    sbias[i] = b;
  }
  for (int i = tid; i < 256; i += kThreads) slut[i] = a.lut[i];
  if (tid == 0) {
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tslot, kCols);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  const bool fast = __syncthreads_and(fast_ok) != 0;
  tc_fence_after();
  const uint32_t tmem = tslot;
  if (tid == 0) pdl_trigger();
  pdl_wait();

  const float rcp = __frcp_rn(a.s_in);
  const uint32_t idesc = idesc_s8_s32(128, CO);
  const uint32_t sb_addr = smem_u32(sbw);
  const int tiles = a.B * static_cast<int>(fd_per.d);
  const int r = tid >> 4, cx = tid & 15;  // this thread's output pixel in the tile
  const StemI8Chunks ch = stem_i8_chunks(a);
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
    const int oy = ty * kTH + r, ox = (rem - ty * static_cast<int>(fd_tx.d)) * kTW + cx;
    const uint32_t tb = tmem + (j & 1) * kAcc + (static_cast<uint32_t>(warp * 32) << 16);
    const bool valid = oy < a.Ho && ox < a.Wo;
    int8_t* o = a.out.p + static_cast<long long>(b) * a.out.bstride +
                (static_cast<long long>(oy) * a.Wo + ox) * a.out.cstride;
#pragma unroll
    for (int u = 0; u < CO / 16; ++u) {
      uint32_t acc[16];
      tc_ld_32x32b_x16(tb + 16u * u, acc);
      tc_wait_ld();
      tc_ld_dep(acc);
      uint32_t pk[4];
      bool exact = true;
      if (fast) exact = requant16_fast<true, false>(acc, make_uint4(0u, 0u, 0u, 0u), sq + 16 * u, slut, nullptr, pk);
      // Warp-uniform: the exact path reloads the accumulators.
      if (__any_sync(0xffffffffu, exact)) {
        const uint4 w = requant16_exact<true, false>(tb + 16u * u, make_uint4(0u, 0u, 0u, 0u), sq + 16 * u,
                                                     sbias + 16 * u, slut, nullptr, 0, 1);
        pk[0] = w.x;
        pk[1] = w.y;
        pk[2] = w.z;
        pk[3] = w.w;
      }
      if (valid) *reinterpret_cast<uint4*>(o + 16 * u) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
    tc_fence_before();
  };
  int it = 0;
  if (static_cast<int>(blockIdx.x) < tiles) stem_fetch(a, ch, sx[0], blockIdx.x, fd_per, fd_tx);
  for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
    const int tn = t + gridDim.x;
    // The next tile's patch goes into the other buffer, quantised by the last
    // iteration before its barriers.
    if (tn < tiles) stem_fetch(a, ch, sx[(it + 1) & 1], tn, fd_per, fd_tx);
    if (tn < tiles) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // the patch has landed; the last iteration's gathers from sqw are done
    const float* px = sx[it & 1];
    for (int i = tid; i < kPR * kPC; i += kThreads)
      sqw[i] = quant_byte(px[i], a.s_in, rcp) | (quant_byte(px[kPR * kPC + i], a.s_in, rcp) << 8) |
               (quant_byte(px[2 * kPR * kPC + i], a.s_in, rcp) << 16);
    __syncthreads();
    // Tap (ky, kx) of output pixel (r, cx): input row 2 r + ky, column
    // 2 cx - 1 + kx of the tile's origin, patch column 2 cx + kx + 3.  A
    // stage it & 1 was last read by the UMMAs of two tiles ago, complete
    // before the last epilogue.
    uint32_t wq[16];
#pragma unroll
    for (int ky = 0; ky < 3; ++ky)
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) wq[ky * 3 + kx] = sqw[(2 * r + ky) * kPC + 2 * cx + kx + 3];
#pragma unroll
    for (int k = 9; k < 16; ++k) wq[k] = 0u;
    const uint32_t sa_addr = smem_u32(sa[it & 1]);
#pragma unroll
    for (int kc = 0; kc < 4; ++kc)
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sa_addr + a_off(tid, kc)), "r"(wq[4 * kc]),
                   "r"(wq[4 * kc + 1]), "r"(wq[4 * kc + 2]), "r"(wq[4 * kc + 3])
                   : "memory");
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint64_t da = kmajor_desc_noswizzle(sa_addr, kALbo, kASbo);
      const uint64_t db = kmajor_desc_noswizzle(sb_addr, kBLbo, 128);
      const uint32_t d = tmem + (it & 1) * kAcc;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
        tc_mma_i8(d, da + ((2u * ks * kALbo) >> 4), db + ((2u * ks * kBLbo) >> 4), idesc, ks != 0 ? 1u : 0u);
      tc_commit(&mbar[it & 1]);
    }
    if (it > 0) epilogue(it - 1);
  }
  if (it > 0) epilogue(it - 1);
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

}  // namespace

cudaError_t init_stem_i8_attributes() { return cudaSuccess; }  // static shared memory only

cudaError_t launch_stem_i8(const StemI8Args& a, cudaStream_t st) {
  if ((a.Co != 16 && a.Co != 32 && a.Co != 64) || a.Ho != (a.H - 1) / 2 + 1 || a.Wo != (a.W - 1) / 2 + 1 ||
      a.out.cstride < a.Co || a.out.cstride % 16 || a.out.bstride % 16 || reinterpret_cast<uintptr_t>(a.out.p) % 16 ||
      !a.lut || !(a.s_in > 0.f))
    return cudaErrorInvalidValue;
  const int tiles_x = (a.Wo + kTW - 1) / kTW, tiles_y = (a.Ho + kTH - 1) / kTH;
  const long long tiles = static_cast<long long>(a.B) * tiles_x * tiles_y;
  if (tiles > 0x7fffffffLL - 4096) return cudaErrorInvalidValue;
  if (tiles == 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long cap = static_cast<long long>(stem_i8_ctas(a.Co)) * sms;
  const unsigned grid = static_cast<unsigned>(tiles < cap ? tiles : cap);
  const FastDiv fd_per(static_cast<uint32_t>(tiles_x * tiles_y)), fd_tx(static_cast<uint32_t>(tiles_x));
  if (a.Co == 16) return launch_pdl(stem_i8_tc_kernel<16>, dim3(grid), dim3(kThreads), 0, st, a, fd_per, fd_tx);
  if (a.Co == 32) return launch_pdl(stem_i8_tc_kernel<32>, dim3(grid), dim3(kThreads), 0, st, a, fd_per, fd_tx);
  return launch_pdl(stem_i8_tc_kernel<64>, dim3(grid), dim3(kThreads), 0, st, a, fd_per, fd_tx);
}

}  // namespace yb
