// Implicit-GEMM convolution for sm_100a on the 5th-generation tensor cores.
//
// Replaces the reference's conv2d_forward (layers.c:41-81: a direct 7-deep
// loop, or tensor_gemm for 1x1) together with the SiLU / residual / concat
// work around it (layers.c:83-108, :145-153, :259-263).
//
// GEMM view: M = B*Ho*Wo output pixels (128 per tile), N = Co (one tile of up
// to 256 channels, so the activation tile is read once), K = kh*kw*Ci ordered
// (ky, kx, ci) and cut in 64-wide chunks.  FP32 semantics come from split
// operands: activations are stored as bf16 hi/lo planes (kernels.h) and the
// weights are packed the same way, and each 16-wide K step issues three
// kind::f16 UMMAs, hi*hi + hi*lo + lo*hi, accumulating in fp32 in tensor
// memory.
//
// Persistent, warp-specialised CTA (288 threads, one CTA per SM):
//   warps 0-3  producers: each K chunk of the activation tile is gathered with
//              16-byte cp.async copies straight from the hi and lo planes into
//              the 128B-swizzled K-major operand layout (zero fill for padding
//              and K tails; upsample and two-source concat in the address
//              computation), kept PD chunks deep, then published on the
//              stage's mbarrier.  Thread 0 also starts one bulk copy (TMA
//              engine) of the pre-packed, pre-swizzled weight chunk.
//   warp 8     allocates tensor memory (two accumulators) and, from one lane,
//              issues the UMMAs; tcgen05.commit frees each smem stage and
//              publishes each finished accumulator.
//   warps 4-7  epilogue: tcgen05.ld of their 32 TMEM lanes (= 32 output
//              pixels), + bias, SiLU, + residual, split (or fp32) NHWC store
//              into the destination channel slice.  Runs while warp 8
//              accumulates the next tile into the other TMEM buffer.
// All barrier waits are bounded (sm100.cuh); a timeout sets *a.err, aborts
// the other roles, drains outstanding copies and UMMAs and frees tensor
// memory.
#include <cstdio>
#include <cstring>
#include <vector>
#include "kernels.h"
#include "sm100.cuh"
#include "split.cuh"

namespace yb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kProducerWarps = 8;  // two per sub-partition: the im2col address stream is the long pole
constexpr int kRowsPerThread = kBM * 8 / (kProducerWarps * 32);  // 16-byte columns per row = 8
constexpr int kEpilogueWarps = 8;  // two per TMEM lane quarter, splitting the columns
constexpr int kMmaWarp = kProducerWarps + kEpilogueWarps;
constexpr int kThreads = (kMmaWarp + 1) * 32;
constexpr uint32_t kAPlaneBytes = kBM * 128;  // one 128 x 64 bf16 plane
constexpr int kSmemLimit = 232448;            // 227 KB opt-in per CTA
constexpr int kSmemExtra = 1024 + 512;

__device__ __forceinline__ void raise_error(int* err, volatile int* abort_flag, int code) {
  *abort_flag = 1;
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Arrives on `bar` (counting as one of its expected arrivals) once every
// cp.async this thread issued so far has landed in shared memory.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) conv_tc_kernel(const ConvArgs a, const int stages) {
  extern __shared__ uint8_t smem_raw[];
  // Swizzle atoms need 1024-byte alignment in the shared window.
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t chunk_bytes = static_cast<uint32_t>(a.n_tile) * 256u;
  const uint32_t stage_bytes = 2u * kAPlaneBytes + chunk_bytes;

  uint8_t* tail = smem + stages * stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  uint32_t ncols = 32;
  while (ncols < 2u * static_cast<uint32_t>(a.n_tile)) ncols <<= 1;
  const uint32_t acc_stride = ncols >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], kProducerWarps * 32);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpilogueWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = a.m_tiles * a.n_tiles;
  const int HoWo = a.Ho * a.Wo;
  const int M = a.B * HoWo;

  if (warp < kProducerWarps) {
    // ------------------------------------------------------------ producers
    // Thread t copies the 16-byte column j = t % 8 (8 K indices) of rows
    // t / 8 + 32 i, i = 0..3, for both planes.  Per tile each row's pixel
    // offset in both sources is computed once; per chunk only the tap and
    // channel of column j change, so a copy costs a few adds and compares.
    const int ptid = threadIdx.x;
    const int j = ptid & 7;
    const int r0 = ptid >> 3;
    uint32_t it = 0;  // chunks issued
    const uint32_t smem_base = smem_u32(smem);
    const int ws0 = a.W >> a.lg_up0, ws1 = a.W >> a.lg_up1;
    const float inv_ci = 1.0f / static_cast<float>(a.Ci);
    uint32_t row_off[kRowsPerThread];
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i)
      row_off[i] = sw128_offset(static_cast<uint32_t>(r0 + 32 * i), static_cast<uint32_t>(j));
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      const int mt = t / a.n_tiles;
      const int nt = t - mt * a.n_tiles;
      int iy0[kRowsPerThread], ix0[kRowsPerThread];
      long long off0[kRowsPerThread], off1[kRowsPerThread];
      {
        // Row r0 of the tile, then step 32 pixels per row without dividing.
        const int m = mt * kBM + r0;
        int b = m / HoWo;
        int r = m - b * HoWo;
        int oy = r / a.Wo;
        int ox = r - oy * a.Wo;
#pragma unroll
        for (int i = 0; i < kRowsPerThread; ++i) {
          const bool valid = m + 32 * i < M;
          const int iy = oy * a.stride - a.pad;
          const int ix = ox * a.stride - a.pad;
          iy0[i] = valid ? iy : -(1 << 28);  // never in bounds
          ix0[i] = ix;
          off0[i] = static_cast<long long>(b) * a.src0.bstride +
                    static_cast<long long>((iy >> a.lg_up0) * ws0 + (ix >> a.lg_up0)) * a.src0.cstride;
          off1[i] = static_cast<long long>(b) * a.src1.bstride +
                    static_cast<long long>((iy >> a.lg_up1) * ws1 + (ix >> a.lg_up1)) * a.src1.cstride;
          ox += 32;
          while (ox >= a.Wo) {
            ox -= a.Wo;
            if (++oy == a.Ho) {
              oy = 0;
              ++b;
            }
          }
        }
      }
      const uint8_t* wsrc = a.wpack + static_cast<size_t>(nt) * a.num_kc * chunk_bytes;
      for (int kc = 0; kc < a.num_kc; ++kc) {
        const uint32_t s = it % stages;
        const uint32_t ph = (it / stages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) {
          raise_error(a.err, abort_flag, kErrWaitEmpty);
          goto producer_done;
        }
        const uint32_t sa_hi = smem_base + s * stage_bytes;
        const uint32_t sa_lo = sa_hi + kAPlaneBytes;
        if (ptid == 0) {
          mbar_expect_tx(&full[s], chunk_bytes);
          bulk_g2s(smem + s * stage_bytes + 2 * kAPlaneBytes, wsrc + static_cast<size_t>(kc) * chunk_bytes,
                   chunk_bytes, &full[s]);
        }
        const int k = kc * kBK + j * 8;
        const bool kvalid = k < a.K;
        // tap = k / Ci via a float reciprocal with an exact integer fix-up.
        int tap = __float2int_rz(static_cast<float>(k) * inv_ci);
        if (tap * a.Ci > k) --tap;
        if ((tap + 1) * a.Ci <= k) ++tap;
        const int c = k - tap * a.Ci;
        int ky = 0;
        while ((ky + 1) * a.kw <= tap) ++ky;
        const int kx = tap - ky * a.kw;
        const bool first = c < a.c_split;
        const uint16_t* sp = first ? a.src0.hi : a.src1.hi;
        const long long splane = first ? a.src0.plane : a.src1.plane;
        const int tap_off = first ? (ky * ws0 + kx) * a.src0.cstride + a.src0.coff + c
                                  : (ky * ws1 + kx) * a.src1.cstride + a.src1.coff + (c - a.c_split);
#pragma unroll
        for (int i = 0; i < kRowsPerThread; ++i) {
          const int iy = iy0[i] + ky;
          const int ix = ix0[i] + kx;
          const bool ok = kvalid && static_cast<unsigned>(iy) < static_cast<unsigned>(a.H) &&
                          static_cast<unsigned>(ix) < static_cast<unsigned>(a.W);
          const uint16_t* p = ok ? sp + (first ? off0[i] : off1[i]) + tap_off : sp;
          cp_async16(sa_hi + row_off[i], p, ok ? 16u : 0u);
          cp_async16(sa_lo + row_off[i], p + (ok ? splane : 0), ok ? 16u : 0u);
        }
        // The stage is published by the copies themselves: this thread's
        // arrival on full[s] fires when all its copies so far have landed.
        cp_async_arrive_noinc(&full[s]);
        ++it;
      }
    }
  producer_done:
    cp_async_wait_all();
  } else if (warp < kMmaWarp) {
    // ------------------------------------------------------------- epilogue
    const int e_idx = warp - kProducerWarps;  // 0..7
    const int q = e_idx & 3;                  // TMEM lane quarter (= warp % 4)
    const int half = e_idx >> 2;              // which 32-column chunks this warp takes
    const bool f32out = a.out_f32.ptr != nullptr;
    int lt = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++lt) {
      const int acc = lt & 1;
      const uint32_t aph = (lt >> 1) & 1;
      if (!mbar_wait(&acc_full[acc], aph, abort_flag)) {
        raise_error(a.err, abort_flag, kErrWaitAccFull);
        break;
      }
      tc_fence_after();
      const int mt = t / a.n_tiles;
      const int nt = t - mt * a.n_tiles;
      const int n0 = nt * a.n_tile;
      const int nvalid = min(a.n_tile, a.Co - n0);
      const int m = mt * kBM + q * 32 + lane;
      const bool valid = m < M;
      int b = 0, p = 0;
      if (valid) {
        b = m / HoWo;
        p = m - b * HoWo;
      }
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * acc_stride;
      for (int c0 = 32 * half; c0 < nvalid; c0 += 64) {
        // Two 16-column TMEM loads, one wait; never past this accumulator.
        uint32_t r[32];
        uint32_t(&r0)[16] = *reinterpret_cast<uint32_t(*)[16]>(&r[0]);
        uint32_t(&r1)[16] = *reinterpret_cast<uint32_t(*)[16]>(&r[16]);
        tc_ld_32x32b_x16(tbase + c0, r0);
        if (c0 + 16 < a.n_tile) tc_ld_32x32b_x16(tbase + c0 + 16, r1);
        tc_wait_ld();
        if (!valid) continue;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int n = c0 + 8 * g;  // column within the tile
          if (n >= nvalid) break;
          float x[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = __uint_as_float(r[8 * g + e]);
          if (a.bias) {
            const float4 b0 = __ldg(reinterpret_cast<const float4*>(a.bias + n0 + n));
            const float4 b1 = __ldg(reinterpret_cast<const float4*>(a.bias + n0 + n + 4));
            x[0] += b0.x;
            x[1] += b0.y;
            x[2] += b0.z;
            x[3] += b0.w;
            x[4] += b1.x;
            x[5] += b1.y;
            x[6] += b1.z;
            x[7] += b1.w;
          }
          if (a.act == kActSiLU) {
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = silu_fast(x[e]);
          }
          if (a.res.hi) {
            float rv[8];
            load8_rw(a.res.hi + static_cast<long long>(b) * a.res.bstride + static_cast<long long>(p) * a.res.cstride +
                         a.res.coff + n0 + n,
                     a.res.plane, rv);
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] += rv[e];
          }
          if (f32out) {
            float* o = a.out_f32.ptr + static_cast<long long>(b) * a.out_f32.bstride +
                       static_cast<long long>(p) * a.out_f32.cstride + a.out_f32.coff + n0 + n;
            *reinterpret_cast<float4*>(o) = make_float4(x[0], x[1], x[2], x[3]);
            if (n + 4 < nvalid) *reinterpret_cast<float4*>(o + 4) = make_float4(x[4], x[5], x[6], x[7]);
          } else {
            store8(a.out.hi + static_cast<long long>(b) * a.out.bstride + static_cast<long long>(p) * a.out.cstride +
                       a.out.coff + n0 + n,
                   a.out.plane, x);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  } else {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kBM, a.n_tile);
      uint32_t it = 0;
      int lt = 0;
      for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++lt) {
        const int acc = lt & 1;
        const uint32_t aph = (lt >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], aph ^ 1u, abort_flag)) {
          raise_error(a.err, abort_flag, kErrWaitAccEmpty);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * acc_stride;
        bool ok = true;
        for (int kc = 0; kc < a.num_kc; ++kc, ++it) {
          const uint32_t s = it % stages;
          const uint32_t ph = (it / stages) & 1u;
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            raise_error(a.err, abort_flag, kErrWaitFull);
            ok = false;
            break;
          }
          // The stage's activation tile was written by cp.async; order it
          // before the tensor core's (async-proxy) operand reads.
          fence_proxy_async_smem();
          tc_fence_after();
          // Descriptors of the stage's four operand planes; a 16-wide K step
          // advances the start address by 32 bytes (2 in the >>4 field).
          const uint32_t a_hi = smem_u32(smem + s * stage_bytes);
          const uint64_t dah0 = sw128_kmajor_desc(a_hi);
          const uint64_t dal0 = sw128_kmajor_desc(a_hi + kAPlaneBytes);
          const uint64_t dbh0 = sw128_kmajor_desc(a_hi + 2 * kAPlaneBytes);
          const uint64_t dbl0 = sw128_kmajor_desc(a_hi + 2 * kAPlaneBytes + static_cast<uint32_t>(a.n_tile) * 128u);
#pragma unroll
          for (int ks = 0; ks < kBK / 16; ++ks) {
            const uint64_t koff = static_cast<uint64_t>(ks * 2);
            tc_mma_bf16(d_tmem, dah0 + koff, dbh0 + koff, idesc, (kc | ks) != 0 ? 1u : 0u);
            tc_mma_bf16(d_tmem, dah0 + koff, dbl0 + koff, idesc, 1u);
            tc_mma_bf16(d_tmem, dal0 + koff, dbh0 + koff, idesc, 1u);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[acc]);
      }
      // Drain: every UMMA issued above completes before tensor memory is freed.
      tc_commit(drain);
      bool drained = mbar_try_wait(drain, 0);
      const uint64_t t0 = globaltimer_ns();
      while (!drained && globaltimer_ns() - t0 < kWaitNs) drained = mbar_try_wait(drain, 0);
      if (!drained) raise_error(a.err, abort_flag, kErrDrain);
    }
    __syncwarp();
  }

  // An aborted producer may have left a bulk copy in flight: give it time to land.
  if (*abort_flag) __nanosleep(100000);
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, ncols);
  }
}

inline uint16_t host_bf16_rn(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return static_cast<uint16_t>(u >> 16);
}
inline float host_bf16_to_float(uint16_t h) {
  const uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

int stages_for(int n_tile) {
  const int stage_bytes = 2 * kAPlaneBytes + static_cast<int>(conv_chunk_bytes(n_tile));
  int stages = (kSmemLimit - kSmemExtra) / stage_bytes;
  return stages > 8 ? 8 : stages;
}

}  // namespace

void choose_n_tiling(int co, int* n_tile, int* n_tiles) {
  const int tiles = (co + 255) / 256;
  const int per = (co + tiles - 1) / tiles;
  *n_tile = ((per + 15) / 16) * 16;
  *n_tiles = tiles;
}

size_t pack_conv_weights(const float* w, int co, int ci, int kh, int kw, int n_tile, uint8_t* dst) {
  const int K = kh * kw * ci;
  const int num_kc = (K + kBK - 1) / kBK;
  const int n_tiles = (co + n_tile - 1) / n_tile;
  const size_t chunk = conv_chunk_bytes(n_tile);
  const size_t total = static_cast<size_t>(n_tiles) * num_kc * chunk;
  if (!dst) return total;
  std::memset(dst, 0, total);
  for (int nt = 0; nt < n_tiles; ++nt) {
    for (int kc = 0; kc < num_kc; ++kc) {
      uint8_t* hi_plane = dst + (static_cast<size_t>(nt) * num_kc + kc) * chunk;
      uint8_t* lo_plane = hi_plane + static_cast<size_t>(n_tile) * 128;
      for (int r = 0; r < n_tile; ++r) {
        const int n = nt * n_tile + r;
        if (n >= co) continue;
        for (int kk = 0; kk < kBK; ++kk) {
          const int k = kc * kBK + kk;
          if (k >= K) break;
          const int tap = k / ci;
          const int c = k - tap * ci;
          const int ky = tap / kw;
          const int kx = tap - ky * kw;
          const float v = w[((static_cast<size_t>(n) * ci + c) * kh + ky) * kw + kx];
          const uint16_t h = host_bf16_rn(v);
          const uint16_t l = host_bf16_rn(v - host_bf16_to_float(h));
          const uint32_t off = sw128_offset(r, kk >> 3) + (kk & 7) * 2;
          std::memcpy(hi_plane + off, &h, 2);
          std::memcpy(lo_plane + off, &l, 2);
        }
      }
    }
  }
  return total;
}

// Opts the kernels into the full 227 KB of shared memory on the current
// device.  Called once per device before any launch (and outside capture).
cudaError_t init_conv_kernel_attributes() {
  return cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
}

cudaError_t launch_conv_tc(const ConvArgs& a, cudaStream_t s, int num_sms) {
  const bool f32 = a.out_f32.ptr != nullptr;
  if (a.n_tile < 16 || a.n_tile > 256 || (a.n_tile % 16) != 0 || a.Ci % 8 != 0 || a.c_split % 8 != 0 ||
      a.Co % (f32 ? 4 : 8) != 0)
    return cudaErrorInvalidValue;
  // Upsampled sources are read by 1x1, stride-1, unpadded convolutions only
  // (the producer resolves their pixel once per row, not per tap).
  if ((a.lg_up0 || a.lg_up1) && (a.kh != 1 || a.kw != 1 || a.stride != 1 || a.pad != 0))
    return cudaErrorInvalidValue;
  const int stages = stages_for(a.n_tile);
  if (stages < 2) return cudaErrorInvalidValue;
  const int stage_bytes = 2 * kAPlaneBytes + static_cast<int>(conv_chunk_bytes(a.n_tile));
  const int smem = kSmemExtra + stages * stage_bytes;
  const int total = a.m_tiles * a.n_tiles;
  if (total <= 0) return cudaSuccess;
  const int grid = total < num_sms ? total : num_sms;
  conv_tc_kernel<<<grid, kThreads, smem, s>>>(a, stages);
  return cudaGetLastError();
}

}  // namespace yb
