// Fused Bottleneck for sm_100a: y = x + SiLU(conv2(SiLU(conv1(x)))) with two
// 3x3 stride-1 pad-1 convolutions, conv1 C -> CM and conv2 CM -> C channels
// ((C, CM) = (16, 16), (32, 32), (32, 16) or (16, 8): the C3k Bottlenecks
// and the e = 0.5 Bottlenecks of C3k2), in one persistent kernel.  Replaces the pair of conv_block_forward calls and the
// residual add of bottleneck_forward (layers.c:92-108) inside the C3k2 and
// C3k blocks (layers.c:110-189, model.c:208-283, :415-557).
//
// Per tile of 16 x 8 output pixels the intermediate never leaves the SM:
//   * the producer thread loads the tile's 20 x 12 input patch (halo 2) once
//     per 8-channel chunk and plane with tiled TMA boxes;
//   * conv1 runs on the tensor cores over the patch read as a linear pixel
//     sequence of row width 12: M row p is intermediate pixel (p / 12, p % 12)
//     and filter tap (ky, kx) is the same operand window shifted by
//     ky * 12 + kx pixels, so each tap is one descriptor offset.  Two M = 128
//     tiles cover the 18 x 10 intermediate (rows with p % 12 >= 10 or
//     p >= 214 are discarded);
//   * eight epilogue warps add the bias, apply SiLU, zero the positions that
//     lie outside the image (conv2's zero padding) and write the split
//     intermediate into shared memory in the 18 x 10 patch layout of the
//     unfused 3x3 kernel;
//   * conv2 runs in that patch mode against the shared-memory intermediate;
//   * four epilogue warps add the bias, apply SiLU, add the residual (the
//     block input, L2-resident) and store the split NHWC output.
// Both weight sets stay resident.  The K order (tap, channel), the stacked
// [B_hi; B_lo] split products and the epilogue arithmetic are those of the
// unfused convolution kernel, so the fused result is bit-identical to the
// two separate launches.
//
// Roles (512 threads, one CTA per SM): warp 0 lane 0 producer, warp 1 TMEM
// allocation and UMMA issue, warps 4-7 and 8-11 the conv1 epilogue (M tile
// 0 and 1), warps 12-15 the output epilogue.  Input patches, intermediates
// and both accumulators are double-buffered, and the issuer orders its work
// conv1(t + 1) before conv2(t) so that the tensor cores stay busy while the
// conv1 epilogue of tile t runs.  Every barrier wait is bounded (sm100.cuh).
#include <cudaTypedefs.h>

#include <mutex>

#include "kernels.h"
#include "pdl.cuh"
#include "sm100.cuh"
#include "split.cuh"

namespace yb {
namespace {

constexpr int kThreads = 512;
constexpr int kInW = 12, kInH = 20;                   // input patch (halo 2)
constexpr int kMidW = 10, kMidH = 18;                 // intermediate patch (halo 1)
constexpr uint32_t kInBox = kInW * kInH * 16;         // 3840 bytes per 8-channel box
constexpr uint32_t kInChunk = 4608;                   // box + slack read by discarded M rows
constexpr uint32_t kMidChunk = 2944;                  // 18 x 10 x 16 bytes, 128-byte multiple
constexpr uint32_t kSmemLimit = 232448;

// N tile of a convolution with co output channels (choose_n_tiling for co <= 256).
__host__ __device__ constexpr int ntile(int co) { return (co + 15) / 16 * 16; }
// Packed weights of a 3x3 convolution ci -> co: 64-wide K chunks of ntile(co)
// hi rows then ntile(co) lo rows of 128 bytes.
__host__ __device__ constexpr uint32_t w_bytes(int ci, int co) {
  return static_cast<uint32_t>((9 * ci + 63) / 64) * static_cast<uint32_t>(ntile(co)) * 256u;
}
__host__ __device__ constexpr uint32_t in_stage_bytes(int c) { return 2u * static_cast<uint32_t>(c / 8) * kInChunk; }
__host__ __device__ constexpr uint32_t mid_stage_bytes(int cm) { return 2u * static_cast<uint32_t>(cm / 8) * kMidChunk; }
__host__ __device__ constexpr uint32_t smem_bytes(int c, int cm) {
  return 1024u + w_bytes(c, cm) + w_bytes(cm, c) + 2u * in_stage_bytes(c) + 2u * mid_stage_bytes(cm) + 256u +
         4u * static_cast<uint32_t>(ntile(cm) + c);
}
static_assert(smem_bytes(32, 32) <= kSmemLimit, "the 32-channel fused bottleneck exceeds the 227 KB opt-in limit");

// One tile's 9 taps x CBS 16-channel K steps, stacked split products, fully
// unrolled (compile-time descriptor offsets; see the unfused kernel).  ROWW is
// the operand's pixel row width, CHUNK the byte stride between its 8-channel
// chunks; the weights are NT hi + NT lo rows per 64-wide K chunk.
template <int CBS, int ROWW, uint32_t CHUNK, int NT>
__device__ __forceinline__ void window_mma(uint32_t d, uint64_t ah, uint64_t al, uint64_t bh, uint32_t idesc) {
  constexpr uint64_t chunk_units = static_cast<uint64_t>(NT) * 256u / 16u;
#pragma unroll
  for (int tap = 0; tap < 9; ++tap) {
#pragma unroll
    for (int cb = 0; cb < CBS; ++cb) {
      const int step = tap * CBS + cb;
      const uint64_t ao = static_cast<uint64_t>((tap / 3) * ROWW + tap % 3) + static_cast<uint64_t>(cb) * (2u * CHUNK / 16u);
      const uint64_t bo = static_cast<uint64_t>(step >> 2) * chunk_units + static_cast<uint64_t>((step & 3) * 2);
      tc_mma_bf16(d, ah + ao, bh + bo, idesc, step != 0 ? 1u : 0u);
      tc_mma_bf16(d, al + ao, bh + bo, idesc_half_n(idesc), 1u);
    }
  }
}

// conv2 with 8 intermediate channels (16 bytes per pixel and plane): two
// taps per 16-wide K step, as the unfused kernel's 8-channel patch mode --
// the A descriptor's second core matrix is the next tap's window (LBO = the
// distance between the windows), tap 8 pairs with zero weights and reads the
// zeroed pad after the box.  hb / lb: hi / lo intermediate descriptors with
// LBO 0; K ordered (tap, channel), so the weights hold the two taps back to
// back.
template <int NT>
__device__ __forceinline__ void pair_mma(uint32_t d, uint64_t hb, uint64_t lb, uint64_t bh, uint32_t idesc) {
  constexpr uint64_t chunk_units = static_cast<uint64_t>(NT) * 256u / 16u;
#pragma unroll
  for (int s2 = 0; s2 < 5; ++s2) {
    const int t0 = 2 * s2, t1 = t0 + 1 < 9 ? t0 + 1 : t0;
    const uint32_t o0 = static_cast<uint32_t>(((t0 / 3) * kMidW + t0 % 3) * 16);
    const uint32_t o1 = static_cast<uint32_t>(((t1 / 3) * kMidW + t1 % 3) * 16);
    const uint32_t lbo = t1 == t0 ? 16u : o1 - o0;
    const uint64_t off = static_cast<uint64_t>(o0 >> 4) | (static_cast<uint64_t>(lbo >> 4) << 16);
    const uint64_t bo = static_cast<uint64_t>(s2 >> 2) * chunk_units + static_cast<uint64_t>((s2 & 3) * 2);
    tc_mma_bf16(d, hb + off, bh + bo, idesc, s2 != 0 ? 1u : 0u);
    tc_mma_bf16(d, lb + off, bh + bo, idesc_half_n(idesc), 1u);
  }
}

__device__ __forceinline__ void raise_error(int* err, volatile int* abort_flag, int code) {
  *abort_flag = 1;
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

template <int C, int CM>
__global__ void __launch_bounds__(kThreads, 1) bottleneck_tc_kernel(const __grid_constant__ BottleneckArgs a) {
  constexpr int NCH = C / 8;     // 8-channel chunks of the input and output
  constexpr int NCM = CM / 8;    // 8-channel chunks of the intermediate
  constexpr int CBS = C / 16;    // 16-channel K steps per tap of conv1
  constexpr int N1 = ntile(CM);  // conv1 N tile (8 intermediate channels: 16, upper half zero weights)
  constexpr int N2 = C;          // conv2 N tile
  constexpr uint32_t WB1 = w_bytes(C, CM);
  constexpr uint32_t WB2 = w_bytes(CM, C);
  constexpr uint32_t INS = in_stage_bytes(C);
  constexpr uint32_t MIDS = mid_stage_bytes(CM);
  // TMEM: acc1 (two M tiles of 2 N1 stacked columns) per slot, then acc2 (2 N2).
  constexpr uint32_t kAcc1 = 4u * N1, kAcc2Base = 8u * N1, kAcc2 = 2u * N2;
  constexpr uint32_t kCols = 8u * N1 + 4u * N2 <= 256u ? 256u : 512u;
  static_assert(8u * N1 + 4u * N2 <= 512u, "accumulators exceed tensor memory");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* w1 = smem;
  uint8_t* w2 = smem + WB1;
  uint8_t* inb = smem + WB1 + WB2;
  uint8_t* midb = inb + 2 * INS;
  uint64_t* bars = reinterpret_cast<uint64_t*>(midb + 2 * MIDS);
  uint64_t* in_full = bars;        // [2]
  uint64_t* in_empty = bars + 2;   // [2] conv1 commit
  uint64_t* acc1_full = bars + 4;  // [2]
  uint64_t* acc1_empty = bars + 6; // [2] 8 conv1-epilogue warps
  uint64_t* mid_full = bars + 8;   // [2] 8 conv1-epilogue warps
  uint64_t* mid_empty = bars + 10; // [2] conv2 commit
  uint64_t* acc2_full = bars + 12; // [2]
  uint64_t* acc2_empty = bars + 14;// [2] 4 output-epilogue warps
  uint64_t* wbar = bars + 16;
  uint64_t* drain = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sb1 = reinterpret_cast<float*>(midb + 2 * MIDS + 256);  // [N1]
  float* sb2 = sb1 + N1;                                          // [C]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < N1; i += kThreads) sb1[i] = (a.b1 && i < CM) ? a.b1[i] : 0.0f;
  for (int i = threadIdx.x; i < C; i += kThreads) sb2[i] = a.b2 ? a.b2[i] : 0.0f;
  if (CM == 8) {
    // conv2's paired tap 8 reads the pixel after the intermediate box
    // (against zero weights): keep that pad zero so no stale NaN survives.
    for (int i = threadIdx.x; i < 2 * 2 * 4; i += kThreads) {
      uint8_t* pad = midb + (i >> 3) * MIDS + ((i >> 2) & 1) * kMidChunk + kMidH * kMidW * 16 + (i & 3) * 16;
      *reinterpret_cast<uint4*>(pad) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  // The slack after each input box is read only by discarded conv1 rows;
  // zero it once so that those rows stay finite.
  for (int i = threadIdx.x; i < 2 * 2 * NCH * static_cast<int>((kInChunk - kInBox) / 16); i += kThreads) {
    const int slack = (kInChunk - kInBox) / 16;
    const int chunk = i / slack;
    *reinterpret_cast<uint4*>(inb + chunk * kInChunk + kInBox + (i - chunk * slack) * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&in_full[s], 1);
      mbar_init(&in_empty[s], 1);
      mbar_init(&acc1_full[s], 1);
      mbar_init(&acc1_empty[s], 8);
      mbar_init(&mid_full[s], 8);
      mbar_init(&mid_empty[s], 1);
      mbar_init(&acc2_full[s], 1);
      mbar_init(&acc2_empty[s], 4);
    }
    mbar_init(wbar, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) {
    // The packed weights are written at plan build: load them before
    // waiting on the previous kernel.
    mbar_arrive_expect_tx(wbar, WB1 + WB2);
    bulk_g2s(w1, a.w1, WB1, wbar);
    bulk_g2s(w2, a.w2, WB2, wbar);
    pdl_trigger();
  }
  pdl_wait();

  const uint64_t wlim = kWaitNs;
  const int per = a.tiles_y * a.tiles_x;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tmap(&a.tm_hi);
      prefetch_tmap(&a.tm_lo);
      int lt = 0;
      for (int t = blockIdx.x; t < a.tiles; t += gridDim.x, ++lt) {
        const int s = lt & 1;
        const uint32_t ph = (lt >> 1) & 1;
        if (!mbar_wait(&in_empty[s], ph ^ 1u, abort_flag, wlim)) {
          raise_error(a.err, abort_flag, kErrWaitEmpty);
          break;
        }
        const int b = static_cast<int>(a.fd_per.div(static_cast<uint32_t>(t)));
        const int rem = t - b * per;
        const int ty = static_cast<int>(a.fd_tx.div(static_cast<uint32_t>(rem)));
        const int tx = rem - ty * a.tiles_x;
        uint8_t* st = inb + s * INS;
        mbar_arrive_expect_tx(&in_full[s], 2u * NCH * kInBox);
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          tma_tile_4d(st + ch * kInChunk, &a.tm_hi, 8 * ch, tx * 8 - 2, ty * 16 - 2, b, &in_full[s]);
          tma_tile_4d(st + (NCH + ch) * kInChunk, &a.tm_lo, 8 * ch, tx * 8 - 2, ty * 16 - 2, b, &in_full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- UMMA issue
    if (lane == 0) {
      const uint32_t idesc1 = idesc_bf16_f32(128, 2 * N1);
      const uint32_t idesc2 = idesc_bf16_f32(128, 2 * N2);
      const uint64_t bw1 = sw128_kmajor_desc(smem_u32(w1));
      const uint64_t bw2 = sw128_kmajor_desc(smem_u32(w2));
      bool ok = mbar_wait(wbar, 0, abort_flag, wlim);
      if (!ok) raise_error(a.err, abort_flag, kErrWaitFull);
      int lt = 0;
      for (int t = blockIdx.x; ok; t += gridDim.x, ++lt) {
        const bool has = t < a.tiles;
        if (has) {
          const int s = lt & 1;
          const uint32_t ph = (lt >> 1) & 1;
          if (!mbar_wait(&in_full[s], ph, abort_flag, wlim)) {
            raise_error(a.err, abort_flag, kErrWaitFull);
            break;
          }
          if (!mbar_wait(&acc1_empty[s], ph ^ 1u, abort_flag, wlim)) {
            raise_error(a.err, abort_flag, kErrWaitAccEmpty);
            break;
          }
          tc_fence_after();
          const uint32_t pa = smem_u32(inb + s * INS);
          const uint64_t ah = kmajor_desc_noswizzle(pa, kInChunk, 128);
          const uint64_t al = kmajor_desc_noswizzle(pa + NCH * kInChunk, kInChunk, 128);
          // M tile m starts 128 pixels (2048 bytes, 128 units) further.
          window_mma<CBS, kInW, kInChunk, N1>(tmem_base + s * kAcc1, ah, al, bw1, idesc1);
          window_mma<CBS, kInW, kInChunk, N1>(tmem_base + s * kAcc1 + 2 * N1, ah + 128, al + 128, bw1, idesc1);
          tc_commit(&in_empty[s]);
          tc_commit(&acc1_full[s]);
        }
        if (lt >= 1) {
          // conv2 of the previous tile, once its intermediate is written.
          const int s = (lt - 1) & 1;
          const uint32_t ph = ((lt - 1) >> 1) & 1;
          if (!mbar_wait(&mid_full[s], ph, abort_flag, wlim)) {
            raise_error(a.err, abort_flag, kErrWaitFull);
            break;
          }
          if (!mbar_wait(&acc2_empty[s], ph ^ 1u, abort_flag, wlim)) {
            raise_error(a.err, abort_flag, kErrWaitAccEmpty);
            break;
          }
          tc_fence_after();
          const uint32_t pm = smem_u32(midb + s * MIDS);
          if (CM == 8) {
            const uint64_t hb = kmajor_desc_noswizzle(pm, 0, kMidW * 16);
            const uint64_t lb = kmajor_desc_noswizzle(pm + kMidChunk, 0, kMidW * 16);
            pair_mma<N2>(tmem_base + kAcc2Base + s * kAcc2, hb, lb, bw2, idesc2);
          } else {
            const uint64_t mh = kmajor_desc_noswizzle(pm, kMidChunk, kMidW * 16);
            const uint64_t ml = kmajor_desc_noswizzle(pm + NCM * kMidChunk, kMidChunk, kMidW * 16);
            window_mma<(CM >= 16 ? CM / 16 : 1), kMidW, kMidChunk, N2>(tmem_base + kAcc2Base + s * kAcc2, mh, ml, bw2,
                                                                      idesc2);
          }
          tc_commit(&mid_empty[s]);
          tc_commit(&acc2_full[s]);
        }
        if (!has) break;
      }
      tc_commit(drain);
      bool drained = mbar_try_wait(drain, 0);
      const uint64_t t0 = globaltimer_ns();
      while (!drained && globaltimer_ns() - t0 < wlim) drained = mbar_try_wait(drain, 0);
      if (!drained) raise_error(a.err, abort_flag, kErrDrain);
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------- conv1 epilogue (2 groups)
    const int m = (warp - 4) >> 2;  // M tile
    const int q = warp & 3;         // TMEM lane quarter
    const int p = m * 128 + q * 32 + lane;
    const int py = p / kInW;
    const int px = p - py * kInW;
    const bool keep = px < kMidW && py < kMidH;
    const uint32_t mid_off = static_cast<uint32_t>(py * kMidW + px) * 16u;
    int lt = 0;
    for (int t = blockIdx.x; t < a.tiles; t += gridDim.x, ++lt) {
      const int s = lt & 1;
      const uint32_t ph = (lt >> 1) & 1;
      if (!mbar_wait(&acc1_full[s], ph, abort_flag, wlim)) {
        raise_error(a.err, abort_flag, kErrWaitAccFull);
        break;
      }
      if (!mbar_wait(&mid_empty[s], ph ^ 1u, abort_flag, wlim)) {
        raise_error(a.err, abort_flag, kErrWaitEmpty);
        break;
      }
      tc_fence_after();
      const int b = static_cast<int>(a.fd_per.div(static_cast<uint32_t>(t)));
      const int rem = t - b * per;
      const int ty = static_cast<int>(a.fd_tx.div(static_cast<uint32_t>(rem)));
      const int tx = rem - ty * a.tiles_x;
      const int gy = ty * 16 - 1 + py, gx = tx * 8 - 1 + px;
      const bool inside = static_cast<unsigned>(gy) < static_cast<unsigned>(a.H) &&
                          static_cast<unsigned>(gx) < static_cast<unsigned>(a.W);
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + s * kAcc1 + m * 2 * N1;
      const uint32_t mid = smem_u32(midb + s * MIDS) + mid_off;
#pragma unroll
      for (int u = 0; u < N1 / 16; ++u) {
        uint32_t r[16], r2[16];
        tc_ld_32x32b_x16(tb + u * 16, r);
        tc_ld_32x32b_x16(tb + N1 + u * 16, r2);
        tc_wait_ld();
        tc_ld_dep(r);
        tc_ld_dep(r2);
        float v[16];
        add_pairs<16>(v, reinterpret_cast<const float*>(r), reinterpret_cast<const float*>(r2));
        add_pairs<16>(v, v, sb1 + u * 16);
        silu_fast_n<16>(v);
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = inside ? v[e] : 0.0f;
        uint32_t hw[8], lw[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) split2(v[2 * i], v[2 * i + 1], hw[i], lw[i]);
        if (keep) {
          const uint32_t c0 = static_cast<uint32_t>(2 * u) * kMidChunk;
          st_shared_v4(mid + c0, hw[0], hw[1], hw[2], hw[3]);
          st_shared_v4(mid + NCM * kMidChunk + c0, lw[0], lw[1], lw[2], lw[3]);
          if (CM > 8) {
            st_shared_v4(mid + c0 + kMidChunk, hw[4], hw[5], hw[6], hw[7]);
            st_shared_v4(mid + NCM * kMidChunk + c0 + kMidChunk, lw[4], lw[5], lw[6], lw[7]);
          }
        }
      }
      // The intermediate is read by the tensor cores (async proxy).
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acc1_empty[s]);
        mbar_arrive(&mid_full[s]);
      }
    }
  } else if (warp >= 12) {
    // ---------------------------------------------------- output epilogue
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int ry = r >> 3, rx = r & 7;
    const bool v8out = (reinterpret_cast<uintptr_t>(a.out.hi) & 31) == 0 && (a.out.cstride & 15) == 0 &&
                       (a.out.coff & 15) == 0 && (a.out.bstride & 15) == 0 && (a.out.plane & 15) == 0;
    int lt = 0;
    for (int t = blockIdx.x; t < a.tiles; t += gridDim.x, ++lt) {
      const int s = lt & 1;
      const uint32_t ph = (lt >> 1) & 1;
      if (!mbar_wait(&acc2_full[s], ph, abort_flag, wlim)) {
        raise_error(a.err, abort_flag, kErrWaitAccFull);
        break;
      }
      tc_fence_after();
      const int b = static_cast<int>(a.fd_per.div(static_cast<uint32_t>(t)));
      const int rem = t - b * per;
      const int ty = static_cast<int>(a.fd_tx.div(static_cast<uint32_t>(rem)));
      const int tx = rem - ty * a.tiles_x;
      const int oy = ty * 16 + ry, ox = tx * 8 + rx;
      const bool valid = oy < a.H && ox < a.W;
      const long long po = static_cast<long long>(b) * a.out.bstride +
                           static_cast<long long>(oy * a.W + ox) * a.out.cstride + a.out.coff;
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + kAcc2Base + s * kAcc2;
      // Residual: the block input at this pixel (L2-resident; its loads are
      // issued before the accumulator is read).  Reading it from global
      // memory rather than from the input patch frees the patch as soon as
      // conv1 has consumed it.
      uint4 rh[NCH], rl[NCH];
      {
        const uint16_t* ip = a.in.hi + static_cast<long long>(b) * a.in.bstride +
                             static_cast<long long>(oy * a.W + ox) * a.in.cstride + a.in.coff;
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          rh[ch] = valid ? *reinterpret_cast<const uint4*>(ip + 8 * ch) : make_uint4(0u, 0u, 0u, 0u);
          rl[ch] = valid ? *reinterpret_cast<const uint4*>(ip + a.in.plane + 8 * ch) : make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int u = 0; u < CBS; ++u) {
        uint32_t rr[16], r2[16];
        tc_ld_32x32b_x16(tb + u * 16, rr);
        tc_ld_32x32b_x16(tb + N2 + u * 16, r2);
        tc_wait_ld();
        tc_ld_dep(rr);
        tc_ld_dep(r2);
        float v[16];
        add_pairs<16>(v, reinterpret_cast<const float*>(rr), reinterpret_cast<const float*>(r2));
        add_pairs<16>(v, v, sb2 + u * 16);
        silu_fast_n<16>(v);
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const uint4 h = rh[2 * u + g];
          const uint4 l = rl[2 * u + g];
          const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
          const uint32_t lw[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[8 * g + 2 * i] =
                __fadd_rn(v[8 * g + 2 * i], bf16_bits_to_f(hw[i] & 0xFFFFu) + bf16_bits_to_f(lw[i] & 0xFFFFu));
            v[8 * g + 2 * i + 1] =
                __fadd_rn(v[8 * g + 2 * i + 1], bf16_bits_to_f(hw[i] >> 16) + bf16_bits_to_f(lw[i] >> 16));
          }
        }
        uint32_t hw[8], lw[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) split2(v[2 * i], v[2 * i + 1], hw[i], lw[i]);
        if (valid) {
          uint16_t* o = a.out.hi + po + u * 16;
          if (v8out) {
            st_global_v8(o, hw);
            st_global_v8(o + a.out.plane, lw);
          } else {
            *reinterpret_cast<uint4*>(o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(o + 8) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
            *reinterpret_cast<uint4*>(o + a.out.plane) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            *reinterpret_cast<uint4*>(o + a.out.plane + 8) = make_uint4(lw[4], lw[5], lw[6], lw[7]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc2_empty[s]);
    }
  }

  if (*abort_flag) __nanosleep(100000);  // let an aborted producer's copies land
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 tiled_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Tiled map over one plane of the input view, dims (C, W, H, B), boxes of 8
// channels x 12 x 20 pixels of one image.
bool encode_in_plane(CUtensorMap* map, const BottleneckArgs& a, const uint16_t* base) {
  const auto enc = tiled_encoder();
  if (!enc) return false;
  const long long cs = a.in.cstride;
  if (reinterpret_cast<uintptr_t>(base) % 16 || (cs * 2) % 16 || (a.in.bstride * 2) % 16) return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.C), static_cast<cuuint64_t>(a.W), static_cast<cuuint64_t>(a.H),
                        static_cast<cuuint64_t>(a.B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(cs * 2), static_cast<cuuint64_t>(cs * 2 * a.W),
                           static_cast<cuuint64_t>(a.in.bstride * 2)};
  cuuint32_t box[4] = {8, kInW, kInH, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<uint16_t*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool bottleneck_supported(int C, int CM) {
  return (C == 16 && (CM == 16 || CM == 8)) || (C == 32 && (CM == 32 || CM == 16));
}

bool bottleneck_setup(BottleneckArgs* a) {
  if (!bottleneck_supported(a->C, a->CM) || a->B < 1 || a->H < 1 || a->W < 1 || !a->in.hi || !a->out.hi ||
      !a->w1 || !a->w2)
    return false;
  if (a->in.coff % 8 || a->out.coff % 8 || a->out.cstride % 8 || a->out.bstride % 8 || a->out.plane % 8 ||
      reinterpret_cast<uintptr_t>(a->out.hi) % 16)
    return false;
  const uint16_t* hi = a->in.hi + a->in.coff;
  if (!encode_in_plane(&a->tm_hi, *a, hi) || !encode_in_plane(&a->tm_lo, *a, hi + a->in.plane)) return false;
  a->tiles_x = (a->W + 7) / 8;
  a->tiles_y = (a->H + 15) / 16;
  const long long tiles = static_cast<long long>(a->B) * a->tiles_x * a->tiles_y;
  if (tiles > (1LL << 30)) return false;
  a->tiles = static_cast<int>(tiles);
  a->fd_per = FastDiv(static_cast<uint32_t>(a->tiles_x * a->tiles_y));
  a->fd_tx = FastDiv(static_cast<uint32_t>(a->tiles_x));
  return true;
}

template <int C, int CM>
cudaError_t set_attr() {
  return cudaFuncSetAttribute(bottleneck_tc_kernel<C, CM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(smem_bytes(C, CM)));
}

cudaError_t init_bottleneck_kernel_attributes() {
  cudaError_t e = set_attr<16, 16>();
  if (e == cudaSuccess) e = set_attr<16, 8>();
  if (e == cudaSuccess) e = set_attr<32, 32>();
  if (e == cudaSuccess) e = set_attr<32, 16>();
  return e;
}

template <int C, int CM>
cudaError_t launch_c(const BottleneckArgs& a, cudaStream_t s, int grid) {
  return launch_pdl(bottleneck_tc_kernel<C, CM>, dim3(grid), dim3(kThreads), static_cast<int>(smem_bytes(C, CM)), s,
                    a);
}

cudaError_t launch_bottleneck(const BottleneckArgs& a, cudaStream_t s, int num_sms) {
  if (!bottleneck_supported(a.C, a.CM) || a.tiles != a.B * a.tiles_x * a.tiles_y || a.tiles_x != (a.W + 7) / 8 ||
      a.tiles_y != (a.H + 15) / 16)
    return cudaErrorInvalidValue;
  if (a.tiles <= 0) return cudaSuccess;
  const int grid = a.tiles < num_sms ? a.tiles : num_sms;
  if (a.C == 16) return a.CM == 16 ? launch_c<16, 16>(a, s, grid) : launch_c<16, 8>(a, s, grid);
  return a.CM == 32 ? launch_c<32, 32>(a, s, grid) : launch_c<32, 16>(a, s, grid);
}

}  // namespace yb
