// Fused INT8 Bottleneck for sm_100a: out = in + requant(conv2(requant(
// conv1(in)))) with two 3x3 stride-1 pad-1 kind::i8 convolutions, conv1
// C -> CM and conv2 CM -> C ((C, CM) = (16, 16), (32, 32), (32, 16) or
// (16, 8)), each with the requantisation and SiLU table of the INT8 graph
// and the residual table term on conv2 -- the Bottleneck of layers.c:92-108
// under the INT8 scheme of yb_int8.h.  The int8 intermediate stays in shared
// memory; the result is bit-identical to the two conv_i8_kernel launches
// (integer accumulation is exact, and the epilogue is the same code,
// i8_requant.cuh).
//
// Layout and pipeline follow the FP32 kernel (bottleneck_tc.cu): per tile of
// 16 x 8 output pixels one thread loads the 20 x 12 input patch (halo 2) as
// 16-channel int8 planes (16 bytes per pixel); conv1 reads it as a linear
// pixel sequence of row width 12 over two M = 128 tiles; eight warps
// requantise the 18 x 10 intermediate into shared memory (zero outside the
// image); conv2 reads it as the unfused patch mode does; four warps
// requantise with the residual term and store.  One UMMA covers a 32-byte K
// step: two 16-channel planes (LBO = plane stride), or with 16 channels two
// taps (the second core matrix at the next tap's window).
// Roles (512 threads, one CTA per SM): warp 0 lane 0 producer, warp 1 TMEM
// and UMMA issue, warps 4-11 conv1 epilogue (M tile 0 / 1), warps 12-15
// output epilogue.  Every barrier wait is bounded (sm100.cuh).
#include <cudaTypedefs.h>

#include <mutex>

#include "i8_requant.cuh"
#include "int8.h"
#include "pdl.cuh"
#include "sm100.cuh"

namespace yb {
namespace {

constexpr int kThreads = 512;
constexpr int kKB = 128;  // K values (bytes) per packed weight chunk
constexpr int kInW = 12, kInH = 20;
constexpr int kMidW = 10, kMidH = 18;
constexpr uint32_t kInBox = kInW * kInH * 16;  // 3840 bytes per 16-channel plane
constexpr uint32_t kInChunk = 4608;            // plane stride: box + slack read by discarded M rows
constexpr uint32_t kMidChunk = 2944;           // 18 x 10 x 16 bytes, 128-byte multiple
constexpr uint32_t kSmemLimit = 232448;

__host__ __device__ constexpr int round16(int c) { return (c + 15) / 16 * 16; }
// Packed weights of a 3x3 convolution ci -> co as the INT8 graph packs it:
// ci <= 16 two taps per 32-byte step (K = 144), else ci padded to 32 (K = 288).
__host__ __device__ constexpr uint32_t w_bytes(int ci, int co) {
  return static_cast<uint32_t>(((ci <= 16 ? 144 : 288) + kKB - 1) / kKB) * static_cast<uint32_t>(round16(co)) * 128u;
}
__host__ __device__ constexpr int planes(int c) { return (c + 15) / 16; }
__host__ __device__ constexpr uint32_t smem_bytes(int c, int cm) {
  return 1024u + w_bytes(c, cm) + w_bytes(cm, c) + 2u * planes(c) * kInChunk + 2u * planes(cm) * kMidChunk + 256u +
         4096u;
}
static_assert(smem_bytes(32, 32) <= kSmemLimit, "fused INT8 bottleneck shared memory");

// One tile's conv K steps: PAIR (16 channels, two taps per 32-byte step) or
// 9 taps of one 32-channel step (two 16-channel planes, LBO = plane stride).
// ROWW: operand row width in pixels; NT: the weights' rows per K chunk.
template <bool PAIR, int ROWW, int NT>
__device__ __forceinline__ void i8_window_mma(uint32_t d, uint64_t base, uint64_t bw, uint32_t idesc) {
  constexpr uint64_t chunk_units = static_cast<uint64_t>(NT) * 128u / 16u;
  if (PAIR) {
#pragma unroll
    for (int s2 = 0; s2 < 5; ++s2) {
      const int t0 = 2 * s2, t1 = 2 * s2 + 1 < 9 ? 2 * s2 + 1 : t0;
      const uint32_t o0 = static_cast<uint32_t>(((t0 / 3) * ROWW + t0 % 3) * 16);
      const uint32_t o1 = static_cast<uint32_t>(((t1 / 3) * ROWW + t1 % 3) * 16);
      const uint32_t lbo = t1 == t0 ? 16u : o1 - o0;
      const uint64_t off = static_cast<uint64_t>(o0 >> 4) | (static_cast<uint64_t>(lbo >> 4) << 16);
      const int k = 32 * s2;
      const uint64_t bo = static_cast<uint64_t>(k / kKB) * chunk_units + static_cast<uint64_t>(((k % kKB) / 32) * 2);
      tc_mma_i8(d, base + off, bw + bo, idesc, s2 != 0 ? 1u : 0u);
    }
  } else {
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
      const uint64_t ao = static_cast<uint64_t>((tap / 3) * ROWW + tap % 3);
      const int k = 32 * tap;
      const uint64_t bo = static_cast<uint64_t>(k / kKB) * chunk_units + static_cast<uint64_t>(((k % kKB) / 32) * 2);
      tc_mma_i8(d, base + ao, bw + bo, idesc, tap != 0 ? 1u : 0u);
    }
  }
}

__device__ __forceinline__ void raise_error(int* err, volatile int* abort_flag, int code) {
  *abort_flag = 1;
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Per-channel requantisation constants (conv_i8_kernel's prologue): qc =
// {M, low and high word of D = bias * M + 2^(shift-1) - 1, shift - 32}, sb =
// bias; returns whether every shift allows the fast path.
__device__ __forceinline__ bool fill_tables(int n, int co, const int32_t* bias, const int32_t* mult,
                                            const int32_t* shift, int4* qc, int32_t* sb) {
  bool fast = true;
  for (int i = threadIdx.x; i < n; i += kThreads) {
    const bool ok = i < co;
    const int b = ok ? bias[i] : 0;
    const int m = ok ? mult[i] : 0;
    const int sh = m == 0 ? 32 : shift[i];
    if (sh < 32) fast = false;
    const long long d = static_cast<long long>(b) * m + ((1LL << (sh - 1)) - 1);
    qc[i] = make_int4(m, static_cast<int>(static_cast<unsigned long long>(d) & 0xFFFFFFFFull),
                      static_cast<int>(d >> 32), sh - 32);
    sb[i] = b;
  }
  return fast;
}

template <int C, int CM>
__global__ void __launch_bounds__(kThreads, 1) bottleneck_i8_kernel(const __grid_constant__ I8BottleneckArgs a) {
  constexpr bool PAIR1 = C <= 16, PAIR2 = CM <= 16;
  constexpr int N1 = round16(CM), N2 = C;
  constexpr int NPI = planes(C), NPM = planes(CM);
  constexpr uint32_t WB1 = w_bytes(C, CM), WB2 = w_bytes(CM, C);
  constexpr uint32_t INS = NPI * kInChunk, MIDS = NPM * kMidChunk;
  // TMEM columns: conv1 slot s, M tile m at 32 (2 s + m); conv2 slot s at 128 + 32 s.
  constexpr uint32_t kCols = 256;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* w1 = smem;
  uint8_t* w2 = smem + WB1;
  uint8_t* inb = smem + WB1 + WB2;
  uint8_t* midb = inb + 2 * INS;
  uint64_t* bars = reinterpret_cast<uint64_t*>(midb + 2 * MIDS);
  uint64_t* in_full = bars;
  uint64_t* in_empty = bars + 2;   // conv1 commit
  uint64_t* acc1_full = bars + 4;
  uint64_t* acc1_empty = bars + 6; // 8 conv1-epilogue warps
  uint64_t* mid_full = bars + 8;   // 8 conv1-epilogue warps
  uint64_t* mid_empty = bars + 10; // conv2 commit
  uint64_t* acc2_full = bars + 12;
  uint64_t* acc2_empty = bars + 14;// 4 output-epilogue warps
  uint64_t* wbar = bars + 16;
  uint64_t* drain = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int4* qc1 = reinterpret_cast<int4*>(midb + 2 * MIDS + 256);  // [N1]
  int4* qc2 = qc1 + N1;                                          // [N2]
  int32_t* sb1 = reinterpret_cast<int32_t*>(qc2 + N2);
  int32_t* sb2 = sb1 + N1;
  int32_t* srtab = sb2 + N2;                                     // [256] residual table
  int8_t* slut1 = reinterpret_cast<int8_t*>(srtab + 256);        // [256]
  int8_t* slut2 = slut1 + 256;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  bool fast_ok = fill_tables(N1, CM, a.b1, a.m1, a.s1, qc1, sb1);
  fast_ok = fill_tables(N2, C, a.b2, a.m2, a.s2, qc2, sb2) && fast_ok;
  if (((128LL * a.res_mult) >> a.res_shift) >= (1LL << 29)) fast_ok = false;
  for (int i = threadIdx.x; i < 256; i += kThreads) {
    slut1[i] = a.lut1[i];
    slut2[i] = a.lut2[i];
    srtab[i] = static_cast<int32_t>(rshift_rne(static_cast<long long>(i - 128) * a.res_mult, a.res_shift));
  }
  // The slack after each input box is read only by discarded conv1 rows.
  for (int i = threadIdx.x; i < 2 * NPI * static_cast<int>((kInChunk - kInBox) / 16); i += kThreads) {
    const int slack = (kInChunk - kInBox) / 16;
    const int chunk = i / slack;
    *reinterpret_cast<uint4*>(inb + chunk * kInChunk + kInBox + (i - chunk * slack) * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
  if (PAIR2) {
    // conv2's paired tap 8 reads the pixel after the intermediate box.
    for (int i = threadIdx.x; i < 2 * 4; i += kThreads) {
      uint8_t* pad = midb + (i >> 2) * MIDS + kMidH * kMidW * 16 + (i & 3) * 16;
      *reinterpret_cast<uint4*>(pad) = make_uint4(0u, 0u, 0u, 0u);
    }
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
  const bool fast = __syncthreads_and(fast_ok ? 1 : 0) != 0;
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) {
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
      prefetch_tmap(&a.tm);
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
        mbar_arrive_expect_tx(&in_full[s], NPI * kInBox);
#pragma unroll
        for (int pl = 0; pl < NPI; ++pl)
          tma_tile_4d(inb + s * INS + pl * kInChunk, &a.tm, 16 * pl, tx * 8 - 2, ty * 16 - 2, b, &in_full[s]);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- UMMA issue
    if (lane == 0) {
      const uint32_t idesc1 = idesc_s8_s32(128, N1);
      const uint32_t idesc2 = idesc_s8_s32(128, N2);
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
          const uint64_t base = kmajor_desc_noswizzle(pa, PAIR1 ? 0u : kInChunk, 128);
          // M tile 1 starts 128 pixels (2048 bytes, 128 units) further.
          i8_window_mma<PAIR1, kInW, N1>(tmem_base + 64u * s, base, bw1, idesc1);
          i8_window_mma<PAIR1, kInW, N1>(tmem_base + 64u * s + 32u, base + 128, bw1, idesc1);
          tc_commit(&in_empty[s]);
          tc_commit(&acc1_full[s]);
        }
        if (lt >= 1) {
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
          const uint64_t base = kmajor_desc_noswizzle(pm, PAIR2 ? 0u : kMidChunk, kMidW * 16);
          i8_window_mma<PAIR2, kMidW, N2>(tmem_base + 128u + 32u * s, base, bw2, idesc2);
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
    const int m = (warp - 4) >> 2;
    const int q = warp & 3;
    const int p = m * 128 + q * 32 + lane;
    const int py = p / kInW;
    const int px = p - py * kInW;
    const bool keep = px < kMidW && py < kMidH;
    const uint32_t mid_off = static_cast<uint32_t>(py * kMidW + px) * 16u;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
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
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + 64u * s + 32u * m;
      const uint32_t mid = smem_u32(midb + s * MIDS) + mid_off;
#pragma unroll
      for (int u = 0; u < N1 / 16; ++u) {
        uint32_t r[16];
        tc_ld_32x32b_x16(tb + 16u * u, r);
        tc_wait_ld();
        tc_ld_dep(r);
        uint32_t pk[4] = {0u, 0u, 0u, 0u};
        bool exact = !fast;
        if (fast) exact = requant16_fast<true, false>(r, zero, qc1 + 16 * u, slut1, srtab, pk);
        // Warp-uniform: the exact path reloads the accumulators.
        if (__any_sync(0xffffffffu, exact)) {
          const uint4 w = requant16_exact<true, false>(tb + 16u * u, zero, qc1 + 16 * u, sb1 + 16 * u, slut1, srtab,
                                                       a.res_mult, a.res_shift);
          pk[0] = w.x;
          pk[1] = w.y;
          pk[2] = w.z;
          pk[3] = w.w;
        }
        if (keep) st_shared_v4(mid + u * kMidChunk, inside ? make_uint4(pk[0], pk[1], pk[2], pk[3]) : zero);
      }
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
      const long long pix = static_cast<long long>(oy * a.W + ox);
      // Residual: the block input at this pixel (L2-resident), 16 channels per word group.
      uint4 rv[NPI];
#pragma unroll
      for (int pl = 0; pl < NPI; ++pl)
        rv[pl] = valid ? *reinterpret_cast<const uint4*>(a.in + static_cast<long long>(b) * a.in_bstride +
                                                         pix * a.in_cstride + 16 * pl)
                       : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + 128u + 32u * s;
#pragma unroll
      for (int u = 0; u < N2 / 16; ++u) {
        uint32_t rr[16];
        tc_ld_32x32b_x16(tb + 16u * u, rr);
        tc_wait_ld();
        tc_ld_dep(rr);
        uint32_t pk[4] = {0u, 0u, 0u, 0u};
        bool exact = !fast;
        if (fast) exact = requant16_fast<true, true>(rr, rv[u], qc2 + 16 * u, slut2, srtab, pk);
        if (__any_sync(0xffffffffu, exact)) {
          const uint4 w = requant16_exact<true, true>(tb + 16u * u, rv[u], qc2 + 16 * u, sb2 + 16 * u, slut2, srtab,
                                                      a.res_mult, a.res_shift);
          pk[0] = w.x;
          pk[1] = w.y;
          pk[2] = w.z;
          pk[3] = w.w;
        }
        if (valid)
          *reinterpret_cast<uint4*>(a.out + static_cast<long long>(b) * a.out_bstride + pix * a.out_cstride + 16 * u) =
              make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc2_empty[s]);
    }
  }

  if (*abort_flag) __nanosleep(100000);
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

template <int C, int CM>
cudaError_t set_attr() {
  return cudaFuncSetAttribute(bottleneck_i8_kernel<C, CM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(smem_bytes(C, CM)));
}
template <int C, int CM>
cudaError_t launch_c(const I8BottleneckArgs& a, cudaStream_t s, int grid) {
  return launch_pdl(bottleneck_i8_kernel<C, CM>, dim3(grid), dim3(kThreads), static_cast<int>(smem_bytes(C, CM)), s,
                    a);
}

}  // namespace

bool i8_bottleneck_supported(int C, int CM) {
  return (C == 16 && (CM == 16 || CM == 8)) || (C == 32 && (CM == 32 || CM == 16));
}

bool i8_bottleneck_setup(I8BottleneckArgs* a) {
  if (!i8_bottleneck_supported(a->C, a->CM) || a->B < 1 || a->H < 1 || a->W < 1 || !a->in || !a->out || !a->w1 ||
      !a->w2 || !a->lut1 || !a->lut2 || a->res_shift < 1 || a->res_shift > 62)
    return false;
  if (a->in_cstride % 16 || a->in_bstride % 16 || reinterpret_cast<uintptr_t>(a->in) % 16 || a->out_cstride % 16 ||
      a->out_bstride % 16 || reinterpret_cast<uintptr_t>(a->out) % 16)
    return false;
  const auto enc = tiled_encoder();
  if (!enc) return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(a->C), static_cast<cuuint64_t>(a->W), static_cast<cuuint64_t>(a->H),
                        static_cast<cuuint64_t>(a->B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(a->in_cstride), static_cast<cuuint64_t>(a->in_cstride * a->W),
                           static_cast<cuuint64_t>(a->in_bstride)};
  cuuint32_t box[4] = {16, kInW, kInH, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  if (enc(&a->tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t*>(a->in), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  a->tiles_x = (a->W + 7) / 8;
  a->tiles_y = (a->H + 15) / 16;
  const long long tiles = static_cast<long long>(a->B) * a->tiles_x * a->tiles_y;
  if (tiles > (1LL << 30)) return false;
  a->tiles = static_cast<int>(tiles);
  a->fd_per = FastDiv(static_cast<uint32_t>(a->tiles_x * a->tiles_y));
  a->fd_tx = FastDiv(static_cast<uint32_t>(a->tiles_x));
  return true;
}

cudaError_t init_i8_bottleneck_attributes() {
  cudaError_t e = set_attr<16, 16>();
  if (e == cudaSuccess) e = set_attr<16, 8>();
  if (e == cudaSuccess) e = set_attr<32, 32>();
  if (e == cudaSuccess) e = set_attr<32, 16>();
  return e;
}

cudaError_t launch_i8_bottleneck(const I8BottleneckArgs& a, cudaStream_t s, int num_sms) {
  if (!i8_bottleneck_supported(a.C, a.CM) || a.tiles != a.B * a.tiles_x * a.tiles_y)
    return cudaErrorInvalidValue;
  if (a.tiles <= 0) return cudaSuccess;
  const int grid = a.tiles < num_sms ? a.tiles : num_sms;
  if (a.C == 16) return a.CM == 16 ? launch_c<16, 16>(a, s, grid) : launch_c<16, 8>(a, s, grid);
  return a.CM == 32 ? launch_c<32, 32>(a, s, grid) : launch_c<32, 16>(a, s, grid);
}

}  // namespace yb
