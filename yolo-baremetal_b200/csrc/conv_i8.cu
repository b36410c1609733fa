// INT8 implicit-GEMM convolution for sm_100a: tcgen05.mma kind::i8 with
// int32 accumulation in tensor memory and the requantisation (bias, 64-bit
// fixed-point multiply, round-half-even shift, optional SiLU table) fused
// into the epilogue.  The reference has no INT8 path; the arithmetic is the
// scheme declared in yb_int8.h.
//
// GEMM view as in conv_tc.cu: M = B*Ho*Wo pixels (128 per tile), N = Co
// (tiles of up to 256), K = kh*kw*ci_pad ordered (ky, kx, ci) in 128-wide
// chunks, one 128-byte operand row per pixel and chunk.  One 32-wide K step
// is one UMMA.  Persistent CTA of 320 threads, one per SM:
//   warp 9     one thread: per chunk the packed weight chunk (bulk copy) and
//              one TMA im2col copy per filter tap of a_cpp channels (32, 64
//              or 128: 32B / 64B / 128B swizzled sub-tiles), all completing
//              on the stage's full barrier.
//   warp 16    TMEM (2-4 accumulators) and, from one lane, the UMMAs.
//   warps 0-15 four epilogue groups taking tiles round robin (as many as
//              there are accumulators), one warp per TMEM lane quarter:
//              tcgen05.ld, requantise, SiLU table, 16-byte int8 stores.
// Every barrier wait is bounded; a timeout sets the error word, stops the
// other roles, drains the tensor core and frees tensor memory.
#include <cudaTypedefs.h>

#include <cfloat>
#include <climits>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "pdl.cuh"
#include "runtime.h"
#include "sm100.cuh"
#include "status.h"
#include "i8_requant.cuh"
#include "int8.h"
#include "yb_int8.h"

namespace yb {
namespace {

constexpr int kBM = 128;
constexpr int kKB = 128;                      // K values (= bytes) per chunk
constexpr uint32_t kATile = kBM * 128;        // activation tile of one chunk
constexpr int kEpiGroups = 3;                 // epilogue groups of 4 warps
constexpr int kMmaWarp = 4 * kEpiGroups, kProdWarp = kMmaWarp + 1;
constexpr int kThreads = 32 * (kProdWarp + 1);
constexpr int kSmemLimit = 232448;
constexpr int kMaxAcc = 4;
constexpr int kMaxCo = 1024;
// Patch mode: one 16-channel plane of a tile's 18 x 10 input patch (16 bytes
// per pixel, pixel-major), padded to a 128-byte multiple.
constexpr int kPatchH = 18, kPatchW = 10;
constexpr uint32_t kPatchBox = kPatchH * kPatchW * 16;  // 2880 bytes written by one box copy
constexpr uint32_t kPatchChunk = 2944;
__host__ __device__ constexpr uint32_t patch_stage_bytes_i8(int ci_pad) {
  return ((static_cast<uint32_t>(ci_pad / 16) * kPatchChunk) + 1023u) & ~1023u;
}
// Stride-2 patch mode: a tile of 16 x 8 output pixels reads input rows
// 2 oy0 - 1 .. 2 oy0 + 31 (33) and columns 2 ox0 - 1 .. 2 ox0 + 15.  Per
// 16-channel chunk two boxes with a column traversal stride of 2 (box 18
// columns -> 9 pixels): plane O holds columns 2 ox0 - 1 + 2i (taps kx = 0 at
// i = c, kx = 2 at i = c + 1), plane E columns 2 ox0 + 2i (kx = 1 at i = c),
// so every tap window is 8 consecutive 16-byte pixels per output row and
// the next output row is two input rows (288 bytes) further.
constexpr int kP2Rows = 33, kP2Cols = 9;
constexpr uint32_t kP2Row = kP2Cols * 16;                 // 144 bytes per plane row
constexpr uint32_t kP2Box = kP2Rows * kP2Row;             // 4752 bytes written by one box copy
constexpr uint32_t kP2Plane = 4864;                       // plane stride (128-byte multiple)
constexpr uint32_t kP2Chunk = 2 * kP2Plane;               // O and E planes of one 16-channel chunk
__host__ __device__ constexpr uint32_t patch2_stage_bytes_i8(int ci_pad) {
  return ((static_cast<uint32_t>(ci_pad / 16) * kP2Chunk) + 1023u) & ~1023u;
}
// Window of tap t (ky = t / 3, kx = t % 3) from the chunk origin.
__host__ __device__ constexpr uint32_t p2_window(int t) {
  return ((t % 3) == 1 ? kP2Plane : 0u) + static_cast<uint32_t>(t / 3) * kP2Row + ((t % 3) == 2 ? 16u : 0u);
}
// K order of the taps for 16 channels (two taps per 32-byte K step): pairs
// with the second window above the first (the descriptor's LBO is unsigned).
__host__ __device__ constexpr int p2_tap(int pos) {
  return pos == 3 ? 4 : pos == 4 ? 3 : pos == 5 ? 7 : pos == 6 ? 5 : pos == 7 ? 6 : pos;
}

// UMMA issue of one patch-mode tile, fully unrolled: each descriptor is a
// compile-time offset (start address, and for paired taps the LBO field)
// from a base descriptor built once per tile, so the issuing thread emits
// little besides the tcgen05.mma instructions (issue-bound otherwise: about
// 45 cycles per UMMA back to back on B200 against about 150 with per-step
// descriptor arithmetic in a rolled loop).
// P2: stride-2 patch (windows p2_window); PAIR: 16 padded channels, two taps
// per 32-byte K step (second core matrix = the next tap's window via LBO);
// else C2 32-channel K steps per tap.  base: descriptor of the patch origin
// with LBO 0 (PAIR) or LBO = the chunk pair stride (C2 steps).
template <bool P2, bool PAIR, int C2>
__device__ __forceinline__ void i8_patch_tile_mma(uint32_t d, uint64_t base, uint64_t db0, uint64_t chunk_units,
                                                  uint32_t idesc) {
  if (PAIR) {
#pragma unroll
    for (int s2 = 0; s2 < 5; ++s2) {
      const int t0 = P2 ? p2_tap(2 * s2) : 2 * s2;
      const int t1 = 2 * s2 + 1 < 9 ? (P2 ? p2_tap(2 * s2 + 1) : 2 * s2 + 1) : t0;
      const uint32_t o0 = P2 ? p2_window(t0) : static_cast<uint32_t>(((t0 / 3) * kPatchW + t0 % 3) * 16);
      const uint32_t o1 = P2 ? p2_window(t1) : static_cast<uint32_t>(((t1 / 3) * kPatchW + t1 % 3) * 16);
      const uint32_t lbo = t1 == t0 ? 16u : o1 - o0;
      const uint64_t off = static_cast<uint64_t>(o0 >> 4) | (static_cast<uint64_t>(lbo >> 4) << 16);
      const int k = 32 * s2;
      const uint64_t boff = static_cast<uint64_t>(k / kKB) * chunk_units + static_cast<uint64_t>(((k % kKB) / 32) * 2);
      tc_mma_i8(d, base + off, db0 + boff, idesc, s2 != 0 ? 1u : 0u);
    }
  } else {
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
#pragma unroll
      for (int c2 = 0; c2 < C2; ++c2) {
        const int step = tap * C2 + c2;
        const uint64_t aoff =
            P2 ? static_cast<uint64_t>((2u * c2 * kP2Chunk + p2_window(tap)) >> 4)
               : static_cast<uint64_t>((tap / 3) * kPatchW + tap % 3 + c2 * (2 * kPatchChunk / 16));
        const int k = tap * 32 * C2 + 32 * c2;
        const uint64_t boff = static_cast<uint64_t>(k / kKB) * chunk_units + static_cast<uint64_t>(((k % kKB) / 32) * 2);
        tc_mma_i8(d, base + aoff, db0 + boff, idesc, step != 0 ? 1u : 0u);
      }
    }
  }
}

}  // namespace

namespace {


__device__ __forceinline__ void raise_err(int* err, volatile int* abort_flag, int code) {
  *abort_flag = 1;
  if (err) atomicCAS(err, 0, code);
}

// EPI: the epilogue, fixed per launch so that each instantiation carries one
// compact loop: bit 1 the SiLU table, bit 0 the residual, 4 = dequantised
// fp32 output (the Detect head's last convolutions).
template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) conv_i8_kernel(const __grid_constant__ I8Args a, const int stages) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t chunk_bytes = static_cast<uint32_t>(a.n_tile) * 128u;
  // Patch mode keeps every weight chunk resident in front of the stages.
  const bool patch = a.patch != 0;
  const bool patch2 = a.patch == 2;
  const int ci_pad = a.K / (a.kh * a.kw);
  const uint32_t wres_bytes = patch ? static_cast<uint32_t>(a.num_kc) * chunk_bytes : 0u;
  const uint32_t stage_bytes = patch2  ? patch2_stage_bytes_i8(ci_pad)
                               : patch ? patch_stage_bytes_i8(ci_pad)
                                       : kATile + chunk_bytes;
  uint8_t* stage0 = smem + wres_bytes;

  // Stride-2 patch mode leaves one plane of slack after the last stage.
  uint8_t* tail = stage0 + stages * stage_bytes + (patch2 ? kP2Plane : 0u);
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;
  uint64_t* acc_empty = acc_full + kMaxAcc;
  uint64_t* drain = acc_empty + kMaxAcc;
  uint64_t* wbar = drain + 1;  // resident weights landed (patch mode)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wbar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Per output channel sq = {multiplier M, low and high word of
  // D = bias * M + 2^(shift-1) - 1, shift - 32} and sb = bias; a zero
  // multiplier gets shift 32 (its result is 0 under any shift).  With
  // shift >= 32 for every channel (fast), y = (acc * M + D) >> shift is the
  // rounded result except at exact ties, which requant16_fast detects.
  const int nq = a.n_tile * a.n_tiles;
  int4* sq = reinterpret_cast<int4*>(tail + 512);
  int32_t* sb = reinterpret_cast<int32_t*>(sq + nq);
  int32_t* srtab = sb + nq;
  int8_t* slut = reinterpret_cast<int8_t*>(srtab + 256);
  int fast_ok = 1;
  for (int i = threadIdx.x; i < nq; i += kThreads) {
    const bool ok = i < a.Co;
    const int b = ok ? a.bias[i] : 0;
    const int m = ok ? a.mult[i] : 0;
    const int sh = m == 0 ? 32 : a.shift[i];
    if (sh < 32) fast_ok = 0;
    const long long d = static_cast<long long>(b) * m + ((1LL << (sh - 1)) - 1);
    sq[i] = make_int4(m, static_cast<int>(static_cast<unsigned long long>(d) & 0xFFFFFFFFull),
                      static_cast<int>(d >> 32), sh - 32);
    sb[i] = b;
  }
  // Residual term rshift_rne(r * res_mult, res_shift) of every int8 r (the
  // fast path needs it below 2^29 in magnitude).
  if (a.res && ((128LL * a.res_mult) >> a.res_shift) >= (1LL << 29)) fast_ok = 0;
  for (int i = threadIdx.x; i < 256; i += kThreads) {
    slut[i] = a.lut ? a.lut[i] : 0;
    srtab[i] = a.res ? static_cast<int32_t>(rshift_rne(static_cast<long long>(i - 128) * a.res_mult, a.res_shift)) : 0;
  }

  uint32_t acc_stride = 32;
  while (acc_stride < static_cast<uint32_t>(a.n_tile)) acc_stride <<= 1;
  const int nacc = min(kMaxAcc, static_cast<int>(512u / acc_stride));
  const uint32_t ncols = static_cast<uint32_t>(nacc) * acc_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < nacc; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(drain, 1);
    mbar_init(wbar, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  const bool fast = __syncthreads_and(fast_ok) != 0;
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) pdl_trigger();
  pdl_wait();

  const int total_tiles = a.m_tiles * a.n_tiles;
  const int ks_last = (a.K - (a.num_kc - 1) * kKB + 31) / 32;
  const int HoWo = a.Ho * a.Wo;
  const int M = a.B * HoWo;

  if (warp == kProdWarp && patch) {
    // ------------------------------------------------------ patch producer
    // One thread: the resident weights once, then per tile one box copy per
    // 16-channel plane of its 18 x 10 input patch (zero outside the image
    // and past the view's channels).
    if (lane == 0) {
      prefetch_tmap(&a.tm);
      mbar_arrive_expect_tx(wbar, wres_bytes);
      for (int kc = 0; kc < a.num_kc; ++kc)
        bulk_g2s(smem + static_cast<size_t>(kc) * chunk_bytes, a.wpack + static_cast<size_t>(kc) * chunk_bytes,
                 chunk_bytes, wbar);
      const int ncb = ci_pad / 16;
      const int per = a.tiles_y * a.tiles_x;
      uint32_t it = 0;
      for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++it) {
        const uint32_t itq = a.fd_stages.div(it);
        const uint32_t s = it - itq * static_cast<uint32_t>(stages);
        const uint32_t ph = itq & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) {
          raise_err(a.err, abort_flag, kErrWaitEmpty);
          break;
        }
        const int b = static_cast<int>(a.fd_per.div(static_cast<uint32_t>(t)));
        const int rem = t - b * per;
        const int ty = static_cast<int>(a.fd_tx.div(static_cast<uint32_t>(rem)));
        const int tx = rem - ty * a.tiles_x;
        uint8_t* stage = stage0 + s * stage_bytes;
        if (patch2) {
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(ncb) * 2u * kP2Box);
          for (int cb = 0; cb < ncb; ++cb) {
            tma_tile_4d(stage + cb * kP2Chunk, &a.tm, 16 * cb, tx * 16 - 1, ty * 32 - 1, b, &full[s]);
            tma_tile_4d(stage + cb * kP2Chunk + kP2Plane, &a.tm, 16 * cb, tx * 16, ty * 32 - 1, b, &full[s]);
          }
          continue;
        }
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(ncb) * kPatchBox);
        for (int cb = 0; cb < ncb; ++cb)
          tma_tile_4d(stage + cb * kPatchChunk, &a.tm, 16 * cb, tx * 8 - 1, ty * 16 - 1, b, &full[s]);
      }
    }
  } else if (warp == kProdWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&a.tm);
      const int taps = a.kh * a.kw;
      const int cpp = a.a_cpp;
      const int tps = cpp == 128 ? 1 : 128 / cpp;
      const int cblocks = cpp == 128 ? (taps == 1 ? a.num_kc : a.Ci / 128) : 1;
      const uint32_t sub_bytes = static_cast<uint32_t>(kBM * cpp);
      uint32_t it = 0;
      for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
        const int mt = static_cast<int>(a.fd_ntiles.div(static_cast<uint32_t>(t)));
        const int nt = t - mt * a.n_tiles;
        const int m0 = mt * kBM;
        const int b = static_cast<int>(a.fd_howo.div(static_cast<uint32_t>(m0)));
        const int r = m0 - b * HoWo;
        const int oy = static_cast<int>(a.fd_wo.div(static_cast<uint32_t>(r)));
        const int ox = r - oy * a.Wo;
        const int w0 = ox * a.stride - a.pad, h0 = oy * a.stride - a.pad;
        const uint8_t* wsrc = a.wpack + static_cast<size_t>(nt) * a.num_kc * chunk_bytes;
        for (int kc = 0; kc < a.num_kc; ++kc, ++it) {
          const uint32_t itq = a.fd_stages.div(it);
          const uint32_t s = it - itq * static_cast<uint32_t>(stages);
          const uint32_t ph = itq & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) {
            raise_err(a.err, abort_flag, kErrWaitEmpty);
            goto producer_done;
          }
          const int t0 = cpp == 128 ? kc / cblocks : kc * tps;
          const int c0 = cpp == 128 ? (kc - t0 * cblocks) * 128 : 0;
          const int ntap = cpp == 128 ? 1 : min(tps, taps - t0);
          uint8_t* stage = stage0 + s * stage_bytes;
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(ntap) * sub_bytes + chunk_bytes);
          bulk_g2s(stage + kATile, wsrc + static_cast<size_t>(kc) * chunk_bytes, chunk_bytes, &full[s]);
          for (int i = 0; i < ntap; ++i) {
            const int tap = t0 + i;
            const int ky = tap / a.kw;
            const int kx = tap - ky * a.kw;
            tma_im2col_4d(stage + i * sub_bytes, &a.tm, c0, w0, h0, b, static_cast<uint16_t>(kx),
                          static_cast<uint16_t>(ky), &full[s]);
          }
        }
      }
    }
  producer_done:;
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_s8_s32(kBM, a.n_tile);
      const int cpp = a.a_cpp;
      const uint32_t layout = cpp == 32 ? 6u : cpp == 64 ? 4u : 2u;
      const uint32_t sbo = cpp == 32 ? 256u : cpp == 64 ? 512u : 1024u;
      uint32_t it = 0;
      int lt = 0;
      for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++lt) {
        const int lq = nacc == 4 ? lt >> 2 : nacc == 2 ? lt >> 1 : nacc == 3 ? lt / 3 : lt;
        const int acc = lt - lq * nacc;
        const uint32_t aph = lq & 1;
        if (!mbar_wait(&acc_empty[acc], aph ^ 1u, abort_flag)) {
          raise_err(a.err, abort_flag, kErrWaitAccEmpty);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * acc_stride;
        bool ok = true;
        if (patch) {
          // One stage per tile: 9 taps x ci_pad / 32 K steps, each A operand
          // a shifted window of the patch (two 16-channel planes), each B step
          // in the resident weights.
          if (lt == 0 && !mbar_wait(wbar, 0, abort_flag)) {
            raise_err(a.err, abort_flag, kErrWaitFull);
            break;
          }
          const uint32_t itq = a.fd_stages.div(it);
          const uint32_t s = it - itq * static_cast<uint32_t>(stages);
          const uint32_t ph = itq & 1u;
          ++it;
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            raise_err(a.err, abort_flag, kErrWaitFull);
            break;
          }
          tc_fence_after();
          // Descriptors at the patch origin and at weight chunk 0; every
          // step adds a start-address offset (16-byte units).
          const uint64_t da0 = kmajor_desc_noswizzle(smem_u32(stage0 + s * stage_bytes), kPatchChunk, kPatchW * 16);
          const uint64_t db0 = sw128_kmajor_desc(smem_u32(smem));
          const uint64_t chunk_units = chunk_bytes >> 4;
          if (patch2) {
            // Stride 2: output row stride 2 input rows (SBO 288 bytes).
            const uint32_t pa = smem_u32(stage0 + s * stage_bytes);
            if (ci_pad == 16) {
              // Two taps per K step in the K order p2_tap (second window
              // above the first); tap 8 pairs with zero weights.
              i8_patch_tile_mma<true, true, 1>(d_tmem, kmajor_desc_noswizzle(pa, 0, 2 * kP2Row), db0, chunk_units,
                                               idesc);
            } else if (ci_pad == 32 || ci_pad == 64) {
              const uint64_t base = kmajor_desc_noswizzle(pa, kP2Chunk, 2 * kP2Row);
              if (ci_pad == 32) i8_patch_tile_mma<true, false, 1>(d_tmem, base, db0, chunk_units, idesc);
              else i8_patch_tile_mma<true, false, 2>(d_tmem, base, db0, chunk_units, idesc);
            } else if (false) {
              for (int s2 = 0; s2 < 5; ++s2) {
                const int t0 = p2_tap(2 * s2), t1 = 2 * s2 + 1 < 9 ? p2_tap(2 * s2 + 1) : t0;
                const uint32_t o0 = p2_window(t0), o1 = p2_window(t1);
                const uint64_t da = kmajor_desc_noswizzle(pa + o0, t1 == t0 ? 16u : o1 - o0, 2 * kP2Row);
                const int k = 32 * s2;
                const uint64_t boff =
                    static_cast<uint64_t>(k / kKB) * chunk_units + static_cast<uint64_t>(((k % kKB) / 32) * 2);
                tc_mma_i8(d_tmem, da, db0 + boff, idesc, s2 != 0 ? 1u : 0u);
              }
            } else {
              // Per tap, 32 channels per K step: the chunks 2 c2 and 2 c2 + 1.
              int step = 0;
              for (int tap = 0; tap < 9; ++tap) {
                for (int c2 = 0; c2 < ci_pad / 32; ++c2, ++step) {
                  const uint64_t da =
                      kmajor_desc_noswizzle(pa + 2u * static_cast<uint32_t>(c2) * kP2Chunk + p2_window(tap), kP2Chunk,
                                            2 * kP2Row);
                  const int k = tap * ci_pad + 32 * c2;
                  const uint64_t boff =
                      static_cast<uint64_t>(k / kKB) * chunk_units + static_cast<uint64_t>(((k % kKB) / 32) * 2);
                  tc_mma_i8(d_tmem, da, db0 + boff, idesc, step != 0 ? 1u : 0u);
                }
              }
            }
            tc_commit(&empty[s]);
            tc_commit(&acc_full[acc]);
            continue;
          }
          if (ci_pad == 16) {
            // At most 16 input channels: two taps per 32-byte K step.  The A
            // operand's second core matrix is the next tap's window (LBO =
            // the distance between the two windows); the weights hold the
            // two taps' 16 channels back to back (K ordered (tap, channel),
            // 16 channels per tap).  Tap 8 pairs with zero weights.
            const uint32_t pa = smem_u32(stage0 + s * stage_bytes);
            i8_patch_tile_mma<false, true, 1>(d_tmem, kmajor_desc_noswizzle(pa, 0, kPatchW * 16), db0, chunk_units,
                                              idesc);
            tc_commit(&empty[s]);
            tc_commit(&acc_full[acc]);
            continue;
          }
          if (ci_pad == 32 || ci_pad == 64) {
            if (ci_pad == 32) i8_patch_tile_mma<false, false, 1>(d_tmem, da0, db0, chunk_units, idesc);
            else i8_patch_tile_mma<false, false, 2>(d_tmem, da0, db0, chunk_units, idesc);
            tc_commit(&empty[s]);
            tc_commit(&acc_full[acc]);
            continue;
          }
          int step = 0;
          for (int tap = 0; tap < 9; ++tap) {
            const uint64_t toff = static_cast<uint64_t>((tap / 3) * kPatchW + tap % 3);  // window shift
            for (int c2 = 0; c2 < ci_pad / 32; ++c2, ++step) {
              const int k = tap * ci_pad + 32 * c2;
              const uint64_t aoff = toff + static_cast<uint64_t>(c2) * (2 * kPatchChunk / 16);
              const uint64_t boff = static_cast<uint64_t>(k / kKB) * chunk_units + static_cast<uint64_t>(((k % kKB) / 32) * 2);
              tc_mma_i8(d_tmem, da0 + aoff, db0 + boff, idesc, step != 0 ? 1u : 0u);
            }
          }
          tc_commit(&empty[s]);
          tc_commit(&acc_full[acc]);
          continue;
        }
        for (int kc = 0; kc < a.num_kc; ++kc, ++it) {
          const uint32_t itq = a.fd_stages.div(it);
          const uint32_t s = it - itq * static_cast<uint32_t>(stages);
          const uint32_t ph = itq & 1u;
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            raise_err(a.err, abort_flag, kErrWaitFull);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(stage0 + s * stage_bytes);
          const uint64_t da0 = kmajor_desc(sa, layout, sbo);
          const uint64_t db0 = sw128_kmajor_desc(sa + kATile);
          const int nks = kc == a.num_kc - 1 ? ks_last : kKB / 32;
#pragma unroll
          for (int ks = 0; ks < kKB / 32; ++ks) {
            if (ks >= nks) break;
            // 16-byte units: a 32-wide K step is one 32B sub-tile, half a 64B
            // row, or a quarter of a 128B row.
            const uint64_t aoff = cpp == 32   ? static_cast<uint64_t>(ks * 256)
                                  : cpp == 64 ? static_cast<uint64_t>((ks >> 1) * 512 + (ks & 1) * 2)
                                              : static_cast<uint64_t>(ks * 2);
            tc_mma_i8(d_tmem, da0 + aoff, db0 + static_cast<uint64_t>(ks * 2), idesc, (kc | ks) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[acc]);
      }
      tc_commit(drain);
      bool drained = mbar_try_wait(drain, 0);
      const uint64_t t0 = globaltimer_ns();
      while (!drained && globaltimer_ns() - t0 < kWaitNs) drained = mbar_try_wait(drain, 0);
      if (!drained) raise_err(a.err, abort_flag, kErrDrain);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    // Groups take tiles round robin; each owns one accumulator, so only
    // min(kEpiGroups, nacc) groups work.
    const int grp = warp >> 2;
    const int ngrp = min(kEpiGroups, nacc);
    // 32-byte stores of whole 32-channel runs when every run is aligned.
    const bool v8out = EPI != 4 && (reinterpret_cast<uintptr_t>(a.out) & 31) == 0 && (a.out_cstride & 31) == 0 &&
                       (a.out_coff & 31) == 0 && (a.n_tile & 31) == 0;
    for (int t = blockIdx.x + grp * gridDim.x, lt = grp; grp < ngrp && t < total_tiles;
         t += ngrp * gridDim.x, lt += ngrp) {
      const int lq = nacc == 4 ? lt >> 2 : nacc == 2 ? lt >> 1 : nacc == 3 ? lt / 3 : lt;
      const int acc = lt - lq * nacc;
      const uint32_t aph = lq & 1;
      if (!mbar_wait(&acc_full[acc], aph, abort_flag)) {
        raise_err(a.err, abort_flag, kErrWaitAccFull);
        break;
      }
      tc_fence_after();
      const int mt = static_cast<int>(a.fd_ntiles.div(static_cast<uint32_t>(t)));
      const int nt = t - mt * a.n_tiles;
      const int n0 = nt * a.n_tile;
      const int nvalid = min(a.n_tile, a.Co - n0);
      bool valid;
      long long pm = 0;
      if (patch) {
        // Tile of 16 rows x 8 columns; TMEM lane r is pixel (r / 8, r % 8).
        const int per = a.tiles_y * a.tiles_x;
        const int tb = static_cast<int>(a.fd_per.div(static_cast<uint32_t>(mt)));
        const int rem = mt - tb * per;
        const int ty = static_cast<int>(a.fd_tx.div(static_cast<uint32_t>(rem)));
        const int r = q * 32 + lane;
        const int oy = ty * 16 + (r >> 3), ox = (rem - ty * a.tiles_x) * 8 + (r & 7);
        valid = oy < a.Ho && ox < a.Wo;
        if (valid) pm = static_cast<long long>(tb) * HoWo + oy * a.Wo + ox;
      } else {
        const int m = mt * kBM + q * 32 + lane;
        valid = m < M;
        if (valid) pm = m;
      }
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * acc_stride;
      const long long po = pm * a.out_cstride + a.out_coff + n0;
      // Units of 32 channels: two TMEM loads, requantise (or dequantise),
      // then lanes 2k and 2k+1 write the two 16-byte halves of one pixel's
      // 32-byte run.
      float rmax = -FLT_MAX;  // dequantised output with a row maximum
      for (int c = 0; c < nvalid; c += 32) {
        const bool two = c + 16 < nvalid;
        if (EPI == 4) {
          uint32_t r[32];
          uint32_t(&r0)[16] = *reinterpret_cast<uint32_t(*)[16]>(&r[0]);
          uint32_t(&r1)[16] = *reinterpret_cast<uint32_t(*)[16]>(&r[16]);
          tc_ld_32x32b_x16(tbase + c, r0);
          if (two) tc_ld_32x32b_x16(tbase + c + 16, r1);
          tc_wait_ld();
          if (valid) {
            const long long fb = pm / HoWo;
            float* of = a.out_f32 + fb * a.f32_bstride + (pm - fb * HoWo) * a.f32_cstride + n0 + c;
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              if (n0 + c + e >= a.f32_co) break;
              float4 v;
              v.x = static_cast<float>(static_cast<long long>(static_cast<int32_t>(r[e])) + sb[n0 + c + e]) *
                    a.deq[n0 + c + e];
              v.y = static_cast<float>(static_cast<long long>(static_cast<int32_t>(r[e + 1])) +
                                       sb[n0 + c + e + 1]) *
                    a.deq[n0 + c + e + 1];
              v.z = static_cast<float>(static_cast<long long>(static_cast<int32_t>(r[e + 2])) +
                                       sb[n0 + c + e + 2]) *
                    a.deq[n0 + c + e + 2];
              v.w = static_cast<float>(static_cast<long long>(static_cast<int32_t>(r[e + 3])) +
                                       sb[n0 + c + e + 3]) *
                    a.deq[n0 + c + e + 3];
              *reinterpret_cast<float4*>(of + e) = v;
              if (a.rowmax) rmax = fmaxf(fmaxf(rmax, fmaxf(v.x, v.y)), fmaxf(v.z, v.w));
            }
          }
          continue;
        }
        uint4 rvv[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
        if (EPI & 1) {
          const int8_t* rp = a.res + pm * a.res_cstride + a.res_coff + n0 + c;
          rvv[0] = *reinterpret_cast<const uint4*>(rp);
          if (two) rvv[1] = *reinterpret_cast<const uint4*>(rp + 16);
        }
        uint32_t p0[4] = {0u, 0u, 0u, 0u}, p1[4] = {0u, 0u, 0u, 0u};
        constexpr int mode = EPI & 3;
        // Two halves of 16 channels: both TMEM loads in flight together, one wait.
        uint32_t ra[16], rb[16];
        tc_ld_32x32b_x16(tbase + c, ra);
        if (two) tc_ld_32x32b_x16(tbase + c + 16, rb);
        tc_wait_ld();
        tc_ld_dep(ra);
        if (two) tc_ld_dep(rb);
        auto half = [&](int hh, uint32_t(&r)[16], uint32_t(&pk)[4]) {
          const int4* qc = sq + n0 + c + 16 * hh;
          const uint4 rh = rvv[hh];
          const int32_t* sbh = sb + n0 + c + 16 * hh;
          bool exact = !fast;
          if (fast) {
            switch (mode) {
              case 0: exact = requant16_fast<false, false>(r, rh, qc, slut, srtab, pk); break;
              case 1: exact = requant16_fast<false, true>(r, rh, qc, slut, srtab, pk); break;
              case 2: exact = requant16_fast<true, false>(r, rh, qc, slut, srtab, pk); break;
              default: exact = requant16_fast<true, true>(r, rh, qc, slut, srtab, pk); break;
            }
          }
          // Warp-uniform: the exact path reloads the accumulators.
          if (__any_sync(0xffffffffu, exact)) {
            const uint32_t ta = tbase + c + 16 * hh;
            uint4 w;
            switch (mode) {
              case 0: w = requant16_exact<false, false>(ta, rh, qc, sbh, slut, srtab, a.res_mult, a.res_shift); break;
              case 1: w = requant16_exact<false, true>(ta, rh, qc, sbh, slut, srtab, a.res_mult, a.res_shift); break;
              case 2: w = requant16_exact<true, false>(ta, rh, qc, sbh, slut, srtab, a.res_mult, a.res_shift); break;
              default: w = requant16_exact<true, true>(ta, rh, qc, sbh, slut, srtab, a.res_mult, a.res_shift); break;
            }
            pk[0] = w.x;
            pk[1] = w.y;
            pk[2] = w.z;
            pk[3] = w.w;
          }
        };
        half(0, ra, p0);
        if (two) half(1, rb, p1);
        if (v8out && two) {
          // The lane's pixel run of 32 channels in one 32-byte store.
          if (valid) {
            const uint32_t w8[8] = {p0[0], p0[1], p0[2], p0[3], p1[0], p1[1], p1[2], p1[3]};
            st_global_v8(a.out + po + c, w8);
          }
          continue;
        }
        const int h = lane & 1;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int src = (lane >> 1) + 16 * i;
          uint32_t w[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t lo = __shfl_sync(0xffffffffu, p0[j], src);
            const uint32_t hi = __shfl_sync(0xffffffffu, p1[j], src);
            w[j] = h ? hi : lo;
          }
          const long long spo = __shfl_sync(0xffffffffu, po, src);
          const bool svalid = __shfl_sync(0xffffffffu, valid, src);
          if (svalid && (h == 0 || two))
            *reinterpret_cast<uint4*>(a.out + spo + c + 16 * h) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      // The same sigmoid as the decode kernel's (accurate expf, IEEE division).
      if (EPI == 4 && a.rowmax && valid) {
        const long long fb = pm / HoWo;
        a.rowmax[fb * a.rm_bstride + (pm - fb * HoWo)] = 1.0f / (1.0f + expf(-rmax));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }

  if (*abort_flag) __nanosleep(100000);
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, ncols);
  }
}

// ------------------------------------------------------------------- host
PFN_cuTensorMapEncodeIm2col_v12000 i8_im2col_encoder() {
  static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(p);
  });
  return fn;
}

PFN_cuTensorMapEncodeTiled_v12000 i8_tiled_encoder() {
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

inline uint32_t sw128_off(uint32_t row, uint32_t chunk16) {
  return (row >> 3) * 1024u + (row & 7u) * 128u + ((chunk16 ^ (row & 7u)) << 4);
}

int stages_for_i8(int n_tile, int n_tiles) {
  const int stage = static_cast<int>(kATile) + n_tile * 128;
  const int extra = 1024 + 512 + 20 * n_tile * n_tiles + 1024 + 256;
  const int st = (kSmemLimit - extra) / stage;
  return st > 8 ? 8 : st;
}


}  // namespace

void i8_tiling_pair(int co, I8Tiling* t) {
  i8_tiling(co, 16, 3, 3, t);
  t->ci_pad = 16;
  t->a_cpp = 16;
  t->K = 9 * 16;
  t->num_kc = (t->K + kKB - 1) / kKB;
}

void i8_tiling_pair_s2(int co, I8Tiling* t) {
  i8_tiling_pair(co, t);
  t->tap_perm = 1;
}

void i8_tiling(int co, int ci, int kh, int kw, I8Tiling* t) {
  const int taps = kh * kw;
  if (taps == 1) {
    // 32 or 64 padded channels: boxes of exactly that width (the TMA
    // engine's smem writes, zero fill included, bound these convolutions).
    t->ci_pad = (ci + 31) / 32 * 32;
    t->a_cpp = t->ci_pad == 32 || t->ci_pad == 64 ? t->ci_pad : 128;
  } else {
    t->ci_pad = ci <= 32 ? 32 : ci <= 64 ? 64 : (ci + 127) / 128 * 128;
    t->a_cpp = t->ci_pad <= 64 ? t->ci_pad : 128;
  }
  t->K = taps * t->ci_pad;
  t->num_kc = (t->K + kKB - 1) / kKB;
  const int tiles = (co + 255) / 256;
  const int per = (co + tiles - 1) / tiles;
  t->n_tile = (per + 15) / 16 * 16;
  t->n_tiles = tiles;
}

std::vector<uint8_t> i8_pack_weights(const int8_t* wq, int co, int ci, int kh, int kw, const I8Tiling& t) {
  const size_t chunk = static_cast<size_t>(t.n_tile) * 128;
  std::vector<uint8_t> pk(static_cast<size_t>(t.n_tiles) * t.num_kc * chunk, 0);
  for (int nt = 0; nt < t.n_tiles; ++nt)
    for (int kc = 0; kc < t.num_kc; ++kc) {
      uint8_t* dst = pk.data() + (static_cast<size_t>(nt) * t.num_kc + kc) * chunk;
      for (int rrow = 0; rrow < t.n_tile; ++rrow) {
        const int n = nt * t.n_tile + rrow;
        if (n >= co) continue;
        for (int kk = 0; kk < kKB; ++kk) {
          const int k = kc * kKB + kk;
          if (k >= t.K) break;
          const int pos = k / t.ci_pad;
          const int tap = t.tap_perm ? p2_tap(pos) : pos;
          const int cc = k - pos * t.ci_pad;
          if (cc >= ci) continue;
          const int ky = tap / kw, kx = tap - (tap / kw) * kw;
          const int8_t v = wq[((static_cast<size_t>(n) * ci + cc) * kh + ky) * kw + kx];
          dst[sw128_off(static_cast<uint32_t>(rrow), static_cast<uint32_t>(kk >> 4)) + (kk & 15)] =
              static_cast<uint8_t>(v);
        }
      }
    }
  return pk;
}

int i8_bias_slots(const I8Tiling& t) { return t.n_tile * t.n_tiles; }

cudaError_t i8_init_kernel() {
  cudaError_t e = cudaSuccess;
  for (auto k : {conv_i8_kernel<0>, conv_i8_kernel<1>, conv_i8_kernel<2>, conv_i8_kernel<3>, conv_i8_kernel<4>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  return e == cudaSuccess ? init_i8_bottleneck_attributes() : e;
}

namespace {
// The kernel instantiation for the launch's epilogue.
using I8ConvKernel = void (*)(I8Args, int);
I8ConvKernel i8_kernel_for(const I8Args& a) {
  if (a.out_f32) return conv_i8_kernel<4>;
  switch ((a.lut ? 2 : 0) | (a.res ? 1 : 0)) {
    case 0: return conv_i8_kernel<0>;
    case 1: return conv_i8_kernel<1>;
    case 2: return conv_i8_kernel<2>;
    default: return conv_i8_kernel<3>;
  }
}

void fill_fastdiv(I8Args& a, int stages) {
  a.fd_stages = FastDiv(static_cast<uint32_t>(stages));
  a.fd_ntiles = FastDiv(static_cast<uint32_t>(a.n_tiles));
  a.fd_howo = FastDiv(static_cast<uint32_t>(a.Ho * a.Wo));
  a.fd_wo = FastDiv(static_cast<uint32_t>(a.Wo));
  a.fd_per = FastDiv(static_cast<uint32_t>(a.tiles_y > 0 && a.tiles_x > 0 ? a.tiles_y * a.tiles_x : 1));
  a.fd_tx = FastDiv(static_cast<uint32_t>(a.tiles_x > 0 ? a.tiles_x : 1));
}
}  // namespace

cudaError_t launch_conv_i8(I8Args& a, const int8_t* x, long long x_cstride, long long x_bstride, cudaStream_t s,
                           int sms, std::string* why) {
  if (a.Co < 16 || a.Co % 16 || a.n_tile < 16 || a.n_tile % 16 || a.n_tiles < 1 || a.n_tile * a.n_tiles < a.Co ||
      (a.out && (a.out_cstride % 16 || a.out_coff % 16)) || (a.res && (a.res_cstride % 16 || a.res_coff % 16)) ||
      (!a.out && !a.out_f32) || (a.out_f32 && (a.f32_cstride % 4 || a.f32_bstride % 4 || a.f32_co % 4 || !a.deq)) ||
      (a.rowmax && (!a.out_f32 || a.n_tiles != 1)) ||
      a.res_shift < 1 ||
      a.res_shift > 62 || x_cstride % 16 || x_bstride % 16 || reinterpret_cast<uintptr_t>(x) % 16) {
    if (why) *why = "int8 conv: unsupported view alignment or tile";
    return cudaErrorInvalidValue;
  }
  const int tail = 512 + 20 * a.n_tile * a.n_tiles + 1024 + 256;
  const int ci_pad = a.K / (a.kh * a.kw);
  // Patch mode: 3x3 stride 1 pad 1, one N tile, 16 (two taps per K step),
  // 32 or 64 padded input channels, enough room for three stages next to
  // the resident weights.  16 padded channels exist only in patch mode.
  a.patch = 0;
  if (a.kh == 3 && a.kw == 3 && a.stride == 1 && a.pad == 1 && a.Ho == a.H && a.Wo == a.W && a.n_tiles == 1 &&
      (ci_pad == 16 || ci_pad == 32 || ci_pad == 64) && a.K == 9 * ci_pad && a.n_tile <= 128 && !a.tap_perm) {
    const int wres = a.num_kc * a.n_tile * 128;
    const int pst = static_cast<int>(patch_stage_bytes_i8(ci_pad));
    int st = (kSmemLimit - 1024 - wres - tail) / pst;
    st = st > 8 ? 8 : st;
    const auto tenc = i8_tiled_encoder();
    if (st >= 3 && tenc) {
      cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.Ci), static_cast<cuuint64_t>(a.W),
                            static_cast<cuuint64_t>(a.H), static_cast<cuuint64_t>(a.B)};
      cuuint64_t strides[3] = {static_cast<cuuint64_t>(x_cstride), static_cast<cuuint64_t>(x_cstride) * a.W,
                               static_cast<cuuint64_t>(x_bstride)};
      cuuint32_t box[4] = {16, kPatchW, kPatchH, 1};
      cuuint32_t estr[4] = {1, 1, 1, 1};
      const CUresult cr = tenc(&a.tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t*>(x), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (cr == CUDA_SUCCESS) {
        a.patch = 1;
        a.tiles_y = (a.Ho + 15) / 16;
        a.tiles_x = (a.Wo + 7) / 8;
        a.m_tiles = a.B * a.tiles_y * a.tiles_x;
        const int smem = 1024 + wres + st * pst + tail;
        if (a.m_tiles <= 0) return cudaSuccess;
        const int grid = a.m_tiles < sms ? a.m_tiles : sms;
        fill_fastdiv(a, st);
        return launch_pdl(i8_kernel_for(a), dim3(grid), dim3(kThreads), smem, s, a, st);
      }
    }
  }
  // Stride-2 patch mode: 3x3 stride 2 pad 1, one N tile, 16 (two taps per K
  // step, taps in the p2_tap order), 32 or 64 padded input channels.
  if (a.kh == 3 && a.kw == 3 && a.stride == 2 && a.pad == 1 && a.Ho == (a.H - 1) / 2 + 1 &&
      a.Wo == (a.W - 1) / 2 + 1 && a.n_tiles == 1 && (ci_pad == 16 || ci_pad == 32 || ci_pad == 64) &&
      a.K == 9 * ci_pad && a.n_tile <= 128 && (ci_pad != 16 || a.tap_perm)) {
    const int wres = a.num_kc * a.n_tile * 128;
    const int pst = static_cast<int>(patch2_stage_bytes_i8(ci_pad));
    int st = (kSmemLimit - 1024 - wres - static_cast<int>(kP2Plane) - tail) / pst;
    st = st > 8 ? 8 : st;
    const auto tenc = i8_tiled_encoder();
    if (st >= 3 && tenc) {
      cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.Ci), static_cast<cuuint64_t>(a.W),
                            static_cast<cuuint64_t>(a.H), static_cast<cuuint64_t>(a.B)};
      cuuint64_t strides[3] = {static_cast<cuuint64_t>(x_cstride), static_cast<cuuint64_t>(x_cstride) * a.W,
                               static_cast<cuuint64_t>(x_bstride)};
      // 18 columns traversed with stride 2: 9 pixels per box row.
      cuuint32_t box[4] = {16, 2 * kP2Cols, kP2Rows, 1};
      cuuint32_t estr[4] = {1, 2, 1, 1};
      const CUresult cr = tenc(&a.tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t*>(x), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (cr == CUDA_SUCCESS) {
        a.patch = 2;
        a.tiles_y = (a.Ho + 15) / 16;
        a.tiles_x = (a.Wo + 7) / 8;
        a.m_tiles = a.B * a.tiles_y * a.tiles_x;
        const int smem = 1024 + wres + st * pst + static_cast<int>(kP2Plane) + tail;
        if (a.m_tiles <= 0) return cudaSuccess;
        const int grid = a.m_tiles < sms ? a.m_tiles : sms;
        fill_fastdiv(a, st);
        return launch_pdl(i8_kernel_for(a), dim3(grid), dim3(kThreads), smem, s, a, st);
      }
    }
  }
  if (ci_pad == 16) {
    if (why) *why = "int8 conv: 16-channel K layout needs patch mode";
    return cudaErrorInvalidValue;
  }
  const auto enc = i8_im2col_encoder();
  if (!enc) {
    if (why) *why = "cuTensorMapEncodeIm2col unavailable";
    return cudaErrorNotSupported;
  }
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.Ci), static_cast<cuuint64_t>(a.W), static_cast<cuuint64_t>(a.H),
                        static_cast<cuuint64_t>(a.B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(x_cstride), static_cast<cuuint64_t>(x_cstride) * a.W,
                           static_cast<cuuint64_t>(x_bstride)};
  int lower[2] = {-a.pad, -a.pad};
  int upper[2] = {a.pad - (a.kw - 1), a.pad - (a.kh - 1)};
  cuuint32_t estr[4] = {1, static_cast<cuuint32_t>(a.stride), static_cast<cuuint32_t>(a.stride), 1};
  const CUtensorMapSwizzle sw = a.a_cpp == 32   ? CU_TENSOR_MAP_SWIZZLE_32B
                                : a.a_cpp == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                : CU_TENSOR_MAP_SWIZZLE_128B;
  const CUresult cr = enc(&a.tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t*>(x), dims, strides, lower,
                          upper, static_cast<cuuint32_t>(a.a_cpp), static_cast<cuuint32_t>(kBM), estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) {
    if (why) *why = "int8 conv: tensor map encoding failed (code " + std::to_string(static_cast<int>(cr)) + ")";
    return cudaErrorInvalidValue;
  }
  const int stages = stages_for_i8(a.n_tile, a.n_tiles);
  if (stages < 2) return cudaErrorInvalidValue;
  const int smem = 1024 + 512 + 20 * a.n_tile * a.n_tiles + 1024 + 256 +
                   stages * (static_cast<int>(kATile) + a.n_tile * 128);
  const int total = a.m_tiles * a.n_tiles;
  if (total <= 0) return cudaSuccess;
  const int grid = total < sms ? total : sms;
  fill_fastdiv(a, stages);
  return launch_pdl(i8_kernel_for(a), dim3(grid), dim3(kThreads), smem, s, a, stages);
}

namespace {
struct Int8Conv {
  int device = 0;
  int co = 0, ci = 0, ci_pad = 0, kh = 1, kw = 1, stride = 1, pad = 0;
  int n_tile = 0, n_tiles = 0, K = 0, num_kc = 0, a_cpp = 0;
  uint8_t* wpack = nullptr;
  int32_t* bias = nullptr;
  int32_t* mult = nullptr;
  int32_t* shift = nullptr;
  int8_t* lut = nullptr;
  int* err = nullptr;
  int sms = 148;
};

status_t free_conv(Int8Conv* c) {
  if (!c) return SUCCESS;
  cudaSetDevice(c->device);
  for (void* p : {static_cast<void*>(c->wpack), static_cast<void*>(c->bias), static_cast<void*>(c->mult),
                  static_cast<void*>(c->shift), static_cast<void*>(c->lut), static_cast<void*>(c->err)})
    if (p) cudaFree(p);
  delete c;
  return SUCCESS;
}

}  // namespace
}  // namespace yb

using namespace yb;

extern "C" status_t yb_int8_quantize_conv(const float* w, const float* b, int co, int ci, int kh, int kw, float s_in,
                                          float s_pre, float s_out, int act_silu, int8_t* wq, int32_t* bq,
                                          int32_t* mult, int32_t* shift, int8_t* lut) {
  if (!w || !wq || !bq || !mult || !shift || (act_silu && !lut)) return ERROR_NULL_POINTER;
  if (co < 1 || ci < 1 || kh < 1 || kw < 1 || !(s_in > 0.f) || !(s_out > 0.f) || (act_silu && !(s_pre > 0.f)))
    return ERROR_INVALID_DIMS;
  const size_t per = static_cast<size_t>(ci) * kh * kw;
  for (int c = 0; c < co; ++c) {
    const float* wc = w + c * per;
    float m = 0.f;
    for (size_t i = 0; i < per; ++i) m = std::fmax(m, std::fabs(wc[i]));
    const float sw = m > 0.f ? m / 127.0f : 1.0f;
    for (size_t i = 0; i < per; ++i) {
      const float qv = std::nearbyint(wc[i] / sw);
      wq[c * per + i] = static_cast<int8_t>(qv < -127.f ? -127 : qv > 127.f ? 127 : static_cast<int>(qv));
    }
    long long bv = b ? std::llrint(static_cast<double>(b[c]) / (static_cast<double>(s_in) * sw)) : 0;
    bv = bv < -INT_MAX ? -INT_MAX : bv > INT_MAX ? INT_MAX : bv;
    bq[c] = static_cast<int32_t>(bv);
    const double ratio = static_cast<double>(s_in) * sw / static_cast<double>(act_silu ? s_pre : s_out);
    int e = 0;
    const double f = std::frexp(ratio, &e);
    long long mm = std::llrint(f * 2147483648.0);
    if (mm == 2147483648LL) {
      mm = 1073741824LL;
      e += 1;
    }
    const int sh = 31 - e;
    if (sh < 1) {
      set_error("int8 requantisation ratio s_in*s_w/s_t is 2^30 or more");
      return ERROR_INVALID_DIMS;
    }
    if (sh > 62) {
      mult[c] = 0;
      shift[c] = 1;
    } else {
      mult[c] = static_cast<int32_t>(mm);
      shift[c] = sh;
    }
  }
  if (act_silu) {
    for (int i = 0; i < 256; ++i) {
      const double x = static_cast<double>(i - 128) * s_pre;
      const double y = x / (1.0 + std::exp(-x));
      const long long qv = std::llrint(y / static_cast<double>(s_out));
      lut[i] = static_cast<int8_t>(qv < -127 ? -127 : qv > 127 ? 127 : qv);
    }
  }
  return SUCCESS;
}

extern "C" status_t yb_int8_conv_create(int device, const int8_t* wq, const int32_t* bq, const int32_t* mult,
                                        const int32_t* shift, const int8_t* lut, int co, int ci, int kh, int kw,
                                        int stride, int pad, void** conv) {
  if (!wq || !bq || !mult || !shift || !conv) return ERROR_NULL_POINTER;
  *conv = nullptr;
  if (co < 16 || co > kMaxCo || co % 16 || ci < 1 || kh != kw || (kh != 1 && kh != 3) || stride < 1 || pad < 0) {
    set_error("int8 conv: co must be a multiple of 16 (<= 1024), kernel 1x1 or 3x3");
    return ERROR_INVALID_DIMS;
  }
  for (int c = 0; c < co; ++c)
    if (shift[c] < 1 || shift[c] > 62) {
      set_error("int8 conv: shift outside [1, 62]");
      return ERROR_INVALID_DIMS;
    }
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  auto* c = new Int8Conv();
  c->device = device;
  c->co = co;
  c->ci = ci;
  c->kh = kh;
  c->kw = kw;
  c->stride = stride;
  c->pad = pad;
  I8Tiling t;
  i8_tiling(co, ci, kh, kw, &t);
  c->ci_pad = t.ci_pad;
  c->a_cpp = t.a_cpp;
  c->K = t.K;
  c->num_kc = t.num_kc;
  c->n_tile = t.n_tile;
  c->n_tiles = t.n_tiles;
  cudaDeviceGetAttribute(&c->sms, cudaDevAttrMultiProcessorCount, device);
  const std::vector<uint8_t> pk = i8_pack_weights(wq, co, ci, kh, kw, t);
  const size_t nq = static_cast<size_t>(i8_bias_slots(t));
  std::vector<int32_t> hb(nq, 0), hm(nq, 0), hs(nq, 1);
  for (int i = 0; i < co; ++i) {
    hb[i] = bq[i];
    hm[i] = mult[i];
    hs[i] = shift[i];
  }
  if ((e = cudaMalloc(&c->wpack, pk.size())) == cudaSuccess &&
      (e = cudaMalloc(&c->bias, nq * 4)) == cudaSuccess && (e = cudaMalloc(&c->mult, nq * 4)) == cudaSuccess &&
      (e = cudaMalloc(&c->shift, nq * 4)) == cudaSuccess && (e = cudaMalloc(&c->err, sizeof(int))) == cudaSuccess &&
      (!lut || (e = cudaMalloc(&c->lut, 256)) == cudaSuccess)) {
    e = cudaMemcpy(c->wpack, pk.data(), pk.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(c->bias, hb.data(), nq * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(c->mult, hm.data(), nq * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(c->shift, hs.data(), nq * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && lut) e = cudaMemcpy(c->lut, lut, 256, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(c->err, 0, sizeof(int));
    if (e == cudaSuccess) e = i8_init_kernel();
  }
  if (e != cudaSuccess) {
    const status_t st = cuda_status(e, "int8 conv upload");
    free_conv(c);
    return st;
  }
  if (stages_for_i8(c->n_tile, c->n_tiles) < 2) {
    free_conv(c);
    set_error("int8 conv: tile does not fit in shared memory");
    return ERROR_INVALID_DIMS;
  }
  *conv = c;
  return SUCCESS;
}

extern "C" int yb_int8_conv_ci_pad(void* conv) { return conv ? static_cast<Int8Conv*>(conv)->ci_pad : 0; }

extern "C" status_t yb_int8_conv_run(void* conv, const int8_t* d_x, int B, int H, int W, int8_t* d_y, void* stream) {
  auto* c = static_cast<Int8Conv*>(conv);
  if (!c || !d_x || !d_y) return ERROR_NULL_POINTER;
  if (B < 1 || H < 1 || W < 1) return ERROR_INVALID_DIMS;
  const int Ho = (H + 2 * c->pad - c->kh) / c->stride + 1, Wo = (W + 2 * c->pad - c->kw) / c->stride + 1;
  if (Ho < 1 || Wo < 1) return ERROR_INVALID_DIMS;
  const long long M = static_cast<long long>(B) * Ho * Wo;
  if (M > INT_MAX - 256 || static_cast<long long>(B) * H * W * c->ci_pad > (1LL << 40)) return ERROR_INVALID_DIMS;
  if (reinterpret_cast<uintptr_t>(d_x) % 16 || reinterpret_cast<uintptr_t>(d_y) % 16) {
    set_error("int8 conv: buffers must be 16-byte aligned");
    return ERROR_INVALID_DIMS;
  }
  cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  I8Args a;
  a.B = B;
  a.H = H;
  a.W = W;
  a.Ci = c->ci_pad;
  a.Co = c->co;
  a.kh = c->kh;
  a.kw = c->kw;
  a.stride = c->stride;
  a.pad = c->pad;
  a.Ho = Ho;
  a.Wo = Wo;
  a.K = c->K;
  a.num_kc = c->num_kc;
  a.n_tile = c->n_tile;
  a.n_tiles = c->n_tiles;
  a.m_tiles = static_cast<int>((M + kBM - 1) / kBM);
  a.a_cpp = c->a_cpp;
  a.wpack = c->wpack;
  a.bias = c->bias;
  a.mult = c->mult;
  a.shift = c->shift;
  a.lut = c->lut;
  a.out = d_y;
  a.out_cstride = c->co;
  a.err = c->err;
  std::string why;
  e = launch_conv_i8(a, d_x, c->ci_pad, static_cast<long long>(c->ci_pad) * H * W, static_cast<cudaStream_t>(stream),
                     c->sms, &why);
  if (e == cudaErrorInvalidValue || e == cudaErrorNotSupported) {
    set_error(why.empty() ? "int8 conv launch rejected" : why);
    return ERROR_INVALID_DIMS;
  }
  return cuda_status(e, "int8 conv launch");
}

extern "C" status_t yb_int8_conv_check(void* conv) {
  auto* c = static_cast<Int8Conv*>(conv);
  if (!c) return ERROR_NULL_POINTER;
  cudaError_t e = cudaSetDevice(c->device);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  int k = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&k, c->err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "int8 conv check");
  if (k) {
    cudaMemset(c->err, 0, sizeof(int));
    set_error("int8 conv kernel reported error code " + std::to_string(k));
    return ERROR_DEVICE;
  }
  return SUCCESS;
}

extern "C" status_t yb_int8_conv_destroy(void* conv) {
  if (!conv) return ERROR_NULL_POINTER;
  const status_t st = yb_int8_conv_check(conv);
  free_conv(static_cast<Int8Conv*>(conv));
  return st;
}
