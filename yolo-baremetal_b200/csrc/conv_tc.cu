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
// Persistent, warp-specialised CTA (544 threads, one CTA per SM):
//   warps 0-3   producers: each K chunk of the activation tile is gathered
//               with 16-byte cp.async copies straight from the hi and lo
//               planes into the 128B-swizzled K-major operand layout (zero
//               fill for padding and K tails; upsample and two-source concat
//               in the address computation), several stages deep; each
//               thread's copies arrive on the stage's mbarrier as they land.
//               Thread 0 also starts one bulk copy (TMA engine) of the
//               pre-packed, pre-swizzled weight chunk.  In the TMA modes one
//               thread issues the tensor copies instead.
//   warp 16     allocates tensor memory (2-3 accumulators) and, from one
//               lane, issues the UMMAs; tcgen05.commit frees each smem stage
//               and publishes each finished accumulator.
//   warps 4-15  epilogue in three groups of four (two when three
//               accumulators do not fit in tensor memory) taking tiles round
//               robin, one warp per TMEM lane quarter (32 output pixels):
//               tcgen05.ld, + bias (staged in shared memory), SiLU,
//               + residual, split (or fp32) NHWC store into the destination
//               channel slice.  Runs while warp 16 accumulates the next tiles
//               into the other TMEM buffers.
// All barrier waits are bounded (sm100.cuh); a timeout sets *a.err, aborts
// the other roles, drains outstanding copies and UMMAs and frees tensor
// memory.
#include <cudaTypedefs.h>

#include <cfloat>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>
#include "pdl.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "split.cuh"

namespace yb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kProducerWarps = 4;  // one per sub-partition (the gather producers; one thread in TMA modes)
constexpr int kRowStep = kProducerWarps * 32 / 8;                // rows per pass: 8 threads per 128-byte row
constexpr int kRowsPerThread = kBM / kRowStep;
constexpr int kEpilogueWarps = 12;  // up to three groups of four (one warp per TMEM lane quarter), round-robin tiles
constexpr int kMaxAcc = 4;         // TMEM accumulators when n_tile allows (4 x n_tile <= 512 columns)
constexpr int kMmaWarp = kProducerWarps + kEpilogueWarps;
constexpr int kThreads = (kMmaWarp + 1) * 32;
constexpr uint32_t kAPlaneBytes = kBM * 128;  // one 128 x 64 bf16 plane
constexpr int kSmemLimit = 232448;            // 227 KB opt-in per CTA
constexpr int kSmemExtra = 1024 + 512;
// Patch mode: one 8-channel chunk of a tile's 18 x 10 input patch (16 bytes
// per pixel, pixel-major), padded to a 128-byte multiple.
constexpr int kPatchH = 18, kPatchW = 10;
constexpr uint32_t kPatchBox = kPatchH * kPatchW * 16;  // 2880 bytes written by one box copy
constexpr uint32_t kPatchChunk = 2944;
__host__ __device__ constexpr uint32_t patch_stage_bytes(int ci) {
  return ((static_cast<uint32_t>(ci / 8) * 2u * kPatchChunk) + 1023u) & ~1023u;
}
// Stride-2 patch mode (a_tma == 3): a tile of 16 x 8 output pixels reads
// input rows 2 oy0 - 1 .. 2 oy0 + 31 (33) and columns 2 ox0 - 1 .. 2 ox0 + 15.
// Per 8-channel chunk and plane two boxes with a column traversal stride of 2
// (box 18 columns -> 9 pixels): O holds columns 2 ox0 - 1 + 2i (taps kx = 0
// at i = c, kx = 2 at i = c + 1), E columns 2 ox0 + 2i (kx = 1 at i = c), so
// every tap window is 8 consecutive 16-byte pixels per output row and the
// next output row is two input rows (288 bytes) further.
constexpr int kP2Rows = 33, kP2Cols = 9;
constexpr uint32_t kP2Row = kP2Cols * 16;      // 144 bytes per row
constexpr uint32_t kP2Box = kP2Rows * kP2Row;  // 4752 bytes written by one box copy
constexpr uint32_t kP2Plane = 4864;            // 128-byte multiple
constexpr uint32_t kP2Chunk = 2 * kP2Plane;    // O and E of one 8-channel chunk
__host__ __device__ constexpr uint32_t patch2_stage_bytes(int ci) {
  return ((static_cast<uint32_t>(ci / 8) * 2u * kP2Chunk) + 1023u) & ~1023u;
}
__host__ __device__ constexpr uint32_t p2_window(int t) {
  return ((t % 3) == 1 ? kP2Plane : 0u) + static_cast<uint32_t>(t / 3) * kP2Row + ((t % 3) == 2 ? 16u : 0u);
}          // alignment slack + barriers; the bias follows


// UMMA issue of one patch-mode tile, fully unrolled: every operand
// descriptor is a compile-time offset from four base descriptors, so the
// issuing thread emits little besides the tcgen05.mma instructions.  Measured
// on B200 (M = 128, K = 16, N <= 32): about 45 cycles per UMMA issued back to
// back this way, against about 150 with per-step descriptor arithmetic in a
// rolled loop, which made the small-channel 3x3 convolutions issue-bound.
// P2: stride-2 patch (odd / even column planes); else the stride-1 patch.
template <int CBS, bool P2, bool ST>
__device__ __forceinline__ void patch_tile_mma(uint32_t d, uint64_t dah0, uint64_t dal0, uint64_t dbh0,
                                               uint64_t dbl0, uint64_t chunk_units, uint32_t idesc) {
#pragma unroll
  for (int tap = 0; tap < 9; ++tap) {
#pragma unroll
    for (int cb = 0; cb < CBS; ++cb) {
      const int step = tap * CBS + cb;
      const uint64_t ao = P2 ? static_cast<uint64_t>((2u * cb * kP2Chunk + p2_window(tap)) >> 4)
                             : static_cast<uint64_t>((tap / 3) * kPatchW + tap % 3 + cb * (2 * kPatchChunk / 16));
      const uint64_t boff = static_cast<uint64_t>(step >> 2) * chunk_units + static_cast<uint64_t>((step & 3) * 2);
      const uint32_t accum = step != 0 ? 1u : 0u;
      if (ST) {
        tc_mma_bf16(d, dah0 + ao, dbh0 + boff, idesc, accum);
        tc_mma_bf16(d, dal0 + ao, dbh0 + boff, idesc_half_n(idesc), 1u);
      } else {
        tc_mma_bf16(d, dah0 + ao, dbh0 + boff, idesc, accum);
        tc_mma_bf16(d, dah0 + ao, dbl0 + boff, idesc, 1u);
        tc_mma_bf16(d, dal0 + ao, dbh0 + boff, idesc, 1u);
      }
    }
  }
}

// Runs patch_tile_mma for cbs in 1..4; false for other channel counts.
template <bool P2, bool ST>
__device__ __forceinline__ bool patch_tile_mma_n(int cbs, uint32_t d, uint64_t dah0, uint64_t dal0, uint64_t dbh0,
                                                 uint64_t dbl0, uint64_t chunk_units, uint32_t idesc) {
  switch (cbs) {
    case 1: patch_tile_mma<1, P2, ST>(d, dah0, dal0, dbh0, dbl0, chunk_units, idesc); return true;
    case 2: patch_tile_mma<2, P2, ST>(d, dah0, dal0, dbh0, dbl0, chunk_units, idesc); return true;
    case 3: patch_tile_mma<3, P2, ST>(d, dah0, dal0, dbh0, dbl0, chunk_units, idesc); return true;
    case 4: patch_tile_mma<4, P2, ST>(d, dah0, dal0, dbh0, dbl0, chunk_units, idesc); return true;
    default: return false;
  }
}

// Eight input channels: two taps per K step (see the caller), unrolled the
// same way; hb / lb are the hi / lo patch descriptors with LBO 0.
template <bool ST>
__device__ __forceinline__ void patch8_tile_mma(uint32_t d, uint64_t hb, uint64_t lb, uint64_t dbh0, uint64_t dbl0,
                                                uint64_t chunk_units, uint32_t idesc) {
#pragma unroll
  for (int s2 = 0; s2 < 5; ++s2) {
    const int t0 = 2 * s2, t1 = t0 + 1 < 9 ? t0 + 1 : t0;
    const uint32_t o0 = static_cast<uint32_t>(((t0 / 3) * kPatchW + t0 % 3) * 16);
    const uint32_t o1 = static_cast<uint32_t>(((t1 / 3) * kPatchW + t1 % 3) * 16);
    const uint32_t lbo = t1 == t0 ? 16u : o1 - o0;
    const uint64_t off = static_cast<uint64_t>(o0 >> 4) | (static_cast<uint64_t>(lbo >> 4) << 16);
    const uint64_t boff = static_cast<uint64_t>(s2 >> 2) * chunk_units + static_cast<uint64_t>((s2 & 3) * 2);
    const uint32_t accum = s2 != 0 ? 1u : 0u;
    if (ST) {
      tc_mma_bf16(d, hb + off, dbh0 + boff, idesc, accum);
      tc_mma_bf16(d, lb + off, dbh0 + boff, idesc_half_n(idesc), 1u);
    } else {
      tc_mma_bf16(d, hb + off, dbh0 + boff, idesc, accum);
      tc_mma_bf16(d, hb + off, dbl0 + boff, idesc, 1u);
      tc_mma_bf16(d, lb + off, dbh0 + boff, idesc, 1u);
    }
  }
}

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

// EPI: the epilogue, fixed per launch so that each instantiation carries one
// compact loop: bit 0 SiLU, bit 1 the residual, bit 2 fp32 output (the Detect
// head's last convolutions), bit 3 calibration statistics.
template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) conv_tc_kernel(const __grid_constant__ ConvArgs a, const int stages) {
  extern __shared__ uint8_t smem_raw[];
  // Swizzle atoms need 1024-byte alignment in the shared window.
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool patch = a.a_tma >= 2;
  const bool patch2 = a.a_tma == 3;
  const uint32_t chunk_bytes = static_cast<uint32_t>(a.n_tile) * 256u;
  // Patch mode keeps every weight chunk resident in front of the stages.
  const uint32_t wres_bytes = patch ? static_cast<uint32_t>(a.num_kc) * chunk_bytes : 0u;
  const uint32_t stage_bytes = patch2  ? patch2_stage_bytes(a.Ci)
                               : patch ? patch_stage_bytes(a.Ci)
                                       : 2u * kAPlaneBytes + chunk_bytes;
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
  float* sbias = reinterpret_cast<float*>(tail + 512);  // n_tile * n_tiles floats, zero past Co
  const int nbias = a.n_tile * a.n_tiles;
  for (int i = threadIdx.x; i < nbias; i += kThreads) sbias[i] = (a.bias && i < a.Co) ? a.bias[i] : 0.0f;

  // Accumulators of acc_stride (power of two >= n_tile) columns, as many as
  // fit in the 512 TMEM columns up to kMaxAcc.
  // Patch mode (MMA-issue bound: many small K steps per tile) with
  // n_tile <= 128: each K step is two UMMAs against the stacked
  // [B_hi; B_lo] chunk, A_hi with N = 2 n_tile (columns [0, n) += A_hi*B_hi,
  // [n, 2n) += A_hi*B_lo) and A_lo with N = n_tile (B_hi only: columns
  // [0, n) += A_lo*B_hi), summed by the epilogue.  Otherwise three UMMAs of N = n_tile, which
  // keeps the epilogue (the long pole there) to one TMEM load per unit.
  // The im2col / gather modes stack too for 3x3 convolutions of at most 64
  // output channels (MMA-issue bound: measured ~45-64 cycles per UMMA at
  // N <= 128, so two UMMAs of 2n beat three of n); 1x1 convolutions keep one
  // TMEM load per unit for their epilogue-bound tiles.  The choice depends on
  // the layer, not on its N tiling (which the engine narrows for small
  // batches), so that every batch size sums the same products in the same
  // order.
  const bool stacked = patch ? a.n_tile <= 128 : (a.kh * a.kw > 1 && a.Co <= 64);
  const uint32_t acc_cols = static_cast<uint32_t>(stacked ? 2 * a.n_tile : a.n_tile);
  uint32_t acc_stride = 32;
  while (acc_stride < acc_cols) acc_stride <<= 1;
  // Three epilogue groups when three accumulators fit (each group then owns
  // one accumulator, so its waits follow that accumulator's phases in
  // order), else two, each owning every other accumulator.
  const int egroups = 3u * acc_stride <= 512u ? 3 : 2;
  const int nacc = egroups == 3 ? 3 : min(kMaxAcc, static_cast<int>(512u / acc_stride));
  uint32_t ncols = 32;  // the allocation is a power of two
  while (ncols < static_cast<uint32_t>(nacc) * acc_stride) ncols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], a.a_tma ? 1 : kProducerWarps * 32);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < nacc; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);  // the four warps of one epilogue group
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
  if (patch && !patch2 && a.Ci == 8) {
    // The paired K step of tap 8 reads the pixel after its window (against
    // zero weights); for the last patch row that is the pad after the box,
    // which no copy writes.  Zero it so that stale bytes (possibly NaN or
    // Inf as bf16) cannot turn the zero products into NaN.
    const int pads = stages * 2;  // per stage: the hi and lo chunk
    for (int i = threadIdx.x; i < pads * 4; i += kThreads) {
      uint8_t* pad = stage0 + (i >> 3) * stage_bytes + ((i >> 2) & 1) * kPatchChunk + kPatchBox + (i & 3) * 16;
      *reinterpret_cast<uint4*>(pad) = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) pdl_trigger();
  pdl_wait();

  const int total_tiles = a.m_tiles * a.n_tiles;
  const uint64_t wlim = a.wait_ns ? a.wait_ns : kWaitNs;
  // The last K chunk holds K - 64 (num_kc - 1) real values: only its first
  // ks_last 16-wide steps are copied and multiplied.
  const int ks_last = (a.K - (a.num_kc - 1) * kBK + 15) / 16;
  const int HoWo = a.Ho * a.Wo;
  const int M = a.B * HoWo;

  if (warp < kProducerWarps && a.debug_withhold) {
    // Test hook: no barrier is armed and no copy issued; the MMA issuer's
    // first wait runs out after wlim.
  } else if (warp < kProducerWarps && patch) {
    // ----------------------------------------------------- patch producer
    // One thread: the resident weights once, then per tile one box copy per
    // 8-channel chunk and plane of its 18 x 10 input patch.
    if (threadIdx.x == 0) {
      prefetch_tmap(&a.tm_hi);
      prefetch_tmap(&a.tm_lo);
      mbar_arrive_expect_tx(wbar, wres_bytes);
      for (int kc = 0; kc < a.num_kc; ++kc)
        bulk_g2s(smem + static_cast<size_t>(kc) * chunk_bytes, a.wpack + static_cast<size_t>(kc) * chunk_bytes,
                 chunk_bytes, wbar);
      const int nch = a.Ci / 8;
      const int per = a.tiles_y * a.tiles_x;
      uint32_t it = 0;
      for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++it) {
        const uint32_t itq = a.fd_stages.div(it);
        const uint32_t s = it - itq * static_cast<uint32_t>(stages);
        const uint32_t ph = itq & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, wlim)) {
          raise_error(a.err, abort_flag, kErrWaitEmpty);
          break;
        }
        const int b = static_cast<int>(a.fd_per.div(static_cast<uint32_t>(t)));
        const int rem = t - b * per;
        const int ty = static_cast<int>(a.fd_tx.div(static_cast<uint32_t>(rem)));
        const int tx = rem - ty * a.tiles_x;
        uint8_t* stage = stage0 + s * stage_bytes;
        if (patch2) {
          mbar_arrive_expect_tx(&full[s], 4u * static_cast<uint32_t>(nch) * kP2Box);
          for (int ch = 0; ch < nch; ++ch) {
            uint8_t* hi = stage + ch * kP2Chunk;
            uint8_t* lo = stage + (nch + ch) * kP2Chunk;
            tma_tile_4d(hi, &a.tm_hi, 8 * ch, tx * 16 - 1, ty * 32 - 1, b, &full[s]);
            tma_tile_4d(hi + kP2Plane, &a.tm_hi, 8 * ch, tx * 16, ty * 32 - 1, b, &full[s]);
            tma_tile_4d(lo, &a.tm_lo, 8 * ch, tx * 16 - 1, ty * 32 - 1, b, &full[s]);
            tma_tile_4d(lo + kP2Plane, &a.tm_lo, 8 * ch, tx * 16, ty * 32 - 1, b, &full[s]);
          }
          continue;
        }
        mbar_arrive_expect_tx(&full[s], 2u * static_cast<uint32_t>(nch) * kPatchBox);
        for (int ch = 0; ch < nch; ++ch) {
          tma_tile_4d(stage + ch * kPatchChunk, &a.tm_hi, 8 * ch, tx * 8 - 1, ty * 16 - 1, b, &full[s]);
          tma_tile_4d(stage + (nch + ch) * kPatchChunk, &a.tm_lo, 8 * ch, tx * 8 - 1, ty * 16 - 1, b, &full[s]);
        }
      }
    }
  } else if (warp < kProducerWarps && a.a_tma) {
    // ------------------------------------------------------- TMA producer
    // One thread: per K chunk, the packed weight chunk (bulk copy) and one
    // im2col copy per filter tap and plane into the chunk's a_cpp-channel
    // sub-tiles, all completing on the stage's full barrier.
    if (threadIdx.x == 0) {
      prefetch_tmap(&a.tm_hi);
      prefetch_tmap(&a.tm_lo);
      const int taps = a.kh * a.kw;
      const int cpp = a.a_cpp;
      const int tps = cpp == 64 ? 1 : 64 / cpp;                   // taps per chunk
      const int cblocks = cpp == 64 ? (taps == 1 ? a.num_kc : a.Ci / 64) : 1;  // chunks per tap
      const uint32_t sub_bytes = static_cast<uint32_t>(kBM * cpp * 2);
      uint32_t it = 0;
      for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
        const int mt = static_cast<int>(a.fd_ntiles.div(static_cast<uint32_t>(t)));
        const int nt = t - mt * a.n_tiles;
        const int m0 = mt * kBM;
        const int b = static_cast<int>(a.fd_howo.div(static_cast<uint32_t>(m0)));
        const int r = m0 - b * HoWo;
        const int oy = static_cast<int>(a.fd_wo.div(static_cast<uint32_t>(r)));
        const int ox = r - oy * a.Wo;
        const int w0 = ox * a.stride - a.pad;
        const int h0 = oy * a.stride - a.pad;
        const uint8_t* wsrc = a.wpack + static_cast<size_t>(nt) * a.num_kc * chunk_bytes;
        for (int kc = 0; kc < a.num_kc; ++kc, ++it) {
          const uint32_t itq = a.fd_stages.div(it);
          const uint32_t s = it - itq * static_cast<uint32_t>(stages);
          const uint32_t ph = itq & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, wlim)) {
            raise_error(a.err, abort_flag, kErrWaitEmpty);
            goto tma_producer_done;
          }
          const int t0 = cpp == 64 ? kc / cblocks : kc * tps;
          const int c0 = cpp == 64 ? (kc - t0 * cblocks) * 64 : 0;
          const int ntap = cpp == 64 ? 1 : min(tps, taps - t0);
          uint8_t* stage = stage0 + s * stage_bytes;
          mbar_arrive_expect_tx(&full[s], 2u * static_cast<uint32_t>(ntap) * sub_bytes + chunk_bytes);
          bulk_g2s(stage + 2 * kAPlaneBytes, wsrc + static_cast<size_t>(kc) * chunk_bytes, chunk_bytes, &full[s]);
          for (int i = 0; i < ntap; ++i) {
            const int tap = t0 + i;
            const int ky = tap / a.kw;
            const int kx = tap - ky * a.kw;
            uint8_t* dst = stage + i * sub_bytes;
            tma_im2col_4d(dst, &a.tm_hi, c0, w0, h0, b, static_cast<uint16_t>(kx), static_cast<uint16_t>(ky),
                          &full[s]);
            tma_im2col_4d(dst + kAPlaneBytes, &a.tm_lo, c0, w0, h0, b, static_cast<uint16_t>(kx),
                          static_cast<uint16_t>(ky), &full[s]);
          }
        }
      }
    }
  tma_producer_done:;
  } else if (warp < kProducerWarps) {
    // ------------------------------------------------------------ producers
    // Thread t copies the 16-byte column j = t % 8 (8 K indices) of rows
    // t / 8 + kRowStep i, i < kRowsPerThread, for both planes.  Per tile each
    // row's pixel offset in both sources is computed once; per chunk only the
    // tap and channel of column j change, so a copy costs a few adds and
    // compares.
    const int ptid = threadIdx.x;
    const int j = ptid & 7;
    const int r0 = ptid >> 3;
    uint32_t it = 0;  // chunks issued
    const uint32_t smem_base = smem_u32(stage0);
    const int ws0 = a.W >> a.lg_up0, ws1 = a.W >> a.lg_up1;
    const float inv_ci = 1.0f / static_cast<float>(a.Ci);
    uint32_t row_off[kRowsPerThread];
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i)
      row_off[i] = sw128_offset(static_cast<uint32_t>(r0 + kRowStep * i), static_cast<uint32_t>(j));
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      const int mt = static_cast<int>(a.fd_ntiles.div(static_cast<uint32_t>(t)));
      const int nt = t - mt * a.n_tiles;
      int iy0[kRowsPerThread], ix0[kRowsPerThread];
      long long off0[kRowsPerThread], off1[kRowsPerThread];
      {
        // Row r0 of the tile, then step kRowStep pixels per row without dividing.
        const int m = mt * kBM + r0;
        int b = static_cast<int>(a.fd_howo.div(static_cast<uint32_t>(m)));
        int r = m - b * HoWo;
        int oy = static_cast<int>(a.fd_wo.div(static_cast<uint32_t>(r)));
        int ox = r - oy * a.Wo;
#pragma unroll
        for (int i = 0; i < kRowsPerThread; ++i) {
          const bool valid = m + kRowStep * i < M;
          const int iy = oy * a.stride - a.pad;
          const int ix = ox * a.stride - a.pad;
          iy0[i] = valid ? iy : -(1 << 28);  // never in bounds
          ix0[i] = ix;
          off0[i] = static_cast<long long>(b) * a.src0.bstride +
                    static_cast<long long>((iy >> a.lg_up0) * ws0 + (ix >> a.lg_up0)) * a.src0.cstride;
          off1[i] = static_cast<long long>(b) * a.src1.bstride +
                    static_cast<long long>((iy >> a.lg_up1) * ws1 + (ix >> a.lg_up1)) * a.src1.cstride;
          ox += kRowStep;
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
        const uint32_t itq = a.fd_stages.div(it);
        const uint32_t s = it - itq * static_cast<uint32_t>(stages);
        const uint32_t ph = itq & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, wlim)) {
          raise_error(a.err, abort_flag, kErrWaitEmpty);
          goto producer_done;
        }
        const uint32_t sa_hi = smem_base + s * stage_bytes;
        const uint32_t sa_lo = sa_hi + kAPlaneBytes;
        if (ptid == 0) {
          mbar_expect_tx(&full[s], chunk_bytes);
          bulk_g2s(stage0 + s * stage_bytes + 2 * kAPlaneBytes, wsrc + static_cast<size_t>(kc) * chunk_bytes,
                   chunk_bytes, &full[s]);
        }
        const int k = kc * kBK + j * 8;
        const bool kvalid = k < a.K;
        if (kc == a.num_kc - 1 && j >= 2 * ks_last) {
          // Past the last multiplied step: nothing to copy.
          cp_async_arrive_noinc(&full[s]);
          ++it;
          continue;
        }
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
    const int e_idx = warp - kProducerWarps;  // 0..11
    const int q = e_idx & 3;                  // TMEM lane quarter (= warp % 4)
    const int grp = e_idx >> 2;               // this group takes every egroups-th tile
    constexpr bool f32out = (EPI & 4) != 0;
    // 32-byte stores of whole 16-channel runs when every run starts on a
    // 32-byte boundary (offsets and strides in elements of 2 bytes).
    const bool v8out = !f32out && (reinterpret_cast<uintptr_t>(a.out.hi) & 31) == 0 && (a.out.cstride & 15) == 0 &&
                       (a.out.coff & 15) == 0 && (a.out.bstride & 15) == 0 && (a.out.plane & 15) == 0;
    float mpre = 0.0f, mout = 0.0f;  // calibration statistics (a.amax)
    for (int t = blockIdx.x + grp * gridDim.x, lt = grp; grp < egroups && t < total_tiles;
         t += egroups * gridDim.x, lt += egroups) {
      const int lq = nacc == 4 ? lt >> 2 : nacc == 2 ? lt >> 1 : nacc == 3 ? lt / 3 : lt;
      const int acc = lt - lq * nacc;
      const uint32_t aph = lq & 1;
      if (!mbar_wait(&acc_full[acc], aph, abort_flag, wlim)) {
        raise_error(a.err, abort_flag, kErrWaitAccFull);
        break;
      }
      tc_fence_after();
      const int mt = static_cast<int>(a.fd_ntiles.div(static_cast<uint32_t>(t)));
      const int nt = t - mt * a.n_tiles;
      const int n0 = nt * a.n_tile;
      const int nvalid = min(a.n_tile, a.Co - n0);
      bool valid;
      int b = 0, p = 0;
      if (patch) {
        // Tile of 16 rows x 8 columns; TMEM lane r is pixel (r / 8, r % 8).
        const int per = a.tiles_y * a.tiles_x;
        const int tb = static_cast<int>(a.fd_per.div(static_cast<uint32_t>(t)));
        const int rem = t - tb * per;
        const int ty = static_cast<int>(a.fd_tx.div(static_cast<uint32_t>(rem)));
        const int r = q * 32 + lane;
        const int oy = ty * 16 + (r >> 3);
        const int ox = (rem - ty * a.tiles_x) * 8 + (r & 7);
        valid = oy < a.Ho && ox < a.Wo;
        if (valid) {
          b = tb;
          p = oy * a.Wo + ox;
        }
      } else {
        const int m = mt * kBM + q * 32 + lane;
        valid = m < M;
        if (valid) {
          b = static_cast<int>(a.fd_howo.div(static_cast<uint32_t>(m)));
          p = m - b * HoWo;
        }
      }
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * acc_stride;
      const float* bias_t = sbias + n0;
      // Output element offset of this lane's pixel (also read by the store
      // shuffle below); invalid lanes compute but never store.
      const long long po = f32out ? static_cast<long long>(b) * a.out_f32.bstride +
                                        static_cast<long long>(p) * a.out_f32.cstride + a.out_f32.coff + n0
                                  : static_cast<long long>(b) * a.out.bstride +
                                        static_cast<long long>(p) * a.out.cstride + a.out.coff + n0;
      // Per 16-column unit: one TMEM load, bias and SiLU, residual loads,
      // then the stores.  The next unit's TMEM load is issued as soon as
      // this unit's registers are consumed, so its latency overlaps this
      // unit's arithmetic and stores.
      uint32_t r[16], r2[16];
      tc_ld_32x32b_x16(tbase, r);
      if (stacked) tc_ld_32x32b_x16(tbase + a.n_tile, r2);
      float rmax = -FLT_MAX;  // fp32 output with a row maximum
      for (int c = 0; c < nvalid; c += 16) {
        tc_wait_ld();
        tc_ld_dep(r);
        if (stacked) tc_ld_dep(r2);
        float v[16];
        if (stacked)
          add_pairs<16>(v, reinterpret_cast<const float*>(r), reinterpret_cast<const float*>(r2));
        else
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = __uint_as_float(r[e]);
        if (c + 16 < nvalid) {
          tc_ld_32x32b_x16(tbase + c + 16, r);
          if (stacked) tc_ld_32x32b_x16(tbase + a.n_tile + c + 16, r2);
        }
#pragma unroll
        for (int e = 0; e < 16; e += 4) {
          const float4 bb = *reinterpret_cast<const float4*>(bias_t + c + e);
          const float2 s0 = __fadd2_rn(make_float2(v[e], v[e + 1]), make_float2(bb.x, bb.y));
          const float2 s1 = __fadd2_rn(make_float2(v[e + 2], v[e + 3]), make_float2(bb.z, bb.w));
          v[e] = s0.x;
          v[e + 1] = s0.y;
          v[e + 2] = s1.x;
          v[e + 3] = s1.y;
        }
        const bool stats = (EPI & 8) != 0 && valid;
        if (stats) {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (c + e < nvalid) mpre = fmaxf(mpre, fabsf(v[e]));
        }
        if (EPI & 1) silu_fast_n<16>(v);
        if (stats) {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (c + e < nvalid) mout = fmaxf(mout, fabsf(v[e]));
        }
        const bool second = c + 8 < nvalid;
        if (EPI & 2) {
          const uint16_t* rb = a.res.hi + static_cast<long long>(b) * a.res.bstride +
                               static_cast<long long>(p) * a.res.cstride + a.res.coff + n0 + c;
          float rv[16];
          load8_rw(rb, a.res.plane, *reinterpret_cast<float(*)[8]>(&rv[0]));
          if (second) load8_rw(rb + 8, a.res.plane, *reinterpret_cast<float(*)[8]>(&rv[8]));
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            if (e < 8 || second) {
              const float2 t = __fadd2_rn(make_float2(v[e], v[e + 1]), make_float2(rv[e], rv[e + 1]));
              v[e] = t.x;
              v[e + 1] = t.y;
            }
          }
          if (stats) {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c + e < nvalid) mout = fmaxf(mout, fabsf(v[e]));
          }
        }
        if (f32out) {
          if (a.out_f32.rowmax) {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c + e < nvalid) rmax = fmaxf(rmax, v[e]);
          }
          if (valid) {
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              const int n = c + 8 * g;
              if (g == 1 && !second) break;
              float* o = a.out_f32.ptr + po + n;
              *reinterpret_cast<float4*>(o) = make_float4(v[8 * g], v[8 * g + 1], v[8 * g + 2], v[8 * g + 3]);
              if (n + 4 < nvalid)
                *reinterpret_cast<float4*>(o + 4) =
                    make_float4(v[8 * g + 4], v[8 * g + 5], v[8 * g + 6], v[8 * g + 7]);
            }
          }
        } else if (v8out && second) {
          // Split to bf16 hi/lo words; each lane writes its pixel's 32-byte
          // runs (16 channels) with one 32-byte store per plane.
          uint32_t hw[8], lw[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) split2(v[2 * i], v[2 * i + 1], hw[i], lw[i]);
          if (valid) {
            uint16_t* o = a.out.hi + po + c;
            st_global_v8(o, hw);
            st_global_v8(o + a.out.plane, lw);
          }
        } else {
          // Split to bf16 hi/lo words (channel pairs), then regroup across
          // the warp so that lanes 2k and 2k+1 write the two 16-byte halves
          // of one pixel's 32-byte run: every store fills whole sectors.
          uint32_t hw[8], lw[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) split2(v[2 * i], v[2 * i + 1], hw[i], lw[i]);
          const int h = lane & 1;
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int src = (lane >> 1) + 16 * i;
            uint32_t oh[4], ol[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t h0 = __shfl_sync(0xffffffffu, hw[j], src);
              const uint32_t h1 = __shfl_sync(0xffffffffu, hw[4 + j], src);
              const uint32_t l0 = __shfl_sync(0xffffffffu, lw[j], src);
              const uint32_t l1 = __shfl_sync(0xffffffffu, lw[4 + j], src);
              oh[j] = h ? h1 : h0;
              ol[j] = h ? l1 : l0;
            }
            const long long spo = __shfl_sync(0xffffffffu, po, src);
            const bool svalid = __shfl_sync(0xffffffffu, valid, src);
            if (svalid && (h == 0 || second)) {
              uint16_t* o = a.out.hi + spo + c + 8 * h;
              *reinterpret_cast<uint4*>(o) = make_uint4(oh[0], oh[1], oh[2], oh[3]);
              *reinterpret_cast<uint4*>(o + a.out.plane) = make_uint4(ol[0], ol[1], ol[2], ol[3]);
            }
          }
        }
      }
      // The same sigmoid as the decode kernel's (accurate expf, IEEE division).
      if (f32out && a.out_f32.rowmax && valid)
        a.out_f32.rowmax[static_cast<long long>(b) * a.out_f32.rm_bstride + p] = 1.0f / (1.0f + expf(-rmax));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
    if (EPI & 8) {
      const unsigned am = __activemask();
      const unsigned wp = __reduce_max_sync(am, __float_as_uint(mpre));
      const unsigned wo = __reduce_max_sync(am, __float_as_uint(mout));
      if (lane == __ffs(am) - 1) {
        atomicMax(a.amax, wp);
        atomicMax(a.amax + 1, wo);
      }
    }
  } else {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kBM, stacked ? 2 * a.n_tile : a.n_tile);
      const int a_cpp = a.a_tma ? a.a_cpp : 64;
      uint32_t it = 0;
      int lt = 0;
      for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++lt) {
        const int lq = nacc == 4 ? lt >> 2 : nacc == 2 ? lt >> 1 : nacc == 3 ? lt / 3 : lt;
        const int acc = lt - lq * nacc;
        const uint32_t aph = lq & 1;
        if (!mbar_wait(&acc_empty[acc], aph ^ 1u, abort_flag, wlim)) {
          raise_error(a.err, abort_flag, kErrWaitAccEmpty);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * acc_stride;
        bool ok = true;
        if (patch) {
          // One stage per tile: 9 taps x Ci/16 K steps, each A operand a
          // shifted window of the patch, each B step in the resident weights.
          if (lt == 0 && !mbar_wait(wbar, 0, abort_flag, wlim)) {
            raise_error(a.err, abort_flag, kErrWaitFull);
            break;
          }
          const uint32_t itq = a.fd_stages.div(it);
          const uint32_t s = it - itq * static_cast<uint32_t>(stages);
          const uint32_t ph = itq & 1u;
          ++it;
          if (!mbar_wait(&full[s], ph, abort_flag, wlim)) {
            raise_error(a.err, abort_flag, kErrWaitFull);
            break;
          }
          tc_fence_after();
          const int nch = a.Ci / 8;
          const int cbs = a.Ci / 16;
          // Descriptors at the patch origin and at weight chunk 0; every
          // step adds a start-address offset (16-byte units) to them.
          const uint32_t pa = smem_u32(stage0 + s * stage_bytes);
          const uint64_t dah0 = kmajor_desc_noswizzle(pa, kPatchChunk, kPatchW * 16);
          const uint64_t dal0 = kmajor_desc_noswizzle(pa + static_cast<uint32_t>(nch) * kPatchChunk, kPatchChunk,
                                                      kPatchW * 16);
          const uint64_t dbh0 = sw128_kmajor_desc(smem_u32(smem));
          const uint64_t dbl0 = sw128_kmajor_desc(smem_u32(smem) + static_cast<uint32_t>(a.n_tile) * 128u);
          const uint64_t chunk_units = chunk_bytes >> 4;
          if (patch2) {
            // Stride 2 (Ci a multiple of 16): per tap, 16 channels per K step
            // = the 8-channel chunks 2 cb and 2 cb + 1 (LBO one chunk); the
            // output row stride is two input rows (SBO 288 bytes).
            const uint64_t p2h = kmajor_desc_noswizzle(pa, kP2Chunk, 2 * kP2Row);
            const uint64_t p2l = kmajor_desc_noswizzle(pa + static_cast<uint32_t>(nch) * kP2Chunk, kP2Chunk, 2 * kP2Row);
            const bool done = stacked ? patch_tile_mma_n<true, true>(cbs, d_tmem, p2h, p2l, dbh0, dbl0, chunk_units, idesc)
                                      : patch_tile_mma_n<true, false>(cbs, d_tmem, p2h, p2l, dbh0, dbl0, chunk_units, idesc);
            int step = 0;
            for (int tap = 0; tap < 9 && !done; ++tap) {
              for (int cb = 0; cb < cbs; ++cb, ++step) {
                const uint32_t ao = 2u * static_cast<uint32_t>(cb) * kP2Chunk + p2_window(tap);
                const uint64_t dah = kmajor_desc_noswizzle(pa + ao, kP2Chunk, 2 * kP2Row);
                const uint64_t dal =
                    kmajor_desc_noswizzle(pa + static_cast<uint32_t>(nch) * kP2Chunk + ao, kP2Chunk, 2 * kP2Row);
                const uint64_t boff =
                    static_cast<uint64_t>(step >> 2) * chunk_units + static_cast<uint64_t>((step & 3) * 2);
                const uint32_t accum = step != 0 ? 1u : 0u;
                if (stacked) {
                  tc_mma_bf16(d_tmem, dah, dbh0 + boff, idesc, accum);
                  tc_mma_bf16(d_tmem, dal, dbh0 + boff, idesc_half_n(idesc), 1u);
                } else {
                  tc_mma_bf16(d_tmem, dah, dbh0 + boff, idesc, accum);
                  tc_mma_bf16(d_tmem, dah, dbl0 + boff, idesc, 1u);
                  tc_mma_bf16(d_tmem, dal, dbh0 + boff, idesc, 1u);
                }
              }
            }
            tc_commit(&empty[s]);
            tc_commit(&acc_full[acc]);
            continue;
          }
          if (a.Ci == 8) {
            // Eight input channels (16 bytes per pixel and plane): two taps
            // per 16-wide K step.  The A operand's second core matrix is the
            // next tap's window (LBO = the distance between the windows);
            // K is ordered (tap, channel) with 8 channels per tap, so the
            // weights already hold the two taps back to back.  Tap 8 pairs
            // with zero weights.
            const uint64_t hb = kmajor_desc_noswizzle(pa, 0, kPatchW * 16);
            const uint64_t lb = kmajor_desc_noswizzle(pa + kPatchChunk, 0, kPatchW * 16);
            if (stacked) patch8_tile_mma<true>(d_tmem, hb, lb, dbh0, dbl0, chunk_units, idesc);
            else patch8_tile_mma<false>(d_tmem, hb, lb, dbh0, dbl0, chunk_units, idesc);
            tc_commit(&empty[s]);
            tc_commit(&acc_full[acc]);
            continue;
          }
          const bool done = stacked ? patch_tile_mma_n<false, true>(cbs, d_tmem, dah0, dal0, dbh0, dbl0, chunk_units, idesc)
                                    : patch_tile_mma_n<false, false>(cbs, d_tmem, dah0, dal0, dbh0, dbl0, chunk_units, idesc);
          int step = 0;
          for (int ky = 0; ky < 3 && !done; ++ky) {
            for (int kx = 0; kx < 3; ++kx) {
              const uint64_t toff = static_cast<uint64_t>(ky * kPatchW + kx);  // window shift, 16-byte rows
              for (int cb = 0; cb < cbs; ++cb, ++step) {
                const uint64_t aoff = toff + static_cast<uint64_t>(cb) * (2 * kPatchChunk / 16);
                const uint64_t boff = static_cast<uint64_t>(step >> 2) * chunk_units + static_cast<uint64_t>((step & 3) * 2);
                const uint32_t accum = step != 0 ? 1u : 0u;
                if (stacked) {
                  tc_mma_bf16(d_tmem, dah0 + aoff, dbh0 + boff, idesc, accum);
                  tc_mma_bf16(d_tmem, dal0 + aoff, dbh0 + boff, idesc_half_n(idesc), 1u);
                } else {
                  tc_mma_bf16(d_tmem, dah0 + aoff, dbh0 + boff, idesc, accum);
                  tc_mma_bf16(d_tmem, dah0 + aoff, dbl0 + boff, idesc, 1u);
                  tc_mma_bf16(d_tmem, dal0 + aoff, dbh0 + boff, idesc, 1u);
                }
              }
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
          if (!mbar_wait(&full[s], ph, abort_flag, wlim)) {
            raise_error(a.err, abort_flag, kErrWaitFull);
            ok = false;
            break;
          }
          // A stage written by cp.async (gather mode) is ordered before the
          // tensor core's (async-proxy) operand reads; TMA writes need no fence.
          if (!a.a_tma) fence_proxy_async_smem();
          tc_fence_after();
          // Descriptors of the stage's four operand planes; a 16-wide K step
          // advances the start address by 32 bytes (2 in the >>4 field).
          const uint32_t a_hi = smem_u32(stage0 + s * stage_bytes);
          // Activation sub-tiles: 128B swizzle (rows of 64 channels) unless
          // TMA copies of 16 or 32 channels per tap (32B / 64B swizzle, one
          // sub-tile per tap).
          const uint32_t a_layout = a_cpp == 16 ? 6u : a_cpp == 32 ? 4u : 2u;
          const uint32_t a_sbo = a_cpp == 16 ? 256u : a_cpp == 32 ? 512u : 1024u;
          const uint64_t dah0 = kmajor_desc(a_hi, a_layout, a_sbo);
          const uint64_t dal0 = kmajor_desc(a_hi + kAPlaneBytes, a_layout, a_sbo);
          const uint64_t dbh0 = sw128_kmajor_desc(a_hi + 2 * kAPlaneBytes);
          const uint64_t dbl0 = sw128_kmajor_desc(a_hi + 2 * kAPlaneBytes + static_cast<uint32_t>(a.n_tile) * 128u);
          const int nks = kc == a.num_kc - 1 ? ks_last : kBK / 16;
#pragma unroll
          for (int ks = 0; ks < kBK / 16; ++ks) {
            if (ks >= nks) break;
            // Start-address advance (16-byte units) of K step ks in A and B.
            const uint64_t koff = static_cast<uint64_t>(ks * 2);
            const uint64_t aoff = a_cpp == 16   ? static_cast<uint64_t>(ks * 256)
                                  : a_cpp == 32 ? static_cast<uint64_t>((ks >> 1) * 512 + (ks & 1) * 2)
                                                : koff;
            if (stacked) {
              tc_mma_bf16(d_tmem, dah0 + aoff, dbh0 + koff, idesc, (kc | ks) != 0 ? 1u : 0u);
              tc_mma_bf16(d_tmem, dal0 + aoff, dbh0 + koff, idesc_half_n(idesc), 1u);
            } else {
              tc_mma_bf16(d_tmem, dah0 + aoff, dbh0 + koff, idesc, (kc | ks) != 0 ? 1u : 0u);
              tc_mma_bf16(d_tmem, dah0 + aoff, dbl0 + koff, idesc, 1u);
              tc_mma_bf16(d_tmem, dal0 + aoff, dbh0 + koff, idesc, 1u);
            }
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
      while (!drained && globaltimer_ns() - t0 < wlim) drained = mbar_try_wait(drain, 0);
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

int bias_bytes(int n_tile, int n_tiles) { return (n_tile * n_tiles * 4 + 15) & ~15; }


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
namespace {

// cuTensorMapEncodeIm2col from the driver, looked up once through the
// runtime (no link-time dependency on libcuda).
PFN_cuTensorMapEncodeIm2col_v12000 im2col_encoder() {
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

// im2col map over one plane of a split NHWC view: dims (C, W, H, N) with
// C = a.Ci channels starting at the view's channel offset.
bool encode_plane(CUtensorMap* map, const ConvArgs& a, const uint16_t* base, int cpp) {
  const auto enc = im2col_encoder();
  if (!enc) return false;
  const uintptr_t addr = reinterpret_cast<uintptr_t>(base);
  const long long cs = a.src0.cstride;
  if (addr % 16 || (cs * 2) % 16 || (a.src0.bstride * 2) % 16) return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.Ci), static_cast<cuuint64_t>(a.W), static_cast<cuuint64_t>(a.H),
                        static_cast<cuuint64_t>(a.B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(cs * 2), static_cast<cuuint64_t>(cs * 2 * a.W),
                           static_cast<cuuint64_t>(a.src0.bstride * 2)};
  // Window origins run from -pad to (extent - 1) + pad - (k - 1).
  int lower[2] = {-a.pad, -a.pad};
  int upper[2] = {a.pad - (a.kw - 1), a.pad - (a.kh - 1)};
  cuuint32_t estr[4] = {1, static_cast<cuuint32_t>(a.stride), static_cast<cuuint32_t>(a.stride), 1};
  const CUtensorMapSwizzle sw = cpp == 16   ? CU_TENSOR_MAP_SWIZZLE_32B
                                : cpp == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                            : CU_TENSOR_MAP_SWIZZLE_128B;
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<uint16_t*>(base), dims, strides, lower,
                         upper, static_cast<cuuint32_t>(cpp), static_cast<cuuint32_t>(kBM), estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
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

// Tiled map over one plane of a split NHWC view, dims (C, W, H, N), with
// boxes of 8 channels x kPatchW x kPatchH pixels of one image.
bool encode_patch_plane(CUtensorMap* map, const ConvArgs& a, const uint16_t* base) {
  const auto enc = tiled_encoder();
  if (!enc) return false;
  const long long cs = a.src0.cstride;
  if (reinterpret_cast<uintptr_t>(base) % 16 || (cs * 2) % 16 || (a.src0.bstride * 2) % 16) return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.Ci), static_cast<cuuint64_t>(a.W), static_cast<cuuint64_t>(a.H),
                        static_cast<cuuint64_t>(a.B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(cs * 2), static_cast<cuuint64_t>(cs * 2 * a.W),
                           static_cast<cuuint64_t>(a.src0.bstride * 2)};
  cuuint32_t box[4] = {8, kPatchW, kPatchH, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<uint16_t*>(base), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int conv_stage_bytes(const ConvArgs& a) {
  return a.a_tma == 3   ? static_cast<int>(patch2_stage_bytes(a.Ci))
         : a.a_tma == 2 ? static_cast<int>(patch_stage_bytes(a.Ci))
                        : 2 * static_cast<int>(kAPlaneBytes) + static_cast<int>(conv_chunk_bytes(a.n_tile));
}
int conv_resident_bytes(const ConvArgs& a) {
  return a.a_tma >= 2 ? a.num_kc * static_cast<int>(conv_chunk_bytes(a.n_tile)) : 0;
}
// Slack after the last stage (stride-2 patch mode).
int conv_slack_bytes(const ConvArgs& a) { return a.a_tma == 3 ? static_cast<int>(kP2Plane) : 0; }
int conv_stages(const ConvArgs& a) {
  const int st = (kSmemLimit - kSmemExtra - bias_bytes(a.n_tile, a.n_tiles) - conv_resident_bytes(a) -
                  conv_slack_bytes(a)) /
                 conv_stage_bytes(a);
  return st > 8 ? 8 : st;
}

// Tiled map over one plane, dims (C, W, H, N), boxes of 8 channels x 18
// columns (traversed with stride 2: 9 pixels) x 33 rows of one image.
bool encode_patch2_plane(CUtensorMap* map, const ConvArgs& a, const uint16_t* base) {
  const auto enc = tiled_encoder();
  if (!enc) return false;
  const long long cs = a.src0.cstride;
  if (reinterpret_cast<uintptr_t>(base) % 16 || (cs * 2) % 16 || (a.src0.bstride * 2) % 16) return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.Ci), static_cast<cuuint64_t>(a.W), static_cast<cuuint64_t>(a.H),
                        static_cast<cuuint64_t>(a.B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(cs * 2), static_cast<cuuint64_t>(cs * 2 * a.W),
                           static_cast<cuuint64_t>(a.src0.bstride * 2)};
  cuuint32_t box[4] = {8, 2 * kP2Cols, kP2Rows, 1};
  cuuint32_t estr[4] = {1, 2, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<uint16_t*>(base), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace

bool conv_setup_patch(ConvArgs* a) {
  if (a->kh != 3 || a->kw != 3 || a->stride != 1 || a->pad != 1) return false;
  if (a->lg_up0 || a->lg_up1 || a->c_split != a->Ci || (a->Ci % 16 && a->Ci != 8) || !a->src0.hi || a->n_tiles != 1)
    return false;
  if (a->K != 9 * a->Ci || a->Ho != a->H || a->Wo != a->W) return false;
  ConvArgs t = *a;
  t.a_tma = 2;
  if (conv_stages(t) < 3) return false;  // resident weights leave too little room
  const uint16_t* hi = a->src0.hi + a->src0.coff;
  if (!encode_patch_plane(&t.tm_hi, t, hi) || !encode_patch_plane(&t.tm_lo, t, hi + a->src0.plane)) return false;
  t.a_cpp = 0;
  t.tiles_y = (a->Ho + 15) / 16;
  t.tiles_x = (a->Wo + 7) / 8;
  t.m_tiles = a->B * t.tiles_y * t.tiles_x;
  *a = t;
  return true;
}

bool conv_setup_patch2(ConvArgs* a) {
  if (a->kh != 3 || a->kw != 3 || a->stride != 2 || a->pad != 1) return false;
  if (a->lg_up0 || a->lg_up1 || a->c_split != a->Ci || a->Ci % 16 || !a->src0.hi || a->n_tiles != 1) return false;
  if (a->K != 9 * a->Ci || a->Ho != (a->H - 1) / 2 + 1 || a->Wo != (a->W - 1) / 2 + 1) return false;
  ConvArgs t = *a;
  t.a_tma = 3;
  if (conv_stages(t) < 3) return false;  // resident weights leave too little room
  const uint16_t* hi = a->src0.hi + a->src0.coff;
  if (!encode_patch2_plane(&t.tm_hi, t, hi) || !encode_patch2_plane(&t.tm_lo, t, hi + a->src0.plane)) return false;
  t.a_cpp = 0;
  t.tiles_y = (a->Ho + 15) / 16;
  t.tiles_x = (a->Wo + 7) / 8;
  t.m_tiles = a->B * t.tiles_y * t.tiles_x;
  *a = t;
  return true;
}

void conv_setup_tma(ConvArgs* a) {
  if (conv_setup_patch(a) || conv_setup_patch2(a)) return;
  if (a->lg_up0 || a->lg_up1 || a->c_split != a->Ci || a->Ci % 16 || !a->src0.hi) return;
  const int taps = a->kh * a->kw;
  if (a->K != taps * a->Ci) return;
  int cpp = 0;
  // 16 or 32 channels take boxes of exactly that width (the TMA engine's
  // smem writes, zero fill included, bound the small 1x1 convolutions);
  // otherwise 64-channel boxes, channels past Ci arriving as zeros.
  if (a->Ci == 16 || a->Ci == 32) cpp = a->Ci;
  else if (taps == 1) cpp = 64;
  else if (a->Ci % 64 == 0) cpp = 64;
  else return;
  // Window origins reach (extent - 1) + upper corner; the corners must give
  // exactly the Ho x Wo output raster.
  if ((a->W - 1 + a->pad - (a->kw - 1) + a->pad) / a->stride + 1 != a->Wo ||
      (a->H - 1 + a->pad - (a->kh - 1) + a->pad) / a->stride + 1 != a->Ho)
    return;
  const uint16_t* hi = a->src0.hi + a->src0.coff;
  if (!encode_plane(&a->tm_hi, *a, hi, cpp) || !encode_plane(&a->tm_lo, *a, hi + a->src0.plane, cpp)) return;
  a->a_tma = 1;
  a->a_cpp = cpp;
}

cudaError_t init_conv_kernel_attributes() {
  cudaError_t e = cudaSuccess;
  for (auto k : {conv_tc_kernel<0>, conv_tc_kernel<1>, conv_tc_kernel<2>, conv_tc_kernel<3>, conv_tc_kernel<4>,
                 conv_tc_kernel<5>, conv_tc_kernel<6>, conv_tc_kernel<7>, conv_tc_kernel<8>, conv_tc_kernel<9>,
                 conv_tc_kernel<10>, conv_tc_kernel<11>, conv_tc_kernel<12>, conv_tc_kernel<13>, conv_tc_kernel<14>,
                 conv_tc_kernel<15>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  if (e != cudaSuccess) return e;
  const cudaError_t e2 = init_bottleneck_kernel_attributes();
  return e2 == cudaSuccess ? init_stem_kernel_attributes() : e2;
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
  if (a.n_tiles < 1 || a.n_tile * a.n_tiles < a.Co) return cudaErrorInvalidValue;
  if (a.out_f32.rowmax && (!f32 || a.n_tiles != 1)) return cudaErrorInvalidValue;
  if (a.a_tma == 2 && (a.n_tiles != 1 || a.kh != 3 || a.kw != 3 || (a.Ci % 16 && a.Ci != 8) || a.tiles_x < 1 || a.tiles_y < 1 ||
                       a.m_tiles != a.B * a.tiles_y * a.tiles_x))
    return cudaErrorInvalidValue;
  if (a.a_tma == 3 && (a.n_tiles != 1 || a.kh != 3 || a.kw != 3 || a.stride != 2 || a.Ci % 16 || a.tiles_x < 1 ||
                       a.tiles_y < 1 || a.m_tiles != a.B * a.tiles_y * a.tiles_x))
    return cudaErrorInvalidValue;
  const int stages = conv_stages(a);
  if (stages < 2) return cudaErrorInvalidValue;
  ConvArgs k = a;
  k.fd_stages = FastDiv(static_cast<uint32_t>(stages));
  k.fd_ntiles = FastDiv(static_cast<uint32_t>(a.n_tiles));
  k.fd_howo = FastDiv(static_cast<uint32_t>(a.Ho * a.Wo));
  k.fd_wo = FastDiv(static_cast<uint32_t>(a.Wo));
  k.fd_per = FastDiv(static_cast<uint32_t>(a.tiles_y > 0 && a.tiles_x > 0 ? a.tiles_y * a.tiles_x : 1));
  k.fd_tx = FastDiv(static_cast<uint32_t>(a.tiles_x > 0 ? a.tiles_x : 1));
  const int smem = kSmemExtra + bias_bytes(a.n_tile, a.n_tiles) + conv_resident_bytes(a) + stages * conv_stage_bytes(a) +
                   conv_slack_bytes(a);
  const int total = a.m_tiles * a.n_tiles;
  if (total <= 0) return cudaSuccess;
  const int grid = total < num_sms ? total : num_sms;
  using ConvKernel = void (*)(ConvArgs, int);
  static const ConvKernel kernels[16] = {
      conv_tc_kernel<0>,  conv_tc_kernel<1>,  conv_tc_kernel<2>,  conv_tc_kernel<3>,
      conv_tc_kernel<4>,  conv_tc_kernel<5>,  conv_tc_kernel<6>,  conv_tc_kernel<7>,
      conv_tc_kernel<8>,  conv_tc_kernel<9>,  conv_tc_kernel<10>, conv_tc_kernel<11>,
      conv_tc_kernel<12>, conv_tc_kernel<13>, conv_tc_kernel<14>, conv_tc_kernel<15>};
  const int epi = (k.act == kActSiLU ? 1 : 0) | (k.res.hi ? 2 : 0) | (k.out_f32.ptr ? 4 : 0) | (k.amax ? 8 : 0);
  return launch_pdl(kernels[epi], dim3(grid), dim3(kThreads), smem, s, k, stages);
}

}  // namespace yb
