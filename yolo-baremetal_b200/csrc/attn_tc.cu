// PSA attention of the FP32 forward (layers.c:310-405) on the tensor cores:
// tcgen05.mma kind::f16 with bf16 operands and fp32 accumulation in tensor
// memory, on the split activation format (value = hi + lo, kernels.h).
//
// One CTA of 128 threads per (128 queries, head, image); thread i owns query
// row i (TMEM lane i).  Keys go in blocks of 64 (72 KB of shared memory and
// 128 TMEM columns, so three CTAs share an SM):
//   pass 1  S = Q K^T as Qh Kh + Qh Kl + Ql Kh (6 UMMAs: 3 products x 2 K
//           steps of 16) -> row maximum of S * kd^-0.5;
//   pass 2  S again; p = exp(S * scale - max) (zero past the last key),
//           l += p; p split into bf16 hi + lo, written as A operands;
//           O += Ph Vh + Ph Vl + Pl Vh (3 products x 4 K steps, N 64).
// Then out = O / l + the positional depthwise term of v (layers.c:373-395,
// same summation order as the reference: bias, then taps ky, kx), split.
// The omitted lo x lo products are below 2^-16 of each term, the precision of
// the split format itself.  Tensor memory: S in columns [0, 64), O in
// [64, 128).  Operands are K-major without swizzle (core matrices of 8 rows
// x 16 bytes, 128 contiguous bytes each, row-group major).  One thread issues
// the UMMAs; completion is one mbarrier every thread waits on with a bound
// (a timeout sets the error word and ends the kernel after freeing TMEM).
#include <atomic>
#include <cfloat>
#include <cstdint>

#include "pdl.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "split.cuh"

namespace yb {
namespace {

constexpr int kTQ = 128;  // queries per CTA (UMMA M)
constexpr int kTK = 64;   // keys per block
constexpr uint32_t kOCol = kTK;  // TMEM column of O (S in [0, kTK))
constexpr uint32_t kTmemCols = kTK + 64 <= 128 ? 128u : 256u;
constexpr int TKD = 32, THD = 64;
constexpr int kErrAttnWaitF = 8;

__device__ __forceinline__ uint32_t opo(int row, int kbyte, int kb) {
  return static_cast<uint32_t>(((row >> 3) * (kb >> 4) + (kbyte >> 4)) * 128 + (row & 7) * 16 + (kbyte & 15));
}

struct AttnTcSmem {
  uint8_t qh[kTQ * TKD * 2], ql[kTQ * TKD * 2];    // A of S: 128 x 32 bf16
  uint8_t kh[kTK * TKD * 2], kl[kTK * TKD * 2];    // B of S: 64 keys x 32 bf16
  uint8_t vh[THD * kTK * 2], vl[THD * kTK * 2];    // B of O: 64 channels x 64 keys bf16
  uint8_t ph[kTQ * kTK * 2], pl[kTQ * kTK * 2];    // A of O: 128 queries x 64 keys bf16
  uint64_t bar;
  uint32_t tmem;
  int abort;
};

__global__ void __launch_bounds__(128, 3) attention_tc_kernel(const AttnArgs a, int* err) {
  extern __shared__ __align__(1024) uint8_t attn_tc_raw[];
  AttnTcSmem& S = *reinterpret_cast<AttnTcSmem*>(attn_tc_raw);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int N = a.H * a.W;
  const int q0 = blockIdx.x * kTQ, h = blockIdx.y, b = blockIdx.z;
  const int blk = 2 * TKD + THD;
  const uint16_t* base = a.qkv.hi + static_cast<long long>(b) * a.qkv.bstride + a.qkv.coff + h * blk;
  const long long pl = a.qkv.plane;
  pdl_wait();
  // Q rows, hi and lo planes (zero past N): 4 16-byte chunks per row each.
  for (int i = tid; i < kTQ * 4; i += 128) {
    const int r = i >> 2, c = i & 3;
    uint4 vh = make_uint4(0u, 0u, 0u, 0u), vl = vh;
    if (q0 + r < N) {
      const uint16_t* p = base + static_cast<long long>(q0 + r) * a.qkv.cstride + 8 * c;
      vh = *reinterpret_cast<const uint4*>(p);
      vl = *reinterpret_cast<const uint4*>(p + pl);
    }
    *reinterpret_cast<uint4*>(S.qh + opo(r, 16 * c, 2 * TKD)) = vh;
    *reinterpret_cast<uint4*>(S.ql + opo(r, 16 * c, 2 * TKD)) = vl;
  }
  if (tid == 0) {
    mbar_init(&S.bar, 1);
    S.abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&S.tmem, kTmemCols);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = S.tmem;
  const uint32_t trow = tbase + (static_cast<uint32_t>(warp * 32) << 16);
  volatile int* abort_flag = &S.abort;
  uint32_t phase = 0;
  bool ok = true;

  auto sync_async = [&]() {
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };
  // Keys [k0, k0 + kTK) into kh / kl (zero past N); with_v also V^T.
  auto stage = [&](int k0, bool with_v) {
    for (int i = tid; i < kTK * 4; i += 128) {
      const int j = i >> 2, c = i & 3;
      uint4 vh = make_uint4(0u, 0u, 0u, 0u), vl = vh;
      if (k0 + j < N) {
        const uint16_t* p = base + static_cast<long long>(k0 + j) * a.qkv.cstride + TKD + 8 * c;
        vh = *reinterpret_cast<const uint4*>(p);
        vl = *reinterpret_cast<const uint4*>(p + pl);
      }
      *reinterpret_cast<uint4*>(S.kh + opo(j, 16 * c, 2 * TKD)) = vh;
      *reinterpret_cast<uint4*>(S.kl + opo(j, 16 * c, 2 * TKD)) = vl;
    }
    if (with_v) {
      // Thread j < kTK transposes key j's 64 values into column j of V^T.
      const int j = tid;
      const bool in = k0 + j < N;
      const uint16_t* p = base + static_cast<long long>(in ? k0 + j : 0) * a.qkv.cstride + 2 * TKD;
#pragma unroll
      for (int c = 0; c < THD / 8; ++c) {
        if (j >= kTK) break;
        uint4 vh = make_uint4(0u, 0u, 0u, 0u), vl = vh;
        if (in) {
          vh = *reinterpret_cast<const uint4*>(p + 8 * c);
          vl = *reinterpret_cast<const uint4*>(p + 8 * c + pl);
        }
        const uint16_t* eh = reinterpret_cast<const uint16_t*>(&vh);
        const uint16_t* el = reinterpret_cast<const uint16_t*>(&vl);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint32_t o = opo(8 * c + e, 2 * j, 2 * kTK);
          *reinterpret_cast<uint16_t*>(S.vh + o) = eh[e];
          *reinterpret_cast<uint16_t*>(S.vl + o) = el[e];
        }
      }
    }
    sync_async();
  };
  auto wait_mma = [&]() {
    if (!ok) return;
    if (!mbar_wait(&S.bar, phase, abort_flag)) {
      *abort_flag = 1;
      if (err) atomicCAS(err, 0, kErrAttnWaitF);
      ok = false;
    }
    phase ^= 1u;
    tc_fence_after();
  };
  auto mma_scores = [&]() {
    if (tid == 0 && ok && !*abort_flag) {
      const uint32_t idesc = idesc_bf16_f32(kTQ, kTK);
      const uint32_t sbo = (2 * TKD / 16) * 128;
      const uint64_t qh = kmajor_desc_noswizzle(smem_u32(S.qh), 128, sbo);
      const uint64_t ql = kmajor_desc_noswizzle(smem_u32(S.ql), 128, sbo);
      const uint64_t kh = kmajor_desc_noswizzle(smem_u32(S.kh), 128, sbo);
      const uint64_t kl = kmajor_desc_noswizzle(smem_u32(S.kl), 128, sbo);
#pragma unroll
      for (int s = 0; s < TKD / 16; ++s) {
        const uint64_t off = static_cast<uint64_t>(16 * s);  // 16 bf16 = two core matrices = 256 bytes
        tc_mma_bf16(tbase, qh + off, kh + off, idesc, s == 0 ? 0u : 1u);
        tc_mma_bf16(tbase, qh + off, kl + off, idesc, 1u);
        tc_mma_bf16(tbase, ql + off, kh + off, idesc, 1u);
      }
      tc_commit(&S.bar);
    }
    wait_mma();
  };
  auto mma_values = [&](bool first) {
    if (tid == 0 && ok && !*abort_flag) {
      const uint32_t idesc = idesc_bf16_f32(kTQ, THD);
      const uint32_t sbo = (2 * kTK / 16) * 128;
      const uint64_t ph = kmajor_desc_noswizzle(smem_u32(S.ph), 128, sbo);
      const uint64_t plo = kmajor_desc_noswizzle(smem_u32(S.pl), 128, sbo);
      const uint64_t vh = kmajor_desc_noswizzle(smem_u32(S.vh), 128, sbo);
      const uint64_t vl = kmajor_desc_noswizzle(smem_u32(S.vl), 128, sbo);
#pragma unroll
      for (int s = 0; s < kTK / 16; ++s) {
        const uint64_t off = static_cast<uint64_t>(16 * s);
        tc_mma_bf16(tbase + kOCol, ph + off, vh + off, idesc, (first && s == 0) ? 0u : 1u);
        tc_mma_bf16(tbase + kOCol, ph + off, vl + off, idesc, 1u);
        tc_mma_bf16(tbase + kOCol, plo + off, vh + off, idesc, 1u);
      }
      tc_commit(&S.bar);
    }
    wait_mma();
  };

  // Pass 1: row maximum of the scaled scores.
  float mx = -FLT_MAX;
  for (int k0 = 0; k0 < N; k0 += kTK) {
    stage(k0, false);
    mma_scores();
#pragma unroll
    for (int cc = 0; cc < kTK; cc += 16) {
      uint32_t r[16];
      tc_ld_32x32b_x16(trow + cc, r);
      tc_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (k0 + cc + e < N) mx = fmaxf(mx, __uint_as_float(r[e]) * a.scale);
    }
    tc_fence_before();
  }
  // Pass 2: weights, their sum, and O.
  float l = 0.f;
  for (int k0 = 0; k0 < N; k0 += kTK) {
    __syncthreads();  // the previous block's UMMAs have completed (waited)
    stage(k0, true);
    mma_scores();
#pragma unroll
    for (int cc = 0; cc < kTK; cc += 16) {
      uint32_t r[16];
      tc_ld_32x32b_x16(trow + cc, r);
      tc_wait_ld();
      uint32_t hw[8], lw[8];
#pragma unroll
      for (int e = 0; e < 16; e += 2) {
        const float p0 = k0 + cc + e < N ? __expf(__uint_as_float(r[e]) * a.scale - mx) : 0.f;
        const float p1 = k0 + cc + e + 1 < N ? __expf(__uint_as_float(r[e + 1]) * a.scale - mx) : 0.f;
        l += p0;
        l += p1;
        split2(p0, p1, hw[e >> 1], lw[e >> 1]);
      }
      *reinterpret_cast<uint4*>(S.ph + opo(tid, 2 * cc, 2 * kTK)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(S.ph + opo(tid, 2 * cc + 16, 2 * kTK)) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
      *reinterpret_cast<uint4*>(S.pl + opo(tid, 2 * cc, 2 * kTK)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      *reinterpret_cast<uint4*>(S.pl + opo(tid, 2 * cc + 16, 2 * kTK)) = make_uint4(lw[4], lw[5], lw[6], lw[7]);
    }
    sync_async();
    mma_values(k0 == 0);
  }
  __syncthreads();
  const bool good = S.abort == 0;
  const int qi = q0 + tid;
  const bool valid = qi < N && good;
  const float inv = l > 1e-12f ? 1.0f / l : 1.0f;
  const int y = qi / a.W, x = qi - (qi / a.W) * a.W;
  uint16_t* op = a.out.hi + static_cast<long long>(b) * a.out.bstride + static_cast<long long>(qi) * a.out.cstride +
                 a.out.coff + h * THD;
  for (int d0 = 0; d0 < THD; d0 += 16) {
    uint32_t ov[16];
    tc_ld_32x32b_x16(trow + kOCol + d0, ov);
    tc_wait_ld();
    if (!valid) continue;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int dd = d0 + 8 * half;
      const int ch = h * THD + dd;
      float pe[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) pe[e] = __ldg(a.pe_b + ch + e);
      for (int ky = 0; ky < 3; ++ky) {
        const int iy = y - 1 + ky;
        if (iy < 0 || iy >= a.H) continue;
        for (int kx = 0; kx < 3; ++kx) {
          const int ix = x - 1 + kx;
          if (ix < 0 || ix >= a.W) continue;
          float v[8];
          load8(base + static_cast<long long>(iy * a.W + ix) * a.qkv.cstride + 2 * TKD + dd, pl, v);
          const float* w = a.pe_w + (ky * 3 + kx) * (a.heads * THD) + ch;
#pragma unroll
          for (int e = 0; e < 8; ++e) pe[e] = __fadd_rn(pe[e], __fmul_rn(v[e], __ldg(w + e)));
        }
      }
      float res[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) res[e] = __uint_as_float(ov[8 * half + e]) * inv + pe[e];
      store8(op + dd, a.out.plane, res);
    }
  }
  if (!good) __nanosleep(100000);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Wide variant for N <= kWideNF keys (the 20 x 20 PSA of a 640 x 640 input):
// 512 threads in four warpgroups.  Q, K and V^T (hi and lo planes) are staged
// once; S for all keys goes to TMEM columns [0, Np) in one pass (N <= 256 per
// UMMA); the warpgroups reduce quarters of the columns to the row maximum.
// P then streams in chunks of 64 keys through two shared-memory slots laid
// over the dead Q and K: every warpgroup writes 16 of a chunk's columns, one
// thread issues the chunk's 12 UMMAs (Ph Vh + Ph Vl + Pl Vh, 4 K steps) into
// O at TMEM columns [0, 64) (chunk 0's scores, read by then) and commits to
// the slot's barrier, which the writers of the chunk two ahead wait on.
// Each warpgroup finishes 16 of the 64 output channels.
constexpr int kWideNF = 448;
constexpr int kWideTF = 512;
constexpr int kChunkF = 64;
constexpr uint32_t kSlotBytes = kTQ * kChunkF * 2;  // one plane of one P chunk

struct AttnWideTcSmem {
  union {
    struct {
      uint8_t qh[kTQ * TKD * 2], ql[kTQ * TKD * 2];
      uint8_t kh[kWideNF * TKD * 2], kl[kWideNF * TKD * 2];
    } s;
    uint8_t p[2][2][kSlotBytes];  // [slot][hi, lo]: 128 x 64 bf16
  } u;
  uint8_t vh[THD * kWideNF * 2 + 128], vl[THD * kWideNF * 2 + 128];  // V^T row groups 16 Np + 16 bytes apart
  float red_max[4][kTQ];
  float red_sum[4][kTQ];
  float pew[9][THD];  // positional weights of this head, [tap][channel]
  float peb[THD];
  uint64_t bar;
  uint64_t slot_bar[2];
  uint32_t tmem;
  int abort;
};

__global__ void __launch_bounds__(kWideTF, 1) attention_wide_tc_kernel(const AttnArgs a, int* err) {
  extern __shared__ __align__(1024) uint8_t attn_wtc_raw[];
  AttnWideTcSmem& S = *reinterpret_cast<AttnWideTcSmem*>(attn_wtc_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = warp >> 2;
  const int row = (warp & 3) * 32 + lane;
  const int N = a.H * a.W;
  const int Np = (N + 63) & ~63;
  const int Nq = Np >> 2;
  const int q0 = blockIdx.x * kTQ, h = blockIdx.y, b = blockIdx.z;
  const int blk = 2 * TKD + THD;
  const uint16_t* base = a.qkv.hi + static_cast<long long>(b) * a.qkv.bstride + a.qkv.coff + h * blk;
  const long long pl = a.qkv.plane;
  for (int i = tid; i < 9 * THD; i += kWideTF) S.pew[i / THD][i % THD] = a.pe_w[(i / THD) * (a.heads * THD) + h * THD + i % THD];
  for (int i = tid; i < THD; i += kWideTF) S.peb[i] = a.pe_b[h * THD + i];
  if (tid == 0) {
    mbar_init(&S.bar, 1);
    mbar_init(&S.slot_bar[0], 1);
    mbar_init(&S.slot_bar[1], 1);
    S.abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&S.tmem, 512);
    tmem_relinquish();
  }
  pdl_wait();
  // Q and K rows: 16-byte asynchronous copies of each plane straight into
  // the K-major operand layout (zero past N).
  auto copy16 = [](void* dst, const uint16_t* src, bool in) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(in ? 16u : 0u)
                 : "memory");
  };
  for (int i = tid; i < kTQ * 4; i += kWideTF) {
    const int r = i >> 2, c = i & 3;
    const bool in = q0 + r < N;
    const uint16_t* p = base + static_cast<long long>(in ? q0 + r : 0) * a.qkv.cstride + 8 * c;
    copy16(S.u.s.qh + opo(r, 16 * c, 2 * TKD), p, in);
    copy16(S.u.s.ql + opo(r, 16 * c, 2 * TKD), p + pl, in);
  }
  for (int i = tid; i < Np * 4; i += kWideTF) {
    const int j = i >> 2, c = i & 3;
    const bool in = j < N;
    const uint16_t* p = base + static_cast<long long>(in ? j : 0) * a.qkv.cstride + TKD + 8 * c;
    copy16(S.u.s.kh + opo(j, 16 * c, 2 * TKD), p, in);
    copy16(S.u.s.kl + opo(j, 16 * c, 2 * TKD), p + pl, in);
  }
  // V^T: item i = key pair i >> 3 (keys 2 jp, 2 jp + 1) x 8 channels
  // 8 (i & 7) .. + 7; each channel's two keys become one 32-bit word.  The
  // row groups of 8 channels are 16 Np + 16 bytes apart, so that the stores
  // of a warp (8 channel groups x 4 key pairs) fall in distinct banks.  Two
  // items' loads in flight per thread.
  const uint32_t vsbo = static_cast<uint32_t>(16 * Np + 16);
  const int nv = (Np / 2) * 8;
  for (int i0 = tid; i0 < nv; i0 += 2 * kWideTF) {
    uint4 v[2][4];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = i0 + u * kWideTF;
      const int jp = i >> 3, c8 = i & 7;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int j = 2 * jp + k;
        v[u][2 * k] = v[u][2 * k + 1] = make_uint4(0u, 0u, 0u, 0u);
        if (i < nv && j < N) {
          const uint16_t* p = base + static_cast<long long>(j) * a.qkv.cstride + 2 * TKD + 8 * c8;
          v[u][2 * k] = *reinterpret_cast<const uint4*>(p);
          v[u][2 * k + 1] = *reinterpret_cast<const uint4*>(p + pl);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = i0 + u * kWideTF;
      if (i >= nv) continue;
      const int jp = i >> 3, c8 = i & 7;
      const uint32_t col = static_cast<uint32_t>((jp >> 2) * 128 + (jp & 3) * 4);  // keys 2 jp, 2 jp + 1
#pragma unroll
      for (int pln = 0; pln < 2; ++pln) {
        const uint4 ka = v[u][pln], kb = v[u][2 + pln];  // key 2 jp, key 2 jp + 1
        const uint32_t wa[4] = {ka.x, ka.y, ka.z, ka.w}, wb[4] = {kb.x, kb.y, kb.z, kb.w};
        uint8_t* vt = (pln == 0 ? S.vh : S.vl) + c8 * vsbo + col;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          // Channel 8 c8 + e: its bf16 of key 2 jp (low half) and 2 jp + 1.
          const uint32_t w = __byte_perm(wa[e >> 1], wb[e >> 1], (e & 1) ? 0x7632 : 0x5410);
          *reinterpret_cast<uint32_t*>(vt + e * 16) = w;
        }
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = S.tmem;
  const uint32_t trow = tbase + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  volatile int* abort_flag = &S.abort;
  bool ok = true;
  auto wait_bar = [&](uint64_t* bar, uint32_t parity) {
    if (!ok) return;
    if (!mbar_wait(bar, parity, abort_flag)) {
      *abort_flag = 1;
      if (err) atomicCAS(err, 0, kErrAttnWaitF);
      ok = false;
    }
    tc_fence_after();
  };
  // S = Q K^T, all keys.
  if (tid == 0) {
    const uint32_t sbo = (2 * TKD / 16) * 128;
    const uint64_t qh = kmajor_desc_noswizzle(smem_u32(S.u.s.qh), 128, sbo);
    const uint64_t ql = kmajor_desc_noswizzle(smem_u32(S.u.s.ql), 128, sbo);
    for (int k0 = 0; k0 < Np; k0 += 256) {
      const int nb = Np - k0 < 256 ? Np - k0 : 256;
      const uint32_t idesc = idesc_bf16_f32(kTQ, nb);
      const uint32_t ko = static_cast<uint32_t>(k0 / 8) * sbo;
      const uint64_t kh = kmajor_desc_noswizzle(smem_u32(S.u.s.kh) + ko, 128, sbo);
      const uint64_t kl = kmajor_desc_noswizzle(smem_u32(S.u.s.kl) + ko, 128, sbo);
      const uint32_t d = tbase + static_cast<uint32_t>(k0);
#pragma unroll
      for (int st = 0; st < TKD / 16; ++st) {
        const uint64_t off = static_cast<uint64_t>(16 * st);
        tc_mma_bf16(d, qh + off, kh + off, idesc, st == 0 ? 0u : 1u);
        tc_mma_bf16(d, qh + off, kl + off, idesc, 1u);
        tc_mma_bf16(d, ql + off, kh + off, idesc, 1u);
      }
    }
    tc_commit(&S.bar);
  }
  // While the score UMMAs run: the positional term of this row's 16
  // channels (bias, then taps in (ky, kx) order, the reference's summation),
  // a depthwise 3x3 of v around the query read from global memory.
  const int qi = q0 + row;
  const int y = qi / a.W, x = qi - (qi / a.W) * a.W;
  const int d0 = 16 * g;
  float pe[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) pe[e] = S.peb[d0 + e];
  if (qi < N) {
    // One filter row at a time: its three pixels' loads (both planes, 16
    // channels) in flight together; taps outside the image are skipped, in
    // the reference's (ky, kx) order.
#pragma unroll
    for (int ky = 0; ky < 3; ++ky) {
      const int iy = y - 1 + ky;
      if (iy < 0 || iy >= a.H) continue;
      uint4 raw[3][4];
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        const int ix = x - 1 + kx;
        const bool in = ix >= 0 && ix < a.W;
        const uint16_t* vp = base + static_cast<long long>(iy * a.W + (in ? ix : x)) * a.qkv.cstride + 2 * TKD + d0;
        raw[kx][0] = *reinterpret_cast<const uint4*>(vp);
        raw[kx][1] = *reinterpret_cast<const uint4*>(vp + pl);
        raw[kx][2] = *reinterpret_cast<const uint4*>(vp + 8);
        raw[kx][3] = *reinterpret_cast<const uint4*>(vp + 8 + pl);
      }
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        const int ix = x - 1 + kx;
        if (ix < 0 || ix >= a.W) continue;
        const float* w = S.pew[ky * 3 + kx] + d0;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const uint4 h = raw[kx][2 * hf], l = raw[kx][2 * hf + 1];
          const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, lw[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int e = 8 * hf + 2 * q;
            const float v0 = bf16_bits_to_f(hw[q] & 0xFFFFu) + bf16_bits_to_f(lw[q] & 0xFFFFu);
            const float v1 = bf16_bits_to_f(hw[q] >> 16) + bf16_bits_to_f(lw[q] >> 16);
            pe[e] = __fadd_rn(pe[e], __fmul_rn(v0, w[e]));
            pe[e + 1] = __fadd_rn(pe[e + 1], __fmul_rn(v1, w[e + 1]));
          }
        }
      }
    }
  }
  wait_bar(&S.bar, 0u);
  // Row maximum of the scaled scores over this warpgroup's quarter.
  float mx = -FLT_MAX;
  for (int cc = 0; cc < Nq; cc += 16) {
    uint32_t r[16];
    tc_ld_32x32b_x16(trow + static_cast<uint32_t>(g * Nq + cc), r);
    tc_wait_ld();
#pragma unroll
    for (int e = 0; e < 16; ++e)
      if (g * Nq + cc + e < N) mx = fmaxf(mx, __uint_as_float(r[e]) * a.scale);
  }
  S.red_max[g][row] = mx;
  __syncthreads();  // also: Q and K are dead from here (their UMMAs completed)
  mx = fmaxf(fmaxf(S.red_max[0][row], S.red_max[1][row]), fmaxf(S.red_max[2][row], S.red_max[3][row]));
  // P in chunks of 64 keys, 16 columns per warpgroup; O += P V per chunk.
  float l = 0.f;
  const int nchunks = Np / kChunkF;
  for (int c = 0; c < nchunks; ++c) {
    const int slot = c & 1;
    if (c >= 2) wait_bar(&S.slot_bar[slot], static_cast<uint32_t>(((c >> 1) - 1) & 1));
    const int col = c * kChunkF + 16 * g;
    uint32_t r[16];
    tc_ld_32x32b_x16(trow + static_cast<uint32_t>(col), r);
    tc_wait_ld();
    uint32_t hw[8], lw[8];
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
      const float p0 = col + e < N ? __expf(__uint_as_float(r[e]) * a.scale - mx) : 0.f;
      const float p1 = col + e + 1 < N ? __expf(__uint_as_float(r[e + 1]) * a.scale - mx) : 0.f;
      l += p0;
      l += p1;
      split2(p0, p1, hw[e >> 1], lw[e >> 1]);
    }
    uint8_t* ph = S.u.p[slot][0];
    uint8_t* plo = S.u.p[slot][1];
    *reinterpret_cast<uint4*>(ph + opo(row, 32 * g, 2 * kChunkF)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(ph + opo(row, 32 * g + 16, 2 * kChunkF)) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
    *reinterpret_cast<uint4*>(plo + opo(row, 32 * g, 2 * kChunkF)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    *reinterpret_cast<uint4*>(plo + opo(row, 32 * g + 16, 2 * kChunkF)) = make_uint4(lw[4], lw[5], lw[6], lw[7]);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0 && ok && !*abort_flag) {
      const uint32_t idesc = idesc_bf16_f32(kTQ, THD);
      const uint32_t psbo = (2 * kChunkF / 16) * 128;
      const uint64_t dph = kmajor_desc_noswizzle(smem_u32(ph), 128, psbo);
      const uint64_t dpl = kmajor_desc_noswizzle(smem_u32(plo), 128, psbo);
      const uint32_t vo = static_cast<uint32_t>(c) * 1024u;  // 64 keys = 8 core matrices along K
      const uint64_t dvh = kmajor_desc_noswizzle(smem_u32(S.vh) + vo, 128, vsbo);
      const uint64_t dvl = kmajor_desc_noswizzle(smem_u32(S.vl) + vo, 128, vsbo);
#pragma unroll
      for (int st = 0; st < kChunkF / 16; ++st) {
        const uint64_t off = static_cast<uint64_t>(16 * st);
        tc_mma_bf16(tbase, dph + off, dvh + off, idesc, (c == 0 && st == 0) ? 0u : 1u);
        tc_mma_bf16(tbase, dph + off, dvl + off, idesc, 1u);
        tc_mma_bf16(tbase, dpl + off, dvh + off, idesc, 1u);
      }
      tc_commit(&S.slot_bar[slot]);
    }
  }
  // The last chunk's UMMAs (and with them every earlier one) have completed.
  wait_bar(&S.slot_bar[(nchunks - 1) & 1], static_cast<uint32_t>(((nchunks - 1) >> 1) & 1));
  S.red_sum[g][row] = l;
  __syncthreads();
  const bool good = S.abort == 0;
  const bool valid = qi < N && good;
  l = S.red_sum[0][row] + S.red_sum[1][row] + S.red_sum[2][row] + S.red_sum[3][row];
  const float inv = l > 1e-12f ? 1.0f / l : 1.0f;
  uint32_t ov[16];
  tc_ld_32x32b_x16(trow + static_cast<uint32_t>(d0), ov);
  tc_wait_ld();
  if (valid) {
    uint16_t* op = a.out.hi + static_cast<long long>(b) * a.out.bstride + static_cast<long long>(qi) * a.out.cstride +
                   a.out.coff + h * THD;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float res[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) res[e] = __uint_as_float(ov[8 * half + e]) * inv + pe[8 * half + e];
      store8(op + d0 + 8 * half, a.out.plane, res);
    }
  }
  if (!good) __nanosleep(100000);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

}  // namespace

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s) {
  const int N = a.H * a.W;
  if (a.kd != TKD || a.hd != THD || N < 1 || a.qkv.cstride % 8 || a.out.cstride % 8 || a.qkv.coff % 8 ||
      a.out.coff % 8 || a.qkv.bstride % 8 || a.out.bstride % 8 || a.qkv.plane % 8 || a.out.plane % 8 ||
      reinterpret_cast<uintptr_t>(a.qkv.hi) % 16 || reinterpret_cast<uintptr_t>(a.out.hi) % 16)
    return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_done{0};
  const cudaError_t e = smem_attr_once(attention_tc_kernel, static_cast<int>(sizeof(AttnTcSmem)), attr_done);
  if (e != cudaSuccess) return e;
  dim3 grid((N + kTQ - 1) / kTQ, a.heads, a.B);
  if (N <= kWideNF) {
    static std::atomic<uint64_t> wide_done{0};
    const cudaError_t e2 =
        smem_attr_once(attention_wide_tc_kernel, static_cast<int>(sizeof(AttnWideTcSmem)), wide_done);
    if (e2 != cudaSuccess) return e2;
    return launch_pdl(attention_wide_tc_kernel, grid, dim3(kWideTF), sizeof(AttnWideTcSmem), s, a, a.err);
  }
  return launch_pdl(attention_tc_kernel, grid, dim3(128), sizeof(AttnTcSmem), s, a, a.err);
}

}  // namespace yb
