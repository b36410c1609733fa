// PSA attention of the INT8 forward (layers.c:310-405 for the graph; the
// integer softmax rules are in i8k.h) with both contractions on the
// tensor cores: tcgen05.mma kind::i8, int32 accumulation in tensor memory.
//
// One CTA of 128 threads per (128 queries, head, image); thread i owns query
// row i (TMEM lane i).  Keys go in blocks of 128:
//   pass 1  S = Q K^T (one UMMA, M 128, N 128, K 32) -> row maximum;
//   pass 2  S again -> t = min(255, rne((max - S) * mt, sht)), p = E[t],
//           l += p, and p split into ph = p >> 6 (0..64) and pl = p & 63,
//           written as int8 A operands; O_h += Ph V, O_l += Pl V (4 UMMAs of
//           K 32 each, N 64).  o = 64 O_h + O_l is exact: |o| <= N 4096 127.
// Then out = div_rne(rne(o * mo, sho), l) + the positional depthwise term,
// clamped.  Tensor memory: S in columns [0, 128), O_h [128, 192), O_l
// [192, 256).  Operands are K-major without swizzle: core matrices of 8 rows
// x 16 bytes, 128 contiguous bytes each, row-group major.  One elected thread
// issues the UMMAs; completion is a tcgen05.commit on one mbarrier that every
// thread waits on with a bound (a timeout sets the error word and ends the
// kernel after freeing tensor memory).
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdint>

#include "pdl.cuh"
#include "i8k.h"
#include "sm100.cuh"

namespace yb {
namespace {

constexpr int kAQ = 128;  // queries per CTA (UMMA M)
constexpr int kAK = 128;  // keys per block
constexpr int KD = 32, HD = 64;
constexpr int kErrAttnWait = 7;

// Byte offset of (row, k) in a K-major no-swizzle operand whose rows hold
// kb bytes: core matrix (row / 8, k / 16), 128 bytes each, row-group major.
__device__ __forceinline__ uint32_t ops_off(int row, int k, int kb) {
  return static_cast<uint32_t>(((row >> 3) * (kb >> 4) + (k >> 4)) * 128 + (row & 7) * 16 + (k & 15));
}

// Load from a shared-memory table that no longer changes (free to schedule).
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ long long rne64(long long p, int sh) {
  return (p + ((1LL << (sh - 1)) - 1) + ((p >> sh) & 1)) >> sh;
}
// a / l rounded half to even (l > 0), floor-based for negative a.
__device__ __forceinline__ long long div_rne64(long long a, long long l) {
  long long q = a / l, r = a % l;
  if (r < 0) {
    q -= 1;
    r += l;
  }
  if (2 * r > l || (2 * r == l && (q & 1))) q += 1;
  return q;
}

struct AttnSmem {
  uint8_t q[kAQ * KD];        // A of S: 128 x 32
  uint8_t k[kAK * KD];        // B of S: 128 keys x 32
  uint8_t vt[HD * kAK];       // B of O: 64 channels x 128 keys
  uint8_t ph[kAQ * kAK];      // A of O_h: 128 queries x 128 keys
  uint8_t pl[kAQ * kAK];      // A of O_l
  int32_t E[256];
  int8_t pe[9 * HD];          // positional weights of this head, [tap][d]
  uint64_t bar;
  uint32_t tmem;
  int abort;
};

__global__ void __launch_bounds__(128, 1) attention_i8_tc_kernel(const I8AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t attn_smem_raw[];
  AttnSmem& S = *reinterpret_cast<AttnSmem*>(attn_smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int N = a.H * a.W;
  const int q0 = blockIdx.x * kAQ, h = blockIdx.y, b = blockIdx.z;
  const int blk = 2 * KD + HD;
  const int8_t* base = a.qkv.p + static_cast<long long>(b) * a.qkv.bstride + h * blk;
  for (int i = tid; i < 256; i += 128) S.E[i] = a.E[i];
  for (int i = tid; i < 9 * HD; i += 128) S.pe[i] = a.pe_w[(i / HD) * a.dim + h * HD + i % HD];
  pdl_wait();
  // Q rows (zero past N), two 16-byte chunks per row.
  for (int i = tid; i < kAQ * 2; i += 128) {
    const int r = i >> 1, c = i & 1;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (q0 + r < N) v = *reinterpret_cast<const uint4*>(base + static_cast<long long>(q0 + r) * a.qkv.cstride + 16 * c);
    *reinterpret_cast<uint4*>(S.q + ops_off(r, 16 * c, KD)) = v;
  }
  if (tid == 0) {
    mbar_init(&S.bar, 1);
    S.abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&S.tmem, 256);
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

  // Keys [k0, k0 + 128) into S.k (zero past N); with_v also V^T into S.vt.
  auto stage = [&](int k0, bool with_v) {
    for (int i = tid; i < kAK * 2; i += 128) {
      const int j = i >> 1, c = i & 1;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (k0 + j < N)
        v = *reinterpret_cast<const uint4*>(base + static_cast<long long>(k0 + j) * a.qkv.cstride + KD + 16 * c);
      *reinterpret_cast<uint4*>(S.k + ops_off(j, 16 * c, KD)) = v;
    }
    if (with_v) {
      // Thread j transposes key j's 64 values into column j of V^T.
      const int j = tid;
      uint4 vv[4] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u),
                     make_uint4(0u, 0u, 0u, 0u)};
      if (k0 + j < N) {
        const uint4* vp = reinterpret_cast<const uint4*>(base + static_cast<long long>(k0 + j) * a.qkv.cstride + 2 * KD);
#pragma unroll
        for (int c = 0; c < 4; ++c) vv[c] = vp[c];
      }
      const uint8_t* vb = reinterpret_cast<const uint8_t*>(vv);
#pragma unroll
      for (int d = 0; d < HD; ++d) S.vt[ops_off(d, j, kAK)] = vb[d];
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };
  auto wait_mma = [&]() {
    if (!ok) return;
    if (!mbar_wait(&S.bar, phase, abort_flag)) {
      *abort_flag = 1;
      if (a.err) atomicCAS(a.err, 0, kErrAttnWait);
      ok = false;
    }
    phase ^= 1u;
    tc_fence_after();
  };
  auto mma_scores = [&]() {
    if (tid == 0 && ok && !*abort_flag) {
      const uint64_t da = kmajor_desc_noswizzle(smem_u32(S.q), 128, (KD / 16) * 128);
      const uint64_t db = kmajor_desc_noswizzle(smem_u32(S.k), 128, (KD / 16) * 128);
      tc_mma_i8(tbase, da, db, idesc_s8_s32(kAQ, kAK), 0u);
      tc_commit(&S.bar);
    }
    wait_mma();
  };
  auto mma_values = [&](bool first) {
    if (tid == 0 && ok && !*abort_flag) {
      const uint32_t idesc = idesc_s8_s32(kAQ, HD);
      const uint64_t dh = kmajor_desc_noswizzle(smem_u32(S.ph), 128, (kAK / 16) * 128);
      const uint64_t dl = kmajor_desc_noswizzle(smem_u32(S.pl), 128, (kAK / 16) * 128);
      const uint64_t dv = kmajor_desc_noswizzle(smem_u32(S.vt), 128, (kAK / 16) * 128);
#pragma unroll
      for (int s = 0; s < kAK / 32; ++s) {
        // 32 keys = two core matrices = 256 bytes = 16 descriptor units.
        const uint64_t off = static_cast<uint64_t>(16 * s);
        const uint32_t acc = (first && s == 0) ? 0u : 1u;
        tc_mma_i8(tbase + 128, dh + off, dv + off, idesc, acc);
        tc_mma_i8(tbase + 192, dl + off, dv + off, idesc, acc);
      }
      tc_commit(&S.bar);
    }
    wait_mma();
  };

  // Pass 1: row maximum of the integer scores.
  int mx = INT_MIN;
  for (int k0 = 0; k0 < N; k0 += kAK) {
    stage(k0, false);
    mma_scores();
#pragma unroll
    for (int cc = 0; cc < kAK; cc += 16) {
      uint32_t r[16];
      tc_ld_32x32b_x16(trow + cc, r);
      tc_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (k0 + cc + e < N) mx = max(mx, static_cast<int>(r[e]));
    }
    tc_fence_before();
  }
  // Pass 2: weights, their sum, and the two value products.
  int l = 0;
  for (int k0 = 0; k0 < N; k0 += kAK) {
    __syncthreads();  // the previous block's UMMAs have completed (waited)
    stage(k0, true);
    mma_scores();
#pragma unroll
    for (int cc = 0; cc < kAK; cc += 16) {
      uint32_t r[16];
      tc_ld_32x32b_x16(trow + cc, r);
      tc_wait_ld();
      uint32_t hw[4] = {0u, 0u, 0u, 0u}, lw[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        int p = 0;
        if (k0 + cc + e < N) {
          const long long t = rne64(static_cast<long long>(mx - static_cast<int>(r[e])) * a.mt, a.sht);
          p = S.E[t > 255 ? 255 : t];
        }
        l += p;
        hw[e >> 2] |= static_cast<uint32_t>(p >> 6) << (8 * (e & 3));
        lw[e >> 2] |= static_cast<uint32_t>(p & 63) << (8 * (e & 3));
      }
      *reinterpret_cast<uint4*>(S.ph + ops_off(tid, cc, kAK)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(S.pl + ops_off(tid, cc, kAK)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    mma_values(k0 == 0);
  }
  __syncthreads();
  const bool good = S.abort == 0;
  const int qi = q0 + tid;
  const bool valid = qi < N && good;
  const int y = qi / a.W, x = qi - (qi / a.W) * a.W;
  int8_t* op = a.out.p + static_cast<long long>(b) * a.out.bstride + static_cast<long long>(qi) * a.out.cstride +
               h * HD;
  for (int d0 = 0; d0 < HD; d0 += 16) {
    uint32_t oh[16], ol[16];
    tc_ld_32x32b_x16(trow + 128 + d0, oh);
    tc_ld_32x32b_x16(trow + 192 + d0, ol);
    tc_wait_ld();
    if (!valid) continue;
    // Positional term: depthwise 3x3 of v (channels h*HD + d) around the query.
    int acc[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[e] = 0;
    for (int tap = 0; tap < 9; ++tap) {
      const int iy = y - 1 + tap / 3, ix = x - 1 + tap % 3;
      if (iy < 0 || iy >= a.H || ix < 0 || ix >= a.W) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(base + static_cast<long long>(iy * a.W + ix) * a.qkv.cstride +
                                                      2 * KD + d0);
      const int8_t* vb = reinterpret_cast<const int8_t*>(&v);
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[e] += static_cast<int>(vb[e]) * static_cast<int>(S.pe[tap * HD + d0 + e]);
    }
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int ch = h * HD + d0 + e;
      const long long o = 64LL * static_cast<int32_t>(oh[e]) + static_cast<int32_t>(ol[e]);
      const long long av = div_rne64(rne64(o * a.mo, a.sho), l);
      const long long pe = rne64((static_cast<long long>(acc[e]) + a.pe_bq[ch]) * a.pe_mult[ch], a.pe_shift[ch]);
      const long long v = av + pe;
      const int c = static_cast<int>(v < -127 ? -127 : v > 127 ? 127 : v);
      w[e >> 2] |= (static_cast<uint32_t>(c) & 0xFFu) << (8 * (e & 3));
    }
    *reinterpret_cast<uint4*>(op + d0) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (!good) __nanosleep(100000);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 256);
  }
}

// ---------------------------------------------------------------------------
// Wide variant for N <= kWideN keys (the 20 x 20 PSA of a 640 x 640 input):
// 512 threads, four warpgroups splitting the key columns, and every phase
// done once.  Q, K and V^T are staged once; S for all keys is computed by one
// or two UMMAs (N <= 256 each) into TMEM columns [0, Np); each warpgroup
// reduces its quarter of the columns to a row maximum, then writes its
// quarter of P = Ph, Pl (int8, shared memory) and its part of l; one thread
// issues O_h += Ph V, O_l += Pl V over all keys (K 32 per UMMA) into TMEM
// columns [0, 128), which S no longer needs; each warpgroup finishes 16 of
// the 64 output channels.  Same integer rules as the kernel above, with two
// exact shortcuts:
//   t   the product d * mt / 2^sht in fp32 (d < 2^21 is exact, the error is
//       below 2^-15 for values up to 256) rounded to nearest even decides t
//       unless it lies within 2^-14 of a half-integer; then the 64-bit rule;
//   div the quotient from a double reciprocal of l, corrected by the integer
//       remainder (and the 64-bit division if it is off by more than 2).
constexpr int kWideN = 512;
constexpr int kWideThreads = 512;

struct AttnWideSmem {
  uint8_t q[kAQ * KD];
  uint8_t k[kWideN * KD];
  uint8_t vt[HD * kWideN];
  uint8_t ph[kAQ * kWideN];
  uint8_t pl[kAQ * kWideN];
  uint32_t E3[257];        // E[t] as (E >> 6) | (E & 63) << 16; E3[256] = 0 (keys past N)
  alignas(16) uint32_t pw[HD][4];  // positional weights of this head per channel: taps 0-3, 4-7, 8
  int32_t pq[3][HD];       // positional bias, multiplier, shift of this head
  int32_t red_max[4][kAQ];
  int32_t red_sum[4][kAQ];  // packed: sum (p >> 6) in the low half, sum (p & 63) in the high half
  uint64_t bar;
  uint32_t tmem;
  int abort;
};

// div_rne64(a, l) for l >= 1 without 64-bit division or fp64 conversions:
// when |a| < 2^30 the fp32 estimate of a / l (relative error below 3 * 2^-24,
// so within one of the floor once l >= 192; attention rows have l >= 4096)
// is corrected once by the exact 32-bit remainder; anything else takes the
// 64-bit rule.
__device__ __forceinline__ long long div_rne_q(long long a, int l, float rlf) {
  if (a > -(1LL << 30) && a < (1LL << 30)) {
    const int ai = static_cast<int>(a);
    int q = __float2int_rd(__fmul_rn(__int2float_rn(ai), rlf));
    int r = ai - q * l;
    if (r < 0) {
      --q;
      r += l;
    } else if (r >= l) {
      ++q;
      r -= l;
    }
    if (r >= 0 && r < l) {
      if (2 * r > l || (2 * r == l && (q & 1))) ++q;
      return q;
    }
  }
  return div_rne64(a, l);
}

// Byte transpose of four words: y[e] byte k = byte e of word k.
__device__ __forceinline__ void transpose4w(uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t (&y)[4]) {
  const uint32_t t0 = __byte_perm(a, b, 0x5140), t1 = __byte_perm(a, b, 0x7362);
  const uint32_t t2 = __byte_perm(c, d, 0x5140), t3 = __byte_perm(c, d, 0x7362);
  y[0] = __byte_perm(t0, t2, 0x5410);
  y[1] = __byte_perm(t0, t2, 0x7632);
  y[2] = __byte_perm(t1, t3, 0x5410);
  y[3] = __byte_perm(t1, t3, 0x7632);
}

__global__ void __launch_bounds__(kWideThreads, 1) attention_i8_wide_kernel(const I8AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t attn_wide_raw[];
  AttnWideSmem& S = *reinterpret_cast<AttnWideSmem*>(attn_wide_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = warp >> 2;                 // warpgroup: quarter of the key columns / channels
  const int row = (warp & 3) * 32 + lane;  // query row = TMEM lane
  const int N = a.H * a.W;
  const int Np = (N + 63) & ~63;  // keys padded to 64 (quarters of 16-column loads)
  const int Nq = Np >> 2;
  const int q0 = blockIdx.x * kAQ, h = blockIdx.y, b = blockIdx.z;
  const int blk = 2 * KD + HD;
  const int8_t* base = a.qkv.p + static_cast<long long>(b) * a.qkv.bstride + h * blk;
  // Constants of this head (not written by earlier kernels): before pdl_wait.
  for (int i = tid; i < 257; i += kWideThreads) {
    const int e = i < 256 ? a.E[i] : 0;
    S.E3[i] = static_cast<uint32_t>(e >> 6) | (static_cast<uint32_t>(e & 63) << 16);
  }
  for (int i = tid; i < HD * 3; i += kWideThreads) {
    const int d = i / 3, wv = i - (i / 3) * 3;  // word wv: taps 4wv .. 4wv+3 (tap 8 alone)
    uint32_t word = 0u;
    for (int k = 0; k < 4 && 4 * wv + k < 9; ++k)
      word |= (static_cast<uint32_t>(a.pe_w[(4 * wv + k) * a.dim + h * HD + d]) & 0xFFu) << (8 * k);
    S.pw[d][wv] = word;
  }
  for (int i = tid; i < HD; i += kWideThreads) {
    S.pq[0][i] = a.pe_bq[h * HD + i];
    S.pq[1][i] = a.pe_mult[h * HD + i];
    S.pq[2][i] = a.pe_shift[h * HD + i];
  }
  if (tid == 0) {
    mbar_init(&S.bar, 1);
    S.abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&S.tmem, 512);
    tmem_relinquish();
  }
  pdl_wait();
  // Q (zero past N), K (zero past N), 16-byte loads.
  for (int i = tid; i < kAQ * 2; i += kWideThreads) {
    const int r = i >> 1, c = i & 1;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (q0 + r < N) v = *reinterpret_cast<const uint4*>(base + static_cast<long long>(q0 + r) * a.qkv.cstride + 16 * c);
    *reinterpret_cast<uint4*>(S.q + ops_off(r, 16 * c, KD)) = v;
  }
  for (int i = tid; i < Np * 2; i += kWideThreads) {
    const int j = i >> 1, c = i & 1;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (j < N) v = *reinterpret_cast<const uint4*>(base + static_cast<long long>(j) * a.qkv.cstride + KD + 16 * c);
    *reinterpret_cast<uint4*>(S.k + ops_off(j, 16 * c, KD)) = v;
  }
  // V^T: one item = 4 keys x 16 channels, transposed into 16 words of 4 keys.
  for (int i = tid; i < Np; i += kWideThreads) {
    const int j0 = (i % (Np >> 2)) * 4, c = i / (Np >> 2);
    uint4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[k] = make_uint4(0u, 0u, 0u, 0u);
      if (j0 + k < N)
        v[k] = *reinterpret_cast<const uint4*>(base + static_cast<long long>(j0 + k) * a.qkv.cstride + 2 * KD + 16 * c);
    }
#pragma unroll
    for (int qd = 0; qd < 4; ++qd) {
      const auto wq = [&](const uint4& u) { return qd == 0 ? u.x : qd == 1 ? u.y : qd == 2 ? u.z : u.w; };
      uint32_t y[4];
      transpose4w(wq(v[0]), wq(v[1]), wq(v[2]), wq(v[3]), y);
#pragma unroll
      for (int e = 0; e < 4; ++e) *reinterpret_cast<uint32_t*>(S.vt + ops_off(16 * c + 4 * qd + e, j0, Np)) = y[e];
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = S.tmem;
  const uint32_t trow = tbase + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  // Score columns preset to the bits of 1.5 * 2^23: the score UMMAs
  // accumulate onto them, so every score arrives as the float 1.5 * 2^23 + S
  // (see the weights below).  This warpgroup presets its quarter of the
  // columns for its warp's lanes.
  const int c0 = g * Nq;
  {
    uint32_t pre[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) pre[e] = 0x4B400000u;
    for (int cc = 0; cc < Nq; cc += 16) tc_st_32x32b_x16(trow + static_cast<uint32_t>(c0 + cc), pre);
    tc_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  volatile int* abort_flag = &S.abort;
  bool ok = true;
  uint32_t phase = 0;
  auto wait_mma = [&]() {
    if (!ok) return;
    if (!mbar_wait(&S.bar, phase, abort_flag)) {
      *abort_flag = 1;
      if (a.err) atomicCAS(a.err, 0, kErrAttnWait);
      ok = false;
    }
    phase ^= 1u;
    tc_fence_after();
  };
  // S = Q K^T for all keys: columns [0, 256) and [256, Np).
  if (tid == 0) {
    const uint64_t da = kmajor_desc_noswizzle(smem_u32(S.q), 128, (KD / 16) * 128);
    for (int k0 = 0; k0 < Np; k0 += 256) {
      const int nb = Np - k0 < 256 ? Np - k0 : 256;
      const uint64_t db = kmajor_desc_noswizzle(smem_u32(S.k) + static_cast<uint32_t>(k0 / 8) * 256u, 128,
                                                (KD / 16) * 128);
      tc_mma_i8(tbase + static_cast<uint32_t>(k0), da, db, idesc_s8_s32(kAQ, nb), 1u);
    }
    tc_commit(&S.bar);
  }
  wait_mma();
  // Row maximum over this warpgroup's quarter of the valid keys (of the
  // preset scores: the same order as of the scores).
  int mx = INT_MIN;
  for (int cc = 0; cc < Nq; cc += 16) {
    uint32_t r[16];
    tc_ld_32x32b_x16(trow + static_cast<uint32_t>(c0 + cc), r);
    tc_wait_ld();
    if (c0 + cc + 16 <= N) {
#pragma unroll
      for (int e = 0; e < 16; ++e) mx = max(mx, static_cast<int>(r[e]));
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (c0 + cc + e < N) mx = max(mx, static_cast<int>(r[e]));
    }
  }
  S.red_max[g][row] = mx;
  __syncthreads();
  mx = max(max(S.red_max[0][row], S.red_max[1][row]), max(S.red_max[2][row], S.red_max[3][row]));
  // Weights of this quarter (keys past N take the zero entry 256): the
  // difference of the preset score from the preset maximum is the exact
  // integer max - S; y = min(255, (max - S) * mt * 2^-sht) from a saturating
  // multiply by mt * 2^-sht / 255 and a fused multiply-add of 255 and
  // 1.5 * 2^23, which rounds to the nearest integer (ties to even) and
  // leaves 1.5 * 2^23 + t in its bits.  With four roundings y is within
  // 2^-13 of the exact value, so a block of 16 keys with a product within
  // 2^-13 of a half-integer is redone with the 64-bit rule.
  const float ratio255 = __fdiv_rn(ldexpf(static_cast<float>(a.mt), -a.sht), 255.0f);
  const float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float fmx = __uint_as_float(static_cast<uint32_t>(mx));
  const int mxs = mx - 0x4B400000;  // the maximum score itself
  const uint32_t e3b = smem_u32(S.E3) - 4u * 0x4B400000u;
  uint32_t lsum = 0u;
  for (int cc = 0; cc < Nq; cc += 16) {
    uint32_t r[16];
    tc_ld_32x32b_x16(trow + static_cast<uint32_t>(c0 + cc), r);
    tc_wait_ld();
    uint32_t t[16];  // 0x4B400000 + t
    bool amb = false;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float d = __fsub_rn(fmx, __uint_as_float(r[e]));
      const float ys = __saturatef(__fmul_rn(d, ratio255));
      const float yb = __fmaf_rn(ys, 255.0f, kMagic);
      const float fr = __fmaf_rn(ys, 255.0f, __fsub_rn(kMagic, yb));  // y - round(y)
      amb = amb || fabsf(fr) > 0.4998779296875f;
      t[e] = __float_as_uint(yb);
    }
    if (amb) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int sv = static_cast<int>(r[e] - 0x4B400000u);
        const long long te = rne64(static_cast<long long>(mxs - sv) * a.mt, a.sht);
        t[e] = 0x4B400000u + static_cast<uint32_t>(te > 255 ? 255 : te);
      }
    }
    if (c0 + cc + 16 > N) {
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (c0 + cc + e >= N) t[e] = 0x4B400000u + 256u;
    }
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      const uint32_t e0 = lds_u32(e3b + 4u * t[4 * q4]), e1 = lds_u32(e3b + 4u * t[4 * q4 + 1]);
      const uint32_t e2 = lds_u32(e3b + 4u * t[4 * q4 + 2]), e3 = lds_u32(e3b + 4u * t[4 * q4 + 3]);
      lsum += e0 + e1 + e2 + e3;
      const uint32_t t01 = __byte_perm(e0, e1, 0x6240), t23 = __byte_perm(e2, e3, 0x6240);
      hw[q4] = __byte_perm(t01, t23, 0x5410);
      lw[q4] = __byte_perm(t01, t23, 0x7632);
    }
    *reinterpret_cast<uint4*>(S.ph + ops_off(row, c0 + cc, Np)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(S.pl + ops_off(row, c0 + cc, Np)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
  S.red_sum[g][row] = static_cast<int32_t>(lsum);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // O_h += Ph V (columns [0, 64)), O_l += Pl V ([64, 128)) over all keys.
  if (tid == 0 && ok && !*abort_flag) {
    const uint32_t idesc = idesc_s8_s32(kAQ, HD);
    const uint32_t sbo = static_cast<uint32_t>(Np / 16) * 128u;
    const uint64_t dh = kmajor_desc_noswizzle(smem_u32(S.ph), 128, sbo);
    const uint64_t dl = kmajor_desc_noswizzle(smem_u32(S.pl), 128, sbo);
    const uint64_t dv = kmajor_desc_noswizzle(smem_u32(S.vt), 128, sbo);
    for (int s = 0; s < Np / 32; ++s) {
      const uint64_t off = static_cast<uint64_t>(16 * s);  // 32 keys = two core matrices = 256 bytes
      tc_mma_i8(tbase, dh + off, dv + off, idesc, s == 0 ? 0u : 1u);
      tc_mma_i8(tbase + 64, dl + off, dv + off, idesc, s == 0 ? 0u : 1u);
    }
    tc_commit(&S.bar);
  }
  // Meanwhile: the positional term of this row's 16 channels, a depthwise
  // 3x3 of v around the query (zero outside the image), as dp4a over taps.
  const int qi = q0 + row;
  const int d0 = 16 * g;
  const int y = qi / a.W, x = qi - (qi / a.W) * a.W;
  int acc[16];
  {
    uint32_t tw[9][4];
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
      const int iy = y - 1 + tap / 3, ix = x - 1 + tap % 3;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (qi < N && iy >= 0 && iy < a.H && ix >= 0 && ix < a.W)
        v = *reinterpret_cast<const uint4*>(base + static_cast<long long>(iy * a.W + ix) * a.qkv.cstride + 2 * KD + d0);
      tw[tap][0] = v.x;
      tw[tap][1] = v.y;
      tw[tap][2] = v.z;
      tw[tap][3] = v.w;
    }
#pragma unroll
    for (int qd = 0; qd < 4; ++qd) {
      uint32_t lo[4], hi[4];
      transpose4w(tw[0][qd], tw[1][qd], tw[2][qd], tw[3][qd], lo);
      transpose4w(tw[4][qd], tw[5][qd], tw[6][qd], tw[7][qd], hi);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = d0 + 4 * qd + e;
        const uint4 w = *reinterpret_cast<const uint4*>(S.pw[d]);
        int s = __dp4a(static_cast<int>(lo[e]), static_cast<int>(w.x), 0);
        s = __dp4a(static_cast<int>(hi[e]), static_cast<int>(w.y), s);
        s += static_cast<int>(static_cast<int8_t>(tw[8][qd] >> (8 * e))) * static_cast<int>(static_cast<int8_t>(w.z));
        acc[4 * qd + e] = s;
      }
    }
  }
  wait_mma();
  __syncthreads();
  const bool good = S.abort == 0;
  const bool valid = qi < N && good;
  int l = 0;
#pragma unroll
  for (int gg = 0; gg < 4; ++gg) {
    const uint32_t ls = static_cast<uint32_t>(S.red_sum[gg][row]);
    l += 64 * static_cast<int>(ls & 0xFFFFu) + static_cast<int>(ls >> 16);
  }
  const float rlf = __frcp_rn(static_cast<float>(l > 0 ? l : 1));
  uint32_t oh[16], ol[16];
  tc_ld_32x32b_x16(trow + static_cast<uint32_t>(d0), oh);
  tc_ld_32x32b_x16(trow + 64u + static_cast<uint32_t>(d0), ol);
  tc_wait_ld();
  if (valid) {
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int d = d0 + e;
      // |o| <= N * 4096 * 127 < 2^31 for N <= 4000.
      const int o = 64 * static_cast<int32_t>(oh[e]) + static_cast<int32_t>(ol[e]);
      const long long av = div_rne_q(rne64(static_cast<long long>(o) * a.mo, a.sho), l > 0 ? l : 1, rlf);
      const long long pe = rne64((static_cast<long long>(acc[e]) + S.pq[0][d]) * S.pq[1][d], S.pq[2][d]);
      const long long v = av + pe;
      const int c = static_cast<int>(v < -127 ? -127 : v > 127 ? 127 : v);
      w[e >> 2] |= (static_cast<uint32_t>(c) & 0xFFu) << (8 * (e & 3));
    }
    int8_t* op = a.out.p + static_cast<long long>(b) * a.out.bstride + static_cast<long long>(qi) * a.out.cstride +
                 h * HD + d0;
    *reinterpret_cast<uint4*>(op) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (!good) __nanosleep(100000);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------------------
// Long variant for kWideN < N <= kLongN keys (the 40 x 40 PSA of a 1280 x 1280
// input).  Q, K and V^T stay resident in shared memory and the keys stream
// through tensor memory in chunks.  Each of the four warpgroups runs its own
// pipeline over its own chunks (chunk c belongs to warpgroup c % 4): its
// first thread issues the warpgroup's UMMAs, so the four pipelines -- tensor
// core, tensor-memory loads and weight arithmetic -- interleave on the SM
// with no thread serialising them.  The value UMMAs of all four accumulate
// into one O (zeroed first); integer sums do not depend on their order.
//   pass 1  S for 128 keys per chunk into the warpgroup's TMEM columns
//           [128 g, 128 g + 128), reduced to row maxima.
//   pass 2  S again for 32 keys per chunk, two TMEM buffers per warpgroup
//           (columns 64 g + 32 b); the warpgroup turns a chunk into Ph / Pl
//           bytes in its shared-memory P buffer and its part of l; its first
//           thread adds Ph V into O_h (columns [256, 320)) and Pl V into O_l
//           ([320, 384)) and refills the score buffer with the chunk eight
//           ahead, whose keys the tensor core multiplies while the
//           warpgroup works on the next chunk.
// Same integer rules as the other variants.  The weight index t comes from
// fp32 arithmetic without conversions or integer work per key: each pass-2
// score buffer is preset to the bit pattern of 1.5 * 2^23 and the score
// UMMAs accumulate onto it, so every score arrives as the float 1.5 * 2^23 +
// S (exact below 2^22 in magnitude) and its difference from the maximum,
// entered the same way, is the exact integer.  y = min(255, (max - S) * mt *
// 2^-sht) comes from a saturating multiply by mt * 2^-sht / 255 and a fused
// multiply-add of 255 and 1.5 * 2^23, which rounds to the nearest integer
// (ties to even, as rintf); the low bits of that sum are t.  With four
// roundings y is within 2^-13 of the exact value, so a block of keys with a
// product within 2^-13 of a half-integer takes the 64-bit rule.
constexpr int kLongN = 1920;
constexpr int kC1 = 128;  // keys per pass-1 chunk
constexpr int kC2 = 32;   // keys per pass-2 chunk
constexpr int kLongThreads = 512;

struct AttnLongSmem {
  uint8_t q[kAQ * KD];
  uint8_t k[kLongN * KD];
  uint8_t vt[HD * kLongN + 128];  // row groups of 8 channels Np * 8 + 16 bytes apart
  uint8_t ph[4][kAQ * kC2];
  uint8_t pl[4][kAQ * kC2];
  uint32_t E3[257];
  alignas(16) uint32_t pw[HD][4];
  int32_t pq[3][HD];
  int32_t red_max[4][kAQ];
  int32_t red_sum[4][kAQ];
  uint64_t s1[4];        // pass-1 scores of the warpgroup's chunk are in TMEM
  uint64_t s2[4][2];     // pass-2 scores in the warpgroup's TMEM buffer b
  uint64_t pv[4];        // the warpgroup's value UMMAs so far have completed
  uint32_t tmem;
  int abort;
};

__device__ __forceinline__ void workers_sync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }
// Barrier of the 128 threads of warpgroup g (named barriers 2 to 5).
__device__ __forceinline__ void group_sync(int g) { asm volatile("bar.sync %0, 128;" ::"r"(2 + g) : "memory"); }

__global__ void __launch_bounds__(kLongThreads, 1) attention_i8_long_kernel(const I8AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t attn_long_raw[];
  AttnLongSmem& S = *reinterpret_cast<AttnLongSmem*>(attn_long_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = warp >> 2;                 // warpgroup
  const int row = (warp & 3) * 32 + lane;  // query row = TMEM lane
  const bool leader = (tid & 127) == 0;    // issues the warpgroup's UMMAs
  const int N = a.H * a.W;
  const int Np = (N + kC2 - 1) & ~(kC2 - 1);
  const int n1 = (Np + kC1 - 1) / kC1, n2 = Np / kC2;
  const int q0 = blockIdx.x * kAQ, h = blockIdx.y, b = blockIdx.z;
  const int blk = 2 * KD + HD;
  const int8_t* base = a.qkv.p + static_cast<long long>(b) * a.qkv.bstride + h * blk;
  for (int i = tid; i < 257; i += kLongThreads) {
    const int e = i < 256 ? a.E[i] : 0;
    S.E3[i] = static_cast<uint32_t>(e >> 6) | (static_cast<uint32_t>(e & 63) << 16);
  }
  for (int i = tid; i < HD * 3; i += kLongThreads) {
    const int d = i / 3, wv = i - (i / 3) * 3;
    uint32_t word = 0u;
    for (int k = 0; k < 4 && 4 * wv + k < 9; ++k)
      word |= (static_cast<uint32_t>(a.pe_w[(4 * wv + k) * a.dim + h * HD + d]) & 0xFFu) << (8 * k);
    S.pw[d][wv] = word;
  }
  for (int i = tid; i < HD; i += kLongThreads) {
    S.pq[0][i] = a.pe_bq[h * HD + i];
    S.pq[1][i] = a.pe_mult[h * HD + i];
    S.pq[2][i] = a.pe_shift[h * HD + i];
  }
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) {
      mbar_init(&S.s1[i], 1);
      mbar_init(&S.s2[i][0], 1);
      mbar_init(&S.s2[i][1], 1);
      mbar_init(&S.pv[i], 1);
    }
    S.abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&S.tmem, 512);
    tmem_relinquish();
  }
  pdl_wait();
  // Q and K: 16-byte asynchronous copies (zero past N).
  for (int i = tid; i < kAQ * 2; i += kLongThreads) {
    const int r = i >> 1, c = i & 1;
    const bool in = q0 + r < N;
    const int8_t* src = base + static_cast<long long>(in ? q0 + r : 0) * a.qkv.cstride + 16 * c;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(S.q + ops_off(r, 16 * c, KD))),
                 "l"(src), "r"(in ? 16u : 0u)
                 : "memory");
  }
  for (int i = tid; i < Np * 2; i += kLongThreads) {
    const int j = i >> 1, c = i & 1;
    const bool in = j < N;
    const int8_t* src = base + static_cast<long long>(in ? j : 0) * a.qkv.cstride + KD + 16 * c;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(S.k + ops_off(j, 16 * c, KD))),
                 "l"(src), "r"(in ? 16u : 0u)
                 : "memory");
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
      if (a.err) atomicCAS(a.err, 0, kErrAttnWait);
      ok = false;
    }
    tc_fence_after();
  };
  auto live = [&]() { return ok && !*abort_flag; };
  const uint64_t da = kmajor_desc_noswizzle(smem_u32(S.q), 128, (KD / 16) * 128);
  const uint64_t db0 = kmajor_desc_noswizzle(smem_u32(S.k), 128, (KD / 16) * 128);
  // Scores of keys [k0, k0 + nb) into TMEM columns [col, col + nb); 8 keys
  // are one 256-byte row group of K (16 descriptor units).
  auto scores = [&](int k0, int nb, uint32_t col, uint64_t* bar, uint32_t accumulate) {
    tc_mma_i8(tbase + col, da, db0 + static_cast<uint64_t>(k0 / 8) * 16u, idesc_s8_s32(kAQ, nb), accumulate);
    tc_commit(bar);
  };
  if (leader && g < n1) scores(g * kC1, min(kC1, Np - g * kC1), static_cast<uint32_t>(g * kC1), &S.s1[g], 0u);

  // V^T while the first scores are computed.  Item i: channel group i & 3,
  // key quad i >> 2, so that the four lanes of a key quad read its 64 bytes
  // together and the stores of a warp spread over the banks (row groups
  // padded by 16 bytes); two items' loads in flight per thread.
  {
    const int nitems = Np;  // (Np / 4) key quads x 4 channel groups
    const uint32_t vsbo = static_cast<uint32_t>(Np * 8 + 16);
    for (int i0 = tid; i0 < nitems; i0 += 2 * kLongThreads) {
      uint4 v[2][4];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = i0 + kLongThreads * u;
        const int j0 = (i >> 2) * 4, c = i & 3;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          v[u][k] = make_uint4(0u, 0u, 0u, 0u);
          if (i < nitems && j0 + k < N)
            v[u][k] =
                *reinterpret_cast<const uint4*>(base + static_cast<long long>(j0 + k) * a.qkv.cstride + 2 * KD + 16 * c);
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = i0 + kLongThreads * u;
        if (i >= nitems) continue;
        const int j0 = (i >> 2) * 4, c = i & 3;
        // Channel d = 16 c + 4 qd + e: row group 2 c + qd / 2, row (4 qd + e) & 7.
        uint8_t* vcol = S.vt + (j0 >> 4) * 128 + (j0 & 15);
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          const auto wq = [&](const uint4& x) { return qd == 0 ? x.x : qd == 1 ? x.y : qd == 2 ? x.z : x.w; };
          uint32_t y[4];
          transpose4w(wq(v[u][0]), wq(v[u][1]), wq(v[u][2]), wq(v[u][3]), y);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            *reinterpret_cast<uint32_t*>(vcol + (2 * c + (qd >> 1)) * vsbo + ((4 * qd + e) & 7) * 16) = y[e];
        }
      }
    }
    fence_proxy_async_smem();
  }

  // Pass 1: row maxima of this warpgroup's chunks.
  int mx = INT_MIN;
  for (int c = g; c < n1; c += 4) {
    wait_bar(&S.s1[g], static_cast<uint32_t>(c >> 2) & 1u);
    const int k0 = c * kC1, nb = min(kC1, Np - k0);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      uint32_t r[4][16];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (64 * hf + 16 * u < nb) tc_ld_32x32b_x16(trow + static_cast<uint32_t>(g * kC1 + 64 * hf + 16 * u), r[u]);
      tc_wait_ld();
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int kb = k0 + 64 * hf + 16 * u;
        if (kb - k0 >= nb) continue;
        tc_ld_dep(r[u]);
        if (kb + 16 <= N) {
#pragma unroll
          for (int e = 0; e < 16; ++e) mx = max(mx, static_cast<int>(r[u][e]));
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (kb + e < N) mx = max(mx, static_cast<int>(r[u][e]));
        }
      }
    }
    tc_fence_before();
    group_sync(g);  // the warpgroup's buffer is read
    if (leader && c + 4 < n1 && live()) {
      tc_fence_after();
      scores((c + 4) * kC1, min(kC1, Np - (c + 4) * kC1), static_cast<uint32_t>(g * kC1), &S.s1[g], 0u);
    }
  }
  S.red_max[g][row] = mx;
  tc_fence_before();
  workers_sync();  // every pass-1 score is read
  tc_fence_after();
  mx = max(max(S.red_max[0][row], S.red_max[1][row]), max(S.red_max[2][row], S.red_max[3][row]));
  // O = 0 (this warpgroup's 32 of its 128 columns, this warp's lanes) and
  // the warpgroup's score buffers preset; then its first two pass-2 chunks.
  uint32_t kPreset[16];  // 1.5 * 2^23 as float bits, the start of every pass-2 score
#pragma unroll
  for (int e = 0; e < 16; ++e) kPreset[e] = 0x4B400000u;
  {
    const uint32_t z[16] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    tc_st_32x32b_x16(trow + 256u + static_cast<uint32_t>(32 * g), z);
    tc_st_32x32b_x16(trow + 256u + static_cast<uint32_t>(32 * g + 16), z);
#pragma unroll
    for (int q = 0; q < 4; ++q) tc_st_32x32b_x16(trow + static_cast<uint32_t>(64 * g + 16 * q), kPreset);
    tc_wait_st();
  }
  tc_fence_before();
  workers_sync();  // O is zero and the score buffers preset before any UMMA
  tc_fence_after();
  if (leader && live()) {
    for (int k = 0; k < 2 && g + 4 * k < n2; ++k)
      scores((g + 4 * k) * kC2, kC2, static_cast<uint32_t>(64 * g + 32 * k), &S.s2[g][k], 1u);
  }

  // Pass 2: weights of this warpgroup's 32-key chunks.
  const float ratio255 = __fdiv_rn(ldexpf(static_cast<float>(a.mt), -a.sht), 255.0f);
  const float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float fmx = __int_as_float(0x4B400000 + mx);
  // Shared-memory address of E3[t] is e3b + 4 * (bits of 1.5 * 2^23 + t).
  const uint32_t e3b = smem_u32(S.E3) - 4u * 0x4B400000u;
  const uint32_t idesc_o = idesc_s8_s32(kAQ, HD);
  const uint64_t dv = kmajor_desc_noswizzle(smem_u32(S.vt), 128, static_cast<uint32_t>(Np * 8 + 16));
  const uint64_t dh = kmajor_desc_noswizzle(smem_u32(S.ph[g]), 128, (kC2 / 16) * 128);
  const uint64_t dl = kmajor_desc_noswizzle(smem_u32(S.pl[g]), 128, (kC2 / 16) * 128);
  uint32_t lsum = 0u;
  int k = 0;
  for (int c = g; c < n2; c += 4, ++k) {
    const int sb = k & 1;
    wait_bar(&S.s2[g][sb], static_cast<uint32_t>(k >> 1) & 1u);
    uint32_t r[2][16];
    tc_ld_32x32b_x16(trow + static_cast<uint32_t>(64 * g + 32 * sb), r[0]);
    tc_ld_32x32b_x16(trow + static_cast<uint32_t>(64 * g + 32 * sb + 16), r[1]);
    tc_wait_ld();
    tc_ld_dep(r[0]);
    tc_ld_dep(r[1]);
    // The buffer is read: preset it for the chunk eight ahead.
    tc_st_32x32b_x16(trow + static_cast<uint32_t>(64 * g + 32 * sb), kPreset);
    tc_st_32x32b_x16(trow + static_cast<uint32_t>(64 * g + 32 * sb + 16), kPreset);
    const int k0 = c * kC2;
    uint32_t hw[8], lw[8];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      uint32_t t[16];  // 0x4B400000 + t
      bool amb = false;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float d = __fsub_rn(fmx, __uint_as_float(r[u][e]));
        const float ys = __saturatef(__fmul_rn(d, ratio255));
        const float yb = __fmaf_rn(ys, 255.0f, kMagic);
        const float fr = __fmaf_rn(ys, 255.0f, __fsub_rn(kMagic, yb));  // y - round(y)
        amb = amb || fabsf(fr) > 0.4998779296875f;
        t[e] = __float_as_uint(yb);
      }
      if (amb) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int sv = static_cast<int>(r[u][e] - 0x4B400000u);
          const long long te = rne64(static_cast<long long>(mx - sv) * a.mt, a.sht);
          t[e] = 0x4B400000u + static_cast<uint32_t>(te > 255 ? 255 : te);
        }
      }
      if (k0 + 16 * u + 16 > N) {
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (k0 + 16 * u + e >= N) t[e] = 0x4B400000u + 256u;
      }
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const uint32_t e0 = lds_u32(e3b + 4u * t[4 * q4]), e1 = lds_u32(e3b + 4u * t[4 * q4 + 1]);
        const uint32_t e2 = lds_u32(e3b + 4u * t[4 * q4 + 2]), e3v = lds_u32(e3b + 4u * t[4 * q4 + 3]);
        lsum += e0 + e1 + e2 + e3v;
        const uint32_t t01 = __byte_perm(e0, e1, 0x6240), t23 = __byte_perm(e2, e3v, 0x6240);
        hw[4 * u + q4] = __byte_perm(t01, t23, 0x5410);
        lw[4 * u + q4] = __byte_perm(t01, t23, 0x7632);
      }
    }
    tc_wait_st();
    if (k >= 1) wait_bar(&S.pv[g], static_cast<uint32_t>(k - 1) & 1u);  // the P buffer is free
    *reinterpret_cast<uint4*>(S.ph[g] + ops_off(row, 0, kC2)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(S.ph[g] + ops_off(row, 16, kC2)) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
    *reinterpret_cast<uint4*>(S.pl[g] + ops_off(row, 0, kC2)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    *reinterpret_cast<uint4*>(S.pl[g] + ops_off(row, 16, kC2)) = make_uint4(lw[4], lw[5], lw[6], lw[7]);
    fence_proxy_async_smem();
    tc_fence_before();
    group_sync(g);  // P written, score buffer sb read
    if (leader && live()) {
      tc_fence_after();
      const uint64_t voff = static_cast<uint64_t>(c * kC2 / 2);  // 32 keys = 256 bytes = 16 units
      tc_mma_i8(tbase + 256u, dh, dv + voff, idesc_o, 1u);
      tc_mma_i8(tbase + 320u, dl, dv + voff, idesc_o, 1u);
      tc_commit(&S.pv[g]);
      if (c + 8 < n2) scores((c + 8) * kC2, kC2, static_cast<uint32_t>(64 * g + 32 * sb), &S.s2[g][sb], 1u);
    }
  }
  // This warpgroup's last value UMMAs (and so all of its earlier ones).
  if (k >= 1) wait_bar(&S.pv[g], static_cast<uint32_t>(k - 1) & 1u);
  S.red_sum[g][row] = static_cast<int32_t>(lsum);
  // The positional term of this row's 16 channels.
  const int qi = q0 + row;
  const int d0 = 16 * g;
  const int y = qi / a.W, x = qi - (qi / a.W) * a.W;
  int acc[16];
  {
    uint32_t tw[9][4];
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
      const int iy = y - 1 + tap / 3, ix = x - 1 + tap % 3;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (qi < N && iy >= 0 && iy < a.H && ix >= 0 && ix < a.W)
        v = *reinterpret_cast<const uint4*>(base + static_cast<long long>(iy * a.W + ix) * a.qkv.cstride + 2 * KD + d0);
      tw[tap][0] = v.x;
      tw[tap][1] = v.y;
      tw[tap][2] = v.z;
      tw[tap][3] = v.w;
    }
#pragma unroll
    for (int qd = 0; qd < 4; ++qd) {
      uint32_t lo[4], hi[4];
      transpose4w(tw[0][qd], tw[1][qd], tw[2][qd], tw[3][qd], lo);
      transpose4w(tw[4][qd], tw[5][qd], tw[6][qd], tw[7][qd], hi);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = d0 + 4 * qd + e;
        const uint4 w = *reinterpret_cast<const uint4*>(S.pw[d]);
        int s = __dp4a(static_cast<int>(lo[e]), static_cast<int>(w.x), 0);
        s = __dp4a(static_cast<int>(hi[e]), static_cast<int>(w.y), s);
        s += static_cast<int>(static_cast<int8_t>(tw[8][qd] >> (8 * e))) * static_cast<int>(static_cast<int8_t>(w.z));
        acc[4 * qd + e] = s;
      }
    }
  }
  tc_fence_before();
  workers_sync();  // every warpgroup's value UMMAs have completed
  tc_fence_after();
  const bool good = S.abort == 0;
  const bool valid = qi < N && good;
  int l = 0;
#pragma unroll
  for (int gg = 0; gg < 4; ++gg) {
    const uint32_t ls = static_cast<uint32_t>(S.red_sum[gg][row]);
    l += 64 * static_cast<int>(ls & 0xFFFFu) + static_cast<int>(ls >> 16);
  }
  const float rlf = __frcp_rn(static_cast<float>(l > 0 ? l : 1));
  uint32_t oh[16], ol[16];
  tc_ld_32x32b_x16(trow + 256u + static_cast<uint32_t>(d0), oh);
  tc_ld_32x32b_x16(trow + 320u + static_cast<uint32_t>(d0), ol);
  tc_wait_ld();
  if (valid) {
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int d = d0 + e;
      const int o = 64 * static_cast<int32_t>(oh[e]) + static_cast<int32_t>(ol[e]);
      const long long av = div_rne_q(rne64(static_cast<long long>(o) * a.mo, a.sho), l > 0 ? l : 1, rlf);
      const long long pe = rne64((static_cast<long long>(acc[e]) + S.pq[0][d]) * S.pq[1][d], S.pq[2][d]);
      const long long v = av + pe;
      const int cl = static_cast<int>(v < -127 ? -127 : v > 127 ? 127 : v);
      w[e >> 2] |= (static_cast<uint32_t>(cl) & 0xFFu) << (8 * (e & 3));
    }
    int8_t* op = a.out.p + static_cast<long long>(b) * a.out.bstride + static_cast<long long>(qi) * a.out.cstride +
                 h * HD + d0;
    *reinterpret_cast<uint4*>(op) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  // A wait that gave up leaves UMMAs possibly in flight: give them time to
  // finish before tensor memory is released.
  if (!good) __nanosleep(100000);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

}  // namespace

cudaError_t launch_attention_i8(const I8AttnArgs& a, cudaStream_t st) {
  const int N = a.H * a.W;
  if (a.kd != KD || a.hd != HD || N < 1 || N > 4000 || a.qkv.cstride % 16 || a.out.cstride % 16 || a.qkv.bstride % 16 ||
      a.out.bstride % 16 || reinterpret_cast<uintptr_t>(a.qkv.p) % 16 || reinterpret_cast<uintptr_t>(a.out.p) % 16 ||
      a.dim != a.heads * HD || a.sht < 1 || a.sho < 1)
    return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_done{0};
  const cudaError_t e = smem_attr_once(attention_i8_tc_kernel, static_cast<int>(sizeof(AttnSmem)), attr_done);
  if (e != cudaSuccess) return e;
  dim3 grid((N + kAQ - 1) / kAQ, a.heads, a.B);
  if (N <= kWideN) {
    static std::atomic<uint64_t> wide_done{0};
    const cudaError_t e2 = smem_attr_once(attention_i8_wide_kernel, static_cast<int>(sizeof(AttnWideSmem)), wide_done);
    if (e2 != cudaSuccess) return e2;
    return launch_pdl(attention_i8_wide_kernel, grid, dim3(kWideThreads), sizeof(AttnWideSmem), st, a);
  }
  if (N <= kLongN) {
    static std::atomic<uint64_t> long_done{0};
    const cudaError_t e2 = smem_attr_once(attention_i8_long_kernel, static_cast<int>(sizeof(AttnLongSmem)), long_done);
    if (e2 != cudaSuccess) return e2;
    return launch_pdl(attention_i8_long_kernel, grid, dim3(kLongThreads), sizeof(AttnLongSmem), st, a);
  }
  return launch_pdl(attention_i8_tc_kernel, grid, dim3(128), sizeof(AttnSmem), st, a);
}

}  // namespace yb
