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

__device__ __forceinline__ long long div_rne_fast(long long a, long long l, double rl) {
  long long q = static_cast<long long>(floor(static_cast<double>(a) * rl));
  long long r = a - q * l;
  if (r < -2 * l || r >= 3 * l) return div_rne64(a, l);
  while (r < 0) {
    --q;
    r += l;
  }
  while (r >= l) {
    ++q;
    r -= l;
  }
  if (2 * r > l || (2 * r == l && (q & 1))) ++q;
  return q;
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
      tc_mma_i8(tbase + static_cast<uint32_t>(k0), da, db, idesc_s8_s32(kAQ, nb), 0u);
    }
    tc_commit(&S.bar);
  }
  wait_mma();
  // Row maximum over this warpgroup's quarter of the valid keys.
  const int c0 = g * Nq;
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
  // Weights of this quarter: t from the fp32 product, clamped to 255 (keys
  // past N take the zero entry 256); a block of 16 keys with a product
  // within 2^-14 of a half-integer is redone with the 64-bit rule.
  const float ratio = ldexpf(static_cast<float>(a.mt), -a.sht);
  uint32_t lsum = 0u;
  for (int cc = 0; cc < Nq; cc += 16) {
    uint32_t r[16];
    tc_ld_32x32b_x16(trow + static_cast<uint32_t>(c0 + cc), r);
    tc_wait_ld();
    int t[16];
    bool amb = false;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float y = fminf(static_cast<float>(mx - static_cast<int>(r[e])) * ratio, 255.0f);
      const float ty = rintf(y);
      amb = amb || fabsf(y - ty) > 0.49993896484375f;
      t[e] = c0 + cc + e < N ? static_cast<int>(ty) : 256;
    }
    if (amb) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        if (t[e] == 256) continue;
        const long long te = rne64(static_cast<long long>(mx - static_cast<int>(r[e])) * a.mt, a.sht);
        t[e] = te > 255 ? 255 : static_cast<int>(te);
      }
    }
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      const uint32_t e0 = S.E3[t[4 * q4]], e1 = S.E3[t[4 * q4 + 1]];
      const uint32_t e2 = S.E3[t[4 * q4 + 2]], e3 = S.E3[t[4 * q4 + 3]];
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
  const double rl = 1.0 / static_cast<double>(l > 0 ? l : 1);
  uint32_t oh[16], ol[16];
  tc_ld_32x32b_x16(trow + static_cast<uint32_t>(d0), oh);
  tc_ld_32x32b_x16(trow + 64u + static_cast<uint32_t>(d0), ol);
  tc_wait_ld();
  if (valid) {
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int d = d0 + e;
      const long long o = 64LL * static_cast<int32_t>(oh[e]) + static_cast<int32_t>(ol[e]);
      const long long av = div_rne_fast(rne64(o * a.mo, a.sho), l, rl);
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
  return launch_pdl(attention_i8_tc_kernel, grid, dim3(128), sizeof(AttnSmem), st, a);
}

}  // namespace yb
