// Inline-PTX building blocks for sm_100a: mbarriers, bulk copies (TMA engine,
// untiled), tcgen05 tensor-memory allocation, UMMA issue/commit and TMEM loads.
// Every barrier wait is bounded: after kWaitNs of polling it reports failure
// so that a kernel can record an error, drain and exit instead of hanging.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace yb {

// Upper bound for any single barrier wait inside a kernel (nanoseconds).
constexpr uint64_t kWaitNs = 2000000000ull;

// Error codes written to the kernel error word.
enum : int {
  kErrNone = 0,
  kErrWaitFull = 1,      // MMA issuer gave up waiting for a filled stage
  kErrWaitEmpty = 2,     // producer gave up waiting for a free stage
  kErrWaitAccFull = 3,   // epilogue gave up waiting for an accumulator
  kErrWaitAccEmpty = 4,  // MMA issuer gave up waiting for a drained accumulator
  kErrDrain = 5,         // teardown gave up waiting for outstanding MMAs
  kErrBadArgs = 6,
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with an explicit suspend-time hint: a thread whose phase is not
// complete sleeps in hardware (up to hint_ns) instead of spinning, so waiting
// warps leave the issue slots to the working ones.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Waits for the phase with the given parity to complete.  Returns false when
// the wait gave up: after kWaitNs, or early once *abort is non-zero.
// limit_ns shortens the bound (a kernel's test hook passes about 1 ms).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint64_t limit_ns = kWaitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint32_t hint = limit_ns < 1000000u ? static_cast<uint32_t>(limit_ns) : 1000000u;
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, hint)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// ------------------------------------------------------------ bulk copies
// Untiled bulk copy global -> shared through the TMA engine; completion is
// signalled as transaction bytes on `bar`.  dst/src 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Arrives on `bar` and adds `bytes` to the transaction count of its current
// phase (the phase completes when the copies have delivered them).
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// TMA load in im2col mode from a 4-D NHWC tensor map (dims C, W, H, N):
// pixelsPerColumn consecutive output pixels starting at the window origin
// (w, h) of image n, channels [c, c + channelsPerPixel), filter tap (ow, oh).
// Out-of-bounds elements arrive as zeros.  c * element size must be a
// multiple of 16 bytes; dst aligned to the map's swizzle span.
__device__ __forceinline__ void tma_im2col_4d(void* dst, const CUtensorMap* map, int c, int w, int h, int n,
                                              uint16_t ow, uint16_t oh, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], {%7, %8};" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c), "r"(w), "r"(h), "r"(n), "r"(smem_u32(bar)), "h"(ow), "h"(oh)
      : "memory");
}

// Brings a tensor map (a __grid_constant__ kernel parameter) into the TMA
// unit's descriptor cache ahead of the first copy that uses it.
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// TMA load of one box of a 4-D tiled tensor map at coordinates (c0..c3),
// innermost first; out-of-bounds elements arrive as zeros.  c0 * element
// size must be a multiple of 16 bytes; dst 128-byte aligned.
__device__ __forceinline__ void tma_tile_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads (tensor-core operand fetch).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulation.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Instruction descriptor, kind::i8: signed 8-bit A and B, int32 D, K-major.
__host__ __device__ constexpr uint32_t idesc_s8_s32(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, signed int8 inputs, int32 accumulation.
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on `bar` when all tcgen05 operations issued so far by this
// thread have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns; thread i of the warp receives
// lane (base_lane + i).
__device__ __forceinline__ void tc_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 lanes x 16 consecutive 32-bit columns from registers (thread i of the
// warp writes lane base_lane + i), and the wait for this thread's stores.
__device__ __forceinline__ void tc_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Ties 16 registers written by an earlier tcgen05.ld to a point after
// tc_wait_ld(), so that no read of them is scheduled before the wait.
__device__ __forceinline__ void tc_ld_dep(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}
// 32-byte global store (sm_100): dst 32-byte aligned.
__device__ __forceinline__ void st_global_v8(void* dst, const uint32_t (&v)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

// Shared-memory matrix descriptor for a K-major operand in the 128-byte
// swizzled canonical layout: rows of 128 bytes (64 bf16 of K), groups of 8
// rows 1024 bytes apart.  Fields: start address >> 4 [0,14), leading byte
// offset >> 4 [16,30) (unused by swizzled K-major, set to 1), stride byte
// offset >> 4 [32,46) = 1024 >> 4, version 1 at [46,48), base offset 0,
// layout type 2 (SWIZZLE_128B) at [61,64).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// K-major operand descriptor for any swizzle mode: layout 2 (128B, rows of
// 128 bytes), 4 (64B) or 6 (32B); 8-row groups sbo bytes apart (8 x row
// bytes when packed).  The tile base must be aligned to 8 x row bytes.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr, uint32_t layout, uint32_t sbo) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(sbo >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(layout) << 61);
}

// K-major operand descriptor without swizzle: core matrices of 8 rows x 16
// bytes stored as 128 contiguous bytes (rows 16 bytes apart), the two core
// matrices of a 16-wide K step lbo bytes apart, 8-row groups sbo bytes apart.
__device__ __forceinline__ uint64_t kmajor_desc_noswizzle(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(lbo >> 4) << 16) |
         (static_cast<uint64_t>(sbo >> 4) << 32) | (static_cast<uint64_t>(1) << 46);
}

// Instruction descriptor for kind::f16 with bf16 A/B, fp32 D, both K-major:
// c_format F32 (1) at [4,6), a_format BF16 (1) at [7,10), b_format BF16 (1)
// at [10,13), N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// The same instruction descriptor with N halved: against a stacked
// [B_hi; B_lo] operand (B_hi rows first) the UMMA then reads B_hi only.
__host__ __device__ constexpr uint32_t idesc_half_n(uint32_t idesc) {
  return (idesc & ~(0x3Fu << 17)) | ((((idesc >> 17) & 0x3Fu) >> 1) << 17);
}

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` inside a
// 128B-swizzled K-major tile whose base is 1024-byte aligned.
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return (row >> 3) * 1024u + (row & 7u) * 128u + ((chunk ^ (row & 7u)) << 4);
}

}  // namespace yb
