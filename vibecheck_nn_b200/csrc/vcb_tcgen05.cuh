// Thin wrappers over the sm_100a primitives the tensor-core kernels share:
// mbarriers with bounded waits, bulk copies, shared-memory matrix
// descriptors, tcgen05.mma (kind::tf32, operands in shared or tensor memory),
// tensor-memory loads / stores and the 3xTF32 operand split.
#pragma once

#include <cstdint>

namespace vcb {
namespace tc5 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Wait for the phase with the given parity; false when `limit` polls pass or
// another role raised *abort (checked every 256 polls).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, unsigned limit,
                                          const volatile int* abort = nullptr) {
  const uint32_t a = smem_u32(bar);
  for (unsigned i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if (abort && (i & 255) == 255 && *abort) return false;
  }
  return false;
}

// As mbar_wait, each poll suspending the thread for up to ~1 us while the
// phase is incomplete (fewer issue slots spent waiting).
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, unsigned parity, unsigned limit,
                                                const volatile int* abort = nullptr) {
  const uint32_t a = smem_u32(bar);
  for (unsigned i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"(1000u)
        : "memory");
    if (done) return true;
    if (abort && (i & 15) == 15 && *abort) return false;
  }
  return false;
}

// Global -> shared bulk copy (16-byte aligned addresses, size a multiple of
// 16) completing on an mbarrier's transaction count.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// K-major operand with 128-byte swizzle: rows of 128 B, 8-row groups 1024 B
// apart (stride byte offset), leading offset unused, descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: D f32, A and B tf32, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// D (tensor memory) (+)= A (shared) B (shared).
__device__ __forceinline__ void mma_tf32_ss(uint32_t tmem_d, uint64_t da, uint64_t db,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}

// D (tensor memory) (+)= A (tensor memory: lane = row, column = K index)
// B (shared).
__device__ __forceinline__ void mma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate));
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has
// completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

#define VCB_R16(r)                                                                          \
  "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),     \
      "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),          \
      "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
#define VCB_RW16(r)                                                                         \
  "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),     \
      "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),          \
      "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
#define VCB_IN16(r)                                                                         \
  "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), \
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),   \
      "r"(r[15])

// 16 consecutive 32-bit columns of this warp's 32 lanes (one row per lane).
// The values may be used only after tmem_wait_ld on the same registers.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : VCB_R16(r)
      : "r"(taddr));
}

#define VCB_R8(r) "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
#define VCB_RW8(r) "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])
#define VCB_IN8(r) "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : VCB_R8(r)
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[8], uint32_t (&s)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : VCB_RW8(r), VCB_RW8(s)::"memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(
                   taddr),
               VCB_IN8(r)
               : "memory");
}

// Completes the loads of this thread; the register operands tie later uses
// of the loaded values to the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : VCB_RW16(r)::"memory");
}

__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[16], uint32_t (&s)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : VCB_RW16(r), VCB_RW16(s)::"memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      VCB_IN16(r)
      : "memory");
}

// Four consecutive columns (short tail chunks).
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[4], uint32_t (&s)[4]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(s[0]), "+r"(s[1]),
                 "+r"(s[2]), "+r"(s[3])::"memory");
}

__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&r)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// x = hi + lo with hi rounded to nearest at TF32 precision (10 explicit
// mantissa bits) and lo the exact fp32 remainder.
__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  const uint32_t u = __float_as_uint(x);
  const bool finite = (u & 0x7F800000u) != 0x7F800000u;
  const uint32_t h = finite ? ((u + 0x1000u) & 0xFFFFE000u) : u;
  hi = h;
  lo = __float_as_uint(finite ? __fsub_rn(x, __uint_as_float(h)) : 0.f);
}

// As tf32_split, with lo also rounded to nearest at TF32 precision (the
// tensor cores read only a TF32 operand's top 19 bits): hi + lo is within
// 2^-24 |x| of x.
__device__ __forceinline__ void tf32_split_rn(float x, uint32_t& hi, uint32_t& lo) {
  tf32_split(x, hi, lo);
  lo = (lo + 0x1000u) & 0xFFFFE000u;
}

}  // namespace tc5
}  // namespace vcb
