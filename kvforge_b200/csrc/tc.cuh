// tc.cuh - 5th-generation tensor-core (tcgen05) building blocks for sm_100a:
// tensor-memory (TMEM) allocation, shared-memory matrix descriptors, the
// instruction descriptor of kind::i8 MMAs, the MMA issue itself, completion
// tracking through mbarriers and TMEM -> register loads.
//
// Descriptor layouts follow the sm100 UMMA definitions (shared-memory matrix
// descriptor: start address, leading/stride byte offsets in 16-byte units,
// version 1, swizzle mode in bits 61-63; instruction descriptor: operand and
// accumulator formats, operand majors, N >> 3 and M >> 4).
#pragma once

#include <cstdint>

namespace kvfb {
namespace tc {

// Swizzle modes of a shared-memory matrix descriptor.
enum : uint32_t { kSwizzleNone = 0, kSwizzle128 = 2, kSwizzle64 = 4, kSwizzle32 = 6 };

// Shared-memory matrix descriptor. `addr` is a shared-window byte address;
// `lbo` / `sbo` are the leading / stride byte offsets of the canonical layout.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t swz) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm100
  d |= (uint64_t)(swz & 7u) << 61;
  return d;
}

// Instruction descriptor of a kind::i8 MMA with an s32 accumulator.
//   a_signed / b_signed: operand is s8 (else u8);  a_mn / b_mn: operand is
//   MN-major (else K-major);  m in {64, 128};  n a multiple of 16 (or 8).
__host__ __device__ constexpr uint32_t idesc_i8(bool a_signed, bool b_signed, bool a_mn, bool b_mn, int m, int n) {
  return (2u << 4)                         // accumulator format: s32
         | ((a_signed ? 1u : 0u) << 7)     // A format
         | ((b_signed ? 1u : 0u) << 10)    // B format
         | ((a_mn ? 1u : 0u) << 15)        // A major
         | ((b_mn ? 1u : 0u) << 16)        // B major
         | ((uint32_t)(n >> 3) << 17)      // N
         | ((uint32_t)(m >> 4) << 24);     // M
}

// D[tmem] (+)= A * B, issued by one thread. `accumulate` false overwrites D.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       bool accumulate) {
  const uint32_t acc = accumulate ? 1u : 0u, z = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
      :
      : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc), "r"(z)
      : "memory");
}

// Arrives (once) on the mbarrier when every MMA this thread issued so far has
// completed.
__device__ __forceinline__ void commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// TMEM allocation by one whole warp; the base address lands in shared memory.
__device__ __forceinline__ void alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp receives lane
// (warp's lane base + i), columns col .. col+15.
__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

} // namespace tc
} // namespace kvfb
