// Fifth-generation tensor core (tcgen05) building blocks for sm_100a:
// tensor-memory (TMEM) allocation, TMEM loads/stores, shared-memory operand
// descriptors, the instruction descriptor of kind::f16 and the MMA/commit
// instructions.  Inline PTX; the encodings follow the public PTX ISA for
// tcgen05 (descriptor bit layout as in CUTLASS cute/arch/mma_sm100_desc.hpp).
//
// TMEM addresses: bits [31:16] lane, [15:0] column (32-bit cells).  A warp
// may touch only its lane quadrant: lanes 32*(warp % 4) .. +31.
#pragma once

#include "qwz_common.cuh"

namespace qwz {
namespace tc {

// ------------------------------------------------------------- allocation
// One full warp allocates `ncols` (power of two, 32..512) columns; the base
// address is written to shared memory at `smem_dst`.
QWZ_DEVINL void tmem_alloc(uint32_t smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_dst),
               "r"(ncols)
               : "memory");
}
QWZ_DEVINL void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
QWZ_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// ----------------------------------------------------------------- fences
// Order tcgen05 operations across a thread synchronisation (barrier or
// mbarrier): `before` ahead of the signal, `after` behind the wait.
QWZ_DEVINL void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
QWZ_DEVINL void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
QWZ_DEVINL void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
QWZ_DEVINL void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// ----------------------------------------------------------- TMEM <-> regs
// 32x32b: thread i of the warp <-> lane (quadrant base + i); consecutive
// registers <-> consecutive columns.
QWZ_DEVINL void st_32x32b_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}
QWZ_DEVINL void st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
QWZ_DEVINL void ld_32x32b_x4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr)
               : "memory");
}
QWZ_DEVINL void st_32x32b_x4(uint32_t taddr, const uint32_t (&r)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}
QWZ_DEVINL void ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
QWZ_DEVINL void ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
      "%13, %14, %15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
// 16x256b: 16 lanes x 8 columns; thread t holds (lane base + t/4, columns
// 2(t%4), 2(t%4)+1) in r0, r1 and (lane base + t/4 + 8, same columns) in
// r2, r3 -- the mma.sync m16n8 accumulator layout.
QWZ_DEVINL void st_16x256b(uint32_t taddr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("tcgen05.st.sync.aligned.16x256b.x1.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(taddr), "r"(r0),
               "r"(r1), "r"(r2), "r"(r3)
               : "memory");
}
QWZ_DEVINL void ld_16x256b(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x1.b32 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr)
               : "memory");
}

// ------------------------------------------------------------ descriptors
// Shared-memory operand, K-major with the 128-byte swizzle: rows of 128 B
// (64 f16 of K), 8-row groups 1 KB apart, group bases 1024-byte aligned.
// A K=16 step inside the 128-byte row advances the start address by 32 B.
QWZ_DEVINL uint64_t smem_desc_k128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
  d |= (uint64_t)1u << 16;                          // leading byte offset (unused when swizzled)
  d |= (uint64_t)(1024u >> 4) << 32;                // stride byte offset: next 8-row group
  d |= (uint64_t)1u << 46;                          // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                          // SWIZZLE_128B
  return d;
}

// Shared-memory operand, MN-major with the 128-byte swizzle: rows of 128 B
// hold 64 f16 of M (or N) for one K index; 8 K rows form a 1 KB atom.
// lbo = byte distance between atoms along M/N (the next 64 elements), sbo =
// byte distance between atoms along K (the next 8 K rows).
QWZ_DEVINL uint64_t smem_desc_mn128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: F16 A and B, F32
// accumulator, M x N; A and B K-major unless a_mn_major / b_mn_major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N, bool b_mn_major = false,
                                                     bool a_mn_major = false) {
  return (1u << 4) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------------- MMA
// D[tmem] (+)= A * B^T with A in TMEM (K-major: lane = row, column = K
// pair) and B from a shared-memory descriptor.  Issued by one thread.
QWZ_DEVINL void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// Both operands from shared-memory descriptors.
QWZ_DEVINL void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// Arrive once on the mbarrier when every tcgen05.mma this thread issued so
// far has completed.
QWZ_DEVINL void commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(mbar)
               : "memory");
}

}  // namespace tc
}  // namespace qwz
