// mr_umma.cuh — tcgen05 (5th-generation tensor core) and tensor-memory
// helpers for sm_100a, written as inline PTX.
//
// Conventions used by the kernels here:
//   - TMEM addresses are (lane << 16) | column. A warp may only touch the 32
//     lanes of its quadrant (warp id % 4) with tcgen05.ld / tcgen05.st.
//   - MMAs are issued by one thread; their completion is observed through
//     tcgen05.commit on an mbarrier.
//   - The A operand lives in TMEM (M = 128 lanes, K pairs of bf16 packed per
//     32-bit column), B in shared memory (K-major, 128-byte swizzle), D in
//     TMEM (fp32, one column per N).
#pragma once

#include "mr_common.cuh"

namespace mr {

// Allocates `ncols` TMEM columns (power of two >= 32) for this CTA and
// writes the base address to shared memory. Whole warp, one warp only.
MR_DEVICE void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
MR_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
MR_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Ordering of tcgen05 operations across a thread synchronisation point.
MR_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MR_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive (once) on `bar` when every tcgen05 operation this thread issued
// before has completed.
MR_DEVICE void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// D[128 x N] (+)= A[128 x 16] . B[16 x N]; A from TMEM, B by shared-memory
// descriptor; kind::f16 (bf16 inputs here), fp32 accumulate. `acc` = 0
// overwrites D. All output lanes enabled.
MR_DEVICE void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                         uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Instruction descriptor of kind::f16: bf16 A and B (both K-major), fp32 D,
// M x N (M = 64 or 128, N a multiple of 8 / 16).
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4)                     // D format: f32
         | (1u << 7)                   // A format: bf16
         | (1u << 10)                  // B format: bf16
         | ((uint32_t)(n >> 3) << 17)  // N / 8
         | ((uint32_t)(m >> 4) << 24); // M / 16
}

// Shared-memory descriptor of a K-major operand in the canonical 128-byte
// swizzled layout: rows of 128 bytes (64 bf16 of K), 8-row atoms of 1024
// bytes stacked along N/M (stride 1024). `addr` is the shared address of
// the K slice the MMA starts at (atom base + 32 bytes per 16-element step).
MR_DEVICE uint64_t umma_desc_sw128(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu)  // start address
         | ((uint64_t)1 << 16)              // leading byte offset (unused with swizzle)
         | ((uint64_t)(1024 >> 4) << 32)    // stride byte offset: 8-row atom
         | ((uint64_t)1 << 46)              // descriptor version (sm_100)
         | ((uint64_t)2 << 61);             // layout: 128-byte swizzle
}

// 32 consecutive 32-bit TMEM columns of this thread's lane <- v.
MR_DEVICE void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
MR_DEVICE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 16 consecutive 32-bit TMEM columns of this thread's lane -> v, waiting for
// the load inside the same statement so no use of v can move above the wait.
MR_DEVICE void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace mr
