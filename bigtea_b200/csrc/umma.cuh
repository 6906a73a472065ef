// 5th-generation tensor cores (tcgen05) for the integer K-quant contractions: shared-memory
// operand descriptors, the instruction descriptor of kind::i8, TMEM allocation, the MMA, its
// commit to an mbarrier and the TMEM -> register loads. Inline PTX for sm_100a.
//
// Operand layout (both operands K-major, no swizzle): a core matrix is 8 rows x 16 bytes,
// stored as 128 contiguous bytes; the two 16-byte halves of one 32-byte K step are LBO bytes
// apart and consecutive groups of 8 rows SBO bytes apart. One MMA of kind::i8 covers K = 32.
#pragma once

#include <stdint.h>

namespace bt {

// Shared-memory matrix descriptor: start address, LBO and SBO in 16-byte units, version 1,
// no swizzle.
__device__ __forceinline__ uint64_t umma_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version for sm_100
    return d;                // base offset 0, absolute LBO mode, layout type 0 (no swizzle)
}

// Instruction descriptor of kind::i8: D s32, A unsigned 8-bit, B signed 8-bit, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_u8s8(int M, int N) {
    return (2u << 4)                        // D format: s32
           | (0u << 7)                      // A: unsigned 8-bit
           | (1u << 10)                     // B: signed 8-bit
           | ((uint32_t)(N >> 3) << 17)     // N / 8
           | ((uint32_t)(M >> 4) << 24);    // M / 16
}

// One warp: allocate `ncols` TMEM columns (a power of two >= 32); the base address lands in
// shared memory at `dst`.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A . B^T for one K step; issued by one thread.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t"
        "}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

// The mbarrier arrives once every MMA this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint32_t mbar_smem) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar_smem)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Warp w reads TMEM lanes 32(w % 4) .. +31, 16 consecutive 32-bit columns from `taddr`
// (lane in the upper 16 bits of the address, column in the lower 16): thread i gets row
// 32 (w % 4) + i.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

// As tmem_ld16 for 8 columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}

// After tcgen05.wait::ld: makes every later use of v depend on this point, so the compiler
// cannot read a loaded register before the wait.
template <int N>
__device__ __forceinline__ void tmem_pin(uint32_t (&v)[N]) {
#pragma unroll
    for (int i = 0; i < N; i++) asm volatile("" : "+r"(v[i]));
}

// Per-thread asynchronous 16-byte copies global -> shared (L1 bypassed), grouped by
// commit_group; wait_group<N> returns once at most N of this thread's newest groups are still
// in flight, and the data of the completed ones is then visible to this thread.
__device__ __forceinline__ void cp_async16(uint32_t dst_smem, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst_smem), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Byte offset of (row, k) in a K-major, no-swizzle operand tile of 32-byte K steps:
// K step s = k / 32 at s * rows * 32; inside it, core matrix (row / 8, (k % 32) / 16).
__host__ __device__ constexpr uint32_t umma_off(int row, int k, int rows) {
    return (uint32_t)((k >> 5) * rows * 32 + (row >> 3) * 256 + ((k >> 4) & 1) * 128 + (row & 7) * 16 + (k & 15));
}

}  // namespace bt
