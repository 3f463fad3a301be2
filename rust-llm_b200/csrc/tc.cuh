// Fifth-generation tensor core (tcgen05) helpers for sm_100a: tensor memory
// allocation, shared-memory matrix descriptors, the kind::f16 MMA in its two
// operand forms, commits to mbarriers, and the 32x32b tensor-memory loads and
// stores.  Written from the PTX ISA's description of these instructions.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace rl {
namespace tc {

// ---- tensor memory ----------------------------------------------------------
// One warp allocates `ncols` columns (a power of two >= 32) and writes the
// base address to `dst` (shared); the same warp frees them.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- descriptors ------------------------------------------------------------
// Shared-memory matrix descriptor (sm_100 layout): start address, leading and
// stride byte offsets (all in 16-byte units), version 1, swizzle mode in bits
// 61-63 (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes,
                                              uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;  // version
    d |= (uint64_t)2 << 61;  // 128-byte swizzle
    return d;
}

// Instruction descriptor of kind::f16 with bf16 A and B and an f32
// accumulator; b_mn_major selects an N-major B.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool b_mn_major) {
    return (1u << 4)                          // D: f32
           | (1u << 7)                        // A: bf16
           | (1u << 10)                       // B: bf16
           | ((b_mn_major ? 1u : 0u) << 16)   // B major
           | ((uint32_t)(N >> 3) << 17)       // N / 8
           | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// ---- MMA ----------------------------------------------------------------------
// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
// Arrive once on `bar` when every MMA this thread issued so far is complete.
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// ---- tensor memory <-> registers (32 lanes x 32 bits per thread-lane) ---------
#define RL_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), \
                 "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
// 32 consecutive columns of this thread's lane
__device__ __forceinline__ void ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : RL_R8(0), RL_R8(8), RL_R8(16), RL_R8(24)
        : "r"(taddr));
}
#undef RL_R8
#define RL_W8(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), \
                 "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])
__device__ __forceinline__ void st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, "
        "%10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, "
        "%27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        RL_W8(0), RL_W8(8), RL_W8(16), RL_W8(24)
        : "memory");
}
__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, "
        "%10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        RL_W8(0), RL_W8(8)
        : "memory");
}
#undef RL_W8
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace tc
}  // namespace rl
