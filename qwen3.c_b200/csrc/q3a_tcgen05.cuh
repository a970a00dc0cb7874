// q3a_tcgen05.cuh -- inline-PTX wrappers for the sm_100a tensor cores
// (tcgen05.mma with fp32 accumulators in tensor memory), shared by the
// prefill and the bf16 decode kernels.
#pragma once

#include "q3a_common.cuh"

namespace q3a {

// Shared-memory matrix descriptor, 128B swizzle, descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D (tensor memory) (+)= A (shared-memory descriptor) . B (shared-memory descriptor)
__device__ __forceinline__ void tc_mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(
            d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}

// D (tensor memory) (+)= A (tensor memory) . B (shared-memory descriptor)
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(
            d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

#define Q3A_TC_LD32(taddr, r, base)                                                               \
    asm volatile(                                                                                 \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14," \
        "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"           \
        : "=r"(r[base + 0]), "=r"(r[base + 1]), "=r"(r[base + 2]), "=r"(r[base + 3]),            \
          "=r"(r[base + 4]), "=r"(r[base + 5]), "=r"(r[base + 6]), "=r"(r[base + 7]),            \
          "=r"(r[base + 8]), "=r"(r[base + 9]), "=r"(r[base + 10]), "=r"(r[base + 11]),          \
          "=r"(r[base + 12]), "=r"(r[base + 13]), "=r"(r[base + 14]), "=r"(r[base + 15]),        \
          "=r"(r[base + 16]), "=r"(r[base + 17]), "=r"(r[base + 18]), "=r"(r[base + 19]),        \
          "=r"(r[base + 20]), "=r"(r[base + 21]), "=r"(r[base + 22]), "=r"(r[base + 23]),        \
          "=r"(r[base + 24]), "=r"(r[base + 25]), "=r"(r[base + 26]), "=r"(r[base + 27]),        \
          "=r"(r[base + 28]), "=r"(r[base + 29]), "=r"(r[base + 30]), "=r"(r[base + 31])         \
        : "r"(taddr))

#define Q3A_TC_ST32(taddr, r, base)                                                               \
    asm volatile(                                                                                 \
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13," \
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(    \
            taddr),                                                                               \
        "r"(r[base + 0]), "r"(r[base + 1]), "r"(r[base + 2]), "r"(r[base + 3]), "r"(r[base + 4]), \
        "r"(r[base + 5]), "r"(r[base + 6]), "r"(r[base + 7]), "r"(r[base + 8]), "r"(r[base + 9]), \
        "r"(r[base + 10]), "r"(r[base + 11]), "r"(r[base + 12]), "r"(r[base + 13]),               \
        "r"(r[base + 14]), "r"(r[base + 15]), "r"(r[base + 16]), "r"(r[base + 17]),               \
        "r"(r[base + 18]), "r"(r[base + 19]), "r"(r[base + 20]), "r"(r[base + 21]),               \
        "r"(r[base + 22]), "r"(r[base + 23]), "r"(r[base + 24]), "r"(r[base + 25]),               \
        "r"(r[base + 26]), "r"(r[base + 27]), "r"(r[base + 28]), "r"(r[base + 29]),               \
        "r"(r[base + 30]), "r"(r[base + 31])                                                     \
        : "memory")

__device__ __forceinline__ void tc_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

#define Q3A_TC_LD8(taddr, r)                                                                  \
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"          \
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),           \
                   "=r"(r[6]), "=r"(r[7])                                                           \
                 : "r"(taddr))

#define Q3A_TC_ST8(taddr, r)                                                                  \
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), \
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),       \
                 "r"(r[7])                                                                          \
                 : "memory")

}  // namespace q3a
