// tc_sm100.cuh -- small tcgen05 / UMMA helpers shared by the tensor-core kernels (sm_100a).
#pragma once
#include <stdint.h>

#include "pipe.cuh"

namespace qq3 {

// K-major, 128-byte swizzle: row r of a tile is 128 B (64 fp16 of K) at r*128; its 16-byte
// chunk c sits at chunk position c ^ (r & 7).  Tiles start on 1024-byte boundaries.
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
    return (uint32_t)row * 128u + (uint32_t)((chunk ^ (row & 7)) << 4);
}

// Shared-memory matrix descriptor (sm100 UMMA): start address >> 4, leading byte offset 1
// (unused for swizzled K-major), stride byte offset 1024 >> 4 between 8-row groups,
// version 1, layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// D (tensor memory) (+)= A . B^T, both fp16 operands from shared memory (kind::f16, f32 accumulate)
__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    const uint32_t mask[4] = {0u, 0u, 0u, 0u};
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(mask[0]), "r"(mask[1]), "r"(mask[2]), "r"(mask[3]));
}

// 16 consecutive 32-bit tensor-memory columns of this thread's lane
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

}  // namespace qq3
