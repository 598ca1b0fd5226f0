// pipe.cuh -- mbarrier / bulk-copy (TMA 1-D) / programmatic-dependent-launch primitives (sm_100a).
//
// Every wait is bounded: after kSpinLimit polls the waiter records an error code in the
// kernel's error word and gives up, so a logic error ends the kernel instead of hanging the GPU.
#pragma once
#include <stdint.h>

namespace qq3 {

constexpr uint32_t kSpinLimit = 1u << 22;

// error codes written to the kernel error word
constexpr int kErrFullWait = 1;
constexpr int kErrEmptyWait = 2;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// arrive (count 1) and add `bytes` to the transaction count of the current phase
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}

// One poll of an mbarrier phase (returns at once or after a short hardware-chosen wait).
constexpr uint32_t kWaitPolls = 1u << 22;  // a wait gives up after this many polls (~seconds)

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for completion of the phase with the given parity; false after kWaitPolls polls.  With
// backoff_ns the waiter sleeps between polls after the first few, leaving issue slots to the
// warps of its SM sub-partition (used by producer threads, whose waits are not latency-critical).
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, uint32_t backoff_ns = 0) {
    const uint32_t a = smem_u32(b);
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(a, parity)) return true;
        if (backoff_ns && i >= 4) __nanosleep(backoff_ns);
    }
    return false;
}

// Bulk global -> shared copy (16-byte aligned addresses, size a multiple of 16) completing
// as transaction bytes on mbarrier `bar`.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// The same with an L2 eviction-priority policy (createpolicy), e.g. evict-first for data read
// once.
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Bulk reduction of a shared-memory f32 vector into global memory (dst[i] += src[i], performed
// at L2), 16-byte aligned, size a multiple of 16; then wait for it to complete and order its
// writes (async proxy) before this thread's later generic accesses.
__device__ __forceinline__ void bulk_add_f32_s2g(float* dst, const float* src, uint32_t bytes) {
    asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(dst),
                 "r"(smem_u32(src)), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Make this thread's generic shared-memory writes visible to later async-proxy (bulk copy)
// reads.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Bulk prefetch of global memory into L2 (16-byte aligned address, size a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch: no-ops when the kernel was launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Named barrier over the first `threads` threads of the CTA (id 0 is __syncthreads).
__device__ __forceinline__ void named_bar(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void set_err(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

}  // namespace qq3
