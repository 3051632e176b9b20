// tma.cuh -- 1-D bulk asynchronous copies (global -> shared) completed on
// an mbarrier, and bounded waits on that mbarrier (sm_90+ PTX; used on
// sm_100a).
//
// A row is brought into shared memory by one thread issuing a few
// cp.async.bulk copies: the copy engine keeps the whole row in flight, so a
// CTA needs no registers or threads to reach full memory-level
// parallelism.  Every wait is bounded by wall time (%globaltimer): on
// timeout the waiter raises a status flag and gives up instead of hanging
// the GPU; the kernel then produces garbage, never a hang or a fault.
#pragma once

#include <stdint.h>

namespace tbk {

constexpr unsigned kFlagTimeout = 0x2u;  // TB_B200_FLAG_WAIT_TIMEOUT: a bounded wait gave up

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Make mbarrier.init visible to the async proxy (the bulk-copy engine).
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses (and,
// after a barrier, the CTA's) before later async-proxy writes.
__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// Bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned)
// from global to shared, completing `bytes` transactions on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// L2 eviction-priority policies for cache-hinted accesses.
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// bulk_g2s with an L2 cache policy for the source lines.
__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Ask L2 to fetch `bytes` (multiple of 16; 16-byte aligned) of global
// memory ahead of use, with an L2 cache policy.  No completion is tracked:
// a later load or copy of the same bytes simply hits L2 if it has landed.
__device__ __forceinline__ void prefetch_l2_hint(const void* src_gmem, uint32_t bytes,
                                                 uint64_t policy) {
    asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(src_gmem),
                 "r"(bytes), "l"(policy)
                 : "memory");
}

// The same prefetch with the default L2 policy.
__device__ __forceinline__ void prefetch_l2(const void* src_gmem, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src_gmem), "r"(bytes)
                 : "memory");
}

// 16-byte global load, not allocated in L1, with an L2 cache policy.
__device__ __forceinline__ float4 ld_f4_hint(const float4* p, uint64_t policy) {
    float4 v;
    asm volatile("ld.global.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p), "l"(policy));
    return v;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// How long a waiting thread may stay suspended in one try_wait (the
// hardware wakes it earlier when the phase completes).
constexpr uint32_t kSuspendHintNs = 100000;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return done != 0;
}

// A counter in shared memory published by one thread and polled by another.
__device__ __forceinline__ void st_release_shared(int* p, int v) {
    asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_addr(p)), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_shared(const int* p) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)) : "memory");
    return v;
}

// Wait for phase `parity` of `bar` to complete, at most `limit_ns`.  On
// timeout raise kFlagTimeout in *status and return false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* status,
                                          uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > limit_ns) {
            atomicOr(status, kFlagTimeout);
            return false;
        }
    }
    return true;
}

}  // namespace tbk
