// ============================================================================
//  mbarrier.cuh -- shared-memory barriers and bulk async copies (sm_100a).
//
//  Thin wrappers over the PTX mbarrier / cp.async.bulk instructions used by
//  the pipelined kernels (tensor-core GEMM, heavy-row gather).  Every wait is
//  bounded in time: after kWaitNs of the global nanosecond timer (2 s; a
//  try_wait may itself suspend for a while, so the bound is not a poll count)
//  it records a code in the caller's device error word and returns false, so
//  a kernel can drain and exit instead of spinning forever.
// ============================================================================
#pragma once

#include <cstdint>

namespace tg {
namespace mb {

constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Makes barrier initialisation visible to the async proxy and other threads.
__device__ __forceinline__ void fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// One arrival that also expects `bytes` of async-copy completions.
__device__ __forceinline__ void arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase of parity `parity` to complete; false (and
// `code` recorded in *err unless one is there already) when it runs out.
__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (try_wait(bar, parity)) return true;
        if ((i & 15) == 0 && global_ns() - t0 > kWaitNs) break;  // the timer read is not free
        if (i > 32) __nanosleep(64);
    }
    atomicCAS(err, 0, code);
    return false;
}

// Bounded wait for a thread whose wait is not on the critical path: it
// sleeps from the first failed poll, leaving issue slots to the warps that
// share its SM sub-partition.
__device__ __forceinline__ bool wait_sleepy(uint64_t* bar, uint32_t parity, int* err, int code, uint32_t sleep_ns) {
    if (try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        __nanosleep(sleep_ns);
        if (try_wait(bar, parity)) return true;
        if ((i & 15) == 0 && global_ns() - t0 > kWaitNs) break;
    }
    atomicCAS(err, 0, code);
    return false;
}

// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned), completion counted on `bar`.  No multicast.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 16-byte global -> shared async copy through the load/store units (L1
// bypassed, L2 policy hint); both addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;"
                 ::"r"(smem_u32(dst)), "l"(src), "l"(policy)
                 : "memory");
}

// 4-byte global -> shared async copy (L1-allocating form; 4-byte aligned).
__device__ __forceinline__ void cp_async4(void* dst, const void* src, uint64_t policy) {
    asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 4, %2;"
                 ::"r"(smem_u32(dst)), "l"(src), "l"(policy)
                 : "memory");
}

// One arrival on `bar` once every cp.async this thread issued so far has
// landed (counts against the barrier's expected arrivals: no increment).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

}  // namespace mb
}  // namespace tg
