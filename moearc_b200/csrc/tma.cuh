// tma.cuh — bulk (TMA) copies global -> shared tracked by an mbarrier, with bounded waits.
//
// Every wait here gives up after a fixed number of polls, records where it gave up in a
// device status word and returns false, so a lost completion turns into an error the host
// reads instead of a kernel that never ends.
#pragma once

#include <cstdint>

namespace moearc {

// Status words a kernel may raise (bit flags, OR-ed into a device-side int).
constexpr int STATUS_WAIT_TIMEOUT = 1;
constexpr int STATUS_RANGE = 2;

__device__ __forceinline__ unsigned smem_addr(const void *p) {
    return (unsigned)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before later async-proxy
// (bulk copy) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// Bulk copy `bytes` (a multiple of 16, both addresses 16-byte aligned) global -> shared,
// completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Hint the L2 to fetch [src, src + bytes) (16-byte aligned, a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(src), "r"(bytes) : "memory");
}

// L2 policies: weights streamed once are marked to leave L2 first; bytes asked into L2 ahead of
// their use, to stay until then.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// bulk_g2s with an L2 cache policy for the bytes read.
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, unsigned bytes, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;\n" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
        : "memory");
}
// bulk_prefetch_l2 with an L2 cache policy.
__device__ __forceinline__ void prefetch_l2_hint(const void *src, unsigned bytes, uint64_t pol) {
    asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;\n" ::"l"(src), "r"(bytes), "l"(pol)
                 : "memory");
}
// CTA c of G asks L2 for its share of [p, p + bytes) (16-byte aligned), in 32 KB requests.
__device__ __forceinline__ void prefetch_share_l2(const uint8_t *p, size_t bytes, int c, int G, uint64_t pol) {
    const size_t n16 = bytes / 16, a = n16 * c / G * 16, b = n16 * (c + 1) / G * 16;
    for (size_t o = a; o < b; o += 32768) prefetch_l2_hint(p + o, (unsigned)(b - o < 32768 ? b - o : 32768), pol);
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete; at most `limit` polls (each try_wait itself
// suspends for a hardware-chosen interval). On timeout sets STATUS_WAIT_TIMEOUT in *status.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity, int *status,
                                          unsigned limit = 1u << 22) {
    for (unsigned i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (status) atomicOr(status, STATUS_WAIT_TIMEOUT);
    return false;
}

}  // namespace moearc
