// tc.cuh — fifth-generation tensor core (tcgen05) building blocks for sm_100a: TMA tile loads,
// mbarrier waits with a time limit, UMMA shared-memory and instruction descriptors, the MMA
// issue and commit, and TMEM loads. Descriptor bit layouts follow the PTX ISA's tcgen05 matrix
// descriptor and instruction descriptor tables (kind::f16).
#pragma once
#include <cuda.h>
#include <cstdint>

namespace moearc {
namespace tc {

constexpr unsigned long long WAIT_NS = 500000000ull;  // a wait gives up after 0.5 s

__device__ __forceinline__ uint32_t sa(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void bar_init(uint64_t *b, unsigned n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(n));
}
__device__ __forceinline__ void bar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void bar_expect_tx(uint64_t *b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t *b, unsigned parity) {
    unsigned ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok)
                 : "r"(sa(b)), "r"(parity)
                 : "memory");
    return ok;
}
// Wait for the phase of `parity` to complete. Gives up (false) when *abort is set by another
// role, or after WAIT_NS, in which case it sets *abort and ORs `code` into *status.
__device__ __forceinline__ bool bar_wait(uint64_t *b, unsigned parity, volatile int *abort, int *status, int code) {
    if (bar_try(b, parity)) return true;
    const unsigned long long t0 = now_ns();
    while (!bar_try(b, parity)) {
        if (*abort) return false;
        if (now_ns() - t0 > WAIT_NS) {
            atomicOr(status, code);
            *abort = 1;
            return false;
        }
    }
    return true;
}
// Bounded wait that ignores aborts (drains before exit).
__device__ __forceinline__ void bar_drain(uint64_t *b, unsigned parity) {
    const unsigned long long t0 = now_ns();
    while (!bar_try(b, parity) && now_ns() - t0 < WAIT_NS) {
    }
}

// 2-D tiled TMA load (box given by the tensor map) into shared memory, completing on `bar`.
// c0 is the innermost coordinate in elements; its byte offset must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            sa(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(sa(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored in the 128-byte swizzle
// canonical layout (rows of 64 bf16, 8-row groups 1024 bytes apart): start address >> 4 in bits
// 0-13, leading byte offset 16 B (>> 4 = 1) in bits 16-29, stride byte offset 1024 B (>> 4) in
// bits 32-45, descriptor version 1 in bits 46-47, base offset 0 (tiles 1024-byte aligned), swizzle
// mode 2 (128 B) in bits 61-63. Advancing the start address by 32 B steps K by 16 elements.
__device__ __forceinline__ uint64_t desc_k_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}
// Instruction descriptor for kind::f16: D f32 (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12 = 1),
// both K-major (bits 15, 16 = 0), N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// The same with A and B f16 (bits 7-9, 10-12 = 0); A and B of one MMA always share a type.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// D[tmem] (+)= A[smem] . B[smem]^T, one elected thread; accumulate = 0 overwrites D.
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
// `bar` gets one arrival once every MMA this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(bar)) : "memory");
}
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Warp-wide TMEM column allocation; the base address lands in *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(slot)), "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols));
}
// 16 consecutive f32 columns of this thread's TMEM lane (warp w reads lanes 32 (w % 4) ..).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace tc
}  // namespace moearc
