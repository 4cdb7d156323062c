// mma_peak.cu — the tensor cores' dense throughput per MMA kind, measured with our own tcgen05 loop.
//
// The roofline of a tensor-core kernel needs the peak of the MMA kind it issues. The pool's
// measured peaks cover bf16 only (a cuBLAS GEMM); the block-scaled kinds have no library
// measurement here, so this probe times them directly: every SM runs one CTA whose elected
// thread issues a long chain of 128 x 256 MMAs from shared-memory operands into one TMEM
// accumulator, then waits (bounded) for their completion. Operand and scale contents are
// irrelevant to the rate (zeros and whatever TMEM holds), so nothing is checked.
//   kind 0  kind::f16, bf16 x bf16 -> f32, K 16 per MMA
//   kind 1  kind::mxf8f6f4.block_scale, E4M3 x E4M3 with E8M0 scales per 32, K 32
//   kind 2  kind::mxf4.block_scale.block32, E2M1 x E2M1 with E8M0 scales per 32, K 64
//   kind 3  kind::mxf8f6f4.block_scale, E4M3 x E2M1 (B in 8-bit containers), K 32
#include "common.cuh"
#include "tc.cuh"
#include "tma.cuh"

using namespace moearc;

namespace {

constexpr int PK_M = 128, PK_N = 256;
constexpr int PK_SMEM = PK_M * 128 + PK_N * 128 + 1024;  // A and B tiles (128-byte rows) + alignment

// Block-scaled instruction descriptor: B scale id 0 (bits 4-5), A / B formats (bits 7-9, 10-12),
// K-major operands, N >> 3 (bits 17-22), E8M0 scales (bit 23), M >> 4 (bits 24-28), A scale id 0.
constexpr uint32_t idesc_block_scaled(int a_fmt, int b_fmt, int M, int N) {
    return ((uint32_t)a_fmt << 7) | ((uint32_t)b_fmt << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
           ((uint32_t)(M >> 4) << 24);
}

template <int KIND>
__device__ __forceinline__ void mma_one(uint32_t d, uint64_t da, uint64_t db, uint32_t sfa, uint32_t sfb, uint32_t acc) {
    if constexpr (KIND == 0) {
        tc::mma_bf16(d, da, db, tc::idesc_bf16_f32(PK_M, PK_N), acc);
    } else if constexpr (KIND == 2) {
        asm volatile(
            "{ .reg .pred p; setp.ne.b32 p, %5, 0;\n"
            " tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %6, [%3], [%4], p; }" ::"r"(d),
            "l"(da), "l"(db), "r"(sfa), "r"(sfb), "r"(acc), "r"(idesc_block_scaled(1, 1, PK_M, PK_N)));
    } else {
        asm volatile(
            "{ .reg .pred p; setp.ne.b32 p, %5, 0;\n"
            " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %6, [%3], [%4], p; }" ::"r"(d),
            "l"(da), "l"(db), "r"(sfa), "r"(sfb), "r"(acc),
            "r"(idesc_block_scaled(0, KIND == 3 ? 5 : 0, PK_M, PK_N)));
    }
}

template <int KIND>
__global__ void __launch_bounds__(128, 1) k_mma_peak(int iters, unsigned long long *ns, int *status) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t tslot;
    __shared__ __align__(8) uint64_t done;
    const uint32_t base = (tc::sa(smem_raw) + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base - tc::sa(smem_raw));
    for (int i = threadIdx.x; i < (PK_M + PK_N) * 128 / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
    if (threadIdx.x < 32) tc::tmem_alloc(&tslot, 512);
    if (threadIdx.x == 0) {
        tc::bar_init(&done, 1);
        tc::bar_init_fence();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // zeros visible to the tensor cores
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tslot;
    if (threadIdx.x == 0) {
        const uint64_t da = tc::desc_k_sw128(base), db = tc::desc_k_sw128(base + PK_M * 128);
        const unsigned long long t0 = tc::now_ns();
        for (int i = 0; i < iters; ++i) {
            const uint64_t step = (uint64_t)((i & 3) * 2);  // 32 bytes of K, >> 4
            mma_one<KIND>(tmem, da + step, db + step, tmem + 256, tmem + 320, i > 0 ? 1u : 0u);
        }
        tc::mma_commit(&done);
        bool ok = false;
        for (long p = 0; p < (1l << 28); ++p)
            if (tc::bar_try(&done, 0)) {
                ok = true;
                break;
            }
        if (!ok) atomicOr(status, STATUS_WAIT_TIMEOUT);
        ns[blockIdx.x] = ok ? tc::now_ns() - t0 : 0ull;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (threadIdx.x < 32) tc::tmem_dealloc(tmem, 512);
}

template <int KIND>
int launch_peak(moearc_ctx *c, int iters, unsigned long long *ns, int *status) {
    static std::atomic<bool> ready[MOEARC_MAX_DEVICES];
    if (once_per_device(ready, [] { return set_smem(k_mma_peak<KIND>, PK_SMEM); }) != cudaSuccess) return ERR;
    k_mma_peak<KIND><<<c->sm_count, 128, PK_SMEM, c->stream>>>(iters, ns, status);
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

}  // namespace

extern "C" int moearc_x_mma_peak(moearc_ctx *c, int kind, int iters, double *tflops) {
    if (!c || !tflops) return ERR;
    if (kind < 0 || kind > 3 || iters < 1 || iters > (1 << 20)) return ERR_ARG;
    unsigned long long *ns = nullptr;
    int *status = nullptr;
    if (cudaMalloc(&ns, sizeof(unsigned long long) * c->sm_count) != cudaSuccess ||
        cudaMalloc(&status, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        if (ns) cudaFree(ns);
        return ERR;
    }
    int rc = cudaMemsetAsync(status, 0, sizeof(int), c->stream) == cudaSuccess ? OK : ERR;
    if (rc == OK) {
        switch (kind) {
        case 0: rc = launch_peak<0>(c, iters, ns, status); break;
        case 1: rc = launch_peak<1>(c, iters, ns, status); break;
        case 2: rc = launch_peak<2>(c, iters, ns, status); break;
        default: rc = launch_peak<3>(c, iters, ns, status); break;
        }
    }
    std::vector<unsigned long long> h(c->sm_count);
    int st = 0;
    if (rc == OK && (cudaMemcpyAsync(h.data(), ns, sizeof(unsigned long long) * c->sm_count, cudaMemcpyDeviceToHost,
                                     c->stream) != cudaSuccess ||
                     cudaMemcpyAsync(&st, status, sizeof(int), cudaMemcpyDeviceToHost, c->stream) != cudaSuccess ||
                     cudaStreamSynchronize(c->stream) != cudaSuccess))
        rc = ERR;
    cudaFree(ns);
    cudaFree(status);
    if (rc != OK) return rc;
    if (st) return ERR;
    unsigned long long worst = 0;
    for (auto v : h) worst = v > worst ? v : worst;
    if (!worst) return ERR;
    const double k = kind == 0 ? 16.0 : (kind == 2 ? 64.0 : 32.0);
    const double flops = 2.0 * PK_M * PK_N * k * (double)iters * (double)c->sm_count;
    *tflops = flops / (double)worst / 1e3;
    return OK;
}
