// router.cu — top-k expert selection and gating weights (kernels.cpp:1495-1588).
//
// One warp per token. Selection is k rounds of a warp-wide argmax over the logits, ordered by
// (value descending, expert id ascending), so an exact tie goes to the lower id
// (reference.rs:612-617); each lane remembers which of its experts are taken in a bitmask.
// Lane r keeps round r's winner, so the gating arithmetic afterwards runs across the warp
// with no per-lane arrays.
#include <cmath>

#include "common.cuh"

using namespace moearc;

namespace {

constexpr int WARPS = 8;
constexpr unsigned MAX_EXPERTS = 1024;  // 32 per lane: one bit each in `taken`

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(WARPS * 32)
    k_topk(unsigned *__restrict__ idx, float *__restrict__ wts, const float *__restrict__ logits,
           size_t n_tokens, unsigned E, unsigned k, unsigned gating) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t t = (size_t)blockIdx.x * WARPS + warp;
    if (t >= n_tokens) return;
    const float *l = logits + t * E;
    const unsigned nper = (E + 31) / 32;
    uint32_t taken = 0;
    float my_v = -INFINITY;
    int my_i = 0;
    for (unsigned r = 0; r < k; ++r) {
        float bv = -INFINITY;
        int bi = 0x7FFFFFFF;
        for (unsigned i = 0; i < nper; ++i) {
            const unsigned j = lane + 32 * i;
            if (j < E && !(taken & (1u << i))) {
                const float v = l[j];
                if (bi == 0x7FFFFFFF || better(v, (int)j, bv, bi)) {
                    bv = v;
                    bi = (int)j;
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7FFFFFFF && (bi == 0x7FFFFFFF || better(ov, oi, bv, bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if ((unsigned)bi % 32 == (unsigned)lane) taken |= 1u << ((unsigned)bi / 32);
        if ((unsigned)lane == r) {
            my_v = bv;
            my_i = bi;
        }
    }
    const bool mine = (unsigned)lane < k;
    if (mine) idx[t * k + lane] = (unsigned)my_i;

    if (gating == 2) {
        // gpt-oss: a softmax over the k selected logits only (kernels.cpp:1541-1556).
        const float smax = warp_max(mine ? my_v : -INFINITY);
        const float e = mine ? expf(my_v - smax) : 0.f;
        const float d2 = warp_sum(e);
        if (mine) wts[t * k + lane] = e / d2;
        return;
    }
    float mx = -INFINITY;
    for (unsigned j = lane; j < E; j += 32) mx = fmaxf(mx, l[j]);
    mx = warp_max(mx);
    float part = 0.f;
    for (unsigned j = lane; j < E; j += 32) part += expf(l[j] - mx);
    const float denom = warp_sum(part);
    float w = mine ? expf(my_v - mx) / denom : 0.f;
    if (gating == 1) {
        // Qwen3: renormalise over the k, the sum clamped up to 2^-14 (kernels.cpp:1566-1574).
        const float s = warp_sum(w);
        w /= fmaxf(s, 6.103515625e-5f);
    }
    if (mine) wts[t * k + lane] = w;
}

}  // namespace

extern "C" {

int moearc_topk_router(moearc_ctx *c, unsigned int *idx, float *weights, const float *logits,
                       unsigned long n_tokens, unsigned long n_expert, unsigned int k,
                       unsigned int gating) {
    if (!c || !idx || !weights || !logits) return ERR;
    if (k == 0 || k > (unsigned)MAX_TOPK || (unsigned long)k > n_expert) return ERR_ARG;
    if (gating > 2u) return ERR_ARG;
    if (n_expert > MAX_EXPERTS) return ERR_ARG;
    if (n_tokens == 0) return OK;
    launch_scope ls(c, "topk_router", n_tokens, k);
    k_topk<<<cdiv(n_tokens, WARPS), WARPS * 32, 0, c->stream>>>(idx, weights, logits, n_tokens,
                                                                (unsigned)n_expert, k, gating);
    return ls.finish();
}

}  // extern "C"
