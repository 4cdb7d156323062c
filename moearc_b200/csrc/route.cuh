// route.cuh — pieces shared by the decode path (moe.cu) and the prefill path (prefill.cu), so
// both select the same experts with the same weights, apply the same activation and read the
// packed expert tiles the same way: warp argmax, the top-k of one token with its gating weights,
// SwiGLU / SwiGLU-OAI, and the E2M1 / Q4_0 decode and block scales of a packed tile.
#pragma once
#include "common.cuh"

namespace moearc {

// SwiGLU (act 0: silu(g) * u, reference.rs:369-372) or SwiGLU-OAI (act 1, reference.rs:386-396).
__device__ __forceinline__ float act_fn(int act, float g, float u, float alpha, float limit) {
    if (act == 1) {
        const float x = fminf(g, limit);
        const float y = fminf(fmaxf(u, -limit), limit);
        return (x / (1.0f + expf(alpha * (-x)))) * (y + 1.0f);
    }
    return (g / (1.0f + expf(-g))) * u;
}

// Argmax across the warp of each lane's candidate (bv at index bi; bi = 0x7FFFFFFF for none),
// the lower index winning a tie, in two integer reductions: the largest order-preserving key of
// the value (-0 counts as +0, so equal logits tie), then the lowest index holding it. Every
// lane gets the winner. NaN logits are outside the contract (reference.rs:616 rejects them).
__device__ __forceinline__ void warp_argmax(float &bv, int &bi) {
    unsigned kb = 0;  // no candidate in this lane
    if (bi != 0x7FFFFFFF) {
        unsigned b = __float_as_uint(bv);
        if (b == 0x80000000u) b = 0;
        kb = max((b & 0x80000000u) ? ~b : (b | 0x80000000u), 1u);
    }
    const unsigned km = __reduce_max_sync(0xffffffffu, kb);
    const unsigned gi = __reduce_min_sync(0xffffffffu, (kb == km && kb != 0) ? (unsigned)bi : 0xFFFFFFFFu);
    bi = (gi == 0xFFFFFFFFu) ? 0x7FFFFFFF : (int)gi;
    bv = __shfl_sync(0xffffffffu, bv, gi & 31);
}

// Top-k of one token by one warp (reference.rs:613-640 semantics, as topk_token): k rounds of
// argmax over the logits held in registers (lower id wins a tie), then the gating weights.
template <int MAXP>  // logits per lane: E <= 32 MAXP
__device__ void xtopk_n(const float *logits, int E, int K, int gating, int lane, unsigned *idx, float *wts) {
    float v[MAXP];
#pragma unroll
    for (int i = 0; i < MAXP; ++i) {
        const int j = lane + 32 * i;
        v[i] = (j < E) ? __ldcg(logits + j) : -INFINITY;
    }
    uint32_t taken = 0;
    float my_v = -INFINITY;
    int my_i = 0;
    for (int r = 0; r < K; ++r) {
        float bv = -INFINITY;
        int bi = 0x7FFFFFFF;
#pragma unroll
        for (int i = 0; i < MAXP; ++i) {
            const int j = lane + 32 * i;
            if (j < E && !(taken & (1u << i)) && (bi == 0x7FFFFFFF || v[i] > bv)) {
                bv = v[i];
                bi = j;
            }
        }
        warp_argmax(bv, bi);
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        if (lane == r) {
            my_v = bv;
            my_i = bi;
        }
    }
    const bool mine = lane < K;
    float w;
    if (gating == 2) {
        const float smax = warp_max(mine ? my_v : -INFINITY);
        const float e = mine ? expf(my_v - smax) : 0.f;
        w = e / warp_sum(e);
    } else {
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < MAXP; ++i) mx = fmaxf(mx, v[i]);
        mx = warp_max(mx);
        float part = 0.f;
#pragma unroll
        for (int i = 0; i < MAXP; ++i)
            if (lane + 32 * i < E) part += expf(v[i] - mx);
        const float denom = warp_sum(part);
        w = mine ? expf(my_v - mx) / denom : 0.f;
        if (gating == 1) w /= fmaxf(warp_sum(w), 6.103515625e-5f);
    }
    if (mine) {
        idx[lane] = (unsigned)my_i;
        wts[lane] = w;
    }
}

__device__ __forceinline__ void xtopk(const float *logits, int E, int K, int gating, int lane, unsigned *idx, float *wts) {
    if (E <= 64) xtopk_n<2>(logits, E, K, gating, lane, idx, wts);
    else if (E <= 128) xtopk_n<4>(logits, E, K, gating, lane, idx, wts);
    else if (E <= 256) xtopk_n<8>(logits, E, K, gating, lane, idx, wts);
    else xtopk_n<32>(logits, E, K, gating, lane, idx, wts);
}

// ---- packed expert tiles (moearc_x_moe_pack's layout): decode of one lane's bytes ----------

// Four E2M1 pairs (the four bytes of w, low nibble first) -> four f16x2 of true values.
__device__ __forceinline__ void e2m1x8(uint32_t w, uint32_t (&r)[4]) {
    asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
        " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
        : "r"(w));
}

// Four Q4_0 byte pairs -> four f16x2 of (nibble - 8), exactly: each nibble is set into the
// mantissa of 1024.0 (0x6400), then 1032 is subtracted.
__device__ __forceinline__ void q4x8(uint32_t w, uint32_t (&r)[4]) {
    const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t b = (w >> (8 * k)) & 0xFFu;
        const uint32_t t = (b & 0x0Fu) | ((b & 0xF0u) << 12) | 0x64006400u;
        __half2 h = *reinterpret_cast<const __half2 *>(&t);
        h = __hsub2(h, bias);
        r[k] = *reinterpret_cast<uint32_t *>(&h);
    }
}

template <int WT>
__device__ __forceinline__ void decode4(uint32_t w, uint32_t (&r)[4]) {
    if constexpr (WT == 39) e2m1x8(w, r);
    else q4x8(w, r);
}

// The scale of (row r or r+8, block b0 or b0+1) from the lane's scale word(s), as the factor
// the block's MMA sum is multiplied by: MXFP4 2 * 2^(e-128) = 2^(e-127) (the E2M1 values
// decoded are the true ones, half the reference's doubled table, reference.rs:51-70), built
// by moving the byte into the f32 exponent field — exact for e >= 1; e = 0 (2^-127, a
// subnormal) becomes 0, an absolute difference below 6 * 2^-127 * sum|x| per block. Q4_0:
// the f16 delta.
template <int WT>
__device__ __forceinline__ void scales4(const uint8_t *tile, int r, float (&s)[4]) {
    if constexpr (WT == 39) {
        const uint32_t e = *reinterpret_cast<const uint32_t *>(tile + 512 + 4 * r);
        s[0] = __uint_as_float((e << 23) & 0x7F800000u);
        s[1] = __uint_as_float((e << 15) & 0x7F800000u);
        s[2] = __uint_as_float((e << 7) & 0x7F800000u);
        s[3] = __uint_as_float((e >> 1) & 0x7F800000u);
    } else {
        const uint2 d = *reinterpret_cast<const uint2 *>(tile + 512 + 8 * r);
        s[0] = f16_bits_to_f32((uint16_t)(d.x & 0xFFFF));
        s[1] = f16_bits_to_f32((uint16_t)(d.x >> 16));
        s[2] = f16_bits_to_f32((uint16_t)(d.y & 0xFFFF));
        s[3] = f16_bits_to_f32((uint16_t)(d.y >> 16));
    }
}

}  // namespace moearc
