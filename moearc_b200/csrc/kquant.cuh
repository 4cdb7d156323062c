// kquant.cuh — device expansion of the K-quant super-blocks (Q4_K 144 B, Q5_K 176 B, Q6_K
// 210 B per 256 elements), eight consecutive elements at a time, in the reference twin's
// arithmetic (reference.rs:154-300, ggml's dequantize_row_q{4,5,6}_K): each product and
// difference is rounded on its own (explicit _rn intrinsics, so no multiply-add is fused),
// which makes the expansion bit-exact with the twin.
#pragma once
#include "common.cuh"

namespace moearc {

__device__ __forceinline__ float kq_f16(const uint8_t *p) { return f16_bits_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

// Scale and min of sub-block j of a Q4_K / Q5_K super-block from its 12 packed bytes.
__device__ __forceinline__ void kq_scale_min(const uint8_t *q, int j, float &sc, float &m) {
    if (j < 4) {
        sc = (float)(q[j] & 63);
        m = (float)(q[j + 4] & 63);
    } else {
        sc = (float)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        m = (float)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

// Elements e0 .. e0 + 7 (e0 % 8 == 0) of the super-block at b.
template <unsigned T>
__device__ __forceinline__ void kq_decode8(const uint8_t *__restrict__ b, int e0, float (&v)[8]) {
    if constexpr (T == T_Q6_K) {
        // half n, quarter k, element l: low four bits from byte l (+32 for odd k) of the half's
        // low-nibble bytes, two high bits from bits 2k, 2k+1 of its high byte l; scale 2k + l/16
        const int n = e0 >> 7, k = (e0 >> 5) & 3, l0 = e0 & 31;
        const float d = kq_f16(b + 208);
        const float ds = __fmul_rn(d, (float)(int8_t)b[192 + 8 * n + 2 * k + (l0 >> 4)]);
        const uint8_t *ql = b + 64 * n + 32 * (k & 1), *qh = b + 128 + 32 * n;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int l = l0 + i;
            const int lo = (k >= 2) ? (ql[l] >> 4) : (ql[l] & 0xF);
            const int q = (lo | (((qh[l] >> (2 * k)) & 3) << 4)) - 32;
            v[i] = __fmul_rn(ds, (float)q);
        }
    } else {
        // run r of four, half h: nibbles of the run's 32 bytes (low first), sub-block 2r + h;
        // Q5_K adds 16 where bit 2r + h of the element's high-plane byte is set
        const int r = e0 >> 6, h = (e0 >> 5) & 1, l0 = e0 & 31;
        float sc, m;
        kq_scale_min(b + 4, 2 * r + h, sc, m);
        const float d1 = __fmul_rn(kq_f16(b), sc), m1 = __fmul_rn(kq_f16(b + 2), m);
        const uint8_t *qs = b + (T == T_Q5_K ? 48 : 16) + 32 * r;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int l = l0 + i;
            int q = h ? (qs[l] >> 4) : (qs[l] & 0xF);
            if (T == T_Q5_K && ((b[16 + l] >> (2 * r + h)) & 1)) q += 16;
            v[i] = __fsub_rn(__fmul_rn(d1, (float)q), m1);
        }
    }
}

}  // namespace moearc
