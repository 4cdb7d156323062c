// xtc.cuh — the batch-1 decode experts on the block-scaled FP4 tensor cores: the tensor-core
// ("tc") layout of the MXFP4 expert banks, the E2M1 digit form of an activation, and the
// launch interface shared by moe.cu (router, forward) and xtc.cu (kernels).
//
// Why: the fragment-layout decode kernels (moe.cu, k_xexpert) decode E2M1 in registers and
// issue one mma.sync per 256 weights, which costs about as many SM cycles as streaming the bytes.
// tcgen05.mma kind::mxf4.block_scale.block32 reads MXFP4 exactly as stored — E2M1 codes, two per
// byte, with one E8M0 scale per 32 elements — so the weights go from HBM to shared memory to the
// tensor core untouched, and one thread issues every MMA of a CTA.
//
// The activation must then also be E2M1 with E8M0 block scales. It enters as digits: for each
// 32-element block, digit 0 is the block rounded to E2M1 under the scale 2^X that puts its largest
// magnitude in (3, 6], digit 1 what digit 0 left over under 2^(X - 2), and so on, each scale four
// times smaller. A remainder is at most one E2M1 spacing at the top, 2^X, i.e. at most 4 of the next
// scale (within E2M1's 6), and is computed exactly in f32, so each digit is an exact part of the
// value and TC_DIGITS_USED = 12 digits leave at most 2^(X - 22) < 2^-23 of the block's largest
// magnitude. The digits are columns of the MMA's N = 16 (the other four zero); the product for
// each is exact and accumulates in f32 in its own column, and the epilogue sums the columns from
// the smallest digit up. The fixed scale schedule keeps one block maximum (a redux) per block
// instead of one per digit: the chain from digit to digit is a multiply, the E2M1 rounding and
// its read-back, and the exact subtraction.
//
// Layouts (probed on B200: kind::mxf4 reads K-major operands in the 32-byte swizzle with 8-row
// groups 256 bytes apart, elements 2q and 2q + 1 of a row in byte q; tcgen05.cp 32x128b.warpx4
// puts byte j of 16-byte row i, word c of a scale block at TMEM lane i (all four quarters), column
// c, byte j; an MMA of scale id 2h reads bytes 2h and 2h + 1 of its scale column):
//   k-step      64 elements of K: one MMA
//   A block     one k-step of a 128-row tile: row m (32 bytes) at 32 m with its two 16-byte
//               halves swapped when bit 2 of m is set (the 32-byte swizzle): 4096 bytes
//   k-pair      two k-steps (A blocks 0, 1) and their scale block: row i (16 bytes), word c =
//               the four 32-element blocks' E8M0 bytes of tile row 32 c + i: 8704 bytes. When
//               K / 64 is odd the last k-pair holds one A block and its scale block (4608 bytes).
//   tile        128 rows x K: the k-pairs in order
//   gate-up     per expert: I / 64 tiles, tile t = gate rows 64 t .. 64 t + 63 then up rows
//               64 t .. 64 t + 63 (K = n_embd)
//   down        per expert: ceil(n_embd / 128) tiles of 128 output rows (K = n_ff); rows past
//               n_embd are zero
//   digits (B)  per k-pair 1536 bytes: two B blocks (16 digit rows x 32 bytes, the same swizzle)
//               and a scale block (row d word 0 = digit d's four block scales)
#pragma once
#include <cuda_fp16.h>
#include <cuda_fp4.h>

#include <cstddef>
#include <cstdint>

#include "common.cuh"

namespace moearc {

constexpr int TC_KSTEP = 64;
constexpr int TC_ABLK = 4096;
constexpr int TC_SFBLK = 512;
constexpr int TC_KPAIR = 2 * TC_ABLK + TC_SFBLK;     // 8704
constexpr int TC_KPAIR_HALF = TC_ABLK + TC_SFBLK;    // 4608
constexpr int TC_BBLK = 512;
constexpr int TC_BKPAIR = 2 * TC_BBLK + TC_SFBLK;    // 1536
constexpr int TC_DIGITS = 16;       // MMA columns
constexpr int TC_DIGITS_USED = 12;  // digits written (the other columns stay zero)

__host__ __device__ inline int tc_ksteps(int K) { return K / TC_KSTEP; }
__host__ __device__ inline int tc_kpairs(int K) { return (tc_ksteps(K) + 1) / 2; }
__host__ __device__ inline size_t tc_tile_bytes(int K) {
    const int ks = tc_ksteps(K);
    return (size_t)(ks / 2) * TC_KPAIR + (size_t)(ks % 2) * TC_KPAIR_HALF;
}
// bytes of one expert's gate-up / down bank in the tc layout
__host__ __device__ inline size_t tc_gu_stride(int H, int I) { return (size_t)(I / 64) * tc_tile_bytes(H); }
__host__ __device__ inline size_t tc_dn_stride(int H, int I) { return (size_t)((H + 127) / 128) * tc_tile_bytes(I); }
// bytes of one activation's digits over K
__host__ __device__ inline size_t tc_digit_bytes(int K) { return (size_t)tc_kpairs(K) * TC_BKPAIR; }

// E8M0 exponent X of an E2M1 block whose largest magnitude is amax: amax / 2^X in (3, 6]
// (6 = 1.5 x 2^2: X = e - 2 when the significand of amax is at most 1.5, else e - 1), at least
// -126 so 2^X stays a normal float.
__device__ __forceinline__ int e2m1_exp(float amax) {
    if (!(amax > 0.f)) return -126;
    const uint32_t b = __float_as_uint(amax);
    const int e = (int)((b >> 23) & 0xFF) - 127;
    return max(-126, e - 2 + (((b & 0x7FFFFF) > 0x400000u) ? 1 : 0));
}

// The TC_DIGITS_USED digits of the 32-element block b of an activation, one element per lane (the
// whole warp calls it), written into the digit buffer B (tc layout, k-pair major; rows and scale
// bytes past the used digits are never written and stay zero). E2M1 rounding by the hardware
// conversion (nearest, ties to even).
__device__ __forceinline__ void tc_write_digits(float x, int lane, uint8_t *B, int b) {
    uint8_t *kp = B + (size_t)(b >> 2) * TC_BKPAIR;
    uint8_t *blk = kp + ((b >> 1) & 1) * TC_BBLK;
    const int half = b & 1;
    int X = e2m1_exp(__uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(x)))));
    float r = x;
    unsigned long long codes = 0;
    int my_x = 0;  // lane d keeps digit d's exponent
#pragma unroll
    for (int d = 0; d < TC_DIGITS_USED; ++d) {
        const float down = __uint_as_float((uint32_t)(127 - X) << 23);  // 2^-X
        const float up = __uint_as_float((uint32_t)(127 + X) << 23);    // 2^X
        const __nv_fp4_storage_t c = __nv_cvt_float_to_fp4(r * down, __NV_E2M1, cudaRoundNearest);
        const float q = __half2float(__half(__nv_cvt_fp4_to_halfraw(c, __NV_E2M1)));
        codes |= (unsigned long long)(c & 15u) << (4 * d);
        r -= q * up;  // exact: q 2^X and r lie within a factor of two of each other, or q = 0
        if (lane == d) my_x = X;
        X = max(-126, X - 2);
    }
#pragma unroll
    for (int d = 0; d < TC_DIGITS_USED; ++d) {
        // bytes: lane 2j holds elements 2j (low nibble) and 2j + 1 (high nibble)
        const uint32_t code = (uint32_t)(codes >> (4 * d)) & 15u;
        const uint32_t byte = code | (__shfl_down_sync(0xffffffffu, code, 1) << 4);
        uint32_t w = byte | (__shfl_down_sync(0xffffffffu, byte, 2) << 8);
        w |= __shfl_down_sync(0xffffffffu, w, 4) << 16;
        if ((lane & 7) == 0) {
            const int chunk = half ^ ((d >> 2) & 1);
            *reinterpret_cast<uint32_t *>(blk + 32 * d + 16 * chunk + (lane >> 1)) = w;
        }
    }
    if (lane < TC_DIGITS_USED) kp[2 * TC_BBLK + 16 * lane + (b & 3)] = (uint8_t)(127 + my_x);
}

// One decode step's expert FFN on the tc layout (xtc.cu). The plan is per MoE layer.
struct xtc_plan;
struct xtc_run {
    const float *logits;      // router logits [E] (top-k derived by the kernels)
    const uint8_t *xdig;      // the routed activation's digits (tc_digit_bytes(H))
    const uint8_t *gu_bank, *dn_bank;  // tc-layout banks, one expert after another
    const float *residual;    // [H] or null
    float *out;               // [H]
    unsigned *idx_out;        // [K] the chosen experts, router order
    float *wts_out;           // [K] their gating weights
    float *act_out;           // [K][I] the activation (inspection)
    const float *bias_gu, *bias_dn;
    unsigned long long poll_ns;
    int phantom;
    unsigned long long *span;  // [2 kernels][span_cta][3] or null
    int span_cta;              // records per kernel (at least the grid)
    int *status;
};
// A plan, or null when the shape has no tc layout (n_embd and n_ff multiples of 64, k <= 8) or
// a CTA's share would touch more tiles than it has accumulators.
xtc_plan *xtc_create(moearc_ctx *c, int H, int I, int E, int K, int gating, int act, float alpha, float limit);
void xtc_destroy(xtc_plan *p);
int xtc_grid(const xtc_plan *p);
uint8_t *xtc_xdig(xtc_plan *p);  // the buffer the router writes the activation's digits into
void xtc_reset(xtc_plan *p);     // empty every partial slot (after a wait gave up), stream-ordered
// Enqueue the gate-up / the down kernel (PDL launches) on the context stream.
int xtc_launch_gu(xtc_plan *p, const xtc_run &r);
int xtc_launch_dn(xtc_plan *p, const xtc_run &r);
// Pack GGUF MXFP4 banks (device memory, [n_expert][rows][K / 32] blocks of 17 bytes) into the tc
// layout (gu_tc: tc_gu_stride bytes per expert, dn_tc: tc_dn_stride).
int xtc_pack(moearc_ctx *c, int H, int I, const void *gate, const void *up, const void *down, unsigned n_expert,
             void *gu_tc, void *dn_tc);

}  // namespace moearc
