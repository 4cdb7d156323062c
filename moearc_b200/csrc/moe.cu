// moe.cu — the fused MoE FFN for decode on B200: route, gate‖up + SwiGLU, down + combine.
//
// Semantics are the reference's MoE block (crates/moearc-engine/src/moe.rs:2074-2427): router
// logits = W_r . x (+ bias before the top-k), top-k with the three gatings, per chosen expert
// g = gate . x, u = up . x, a = act(g, u), o = down . a, out = sum over the k experts, in
// router order, of w_m * o_m — plus the residual add that follows it (moe.rs:2422-2425).
//
// What is B200-specific is everything else:
//
// * The expert banks are re-laid once at load into tensor-core fragment order ("packed"): a
//   tile is 16 rows x 64 columns (two quantisation blocks), its 512 bytes of nibbles ordered
//   so that lane l's 16 contiguous bytes are exactly the A-fragment bytes of two
//   m16n8k16 MMAs per block, followed by the tile's 16x2 scales. Bytes per block are unchanged
//   (17 for MXFP4, 18 for Q4_0). Gate and up tiles of the same rows are interleaved, so one
//   warp streams one contiguous run for both.
// * There is no host readback of the router's choice (the reference's largest phase,
//   moe.rs:2121-2149): the routing kernel writes a device-side slot table, and the expert
//   kernels read it.
// * The expert kernels are persistent grouped GEMVs. Each warp owns a sequence of items
//   (expert slot, 16-row tile-row, chunk of k-tiles), pulls each item's contiguous weight run
//   and activation fragments into its shared memory with one TMA bulk copy per run (two
//   stages, mbarrier-tracked), decodes E2M1 with the hardware converter (Q4_0 with an exact
//   f16 bias trick) and multiplies on the tensor cores. The activation enters the MMA as two
//   f16 columns, its f16 rounding and the rounding residual, so the product carries ~22 bits
//   of the f32 activation (f32 check-mode accuracy, 1e-4); the weights are exact in f16.
// * Split-K partials go to scratch and the last warp to finish a unit (found with one atomic
//   counter per unit, reset by that warp) reduces them in a fixed order: deterministic, no
//   floating-point atomics. For gate‖up that warp applies the activation; for down it applies
//   the router weights in router order and the residual.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <vector>

#include "common.cuh"
#include "tma.cuh"

using namespace moearc;

// ---- the state behind the opaque moearc_x_moe handle of include/moearc.h -------------------
struct moearc_x_moe {
    moearc_ctx *ctx;
    // shape
    int H, I, E, K, wtype, gating, act;
    float alpha, limit;
    int T_max;
    // derived
    int tile_bytes;  // one packed tile (16 rows x 64 cols)
    int nkt_h, nkt_i, ntr_h, ntr_i;
    int kc_gu, nch_gu, kc_dn, nch_dn;
    int stage_gu, stage_dn;  // bytes per warp per stage
    int grid_gu, grid_dn;
    // device scratch (one allocation)
    void *mem;
    size_t mem_bytes;
    float *logits;     // [T_max][E]
    unsigned *idx;     // [T_max][K]
    float *wts;        // [T_max][K]
    int *tables;       // slot / group / column tables, see k_route
    uint32_t *xfrag;   // [T_max][H/32][2][4][4] u32
    uint32_t *actfrag; // [T_max*K][I/32][2][4][4] u32
    float *act_f32;    // [T_max*K][I], the activation, kept for inspection
    float *part_gu;    // [nch_gu][T_max*K][I][2]
    float *part_dn;    // [nch_dn][T_max*K][H]
    unsigned *ctr;     // route done counter, gate-up unit counters, down unit counters
    int *status;
};

namespace {

constexpr int WARPS = 4;   // per CTA of the expert kernels
constexpr int STAGES = 2;
constexpr int GROUP = 4;   // tokens per column group (2 MMA columns each)

// Layout of the int tables written by k_route (offsets in ints):
//   [0] n_slots, [1] n_groups, [2] n_cols
//   grp_slot[G], grp_col0[G], grp_ntok[G], slot_expert[S], col_tok[C], col_of[T*K]
struct tab_view {
    int *base;
    int G, S, C, TK;
    __host__ __device__ int *n_slots() const { return base; }
    __host__ __device__ int *n_groups() const { return base + 1; }
    __host__ __device__ int *n_cols() const { return base + 2; }
    __host__ __device__ int *grp_slot() const { return base + 4; }
    __host__ __device__ int *grp_col0() const { return grp_slot() + G; }
    __host__ __device__ int *grp_ntok() const { return grp_col0() + G; }
    __host__ __device__ int *slot_expert() const { return grp_ntok() + G; }
    __host__ __device__ int *col_tok() const { return slot_expert() + S; }
    __host__ __device__ int *col_of() const { return col_tok() + C; }
    static size_t ints(int G, int S, int C, int TK) { return 4 + 3 * (size_t)G + S + C + TK; }
};

// ---- packing ------------------------------------------------------------------------------

// Packed tile (16 rows r0..r0+15 x 64 columns = blocks b0, b0+1):
//   bytes [16 l, 16 l + 16) for lane l = 4 r + q (r < 8, q < 4):
//     [0..4)  qs bytes 4q..4q+3 of row r,   block b0
//     [4..8)  qs bytes 4q..4q+3 of row r+8, block b0
//     [8..12) qs bytes 4q..4q+3 of row r,   block b0+1
//     [12..16) qs bytes 4q..4q+3 of row r+8, block b0+1
//   then the scales of rows r and r+8 for blocks b0, b0+1:
//     MXFP4: 4 bytes at 512 + 4 r: e(r,b0), e(r+8,b0), e(r,b0+1), e(r+8,b0+1)
//     Q4_0:  8 bytes at 512 + 8 r: the four f16 deltas in the same order
__global__ void k_pack(uint8_t *dst, const uint8_t *src, size_t n_tiles_per_mat, int n_mat,
                       int ntr, int nkt, int bb, int qs_off, int tile_bytes, int dst_stride_tiles,
                       int dst_tile_step, int dst_tile_off) {
    // one thread per (matrix, tile, lane)
    const size_t total = (size_t)n_mat * n_tiles_per_mat * 32;
    const size_t nb = (size_t)nkt * 2;  // blocks per row
    const int sb = bb - 16;             // scale bytes per block (1 or 2)
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < total; g += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(g & 31);
        const size_t t = (g >> 5) % n_tiles_per_mat;
        const size_t m = (g >> 5) / n_tiles_per_mat;
        const int tr = (int)(t / nkt), tk = (int)(t % nkt);
        const int r = lane >> 2, q = lane & 3;
        const uint8_t *mat = src + m * (size_t)ntr * 16 * nb * bb;
        uint8_t *tile = dst + (m * (size_t)dst_stride_tiles + t * dst_tile_step + dst_tile_off) * tile_bytes;
        const size_t rowA = (size_t)tr * 16 + r, rowB = rowA + 8;
        const size_t bA = (size_t)tk * 2, bB = bA + 1;
        const uint8_t *pA0 = mat + (rowA * nb + bA) * bb, *pB0 = mat + (rowB * nb + bA) * bb;
        const uint8_t *pA1 = mat + (rowA * nb + bB) * bb, *pB1 = mat + (rowB * nb + bB) * bb;
        uint8_t *o = tile + lane * 16;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            o[j] = pA0[qs_off + 4 * q + j];
            o[4 + j] = pB0[qs_off + 4 * q + j];
            o[8 + j] = pA1[qs_off + 4 * q + j];
            o[12 + j] = pB1[qs_off + 4 * q + j];
        }
        if (q == 0) {
            uint8_t *s = tile + 512 + r * 4 * sb;
            const uint8_t *src4[4] = {pA0, pB0, pA1, pB1};
#pragma unroll
            for (int i = 0; i < 4; ++i)
                for (int k = 0; k < sb; ++k) s[i * sb + k] = src4[i][k];
        }
    }
}

// ---- device helpers ---------------------------------------------------------------------

__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

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
// the block's MMA sum is multiplied by: MXFP4 2 * 2^(e-128) (the E2M1 values decoded are
// the true ones, half the reference's doubled table, reference.rs:51-70); Q4_0 the delta.
template <int WT>
__device__ __forceinline__ void scales4(const uint8_t *tile, int r, float (&s)[4]) {
    if constexpr (WT == 39) {
        const uint32_t e = *reinterpret_cast<const uint32_t *>(tile + 512 + 4 * r);
#pragma unroll
        for (int i = 0; i < 4; ++i) s[i] = 2.0f * e8m0_half((e >> (8 * i)) & 0xFFu);
    } else {
        const uint2 d = *reinterpret_cast<const uint2 *>(tile + 512 + 8 * r);
        s[0] = f16_bits_to_f32((uint16_t)(d.x & 0xFFFF));
        s[1] = f16_bits_to_f32((uint16_t)(d.x >> 16));
        s[2] = f16_bits_to_f32((uint16_t)(d.y & 0xFFFF));
        s[3] = f16_bits_to_f32((uint16_t)(d.y >> 16));
    }
}

// One packed tile against the column group's B fragments: acc[c] += tile . x for rows
// r, r+8 (c0,c1 row r; c2,c3 row r+8), columns 2q, 2q+1.
// bfr: the lane's B registers for this k-tile: [block][mma][2].
template <int WT>
__device__ __forceinline__ void tile_mma(const uint8_t *tile, int lane, const uint32_t (&bfr)[2][2][2],
                                         float (&acc)[4]) {
    const uint4 w = *reinterpret_cast<const uint4 *>(tile + lane * 16);
    float s[4];
    scales4<WT>(tile, lane >> 2, s);
    uint32_t a[4][4];
    decode4<WT>(w.x, a[0]);  // row r,   block 0
    decode4<WT>(w.y, a[1]);  // row r+8, block 0
    decode4<WT>(w.z, a[2]);  // row r,   block 1
    decode4<WT>(w.w, a[3]);  // row r+8, block 1
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t(&ar)[4] = a[2 * blk];
        const uint32_t(&br)[4] = a[2 * blk + 1];
        // k-slots (2q, 2q+1) <- byte 4q+j's pair (elements 4q+j, 4q+j+16), j = 0 for a0/a1 of
        // the first MMA, j = 1 for a2/a3; the second MMA takes j = 2, 3.
        mma_f16(d, ar[0], br[0], ar[1], br[1], bfr[blk][0][0], bfr[blk][0][1]);
        mma_f16(d, ar[2], br[2], ar[3], br[3], bfr[blk][1][0], bfr[blk][1][1]);
        const float sr = s[blk * 2], sr8 = s[blk * 2 + 1];
        acc[0] = fmaf(d[0], sr, acc[0]);
        acc[1] = fmaf(d[1], sr, acc[1]);
        acc[2] = fmaf(d[2], sr8, acc[2]);
        acc[3] = fmaf(d[3], sr8, acc[3]);
    }
}

// B fragment registers of lane (n = lane/4, q = lane%4) for one k-tile (two blocks) from a
// staged fragment buffer laid [token][block][part][q][4 x u32], where the token is column
// group member n/2 and part = n%2 (0: f16 rounding, 1: residual). Members past ntok get zero.
__device__ __forceinline__ void load_b(const uint32_t *bsm, int blocks_staged, int kt, int lane, int ntok,
                                       uint32_t (&bfr)[2][2][2]) {
    const int n = lane >> 2, q = lane & 3, tt = n >> 1, part = n & 1;
    if (tt < ntok) {
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
            const uint4 v = *reinterpret_cast<const uint4 *>(
                bsm + ((((size_t)tt * blocks_staged + 2 * kt + blk) * 2 + part) * 4 + q) * 4);
            bfr[blk][0][0] = v.x;
            bfr[blk][0][1] = v.y;
            bfr[blk][1][0] = v.z;
            bfr[blk][1][1] = v.w;
        }
    } else {
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) bfr[blk][0][0] = bfr[blk][0][1] = bfr[blk][1][0] = bfr[blk][1][1] = 0u;
    }
}

// f32 -> (f16 rounding, f16 of the residual) for two values, packed as two f16x2.
__device__ __forceinline__ void split_f16x2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half ah = __float2half_rn(a), bh = __float2half_rn(b);
    const __half al = __float2half_rn(a - __half2float(ah)), bl = __float2half_rn(b - __half2float(bh));
    hi = (uint32_t)__half_as_ushort(ah) | ((uint32_t)__half_as_ushort(bh) << 16);
    lo = (uint32_t)__half_as_ushort(al) | ((uint32_t)__half_as_ushort(bl) << 16);
}

__device__ __forceinline__ float act_fn(int act, float g, float u, float alpha, float limit) {
    if (act == 1) {
        const float x = fminf(g, limit);
        const float y = fminf(fmaxf(u, -limit), limit);
        return (x / (1.0f + expf(alpha * (-x)))) * (y + 1.0f);
    }
    return (g / (1.0f + expf(-g))) * u;
}

// ---- kernel 1: routing --------------------------------------------------------------------

struct route_args {
    const float *x;       // [T][H]
    const float *router;  // [E][H]
    const float *rbias;   // [E] or null
    int T, H, E, K, gating;
    float *logits;
    unsigned *idx;
    float *wts;
    uint32_t *xfrag;
    tab_view tab;
    unsigned *done;
};

__device__ void topk_token(const route_args &a, int t, int lane) {
    const float *l = a.logits + (size_t)t * a.E;
    const unsigned nper = (a.E + 31) / 32;
    uint32_t taken = 0;
    float my_v = -INFINITY;
    int my_i = 0;
    for (int r = 0; r < a.K; ++r) {
        float bv = -INFINITY;
        int bi = 0x7FFFFFFF;
        for (unsigned i = 0; i < nper; ++i) {
            const int j = lane + 32 * i;
            if (j < a.E && !(taken & (1u << i))) {
                const float v = __ldcg(l + j);
                if (bi == 0x7FFFFFFF || v > bv || (v == bv && j < bi)) {
                    bv = v;
                    bi = j;
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7FFFFFFF && (bi == 0x7FFFFFFF || ov > bv || (ov == bv && oi < bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        if (lane == r) {
            my_v = bv;
            my_i = bi;
        }
    }
    const bool mine = lane < a.K;
    if (mine) a.idx[(size_t)t * a.K + lane] = (unsigned)my_i;
    float w;
    if (a.gating == 2) {
        const float smax = warp_max(mine ? my_v : -INFINITY);
        const float e = mine ? expf(my_v - smax) : 0.f;
        w = e / warp_sum(e);
    } else {
        float mx = -INFINITY;
        for (int j = lane; j < a.E; j += 32) mx = fmaxf(mx, __ldcg(l + j));
        mx = warp_max(mx);
        float part = 0.f;
        for (int j = lane; j < a.E; j += 32) part += expf(__ldcg(l + j) - mx);
        const float denom = warp_sum(part);
        w = mine ? expf(my_v - mx) / denom : 0.f;
        if (a.gating == 1) w /= fmaxf(warp_sum(w), 6.103515625e-5f);
    }
    if (mine) a.wts[(size_t)t * a.K + lane] = w;
}

__global__ void __launch_bounds__(256) k_route(route_args a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = blockIdx.x * 8 + warp, nw = gridDim.x * 8;
    // (a) router logits, the fixed order of moearc_matvec_f32 (reproducible on the host)
    for (int row = gw; row < a.T * a.E; row += nw) {
        const int t = row / a.E, e = row % a.E;
        const float *wr = a.router + (size_t)e * a.H;
        const float *xr = a.x + (size_t)t * a.H;
        float acc = 0.f;
        for (int c4 = lane; c4 < a.H / 4; c4 += 32) {
            const float4 w4 = __ldg(reinterpret_cast<const float4 *>(wr) + c4);
            const float4 x4 = __ldg(reinterpret_cast<const float4 *>(xr) + c4);
            acc = fmaf(w4.x, x4.x, acc);
            acc = fmaf(w4.y, x4.y, acc);
            acc = fmaf(w4.z, x4.z, acc);
            acc = fmaf(w4.w, x4.w, acc);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) a.logits[row] = a.rbias ? acc + a.rbias[e] : acc;
    }
    // (b) x -> B fragments: [t][block][part][q][j] = pair (x[32b+4q+j], x[32b+4q+16+j])
    const int nblk = a.H / 32;
    for (int i = blockIdx.x * 256 + threadIdx.x; i < a.T * nblk * 16; i += gridDim.x * 256) {
        const int j = i & 3, q = (i >> 2) & 3;
        const int tb = i >> 4, t = tb / nblk, b = tb % nblk;
        const float *xr = a.x + (size_t)t * a.H + 32 * b;
        uint32_t hi, lo;
        split_f16x2(xr[4 * q + j], xr[4 * q + 16 + j], hi, lo);
        a.xfrag[((((size_t)t * nblk + b) * 2 + 0) * 4 + q) * 4 + j] = hi;
        a.xfrag[((((size_t)t * nblk + b) * 2 + 1) * 4 + q) * 4 + j] = lo;
    }
    // the last CTA to finish does the top-k and builds the slot tables
    __shared__ unsigned last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = (atomicAdd(a.done, 1u) == gridDim.x - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int t = warp; t < a.T; t += 8) topk_token(a, t, lane);
    __threadfence_block();
    __syncthreads();
    // slots: distinct experts ascending; a slot's columns are its tokens in token order
    __shared__ int cnt[1024];
    for (int e = threadIdx.x; e < a.E; e += 256) cnt[e] = 0;
    __syncthreads();
    const int TK = a.T * a.K;
    for (int e = threadIdx.x; e < a.E; e += 256) {
        int c = 0;
        for (int i = 0; i < TK; ++i) c += (a.idx[i] == (unsigned)e);
        cnt[e] = c;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int s = 0, g = 0, col = 0;
        for (int e = 0; e < a.E; ++e) {
            const int n = cnt[e];
            if (!n) continue;
            a.tab.slot_expert()[s] = e;
            for (int m0 = 0; m0 < n; m0 += GROUP) {
                a.tab.grp_slot()[g] = s;
                a.tab.grp_col0()[g] = col + m0;
                a.tab.grp_ntok()[g] = min(GROUP, n - m0);
                ++g;
            }
            cnt[e] = col;  // from here on: the next free column of expert e's slot
            col += n;
            ++s;
        }
        *a.tab.n_slots() = s;
        *a.tab.n_groups() = g;
        *a.tab.n_cols() = col;
        // a slot's columns are its tokens in token order (i runs token-major)
        for (int i = 0; i < TK; ++i) {
            const int e = (int)a.idx[i];
            const int c = cnt[e]++;
            a.tab.col_of()[i] = c;
            a.tab.col_tok()[c] = i / a.K;
        }
        *a.done = 0;
    }
}

// ---- kernels 2 and 3: the grouped expert GEMVs ---------------------------------------------

struct gemv_args {
    const uint8_t *bank;      // packed gate-up (2 tiles per k-tile) or down bank
    size_t bank_stride;       // bytes per expert
    int mats;                 // 2 for gate-up, 1 for down
    int ntr, nkt, kc, nch;    // tile-rows, k-tiles per row, k-tiles per chunk, chunks
    int tile_bytes;
    int stage_bytes;
    const uint32_t *bsrc;     // B fragments, indexed by token (gate-up) or column (down)
    int b_by_column;          // 0: bsrc row = token of the column, 1: row = the column itself
    int nblk_b;               // blocks per B row
    tab_view tab;
    // gate-up epilogue
    int act;
    float alpha, limit;
    uint32_t *actfrag;        // [col][I/32][2][4][4]
    float *act_out;           // [col][I] f32, optional
    int I;
    // down epilogue
    const float *wts;         // [T][K]
    const float *residual;    // [T][H] or null
    float *out;               // [T][H]
    int T, K, H;
    float *part;
    unsigned *ctr;
    int *status;
};

// Item i -> (group, tile-row, chunk).
__device__ __forceinline__ void item_of(const gemv_args &a, int i, int &g, int &tr, int &ch) {
    ch = i % a.nch;
    const int r = i / a.nch;
    tr = r % a.ntr;
    g = r / a.ntr;
}

__device__ __forceinline__ void issue_item(const gemv_args &a, int item, uint8_t *stage, uint64_t *bar,
                                           int lane) {
    int g, tr, ch;
    item_of(a, item, g, tr, ch);
    const int slot = a.tab.grp_slot()[g];
    const int expert = a.tab.slot_expert()[slot];
    const int col0 = a.tab.grp_col0()[g], ntok = a.tab.grp_ntok()[g];
    const int k0 = ch * a.kc;
    const int kn = min(a.kc, a.nkt - k0);
    const unsigned wbytes = (unsigned)(kn * a.mats * a.tile_bytes);
    const unsigned bbytes_tok = (unsigned)(2 * kn * 128);
    if (lane == 0) {
        fence_proxy_async();
        mbar_expect_tx(bar, wbytes + bbytes_tok * ntok);
        const uint8_t *w = a.bank + (size_t)expert * a.bank_stride +
                           ((size_t)tr * a.nkt + k0) * a.mats * a.tile_bytes;
        bulk_g2s(stage, w, wbytes, bar);
        uint8_t *bs = stage + a.kc * a.mats * a.tile_bytes;
        for (int t = 0; t < ntok; ++t) {
            const int col = col0 + t;
            const int row = a.b_by_column ? col : a.tab.col_tok()[col];
            const uint32_t *src = a.bsrc + ((size_t)row * a.nblk_b + 2 * k0) * 32;
            bulk_g2s(bs + (size_t)t * a.kc * 2 * 128, src, bbytes_tok, bar);
        }
    }
}

template <int WT>
__global__ void __launch_bounds__(WARPS * 32) k_expert_gemv(gemv_args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[WARPS][STAGES];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = blockIdx.x * WARPS + warp, nw = gridDim.x * WARPS;
    uint8_t *my = smem + (size_t)warp * STAGES * a.stage_bytes;
    if (lane == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    const int n_items = *a.tab.n_groups() * a.ntr * a.nch;
    unsigned phase[STAGES] = {0u, 0u};
    bool pending[STAGES] = {false, false};
    // prologue: the first two items
    for (int s = 0; s < STAGES; ++s) {
        const int it = gw + s * nw;
        if (it < n_items) {
            issue_item(a, it, my + s * a.stage_bytes, &bars[warp][s], lane);
            pending[s] = true;
        }
    }
    int stage = 0;
    for (int it = gw; it < n_items; it += nw) {
        uint8_t *st = my + stage * a.stage_bytes;
        const bool ok = mbar_wait(&bars[warp][stage], phase[stage], a.status);
        phase[stage] ^= 1u;
        pending[stage] = false;
        if (!ok) break;  // status raised; the host reports it
        int g, tr, ch;
        item_of(a, it, g, tr, ch);
        const int ntok = a.tab.grp_ntok()[g], col0 = a.tab.grp_col0()[g];
        const int k0 = ch * a.kc, kn = min(a.kc, a.nkt - k0);
        const uint32_t *bsm = reinterpret_cast<const uint32_t *>(st + a.kc * a.mats * a.tile_bytes);
        float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
        for (int kt = 0; kt < kn; ++kt) {
            uint32_t bfr[2][2][2];
            load_b(bsm, 2 * a.kc, kt, lane, ntok, bfr);
            const uint8_t *tile = st + (size_t)kt * a.mats * a.tile_bytes;
            tile_mma<WT>(tile, lane, bfr, acc0);
            if (a.mats == 2) tile_mma<WT>(tile + a.tile_bytes, lane, bfr, acc1);
        }
        __syncwarp();
        // the stage is free: start the item after next into it
        const int nxt = it + STAGES * nw;
        if (nxt < n_items) {
            issue_item(a, nxt, st, &bars[warp][stage], lane);
            pending[stage] = true;
        }
        stage = (stage + 1) % STAGES;

        // partial: lane (r, q) holds column pair (2q, 2q+1) = (f16 part, residual part) of
        // group member q, rows r and r+8.
        const int r = lane >> 2, q = lane & 3;
        const int row0 = tr * 16 + r;
        const int ncol = *a.tab.n_cols();
        if (q < ntok) {
            const int col = col0 + q;
            if (a.mats == 2) {
                float *p = a.part + (((size_t)ch * ncol + col) * a.I) * 2;
                p[(size_t)row0 * 2] = acc0[0] + acc0[1];
                p[(size_t)row0 * 2 + 1] = acc1[0] + acc1[1];
                p[(size_t)(row0 + 8) * 2] = acc0[2] + acc0[3];
                p[(size_t)(row0 + 8) * 2 + 1] = acc1[2] + acc1[3];
            } else {
                float *p = a.part + ((size_t)ch * ncol + col) * a.H;
                p[row0] = acc0[0] + acc0[1];
                p[row0 + 8] = acc0[2] + acc0[3];
            }
        }
        __threadfence();
        __syncwarp();
        // the unit: (group, tile-row) for gate-up, tile-row for down
        unsigned prev = 0;
        const int unit = (a.mats == 2) ? g * a.ntr + tr : tr;
        const unsigned target = (a.mats == 2) ? (unsigned)a.nch : (unsigned)(*a.tab.n_groups() * a.nch);
        if (lane == 0) prev = atomicAdd(a.ctr + unit, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev != target - 1) continue;
        __threadfence();
        if (lane == 0) a.ctr[unit] = 0;  // ready for the next call
        if (a.mats == 2) {
            // gate-up unit complete: reduce the chunks in order, apply the activation, write
            // the activation both as f32 and as the down GEMV's B fragments.
            const int nblk_i = a.I / 32;
            for (int e = lane; e < ntok * 16; e += 32) {
                const int t = e / 16, rr = e % 16;
                const int col = col0 + t, row = tr * 16 + rr;
                float gsum = 0.f, usum = 0.f;
                for (int c = 0; c < a.nch; ++c) {
                    const float *p = a.part + (((size_t)c * ncol + col) * a.I + row) * 2;
                    gsum += __ldcg(p);
                    usum += __ldcg(p + 1);
                }
                const float v = act_fn(a.act, gsum, usum, a.alpha, a.limit);
                if (a.act_out) a.act_out[(size_t)col * a.I + row] = v;
                const __half hh = __float2half_rn(v);
                const __half hl = __float2half_rn(v - __half2float(hh));
                // element el of block blk sits in pair j = el & 3 of lane q = (el & 15) >> 2,
                // in the low half for el < 16 and the high half for el >= 16
                const int blk = row / 32, el = row % 32;
                const int qq = (el & 15) >> 2, jj = el & 3, half = el >> 4;
                const size_t ihi = ((((size_t)col * nblk_i + blk) * 2 + 0) * 4 + qq) * 4 + jj;
                const size_t ilo = ((((size_t)col * nblk_i + blk) * 2 + 1) * 4 + qq) * 4 + jj;
                reinterpret_cast<uint16_t *>(a.actfrag + ihi)[half] = __half_as_ushort(hh);
                reinterpret_cast<uint16_t *>(a.actfrag + ilo)[half] = __half_as_ushort(hl);
            }
        } else {
            // down tile-row complete: out[t][row] = residual + sum_m w[t][m] * o_(t,m)[row],
            // m ascending (router order), each o the chunks summed in order.
            for (int e = lane; e < a.T * 16; e += 32) {
                const int t = e / 16, row = tr * 16 + e % 16;
                float acc = 0.f;
                for (int m = 0; m < a.K; ++m) {
                    const int col = a.tab.col_of()[t * a.K + m];
                    float o = 0.f;
                    for (int c = 0; c < a.nch; ++c) o += __ldcg(a.part + ((size_t)c * ncol + col) * a.H + row);
                    acc = fmaf(a.wts[t * a.K + m], o, acc);
                }
                a.out[(size_t)t * a.H + row] = a.residual ? a.residual[(size_t)t * a.H + row] + acc : acc;
            }
        }
    }
    // no bulk copy may still be landing in this warp's shared memory when the CTA exits
    for (int s = 0; s < STAGES; ++s)
        if (pending[s]) mbar_wait(&bars[warp][s], phase[s], a.status);
}

// Choose the chunk length (k-tiles per item) that best balances `units` rows of `nkt` k-tiles
// over `nw` warps: the makespan in k-tiles plus a fixed per-item cost, minimised.
int pick_kc(long units, int nkt, long nw, int kc_max) {
    int best = 1;
    double best_cost = 1e30;
    for (int kc = 1; kc <= std::min(kc_max, nkt); ++kc) {
        const long nch = (nkt + kc - 1) / kc;
        const long items = units * nch;
        const long per_warp = (items + nw - 1) / nw;
        const double cost = (double)per_warp * (kc + 1.5);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = kc;
        }
    }
    return best;
}

}  // namespace

// ---- host side ----------------------------------------------------------------------------

namespace {

tab_view make_tab(const moearc_x_moe *m) {
    const int TK = m->T_max * m->K;
    tab_view t;
    t.base = m->tables;
    t.G = TK;
    t.S = std::min(TK, m->E);
    t.C = TK;
    t.TK = TK;
    return t;
}

int occupancy_grid(moearc_ctx *c, int smem_per_cta) {
    // 228 KB of shared memory per SM, 1 KB of it reserved per resident CTA
    int per_sm = (228 * 1024) / (std::max(smem_per_cta, 1) + 1024 + 64);
    per_sm = std::max(1, std::min(per_sm, 4));
    return c->sm_count * per_sm;
}

}  // namespace

extern "C" {

moearc_x_moe *moearc_x_moe_create(moearc_ctx *c, const moearc_x_moe_desc *d) {
    if (!c || !d) return nullptr;
    if (d->wtype != T_MXFP4 && d->wtype != T_Q4_0) return nullptr;
    if (d->n_embd % 64 || d->n_ff % 64 || d->n_embd % 4) return nullptr;
    if (d->k == 0 || d->k > (unsigned)MAX_TOPK || d->k > d->n_expert || d->n_expert > 1024) return nullptr;
    if (d->gating > 2 || d->act > 1 || d->max_tokens == 0) return nullptr;
    auto *m = new moearc_x_moe();
    m->ctx = c;
    m->H = (int)d->n_embd;
    m->I = (int)d->n_ff;
    m->E = (int)d->n_expert;
    m->K = (int)d->k;
    m->wtype = (int)d->wtype;
    m->gating = (int)d->gating;
    m->act = (int)d->act;
    m->alpha = d->alpha;
    m->limit = d->limit;
    m->T_max = (int)d->max_tokens;
    m->tile_bytes = (d->wtype == T_MXFP4) ? 544 : 576;
    m->nkt_h = m->H / 64;
    m->nkt_i = m->I / 64;
    m->ntr_h = m->H / 16;
    m->ntr_i = m->I / 16;
    const int TK = m->T_max * m->K;
    const int tok_group = std::min(GROUP, m->T_max);
    // Balance the chunking for the expected number of column groups (k at batch 1).
    const long groups = std::min<long>(TK, std::max<long>(m->K, std::min(m->E, TK)));
    const long nw = (long)c->sm_count * 2 * WARPS;
    m->kc_gu = pick_kc(groups * m->ntr_i, m->nkt_h, nw, 8);
    m->kc_dn = pick_kc(groups * m->ntr_h, m->nkt_i, nw, 16);
    m->nch_gu = (m->nkt_h + m->kc_gu - 1) / m->kc_gu;
    m->nch_dn = (m->nkt_i + m->kc_dn - 1) / m->kc_dn;
    auto round128 = [](int b) { return (b + 127) & ~127; };
    m->stage_gu = round128(m->kc_gu * 2 * m->tile_bytes + tok_group * 2 * m->kc_gu * 128);
    m->stage_dn = round128(m->kc_dn * 1 * m->tile_bytes + tok_group * 2 * m->kc_dn * 128);
    m->grid_gu = occupancy_grid(c, WARPS * STAGES * m->stage_gu);
    m->grid_dn = occupancy_grid(c, WARPS * STAGES * m->stage_dn);

    // one scratch allocation
    const size_t n_tab = tab_view::ints(TK, std::min(TK, m->E), TK, TK);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) & ~size_t(255);
        return o;
    };
    const size_t o_logits = take(sizeof(float) * m->T_max * m->E);
    const size_t o_idx = take(sizeof(unsigned) * TK);
    const size_t o_wts = take(sizeof(float) * TK);
    const size_t o_tab = take(sizeof(int) * n_tab);
    const size_t o_xf = take((size_t)m->T_max * (m->H / 32) * 128);
    const size_t o_af = take((size_t)TK * (m->I / 32) * 128);
    const size_t o_act = take(sizeof(float) * (size_t)TK * m->I);
    const size_t o_pgu = take(sizeof(float) * (size_t)m->nch_gu * TK * m->I * 2);
    const size_t o_pdn = take(sizeof(float) * (size_t)m->nch_dn * TK * m->H);
    const size_t n_ctr = 1 + (size_t)TK * m->ntr_i + m->ntr_h;
    const size_t o_ctr = take(sizeof(unsigned) * n_ctr);
    const size_t o_st = take(sizeof(int));
    m->mem_bytes = off;
    if (cudaMalloc(&m->mem, off) != cudaSuccess) {
        cudaGetLastError();
        delete m;
        return nullptr;
    }
    uint8_t *b = static_cast<uint8_t *>(m->mem);
    m->logits = reinterpret_cast<float *>(b + o_logits);
    m->idx = reinterpret_cast<unsigned *>(b + o_idx);
    m->wts = reinterpret_cast<float *>(b + o_wts);
    m->tables = reinterpret_cast<int *>(b + o_tab);
    m->xfrag = reinterpret_cast<uint32_t *>(b + o_xf);
    m->actfrag = reinterpret_cast<uint32_t *>(b + o_af);
    m->part_gu = reinterpret_cast<float *>(b + o_pgu);
    m->part_dn = reinterpret_cast<float *>(b + o_pdn);
    m->ctr = reinterpret_cast<unsigned *>(b + o_ctr);
    m->status = reinterpret_cast<int *>(b + o_st);
    m->act_f32 = reinterpret_cast<float *>(b + o_act);
    cudaMemsetAsync(m->mem, 0, off, c->stream);
    const int smem_max = WARPS * STAGES * std::max(m->stage_gu, m->stage_dn);
    if (cudaFuncSetAttribute(k_expert_gemv<39>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max) != cudaSuccess ||
        cudaFuncSetAttribute(k_expert_gemv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(m->mem);
        delete m;
        return nullptr;
    }
    return m;
}

void moearc_x_moe_destroy(moearc_x_moe *m) {
    if (!m) return;
    cudaStreamSynchronize(m->ctx->stream);
    cudaFree(m->mem);
    delete m;
}

unsigned long moearc_x_moe_packed_bytes(const moearc_x_moe_desc *d, int which) {
    if (!d) return 0;
    const unsigned long bb = (d->wtype == T_MXFP4) ? 17 : (d->wtype == T_Q4_0 ? 18 : 0);
    const unsigned long blocks = (unsigned long)d->n_embd * d->n_ff / 32;
    return which == 0 ? 2 * blocks * bb : blocks * bb;
}

int moearc_x_moe_pack(moearc_x_moe *m, const void *gate, const void *up, const void *down,
                      unsigned n_expert, void *gateup_packed, void *down_packed) {
    if (!m || !gate || !up || !down || !gateup_packed || !down_packed) return ERR;
    if ((reinterpret_cast<uintptr_t>(gateup_packed) | reinterpret_cast<uintptr_t>(down_packed)) & 15) return ERR_ARG;
    moearc_ctx *c = m->ctx;
    const int bb = (m->wtype == T_MXFP4) ? 17 : 18, qs_off = bb - 16;
    const size_t tiles_gu = (size_t)m->ntr_i * m->nkt_h, tiles_dn = (size_t)m->ntr_h * m->nkt_i;
    launch_scope ls(c, "moe_pack", (unsigned long)n_expert, 3);
    const unsigned th = 256;
    auto grid = [&](size_t work) { return (unsigned)std::min<size_t>((work + th - 1) / th, (size_t)c->sm_count * 64); };
    auto *gu = static_cast<uint8_t *>(gateup_packed);
    k_pack<<<grid(n_expert * tiles_gu * 32), th, 0, c->stream>>>(gu, static_cast<const uint8_t *>(gate), tiles_gu, (int)n_expert, m->ntr_i, m->nkt_h, bb, qs_off, m->tile_bytes, (int)(2 * tiles_gu), 2, 0);
    k_pack<<<grid(n_expert * tiles_gu * 32), th, 0, c->stream>>>(gu, static_cast<const uint8_t *>(up), tiles_gu, (int)n_expert, m->ntr_i, m->nkt_h, bb, qs_off, m->tile_bytes, (int)(2 * tiles_gu), 2, 1);
    k_pack<<<grid(n_expert * tiles_dn * 32), th, 0, c->stream>>>(static_cast<uint8_t *>(down_packed), static_cast<const uint8_t *>(down), tiles_dn, (int)n_expert, m->ntr_h, m->nkt_i, bb, qs_off, m->tile_bytes, (int)tiles_dn, 1, 0);
    return ls.finish();
}

int moearc_x_moe_forward(moearc_x_moe *m, const float *x, unsigned n_tokens, const float *router_w,
                         const float *router_b, const void *gateup_packed, const void *down_packed,
                         const float *residual, float *out) {
    if (!m || !x || !router_w || !gateup_packed || !down_packed || !out) return ERR;
    if (n_tokens == 0) return OK;
    if ((int)n_tokens > m->T_max) return ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(router_w) |
         reinterpret_cast<uintptr_t>(gateup_packed) | reinterpret_cast<uintptr_t>(down_packed)) & 15)
        return ERR_ARG;
    moearc_ctx *c = m->ctx;
    const int T = (int)n_tokens;
    const tab_view tab = make_tab(m);
    launch_scope ls(c, "moe_forward", (unsigned long)m->H, (unsigned)T);

    route_args ra{x, router_w, router_b, T, m->H, m->E, m->K, m->gating, m->logits, m->idx, m->wts,
                  m->xfrag, tab, m->ctr};
    const int rows_ctas = (T * m->E + 7) / 8;
    const int conv_ctas = (T * (m->H / 32) * 16 + 255) / 256;
    const int grid_r = std::max(1, std::min(std::max(rows_ctas, conv_ctas), c->sm_count * 2));
    k_route<<<grid_r, 256, 0, c->stream>>>(ra);

    gemv_args ga{};
    ga.bank = static_cast<const uint8_t *>(gateup_packed);
    ga.bank_stride = (size_t)2 * m->ntr_i * m->nkt_h * m->tile_bytes;
    ga.mats = 2;
    ga.ntr = m->ntr_i;
    ga.nkt = m->nkt_h;
    ga.kc = m->kc_gu;
    ga.nch = m->nch_gu;
    ga.tile_bytes = m->tile_bytes;
    ga.stage_bytes = m->stage_gu;
    ga.bsrc = m->xfrag;
    ga.b_by_column = 0;
    ga.nblk_b = m->H / 32;
    ga.tab = tab;
    ga.act = m->act;
    ga.alpha = m->alpha;
    ga.limit = m->limit;
    ga.actfrag = m->actfrag;
    ga.act_out = m->act_f32;
    ga.I = m->I;
    ga.T = T;
    ga.K = m->K;
    ga.H = m->H;
    ga.part = m->part_gu;
    ga.ctr = m->ctr + 1;
    ga.status = m->status;
    const size_t smem_gu = (size_t)WARPS * STAGES * m->stage_gu;
    if (m->wtype == T_MXFP4) k_expert_gemv<39><<<m->grid_gu, WARPS * 32, smem_gu, c->stream>>>(ga);
    else k_expert_gemv<2><<<m->grid_gu, WARPS * 32, smem_gu, c->stream>>>(ga);

    gemv_args da = ga;
    da.bank = static_cast<const uint8_t *>(down_packed);
    da.bank_stride = (size_t)m->ntr_h * m->nkt_i * m->tile_bytes;
    da.mats = 1;
    da.ntr = m->ntr_h;
    da.nkt = m->nkt_i;
    da.kc = m->kc_dn;
    da.nch = m->nch_dn;
    da.stage_bytes = m->stage_dn;
    da.bsrc = m->actfrag;
    da.b_by_column = 1;
    da.nblk_b = m->I / 32;
    da.wts = m->wts;
    da.residual = residual;
    da.out = out;
    da.part = m->part_dn;
    da.ctr = m->ctr + 1 + (size_t)m->T_max * m->K * m->ntr_i;
    const size_t smem_dn = (size_t)WARPS * STAGES * m->stage_dn;
    if (m->wtype == T_MXFP4) k_expert_gemv<39><<<m->grid_dn, WARPS * 32, smem_dn, c->stream>>>(da);
    else k_expert_gemv<2><<<m->grid_dn, WARPS * 32, smem_dn, c->stream>>>(da);
    return ls.finish();
}

void *moearc_x_moe_buffer(moearc_x_moe *m, int which) {
    if (!m) return nullptr;
    switch (which) {
    case 0: return m->idx;
    case 1: return m->wts;
    case 2: return m->act_f32;
    case 3: return m->logits;
    case 4: return m->tables;
    default: return nullptr;
    }
}

int moearc_x_moe_status(moearc_x_moe *m) {
    if (!m) return ERR;
    int st = 0;
    if (cudaMemcpyAsync(&st, m->status, sizeof(int), cudaMemcpyDeviceToHost, m->ctx->stream) != cudaSuccess) return ERR;
    if (cudaStreamSynchronize(m->ctx->stream) != cudaSuccess) return ERR;
    if (st) cudaMemsetAsync(m->status, 0, sizeof(int), m->ctx->stream);
    return st;
}

}  // extern "C"
