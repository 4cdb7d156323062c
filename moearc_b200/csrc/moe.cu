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
#include "route.cuh"

#include <climits>
#include "tma.cuh"
#include "xtc.cuh"

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
    // gate-up (mode 0) and down (mode 1) kernel plans
    int warps_gu, ranges_gu, tpr_gu, stages_gu, stage_gu, smem_gu, grid_gu;
    int warps_dn, ranges_dn, tpr_dn, stages_dn, stage_dn, smem_dn, grid_dn;
    // decode path (T_max * K <= MAX_TK columns): k_xroute + k_xexpert
    bool xpath;
    int x_grid, x_warps, x_route_grid, x_route_smem, x_ch_gu, x_ch_dn, x_stage_gu, x_stage_dn, x_ntok;
    float *x_part_gu, *x_part_dn;  // expert kernels' piece partials (PART_EMPTY when idle)
    unsigned long long x_poll_ns = XPOLL_NS;  // their wait for one another's partials
    const float *bias_gu = nullptr, *bias_dn = nullptr;  // moearc_x_moe_set_bias
    int x_phantom = 0;                        // testing: every such wait runs out
    size_t x_part_gu_n, x_part_dn_n;
    float *f_part_gu, *f_part_dn;  // the opt-in fused kernels' (arrival counters instead)
    void *x_tab_pub;               // the gate-up kernel's routing tables, read by the down kernel
    unsigned *x_ctr_gu, *x_ctr_dn;
    // the fused decode kernel (k_moe_fused): one cooperative launch per layer
    bool fused;
    bool fused_gd;  // gate-up + down in one launch after k_xroute (opt-in)
    int f_grid, f_stage, f_smem, f_bsmem;
    unsigned *f_ready, *f_bar;
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
    unsigned *ctr;     // route done counter, gate-up unit counters, down unit counters
    int *status;
    // the batch-1 decode path on the block-scaled FP4 tensor cores (xtc.cu), for MXFP4 banks
    // packed in the tc layout; null when the shape has none
    xtc_plan *xtc = nullptr;
};

namespace {

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
    __host__ __device__ static size_t ints(int G, int S, int C, int TK) { return 4 + 3 * (size_t)G + S + C + TK; }
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


// ---- kernel 1: routing --------------------------------------------------------------------

struct route_args {
    const float *x;       // [T][H]
    const float *norm_w;  // [H]: route rmsnorm(x) * norm_w instead of x (null: x as is)
    float eps;
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
        warp_argmax(bv, bi);
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

constexpr int ROUTE_NORM_TOKENS = 64;

constexpr int ROUTE_WARPS = 4;

__global__ void __launch_bounds__(ROUTE_WARPS * 32) k_route(route_args a) {
    const int trace_row = (int)blockIdx.x;
    (void)trace_row;
    TRACE(0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = blockIdx.x * ROUTE_WARPS + warp, nw = gridDim.x * ROUTE_WARPS;
    // The router weights are static: have L2 fetch this warp's rows while the previous kernel
    // finishes.
    if (lane == 0)
        for (int row = gw; row < a.T * a.E; row += nw)
            bulk_prefetch_l2(a.router + (size_t)(row % a.E) * a.H, (unsigned)(a.H * 4));
    pdl_trigger();
    pdl_wait();
    TRACE(1);
    // (0) the RMSNorm scale of every token, when routing the normalised residual stream
    // (moe.rs:2074-2076): f32 sum of squares, 1/sqrt(mean + eps)
    __shared__ float nscale[ROUTE_NORM_TOKENS];
    if (a.norm_w) {
        for (int t = warp; t < a.T; t += ROUTE_WARPS) {
            const float4 *xr = reinterpret_cast<const float4 *>(a.x + (size_t)t * a.H);
            float ss = 0.f;
#pragma unroll 8
            for (int c = lane; c < a.H / 4; c += 32) {
                const float4 v = __ldcg(xr + c);
                ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
            }
            ss = warp_sum(ss);
            if (lane == 0) nscale[t] = 1.0f / sqrtf(ss / (float)a.H + a.eps);
        }
        __syncthreads();
    }
    // (a) router logits, the fixed order of moearc_matvec_f32 (reproducible on the host):
    // lane l folds float4 columns l, l + 32, l + 64, ... in that order; loads are batched
    // eight deep ahead of the multiply-adds, which keeps the order
    const int n4 = a.H / 4;
    for (int row = gw; row < a.T * a.E; row += nw) {
        const int t = row / a.E, e = row % a.E;
        const float4 *wr = reinterpret_cast<const float4 *>(a.router + (size_t)e * a.H);
        const float4 *xr = reinterpret_cast<const float4 *>(a.x + (size_t)t * a.H);
        const float4 *nr = reinterpret_cast<const float4 *>(a.norm_w);
        float acc = 0.f;
        for (int c0 = lane; c0 < n4; c0 += 32 * 8) {
            float4 wv[8], xv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c4 = c0 + 32 * u;
                if (c4 < n4) {
                    wv[u] = __ldg(wr + c4);
                    xv[u] = __ldcg(xr + c4);
                    if (a.norm_w) {
                        const float s = nscale[t];
                        const float4 n = __ldg(nr + c4);
                        xv[u] = make_float4((xv[u].x * s) * n.x, (xv[u].y * s) * n.y, (xv[u].z * s) * n.z,
                                            (xv[u].w * s) * n.w);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (c0 + 32 * u < n4) {
                    acc = fmaf(wv[u].x, xv[u].x, acc);
                    acc = fmaf(wv[u].y, xv[u].y, acc);
                    acc = fmaf(wv[u].z, xv[u].z, acc);
                    acc = fmaf(wv[u].w, xv[u].w, acc);
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) a.logits[row] = a.rbias ? acc + a.rbias[e] : acc;
    }
    TRACE(2);
    // (b) x -> B fragments: [t][block][part][q][j] = pair (x[32b+4q+j], x[32b+4q+16+j])
    const int nblk = a.H / 32;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.T * nblk * 16; i += gridDim.x * blockDim.x) {
        const int j = i & 3, q = (i >> 2) & 3;
        const int tb = i >> 4, t = tb / nblk, b = tb % nblk;
        const float *xr = a.x + (size_t)t * a.H + 32 * b;
        float v0 = xr[4 * q + j], v1 = xr[4 * q + 16 + j];
        if (a.norm_w) {
            const float s = nscale[t];
            v0 = (v0 * s) * a.norm_w[32 * b + 4 * q + j];
            v1 = (v1 * s) * a.norm_w[32 * b + 4 * q + 16 + j];
        }
        uint32_t hi, lo;
        split_f16x2(v0, v1, hi, lo);
        a.xfrag[((((size_t)t * nblk + b) * 2 + 0) * 4 + q) * 4 + j] = hi;
        a.xfrag[((((size_t)t * nblk + b) * 2 + 1) * 4 + q) * 4 + j] = lo;
    }
    // the last CTA to finish does the top-k and builds the slot tables
    TRACE(3);
    __shared__ unsigned last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = (atomicAdd(a.done, 1u) == gridDim.x - 1);
    __syncthreads();
    TRACE(4);
    if (!last) return;
    __threadfence();
    for (int t = warp; t < a.T; t += ROUTE_WARPS) topk_token(a, t, lane);
    TRACE(5);
    __threadfence_block();
    __syncthreads();
    // slots: distinct experts ascending; a slot's columns are its tokens in token order
    __shared__ int cnt[1024];
    for (int e = threadIdx.x; e < a.E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    const int TK = a.T * a.K;
    for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
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
        TRACE(6);
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
//
// A CTA owns a unit of output rows and nothing else touches them:
//   gate-up  unit (column group, tile-row): 16 rows of gate and up for <= 4 tokens
//   down     unit tile-row: 16 output rows for every token
// The unit's K extent is cut into `ranges` contiguous runs of k-tiles; an item is one run of
// one column group. The CTA's warps take the unit's items round-robin, each warp streaming
// its items' weight runs (and activation fragments) through its own ring of `stages`
// shared-memory buffers, filled by TMA bulk copies and tracked by mbarriers. The ring runs
// ahead across unit boundaries, so a warp's next unit is already in flight while the CTA
// reduces the current one. Partial sums go to shared memory; after a CTA barrier the unit is
// reduced in a fixed order (range ascending) and finished: SwiGLU into the down kernel's
// fragments, or the router-weighted combine in router order plus the residual.

struct rows_args {
    const uint8_t *bank;      // packed gate-up (2 tiles per k-tile) or down bank
    size_t bank_stride;       // bytes per expert
    int mats;                 // 2 for gate-up, 1 for down
    int ntr, nkt;             // tile-rows, k-tiles (64 columns) per row
    int ranges, tpr;          // K runs per item row, most k-tiles in one run
    int tile_bytes;
    int stages, stage_bytes;  // per-warp ring
    int n_units_hint;         // units the grid was sized for
    const uint32_t *bsrc;     // B fragments, indexed by token (gate-up) or column (down)
    int b_by_column;
    int nblk_b;
    tab_view tab;             // in global memory; copied to shared memory at start
    // gate-up epilogue
    int act;
    float alpha, limit;
    uint32_t *actfrag;        // [col][I/32][2][4][4]
    float *act_out;           // [col][I] f32
    int I;
    // down epilogue
    const float *wts;         // [T][K]
    const float *residual;    // [T][H] or null
    float *out;               // [T][H]
    int T, K, H;
    // per-expert biases (moe.rs:2310-2331, 2362-2372) or null: gate rows of expert e at e, up
    // rows at E + e ([2E][I]); down [E][H]
    const float *bias_gu, *bias_dn;
    int E;
    int *status;
};

__device__ __forceinline__ int range_lo(int r, int nkt, int ranges) { return (int)(((long)r * nkt) / ranges); }

struct item_pos {
    int u, i;
};

template <int WT>
__global__ void __launch_bounds__(256) k_moe_rows(rows_args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[8][4];
    const int trace_row = (int)blockIdx.x + (a.mats == 2 ? 1024 : 2048);
    (void)trace_row;
    TRACE(0);
    const int nwarps = blockDim.x >> 5;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool down = a.mats == 1;

    // gate-up consumes the routing tables of the kernel before it: wait, then release the
    // down kernel, which may then read the same tables before its own wait.
    if (!down) {
        pdl_wait();
        pdl_trigger();
    }
    // routing tables into shared memory
    const int n_tab = (int)tab_view::ints(a.tab.G, a.tab.S, a.tab.C, a.tab.TK);
    int *tabs = reinterpret_cast<int *>(smem);
    for (int i = threadIdx.x; i < n_tab; i += blockDim.x) tabs[i] = __ldcg(a.tab.base + i);
    __syncthreads();
    tab_view tb = a.tab;
    tb.base = tabs;
    const int G = *tb.n_groups(), ncol = *tb.n_cols();
    const size_t tab_bytes = ((size_t)n_tab * 4 + 127) / 128 * 128;
    float *part = reinterpret_cast<float *>(smem + tab_bytes);
    const size_t part_floats = down ? (size_t)a.tab.G * a.ranges * 16 * GROUP : (size_t)a.ranges * 2 * 16 * GROUP;
    float *osum = part + part_floats;  // down: [col][16]
    const size_t part_bytes = ((part_floats + (down ? (size_t)a.tab.C * 16 : 0)) * 4 + 127) / 128 * 128;
    uint8_t *ring = smem + tab_bytes + part_bytes + (size_t)warp * a.stages * a.stage_bytes;

    const int n_units = down ? a.ntr : G * a.ntr;
    const int items_per_unit = down ? G * a.ranges : a.ranges;
    if (lane == 0) {
        for (int s = 0; s < a.stages; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    auto valid = [&](const item_pos &p) { return p.u < n_units; };
    auto advance = [&](item_pos &p) {
        p.i += nwarps;
        while (p.u < n_units && p.i >= items_per_unit) {
            p.u += gridDim.x;
            p.i = warp;
        }
    };
    auto first = [&]() {
        item_pos p{(int)blockIdx.x, warp};
        if (p.i >= items_per_unit) p.u = n_units;  // this warp has no item in any unit
        return p;
    };
    // (unit, item) -> group, tile-row, K run
    auto decode = [&](const item_pos &p, int &g, int &tr, int &rg) {
        if (down) {
            tr = p.u;
            g = p.i / a.ranges;
            rg = p.i % a.ranges;
        } else {
            g = p.u / a.ntr;
            tr = p.u % a.ntr;
            rg = p.i;
        }
    };
    auto issue = [&](const item_pos &p, int stage, bool weights, bool acts) {
        if (lane != 0) return;
        int g, tr, rg;
        decode(p, g, tr, rg);
        const int slot = tb.grp_slot()[g];
        const int expert = tb.slot_expert()[slot];
        const int col0 = tb.grp_col0()[g], ntok = tb.grp_ntok()[g];
        const int k0 = range_lo(rg, a.nkt, a.ranges), kn = range_lo(rg + 1, a.nkt, a.ranges) - k0;
        const unsigned wbytes = (unsigned)(kn * a.mats * a.tile_bytes);
        const unsigned bbytes = (unsigned)(2 * kn * 128);
        uint8_t *st = ring + (size_t)stage * a.stage_bytes;
        uint64_t *bar = &bars[warp][stage];
        if (weights) {
            fence_proxy_async();
            mbar_expect_tx(bar, wbytes + bbytes * ntok);
            bulk_g2s(st, a.bank + (size_t)expert * a.bank_stride + ((size_t)tr * a.nkt + k0) * a.mats * a.tile_bytes,
                     wbytes, bar);
        }
        if (acts) {
            uint8_t *bs = st + (size_t)a.tpr * a.mats * a.tile_bytes;
            for (int t = 0; t < ntok; ++t) {
                const int col = col0 + t;
                const int row = a.b_by_column ? col : tb.col_tok()[col];
                bulk_g2s(bs + (size_t)t * a.tpr * 2 * 128, a.bsrc + ((size_t)row * a.nblk_b + 2 * k0) * 32, bbytes, bar);
            }
        }
    };

    // prologue: the first `stages` items of this warp (down: weights now, fragments after the wait)
    item_pos iss = first();
    const item_pos start = iss;
    int issued = 0, n_issued = 0;
    for (int s = 0; s < a.stages && valid(iss); ++s) {
        issue(iss, s, true, !down);
        advance(iss);
        ++issued;
        ++n_issued;
    }
    TRACE(1);
    if (down) {
        pdl_trigger();
        pdl_wait();
        TRACE(2);
        item_pos p = start;
        for (int s = 0; s < issued; ++s) {
            issue(p, s, false, true);
            advance(p);
        }
    }

    // Item j of this warp's sequence lives in stage j % stages and completes that stage's
    // barrier phase number j / stages, parity (j / stages) & 1.
    int k = 0;        // items this warp has consumed
    int kf = -1;      // the first item whose wait gave up (-1: none)
    bool failed = false;
    const int r = lane >> 2, q = lane & 3;
    int un = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++un) {
        if (un < 5) TRACE(4 + 2 * un);
        for (int i = warp; i < items_per_unit; i += nwarps) {
            const int stage = k % a.stages;
            if (k < 8) TRACE(14 + 2 * k);
            if (!failed && !mbar_wait(&bars[warp][stage], (unsigned)(k / a.stages) & 1u, a.status)) {
                failed = true;
                kf = k;
            }
            if (k < 8) TRACE(15 + 2 * k);
            ++k;
            int g, tr, rg;
            decode(item_pos{u, i}, g, tr, rg);
            const int ntok = tb.grp_ntok()[g];
            const int kn = range_lo(rg + 1, a.nkt, a.ranges) - range_lo(rg, a.nkt, a.ranges);
            const uint8_t *st = ring + (size_t)stage * a.stage_bytes;
            const uint32_t *bsm = reinterpret_cast<const uint32_t *>(st + (size_t)a.tpr * a.mats * a.tile_bytes);
            float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
            if (!failed) {
                for (int kt = 0; kt < kn; ++kt) {
                    uint32_t bfr[2][2][2];
                    load_b(bsm, 2 * a.tpr, kt, lane, ntok, bfr);
                    const uint8_t *tile = st + (size_t)kt * a.mats * a.tile_bytes;
                    tile_mma<WT>(tile, lane, bfr, acc0);
                    if (a.mats == 2) tile_mma<WT>(tile + a.tile_bytes, lane, bfr, acc1);
                }
            }
            __syncwarp();
            if (valid(iss) && !failed) {
                issue(iss, stage, true, true);
                advance(iss);
                ++n_issued;
            }
            // lane (r, q) holds column pair (2q, 2q+1) = (f16 part, residual part) of group
            // member q for rows r and r+8
            if (q < ntok) {
                if (down) {
                    float *p = part + (size_t)i * 16 * GROUP;
                    p[r * GROUP + q] = acc0[0] + acc0[1];
                    p[(r + 8) * GROUP + q] = acc0[2] + acc0[3];
                } else {
                    float *pg = part + ((size_t)rg * 2 + 0) * 16 * GROUP;
                    float *pu = part + ((size_t)rg * 2 + 1) * 16 * GROUP;
                    pg[r * GROUP + q] = acc0[0] + acc0[1];
                    pg[(r + 8) * GROUP + q] = acc0[2] + acc0[3];
                    pu[r * GROUP + q] = acc1[0] + acc1[1];
                    pu[(r + 8) * GROUP + q] = acc1[2] + acc1[3];
                }
            }
        }
        __syncthreads();
        if (un < 5) TRACE(5 + 2 * un);
        if (!down) {
            // gate-up unit: sum the K runs in order, apply the activation, write the f32
            // activation and the down kernel's B fragments (f16 rounding + residual halves)
            const int g = u / a.ntr, tr = u % a.ntr;
            const int ntok = tb.grp_ntok()[g], col0 = tb.grp_col0()[g];
            const int nblk_i = a.I / 32;
            for (int e = threadIdx.x; e < ntok * 16; e += blockDim.x) {
                const int t = e / 16, rr = e % 16;
                float gs = 0.f, us = 0.f;
                for (int rg = 0; rg < a.ranges; ++rg) {
                    gs += part[((size_t)rg * 2 + 0) * 16 * GROUP + rr * GROUP + t];
                    us += part[((size_t)rg * 2 + 1) * 16 * GROUP + rr * GROUP + t];
                }
                const int col = col0 + t, row = tr * 16 + rr;
                if (a.bias_gu) {
                    // ggml_add_id right after each expert matvec, before the activation
                    const int ex = tb.slot_expert()[tb.grp_slot()[g]];
                    gs += a.bias_gu[(size_t)ex * a.I + row];
                    us += a.bias_gu[(size_t)(a.E + ex) * a.I + row];
                }
                const float v = act_fn(a.act, gs, us, a.alpha, a.limit);
                a.act_out[(size_t)col * a.I + row] = v;
                const __half hh = __float2half_rn(v);
                const __half hl = __float2half_rn(v - __half2float(hh));
                // element el of block blk sits in pair j = el & 3 of lane q = (el & 15) >> 2, in
                // the low half for el < 16 and the high half for el >= 16
                const int blk = row / 32, el = row % 32;
                const int qq = (el & 15) >> 2, jj = el & 3, half = el >> 4;
                const size_t ihi = ((((size_t)col * nblk_i + blk) * 2 + 0) * 4 + qq) * 4 + jj;
                const size_t ilo = ((((size_t)col * nblk_i + blk) * 2 + 1) * 4 + qq) * 4 + jj;
                reinterpret_cast<uint16_t *>(a.actfrag + ihi)[half] = __half_as_ushort(hh);
                reinterpret_cast<uint16_t *>(a.actfrag + ilo)[half] = __half_as_ushort(hl);
            }
        } else {
            // down unit: each column's output = its K runs in order; then per token the
            // router-weighted sum over its k experts in router order, plus the residual
            const int tr = u;
            for (int e = threadIdx.x; e < G * 16 * GROUP; e += blockDim.x) {
                const int g = e / (16 * GROUP), rr = (e / GROUP) % 16, t = e % GROUP;
                if (t >= tb.grp_ntok()[g]) continue;
                float o = 0.f;
                for (int rg = 0; rg < a.ranges; ++rg) o += part[((size_t)g * a.ranges + rg) * 16 * GROUP + rr * GROUP + t];
                // the down bias inside the router weighting: added to each expert's output
                if (a.bias_dn) o += a.bias_dn[(size_t)tb.slot_expert()[tb.grp_slot()[g]] * a.H + tr * 16 + rr];
                osum[(size_t)(tb.grp_col0()[g] + t) * 16 + rr] = o;
            }
            __syncthreads();
            for (int e = threadIdx.x; e < a.T * 16; e += blockDim.x) {
                const int t = e / 16, rr = e % 16;
                float acc = 0.f;
                for (int m = 0; m < a.K; ++m)
                    acc = fmaf(a.wts[t * a.K + m], osum[(size_t)tb.col_of()[t * a.K + m] * 16 + rr], acc);
                const size_t o = (size_t)t * a.H + tr * 16 + rr;
                a.out[o] = a.residual ? a.residual[o] + acc : acc;
            }
            (void)ncol;
        }
        __syncthreads();
    }
    // no bulk copy may still be landing in this warp's ring when the CTA exits: wait (bounded)
    // for any that were issued and not consumed (only after a failed wait)
    if (failed)
        for (int j = kf; j < n_issued; ++j) mbar_wait(&bars[warp][j % a.stages], (unsigned)(j / a.stages) & 1u, a.status);
    TRACE(31);
}

// ---- the decode path: T x K <= 32 columns --------------------------------------------------
//
// Three kernels per layer, each one CTA per SM at most, each sized to share an SM with its
// neighbours so a kernel's CTAs become resident (and start their weight copies) while the
// kernel before it still runs:
//   x_route   router logits (+ bias) and the activation's B fragments; the router rows are
//             bulk-copied to shared memory before the wait, so after it only the activation
//             is read
//   x_expert  gate-up (mode 0) or down (mode 1). Every CTA derives the top-k and the slot
//             tables itself from the logits (warp-parallel, in shared memory) instead of one
//             CTA building them for all. The work is one flattened sequence — gate-up
//             (group, tile-row, k-tile) pairs of gate and up tiles, down (tile-row, group,
//             k-tile) tiles — cut into equal contiguous ranges, one per warp, streamed through
//             a per-warp ring of bulk copies (down issues its first stages before the wait).
//             A warp writes one partial per segment (nkt consecutive elements: one k-extent)
//             it touches, then fences once and arrives on the segment's counter (gate-up) or
//             the tile-row's (down); the last warp to arrive finishes: the activation into the
//             down kernel's fragments, or the router-weighted combine plus the residual.

constexpr int XW = 16;         // most warps per expert CTA (the plan takes 8 when 16 rings do not fit)
constexpr int XSTAGES = 3;     // ring stages per warp
constexpr int MAX_TK = 32;     // columns (token, expert choices) of the decode path
constexpr int XREC_GU = 2 * 16 * GROUP;  // floats in one gate-up partial (gate, up x 16 rows x 4 cols)
constexpr int XREC_DN = 16 * GROUP;      // floats in one down partial
constexpr int XREC_XDN = 4 * 8 * GROUP;  // the expert kernel's down partial: 4 accumulators a lane
constexpr int XROUTE_WARPS = 4;
constexpr int XMAX_PIECES = 24;          // pieces per segment (k-extent / piece length)
constexpr int XMAX_K = 8;                // experts per token the decode path's combine unrolls
constexpr int XEXCLUSIVE_SMEM = 116 * 1024;  // > half of the 228 KB an SM has: one CTA per SM

struct xroute_args {
    const float *x;       // [T][H]
    const float *norm_w;  // [H] or null
    float eps;
    const float *router;  // [E][H]
    const float *rbias;   // [E] or null
    int T, H, E;
    float *logits;        // [T][E]
    uint32_t *xfrag;      // [T][H/32][2][4][4]
    float *x_out;         // [T][H]: the routed activation (normalised), for the host's experts; or null
    int *status;
    uint8_t *xdig;        // one token: its E2M1 digits for the tc path (xtc.cuh) in place of xfrag; or null
};

// One router row per warp, staged in shared memory by a bulk copy issued before the wait; the
// activation row is read once per CTA after it. The dot product keeps the fixed order of
// moearc_matvec_f32 (lane l folds float4 columns l, l + 32, ... in order, then a butterfly).
__global__ void __launch_bounds__(XROUTE_WARPS * 32) k_xroute(xroute_args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bar[XROUTE_WARPS];
    __shared__ float red[XROUTE_WARPS];
    const int trace_row = (int)blockIdx.x;
    (void)trace_row;
    TRACE(0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = a.H, n4 = H / 4;
    float *wrow = reinterpret_cast<float *>(smem) + (size_t)warp * H;
    float *xs = reinterpret_cast<float *>(smem) + (size_t)XROUTE_WARPS * H;
    float *nws = xs + H;  // the norm weights, static: staged before the wait
    const int e0 = blockIdx.x * XROUTE_WARPS + warp;
    const int nw = gridDim.x * XROUTE_WARPS;
    if (lane == 0) {
        mbar_init(&bar[warp], 1);
        fence_mbar_init();
        if (e0 < a.E) {
            mbar_expect_tx(&bar[warp], (unsigned)(H * 4));
            bulk_g2s(wrow, a.router + (size_t)e0 * H, (unsigned)(H * 4), &bar[warp]);
        }
    }
    if (a.norm_w)
        for (int c = threadIdx.x; c < n4; c += XROUTE_WARPS * 32)
            reinterpret_cast<float4 *>(nws)[c] = __ldg(reinterpret_cast<const float4 *>(a.norm_w) + c);
    __syncwarp();
    pdl_trigger();
    pdl_wait();
    TRACE(1);
    bool have_row = true;
    for (int t = 0; t < a.T; ++t) {
        // the token's activation (normalised when routing rmsnorm(x) * norm_w)
        const float4 *xr = reinterpret_cast<const float4 *>(a.x + (size_t)t * H);
        float ss = 0.f;
        for (int c = threadIdx.x; c < n4; c += XROUTE_WARPS * 32) {
            const float4 v = __ldcg(xr + c);
            reinterpret_cast<float4 *>(xs)[c] = v;
            ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
        }
        if (a.norm_w) {
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            float tot = 0.f;
            for (int w = 0; w < XROUTE_WARPS; ++w) tot += red[w];
            const float s = 1.0f / sqrtf(tot / (float)H + a.eps);
            for (int c = threadIdx.x; c < n4; c += XROUTE_WARPS * 32) {
                float4 v = reinterpret_cast<float4 *>(xs)[c];
                const float4 n = reinterpret_cast<const float4 *>(nws)[c];
                v = make_float4((v.x * s) * n.x, (v.y * s) * n.y, (v.z * s) * n.z, (v.w * s) * n.w);
                reinterpret_cast<float4 *>(xs)[c] = v;
            }
        }
        __syncthreads();
        TRACE(3);
        if (a.x_out && blockIdx.x == 0)
            for (int c = threadIdx.x; c < n4; c += XROUTE_WARPS * 32)
                reinterpret_cast<float4 *>(a.x_out + (size_t)t * H)[c] = reinterpret_cast<const float4 *>(xs)[c];
        for (int e = e0; e < a.E; e += nw) {
            const float *w = wrow;
            if (e != e0) {
                // more experts than warps: the row comes straight from global memory
                w = a.router + (size_t)e * H;
            } else if (t == 0) {
                have_row = mbar_wait(&bar[warp], 0, a.status);
            }
            if (!have_row && e == e0) continue;
            float acc = 0.f;
            for (int c = lane; c < n4; c += 32) {
                const float4 wv = (e == e0) ? reinterpret_cast<const float4 *>(w)[c] : __ldg(reinterpret_cast<const float4 *>(w) + c);
                const float4 xv = reinterpret_cast<const float4 *>(xs)[c];
                acc = fmaf(wv.x, xv.x, acc);
                acc = fmaf(wv.y, xv.y, acc);
                acc = fmaf(wv.z, xv.z, acc);
                acc = fmaf(wv.w, xv.w, acc);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (lane == 0) a.logits[(size_t)t * a.E + e] = a.rbias ? acc + a.rbias[e] : acc;
        }
        TRACE(4);
        const int nblk = H / 32;
        if (a.xdig) {
            // the tc path: each 32-element block's digits, one warp a block
            for (int b = blockIdx.x * XROUTE_WARPS + warp; b < nblk; b += gridDim.x * XROUTE_WARPS)
                tc_write_digits(xs[32 * b + lane], lane, a.xdig, b);
            __syncthreads();
            continue;
        }
        // B fragments of this token: [block][part][q][j] = pair (x[32b+4q+j], x[32b+4q+16+j])
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nblk * 16; i += gridDim.x * blockDim.x) {
            const int j = i & 3, q = (i >> 2) & 3, b = i >> 4;
            uint32_t hi, lo;
            split_f16x2(xs[32 * b + 4 * q + j], xs[32 * b + 4 * q + 16 + j], hi, lo);
            a.xfrag[((((size_t)t * nblk + b) * 2 + 0) * 4 + q) * 4 + j] = hi;
            a.xfrag[((((size_t)t * nblk + b) * 2 + 1) * 4 + q) * 4 + j] = lo;
        }
        __syncthreads();
    }
    // a row copy that was issued and never waited for (no tokens) must land before exit
    if (a.T == 0 && lane == 0 && e0 < a.E) mbar_wait(&bar[warp], 0, a.status);
    TRACE(2);
}

// Routing tables of the decode path, in shared memory.
struct xtab {
    int G, C;                         // groups, columns (T * K less the choices the host takes)
    int n_slots;                      // distinct experts, ascending
    int grp_slot[MAX_TK], slot_expert[MAX_TK];
    int grp_expert[MAX_TK], grp_col0[MAX_TK], grp_ntok[MAX_TK];
    int col_tok[MAX_TK], col_grp[MAX_TK];
    int col_of[MAX_TK];               // column of choice i = t * K + m
    float wts[MAX_TK];                // gating weight of choice i
    unsigned idx[MAX_TK];             // expert of choice i
    int key[32];                      // sort keys of the rank step (expert * 64 + token)
};


// Every token's top-k (warp t of nw takes tokens t, t + nw, ...), then the tables by warp 0: the
// columns are the choices sorted by (expert, token) — distinct experts ascending, a slot's
// tokens in token order — cut into groups of at most GROUP columns of one expert. Choices whose
// bit is set in `hmask` (bit t * K + m) are computed on the host: they get no column
// (col_of = -1) and their experts no slot unless another choice keeps them.
// Not inlined: the gate-up kernel runs it twice (a dry run before its wait, then the real one)
// and the second call finds the code in the instruction cache.
__device__ __noinline__ void xbuild(xtab &tb, const float *logits, int T, int E, int K, int gating, int warp, int lane,
                                   unsigned hmask = 0u) {
    const int nw = (int)(blockDim.x >> 5);
    for (int t = warp; t < T; t += nw) xtopk(logits + (size_t)t * E, E, K, gating, lane, tb.idx + t * K, tb.wts + t * K);
    __syncthreads();
    if (warp == 0) {
        const bool chosen = lane < T * K && !((hmask >> lane) & 1u);
        const int C = __popc(__ballot_sync(0xffffffffu, chosen));
        const int key = chosen ? (int)tb.idx[lane] * 64 + lane / K : 0x7FFFFFFF;
        // rank = number of smaller keys; the keys go through shared memory, which the unrolled
        // compares read as broadcasts (a loop of 32 shuffles took several times as long)
        tb.key[lane] = key;
        __syncwarp();
        int rank = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) rank += (tb.key[j] < key);
        if (chosen) {
            tb.col_of[lane] = rank;
            tb.col_tok[rank] = lane / K;
            tb.grp_expert[rank] = (int)tb.idx[lane];  // expert of column `rank`, for now
        } else if (lane < T * K) {
            tb.col_of[lane] = -1;
        }
        __syncwarp();
        const bool live = lane < C;  // from here on a lane is a column
        const int ex = live ? tb.grp_expert[lane] : -1;
        const int prev = __shfl_up_sync(0xffffffffu, ex, 1);
        const bool start = live && (lane == 0 || prev != ex);
        const unsigned starts = __ballot_sync(0xffffffffu, start);
        const unsigned le = (lane == 31) ? 0xffffffffu : ((2u << lane) - 1u);
        const int first = live ? 31 - __clz(starts & le) : 0;  // first column of this expert
        const bool gstart = live && ((lane - first) % GROUP == 0);
        const unsigned gs = __ballot_sync(0xffffffffu, gstart);
        const int g = __popc(gs & le) - 1;
        __syncwarp();
        if (live) tb.col_grp[lane] = g;
        if (gstart) {
            const unsigned after = gs & ~le;
            const int nxt = after ? __ffs(after) - 1 : C;
            // a group ends at the next group start or at the expert's end, whichever is first
            const unsigned next_exp = starts & ~le;
            const int exp_end = next_exp ? __ffs(next_exp) - 1 : C;
            tb.grp_expert[g] = ex;
            tb.grp_col0[g] = lane;
            tb.grp_ntok[g] = min(nxt, exp_end) - lane;
        }
        if (lane == 0) {
            tb.G = __popc(gs);
            tb.C = C;
        }
        __syncwarp();
        // slots: the distinct experts in ascending order (groups of one expert are adjacent)
        const int G = __popc(gs);
        const int ge = lane < G ? tb.grp_expert[lane] : -1;
        const int gprev = __shfl_up_sync(0xffffffffu, ge, 1);
        const bool new_slot = lane < G && (lane == 0 || gprev != ge);
        const unsigned ns = __ballot_sync(0xffffffffu, new_slot);
        if (lane < G) tb.grp_slot[lane] = __popc(ns & le) - 1;
        if (new_slot) tb.slot_expert[__popc(ns & le) - 1] = ge;
        if (lane == 0) tb.n_slots = __popc(ns);
    }
    __syncthreads();
}

struct xexp_args {
    const uint8_t *bank;      // packed gate-up (pairs) or down (tiles)
    size_t bank_stride;       // bytes per expert
    int ntr, nkt;             // tile-rows and k-tiles per row of one expert matrix
    int tile_bytes, elem_bytes;
    int ch, stage_bytes, ntok_max;
    int nblk_b;               // B fragment blocks per row (H/32 gate-up, I/32 down)
    const uint32_t *bsrc;     // xfrag (gate-up, by token) or actfrag (down, by column)
    const float *logits;
    int T, E, K, gating;
    // gate-up epilogue
    int act;
    float alpha, limit;
    uint32_t *actfrag;
    float *act_out;
    int I;
    unsigned *idx_out;
    float *wts_out;
    // down epilogue
    const float *residual;
    float *out;
    int H;
    float *part;              // piece partials, PART_EMPTY where none is pending
    xtab *tab_pub;            // gate-up: CTA 0 publishes its tables here; down: read them (or null)
    const int *slot_of;       // residency cache: expert -> slot of the bank (or null)
    int by_slot;              // bank holds one expert per slot (staged offload), not all experts
    const unsigned *hmask;    // choices the host computes (bit t * K + m), or null
    unsigned long long poll_ns;  // the wait for other warps' partials (XPOLL_NS in use)
    int phantom;                 // 1: every such wait runs out (testing)
    // per-expert biases or null: gate rows of expert e at e, up rows at E + e ([2E][I]); down
    // [E][H] (moe.rs:2310-2331, 2362-2372)
    const float *bias_gu, *bias_dn;
    // per CTA [start, dependency wait over, end] in ns of %globaltimer (the end the last warp's),
    // rewritten every launch, or null
    unsigned long long *span;
    int *status;
};

__device__ __forceinline__ int xcta(long P, long NW, long p) { return (int)(((p + 1) * NW - 1) / P); }

// The np piece partials of one (record run, float4): pieces seg * np .. + np - 1, rec floats
// apart, the float4 at offset off of each; read as soon as every one has been stored and summed
// in piece order from 0, per component (sum[0..3]) or, PAIR, per pair (sum[0] = x + y, sum[1] =
// z + w). False (and STATUS_WAIT_TIMEOUT) when a piece does not arrive within poll_ns
// (`phantom`: as if one never did — a test of this path).
template <bool PAIR>
__device__ bool take_quads(const float *part, int rec, int np, int seg, int off, float (&sum)[4], int *status,
                           unsigned long long poll_ns, int phantom, int *rounds = nullptr) {
    uint4 v[XMAX_PIECES];
    unsigned long long t0 = 0;
    for (;;) {
        if (rounds) ++*rounds;
        // every load issued before any is looked at; the check has no branch per value
#pragma unroll
        for (int j = 0; j < XMAX_PIECES; ++j)
            v[j] = j < np ? ld_part4(part + ((size_t)seg * np + j) * rec + off) : make_uint4(0u, 0u, 0u, 0u);
        uint32_t empty = 0;
#pragma unroll
        for (int j = 0; j < XMAX_PIECES; ++j)
            empty |= (uint32_t)(v[j].x == PART_EMPTY) | (uint32_t)(v[j].y == PART_EMPTY) |
                     (uint32_t)(v[j].z == PART_EMPTY) | (uint32_t)(v[j].w == PART_EMPTY);
        if (!empty && !phantom) break;
        const unsigned long long t = xnow();
        if (t0 == 0) {
            t0 = t;
        } else if (t - t0 > poll_ns) {
            atomicOr(status, STATUS_WAIT_TIMEOUT);
            return false;
        }
    }
    sum[0] = sum[1] = sum[2] = sum[3] = 0.f;
#pragma unroll
    for (int j = 0; j < XMAX_PIECES; ++j)
        if (j < np) {
            const float x = __uint_as_float(v[j].x), y = __uint_as_float(v[j].y);
            const float z = __uint_as_float(v[j].z), w = __uint_as_float(v[j].w);
            if (PAIR) {
                sum[0] += x + y;
                sum[1] += z + w;
            } else {
                sum[0] += x;
                sum[1] += y;
                sum[2] += z;
                sum[3] += w;
            }
        }
    return true;
}

template <int WT, int MODE>
__global__ void __launch_bounds__(XW * 32, 1) k_xexpert(xexp_args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[XW][XSTAGES];
    __shared__ xtab tb;
    const int trace_row = (int)blockIdx.x + (MODE == 0 ? 1024 : 2048);
    (void)trace_row;
    TRACE(0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int MATS = MODE == 0 ? 2 : 1;
    unsigned long long *span = a.span ? a.span + (size_t)blockIdx.x * 3 : nullptr;
    if (span && threadIdx.x == 0) {
        span[0] = xnow();
        span[2] = 0;  // before the CTA's first barrier; the warps' ends are taken after it
    }
    // the CTA's end: the latest of its warps' returns
#define XSPAN_END()                                          \
    do {                                                     \
        if (span && lane == 0) atomicMax(span + 2, xnow()); \
    } while (0)
    if (MODE == 0) {
        // Before the wait, a dry run of the table build on whatever the logits hold now (the
        // router kernel is still writing them; these tables are discarded): it brings the
        // code into the instruction cache while the router runs.
        xbuild(tb, a.logits, a.T, a.E, a.K, a.gating, warp, lane);
        TRACE(13);
        // the logits are the previous kernel's output
        pdl_wait();
        if (span && threadIdx.x == 0) span[1] = xnow();
        TRACE(12);
        // CTA 0 releases the down kernel only once it has published the tables (below)
        if (blockIdx.x != 0 || !a.tab_pub) pdl_trigger();
    }
    // final before this kernel's wait (gate-up) or before it was launched (down)
    const unsigned hm = a.hmask ? __ldcg(a.hmask) : 0u;
    if (MODE == 1 && a.tab_pub) {
        // the gate-up kernel's published tables: final before this kernel was launched
        const uint32_t *src = reinterpret_cast<const uint32_t *>(a.tab_pub);
        uint32_t *dst = reinterpret_cast<uint32_t *>(&tb);
        for (int i = threadIdx.x; i < (int)(sizeof(xtab) / 4); i += blockDim.x) dst[i] = __ldcg(src + i);
        __syncthreads();
    } else {
        xbuild(tb, a.logits, a.T, a.E, a.K, a.gating, warp, lane, hm);
    }
    TRACE(1);
    if (MODE == 0 && blockIdx.x == 0 && a.tab_pub) {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(&tb);
        uint32_t *dst = reinterpret_cast<uint32_t *>(a.tab_pub);
        for (int i = threadIdx.x; i < (int)(sizeof(xtab) / 4); i += blockDim.x) dst[i] = src[i];
        __threadfence();
        __syncthreads();
        pdl_trigger();
    }
    if (MODE == 0 && blockIdx.x == 0)
        for (int i = threadIdx.x; i < a.T * a.K; i += blockDim.x) {
            a.idx_out[i] = tb.idx[i];
            a.wts_out[i] = tb.wts[i];
        }

    // Work: segments (gate-up: group * ntr + tile-row; down: tile-row * G + group), each one
    // k-extent of nkt elements cut into np pieces of a.ch elements at fixed places. A warp
    // takes a contiguous run of pieces; every piece leaves its own partial, so the sums do not
    // depend on how pieces fall to warps (the batch, the grid).
    const int G = tb.G, nkt = a.nkt, ntr = a.ntr, ch = a.ch;
    const int np = (nkt + ch - 1) / ch;
    const long Q = (long)G * ntr * np;
    const int nw = (int)(blockDim.x >> 5);
    const long NW = (long)gridDim.x * nw, gw = (long)blockIdx.x * nw + warp;
    const long qa = Q * gw / NW, qb = Q * (gw + 1) / NW;
    uint8_t *ring = smem + (size_t)warp * XSTAGES * a.stage_bytes;
    const int wmax = ch * a.elem_bytes;  // B region offset inside a stage
    if (lane == 0) {
        for (int s = 0; s < XSTAGES; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    auto piece_len = [&](int j) { return min(ch, nkt - j * ch); };
    // piece cursor: piece q is index j of segment (group g, tile-row tr); it advances without
    // division (the issuing lane runs it once per piece while the warp's other lanes wait)
    struct cur {
        long q;
        int j, g, tr;
    };
    auto at = [&](long q) {
        cur c;
        c.q = q;
        const long seg = q / np;
        c.j = (int)(q - seg * np);
        if (MODE == 0) {
            c.g = (int)(seg / ntr);
            c.tr = (int)(seg - (long)c.g * ntr);
        } else {
            c.tr = (int)(seg / G);
            c.g = (int)(seg - (long)c.tr * G);
        }
        return c;
    };
    auto step = [&](cur &c) {
        ++c.q;
        if (++c.j == np) {
            c.j = 0;
            if (MODE == 0) {
                if (++c.tr == ntr) {
                    c.tr = 0;
                    ++c.g;
                }
            } else if (++c.g == G) {
                c.g = 0;
                ++c.tr;
            }
        }
    };
    auto issue = [&](const cur &c, int stage, bool weights, bool acts) {
        const int n = piece_len(c.j), kt = c.j * ch;
        const int ntok = tb.grp_ntok[c.g];
        uint8_t *st = ring + (size_t)stage * a.stage_bytes;
        uint64_t *bar = &bars[warp][stage];
        if (weights) {
            fence_proxy_async();
            mbar_expect_tx(bar, (unsigned)(n * a.elem_bytes + ntok * n * 256));
            const int bank_ix = a.by_slot ? tb.grp_slot[c.g] : tb.grp_expert[c.g];
            bulk_g2s_hint(st, a.bank + (size_t)bank_ix * a.bank_stride + (size_t)((c.tr * nkt + kt) * a.elem_bytes),
                          (unsigned)(n * a.elem_bytes), bar, policy_evict_first());
        }
        if (acts)
            for (int t = 0; t < ntok; ++t) {
                const int col = tb.grp_col0[c.g] + t;
                const int row = MODE == 0 ? tb.col_tok[col] : col;
                bulk_g2s(st + wmax + t * ch * 256, a.bsrc + (size_t)((row * a.nblk_b + 2 * kt) * 32), (unsigned)(n * 256), bar);
            }
    };
    const cur start = at(qa);
    cur ic = start;
    long n_issued = 0;  // lane 0's count
    if (MODE == 1 && a.by_slot) {
        // staged down banks are the previous kernel's output: nothing streams before the wait
        pdl_trigger();
        pdl_wait();
        if (span && threadIdx.x == 0) span[1] = xnow();
    }
    if (MODE == 1 && a.by_slot && G == 0) {
        // the host took every choice: the device's share is zero
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.T * a.H; i += gridDim.x * blockDim.x)
            a.out[i] = a.residual ? a.residual[i] : 0.f;
        XSPAN_END();
        return;
    }
    if (a.slot_of) {
        // cached offload: the block's residency table (final before either kernel's wait
        // returned) names each expert's slot
        // (an unplaced expert, possible only after a reported planning error, reads slot 0)
        if ((int)threadIdx.x < tb.G) tb.grp_slot[threadIdx.x] = max(0, __ldcg(a.slot_of + tb.grp_expert[threadIdx.x]));
        __syncthreads();
    }
    if (lane == 0)
        for (int s = 0; s < XSTAGES && ic.q < qb; ++s) {
            issue(ic, s, true, MODE == 0);
            step(ic);
            ++n_issued;
        }

    if (MODE == 1) {
        // the weights are static and stream now; the activation fragments are the gate-up
        // kernel's output and follow the wait
        pdl_trigger();
        pdl_wait();
        if (span && threadIdx.x == 0 && !a.by_slot) span[1] = xnow();
        TRACE(2);
        if (lane == 0) {
            cur c = start;
            for (long s = 0; s < n_issued; ++s) {
                issue(c, (int)s, false, true);
                step(c);
            }
        }
    }
    // consume: lane (r = lane / 4, q = lane % 4) holds rows r, r + 8 of column q; B column
    // n = lane / 4 is token n / 2, part n % 2
    const int r = lane >> 2, qd = lane & 3;
    const int rec = MODE == 0 ? XREC_GU : XREC_XDN;
    cur cc = start;
    long k = 0, kf = -1;
    while (cc.q < qb) {
        const int stage = (int)(k % XSTAGES);
        if (!mbar_wait(&bars[warp][stage], (unsigned)((k / XSTAGES) & 1), a.status)) {
            kf = k;
            break;
        }
        if (k < 6) TRACE(3 + k);
        const int n = piece_len(cc.j);
        const int ntok = tb.grp_ntok[cc.g];
        const uint8_t *st = ring + (size_t)stage * a.stage_bytes;
        const uint32_t *bsm = reinterpret_cast<const uint32_t *>(st + wmax);
        float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
        for (int i = 0; i < n; ++i) {
            uint32_t bfr[2][2][2];
            load_b(bsm, 2 * ch, i, lane, ntok, bfr);
            const uint8_t *tile = st + i * a.elem_bytes;
            tile_mma<WT>(tile, lane, bfr, acc0);
            if (MATS == 2) tile_mma<WT>(tile + a.tile_bytes, lane, bfr, acc1);
        }
        __syncwarp();
        ++k;
        if (lane == 0 && ic.q < qb) {
            issue(ic, stage, true, true);
            step(ic);
            ++n_issued;
        }
        // the piece's partial of column q and rows r, r + 8, laid [column][r][4] so the columns
        // in use fill whole 128-byte lines: gate-up stores the sums (f16 part + residual part)
        // of gate r, gate r + 8, up r, up r + 8; down stores its four accumulators (row r is
        // [0] + [1], row r + 8 is [2] + [3], added by the reader)
        float *pr = a.part + (size_t)cc.q * rec;  // piece q = segment * np + j
        if (qd < ntok) {
            if (MATS == 2)
                st_part4(pr + (qd * 8 + r) * 4, acc0[0] + acc0[1], acc0[2] + acc0[3], acc1[0] + acc1[1],
                         acc1[2] + acc1[3]);
            else
                st_part4(pr + (qd * 8 + r) * 4, acc0[0], acc0[1], acc0[2], acc0[3]);
        }
        step(cc);
    }
    if (kf >= 0) {
        // a copy did not complete in time: wait (bounded) for every copy issued, so none lands
        // after the CTA exits, and finish nothing
        n_issued = __shfl_sync(0xffffffffu, n_issued, 0);
        for (long j = kf; j < n_issued; ++j) mbar_wait(&bars[warp][j % XSTAGES], (unsigned)((j / XSTAGES) & 1), a.status);
        return;
    }
    if (qb <= qa) {
        XSPAN_END();
        return;
    }
    TRACE(10);
    TRACE_WARP(14 + warp);
    // This warp finishes the units (gate-up: segment; down: tile-row) whose last piece lies in
    // its run, reading every piece's partial as soon as it has landed: no arrival count and no
    // fence stand between the last piece and the unit's result.
    const long upc = MODE == 0 ? (long)np : (long)G * np;  // pieces per unit
    const int u_lo = (int)((qa + upc) / upc) - 1, u_hi = (int)(qb / upc) - 1;
    if (u_lo > u_hi) {
        XSPAN_END();
        return;
    }
#ifdef MOEARC_TRACE
    int n_rounds = 0;
#define TRACE_ROUNDS (&n_rounds)
    if (lane == 0 && g_trace) atomicMax(&g_trace[(size_t)trace_row * 32 + 9], xnow());
#else
#define TRACE_ROUNDS nullptr
#endif
    for (int u = u_lo; u <= u_hi; ++u) {
        bool failed = false;
        if (MODE == 0) {
            // gate-up segment (group g, tile-row tr): the activation of 16 rows x ntok columns;
            // lane t * 8 + r takes column t, rows r and r + 8 (one float4 a piece)
            const int g = u / ntr, tr = u % ntr;
            const int ntok = tb.grp_ntok[g], col0 = tb.grp_col0[g];
            const int nblk_i = a.I / 32;
            for (int e = lane; e < 8 * ntok; e += 32) {
                const int r = e & 7, t = e >> 3;
                float gu[4];  // gate r, gate r + 8, up r, up r + 8
                if (!take_quads<false>(a.part, rec, np, u, e * 4, gu, a.status, a.poll_ns, a.phantom, TRACE_ROUNDS)) {
                    failed = true;
                    break;
                }
                const int col = col0 + t;
                if (a.bias_gu) {
                    const int ex = tb.grp_expert[g];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int row = tr * 16 + r + 8 * h;
                        gu[h] += a.bias_gu[(size_t)ex * a.I + row];
                        gu[2 + h] += a.bias_gu[(size_t)(a.E + ex) * a.I + row];
                    }
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int row = tr * 16 + r + 8 * h;
                    const float v = act_fn(a.act, gu[h], gu[2 + h], a.alpha, a.limit);
                    a.act_out[(size_t)col * a.I + row] = v;
                    const __half hh = __float2half_rn(v);
                    const __half hl = __float2half_rn(v - __half2float(hh));
                    // element el of block blk sits in pair j = el & 3 of lane q = (el & 15) >> 2, in
                    // the low half for el < 16 and the high half for el >= 16
                    const int blk = row / 32, el = row % 32;
                    const int qq = (el & 15) >> 2, jj = el & 3, half = el >> 4;
                    const size_t ihi = ((((size_t)col * nblk_i + blk) * 2 + 0) * 4 + qq) * 4 + jj;
                    const size_t ilo = ((((size_t)col * nblk_i + blk) * 2 + 1) * 4 + qq) * 4 + jj;
                    reinterpret_cast<uint16_t *>(a.actfrag + ihi)[half] = __half_as_ushort(hh);
                    reinterpret_cast<uint16_t *>(a.actfrag + ilo)[half] = __half_as_ushort(hl);
                }
            }
            if (__any_sync(0xffffffffu, failed)) return;
#ifdef MOEARC_TRACE
            {
                const int mr = __reduce_max_sync(0xffffffffu, n_rounds);
                if (lane == 0 && g_trace && u == u_lo) {
                    atomicMax(&g_trace[(size_t)trace_row * 32 + 11], xnow());
                    atomicMax(&g_trace[(size_t)trace_row * 32 + 13], (unsigned long long)mr);
                }
            }
#endif
            // the segment's records, the columns in use, back to empty
            empty_recs(a.part + (size_t)u * np * rec, np, rec, ntok * 8, lane);
        } else {
            // down tile-row tr: per token, the router-weighted sum over its k experts in router
            // order (moe.rs:2395-2421), plus the residual. Lane (t, m, r) sums the outputs of
            // rows r and r + 8 for token t's m-th expert (one float4 a piece) into this warp's
            // ring (all its copies have landed), staged [T][16][K]; then per (token, row) the
            // fmaf chain in router order. The residual of the lane's first (token, row) is
            // read before the poll.
            const int tr = u;
            float *os = reinterpret_cast<float *>(ring);
            const int n_q = a.T * a.K * 8;
            const float res_first = (a.residual && lane < a.T * 16)
                                        ? a.residual[(size_t)(lane >> 4) * a.H + tr * 16 + (lane & 15)]
                                        : 0.f;
            for (int e = lane; e < n_q; e += 32) {
                const int r = e & 7, m = (e >> 3) % a.K, t = (e >> 3) / a.K;
                const int col = tb.col_of[t * a.K + m];
                if (col < 0) {
                    // a choice the host computes: nothing here (fmaf(w, 0, acc) leaves acc as it is)
                    os[(t * 16 + r) * a.K + m] = 0.f;
                    os[(t * 16 + r + 8) * a.K + m] = 0.f;
                    continue;
                }
                const int g = tb.col_grp[col];
                float o[4];
                if (!take_quads<true>(a.part, rec, np, tr * G + g, ((col - tb.grp_col0[g]) * 8 + r) * 4, o, a.status,
                                      a.poll_ns, a.phantom,
                                      TRACE_ROUNDS)) {
                    failed = true;
                    break;
                }
                if (a.bias_dn) {
                    const float *bd = a.bias_dn + (size_t)tb.idx[t * a.K + m] * a.H + tr * 16 + r;
                    o[0] += bd[0];
                    o[1] += bd[8];
                }
                os[(t * 16 + r) * a.K + m] = o[0];
                os[(t * 16 + r + 8) * a.K + m] = o[1];
            }
            if (__any_sync(0xffffffffu, failed)) return;
#ifdef MOEARC_TRACE
            {
                const int mr = __reduce_max_sync(0xffffffffu, n_rounds);
                if (lane == 0 && g_trace && u == u_lo) {
                    atomicMax(&g_trace[(size_t)trace_row * 32 + 11], xnow());
                    atomicMax(&g_trace[(size_t)trace_row * 32 + 13], (unsigned long long)mr);
                }
            }
#endif
            __syncwarp();
            for (int e = lane; e < a.T * 16; e += 32) {
                const int t = e >> 4, rr = e & 15;
                const size_t oi = (size_t)t * a.H + tr * 16 + rr;
                const float res = a.residual ? (e == lane ? res_first : a.residual[oi]) : 0.f;
                float acc = 0.f;
                for (int m = 0; m < a.K; ++m) acc = fmaf(tb.wts[t * a.K + m], os[e * a.K + m], acc);
                a.out[oi] = a.residual ? res + acc : acc;
            }
            // the tile-row's records (every group's, the columns in use) back to empty
            for (int g = 0; g < G; ++g)
                empty_recs(a.part + (size_t)(tr * G + g) * np * rec, np, rec, tb.grp_ntok[g] * 8, lane);
            __syncwarp();
        }
    }
#undef TRACE_ROUNDS
    XSPAN_END();
#undef XSPAN_END
#ifdef MOEARC_TRACE
    if (lane == 0 && g_trace) {
        unsigned long long t_;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));
        atomicMax(&g_trace[(size_t)trace_row * 32 + 30], t_);
    }
#endif
    TRACE(31);
}

// ---- the decode path, fused: route, gate-up and down in one cooperative launch -------------
//
// One CTA per SM, all resident at once (cooperative launch), so CTAs may wait on one another:
//   route    router rows spread one per warp over the grid (the lane order of moearc_matvec_f32,
//            so the logits match the oracle bit for bit); the activation's gate-up B fragments
//            are built in every CTA's shared memory (or, past two tokens, in global memory);
//            then a grid barrier
//   tables   every CTA derives the top-k and the slot tables from the logits (xbuild)
//   stream   every warp takes an equal run of gate-up pieces and then of down pieces and
//            streams both through one ring of bulk copies, so down weights are in flight while
//            gate-up finishes. Gate-up pieces leave partials; the last warp on a segment
//            applies the activation, writes the down kernel's fragments and bumps the ready
//            count of the down k-range those rows feed. A down piece waits (bounded) for its
//            k-range's count, copies its fragments from global memory and multiplies; the last
//            warp on a tile-row combines in router order and adds the residual.

struct xfused_args {
    const float *x;        // [T][H]
    const float *norm_w;   // [H] or null
    float eps;
    const float *router;   // [E][H]
    const float *rbias;    // [E] or null
    int T, H, E, K, gating, I;
    float *logits;         // [T][E]
    const uint8_t *gu_bank, *dn_bank;
    size_t gu_stride, dn_stride;
    int ntr_i, nkt_h, ntr_h, nkt_i, tile_bytes;
    int ch_gu, ch_dn, stage_bytes, ntok_max, b_smem;
    uint32_t *xfrag;       // [T][H/32][2][4][4], used when !b_smem
    int act;
    float alpha, limit;
    uint32_t *actfrag;     // [col][I/32][2][4][4]
    float *act_out;        // [col][I]
    unsigned *idx_out;
    float *wts_out;
    const float *residual;
    float *out;
    float *part_gu, *part_dn;
    unsigned *ctr_gu, *ctr_dn, *ready, *bar;
    int *status;
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- expert offload: the routed experts of a block fetched from pinned host memory ------
//
// The -ncmoe mirror (moe.rs:1179-1299 StaticSplit, stage() 2521-2564): the packed banks of an
// offloaded block live in pinned, device-mapped host memory. Instead of reading the routing back
// to the host and issuing copies (moe.rs:2121-2149), each fetch kernel builds the block's
// routing tables itself and copies the distinct routed experts' banks over PCIe into device
// slots (slot s = the s-th distinct expert, ascending), so an offloaded block is still a chain
// of kernels with no host round trip. Gate-up banks are fetched before the gate-up kernel; the
// down banks are fetched while the gate-up kernel computes.

constexpr int XFETCH_THREADS = 256;

struct xfetch_args {
    const float *logits;  // [T][E], the router kernel's output
    int T, E, K, gating;
    const uint8_t *host;  // device-visible pointer of the pinned bank (all experts)
    size_t stride;        // packed bytes per expert (a multiple of 16)
    uint8_t *stage;       // device slots, one per distinct routed expert (or the cache's)
    const int *plan;      // residency cache: the misses to copy, (expert, slot) pairs (or null)
    const unsigned *hmask;  // choices the host computes (their experts are not copied), or null
};

// Copy n16 16-byte words, the grid's threads striding, eight loads in flight per thread (host
// memory answers over PCIe with a latency of microseconds).
__device__ __forceinline__ void copy16(const uint4 *src, uint4 *dst, size_t n16) {
    const size_t nt = (size_t)gridDim.x * blockDim.x;
    size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    for (; i + 7 * nt < n16; i += 8 * nt) {
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = __ldcs(src + i + u * nt);
#pragma unroll
        for (int u = 0; u < 8; ++u) dst[i + u * nt] = v[u];
    }
    for (; i < n16; i += nt) dst[i] = __ldcs(src + i);
}

// MODE 0 (gate-up banks) follows the router kernel; MODE 1 (down banks) follows the gate-up
// kernel and needs nothing from it: the logits it reads were final before the gate-up kernel
// got past its own wait. MODE 1 waits for the gate-up kernel at its end, so the down kernel's
// wait on this one covers both.
// At most 48 registers a thread, so that a down-fetch CTA fits on an SM beside a gate-up CTA
// (512 threads x 96 registers) and the two run together.
template <int MODE>
__global__ void __launch_bounds__(XFETCH_THREADS, 5) k_xfetch(xfetch_args a) {
    __shared__ xtab tb;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (MODE == 0) {
        pdl_wait();
        pdl_trigger();
    }
    const size_t n16 = a.stride / 16;
    if (a.plan) {
        // cached: only the plan's misses, each into the slot the plan gave it
        const int n = __ldcg(a.plan);
        for (int i = 0; i < n; ++i)
            copy16(reinterpret_cast<const uint4 *>(a.host + (size_t)__ldcg(a.plan + 1 + 2 * i) * a.stride),
                   reinterpret_cast<uint4 *>(a.stage + (size_t)__ldcg(a.plan + 2 + 2 * i) * a.stride), n16);
    } else {
        xbuild(tb, a.logits, a.T, a.E, a.K, a.gating, warp, lane, a.hmask ? __ldcg(a.hmask) : 0u);
        for (int s = 0; s < tb.n_slots; ++s)
            copy16(reinterpret_cast<const uint4 *>(a.host + (size_t)tb.slot_expert[s] * a.stride),
                   reinterpret_cast<uint4 *>(a.stage + (size_t)s * a.stride), n16);
    }
    if (MODE == 1) {
        pdl_trigger();
        pdl_wait();
    }
}

// ---- residency cache of an offloaded block (the reference's ExpertCache, cache.rs:177, with
// StaticSplit's rule that a step never evicts an expert it still needs, moe.rs:1226-1255) ------
//
// One warp, after the router: the step's distinct experts (ascending) that are resident keep
// their slots and are stamped with the current position; each one that is not takes the least
// recently used slot no expert of this step holds (an empty slot first, the lowest index on a
// tie), evicting its owner, and is listed in the plan for the fetch kernels. Deterministic, so
// the slot tables are the same for any timing.
// The reference's host split (moe.rs:2180-2193 with HostPolicy::host_count,
// host_experts.rs:111-118): of one token's choices whose experts the device does not hold (bit
// m of `miss`, lane m holding choice m), the first host_count(misses) in router order are
// computed on the host. kind: 0 none, 1 ceil(misses x frac) (frac clamped to [0, 1]), 2 misses -
// over. Leaves the mask in h.hmask; with a nonzero mask, posts the job to the host's mail — the
// block, the experts and their gating weights in router order, the routed activation x (H
// floats, device memory) — and then, after a system-scope fence, the next sequence number.
// Returns the mask. One warp.
__device__ unsigned host_split(unsigned miss, const unsigned *idx, const float *wts, int K, const moe_host &h,
                               const float *x, int H, int lane) {
    const int misses = __popc(miss);
    int n = 0;
    if (h.kind == 1) n = min((int)ceilf((float)misses * fminf(fmaxf(h.frac, 0.f), 1.f)), misses);
    else if (h.kind == 2) n = max(misses - h.over, 0);
    unsigned hm = 0u, mm = miss;
    for (int i = 0; i < n; ++i) {
        hm |= mm & (0u - mm);
        mm &= mm - 1u;
    }
    if (lane == 0) *h.hmask = hm;
    if (!hm) return 0u;
    if (lane < K && ((hm >> lane) & 1u)) {
        const int p = __popc(hm & ((1u << lane) - 1u));
        reinterpret_cast<unsigned *>(h.mail + MAIL_IDS)[p] = idx[lane];
        reinterpret_cast<float *>(h.mail + MAIL_WTS)[p] = wts[lane];
    }
    if (lane == 0) {
        *reinterpret_cast<unsigned *>(h.mail + MAIL_N) = (unsigned)n;
        *reinterpret_cast<unsigned *>(h.mail + MAIL_BLOCK) = (unsigned)h.block;
    }
    for (int c = lane; c < H / 4; c += 32)
        reinterpret_cast<float4 *>(h.mail + MAIL_X)[c] = __ldcg(reinterpret_cast<const float4 *>(x) + c);
    __threadfence_system();  // every lane's writes reach host memory before the number below
    __syncwarp();
    if (lane == 0) {
        const unsigned long long seq = *h.seq + 1;
        *h.seq = seq;
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(h.mail + MAIL_SEQ), "l"(seq) : "memory");
    }
    return hm;
}

struct xplan_args {
    const float *logits;
    int T, E, K, gating;
    const int *pos;  // the decode position: the cache's clock
    int *slot_of, *owner, *stamp, *plan;
    int n_cache;
    unsigned long long *fetched;
    // host split (one token) when has_host; x: the routed activation (device)
    int has_host;
    moe_host host;
    const float *x;
    int H;
    int *status;
};

__global__ void __launch_bounds__(32) k_xplan(xplan_args a) {
    __shared__ xtab tb;
    extern __shared__ unsigned char used[];  // [n_cache]: a slot this step's experts hold
    const int lane = threadIdx.x;
    pdl_wait();
    pdl_trigger();
    xbuild(tb, a.logits, a.T, a.E, a.K, a.gating, 0, lane);
    if (a.has_host && a.T == 1) {
        // the host takes some of the choices that miss the cache; only the device's are admitted
        const bool miss = lane < a.K && a.slot_of[tb.idx[lane]] < 0;
        const unsigned hm = host_split(__ballot_sync(0xffffffffu, miss), tb.idx, tb.wts, a.K, a.host, a.x, a.H, lane);
        __syncwarp();
        if (hm) xbuild(tb, a.logits, a.T, a.E, a.K, a.gating, 0, lane, hm);
    }
    const int clock = *a.pos;
    for (int j = lane; j < a.n_cache; j += 32) used[j] = 0;
    __syncwarp();
    const int S = tb.n_slots;
    const int e = lane < S ? tb.slot_expert[lane] : -1;
    int slot = e >= 0 ? a.slot_of[e] : -1;
    if (slot >= 0) {
        used[slot] = 1;
        a.stamp[slot] = clock;
    }
    __syncwarp();
    unsigned misses = __ballot_sync(0xffffffffu, e >= 0 && slot < 0);
    int n = 0;
    while (misses) {
        const int ml = __ffs(misses) - 1;
        misses &= misses - 1;
        const int me = __shfl_sync(0xffffffffu, e, ml);
        // least recently used free slot: smallest stamp (empty slots hold INT_MIN), lowest index
        int best = INT_MAX, bi = INT_MAX;
        for (int j = lane; j < a.n_cache; j += 32) {
            const int key = used[j] ? INT_MAX : a.stamp[j];
            if (key < best) {
                best = key;
                bi = j;
            }
        }
        const int kmin = __reduce_min_sync(0xffffffffu, best);
        const int v = (int)__reduce_min_sync(0xffffffffu, best == kmin ? (unsigned)bi : 0xFFFFFFFFu);
        if (kmin == INT_MAX) {
            // every slot is held by this step (fewer slots than distinct experts): refused by
            // the host at create; reported, and the expert stays unplaced
            if (lane == 0) atomicOr(a.status, STATUS_RANGE);
            break;
        }
        if (lane == 0) {
            const int old = a.owner[v];
            if (old >= 0) a.slot_of[old] = -1;
            a.owner[v] = me;
            a.slot_of[me] = v;
            a.stamp[v] = clock;
            used[v] = 1;
            a.plan[1 + 2 * n] = me;
            a.plan[2 + 2 * n] = v;
        }
        ++n;
        __syncwarp();
    }
    if (lane == 0) {
        a.plan[0] = n;
        if (a.fetched) *a.fetched += (unsigned long long)n;
    }
}

// Host split of an offloaded block without a residency cache: every choice misses the device.
struct xsplit_args {
    const float *logits;  // [1][E]
    int E, K, gating;
    moe_host host;
    const float *x;       // [H], the routed activation
    int H;
};

__global__ void __launch_bounds__(32) k_xsplit(xsplit_args a) {
    __shared__ unsigned idx[32];
    __shared__ float wts[32];
    const int lane = threadIdx.x;
    pdl_wait();
    pdl_trigger();
    xtopk(a.logits, a.E, a.K, a.gating, lane, idx, wts);
    __syncwarp();
    host_split(a.K >= 32 ? 0xffffffffu : (1u << a.K) - 1u, idx, wts, a.K, a.host, a.x, a.H, lane);
}

// The fold of the host's share (moe.rs:2389-2420): ffn += host part, then h += ffn. The wait
// for the host's answer (its sequence number in the done record) starts before the dependency
// wait, so it overlaps the device's share; it is bounded by host.wait_ns, after which the
// status is raised and the host's share left out.
struct xfold_args {
    float *out;
    const float *residual;  // or null
    moe_host host;
    int n;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const void *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float ld_relaxed_sys_f32(const void *p) {
    float v;
    asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(256) k_xfold(xfold_args a) {
    __shared__ int take;  // 1: the host answered for this block; 0: no host share or no answer
    if (threadIdx.x == 0) {
        // the split kernel finished before the kernel this one follows was allowed to start
        const unsigned hm = __ldcg(a.host.hmask);
        int ok = 0;
        if (hm) {
            const unsigned long long want = __ldcg(a.host.seq);
            const unsigned long long t0 = xnow();
            for (;;) {
                if (ld_acquire_sys_u64(a.host.done + DONE_SEQ) == want) {
                    ok = 1;
                    break;
                }
                if (xnow() - t0 > a.host.wait_ns) {
                    atomicOr(a.host.status, STATUS_WAIT_TIMEOUT);
                    break;
                }
                __nanosleep(256);
            }
        }
        take = ok;
    }
    __syncthreads();
    const int ok = take;
    if (ok) (void)ld_acquire_sys_u64(a.host.done + DONE_SEQ);  // this thread's own acquire
    pdl_wait();  // the device's share is the previous kernel's output
    const float *host = reinterpret_cast<const float *>(a.host.done + DONE_OUT);
    for (int i = threadIdx.x; i < a.n; i += blockDim.x) {
        const float f = a.host.ffn[i] + (ok ? ld_relaxed_sys_f32(host + i) : 0.f);
        a.out[i] = a.residual ? a.residual[i] + f : f;
    }
    pdl_trigger();
}

constexpr unsigned long long XWAIT_NS = 200000000ull;  // a wait on other CTAs gives up after 0.2 s

// Grid barrier of a cooperative launch (arrivals counter + generation word, reusable across
// launches): every CTA's writes before it are visible to every CTA after it. A CTA that waits
// longer than XWAIT_NS sets STATUS_WAIT_TIMEOUT and goes on.
__device__ void grid_barrier(unsigned *bar, int *status) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned gen = ld_acquire_u32(bar + 1);
        __threadfence();
        if (atomicAdd(bar, 1u) == gridDim.x - 1) {
            atomicExch(bar, 0u);
            __threadfence();
            atomicAdd(bar + 1, 1u);
        } else {
            const unsigned long long t0 = gtimer();
            while (ld_acquire_u32(bar + 1) == gen) {
                if (gtimer() - t0 > XWAIT_NS) {
                    atomicOr(status, STATUS_WAIT_TIMEOUT);
                    break;
                }
                __nanosleep(32);
            }
        }
        __threadfence();
    }
    __syncthreads();
}

// Wait (one lane) until *p >= target; false (and STATUS_WAIT_TIMEOUT) after XWAIT_NS.
__device__ bool wait_count(const unsigned *p, unsigned target, int *status) {
    if (ld_acquire_u32(p) >= target) return true;
    const unsigned long long t0 = gtimer();
    while (ld_acquire_u32(p) < target) {
        if (gtimer() - t0 > XWAIT_NS) {
            atomicOr(status, STATUS_WAIT_TIMEOUT);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// B fragments of one k-tile for lane (n = lane / 4, q = lane % 4) from a fragment row
// [block][part][q][4 x u32] (null: a column past the group, zeros)
__device__ __forceinline__ void load_b_row(const uint32_t *brow, int kt, int lane, uint32_t (&bfr)[2][2][2]) {
    const int part = (lane >> 2) & 1, q = lane & 3;
    if (brow) {
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
            const uint4 v = *reinterpret_cast<const uint4 *>(brow + ((2 * kt + blk) * 2 + part) * 16 + q * 4);
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

// ROUTE = false: the gate-up and down phases only, after k_xroute (logits and the gate-up B
// fragments are its output). That launch is not cooperative but PDL-chained, so it starts under
// the router kernel; its CTAs still wait on one another (down pieces on ready counts), which
// needs them all resident: the grid is at most one CTA per SM, each CTA takes more than half an
// SM's shared memory, and a CTA lets the next kernel launch only once it runs, so the next
// kernel cannot take an SM before every CTA of this one has one. Every wait is bounded. With no
// grid barrier, the ready counts are reset by the last warp to leave, for the next launch.
template <int WT, bool ROUTE>
__global__ void __launch_bounds__(XW * 32, 1) k_moe_fused(xfused_args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[XW][XSTAGES];
    __shared__ xtab tb;
    __shared__ float red[XW];
    const int trace_row = (int)blockIdx.x + 1024;
    (void)trace_row;
    TRACE(0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = a.H, n4 = H / 4, nblk_h = H / 32, nblk_i = a.I / 32;
    const long NW = (long)gridDim.x * XW, gw = (long)blockIdx.x * XW + warp;
    const int chmax = max(a.ch_gu, a.ch_dn);
    uint8_t *ring = smem + (size_t)warp * XSTAGES * a.stage_bytes;
    const size_t ring_all = (size_t)XW * XSTAGES * a.stage_bytes;
    uint32_t *bbuf = reinterpret_cast<uint32_t *>(smem + ring_all) + (size_t)warp * a.ntok_max * chmax * 64;
    uint32_t *xf = reinterpret_cast<uint32_t *>(smem + ring_all + (size_t)XW * a.ntok_max * chmax * 256);
    float *xs = reinterpret_cast<float *>(smem);  // the route phase only: aliases the ring
    if (lane == 0) {
        for (int s = 0; s < XSTAGES; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
    }
    // router rows of this warp: e with floor(e * NW / E) == gw; fetch them to L2 now (static)
    const int e_lo = (int)((gw * a.E + NW - 1) / NW), e_hi = (int)(((gw + 1) * a.E + NW - 1) / NW);
    if (ROUTE && lane == 0)
        for (int e = e_lo; e < e_hi; ++e) bulk_prefetch_l2(a.router + (size_t)e * H, (unsigned)(H * 4));
    const int np_dn = (a.nkt_i + a.ch_dn - 1) / a.ch_dn;
    if (ROUTE && blockIdx.x == 0)
        for (int i = threadIdx.x; i < a.K * a.T * np_dn; i += blockDim.x) a.ready[i] = 0u;
    pdl_wait();
    TRACE(1);
    if (!ROUTE) {
        pdl_trigger();
        // the router kernel's gate-up B fragments of every token, into shared memory (xbuild's
        // barrier orders the copy before the first use)
        if (a.b_smem) {
            const uint4 *src = reinterpret_cast<const uint4 *>(a.xfrag);
            uint4 *dst = reinterpret_cast<uint4 *>(xf);
            for (int i = threadIdx.x; i < a.T * nblk_h * 8; i += blockDim.x) dst[i] = __ldcg(src + i);
        }
    }

    // ---- route ----
    for (int t = 0; ROUTE && t < a.T; ++t) {
        const float4 *xr = reinterpret_cast<const float4 *>(a.x + (size_t)t * H);
        float ss = 0.f;
        for (int c = threadIdx.x; c < n4; c += XW * 32) {
            const float4 v = __ldcg(xr + c);
            reinterpret_cast<float4 *>(xs)[c] = v;
            ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
        }
        if (a.norm_w) {
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            float tot = 0.f;
            for (int w = 0; w < XW; ++w) tot += red[w];
            const float s = 1.0f / sqrtf(tot / (float)H + a.eps);
            for (int c = threadIdx.x; c < n4; c += XW * 32) {
                float4 v = reinterpret_cast<float4 *>(xs)[c];
                const float4 n = __ldg(reinterpret_cast<const float4 *>(a.norm_w) + c);
                v = make_float4((v.x * s) * n.x, (v.y * s) * n.y, (v.z * s) * n.z, (v.w * s) * n.w);
                reinterpret_cast<float4 *>(xs)[c] = v;
            }
        }
        __syncthreads();
        for (int e = e_lo; e < e_hi; ++e) {
            const float4 *wr = reinterpret_cast<const float4 *>(a.router + (size_t)e * H);
            float acc = 0.f;
            for (int c = lane; c < n4; c += 32) {
                const float4 wv = __ldg(wr + c);
                const float4 xv = reinterpret_cast<const float4 *>(xs)[c];
                acc = fmaf(wv.x, xv.x, acc);
                acc = fmaf(wv.y, xv.y, acc);
                acc = fmaf(wv.z, xv.z, acc);
                acc = fmaf(wv.w, xv.w, acc);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (lane == 0) a.logits[(size_t)t * a.E + e] = a.rbias ? acc + a.rbias[e] : acc;
        }
        // gate-up B fragments: [block][part][q][j] = pair (x[32b+4q+j], x[32b+4q+16+j])
        if (a.b_smem) {
            for (int i = threadIdx.x; i < nblk_h * 16; i += blockDim.x) {
                const int j = i & 3, q = (i >> 2) & 3, b = i >> 4;
                uint32_t hi, lo;
                split_f16x2(xs[32 * b + 4 * q + j], xs[32 * b + 4 * q + 16 + j], hi, lo);
                xf[(((size_t)t * nblk_h + b) * 2 + 0) * 16 + q * 4 + j] = hi;
                xf[(((size_t)t * nblk_h + b) * 2 + 1) * 16 + q * 4 + j] = lo;
            }
        } else {
            for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nblk_h * 16; i += gridDim.x * blockDim.x) {
                const int j = i & 3, q = (i >> 2) & 3, b = i >> 4;
                uint32_t hi, lo;
                split_f16x2(xs[32 * b + 4 * q + j], xs[32 * b + 4 * q + 16 + j], hi, lo);
                a.xfrag[(((size_t)t * nblk_h + b) * 2 + 0) * 16 + q * 4 + j] = hi;
                a.xfrag[(((size_t)t * nblk_h + b) * 2 + 1) * 16 + q * 4 + j] = lo;
            }
        }
        __syncthreads();
    }
    if (ROUTE) {
        grid_barrier(a.bar, a.status);
        // every CTA is resident and past the route: the next kernel may launch
        pdl_trigger();
    }
    TRACE(2);

    // ---- tables ----
    xbuild(tb, a.logits, a.T, a.E, a.K, a.gating, warp, lane);
    TRACE(3);
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < tb.C; i += blockDim.x) {
            a.idx_out[i] = tb.idx[i];
            a.wts_out[i] = tb.wts[i];
        }
    const int G = tb.G;
    const int np_gu = (a.nkt_h + a.ch_gu - 1) / a.ch_gu;
    const long Qg = (long)G * a.ntr_i * np_gu, Qd = (long)a.ntr_h * G * np_dn;
    const long ga = Qg * gw / NW, gb = Qg * (gw + 1) / NW;  // this warp's gate-up pieces
    const long da = Qd * gw / NW, db = Qd * (gw + 1) / NW;  // and down pieces
    const long n_gu = gb - ga, n_all = n_gu + (db - da);

    // piece cursor over the warp's gate-up run, then its down run: piece q of a run is index j
    // of segment (g, tr) — gate-up segments (group, tile-row of I), down (tile-row of H, group)
    struct cur {
        long q;      // position in the warp's sequence
        int j, g, tr;
        bool dn;
    };
    auto locate = [&](long k) {
        cur c;
        c.q = k;
        c.dn = k >= n_gu;
        const long p = c.dn ? da + (k - n_gu) : ga + k;
        const int np = c.dn ? np_dn : np_gu;
        const long seg = p / np;
        c.j = (int)(p - seg * np);
        if (!c.dn) {
            c.g = (int)(seg / a.ntr_i);
            c.tr = (int)(seg - (long)c.g * a.ntr_i);
        } else {
            c.tr = (int)(seg / G);
            c.g = (int)(seg - (long)c.tr * G);
        }
        return c;
    };
    auto step = [&](cur &c) {
        ++c.q;
        if (c.q == n_gu) {
            c = locate(c.q);  // from the gate-up run to the down run
            return;
        }
        const int np = c.dn ? np_dn : np_gu;
        if (++c.j == np) {
            c.j = 0;
            if (!c.dn) {
                if (++c.tr == a.ntr_i) {
                    c.tr = 0;
                    ++c.g;
                }
            } else if (++c.g == G) {
                c.g = 0;
                ++c.tr;
            }
        }
    };
    auto plen = [&](const cur &c) {
        return c.dn ? min(a.ch_dn, a.nkt_i - c.j * a.ch_dn) : min(a.ch_gu, a.nkt_h - c.j * a.ch_gu);
    };
    auto issue = [&](const cur &c, int stage) {
        const int n = plen(c);
        const int elem = c.dn ? a.tile_bytes : 2 * a.tile_bytes;
        const int nkt = c.dn ? a.nkt_i : a.nkt_h;
        const int kt = c.j * (c.dn ? a.ch_dn : a.ch_gu);
        const uint8_t *src = (c.dn ? a.dn_bank + (size_t)tb.grp_expert[c.g] * a.dn_stride
                                   : a.gu_bank + (size_t)tb.grp_expert[c.g] * a.gu_stride) +
                             (size_t)(c.tr * nkt + kt) * elem;
        uint64_t *bar = &bars[warp][stage];
        fence_proxy_async();
        mbar_expect_tx(bar, (unsigned)(n * elem));
        bulk_g2s(ring + (size_t)stage * a.stage_bytes, src, (unsigned)(n * elem), bar);
    };
    cur ic = locate(0);
    long n_issued = 0;
    if (lane == 0)
        for (int s = 0; s < XSTAGES && ic.q < n_all; ++s) {
            issue(ic, s);
            step(ic);
            ++n_issued;
        }
    const int r = lane >> 2, qd = lane & 3, tt = (lane >> 3);  // tt: group member of B column lane / 4
    cur cc = locate(0);
    long kf = -1;
    bool gu_done = n_gu == 0;
    bool leave_last = false;
    // finishing steps shared by both runs: fence the warp's partials, arrive on its counters and
    // finish the units it completed last
    // warps holding pieces of segment s: with at least one piece per warp, the run from the
    // first piece's owner to the last's; with fewer pieces than warps every piece has its own
    auto seg_warps = [&](long Q, int np, long s) {
        if (Q < NW) return (unsigned)np;
        return (unsigned)(xcta(Q, NW, (s + 1) * np - 1) - xcta(Q, NW, s * np) + 1);
    };
    auto sum_seg = [&](const float *base, int rec, int np, int s, int off) {
        const float *pp = base + (size_t)s * np * rec + off;
        float t[XMAX_PIECES];
#pragma unroll
        for (int j = 0; j < XMAX_PIECES; ++j) t[j] = (j < np) ? __ldcg(pp + (size_t)j * rec) : 0.f;
        float v = 0.f;
#pragma unroll
        for (int j = 0; j < XMAX_PIECES; ++j)
            if (j < np) v += t[j];
        return v;
    };
    auto finish_gu = [&]() {
        if (gb <= ga) return;
        __threadfence();
        __syncwarp();
        const int s_first = (int)(ga / np_gu), s_last = (int)((gb - 1) / np_gu);
        bool mine = false;
        if (lane <= s_last - s_first) {
            const int u = s_first + lane;
            const unsigned target = seg_warps(Qg, np_gu, u);
            if (atomicAdd(a.ctr_gu + u, 1u) + 1 == target) {
                mine = true;
                a.ctr_gu[u] = 0;
            }
        }
        unsigned done = __ballot_sync(0xffffffffu, mine);
        if (!done) return;
        __threadfence();
        while (done) {
            const int u = s_first + __ffs(done) - 1;
            done &= done - 1;
            const int g = u / a.ntr_i, tr = u % a.ntr_i;
            const int ntok = tb.grp_ntok[g], col0 = tb.grp_col0[g];
            for (int e = lane; e < 16 * ntok; e += 32) {
                const int rr = e & 15, t = e >> 4;
                const float gs = sum_seg(a.part_gu, XREC_GU, np_gu, u, rr * GROUP + t);
                const float us = sum_seg(a.part_gu, XREC_GU, np_gu, u, 64 + rr * GROUP + t);
                const int col = col0 + t, row = tr * 16 + rr;
                const float v = act_fn(a.act, gs, us, a.alpha, a.limit);
                a.act_out[(size_t)col * a.I + row] = v;
                const __half hh = __float2half_rn(v);
                const __half hl = __float2half_rn(v - __half2float(hh));
                const int blk = row / 32, el = row % 32;
                const int qq = (el & 15) >> 2, jj = el & 3, half = el >> 4;
                const size_t ihi = ((((size_t)col * nblk_i + blk) * 2 + 0) * 4 + qq) * 4 + jj;
                const size_t ilo = ((((size_t)col * nblk_i + blk) * 2 + 1) * 4 + qq) * 4 + jj;
                reinterpret_cast<uint16_t *>(a.actfrag + ihi)[half] = __half_as_ushort(hh);
                reinterpret_cast<uint16_t *>(a.actfrag + ilo)[half] = __half_as_ushort(hl);
            }
            // publish: these 16 rows feed down k-tile tr / 4, i.e. down piece (tr / 4) / ch_dn
            __threadfence();
            __syncwarp();
            if (lane == 0) atomicAdd(a.ready + g * np_dn + (tr / 4) / a.ch_dn, 1u);
        }
    };
    auto finish_dn = [&]() {
        if (db <= da) return;
        __threadfence();
        __syncwarp();
        const int s_first = (int)(da / np_dn), s_last = (int)((db - 1) / np_dn);
        const int u_first = s_first / G, u_last = s_last / G;
        bool mine = false;
        if (lane <= u_last - u_first) {
            const int u = u_first + lane;
            unsigned target = 0, inc = 0;
            for (int gg = 0; gg < G; ++gg) {
                const int s = u * G + gg;
                target += seg_warps(Qd, np_dn, s);
                if (s >= s_first && s <= s_last) ++inc;
            }
            if (atomicAdd(a.ctr_dn + u, inc) + inc == target) {
                mine = true;
                a.ctr_dn[u] = 0;
            }
        }
        unsigned done = __ballot_sync(0xffffffffu, mine);
        if (!done) return;
        __threadfence();
        while (done) {
            const int tr = u_first + __ffs(done) - 1;
            done &= done - 1;
            // the router-weighted sum over the token's k experts in router order
            // (moe.rs:2395-2421), plus the residual
            for (int e = lane; e < a.T * 16; e += 32) {
                const int t = e >> 4, rr = e & 15;
                float acc = 0.f;
                for (int m = 0; m < a.K; ++m) {
                    const int col = tb.col_of[t * a.K + m];
                    const int g = tb.col_grp[col];
                    const float o = sum_seg(a.part_dn, XREC_DN, np_dn, tr * G + g, rr * GROUP + (col - tb.grp_col0[g]));
                    acc = fmaf(tb.wts[t * a.K + m], o, acc);
                }
                const size_t o = (size_t)t * H + tr * 16 + rr;
                a.out[o] = a.residual ? a.residual[o] + acc : acc;
            }
        }
    };

    // the last warp of the grid to leave resets the ready counts (launches without a barrier)
    auto leave = [&]() {
        if (ROUTE) return;
        __syncwarp();
        if (lane == 0) {
            __threadfence();
            leave_last = atomicAdd(a.bar, 1u) == (unsigned)NW - 1;
        }
        if (__shfl_sync(0xffffffffu, leave_last ? 1 : 0, 0)) {
            for (int i = lane; i < G * np_dn; i += 32) a.ready[i] = 0u;
            if (lane == 0) a.bar[0] = 0u;
        }
    };

    float acc0[4], acc1[4];
    while (cc.q < n_all) {
        if (cc.dn && !gu_done) {
            finish_gu();
            gu_done = true;
            TRACE(8);
        }
        const int n = plen(cc);
        const int ntok = tb.grp_ntok[cc.g], col0 = tb.grp_col0[cc.g];
        const uint32_t *brow = nullptr;
        if (!cc.dn && a.b_smem) {
            if (tt < ntok) brow = xf + (size_t)tb.col_tok[col0 + tt] * nblk_h * 32 + (size_t)cc.j * a.ch_gu * 64;
        } else {
            // fragments of this piece from global memory: down waits for its k-range first
            const int kt0 = cc.j * (cc.dn ? a.ch_dn : a.ch_gu);
            if (cc.dn) {
                const unsigned target = 4u * (unsigned)n;
                bool ok = true;
                if (lane == 0) ok = wait_count(a.ready + cc.g * np_dn + cc.j, target, a.status);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    kf = cc.q;
                    break;
                }
            }
            __syncwarp();
            const int nb = cc.dn ? nblk_i : nblk_h;
            const uint32_t *src_base = cc.dn ? a.actfrag : a.xfrag;
            for (int t = 0; t < ntok; ++t) {
                const int row = cc.dn ? col0 + t : tb.col_tok[col0 + t];
                const uint4 *src = reinterpret_cast<const uint4 *>(src_base + ((size_t)row * nb + 2 * kt0) * 32);
                uint4 *dst = reinterpret_cast<uint4 *>(bbuf + (size_t)t * chmax * 64);
                for (int i = lane; i < n * 16; i += 32) dst[i] = __ldcg(src + i);
            }
            __syncwarp();
            if (tt < ntok) brow = bbuf + (size_t)tt * chmax * 64;
        }
        const int stage = (int)(cc.q % XSTAGES);
        if (!mbar_wait(&bars[warp][stage], (unsigned)((cc.q / XSTAGES) & 1), a.status)) {
            kf = cc.q;
            break;
        }
        if (cc.q < 4) TRACE(4 + cc.q);
        const uint8_t *st = ring + (size_t)stage * a.stage_bytes;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc0[e] = acc1[e] = 0.f;
        if (!cc.dn) {
            for (int i = 0; i < n; ++i) {
                uint32_t bfr[2][2][2];
                load_b_row(brow, i, lane, bfr);
                const uint8_t *tile = st + i * 2 * a.tile_bytes;
                tile_mma<WT>(tile, lane, bfr, acc0);
                tile_mma<WT>(tile + a.tile_bytes, lane, bfr, acc1);
            }
        } else {
            for (int i = 0; i < n; ++i) {
                uint32_t bfr[2][2][2];
                load_b_row(brow, i, lane, bfr);
                tile_mma<WT>(st + i * a.tile_bytes, lane, bfr, acc0);
            }
        }
        __syncwarp();
        if (lane == 0 && ic.q < n_all) {
            issue(ic, stage);
            step(ic);
            ++n_issued;
        }
        // the piece's partial: column q = (f16 part + residual part) of rows r and r + 8
        if (!cc.dn) {
            float *pr = a.part_gu + (size_t)(ga + cc.q) * XREC_GU;
            if (qd < ntok) {
                pr[r * GROUP + qd] = acc0[0] + acc0[1];
                pr[(r + 8) * GROUP + qd] = acc0[2] + acc0[3];
                pr[64 + r * GROUP + qd] = acc1[0] + acc1[1];
                pr[64 + (r + 8) * GROUP + qd] = acc1[2] + acc1[3];
            }
        } else {
            float *pr = a.part_dn + (size_t)(da + cc.q - n_gu) * XREC_DN;
            if (qd < ntok) {
                pr[r * GROUP + qd] = acc0[0] + acc0[1];
                pr[(r + 8) * GROUP + qd] = acc0[2] + acc0[3];
            }
        }
        step(cc);
    }
    if (kf >= 0) {
        // a wait gave up: let every issued copy land before the CTA exits, finish nothing
        n_issued = __shfl_sync(0xffffffffu, n_issued, 0);
        for (long j = kf; j < n_issued; ++j) mbar_wait(&bars[warp][j % XSTAGES], (unsigned)((j / XSTAGES) & 1), a.status);
        if (!gu_done) finish_gu();  // down warps elsewhere may be waiting on these rows
        leave();
        return;
    }
    if (!gu_done) finish_gu();
    TRACE(9);
    finish_dn();
    leave();
    TRACE(31);
}

}  // namespace

// ---- host side ----------------------------------------------------------------------------

TRACE_SETTER(moe)

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

// Every partial slot of the expert kernels back to PART_EMPTY (at creation, and after a wait
// gave up).
void x_parts_empty(moearc_x_moe *m) {
    parts_empty(m->x_part_gu, m->x_part_gu_n, m->ctx->stream, m->ctx->sm_count);
    parts_empty(m->x_part_dn, m->x_part_dn_n, m->ctx->stream, m->ctx->sm_count);
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
    const size_t n_tab = tab_view::ints(TK, std::min(TK, m->E), TK, TK);
    const int tab_bytes = (int)((n_tab * 4 + 127) / 128 * 128);
    auto round128 = [](long b) { return (int)((b + 127) & ~127L); };
    // gate-up: 8 warps, one K run each; down: 4 warps, 4 K runs per column group
    m->warps_gu = 8;
    m->ranges_gu = 8;
    m->tpr_gu = (m->nkt_h + m->ranges_gu - 1) / m->ranges_gu;
    m->stage_gu = round128((long)m->tpr_gu * 2 * m->tile_bytes + (long)tok_group * 2 * m->tpr_gu * 128);
    const int part_gu = round128((long)m->ranges_gu * 2 * 16 * GROUP * 4);
    m->warps_dn = 4;
    m->ranges_dn = 4;
    m->tpr_dn = (m->nkt_i + m->ranges_dn - 1) / m->ranges_dn;
    m->stage_dn = round128((long)m->tpr_dn * m->tile_bytes + (long)tok_group * 2 * m->tpr_dn * 128);
    const int part_dn = round128(((long)TK * m->ranges_dn * 16 * GROUP + (long)TK * 16) * 4);
    const int budget = 220 * 1024;
    m->stages_gu = std::max(1, std::min(3, (budget - tab_bytes - part_gu) / (m->warps_gu * m->stage_gu)));
    m->stages_dn = std::max(1, std::min(3, (budget - tab_bytes - part_dn) / (m->warps_dn * m->stage_dn)));
    m->smem_gu = tab_bytes + part_gu + m->warps_gu * m->stages_gu * m->stage_gu;
    m->smem_dn = tab_bytes + part_dn + m->warps_dn * m->stages_dn * m->stage_dn;
    // grids: as many CTAs as fit, then shrunk so every CTA gets the same number of units
    const long groups = std::min<long>(TK, std::max<long>(m->K, std::min(m->E, TK)));
    auto balanced = [&](long units, int smem) {
        const long cap = occupancy_grid(c, smem);
        const long rounds = (units + cap - 1) / cap;
        return (int)std::max<long>(1, (units + rounds - 1) / rounds);
    };
    m->grid_gu = balanced(groups * m->ntr_i, m->smem_gu);
    m->grid_dn = balanced(m->ntr_h, m->smem_dn);
    if (m->smem_gu > 226 * 1024 || m->smem_dn > 226 * 1024 || m->stages_gu < 1 || m->stages_dn < 1) {
        delete m;
        return nullptr;
    }

    // decode path plan: one CTA per SM (fewer when a warp would get under two elements), a
    // ring of XSTAGES stages per warp, each ch elements and their B fragments
    m->xpath = TK <= MAX_TK && m->T_max <= 32 && m->K <= XMAX_K;
    const long x_pmin = (long)m->K * m->ntr_i * m->nkt_h;  // fewest elements of a launch (both modes)
    m->x_ntok = tok_group;
    m->x_ch_gu = 3;
    m->x_ch_dn = 5;
    m->x_stage_gu = round128((long)m->x_ch_gu * 2 * m->tile_bytes + (long)m->x_ntok * m->x_ch_gu * 256);
    m->x_stage_dn = round128((long)m->x_ch_dn * m->tile_bytes + (long)m->x_ntok * m->x_ch_dn * 256);
    m->x_route_grid = (m->E + XROUTE_WARPS - 1) / XROUTE_WARPS;
    m->x_route_smem = (XROUTE_WARPS + 2) * m->H * 4;  // router rows, the activation, the norm weights
    // 16 warps per CTA when their rings fit (one token: 192 KB for gpt-oss-120b), else 8
    m->x_warps = XW * XSTAGES * std::max(m->x_stage_gu, m->x_stage_dn) <= 200 * 1024 ? XW : XW / 2;
    m->x_grid = (int)std::max(1L, std::min<long>(c->sm_count, x_pmin / (m->x_warps * 2 * 5)));
    if (m->xpath && (m->x_warps * XSTAGES * std::max(m->x_stage_gu, m->x_stage_dn) > 200 * 1024 || m->x_route_smem > 200 * 1024 ||
                     (m->nkt_h + m->x_ch_gu - 1) / m->x_ch_gu > XMAX_PIECES ||
                     (m->nkt_i + m->x_ch_dn - 1) / m->x_ch_dn > XMAX_PIECES))
        m->xpath = false;

    // fused decode kernel: one CTA per SM, all resident; a ring stage holds one piece of either
    // kind; the gate-up B fragments of up to 24 KB of tokens stay in shared memory
    {
        const int chmax = std::max(m->x_ch_gu, m->x_ch_dn);
        m->f_stage = round128(std::max((long)m->x_ch_gu * 2 * m->tile_bytes, (long)m->x_ch_dn * m->tile_bytes));
        m->f_bsmem = (long)m->T_max * (m->H / 32) * 128 <= 24 * 1024;
        m->f_smem = XW * XSTAGES * m->f_stage + XW * m->x_ntok * chmax * 256 +
                    (m->f_bsmem ? m->T_max * (m->H / 32) * 128 : 0);
        int occ = 0;
        const bool ok = m->xpath && m->f_smem <= 200 * 1024 && XW * XSTAGES * m->f_stage >= m->H * 4 &&
                        cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                            &occ, m->wtype == T_MXFP4 ? k_moe_fused<39, true> : k_moe_fused<2, true>, XW * 32,
                            0) == cudaSuccess;
        cudaGetLastError();
        // one CTA per SM, fewer when even the smallest launch (one group per chosen expert)
        // would leave warps without a piece
        const long qmin = std::min((long)m->K * m->ntr_i * ((m->nkt_h + m->x_ch_gu - 1) / m->x_ch_gu),
                                   (long)m->K * m->ntr_h * ((m->nkt_i + m->x_ch_dn - 1) / m->x_ch_dn));
        m->f_grid = (int)std::max(1L, std::min<long>(c->sm_count, qmin / XW));
        // opt-in: correct (the same tests pass) but, as a cooperative launch, it cannot start
        // while the kernel before it finishes, and it measured slower than the three kernels
        const char *fz = std::getenv("MOEARC_FUSED_MOE");
        m->fused = ok && occ >= 1 && fz && fz[0] == '1';
        // opt-in (MOEARC_MOE_FUSED_GD=1): k_xroute, then gate-up and down as one PDL-chained
        // launch (its CTAs wait on one another, so it needs every CTA resident: one per SM, and
        // more than half an SM's shared memory each, so no SM takes two). Correct (the same
        // tests pass) but measured slower than separate gate-up and down kernels: each warp
        // runs its gate-up and its down pieces in series, and the down pieces wait for the
        // slowest gate-up segment of their k-range.
        const char *gd = std::getenv("MOEARC_MOE_FUSED_GD");
        m->fused_gd = m->xpath && m->f_smem <= 200 * 1024 && m->f_smem > 114 * 1024 && m->f_bsmem &&
                      m->f_grid <= c->sm_count && gd && gd[0] == '1';
    }

    // one scratch allocation
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
    const size_t n_ctr = 1 + (size_t)TK * m->ntr_i + m->ntr_h;
    const size_t o_ctr = take(sizeof(unsigned) * n_ctr);
    const size_t o_st = take(sizeof(int));
    const size_t x_segs_gu = (size_t)TK * m->ntr_i, x_segs_dn = (size_t)m->ntr_h * TK;
    const size_t np_gu = (m->nkt_h + m->x_ch_gu - 1) / m->x_ch_gu, np_dn = (m->nkt_i + m->x_ch_dn - 1) / m->x_ch_dn;
    const size_t o_xpg = take(m->xpath ? sizeof(float) * x_segs_gu * np_gu * XREC_GU : 0);
    const size_t o_xpd = take(m->xpath ? sizeof(float) * x_segs_dn * np_dn * XREC_XDN : 0);
    const bool fz_any = m->fused || m->fused_gd;
    const size_t o_fpg = take(fz_any ? sizeof(float) * x_segs_gu * np_gu * XREC_GU : 0);
    const size_t o_fpd = take(fz_any ? sizeof(float) * x_segs_dn * np_dn * XREC_DN : 0);
    const size_t o_xtp = take(m->xpath ? sizeof(xtab) : 0);
    const size_t o_xcg = take(m->xpath ? sizeof(unsigned) * x_segs_gu : 0);
    const size_t o_xcd = take(m->xpath ? sizeof(unsigned) * m->ntr_h : 0);
    const size_t o_frd = take(m->xpath ? sizeof(unsigned) * (size_t)TK * np_dn : 0);
    const size_t o_fbar = take(sizeof(unsigned) * 2);
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
    m->ctr = reinterpret_cast<unsigned *>(b + o_ctr);
    m->status = reinterpret_cast<int *>(b + o_st);
    m->act_f32 = reinterpret_cast<float *>(b + o_act);
    m->x_part_gu = reinterpret_cast<float *>(b + o_xpg);
    m->x_part_dn = reinterpret_cast<float *>(b + o_xpd);
    m->x_part_gu_n = m->xpath ? x_segs_gu * np_gu * XREC_GU : 0;
    m->x_part_dn_n = m->xpath ? x_segs_dn * np_dn * XREC_XDN : 0;
    m->x_tab_pub = m->xpath ? b + o_xtp : nullptr;
    m->f_part_gu = reinterpret_cast<float *>(b + o_fpg);
    m->f_part_dn = reinterpret_cast<float *>(b + o_fpd);
    m->x_ctr_gu = reinterpret_cast<unsigned *>(b + o_xcg);
    m->x_ctr_dn = reinterpret_cast<unsigned *>(b + o_xcd);
    m->f_ready = reinterpret_cast<unsigned *>(b + o_frd);
    m->f_bar = reinterpret_cast<unsigned *>(b + o_fbar);
    cudaMemsetAsync(m->mem, 0, off, c->stream);
    x_parts_empty(m);
    if (m->wtype == T_MXFP4 && m->xpath)
        m->xtc = xtc_create(c, m->H, m->I, m->E, m->K, m->gating, m->act, m->alpha, m->limit);
    // per-kernel attribute shared by every layer object: the most any of them may use
    const int smem_attr = 226 * 1024;
    if (set_smem(k_moe_rows<39>, smem_attr) != cudaSuccess ||
        set_smem(k_moe_rows<2>, smem_attr) != cudaSuccess ||
        set_smem(k_xexpert<39, 0>, 200 * 1024) != cudaSuccess ||
        set_smem(k_xexpert<39, 1>, 200 * 1024) != cudaSuccess ||
        set_smem(k_xexpert<2, 0>, 200 * 1024) != cudaSuccess ||
        set_smem(k_xexpert<2, 1>, 200 * 1024) != cudaSuccess ||
        set_smem(k_xroute, 200 * 1024) != cudaSuccess ||
        set_smem(k_moe_fused<39, true>, 200 * 1024) != cudaSuccess ||
        set_smem(k_moe_fused<2, true>, 200 * 1024) != cudaSuccess ||
        set_smem(k_moe_fused<39, false>, 200 * 1024) != cudaSuccess ||
        set_smem(k_moe_fused<2, false>, 200 * 1024) != cudaSuccess ||
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
    xtc_destroy(m->xtc);
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

}  // extern "C"

namespace moearc {

// The forward pass; norm_w (may be null) routes rmsnorm(x) * norm_w instead of x.
int moe_forward_impl(moearc_x_moe *m, const float *x, unsigned n_tokens, const float *norm_w, float eps,
                     const float *router_w, const float *router_b, const void *gateup_packed,
                     const void *down_packed, const float *residual, float *out,
                     std::vector<cudaEvent_t> *marks, std::vector<int> *kinds, const moe_offload *off,
                     unsigned long long *span, bool tc, int span_cta) {
    auto mark = [&](int k) {
        if (!marks) return;
        cudaEvent_t e;
        cudaEventCreate(&e);
        cudaEventRecord(e, m->ctx->stream);
        marks->push_back(e);
        kinds->push_back(k);
    };
    if (!m || !x || !router_w || !gateup_packed || !down_packed || !out) return ERR;
    if (n_tokens == 0) return OK;
    if ((int)n_tokens > m->T_max) return ERR_ARG;
    if (norm_w && n_tokens > (unsigned)ROUTE_NORM_TOKENS) return ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(router_w) |
         reinterpret_cast<uintptr_t>(gateup_packed) | reinterpret_cast<uintptr_t>(down_packed)) & 15)
        return ERR_ARG;
    moearc_ctx *c = m->ctx;
    const int T = (int)n_tokens;
    const tab_view tab = make_tab(m);
    launch_scope ls(c, "moe_forward", (unsigned long)m->H, (unsigned)T);

    // an offloaded block runs the decode path with the fetch kernels (gateup_packed and
    // down_packed are then device-visible pointers of pinned host banks)
    if (off && (!m->xpath || !off->gu_stage || !off->dn_stage)) return ERR_ARG;
    if (tc) {
        // banks in the tc layout: one token, resident (xtc.cu)
        if (!m->xtc || T != 1 || off) return ERR_ARG;
        xroute_args xr{x, norm_w, eps, router_w, router_b, T, m->H, m->E, m->logits, m->xfrag, nullptr, m->status,
                       xtc_xdig(m->xtc)};
        if (launch_pdl(k_xroute, dim3(m->x_route_grid), dim3(XROUTE_WARPS * 32), (size_t)m->x_route_smem, c->stream,
                       xr) != cudaSuccess)
            return ERR;
        mark(3);
        xtc_run r{};
        r.logits = m->logits;
        r.xdig = xtc_xdig(m->xtc);
        r.gu_bank = static_cast<const uint8_t *>(gateup_packed);
        r.dn_bank = static_cast<const uint8_t *>(down_packed);
        r.residual = residual;
        r.out = out;
        r.idx_out = m->idx;
        r.wts_out = m->wts;
        r.act_out = m->act_f32;
        r.bias_gu = m->bias_gu;
        r.bias_dn = m->bias_dn;
        r.poll_ns = m->x_poll_ns;
        r.phantom = m->x_phantom;
        r.span = span;
        r.span_cta = span_cta ? span_cta : xtc_grid(m->xtc);
        r.status = m->status;
        if (xtc_launch_gu(m->xtc, r) != OK) return ERR;
        mark(4);
        if (xtc_launch_dn(m->xtc, r) != OK) return ERR;
        mark(5);
        return ls.finish();
    }
    auto fused_args = [&]() {
        xfused_args f{};
        f.x = x;
        f.norm_w = norm_w;
        f.eps = eps;
        f.router = router_w;
        f.rbias = router_b;
        f.T = T;
        f.H = m->H;
        f.E = m->E;
        f.K = m->K;
        f.gating = m->gating;
        f.I = m->I;
        f.logits = m->logits;
        f.gu_bank = static_cast<const uint8_t *>(gateup_packed);
        f.dn_bank = static_cast<const uint8_t *>(down_packed);
        f.gu_stride = (size_t)2 * m->ntr_i * m->nkt_h * m->tile_bytes;
        f.dn_stride = (size_t)m->ntr_h * m->nkt_i * m->tile_bytes;
        f.ntr_i = m->ntr_i;
        f.nkt_h = m->nkt_h;
        f.ntr_h = m->ntr_h;
        f.nkt_i = m->nkt_i;
        f.tile_bytes = m->tile_bytes;
        f.ch_gu = m->x_ch_gu;
        f.ch_dn = m->x_ch_dn;
        f.stage_bytes = m->f_stage;
        f.ntok_max = m->x_ntok;
        f.b_smem = m->f_bsmem;
        f.xfrag = m->xfrag;
        f.act = m->act;
        f.alpha = m->alpha;
        f.limit = m->limit;
        f.actfrag = m->actfrag;
        f.act_out = m->act_f32;
        f.idx_out = m->idx;
        f.wts_out = m->wts;
        f.residual = residual;
        f.out = out;
        f.part_gu = m->f_part_gu;
        f.part_dn = m->f_part_dn;
        f.ctr_gu = m->x_ctr_gu;
        f.ctr_dn = m->x_ctr_dn;
        f.ready = m->f_ready;
        f.bar = m->f_bar;
        f.status = m->status;
        return f;
    };
    const bool biased = m->bias_gu || m->bias_dn;  // the opt-in single-launch kernels have no biases
    if (m->fused && !off && !biased) {
        if (launch_coop(m->wtype == T_MXFP4 ? k_moe_fused<39, true> : k_moe_fused<2, true>, dim3(m->f_grid),
                        dim3(XW * 32), (size_t)m->f_smem, c->stream, fused_args()) != cudaSuccess)
            return ERR;
        mark(4);
        return ls.finish();
    }
    if (m->xpath) {
        // part of an offloaded block's experts on the host cores (one token per call)
        const moe_host *hs = (off && off->host && off->host->kind && T == 1) ? off->host : nullptr;
        if (hs && biased) return ERR_ARG;  // the host pool has no expert biases
        // the routed activation goes to the host through the device's-share buffer, which the
        // down kernel overwrites only after the split kernel has read it
        xroute_args xr{x, norm_w, eps, router_w, router_b, T, m->H, m->E, m->logits, m->xfrag,
                       hs ? hs->ffn : nullptr, m->status};
        if (launch_pdl(k_xroute, dim3(m->x_route_grid), dim3(XROUTE_WARPS * 32), (size_t)m->x_route_smem, c->stream,
                       xr) != cudaSuccess)
            return ERR;
        mark(3);
        if (m->fused_gd && !off && !biased) {
            // gate-up and down in one launch: down weights stream while gate-up finishes
            if (launch_pdl(m->wtype == T_MXFP4 ? k_moe_fused<39, false> : k_moe_fused<2, false>, dim3(m->f_grid),
                           dim3(XW * 32), (size_t)m->f_smem, c->stream, fused_args()) != cudaSuccess)
                return ERR;
            mark(4);
            return ls.finish();
        }
        const size_t gu_stride = (size_t)2 * m->ntr_i * m->nkt_h * m->tile_bytes;
        const size_t dn_stride = (size_t)m->ntr_h * m->nkt_i * m->tile_bytes;
        xfetch_args fa{m->logits, T, m->E, m->K, m->gating, nullptr, 0, nullptr, nullptr, hs ? hs->hmask : nullptr};
        if (off && off->slot_of) {
            // residency cache: plan the step's slots (hits stay, misses evict the least recently
            // used slot), then fetch only the misses; with a host policy the host first takes its
            // share of the misses, which are neither admitted nor fetched
            xplan_args pa{m->logits, T, m->E, m->K, m->gating, off->clock, off->slot_of, off->owner, off->stamp,
                          off->plan, off->n_cache, off->fetched, hs ? 1 : 0, hs ? *hs : moe_host{},
                          hs ? hs->ffn : nullptr, m->H, m->status};
            if (launch_pdl(k_xplan, dim3(1), dim3(32), (size_t)off->n_cache, c->stream, pa) != cudaSuccess)
                return ERR;
            fa.plan = off->plan;
        } else if (hs) {
            xsplit_args sa{m->logits, m->E, m->K, m->gating, *hs, hs->ffn, m->H};
            if (launch_pdl(k_xsplit, dim3(1), dim3(32), 0, c->stream, sa) != cudaSuccess) return ERR;
        }
        if (off) {
            fa.host = static_cast<const uint8_t *>(gateup_packed);
            fa.stride = gu_stride;
            fa.stage = off->gu_stage;
            if (launch_pdl(k_xfetch<0>, dim3(c->sm_count), dim3(XFETCH_THREADS), 0, c->stream, fa) != cudaSuccess)
                return ERR;
            mark(7);
        }
        xexp_args xa{};
        xa.bank = off ? off->gu_stage : static_cast<const uint8_t *>(gateup_packed);
        xa.bank_stride = gu_stride;
        xa.by_slot = off ? 1 : 0;
        xa.ntr = m->ntr_i;
        xa.nkt = m->nkt_h;
        xa.tile_bytes = m->tile_bytes;
        xa.elem_bytes = 2 * m->tile_bytes;
        xa.ch = m->x_ch_gu;
        xa.stage_bytes = m->x_stage_gu;
        xa.ntok_max = m->x_ntok;
        xa.nblk_b = m->H / 32;
        xa.bsrc = m->xfrag;
        xa.logits = m->logits;
        xa.T = T;
        xa.E = m->E;
        xa.K = m->K;
        xa.gating = m->gating;
        xa.act = m->act;
        xa.alpha = m->alpha;
        xa.limit = m->limit;
        xa.actfrag = m->actfrag;
        xa.act_out = m->act_f32;
        xa.I = m->I;
        xa.idx_out = m->idx;
        xa.wts_out = m->wts;
        xa.H = m->H;
        xa.part = m->x_part_gu;
        // offloaded blocks: the down fetch runs between the two kernels and the down kernel
        // builds its own tables after its wait
        xa.tab_pub = off ? nullptr : static_cast<xtab *>(m->x_tab_pub);
        xa.slot_of = off ? off->slot_of : nullptr;
        xa.hmask = hs ? hs->hmask : nullptr;
        xa.poll_ns = m->x_poll_ns;
        xa.phantom = m->x_phantom;
        xa.bias_gu = m->bias_gu;
        xa.bias_dn = m->bias_dn;
        xa.status = m->status;
        xa.span = span;  // the gate-up kernel's CTAs, then the down kernel's
        const bool mx = m->wtype == T_MXFP4;
        // More than half an SM's shared memory, so no SM takes two gate-up CTAs: at launch the
        // router's CTAs still hold some SMs, and a CTA that fits beside another gate-up CTA
        // would start there, leaving its SM's share of the stream to be split with a neighbour
        // while other SMs go without. One down CTA still fits beside it.
        const size_t smem_gu = std::max((size_t)m->x_warps * XSTAGES * m->x_stage_gu, (size_t)XEXCLUSIVE_SMEM);
        if (launch_pdl(mx ? k_xexpert<39, 0> : k_xexpert<2, 0>, dim3(m->x_grid), dim3(m->x_warps * 32), smem_gu,
                       c->stream, xa) != cudaSuccess)
            return ERR;
        mark(4);
        if (off) {
            fa.host = static_cast<const uint8_t *>(down_packed);
            fa.stride = dn_stride;
            fa.stage = off->dn_stage;
            if (launch_pdl(k_xfetch<1>, dim3(c->sm_count), dim3(XFETCH_THREADS), 0, c->stream, fa) != cudaSuccess)
                return ERR;
            mark(7);
        }
        xexp_args xd = xa;
        xd.span = span ? span + (size_t)m->x_grid * 3 : nullptr;
        xd.bank = off ? off->dn_stage : static_cast<const uint8_t *>(down_packed);
        xd.bank_stride = dn_stride;
        xd.ntr = m->ntr_h;
        xd.nkt = m->nkt_i;
        xd.elem_bytes = m->tile_bytes;
        xd.ch = m->x_ch_dn;
        xd.stage_bytes = m->x_stage_dn;
        xd.nblk_b = m->I / 32;
        xd.bsrc = m->actfrag;
        xd.residual = hs ? nullptr : residual;  // with a host share: the device's share alone, folded below
        xd.out = hs ? hs->ffn : out;
        xd.part = m->x_part_dn;
        if (launch_pdl(mx ? k_xexpert<39, 1> : k_xexpert<2, 1>, dim3(m->x_grid), dim3(m->x_warps * 32),
                       (size_t)m->x_warps * XSTAGES * m->x_stage_dn, c->stream, xd) != cudaSuccess)
            return ERR;
        mark(5);
        if (hs) {
            if (launch_pdl(k_xfold, dim3(1), dim3(256), 0, c->stream, xfold_args{out, residual, *hs, m->H}) !=
                cudaSuccess)
                return ERR;
            mark(8);
        }
        return ls.finish();
    }

    route_args ra{x, norm_w, eps, router_w, router_b, T, m->H, m->E, m->K, m->gating, m->logits, m->idx,
                  m->wts, m->xfrag, tab, m->ctr};
    // one router row per warp, one pass of the fragment conversion
    const int rows_ctas = (T * m->E + ROUTE_WARPS - 1) / ROUTE_WARPS;
    const int conv_ctas = (T * (m->H / 32) * 16 + ROUTE_WARPS * 32 - 1) / (ROUTE_WARPS * 32);
    const int grid_r = std::max(1, std::min(std::max(rows_ctas, conv_ctas), c->sm_count * 4));
    if (launch_pdl(k_route, dim3(grid_r), dim3(ROUTE_WARPS * 32), 0, c->stream, ra) != cudaSuccess) return ERR;
    mark(3);

    rows_args ga{};
    ga.bank = static_cast<const uint8_t *>(gateup_packed);
    ga.bank_stride = (size_t)2 * m->ntr_i * m->nkt_h * m->tile_bytes;
    ga.mats = 2;
    ga.ntr = m->ntr_i;
    ga.nkt = m->nkt_h;
    ga.ranges = m->ranges_gu;
    ga.tpr = m->tpr_gu;
    ga.tile_bytes = m->tile_bytes;
    ga.stages = m->stages_gu;
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
    ga.bias_gu = m->bias_gu;
    ga.bias_dn = m->bias_dn;
    ga.E = m->E;
    ga.status = m->status;
    if (launch_pdl(m->wtype == T_MXFP4 ? k_moe_rows<39> : k_moe_rows<2>, dim3(m->grid_gu), dim3(m->warps_gu * 32),
                   (size_t)m->smem_gu, c->stream, ga) != cudaSuccess)
        return ERR;
    mark(4);

    rows_args da = ga;
    da.bank = static_cast<const uint8_t *>(down_packed);
    da.bank_stride = (size_t)m->ntr_h * m->nkt_i * m->tile_bytes;
    da.mats = 1;
    da.ntr = m->ntr_h;
    da.nkt = m->nkt_i;
    da.ranges = m->ranges_dn;
    da.tpr = m->tpr_dn;
    da.stages = m->stages_dn;
    da.stage_bytes = m->stage_dn;
    da.bsrc = m->actfrag;
    da.b_by_column = 1;
    da.nblk_b = m->I / 32;
    da.wts = m->wts;
    da.residual = residual;
    da.out = out;
    if (launch_pdl(m->wtype == T_MXFP4 ? k_moe_rows<39> : k_moe_rows<2>, dim3(m->grid_dn), dim3(m->warps_dn * 32),
                   (size_t)m->smem_dn, c->stream, da) != cudaSuccess)
        return ERR;
    mark(5);
    return ls.finish();
}

// CTAs of each decode-path expert kernel (their span records, per kernel).
int moe_decode_grid(moearc_x_moe *m) { return m && m->xpath ? std::max(m->x_grid, xtc_grid(m->xtc)) : 0; }

}  // namespace moearc

extern "C" {

int moearc_x_moe_forward(moearc_x_moe *m, const float *x, unsigned n_tokens, const float *router_w,
                         const float *router_b, const void *gateup_packed, const void *down_packed,
                         const float *residual, float *out) {
    return moe_forward_impl(m, x, n_tokens, nullptr, 0.f, router_w, router_b, gateup_packed, down_packed,
                            residual, out, nullptr, nullptr, nullptr, nullptr, false, 0);
}

unsigned long moearc_x_moe_tc_bytes(const moearc_x_moe_desc *d, int which) {
    if (!d || d->wtype != T_MXFP4 || d->n_embd % 64 || d->n_ff % 64) return 0;
    return which == 0 ? (unsigned long)tc_gu_stride((int)d->n_embd, (int)d->n_ff) * d->n_expert
                      : (unsigned long)tc_dn_stride((int)d->n_embd, (int)d->n_ff) * d->n_expert;
}

int moearc_x_moe_has_tc(moearc_x_moe *m) { return m && m->xtc ? 1 : 0; }

int moearc_x_moe_pack_tc(moearc_x_moe *m, const void *gate, const void *up, const void *down, unsigned n_expert,
                         void *gateup_tc, void *down_tc) {
    if (!m || !gate || !up || !down || !gateup_tc || !down_tc) return ERR;
    if (m->wtype != T_MXFP4 || m->H % 64 || m->I % 64 || n_expert == 0) return ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(gateup_tc) | reinterpret_cast<uintptr_t>(down_tc)) & 15) return ERR_ARG;
    launch_scope ls(m->ctx, "moe_pack_tc", (unsigned long)n_expert, 2);
    const int rc = xtc_pack(m->ctx, m->H, m->I, gate, up, down, n_expert, gateup_tc, down_tc);
    return rc ? rc : ls.finish();
}

int moearc_x_moe_forward_tc(moearc_x_moe *m, const float *x, unsigned n_tokens, const float *router_w,
                            const float *router_b, const void *gateup_tc, const void *down_tc, const float *residual,
                            float *out) {
    if (!m) return ERR;
    if (!m->xtc || n_tokens > 1) return ERR_ARG;
    return moe_forward_impl(m, x, n_tokens, nullptr, 0.f, router_w, router_b, gateup_tc, down_tc, residual, out,
                            nullptr, nullptr, nullptr, nullptr, true, 0);
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

int moearc_x_moe_set_bias(moearc_x_moe *m, const float *gate_up_bias, const float *down_bias) {
    if (!m) return ERR;
    if ((reinterpret_cast<uintptr_t>(gate_up_bias) | reinterpret_cast<uintptr_t>(down_bias)) & 3) return ERR_ARG;
    m->bias_gu = gate_up_bias;
    m->bias_dn = down_bias;
    return OK;
}

int moearc_x_moe_set_wait(moearc_x_moe *m, unsigned long long poll_ns, int phantom) {
    if (!m) return ERR;
    m->x_poll_ns = poll_ns ? poll_ns : XPOLL_NS;
    m->x_phantom = phantom ? 1 : 0;
    return OK;
}

int moearc_x_moe_status(moearc_x_moe *m) {
    if (!m) return ERR;
    int st = 0;
    if (cudaMemcpyAsync(&st, m->status, sizeof(int), cudaMemcpyDeviceToHost, m->ctx->stream) != cudaSuccess) return ERR;
    if (cudaStreamSynchronize(m->ctx->stream) != cudaSuccess) return ERR;
    if (st) {
        // a wait that gave up can leave partial slots stored and never read: empty them all
        cudaMemsetAsync(m->status, 0, sizeof(int), m->ctx->stream);
        x_parts_empty(m);
        xtc_reset(m->xtc);
    }
    return st;
}

}  // extern "C"
