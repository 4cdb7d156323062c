// dense.cu — packed bf16 tensor-core GEMVs for the decoder's attention projections.
// See dense.cuh for the structure.
#include <algorithm>
#include <cmath>

#include "dense.cuh"
#include "tma.cuh"

namespace moearc {

namespace {

constexpr int WARPS = 8;
constexpr int CH = 2;          // tiles per ring stage (4 KB bulk copies)
constexpr int STAGES = 3;      // ring stages per warp
constexpr int PARTS = 3;       // bf16 rounding + two residuals
constexpr int MAX_LOCAL = 8;   // tile-rows (hence units) one CTA may touch; <= WARPS
constexpr int MAX_ITEMS = 8;   // B-fragment items per thread: n_cols / 2 <= 8 x 256
constexpr int MAX_COLS = 2 * MAX_ITEMS * WARPS * 32;
constexpr int RING_BYTES = WARPS * STAGES * CH * DENSE_TILE;
constexpr int MAX_CONTRIB = 4;  // CTAs that may share one tile-row (checked at plan time)

__global__ void k_dense_pack(uint8_t *dst, const uint16_t *src, int n_rows, int n_cols) {
    const int nkt = n_cols / 64;
    const size_t total = (size_t)(n_rows / 16) * nkt * 128;  // (tile, sub-block, lane)
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < total; g += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(g & 31), s = (int)((g >> 5) & 3);
        const size_t tile = g >> 7;
        const int tr = (int)(tile / nkt), tk = (int)(tile % nkt);
        const int r = lane >> 2, q = lane & 3;
        uint32_t *o = reinterpret_cast<uint32_t *>(dst + tile * DENSE_TILE + s * 512 + lane * 16);
        const uint16_t *rowA = src + (size_t)(tr * 16 + r) * n_cols + tk * 64;
        const uint16_t *rowB = rowA + (size_t)8 * n_cols;
        const int c0 = 16 * s + 2 * q, c1 = c0 + 8;
        o[0] = (uint32_t)rowA[c0] | ((uint32_t)rowA[c0 + 1] << 16);
        o[1] = (uint32_t)rowB[c0] | ((uint32_t)rowB[c0 + 1] << 16);
        o[2] = (uint32_t)rowA[c1] | ((uint32_t)rowA[c1 + 1] << 16);
        o[3] = (uint32_t)rowB[c1] | ((uint32_t)rowB[c1 + 1] << 16);
    }
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint16_t bf(float v) { return f32_to_bf16_bits(v); }

struct dense_args {
    const uint8_t *w;
    int n_rows, n_cols, ntr, nkt;
    long T;         // tiles
    int mode;
    int unit_trs;   // tile-rows per unit
    int maxc;       // partial slots per tile-row (the most CTAs that touch one tile-row)
    const float *in;
    const float *norm_w;
    float eps;
    float *out;
    const float *residual;
    const int *pos;
    dense_rope rope;
    dense_kv kv;
    float *part;    // [ntr][maxc][16] partial slots, PART_EMPTY when free
    int *status;
};

// First tile of CTA c's range (ranges are [T c / G, T (c + 1) / G)), and the CTA whose range
// holds tile t.
__host__ __device__ __forceinline__ long tile_lo(long T, int G, int c) { return T * c / G; }
__host__ __device__ __forceinline__ int cta_of(long T, int G, long t) { return (int)(((t + 1) * G - 1) / T); }

__global__ void __launch_bounds__(WARPS * 32, 1) k_dense(dense_args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[WARPS][STAGES];
    __shared__ float red[WARPS];
    const int trace_row = (int)blockIdx.x + (a.mode == 0 ? 0 : 1024);
    (void)trace_row;
    TRACE(0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const long ta = tile_lo(a.T, G, cta), tb = tile_lo(a.T, G, cta + 1);
    const long wa = ta + (tb - ta) * warp / WARPS, wb = ta + (tb - ta) * (warp + 1) / WARPS;
    const int nkb = a.n_cols / 16;
    uint8_t *ring = smem + (size_t)warp * STAGES * CH * DENSE_TILE;
    uint32_t *bsm = reinterpret_cast<uint32_t *>(smem + RING_BYTES);  // [nkb][3][4][2]
    float *psm = reinterpret_cast<float *>(smem + RING_BYTES + (size_t)nkb * PARTS * 32);  // [WARPS][MAX_LOCAL][16]
    const int tr0 = (int)(ta / a.nkt), tr1 = (int)((tb - 1) / a.nkt);  // tile-rows this CTA touches

    if (lane == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    const long nch = (wb - wa + CH - 1) / CH;
    auto issue = [&](long j, int s) {
        const long t0 = wa + j * CH;
        const long n = (wb - t0 < CH) ? wb - t0 : CH;
        const unsigned bytes = (unsigned)(n * DENSE_TILE);
        fence_proxy_async();
        mbar_expect_tx(&bars[warp][s], bytes);
        bulk_g2s(ring + (size_t)s * CH * DENSE_TILE, a.w + t0 * DENSE_TILE, bytes, &bars[warp][s]);
    };
    // the weights do not depend on the previous kernel: stream the first stages now
    long issued = nch < STAGES ? nch : STAGES;
    if (lane == 0)
        for (long j = 0; j < issued; ++j) issue(j, (int)j);
    for (int i = threadIdx.x; i < WARPS * MAX_LOCAL * 16; i += WARPS * 32) psm[i] = 0.f;
    // B-fragment item i of this thread: (k16 block kb, q, register reg) -> columns c, c + 1
    // with c = 16 kb + 2q + 8 reg. The norm weights are static and load before the wait too.
    const int n_items = nkb * 8;
    float2 nw[MAX_ITEMS];
#pragma unroll
    for (int m = 0; m < MAX_ITEMS; ++m) {
        const int i = threadIdx.x + m * WARPS * 32;
        nw[m] = make_float2(1.f, 1.f);
        if (a.norm_w && i < n_items) {
            const int reg = i & 1, q = (i >> 1) & 3, kb = i >> 3;
            nw[m] = __ldg(reinterpret_cast<const float2 *>(a.norm_w + 16 * kb + 2 * q + 8 * reg));
        }
    }
    // the position and this step's K/V page: the position advances only at the end of a step,
    // after the last kernel of the step, so both can be read before the wait
    int pos = 0;
    size_t page = 0;
    if (a.mode == 0) {
        pos = *a.pos;
        page = a.kv.table[pos / a.kv.page_tokens];
    }
    // Warp i finishes the i-th unit this CTA touches if the CTA turns out to be the unit's last
    // to arrive; for a query or key head the rotations of its RoPE pairs are known now, before
    // the wait. NeoX RoPE: pairs (d, d + D/2), the lane holding d = lane + 32 i; the angle of
    // pair p is pos * freq[p] (the YaRN blend folded into freq on the host), reduced by 2 pi in
    // two steps before the sine and cosine so large positions keep full precision; both
    // factors carry mscale.
    const int u0 = tr0 / a.unit_trs, u1 = tr1 / a.unit_trs;
    double rot_c[2] = {1.0, 1.0}, rot_s[2] = {0.0, 0.0};
    if (a.mode == 0 && warp <= u1 - u0 && u0 + warp < a.rope.n_q_heads + a.rope.n_kv_heads) {
#pragma unroll
        for (int i = 0; i < 2; ++i)
            if (i < a.rope.head_dim / 64) {
                const int p = lane + 32 * i;  // pair index < D/2
                const double th = (double)pos * __ldg(a.rope.freq + p);
                const double k = rint(th * 0.15915494309189535);
                double r = fma(-k, 6.283185307179586, th);
                r = fma(-k, 2.4492935982947064e-16, r);
                double sn, cs;
                sincos(r, &sn, &cs);
                rot_c[i] = cs * a.rope.mscale;
                rot_s[i] = sn * a.rope.mscale;
            }
    }
    pdl_trigger();
    pdl_wait();
    TRACE(1);
    float2 xv[MAX_ITEMS];
#pragma unroll
    for (int m = 0; m < MAX_ITEMS; ++m) {
        const int i = threadIdx.x + m * WARPS * 32;
        xv[m] = make_float2(0.f, 0.f);
        if (i < n_items) {
            const int reg = i & 1, q = (i >> 1) & 3, kb = i >> 3;
            xv[m] = __ldcg(reinterpret_cast<const float2 *>(a.in + 16 * kb + 2 * q + 8 * reg));
        }
    }
    float scale = 1.f;
    if (a.norm_w) {
        // RMSNorm (moe.rs:1936-1940): f32 sum of squares, 1 / sqrt(mean + eps)
        float ss = 0.f;
#pragma unroll
        for (int m = 0; m < MAX_ITEMS; ++m) ss = fmaf(xv[m].x, xv[m].x, fmaf(xv[m].y, xv[m].y, ss));
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float t = 0.f;
        for (int w = 0; w < WARPS; ++w) t += red[w];
        scale = 1.0f / sqrtf(t / (float)a.n_cols + a.eps);
    }
#pragma unroll
    for (int m = 0; m < MAX_ITEMS; ++m) {
        const int i = threadIdx.x + m * WARPS * 32;
        if (i < n_items) {
            const int reg = i & 1, q = (i >> 1) & 3, kb = i >> 3;
            float v0 = xv[m].x, v1 = xv[m].y;
            if (a.norm_w) {
                v0 = (v0 * scale) * nw[m].x;
                v1 = (v1 * scale) * nw[m].y;
            }
            const uint16_t h0 = bf(v0), h1 = bf(v1);
            float r0 = v0 - bf16_bits_to_f32(h0), r1 = v1 - bf16_bits_to_f32(h1);
            const uint16_t m0 = bf(r0), m1 = bf(r1);
            r0 -= bf16_bits_to_f32(m0);
            r1 -= bf16_bits_to_f32(m1);
            const uint16_t l0 = bf(r0), l1 = bf(r1);
            bsm[(((size_t)kb * PARTS + 0) * 4 + q) * 2 + reg] = (uint32_t)h0 | ((uint32_t)h1 << 16);
            bsm[(((size_t)kb * PARTS + 1) * 4 + q) * 2 + reg] = (uint32_t)m0 | ((uint32_t)m1 << 16);
            bsm[(((size_t)kb * PARTS + 2) * 4 + q) * 2 + reg] = (uint32_t)l0 | ((uint32_t)l1 << 16);
        }
    }
    __syncthreads();
    TRACE(2);

    // body: lane (n = lane / 4, q = lane % 4) feeds B column n (part n; zero past the three);
    // sub-blocks alternate between two accumulators to halve the MMA dependency chain
    const int n8 = lane >> 2, qd = lane & 3;
    float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
    int cur = -1;
    long kf = -1;
    // (tile-row, k-tile) of the warp's next tile, advanced per tile (a 64-bit division per
    // tile would cost more than the tile's multiply)
    int wtr = (int)(wa / a.nkt), wkt = (int)(wa % a.nkt);
    // row r of the tile-row = columns 0 + 1 (lane q = 0) + column 2 (lane q = 1)
    auto flush = [&](int ltr) {
        const float a0 = acc0[0] + acc1[0], a1 = acc0[1] + acc1[1];
        const float a2 = acc0[2] + acc1[2], a3 = acc0[3] + acc1[3];
        const float p0 = __shfl_xor_sync(0xffffffffu, a0, 1);
        const float p2 = __shfl_xor_sync(0xffffffffu, a2, 1);
        if (qd == 0) {
            float *ps = psm + ((size_t)warp * MAX_LOCAL + ltr) * 16;
            ps[n8] = (a0 + a1) + p0;
            ps[n8 + 8] = (a2 + a3) + p2;
        }
    };
    for (long j = 0; j < nch; ++j) {
        const int s = (int)(j % STAGES);
        if (!mbar_wait(&bars[warp][s], (unsigned)((j / STAGES) & 1), a.status)) {
            kf = j;
            break;
        }
        if (j < 4) TRACE(3 + j);
        const long t0 = wa + j * CH;
        const int n = (int)((wb - t0 < CH) ? wb - t0 : CH);
        const uint8_t *st = ring + (size_t)s * CH * DENSE_TILE + lane * 16;
        for (int i = 0; i < n; ++i) {
            const int ltr = wtr - tr0, kt = wkt;
            if (++wkt == a.nkt) {
                wkt = 0;
                ++wtr;
            }
            if (ltr != cur) {
                if (cur >= 0) flush(cur);
                cur = ltr;
#pragma unroll
                for (int e = 0; e < 4; ++e) acc0[e] = acc1[e] = 0.f;
            }
            const uint8_t *tile = st + (size_t)i * DENSE_TILE;
            uint4 av[4];
            uint2 bv[4];
#pragma unroll
            for (int sb = 0; sb < 4; ++sb) {
                av[sb] = *reinterpret_cast<const uint4 *>(tile + sb * 512);
                bv[sb] = make_uint2(0u, 0u);
                if (n8 < PARTS)
                    bv[sb] = *reinterpret_cast<const uint2 *>(bsm + (((size_t)(kt * 4 + sb) * PARTS + n8) * 4 + qd) * 2);
            }
            mma_bf16(acc0, av[0], bv[0].x, bv[0].y);
            mma_bf16(acc1, av[1], bv[1].x, bv[1].y);
            mma_bf16(acc0, av[2], bv[2].x, bv[2].y);
            mma_bf16(acc1, av[3], bv[3].x, bv[3].y);
        }
        __syncwarp();
        if (issued < nch) {
            if (lane == 0) issue(issued, s);
            ++issued;
        }
    }
    if (kf >= 0) {
        // a copy did not complete in time: no bulk copy may still land in this warp's ring
        // when the CTA exits, so wait (bounded) for every one issued, then skip the epilogue
        for (long j = kf; j < issued; ++j) mbar_wait(&bars[warp][j % STAGES], (unsigned)((j / STAGES) & 1), a.status);
    } else if (cur >= 0) {
        flush(cur);
    }
    if (__syncthreads_or(kf >= 0)) return;
    TRACE(8);

    // the CTA's partial of every tile-row it touched: its warps summed in order
    const int n_local = tr1 - tr0 + 1;
    for (int e = threadIdx.x; e < n_local * 16; e += WARPS * 32) {
        const int ltr = e >> 4, row = e & 15;
        float s = 0.f;
        for (int w = 0; w < WARPS; ++w) s += psm[((size_t)w * MAX_LOCAL + ltr) * 16 + row];
        const int tr = tr0 + ltr;
        const int slot = cta - cta_of(a.T, G, (long)tr * a.nkt);
        st_part(a.part + ((size_t)tr * a.maxc + slot) * 16 + row, s);
    }
    __syncthreads();
    TRACE(9);
    // The unit's finisher is the CTA holding its first tile: warp i takes the i-th unit touched
    // when this CTA is that one, and polls every contributor's partial slot (bounded), with no
    // fence or arrival count between the last partial and the unit's result.
    if (warp > u1 - u0) return;
    const int unit = u0 + warp;
    if (cta_of(a.T, G, (long)unit * a.unit_trs * a.nkt) != cta) return;
    // a row's contributors summed in CTA order; each slot is taken once stored, then emptied
    auto row_value = [&](int row) {
        const int tr = row >> 4;
        const int c0 = cta_of(a.T, G, (long)tr * a.nkt), c1 = cta_of(a.T, G, (long)(tr + 1) * a.nkt - 1);
        const int nc = c1 - c0 + 1;
        float *pp = a.part + (size_t)tr * a.maxc * 16 + (row & 15);
        static_assert(MAX_CONTRIB == 4, "four slots below");
        uint32_t v0 = 0, v1 = 0, v2 = 0, v3 = 0;
        unsigned long long t0 = 0;
        for (;;) {
            v0 = ld_part(pp);
            v1 = nc > 1 ? ld_part(pp + 16) : 0u;
            v2 = nc > 2 ? ld_part(pp + 32) : 0u;
            v3 = nc > 3 ? ld_part(pp + 48) : 0u;
            if (v0 != PART_EMPTY && v1 != PART_EMPTY && v2 != PART_EMPTY && v3 != PART_EMPTY) break;
            const unsigned long long now = xnow();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > XPOLL_NS) {
                atomicOr(a.status, STATUS_WAIT_TIMEOUT);  // the step's output is then invalid
                break;
            }
        }
        const float e = __uint_as_float(PART_EMPTY);
        float s = __uint_as_float(v0);
        st_part(pp, e);
        if (nc > 1) {
            s += __uint_as_float(v1);
            st_part(pp + 16, e);
        }
        if (nc > 2) {
            s += __uint_as_float(v2);
            st_part(pp + 32, e);
        }
        if (nc > 3) {
            s += __uint_as_float(v3);
            st_part(pp + 48, e);
        }
        return s;
    };
    if (a.mode == 1) {
        for (int rr = lane; rr < a.unit_trs * 16; rr += 32) {
            const int row = unit * a.unit_trs * 16 + rr;
            const float s = row_value(row);
            a.out[row] = a.residual ? a.residual[row] + s : s;
        }
        return;
    }
    // Q/K/V head complete: unit < n_q_heads is a query head, then the K heads, then V.
    const int D = a.rope.head_dim;
    const int per = D / 32;  // values per lane: d = lane + 32 i
    const int row0 = unit * D;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = (i < per) ? row_value(row0 + lane + 32 * i) : 0.f;
    const int hq = a.rope.n_q_heads, hk = a.rope.n_kv_heads;
    if (unit < hq + hk && a.rope.q_norm) {
        // QK-norm: the head's mean square over its D values (a fixed butterfly), then the
        // reference's (x * scale) * w
        const float *w = unit < hq ? a.rope.q_norm : a.rope.k_norm;
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (i < per) ss = fmaf(v[i], v[i], ss);
        ss = warp_sum(ss);
        const float sc = 1.0f / sqrtf(ss / (float)D + a.rope.norm_eps);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (i < per) v[i] = (v[i] * sc) * __ldg(w + lane + 32 * i);
    }
    if (unit < hq + hk) {
        // the rotations computed before the wait
        if (per == 2) {
            const double x0 = v[0], x1 = v[1];
            v[0] = (float)(x0 * rot_c[0] - x1 * rot_s[0]);
            v[1] = (float)(x0 * rot_s[0] + x1 * rot_c[0]);
        } else {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const double x0 = v[i], x1 = v[i + 2];
                v[i] = (float)(x0 * rot_c[i] - x1 * rot_s[i]);
                v[i + 2] = (float)(x0 * rot_s[i] + x1 * rot_c[i]);
            }
        }
    }
    if (unit < hq) {
        for (int i = 0; i < per; ++i) a.out[(size_t)unit * D + lane + 32 * i] = v[i];
    } else {
        const int kvh = (unit < hq + hk) ? unit - hq : unit - hq - hk;
        uint16_t *pool = (unit < hq + hk) ? a.kv.k_pages : a.kv.v_pages;
        const int pt = a.kv.page_tokens;
        const size_t slot = pos % pt;
        uint16_t *dst = pool + ((page * pt + slot) * hk + kvh) * D;
        for (int i = 0; i < per; ++i) dst[lane + 32 * i] = bf(v[i]);
    }
    TRACE(31);
}

}  // namespace

TRACE_SETTER(dense)

struct dense_gemv {
    moearc_ctx *c;
    int n_rows, n_cols, mode;
    int ntr, nkt, grid, smem, maxc;
    long T;
    float *part;
    int *status;
    void *mem;
};

int dense_pack(moearc_ctx *c, void *dst, const void *src, int n_rows, int n_cols) {
    if (n_rows % 16 || n_cols % 64) return ERR_ARG;
    const size_t work = (size_t)(n_rows / 16) * (n_cols / 64) * 128;
    const unsigned g = (unsigned)std::min<size_t>((work + 255) / 256, (size_t)c->sm_count * 64);
    k_dense_pack<<<g, 256, 0, c->stream>>>(static_cast<uint8_t *>(dst), static_cast<const uint16_t *>(src), n_rows, n_cols);
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

// Units: mode 0 heads of head_dim rows (head_dim a multiple of 64, at most 128, from
// dense_run's rope), mode 1 single tile-rows.
dense_gemv *dense_create(moearc_ctx *c, int n_rows, int n_cols, int mode) {
    if (n_rows % 16 || n_cols % 64 || n_cols > MAX_COLS) return nullptr;
    auto *g = new dense_gemv();
    g->c = c;
    g->n_rows = n_rows;
    g->n_cols = n_cols;
    g->mode = mode;
    g->ntr = n_rows / 16;
    g->nkt = n_cols / 64;
    g->T = (long)g->ntr * g->nkt;
    // one CTA per SM with a few stages of tiles per warp; more CTAs only when a CTA's range
    // would touch more than MAX_LOCAL tile-rows (short rows)
    auto fits = [&](int grid) {
        for (int cta = 0; cta < grid; ++cta) {
            const long ta = tile_lo(g->T, grid, cta), tb = tile_lo(g->T, grid, cta + 1);
            if (tb <= ta || (tb - 1) / g->nkt - ta / g->nkt + 1 > MAX_LOCAL) return false;
        }
        return true;
    };
    int grid = (int)std::max(1L, std::min<long>(c->sm_count, g->T / (WARPS * CH)));
    while (!fits(grid) && grid < g->T) ++grid;
    if (!fits(grid)) {
        delete g;
        return nullptr;
    }
    g->grid = grid;
    int maxc = 1;
    for (int tr = 0; tr < g->ntr; ++tr)
        maxc = std::max(maxc, cta_of(g->T, grid, (long)(tr + 1) * g->nkt - 1) - cta_of(g->T, grid, (long)tr * g->nkt) + 1);
    if (maxc > MAX_CONTRIB) {
        delete g;
        return nullptr;
    }
    g->maxc = maxc;
    g->smem = RING_BYTES + (n_cols / 16) * PARTS * 32 + WARPS * MAX_LOCAL * 16 * 4;
    const size_t part_b = sizeof(float) * (size_t)g->ntr * maxc * 16;
    if (cudaMalloc(&g->mem, part_b + 256) != cudaSuccess) {
        cudaGetLastError();
        delete g;
        return nullptr;
    }
    g->part = static_cast<float *>(g->mem);
    g->status = reinterpret_cast<int *>(static_cast<uint8_t *>(g->mem) + part_b);
    cudaMemsetAsync(g->mem, 0, part_b + 256, c->stream);
    parts_empty(g->part, (size_t)g->ntr * maxc * 16, c->stream, c->sm_count);
    // The attribute is per kernel, shared by every plan: set it to the most any plan may use,
    // not to this plan's need.
    if (g->smem > 200 * 1024 ||
        set_smem(k_dense, 200 * 1024) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(g->mem);
        delete g;
        return nullptr;
    }
    return g;
}

int dense_status(dense_gemv *g) {
    int st = 0;
    if (cudaMemcpyAsync(&st, g->status, sizeof(int), cudaMemcpyDeviceToHost, g->c->stream) != cudaSuccess ||
        cudaStreamSynchronize(g->c->stream) != cudaSuccess)
        return ERR;
    if (st) {
        // a wait that gave up can leave partials stored and never taken: empty every slot
        cudaMemsetAsync(g->status, 0, sizeof(int), g->c->stream);
        parts_empty(g->part, (size_t)g->ntr * g->maxc * 16, g->c->stream, g->c->sm_count);
    }
    return st;
}

void dense_destroy(dense_gemv *g) {
    if (!g) return;
    cudaFree(g->mem);
    delete g;
}

int dense_run(dense_gemv *g, const void *w_packed, const float *in, const float *norm_w, float eps,
              float *out, const float *residual, const int *pos, const dense_rope *rope,
              const dense_kv *kv) {
    dense_args a{};
    a.w = static_cast<const uint8_t *>(w_packed);
    a.n_rows = g->n_rows;
    a.n_cols = g->n_cols;
    a.ntr = g->ntr;
    a.nkt = g->nkt;
    a.T = g->T;
    a.mode = g->mode;
    a.maxc = g->maxc;
    a.unit_trs = 1;
    if (g->mode == 0) {
        if (!rope || !kv || rope->head_dim % 64 != 0 || rope->head_dim > 128 ||
            g->n_rows != (rope->n_q_heads + 2 * rope->n_kv_heads) * rope->head_dim)
            return ERR_ARG;
        a.unit_trs = rope->head_dim / 16;
    }
    a.in = in;
    a.norm_w = norm_w;
    a.eps = eps;
    a.out = out;
    a.residual = residual;
    a.pos = pos;
    if (rope) a.rope = *rope;
    if (kv) a.kv = *kv;
    a.part = g->part;
    a.status = g->status;
    return launch_pdl(k_dense, dim3(g->grid), dim3(WARPS * 32), (size_t)g->smem, g->c->stream, a) == cudaSuccess
               ? OK
               : ERR;
}

}  // namespace moearc
