// step.cu — the batch-1 decode step as one persistent cooperative kernel (see step.cuh).
#include <algorithm>
#include <cmath>
#include <vector>

#include "route.cuh"
#include "step.cuh"
#include "tma.cuh"

namespace moearc {

namespace {

constexpr int NW = 16;           // warps per CTA
constexpr int RS = 3;            // ring stages per warp
constexpr int SB = 4096;         // bytes per ring stage
constexpr int AW = 4;            // attention warps (0 .. AW-1); the O projection uses the others
constexpr int WSEG = 4;          // partial records a warp may hold in one phase
constexpr int DT = 2048;         // packed bf16 tile: 16 rows x 64 columns
constexpr int DCH = 2;           // dense tiles per stage
constexpr int HD = 64;           // head_dim
constexpr int TK = 16;           // keys per attention tile
constexpr int HMAX = 8;          // residual values per thread: n_embd <= 8 x 512
constexpr int MAXG = 8;          // query heads per KV head
constexpr int NPH = 6;           // traced phases: QKV, ATT, O, ROUTE, GU, DN
enum { R_QKV = 0, R_O = 1, R_RT = 2, R_GU = 3, R_DN = 4, R_END = 5 };  // ring phases of a block

struct step_args {
    const step_layer *L;
    int n_layer;
    int H, Dq, Dkv, n_head, n_kv, group;
    int E, K, I, gating, act;
    float alpha, limit, eps, scale;
    const double *rope_freq;
    double mscale;
    int q_ntr, q_nkt, o_ntr, o_nkt;
    long q_T, o_T;
    int q_maxc, o_maxc;
    int tile_bytes, pair_bytes, ch_gu, ch_dn;
    int gu_ntr, gu_nkt, dn_ntr, dn_nkt;
    size_t gu_stride, dn_stride;
    int max_splits;
    int xs_bytes;
    const float *in;
    float *out;
    const float *out_norm;
    int *pos;
    float *hbuf, *hmid, *qkv_part, *o_part, *att, *att_ml, *att_acc;
    unsigned *att_ctr;
    float *logits;
    uint32_t *actfrag;
    float *down_out;
    unsigned *route_idx;
    float *route_w;
    unsigned *sync;  // [0] barrier arrivals, [1] abort; zeroed before every launch
    int *status;
    unsigned long long limit_ns;
    unsigned phantom;
    unsigned long long *trace;
};

// ---- small device helpers -------------------------------------------------------------------

__device__ __forceinline__ unsigned ld_acq(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_rlx(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Generic-proxy writes of other CTAs (made visible here by the grid barrier) before this
// thread's later bulk copies read them.
__device__ __forceinline__ void fence_proxy_all() { asm volatile("fence.proxy.async;\n" ::: "memory"); }
__device__ __forceinline__ void bar_att() { asm volatile("bar.sync 1, %0;" ::"n"(AW * 32) : "memory"); }

// The CTA (of G) whose share [T c / G, T (c + 1) / G) holds item t.
__host__ __device__ __forceinline__ int owner_of(long T, int G, long t) { return (int)(((t + 1) * G - 1) / T); }

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16r(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One packed expert tile (16 rows x 64 columns, two quantisation blocks) against the
// activation's B registers for that k-tile: acc[0..1] row r, acc[2..3] row r + 8 (columns 0
// and 1 of the MMA carry the activation's f16 rounding and its residual).
template <int WT>
__device__ __forceinline__ void etile(const uint8_t *tile, int lane, const uint32_t (&b)[2][4], float (&acc)[4]) {
    const uint4 w = *reinterpret_cast<const uint4 *>(tile + lane * 16);
    float s[4];
    scales4<WT>(tile, lane >> 2, s);
    uint32_t q[4][4];
    decode4<WT>(w.x, q[0]);
    decode4<WT>(w.y, q[1]);
    decode4<WT>(w.z, q[2]);
    decode4<WT>(w.w, q[3]);
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t(&ar)[4] = q[2 * blk];
        const uint32_t(&br)[4] = q[2 * blk + 1];
        mma_f16(d, ar[0], br[0], ar[1], br[1], b[blk][0], b[blk][1]);
        mma_f16(d, ar[2], br[2], ar[3], br[3], b[blk][2], b[blk][3]);
        acc[0] = fmaf(d[0], s[blk * 2], acc[0]);
        acc[1] = fmaf(d[1], s[blk * 2], acc[1]);
        acc[2] = fmaf(d[2], s[blk * 2 + 1], acc[2]);
        acc[3] = fmaf(d[3], s[blk * 2 + 1], acc[3]);
    }
}

// B registers of one k-tile from expert-activation fragments laid [block][part][q][4 x u32]
// (part 0 the f16 rounding, 1 the residual): lane n = lane / 4 < 2 feeds column n, the others 0.
__device__ __forceinline__ void eload_b(const uint8_t *frag, int kt, int lane, uint32_t (&b)[2][4]) {
    const int n = lane >> 2, q = lane & 3;
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (n < 2) v = *reinterpret_cast<const uint4 *>(frag + (((2 * kt + blk) * 2 + n) * 4 + q) * 16);
        b[blk][0] = v.x;
        b[blk][1] = v.y;
        b[blk][2] = v.z;
        b[blk][3] = v.w;
    }
}

// Element i of a dense input as its three bf16 parts (rounding and two residuals) into the
// packed B-fragment buffer [16-column block][part][q][reg] of u32 pairs.
__device__ __forceinline__ void dense_frag_put(uint16_t *xs16, int i, float v) {
    const uint16_t h = f32_to_bf16_bits(v);
    float r = v - bf16_bits_to_f32(h);
    const uint16_t m = f32_to_bf16_bits(r);
    r -= bf16_bits_to_f32(m);
    const uint16_t lo = f32_to_bf16_bits(r);
    const int kb = i >> 4, cc = i & 15, reg = cc >> 3, q = (cc & 7) >> 1, half = cc & 1;
    const int base = ((kb * 3) * 4 + q) * 2 + reg;  // u32 index of part 0
    xs16[2 * base + half] = h;
    xs16[2 * (base + 8) + half] = m;
    xs16[2 * (base + 16) + half] = lo;
}

// Element i of an expert input as (f16 rounding, f16 residual) into [block][part][q][4 x u32].
__device__ __forceinline__ void expert_frag_put(uint16_t *f16buf, int i, float v) {
    const __half hh = __float2half_rn(v);
    const __half hl = __float2half_rn(v - __half2float(hh));
    const int blk = i >> 5, el = i & 31, q = (el & 15) >> 2, j = el & 3, half = el >> 4;
    const int u0 = ((blk * 2 + 0) * 4 + q) * 4 + j, u1 = ((blk * 2 + 1) * 4 + q) * 4 + j;
    f16buf[2 * u0 + half] = __half_as_ushort(hh);
    f16buf[2 * u1 + half] = __half_as_ushort(hl);
}

template <bool BF>
__device__ __forceinline__ uint16_t to16(float v) {
    if constexpr (BF) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
    else return __half_as_ushort(__float2half_rn(v));
}
__device__ __forceinline__ void split_bf16(float a, float b, uint32_t &hi, uint32_t &lo) {
    const uint16_t ah = to16<true>(a), bh = to16<true>(b);
    const uint16_t al = to16<true>(a - bf16_bits_to_f32(ah)), bl = to16<true>(b - bf16_bits_to_f32(bh));
    hi = (uint32_t)ah | ((uint32_t)bh << 16);
    lo = (uint32_t)al | ((uint32_t)bl << 16);
}
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(s));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(s));
}

constexpr float LOG2E = 1.4426950408889634f;

// ---- the kernel ----------------------------------------------------------------------------

template <int WT>
__global__ void __launch_bounds__(NW * 32, 1) k_step(const __grid_constant__ step_args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[NW][RS];
    __shared__ unsigned s_idx[8];
    __shared__ float s_wts[8];
    __shared__ float s_red[NW];
    __shared__ int s_rec_lo[NW], s_rec_n[NW];
    __shared__ int s_flag;
    __shared__ int s_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int c = blockIdx.x, G = gridDim.x;
    uint8_t *ring = smem + (size_t)warp * RS * SB;
    uint8_t *xs = smem + (size_t)NW * RS * SB;
    float *red = reinterpret_cast<float *>(xs + a.xs_bytes);  // [NW][WSEG][32]
    const int H = a.H;

    if (lane == 0) {
        for (int s = 0; s < RS; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    const int pos = *a.pos;

    // ---- this warp's item ranges (the same in every block) ----
    long rq_lo, rq_hi, ro_lo = 0, ro_hi = 0, rg_lo, rg_hi, rd_lo, rd_hi;
    {
        const long GW = (long)G * NW, gw = (long)c * NW + warp;
        rq_lo = a.q_T * gw / GW;
        rq_hi = a.q_T * (gw + 1) / GW;
        if (warp >= AW) {
            const long GWo = (long)G * (NW - AW), gwo = (long)c * (NW - AW) + (warp - AW);
            ro_lo = a.o_T * gwo / GWo;
            ro_hi = a.o_T * (gwo + 1) / GWo;
        }
        const long Sg = (long)a.K * a.gu_ntr, sg0 = Sg * c / G, sg1 = Sg * (c + 1) / G;
        const long Pg = (sg1 - sg0) * a.gu_nkt;
        rg_lo = sg0 * a.gu_nkt + Pg * warp / NW;
        rg_hi = sg0 * a.gu_nkt + Pg * (warp + 1) / NW;
        const long Sd = (long)a.K * a.dn_ntr, sd0 = Sd * c / G, sd1 = Sd * (c + 1) / G;
        const long Pd = (sd1 - sd0) * a.dn_nkt;
        rd_lo = sd0 * a.dn_nkt + Pd * warp / NW;
        rd_hi = sd0 * a.dn_nkt + Pd * (warp + 1) / NW;
    }
    const int n_rt = c < a.E ? (a.E - 1 - c) / G + 1 : 0;  // router rows c, c + G, ...

    // ---- the warp's ring: issue side ----
    long n_iss = 0, n_con = 0;        // pieces issued / consumed (warp-uniform)
    int att_done = -1, routed = -1, acts_ok = -1;
    int n_def = 0;                    // down pieces of the current block issued without their activations
    long dn_k0 = 0;                   // sequence number of the first of them
    struct cursor {
        int l, ph;
        long it, hi;
        bool done;
    } ic{0, R_QKV, rq_lo, rq_hi, a.n_layer == 0};
    auto range_of = [&](int ph, long &lo, long &hi) {
        switch (ph) {
        case R_QKV: lo = rq_lo; hi = rq_hi; break;
        case R_O: lo = ro_lo; hi = ro_hi; break;
        case R_RT: lo = 0; hi = n_rt; break;
        case R_GU: lo = rg_lo; hi = rg_hi; break;
        default: lo = rd_lo; hi = rd_hi; break;
        }
    };
    struct piece {
        const uint8_t *src, *asrc;
        unsigned bytes, abytes;
        int n;
    };
    auto describe = [&](int l, int ph, long it, long hi) {
        piece p{nullptr, nullptr, 0u, 0u, 1};
        const step_layer &Lb = a.L[l];
        if (ph == R_QKV || ph == R_O) {
            p.n = (int)min((long)DCH, hi - it);
            p.src = (ph == R_QKV ? Lb.wqkv : Lb.wo) + (size_t)it * DT;
            p.bytes = (unsigned)(p.n * DT);
        } else if (ph == R_RT) {
            const long e = c + (long)G * it;
            p.src = reinterpret_cast<const uint8_t *>(Lb.router + (size_t)e * H + (size_t)warp * (H / NW));
            p.bytes = (unsigned)(H / NW * 4);
        } else if (ph == R_GU) {
            const long seg = it / a.gu_nkt;
            const int kt = (int)(it - seg * a.gu_nkt);
            p.n = (int)min(min((long)a.ch_gu, (long)(a.gu_nkt - kt)), hi - it);
            const int m = (int)(seg / a.gu_ntr), tr = (int)(seg - (long)m * a.gu_ntr);
            p.src = Lb.gateup + (size_t)s_idx[m] * a.gu_stride + ((size_t)tr * a.gu_nkt + kt) * a.pair_bytes;
            p.bytes = (unsigned)(p.n * a.pair_bytes);
        } else {
            const long seg = it / a.dn_nkt;
            const int kt = (int)(it - seg * a.dn_nkt);
            p.n = (int)min(min((long)a.ch_dn, (long)(a.dn_nkt - kt)), hi - it);
            const int m = (int)(seg / a.dn_ntr), tr = (int)(seg - (long)m * a.dn_ntr);
            p.src = Lb.down + (size_t)s_idx[m] * a.dn_stride + ((size_t)tr * a.dn_nkt + kt) * a.tile_bytes;
            p.bytes = (unsigned)(p.n * a.tile_bytes);
            p.asrc = reinterpret_cast<const uint8_t *>(a.actfrag + (size_t)m * (a.I / 32) * 32 + (size_t)kt * 64);
            p.abytes = (unsigned)(p.n * 256);
        }
        return p;
    };
    auto can_issue = [&](int l, int ph) {
        if (ph == R_RT && warp < AW) return att_done >= l;  // warps 0-3 lend their ring to attention
        if (ph == R_GU || ph == R_DN) return routed >= l;    // expert addresses need the routing
        return true;
    };
    // Keep the ring full: issue pieces in sequence while a stage is free and the next piece's
    // addresses are known. A down piece issued before its block's activations exist gets them later.
    auto pump = [&]() {
        while (!ic.done && n_iss - n_con < RS) {
            if (ic.it >= ic.hi) {
                if (++ic.ph == R_END) {
                    ic.ph = R_QKV;
                    if (++ic.l == a.n_layer) {
                        ic.done = true;
                        break;
                    }
                }
                range_of(ic.ph, ic.it, ic.hi);
                continue;
            }
            if (!can_issue(ic.l, ic.ph)) break;
            const piece p = describe(ic.l, ic.ph, ic.it, ic.hi);
            const int stage = (int)(n_iss % RS);
            const bool with_acts = p.abytes && acts_ok >= ic.l;
            if (p.abytes && !with_acts) {
                if (n_def == 0) dn_k0 = n_iss;
                ++n_def;
            }
            if (lane == 0) {
                uint64_t *bar = &bars[warp][stage];
                uint8_t *st = ring + (size_t)stage * SB;
                fence_proxy_async();
                mbar_expect_tx(bar, p.bytes + p.abytes);
                bulk_g2s(st, p.src, p.bytes, bar);
                if (with_acts) bulk_g2s(st + p.bytes, p.asrc, p.abytes, bar);
            }
            ic.it += p.n;
            ++n_iss;
        }
        __syncwarp();
    };
    // The deferred activation copies of block l's first down pieces, once the activations exist.
    auto issue_deferred = [&](int l) {
        long it = rd_lo;
        for (int j = 0; j < n_def; ++j) {
            const piece p = describe(l, R_DN, it, rd_hi);
            const int stage = (int)((dn_k0 + j) % RS);
            if (lane == 0) bulk_g2s(ring + (size_t)stage * SB + p.bytes, p.asrc, p.abytes, &bars[warp][stage]);
            it += p.n;
        }
        n_def = 0;
        __syncwarp();
    };
    bool alive = true;  // no wait has given up in this CTA
    auto wait_piece = [&]() -> const uint8_t * {
        const int stage = (int)(n_con % RS);
        if (!mbar_wait(&bars[warp][stage], (unsigned)((n_con / RS) & 1), a.status)) {
            alive = false;
            if (lane == 0) atomicExch(a.sync + 1, 1u);
            return nullptr;
        }
        return ring + (size_t)stage * SB;
    };
    auto release = [&]() {
        __syncwarp();
        ++n_con;
        pump();
    };

    // ---- grid barrier: every CTA arrives, then waits (bounded) for all. False (the same in
    // every thread of the CTA) when a wait of this CTA or of another has given up. ----
    unsigned nbar = 0;
    auto gsync = [&]() -> bool {
        const bool all_alive = __syncthreads_and(alive);
        ++nbar;
        if (tid == 0 && !all_alive) {
            atomicExch(a.sync + 1, 1u);
            s_flag = 0;
        } else if (tid == 0) {
            __threadfence();
            atomicAdd(a.sync, 1u);
            const unsigned target = nbar * (unsigned)G + a.phantom;
            int ok = 1;
            unsigned long long t0 = 0;
            for (;;) {
                if (ld_acq(a.sync) >= target) break;
                if (ld_rlx(a.sync + 1)) {
                    ok = 0;
                    break;
                }
                const unsigned long long t = xnow();
                if (t0 == 0) {
                    t0 = t;
                } else if (t - t0 > a.limit_ns) {
                    atomicOr(a.status, STATUS_WAIT_TIMEOUT);
                    atomicExch(a.sync + 1, 1u);
                    ok = 0;
                    break;
                }
            }
            __threadfence();
            s_flag = ok;
        }
        __syncthreads();
        return s_flag != 0;
    };
    auto stamp = [&](int l, int ph, int end) {
        if (a.trace && tid == 0) a.trace[(((size_t)l * NPH + ph) * 2 + end) * G + c] = xnow();
    };

    // ---- per-warp partial records ----
    auto rec = [&](int w, int slot) { return red + ((size_t)w * WSEG + slot) * 32; };

    // A dense phase's share of this warp: tiles [lo, hi) of a matrix with nkt k-tiles a row,
    // against the B fragments in xs; per tile-row touched one record of 16 row sums.
    auto dense_consume = [&](long lo, long hi, int nkt) {
        int rec_lo = -1, nrec = 0, cur = -1;
        float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
        const int n8 = lane >> 2, qd = lane & 3;
        const uint32_t *bsm = reinterpret_cast<const uint32_t *>(xs);
        auto flush = [&]() {
            const float a0 = acc0[0] + acc1[0], a1 = acc0[1] + acc1[1];
            const float a2 = acc0[2] + acc1[2], a3 = acc0[3] + acc1[3];
            const float p0 = __shfl_xor_sync(0xffffffffu, a0, 1);
            const float p2 = __shfl_xor_sync(0xffffffffu, a2, 1);
            if (qd == 0) {
                float *r = rec(warp, cur - rec_lo);
                r[n8] = (a0 + a1) + p0;
                r[n8 + 8] = (a2 + a3) + p2;
            }
        };
        int tr = (int)(lo / nkt), kt = (int)(lo - (long)tr * nkt);
        for (long t = lo; t < hi && alive;) {
            const uint8_t *st = wait_piece();
            if (!st) break;
            const int n = (int)min((long)DCH, hi - t);
            for (int i = 0; i < n; ++i) {
                if (tr != cur) {
                    if (cur >= 0) flush();
                    if (rec_lo < 0) rec_lo = tr;
                    cur = tr;
                    nrec = cur - rec_lo + 1;
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc0[e] = acc1[e] = 0.f;
                }
                const uint8_t *tile = st + (size_t)i * DT + lane * 16;
                uint4 av[4];
                uint2 bv[4];
#pragma unroll
                for (int sb = 0; sb < 4; ++sb) {
                    av[sb] = *reinterpret_cast<const uint4 *>(tile + sb * 512);
                    bv[sb] = make_uint2(0u, 0u);
                    if (n8 < 3) bv[sb] = *reinterpret_cast<const uint2 *>(bsm + (((kt * 4 + sb) * 3 + n8) * 4 + qd) * 2);
                }
                mma_bf16(acc0, av[0], bv[0].x, bv[0].y);
                mma_bf16(acc1, av[1], bv[1].x, bv[1].y);
                mma_bf16(acc0, av[2], bv[2].x, bv[2].y);
                mma_bf16(acc1, av[3], bv[3].x, bv[3].y);
                if (++kt == nkt) {
                    kt = 0;
                    ++tr;
                }
            }
            t += n;
            release();
        }
        if (cur >= 0) flush();
        if (lane == 0) {
            s_rec_lo[warp] = rec_lo;
            s_rec_n[warp] = nrec;
        }
    };
    // After dense_consume in every warp: the CTA's partial of each tile-row it touched, its
    // warps summed in order, into part[tile-row][contributor][16].
    auto dense_reduce = [&](long T, int nkt, int maxc, float *part) {
        __syncthreads();
        const long ta = T * c / G, tb = T * (c + 1) / G;
        if (tb <= ta) return;
        const int tr0 = (int)(ta / nkt), tr1 = (int)((tb - 1) / nkt);
        for (int e = tid; e < (tr1 - tr0 + 1) * 16; e += NW * 32) {
            const int tr = tr0 + (e >> 4), r = e & 15;
            float s = 0.f;
            for (int w = 0; w < NW; ++w) {
                const int k = tr - s_rec_lo[w];
                if (s_rec_n[w] > 0 && k >= 0 && k < s_rec_n[w]) s += rec(w, k)[r];
            }
            const int slot = c - owner_of(T, G, (long)tr * nkt);
            part[((size_t)tr * maxc + slot) * 16 + r] = s;
        }
    };
    // Row `row` of a dense phase's output: its contributors' partials summed in CTA order.
    auto dense_row = [&](long T, int nkt, int maxc, const float *part, int row) {
        const int tr = row >> 4;
        const int c0 = owner_of(T, G, (long)tr * nkt), c1 = owner_of(T, G, (long)(tr + 1) * nkt - 1);
        float s = 0.f;
        for (int k = 0; k <= c1 - c0; ++k) s += __ldcg(part + ((size_t)tr * maxc + k) * 16 + (row & 15));
        return s;
    };
    auto block_sum = [&](float v) {
        v = warp_sum(v);
        if (lane == 0) s_red[warp] = v;
        __syncthreads();
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) t += s_red[w];
        __syncthreads();
        return t;
    };
    // h entering block l: the input, or the previous block's residual plus its router-order combine.
    auto residual_in = [&](int l, int i) {
        if (l == 0) return __ldcg(a.in + i);
        float acc = 0.f;
        for (int m = 0; m < a.K; ++m) acc = fmaf(s_wts[m], __ldcg(a.down_out + (size_t)m * H + i), acc);
        return __ldcg(a.hmid + i) + acc;
    };

    pump();  // the first block's Q/K/V weights start streaming now

    bool synced = true;  // every grid barrier so far opened (uniform across the CTA)
    for (int l = 0; l < a.n_layer; ++l) {
        const step_layer &Lb = a.L[l];
        // ================= QKV =================
        if (l > 0 && !(synced = gsync())) break;
        stamp(l, 0, 0);
        {
            float hv[HMAX];
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < HMAX; ++j) {
                const int i = tid + j * NW * 32;
                hv[j] = 0.f;
                if (i < H) {
                    hv[j] = residual_in(l, i);
                    ss = fmaf(hv[j], hv[j], ss);
                }
            }
            const float scale = 1.0f / sqrtf(block_sum(ss) / (float)H + a.eps);
            const int h0 = (int)((long)H * c / G), h1 = (int)((long)H * (c + 1) / G);
            uint16_t *xs16 = reinterpret_cast<uint16_t *>(xs);
#pragma unroll
            for (int j = 0; j < HMAX; ++j) {
                const int i = tid + j * NW * 32;
                if (i < H) {
                    if (i >= h0 && i < h1) a.hbuf[i] = hv[j];
                    dense_frag_put(xs16, i, (hv[j] * scale) * __ldg(Lb.attn_norm + i));
                }
            }
            __syncthreads();
        }
        dense_consume(rq_lo, rq_hi, a.q_nkt);
        dense_reduce(a.q_T, a.q_nkt, a.q_maxc, a.qkv_part);
        stamp(l, 0, 1);
        // ================= ATT =================
        if (!(synced = gsync())) break;
        stamp(l, 1, 0);
        {
            const size_t n_tok = (size_t)pos + 1;
            const size_t kv_begin = (Lb.window > 0 && n_tok > (size_t)Lb.window) ? n_tok - (size_t)Lb.window : 0;
            const size_t span = n_tok - kv_begin;
            size_t kps = (span + a.max_splits - 1) / a.max_splits;
            kps = ((kps + 255) / 256) * 256;
            const int n_splits = (int)((span + kps - 1) / kps);
            const bool unit = c < a.n_kv * n_splits;
            if (warp < AW && unit) {
                const int kvh = c / n_splits, split = c - kvh * n_splits;
                const int group = a.group;
                const size_t s0 = kv_begin + (size_t)split * kps, s1 = min(s0 + kps, n_tok);
                const bool last = split == n_splits - 1;
                float *qf = red;             // [group][64] f32
                float *kf = red + MAXG * HD; // [64]
                float *vf = kf + HD;         // [64]
                const int t = tid;           // 0 .. 127
                // q (every split) and, for the split holding the step's token, k and v: rows of
                // the Q/K/V output, RoPE (NeoX pairs d, d + 32) on q and k
                const int n_pairs = group * 32 + (last ? 32 : 0);
                for (int i = t; i < n_pairs; i += AW * 32) {
                    const int hs = i >> 5, p = i & 31;
                    const int row0 = hs < group ? (kvh * group + hs) * HD : a.Dq + kvh * HD;
                    const double x0 = dense_row(a.q_T, a.q_nkt, a.q_maxc, a.qkv_part, row0 + p);
                    const double x1 = dense_row(a.q_T, a.q_nkt, a.q_maxc, a.qkv_part, row0 + p + 32);
                    const double th = (double)pos * __ldg(a.rope_freq + p);
                    const double k2 = rint(th * 0.15915494309189535);
                    double r = fma(-k2, 6.283185307179586, th);
                    r = fma(-k2, 2.4492935982947064e-16, r);
                    double sn, cs;
                    sincos(r, &sn, &cs);
                    cs *= a.mscale;
                    sn *= a.mscale;
                    float *dst = hs < group ? qf + hs * HD : kf;
                    dst[p] = (float)(x0 * cs - x1 * sn);
                    dst[p + 32] = (float)(x0 * sn + x1 * cs);
                }
                if (last)
                    for (int i = t; i < HD; i += AW * 32)
                        vf[i] = dense_row(a.q_T, a.q_nkt, a.q_maxc, a.qkv_part, a.Dq + a.Dkv + kvh * HD + i);
                bar_att();
                if (last) {
                    const size_t page = Lb.table[pos / 32];
                    const size_t off = ((page * 32 + (size_t)(pos % 32)) * a.n_kv + kvh) * HD;
                    for (int i = t; i < HD; i += AW * 32) {
                        Lb.k_pages[off + i] = f32_to_bf16_bits(kf[i]);
                        Lb.v_pages[off + i] = f32_to_bf16_bits(vf[i]);
                    }
                    __threadfence();
                }
                bar_att();
                // flash decode over [s0, s1): warp w takes tiles s0 + 16 w, + 64, ...; its ring
                // holds two stages of K and V tiles (16 keys x 64, rows swizzled in 16-byte chunks)
                const int qd = lane & 3, hr = lane >> 2;
                uint16_t *ws = reinterpret_cast<uint16_t *>(ring);
                uint32_t qa[HD / 16][4];
                {
                    const bool live = hr < group;
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk) {
                        const int c0 = 16 * kk + 2 * qd, c1 = c0 + 8;
                        const float *qh = qf + (live ? hr : 0) * HD;
                        split_bf16(live ? qh[c0] : 0.f, live ? qh[c0 + 1] : 0.f, qa[kk][0], qa[kk][1]);
                        split_bf16(live ? qh[c1] : 0.f, live ? qh[c1 + 1] : 0.f, qa[kk][2], qa[kk][3]);
                    }
                }
                float o[HD / 8][4];
#pragma unroll
                for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
                float m = -INFINITY, lsum = 0.f;
                const size_t row_elems = (size_t)a.n_kv * HD;
                constexpr int CH = HD / 8;
                auto load_tile = [&](size_t t0, int stg) {
                    uint16_t *kt = ws + stg * 2 * TK * HD, *vt = kt + TK * HD;
#pragma unroll
                    for (int cc = lane; cc < TK * CH; cc += 32) {
                        const int r = cc / CH, ch = cc % CH;
                        const size_t j = t0 + r;
                        const bool valid = j < s1;
                        const size_t jj = valid ? j : s0;
                        const size_t off = ((size_t)Lb.table[jj / 32] * 32 + jj % 32) * row_elems + (size_t)kvh * HD + ch * 8;
                        const int dst = r * HD + ((ch ^ (r & 7)) * 8);
                        cp_async16(kt + dst, Lb.k_pages + off, valid);
                        cp_async16(vt + dst, Lb.v_pages + off, valid);
                    }
                };
                size_t t0 = s0 + (size_t)warp * TK;
                int stg = 0;
                if (t0 < s1) load_tile(t0, 0);
                cp_async_commit();
                for (; t0 < s1; t0 += AW * TK) {
                    const size_t tn = t0 + AW * TK;
                    if (tn < s1) load_tile(tn, stg ^ 1);
                    cp_async_commit();
                    cp_async_wait<1>();
                    __syncwarp();
                    const uint16_t *kt = ws + stg * 2 * TK * HD, *vt = kt + TK * HD;
                    float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk) {
                        const int mi = lane >> 3, r = ((mi >> 1) << 3) | (lane & 7);
                        const int ch = 2 * kk + (mi & 1);
                        uint32_t b[4];
                        ldsm_x4(b, kt + r * HD + ((ch ^ (r & 7)) * 8));
                        mma_bf16r(sacc[0], qa[kk], b[0], b[1]);
                        mma_bf16r(sacc[1], qa[kk], b[2], b[3]);
                    }
                    float sc[4];
#pragma unroll
                    for (int nn = 0; nn < 2; ++nn)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const size_t j = t0 + 8 * nn + 2 * qd + e;
                            const float v = (sacc[nn][e] + sacc[nn][e + 2]) * a.scale;
                            sc[2 * nn + e] = j < s1 ? v : -INFINITY;
                        }
                    float mt = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
                    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
                    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
                    const float mn = fmaxf(m, mt);
                    const float corr = (mn == -INFINITY) ? 1.f : exp2f((m - mn) * LOG2E);
                    float p[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) p[e] = (sc[e] == -INFINITY) ? 0.f : exp2f((sc[e] - mn) * LOG2E);
                    lsum = lsum * corr + (p[0] + p[1]) + (p[2] + p[3]);
                    m = mn;
#pragma unroll
                    for (int i = 0; i < HD / 8; ++i) {
                        o[i][0] *= corr;
                        o[i][1] *= corr;
                        o[i][2] *= corr;
                        o[i][3] *= corr;
                    }
                    uint32_t pa[4];
                    split_bf16(p[0], p[1], pa[0], pa[1]);
                    split_bf16(p[2], p[3], pa[2], pa[3]);
#pragma unroll
                    for (int dn = 0; dn < HD / 16; ++dn) {
                        const int mi = lane >> 3, r = ((mi & 1) << 3) | (lane & 7);
                        const int ch = 2 * dn + (mi >> 1);
                        uint32_t b[4];
                        ldsm_x4_t(b, vt + r * HD + ((ch ^ (r & 7)) * 8));
                        mma_bf16r(o[2 * dn], pa, b[0], b[1]);
                        mma_bf16r(o[2 * dn + 1], pa, b[2], b[3]);
                    }
                    __syncwarp();
                    stg ^= 1;
                }
                cp_async_wait<0>();
                lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
                lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
                // the four warps merged through the first two warps' rings (tiles done with)
                bar_att();
                float *fm = reinterpret_cast<float *>(smem);  // [AW][8] m, [AW][8] l, [AW][8][HD] acc
                float *fl = fm + AW * 8, *fo = fm + 2 * AW * 8;
                if (qd == 0) {
                    fm[warp * 8 + hr] = m;
                    fl[warp * 8 + hr] = lsum;
                }
#pragma unroll
                for (int i = 0; i < HD / 8; ++i) {
                    const int d = 8 * i + 2 * qd;
                    fo[(warp * 8 + hr) * HD + d] = o[i][0] + o[i][2];
                    fo[(warp * 8 + hr) * HD + d + 1] = o[i][1] + o[i][3];
                }
                bar_att();
                for (int e = t; e < group * HD; e += AW * 32) {
                    const int h = e / HD, d = e % HD;
                    float M = -INFINITY;
                    for (int w = 0; w < AW; ++w) M = fmaxf(M, fm[w * 8 + h]);
                    float Lsum = 0.f, v = 0.f;
                    for (int w = 0; w < AW; ++w) {
                        const float mw = fm[w * 8 + h];
                        if (mw == -INFINITY) continue;
                        const float f = exp2f((mw - M) * LOG2E);
                        Lsum += fl[w * 8 + h] * f;
                        v += fo[(w * 8 + h) * HD + d] * f;
                    }
                    const int hq = kvh * group + h;
                    if (n_splits == 1) {
                        float fs = 1.f;
                        if (Lb.sinks) {
                            const float sk = __ldg(Lb.sinks + hq);
                            const float Mf = fmaxf(M, sk);
                            fs = (M == -INFINITY) ? 0.f : exp2f((M - Mf) * LOG2E);
                            Lsum = Lsum * fs + exp2f((sk - Mf) * LOG2E);
                        }
                        a.att[(size_t)hq * HD + d] = v * fs / Lsum;
                    } else {
                        if (d == 0) {
                            a.att_ml[((size_t)hq * n_splits + split) * 2] = M;
                            a.att_ml[((size_t)hq * n_splits + split) * 2 + 1] = Lsum;
                        }
                        a.att_acc[((size_t)hq * n_splits + split) * HD + d] = v;
                    }
                }
                if (n_splits > 1) {
                    // the last split of this KV head to arrive merges all of them (the sink joins
                    // as one more logit with no value) and re-arms the counter
                    fence_acq_rel_gpu();
                    bar_att();
                    if (t == 0) s_last = atomicAdd(a.att_ctr + kvh, 1u) == (unsigned)n_splits - 1;
                    bar_att();
                    if (s_last) {
                        fence_acq_rel_gpu();
                        for (int e = t; e < group * HD; e += AW * 32) {
                            const int h = e / HD, d = e % HD, hq = kvh * group + h;
                            const float *ml = a.att_ml + (size_t)hq * n_splits * 2;
                            float M = Lb.sinks ? __ldg(Lb.sinks + hq) : -INFINITY;
                            for (int sp = 0; sp < n_splits; ++sp) M = fmaxf(M, __ldcg(ml + 2 * sp));
                            float Lsum = Lb.sinks ? exp2f((__ldg(Lb.sinks + hq) - M) * LOG2E) : 0.f, v = 0.f;
                            for (int sp = 0; sp < n_splits; ++sp) {
                                const float ms = __ldcg(ml + 2 * sp);
                                if (ms == -INFINITY) continue;
                                const float f = exp2f((ms - M) * LOG2E);
                                Lsum += __ldcg(ml + 2 * sp + 1) * f;
                                v += __ldcg(a.att_acc + ((size_t)hq * n_splits + sp) * HD + d) * f;
                            }
                            a.att[(size_t)hq * HD + d] = v / Lsum;
                        }
                        if (t == 0) a.att_ctr[kvh] = 0;
                    }
                }
                bar_att();  // the rings are free again
            }
            if (warp < AW) {
                att_done = l;
                pump();
            }
        }
        stamp(l, 1, 1);
        // ================= O =================
        if (!(synced = gsync())) break;
        stamp(l, 2, 0);
        {
            uint16_t *xs16 = reinterpret_cast<uint16_t *>(xs);
            for (int i = tid; i < a.Dq; i += NW * 32) dense_frag_put(xs16, i, __ldcg(a.att + i));
            __syncthreads();
        }
        dense_consume(ro_lo, ro_hi, a.o_nkt);
        dense_reduce(a.o_T, a.o_nkt, a.o_maxc, a.o_part);
        stamp(l, 2, 1);
        // ================= ROUTE =================
        if (!(synced = gsync())) break;
        stamp(l, 3, 0);
        float *xf = reinterpret_cast<float *>(xs);                 // [H] the MoE input, f32
        uint16_t *xg = reinterpret_cast<uint16_t *>(xs + 4 * H);   // its expert fragments
        {
            float hv[HMAX];
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < HMAX; ++j) {
                const int i = tid + j * NW * 32;
                hv[j] = 0.f;
                if (i < H) {
                    hv[j] = __ldcg(a.hbuf + i) + dense_row(a.o_T, a.o_nkt, a.o_maxc, a.o_part, i);
                    ss = fmaf(hv[j], hv[j], ss);
                }
            }
            const float scale = 1.0f / sqrtf(block_sum(ss) / (float)H + a.eps);
            const int h0 = (int)((long)H * c / G), h1 = (int)((long)H * (c + 1) / G);
#pragma unroll
            for (int j = 0; j < HMAX; ++j) {
                const int i = tid + j * NW * 32;
                if (i < H) {
                    if (i >= h0 && i < h1) a.hmid[i] = hv[j];
                    const float x = (hv[j] * scale) * __ldg(Lb.ffn_norm + i);
                    xf[i] = x;
                    expert_frag_put(xg, i, x);
                }
            }
            __syncthreads();
        }
        // router row c + G j, slice `warp` of it (H / 16 columns), one piece each
        for (int j = 0; j < n_rt && alive; ++j) {
            const uint8_t *st = wait_piece();
            if (!st) break;
            const float4 *w4 = reinterpret_cast<const float4 *>(st);
            const float4 *x4 = reinterpret_cast<const float4 *>(xf + warp * (H / NW));
            float acc = 0.f;
            for (int f = lane; f < H / (NW * 4); f += 32) {
                const float4 wv = w4[f], xv = x4[f];
                acc = fmaf(wv.x, xv.x, acc);
                acc = fmaf(wv.y, xv.y, acc);
                acc = fmaf(wv.z, xv.z, acc);
                acc = fmaf(wv.w, xv.w, acc);
            }
            acc = warp_sum(acc);
            if (lane == 0) rec(warp, 0)[j] = acc;  // j < 32 WSEG: checked at plan time
            release();
        }
        __syncthreads();
        for (int j = tid; j < n_rt; j += NW * 32) {
            float s = 0.f;
            for (int w = 0; w < NW; ++w) s += rec(w, 0)[j];
            a.logits[c + (size_t)G * j] = s;
        }
        stamp(l, 3, 1);
        // ================= GU =================
        if (!(synced = gsync())) break;
        stamp(l, 4, 0);
        if (warp == 0) {
            xtopk(a.logits, a.E, a.K, a.gating, lane, s_idx, s_wts);
            __syncwarp();
            // an id out of range (NaN logits, outside the router's contract) reads expert 0
            // rather than memory past the bank, and is reported
            if (lane < a.K && s_idx[lane] >= (unsigned)a.E) {
                s_idx[lane] = 0;
                atomicOr(a.status, STATUS_RANGE);
            }
            __syncwarp();
            if (c == 0 && lane < a.K) {
                a.route_idx[(size_t)l * a.K + lane] = s_idx[lane];
                a.route_w[(size_t)l * a.K + lane] = s_wts[lane];
            }
        }
        __syncthreads();
        routed = l;
        pump();
        {
            // pairs [rg_lo, rg_hi): (gate, up) tiles of segment (expert m, tile-row tr)
            int rec_lo = -1, nrec = 0;
            long cur = -1;
            float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
            const int r = lane >> 2, qd = lane & 3;
            auto flush = [&]() {
                if (qd == 0) {
                    float *p = rec(warp, (int)(cur - rec_lo));
                    p[r] = ag[0] + ag[1];
                    p[r + 8] = ag[2] + ag[3];
                    p[16 + r] = au[0] + au[1];
                    p[16 + r + 8] = au[2] + au[3];
                }
            };
            long seg = rg_lo / a.gu_nkt;
            int kt = (int)(rg_lo - seg * a.gu_nkt);
            for (long it = rg_lo; it < rg_hi && alive;) {
                const uint8_t *st = wait_piece();
                if (!st) break;
                const int n = (int)min(min((long)a.ch_gu, (long)(a.gu_nkt - kt)), rg_hi - it);
                if (seg != cur) {
                    if (cur >= 0) flush();
                    if (rec_lo < 0) rec_lo = (int)seg;
                    cur = seg;
                    nrec = (int)(cur - rec_lo) + 1;
#pragma unroll
                    for (int e = 0; e < 4; ++e) ag[e] = au[e] = 0.f;
                }
                for (int i = 0; i < n; ++i) {
                    uint32_t b[2][4];
                    eload_b(reinterpret_cast<const uint8_t *>(xg), kt + i, lane, b);
                    const uint8_t *pr = st + (size_t)i * a.pair_bytes;
                    etile<WT>(pr, lane, b, ag);
                    etile<WT>(pr + a.tile_bytes, lane, b, au);
                }
                it += n;
                kt += n;
                if (kt == a.gu_nkt) {
                    kt = 0;
                    ++seg;
                }
                release();
            }
            if (cur >= 0) flush();
            if (lane == 0) {
                s_rec_lo[warp] = rec_lo;
                s_rec_n[warp] = nrec;
            }
            __syncthreads();
            // the CTA's segments: gate and up summed over warps in order, the activation, its
            // fragments for the down phase
            const long Sg = (long)a.K * a.gu_ntr, sg0 = Sg * c / G, sg1 = Sg * (c + 1) / G;
            uint16_t *af = reinterpret_cast<uint16_t *>(a.actfrag);
            for (int e = tid; e < (int)(sg1 - sg0) * 16; e += NW * 32) {
                const long sg = sg0 + (e >> 4);
                const int rr = e & 15;
                float g = 0.f, u = 0.f;
                for (int w = 0; w < NW; ++w) {
                    const long k = sg - s_rec_lo[w];
                    if (s_rec_n[w] > 0 && k >= 0 && k < s_rec_n[w]) {
                        g += rec(w, (int)k)[rr];
                        u += rec(w, (int)k)[16 + rr];
                    }
                }
                const int m = (int)(sg / a.gu_ntr), tr = (int)(sg - (long)m * a.gu_ntr);
                expert_frag_put(af + (size_t)m * a.I * 2, tr * 16 + rr, act_fn(a.act, g, u, a.alpha, a.limit));
            }
        }
        stamp(l, 4, 1);
        // ================= DN =================
        if (!(synced = gsync())) break;
        stamp(l, 5, 0);
        acts_ok = l;
        if (lane == 0) fence_proxy_all();
        __syncwarp();
        issue_deferred(l);
        pump();
        {
            int rec_lo = -1, nrec = 0;
            long cur = -1;
            float ac[4] = {0.f, 0.f, 0.f, 0.f};
            const int r = lane >> 2, qd = lane & 3;
            auto flush = [&]() {
                if (qd == 0) {
                    float *p = rec(warp, (int)(cur - rec_lo));
                    p[r] = ac[0] + ac[1];
                    p[r + 8] = ac[2] + ac[3];
                }
            };
            long seg = rd_lo / a.dn_nkt;
            int kt = (int)(rd_lo - seg * a.dn_nkt);
            for (long it = rd_lo; it < rd_hi && alive;) {
                const uint8_t *st = wait_piece();
                if (!st) break;
                const int n = (int)min(min((long)a.ch_dn, (long)(a.dn_nkt - kt)), rd_hi - it);
                if (seg != cur) {
                    if (cur >= 0) flush();
                    if (rec_lo < 0) rec_lo = (int)seg;
                    cur = seg;
                    nrec = (int)(cur - rec_lo) + 1;
#pragma unroll
                    for (int e = 0; e < 4; ++e) ac[e] = 0.f;
                }
                const uint8_t *acts = st + (size_t)n * a.tile_bytes;
                for (int i = 0; i < n; ++i) {
                    uint32_t b[2][4];
                    eload_b(acts, i, lane, b);
                    etile<WT>(st + (size_t)i * a.tile_bytes, lane, b, ac);
                }
                it += n;
                kt += n;
                if (kt == a.dn_nkt) {
                    kt = 0;
                    ++seg;
                }
                release();
            }
            if (cur >= 0) flush();
            if (lane == 0) {
                s_rec_lo[warp] = rec_lo;
                s_rec_n[warp] = nrec;
            }
            __syncthreads();
            const long Sd = (long)a.K * a.dn_ntr, sd0 = Sd * c / G, sd1 = Sd * (c + 1) / G;
            for (int e = tid; e < (int)(sd1 - sd0) * 16; e += NW * 32) {
                const long sd = sd0 + (e >> 4);
                const int rr = e & 15;
                float s = 0.f;
                for (int w = 0; w < NW; ++w) {
                    const long k = sd - s_rec_lo[w];
                    if (s_rec_n[w] > 0 && k >= 0 && k < s_rec_n[w]) s += rec(w, (int)k)[rr];
                }
                const int m = (int)(sd / a.dn_ntr), tr = (int)(sd - (long)m * a.dn_ntr);
                a.down_out[(size_t)m * H + tr * 16 + rr] = s;
            }
        }
        stamp(l, 5, 1);
    }
    // ================= final norm =================
    if (synced && gsync() && c == 0) {
        float hv[HMAX];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < HMAX; ++j) {
            const int i = tid + j * NW * 32;
            hv[j] = 0.f;
            if (i < H) {
                hv[j] = residual_in(a.n_layer, i);
                ss = fmaf(hv[j], hv[j], ss);
            }
        }
        const float scale = 1.0f / sqrtf(block_sum(ss) / (float)H + a.eps);
#pragma unroll
        for (int j = 0; j < HMAX; ++j) {
            const int i = tid + j * NW * 32;
            if (i < H) a.out[i] = (hv[j] * scale) * __ldg(a.out_norm + i);
        }
        if (tid == 0) *a.pos = pos + 1;
    }
    // no bulk copy may still be landing in this CTA's shared memory when it exits: a down
    // piece still waiting for its activations gets them (from the buffer as it is), then every
    // issued piece is waited for (bounded)
    if (n_def > 0) issue_deferred(ic.l < a.n_layer ? ic.l : a.n_layer - 1);
    for (long k = n_con; k < n_iss; ++k) mbar_wait(&bars[warp][k % RS], (unsigned)((k / RS) & 1), a.status);
}

}  // namespace

// ---- host side -------------------------------------------------------------------------------

struct step_plan {
    moearc_ctx *c = nullptr;
    step_args a{};
    int G = 0, smem = 0, wtype = 0;
    void *mem = nullptr;
    step_layer *dL = nullptr;
    unsigned long long limit_ns = XPOLL_NS;
    unsigned phantom = 0;
    unsigned long long *trace = nullptr;
};

namespace {

// Most distinct units (tile-rows or segments) one warp's item range [lo, hi) touches, units of
// `per` items.
int units_touched(long lo, long hi, long per) { return hi <= lo ? 0 : (int)((hi - 1) / per - lo / per + 1); }

}  // namespace

step_plan *step_create(moearc_ctx *c, const step_shape &s, const step_layer *layers) {
    if (!c || !layers || s.n_layer <= 0) return nullptr;
    const int H = s.H, Dq = s.n_head * s.head_dim, Dkv = s.n_kv * s.head_dim;
    if (s.head_dim != HD || H % 64 || s.I % 64 || H > HMAX * NW * 32 || s.n_kv <= 0 || s.n_head % s.n_kv ||
        s.n_head / s.n_kv > MAXG || s.K < 1 || s.K > 8 || s.E < s.K || s.E > 256 ||
        (s.wtype != T_MXFP4 && s.wtype != T_Q4_0))
        return nullptr;
    const int G = c->sm_count;
    if (s.n_kv > G) return nullptr;
    auto *p = new step_plan();
    p->c = c;
    p->G = G;
    p->wtype = s.wtype;
    step_args &a = p->a;
    a.n_layer = s.n_layer;
    a.H = H;
    a.Dq = Dq;
    a.Dkv = Dkv;
    a.n_head = s.n_head;
    a.n_kv = s.n_kv;
    a.group = s.n_head / s.n_kv;
    a.E = s.E;
    a.K = s.K;
    a.I = s.I;
    a.gating = s.gating;
    a.act = s.act;
    a.alpha = s.alpha;
    a.limit = s.limit;
    a.eps = s.eps;
    a.scale = 1.0f / std::sqrt((float)HD);
    a.rope_freq = s.rope_freq;
    a.mscale = s.mscale;
    a.q_ntr = (Dq + 2 * Dkv) / 16;
    a.q_nkt = H / 64;
    a.q_T = (long)a.q_ntr * a.q_nkt;
    a.o_ntr = H / 16;
    a.o_nkt = Dq / 64;
    a.o_T = (long)a.o_ntr * a.o_nkt;
    const bool mx = s.wtype == T_MXFP4;
    a.tile_bytes = mx ? 544 : 576;
    a.pair_bytes = 2 * a.tile_bytes;
    a.ch_gu = std::max(1, std::min(3, SB / a.pair_bytes));
    a.ch_dn = std::max(1, SB / (a.tile_bytes + 256));
    a.gu_ntr = s.I / 16;
    a.gu_nkt = H / 64;
    a.dn_ntr = H / 16;
    a.dn_nkt = s.I / 64;
    a.gu_stride = (size_t)a.gu_ntr * a.gu_nkt * a.pair_bytes;
    a.dn_stride = (size_t)a.dn_ntr * a.dn_nkt * a.tile_bytes;
    a.max_splits = std::max(1, G / s.n_kv);
    a.xs_bytes = (std::max({6 * H, 6 * Dq, 8 * H}) + 127) / 128 * 128;
    // every warp's share of every phase must fit its partial records
    auto fits = [&]() {
        const long GW = (long)G * NW, GWo = (long)G * (NW - AW);
        for (int cc = 0; cc < G; ++cc) {
            for (int w = 0; w < NW; ++w) {
                const long gw = (long)cc * NW + w;
                if (units_touched(a.q_T * gw / GW, a.q_T * (gw + 1) / GW, a.q_nkt) > WSEG) return false;
                if (w >= AW) {
                    const long g2 = (long)cc * (NW - AW) + (w - AW);
                    if (units_touched(a.o_T * g2 / GWo, a.o_T * (g2 + 1) / GWo, a.o_nkt) > WSEG) return false;
                }
                const long Sg = (long)a.K * a.gu_ntr, s0 = Sg * cc / G, s1 = Sg * (cc + 1) / G;
                const long Pg = (s1 - s0) * a.gu_nkt;
                if (units_touched(s0 * a.gu_nkt + Pg * w / NW, s0 * a.gu_nkt + Pg * (w + 1) / NW, a.gu_nkt) > WSEG)
                    return false;
                const long Sd = (long)a.K * a.dn_ntr, d0 = Sd * cc / G, d1 = Sd * (cc + 1) / G;
                const long Pd = (d1 - d0) * a.dn_nkt;
                if (units_touched(d0 * a.dn_nkt + Pd * w / NW, d0 * a.dn_nkt + Pd * (w + 1) / NW, a.dn_nkt) > WSEG)
                    return false;
            }
        }
        return (s.E + G - 1) / G <= WSEG * 32;
    };
    auto maxc_of = [&](long T, int nkt, int ntr) {
        int m = 1;
        for (int tr = 0; tr < ntr; ++tr)
            m = std::max(m, owner_of(T, G, (long)(tr + 1) * nkt - 1) - owner_of(T, G, (long)tr * nkt) + 1);
        return m;
    };
    if (!fits()) {
        delete p;
        return nullptr;
    }
    a.q_maxc = maxc_of(a.q_T, a.q_nkt, a.q_ntr);
    a.o_maxc = maxc_of(a.o_T, a.o_nkt, a.o_ntr);
    p->smem = NW * RS * SB + a.xs_bytes + NW * WSEG * 32 * 4;

    // device state, one allocation
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) / 256 * 256;
        return o;
    };
    const size_t o_sync = take(16), o_status = take(16), o_ctr = take(4 * (size_t)s.n_kv);
    const size_t o_hbuf = take(4 * (size_t)H), o_hmid = take(4 * (size_t)H);
    const size_t o_qp = take(4 * 16 * (size_t)a.q_ntr * a.q_maxc), o_op = take(4 * 16 * (size_t)a.o_ntr * a.o_maxc);
    const size_t o_att = take(4 * (size_t)Dq);
    const size_t o_ml = take(4 * 2 * (size_t)s.n_head * a.max_splits), o_acc = take(4 * (size_t)HD * s.n_head * a.max_splits);
    const size_t o_lg = take(4 * (size_t)s.E), o_af = take(4 * (size_t)s.K * s.I), o_do = take(4 * (size_t)s.K * H);
    const size_t o_ri = take(4 * (size_t)s.n_layer * s.K), o_rw = take(4 * (size_t)s.n_layer * s.K);
    const size_t o_L = take(sizeof(step_layer) * (size_t)s.n_layer);
    if (cudaMalloc(&p->mem, off) != cudaSuccess) {
        cudaGetLastError();
        delete p;
        return nullptr;
    }
    uint8_t *b = static_cast<uint8_t *>(p->mem);
    a.sync = reinterpret_cast<unsigned *>(b + o_sync);
    a.status = reinterpret_cast<int *>(b + o_status);
    a.att_ctr = reinterpret_cast<unsigned *>(b + o_ctr);
    a.hbuf = reinterpret_cast<float *>(b + o_hbuf);
    a.hmid = reinterpret_cast<float *>(b + o_hmid);
    a.qkv_part = reinterpret_cast<float *>(b + o_qp);
    a.o_part = reinterpret_cast<float *>(b + o_op);
    a.att = reinterpret_cast<float *>(b + o_att);
    a.att_ml = reinterpret_cast<float *>(b + o_ml);
    a.att_acc = reinterpret_cast<float *>(b + o_acc);
    a.logits = reinterpret_cast<float *>(b + o_lg);
    a.actfrag = reinterpret_cast<uint32_t *>(b + o_af);
    a.down_out = reinterpret_cast<float *>(b + o_do);
    a.route_idx = reinterpret_cast<unsigned *>(b + o_ri);
    a.route_w = reinterpret_cast<float *>(b + o_rw);
    p->dL = reinterpret_cast<step_layer *>(b + o_L);
    a.L = p->dL;
    bool ok = cudaMemsetAsync(p->mem, 0, off, c->stream) == cudaSuccess &&
              cudaMemcpyAsync(p->dL, layers, sizeof(step_layer) * s.n_layer, cudaMemcpyHostToDevice, c->stream) ==
                  cudaSuccess &&
              cudaStreamSynchronize(c->stream) == cudaSuccess;
    const cudaError_t e = mx ? set_smem(k_step<39>, p->smem) : set_smem(k_step<2>, p->smem);
    ok &= e == cudaSuccess;
    if (ok) {
        int per_sm = 0;
        ok = (mx ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_step<39>, NW * 32, p->smem)
                 : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_step<2>, NW * 32, p->smem)) ==
                 cudaSuccess &&
             per_sm >= 1;
    }
    if (!ok) {
        cudaGetLastError();
        cudaFree(p->mem);
        delete p;
        return nullptr;
    }
    return p;
}

void step_destroy(step_plan *p) {
    if (!p) return;
    cudaFree(p->mem);
    delete p;
}

int step_run(step_plan *p, const float *in, float *out, const float *out_norm, int *pos) {
    if (!p || !in || !out || !out_norm || !pos) return ERR;
    step_args a = p->a;
    a.in = in;
    a.out = out;
    a.out_norm = out_norm;
    a.pos = pos;
    a.limit_ns = p->limit_ns;
    a.phantom = p->phantom;
    a.trace = p->trace;
    moearc_ctx *c = p->c;
    if (cudaMemsetAsync(a.sync, 0, 2 * sizeof(unsigned), c->stream) != cudaSuccess) return ERR;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)p->G);
    cfg.blockDim = dim3(NW * 32);
    cfg.dynamicSmemBytes = (size_t)p->smem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = p->wtype == T_MXFP4 ? cudaLaunchKernelEx(&cfg, k_step<39>, a) : cudaLaunchKernelEx(&cfg, k_step<2>, a);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return ERR;
    }
    return OK;
}

int step_status(step_plan *p) {
    if (!p) return ERR;
    int s = 0;
    if (cudaMemcpyAsync(&s, p->a.status, sizeof(int), cudaMemcpyDeviceToHost, p->c->stream) != cudaSuccess ||
        cudaMemsetAsync(p->a.status, 0, sizeof(int), p->c->stream) != cudaSuccess ||
        cudaStreamSynchronize(p->c->stream) != cudaSuccess)
        return ERR;
    return s;
}

void step_set_wait(step_plan *p, unsigned long long limit_ns, unsigned phantom) {
    if (!p) return;
    p->limit_ns = limit_ns ? limit_ns : XPOLL_NS;
    p->phantom = phantom;
}

size_t step_trace_words(step_plan *p) { return p ? (size_t)p->a.n_layer * NPH * 2 * p->G : 0; }

void step_set_trace(step_plan *p, unsigned long long *buf) {
    if (p) p->trace = buf;
}

void *step_buffer(step_plan *p, int which) {
    if (!p) return nullptr;
    return which == 0 ? static_cast<void *>(p->a.route_idx) : which == 1 ? static_cast<void *>(p->a.route_w) : nullptr;
}

}  // namespace moearc
