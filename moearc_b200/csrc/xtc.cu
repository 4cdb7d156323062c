// xtc.cu — batch-1 decode experts on the block-scaled FP4 tensor cores (tcgen05.mma
// kind::mxf4.block_scale.block32). Layouts and the digit form of the activation: xtc.cuh.
//
// Semantics are the decode path's (moe.cu; crates/moearc-engine/src/moe.rs:2074-2427): the
// token's top-k from the router logits, per chosen expert act(gate . x, up . x), down . that,
// and the router-weighted sum over the k experts in router order plus the residual.
//
// Two kernels per layer, one CTA per SM, each a flat run of work units (one k-pair of one tile)
// cut into equal contiguous shares:
//   gate-up  units (expert slot, tile, k-pair); after its wait every CTA derives the top-k
//            (CTA 0 publishes it for the down kernel), then streams its share
//   down     units (row tile, expert slot, k-pair); its weights stream before its wait (the
//            experts are known from the published top-k), the digits of the activation after
// Roles: warp 0 lane 0 issues the bulk copies of each piece (up to XT_PK k-pairs of one tile:
// the weights and the matching activation digits) into a ring of XT_STAGES stages; warp 1 lane 0
// copies each k-pair's scale blocks into TMEM and issues its MMAs (128 rows x 16 digit columns x
// 64 per MMA) into the accumulator of the tile; warps 2-5 read each finished accumulator (lane =
// row), sum its digit columns, and finish the tile: a tile shared by several CTAs (split K)
// leaves partials, and the last CTA to arrive on the tile's counter (the row tile's, for down)
// sums them in CTA order — deterministic, no floating-point atomics.
//   gate-up finish: act(gate, up) (+ biases) into the down kernel's digits
//   down finish:    per row, the router-weighted sum over the k experts (+ biases) + residual
#include <algorithm>
#include <atomic>
#include <vector>

#include "route.cuh"
#include "tc.cuh"
#include "tma.cuh"
#include "xtc.cuh"

namespace moearc {

namespace {

constexpr int XT_PK = 4;                                  // k-pairs per piece: one bulk copy, one ring stage
constexpr int XT_STAGES = 5;                              // most ring stages (fewer when the digits take room)
constexpr int XT_STAGE_A = XT_PK * TC_KPAIR;              // 34816
constexpr int XT_SMEM_MAX = 226 * 1024;             // dynamic shared memory limit (static use beside it)
constexpr int XT_MAXSEG = 4;                              // tiles one CTA's share may touch
constexpr int XT_MAXUNITS = 40;                           // k-pairs one CTA's share may hold
// Two threads in different warps issue the MMAs, alternating pieces, each into its own
// accumulator: one thread's tcgen05 instructions issue in series (about 60 ns an MMA measured),
// two overlap (22 ns an MMA between them).
constexpr int XT_ISSUERS = 2;
// TMEM columns: per tile of the share one 16-column accumulator per issuer, then the weights'
// scale blocks (4 columns per k-pair of a ring stage), then the digits' scale blocks (4 columns
// per k-pair of the share, copied once).
constexpr int XT_SEGCOLS = XT_ISSUERS * TC_DIGITS;
constexpr int XT_ASC = XT_MAXSEG * XT_SEGCOLS;            // 128
constexpr int XT_BSC = XT_ASC + XT_STAGES * XT_PK * 4;    // 208
constexpr int XT_TMEM = 512;
static_assert(XT_BSC + XT_MAXUNITS * 4 <= XT_TMEM, "TMEM columns");
constexpr int XT_THREADS = 224;  // warp 0 producer, warps 1 and 6 MMA issuers, warps 2-5 epilogue
constexpr int XT_MAXK = 8;

struct xtc_args {
    const uint8_t *bank;
    size_t bank_stride, tile_bytes;
    int tiles, nkp, ksteps;
    int stages;                // ring stages (the share's digits take the rest of the shared memory)
    int rows_last;             // rows of the last tile that exist (down), else 128
    const uint8_t *b_in;       // digits: gate-up one activation; down [K] activations
    size_t b_stride;           // bytes per expert slot of b_in (0 for gate-up)
    uint8_t *b_out;            // gate-up: the down kernel's digits
    size_t b_out_stride;
    const float *logits;
    int E, K, gating;
    unsigned *idx_pub;
    float *wts_pub;
    int act;
    float alpha, limit;
    float *act_out;
    int H, I;
    const float *bias_gu, *bias_dn;
    const float *residual;
    float *out;
    float *part;               // partial slots [tile][contributor][128], PART_EMPTY when free
    int maxc;
    unsigned long long poll_ns;
    int phantom;
    unsigned long long *span;
    int *status;
};

// The CTA of G whose share [U c / G, U (c + 1) / G) holds unit u.
__host__ __device__ __forceinline__ int unit_cta(long U, int G, long u) { return (int)(((u + 1) * G - 1) / U); }

__device__ __forceinline__ uint64_t desc_sw32(uint32_t addr) {
    // start >> 4, leading offset 16 B (unused by swizzled K-major), 8-row groups 256 B apart,
    // descriptor version 1, layout 6 (32-byte swizzle)
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(256 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)6 << 61);
}
__device__ __forceinline__ uint64_t desc_sfblk(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 32) | ((uint64_t)1 << 46);
}
// kind::mxf4 instruction descriptor: scale ids (A bits 29-30, B bits 4-5), A and B E2M1 (1),
// K-major, N = 16 (bits 17-22: N >> 3), E8M0 scales (bit 23), M = 128 (bits 24-28: M >> 4).
__device__ __forceinline__ uint32_t idesc_mxf4(int sf_id) {
    return ((uint32_t)sf_id << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_DIGITS >> 3) << 17) | (1u << 23) |
           ((uint32_t)(128 >> 4) << 24) | ((uint32_t)sf_id << 29);
}
__device__ __forceinline__ void mma_mxf4(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t sfa,
                                         uint32_t sfb, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %6, 0;\n"
        " tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%4], [%5], p; }" ::"r"(d),
        "l"(da), "l"(db), "r"(idesc), "r"(sfa), "r"(sfb), "r"(acc));
}
__device__ __forceinline__ void cp_sf(uint32_t taddr, uint32_t saddr) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc_sfblk(saddr)));
}
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Phase timestamps of one CTA (-DMOEARC_TRACE builds only): any thread may record a slot.
#ifdef MOEARC_TRACE
#define XT_TRACE(slot)                                                          \
    do {                                                                        \
        if (g_trace) g_trace[(size_t)trace_row * 32 + (slot)] = xnow();         \
    } while (0)
#else
#define XT_TRACE(slot) \
    do {               \
    } while (0)
#endif

// The top-k, not inlined: the gate-up kernel runs it twice (a dry run before its wait, then the
// real one), and the second call finds the code in the instruction cache.
__device__ __noinline__ void xt_topk(const float *logits, int E, int K, int gating, int lane, unsigned *idx, float *wts) {
    xtopk(logits, E, K, gating, lane, idx, wts);
}

// The CTA's share as segments (one per tile it touches): the tile (group) and its k-pairs
// [lo, hi); b is the segment's first k-pair within the share (the digit buffer and the digits'
// scale columns are laid out by position within the share).
struct xt_share {
    int n;
    int g[XT_MAXSEG], lo[XT_MAXSEG], hi[XT_MAXSEG], b[XT_MAXSEG];
};

template <int MODE>
__global__ void __launch_bounds__(XT_THREADS, 1) k_xtc(xtc_args a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full[XT_STAGES], empty[XT_STAGES], seg_full[XT_MAXSEG], bfull, bsf,
        done[XT_ISSUERS], never;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_;
    __shared__ unsigned s_idx[XT_MAXK];
    __shared__ float s_wts[XT_MAXK];
    __shared__ float s_up[64];
    __shared__ int s_ok;
    __shared__ xt_share sh;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int trace_row = (int)blockIdx.x + (MODE == 0 ? 0 : 1024);
    (void)trace_row;
    if (threadIdx.x == 0) XT_TRACE(0);
    unsigned long long *span = a.span ? a.span + (size_t)blockIdx.x * 3 : nullptr;
    if (span && threadIdx.x == 0) {
        span[0] = xnow();
        span[2] = 0;
    }
    const int nkp = a.nkp, K = a.K, S = a.stages;
    const long U = (long)K * a.tiles * nkp;
    const int NC = gridDim.x;
    const long ua = U * blockIdx.x / NC, ub = U * (blockIdx.x + 1) / NC;
    const int units = (int)(ub - ua);
    uint8_t *bsm = smem + (size_t)S * XT_STAGE_A;  // the share's digits, k-pair by k-pair
    if (threadIdx.x == 0) {
        for (int s = 0; s < XT_STAGES; ++s) {
            tc::bar_init(&full[s], 1);
            tc::bar_init(&empty[s], 1);
        }
        for (int s = 0; s < XT_MAXSEG; ++s) tc::bar_init(&seg_full[s], XT_ISSUERS);
        tc::bar_init(&bfull, 1);
        tc::bar_init(&bsf, 1);
        for (int c = 0; c < XT_ISSUERS; ++c) tc::bar_init(&done[c], 1);
        tc::bar_init(&never, 1);
        abort_ = 0;
        tc::bar_init_fence();
        int n = 0, b = 0;
        for (long u = ua; u < ub && n < XT_MAXSEG; ++n) {
            const int g = (int)(u / nkp);
            const long e = min(ub, (long)(g + 1) * nkp);
            sh.g[n] = g;
            sh.lo[n] = (int)(u - (long)g * nkp);
            sh.hi[n] = (int)(e - (long)g * nkp);
            sh.b[n] = b;
            b += (int)(e - u);
            u = e;
        }
        sh.n = n;
    }
    if (warp == 1) tc::tmem_alloc(&tmem_slot, XT_TMEM);
    if (MODE == 1) {
        // the gate-up kernel's CTA 0 published the top-k before it let this kernel launch
        if (threadIdx.x < K) {
            s_idx[threadIdx.x] = __ldcg(a.idx_pub + threadIdx.x);
            s_wts[threadIdx.x] = __ldcg(a.wts_pub + threadIdx.x);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    const int nseg = sh.n;

    if (MODE == 0) {
        // a dry run of the top-k on whatever the logits hold now (the router is still writing
        // them; the result is overwritten below) brings its code into the instruction cache
        if (warp == 0) xt_topk(a.logits, a.E, K, a.gating, lane, s_idx, s_wts);
        // the logits and the activation's digits are the router's output
        pdl_wait();
        if (span && threadIdx.x == 0) span[1] = xnow();
        if (threadIdx.x == 0) XT_TRACE(1);
        if (warp == 0) xt_topk(a.logits, a.E, K, a.gating, lane, s_idx, s_wts);
        __syncthreads();
        if (threadIdx.x == 0) XT_TRACE(2);
        if (blockIdx.x == 0) {
            if (threadIdx.x < K) {
                a.idx_pub[threadIdx.x] = s_idx[threadIdx.x];
                a.wts_pub[threadIdx.x] = s_wts[threadIdx.x];
            }
            __threadfence();
            __syncthreads();
        }
        pdl_trigger();
    }

    auto expert_of = [&](int g) { return MODE == 0 ? g / a.tiles : g % K; };  // expert slot
    auto tile_of = [&](int g) { return MODE == 0 ? g % a.tiles : g / K; };
    // piece q of the share: its segment, first k-pair and k-pairs (pieces never span segments)
    auto piece_of = [&](int q, int &sg, int &kp0, int &n) {
        for (sg = 0; sg < nseg; ++sg) {
            const int np = (sh.hi[sg] - sh.lo[sg] + XT_PK - 1) / XT_PK;
            if (q < np) break;
            q -= np;
        }
        kp0 = sh.lo[sg] + q * XT_PK;
        n = min(XT_PK, sh.hi[sg] - kp0);
    };
    int n_pieces = 0;
    for (int sg = 0; sg < nseg; ++sg) n_pieces += (sh.hi[sg] - sh.lo[sg] + XT_PK - 1) / XT_PK;

    if (warp == 0) {
        // ---- producer: one bulk copy per piece; the first S pieces from S lanes at once -------
        auto issue_a = [&](int q) {
            int sg, kp0, n;
            piece_of(q, sg, kp0, n);
            const int g = sh.g[sg], s = q % S;
            const bool half_last = (kp0 + n == nkp) && (a.ksteps & 1);
            const unsigned bytes = (unsigned)(n * TC_KPAIR - (half_last ? TC_KPAIR - TC_KPAIR_HALF : 0));
            const uint8_t *src = a.bank + (size_t)s_idx[expert_of(g)] * a.bank_stride +
                                 (size_t)tile_of(g) * a.tile_bytes + (size_t)kp0 * TC_KPAIR;
            tc::bar_expect_tx(&full[s], bytes);
            bulk_g2s(smem + (size_t)s * XT_STAGE_A, src, bytes, &full[s]);
        };
        auto issue_b = [&]() {
            // the digits of every segment's k-pairs, once: gate-up one activation, down the
            // segment's expert's
            tc::bar_expect_tx(&bfull, (unsigned)(units * TC_BKPAIR));
            for (int sg = 0; sg < nseg; ++sg)
                bulk_g2s(bsm + (size_t)sh.b[sg] * TC_BKPAIR,
                         a.b_in + (size_t)expert_of(sh.g[sg]) * a.b_stride + (size_t)sh.lo[sg] * TC_BKPAIR,
                         (unsigned)((sh.hi[sg] - sh.lo[sg]) * TC_BKPAIR), &bfull);
        };
        // A CTA's bulk copies complete in issue order: the gate-up kernel's digits (in L2, and
        // needed by the first MMA) go before the weights; the down kernel's weights go before its
        // wait, its digits after it.
        const int burst = min(S, n_pieces);
        if (MODE == 0 && lane == 0) issue_b();
        __syncwarp();
        if (lane < burst) issue_a(lane);
        __syncwarp();
        if (MODE == 1) {
            pdl_wait();  // the digits are the gate-up kernel's output
            if (span && lane == 0) span[1] = xnow();
            if (lane == 0) XT_TRACE(1);
            if (lane == 0) issue_b();
        }
        if (lane == 0) {
            XT_TRACE(3);
            int q = burst;
            for (; q < n_pieces; ++q) {
                const int s = q % S;
                if (!tc::bar_wait(&empty[s], (unsigned)(((q / S) - 1) & 1), &abort_, a.status, STATUS_WAIT_TIMEOUT))
                    break;
                issue_a(q);
            }
            XT_TRACE(10);
            // every copy issued lands before the CTA exits
            for (int r = max(0, q - S); r < q; ++r) tc::bar_drain(&full[r % S], (unsigned)((r / S) & 1));
            tc::bar_drain(&bfull, 0);
        }
    } else if (warp == 1 || warp == 6) {
        // ---- MMA issuers: issuer c takes the pieces q with q % 2 == c ------------------------
        const int c = warp == 1 ? 0 : 1;
        if (MODE == 1) pdl_wait();
        if (lane == 0) {
            bool ok = tc::bar_wait(&bfull, 0, &abort_, a.status, STATUS_WAIT_TIMEOUT);
            if (ok && c == 0) {
                // the digits' scale blocks, once, then released to the other issuer
                tc::fence_after_sync();
                XT_TRACE(11);
                const uint32_t b0 = tc::sa(bsm);
                for (int j = 0; j < units; ++j)
                    cp_sf(tmem + (uint32_t)(XT_BSC + 4 * j), b0 + (uint32_t)(j * TC_BKPAIR + 2 * TC_BBLK));
                tc::mma_commit(&bsf);
            }
            if (ok && c == 1) ok = tc::bar_wait(&bsf, 0, &abort_, a.status, STATUS_WAIT_TIMEOUT);
            // descriptors advance by address: a 16-byte unit is 1 in the start field (bits 0-13)
            const uint32_t a_base = tc::sa(smem), b_base = tc::sa(bsm);
            const uint32_t id0 = idesc_mxf4(0), id2 = idesc_mxf4(2);
            const bool odd = a.ksteps & 1;
            int q = 0, s = 0, ph = 0;  // piece, its stage and the stage's phase parity
            for (int sg = 0; sg < nseg && ok; ++sg) {
                const int lo = sh.lo[sg], hi = sh.hi[sg], jb = sh.b[sg] - lo;
                const uint32_t dcol = tmem + (uint32_t)(sg * XT_SEGCOLS + c * TC_DIGITS);
                uint32_t acc = 0u;
                for (int kp0 = lo; kp0 < hi && ok; kp0 += XT_PK, ++q) {
                    if ((q & 1) == c) {
                        const int n = min(XT_PK, hi - kp0);
                        if (!tc::bar_wait(&full[s], (unsigned)ph, &abort_, a.status, STATUS_WAIT_TIMEOUT)) {
                            ok = false;
                            break;
                        }
                        if (c == 0 && q < 7) XT_TRACE(12 + q);
                        tc::fence_after_sync();
                        uint32_t a_kp = a_base + (uint32_t)(s * XT_STAGE_A);
                        uint32_t b_kp = b_base + (uint32_t)((kp0 + jb) * TC_BKPAIR);
                        uint32_t sfa = tmem + (uint32_t)(XT_ASC + s * XT_PK * 4);
                        uint32_t sfb = tmem + (uint32_t)(XT_BSC + 4 * (kp0 + jb));
                        for (int i = 0; i < n; ++i) {
                            const bool half = odd && (kp0 + i == nkp - 1);
                            cp_sf(sfa, a_kp + (half ? TC_ABLK : 2 * TC_ABLK));
                            const uint64_t da = desc_sw32(a_kp), db = desc_sw32(b_kp);
                            mma_mxf4(dcol, da, db, id0, sfa, sfb, acc);
                            acc = 1u;
                            if (!half) mma_mxf4(dcol, da + (TC_ABLK >> 4), db + (TC_BBLK >> 4), id2, sfa, sfb, 1u);
                            a_kp += TC_KPAIR;
                            b_kp += TC_BKPAIR;
                            sfa += 4;
                            sfb += 4;
                        }
                        tc::mma_commit(&empty[s]);
                    }
                    if (++s == S) {
                        s = 0;
                        ph ^= 1;
                    }
                }
                if (ok) tc::mma_commit(&seg_full[sg]);  // an issuer with no piece in the tile arrives at once
            }
            if (c == 0) XT_TRACE(19);
            tc::mma_commit(&done[c]);
            tc::bar_drain(&done[c], 0);
            if (c == 0) XT_TRACE(20);
        }
    } else {
        // ---- epilogue: warps 2-5, TMEM lane quarter warp % 4, tile row m = 32 quarter + lane --
        if (MODE == 1) pdl_wait();
        const int quarter = warp & 3, m = 32 * quarter + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * quarter) << 16);
        bool stop = false;
        if (a.phantom) {
            // testing: a wait that nothing ends gives up after poll_ns
            const unsigned long long t0 = xnow();
            while (!tc::bar_try(&never, 0))
                if (xnow() - t0 > a.poll_ns) break;
            if (threadIdx.x == 64) atomicOr(a.status, STATUS_WAIT_TIMEOUT);
            abort_ = 1;
            stop = true;
        }
        for (int seg = 0; seg < nseg && !stop; ++seg) {
            const int g = sh.g[seg];
            // one thread waits for the accumulator, so the four warps take the same branch
            if (threadIdx.x == 64) s_ok = tc::bar_wait(&seg_full[seg], 0, &abort_, a.status, STATUS_WAIT_TIMEOUT);
            epi_sync();
            if (!s_ok) break;
            if (threadIdx.x == 64 && seg < 3) XT_TRACE(21 + seg);
            tc::fence_after_sync();
            // the issuers that took a piece of this tile: both, unless it has one piece
            int q0 = 0;
            for (int j = 0; j < seg; ++j) q0 += (sh.hi[j] - sh.lo[j] + XT_PK - 1) / XT_PK;
            const int np = (sh.hi[seg] - sh.lo[seg] + XT_PK - 1) / XT_PK;
            float dsum[TC_DIGITS];
#pragma unroll
            for (int d = 0; d < TC_DIGITS; ++d) dsum[d] = 0.f;
            for (int c = 0; c < XT_ISSUERS; ++c) {
                if (np == 1 && (q0 & 1) != c) continue;
                float v[TC_DIGITS];
                tc::tmem_ld16(lane_base + (uint32_t)(seg * XT_SEGCOLS + c * TC_DIGITS), v);
#pragma unroll
                for (int d = 0; d < TC_DIGITS; ++d) dsum[d] += v[d];
            }
            float s = 0.f;
#pragma unroll
            for (int d = TC_DIGITS - 1; d >= 0; --d) s += dsum[d];
            // The tile's contributors are the CTAs c0 .. c0 + nc - 1 (c0 holds its first k-pairs, at
            // the end of its share, so it finishes its part last). Each other contributor stores its
            // partial into its slot (whole lines, relaxed); c0 polls the slots (bounded), sums them in
            // contributor order, empties them and finishes the tile. Down: the row tile's finisher is
            // the CTA holding its first unit, after its last segment in that row tile.
            const long g_lo = (long)g * nkp;
            const int c0 = unit_cta(U, NC, g_lo), nc = unit_cta(U, NC, g_lo + nkp - 1) - c0 + 1;
            const int slot = (int)blockIdx.x - c0;
            const int em = expert_of(g), t = tile_of(g);
            bool fin;
            if (MODE == 0) {
                fin = slot == 0;
            } else {
                const long t_lo = (long)t * K * nkp;
                fin = (int)blockIdx.x == unit_cta(U, NC, t_lo) && (seg + 1 == nseg || tile_of(sh.g[seg + 1]) != t);
            }
            if (!fin) st_part(a.part + ((size_t)g * a.maxc + slot) * 128 + m, s);
            // the slot's value once it has been stored (testing: a phantom wait never sees one)
            auto take = [&](float *p, float &v) {
                const unsigned long long t0 = xnow();
                uint32_t w;
                while ((w = ld_part(p)) == PART_EMPTY) {
                    if (xnow() - t0 > a.poll_ns) {
                        atomicOr(a.status, STATUS_WAIT_TIMEOUT);
                        return false;
                    }
                }
                st_part(p, __uint_as_float(PART_EMPTY));
                v = __uint_as_float(w);
                return true;
            };
            bool ok = true;
            if (fin && MODE == 0) {
                // gate-up tile (expert slot em, tile t): rows 0-63 gate, 64-127 up of 64 t + (m % 64)
                float tot = s;
                for (int k = 1; k < nc && ok; ++k) {
                    float v;
                    ok = take(a.part + ((size_t)g * a.maxc + k) * 128 + m, v);
                    tot += v;
                }
                if (threadIdx.x == 128) XT_TRACE(28);
                const int e = (int)s_idx[em], row = 64 * t + (m & 63);
                if (m >= 64) {
                    if (a.bias_gu) tot += a.bias_gu[(size_t)(a.E + e) * a.I + row];
                    s_up[m - 64] = tot;
                }
                epi_sync();
                if (m < 64) {
                    if (a.bias_gu) tot += a.bias_gu[(size_t)e * a.I + row];
                    const float act = act_fn(a.act, tot, s_up[m], a.alpha, a.limit);
                    // inspection copy, columns in ascending expert order as the fragment path's
                    int col = 0;
                    for (int e2 = 0; e2 < K; ++e2) col += s_idx[e2] < (unsigned)e;
                    a.act_out[(size_t)col * a.I + row] = act;
                    if (threadIdx.x == 128) XT_TRACE(29);
                    tc_write_digits(act, lane, a.b_out + (size_t)em * a.b_out_stride, 2 * t + quarter);
                    if (threadIdx.x == 128) XT_TRACE(30);
                }
            } else if (fin) {
                // row tile t: every expert's rows summed over its contributors, then the
                // router-weighted sum in router order and the residual (moe.rs:2395-2425)
                const int rows = (t == a.tiles - 1) ? a.rows_last : 128;
                const int row = 128 * t + m;
                float acc = 0.f;
                for (int e2 = 0; e2 < K; ++e2) {
                    const int h = t * K + e2;
                    const long h_lo = (long)h * nkp;
                    const int d0 = unit_cta(U, NC, h_lo), dn = unit_cta(U, NC, h_lo + nkp - 1) - d0 + 1;
                    float o = 0.f;
                    for (int k = 0; k < dn; ++k) {
                        float v = s;
                        if (!(h == g && k == slot) && !take(a.part + ((size_t)h * a.maxc + k) * 128 + m, v)) ok = false;
                        o += v;
                    }
                    if (m < rows && a.bias_dn) o += a.bias_dn[(size_t)s_idx[e2] * a.H + row];
                    acc = fmaf(s_wts[e2], o, acc);
                }
                if (m < rows) a.out[row] = a.residual ? a.residual[row] + acc : acc;
            }
            // a slot that never filled has raised the status; the step's output is then invalid
            (void)ok;
            epi_sync();  // the shared words are rewritten by the next tile
            if (threadIdx.x == 64 && seg < 3) XT_TRACE(24 + seg);
        }
        if (threadIdx.x == 64) XT_TRACE(27);
    }
    if (MODE == 1) pdl_trigger();
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, XT_TMEM);
    }
    if (span && threadIdx.x == 0) atomicMax(span + 2, xnow());
    if (threadIdx.x == 0) XT_TRACE(31);
}

// ---- packing -------------------------------------------------------------------------------

// One 16-byte half of a k-step row (32 elements: one MXFP4 block) per thread. Gate-up (MODE 0):
// tile t row m is gate row 64 t + m (m < 64) or up row 64 t + m - 64; down (MODE 1): row 128 t + m,
// zero past the matrix. GGUF MXFP4 block: e8m0 byte, then qs[16] with element j in the low and
// element j + 16 in the high nibble of qs[j]; the tc layout wants elements 2q, 2q + 1 in byte q.
template <int MODE>
__global__ void k_xtc_pack(uint8_t *dst, const uint8_t *src0, const uint8_t *src1, int rows, int K, int tiles,
                           size_t stride, unsigned n_expert) {
    const int ks_n = tc_ksteps(K), nkp = tc_kpairs(K), nblk = K / 32;
    const size_t tile_bytes = tc_tile_bytes(K);
    const size_t per_tile = (size_t)ks_n * 128 * 2;
    const size_t total = (size_t)n_expert * tiles * per_tile;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int half = (int)(i & 1);
        const int m = (int)((i >> 1) & 127);
        const size_t r = i >> 8;
        const int ks = (int)(r % ks_n);
        const size_t et = r / ks_n;
        const int t = (int)(et % tiles);
        const unsigned e = (unsigned)(et / tiles);
        const uint8_t *src;
        int row;
        if (MODE == 0) {
            src = m < 64 ? src0 : src1;
            row = 64 * t + (m & 63);
        } else {
            src = src0;
            row = 128 * t + m;
        }
        uint8_t *tile = dst + (size_t)e * stride + (size_t)t * tile_bytes;
        const int kp = ks >> 1;
        const bool half_kp = (kp == nkp - 1) && (ks_n & 1);
        uint8_t *ab = tile + (size_t)kp * TC_KPAIR + (ks & 1) * TC_ABLK;
        uint8_t *sf = tile + (size_t)kp * TC_KPAIR + (half_kp ? TC_ABLK : 2 * TC_ABLK);
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        uint8_t scale = 0;
        if (row < rows) {
            const uint8_t *blk = src + (((size_t)e * rows + row) * nblk + 2 * ks + half) * 17;
            scale = blk[0];
            const uint8_t *qs = blk + 1;
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                const uint32_t lo = q < 8 ? (qs[2 * q] & 15u) : (qs[2 * q - 16] >> 4);
                const uint32_t hi = q < 8 ? (qs[2 * q + 1] & 15u) : (qs[2 * q - 15] >> 4);
                w[q >> 2] |= (lo | (hi << 4)) << (8 * (q & 3));
            }
        }
        *reinterpret_cast<uint4 *>(ab + 32 * m + 16 * (half ^ ((m >> 2) & 1))) = make_uint4(w[0], w[1], w[2], w[3]);
        sf[(m & 31) * 16 + (m >> 5) * 4 + 2 * (ks & 1) + half] = scale;
    }
}

}  // namespace

TRACE_SETTER(xtc)

struct xtc_plan {
    moearc_ctx *c;
    int H, I, E, K, gating, act;
    float alpha, limit;
    int grid_gu, grid_dn;  // at most the units of the launch: every CTA's share is non-empty
    int stages_gu, stages_dn, smem_gu, smem_dn;
    int tiles_gu, tiles_dn;
    int maxc_gu, maxc_dn;
    void *mem;
    uint8_t *xdig, *adig;
    float *part_gu, *part_dn;

};

namespace {

// Most contributors of a tile and most tiles of one CTA's share, for U units in groups of nkp.
void share_stats(long U, int G, int nkp, int &maxc, int &maxseg) {
    maxc = 1;
    maxseg = 0;
    for (long g = 0; g * nkp < U; ++g)
        maxc = std::max(maxc, unit_cta(U, G, g * nkp + nkp - 1) - unit_cta(U, G, g * nkp) + 1);
    for (int c = 0; c < G; ++c) {
        const long ua = U * c / G, ub = U * (c + 1) / G;
        if (ub > ua) maxseg = std::max(maxseg, (int)((ub - 1) / nkp - ua / nkp + 1));
    }
}

}  // namespace

xtc_plan *xtc_create(moearc_ctx *c, int H, int I, int E, int K, int gating, int act, float alpha, float limit) {
    if (H % 64 || I % 64 || K < 1 || K > XT_MAXK || E < K) return nullptr;
    auto *p = new xtc_plan();
    p->c = c;
    p->H = H;
    p->I = I;
    p->E = E;
    p->K = K;
    p->gating = gating;
    p->act = act;
    p->alpha = alpha;
    p->limit = limit;
    p->tiles_gu = I / 64;
    p->tiles_dn = (H + 127) / 128;
    // a tile's contributors are the run of CTAs between its first and last unit's, so no CTA of
    // the grid may have an empty share (it would never arrive on the tile's counter)
    const long u_gu = (long)K * p->tiles_gu * tc_kpairs(H), u_dn = (long)K * p->tiles_dn * tc_kpairs(I);
    p->grid_gu = (int)std::min<long>(c->sm_count, u_gu);
    p->grid_dn = (int)std::min<long>(c->sm_count, u_dn);
    int seg_gu = 0, seg_dn = 0;
    share_stats(u_gu, p->grid_gu, tc_kpairs(H), p->maxc_gu, seg_gu);
    share_stats(u_dn, p->grid_dn, tc_kpairs(I), p->maxc_dn, seg_dn);
    // shared memory: the ring, then the share's digits (at most ceil(U / grid) k-pairs)
    const int mu_gu = (int)((u_gu + p->grid_gu - 1) / p->grid_gu), mu_dn = (int)((u_dn + p->grid_dn - 1) / p->grid_dn);
    auto stages = [](int mu) { return std::min(XT_STAGES, (XT_SMEM_MAX - 1024 - mu * TC_BKPAIR) / XT_STAGE_A); };
    p->stages_gu = stages(mu_gu);
    p->stages_dn = stages(mu_dn);
    p->smem_gu = p->stages_gu * XT_STAGE_A + mu_gu * TC_BKPAIR + 1024;
    p->smem_dn = p->stages_dn * XT_STAGE_A + mu_dn * TC_BKPAIR + 1024;
    if (seg_gu > XT_MAXSEG || seg_dn > XT_MAXSEG || mu_gu > XT_MAXUNITS || mu_dn > XT_MAXUNITS || p->stages_gu < 2 ||
        p->stages_dn < 2) {
        delete p;
        return nullptr;
    }
    const size_t xd = tc_digit_bytes(H), ad = (size_t)K * tc_digit_bytes(I);
    const size_t pg = sizeof(float) * (size_t)K * p->tiles_gu * p->maxc_gu * 128;
    const size_t pd = sizeof(float) * (size_t)K * p->tiles_dn * p->maxc_dn * 128;
    auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t total = up(xd) + up(ad) + up(pg) + up(pd);
    if (cudaMalloc(&p->mem, total) != cudaSuccess) {
        cudaGetLastError();
        delete p;
        return nullptr;
    }
    uint8_t *b = static_cast<uint8_t *>(p->mem);
    p->xdig = b;
    b += up(xd);
    p->adig = b;
    b += up(ad);
    p->part_gu = reinterpret_cast<float *>(b);
    b += up(pg);
    p->part_dn = reinterpret_cast<float *>(b);
    static std::atomic<bool> ready[MOEARC_MAX_DEVICES];
    if (cudaMemsetAsync(p->mem, 0, total, c->stream) != cudaSuccess ||
        once_per_device(ready, [] {
            cudaError_t e = set_smem(k_xtc<0>, XT_SMEM_MAX);
            return e == cudaSuccess ? set_smem(k_xtc<1>, XT_SMEM_MAX) : e;
        }) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p->mem);
        delete p;
        return nullptr;
    }
    xtc_reset(p);
    return p;
}

void xtc_destroy(xtc_plan *p) {
    if (!p) return;
    cudaFree(p->mem);
    delete p;
}

int xtc_grid(const xtc_plan *p) { return p ? std::max(p->grid_gu, p->grid_dn) : 0; }
uint8_t *xtc_xdig(xtc_plan *p) { return p ? p->xdig : nullptr; }

void xtc_reset(xtc_plan *p) {
    if (!p) return;
    parts_empty(p->part_gu, (size_t)p->K * p->tiles_gu * p->maxc_gu * 128, p->c->stream, p->c->sm_count);
    parts_empty(p->part_dn, (size_t)p->K * p->tiles_dn * p->maxc_dn * 128, p->c->stream, p->c->sm_count);
}

namespace {

xtc_args common_args(xtc_plan *p, const xtc_run &r) {
    xtc_args a{};
    a.logits = r.logits;
    a.E = p->E;
    a.K = p->K;
    a.gating = p->gating;
    a.idx_pub = r.idx_out;
    a.wts_pub = r.wts_out;
    a.act = p->act;
    a.alpha = p->alpha;
    a.limit = p->limit;
    a.act_out = r.act_out;
    a.H = p->H;
    a.I = p->I;
    a.bias_gu = r.bias_gu;
    a.bias_dn = r.bias_dn;
    a.poll_ns = r.poll_ns;
    a.phantom = r.phantom;
    a.status = r.status;
    return a;
}

}  // namespace

int xtc_launch_gu(xtc_plan *p, const xtc_run &r) {
    xtc_args a = common_args(p, r);
    a.bank = r.gu_bank;
    a.bank_stride = tc_gu_stride(p->H, p->I);
    a.tile_bytes = tc_tile_bytes(p->H);
    a.tiles = p->tiles_gu;
    a.nkp = tc_kpairs(p->H);
    a.ksteps = tc_ksteps(p->H);
    a.stages = p->stages_gu;
    a.rows_last = 128;
    a.b_in = r.xdig;
    a.b_stride = 0;
    a.b_out = p->adig;
    a.b_out_stride = tc_digit_bytes(p->I);
    a.part = p->part_gu;
    a.maxc = p->maxc_gu;
    a.span = r.span;
    return launch_pdl(k_xtc<0>, dim3(p->grid_gu), dim3(XT_THREADS), (size_t)p->smem_gu, p->c->stream, a) == cudaSuccess ? OK
                                                                                                                : ERR;
}

int xtc_launch_dn(xtc_plan *p, const xtc_run &r) {
    xtc_args a = common_args(p, r);
    a.bank = r.dn_bank;
    a.bank_stride = tc_dn_stride(p->H, p->I);
    a.tile_bytes = tc_tile_bytes(p->I);
    a.tiles = p->tiles_dn;
    a.nkp = tc_kpairs(p->I);
    a.ksteps = tc_ksteps(p->I);
    a.stages = p->stages_dn;
    a.rows_last = p->H - 128 * (p->tiles_dn - 1);
    a.b_in = p->adig;
    a.b_stride = tc_digit_bytes(p->I);
    a.residual = r.residual;
    a.out = r.out;
    a.part = p->part_dn;
    a.maxc = p->maxc_dn;
    a.span = r.span ? r.span + (size_t)r.span_cta * 3 : nullptr;
    return launch_pdl(k_xtc<1>, dim3(p->grid_dn), dim3(XT_THREADS), (size_t)p->smem_dn, p->c->stream, a) == cudaSuccess ? OK
                                                                                                                : ERR;
}

int xtc_pack(moearc_ctx *c, int H, int I, const void *gate, const void *up, const void *down, unsigned n_expert,
             void *gu_tc, void *dn_tc) {
    if (H % 64 || I % 64 || !n_expert) return ERR_ARG;
    const size_t sg = tc_gu_stride(H, I), sd = tc_dn_stride(H, I);
    if (cudaMemsetAsync(gu_tc, 0, sg * n_expert, c->stream) != cudaSuccess ||
        cudaMemsetAsync(dn_tc, 0, sd * n_expert, c->stream) != cudaSuccess)
        return ERR;
    const int grid = c->sm_count * 8;
    k_xtc_pack<0><<<grid, 256, 0, c->stream>>>(static_cast<uint8_t *>(gu_tc), static_cast<const uint8_t *>(gate),
                                              static_cast<const uint8_t *>(up), I, H, I / 64, sg, n_expert);
    k_xtc_pack<1><<<grid, 256, 0, c->stream>>>(static_cast<uint8_t *>(dn_tc), static_cast<const uint8_t *>(down),
                                              nullptr, H, I, (H + 127) / 128, sd, n_expert);
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

}  // namespace moearc
