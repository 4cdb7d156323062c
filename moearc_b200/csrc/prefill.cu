// prefill.cu — the MoE FFN for prefill (many tokens per call) on the fifth-generation tensor
// cores: route every token, group the (token, expert) pairs by expert, and run the expert FFN as
// two grouped GEMMs on tcgen05 with operands loaded by TMA and accumulators in TMEM.
//
// The reference has no prefill path (its decode loop, crates/moearc-engine/src/moe.rs:2074-2427,
// runs one token at a time through matvec kernels); this is the same MoE block, token for token:
//   logits = router . x (+ bias)                         (the decode router's fixed fold order)
//   top-k, gating weights                                (reference.rs:599-639, shared route.cuh)
//   a[t,m] = act(W_gate[e] x, W_up[e] x)                 (SwiGLU / SwiGLU-OAI, reference.rs:369-396)
//   out[t] = residual[t] + sum_m w[t,m] (W_down[e] a[t,m])   (router order, moe.rs:2395-2421)
//
// Kernels, in stream order (no host round trip; the GEMMs read their tile counts on the device):
//   k_pf_logits   16 tokens x 32 experts per CTA; bf16 x -> f32, fixed lane order
//   k_pf_topk     one warp per token; expert counts
//   k_pf_scan     row offsets and 128-token tile counts per expert
//   k_pf_scatter  each (token, choice) gets a row of its expert's segment; x copied there (bf16)
//   k_pf_gemm<0>  gate-up: W_gate and W_up tiles of the same 128 features against 128 rows,
//                 two TMEM accumulators, SwiGLU in the epilogue, bf16 activations out
//   k_pf_gemm<1>  down: W_down tiles against the activations, f32 rows out
//   k_pf_combine  per token the router-weighted sum of its k rows, plus the residual
//
// Precision: expert weights are MXFP4 (E2M1 x e8m0: exact in bf16) or Q4_0 ((n - 8) d: rounded
// to bf16); activations are bf16 (the inputs as given; SwiGLU outputs rounded once); products
// accumulate in f32 in TMEM. The bound is the reference's bf16-activation tolerance.
//
// Weights: moearc_x_prefill_load expands a block's packed banks (moearc_x_moe_pack layout) into
// bf16 K-major matrices [E][2][n_ff][n_embd] (gate block, up block) and [E][n_embd][n_ff].
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "route.cuh"
#include "tc.cuh"
#include "tma.cuh"

using namespace moearc;

namespace {

constexpr int PF_BM = 128, PF_BN = 128, PF_BK = 64;
constexpr int PF4_BN_SMALL = 32;    // the 4-bit form's tile rows for decode-sized batches
constexpr int PF4_SMALL_ROWS = 16;  // ... taken while the mean rows per expert is at most this
constexpr int PF_TILE_BYTES = PF_BM * PF_BK * 2;  // one 128 x 64 bf16 operand tile (16 KB)
constexpr int PF_LOGIT_TOK = 16;                  // tokens per router CTA
constexpr int PF_LOGIT_EXP = 4;                   // experts a warp folds at once
constexpr int PF_STATUS_WAIT = 1;                 // a pipeline wait gave up
constexpr int PF_STATUS_RANGE = 2;                // 4-bit weights whose scaled values leave f16

__device__ __forceinline__ uint16_t f32_to_bf16_rn(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// ---- routing -------------------------------------------------------------------------------

struct pf_route_args {
    const uint16_t *x;  // [T][H] bf16
    const float *x32;   // [T][H] f32 the logits are taken from instead of x (null: x)
    const float *router, *rbias;
    int T, H, E, K, gating;
    float *logits;      // [T][E]
    unsigned *idx;      // [T][K]
    float *wts;         // [T][K]
    int *cnt;           // [E] counts by position, zeroed before
    const int *epos;    // [E] position of each expert in the row order
};

// Logits of PF_LOGIT_TOK tokens against every expert. Per (token, expert) the fold is that of
// moearc_matvec_f32 / the decode router: lane l accumulates float4 columns l, l + 32, ... with
// fmaf over x, y, z, w in turn, then an xor-shuffle tree. A warp folds PF_LOGIT_EXP experts
// against all PF_LOGIT_TOK tokens at once (64 accumulators a lane), so each router load from
// L2 and each activation load from shared memory feeds 16 and 4 folds.
__global__ void __launch_bounds__(256) k_pf_logits(pf_route_args a) {
    extern __shared__ __align__(16) float xs[];  // [PF_LOGIT_TOK][H]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * PF_LOGIT_TOK, nt = min(PF_LOGIT_TOK, a.T - t0);
    const int H = a.H, n4 = H / 4;
    // staged with 16-byte loads, eight in flight per thread (H is a multiple of 64)
    if (a.x32) {
        const float4 *src = reinterpret_cast<const float4 *>(a.x32 + (size_t)t0 * H);
        float4 *dst = reinterpret_cast<float4 *>(xs);
        const int n = nt * H / 4;
        for (int i0 = threadIdx.x; i0 < n; i0 += 8 * blockDim.x) {
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = i0 + j * blockDim.x;
                if (i < n) v[j] = src[i];
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = i0 + j * blockDim.x;
                if (i < n) dst[i] = v[j];
            }
        }
    } else {
        const uint4 *src = reinterpret_cast<const uint4 *>(a.x + (size_t)t0 * H);
        const int n = nt * H / 8;
        for (int i0 = threadIdx.x; i0 < n; i0 += 4 * blockDim.x) {
            uint4 v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = i0 + j * blockDim.x;
                if (i < n) v[j] = src[i];
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = i0 + j * blockDim.x;
                if (i < n) {
                    const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        xs[8 * i + 2 * e] = __uint_as_float(w[e] << 16);
                        xs[8 * i + 2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
                    }
                }
            }
        }
    }
    __syncthreads();
    const int nwarps = blockDim.x >> 5;
    // blockIdx.y: a group of nwarps * PF_LOGIT_EXP experts (a decode-sized batch has few token
    // groups, so the experts spread the work over more SMs)
    for (int e0 = (blockIdx.y * nwarps + warp) * PF_LOGIT_EXP; e0 < a.E; e0 += gridDim.y * nwarps * PF_LOGIT_EXP) {
        float acc[PF_LOGIT_EXP][PF_LOGIT_TOK];
#pragma unroll
        for (int j = 0; j < PF_LOGIT_EXP; ++j)
#pragma unroll
            for (int t = 0; t < PF_LOGIT_TOK; ++t) acc[j][t] = 0.f;
        // the router columns are loaded three steps ahead (few warps share an SM, and each step
        // would otherwise wait out a whole memory latency); every lane still adds its columns
        // c = lane, lane + 32, ... in ascending order
        auto load_w = [&](int c, float4 (&w)[PF_LOGIT_EXP]) {
#pragma unroll
            for (int j = 0; j < PF_LOGIT_EXP; ++j)
                w[j] = (c < n4 && e0 + j < a.E) ? __ldg(reinterpret_cast<const float4 *>(a.router + (size_t)(e0 + j) * H) + c)
                                                : make_float4(0.f, 0.f, 0.f, 0.f);
        };
        auto step = [&](int c, const float4 (&wv)[PF_LOGIT_EXP]) {
            if (c >= n4) return;
#pragma unroll
            for (int t = 0; t < PF_LOGIT_TOK; ++t) {
                const float4 xv = reinterpret_cast<const float4 *>(xs + (size_t)t * H)[c];
#pragma unroll
                for (int j = 0; j < PF_LOGIT_EXP; ++j) {
                    acc[j][t] = fmaf(wv[j].x, xv.x, acc[j][t]);
                    acc[j][t] = fmaf(wv[j].y, xv.y, acc[j][t]);
                    acc[j][t] = fmaf(wv[j].z, xv.z, acc[j][t]);
                    acc[j][t] = fmaf(wv[j].w, xv.w, acc[j][t]);
                }
            }
        };
        float4 w0[PF_LOGIT_EXP], w1[PF_LOGIT_EXP], w2[PF_LOGIT_EXP];
        load_w(lane, w0);
        load_w(lane + 32, w1);
        load_w(lane + 64, w2);
        for (int c = lane; c < n4; c += 96) {
            step(c, w0);
            load_w(c + 96, w0);
            step(c + 32, w1);
            load_w(c + 128, w1);
            step(c + 64, w2);
            load_w(c + 160, w2);
        }
#pragma unroll
        for (int j = 0; j < PF_LOGIT_EXP; ++j)
#pragma unroll
            for (int t = 0; t < PF_LOGIT_TOK; ++t) {
                float v = acc[j][t];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                const int e = e0 + j;
                if (lane == 0 && t < nt && e < a.E) a.logits[(size_t)(t0 + t) * a.E + e] = a.rbias ? v + a.rbias[e] : v;
            }
    }
}

// Token groups x expert groups (8 warps of PF_LOGIT_EXP experts each).
inline dim3 logit_grid(int T, int E) {
    return dim3((unsigned)((T + PF_LOGIT_TOK - 1) / PF_LOGIT_TOK), (unsigned)((E + 8 * PF_LOGIT_EXP - 1) / (8 * PF_LOGIT_EXP)));
}

// Top-k of each token (one warp per token) and the per-expert counts.
__global__ void __launch_bounds__(256) k_pf_topk(pf_route_args a) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= a.T) return;
    xtopk(a.logits + (size_t)t * a.E, a.E, a.K, a.gating, lane, a.idx + (size_t)t * a.K, a.wts + (size_t)t * a.K);
    __syncwarp();
    if (lane < a.K) atomicAdd(a.cnt + a.epos[__ldcg(a.idx + (size_t)t * a.K + lane)], 1);
}

// Row offsets (off[e], off[E] = T K), 128-row tile offsets (toff[e], toff[E] = all tiles) and
// zeroed cursors. One CTA; E <= 1024.
__global__ void k_pf_scan(const int *cnt, int E, int *off, int *toff, int *cursor, int bn = PF_BN) {
    __shared__ int s_c[1024], s_t[1024];
    const int e = threadIdx.x;
    const int c = e < E ? cnt[e] : 0;
    s_c[e] = c;
    s_t[e] = (c + bn - 1) / bn;
    __syncthreads();
    // inclusive scans (Hillis-Steele; E is small)
    for (int d = 1; d < (int)blockDim.x; d <<= 1) {
        const int vc = e >= d ? s_c[e - d] : 0, vt = e >= d ? s_t[e - d] : 0;
        __syncthreads();
        s_c[e] += vc;
        s_t[e] += vt;
        __syncthreads();
    }
    if (e < E) {
        off[e + 1] = s_c[e];
        toff[e + 1] = s_t[e];
        cursor[e] = 0;
    }
    if (e == 0) {
        off[0] = 0;
        toff[0] = 0;
    }
}

// One warp per (token, choice): its row in the segment of its expert's position (experts sit in
// the row order at epos[e]: the identity on one GPU, owner-major under expert parallelism), and
// the token's bf16 activation copied there. Rows within a segment are in arrival order; every row's results depend only on
// its own activation, so the order does not reach the output.
// Under expert parallelism with peer memory (dst_rows set): the row does not stay here but is
// stored straight into the receive buffer of the rank owning its position (positions are
// owner-major, n_local per rank): dst_rows[r] + (dst_base[r] + row - off[r * n_local]) rows.
__global__ void __launch_bounds__(256) k_pf_scatter(const uint16_t *x, const unsigned *idx, const int *epos, int T,
                                                    int K, int H, const int *off, int *cursor, int *perm,
                                                    uint16_t *xp, int to_f16, uint16_t *const *dst_rows,
                                                    const int *dst_base, int n_local) {
    const int lane = threadIdx.x & 31;
    const long p = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (p >= (long)T * K) return;
    int row = 0, pos = 0;
    if (lane == 0) {
        pos = epos[idx[p]];
        row = off[pos] + atomicAdd(cursor + pos, 1);
        perm[p] = row;
    }
    row = __shfl_sync(0xffffffffu, row, 0);
    pos = __shfl_sync(0xffffffffu, pos, 0);
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)(p / K) * H);
    uint4 *dst;
    if (dst_rows) {
        const int r = pos / n_local;
        dst = reinterpret_cast<uint4 *>(dst_rows[r] + (size_t)(dst_base[r] + row - off[r * n_local]) * H);
    } else {
        dst = reinterpret_cast<uint4 *>(xp + (size_t)row * H);
    }
    if (!to_f16) {
        for (int i = lane; i < H / 8; i += 32) dst[i] = __ldg(src + i);
        if (dst_rows) __threadfence_system();  // peer stores performed before the kernel ends
        return;
    }
    // the 4-bit path's f16 operands: bf16 -> f16 (exact within f16's range)
    for (int i = lane; i < H / 8; i += 32) {
        const uint4 v = __ldg(src + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 h = __floats2half2_rn(__uint_as_float(w[j] << 16), __uint_as_float(w[j] & 0xFFFF0000u));
            o[j] = *reinterpret_cast<const uint32_t *>(&h);
        }
        dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    if (dst_rows) __threadfence_system();
}

// out[t] = residual[t] + sum_m w[t,m] y[perm[t,m]] (fmaf chain, m ascending).
__global__ void __launch_bounds__(256) k_pf_combine(const float *y, const int *perm, const float *wts, const float *residual,
                                                    float *out, int T, int K, int H) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)T * H) return;
    const int t = (int)(i / H), h = (int)(i - (long)t * H);
    float acc = 0.f;
    for (int m = 0; m < K; ++m) acc = fmaf(wts[t * K + m], y[(size_t)perm[t * K + m] * H + h], acc);
    out[i] = residual ? residual[i] + acc : acc;
}

// ---- weights: packed tiles -> bf16 K-major -----------------------------------------------

// One warp per packed tile (16 rows x 64 columns). mats = 2: gate-up pairs (gate tile, up
// tile) -> dst [E][2][R][Kc]; mats = 1: down tiles -> dst [E][R][Kc]. R rows, Kc columns per
// matrix; tiles run tile-row-major per expert. The warp decodes its tile into shared memory and
// writes it out as 16 rows of 128 contiguous bytes (16-byte stores).
template <int WT>
__global__ void __launch_bounds__(256) k_pf_unpack(const uint8_t *bank, int E, int R, int Kc, int mats, int tile_bytes,
                                                   uint16_t *dst) {
    __shared__ __align__(16) uint16_t stage[8][16 * 64];
    const int lane = threadIdx.x & 31, r = lane >> 2, q = lane & 3;
    uint16_t *tl = stage[threadIdx.x >> 5];
    const long ntr = R / 16, nkt = Kc / 64;
    const long per_e = ntr * nkt * mats;
    const long g = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (g >= (long)E * per_e) return;
    const int e = (int)(g / per_e);
    const long rem = g - e * per_e;
    const long pair = rem / mats;
    const int mat = (int)(rem - pair * mats);
    const int tr = (int)(pair / nkt), kt = (int)(pair - (long)tr * nkt);
    const uint8_t *tile = bank + (size_t)g * tile_bytes;
    const uint4 w = *reinterpret_cast<const uint4 *>(tile + lane * 16);
    float s[4];
    scales4<WT>(tile, r, s);
    uint16_t *m = dst + ((size_t)e * mats + mat) * (size_t)R * Kc;
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};  // (row r, blk 0), (r+8, 0), (r, 1), (r+8, 1)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t pr[4];
        decode4<WT>(words[i], pr);
        const int lrow = r + ((i & 1) ? 8 : 0), blk = i >> 1;
        const float sc = s[blk * 2 + (i & 1)];
        uint16_t *dr = tl + lrow * 64 + blk * 32;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 h = *reinterpret_cast<const __half2 *>(&pr[j]);
            dr[4 * q + j] = f32_to_bf16_rn(__low2float(h) * sc);
            dr[4 * q + j + 16] = f32_to_bf16_rn(__high2float(h) * sc);
        }
    }
    __syncwarp();
    // 16 rows x 8 chunks of 16 bytes: lane takes chunks lane, lane + 32, ...
#pragma unroll
    for (int c = lane; c < 128; c += 32) {
        const int row = c >> 3, ch = c & 7;
        *reinterpret_cast<uint4 *>(m + (size_t)(tr * 16 + row) * Kc + kt * 64 + ch * 8) =
            *reinterpret_cast<const uint4 *>(tl + row * 64 + ch * 8);
    }
}

// ---- the grouped GEMM on tcgen05 ------------------------------------------------------------

struct pf_gemm_args {
    int Mrows;        // feature rows of one matrix per expert (gate-up: n_ff; down: n_embd)
    int K;            // reduction length (gate-up: n_embd; down: n_ff)
    int E;            // segments (runs of rows of one expert; one per expert on one GPU)
    const int *off;   // [E + 1] row offsets of the segments
    const int *toff;  // [E + 1] 128-row tile offsets
    const int *seg_w; // [E] expert (weight block) of each segment; null: segment e is expert e
    int act;          // gate-up epilogue
    float alpha, limit;
    uint16_t *act_out;  // gate-up: [rows][n_ff] bf16
    float *y_out;       // down: [rows][n_embd] f32
    float *const *seg_y;  // down, if set: segment e's rows go to seg_y[e] + n * n_embd instead (a peer
                          // rank's memory under expert parallelism: the return leg of the exchange)
    // per-expert biases indexed by weight block w (moe.rs:2310-2331, 2362-2372), or null:
    // gate-up: gate rows of block w at w, up rows at n_blocks + w ([2 n_blocks][Mrows]), added
    // before the activation; down: [n_blocks][Mrows], added to each row before the combine
    const float *bias;
    int n_blocks;
    int *status;
    // down only (the dense projections of a decode-sized batch): the K blocks split into ksplit
    // runs (<= K / 64), each tile's partial sum written to y_out + ks * split_stride; 0 or 1: none
    int ksplit;
    size_t split_stride;
};

template <int MODE>
struct pf_cfg {
    static constexpr int NA = MODE == 0 ? 2 : 1;  // A tiles per stage (gate and up, or down)
    static constexpr int STAGE = (NA + 1) * PF_TILE_BYTES;
    static constexpr int STAGES = MODE == 0 ? 4 : 6;
    static constexpr int SMEM = STAGES * STAGE + 1024;
    static constexpr int ACC_COLS = NA * PF_BN;      // one accumulator set (gate + up, or down)
    static constexpr int TMEM_COLS = 2 * ACC_COLS;   // two sets: the epilogue of tile i overlaps
                                                     // the MMAs of tile i + 1
};

// Persistent: CTA b takes tiles b, b + grid, ...; tile = (n-tile over all experts' segments,
// m-tile of features), features fastest so CTAs running together share a row block in L2.
// Warp 0: TMA producer (and TMEM owner); warp 1: MMA issuer; warps 2-5: epilogue (warp w reads
// TMEM lanes 32 (w % 4) ..). Stages cycle across tiles; two accumulator sets (tile i uses set
// i % 2), each handed between the MMA issuer and the epilogue by acc_full (tcgen05.commit) and
// acc_empty (4 epilogue warps).
template <int MODE>
__global__ void __launch_bounds__(192, 1) k_pf_gemm(const __grid_constant__ CUtensorMap wmap,
                                                    const __grid_constant__ CUtensorMap xmap, pf_gemm_args a) {
    using C = pf_cfg<MODE>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full[C::STAGES], empty[C::STAGES], acc_full[2], acc_empty[2], done;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_;
    __shared__ int s_toff[1025];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i <= a.E; i += blockDim.x) s_toff[i] = a.toff[i];
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            tc::bar_init(&full[s], 1);
            tc::bar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::bar_init(&acc_full[b], 1);
            tc::bar_init(&acc_empty[b], 4);
        }
        tc::bar_init(&done, 1);
        abort_ = 0;
        tc::bar_init_fence();
    }
    if (warp == 0) tc::tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    const int MT = (a.Mrows + PF_BM - 1) / PF_BM, KB = a.K / PF_BK;
    const int KS = (MODE == 1 && a.ksplit > 1) ? a.ksplit : 1;  // K runs (tile % KS: the run)
    const long total = (long)s_toff[a.E] * MT * KS;
    // tile -> expert, n-tile within the expert, m-tile
    auto locate = [&](long tile, int &e, int &nt, int &mt) {
        const int ntg = (int)(tile / MT);
        mt = (int)(tile - (long)ntg * MT);
        int lo = 0, hi = a.E;  // largest e with s_toff[e] <= ntg (empty experts skipped)
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (s_toff[mid] <= ntg) lo = mid;
            else hi = mid;
        }
        e = lo;
        nt = ntg - s_toff[e];
    };

    if (warp == 0) {
        long g = 0;  // k-blocks issued (lane 0)
        if (lane == 0) {
            for (long tile = blockIdx.x; tile < total && !abort_; tile += gridDim.x) {
                int e, nt, mt;
                const int ks = (int)(tile % KS);
                locate(tile / KS, e, nt, mt);
                const int we = a.seg_w ? a.seg_w[e] : e;
                const int rowA = MODE == 0 ? we * 2 * a.Mrows + mt * PF_BM : we * a.Mrows + mt * PF_BM;
                const int rowB = a.off[e] + nt * PF_BN;
                for (int kb = ks * KB / KS; kb < (ks + 1) * KB / KS; ++kb, ++g) {
                    const int s = (int)(g % C::STAGES);
                    if (g >= C::STAGES && !tc::bar_wait(&empty[s], (unsigned)(((g / C::STAGES) - 1) & 1), &abort_, a.status, PF_STATUS_WAIT))
                        break;
                    uint8_t *st = smem + (size_t)s * C::STAGE;
                    tc::bar_expect_tx(&full[s], C::STAGE);
                    tc::tma_load_2d(st, &wmap, kb * PF_BK, rowA, &full[s]);
                    if (MODE == 0) tc::tma_load_2d(st + PF_TILE_BYTES, &wmap, kb * PF_BK, rowA + a.Mrows, &full[s]);
                    tc::tma_load_2d(st + C::NA * PF_TILE_BYTES, &xmap, kb * PF_BK, rowB, &full[s]);
                }
            }
            if (abort_)  // let every issued copy land (bounded) before the CTA exits
                for (long j = std::max(0L, g - C::STAGES); j < g; ++j)
                    tc::bar_drain(&full[j % C::STAGES], (unsigned)((j / C::STAGES) & 1));
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_bf16_f32(PF_BM, PF_BN);
            long g = 0, i = 0;
            for (long tile = blockIdx.x; tile < total && !abort_; tile += gridDim.x, ++i) {
                const int ab = (int)(i & 1);
                const uint32_t dcol = tmem + (uint32_t)(ab * C::ACC_COLS);
                if (i >= 2 && !tc::bar_wait(&acc_empty[ab], (unsigned)(((i >> 1) - 1) & 1), &abort_, a.status, PF_STATUS_WAIT))
                    break;
                tc::fence_after_sync();
                bool ok = true;
                const int ks = (int)(tile % KS), kb0 = ks * KB / KS;
                for (int kb = kb0; kb < (ks + 1) * KB / KS; ++kb, ++g) {
                    const int s = (int)(g % C::STAGES);
                    if (!tc::bar_wait(&full[s], (unsigned)((g / C::STAGES) & 1), &abort_, a.status, PF_STATUS_WAIT)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t a0 = tc::sa(smem + (size_t)s * C::STAGE);
                    const uint32_t b0 = a0 + C::NA * PF_TILE_BYTES;
#pragma unroll
                    for (int k = 0; k < PF_BK / 16; ++k) {
                        const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
                        tc::mma_bf16(dcol, tc::desc_k_sw128(a0 + k * 32), tc::desc_k_sw128(b0 + k * 32), idesc, acc);
                        if (MODE == 0)
                            tc::mma_bf16(dcol + PF_BN, tc::desc_k_sw128(a0 + PF_TILE_BYTES + k * 32),
                                         tc::desc_k_sw128(b0 + k * 32), idesc, acc);
                    }
                    tc::mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
                }
                if (!ok) break;
                tc::mma_commit(&acc_full[ab]);
            }
            // every MMA issued has completed before the columns can be freed
            tc::mma_commit(&done);
            tc::bar_drain(&done, 0);
        }
        __syncwarp();
    } else {
        const int qd = warp & 3;  // TMEM lane quarter
        const uint32_t lane_base = tmem + ((uint32_t)(32 * qd) << 16);
        long i = 0;
        for (long tile = blockIdx.x; tile < total; tile += gridDim.x, ++i) {
            const int ab = (int)(i & 1);
            if (!tc::bar_wait(&acc_full[ab], (unsigned)((i >> 1) & 1), &abort_, a.status, PF_STATUS_WAIT)) break;
            tc::fence_after_sync();
            int e, nt, mt;
            const int ks = (int)(tile % KS);
            locate(tile / KS, e, nt, mt);
            const int seg = a.off[e], n_rows = a.off[e + 1] - seg;
            const int f = mt * PF_BM + 32 * qd + lane;  // this thread's feature row
            const bool fok = f < a.Mrows;
            const uint32_t acc_base = lane_base + (uint32_t)(ab * C::ACC_COLS);
            // this row's biases (gate-up: gate, up; down: the row's)
            const int wblk = a.seg_w ? a.seg_w[e] : e;
            const float bg = (a.bias && fok) ? a.bias[(size_t)wblk * a.Mrows + f] : 0.f;
            const float bu = (MODE == 0 && a.bias && fok) ? a.bias[(size_t)(a.n_blocks + wblk) * a.Mrows + f] : 0.f;
            for (int c0 = 0; c0 < PF_BN; c0 += 16) {
                float d[16];
                tc::tmem_ld16(acc_base + c0, d);
                if (MODE == 0) {
                    float u[16];
                    tc::tmem_ld16(acc_base + PF_BN + c0, u);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = nt * PF_BN + c0 + j;
                        if (fok && n < n_rows)
                            a.act_out[(size_t)(seg + n) * a.Mrows + f] =
                                f32_to_bf16_rn(act_fn(a.act, d[j] + bg, u[j] + bu, a.alpha, a.limit));
                    }
                } else {
                    float *ybase = a.seg_y ? a.seg_y[e] : a.y_out + ks * a.split_stride + (size_t)seg * a.Mrows;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = nt * PF_BN + c0 + j;
                        if (fok && n < n_rows) ybase[(size_t)n * a.Mrows + f] = d[j] + bg;
                    }
                }
            }
            if (MODE == 1 && a.seg_y) __threadfence_system();  // peer stores performed
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::bar_arrive(&acc_empty[ab]);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ---- 4-bit expert weights on the tensor cores ---------------------------------------------------
//
// "tc4" layout of one weight matrix [R][K] (R rounded up to 128): chunks of 128 rows x 64 columns,
// chunk (rb, kb) at index rb * (K / 64) + kb, each one contiguous run: 128 rows of 32 bytes (byte j
// holds column 2j in its low nibble and 2j + 1 in its high nibble), then the rows' two block
// scales (MXFP4: one e8m0 byte per 32 columns; Q4_0: one f16 delta). Rows past R are zeros. A
// chunk is one bulk copy; decoder warps turn it into an f16 operand tile for the MMA (one
// conversion and one multiply per pair of weights). The whole 4-bit path runs in f16 (weights,
// activations, SwiGLU outputs; A and B of an MMA always share the type): the MXFP4 weights are
// exact in f16 while their e8m0 exponents lie in [105, 140] (the pack kernel checks, and the load
// refuses weights outside it), Q4_0's (n - 8) d rounds once to f16, and bf16 activations convert
// exactly.

constexpr int TC4_NIB = 128 * 32;  // nibble bytes of a chunk

template <int WT>
constexpr int tc4_sb() { return WT == 39 ? 1 : 2; }
template <int WT>
constexpr int tc4_chunk() { return TC4_NIB + 128 * 2 * tc4_sb<WT>(); }  // 4352 (MXFP4) or 4608 (Q4_0)

// One thread per (chunk, row): the row's 64 nibbles and 2 scales gathered from the packed tiles
// (moearc_x_moe_pack layout; mats = 2: gate-up pairs, 1: down tiles) of experts[i] -> slot i.
template <int WT>
__global__ void k_pf_pack4(const uint8_t *bank, const int *experts, int n_exp, int R, int K, int mats,
                           int tile_bytes, uint8_t *dst, int *status) {
    constexpr int sb = tc4_sb<WT>();
    const int RB = (R + 127) / 128, KB = K / 64;
    const long per_mat = (long)RB * KB;
    const long gid = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (gid >= (long)n_exp * mats * per_mat * 128) return;
    const int row = (int)(gid & 127);
    const long chunk = gid >> 7;
    const long em = chunk / per_mat;
    const int slot = (int)(em / mats), mat = (int)(em - (long)slot * mats);
    const long rk = chunk - em * per_mat;
    const int rb = (int)(rk / KB), kb = (int)(rk - (long)rb * KB);
    uint8_t *out = dst + (size_t)chunk * tc4_chunk<WT>();
    const int grow = rb * 128 + row;
    uint32_t nib[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    uint8_t sc[2 * sb];
    if (grow >= R) {
        for (int i = 0; i < 8; ++i) nib[i] = WT == 39 ? 0u : 0x88888888u;
        for (int i = 0; i < 2 * sb; ++i) sc[i] = 0;
    } else {
        const int e = experts ? experts[slot] : slot;
        const long ntr = R / 16, nkt = K / 64;
        const int tr = grow >> 4, lr = grow & 15, r = lr & 7, half = lr >> 3;
        const uint8_t *tile = bank + (((size_t)e * ntr * nkt + (size_t)tr * nkt + kb) * mats + mat) * tile_bytes;
        for (int k = 0; k < 64; ++k) {
            const int b = k >> 5, kk = k & 31, j = kk & 15;
            const uint8_t byte = tile[(4 * r + (j >> 2)) * 16 + (half + 2 * b) * 4 + (j & 3)];
            const uint32_t v = (kk >= 16) ? (byte >> 4) : (byte & 15u);
            nib[k >> 3] |= v << (4 * (k & 7));
        }
        for (int b = 0; b < 2; ++b)
            for (int i = 0; i < sb; ++i) sc[b * sb + i] = tile[512 + r * 4 * sb + (half + 2 * b) * sb + i];
        // f16 must hold every scaled value exactly (MXFP4: 0.5 .. 6 times 2^(e - 127), e = 0 for an
        // all-zero block) or at least in range (Q4_0: 8 |d| <= 65504)
        bool bad = false;
        for (int b = 0; b < 2; ++b) {
            if constexpr (WT == 39) {
                const int e = sc[b];
                bad |= e != 0 && (e < 105 || e > 140);
            } else {
                const float d = fabsf(f16_bits_to_f32((uint16_t)(sc[2 * b] | (sc[2 * b + 1] << 8))));
                bad |= !(d * 8.0f <= 65504.0f);
            }
        }
        if (bad) atomicOr(status, PF_STATUS_RANGE);
    }
    uint4 *o = reinterpret_cast<uint4 *>(out + row * 32);
    o[0] = make_uint4(nib[0], nib[1], nib[2], nib[3]);
    o[1] = make_uint4(nib[4], nib[5], nib[6], nib[7]);
    for (int i = 0; i < 2 * sb; ++i) out[TC4_NIB + row * 2 * sb + i] = sc[i];
}

// ---- MXFP8 mode: block-scaled FP8 GEMMs (tcgen05.mma kind::mxf8f6f4) ----------------------
//
// A perf mode beside the exact bf16 one. Weights: MXFP4 elements are E2M1 values, each exactly an
// E4M3 value, and their E8M0 block scale is the MMA's block scale, so the weights enter the MMA
// exactly (1 byte an element, the scale a byte per 32). Activations (the expert rows and the
// SwiGLU output) are quantised to MXFP8 per 32 along K: scale 2^X with X the smallest exponent
// that keeps the block's largest magnitude within E4M3's 448 (no saturation), elements E4M3 round
// to nearest even. The quantisation of the activations is the mode's only change of arithmetic;
// the oracle restates it (or_moe_ffn_token_mx8).
//
// Scale factors in TMEM (measured on B200): for M = 128, row m's scale for the MMA's K block is
// byte sf_id of lane m, column base + m / 32; for N <= 128, column n's at lane n % 32, column
// base + n / 32. tcgen05.cp.32x128b.warpx4 copies a 32-row x 16-byte shared-memory block to every
// lane quarter (row i, word c -> lane 32 q + i, column c), so one 512-byte block — row i, word
// c = the 4 K blocks' scales of matrix row 32 c + i — feeds one operand's scales for a 128-wide
// K stage (sf_id = K block 0..3).
constexpr int PF8_BN = 96, PF8_BK = 128;           // token rows per tile; K elements (bytes) a stage
constexpr int PF8_ATILE = PF_BM * PF8_BK;          // 16 KB: 128 feature rows x 128 E4M3
constexpr int PF8_BTILE = PF8_BN * PF8_BK;         // 12 KB
constexpr int PF8_SFBLK = 512;                     // one 32 x 16-byte scale block

template <int MODE>
struct pf8_cfg {
    static constexpr int NA = MODE == 0 ? 2 : 1;
    static constexpr int STAGE = ((NA * PF8_ATILE + PF8_BTILE + (NA + 1) * PF8_SFBLK + 1023) / 1024) * 1024;
    static constexpr int STAGES = MODE == 0 ? 4 : 6;
    static constexpr int SMEM = STAGES * STAGE + 1024;
    static constexpr int ACC_COLS = NA * PF8_BN;
    static constexpr int SF_BASE = 2 * ACC_COLS;    // after the two accumulator sets
    static constexpr int SF_SLOT = (NA + 1) * 4;    // one stage's scale columns (two slots alternate)
    static constexpr int TMEM_COLS = MODE == 0 ? 512 : 256;
    static_assert(SF_BASE + 2 * SF_SLOT <= TMEM_COLS, "TMEM columns");
};

// Scales are stored the way a stage consumes them: per (row tile, K stage) one 512-byte block,
// row i (16 bytes) word c = the 4 scale bytes (K blocks 4 kb .. 4 kb + 3) of tile row 32 c + i.
// A stage then fetches each operand's scales with one bulk copy. Byte offset of (tile row r,
// 32-element K block b) inside tile t of a matrix with kbs stages: ((t kbs + b / 4) 512 + (r % 32)
// 16 + (r / 32) 4 + b % 4. Unwritten bytes (rows past the matrix, K blocks past its end) hold
// 127, a scale of 1 on zeros.
__host__ __device__ __forceinline__ size_t sf_at(long tile, int kbs, int r, int b) {
    return ((size_t)tile * kbs + (b >> 2)) * PF8_SFBLK + (size_t)(r & 31) * 16 + (size_t)(r >> 5) * 4 + (b & 3);
}
__host__ __device__ __forceinline__ int sf_stages(int k) { return (k + PF8_BK - 1) / PF8_BK; }

// MXFP8 scale exponent of a block whose largest magnitude is amax: the smallest X with
// amax / 2^X <= 448 (448 = 1.75 x 2^8): X = e - 8 if the significand of amax is at most 1.75,
// else e - 7. 0 for a zero block.
__device__ __forceinline__ int mx8_exp(float amax) {
    const uint32_t b = __float_as_uint(amax);
    if (amax == 0.f) return 0;
    const int e = (int)((b >> 23) & 0xFF) - 127;
    return max(-127, e - 8 + (((b & 0x7FFFFF) > 0x600000u) ? 1 : 0));
}

__device__ __forceinline__ uint8_t to_e4m3(float v) {
    return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

// 2^-X for X in [-127, 126], built from the exponent bits: v * pow2_neg(X) is v scaled exactly
// (rounded once, as ldexpf would, when the product leaves the normal range).
__device__ __forceinline__ float pow2_neg(int X) { return __int_as_float((127 - X) << 23); }

// One warp per packed tile (16 rows x 64 columns): MXFP4 -> E4M3 rows dst[E][mats][R][Kc] and
// the scale bytes (the e8m0 byte itself: E2M1 value x 2^(e - 127)) in blocks per (expert, matrix,
// 128-row tile, K stage).
__global__ void __launch_bounds__(256) k_pf_unpack8(const uint8_t *bank, int E, int R, int Kc, int mats, int tile_bytes,
                                                    uint8_t *dst, uint8_t *sdst) {
    // E2M1 code -> E4M3 byte of the same value: 0, 0.5 = 0x30, and m / 2 = (m >= 2) 0x30 + 4 m
    auto e4 = [](uint32_t code) -> uint32_t {
        const uint32_t m = code & 7;
        return ((code & 8) << 4) | (m == 0 ? 0u : (m == 1 ? 0x30u : 0x30u + 4u * m));
    };
    const int lane = threadIdx.x & 31, r = lane >> 2, q = lane & 3;
    const long ntr = R / 16, nkt = Kc / 64;
    const long per_e = ntr * nkt * mats;
    const long g = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (g >= (long)E * per_e) return;
    const int e = (int)(g / per_e);
    const long rem = g - e * per_e;
    const long pair = rem / mats;
    const int mat = (int)(rem - pair * mats);
    const int tr = (int)(pair / nkt), kt = (int)(pair - (long)tr * nkt);
    const uint8_t *tile = bank + (size_t)g * tile_bytes;
    const uint4 w = *reinterpret_cast<const uint4 *>(tile + lane * 16);
    const size_t mbase = ((size_t)e * mats + mat) * (size_t)R;
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};  // (row r, blk 0), (r+8, 0), (r, 1), (r+8, 1)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = tr * 16 + r + ((i & 1) ? 8 : 0), blk = i >> 1;
        uint8_t *d = dst + (mbase + row) * (size_t)Kc + kt * 64 + blk * 32;
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t byte = (words[i] >> (8 * j)) & 0xFF;
            lo |= e4(byte & 15) << (8 * j);
            hi |= e4(byte >> 4) << (8 * j);
        }
        *reinterpret_cast<uint32_t *>(d + 4 * q) = lo;        // elements 4q .. 4q + 3
        *reinterpret_cast<uint32_t *>(d + 16 + 4 * q) = hi;   // elements 16 + 4q ..
        if (q == 0)
            sdst[sf_at(((long)e * mats + mat) * ((R + PF_BM - 1) / PF_BM) + row / PF_BM, sf_stages(Kc), row % PF_BM,
                       kt * 2 + blk)] = tile[512 + 4 * r + i];
    }
}

// k_pf_scatter with MXFP8 rows: one warp per (token, choice), its row as k_pf_scatter places it;
// each 32-element block of the token's bf16 activation quantised (x8 [rows][H] E4M3; the scales
// in the blocks of the row's 96-row tile, toff the segments' tile offsets).
__global__ void __launch_bounds__(256) k_pf_scatter8(const uint16_t *x, const unsigned *idx, const int *epos, int T,
                                                     int K, int H, const int *off, const int *toff, int *cursor,
                                                     int *perm, uint8_t *x8, uint8_t *sx) {
    const int lane = threadIdx.x & 31;
    const long p = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (p >= (long)T * K) return;
    int row = 0, pos = 0, n = 0;
    if (lane == 0) {
        pos = epos[idx[p]];
        n = atomicAdd(cursor + pos, 1);
        row = off[pos] + n;
        perm[p] = row;
    }
    row = __shfl_sync(0xffffffffu, row, 0);
    pos = __shfl_sync(0xffffffffu, pos, 0);
    n = __shfl_sync(0xffffffffu, n, 0);
    const long tile = toff[pos] + n / PF8_BN;
    const int kbs = sf_stages(H);
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)(p / K) * H);
    // lane l takes elements 8 l .. 8 l + 7 of each 256-element chunk: four lanes form a block
    for (int c0 = 0; c0 < H; c0 += 256) {
        const int e0 = c0 + 8 * lane;
        const bool live = e0 < H;
        float v[8];
        if (live) {
            const uint4 w = __ldg(src + e0 / 8);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[2 * j] = __uint_as_float(ws[j] << 16);
                v[2 * j + 1] = __uint_as_float(ws[j] & 0xFFFF0000u);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = 0.f;
        }
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[j]));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        const int X = mx8_exp(m);
        if (live) {
            uint32_t lo = 0, hi = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                lo |= (uint32_t)to_e4m3(v[j] * pow2_neg(X)) << (8 * j);
                hi |= (uint32_t)to_e4m3(v[4 + j] * pow2_neg(X)) << (8 * j);
            }
            *reinterpret_cast<uint2 *>(x8 + (size_t)row * H + e0) = make_uint2(lo, hi);
            if ((lane & 3) == 0) sx[sf_at(tile, kbs, n % PF8_BN, e0 / 32)] = (uint8_t)(127 + X);
        }
    }
}

struct pf8_args {
    int Mrows, K, E;
    const int *off, *toff, *seg_w;
    int act;
    float alpha, limit;
    const uint8_t *sfw;    // weight scale blocks [expert][NA][128-row tile][K stage]
    const uint8_t *sfx;    // activation scale blocks [96-row tile][K stage]
    uint8_t *act8;         // gate-up: E4M3 activations [rows][Mrows]
    uint8_t *sact;         // gate-up: their scale blocks [96-row tile][Mrows stage]
    float *y_out;          // down: [rows][Mrows] f32
    const float *bias;     // as pf_gemm_args
    int n_blocks;
    int *status;
};

// Shared-memory descriptor of a 32-row x 16-byte block (no swizzle: rows 16 bytes apart, 8-row
// core matrices 128 bytes apart), the source of tcgen05.cp.32x128b.
__device__ __forceinline__ uint64_t desc_sfblk(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 32) | ((uint64_t)1 << 46);
}

// Block-scaled instruction descriptor (kind::mxf8f6f4): A and B E4M3 (formats 0), K-major, N >> 3
// in bits 17-22, E8M0 scales (bit 23), M >> 4 in bits 24-28, scale ids for B (bits 4-5) and A
// (bits 29-30).
__host__ __device__ constexpr uint32_t idesc_mx8(int M, int N, int sf_id) {
    return ((uint32_t)sf_id << 4) | ((uint32_t)(N >> 3) << 17) | (1u << 23) | ((uint32_t)(M >> 4) << 24) |
           ((uint32_t)sf_id << 29);
}

__device__ __forceinline__ void mma_mx8(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                        uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %6, 0;\n"
        " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], p; }" ::"r"(d),
        "l"(da), "l"(db), "r"(idesc), "r"(sfa), "r"(sfb), "r"(acc));
}

__device__ __forceinline__ void cp_sf(uint32_t taddr, uint32_t saddr) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc_sfblk(saddr)));
}

// The MXFP8 GEMMs, laid out as k_pf_gemm (persistent, warp 0 producer and TMEM owner, warp 1 MMA
// issuer, two accumulator sets) but with eight epilogue warps (2-9: warp w reads TMEM lane quarter
// w % 4, columns of half (w - 2) / 4 of the tile) with tiles of 128 features x 96 rows and K
// stages of 128 bytes. Warp 0's lanes also gather each stage's scale blocks (lane i: matrix rows
// 32 c + i) into shared memory; the stage's full barrier waits for the TMA bytes and for that.
// The MMA issuer copies the blocks into TMEM (two slots, alternating by stage) ahead of the
// stage's MMAs; tcgen05 operations of one thread run in issue order. Gate-up's epilogue writes
// the SwiGLU output as MXFP8 (a warp's 32 lanes are one 32-feature block).
constexpr int PF8_THREADS = 320;

template <int MODE>
__global__ void __launch_bounds__(PF8_THREADS, 1) k_pf_gemm8(const __grid_constant__ CUtensorMap wmap,
                                                     const __grid_constant__ CUtensorMap xmap, pf8_args a) {
    using C = pf8_cfg<MODE>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full[C::STAGES], empty[C::STAGES], acc_full[2], acc_empty[2], done;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_;
    __shared__ int s_toff[1025];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i <= a.E; i += blockDim.x) s_toff[i] = a.toff[i];
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            tc::bar_init(&full[s], 1);
            tc::bar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::bar_init(&acc_full[b], 1);
            tc::bar_init(&acc_empty[b], 8);
        }
        tc::bar_init(&done, 1);
        abort_ = 0;
        tc::bar_init_fence();
    }
    if (warp == 0) tc::tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    const int MT = (a.Mrows + PF_BM - 1) / PF_BM, KB = sf_stages(a.K);
    const long total = (long)s_toff[a.E] * MT;
    auto locate = [&](long tile, int &e, int &nt, int &mt) {
        const int ntg = (int)(tile / MT);
        mt = (int)(tile - (long)ntg * MT);
        int lo = 0, hi = a.E;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (s_toff[mid] <= ntg) lo = mid;
            else hi = mid;
        }
        e = lo;
        nt = ntg - s_toff[e];
    };

    if (warp == 0) {
        long g = 0;  // k-blocks issued (lane 0)
        if (lane == 0) {
            for (long tile = blockIdx.x; tile < total && !abort_; tile += gridDim.x) {
                int e, nt, mt;
                locate(tile, e, nt, mt);
                const int we = a.seg_w ? a.seg_w[e] : e;
                const long rowA = MODE == 0 ? (long)we * 2 * a.Mrows + mt * PF_BM : (long)we * a.Mrows + mt * PF_BM;
                const long rowB = a.off[e] + (long)nt * PF8_BN;
                const uint8_t *sfa = a.sfw + (((size_t)we * C::NA) * MT + mt) * KB * PF8_SFBLK;
                const uint8_t *sfb = a.sfx + (size_t)(s_toff[e] + nt) * KB * PF8_SFBLK;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int s = (int)(g % C::STAGES);
                    if (g >= C::STAGES &&
                        !tc::bar_wait(&empty[s], (unsigned)(((g / C::STAGES) - 1) & 1), &abort_, a.status, PF_STATUS_WAIT))
                        break;
                    uint8_t *st = smem + (size_t)s * C::STAGE;
                    uint8_t *sfs = st + C::NA * PF8_ATILE + PF8_BTILE;
                    tc::bar_expect_tx(&full[s], C::NA * PF8_ATILE + PF8_BTILE + (C::NA + 1) * PF8_SFBLK);
                    tc::tma_load_2d(st, &wmap, kb * PF8_BK, (int)rowA, &full[s]);
                    if (MODE == 0) tc::tma_load_2d(st + PF8_ATILE, &wmap, kb * PF8_BK, (int)(rowA + a.Mrows), &full[s]);
                    tc::tma_load_2d(st + C::NA * PF8_ATILE, &xmap, kb * PF8_BK, (int)rowB, &full[s]);
#pragma unroll
                    for (int mat = 0; mat < C::NA; ++mat)
                        bulk_g2s(sfs + mat * PF8_SFBLK, sfa + ((size_t)mat * MT * KB + kb) * PF8_SFBLK, PF8_SFBLK, &full[s]);
                    bulk_g2s(sfs + C::NA * PF8_SFBLK, sfb + (size_t)kb * PF8_SFBLK, PF8_SFBLK, &full[s]);
                }
            }
            if (abort_)  // let every issued copy land (bounded) before the CTA exits
                for (long j = std::max(0L, g - C::STAGES); j < g; ++j)
                    tc::bar_drain(&full[j % C::STAGES], (unsigned)((j / C::STAGES) & 1));
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            long g = 0, i = 0;
            for (long tile = blockIdx.x; tile < total && !abort_; tile += gridDim.x, ++i) {
                const int ab = (int)(i & 1);
                const uint32_t dcol = tmem + (uint32_t)(ab * C::ACC_COLS);
                if (i >= 2 && !tc::bar_wait(&acc_empty[ab], (unsigned)(((i >> 1) - 1) & 1), &abort_, a.status, PF_STATUS_WAIT))
                    break;
                tc::fence_after_sync();
                bool ok = true;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int s = (int)(g % C::STAGES);
                    if (!tc::bar_wait(&full[s], (unsigned)((g / C::STAGES) & 1), &abort_, a.status, PF_STATUS_WAIT)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t a0 = tc::sa(smem + (size_t)s * C::STAGE);
                    const uint32_t b0 = a0 + C::NA * PF8_ATILE, sfs = b0 + PF8_BTILE;
                    const uint32_t sfc = tmem + (uint32_t)(C::SF_BASE + (int)(g & 1) * C::SF_SLOT);
#pragma unroll
                    for (int mat = 0; mat <= C::NA; ++mat) cp_sf(sfc + 4 * mat, sfs + mat * PF8_SFBLK);
#pragma unroll
                    for (int k = 0; k < PF8_BK / 32; ++k) {
                        const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
                        const uint32_t id = idesc_mx8(PF_BM, PF8_BN, k);
                        mma_mx8(dcol, tc::desc_k_sw128(a0 + k * 32), tc::desc_k_sw128(b0 + k * 32), id, sfc,
                                sfc + 4 * C::NA, acc);
                        if (MODE == 0)
                            mma_mx8(dcol + PF8_BN, tc::desc_k_sw128(a0 + PF8_ATILE + k * 32), tc::desc_k_sw128(b0 + k * 32),
                                    id, sfc + 4, sfc + 4 * C::NA, acc);
                    }
                    tc::mma_commit(&empty[s]);
                }
                if (!ok) break;
                tc::mma_commit(&acc_full[ab]);
            }
            tc::mma_commit(&done);
            tc::bar_drain(&done, 0);
        }
        __syncwarp();
    } else {
        const int qd = warp & 3;  // TMEM lane quarter
        const int half = (warp - 2) >> 2;  // columns [48 half, 48 half + 48)
        const uint32_t lane_base = tmem + ((uint32_t)(32 * qd) << 16);
        const int kb_act = sf_stages(a.Mrows);  // the down GEMM's K stages
        long i = 0;
        for (long tile = blockIdx.x; tile < total; tile += gridDim.x, ++i) {
            const int ab = (int)(i & 1);
            if (!tc::bar_wait(&acc_full[ab], (unsigned)((i >> 1) & 1), &abort_, a.status, PF_STATUS_WAIT)) break;
            tc::fence_after_sync();
            int e, nt, mt;
            locate(tile, e, nt, mt);
            const int seg = a.off[e], n_rows = a.off[e + 1] - seg;
            const int f = mt * PF_BM + 32 * qd + lane;  // this thread's feature row
            const bool fok = f < a.Mrows;
            const uint32_t acc_base = lane_base + (uint32_t)(ab * C::ACC_COLS);
            const int wblk = a.seg_w ? a.seg_w[e] : e;
            const float bg = (a.bias && fok) ? a.bias[(size_t)wblk * a.Mrows + f] : 0.f;
            const float bu = (MODE == 0 && a.bias && fok) ? a.bias[(size_t)(a.n_blocks + wblk) * a.Mrows + f] : 0.f;
            for (int c0 = half * (PF8_BN / 2); c0 < (half + 1) * (PF8_BN / 2); c0 += 16) {
                float d[16];
                tc::tmem_ld16(acc_base + c0, d);
                if (MODE == 0) {
                    float u[16];
                    tc::tmem_ld16(acc_base + PF8_BN + c0, u);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = nt * PF8_BN + c0 + j;
                        const float v = fok ? act_fn(a.act, d[j] + bg, u[j] + bu, a.alpha, a.limit) : 0.f;
                        // the block's largest magnitude: non-negative floats order as their bits
                        const float m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))));
                        const int X = mx8_exp(m);
                        if (n < n_rows) {
                            if (fok) a.act8[(size_t)(seg + n) * a.Mrows + f] = to_e4m3(v * pow2_neg(X));
                            if (lane == 0) a.sact[sf_at(s_toff[e] + nt, kb_act, c0 + j, f / 32)] = (uint8_t)(127 + X);
                        }
                    }
                } else {
                    float *ybase = a.y_out + (size_t)seg * a.Mrows;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = nt * PF8_BN + c0 + j;
                        if (fok && n < n_rows) ybase[(size_t)n * a.Mrows + f] = d[j] + bg;
                    }
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::bar_arrive(&acc_empty[ab]);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tmem, C::TMEM_COLS);
}

struct pf_gemm4_args {
    pf_gemm_args g;
    const uint8_t *w4;  // the matrix set's chunks: [slot][mat][rb][kb]
    int RB, KB;         // row blocks and 64-column blocks of one matrix
};

// BN: rows (tokens) per tile. 128 for prefill; 32 for decode-sized batches (a few rows per
// expert), where the issue of the small MMAs bounds the kernel: a stage's MMAs are split between
// ISS = 4 issuing threads, each into its own accumulator (gate-up: issuer i takes matrix i / 2,
// K steps 2 (i % 2) and 2 (i % 2) + 1; down: K step i), the epilogue adding them in a fixed order.
//
// Stages: RS raw stages (the B tile and the stage's 4-bit chunks, filled by the producer's
// copies) and TS f16 tile stages (written by the decoder warps). With RS == TS (both variants)
// stage s is one unit: the MMAs' one commit per issuer releases both, and the decoders wait for
// that release before rewriting the tile.
template <int MODE, int WT, int BN = PF_BN>
struct pf4_cfg {
    static constexpr int NA = MODE == 0 ? 2 : 1;
    static constexpr int ISS = BN < PF_BN ? 4 : 1;
    static constexpr int CB = tc4_chunk<WT>();
    static constexpr int B_BYTES = BN * PF_BK * 2;
    static constexpr int RSTAGE = ((B_BYTES + NA * CB + 1023) / 1024) * 1024;  // B tile, then 4-bit chunks
    static constexpr int TSTAGE = NA * PF_TILE_BYTES;                          // f16 A tiles
    static constexpr int TS = BN == PF_BN ? (MODE == 0 ? 3 : 5) : (MODE == 0 ? 4 : 8);
    static constexpr int RS = TS;
    static constexpr int SMEM = TS * TSTAGE + RS * RSTAGE + 1024;
    static constexpr int ACC_COLS = (NA > ISS ? NA : ISS) * BN;
    static constexpr int TMEM_COLS = 2 * ACC_COLS;
    static constexpr int DEC_WARPS = 8;
    static constexpr int ISS_WARP1 = 6 + DEC_WARPS;  // issuers 1 .. ISS - 1 (issuer 0: warp 1)
    static constexpr int THREADS = (6 + DEC_WARPS + ISS - 1) * 32;
};

// Decode a quarter row (16 columns: half a scale block) of a staged chunk into the f16 A tile in
// the 128-byte swizzle layout (row `row`, 16-byte unit u at (u ^ (row & 7)) * 16).
template <int WT>
__device__ __forceinline__ void tc4_decode_quarter(const uint8_t *chunk, uint8_t *tile, int row, int qtr) {
    const uint2 w = *reinterpret_cast<const uint2 *>(chunk + row * 32 + qtr * 8);
    const int half = qtr >> 1;
    __half2 s2;
    if constexpr (WT == 39) {
        // 2^(e - 127) (e = 0: a zero block), exact in f16 for the exponents the load accepts
        s2 = __float2half2_rn(__uint_as_float((uint32_t)chunk[TC4_NIB + row * 2 + half] << 23));
    } else {
        const __half d = __ushort_as_half(*reinterpret_cast<const uint16_t *>(chunk + TC4_NIB + row * 4 + half * 2));
        s2 = __halves2half2(d, d);
    }
    const uint32_t words[2] = {w.x, w.y};
#pragma unroll
    for (int i = 0; i < 2; ++i) {  // 8 columns: bytes 4i .. 4i+3 of the quarter row
        uint32_t pr[4];
        decode4<WT>(words[i], pr);  // pr[j]: (column 2j, 2j + 1) of these 8, true values
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 h = __hmul2(*reinterpret_cast<const __half2 *>(&pr[j]), s2);
            o[j] = *reinterpret_cast<const uint32_t *>(&h);
        }
        const int u = qtr * 2 + i;
        *reinterpret_cast<uint4 *>(tile + row * 128 + ((u ^ (row & 7)) * 16)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// As k_pf_gemm, with the A operand (expert weights) staged as 4-bit chunks by bulk copies and
// expanded to bf16 tiles in shared memory by DEC_WARPS decoder warps (warps 6 ..): per stage the
// producer's copies complete on full[s]; the decoders wait for it, write the tiles, fence them to
// the async proxy and arrive on dec[s] (one arrival per decoder warp); the MMA issuer waits for
// both.
template <int MODE, int WT, int BN = PF_BN>
__global__ void __launch_bounds__(pf4_cfg<MODE, WT, BN>::THREADS, 1)
    k_pf_gemm4(const __grid_constant__ CUtensorMap xmap, pf_gemm4_args a4) {
    using C = pf4_cfg<MODE, WT, BN>;
    const pf_gemm_args &a = a4.g;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    static_assert(C::RS == C::TS, "one commit per stage releases the raw and the tile stage together");
    __shared__ __align__(8) uint64_t full[C::RS], empty[C::RS], dec[C::TS], acc_full[2], acc_empty[2], done[C::ISS];
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_;
    __shared__ int s_toff[1025];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i <= a.E; i += blockDim.x) s_toff[i] = a.toff[i];
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::RS; ++s) {
            tc::bar_init(&full[s], 1);
            tc::bar_init(&empty[s], C::ISS);  // one commit per issuer
        }
        for (int s = 0; s < C::TS; ++s) tc::bar_init(&dec[s], C::DEC_WARPS);
        for (int b = 0; b < 2; ++b) {
            tc::bar_init(&acc_full[b], C::ISS);
            tc::bar_init(&acc_empty[b], 4);
        }
        for (int i = 0; i < C::ISS; ++i) tc::bar_init(&done[i], 1);
        abort_ = 0;
        tc::bar_init_fence();
    }
    if (warp == 0) tc::tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    const int MT = (a.Mrows + PF_BM - 1) / PF_BM, KB = a.K / PF_BK;
    const long total = (long)s_toff[a.E] * MT;
    auto locate = [&](long tile, int &e, int &nt, int &mt) {
        const int ntg = (int)(tile / MT);
        mt = (int)(tile - (long)ntg * MT);
        int lo = 0, hi = a.E;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (s_toff[mid] <= ntg) lo = mid;
            else hi = mid;
        }
        e = lo;
        nt = ntg - s_toff[e];
    };
    auto stage_a = [&](int t) { return smem + (size_t)t * C::TSTAGE; };                       // f16 A tiles
    auto stage_b = [&](int s) { return smem + (size_t)C::TS * C::TSTAGE + (size_t)s * C::RSTAGE; };  // B tile
    auto stage_raw = [&](int s) { return stage_b(s) + C::B_BYTES; };                            // 4-bit chunks

    if (warp == 0) {
        long g = 0;
        if (lane == 0) {
            for (long tile = blockIdx.x; tile < total && !abort_; tile += gridDim.x) {
                int e, nt, mt;
                locate(tile, e, nt, mt);
                const int we = a.seg_w ? a.seg_w[e] : e;
                const int rowB = a.off[e] + nt * BN;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int s = (int)(g % C::RS);
                    if (g >= C::RS &&
                        !tc::bar_wait(&empty[s], (unsigned)(((g / C::RS) - 1) & 1), &abort_, a.status, PF_STATUS_WAIT))
                        break;
                    tc::bar_expect_tx(&full[s], C::NA * C::CB + C::B_BYTES);
                    for (int m = 0; m < C::NA; ++m) {
                        const uint8_t *src = a4.w4 + ((((size_t)we * C::NA + m) * a4.RB + mt) * a4.KB + kb) * C::CB;
                        bulk_g2s(stage_raw(s) + m * C::CB, src, (unsigned)C::CB, &full[s]);
                    }
                    tc::tma_load_2d(stage_b(s), &xmap, kb * PF_BK, rowB, &full[s]);
                }
            }
            if (abort_)
                for (long j = std::max(0L, g - C::RS); j < g; ++j)
                    tc::bar_drain(&full[j % C::RS], (unsigned)((j / C::RS) & 1));
        }
        __syncwarp();
    } else if (warp == 1 || (C::ISS > 1 && warp >= C::ISS_WARP1)) {
        const int iss = warp == 1 ? 0 : 1 + warp - C::ISS_WARP1;
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16_f32(PF_BM, BN);  // A and B both f16
            long g = 0, i = 0;
            for (long tile = blockIdx.x; tile < total && !abort_; tile += gridDim.x, ++i) {
                const int ab = (int)(i & 1);
                const uint32_t dcol = tmem + (uint32_t)(ab * C::ACC_COLS);
                if (i >= 2 && !tc::bar_wait(&acc_empty[ab], (unsigned)(((i >> 1) - 1) & 1), &abort_, a.status, PF_STATUS_WAIT))
                    break;
                tc::fence_after_sync();
                bool ok = true;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int s = (int)(g % C::RS), ts = (int)(g % C::TS);
                    if (!tc::bar_wait(&full[s], (unsigned)((g / C::RS) & 1), &abort_, a.status, PF_STATUS_WAIT) ||
                        !tc::bar_wait(&dec[ts], (unsigned)((g / C::TS) & 1), &abort_, a.status, PF_STATUS_WAIT)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t a0 = tc::sa(stage_a(ts)), b0 = tc::sa(stage_b(s));
                    if constexpr (C::ISS == 1) {
#pragma unroll
                        for (int k = 0; k < PF_BK / 16; ++k) {
                            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
                            tc::mma_bf16(dcol, tc::desc_k_sw128(a0 + k * 32), tc::desc_k_sw128(b0 + k * 32), idesc, acc);
                            if (MODE == 0)
                                tc::mma_bf16(dcol + BN, tc::desc_k_sw128(a0 + PF_TILE_BYTES + k * 32),
                                             tc::desc_k_sw128(b0 + k * 32), idesc, acc);
                        }
                    } else if constexpr (MODE == 0) {
                        // issuer iss: matrix iss / 2 (gate or up), K steps 2 (iss % 2), 2 (iss % 2) + 1
                        const uint32_t am = a0 + (uint32_t)((iss >> 1) * PF_TILE_BYTES);
#pragma unroll
                        for (int k = 0; k < 2; ++k) {
                            const int kk = 2 * (iss & 1) + k;
                            tc::mma_bf16(dcol + iss * BN, tc::desc_k_sw128(am + kk * 32), tc::desc_k_sw128(b0 + kk * 32),
                                         idesc, (kb > 0 || k > 0) ? 1u : 0u);
                        }
                    } else {
                        // issuer iss: K step iss into accumulator iss
                        tc::mma_bf16(dcol + iss * BN, tc::desc_k_sw128(a0 + iss * 32), tc::desc_k_sw128(b0 + iss * 32),
                                     idesc, kb > 0 ? 1u : 0u);
                    }
                    tc::mma_commit(&empty[s]);  // releases the raw stage and the tile stage
                }
                if (!ok) break;
                tc::mma_commit(&acc_full[ab]);
            }
            tc::mma_commit(&done[iss]);
            tc::bar_drain(&done[iss], 0);
        }
        __syncwarp();
    } else if (warp < 6) {
        const int qd = warp & 3;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * qd) << 16);
        long i = 0;
        for (long tile = blockIdx.x; tile < total; tile += gridDim.x, ++i) {
            const int ab = (int)(i & 1);
            if (!tc::bar_wait(&acc_full[ab], (unsigned)((i >> 1) & 1), &abort_, a.status, PF_STATUS_WAIT)) break;
            tc::fence_after_sync();
            int e, nt, mt;
            locate(tile, e, nt, mt);
            const int seg = a.off[e], n_rows = a.off[e + 1] - seg;
            const int f = mt * PF_BM + 32 * qd + lane;
            const bool fok = f < a.Mrows;
            const uint32_t acc_base = lane_base + (uint32_t)(ab * C::ACC_COLS);
            // this row's biases (gate-up: gate, up; down: the row's)
            const int wblk = a.seg_w ? a.seg_w[e] : e;
            const float bg = (a.bias && fok) ? a.bias[(size_t)wblk * a.Mrows + f] : 0.f;
            const float bu = (MODE == 0 && a.bias && fok) ? a.bias[(size_t)(a.n_blocks + wblk) * a.Mrows + f] : 0.f;
            for (int c0 = 0; c0 < BN; c0 += 16) {
                float d[16];
                tc::tmem_ld16(acc_base + c0, d);
                if (MODE == 1 && C::ISS == 4) {  // the other issuers' K steps, in order
                    float d2[16];
#pragma unroll
                    for (int i = 1; i < 4; ++i) {
                        tc::tmem_ld16(acc_base + i * BN + c0, d2);
#pragma unroll
                        for (int j = 0; j < 16; ++j) d[j] += d2[j];
                    }
                }
                if (MODE == 0) {
                    float u[16];
                    if constexpr (C::ISS == 4) {  // gate = acc 0 + acc 1, up = acc 2 + acc 3
                        float d2[16];
                        tc::tmem_ld16(acc_base + BN + c0, d2);
#pragma unroll
                        for (int j = 0; j < 16; ++j) d[j] += d2[j];
                        tc::tmem_ld16(acc_base + 2 * BN + c0, u);
                        tc::tmem_ld16(acc_base + 3 * BN + c0, d2);
#pragma unroll
                        for (int j = 0; j < 16; ++j) u[j] += d2[j];
                    } else {
                        tc::tmem_ld16(acc_base + BN + c0, u);
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = nt * BN + c0 + j;
                        if (fok && n < n_rows)
                            a.act_out[(size_t)(seg + n) * a.Mrows + f] =
                                __half_as_ushort(__float2half_rn(act_fn(a.act, d[j] + bg, u[j] + bu, a.alpha, a.limit)));
                    }
                } else {
                    float *ybase = a.seg_y ? a.seg_y[e] : a.y_out + (size_t)seg * a.Mrows;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = nt * BN + c0 + j;
                        if (fok && n < n_rows) ybase[(size_t)n * a.Mrows + f] = d[j] + bg;
                    }
                }
            }
            if (MODE == 1 && a.seg_y) __threadfence_system();  // peer stores performed
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::bar_arrive(&acc_empty[ab]);
        }
    } else {
        // decoder warps: quarter rows (16 columns) t, t + 32 DEC_WARPS, ... of the stage's chunks
        const int t = threadIdx.x - 6 * 32;
        long g = 0;
        for (long tile = blockIdx.x; tile < total && !abort_; tile += gridDim.x) {
            bool ok = true;
            for (int kb = 0; kb < KB; ++kb, ++g) {
                const int s = (int)(g % C::RS), ts = (int)(g % C::TS);
                // the tile stage is free once the MMAs of its previous use have completed
                if (!tc::bar_wait(&full[s], (unsigned)((g / C::RS) & 1), &abort_, a.status, PF_STATUS_WAIT) ||
                    (g >= C::TS &&
                     !tc::bar_wait(&empty[ts], (unsigned)(((g / C::TS) - 1) & 1), &abort_, a.status, PF_STATUS_WAIT))) {
                    ok = false;
                    break;
                }
#pragma unroll
                for (int q = t; q < C::NA * 512; q += C::DEC_WARPS * 32) {
                    const int m = q >> 9, row = (q & 511) >> 2;
                    tc4_decode_quarter<WT>(stage_raw(s) + m * C::CB, stage_a(ts) + m * PF_TILE_BYTES, row, q & 3);
                }
                fence_proxy_async();  // the generic-proxy tile writes, visible to the MMA's reads
                __syncwarp();
                if (lane == 0) tc::bar_arrive(&dec[ts]);
            }
            if (!ok) break;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ---- host ---------------------------------------------------------------------------------

typedef CUresult (*encode_tiled_fn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

encode_tiled_fn encoder() {
    static encode_tiled_fn fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<encode_tiled_fn>(p);
        cudaGetLastError();
    }
    return fn;
}

// An E4M3 row-major [rows][cols] matrix read as box_rows-row x 128-byte boxes, 128-byte swizzle;
// rows and columns past the end read as zeros.
bool make_map8(CUtensorMap *map, const void *base, long rows, int cols, int box_rows) {
    encode_tiled_fn enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols};
    const cuuint32_t box[2] = {PF8_BK, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A bf16 (or f16) row-major [rows][cols] matrix read as box_rows-row x 64-column boxes, 128-byte
// swizzle (the UMMA K-major canonical layout); rows past the end read as zeros.
bool make_map(CUtensorMap *map, const void *base, long rows, int cols, int box_rows = PF_BM) {
    encode_tiled_fn enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {PF_BK, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

namespace moearc {

// For other translation units (the batched decoder): the 128 x 64 bf16 K-major tensor map, and a
// dense GEMM on the same kernel, out[n][m] = sum_k W[m][k] x[n][k] (f32), as one segment of
// n rows: seg_off = {0, n} and seg_toff = {0, ceil(n / 128)} in device memory. With ksplit > 1
// the K blocks are split into ksplit runs and run j's partial sums go to out + j * split_stride
// (the caller adds them, in order).
bool tc_make_map_bf16(CUtensorMap *map, const void *base, long rows, int cols) { return make_map(map, base, rows, cols); }

int tc_dense_gemm(moearc_ctx *c, const CUtensorMap &w, int M, int K, const CUtensorMap &x, const int *seg_off,
                  const int *seg_toff, float *out, int *status, int ksplit, size_t split_stride) {
    static std::atomic<bool> ready[MOEARC_MAX_DEVICES];
    if (once_per_device(ready, [] { return set_smem(k_pf_gemm<1>, pf_cfg<1>::SMEM); }) != cudaSuccess) return ERR;
    if (K % PF_BK) return ERR_ARG;
    pf_gemm_args g{};
    g.Mrows = M;
    g.K = K;
    g.E = 1;
    g.off = seg_off;
    g.toff = seg_toff;
    g.y_out = out;
    g.status = status;
    if (ksplit > K / PF_BK) return ERR_ARG;
    g.ksplit = ksplit;
    g.split_stride = split_stride;
    const int grid = std::min(c->sm_count, (M + PF_BM - 1) / PF_BM * std::max(8, ksplit));  // n is small
    k_pf_gemm<1><<<grid, 192, pf_cfg<1>::SMEM, c->stream>>>(w, x, g);
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

}  // namespace moearc

struct moearc_x_prefill {
    moearc_ctx *c;
    int H, I, E, K, wtype, gating, act;
    float alpha, limit;
    int T_max, tile_bytes;
    void *mem = nullptr;
    float *logits, *y, *wts;
    unsigned *idx;
    int *cnt, *off, *toff, *cursor, *perm, *status;
    int *seg_cnt, *seg_off, *seg_toff, *seg_w, *seg_cur;  // expert-parallel segments (<= 1024)
    int *epos;                                          // [E] position of each expert in the row order
    bool order_identity = true;
    uint16_t *xp, *actb;
    CUtensorMap map_xp, map_act;
    CUtensorMap map_xp32, map_act32;  // the same with 32-row boxes (the 4-bit form's decode-sized tiles)
    // expert weights, allocated by the first load of each form: the bf16 expansion
    // ([E][2][I][H] and [E][H][I]) or the 4-bit chunks (tc4 layout); the last load picks the form
    void *w16 = nullptr;
    uint16_t *wgu = nullptr, *wdn = nullptr;
    CUtensorMap map_wgu, map_wdn;
    uint8_t *w4 = nullptr, *w4gu = nullptr, *w4dn = nullptr;
    bool mode4 = false;
    int *elist = nullptr;  // [E] device copy of a load list
    // peer-memory exchange: destination row pointers and bases per rank, y pointers per segment
    uint16_t **dst_rows = nullptr;
    int *dst_base = nullptr;
    float **seg_y = nullptr;
    const uint16_t *route_x = nullptr;  // the activations of the last route_begin call
    int route_T = 0;
    // per-expert biases (moearc_x_prefill_set_bias), indexed by weight block: gate-up
    // [2E][I] (gate of block w at w, up at E + w), down [E][H]; null: none
    const float *bias_gu = nullptr, *bias_dn = nullptr;
    // MXFP8 mode (moearc_x_prefill_load8): E4M3 weights [E][2][I][H] and [E][H][I] with their
    // scale bytes, the activations' scale bytes (the E4M3 rows reuse xp and actb)
    void *w8 = nullptr;
    uint8_t *w8gu = nullptr, *w8dn = nullptr, *s8gu = nullptr, *s8dn = nullptr, *s8x = nullptr, *s8a = nullptr;
    CUtensorMap map8_wgu, map8_wdn, map8_x, map8_act;
    bool mode8 = false;
};

namespace {

bool ensure_bf16(moearc_x_prefill *p) {
    if (p->w16) return true;
    const size_t ngu = (size_t)p->E * 2 * p->I * p->H, ndn = (size_t)p->E * p->H * p->I;
    if (cudaMalloc(&p->w16, 2 * (ngu + ndn)) != cudaSuccess) {
        cudaGetLastError();
        p->w16 = nullptr;
        return false;
    }
    p->wgu = static_cast<uint16_t *>(p->w16);
    p->wdn = p->wgu + ngu;
    return make_map(&p->map_wgu, p->wgu, (long)p->E * 2 * p->I, p->H) && make_map(&p->map_wdn, p->wdn, (long)p->E * p->H, p->I);
}

// The MXFP8 form's memory (first load8): weights and scales, the activation scales (the pad bytes
// of every scale row hold 127), and the four tensor maps.
bool ensure_fp8(moearc_x_prefill *p) {
    if (p->w8) return true;
    const size_t rows = (size_t)p->T_max * p->K;
    const size_t ngu = (size_t)p->E * 2 * p->I * p->H, ndn = (size_t)p->E * p->H * p->I;
    const size_t mt_i = (p->I + PF_BM - 1) / PF_BM, mt_h = (p->H + PF_BM - 1) / PF_BM;
    const size_t sgu = (size_t)p->E * 2 * mt_i * sf_stages(p->H) * PF8_SFBLK;
    const size_t sdn = (size_t)p->E * mt_h * sf_stages(p->I) * PF8_SFBLK;
    const size_t tiles = (rows + PF8_BN - 1) / PF8_BN + p->E;  // 96-row tiles over all segments, at most
    const size_t sx = tiles * sf_stages(p->H) * PF8_SFBLK, sa = tiles * sf_stages(p->I) * PF8_SFBLK;
    const size_t total = ngu + ndn + sgu + sdn + sx + sa;
    if (cudaMalloc(&p->w8, total) != cudaSuccess) {
        cudaGetLastError();
        p->w8 = nullptr;
        return false;
    }
    uint8_t *b = static_cast<uint8_t *>(p->w8);
    p->w8gu = b;
    p->w8dn = b + ngu;
    p->s8gu = p->w8dn + ndn;
    p->s8dn = p->s8gu + sgu;
    p->s8x = p->s8dn + sdn;
    p->s8a = p->s8x + sx;
    if (cudaMemsetAsync(p->s8gu, 0x7F, sgu + sdn + sx + sa, p->c->stream) != cudaSuccess) return false;
    const bool ok = make_map8(&p->map8_wgu, p->w8gu, (long)p->E * 2 * p->I, p->H, PF_BM) &&
                    make_map8(&p->map8_wdn, p->w8dn, (long)p->E * p->H, p->I, PF_BM) &&
                    make_map8(&p->map8_x, p->xp, (long)rows, p->H, PF8_BN) &&
                    make_map8(&p->map8_act, p->actb, (long)rows, p->I, PF8_BN) &&
                    set_smem(k_pf_gemm8<0>, pf8_cfg<0>::SMEM) == cudaSuccess &&
                    set_smem(k_pf_gemm8<1>, pf8_cfg<1>::SMEM) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        cudaFree(p->w8);
        p->w8 = nullptr;
    }
    return ok;
}

int tc4_bytes(const moearc_x_prefill *p) { return p->wtype == T_MXFP4 ? tc4_chunk<39>() : tc4_chunk<2>(); }

bool ensure_4bit(moearc_x_prefill *p) {
    if (p->w4) return true;
    const size_t cb = (size_t)tc4_bytes(p);
    const size_t gu = (size_t)p->E * 2 * ((p->I + 127) / 128) * (p->H / 64) * cb;
    const size_t dn = (size_t)p->E * ((p->H + 127) / 128) * (p->I / 64) * cb;
    if (cudaMalloc(reinterpret_cast<void **>(&p->w4), gu + dn) != cudaSuccess) {
        cudaGetLastError();
        p->w4 = nullptr;
        return false;
    }
    p->w4gu = p->w4;
    p->w4dn = p->w4 + gu;
    return true;
}

// The grouped GEMM of one matrix set (MODE 0 gate-up, 1 down) on whichever weight form is loaded.
// bn: rows per tile, PF_BN or (4-bit form only) PF4_BN_SMALL, as the tile offsets were counted.
int launch_gemm(moearc_x_prefill *p, int mode, const pf_gemm_args &g_in, const CUtensorMap &xmap, int bn = PF_BN) {
    moearc_ctx *c = p->c;
    cudaStream_t st = c->stream;
    pf_gemm_args g = g_in;
    g.bias = mode == 0 ? p->bias_gu : p->bias_dn;  // indexed by weight block (E of them)
    g.n_blocks = p->E;
    if (!p->mode4) {
        if (mode == 0) k_pf_gemm<0><<<c->sm_count, 192, pf_cfg<0>::SMEM, st>>>(p->map_wgu, xmap, g);
        else k_pf_gemm<1><<<c->sm_count, 192, pf_cfg<1>::SMEM, st>>>(p->map_wdn, xmap, g);
        return cudaGetLastError() == cudaSuccess ? OK : ERR;
    }
    pf_gemm4_args a4{g, mode == 0 ? p->w4gu : p->w4dn, 0, 0};
    a4.RB = mode == 0 ? (p->I + 127) / 128 : (p->H + 127) / 128;
    a4.KB = mode == 0 ? p->H / 64 : p->I / 64;
    if (bn == PF4_BN_SMALL) {
        constexpr int S = PF4_BN_SMALL;
        if (p->wtype == T_MXFP4) {
            if (mode == 0) k_pf_gemm4<0, 39, S><<<c->sm_count, pf4_cfg<0, 39, S>::THREADS, pf4_cfg<0, 39, S>::SMEM, st>>>(xmap, a4);
            else k_pf_gemm4<1, 39, S><<<c->sm_count, pf4_cfg<1, 39, S>::THREADS, pf4_cfg<1, 39, S>::SMEM, st>>>(xmap, a4);
        } else {
            if (mode == 0) k_pf_gemm4<0, 2, S><<<c->sm_count, pf4_cfg<0, 2, S>::THREADS, pf4_cfg<0, 2, S>::SMEM, st>>>(xmap, a4);
            else k_pf_gemm4<1, 2, S><<<c->sm_count, pf4_cfg<1, 2, S>::THREADS, pf4_cfg<1, 2, S>::SMEM, st>>>(xmap, a4);
        }
        return cudaGetLastError() == cudaSuccess ? OK : ERR;
    }
    if (bn != PF_BN) return ERR_ARG;
    if (p->wtype == T_MXFP4) {
        if (mode == 0) k_pf_gemm4<0, 39><<<c->sm_count, pf4_cfg<0, 39>::THREADS, pf4_cfg<0, 39>::SMEM, st>>>(xmap, a4);
        else k_pf_gemm4<1, 39><<<c->sm_count, pf4_cfg<1, 39>::THREADS, pf4_cfg<1, 39>::SMEM, st>>>(xmap, a4);
    } else {
        if (mode == 0) k_pf_gemm4<0, 2><<<c->sm_count, pf4_cfg<0, 2>::THREADS, pf4_cfg<0, 2>::SMEM, st>>>(xmap, a4);
        else k_pf_gemm4<1, 2><<<c->sm_count, pf4_cfg<1, 2>::THREADS, pf4_cfg<1, 2>::SMEM, st>>>(xmap, a4);
    }
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

}  // namespace

extern "C" {

moearc_x_prefill *moearc_x_prefill_create(moearc_ctx *c, const moearc_x_moe_desc *d) {
    if (!c || !d) return nullptr;
    if (d->wtype != T_MXFP4 && d->wtype != T_Q4_0) return nullptr;
    // the router kernel holds PF_LOGIT_TOK f32 activations in shared memory (n_embd <= 3584)
    if (d->n_embd % 64 || d->n_ff % 64 || d->n_expert == 0 || d->n_expert > 1024 || d->k == 0 || d->k > 32 ||
        d->k > d->n_expert || d->max_tokens == 0 || (size_t)PF_LOGIT_TOK * d->n_embd * 4 > 227 * 1024)
        return nullptr;
    auto *p = new moearc_x_prefill();
    p->c = c;
    p->H = (int)d->n_embd;
    p->I = (int)d->n_ff;
    p->E = (int)d->n_expert;
    p->K = (int)d->k;
    p->wtype = (int)d->wtype;
    p->gating = (int)d->gating;
    p->act = (int)d->act;
    p->alpha = d->alpha;
    p->limit = d->limit;
    p->T_max = (int)d->max_tokens;
    p->tile_bytes = d->wtype == T_MXFP4 ? 544 : 576;
    const size_t rows = (size_t)p->T_max * p->K;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 1023) & ~(size_t)1023;
        return o;
    };
    const size_t o_lg = take(sizeof(float) * p->T_max * p->E), o_y = take(sizeof(float) * rows * p->H);
    const size_t o_w = take(sizeof(float) * rows), o_i = take(sizeof(unsigned) * rows);
    const size_t o_cnt = take(sizeof(int) * (p->E + 1)), o_off = take(sizeof(int) * (p->E + 1));
    const size_t o_toff = take(sizeof(int) * (p->E + 1)), o_cur = take(sizeof(int) * (p->E + 1));
    const size_t o_perm = take(sizeof(int) * rows), o_st = take(sizeof(int));
    const size_t o_seg = take(sizeof(int) * 7 * 1025);
    const size_t o_ptrs = take(sizeof(void *) * (1024 + 1024) + sizeof(int) * 1024);
    const size_t o_xp = take(2 * rows * p->H), o_act = take(2 * rows * p->I);
    if (cudaMalloc(&p->mem, off) != cudaSuccess) {
        cudaGetLastError();
        delete p;
        return nullptr;
    }
    uint8_t *b = static_cast<uint8_t *>(p->mem);
    p->logits = reinterpret_cast<float *>(b + o_lg);
    p->y = reinterpret_cast<float *>(b + o_y);
    p->wts = reinterpret_cast<float *>(b + o_w);
    p->idx = reinterpret_cast<unsigned *>(b + o_i);
    p->cnt = reinterpret_cast<int *>(b + o_cnt);
    p->off = reinterpret_cast<int *>(b + o_off);
    p->toff = reinterpret_cast<int *>(b + o_toff);
    p->cursor = reinterpret_cast<int *>(b + o_cur);
    p->perm = reinterpret_cast<int *>(b + o_perm);
    p->status = reinterpret_cast<int *>(b + o_st);
    p->seg_cnt = reinterpret_cast<int *>(b + o_seg);
    p->seg_off = p->seg_cnt + 1025;
    p->seg_toff = p->seg_off + 1025;
    p->seg_w = p->seg_toff + 1025;
    p->seg_cur = p->seg_w + 1025;
    p->epos = p->seg_cur + 1025;
    p->elist = p->epos + 1025;
    p->dst_rows = reinterpret_cast<uint16_t **>(b + o_ptrs);
    p->seg_y = reinterpret_cast<float **>(b + o_ptrs + sizeof(void *) * 1024);
    p->dst_base = reinterpret_cast<int *>(b + o_ptrs + sizeof(void *) * 2048);
    p->xp = reinterpret_cast<uint16_t *>(b + o_xp);
    p->actb = reinterpret_cast<uint16_t *>(b + o_act);
    constexpr int S = PF4_BN_SMALL;
    const bool ok = make_map(&p->map_xp, p->xp, (long)rows, p->H) &&
                    make_map(&p->map_act, p->actb, (long)rows, p->I) &&
                    make_map(&p->map_xp32, p->xp, (long)rows, p->H, S) &&
                    make_map(&p->map_act32, p->actb, (long)rows, p->I, S) &&
                    set_smem(k_pf_gemm4<0, 39, S>, pf4_cfg<0, 39, S>::SMEM) == cudaSuccess &&
                    set_smem(k_pf_gemm4<1, 39, S>, pf4_cfg<1, 39, S>::SMEM) == cudaSuccess &&
                    set_smem(k_pf_gemm4<0, 2, S>, pf4_cfg<0, 2, S>::SMEM) == cudaSuccess &&
                    set_smem(k_pf_gemm4<1, 2, S>, pf4_cfg<1, 2, S>::SMEM) == cudaSuccess &&
                    set_smem(k_pf_gemm4<0, 39>, pf4_cfg<0, 39>::SMEM) == cudaSuccess &&
                    set_smem(k_pf_gemm4<1, 39>, pf4_cfg<1, 39>::SMEM) == cudaSuccess &&
                    set_smem(k_pf_gemm4<0, 2>, pf4_cfg<0, 2>::SMEM) == cudaSuccess &&
                    set_smem(k_pf_gemm4<1, 2>, pf4_cfg<1, 2>::SMEM) == cudaSuccess &&
                    set_smem(k_pf_gemm<0>, pf_cfg<0>::SMEM) == cudaSuccess &&
                    set_smem(k_pf_gemm<1>, pf_cfg<1>::SMEM) == cudaSuccess &&
                    set_smem(k_pf_logits, PF_LOGIT_TOK * p->H * 4) == cudaSuccess &&
                    cudaMemsetAsync(p->mem, 0, off, c->stream) == cudaSuccess;
    std::vector<int> ident(p->E);
    for (int e = 0; e < p->E; ++e) ident[e] = e;
    const bool ok2 = ok && cudaMemcpyAsync(p->epos, ident.data(), sizeof(int) * p->E, cudaMemcpyHostToDevice,
                                           c->stream) == cudaSuccess &&
                     cudaStreamSynchronize(c->stream) == cudaSuccess;
    if (!ok2) {
        cudaGetLastError();
        cudaFree(p->mem);
        delete p;
        return nullptr;
    }
    return p;
}

void moearc_x_prefill_destroy(moearc_x_prefill *p) {
    if (!p) return;
    cudaStreamSynchronize(p->c->stream);
    cudaFree(p->w16);
    cudaFree(p->w4);
    cudaFree(p->w8);
    cudaFree(p->mem);
    delete p;
}

int moearc_x_prefill_load8(moearc_x_prefill *p, const void *gateup_packed, const void *down_packed) {
    if (!p || !gateup_packed || !down_packed) return ERR;
    if (p->wtype != T_MXFP4 || p->H % 64 || p->I % 64) return ERR_ARG;  // E2M1 elements carry over exactly
    if (!ensure_fp8(p)) return ERR;
    moearc_ctx *c = p->c;
    const long gu_tiles = (long)p->E * (p->I / 16) * (p->H / 64) * 2, dn_tiles = (long)p->E * (p->H / 16) * (p->I / 64);
    auto grid = [](long warps) { return dim3((unsigned)((warps + 7) / 8)); };
    k_pf_unpack8<<<grid(gu_tiles), 256, 0, c->stream>>>(static_cast<const uint8_t *>(gateup_packed), p->E, p->I, p->H,
                                                         2, p->tile_bytes, p->w8gu, p->s8gu);
    k_pf_unpack8<<<grid(dn_tiles), 256, 0, c->stream>>>(static_cast<const uint8_t *>(down_packed), p->E, p->H, p->I, 1,
                                                         p->tile_bytes, p->w8dn, p->s8dn);
    p->mode4 = false;
    p->mode8 = true;
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

int moearc_x_prefill_load_range(moearc_x_prefill *p, const void *gateup_packed, const void *down_packed,
                                unsigned e_first, unsigned n) {
    if (!p || !gateup_packed || !down_packed) return ERR;
    if (n == 0 || e_first + n > (unsigned)p->E) return ERR_ARG;
    if (!ensure_bf16(p)) return ERR;
    p->mode4 = false;
    p->mode8 = false;
    moearc_ctx *c = p->c;
    const int E = (int)n;
    const size_t gu_e = (size_t)(p->I / 16) * (p->H / 64) * 2 * p->tile_bytes, dn_e = (size_t)(p->H / 16) * (p->I / 64) * p->tile_bytes;
    const uint8_t *gu = static_cast<const uint8_t *>(gateup_packed) + e_first * gu_e;
    const uint8_t *dn = static_cast<const uint8_t *>(down_packed) + e_first * dn_e;
    const long gu_tiles = (long)E * (p->I / 16) * (p->H / 64) * 2, dn_tiles = (long)E * (p->H / 16) * (p->I / 64);
    const bool mx = p->wtype == T_MXFP4;
    auto grid = [](long warps) { return dim3((unsigned)((warps + 7) / 8)); };
    if (mx) {
        k_pf_unpack<39><<<grid(gu_tiles), 256, 0, c->stream>>>(gu, E, p->I, p->H, 2, p->tile_bytes, p->wgu);
        k_pf_unpack<39><<<grid(dn_tiles), 256, 0, c->stream>>>(dn, E, p->H, p->I, 1, p->tile_bytes, p->wdn);
    } else {
        k_pf_unpack<2><<<grid(gu_tiles), 256, 0, c->stream>>>(gu, E, p->I, p->H, 2, p->tile_bytes, p->wgu);
        k_pf_unpack<2><<<grid(dn_tiles), 256, 0, c->stream>>>(dn, E, p->H, p->I, 1, p->tile_bytes, p->wdn);
    }
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

// Expert experts[i] into weight slot i, for i < n (host array of distinct expert ids).
int moearc_x_prefill_load_list(moearc_x_prefill *p, const void *gateup_packed, const void *down_packed,
                               const int *experts, unsigned n) {
    if (!p || !gateup_packed || !down_packed || !experts) return ERR;
    if (n == 0 || n > (unsigned)p->E) return ERR_ARG;
    for (unsigned i = 0; i < n; ++i)
        if (experts[i] < 0 || experts[i] >= p->E) return ERR_ARG;
    if (!ensure_bf16(p)) return ERR;
    p->mode4 = false;
    p->mode8 = false;
    moearc_ctx *c = p->c;
    const size_t gu_e = (size_t)(p->I / 16) * (p->H / 64) * 2 * p->tile_bytes, dn_e = (size_t)(p->H / 16) * (p->I / 64) * p->tile_bytes;
    const long gu_tiles = (long)(p->I / 16) * (p->H / 64) * 2, dn_tiles = (long)(p->H / 16) * (p->I / 64);
    const bool mx = p->wtype == T_MXFP4;
    auto grid = [](long warps) { return dim3((unsigned)((warps + 7) / 8)); };
    for (unsigned i = 0; i < n; ++i) {
        const uint8_t *gu = static_cast<const uint8_t *>(gateup_packed) + experts[i] * gu_e;
        const uint8_t *dn = static_cast<const uint8_t *>(down_packed) + experts[i] * dn_e;
        uint16_t *wg = p->wgu + (size_t)i * 2 * p->I * p->H, *wd = p->wdn + (size_t)i * p->H * p->I;
        if (mx) {
            k_pf_unpack<39><<<grid(gu_tiles), 256, 0, c->stream>>>(gu, 1, p->I, p->H, 2, p->tile_bytes, wg);
            k_pf_unpack<39><<<grid(dn_tiles), 256, 0, c->stream>>>(dn, 1, p->H, p->I, 1, p->tile_bytes, wd);
        } else {
            k_pf_unpack<2><<<grid(gu_tiles), 256, 0, c->stream>>>(gu, 1, p->I, p->H, 2, p->tile_bytes, wg);
            k_pf_unpack<2><<<grid(dn_tiles), 256, 0, c->stream>>>(dn, 1, p->H, p->I, 1, p->tile_bytes, wd);
        }
    }
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

// The row order of the route step: expert e's rows form segment pos[e] (host array, a permutation
// of 0 .. E-1). The identity at create; moearc_x_prefill_forward needs the identity.
int moearc_x_prefill_set_order(moearc_x_prefill *p, const int *pos) {
    if (!p || !pos) return ERR;
    std::vector<char> seen(p->E, 0);
    for (int e = 0; e < p->E; ++e) {
        if (pos[e] < 0 || pos[e] >= p->E || seen[pos[e]]) return ERR_ARG;
        seen[pos[e]] = 1;
    }
    p->order_identity = true;
    for (int e = 0; e < p->E; ++e) p->order_identity = p->order_identity && pos[e] == e;
    return cudaMemcpyAsync(p->epos, pos, sizeof(int) * p->E, cudaMemcpyHostToDevice, p->c->stream) == cudaSuccess &&
                   cudaStreamSynchronize(p->c->stream) == cudaSuccess
               ? OK
               : ERR;
}

// The 4-bit form: experts[i] (host array) repacked into chunk slot i of the tc4 layout; the
// GEMMs then decode the chunks on the fly (same values as the bf16 expansion).
int moearc_x_prefill_load4_list(moearc_x_prefill *p, const void *gateup_packed, const void *down_packed,
                                const int *experts, unsigned n) {
    if (!p || !gateup_packed || !down_packed || !experts) return ERR;
    if (n == 0 || n > (unsigned)p->E) return ERR_ARG;
    for (unsigned i = 0; i < n; ++i)
        if (experts[i] < 0 || experts[i] >= p->E) return ERR_ARG;
    if (!ensure_4bit(p)) return ERR;
    moearc_ctx *c = p->c;
    if (cudaMemcpyAsync(p->elist, experts, sizeof(int) * n, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) return ERR;
    const uint8_t *gu = static_cast<const uint8_t *>(gateup_packed), *dn = static_cast<const uint8_t *>(down_packed);
    const long rows_gu = (long)n * 2 * ((p->I + 127) / 128) * (p->H / 64) * 128;
    const long rows_dn = (long)n * ((p->H + 127) / 128) * (p->I / 64) * 128;
    auto grid = [](long t) { return dim3((unsigned)((t + 255) / 256)); };
    if (cudaMemsetAsync(p->status, 0, sizeof(int), c->stream) != cudaSuccess) return ERR;
    if (p->wtype == T_MXFP4) {
        k_pf_pack4<39><<<grid(rows_gu), 256, 0, c->stream>>>(gu, p->elist, (int)n, p->I, p->H, 2, p->tile_bytes, p->w4gu, p->status);
        k_pf_pack4<39><<<grid(rows_dn), 256, 0, c->stream>>>(dn, p->elist, (int)n, p->H, p->I, 1, p->tile_bytes, p->w4dn, p->status);
    } else {
        k_pf_pack4<2><<<grid(rows_gu), 256, 0, c->stream>>>(gu, p->elist, (int)n, p->I, p->H, 2, p->tile_bytes, p->w4gu, p->status);
        k_pf_pack4<2><<<grid(rows_dn), 256, 0, c->stream>>>(dn, p->elist, (int)n, p->H, p->I, 1, p->tile_bytes, p->w4dn, p->status);
    }
    if (cudaGetLastError() != cudaSuccess) return ERR;
    int st = 0;
    if (cudaMemcpyAsync(&st, p->status, sizeof(int), cudaMemcpyDeviceToHost, c->stream) != cudaSuccess ||
        cudaMemsetAsync(p->status, 0, sizeof(int), c->stream) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess)
        return ERR;
    if (st & PF_STATUS_RANGE) return ERR_ARG;  // scales f16 cannot hold: keep the bf16 form
    p->mode4 = true;
    p->mode8 = false;
    return OK;
}

int moearc_x_prefill_load4(moearc_x_prefill *p, const void *gateup_packed, const void *down_packed) {
    if (!p) return ERR;
    std::vector<int> all(p->E);
    for (int e = 0; e < p->E; ++e) all[e] = e;
    return moearc_x_prefill_load4_list(p, gateup_packed, down_packed, all.data(), (unsigned)p->E);
}

int moearc_x_prefill_set_bias(moearc_x_prefill *p, const float *gate_up_bias, const float *down_bias) {
    if (!p) return ERR;
    if ((reinterpret_cast<uintptr_t>(gate_up_bias) | reinterpret_cast<uintptr_t>(down_bias)) & 3) return ERR_ARG;
    p->bias_gu = gate_up_bias;
    p->bias_dn = down_bias;
    return OK;
}

int moearc_x_prefill_load(moearc_x_prefill *p, const void *gateup_packed, const void *down_packed) {
    return p ? moearc_x_prefill_load_range(p, gateup_packed, down_packed, 0, (unsigned)p->E) : ERR;
}

}  // extern "C"

namespace {

// The forward sequence; with `ev`, an event is recorded before the first kernel and after each
// of the 7 kernels (routing, top-k, scan, scatter, gate-up GEMM, down GEMM, combine).
int prefill_forward(moearc_x_prefill *p, const uint16_t *x, unsigned n_tokens, const float *router_w,
                    const float *router_b, const float *residual, float *out, cudaEvent_t *ev,
                    const float *x32 = nullptr) {
    if (!p || !x || !router_w || !out) return ERR;
    if (n_tokens == 0) return OK;
    if ((int)n_tokens > p->T_max || !p->order_identity) return ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(router_w)) & 15) return ERR_ARG;
    moearc_ctx *c = p->c;
    cudaStream_t st = c->stream;
    const int T = (int)n_tokens;
    launch_scope ls(c, "moe_prefill", (unsigned long)p->H, (unsigned)T);
    auto mark = [&](int i) {
        if (ev) cudaEventRecord(ev[i], st);
    };
    if (cudaMemsetAsync(p->cnt, 0, sizeof(int) * (p->E + 1), st) != cudaSuccess) return ERR;
    mark(0);
    pf_route_args ra{x, x32, router_w, router_b, T, p->H, p->E, p->K, p->gating, p->logits, p->idx, p->wts, p->cnt, p->epos};
    k_pf_logits<<<logit_grid(T, p->E), 256, PF_LOGIT_TOK * p->H * 4, st>>>(ra);
    mark(1);
    k_pf_topk<<<(T + 7) / 8, 256, 0, st>>>(ra);
    mark(2);
    // the 4-bit form takes 32-row tiles when the rows per expert are few (decode-sized batches)
    const int bn = p->mode8 ? PF8_BN : (p->mode4 && (long)T * p->K <= (long)PF4_SMALL_ROWS * p->E) ? PF4_BN_SMALL : PF_BN;
    k_pf_scan<<<1, 1024, 0, st>>>(p->cnt, p->E, p->off, p->toff, p->cursor, bn);
    mark(3);
    const long pairs = (long)T * p->K;
    if (p->mode8) {
        // MXFP8: quantised rows, then the block-scaled GEMMs
        k_pf_scatter8<<<(unsigned)((pairs + 7) / 8), 256, 0, st>>>(x, p->idx, p->epos, T, p->K, p->H, p->off, p->toff,
                                                                   p->cursor, p->perm, reinterpret_cast<uint8_t *>(p->xp),
                                                                   p->s8x);
        mark(4);
        pf8_args g{};
        g.E = p->E;
        g.off = p->off;
        g.toff = p->toff;
        g.act = p->act;
        g.alpha = p->alpha;
        g.limit = p->limit;
        g.status = p->status;
        g.n_blocks = p->E;
        g.Mrows = p->I;
        g.K = p->H;
        g.sfw = p->s8gu;
        g.sfx = p->s8x;
        g.act8 = reinterpret_cast<uint8_t *>(p->actb);
        g.sact = p->s8a;
        g.bias = p->bias_gu;
        k_pf_gemm8<0><<<c->sm_count, PF8_THREADS, pf8_cfg<0>::SMEM, st>>>(p->map8_wgu, p->map8_x, g);
        mark(5);
        g.Mrows = p->H;
        g.K = p->I;
        g.sfw = p->s8dn;
        g.sfx = p->s8a;
        g.y_out = p->y;
        g.bias = p->bias_dn;
        k_pf_gemm8<1><<<c->sm_count, PF8_THREADS, pf8_cfg<1>::SMEM, st>>>(p->map8_wdn, p->map8_act, g);
        mark(6);
        const long n = (long)T * p->H;
        k_pf_combine<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(p->y, p->perm, p->wts, residual, out, T, p->K, p->H);
        mark(7);
        if (cudaGetLastError() != cudaSuccess) return ERR;
        return ls.finish();
    }
    k_pf_scatter<<<(unsigned)((pairs + 7) / 8), 256, 0, st>>>(x, p->idx, p->epos, T, p->K, p->H, p->off, p->cursor,
                                                              p->perm, p->xp, p->mode4 ? 1 : 0, nullptr, nullptr, 0);
    mark(4);
    pf_gemm_args g{};
    g.E = p->E;
    g.off = p->off;
    g.toff = p->toff;
    g.act = p->act;
    g.alpha = p->alpha;
    g.limit = p->limit;
    g.act_out = p->actb;
    g.y_out = p->y;
    g.status = p->status;
    g.Mrows = p->I;
    g.K = p->H;
    if (!p->w16 && !p->w4) return ERR_ARG;  // no weights loaded
    const bool small = bn == PF4_BN_SMALL;
    if (launch_gemm(p, 0, g, small ? p->map_xp32 : p->map_xp, bn) != OK) return ERR;
    mark(5);
    g.Mrows = p->H;
    g.K = p->I;
    if (launch_gemm(p, 1, g, small ? p->map_act32 : p->map_act, bn) != OK) return ERR;
    mark(6);
    const long n = (long)T * p->H;
    k_pf_combine<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(p->y, p->perm, p->wts, residual, out, T, p->K, p->H);
    mark(7);
    return ls.finish();
}

}  // namespace

namespace moearc {
// moearc_x_prefill_forward with the router logits taken from x32 (f32 [T][H]) instead of the bf16
// activations: for a caller whose decode path routes on f32 activations.
int prefill_forward_x32(moearc_x_prefill *p, const uint16_t *x, const float *x32, unsigned n_tokens,
                        const float *router_w, const float *router_b, const float *residual, float *out) {
    return prefill_forward(p, x, n_tokens, router_w, router_b, residual, out, nullptr, x32);
}
int prefill_route_x32(moearc_x_prefill *p, const uint16_t *x, const float *x32, unsigned n_tokens,
                      const float *router_w, const float *router_b);
}  // namespace moearc

extern "C" {

int moearc_x_prefill_forward(moearc_x_prefill *p, const uint16_t *x, unsigned n_tokens, const float *router_w,
                             const float *router_b, const float *residual, float *out) {
    return prefill_forward(p, x, n_tokens, router_w, router_b, residual, out, nullptr);
}

// One forward with an event between kernels; ms[i] = device time of kernel i (0 routing logits,
// 1 top-k, 2 scan, 3 scatter, 4 gate-up GEMM, 5 down GEMM, 6 combine); n >= 7. Waits for it.
int moearc_x_prefill_profile(moearc_x_prefill *p, const uint16_t *x, unsigned n_tokens, const float *router_w,
                             const float *router_b, const float *residual, float *out, float *ms, int n) {
    if (!p || !ms || n < 7) return ERR;
    cudaEvent_t ev[8];
    for (auto &e : ev) cudaEventCreate(&e);
    int rc = prefill_forward(p, x, n_tokens, router_w, router_b, residual, out, ev);
    if (cudaStreamSynchronize(p->c->stream) != cudaSuccess) rc = ERR;
    for (int i = 0; i < 7; ++i) {
        ms[i] = 0.f;
        if (rc == OK) cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]);
    }
    for (auto &e : ev) cudaEventDestroy(e);
    return rc;
}

// Routing and grouping only (the first four kernels of moearc_x_prefill_forward): the tokens'
// activations end up in expert order (buffer 6), with the counts (3), the segment offsets (10)
// and the row of each (token, choice) (9). For expert parallelism, where the rows of each
// expert range travel to the rank that owns it before moearc_x_prefill_experts.
int moearc_x_prefill_route(moearc_x_prefill *p, const uint16_t *x, unsigned n_tokens, const float *router_w,
                           const float *router_b) {
    return prefill_route_x32(p, x, nullptr, n_tokens, router_w, router_b);
}
}  // extern "C"

namespace moearc {
// moearc_x_prefill_route with the router logits taken from x32 (f32 [T][H]) when it is given.
int prefill_route_x32(moearc_x_prefill *p, const uint16_t *x, const float *x32, unsigned n_tokens,
                      const float *router_w, const float *router_b) {
    if (p && p->mode8) return ERR_ARG;  // the expert-parallel steps take the bf16 and 4-bit forms
    if (!p || !x || !router_w) return ERR;
    if (n_tokens == 0) return OK;
    if ((int)n_tokens > p->T_max) return ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(router_w)) & 15) return ERR_ARG;
    cudaStream_t st = p->c->stream;
    const int T = (int)n_tokens;
    if (cudaMemsetAsync(p->cnt, 0, sizeof(int) * (p->E + 1), st) != cudaSuccess) return ERR;
    pf_route_args ra{x, x32, router_w, router_b, T, p->H, p->E, p->K, p->gating, p->logits, p->idx, p->wts, p->cnt, p->epos};
    k_pf_logits<<<logit_grid(T, p->E), 256, PF_LOGIT_TOK * p->H * 4, st>>>(ra);
    k_pf_topk<<<(T + 7) / 8, 256, 0, st>>>(ra);
    k_pf_scan<<<1, 1024, 0, st>>>(p->cnt, p->E, p->off, p->toff, p->cursor);
    const long pairs = (long)T * p->K;
    k_pf_scatter<<<(unsigned)((pairs + 7) / 8), 256, 0, st>>>(x, p->idx, p->epos, T, p->K, p->H, p->off, p->cursor,
                                                              p->perm, p->xp, p->mode4 ? 1 : 0, nullptr, nullptr, 0);
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

// The expert FFN of the 4-bit form over segments described in device memory, for a caller whose
// row counts never reach the host (the batched decoder's expert-parallel step, inside a captured
// graph): segment i is rows off[i] .. off[i+1] of rows (f16 [n_rows][n_embd]) for weight slot
// seg_w[i], toff its 32-row tile offsets (a segment with no tiles is skipped: gaps between the
// segments). act (f16 [n_rows][n_ff]) and y (f32 [n_rows][n_embd]) are indexed like rows.
int prefill_experts_dev(moearc_x_prefill *p, const uint16_t *rows, long n_rows, const int *off, const int *toff,
                        const int *seg_w, int n_seg, uint16_t *act, float *y) {
    if (!p || !rows || !off || !toff || !seg_w || !act || !y) return ERR;
    if (!p->mode4 || n_seg < 1 || n_seg > 1024) return ERR_ARG;
    CUtensorMap map_rows, map_act;
    if (!make_map(&map_rows, rows, n_rows, p->H, PF4_BN_SMALL) || !make_map(&map_act, act, n_rows, p->I, PF4_BN_SMALL))
        return ERR_ARG;
    pf_gemm_args g{};
    g.E = n_seg;
    g.off = off;
    g.toff = toff;
    g.seg_w = seg_w;
    g.act = p->act;
    g.alpha = p->alpha;
    g.limit = p->limit;
    g.act_out = act;
    g.y_out = y;
    g.status = p->status;
    g.Mrows = p->I;
    g.K = p->H;
    if (launch_gemm(p, 0, g, map_rows, PF4_BN_SMALL) != OK) return ERR;
    g.Mrows = p->H;
    g.K = p->I;
    return launch_gemm(p, 1, g, map_act, PF4_BN_SMALL);
}
}  // namespace moearc

extern "C" {

// The expert FFN over rows given in segments: segment s holds seg_counts[s] consecutive rows of
// rows_in (bf16 [n_rows][n_embd]) for expert seg_expert[s], an index into the experts last
// loaded by moearc_x_prefill_load_range (0 = its e_first). y_out (f32 [n_rows][n_embd]) gets one
// row per input row, in the same order; act_scratch is bf16 [n_rows][n_ff]. seg_counts and
// seg_expert are host arrays of n_seg <= 1024 entries whose counts sum to n_rows.
int moearc_x_prefill_experts(moearc_x_prefill *p, const uint16_t *rows_in, unsigned n_rows, const int *seg_counts,
                             const int *seg_expert, unsigned n_seg, uint16_t *act_scratch, float *y_out) {
    if (p && p->mode8) return ERR_ARG;  // the expert-parallel steps take the bf16 and 4-bit forms
    if (!p || !seg_counts || !seg_expert) return ERR;
    if (n_seg == 0 || n_seg > 1024) return ERR_ARG;
    long sum = 0;
    for (unsigned s = 0; s < n_seg; ++s) {
        if (seg_counts[s] < 0 || seg_expert[s] < 0 || seg_expert[s] >= p->E) return ERR_ARG;
        sum += seg_counts[s];
    }
    if (sum != (long)n_rows) return ERR_ARG;
    if (n_rows == 0) return OK;
    if (!rows_in || !act_scratch || !y_out) return ERR;
    if ((reinterpret_cast<uintptr_t>(rows_in) | reinterpret_cast<uintptr_t>(act_scratch)) & 15) return ERR_ARG;
    moearc_ctx *c = p->c;
    cudaStream_t st = c->stream;
    CUtensorMap map_rows, map_act;
    if (!make_map(&map_rows, rows_in, (long)n_rows, p->H) || !make_map(&map_act, act_scratch, (long)n_rows, p->I))
        return ERR_ARG;
    if (cudaMemcpyAsync(p->seg_cnt, seg_counts, sizeof(int) * n_seg, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(p->seg_w, seg_expert, sizeof(int) * n_seg, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return ERR;
    launch_scope ls(c, "moe_prefill_experts", (unsigned long)p->H, n_rows);
    k_pf_scan<<<1, 1024, 0, st>>>(p->seg_cnt, (int)n_seg, p->seg_off, p->seg_toff, p->seg_cur);
    pf_gemm_args g{};
    g.E = (int)n_seg;
    g.off = p->seg_off;
    g.toff = p->seg_toff;
    g.seg_w = p->seg_w;
    g.act = p->act;
    g.alpha = p->alpha;
    g.limit = p->limit;
    g.act_out = act_scratch;
    g.y_out = y_out;
    g.status = p->status;
    g.Mrows = p->I;
    g.K = p->H;
    if (!p->w16 && !p->w4) return ERR_ARG;
    if (launch_gemm(p, 0, g, map_rows) != OK) return ERR;
    g.Mrows = p->H;
    g.K = p->I;
    if (launch_gemm(p, 1, g, map_act) != OK) return ERR;
    return ls.finish();
}

// ---- expert parallelism over peer memory ----------------------------------------------------
//
// The exchange without a collective library: route_begin counts the rows per position; once the
// counts of every rank are known (the caller all-gathers them), route_dispatch's scatter stores
// each row straight into the receive buffer of the rank that owns it (peer memory, opened with
// moearc_x_ipc_open), and experts_to's down GEMM stores each result row straight into the
// y buffer of the rank it came from, at the row that rank's combine reads. The caller
// synchronises the ranks between the three steps (every rank's stream done, then a barrier).

int moearc_x_prefill_route_begin(moearc_x_prefill *p, const uint16_t *x, unsigned n_tokens, const float *router_w,
                                 const float *router_b) {
    if (!p || !x || !router_w) return ERR;
    if ((int)n_tokens > p->T_max) return ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(router_w)) & 15) return ERR_ARG;
    p->route_x = x;
    p->route_T = (int)n_tokens;
    cudaStream_t st = p->c->stream;
    if (cudaMemsetAsync(p->cnt, 0, sizeof(int) * (p->E + 1), st) != cudaSuccess) return ERR;
    if (n_tokens == 0) return OK;
    const int T = (int)n_tokens;
    const float *x32 = nullptr;
    pf_route_args ra{x, x32, router_w, router_b, T, p->H, p->E, p->K, p->gating, p->logits, p->idx, p->wts, p->cnt, p->epos};
    k_pf_logits<<<logit_grid(T, p->E), 256, PF_LOGIT_TOK * p->H * 4, st>>>(ra);
    k_pf_topk<<<(T + 7) / 8, 256, 0, st>>>(ra);
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

// dst_rows[r]: rank r's receive buffer (device or peer pointer, n_embd 16-bit words a row);
// dst_base[r]: the row of that buffer where this rank's rows start; positions are owner-major,
// n_local per rank (host arrays of n_ranks entries, n_ranks * n_local == E).
int moearc_x_prefill_route_dispatch(moearc_x_prefill *p, void *const *dst_rows, const int *dst_base, unsigned n_ranks,
                                    unsigned n_local) {
    if (!p || !dst_rows || !dst_base) return ERR;
    if (n_ranks == 0 || n_ranks > 1024 || n_ranks * n_local != (unsigned)p->E) return ERR_ARG;
    cudaStream_t st = p->c->stream;
    if (cudaMemcpyAsync(p->dst_rows, dst_rows, sizeof(void *) * n_ranks, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(p->dst_base, dst_base, sizeof(int) * n_ranks, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return ERR;
    k_pf_scan<<<1, 1024, 0, st>>>(p->cnt, p->E, p->off, p->toff, p->cursor);
    const long pairs = (long)p->route_T * p->K;
    if (pairs > 0)
        k_pf_scatter<<<(unsigned)((pairs + 7) / 8), 256, 0, st>>>(p->route_x, p->idx, p->epos, p->route_T, p->K, p->H,
                                                                  p->off, p->cursor, p->perm, p->xp, p->mode4 ? 1 : 0,
                                                                  p->dst_rows, p->dst_base, (int)n_local);
    if (cudaGetLastError() != cudaSuccess) return ERR;
    // the host arrays may go once the copies have been made
    return cudaStreamSynchronize(st) == cudaSuccess ? OK : ERR;
}

// moearc_x_prefill_experts with segment s's result rows stored to seg_dst[s] (host array of
// n_seg device or peer pointers, f32 rows of n_embd) instead of y_out.
int moearc_x_prefill_experts_to(moearc_x_prefill *p, const uint16_t *rows_in, unsigned n_rows, const int *seg_counts,
                                const int *seg_expert, unsigned n_seg, uint16_t *act_scratch, float *const *seg_dst) {
    if (p && p->mode8) return ERR_ARG;  // the expert-parallel steps take the bf16 and 4-bit forms
    if (!p || !seg_counts || !seg_expert || !seg_dst) return ERR;
    if (n_seg == 0 || n_seg > 1024) return ERR_ARG;
    long sum = 0;
    for (unsigned s = 0; s < n_seg; ++s) {
        if (seg_counts[s] < 0 || seg_expert[s] < 0 || seg_expert[s] >= p->E) return ERR_ARG;
        sum += seg_counts[s];
    }
    if (sum != (long)n_rows) return ERR_ARG;
    if (n_rows == 0) return OK;
    if (!rows_in || !act_scratch) return ERR;
    if ((reinterpret_cast<uintptr_t>(rows_in) | reinterpret_cast<uintptr_t>(act_scratch)) & 15) return ERR_ARG;
    if (!p->w16 && !p->w4) return ERR_ARG;
    moearc_ctx *c = p->c;
    cudaStream_t st = c->stream;
    CUtensorMap map_rows, map_act;
    if (!make_map(&map_rows, rows_in, (long)n_rows, p->H) || !make_map(&map_act, act_scratch, (long)n_rows, p->I))
        return ERR_ARG;
    if (cudaMemcpyAsync(p->seg_cnt, seg_counts, sizeof(int) * n_seg, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(p->seg_w, seg_expert, sizeof(int) * n_seg, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(p->seg_y, seg_dst, sizeof(float *) * n_seg, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return ERR;
    k_pf_scan<<<1, 1024, 0, st>>>(p->seg_cnt, (int)n_seg, p->seg_off, p->seg_toff, p->seg_cur);
    pf_gemm_args g{};
    g.E = (int)n_seg;
    g.off = p->seg_off;
    g.toff = p->seg_toff;
    g.seg_w = p->seg_w;
    g.act = p->act;
    g.alpha = p->alpha;
    g.limit = p->limit;
    g.act_out = act_scratch;
    g.status = p->status;
    g.Mrows = p->I;
    g.K = p->H;
    if (launch_gemm(p, 0, g, map_rows) != OK) return ERR;
    g.Mrows = p->H;
    g.K = p->I;
    g.seg_y = p->seg_y;
    if (launch_gemm(p, 1, g, map_act) != OK) return ERR;
    return cudaStreamSynchronize(st) == cudaSuccess ? OK : ERR;
}

// Device memory shared between the processes of one node: the 64-byte handle of an allocation
// (cudaMalloc'd, its start), its mapping in another process, and the mapping's release.
int moearc_x_ipc_handle(const void *ptr, void *handle) {
    if (!ptr || !handle) return ERR;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, const_cast<void *>(ptr)) != cudaSuccess) {
        cudaGetLastError();
        return ERR;
    }
    std::memcpy(handle, &h, sizeof(h));
    return OK;
}

int moearc_x_ipc_open(const void *handle, void **ptr) {
    if (!handle || !ptr) return ERR;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        *ptr = nullptr;
        return ERR;
    }
    return OK;
}

int moearc_x_ipc_close(void *ptr) {
    if (!ptr) return ERR;
    return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? OK : ERR;
}

// out[t] = residual[t] (if not NULL) + sum_m w[t,m] y[row(t,m)] for the tokens of the last
// moearc_x_prefill_route call, y_rows (f32 [T k][n_embd]) in the expert order that call produced.
int moearc_x_prefill_combine(moearc_x_prefill *p, const float *y_rows, unsigned n_tokens, const float *residual,
                             float *out) {
    if (!p || !y_rows || !out) return ERR;
    if (n_tokens == 0) return OK;
    if ((int)n_tokens > p->T_max) return ERR_ARG;
    const long n = (long)n_tokens * p->H;
    k_pf_combine<<<(unsigned)((n + 255) / 256), 256, 0, p->c->stream>>>(y_rows, p->perm, p->wts, residual, out,
                                                                        (int)n_tokens, p->K, p->H);
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

// 0 expert ids [T x k] (u32), 1 gating weights [T x k], 2 logits [T x E], 3 per-expert counts
// [E] (int), 4 expanded gate-up weights [E][2][n_ff][n_embd] (bf16), 5 expanded down weights,
// 6 the activations in expert order [T k][n_embd] (bf16), 7 the SwiGLU outputs [T k][n_ff]
// (bf16), 8 the down rows [T k][n_embd] (f32), 9 the row of each (token, choice) [T k] (int),
// 10 the expert segment offsets [E + 1] (int).
void *moearc_x_prefill_buffer(moearc_x_prefill *p, int which) {
    if (!p) return nullptr;
    switch (which) {
    case 0: return p->idx;
    case 1: return p->wts;
    case 2: return p->logits;
    case 3: return p->cnt;
    case 4: return p->wgu;
    case 5: return p->wdn;
    case 6: return p->xp;
    case 7: return p->actb;
    case 8: return p->y;
    case 9: return p->perm;
    case 10: return p->off;
    default: return nullptr;
    }
}

int moearc_x_prefill_status(moearc_x_prefill *p) {
    if (!p) return ERR;
    int s = 0;
    if (cudaMemcpyAsync(&s, p->status, sizeof(int), cudaMemcpyDeviceToHost, p->c->stream) != cudaSuccess ||
        cudaMemsetAsync(p->status, 0, sizeof(int), p->c->stream) != cudaSuccess ||
        cudaStreamSynchronize(p->c->stream) != cudaSuccess)
        return ERR;
    return s;
}

}  // extern "C"
