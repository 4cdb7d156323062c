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
constexpr int WSEG = 3;          // partial records a warp may hold in one phase
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
    int q_mp, o_mp;  // slots per row of the partial arrays: maxc rounded up to a multiple of 4
    int KP;          // slots per row of the expert outputs: K rounded up to 4 or 8
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

// The key span of a decode step at position pos (window 0: all keys) and its split into runs of
// a multiple of 256 keys over at most max_splits CTAs (a shorter split costs more in partials and
// merging than the keys it takes off the others).
struct att_span {
    int kv_begin, n_tok, kps, n_splits;
};
__device__ __forceinline__ att_span span_of(int pos, int window, int max_splits) {
    att_span r;
    r.n_tok = pos + 1;
    r.kv_begin = (window > 0 && r.n_tok > window) ? r.n_tok - window : 0;
    const int span = r.n_tok - r.kv_begin;
    const int kps = (span + max_splits - 1) / max_splits;
    r.kps = (kps + 255) / 256 * 256;
    r.n_splits = (span + r.kps - 1) / r.kps;
    return r;
}

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

// One warp's ring: the piece sequence it has issued and consumed, the issue cursor over the
// step's phases, and the gates that hold the cursor (kept in shared memory so the issue code,
// one copy shared by every call site, can update it).
struct wring {
    int n_iss, n_con;           // pieces issued / consumed
    int l, ph, it, hi, done;    // issue cursor: block, ring phase, next item, end of the range
    int att_done, routed, acts_ok;
    int n_def, dn_k0;           // down pieces of block `routed` issued before their activations
    int lo[5], hiR[5];          // this warp's item range per ring phase (the same in every block)
    const uint8_t *base;        // the weights of the cursor's (block, phase), read once per phase
};

struct cta_state {
    uint64_t bars[NW][RS];
    wring R[NW];
    double rot_c[HD / 2], rot_s[HD / 2];  // RoPE rotation at this step's position, x mscale
    unsigned idx[8];
    float wts[8];
    float red1[NW];
    int rec_lo[NW], rec_n[NW];
    int flag, last;
};

struct piece {
    const uint8_t *src, *asrc;
    unsigned bytes, abytes;
    int n;
};

// The weights a ring phase of block l streams from.
__device__ __forceinline__ const uint8_t *phase_base(const step_args &a, int l, int ph) {
    const step_layer &Lb = a.L[l];
    switch (ph) {
    case R_QKV: return Lb.wqkv;
    case R_O: return Lb.wo;
    case R_RT: return reinterpret_cast<const uint8_t *>(Lb.router);
    case R_GU: return Lb.gateup;
    default: return Lb.down;
    }
}

__device__ __forceinline__ piece describe(const step_args &a, const cta_state &S, int warp, int c, int G,
                                          const uint8_t *base, int ph, int it, int hi) {
    piece p{nullptr, nullptr, 0u, 0u, 1};
    if (ph == R_QKV || ph == R_O) {
        p.n = min(DCH, hi - it);
        p.src = base + (size_t)it * DT;
        p.bytes = (unsigned)(p.n * DT);
    } else if (ph == R_RT) {
        const int e = c + G * it;
        p.src = base + ((size_t)e * a.H + (size_t)warp * (a.H / NW)) * 4;
        p.bytes = (unsigned)(a.H / NW * 4);
    } else if (ph == R_GU) {
        const int seg = it / a.gu_nkt, kt = it - seg * a.gu_nkt;
        p.n = min(min(a.ch_gu, a.gu_nkt - kt), hi - it);
        const int m = seg / a.gu_ntr, tr = seg - m * a.gu_ntr;
        p.src = base + (size_t)S.idx[m] * a.gu_stride + ((size_t)tr * a.gu_nkt + kt) * a.pair_bytes;
        p.bytes = (unsigned)(p.n * a.pair_bytes);
    } else {
        const int seg = it / a.dn_nkt, kt = it - seg * a.dn_nkt;
        p.n = min(min(a.ch_dn, a.dn_nkt - kt), hi - it);
        const int m = seg / a.dn_ntr, tr = seg - m * a.dn_ntr;
        p.src = base + (size_t)S.idx[m] * a.dn_stride + ((size_t)tr * a.dn_nkt + kt) * a.tile_bytes;
        p.bytes = (unsigned)(p.n * a.tile_bytes);
        p.asrc = reinterpret_cast<const uint8_t *>(a.actfrag + (size_t)m * (a.I / 32) * 32 + (size_t)kt * 64);
        p.abytes = (unsigned)(p.n * 256);
    }
    return p;
}

// Keep the warp's ring full: issue pieces in sequence while a stage is free and the next
// piece's addresses are known (warps 0-3 lend their rings to attention until it is done;
// expert pieces need the block's routing). A down piece issued before its block's
// activations exist gets them later (issue_deferred). Called by the whole warp.
__device__ __noinline__ void pump(const step_args &a, cta_state &S, uint8_t *ring, int warp, int lane, int c, int G) {
    __syncwarp();
    if (lane == 0) {  // the warp's lane 0 alone runs the cursor and issues
        wring &w = S.R[warp];
        while (!w.done && w.n_iss - w.n_con < RS) {
            if (w.it >= w.hi) {
                if (++w.ph == R_END) {
                    w.ph = R_QKV;
                    if (++w.l == a.n_layer) {
                        w.done = 1;
                        break;
                    }
                }
                w.it = w.lo[w.ph];
                w.hi = w.hiR[w.ph];
                if (w.it < w.hi) w.base = phase_base(a, w.l, w.ph);
                continue;
            }
            if (w.ph == R_RT && warp < AW && w.att_done < w.l) break;
            if ((w.ph == R_GU || w.ph == R_DN) && w.routed < w.l) break;
            const piece p = describe(a, S, warp, c, G, w.base, w.ph, w.it, w.hi);
            const int stage = w.n_iss % RS;
            const bool with_acts = p.abytes && w.acts_ok >= w.l;
            if (p.abytes && !with_acts) {
                if (w.n_def == 0) w.dn_k0 = w.n_iss;
                ++w.n_def;
            }
            uint64_t *bar = &S.bars[warp][stage];
            uint8_t *st = ring + (size_t)stage * SB;
            fence_proxy_async();
            mbar_expect_tx(bar, p.bytes + p.abytes);
            if (w.ph == R_RT) bulk_g2s(st, p.src, p.bytes, bar);
            else bulk_g2s_hint(st, p.src, p.bytes, bar, policy_evict_first());
            if (with_acts) bulk_g2s(st + p.bytes, p.asrc, p.abytes, bar);
            w.it += p.n;
            ++w.n_iss;
        }
    }
    __syncwarp();
}

// The activation copies of block l's down pieces that were issued before the activations
// existed (after the grid barrier that follows the gate-up phase).
__device__ __noinline__ void issue_deferred(const step_args &a, cta_state &S, uint8_t *ring, int warp, int lane, int c,
                                            int G, int l) {
    wring &w = S.R[warp];
    __syncwarp();
    if (lane == 0) {
        int it = w.lo[R_DN];
#pragma unroll 1
        for (int j = 0; j < w.n_def; ++j) {
            const piece p = describe(a, S, warp, c, G, a.L[l].down, R_DN, it, w.hiR[R_DN]);
            const int stage = (w.dn_k0 + j) % RS;
            bulk_g2s(ring + (size_t)stage * SB + p.bytes, p.asrc, p.abytes, &S.bars[warp][stage]);
            it += p.n;
        }
        w.n_def = 0;
    }
    __syncwarp();
}

// Ask L2 for block l's tensors this CTA reads first in that block: its shares of the Q/K/V and
// O tiles, the norms (one CTA each), and, for the CTA that will attend over a short span, that
// span's K/V rows. Run by one lane while the CTA waits on something else; the bytes then stream
// while HBM would otherwise idle (attention, the router, the barriers), and the phases that use
// them find them in L2.
__device__ __noinline__ void prefetch_block(const step_args &a, int l, int pos) {
    const int c = blockIdx.x, G = gridDim.x;
    const step_layer &Lb = a.L[l];
    const uint64_t pol = policy_evict_last();
    auto range = [&](const uint8_t *base, long T) {
        const long t0 = T * c / G, t1 = T * (c + 1) / G;
#pragma unroll 1
        for (long t = t0; t < t1; t += 16) prefetch_l2_hint(base + (size_t)t * DT, (unsigned)(min(16L, t1 - t) * DT), pol);
    };
    range(Lb.wqkv, a.q_T);
    range(Lb.wo, a.o_T);
    if (c == 0) prefetch_l2_hint(Lb.attn_norm, (unsigned)(a.H * 4), pol);
    if (c == 1 % G) prefetch_l2_hint(Lb.ffn_norm, (unsigned)(a.H * 4), pol);
    // the attention span of this CTA's (KV head, split) unit, when short: whole pages of 32
    // keys, the unit's head only (64 bf16 = 128 bytes of each key's row)
    const att_span sp = span_of(pos, Lb.window, a.max_splits);
    if (sp.n_tok - sp.kv_begin > 4096 || c >= a.n_kv * sp.n_splits) return;
    const int kvh = c / sp.n_splits, split = c % sp.n_splits;
    const int s0 = sp.kv_begin + split * sp.kps, s1 = min(s0 + sp.kps, sp.n_tok);
#pragma unroll 1
    for (int j = s0; j < s1; ++j) {
        const size_t off = ((size_t)Lb.table[j >> 5] * 32 + (j & 31)) * a.n_kv * HD + (size_t)kvh * HD;
        prefetch_l2_hint(Lb.k_pages + off, HD * 2, pol);
        prefetch_l2_hint(Lb.v_pages + off, HD * 2, pol);
    }
}

__device__ __noinline__ void trace_point(unsigned long long *trace, int i) { trace[i] = xnow(); }

// Grid barrier: every CTA arrives, then waits (bounded) for all. False (the same in every
// thread of the CTA) when a wait of this CTA or of another has given up. All threads call it.
__device__ __noinline__ bool gsync(const step_args &a, cta_state &S, unsigned nbar, bool alive) {
    const bool all_alive = __syncthreads_and(alive);
    if (threadIdx.x == 0) {
        int ok = 0;
        if (!all_alive) {
            atomicExch(a.sync + 1, 1u);
        } else {
            __threadfence();
            atomicAdd(a.sync, 1u);
            const unsigned target = nbar * gridDim.x + a.phantom;
            ok = 1;
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
        }
        S.flag = ok;
    }
    __syncthreads();
    return S.flag != 0;
}

__device__ __forceinline__ float *rec(float *red, int w, int slot) { return red + ((size_t)w * WSEG + slot) * 32; }

// Wait (bounded) for the warp's next piece; null when the wait gave up (the abort word is then
// raised so every CTA stops at its next barrier).
__device__ __forceinline__ const uint8_t *wait_piece(const step_args &a, cta_state &S, uint8_t *ring, int warp, int lane,
                                                     bool &alive) {
    const int n = S.R[warp].n_con;
    const int stage = n % RS;
    // the outcome is made the warp's (all lanes poll; every lane must take the same path)
    if (!__all_sync(0xffffffffu, mbar_wait(&S.bars[warp][stage], (unsigned)((n / RS) & 1), a.status))) {
        alive = false;
        if (lane == 0) atomicExch(a.sync + 1, 1u);
        return nullptr;
    }
    return ring + (size_t)stage * SB;
}
__device__ __forceinline__ void release(const step_args &a, cta_state &S, uint8_t *ring, int warp, int lane, int c,
                                        int G) {
    __syncwarp();
    if (lane == 0) ++S.R[warp].n_con;
    __syncwarp();
    pump(a, S, ring, warp, lane, c, G);
}

// A dense phase's share of this warp: packed bf16 tiles [lo, hi) of a matrix with nkt k-tiles a
// row, against the B fragments in xs; per tile-row touched, one record of 16 row sums.
__device__ __noinline__ void dense_consume(const step_args &a, cta_state &S, uint8_t *ring, const uint8_t *xs,
                                           float *red, int warp, int lane, int c, int G, int lo, int hi, int nkt,
                                           bool &alive) {
    int rec_lo = -1, nrec = 0, cur = -1;
    float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
    const int n8 = lane >> 2, qd = lane & 3;
    const uint32_t *bsm = reinterpret_cast<const uint32_t *>(xs);
    int tr = lo / nkt, kt = lo - tr * nkt;
    for (int t = lo; t < hi && alive;) {
        const uint8_t *st = wait_piece(a, S, ring, warp, lane, alive);
        if (!st) break;
        const int n = min(DCH, hi - t);
#pragma unroll 1
        for (int i = 0; i < n; ++i) {
            if (tr != cur) {
                if (cur >= 0) {
                    const float a0 = acc0[0] + acc1[0], a1 = acc0[1] + acc1[1];
                    const float a2 = acc0[2] + acc1[2], a3 = acc0[3] + acc1[3];
                    const float p0 = __shfl_xor_sync(0xffffffffu, a0, 1);
                    const float p2 = __shfl_xor_sync(0xffffffffu, a2, 1);
                    if (qd == 0) {
                        float *r = rec(red, warp, cur - rec_lo);
                        r[n8] = (a0 + a1) + p0;
                        r[n8 + 8] = (a2 + a3) + p2;
                    }
                }
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
        release(a, S, ring, warp, lane, c, G);
    }
    if (cur >= 0) {
        const float a0 = acc0[0] + acc1[0], a1 = acc0[1] + acc1[1];
        const float a2 = acc0[2] + acc1[2], a3 = acc0[3] + acc1[3];
        const float p0 = __shfl_xor_sync(0xffffffffu, a0, 1);
        const float p2 = __shfl_xor_sync(0xffffffffu, a2, 1);
        if (qd == 0) {
            float *r = rec(red, warp, cur - rec_lo);
            r[n8] = (a0 + a1) + p0;
            r[n8 + 8] = (a2 + a3) + p2;
        }
    }
    if (lane == 0) {
        S.rec_lo[warp] = rec_lo;
        S.rec_n[warp] = nrec;
    }
}

// After every warp's records: the CTA's partial of each unit (tile-row or segment) it touched,
// its warps summed in order. Units [u0, u1) with `width` values each (16 or 32) per record.
// Returns the sum of record value v of unit u through out(u, v, s).
template <typename F>
__device__ __forceinline__ void cta_reduce(const cta_state &S, const float *red, int u0, int u1, int width, F &&out) {
#pragma unroll 1
    for (int e = threadIdx.x; e < (u1 - u0) * width; e += NW * 32) {
        const int u = u0 + e / width, v = e % width;
        float s = 0.f;
#pragma unroll 1
        for (int w = 0; w < NW; ++w) {
            const int k = u - S.rec_lo[w];
            if (S.rec_n[w] > 0 && k >= 0 && k < S.rec_n[w]) s += red[((size_t)w * WSEG + k) * 32 + v];
        }
        out(u, v, s);
    }
}

// Row `row` of a dense phase's output: part is laid [row][mp], slot k holding the k-th
// contributing CTA's partial (slots past a row's contributors stay zero), summed in slot order.
__device__ __forceinline__ float row_slots(const float *part, int mp, int row) {
    const float4 *p = reinterpret_cast<const float4 *>(part + (size_t)row * mp);
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q)
        if (q < mp / 4) {
            const float4 v = __ldcg(p + q);
            s += v.x;
            s += v.y;
            s += v.z;
            s += v.w;
        }
    return s;
}

// Rows r0 + i (i < nr) of a dense phase's output into dst: thread t of a group of nt takes rows
// t, t + nt, ..., four rows' loads issued before any is summed. One copy of the code serves every
// caller (the instruction cache, not the arithmetic, bounds these short phases).
__device__ __noinline__ void gather_rows(const float *part, int mp, int r0, int nr, int t, int nt, float *dst) {
#pragma unroll 1
    for (int i0 = t; i0 < nr; i0 += 4 * nt) {
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = row_slots(part, mp, r0 + min(i0 + j * nt, nr - 1));
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (i0 + j * nt < nr) dst[i0 + j * nt] = v[j];
    }
}

__device__ __forceinline__ float block_sum(cta_state &S, float v, int warp, int lane) {
    v = warp_sum(v);
    if (lane == 0) S.red1[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) t += S.red1[w];
    __syncthreads();
    return t;
}

// h entering block l (the input, or the previous block's residual plus the router-order combine
// of its experts' outputs, laid [row][KP]), for this thread's values i = tid + 512 j: four
// values' loads issued before any is summed.
__device__ __noinline__ void residual_in(const step_args &a, const cta_state &S, int l, float (&hv)[HMAX]) {
    const int tid = threadIdx.x;
    const float *base = l == 0 ? a.in : a.hmid;
#pragma unroll 1
    for (int j0 = 0; j0 < HMAX; j0 += 4) {
        float hm[4];
        float4 d[4][2];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = min(tid + (j0 + j) * NW * 32, a.H - 1);
            hm[j] = __ldcg(base + i);
            const float4 *dp = reinterpret_cast<const float4 *>(a.down_out + (size_t)i * a.KP);
            d[j][0] = l > 0 ? __ldcg(dp) : make_float4(0.f, 0.f, 0.f, 0.f);
            d[j][1] = (l > 0 && a.KP > 4) ? __ldcg(dp + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float o[8] = {d[j][0].x, d[j][0].y, d[j][0].z, d[j][0].w, d[j][1].x, d[j][1].y, d[j][1].z, d[j][1].w};
            float acc = 0.f;
#pragma unroll
            for (int m = 0; m < 8; ++m)
                if (m < a.K) acc = fmaf(S.wts[m], o[m], acc);
            const bool in = tid + (j0 + j) * NW * 32 < a.H;
            hv[j0 + j] = !in ? 0.f : (l == 0 ? hm[j] : hm[j] + acc);
        }
    }
}

// Split-K flash decode of one (KV head, key split) by warps 0-3 (see step.cuh): q, and for the
// split holding the step's token k and v, from the Q/K/V partials; RoPE; the step's K/V into
// the paged cache; tensor-core score and value products over the split's keys; the four warps
// merged; the head group's output, or the split's partial and, for the last split to finish,
// the merge of all splits.
__device__ __noinline__ void attention_unit(const step_args &a, cta_state &S, const step_layer &Lb, uint8_t *smem,
                                            float *red, int pos, int kvh, int split, const att_span &sp) {
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int group = a.group, n_splits = sp.n_splits;
    const int s0 = sp.kv_begin + split * sp.kps, s1 = min(s0 + sp.kps, sp.n_tok);
    const bool last = split == n_splits - 1;
    float *qf = red;                   // [group][64] f32, then k [64], v [64]
    float *kf = red + MAXG * HD, *vf = kf + HD;
    // raw q (and k, v) rows: the group's query heads, then this head's key and value rows
    {
        // q rows of the group's heads, then (last split) this head's k and v rows: every load
        // issued before any is summed
        const int nq = group * HD, n = nq + (last ? 2 * HD : 0);
        constexpr int PER = (MAXG + 2) * HD / (AW * 32);  // rows per thread at most
        float v[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int i = t + j * AW * 32;
            const int row = i < nq ? kvh * nq + i : (i < nq + HD ? a.Dq + kvh * HD + (i - nq) : a.Dq + a.Dkv + kvh * HD + (i - nq - HD));
            v[j] = i < n ? row_slots(a.qkv_part, a.q_mp, row) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int i = t + j * AW * 32;
            if (i < n) (i < nq ? qf[i] : (i < nq + HD ? kf[i - nq] : vf[i - nq - HD])) = v[j];
        }
    }
    bar_att();
    // NeoX RoPE on q and k: pairs (d, d + 32) turn by the step's precomputed rotation of pair d
    const int n_pairs = group * 32 + (last ? 32 : 0);
#pragma unroll 1
    for (int i = t; i < n_pairs; i += AW * 32) {
        const int hs = i >> 5, p = i & 31;
        float *row = hs < group ? qf + hs * HD : kf;
        const double x0 = row[p], x1 = row[p + 32];
        row[p] = (float)(x0 * S.rot_c[p] - x1 * S.rot_s[p]);
        row[p + 32] = (float)(x0 * S.rot_s[p] + x1 * S.rot_c[p]);
    }
    if (last) {
        // the step's K/V into the cache (read by later steps), and the same bf16 values for
        // this step's own key, which joins below rather than through the cache
        const size_t page = Lb.table[pos / 32];
        const size_t off = ((page * 32 + (size_t)(pos % 32)) * a.n_kv + kvh) * HD;
#pragma unroll 1
        for (int i = t; i < HD; i += AW * 32) {
            const uint16_t kb = f32_to_bf16_bits(kf[i]), vb = f32_to_bf16_bits(vf[i]);
            Lb.k_pages[off + i] = kb;
            Lb.v_pages[off + i] = vb;
            kf[i] = bf16_bits_to_f32(kb);
            vf[i] = bf16_bits_to_f32(vb);
        }
    }
    bar_att();
    const int s1c = last ? sp.n_tok - 1 : s1;  // keys read from the cache
    const int qd = lane & 3, hr = lane >> 2;
    uint16_t *ws = reinterpret_cast<uint16_t *>(smem + (size_t)warp * RS * SB);
    uint32_t qa[HD / 16][4];
    {
        const bool live = hr < group;
        const float *qh = qf + (live ? hr : 0) * HD;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
            const int c0 = 16 * kk + 2 * qd, c1 = c0 + 8;
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
    auto load_tile = [&](int t0, int stg) {
        uint16_t *kt = ws + stg * 2 * TK * HD, *vt = kt + TK * HD;
#pragma unroll
        for (int cc = lane; cc < TK * CH; cc += 32) {
            const int r = cc / CH, ch = cc % CH;
            const int j = t0 + r;
            const bool valid = j < s1c;
            const int jj = valid ? j : s0;
            const size_t off = ((size_t)Lb.table[jj >> 5] * 32 + (jj & 31)) * row_elems + (size_t)kvh * HD + ch * 8;
            const int dst = r * HD + ((ch ^ (r & 7)) * 8);
            cp_async16(kt + dst, Lb.k_pages + off, valid);
            cp_async16(vt + dst, Lb.v_pages + off, valid);
        }
    };
    int t0 = s0 + warp * TK;
    int stg = 0;
    if (t0 < s1c) load_tile(t0, 0);
    cp_async_commit();
    for (; t0 < s1c; t0 += AW * TK) {
        const int tn = t0 + AW * TK;
        if (tn < s1c) load_tile(tn, stg ^ 1);
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
                const int j = t0 + 8 * nn + 2 * qd + e;
                const float v = (sacc[nn][e] + sacc[nn][e + 2]) * a.scale;
                sc[2 * nn + e] = j < s1c ? v : -INFINITY;
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
    // the four warps' partials, and for the last split the step's own key as a fifth (its
    // score, weight 1, its value), merged through warp 0's ring (every warp's tiles are done with)
    bar_att();
    float *fm = reinterpret_cast<float *>(smem);  // [AW + 1][8] m, [AW + 1][8] l, [AW + 1][8][HD] acc
    float *fl = fm + (AW + 1) * 8, *fo = fm + 2 * (AW + 1) * 8;
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
    const int nent = last ? AW + 1 : AW;
    if (last)
#pragma unroll 1
        for (int h = warp; h < 8; h += AW) {
            float dot = 0.f;
            if (h < group) dot = fmaf(qf[h * HD + lane], kf[lane], qf[h * HD + lane + 32] * kf[lane + 32]);
            dot = warp_sum(dot);
            if (lane == 0) {
                fm[AW * 8 + h] = h < group ? dot * a.scale : -INFINITY;
                fl[AW * 8 + h] = 1.f;
            }
            fo[(AW * 8 + h) * HD + lane] = vf[lane];
            fo[(AW * 8 + h) * HD + lane + 32] = vf[lane + 32];
        }
    bar_att();
#pragma unroll 1
    for (int e = t; e < group * HD; e += AW * 32) {
        const int h = e / HD, d = e % HD;
        float M = -INFINITY;
        for (int w = 0; w < nent; ++w) M = fmaxf(M, fm[w * 8 + h]);
        float Lsum = 0.f, v = 0.f;
        for (int w = 0; w < nent; ++w) {
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
        // the last split of this KV head to arrive merges all of them (the sink joins as one
        // more logit with no value) and re-arms the counter
        fence_acq_rel_gpu();
        bar_att();
        if (t == 0) S.last = atomicAdd(a.att_ctr + kvh, 1u) == (unsigned)n_splits - 1;
        bar_att();
        if (S.last) {
            fence_acq_rel_gpu();
#pragma unroll 1
            for (int e = t; e < group * HD; e += AW * 32) {
                const int h = e / HD, d = e % HD, hq = kvh * group + h;
                const float *ml = a.att_ml + (size_t)hq * n_splits * 2;
                const float sk = Lb.sinks ? __ldg(Lb.sinks + hq) : -INFINITY;
                float M = sk;
#pragma unroll 1
                for (int sp = 0; sp < n_splits; ++sp) M = fmaxf(M, __ldcg(ml + 2 * sp));
                float Lsum = Lb.sinks ? exp2f((sk - M) * LOG2E) : 0.f, v = 0.f;
#pragma unroll 1
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

template <int WT>
__global__ void __launch_bounds__(NW * 32, 1) k_step(const __grid_constant__ step_args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ cta_state S;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int c = blockIdx.x, G = gridDim.x;
    uint8_t *ring = smem + (size_t)warp * RS * SB;
    uint8_t *xs = smem + (size_t)NW * RS * SB;
    float *red = reinterpret_cast<float *>(xs + a.xs_bytes);  // [NW][WSEG][32]
    const int H = a.H;
    const int pos = *a.pos;

    // ---- this warp's ring: its item ranges (the same in every block) and cursor ----
    if (lane == 0) {
        for (int s = 0; s < RS; ++s) mbar_init(&S.bars[warp][s], 1);
        fence_mbar_init();
        wring &w = S.R[warp];
        const long GW = (long)G * NW, gw = (long)c * NW + warp;
        w.lo[R_QKV] = (int)(a.q_T * gw / GW);
        w.hiR[R_QKV] = (int)(a.q_T * (gw + 1) / GW);
        w.lo[R_O] = w.hiR[R_O] = 0;
        if (warp >= AW) {
            const long GWo = (long)G * (NW - AW), gwo = (long)c * (NW - AW) + (warp - AW);
            w.lo[R_O] = (int)(a.o_T * gwo / GWo);
            w.hiR[R_O] = (int)(a.o_T * (gwo + 1) / GWo);
        }
        w.lo[R_RT] = 0;
        w.hiR[R_RT] = c < a.E ? (a.E - 1 - c) / G + 1 : 0;
        const long Sg = (long)a.K * a.gu_ntr, sg0 = Sg * c / G, sg1 = Sg * (c + 1) / G;
        const long Pg = (sg1 - sg0) * a.gu_nkt;
        w.lo[R_GU] = (int)(sg0 * a.gu_nkt + Pg * warp / NW);
        w.hiR[R_GU] = (int)(sg0 * a.gu_nkt + Pg * (warp + 1) / NW);
        const long Sd = (long)a.K * a.dn_ntr, sd0 = Sd * c / G, sd1 = Sd * (c + 1) / G;
        const long Pd = (sd1 - sd0) * a.dn_nkt;
        w.lo[R_DN] = (int)(sd0 * a.dn_nkt + Pd * warp / NW);
        w.hiR[R_DN] = (int)(sd0 * a.dn_nkt + Pd * (warp + 1) / NW);
        w.n_iss = w.n_con = 0;
        w.l = 0;
        w.ph = R_QKV;
        w.it = w.lo[R_QKV];
        w.hi = w.hiR[R_QKV];
        w.done = a.n_layer == 0;
        w.att_done = w.routed = w.acts_ok = -1;
        w.n_def = w.dn_k0 = 0;
        w.base = phase_base(a, 0, R_QKV);
    }
    __syncwarp();
    pump(a, S, ring, warp, lane, c, G);  // the first block's Q/K/V weights start streaming now
    if (warp == NW - 2 && lane == 0) prefetch_block(a, 0, pos);
    // the RoPE rotation of this step's position, pair p: the angle pos * freq[p] (the YaRN blend
    // folded into freq), reduced by 2 pi in two steps so large positions keep full precision
    if (warp == NW - 1) {
        const double th = (double)pos * __ldg(a.rope_freq + lane);
        const double k2 = rint(th * 0.15915494309189535);
        double r = fma(-k2, 6.283185307179586, th);
        r = fma(-k2, 2.4492935982947064e-16, r);
        double sn, cs;
        sincos(r, &sn, &cs);
        S.rot_c[lane] = cs * a.mscale;
        S.rot_s[lane] = sn * a.mscale;
    }

    bool alive = true;  // none of this warp's waits has given up
    bool synced = true; // every grid barrier so far opened (the same in the whole CTA)
    unsigned nbar = 0;
    // trace point k of phase ph: 0 start (the barrier opened), 1 inputs ready, 2 warp 0 done
    // with its share, 3 end (before the barrier)
    auto stamp = [&](int l, int ph, int k) {
        if (a.trace && tid == 0) trace_point(a.trace, ((l * NPH + ph) * 4 + k) * G + c);
    };

    for (int l = 0; l < a.n_layer; ++l) {
        const step_layer &Lb = a.L[l];
        // ================= QKV =================
        if (l > 0 && !(synced = gsync(a, S, ++nbar, alive))) break;
        stamp(l, 0, 0);
        {
            float hv[HMAX];
            residual_in(a, S, l, hv);
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < HMAX; ++j) ss = fmaf(hv[j], hv[j], ss);
            const float scale = 1.0f / sqrtf(block_sum(S, ss, warp, lane) / (float)H + a.eps);
            const int h0 = (int)((long)H * c / G), h1 = (int)((long)H * (c + 1) / G);
            uint16_t *xs16 = reinterpret_cast<uint16_t *>(xs);
#pragma unroll 2
            for (int j = 0; j < HMAX; ++j) {
                const int i = tid + j * NW * 32;
                if (i < H) {
                    if (i >= h0 && i < h1) a.hbuf[i] = hv[j];
                    dense_frag_put(xs16, i, (hv[j] * scale) * __ldg(Lb.attn_norm + i));
                }
            }
            __syncthreads();
        }
        stamp(l, 0, 1);
        const wring &W = S.R[warp];
        dense_consume(a, S, ring, xs, red, warp, lane, c, G, W.lo[R_QKV], W.hiR[R_QKV], a.q_nkt, alive);
        stamp(l, 0, 2);
        __syncthreads();
        {
            const long ta = a.q_T * c / G, tb = a.q_T * (c + 1) / G;
            if (tb > ta) {
                const int tr0 = (int)(ta / a.q_nkt), tr1 = (int)((tb - 1) / a.q_nkt);
                cta_reduce(S, red, tr0, tr1 + 1, 16, [&](int tr, int r, float s) {
                    const int slot = c - owner_of(a.q_T, G, (long)tr * a.q_nkt);
                    a.qkv_part[((size_t)tr * 16 + r) * a.q_mp + slot] = s;
                });
            }
        }
        stamp(l, 0, 3);
        // ================= ATT =================
        if (!(synced = gsync(a, S, ++nbar, alive))) break;
        stamp(l, 1, 0);
        if (warp == NW - 1 && lane == 0 && l + 1 < a.n_layer) prefetch_block(a, l + 1, pos);
        {
            const att_span sp = span_of(pos, Lb.window, a.max_splits);
            const int n_splits = sp.n_splits;
            stamp(l, 1, 1);
            if (warp < AW && c < a.n_kv * n_splits)
                attention_unit(a, S, Lb, smem, red, pos, c / n_splits, c % n_splits, sp);
            stamp(l, 1, 2);
            if (warp < AW) {
                if (lane == 0) S.R[warp].att_done = l;
                __syncwarp();
                pump(a, S, ring, warp, lane, c, G);
            }
        }
        stamp(l, 1, 3);
        // ================= O =================
        if (!(synced = gsync(a, S, ++nbar, alive))) break;
        stamp(l, 2, 0);
        {
            uint16_t *xs16 = reinterpret_cast<uint16_t *>(xs);
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = tid + j * NW * 32;
                v[j] = i < a.Dq ? __ldcg(a.att + i) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = tid + j * NW * 32;
                if (i < a.Dq) dense_frag_put(xs16, i, v[j]);
            }
            __syncthreads();
        }
        stamp(l, 2, 1);
        dense_consume(a, S, ring, xs, red, warp, lane, c, G, W.lo[R_O], W.hiR[R_O], a.o_nkt, alive);
        stamp(l, 2, 2);
        __syncthreads();
        {
            const long ta = a.o_T * c / G, tb = a.o_T * (c + 1) / G;
            if (tb > ta) {
                const int tr0 = (int)(ta / a.o_nkt), tr1 = (int)((tb - 1) / a.o_nkt);
                cta_reduce(S, red, tr0, tr1 + 1, 16, [&](int tr, int r, float s) {
                    const int slot = c - owner_of(a.o_T, G, (long)tr * a.o_nkt);
                    a.o_part[((size_t)tr * 16 + r) * a.o_mp + slot] = s;
                });
            }
        }
        stamp(l, 2, 3);
        // ================= ROUTE =================
        if (!(synced = gsync(a, S, ++nbar, alive))) break;
        stamp(l, 3, 0);
        float *xf = reinterpret_cast<float *>(xs);                // [H] the MoE input, f32
        uint16_t *xg = reinterpret_cast<uint16_t *>(xs + 4 * H);  // its expert fragments
        {
            // h + O, each value's contributors loaded at once, into xf first
            gather_rows(a.o_part, a.o_mp, 0, H, tid, NW * 32, xf);
            float hv[HMAX];
#pragma unroll
            for (int j = 0; j < HMAX; ++j) {
                const int i = tid + j * NW * 32;
                hv[j] = i < H ? __ldcg(a.hbuf + i) : 0.f;
            }
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < HMAX; ++j) {
                const int i = tid + j * NW * 32;
                if (i < H) hv[j] += xf[i];
                ss = fmaf(hv[j], hv[j], ss);
            }
            const float scale = 1.0f / sqrtf(block_sum(S, ss, warp, lane) / (float)H + a.eps);
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
        stamp(l, 3, 1);
        // router row c + G j, slice `warp` of it (H / 16 columns), one piece each
        const int n_rt = W.hiR[R_RT];
#pragma unroll 1
        for (int j = 0; j < n_rt && alive; ++j) {
            const uint8_t *st = wait_piece(a, S, ring, warp, lane, alive);
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
            if (lane == 0) rec(red, warp, 0)[j] = acc;  // j < 32 WSEG: checked at plan time
            release(a, S, ring, warp, lane, c, G);
        }
        stamp(l, 3, 2);
        __syncthreads();
#pragma unroll 1
        for (int j = tid; j < n_rt; j += NW * 32) {
            float s = 0.f;
            for (int w = 0; w < NW; ++w) s += rec(red, w, 0)[j];
            a.logits[c + (size_t)G * j] = s;
        }
        stamp(l, 3, 3);
        // ================= GU =================
        if (!(synced = gsync(a, S, ++nbar, alive))) break;
        stamp(l, 4, 0);
        if (warp == 0) {
            xtopk_n<8>(a.logits, a.E, a.K, a.gating, lane, S.idx, S.wts);  // E <= 256
            __syncwarp();
            // an id out of range (NaN logits, outside the router's contract) reads expert 0
            // rather than memory past the bank, and is reported
            if (lane < a.K && S.idx[lane] >= (unsigned)a.E) {
                S.idx[lane] = 0;
                atomicOr(a.status, STATUS_RANGE);
            }
            __syncwarp();
            if (c == 0 && lane < a.K) {
                a.route_idx[(size_t)l * a.K + lane] = S.idx[lane];
                a.route_w[(size_t)l * a.K + lane] = S.wts[lane];
            }
        }
        __syncthreads();
        stamp(l, 4, 1);
        if (lane == 0) S.R[warp].routed = l;
        __syncwarp();
        pump(a, S, ring, warp, lane, c, G);
        {
            // pairs [lo, hi): (gate, up) tiles of segment (expert m, tile-row tr)
            int rec_lo = -1, nrec = 0, cur = -1;
            float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
            const int r = lane >> 2, qd = lane & 3;
            const int lo = W.lo[R_GU], hi = W.hiR[R_GU];
            int seg = lo / a.gu_nkt, kt = lo - seg * a.gu_nkt;
            for (int it = lo; it < hi && alive;) {
                const uint8_t *st = wait_piece(a, S, ring, warp, lane, alive);
                if (!st) break;
                const int n = min(min(a.ch_gu, a.gu_nkt - kt), hi - it);
                if (seg != cur) {
                    if (cur >= 0 && qd == 0) {
                        float *p = rec(red, warp, cur - rec_lo);
                        p[r] = ag[0] + ag[1];
                        p[r + 8] = ag[2] + ag[3];
                        p[16 + r] = au[0] + au[1];
                        p[16 + r + 8] = au[2] + au[3];
                    }
                    if (rec_lo < 0) rec_lo = seg;
                    cur = seg;
                    nrec = cur - rec_lo + 1;
#pragma unroll
                    for (int e = 0; e < 4; ++e) ag[e] = au[e] = 0.f;
                }
#pragma unroll 1
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
                release(a, S, ring, warp, lane, c, G);
            }
            stamp(l, 4, 2);
            if (cur >= 0 && qd == 0) {
                float *p = rec(red, warp, cur - rec_lo);
                p[r] = ag[0] + ag[1];
                p[r + 8] = ag[2] + ag[3];
                p[16 + r] = au[0] + au[1];
                p[16 + r + 8] = au[2] + au[3];
            }
            if (lane == 0) {
                S.rec_lo[warp] = rec_lo;
                S.rec_n[warp] = nrec;
            }
            __syncthreads();
            // the CTA's segments: gate and up summed over warps in order, the activation, its
            // fragments for the down phase
            const long Sg = (long)a.K * a.gu_ntr;
            const int sg0 = (int)(Sg * c / G), sg1 = (int)(Sg * (c + 1) / G);
            uint16_t *af = reinterpret_cast<uint16_t *>(a.actfrag);
#pragma unroll 1
            for (int e = tid; e < (sg1 - sg0) * 16; e += NW * 32) {
                const int sg = sg0 + (e >> 4), rr = e & 15;
                float g = 0.f, u = 0.f;
#pragma unroll 1
                for (int w = 0; w < NW; ++w) {
                    const int k = sg - S.rec_lo[w];
                    if (S.rec_n[w] > 0 && k >= 0 && k < S.rec_n[w]) {
                        g += rec(red, w, k)[rr];
                        u += rec(red, w, k)[16 + rr];
                    }
                }
                const int m = sg / a.gu_ntr, tr = sg - m * a.gu_ntr;
                expert_frag_put(af + (size_t)m * a.I * 2, tr * 16 + rr, act_fn(a.act, g, u, a.alpha, a.limit));
            }
        }
        stamp(l, 4, 3);
        // ================= DN =================
        if (!(synced = gsync(a, S, ++nbar, alive))) break;
        stamp(l, 5, 0);
        if (lane == 0) {
            S.R[warp].acts_ok = l;
            fence_proxy_all();
        }
        __syncwarp();
        issue_deferred(a, S, ring, warp, lane, c, G, l);
        pump(a, S, ring, warp, lane, c, G);
        stamp(l, 5, 1);
        {
            int rec_lo = -1, nrec = 0, cur = -1;
            float ac[4] = {0.f, 0.f, 0.f, 0.f};
            const int r = lane >> 2, qd = lane & 3;
            const int lo = W.lo[R_DN], hi = W.hiR[R_DN];
            int seg = lo / a.dn_nkt, kt = lo - seg * a.dn_nkt;
            for (int it = lo; it < hi && alive;) {
                const uint8_t *st = wait_piece(a, S, ring, warp, lane, alive);
                if (!st) break;
                const int n = min(min(a.ch_dn, a.dn_nkt - kt), hi - it);
                if (seg != cur) {
                    if (cur >= 0 && qd == 0) {
                        float *p = rec(red, warp, cur - rec_lo);
                        p[r] = ac[0] + ac[1];
                        p[r + 8] = ac[2] + ac[3];
                    }
                    if (rec_lo < 0) rec_lo = seg;
                    cur = seg;
                    nrec = cur - rec_lo + 1;
#pragma unroll
                    for (int e = 0; e < 4; ++e) ac[e] = 0.f;
                }
                const uint8_t *acts = st + (size_t)n * a.tile_bytes;
#pragma unroll 1
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
                release(a, S, ring, warp, lane, c, G);
            }
            stamp(l, 5, 2);
            if (cur >= 0 && qd == 0) {
                float *p = rec(red, warp, cur - rec_lo);
                p[r] = ac[0] + ac[1];
                p[r + 8] = ac[2] + ac[3];
            }
            if (lane == 0) {
                S.rec_lo[warp] = rec_lo;
                S.rec_n[warp] = nrec;
            }
            __syncthreads();
            const long Sd = (long)a.K * a.dn_ntr;
            const int sd0 = (int)(Sd * c / G), sd1 = (int)(Sd * (c + 1) / G);
            cta_reduce(S, red, sd0, sd1, 16, [&](int sd, int rr, float s) {
                const int m = sd / a.dn_ntr, tr = sd - m * a.dn_ntr;
                a.down_out[((size_t)tr * 16 + rr) * a.KP + m] = s;
            });
        }
        stamp(l, 5, 3);
    }
    // ================= final norm =================
    if (synced && gsync(a, S, ++nbar, alive) && c == 0) {
        float hv[HMAX];
        residual_in(a, S, a.n_layer, hv);
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < HMAX; ++j) ss = fmaf(hv[j], hv[j], ss);
        const float scale = 1.0f / sqrtf(block_sum(S, ss, warp, lane) / (float)H + a.eps);
#pragma unroll
        for (int j = 0; j < HMAX; ++j) {
            const int i = tid + j * NW * 32;
            if (i < H) a.out[i] = (hv[j] * scale) * __ldg(a.out_norm + i);
        }
        if (tid == 0) *a.pos = pos + 1;
    }
    // no bulk copy may still be landing in this CTA's shared memory when it exits: down pieces
    // still waiting for their activations get them (from the buffer as it is), then every issued
    // piece is waited for (bounded)
    const wring &W = S.R[warp];
    if (W.n_def > 0) issue_deferred(a, S, ring, warp, lane, c, G, W.l < a.n_layer ? W.l : a.n_layer - 1);
#pragma unroll 1
    for (int k = W.n_con; k < W.n_iss; ++k) mbar_wait(&S.bars[warp][k % RS], (unsigned)((k / RS) & 1), a.status);
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
    a.q_mp = (a.q_maxc + 3) / 4 * 4;
    a.o_mp = (a.o_maxc + 3) / 4 * 4;
    a.KP = s.K <= 4 ? 4 : 8;
    if (a.q_T >= (1L << 30) || a.o_T >= (1L << 30) || a.q_maxc > 16 || a.o_maxc > 16) {
        delete p;
        return nullptr;
    }
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
    const size_t o_qp = take(4 * 16 * (size_t)a.q_ntr * a.q_mp), o_op = take(4 * 16 * (size_t)a.o_ntr * a.o_mp);
    const size_t o_att = take(4 * (size_t)Dq);
    const size_t o_ml = take(4 * 2 * (size_t)s.n_head * a.max_splits), o_acc = take(4 * (size_t)HD * s.n_head * a.max_splits);
    const size_t o_lg = take(4 * (size_t)s.E), o_af = take(4 * (size_t)s.K * s.I), o_do = take(4 * (size_t)(s.K <= 4 ? 4 : 8) * H);
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

size_t step_trace_words(step_plan *p) { return p ? (size_t)p->a.n_layer * NPH * 4 * p->G : 0; }

void step_set_trace(step_plan *p, unsigned long long *buf) {
    if (p) p->trace = buf;
}

void *step_buffer(step_plan *p, int which) {
    if (!p) return nullptr;
    return which == 0 ? static_cast<void *>(p->a.route_idx) : which == 1 ? static_cast<void *>(p->a.route_w) : nullptr;
}

}  // namespace moearc
