// attention.cu — paged KV append and single-query decode attention
// (kernels.cpp:1782-1919; twin reference.rs:767-873).
//
// The reference runs one work-group of head_dim lanes per query head and walks every key with a
// group reduction per key. Here the key span [kv_begin, n_kv) is split across CTAs (split-K
// flash-decode): CTA (kv_head, split) serves all query heads of the GQA group, so each K/V row
// is read from HBM once per group rather than once per query head. Partial (max, sum, acc)
// triples are merged by a second kernel; the attention sink (kernels.cpp:1856-1880) joins there
// as one more logit with no value.
//
// bf16/f16 caches with group <= 8 and head_dim 64 or 128 take the tensor-core kernel:
// per warp, S = Q K^T and O += P V are m16n8k16 MMAs. The 16 MMA rows hold the group's query
// heads twice — rows 0-7 the head rounded to the cache type (hi), rows 8-15 the rounding
// residual (lo) — so S_h = S[h] + S[h+8] carries ~16 significant bits of q instead of 8, and
// the same split of P keeps the softmax weights as accurate. Both halves of a head land in the
// same lane of the accumulator fragment, so combining them costs one add.
#include <cmath>

#include "common.cuh"

using namespace moearc;

namespace {

// ---- paged KV append (kernels.cpp:1782-1799) ----------------------------------------------

__global__ void k_kv_append(void *kp, void *vp, const float *k, const float *v, size_t base,
                            size_t n, unsigned kv_type) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        if (kv_type == T_F32) {
            static_cast<float *>(kp)[base + i] = k[i];
            static_cast<float *>(vp)[base + i] = v[i];
        } else if (kv_type == T_F16) {
            static_cast<uint16_t *>(kp)[base + i] = __half_as_ushort(__float2half_rn(k[i]));
            static_cast<uint16_t *>(vp)[base + i] = __half_as_ushort(__float2half_rn(v[i]));
        } else {
            static_cast<uint16_t *>(kp)[base + i] = f32_to_bf16_bits(k[i]);
            static_cast<uint16_t *>(vp)[base + i] = f32_to_bf16_bits(v[i]);
        }
    }
}

__device__ __forceinline__ float kv_get(const void *base, size_t i, unsigned t) {
    if (t == T_F16) return f16_bits_to_f32(static_cast<const uint16_t *>(base)[i]);
    if (t == T_BF16) return bf16_bits_to_f32(static_cast<const uint16_t *>(base)[i]);
    return static_cast<const float *>(base)[i];
}

constexpr float LOG2E = 1.4426950408889634f;

// The key span of a decode step whose position lives in device memory: n_kv = pos + 1, a
// window of `window` keys (0 = full causal), split over at most max_splits CTAs in runs of a
// multiple of 64 keys. Returns false for a CTA past the last split.
__device__ __forceinline__ bool device_span(const int *dpos, int window, int max_splits, size_t &kv_begin,
                                            size_t &n_kv, size_t &kps, int &n_splits) {
    n_kv = (size_t)(*dpos) + 1;
    kv_begin = (window > 0 && n_kv > (size_t)window) ? n_kv - (size_t)window : 0;
    const size_t span = n_kv - kv_begin;
    // at least 256 keys a split: below that a second split costs more (its partials, the
    // arrival and the merge) than the keys it takes off the first
    kps = (span + max_splits - 1) / max_splits;
    kps = ((kps + 255) / 256) * 256;
    n_splits = (int)((span + kps - 1) / kps);
    return (int)blockIdx.y < n_splits;
}

// Merge the n_splits partial (max, sum, acc) triples of heads [h0, h0 + nh) into out, with
// the sink as one extra logit (kernels.cpp:1856-1880). Run by one whole CTA. The splits'
// (max, sum) pairs are staged in shared memory and turned into per-split weights first, so the
// accumulator loads (independent of one another) are issued in batches, not one round trip
// per split.
constexpr int MERGE_MAX = 8 * 64;  // heads x splits the staged weights cover
__device__ void merge_heads(float *out, const float *part_ml, const float *part_acc, const float *sinks,
                            int h0, int nh, int hd, int n_splits) {
    __shared__ float wgt[MERGE_MAX];  // [head][split] exp(m_s - M)
    __shared__ float inv_l[8];
    const bool staged = nh <= 8 && nh * n_splits <= MERGE_MAX;
    if (staged) {
        for (int i = threadIdx.x; i < nh * n_splits; i += blockDim.x)
            wgt[i] = __ldcg(part_ml + ((size_t)(h0 + i / n_splits) * n_splits + i % n_splits) * 2);
        __syncthreads();
        // one warp per head: the max, the weights and 1 / (sum of weighted l + sink)
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int h = warp; h < nh; h += blockDim.x >> 5) {
            float M = sinks ? sinks[h0 + h] : -INFINITY;
            for (int sp = lane; sp < n_splits; sp += 32) M = fmaxf(M, wgt[h * n_splits + sp]);
            M = warp_max(M);
            float L = 0.f;
            for (int sp = lane; sp < n_splits; sp += 32) {
                const float ms = wgt[h * n_splits + sp];
                const float f = (ms == -INFINITY) ? 0.f : exp2f((ms - M) * LOG2E);
                L += __ldcg(part_ml + ((size_t)(h0 + h) * n_splits + sp) * 2 + 1) * f;
                wgt[h * n_splits + sp] = f;
            }
            L = warp_sum(L);
            if (lane == 0) inv_l[h] = 1.f / (L + (sinks ? exp2f((sinks[h0 + h] - M) * LOG2E) : 0.f));
        }
        __syncthreads();
        for (int e = threadIdx.x; e < nh * hd; e += blockDim.x) {
            const int h = e / hd, d = e % hd;
            const float *pa = part_acc + (size_t)(h0 + h) * n_splits * hd + d;
            float v = 0.f;
#pragma unroll 8
            for (int sp = 0; sp < n_splits; ++sp) {
                const float w = wgt[h * n_splits + sp];
                if (w != 0.f) v += __ldcg(pa + (size_t)sp * hd) * w;  // a split with no keys adds nothing
            }
            out[(size_t)(h0 + h) * hd + d] = v * inv_l[h];
        }
        return;
    }
    for (int e = threadIdx.x; e < nh * hd; e += blockDim.x) {
        const int h = h0 + e / hd, d = e % hd;
        const float *ml = part_ml + (size_t)h * n_splits * 2;
        float M = sinks ? sinks[h] : -INFINITY;
        for (int sp = 0; sp < n_splits; ++sp) M = fmaxf(M, __ldcg(ml + 2 * sp));
        float L = sinks ? exp2f((sinks[h] - M) * LOG2E) : 0.f;
        float v = 0.f;
        for (int sp = 0; sp < n_splits; ++sp) {
            const float ms = __ldcg(ml + 2 * sp);
            if (ms == -INFINITY) continue;
            const float f = exp2f((ms - M) * LOG2E);
            L += __ldcg(ml + 2 * sp + 1) * f;
            v += __ldcg(part_acc + ((size_t)h * n_splits + sp) * hd + d) * f;
        }
        out[(size_t)h * hd + d] = v / L;
    }
}

// After a CTA wrote its partials: count it in; the last CTA of `unit` merges the unit's heads
// and resets the counter for the next call.
__device__ __forceinline__ void arrive_and_merge(unsigned *ctr, int unit, int n_splits, float *out,
                                                 const float *part_ml, const float *part_acc,
                                                 const float *sinks, int h0, int nh, int hd) {
    __shared__ unsigned last;
    fence_acq_rel_gpu();
    __syncthreads();
    if (threadIdx.x == 0) last = (atomicAdd(ctr + unit, 1u) == (unsigned)n_splits - 1);
    __syncthreads();
    if (!last) return;
    fence_acq_rel_gpu();
    merge_heads(out, part_ml, part_acc, sinks, h0, nh, hd, n_splits);
    if (threadIdx.x == 0) ctr[unit] = 0;
}

// ---- the generic split-K kernel (any cache type, group, head_dim <= 1024) ----------------
//
// CTA (query head, split), 4 warps; warp w walks keys s0+w, s0+w+4, ...; lanes hold NPL
// channels each. Online softmax per warp, merged across the warps in shared memory.
template <int NPL>
__global__ void __launch_bounds__(128)
    k_attn_generic(float *part_ml, float *part_acc, float *out, const float *q, const void *kp,
                   const void *vp, const unsigned *table, const float *sinks, int n_heads,
                   int n_kv_heads, int hd, size_t kv_begin, size_t n_kv, size_t pt, float scale,
                   unsigned kv_type, size_t kps, int n_splits, const int *dpos, int window, unsigned *ctr) {
    extern __shared__ float sm[];  // [4][2] m,l then [4][hd] acc
    const int h = blockIdx.x, split = blockIdx.y;
    pdl_trigger();
    pdl_wait();
    if (dpos && !device_span(dpos, window, gridDim.y, kv_begin, n_kv, kps, n_splits)) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int group = n_heads / n_kv_heads, kvh = h / group;
    const size_t s0 = kv_begin + (size_t)split * kps;
    const size_t s1 = min(s0 + kps, n_kv);
    float qr[NPL], acc[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
        const int d = lane + 32 * i;
        qr[i] = d < hd ? q[(size_t)h * hd + d] : 0.f;
        acc[i] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    const size_t row = (size_t)n_kv_heads * hd;
    for (size_t j = s0 + warp; j < s1; j += 4) {
        const size_t base = ((size_t)table[j / pt] * pt + j % pt) * row + (size_t)kvh * hd;
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            const int d = lane + 32 * i;
            if (d < hd) dot = fmaf(qr[i], kv_get(kp, base + d, kv_type), dot);
        }
        const float s = warp_sum(dot) * scale;
        const float mn = fmaxf(m, s);
        const float corr = exp2f((m - mn) * LOG2E);
        const float p = exp2f((s - mn) * LOG2E);
        l = l * corr + p;
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            const int d = lane + 32 * i;
            acc[i] = acc[i] * corr + (d < hd ? p * kv_get(vp, base + d, kv_type) : 0.f);
        }
        m = mn;
    }
    float *wm = sm, *wacc = sm + 8;
    if (lane == 0) {
        wm[2 * warp] = m;
        wm[2 * warp + 1] = l;
    }
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
        const int d = lane + 32 * i;
        if (d < hd) wacc[warp * hd + d] = acc[i];
    }
    __syncthreads();
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[2 * w]);
    float L = 0.f, fw[4];
    for (int w = 0; w < 4; ++w) {
        fw[w] = (wm[2 * w] == -INFINITY) ? 0.f : exp2f((wm[2 * w] - M) * LOG2E);
        L += wm[2 * w + 1] * fw[w];
    }
    if (n_splits == 1) {
        float Mf = M, Lf = L, fs = 1.f;
        if (sinks) {
            const float sk = sinks[h];
            Mf = fmaxf(M, sk);
            fs = (M == -INFINITY) ? 0.f : exp2f((M - Mf) * LOG2E);
            Lf = L * fs + exp2f((sk - Mf) * LOG2E);
        }
        for (int d = threadIdx.x; d < hd; d += 128) {
            float v = 0.f;
            for (int w = 0; w < 4; ++w) v += wacc[w * hd + d] * fw[w];
            out[(size_t)h * hd + d] = v * fs / Lf;
        }
    } else {
        if (threadIdx.x == 0) {
            part_ml[((size_t)h * n_splits + split) * 2] = M;
            part_ml[((size_t)h * n_splits + split) * 2 + 1] = L;
        }
        for (int d = threadIdx.x; d < hd; d += 128) {
            float v = 0.f;
            for (int w = 0; w < 4; ++w) v += wacc[w * hd + d] * fw[w];
            part_acc[((size_t)h * n_splits + split) * hd + d] = v;
        }
        if (ctr) arrive_and_merge(ctr, h, n_splits, out, part_ml, part_acc, sinks, h, 1, hd);
    }
}

// Merge the splits of every query head, with the sink as one extra logit.
__global__ void k_attn_combine(float *out, const float *part_ml, const float *part_acc,
                               const float *sinks, int hd, int n_splits, const int *dpos, int window,
                               int max_splits) {
    const int h = blockIdx.x;
    if (dpos) {
        size_t b = 0, n = 0, kps = 0;
        if (!device_span(dpos, window, max_splits, b, n, kps, n_splits) || n_splits == 1) return;
    }
    const float *ml = part_ml + (size_t)h * n_splits * 2;
    float M = sinks ? sinks[h] : -INFINITY;
    for (int s = 0; s < n_splits; ++s) M = fmaxf(M, ml[2 * s]);
    float L = sinks ? exp2f((sinks[h] - M) * LOG2E) : 0.f;
    for (int s = 0; s < n_splits; ++s)
        if (ml[2 * s] != -INFINITY) L += ml[2 * s + 1] * exp2f((ml[2 * s] - M) * LOG2E);
    const float inv = 1.f / L;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float v = 0.f;
        for (int s = 0; s < n_splits; ++s)
            if (ml[2 * s] != -INFINITY)
                v += part_acc[((size_t)h * n_splits + s) * hd + d] * exp2f((ml[2 * s] - M) * LOG2E);
        out[(size_t)h * hd + d] = v * inv;
    }
}

// ---- the tensor-core split-K kernel -------------------------------------------------------

template <bool BF>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (BF)
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// value -> (hi, lo) halves in the cache's 16-bit type, packed two per register.
template <bool BF>
__device__ __forceinline__ uint16_t to16(float v) {
    if constexpr (BF) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
    else return __half_as_ushort(__float2half_rn(v));
}
template <bool BF>
__device__ __forceinline__ float from16(uint16_t b) {
    if constexpr (BF) return bf16_bits_to_f32(b);
    else return f16_bits_to_f32(b);
}
template <bool BF>
__device__ __forceinline__ void split2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const uint16_t ah = to16<BF>(a), bh = to16<BF>(b);
    const uint16_t al = to16<BF>(a - from16<BF>(ah)), bl = to16<BF>(b - from16<BF>(bh));
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

constexpr int TK = 16;  // keys per warp tile

// Shared memory per warp: 2 stages x (K tile + V tile), each TK x D 16-bit values, rows
// swizzled in 16-byte chunks (chunk c of row r lives at c ^ (r & 7)) so ldmatrix's eight rows
// hit eight different bank groups.
template <int D>
constexpr int warp_smem_elems() { return 2 * 2 * TK * D; }

template <int D, bool BF>
__global__ void __launch_bounds__(128)
    k_attn_mma(float *part_ml, float *part_acc, float *out, const float *q, const uint16_t *kp,
               const uint16_t *vp, const unsigned *table, const float *sinks, int n_heads,
               int n_kv_heads, int group, size_t kv_begin, size_t n_kv, size_t pt, float scale,
               size_t kps, int n_splits, const int *dpos, int window, unsigned *ctr, size_t bs_tab) {
    extern __shared__ __align__(16) uint16_t smem[];
    constexpr int CH = D / 8;  // 16-byte chunks per row
    const int kvh = blockIdx.x, split = blockIdx.y;
    if (gridDim.z > 1) {
        // sequence blockIdx.z of a batch: its own query and output rows, page table, position,
        // split partials and merge counters; the page pool and the sinks are shared
        const size_t bz = blockIdx.z;
        q += bz * n_heads * D;
        out += bz * n_heads * D;
        table += bz * bs_tab;
        if (dpos) dpos += bz;
        part_ml += bz * n_heads * gridDim.y * 2;
        part_acc += bz * n_heads * gridDim.y * D;
        if (ctr) ctr += bz * n_kv_heads;
    }
    const int trace_row = (int)(blockIdx.y * gridDim.x + blockIdx.x);
    (void)trace_row;
    TRACE(0);
    // Before the wait only what the kernel before this one (the Q/K/V projection) does not
    // write: the sinks (weights) and the key span (the position advances only at the end of a
    // step).
    __shared__ float s_sink[8];
    if (threadIdx.x < group) s_sink[threadIdx.x] = sinks ? sinks[kvh * group + threadIdx.x] : 0.f;
    const bool live = !dpos || device_span(dpos, window, gridDim.y, kv_begin, n_kv, kps, n_splits);
    pdl_trigger();
    if (!live) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qd = lane & 3, hr = lane >> 2;  // quad position, head row
    const size_t s0 = kv_begin + (size_t)split * kps;
    const size_t s1 = min(s0 + kps, n_kv);
    uint16_t *ws = smem + warp * warp_smem_elems<D>();

    float o[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m = -INFINITY, lsum = 0.f;

    // sel 0: every row of the tile; 1: all but the newest key's; 2: the newest key's only
    const size_t row_elems = (size_t)n_kv_heads * D;
    const size_t newest = n_kv - 1;
    auto load_tile = [&](size_t t0, int stage, int sel) {
        uint16_t *kt = ws + stage * 2 * TK * D, *vt = kt + TK * D;
#pragma unroll
        for (int c = lane; c < TK * CH; c += 32) {
            const int r = c / CH, ch = c % CH;
            const size_t j = t0 + r;
            if ((sel == 1 && j == newest) || (sel == 2 && j != newest)) continue;
            const bool valid = j < s1;
            const size_t jj = valid ? j : s0;
            const size_t off = ((size_t)table[jj / pt] * pt + jj % pt) * row_elems + (size_t)kvh * D + ch * 8;
            const int dst = r * D + ((ch ^ (r & 7)) * 8);
            cp_async16(kt + dst, kp + off, valid);
            cp_async16(vt + dst, vp + off, valid);
        }
    };

    size_t t0 = s0 + (size_t)warp * TK;
    int stage = 0;
    // With the decoder's device position the Q/K/V kernel before this one wrote only this step's
    // key (n_kv - 1); the older keys' rows (pages and ring slots the step does not touch) are
    // copied before the wait, the newest after it.
    const bool pre = dpos != nullptr;
    if (pre) {
        if (t0 < s1) load_tile(t0, 0, 1);
        cp_async_commit();
    }
    pdl_wait();
    TRACE(1);
    TRACE(2);
    if (t0 < s1) load_tile(t0, 0, pre ? 2 : 0);
    cp_async_commit();
    // q after the first tile's copies are in flight: the two reads overlap
    // Q as the A operand: rows 0-7 hi, rows 8-15 lo; k = channel.
    uint32_t qa[D / 16][4];
    {
        const bool live = hr < group;
        const float *qh = q + (size_t)(kvh * group + (live ? hr : 0)) * D;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
            const int c0 = 16 * kk + 2 * qd, c1 = c0 + 8;
            const float x0 = live ? qh[c0] : 0.f, x1 = live ? qh[c0 + 1] : 0.f;
            const float y0 = live ? qh[c1] : 0.f, y1 = live ? qh[c1 + 1] : 0.f;
            split2<BF>(x0, x1, qa[kk][0], qa[kk][1]);
            split2<BF>(y0, y1, qa[kk][2], qa[kk][3]);
        }
    }

    for (; t0 < s1; t0 += 4 * TK) {
        const size_t tn = t0 + 4 * TK;
        if (tn < s1) load_tile(tn, stage ^ 1, 0);
        cp_async_commit();
        cp_async_wait<1>();
        __syncwarp();
        const uint16_t *kt = ws + stage * 2 * TK * D, *vt = kt + TK * D;

        // S = Q K^T for keys t0..t0+15 (two n8 tiles).
        float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
            const int mi = lane >> 3, r = ((mi >> 1) << 3) | (lane & 7);
            const int ch = 2 * kk + (mi & 1);
            uint32_t b[4];
            ldsm_x4(b, kt + r * D + ((ch ^ (r & 7)) * 8));
            mma16816<BF>(sacc[0], qa[kk], b[0], b[1]);
            mma16816<BF>(sacc[1], qa[kk], b[2], b[3]);
        }
        // Scores of head hr for keys 2qd, 2qd+1 (tile 0) and 8+2qd, 8+2qd+1 (tile 1).
        float s[4];
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const size_t j = t0 + 8 * n + 2 * qd + e;
                const float v = (sacc[n][e] + sacc[n][e + 2]) * scale;
                s[2 * n + e] = j < s1 ? v : -INFINITY;
            }
        float mt = fmaxf(fmaxf(s[0], s[1]), fmaxf(s[2], s[3]));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
        const float mn = fmaxf(m, mt);
        const float corr = (mn == -INFINITY) ? 1.f : exp2f((m - mn) * LOG2E);
        float p[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) p[e] = (s[e] == -INFINITY) ? 0.f : exp2f((s[e] - mn) * LOG2E);
        lsum = lsum * corr + (p[0] + p[1]) + (p[2] + p[3]);
        m = mn;
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
            o[i][0] *= corr;
            o[i][1] *= corr;
            o[i][2] *= corr;
            o[i][3] *= corr;
        }
        // P as the A operand (rows 0-7 hi, 8-15 lo; k = key).
        uint32_t pa[4];
        split2<BF>(p[0], p[1], pa[0], pa[1]);
        split2<BF>(p[2], p[3], pa[2], pa[3]);
        // O += P V.
#pragma unroll
        for (int dn = 0; dn < D / 16; ++dn) {
            const int mi = lane >> 3, r = ((mi & 1) << 3) | (lane & 7);
            const int ch = 2 * dn + (mi >> 1);
            uint32_t b[4];
            ldsm_x4_t(b, vt + r * D + ((ch ^ (r & 7)) * 8));
            mma16816<BF>(o[2 * dn], pa, b[0], b[1]);
            mma16816<BF>(o[2 * dn + 1], pa, b[2], b[3]);
        }
        __syncwarp();
        stage ^= 1;
    }
    cp_async_wait<0>();
    TRACE(3);
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);

    // Merge the four warps through shared memory (the tile buffers are free now).
    __syncthreads();
    float *fm = reinterpret_cast<float *>(smem);  // [4][8] m, [4][8] l, [4][8][D] acc
    float *fl = fm + 32, *fo = fm + 64;
    if (qd == 0) {
        fm[warp * 8 + hr] = m;
        fl[warp * 8 + hr] = lsum;
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
        const int d = 8 * i + 2 * qd;
        fo[(warp * 8 + hr) * D + d] = o[i][0] + o[i][2];
        fo[(warp * 8 + hr) * D + d + 1] = o[i][1] + o[i][3];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < group * D; e += 128) {
        const int h = e / D, d = e % D;
        float M = -INFINITY;
        for (int w = 0; w < 4; ++w) M = fmaxf(M, fm[w * 8 + h]);
        float L = 0.f, v = 0.f;
        for (int w = 0; w < 4; ++w) {
            const float mw = fm[w * 8 + h];
            if (mw == -INFINITY) continue;
            const float f = exp2f((mw - M) * LOG2E);
            L += fl[w * 8 + h] * f;
            v += fo[(w * 8 + h) * D + d] * f;
        }
        const int hq = kvh * group + h;
        if (n_splits == 1) {
            float fs = 1.f;
            if (sinks) {
                const float sk = s_sink[h];
                const float Mf = fmaxf(M, sk);
                fs = (M == -INFINITY) ? 0.f : exp2f((M - Mf) * LOG2E);
                L = L * fs + exp2f((sk - Mf) * LOG2E);
            }
            out[(size_t)hq * D + d] = v * fs / L;
        } else {
            if (d == 0) {
                part_ml[((size_t)hq * n_splits + split) * 2] = M;
                part_ml[((size_t)hq * n_splits + split) * 2 + 1] = L;
            }
            part_acc[((size_t)hq * n_splits + split) * D + d] = v;
        }
    }
    TRACE(4);
    if (n_splits > 1 && ctr) arrive_and_merge(ctr, kvh, n_splits, out, part_ml, part_acc, sinks, kvh * group, group, D);
    TRACE(5);
}

// The tensor-core kernel's shared-memory limit (64 KiB at head_dim 128, above the default 48),
// set once on each device that launches it.
template <int D, bool BF>
cudaError_t set_mma_smem() {
    static std::atomic<bool> done[MOEARC_MAX_DEVICES];
    return once_per_device(done, [] { return set_smem(k_attn_mma<D, BF>, 4 * warp_smem_elems<D>() * 2); });
}

}  // namespace

TRACE_SETTER(attn)

namespace moearc {

// Shared by the ABI entry point and the decoder: chooses the kernel and the split count, and
// uses `scratch` (at least attn_scratch_bytes) for the partials.
size_t attn_scratch_bytes(size_t n_heads, size_t head_dim, int n_splits) {
    return (size_t)n_heads * n_splits * (head_dim + 2) * sizeof(float);
}

int attn_splits(moearc_ctx *c, size_t n_kv_heads, size_t n_heads, size_t span, bool mma, size_t *kps_out) {
    const size_t units = mma ? n_kv_heads : n_heads;
    const size_t want = (size_t)(2 * c->sm_count + units - 1) / units;
    size_t kps = (span + want - 1) / want;
    kps = ((kps + 63) / 64) * 64;
    if (kps < 64) kps = 64;
    *kps_out = kps;
    return (int)((span + kps - 1) / kps);
}

bool attn_mma_ok(size_t n_heads, size_t n_kv_heads, size_t head_dim, unsigned kv_type,
                 const void *kp, const void *vp) {
    if (kv_type != T_BF16 && kv_type != T_F16) return false;
    if (n_heads / n_kv_heads > 8) return false;
    if (head_dim != 64 && head_dim != 128) return false;
    return ((reinterpret_cast<uintptr_t>(kp) | reinterpret_cast<uintptr_t>(vp)) & 15) == 0;
}

int attn_launch(moearc_ctx *c, float *out, const float *q, const void *kp, const void *vp,
                const unsigned *table, const float *sinks, size_t n_heads, size_t n_kv_heads,
                size_t hd, size_t kv_begin, size_t n_kv, size_t pt, float scale, unsigned kv_type,
                float *scratch, size_t scratch_bytes, const int *dpos, int window, int max_splits,
                unsigned *ctr) {
    const bool mma = attn_mma_ok(n_heads, n_kv_heads, hd, kv_type, kp, vp);
    cudaError_t err = cudaSuccess;
    size_t kps = 0;
    // With the position on the device the split count is decided there; the grid is sized
    // for the most splits the caller allows.
    const int n_splits = dpos ? max_splits : attn_splits(c, n_kv_heads, n_heads, n_kv - kv_begin, mma, &kps);
    float *ml = nullptr, *acc = nullptr;
    if (n_splits > 1) {
        if (!scratch || scratch_bytes < attn_scratch_bytes(n_heads, hd, n_splits)) return ERR;
        ml = scratch;
        acc = scratch + n_heads * n_splits * 2;
    }
    const int group = (int)(n_heads / n_kv_heads);
    if (mma) {
        const dim3 grid((unsigned)n_kv_heads, (unsigned)n_splits);
        const auto *k16 = static_cast<const uint16_t *>(kp);
        const auto *v16 = static_cast<const uint16_t *>(vp);
        if (hd == 64) {
            constexpr size_t sm = 4 * warp_smem_elems<64>() * 2;
            if (kv_type == T_BF16) {
                err = set_mma_smem<64, true>();
                if (err == cudaSuccess) err = launch_pdl(k_attn_mma<64, true>, grid, dim3(128), sm, c->stream, ml, acc, out, q, k16, v16, table, sinks, (int)n_heads, (int)n_kv_heads, group, kv_begin, n_kv, pt, scale, kps, n_splits, dpos, window, ctr, (size_t)0);
            } else {
                err = set_mma_smem<64, false>();
                if (err == cudaSuccess) err = launch_pdl(k_attn_mma<64, false>, grid, dim3(128), sm, c->stream, ml, acc, out, q, k16, v16, table, sinks, (int)n_heads, (int)n_kv_heads, group, kv_begin, n_kv, pt, scale, kps, n_splits, dpos, window, ctr, (size_t)0);
            }
        } else {
            constexpr size_t sm = 4 * warp_smem_elems<128>() * 2;
            if (kv_type == T_BF16) {
                err = set_mma_smem<128, true>();
                if (err == cudaSuccess) err = launch_pdl(k_attn_mma<128, true>, grid, dim3(128), sm, c->stream, ml, acc, out, q, k16, v16, table, sinks, (int)n_heads, (int)n_kv_heads, group, kv_begin, n_kv, pt, scale, kps, n_splits, dpos, window, ctr, (size_t)0);
            } else {
                err = set_mma_smem<128, false>();
                if (err == cudaSuccess) err = launch_pdl(k_attn_mma<128, false>, grid, dim3(128), sm, c->stream, ml, acc, out, q, k16, v16, table, sinks, (int)n_heads, (int)n_kv_heads, group, kv_begin, n_kv, pt, scale, kps, n_splits, dpos, window, ctr, (size_t)0);
            }
        }
    } else {
        const dim3 grid((unsigned)n_heads, (unsigned)n_splits);
        const size_t sm = (8 + 4 * hd) * sizeof(float);
        const int npl = (int)((hd + 31) / 32);
#define GEN(N) err = launch_pdl(k_attn_generic<N>, grid, dim3(128), sm, c->stream, ml, acc, out, q, kp, vp, table, sinks, (int)n_heads, (int)n_kv_heads, (int)hd, kv_begin, n_kv, pt, scale, kv_type, kps, n_splits, dpos, window, ctr)
        if (npl <= 2) GEN(2);
        else if (npl <= 4) GEN(4);
        else if (npl <= 8) GEN(8);
        else {
            cudaFuncSetAttribute(k_attn_generic<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
            GEN(32);
        }
#undef GEN
    }
    if (err != cudaSuccess) {
        cudaGetLastError();  // the failed launch's error, not left for an unrelated later check
        return ERR;
    }
    // with counters the last split of each head group merges in the kernel; without, a
    // second kernel merges
    if (n_splits > 1 && !ctr) {
        k_attn_combine<<<(unsigned)n_heads, 128, 0, c->stream>>>(out, ml, acc, sinks, (int)hd, n_splits, dpos,
                                                                window, n_splits);
        if (cudaPeekAtLastError() != cudaSuccess) {
            cudaGetLastError();
            return ERR;
        }
    }
    return OK;
}

// n_batch sequences at once (bf16 KV, head_dim 64 or 128, tensor-core kernel): sequence b reads
// q + b n_heads hd, writes out + b n_heads hd, pages through table + b table_stride, attends over
// [window-limited start, dpos[b]]; scratch holds n_batch x n_heads x max_splits x (hd + 2) floats,
// ctr n_batch x n_kv_heads zeroed counters (the last split of a head group merges and re-zeroes).
int attn_launch_batched(moearc_ctx *c, float *out, const float *q, const void *kp, const void *vp,
                        const unsigned *table, size_t table_stride, const float *sinks, size_t n_heads,
                        size_t n_kv_heads, size_t hd, size_t n_ctx, size_t pt, float scale, float *scratch,
                        size_t scratch_bytes, const int *dpos, int window, int max_splits, unsigned *ctr,
                        int n_batch) {
    if (!attn_mma_ok(n_heads, n_kv_heads, hd, T_BF16, kp, vp) || !dpos || !ctr || n_batch < 1 || max_splits < 1)
        return ERR_ARG;
    if (scratch_bytes < (size_t)n_batch * attn_scratch_bytes(n_heads, hd, max_splits)) return ERR_ARG;
    const int group = (int)(n_heads / n_kv_heads);
    float *ml = scratch, *acc = scratch + (size_t)n_batch * n_heads * max_splits * 2;
    const dim3 grid((unsigned)n_kv_heads, (unsigned)max_splits, (unsigned)n_batch);
    const auto *k16 = static_cast<const uint16_t *>(kp);
    const auto *v16 = static_cast<const uint16_t *>(vp);
    cudaError_t err;
    if (hd == 64) {
        constexpr size_t sm = 4 * warp_smem_elems<64>() * 2;
        err = set_mma_smem<64, true>();
        if (err == cudaSuccess) err = launch_pdl(k_attn_mma<64, true>, grid, dim3(128), sm, c->stream, ml, acc, out, q, k16, v16, table, sinks,
                         (int)n_heads, (int)n_kv_heads, group, (size_t)0, n_ctx, pt, scale, (size_t)0, max_splits, dpos,
                         window, ctr, table_stride);
    } else {
        constexpr size_t sm = 4 * warp_smem_elems<128>() * 2;
        err = set_mma_smem<128, true>();
        if (err == cudaSuccess) err = launch_pdl(k_attn_mma<128, true>, grid, dim3(128), sm, c->stream, ml, acc, out, q, k16, v16, table, sinks,
                         (int)n_heads, (int)n_kv_heads, group, (size_t)0, n_ctx, pt, scale, (size_t)0, max_splits, dpos,
                         window, ctr, table_stride);
    }
    return err == cudaSuccess ? OK : ERR;
}

}  // namespace moearc

extern "C" {

int moearc_kv_append(moearc_ctx *c, void *k_pages, void *v_pages, const float *k,
                     const float *v, unsigned int page_id, unsigned int slot,
                     unsigned long n_kv_heads, unsigned long head_dim, unsigned long page_tokens,
                     unsigned int kv_type) {
    if (!c || !k_pages || !v_pages || !k || !v) return ERR;
    if (kv_type != T_F32 && kv_type != T_F16 && kv_type != T_BF16) return ERR_ARG;
    if (page_tokens == 0 || slot >= page_tokens) return ERR_ARG;
    if (n_kv_heads == 0 || head_dim == 0) return ERR_ARG;
    const size_t n = (size_t)n_kv_heads * head_dim;
    const size_t base = ((size_t)page_id * page_tokens + slot) * n;
    launch_scope ls(c, "kv_append", n_kv_heads, (unsigned)head_dim);
    k_kv_append<<<cdiv(n, 256), 256, 0, c->stream>>>(k_pages, v_pages, k, v, base, n, kv_type);
    return ls.finish();
}

int moearc_attn_decode(moearc_ctx *c, float *out, const float *q, const void *k_pages,
                       const void *v_pages, const unsigned int *block_table, const float *sinks,
                       unsigned long n_heads, unsigned long n_kv_heads, unsigned long head_dim,
                       unsigned long kv_begin, unsigned long n_kv, unsigned long page_tokens,
                       float scale, unsigned int kv_type) {
    if (!c || !out || !q || !k_pages || !v_pages || !block_table) return ERR;
    if (kv_type != T_F32 && kv_type != T_F16 && kv_type != T_BF16) return ERR_ARG;
    if (n_heads == 0 || n_kv_heads == 0 || head_dim == 0 || n_kv == 0 || page_tokens == 0) return ERR_ARG;
    if (n_heads % n_kv_heads != 0) return ERR_ARG;
    if (kv_begin >= n_kv) return ERR_ARG;
    if (head_dim > 1024) return ERR_ARG;
    const bool mma = attn_mma_ok(n_heads, n_kv_heads, head_dim, kv_type, k_pages, v_pages);
    size_t kps = 0;
    const int n_splits = attn_splits(c, n_kv_heads, n_heads, n_kv - kv_begin, mma, &kps);
    float *scratch = nullptr;
    size_t sb = 0;
    if (n_splits > 1) {
        sb = attn_scratch_bytes(n_heads, head_dim, n_splits);
        scratch = static_cast<float *>(ctx_scratch(c, sb));
        if (!scratch) return ERR;
    }
    launch_scope ls(c, "attn_decode", n_heads, (unsigned)head_dim);
    const int rc = attn_launch(c, out, q, k_pages, v_pages, block_table, sinks, n_heads, n_kv_heads,
                               head_dim, kv_begin, n_kv, page_tokens, scale, kv_type, scratch, sb,
                               nullptr, 0, 0, nullptr);
    const int rc2 = ls.finish();
    return rc ? rc : rc2;
}

}  // extern "C"
