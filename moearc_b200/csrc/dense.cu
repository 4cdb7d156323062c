// dense.cu — packed bf16 tensor-core GEMVs for the decoder's attention projections.
// See dense.cuh for the structure; the persistent/TMA/last-arriver scheme is moe.cu's.
#include <algorithm>
#include <cmath>

#include "dense.cuh"
#include "tma.cuh"

namespace moearc {

namespace {

constexpr int WARPS = 4;
constexpr int STAGES = 2;
constexpr int PARTS = 3;  // bf16 rounding + two residuals

__global__ void k_dense_pack(uint8_t *dst, const uint16_t *src, int n_rows, int n_cols) {
    const int nkt = n_cols / 64;
    const size_t total = (size_t)(n_rows / 16) * nkt * 32;
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < total; g += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(g & 31);
        const size_t tile = g >> 5;
        const int tr = (int)(tile / nkt), tk = (int)(tile % nkt);
        const int r = lane >> 2, q = lane & 3;
        uint32_t *o = reinterpret_cast<uint32_t *>(dst + tile * DENSE_TILE + lane * 64);
        const uint16_t *rowA = src + (size_t)(tr * 16 + r) * n_cols + tk * 64;
        const uint16_t *rowB = rowA + (size_t)8 * n_cols;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int c0 = 16 * s + 2 * q, c1 = c0 + 8;
            o[4 * s + 0] = (uint32_t)rowA[c0] | ((uint32_t)rowA[c0 + 1] << 16);
            o[4 * s + 1] = (uint32_t)rowB[c0] | ((uint32_t)rowB[c0 + 1] << 16);
            o[4 * s + 2] = (uint32_t)rowA[c1] | ((uint32_t)rowA[c1 + 1] << 16);
            o[4 * s + 3] = (uint32_t)rowB[c1] | ((uint32_t)rowB[c1 + 1] << 16);
        }
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
    int n_rows, n_cols, ntr, nkt, kc, nch;
    int stage_bytes;
    int mode;
    const float *in;
    const float *norm_w;
    float eps;
    float *out;
    const float *residual;
    const int *pos;
    dense_rope rope;
    dense_kv kv;
    float *part;     // [nch][n_rows]
    unsigned *ctr;   // per unit
    int *status;
};

__device__ __forceinline__ void issue(const dense_args &a, int item, uint8_t *stage, uint64_t *bar, int lane) {
    const int ch = item % a.nch, tr = item / a.nch;
    const int k0 = ch * a.kc, kn = min(a.kc, a.nkt - k0);
    if (lane == 0) {
        fence_proxy_async();
        mbar_expect_tx(bar, (unsigned)(kn * DENSE_TILE));
        bulk_g2s(stage, a.w + ((size_t)tr * a.nkt + k0) * DENSE_TILE, (unsigned)(kn * DENSE_TILE), bar);
    }
}

__global__ void __launch_bounds__(WARPS * 32) k_dense(dense_args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int trace_row = (int)blockIdx.x + (a.mode == 0 ? 0 : 1024);
    (void)trace_row;
    TRACE(0);
    __shared__ __align__(8) uint64_t bars[WARPS][STAGES];
    __shared__ float red[WARPS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = blockIdx.x * WARPS + warp, nw = gridDim.x * WARPS;
    const int nkb = a.n_cols / 16;
    uint32_t *bsm = reinterpret_cast<uint32_t *>(smem);                   // [nkb][3][4][2]
    const size_t bsm_bytes = ((size_t)nkb * PARTS * 4 * 8 + 127) / 128 * 128;
    float *xs = reinterpret_cast<float *>(smem + bsm_bytes);              // [n_cols]
    const size_t xs_bytes = ((size_t)a.n_cols * 8 + 127) / 128 * 128;  // activation + norm weights
    uint8_t *my = smem + bsm_bytes + xs_bytes + (size_t)warp * STAGES * a.stage_bytes;
    const int n_items = a.ntr * a.nch;
    if (lane == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[warp][s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    unsigned phase[STAGES] = {0u, 0u};
    bool pending[STAGES] = {false, false};
    // The weights do not depend on the previous kernel: start streaming them before waiting.
    for (int s = 0; s < STAGES; ++s) {
        const int it = gw + s * nw;
        if (it < n_items) {
            issue(a, it, my + s * a.stage_bytes, &bars[warp][s], lane);
            pending[s] = true;
        }
    }
    pdl_trigger();
    pdl_wait();
    TRACE(1);
    // The activation (and the norm weights) into shared memory, all loads in flight at once.
    const int n4 = a.n_cols / 4;
    float ss = 0.f;
    float *ns = xs + a.n_cols;  // norm weights, when present
    {
        constexpr int U = 8;  // float4 per thread per batch; 128 threads x 8 x 4 = 4096 values
        for (int base = threadIdx.x; base < n4; base += WARPS * 32 * U) {
            float4 v[U], w[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = base + u * WARPS * 32;
                if (i < n4) {
                    v[u] = __ldcg(reinterpret_cast<const float4 *>(a.in) + i);
                    if (a.norm_w) w[u] = __ldg(reinterpret_cast<const float4 *>(a.norm_w) + i);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = base + u * WARPS * 32;
                if (i < n4) {
                    reinterpret_cast<float4 *>(xs)[i] = v[u];
                    if (a.norm_w) reinterpret_cast<float4 *>(ns)[i] = w[u];
                    ss = fmaf(v[u].x, v[u].x, fmaf(v[u].y, v[u].y, fmaf(v[u].z, v[u].z, fmaf(v[u].w, v[u].w, ss))));
                }
            }
        }
    }
    float scale = 1.f;
    if (a.norm_w) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
    }
    __syncthreads();
    if (a.norm_w) {
        float t = 0.f;
        for (int w = 0; w < WARPS; ++w) t += red[w];
        scale = 1.0f / sqrtf(t / (float)a.n_cols + a.eps);
    }
    // B fragments: (k16 block, q, register) -> the pair (x[16kb + 2q + 8reg], x[... + 1]),
    // RMSNorm applied for the Q/K/V projection, split into three bf16 parts
    for (int i = threadIdx.x; i < nkb * 4 * 2; i += WARPS * 32) {
        const int reg = i & 1, q = (i >> 1) & 3, kb = i >> 3;
        const int c = 16 * kb + 2 * q + 8 * reg;
        float v0 = xs[c], v1 = xs[c + 1];
        if (a.norm_w) {
            v0 = (v0 * scale) * ns[c];
            v1 = (v1 * scale) * ns[c + 1];
        }
        uint16_t h0 = bf(v0), h1 = bf(v1);
        float r0 = v0 - bf16_bits_to_f32(h0), r1 = v1 - bf16_bits_to_f32(h1);
        uint16_t m0 = bf(r0), m1 = bf(r1);
        r0 -= bf16_bits_to_f32(m0);
        r1 -= bf16_bits_to_f32(m1);
        uint16_t l0 = bf(r0), l1 = bf(r1);
        bsm[(((size_t)kb * PARTS + 0) * 4 + q) * 2 + reg] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        bsm[(((size_t)kb * PARTS + 1) * 4 + q) * 2 + reg] = (uint32_t)m0 | ((uint32_t)m1 << 16);
        bsm[(((size_t)kb * PARTS + 2) * 4 + q) * 2 + reg] = (uint32_t)l0 | ((uint32_t)l1 << 16);
    }
    __syncthreads();

    TRACE(2);
    const int n = lane >> 2, qd = lane & 3, r = lane >> 2;
    int stage = 0;
    int itn = 0;
    for (int it = gw; it < n_items; it += nw, ++itn) {
        uint8_t *st = my + stage * a.stage_bytes;
        const bool ok = mbar_wait(&bars[warp][stage], phase[stage], a.status);
        phase[stage] ^= 1u;
        pending[stage] = false;
        if (!ok) break;
        if (itn < 6) TRACE(3 + 4 * itn);
        const int ch = it % a.nch, tr = it / a.nch;
        const int k0 = ch * a.kc, kn = min(a.kc, a.nkt - k0);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int kt = 0; kt < kn; ++kt) {
            const uint8_t *tile = st + (size_t)kt * DENSE_TILE + lane * 64;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const uint4 av = *reinterpret_cast<const uint4 *>(tile + 16 * s);
                const int kb = (k0 + kt) * 4 + s;
                uint2 bv = make_uint2(0u, 0u);
                if (n < PARTS) bv = *reinterpret_cast<const uint2 *>(bsm + (((size_t)kb * PARTS + n) * 4 + qd) * 2);
                mma_bf16(acc, av, bv.x, bv.y);
            }
        }
        __syncwarp();
        const int nxt = it + STAGES * nw;
        if (nxt < n_items) {
            issue(a, nxt, st, &bars[warp][stage], lane);
            pending[stage] = true;
        }
        stage ^= 1;
        // columns 0,1 (lane q = 0) and 2 (lane q = 1, c0) are the three parts
        const float lo_r = __shfl_xor_sync(0xffffffffu, acc[0], 1);
        const float lo_r8 = __shfl_xor_sync(0xffffffffu, acc[2], 1);
        if (qd == 0) {
            a.part[(size_t)ch * a.n_rows + tr * 16 + r] = (acc[0] + acc[1]) + lo_r;
            a.part[(size_t)ch * a.n_rows + tr * 16 + r + 8] = (acc[2] + acc[3]) + lo_r8;
        }
        if (itn < 6) TRACE(4 + 4 * itn);
        __threadfence();
        __syncwarp();
        if (itn < 6) TRACE(5 + 4 * itn);
        const int rows_per_unit = (a.mode == 0) ? a.rope.head_dim : 16;
        const int tr_per_unit = rows_per_unit / 16;
        const int unit = tr / tr_per_unit;
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(a.ctr + unit, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev != (unsigned)(tr_per_unit * a.nch) - 1) continue;
        if (itn < 6) TRACE(6 + 4 * itn);
        __threadfence();
        if (lane == 0) a.ctr[unit] = 0;
        const int row0 = unit * rows_per_unit;
        if (a.mode == 1) {
            if (lane < 16) {
                const int row = row0 + lane;
                float s = 0.f;
                for (int c = 0; c < a.nch; ++c) s += __ldcg(a.part + (size_t)c * a.n_rows + row);
                a.out[row] = a.residual ? a.residual[row] + s : s;
            }
            continue;
        }
        // Q/K/V head complete: unit < n_q_heads is a query head, then the K heads, then V.
        const int D = a.rope.head_dim, half = D / 2;
        float v[4];
        const int per = D / 32;  // values per lane: d = lane + 32 i
        for (int i = 0; i < per; ++i) {
            const int row = row0 + lane + 32 * i;
            float s = 0.f;
            for (int c = 0; c < a.nch; ++c) s += __ldcg(a.part + (size_t)c * a.n_rows + row);
            v[i] = s;
        }
        const int hq = a.rope.n_q_heads, hk = a.rope.n_kv_heads;
        const int pos = *a.pos;
        if (unit < hq + hk) {
            // NeoX RoPE: pairs (d, d + half); this lane holds d = lane + 32 i.
            for (int i = 0; i < per / 2; ++i) {
                const int p = lane + 32 * i;  // pair index < half
                const double te = (double)pos * pow(a.rope.theta_scale, (double)p);
                double th = (double)a.rope.freq_scale * te, ms = a.rope.attn_factor;
                if (a.rope.ext_factor != 0.0f) {
                    const double y = ((double)p - a.rope.corr_lo) / fmax(0.001, (double)a.rope.corr_hi - a.rope.corr_lo);
                    const double ramp = 1.0 - fmin(1.0, fmax(0.0, y));
                    const double mix = ramp * a.rope.ext_factor;
                    th = th * (1.0 - mix) + te * mix;
                    ms *= 1.0 + 0.1 * log(1.0 / (double)a.rope.freq_scale);
                }
                double sn, cs;
                sincos(th, &sn, &cs);
                cs *= ms;
                sn *= ms;
                const double x0 = v[i], x1 = v[i + per / 2];
                v[i] = (float)(x0 * cs - x1 * sn);
                v[i + per / 2] = (float)(x0 * sn + x1 * cs);
            }
            (void)half;
        }
        if (unit < hq) {
            for (int i = 0; i < per; ++i) a.out[(size_t)unit * D + lane + 32 * i] = v[i];
        } else {
            const int kvh = (unit < hq + hk) ? unit - hq : unit - hq - hk;
            uint16_t *pool = (unit < hq + hk) ? a.kv.k_pages : a.kv.v_pages;
            const int pt = a.kv.page_tokens;
            const size_t page = a.kv.table[pos / pt], slot = pos % pt;
            uint16_t *dst = pool + ((page * pt + slot) * hk + kvh) * D;
            for (int i = 0; i < per; ++i) dst[lane + 32 * i] = bf(v[i]);
        }
    }
    for (int s = 0; s < STAGES; ++s)
        if (pending[s]) mbar_wait(&bars[warp][s], phase[s], a.status);
    TRACE(31);
}

}  // namespace

TRACE_SETTER(dense)

struct dense_gemv {
    moearc_ctx *c;
    int n_rows, n_cols, mode;
    int ntr, nkt, kc, nch, stage_bytes, grid, smem;
    float *part;
    unsigned *ctr;
    int *status;
    void *mem;
};

int dense_pack(moearc_ctx *c, void *dst, const void *src, int n_rows, int n_cols) {
    if (n_rows % 16 || n_cols % 64) return ERR_ARG;
    const size_t work = (size_t)(n_rows / 16) * (n_cols / 64) * 32;
    const unsigned g = (unsigned)std::min<size_t>((work + 255) / 256, (size_t)c->sm_count * 64);
    k_dense_pack<<<g, 256, 0, c->stream>>>(static_cast<uint8_t *>(dst), static_cast<const uint16_t *>(src), n_rows, n_cols);
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

dense_gemv *dense_create(moearc_ctx *c, int n_rows, int n_cols, int mode) {
    if (n_rows % 16 || n_cols % 64) return nullptr;
    auto *g = new dense_gemv();
    g->c = c;
    g->n_rows = n_rows;
    g->n_cols = n_cols;
    g->mode = mode;
    g->ntr = n_rows / 16;
    g->nkt = n_cols / 64;
    // chunking: balance ntr * nch items over the grid's warps
    const int bsm = ((n_cols / 16) * PARTS * 4 * 8 + 127) / 128 * 128 + (n_cols * 8 + 127) / 128 * 128;
    int best = 1;
    double best_cost = 1e30;
    for (int kc = 1; kc <= std::min(8, g->nkt); ++kc) {
        const int stage = kc * DENSE_TILE;
        const int smem = bsm + WARPS * STAGES * stage;
        const int per_sm = std::max(1, std::min(4, (228 * 1024) / (smem + 1024 + 128)));
        const long nw = (long)c->sm_count * per_sm * WARPS;
        const long items = (long)g->ntr * ((g->nkt + kc - 1) / kc);
        const double cost = (double)((items + nw - 1) / nw) * (kc + 1.0);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = kc;
        }
    }
    g->kc = best;
    g->nch = (g->nkt + best - 1) / best;
    g->stage_bytes = best * DENSE_TILE;
    g->smem = bsm + WARPS * STAGES * g->stage_bytes;
    const int per_sm = std::max(1, std::min(4, (228 * 1024) / (g->smem + 1024 + 128)));
    g->grid = c->sm_count * per_sm;
    const size_t part_b = sizeof(float) * (size_t)g->nch * n_rows;
    const size_t ctr_b = sizeof(unsigned) * (size_t)g->ntr;
    if (cudaMalloc(&g->mem, part_b + ctr_b + 256) != cudaSuccess) {
        cudaGetLastError();
        delete g;
        return nullptr;
    }
    g->part = static_cast<float *>(g->mem);
    g->ctr = reinterpret_cast<unsigned *>(static_cast<uint8_t *>(g->mem) + part_b);
    g->status = reinterpret_cast<int *>(static_cast<uint8_t *>(g->mem) + part_b + ctr_b);
    cudaMemsetAsync(g->mem, 0, part_b + ctr_b + 256, c->stream);
    // The attribute is per kernel, shared by every plan: set it to the most any plan may use
    // (227 KB less the kernel's static shared memory), not to this plan's need.
    if (g->smem > 226 * 1024 ||
        cudaFuncSetAttribute(k_dense, cudaFuncAttributeMaxDynamicSharedMemorySize, 226 * 1024) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(g->mem);
        delete g;
        return nullptr;
    }
    return g;
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
    a.kc = g->kc;
    a.nch = g->nch;
    a.stage_bytes = g->stage_bytes;
    a.mode = g->mode;
    a.in = in;
    a.norm_w = norm_w;
    a.eps = eps;
    a.out = out;
    a.residual = residual;
    a.pos = pos;
    if (rope) a.rope = *rope;
    if (kv) a.kv = *kv;
    a.part = g->part;
    a.ctr = g->ctr;
    a.status = g->status;
    return launch_pdl(k_dense, dim3(g->grid), dim3(WARPS * 32), (size_t)g->smem, g->c->stream, a) == cudaSuccess
               ? OK
               : ERR;
}

}  // namespace moearc
