// batch.cu — batched decode: B independent sequences each decode one token per step through the
// same routed-MoE decoder (configs[4] of the benchmark description: 64 streams of a
// Qwen3-MoE-shaped model at depth 4096). Per block, for all B tokens at once:
//
//   xb = bf16(rmsnorm(h) * attn_norm)                              k_bd_norm
//   qkv = Wqkv xb                                                  tcgen05 GEMM (bf16, f32 out)
//   q, k = rope(q, k) at each stream's position; k, v -> its pages k_bd_rope_kv
//   att = attention of each stream over its own pages              k_attn_mma, one launch
//   h += Wo bf16(att)                                              k_bd_to_bf16, GEMM, k_bd_add
//   h = h + MoE(bf16(rmsnorm(h) * ffn_norm))                       the prefill MoE block (experts
//                                                                  at 4 bits, or the bf16 expansion)
//   out = rmsnorm(h) * output_norm; positions advance              k_bd_final
//
// The per-token semantics are the single-stream decoder's (decoder.cu; moe.rs:1862-2443) with
// bf16 activations into the projections and the experts (the reference's bf16-activation mode).
// Weights come from the same seeds and kinds as moearc_x_decoder's, so a batch decoder and a
// single-stream decoder of the same configuration hold the same values. The whole step is
// captured once as a CUDA graph.
#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "common.cuh"

namespace moearc {
bool tc_make_map_bf16(CUtensorMap *map, const void *base, long rows, int cols);
int tc_dense_gemm(moearc_ctx *c, const CUtensorMap &w, int M, int K, const CUtensorMap &x, const int *seg_off,
                  const int *seg_toff, float *out, int *status, int ksplit, size_t split_stride);
size_t attn_scratch_bytes(size_t n_heads, size_t head_dim, int n_splits);
int attn_launch_batched(moearc_ctx *c, float *out, const float *q, const void *kp, const void *vp,
                        const unsigned *table, size_t table_stride, const float *sinks, size_t n_heads,
                        size_t n_kv_heads, size_t hd, size_t n_ctx, size_t pt, float scale, float *scratch,
                        size_t scratch_bytes, const int *dpos, int window, int max_splits, unsigned *ctr,
                        int n_batch);
int prefill_forward_x32(moearc_x_prefill *p, const uint16_t *x, const float *x32, unsigned n_tokens,
                        const float *router_w, const float *router_b, const float *residual, float *out);
int prefill_route_x32(moearc_x_prefill *p, const uint16_t *x, const float *x32, unsigned n_tokens,
                      const float *router_w, const float *router_b);
int prefill_experts_dev(moearc_x_prefill *p, const uint16_t *rows, long n_rows, const int *off, const int *toff,
                        const int *seg_w, int n_seg, uint16_t *act, float *y);
int ep_all_gather(void *comm, const void *send, void *recv, size_t bytes, cudaStream_t s);
int ep_exchange(void *comm, int world, const void *send, size_t send_stride, void *recv, size_t recv_stride,
                size_t bytes, cudaStream_t s);
}  // namespace moearc

using namespace moearc;

namespace {

constexpr int BD_PAGE = 32;  // tokens per KV page (moe.rs:153)

__device__ __forceinline__ uint16_t bf16_rn(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }

// xb[b] = bf16(rmsnorm(h[b]) * w) (and x32[b] the f32 values, if given): one CTA per stream.
__global__ void __launch_bounds__(256) k_bd_norm(const float *h, const float *w, float eps, int H, uint16_t *xb,
                                                 float *x32) {
    __shared__ float red[8];
    const float *hb = h + (size_t)blockIdx.x * H;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ss = fmaf(hb[i], hb[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    const float s = 1.0f / sqrtf(t / (float)H + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float v = (hb[i] * s) * w[i];
        xb[(size_t)blockIdx.x * H + i] = bf16_rn(v);
        if (x32) x32[(size_t)blockIdx.x * H + i] = v;
    }
}

// NeoX RoPE at each stream's position on its q heads (-> q) and k heads, and k, v appended to the
// stream's pages (bf16). Block (head, stream), D / 2 threads; the angle of pair p is pos * freq[p]
// (YaRN folded into freq on the host), reduced by 2 pi in double before the sine and cosine.
// With QK-norm weights (q_norm, k_norm [D]; moe.rs:1961-1985) each q and k head is first
// RMS-normalised over its D values and scaled by them.
__global__ void k_bd_rope_kv(const float *qkv, int ksplit, size_t split_stride, int nq, int nkv, int D,
                             const double *freq, double mscale, const int *pos, const unsigned *tables,
                             int table_stride, float *q, uint16_t *kpool, uint16_t *vpool, const float *q_norm,
                             const float *k_norm, float eps) {
    __shared__ float red[32];
    const int head = blockIdx.x, b = blockIdx.y, p = threadIdx.x, half = D / 2;
    const int n_qkv = (nq + 2 * nkv) * D;
    const float *row = qkv + (size_t)b * n_qkv + (size_t)head * D;
    const int ps = pos[b];
    const unsigned page = tables[(size_t)b * table_stride + ps / BD_PAGE];
    const size_t slot = (size_t)page * BD_PAGE + ps % BD_PAGE;
    // the projection's K runs, added in order
    float a0 = row[p], a1 = row[p + half];
    for (int j = 1; j < ksplit; ++j) {
        a0 += row[j * split_stride + p];
        a1 += row[j * split_stride + p + half];
    }
    if (head < nq + nkv && q_norm) {
        float ss = warp_sum(fmaf(a0, a0, a1 * a1));
        if ((p & 31) == 0) red[p >> 5] = ss;
        __syncthreads();
        ss = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) ss += red[w];
        const float sc = 1.0f / sqrtf(ss / (float)D + eps);
        const float *w = head < nq ? q_norm : k_norm;
        a0 = (a0 * sc) * w[p];
        a1 = (a1 * sc) * w[p + half];
    }
    if (head < nq + nkv) {
        const double th = (double)ps * freq[p];
        const double k = rint(th * 0.15915494309189535);
        double r = fma(-k, 6.283185307179586, th);
        r = fma(-k, 2.4492935982947064e-16, r);
        double sn, cs;
        sincos(r, &sn, &cs);
        cs *= mscale;
        sn *= mscale;
        const double x0 = a0, x1 = a1;
        const float y0 = (float)(x0 * cs - x1 * sn), y1 = (float)(x0 * sn + x1 * cs);
        if (head < nq) {
            q[((size_t)b * nq + head) * D + p] = y0;
            q[((size_t)b * nq + head) * D + p + half] = y1;
        } else {
            uint16_t *dst = kpool + (slot * nkv + (head - nq)) * D;
            dst[p] = bf16_rn(y0);
            dst[p + half] = bf16_rn(y1);
        }
    } else {
        uint16_t *dst = vpool + (slot * nkv + (head - nq - nkv)) * D;
        dst[p] = bf16_rn(a0);
        dst[p + half] = bf16_rn(a1);
    }
}

__global__ void k_bd_to_bf16(const float *x, uint16_t *y, long n) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) y[i] = bf16_rn(x[i]);
}

// h += the O projection, its ksplit K runs (n apart) added in order first
__global__ void k_bd_add(float *h, const float *o, int ksplit, long n) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        float v = o[i];
        for (int j = 1; j < ksplit; ++j) v += o[j * n + i];
        h[i] += v;
    }
}

// out[b] = rmsnorm(h[b]) * w; stream b's position advances.
__global__ void __launch_bounds__(256) k_bd_final(const float *h, const float *w, float eps, int H, float *out, int *pos) {
    __shared__ float red[8];
    const float *hb = h + (size_t)blockIdx.x * H;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ss = fmaf(hb[i], hb[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    const float s = 1.0f / sqrtf(t / (float)H + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) out[(size_t)blockIdx.x * H + i] = (hb[i] * s) * w[i];
    __syncthreads();
    if (threadIdx.x == 0) pos[blockIdx.x] += 1;
}

// ---- expert parallelism (moearc_x_batch_decoder_create_ep) ----------------------------------
//
// Every rank routes its own streams' tokens; its P = n_batch k rows (in expert order, f16) and
// their E + 1 row offsets form one block of R rows (P rows, then the offsets in the tail rows),
// all-gathered so that each rank holds every rank's block. The owner of experts lo .. lo + nl - 1
// gathers its experts' rows of every block into one segment per expert (so an expert's weights
// stream once, whatever the number of sources), runs them, puts the result rows back in source
// order and returns block s's rows to rank s in one grouped exchange; each rank then combines its
// tokens' k rows in router order, reading row i of its expert order from the block of the
// expert's owner. Fixed sizes throughout: nothing is read back to the host, so the whole step
// stays one captured graph.

// The plan of this rank's experts over the gathered blocks (one CTA): per local expert j its rows
// from every source, contiguous in source order (segment j: rows off[j] .. off[j + 1], 32-row
// tile offsets toff, weight slot j), and map[s P + i] = the segment row of source s's row i, or
// -1 for rows of other owners' experts.
__global__ void __launch_bounds__(256) k_ep_plan(const uint16_t *rows, int W, int R, int P, int H, int lo, int nl,
                                                 int *off, int *toff, int *seg_w, int *map) {
    extern __shared__ int sh[];  // cnt [W][nl], then base [W][nl]
    int *cnt = sh, *base = sh + W * nl;
    auto offs = [&](int s) { return reinterpret_cast<const int *>(rows + ((size_t)s * R + P) * H); };
    for (int q = threadIdx.x; q < W * nl; q += blockDim.x) {
        const int s = q / nl, j = q - s * nl;
        const int *o = offs(s);
        cnt[q] = o[lo + j + 1] - o[lo + j];
    }
    for (int q = threadIdx.x; q < W * P; q += blockDim.x) map[q] = -1;
    __syncthreads();
    if (threadIdx.x == 0) {
        int r = 0, t = 0;
        for (int j = 0; j < nl; ++j) {
            off[j] = r;
            toff[j] = t;
            seg_w[j] = j;
            const int r0 = r;
            for (int s = 0; s < W; ++s) {
                base[s * nl + j] = r;
                r += cnt[s * nl + j];
            }
            t += (r - r0 + 31) / 32;
        }
        off[nl] = r;
        toff[nl] = t;
    }
    __syncthreads();
    for (int q = threadIdx.x; q < W * nl; q += blockDim.x) {
        const int s = q / nl, j = q - s * nl;
        const int i0 = offs(s)[lo + j];
        for (int i = 0; i < cnt[q]; ++i) map[s * P + i0 + i] = base[q] + i;
    }
}

// rows_e[map[r]] = the gathered row r (source r / P, row r % P) for this rank's rows.
__global__ void __launch_bounds__(128) k_ep_rows(const uint16_t *rows, int R, int P, int H, const int *map,
                                                 uint16_t *rows_e) {
    const int r = blockIdx.x, dst = map[r];
    if (dst < 0) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(rows + ((size_t)(r / P) * R + r % P) * H);
    uint4 *d = reinterpret_cast<uint4 *>(rows_e + (size_t)dst * H);
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) d[c] = src[c];
}

// y_src[r] = y_e[map[r]]: the result rows back in source order for the return exchange.
__global__ void __launch_bounds__(256) k_ep_back(const float *y_e, int H, const int *map, float *y_src) {
    const int r = blockIdx.x, dst = map[r];
    if (dst < 0) return;
    const float4 *src = reinterpret_cast<const float4 *>(y_e + (size_t)dst * H);
    float4 *d = reinterpret_cast<float4 *>(y_src + (size_t)r * H);
    for (int c = threadIdx.x; c < H / 4; c += blockDim.x) d[c] = src[c];
}

// h[t] += sum over m of w[t, m] y(t, m) in router order, y(t, m) the row perm[t k + m] of the
// block returned by the owner of expert idx[t k + m] (as k_pf_combine, with the rows gathered
// from the owners' blocks).
__global__ void __launch_bounds__(256) k_ep_combine(const float *yb, int P, int nl, const unsigned *idx,
                                                    const int *perm, const float *wts, float *h, int T, int K, int H) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)T * H) return;
    const int t = (int)(i / H), c = (int)(i - (long)t * H);
    float acc = 0.f;
    for (int m = 0; m < K; ++m) {
        const int r = (int)(idx[t * K + m] / (unsigned)nl);
        acc = fmaf(wts[t * K + m], yb[((size_t)r * P + perm[t * K + m]) * H + c], acc);
    }
    h[i] = h[i] + acc;
}

__global__ void k_bd_set_pos(int *pos, int v, int n) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) pos[i] = v;
}

}  // namespace

struct moearc_x_batch_decoder {
    moearc_ctx *c;
    moearc_x_decoder_cfg cfg;
    int B, Dq, Dkv, n_qkv, pages, max_splits;
    int ks_qkv = 1, ks_o = 1;  // K runs of the Q/K/V and O projections (one row block per SM or so)
    struct layer {
        float *attn_norm, *ffn_norm, *router;
        float *q_norm, *k_norm;  // QK-norm weights [head_dim] or null
        uint16_t *wqkv, *wo;
        CUtensorMap map_qkv, map_o;
        uint16_t *k_pages, *v_pages;
        moearc_x_prefill *moe;
    };
    std::vector<layer> L;
    std::vector<void *> allocs;
    float *x32 = nullptr;
    float *h = nullptr, *qkv = nullptr, *q = nullptr, *att = nullptr, *o = nullptr, *in = nullptr, *out = nullptr;
    float *output_norm = nullptr, *attn_scratch = nullptr;
    size_t attn_scratch_b = 0;
    uint16_t *xb = nullptr, *attb = nullptr;
    CUtensorMap map_xb, map_attb;
    unsigned *tables = nullptr, *attn_ctr = nullptr;
    int *dpos = nullptr, *seg = nullptr, *status = nullptr;
    double *rope_freq = nullptr;
    double rope_mscale = 1.0;
    int pos = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    // expert parallelism: world ranks over comm (an ncclComm_t), this rank's nl experts
    void *comm = nullptr;
    int rank = 0, world = 1, nl = 0, P = 0, R = 0;  // rows per rank (n_batch k); rows per gathered block
    uint16_t *ep_send = nullptr, *ep_rows = nullptr, *ep_rows_e = nullptr, *ep_act = nullptr;
    float *ep_y = nullptr, *ep_ysrc = nullptr, *ep_back = nullptr;
    int *ep_off = nullptr, *ep_toff = nullptr, *ep_w = nullptr, *ep_map = nullptr;

    void *alloc(size_t bytes) {
        void *p = nullptr;
        if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        allocs.push_back(p);
        return p;
    }
};

namespace {

int enqueue(moearc_x_batch_decoder *d) {
    moearc_ctx *c = d->c;
    cudaStream_t st = c->stream;
    const auto &g = d->cfg;
    const int B = d->B, H = (int)g.n_embd, D = (int)g.head_dim;
    if (cudaMemcpyAsync(d->h, d->in, sizeof(float) * B * H, cudaMemcpyDeviceToDevice, st) != cudaSuccess) return ERR;
    const float scale = 1.0f / std::sqrt((float)D);
    const long nh = (long)B * H;
    for (unsigned l = 0; l < g.n_layer; ++l) {
        auto &b = d->L[l];
        k_bd_norm<<<B, 256, 0, st>>>(d->h, b.attn_norm, g.rms_eps, H, d->xb, nullptr);
        const size_t qkv_stride = (size_t)B * d->n_qkv;
        int rc = tc_dense_gemm(c, b.map_qkv, d->n_qkv, H, d->map_xb, d->seg, d->seg + 2, d->qkv, d->status,
                               d->ks_qkv, qkv_stride);
        if (rc) return rc;
        k_bd_rope_kv<<<dim3((unsigned)(g.n_head + 2 * g.n_head_kv), (unsigned)B), (unsigned)(D / 2), 0, st>>>(
            d->qkv, d->ks_qkv, qkv_stride, (int)g.n_head, (int)g.n_head_kv, D, d->rope_freq, d->rope_mscale, d->dpos,
            d->tables, d->pages, d->q, b.k_pages, b.v_pages, b.q_norm, b.k_norm, g.rms_eps);
        rc = attn_launch_batched(c, d->att, d->q, b.k_pages, b.v_pages, d->tables, (size_t)d->pages, nullptr,
                                 g.n_head, g.n_head_kv, D, g.n_ctx, BD_PAGE, scale, d->attn_scratch,
                                 d->attn_scratch_b, d->dpos, 0, d->max_splits, d->attn_ctr, B);
        if (rc) return rc;
        k_bd_to_bf16<<<std::max(1, (int)((long)B * d->Dq / 256)), 256, 0, st>>>(d->att, d->attb, (long)B * d->Dq);
        rc = tc_dense_gemm(c, b.map_o, H, d->Dq, d->map_attb, d->seg, d->seg + 2, d->o, d->status, d->ks_o,
                           (size_t)nh);
        if (rc) return rc;
        k_bd_add<<<std::max(1, (int)(nh / 256)), 256, 0, st>>>(d->h, d->o, d->ks_o, nh);
        // the router sees the f32 normalised activations (as the single-stream decoder's does),
        // the expert GEMMs their bf16 rounding
        k_bd_norm<<<B, 256, 0, st>>>(d->h, b.ffn_norm, g.rms_eps, H, d->xb, d->x32);
        if (d->world == 1) {
            rc = prefill_forward_x32(b.moe, d->xb, d->x32, (unsigned)B, b.router, nullptr, d->h, d->h);
            if (rc) return rc;
            continue;
        }
        // expert parallelism: route, all-gather the blocks, this rank's experts, return, combine
        const int E = (int)g.n_expert, K = (int)g.n_expert_used, W = d->world;
        rc = prefill_route_x32(b.moe, d->xb, d->x32, (unsigned)B, b.router, nullptr);
        if (rc) return rc;
        const auto *xp = static_cast<const uint16_t *>(moearc_x_prefill_buffer(b.moe, 6));
        const auto *offs = static_cast<const int *>(moearc_x_prefill_buffer(b.moe, 10));
        if (cudaMemcpyAsync(d->ep_send, xp, (size_t)d->P * H * 2, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(d->ep_send + (size_t)d->P * H, offs, sizeof(int) * (E + 1), cudaMemcpyDeviceToDevice, st) !=
                cudaSuccess)
            return ERR;
        if (ep_all_gather(d->comm, d->ep_send, d->ep_rows, (size_t)d->R * H * 2, st) != OK) return ERR;
        k_ep_plan<<<1, 256, sizeof(int) * 2 * W * d->nl, st>>>(d->ep_rows, W, d->R, d->P, H, d->rank * d->nl, d->nl,
                                                               d->ep_off, d->ep_toff, d->ep_w, d->ep_map);
        k_ep_rows<<<W * d->P, 128, 0, st>>>(d->ep_rows, d->R, d->P, H, d->ep_map, d->ep_rows_e);
        rc = prefill_experts_dev(b.moe, d->ep_rows_e, (long)W * d->P, d->ep_off, d->ep_toff, d->ep_w, d->nl,
                                 d->ep_act, d->ep_y);
        if (rc) return rc;
        k_ep_back<<<W * d->P, 256, 0, st>>>(d->ep_y, H, d->ep_map, d->ep_ysrc);
        if (ep_exchange(d->comm, W, d->ep_ysrc, sizeof(float) * d->P * H, d->ep_back, sizeof(float) * d->P * H,
                        sizeof(float) * d->P * H, st) != OK)
            return ERR;
        k_ep_combine<<<(unsigned)((nh + 255) / 256), 256, 0, st>>>(
            d->ep_back, d->P, d->nl, static_cast<const unsigned *>(moearc_x_prefill_buffer(b.moe, 0)),
            static_cast<const int *>(moearc_x_prefill_buffer(b.moe, 9)),
            static_cast<const float *>(moearc_x_prefill_buffer(b.moe, 1)), d->h, B, K, H);
    }
    k_bd_final<<<B, 256, 0, st>>>(d->h, d->output_norm, g.rms_eps, H, d->out, d->dpos);
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

}  // namespace

extern "C" {

void moearc_x_batch_decoder_destroy(moearc_x_batch_decoder *d);
}  // extern "C"

namespace {

moearc_x_batch_decoder *create_impl(moearc_ctx *c, const moearc_x_decoder_cfg *cfg, unsigned n_batch, void *comm,
                                    int rank, int world) {
    if (!c || !cfg || n_batch == 0 || n_batch > 128) return nullptr;
    const auto &g = *cfg;
    if (g.n_layer == 0 || g.n_head_kv == 0 || g.n_head % g.n_head_kv || (g.head_dim != 64 && g.head_dim != 128) ||
        g.n_head / g.n_head_kv > 8 || g.n_ctx == 0 || g.n_swa != 0 || g.has_sinks || g.n_offload || g.n_vocab)
        return nullptr;
    if (g.n_embd % 64 || ((g.n_head * g.head_dim) % 64)) return nullptr;
    if (world < 1 || rank < 0 || rank >= world) return nullptr;
    if (g.expert_layout > 1) return nullptr;
    if (world > 1 && (!comm || g.n_expert % world || g.expert_layout != 0 || g.n_expert > 1000)) return nullptr;
    auto *d = new moearc_x_batch_decoder();
    d->c = c;
    d->cfg = g;
    d->B = (int)n_batch;
    d->comm = comm;
    d->rank = rank;
    d->world = world;
    d->Dq = (int)(g.n_head * g.head_dim);
    d->Dkv = (int)(g.n_head_kv * g.head_dim);
    d->n_qkv = d->Dq + 2 * d->Dkv;
    const int B = d->B, H = (int)g.n_embd;
    d->pages = (int)((g.n_ctx + BD_PAGE - 1) / BD_PAGE);
    auto fail = [&]() {
        moearc_x_batch_decoder_destroy(d);
        return (moearc_x_batch_decoder *)nullptr;
    };
    // activations, scratch, positions, page tables (stream b's pages: a seeded permutation of
    // b * pages .. (b + 1) * pages - 1)
    d->in = static_cast<float *>(d->alloc(sizeof(float) * B * H));
    d->out = static_cast<float *>(d->alloc(sizeof(float) * B * H));
    d->h = static_cast<float *>(d->alloc(sizeof(float) * B * H));
    // a decode-sized batch is one 128-row tile: the projections' K blocks are split so that their
    // row blocks x K runs fill the SMs (a deterministic sum of the runs follows each)
    d->ks_qkv = std::max(1, std::min((int)H / 64, c->sm_count / ((d->n_qkv + 127) / 128)));
    d->ks_o = std::max(1, std::min(d->Dq / 64, c->sm_count / ((H + 127) / 128)));
    d->o = static_cast<float *>(d->alloc(sizeof(float) * B * H * d->ks_o));
    d->x32 = static_cast<float *>(d->alloc(sizeof(float) * B * H));
    d->qkv = static_cast<float *>(d->alloc(sizeof(float) * B * d->n_qkv * d->ks_qkv));
    d->q = static_cast<float *>(d->alloc(sizeof(float) * B * d->Dq));
    d->att = static_cast<float *>(d->alloc(sizeof(float) * B * d->Dq));
    d->xb = static_cast<uint16_t *>(d->alloc(2 * (size_t)B * H));
    d->attb = static_cast<uint16_t *>(d->alloc(2 * (size_t)B * d->Dq));
    d->output_norm = static_cast<float *>(d->alloc(sizeof(float) * H));
    d->dpos = static_cast<int *>(d->alloc(sizeof(int) * B));
    d->seg = static_cast<int *>(d->alloc(sizeof(int) * 4));
    d->status = static_cast<int *>(d->alloc(sizeof(int)));
    d->tables = static_cast<unsigned *>(d->alloc(sizeof(unsigned) * B * d->pages));
    d->max_splits = std::max(1, (8 * c->sm_count) / (B * (int)g.n_head_kv));
    d->attn_scratch_b = (size_t)B * attn_scratch_bytes(g.n_head, g.head_dim, d->max_splits);
    d->attn_scratch = static_cast<float *>(d->alloc(d->attn_scratch_b));
    d->attn_ctr = static_cast<unsigned *>(d->alloc(sizeof(unsigned) * B * g.n_head_kv));
    if (!d->in || !d->out || !d->h || !d->o || !d->x32 || !d->qkv || !d->q || !d->att || !d->xb || !d->attb || !d->output_norm ||
        !d->dpos || !d->seg || !d->status || !d->tables || !d->attn_scratch || !d->attn_ctr)
        return fail();
    if (world > 1) {
        // one block: P rows of f16 activations, then the E + 1 offsets in whole rows
        d->nl = (int)g.n_expert / world;
        d->P = B * (int)g.n_expert_used;
        d->R = d->P + (int)((sizeof(int) * (g.n_expert + 1) + 2 * H - 1) / (2 * H));
        const size_t WR = (size_t)world * d->R, WP = (size_t)world * d->P, nseg = (size_t)d->nl + 1;
        d->ep_send = static_cast<uint16_t *>(d->alloc(2 * (size_t)d->R * H));
        d->ep_rows = static_cast<uint16_t *>(d->alloc(2 * WR * H));
        d->ep_rows_e = static_cast<uint16_t *>(d->alloc(2 * WP * H));
        d->ep_act = static_cast<uint16_t *>(d->alloc(2 * WP * g.n_ff));
        d->ep_y = static_cast<float *>(d->alloc(sizeof(float) * WP * H));
        d->ep_ysrc = static_cast<float *>(d->alloc(sizeof(float) * WP * H));
        d->ep_back = static_cast<float *>(d->alloc(sizeof(float) * WP * H));
        d->ep_off = static_cast<int *>(d->alloc(sizeof(int) * nseg));
        d->ep_toff = static_cast<int *>(d->alloc(sizeof(int) * nseg));
        d->ep_w = static_cast<int *>(d->alloc(sizeof(int) * nseg));
        d->ep_map = static_cast<int *>(d->alloc(sizeof(int) * WP));
        if (!d->ep_send || !d->ep_rows || !d->ep_rows_e || !d->ep_act || !d->ep_y || !d->ep_ysrc || !d->ep_back ||
            !d->ep_off || !d->ep_toff || !d->ep_w || !d->ep_map ||
            cudaMemset(d->ep_send, 0, 2 * (size_t)d->R * H) != cudaSuccess)
            return fail();
    }
    bool ok = true;
    {
        std::vector<unsigned> t((size_t)B * d->pages);
        uint64_t st = g.seed ^ 0xBA7C4ull;
        for (int b = 0; b < B; ++b) {
            unsigned *tb = t.data() + (size_t)b * d->pages;
            for (int i = 0; i < d->pages; ++i) tb[i] = (unsigned)(b * d->pages + i);
            for (int i = d->pages - 1; i > 0; --i) {
                st = st * 6364136223846793005ull + 1442695040888963407ull;
                std::swap(tb[i], tb[(int)((st >> 33) % (uint64_t)(i + 1))]);
            }
        }
        const int seg[4] = {0, B, 0, (B + 127) / 128};
        ok &= cudaMemcpy(d->tables, t.data(), sizeof(unsigned) * t.size(), cudaMemcpyHostToDevice) == cudaSuccess;
        ok &= cudaMemcpy(d->seg, seg, sizeof(seg), cudaMemcpyHostToDevice) == cudaSuccess;
        ok &= cudaMemset(d->dpos, 0, sizeof(int) * B) == cudaSuccess;
        ok &= cudaMemset(d->status, 0, sizeof(int)) == cudaSuccess;
        ok &= cudaMemset(d->attn_ctr, 0, sizeof(unsigned) * B * g.n_head_kv) == cudaSuccess;
        ok &= cudaMemset(d->in, 0, sizeof(float) * B * H) == cudaSuccess;
    }
    // RoPE angle table (as the single-stream decoder builds it)
    {
        const int half = (int)g.head_dim / 2;
        std::vector<double> fr(half);
        const double ts = std::pow((double)g.rope_base, -2.0 / (double)g.head_dim);
        double ms = g.rope_attn_factor;
        for (int p = 0; p < half; ++p) {
            double f = (double)g.rope_freq_scale;
            if (g.rope_ext_factor != 0.0f) {
                const double den = std::fmax(0.001, (double)g.rope_corr_hi - (double)g.rope_corr_lo);
                const double y = ((double)p - (double)g.rope_corr_lo) / den;
                const double ramp = 1.0 - std::fmin(1.0, std::fmax(0.0, y));
                const double mix = ramp * (double)g.rope_ext_factor;
                f = f * (1.0 - mix) + mix;
            }
            fr[p] = std::pow(ts, (double)p) * f;
        }
        if (g.rope_ext_factor != 0.0f) ms *= 1.0 + 0.1 * std::log(1.0 / (double)g.rope_freq_scale);
        d->rope_mscale = ms;
        d->rope_freq = static_cast<double *>(d->alloc(sizeof(double) * half));
        ok &= d->rope_freq &&
              cudaMemcpy(d->rope_freq, fr.data(), sizeof(double) * half, cudaMemcpyHostToDevice) == cudaSuccess;
    }
    ok &= tc_make_map_bf16(&d->map_xb, d->xb, B, H) && tc_make_map_bf16(&d->map_attb, d->attb, B, d->Dq);
    auto seed = [&](int kind, unsigned l) { return moearc_x_decoder_seed(nullptr, kind, l, g.seed); };
    ok &= moearc_x_synth(c, d->output_norm, H, 4, seed(11, 0), 0.1f, 0, 0) == OK;
    // per block: the same tensors and seeds as moearc_x_decoder; expert banks packed, expanded to
    // bf16 by the block's prefill object, and the packed copies dropped
    moearc_x_moe_desc md{g.n_embd, g.n_ff, g.n_expert, g.n_expert_used, g.gating, g.act, g.alpha, g.limit,
                         g.expert_type, (unsigned)B};
    moearc_x_moe_desc md1 = md;
    md1.max_tokens = 1;
    moearc_x_moe *packer = moearc_x_moe_create(c, &md1);
    const size_t bb = (g.expert_type == T_MXFP4) ? 17 : 18;
    const size_t blocks = (size_t)g.n_expert * g.n_ff * g.n_embd / 32, bank = blocks * bb;
    const unsigned ekind = (g.expert_type == T_MXFP4) ? 2 : 3;
    void *staging = nullptr, *packed = nullptr;
    if (!packer || cudaMalloc(&staging, std::max(3 * bank, (size_t)d->n_qkv * H * 2)) != cudaSuccess ||
        cudaMalloc(&packed, 3 * bank) != cudaSuccess) {
        cudaGetLastError();
        if (packer) moearc_x_moe_destroy(packer);
        cudaFree(staging);
        return fail();
    }
    const size_t pool = (size_t)B * d->pages * BD_PAGE * d->Dkv;
    d->L.resize(g.n_layer);
    for (unsigned l = 0; l < g.n_layer && ok; ++l) {
        auto &b = d->L[l];
        b.moe = nullptr;
        b.attn_norm = static_cast<float *>(d->alloc(sizeof(float) * H));
        b.ffn_norm = static_cast<float *>(d->alloc(sizeof(float) * H));
        b.router = static_cast<float *>(d->alloc(sizeof(float) * g.n_expert * H));
        b.q_norm = g.has_qk_norm ? static_cast<float *>(d->alloc(sizeof(float) * g.head_dim)) : nullptr;
        b.k_norm = g.has_qk_norm ? static_cast<float *>(d->alloc(sizeof(float) * g.head_dim)) : nullptr;
        b.wqkv = static_cast<uint16_t *>(d->alloc(2 * (size_t)d->n_qkv * H));
        b.wo = static_cast<uint16_t *>(d->alloc(2 * (size_t)H * d->Dq));
        b.k_pages = static_cast<uint16_t *>(d->alloc(2 * pool));
        b.v_pages = static_cast<uint16_t *>(d->alloc(2 * pool));
        b.moe = moearc_x_prefill_create(c, &md);
        if (!b.attn_norm || !b.ffn_norm || !b.router || !b.wqkv || !b.wo || !b.k_pages || !b.v_pages || !b.moe) {
            ok = false;
            break;
        }
        ok &= moearc_x_synth(c, b.attn_norm, H, 4, seed(0, l), 0.1f, 0, 0) == OK;
        ok &= moearc_x_synth(c, b.ffn_norm, H, 4, seed(1, l), 0.1f, 0, 0) == OK;
        ok &= moearc_x_synth(c, b.router, (size_t)g.n_expert * H, 0, seed(7, l), 0.02f, 0, 0) == OK;
        if (g.has_qk_norm) {
            ok &= b.q_norm && b.k_norm;
            ok &= ok && moearc_x_synth(c, b.q_norm, g.head_dim, 4, seed(14, l), 0.1f, 0, 0) == OK;
            ok &= ok && moearc_x_synth(c, b.k_norm, g.head_dim, 4, seed(15, l), 0.1f, 0, 0) == OK;
        }
        ok &= moearc_x_synth(c, b.wqkv, (size_t)d->Dq * H, 1, seed(2, l), 0.02f, 0, 0) == OK;
        ok &= moearc_x_synth(c, b.wqkv + (size_t)d->Dq * H, (size_t)d->Dkv * H, 1, seed(3, l), 0.02f, 0, 0) == OK;
        ok &= moearc_x_synth(c, b.wqkv + (size_t)(d->Dq + d->Dkv) * H, (size_t)d->Dkv * H, 1, seed(4, l), 0.02f, 0, 0) == OK;
        ok &= moearc_x_synth(c, b.wo, (size_t)H * d->Dq, 1, seed(5, l), 0.02f, 0, 0) == OK;
        uint8_t *s8 = static_cast<uint8_t *>(staging), *p8 = static_cast<uint8_t *>(packed);
        ok &= moearc_x_synth(c, s8, blocks, ekind, seed(8, l), 0.01f, -8, -4) == OK;
        ok &= moearc_x_synth(c, s8 + bank, blocks, ekind, seed(9, l), 0.01f, -8, -4) == OK;
        ok &= moearc_x_synth(c, s8 + 2 * bank, blocks, ekind, seed(10, l), 0.01f, -8, -4) == OK;
        ok &= moearc_x_moe_pack(packer, s8, s8 + bank, s8 + 2 * bank, g.n_expert, p8, p8 + 2 * bank) == OK;
        // expert_layout 0: the 4-bit form (read at 4 bits, expanded to f16 tiles in shared memory,
        // 32-row tiles for the few rows per expert of a decode step); 1: the bf16 expansion
        if (world > 1) {  // this rank's experts rank * nl .. into slots 0 .. nl - 1
            std::vector<int> mine(d->nl);
            for (int j = 0; j < d->nl; ++j) mine[j] = rank * d->nl + j;
            ok &= moearc_x_prefill_load4_list(b.moe, p8, p8 + 2 * bank, mine.data(), (unsigned)d->nl) == OK;
        } else {
            ok &= (g.expert_layout == 0 ? moearc_x_prefill_load4(b.moe, p8, p8 + 2 * bank)
                                        : moearc_x_prefill_load(b.moe, p8, p8 + 2 * bank)) == OK;
        }
        ok &= cudaMemsetAsync(b.k_pages, 0, 2 * pool, c->stream) == cudaSuccess;
        ok &= cudaMemsetAsync(b.v_pages, 0, 2 * pool, c->stream) == cudaSuccess;
        ok &= tc_make_map_bf16(&b.map_qkv, b.wqkv, d->n_qkv, H) && tc_make_map_bf16(&b.map_o, b.wo, H, d->Dq);
        ok &= cudaStreamSynchronize(c->stream) == cudaSuccess;  // the staging buffers are reused
    }
    moearc_x_moe_destroy(packer);
    cudaFree(staging);
    cudaFree(packed);
    if (!ok) return fail();
    return d;
}

}  // namespace

extern "C" {

moearc_x_batch_decoder *moearc_x_batch_decoder_create(moearc_ctx *c, const moearc_x_decoder_cfg *cfg,
                                                      unsigned n_batch) {
    return create_impl(c, cfg, n_batch, nullptr, 0, 1);
}

moearc_x_batch_decoder *moearc_x_batch_decoder_create_ep(moearc_ctx *c, const moearc_x_decoder_cfg *cfg,
                                                         unsigned n_batch, void *comm, int rank, int n_ranks) {
    return create_impl(c, cfg, n_batch, comm, rank, n_ranks);
}

void moearc_x_batch_decoder_destroy(moearc_x_batch_decoder *d) {
    if (!d) return;
    cudaStreamSynchronize(d->c->stream);
    if (d->exec) cudaGraphExecDestroy(d->exec);
    if (d->graph) cudaGraphDestroy(d->graph);
    for (auto &b : d->L)
        if (b.moe) moearc_x_prefill_destroy(b.moe);
    for (void *p : d->allocs) cudaFree(p);
    delete d;
}

void *moearc_x_batch_decoder_input(moearc_x_batch_decoder *d) { return d ? d->in : nullptr; }
void *moearc_x_batch_decoder_output(moearc_x_batch_decoder *d) { return d ? d->out : nullptr; }

// Every stream at position pos (a sequence that has decoded pos tokens); with fill, every KV
// page gets synthetic bf16 N(0, 0.02) contents from `seed` first.
int moearc_x_batch_decoder_set_pos(moearc_x_batch_decoder *d, unsigned pos, int fill, unsigned long long seed) {
    if (!d) return ERR;
    if (pos >= d->cfg.n_ctx) return ERR_ARG;
    if (fill) {
        const size_t n = (size_t)d->B * d->pages * BD_PAGE * d->Dkv;
        for (unsigned l = 0; l < d->cfg.n_layer; ++l) {
            if (moearc_x_synth(d->c, d->L[l].k_pages, n, 1, moearc_x_decoder_seed(nullptr, 12, l, seed), 0.02f, 0, 0) != OK ||
                moearc_x_synth(d->c, d->L[l].v_pages, n, 1, moearc_x_decoder_seed(nullptr, 13, l, seed), 0.02f, 0, 0) != OK)
                return ERR;
        }
    }
    k_bd_set_pos<<<1, 256, 0, d->c->stream>>>(d->dpos, (int)pos, d->B);
    d->pos = (int)pos;
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

// One token for every stream (inputs: n_batch x n_embd f32 at moearc_x_batch_decoder_input;
// outputs at _output). The first call captures the step as a CUDA graph, later calls replay it.
int moearc_x_batch_decoder_step(moearc_x_batch_decoder *d) {
    if (!d) return ERR;
    if ((unsigned)d->pos >= d->cfg.n_ctx) return ERR_ARG;
    moearc_ctx *c = d->c;
    if (!d->exec) {
        if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return ERR;
        const int rc = enqueue(d);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(c->stream, &g);
        if (rc || e != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
            return rc ? rc : ERR;
        }
        d->graph = g;
        if (cudaGraphInstantiate(&d->exec, g, 0) != cudaSuccess) {
            cudaGetLastError();
            return ERR;
        }
    }
    if (cudaGraphLaunch(d->exec, c->stream) != cudaSuccess) return ERR;
    d->pos += 1;
    return OK;
}

// Reads and clears the status words of the step's kernels (GEMM waits and the MoE blocks'):
// 0, or a nonzero bit pattern when a bounded wait gave up.
void *moearc_x_batch_decoder_routing(moearc_x_batch_decoder *d, unsigned int layer) {
    if (!d || layer >= d->L.size()) return nullptr;
    return moearc_x_prefill_buffer(d->L[layer].moe, 0);
}

int moearc_x_batch_decoder_status(moearc_x_batch_decoder *d) {
    if (!d) return ERR;
    int s = 0;
    if (cudaMemcpy(&s, d->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return ERR;
    cudaMemset(d->status, 0, sizeof(int));
    for (auto &b : d->L) {
        const int m = moearc_x_prefill_status(b.moe);
        if (m < 0) return ERR;
        s |= m;
    }
    return s;
}

}  // extern "C"
