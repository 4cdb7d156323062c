// decoder.cu — a synthetic routed-MoE decoder (gpt-oss / Qwen3-MoE shaped) decoding one token
// per step on the device, the per-block sequence of crates/moearc-engine/src/moe.rs:1862-2443:
//
//   h = input embedding
//   for each block: x = rmsnorm(h) ; q,k,v = W x ; rope(q), rope(k) ; append K,V at (page,slot)
//                   attn = attention over [kv_begin, n_kv) (+ sinks) ; h += Wo attn
//                   h += MoE(rmsnorm(h))
//   out = rmsnorm(h)
//
// Blocks with l % swa_pattern < swa_pattern - 1 attend through a window of n_swa keys
// (moe.rs:687-699) kept in a ring of ceil(n_swa / page) pages addressed through a cyclic page
// table (moe.rs:1420-1438, 1506-1513); the others through the sequence's page table.
//
// Weights are random (seeded) and generated on the device; nothing is read from a model file.
// The position lives in device memory and is advanced by the step's last kernel, so the whole
// step — 7 kernels per block — is captured once as a CUDA graph and replayed.
//
// Blocks below cfg.n_offload keep their packed expert banks in pinned, device-mapped host memory
// (the -ncmoe mirror, moe.rs:1179-1299 StaticSplit with every expert of the block streamed);
// their MoE adds two fetch kernels that copy the routed experts over PCIe into device slots, so
// the step stays one graph with no host round trip. With a host policy
// (moearc_x_decoder_host_experts) part of those experts is computed by a pool of host threads
// from the same pinned banks while the device streams the rest (moe.rs:2169-2211, 2389-2420):
// the split and the answer pass through a mailbox in pinned memory that a host thread polls, so
// the step stays one graph with no host function in it.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include <unistd.h>

#include "common.cuh"
#include "dense.cuh"
#include "host_experts.hpp"
#include "step.cuh"
#include "tma.cuh"

namespace moearc {
int moe_forward_impl(moearc_x_moe *m, const float *x, unsigned n_tokens, const float *norm_w, float eps,
                     const float *router_w, const float *router_b, const void *gateup_packed,
                     const void *down_packed, const float *residual, float *out,
                     std::vector<cudaEvent_t> *marks = nullptr, std::vector<int> *kinds = nullptr,
                     const moe_offload *off = nullptr, unsigned long long *span = nullptr, bool tc = false,
                     int span_cta = 0);
int moe_decode_grid(moearc_x_moe *m);
size_t attn_scratch_bytes(size_t n_heads, size_t head_dim, int n_splits);
int attn_launch(moearc_ctx *c, float *out, const float *q, const void *kp, const void *vp,
                const unsigned *table, const float *sinks, size_t n_heads, size_t n_kv_heads,
                size_t hd, size_t kv_begin, size_t n_kv, size_t pt, float scale, unsigned kv_type,
                float *scratch, size_t scratch_bytes, const int *dpos, int window, int max_splits,
                unsigned *ctr);
}  // namespace moearc

using namespace moearc;

namespace {

constexpr int PAGE_TOKENS = 32;  // moe.rs:153

// Seed of one tensor: the model seed, the tensor kind and the layer, mixed.
uint64_t tensor_seed(uint64_t seed, int kind, int layer) {
    uint64_t z = seed ^ ((uint64_t)(kind + 1) << 40) ^ ((uint64_t)(layer + 1) * 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 31)) * 0xBF58476D1CE4E5B9ull;
    return z ^ (z >> 29);
}

__global__ void k_step_end(float *out, const float *h, const float *w, int n, float eps, int *pos) {
    __shared__ float red[32];
    pdl_wait();
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(h[i], h[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    const float scale = 1.0f / sqrtf(t / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = (h[i] * scale) * w[i];
    __syncthreads();
    if (threadIdx.x == 0) *pos += 1;
}

__global__ void k_set_pos(int *pos, int v) { *pos = v; }

}  // namespace

struct moearc_x_decoder {
    moearc_ctx *c;
    moearc_x_decoder_cfg cfg;
    int Dq, Dkv, n_qkv;
    struct layer {
        float *attn_norm, *ffn_norm, *sinks, *router;
        float *q_norm, *k_norm;           // QK-norm weights [head_dim] (has_qk_norm) or null
        void *wqkv, *wo, *gateup, *down;  // gateup/down: device-visible host banks when offloaded
        void *gu_host, *dn_host;           // pinned host allocations of an offloaded block
        moe_offload off;                   // an offloaded block's own residency cache (n_cache)
        uint16_t *k_pages, *v_pages;
        const unsigned *table;
        int window;
        size_t pool_tokens;
    };
    std::vector<layer> L;
    float *output_norm = nullptr;
    dense_gemv *qkv = nullptr, *wo = nullptr;
    dense_gemv *head = nullptr;  // the output head (n_vocab rows), or null
    void *w_out = nullptr;       // its packed bf16 weights
    float *logits = nullptr;     // [n_vocab]
    moearc_x_moe *moe = nullptr;
    int *dpos = nullptr;
    unsigned *table_full = nullptr, *table_swa = nullptr;
    float *in = nullptr, *h = nullptr, *q = nullptr, *att = nullptr, *out = nullptr;
    float *attn_scratch = nullptr;
    size_t attn_scratch_b = 0;
    unsigned *attn_ctr = nullptr;  // one split counter per KV head, zero between steps
    double *rope_freq = nullptr;   // head_dim / 2 angle multipliers (see dense_rope)
    double rope_mscale = 1.0;
    int max_splits = 1;
    int pos = 0;
    std::vector<void *> allocs;
    std::vector<void *> host_allocs;  // pinned (cudaHostAlloc) banks of offloaded blocks
    moe_offload off{};                // device slots the offloaded blocks' experts are fetched into
    unsigned long long *fetched = nullptr;  // experts the residency caches fetched
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    // moearc_x_decoder_step_host: pinned staging of one input and one output row, and the step
    // captured with its two copies (host -> in, out -> host) as one graph
    float *pin_in = nullptr, *pin_out = nullptr;
    float *pin_in_dev = nullptr, *pin_out_dev = nullptr;  // their device mappings
    cudaGraph_t graph_io = nullptr;
    cudaGraphExec_t exec_io = nullptr;
    bool use_graph = true;
    // the whole step as one persistent kernel (step.cuh) when the shape allows it; the chain
    // of per-block kernels otherwise (offloaded experts, head_dim 128, ...) or on request
    step_plan *step = nullptr;
    bool use_step = false;
    // resident blocks' expert banks in the tc layout, run on the block-scaled FP4 tensor cores
    bool tc = false;
    // the chain's expert kernels' CTA timestamps per block (moearc_x_decoder_kernel_spans), or null
    unsigned long long *spans = nullptr;
    int span_cta = 0;
    // host execution of part of the offloaded blocks' experts (moearc_x_decoder_host_experts):
    // the pool, the per-block split records, the pinned mail and done records (host pointers),
    // and the thread that polls the mail
    host_pool *pool = nullptr;
    std::vector<moe_host> hosts;  // per offloaded block (kind 0: off)
    uint8_t *mail = nullptr, *done = nullptr;
    unsigned *hmask = nullptr;
    unsigned long long *hseq = nullptr;
    float *hffn = nullptr;
    int *hstatus = nullptr;
    std::thread poller;
    std::atomic<bool> poll_stop{false}, poll_hold{false};
    std::atomic<int> host_failed{0};
    host_shape hshape{};

    // The host side of the mailbox: a new sequence number in the mail is a job; its answer (the
    // host's share, then the same number) goes to the done record. Polls continuously while
    // jobs come; after 20 ms without one it naps 50 us between polls.
    void poll_mail() {
        const auto *seqp = reinterpret_cast<const std::atomic<unsigned long long> *>(mail + MAIL_SEQ);
        auto *donep = reinterpret_cast<std::atomic<unsigned long long> *>(done + DONE_SEQ);
        unsigned long long last = seqp->load(std::memory_order_acquire);
        auto idle0 = std::chrono::steady_clock::now();
        while (!poll_stop.load(std::memory_order_relaxed)) {
            const unsigned long long sq = seqp->load(std::memory_order_acquire);
            if (sq == last || poll_hold.load(std::memory_order_relaxed)) {
                if (std::chrono::steady_clock::now() - idle0 > std::chrono::milliseconds(20))
                    std::this_thread::sleep_for(std::chrono::microseconds(50));
                else
                    __builtin_ia32_pause();
                continue;
            }
            last = sq;
            unsigned n, blk;
            std::memcpy(&n, mail + MAIL_N, 4);
            std::memcpy(&blk, mail + MAIL_BLOCK, 4);
            float *out = reinterpret_cast<float *>(done + DONE_OUT);
            if (n == 0 || n > 32 || blk >= cfg.n_offload ||
                host_submit(pool, hshape, static_cast<const uint8_t *>(L[blk].gu_host),
                            static_cast<const uint8_t *>(L[blk].dn_host),
                            reinterpret_cast<const unsigned *>(mail + MAIL_IDS),
                            reinterpret_cast<const float *>(mail + MAIL_WTS), n,
                            reinterpret_cast<const float *>(mail + MAIL_X)) != 0 ||
                host_sync(pool, out) != 0) {
                for (unsigned i = 0; i < cfg.n_embd; ++i) out[i] = NAN;
                host_failed.store(1);
            }
            donep->store(sq, std::memory_order_release);
            idle0 = std::chrono::steady_clock::now();
        }
    }

    void stop_poller() {
        if (poller.joinable()) {
            poll_stop.store(true);
            poller.join();
        }
    }

    void drop_graph() {
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
        if (exec_io) cudaGraphExecDestroy(exec_io);
        if (graph_io) cudaGraphDestroy(graph_io);
        exec = nullptr;
        graph = nullptr;
        exec_io = nullptr;
        graph_io = nullptr;
    }

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

bool is_swa(const moearc_x_decoder_cfg &c, unsigned l) {
    return c.n_swa > 0 && c.swa_pattern > 0 && (l % c.swa_pattern) < c.swa_pattern - 1;
}

// Profiling: an event after each launch, tagged with the launch's kind.
struct step_marks {
    std::vector<cudaEvent_t> ev;
    std::vector<int> kind;
    void mark(cudaStream_t s, int k) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        cudaEventRecord(e, s);
        ev.push_back(e);
        kind.push_back(k);
    }
};

// Everything one step enqueues, in order (captured into a graph on first use). With `pm`,
// an event follows every kernel: kinds 0 qkv, 1 attention (+ combine), 2 o-proj, 3 MoE route,
// 4 MoE gate-up, 5 MoE down, 6 final norm, 7 expert fetch (offloaded blocks).
int enqueue_step(moearc_x_decoder *d, step_marks *pm = nullptr) {
    moearc_ctx *c = d->c;
    const auto &cfg = d->cfg;
    if (d->step && d->use_step && !pm) {
        int rc = step_run(d->step, d->in, d->out, d->output_norm, d->dpos);
        if (rc == OK && d->head)
            rc = dense_run(d->head, d->w_out, d->out, nullptr, 0.f, d->logits, nullptr, d->dpos, nullptr, nullptr);
        return rc;
    }
    if (cudaMemcpyAsync(d->h, d->in, sizeof(float) * cfg.n_embd, cudaMemcpyDeviceToDevice, c->stream) != cudaSuccess)
        return ERR;
    if (pm) pm->mark(c->stream, -1);
    dense_rope rope;
    rope.n_q_heads = (int)cfg.n_head;
    rope.n_kv_heads = (int)cfg.n_head_kv;
    rope.head_dim = (int)cfg.head_dim;
    rope.freq = d->rope_freq;
    rope.mscale = d->rope_mscale;
    const float scale = 1.0f / std::sqrt((float)cfg.head_dim);
    for (unsigned l = 0; l < cfg.n_layer; ++l) {
        auto &b = d->L[l];
        dense_kv kv{b.k_pages, b.v_pages, b.table, PAGE_TOKENS};
        rope.q_norm = b.q_norm;
        rope.k_norm = b.k_norm;
        rope.norm_eps = cfg.rms_eps;
        int rc = dense_run(d->qkv, b.wqkv, d->h, b.attn_norm, cfg.rms_eps, d->q, nullptr, d->dpos, &rope, &kv);
        if (rc) return rc;
        if (pm) pm->mark(c->stream, 0);
        rc = attn_launch(c, d->att, d->q, b.k_pages, b.v_pages, b.table, b.sinks, cfg.n_head, cfg.n_head_kv,
                         cfg.head_dim, 0, 1, PAGE_TOKENS, scale, T_BF16, d->attn_scratch, d->attn_scratch_b,
                         d->dpos, b.window, d->max_splits, d->attn_ctr);
        if (rc) return rc;
        if (pm) pm->mark(c->stream, 1);
        rc = dense_run(d->wo, b.wo, d->att, nullptr, 0.f, d->h, d->h, d->dpos, nullptr, nullptr);
        if (rc) return rc;
        if (pm) pm->mark(c->stream, 2);
        moe_offload off{};
        if (l < cfg.n_offload) {
            off = cfg.n_cache ? b.off : d->off;
            off.host = l < d->hosts.size() && d->hosts[l].kind ? &d->hosts[l] : nullptr;
        }
        rc = moe_forward_impl(d->moe, d->h, 1, b.ffn_norm, cfg.rms_eps, b.router, nullptr, b.gateup, b.down,
                              d->h, d->h, pm ? &pm->ev : nullptr, pm ? &pm->kind : nullptr,
                              l < cfg.n_offload ? &off : nullptr,
                              d->spans ? d->spans + (size_t)l * 2 * d->span_cta * 3 : nullptr,
                              d->tc && l >= cfg.n_offload, d->span_cta);
        if (rc) return rc;
    }
    if (launch_pdl(k_step_end, dim3(1), dim3(512), 0, c->stream, d->out, (const float *)d->h,
                   (const float *)d->output_norm, (int)cfg.n_embd, cfg.rms_eps, d->dpos) != cudaSuccess)
        return ERR;
    if (d->head) {
        // the output head on the normalised final state (moe.rs:2434-2437)
        const int rc = dense_run(d->head, d->w_out, d->out, nullptr, 0.f, d->logits, nullptr, d->dpos, nullptr, nullptr);
        if (rc) return rc;
    }
    if (pm) pm->mark(c->stream, 6);
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

int synth(moearc_ctx *c, void *dst, size_t n, unsigned kind, uint64_t seed, float sigma, int lo = -8, int hi = -4) {
    return moearc_x_synth(c, dst, n, kind, seed, sigma, lo, hi);
}

}  // namespace

extern "C" {

moearc_x_decoder *moearc_x_decoder_create(moearc_ctx *c, const moearc_x_decoder_cfg *cfg) {
    if (!c || !cfg) return nullptr;
    const auto &g = *cfg;
    if (g.n_layer == 0 || g.n_head % std::max(1u, g.n_head_kv) || (g.head_dim != 64 && g.head_dim != 128))
        return nullptr;
    if (g.n_head / g.n_head_kv > 8 || g.n_ctx == 0 || g.n_offload > g.n_layer) return nullptr;
    if (g.n_cache && (g.n_cache < g.n_expert_used || g.n_cache > g.n_expert || !g.n_offload)) return nullptr;
    if (g.n_vocab % 16) return nullptr;
    auto *d = new moearc_x_decoder();
    d->c = c;
    d->cfg = g;
    d->Dq = (int)(g.n_head * g.head_dim);
    d->Dkv = (int)(g.n_head_kv * g.head_dim);
    d->n_qkv = d->Dq + 2 * d->Dkv;
    const int H = (int)g.n_embd;
    bool ok = true;
    auto fail = [&]() {
        moearc_x_decoder_destroy(d);
        return (moearc_x_decoder *)nullptr;
    };
    moearc_x_moe_desc md{g.n_embd, g.n_ff, g.n_expert, g.n_expert_used, g.gating, g.act, g.alpha, g.limit,
                         g.expert_type, 1};
    d->moe = moearc_x_moe_create(c, &md);
    set_smem(k_step_end, 0);
    cudaGetLastError();
    d->qkv = dense_create(c, d->n_qkv, H, 0);
    d->wo = dense_create(c, H, d->Dq, 1);
    if (!d->moe || !d->qkv || !d->wo) return fail();
    d->tc = g.expert_layout == 0 && g.expert_type == T_MXFP4 && moearc_x_moe_has_tc(d->moe) &&
            g.n_offload < g.n_layer;
    if (g.n_vocab) {
        d->head = dense_create(c, (int)g.n_vocab, H, 1);
        d->w_out = d->alloc((size_t)g.n_vocab * H * 2);
        d->logits = static_cast<float *>(d->alloc(sizeof(float) * g.n_vocab));
        if (!d->head || !d->w_out || !d->logits) return fail();
    }

    // page tables: the sequence's (a seeded permutation, so pages are scattered as a pool that
    // has served other sequences would hand them out) and the windowed blocks' ring
    const int pages = (int)((g.n_ctx + PAGE_TOKENS - 1) / PAGE_TOKENS);
    const int swa_pages = g.n_swa ? std::min(pages, (int)((g.n_swa + PAGE_TOKENS - 1) / PAGE_TOKENS)) : pages;
    std::vector<unsigned> tf(pages), ts(pages);
    for (int i = 0; i < pages; ++i) tf[i] = (unsigned)i;
    uint64_t st = g.seed ^ 0x7AB1Eull;
    for (int i = pages - 1; i > 0; --i) {
        st = st * 6364136223846793005ull + 1442695040888963407ull;
        std::swap(tf[i], tf[(int)((st >> 33) % (uint64_t)(i + 1))]);
    }
    for (int i = 0; i < pages; ++i) ts[i] = (unsigned)(i % swa_pages);
    d->table_full = static_cast<unsigned *>(d->alloc(sizeof(unsigned) * pages));
    d->table_swa = static_cast<unsigned *>(d->alloc(sizeof(unsigned) * pages));
    d->dpos = static_cast<int *>(d->alloc(sizeof(int)));
    d->in = static_cast<float *>(d->alloc(sizeof(float) * H));
    d->h = static_cast<float *>(d->alloc(sizeof(float) * H));
    d->out = static_cast<float *>(d->alloc(sizeof(float) * H));
    d->q = static_cast<float *>(d->alloc(sizeof(float) * d->Dq));
    d->att = static_cast<float *>(d->alloc(sizeof(float) * d->Dq));
    d->output_norm = static_cast<float *>(d->alloc(sizeof(float) * H));
    d->max_splits = std::max(1, (2 * c->sm_count + (int)g.n_head_kv - 1) / (int)g.n_head_kv);
    d->attn_scratch_b = attn_scratch_bytes(g.n_head, g.head_dim, d->max_splits);
    d->attn_scratch = static_cast<float *>(d->alloc(d->attn_scratch_b));
    d->attn_ctr = static_cast<unsigned *>(d->alloc(sizeof(unsigned) * g.n_head));
    // RoPE angle of pair p at position pos = pos * freq[p]: base^(-2p/head_dim), blended per
    // pair by the YaRN ramp (the closed form of reference.rs rope_ext, folded per pair)
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
        ok &= d->rope_freq && cudaMemcpy(d->rope_freq, fr.data(), sizeof(double) * half, cudaMemcpyHostToDevice) == cudaSuccess;
    }
    if (!d->table_full || !d->table_swa || !d->dpos || !d->in || !d->h || !d->out || !d->q || !d->att ||
        !d->output_norm || !d->attn_scratch)
        return fail();
    ok &= cudaMemcpy(d->table_full, tf.data(), sizeof(unsigned) * pages, cudaMemcpyHostToDevice) == cudaSuccess;
    ok &= cudaMemcpy(d->table_swa, ts.data(), sizeof(unsigned) * pages, cudaMemcpyHostToDevice) == cudaSuccess;
    ok &= cudaMemset(d->dpos, 0, sizeof(int)) == cudaSuccess;
    ok &= d->attn_ctr && cudaMemset(d->attn_ctr, 0, sizeof(unsigned) * g.n_head) == cudaSuccess;
    ok &= cudaMemset(d->in, 0, sizeof(float) * H) == cudaSuccess;
    ok &= synth(c, d->output_norm, H, 4, tensor_seed(g.seed, 11, 0), 0.1f) == OK;

    // per-layer weights: generated in GGUF/row-major layout into a staging buffer, then packed
    const size_t bb = (g.expert_type == T_MXFP4) ? 17 : 18;
    const size_t blocks = (size_t)g.n_expert * g.n_ff * g.n_embd / 32;
    const size_t bank_bytes = blocks * bb;
    const size_t qkv_elems = (size_t)d->n_qkv * H, wo_elems = (size_t)H * d->Dq;
    const size_t stage_bytes = std::max({3 * bank_bytes, qkv_elems * 2, wo_elems * 2, (size_t)g.n_vocab * H * 2});
    void *staging = nullptr;
    if (cudaMalloc(&staging, stage_bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail();
    }
    // offloaded blocks: packed on the device into pack_tmp, then copied to pinned host banks;
    // one device slot per expert a token routes to
    const size_t gu_stride = moearc_x_moe_packed_bytes(&md, 0), dn_stride = moearc_x_moe_packed_bytes(&md, 1);
    void *pack_tmp = nullptr;
    if (g.n_offload && g.n_cache) {
        // one residency cache per offloaded block: its slots, the tables (every expert out,
        // every slot empty and older than any position) and a plan; one shared fetch count
        d->L.resize(g.n_layer);
        d->fetched = static_cast<unsigned long long *>(d->alloc(sizeof(unsigned long long)));
        const std::vector<int> older(g.n_cache, INT_MIN);
        bool okc = d->fetched && cudaMemset(d->fetched, 0, sizeof(unsigned long long)) == cudaSuccess;
        for (unsigned l = 0; l < g.n_offload && okc; ++l) {
            moe_offload &o = d->L[l].off;
            o.gu_stage = static_cast<uint8_t *>(d->alloc(g.n_cache * gu_stride));
            o.dn_stage = static_cast<uint8_t *>(d->alloc(g.n_cache * dn_stride));
            o.slot_of = static_cast<int *>(d->alloc(sizeof(int) * g.n_expert));
            o.owner = static_cast<int *>(d->alloc(sizeof(int) * g.n_cache));
            o.stamp = static_cast<int *>(d->alloc(sizeof(int) * g.n_cache));
            o.plan = static_cast<int *>(d->alloc(sizeof(int) * (1 + 2 * 32)));
            o.fetched = d->fetched;
            o.clock = d->dpos;
            o.n_cache = (int)g.n_cache;
            okc = o.gu_stage && o.dn_stage && o.slot_of && o.owner && o.stamp && o.plan &&
                  cudaMemset(o.slot_of, 0xFF, sizeof(int) * g.n_expert) == cudaSuccess &&
                  cudaMemset(o.owner, 0xFF, sizeof(int) * g.n_cache) == cudaSuccess &&
                  cudaMemcpy(o.stamp, older.data(), sizeof(int) * g.n_cache, cudaMemcpyHostToDevice) == cudaSuccess;
        }
        if (!okc) {
            cudaGetLastError();
            cudaFree(staging);
            return fail();
        }
    }
    if (g.n_offload) {
        d->off.gu_stage = static_cast<uint8_t *>(d->alloc(g.n_expert_used * gu_stride));
        d->off.dn_stage = static_cast<uint8_t *>(d->alloc(g.n_expert_used * dn_stride));
        if (!d->off.gu_stage || !d->off.dn_stage || cudaMalloc(&pack_tmp, g.n_expert * (gu_stride + dn_stride)) != cudaSuccess) {
            cudaGetLastError();
            cudaFree(staging);
            return fail();
        }
    }
    const unsigned ekind = (g.expert_type == T_MXFP4) ? 2 : 3;
    const float esig = 0.01f;
    d->L.resize(g.n_layer);
    for (unsigned l = 0; l < g.n_layer && ok; ++l) {
        auto &b = d->L[l];
        const int window = is_swa(g, l) ? (int)g.n_swa : 0;
        b.window = window;
        b.table = window ? d->table_swa : d->table_full;
        b.pool_tokens = (size_t)(window ? swa_pages : pages) * PAGE_TOKENS;
        b.attn_norm = static_cast<float *>(d->alloc(sizeof(float) * H));
        b.ffn_norm = static_cast<float *>(d->alloc(sizeof(float) * H));
        b.sinks = g.has_sinks ? static_cast<float *>(d->alloc(sizeof(float) * g.n_head)) : nullptr;
        b.q_norm = g.has_qk_norm ? static_cast<float *>(d->alloc(sizeof(float) * g.head_dim)) : nullptr;
        b.k_norm = g.has_qk_norm ? static_cast<float *>(d->alloc(sizeof(float) * g.head_dim)) : nullptr;
        b.router = static_cast<float *>(d->alloc(sizeof(float) * g.n_expert * H));
        b.wqkv = d->alloc(qkv_elems * 2);
        b.wo = d->alloc(wo_elems * 2);
        const bool offl = l < g.n_offload;
        b.gu_host = b.dn_host = nullptr;
        if (offl) {
            b.gateup = static_cast<uint8_t *>(pack_tmp);
            b.down = static_cast<uint8_t *>(pack_tmp) + g.n_expert * gu_stride;
        } else if (d->tc) {
            b.gateup = d->alloc(moearc_x_moe_tc_bytes(&md, 0));
            b.down = d->alloc(moearc_x_moe_tc_bytes(&md, 1));
        } else {
            b.gateup = d->alloc(2 * bank_bytes);
            b.down = d->alloc(bank_bytes);
        }
        b.k_pages = static_cast<uint16_t *>(d->alloc(b.pool_tokens * d->Dkv * 2));
        b.v_pages = static_cast<uint16_t *>(d->alloc(b.pool_tokens * d->Dkv * 2));
        if (!b.attn_norm || !b.ffn_norm || (g.has_sinks && !b.sinks) || !b.router || !b.wqkv || !b.wo ||
            !b.gateup || !b.down || !b.k_pages || !b.v_pages) {
            ok = false;
            break;
        }
        ok &= synth(c, b.attn_norm, H, 4, tensor_seed(g.seed, 0, l), 0.1f) == OK;
        ok &= synth(c, b.ffn_norm, H, 4, tensor_seed(g.seed, 1, l), 0.1f) == OK;
        if (b.sinks) ok &= synth(c, b.sinks, g.n_head, 0, tensor_seed(g.seed, 6, l), 1.0f) == OK;
        if (g.has_qk_norm) {
            ok &= b.q_norm && b.k_norm;
            ok &= ok && synth(c, b.q_norm, g.head_dim, 4, tensor_seed(g.seed, 14, l), 0.1f) == OK;
            ok &= ok && synth(c, b.k_norm, g.head_dim, 4, tensor_seed(g.seed, 15, l), 0.1f) == OK;
        }
        ok &= synth(c, b.router, (size_t)g.n_expert * H, 0, tensor_seed(g.seed, 7, l), 0.02f) == OK;
        // Q, K, V rows concatenated into one [Dq + 2 Dkv] x H matrix
        uint16_t *s16 = static_cast<uint16_t *>(staging);
        ok &= synth(c, s16, (size_t)d->Dq * H, 1, tensor_seed(g.seed, 2, l), 0.02f) == OK;
        ok &= synth(c, s16 + (size_t)d->Dq * H, (size_t)d->Dkv * H, 1, tensor_seed(g.seed, 3, l), 0.02f) == OK;
        ok &= synth(c, s16 + (size_t)(d->Dq + d->Dkv) * H, (size_t)d->Dkv * H, 1, tensor_seed(g.seed, 4, l), 0.02f) == OK;
        ok &= dense_pack(c, b.wqkv, staging, d->n_qkv, H) == OK;
        ok &= synth(c, s16, wo_elems, 1, tensor_seed(g.seed, 5, l), 0.02f) == OK;
        ok &= dense_pack(c, b.wo, staging, H, d->Dq) == OK;
        uint8_t *s8 = static_cast<uint8_t *>(staging);
        ok &= synth(c, s8, blocks, ekind, tensor_seed(g.seed, 8, l), esig) == OK;
        ok &= synth(c, s8 + bank_bytes, blocks, ekind, tensor_seed(g.seed, 9, l), esig) == OK;
        ok &= synth(c, s8 + 2 * bank_bytes, blocks, ekind, tensor_seed(g.seed, 10, l), esig) == OK;
        if (d->tc && !offl)
            ok &= moearc_x_moe_pack_tc(d->moe, s8, s8 + bank_bytes, s8 + 2 * bank_bytes, g.n_expert, b.gateup, b.down) == OK;
        else
            ok &= moearc_x_moe_pack(d->moe, s8, s8 + bank_bytes, s8 + 2 * bank_bytes, g.n_expert, b.gateup, b.down) == OK;
        if (offl && ok) {
            const size_t gb = g.n_expert * gu_stride, db = g.n_expert * dn_stride;
            void *gdev = nullptr, *ddev = nullptr;
            if (cudaHostAlloc(&b.gu_host, gb, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) b.gu_host = nullptr;
            else d->host_allocs.push_back(b.gu_host);
            if (cudaHostAlloc(&b.dn_host, db, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) b.dn_host = nullptr;
            else d->host_allocs.push_back(b.dn_host);
            ok = b.gu_host && b.dn_host && cudaStreamSynchronize(c->stream) == cudaSuccess &&
                 cudaMemcpy(b.gu_host, b.gateup, gb, cudaMemcpyDeviceToHost) == cudaSuccess &&
                 cudaMemcpy(b.dn_host, b.down, db, cudaMemcpyDeviceToHost) == cudaSuccess &&
                 cudaHostGetDevicePointer(&gdev, b.gu_host, 0) == cudaSuccess &&
                 cudaHostGetDevicePointer(&ddev, b.dn_host, 0) == cudaSuccess;
            cudaGetLastError();
            b.gateup = gdev;
            b.down = ddev;
        }
        // an empty cache reads as zeros; fill_kv writes synthetic contents
        ok &= cudaMemsetAsync(b.k_pages, 0, b.pool_tokens * d->Dkv * 2, c->stream) == cudaSuccess;
        ok &= cudaMemsetAsync(b.v_pages, 0, b.pool_tokens * d->Dkv * 2, c->stream) == cudaSuccess;
    }
    if (g.n_vocab && ok) {
        ok &= synth(c, staging, (size_t)g.n_vocab * H, 1, tensor_seed(g.seed, 16, 0), 0.02f) == OK;
        ok &= dense_pack(c, d->w_out, staging, (int)g.n_vocab, H) == OK;
    }
    ok &= cudaStreamSynchronize(c->stream) == cudaSuccess;
    cudaFree(staging);
    if (pack_tmp) cudaFree(pack_tmp);
    if (!ok) return fail();
    if (!g.n_offload && !g.has_qk_norm && !d->tc) {
        std::vector<step_layer> sl(g.n_layer);
        for (unsigned l = 0; l < g.n_layer; ++l) {
            const auto &b = d->L[l];
            sl[l] = step_layer{b.attn_norm, b.ffn_norm, b.sinks, b.router,
                               static_cast<const uint8_t *>(b.wqkv), static_cast<const uint8_t *>(b.wo),
                               static_cast<const uint8_t *>(b.gateup), static_cast<const uint8_t *>(b.down),
                               b.k_pages, b.v_pages, b.table, b.window};
        }
        const step_shape ss{(int)g.n_layer, H, (int)g.n_head, (int)g.n_head_kv, (int)g.head_dim, (int)g.n_expert,
                            (int)g.n_expert_used, (int)g.n_ff, (int)g.gating, (int)g.act, (int)g.expert_type,
                            g.alpha, g.limit, g.rms_eps, d->rope_freq, d->rope_mscale};
        d->step = step_create(c, ss, sl.data());
        // the kernel chain is the default (measured faster at the gpt-oss-120b shape); the
        // persistent kernel on request
        const char *e = std::getenv("MOEARC_STEP_KERNEL");
        d->use_step = e && e[0] == '1';

    }
    return d;
}

void moearc_x_decoder_destroy(moearc_x_decoder *d) {
    if (!d) return;
    cudaStreamSynchronize(d->c->stream);
    d->drop_graph();
    step_destroy(d->step);
    if (d->spans) cudaFree(d->spans);
    d->stop_poller();
    if (d->mail) cudaFreeHost(d->mail);
    if (d->done) cudaFreeHost(d->done);
    host_pool_destroy(d->pool);
    if (d->moe) moearc_x_moe_destroy(d->moe);
    if (d->qkv) dense_destroy(d->qkv);
    if (d->wo) dense_destroy(d->wo);
    if (d->head) dense_destroy(d->head);
    for (void *p : d->allocs) cudaFree(p);
    for (void *p : d->host_allocs) cudaFreeHost(p);
    delete d;
}

void *moearc_x_decoder_input(moearc_x_decoder *d) { return d ? d->in : nullptr; }
void *moearc_x_decoder_output(moearc_x_decoder *d) { return d ? d->out : nullptr; }
void *moearc_x_decoder_logits(moearc_x_decoder *d) { return d ? d->logits : nullptr; }

int moearc_x_decoder_pos(moearc_x_decoder *d) { return d ? d->pos : -1; }

int moearc_x_decoder_set_pos(moearc_x_decoder *d, unsigned pos) {
    if (!d) return ERR;
    if (pos >= d->cfg.n_ctx) return ERR_ARG;
    k_set_pos<<<1, 1, 0, d->c->stream>>>(d->dpos, (int)pos);
    d->pos = (int)pos;
    return cudaGetLastError() == cudaSuccess ? OK : ERR;
}

// Synthetic K/V bf16 N(0, 0.02) in every page of every block, and the position set to depth:
// the state of a sequence that has already decoded `depth` tokens.
int moearc_x_decoder_fill_kv(moearc_x_decoder *d, unsigned depth, unsigned long long seed) {
    if (!d) return ERR;
    if (depth >= d->cfg.n_ctx) return ERR_ARG;
    for (unsigned l = 0; l < d->cfg.n_layer; ++l) {
        auto &b = d->L[l];
        const size_t n = b.pool_tokens * d->Dkv;
        if (synth(d->c, b.k_pages, n, 1, tensor_seed(seed, 12, l), 0.02f) != OK) return ERR;
        if (synth(d->c, b.v_pages, n, 1, tensor_seed(seed, 13, l), 0.02f) != OK) return ERR;
    }
    return moearc_x_decoder_set_pos(d, depth);
}

unsigned long long moearc_x_decoder_fetched(moearc_x_decoder *d) {
    if (!d || !d->fetched) return 0;
    unsigned long long n = 0;
    if (cudaMemcpyAsync(&n, d->fetched, sizeof(n), cudaMemcpyDeviceToHost, d->c->stream) != cudaSuccess ||
        cudaStreamSynchronize(d->c->stream) != cudaSuccess)
        return 0;
    return n;
}

int moearc_x_decoder_status(moearc_x_decoder *d) {
    if (!d) return ERR;
    const int sm = moearc_x_moe_status(d->moe), sq = dense_status(d->qkv), so = dense_status(d->wo);
    const int sd = d->head ? dense_status(d->head) : 0;
    if (sd < 0) return ERR;
    const int st = d->step ? step_status(d->step) : 0;
    if (sm < 0 || sq < 0 || so < 0 || st < 0) return ERR;
    // a host job the pool refused (the block's output was then NaN), or a fold that gave up
    // waiting for the host's answer
    int sh = d->host_failed.exchange(0) ? STATUS_RANGE : 0;
    if (d->hstatus) {
        int v = 0;
        if (cudaMemcpy(&v, d->hstatus, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess ||
            cudaMemset(d->hstatus, 0, sizeof(int)) != cudaSuccess)
            return ERR;
        sh |= v;
    }
    return sm | sq | so | st | sh | sd;
}

int moearc_x_decoder_host_experts(moearc_x_decoder *d, int kind, float fraction, unsigned over, int n_threads) {
    if (!d) return ERR;
    const auto &g = d->cfg;
    if (kind < 0 || kind > 2 || !g.n_offload || (kind == 1 && !(fraction >= 0.f))) return ERR_ARG;
    if (cudaStreamSynchronize(d->c->stream) != cudaSuccess) return ERR;
    d->drop_graph();
    if (kind == 0) {
        for (auto &h : d->hosts) h.kind = 0;
        return OK;
    }
    if (d->pool && n_threads > 0 && host_pool_threads(d->pool) != n_threads) {
        d->stop_poller();
        host_pool_destroy(d->pool);
        d->pool = nullptr;
    }
    if (n_threads <= 0 && !std::getenv("MOEARC_HOST_THREADS")) {
        // the online cores less two: one for the thread polling the mail (which works in every
        // job too) and one for the thread driving the device
        const long nc = sysconf(_SC_NPROCESSORS_ONLN);
        n_threads = nc > 3 ? (int)(nc - 2) : 1;
    }
    if (!d->pool && !(d->pool = host_pool_create(n_threads))) return ERR;
    if (!d->mail) {
        // one mailbox for every block: a block's job is answered before the next block posts
        const size_t mail_bytes = MAIL_X + sizeof(float) * g.n_embd, done_bytes = DONE_OUT + sizeof(float) * g.n_embd;
        void *m = nullptr, *dn = nullptr;
        if (cudaHostAlloc(&m, mail_bytes, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) m = nullptr;
        if (m && cudaHostAlloc(&dn, done_bytes, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) dn = nullptr;
        if (!m || !dn) {
            cudaGetLastError();
            if (m) cudaFreeHost(m);
            return ERR;
        }
        std::memset(m, 0, mail_bytes);
        std::memset(dn, 0, done_bytes);
        d->mail = static_cast<uint8_t *>(m);
        d->done = static_cast<uint8_t *>(dn);
        d->hmask = static_cast<unsigned *>(d->alloc(sizeof(unsigned) * g.n_offload));
        d->hseq = static_cast<unsigned long long *>(d->alloc(sizeof(unsigned long long)));
        d->hffn = static_cast<float *>(d->alloc(sizeof(float) * g.n_embd));
        d->hstatus = static_cast<int *>(d->alloc(sizeof(int)));
        void *mail_dev = nullptr, *done_dev = nullptr;
        if (!d->hmask || !d->hseq || !d->hffn || !d->hstatus ||
            cudaMemset(d->hmask, 0, sizeof(unsigned) * g.n_offload) != cudaSuccess ||
            cudaMemset(d->hseq, 0, sizeof(unsigned long long)) != cudaSuccess ||
            cudaMemset(d->hstatus, 0, sizeof(int)) != cudaSuccess ||
            cudaHostGetDevicePointer(&mail_dev, d->mail, 0) != cudaSuccess ||
            cudaHostGetDevicePointer(&done_dev, d->done, 0) != cudaSuccess) {
            cudaGetLastError();
            return ERR;
        }
        d->hosts.assign(g.n_offload, moe_host{});
        for (unsigned l = 0; l < g.n_offload; ++l) {
            moe_host &h = d->hosts[l];
            h.block = (int)l;
            h.hmask = d->hmask + l;
            h.seq = d->hseq;
            h.mail = static_cast<uint8_t *>(mail_dev);
            h.done = static_cast<const uint8_t *>(done_dev);
            h.ffn = d->hffn;
            h.wait_ns = 2000000000ull;
            h.status = d->hstatus;
        }
    }
    d->hshape = host_shape{(int)g.n_embd, (int)g.n_ff, (int)g.expert_type, (int)g.act, g.alpha, g.limit};
    for (auto &h : d->hosts) {
        h.kind = kind;
        h.frac = fraction;
        h.over = (int)std::min(over, 64u);
    }
    if (!d->poller.joinable()) {
        d->poll_stop.store(false);
        try {
            d->poller = std::thread([d] { d->poll_mail(); });
        } catch (...) {
            for (auto &h : d->hosts) h.kind = 0;
            return ERR;
        }
    }
    return OK;
}

int moearc_x_decoder_host_wait(moearc_x_decoder *d, unsigned long long limit_ns, int hold) {
    if (!d || d->hosts.empty()) return ERR;
    if (cudaStreamSynchronize(d->c->stream) != cudaSuccess) return ERR;
    for (auto &h : d->hosts) h.wait_ns = limit_ns ? limit_ns : 2000000000ull;
    d->poll_hold.store(hold != 0);
    d->drop_graph();
    return OK;
}

int moearc_x_decoder_host_stats(moearc_x_decoder *d, unsigned long long *out4) {
    if (!d || !out4) return ERR;
    if (cudaStreamSynchronize(d->c->stream) != cudaSuccess) return ERR;
    host_stats(d->pool, out4);
    return OK;
}

int moearc_x_decoder_uses_step_kernel(moearc_x_decoder *d) { return d && d->step && d->use_step ? 1 : 0; }

int moearc_x_decoder_has_step_kernel(moearc_x_decoder *d) { return d && d->step ? 1 : 0; }

int moearc_x_decoder_use_step_kernel(moearc_x_decoder *d, int on) {
    if (!d) return ERR;
    if (on && !d->step) return ERR_ARG;
    if (d->use_step != (on != 0)) d->drop_graph();
    d->use_step = on != 0;
    return OK;
}

int moearc_x_decoder_set_wait(moearc_x_decoder *d, unsigned long long limit_ns, unsigned int phantom) {
    if (!d) return ERR;
    if (cudaStreamSynchronize(d->c->stream) != cudaSuccess) return ERR;
    if (d->step) step_set_wait(d->step, limit_ns, phantom);
    moearc_x_moe_set_wait(d->moe, limit_ns, phantom ? 1 : 0);
    d->drop_graph();
    return OK;
}

unsigned long moearc_x_decoder_trace_words(moearc_x_decoder *d) {
    return d && d->step ? (unsigned long)step_trace_words(d->step) : 0;
}

int moearc_x_decoder_set_trace(moearc_x_decoder *d, void *device_buffer) {
    if (!d || !d->step) return ERR;
    if (cudaStreamSynchronize(d->c->stream) != cudaSuccess) return ERR;
    step_set_trace(d->step, static_cast<unsigned long long *>(device_buffer));
    d->drop_graph();
    return OK;
}

int moearc_x_decoder_kernel_spans(moearc_x_decoder *d, int on) {
    if (!d) return ERR;
    if (cudaStreamSynchronize(d->c->stream) != cudaSuccess) return ERR;
    if (on && !d->spans) {
        d->span_cta = moe_decode_grid(d->moe);
        if (!d->span_cta) return ERR_ARG;
        const size_t bytes = sizeof(unsigned long long) * d->cfg.n_layer * 2 * d->span_cta * 3;
        if (cudaMalloc(&d->spans, bytes) != cudaSuccess) {
            cudaGetLastError();
            d->spans = nullptr;
            return ERR;
        }
        if (cudaMemset(d->spans, 0, bytes) != cudaSuccess) return ERR;
    } else if (!on && d->spans) {
        cudaFree(d->spans);
        d->spans = nullptr;
    }
    d->drop_graph();
    return OK;
}

int moearc_x_decoder_use_graph(moearc_x_decoder *d, int on) {
    if (!d) return ERR;
    d->use_graph = on != 0;
    return OK;
}

int moearc_x_decoder_step(moearc_x_decoder *d) {
    if (!d) return ERR;
    if ((unsigned)d->pos >= d->cfg.n_ctx) return ERR_ARG;
    moearc_ctx *c = d->c;
    int rc = OK;
    if (!d->use_graph) {
        rc = enqueue_step(d);
    } else {
        if (!d->exec) {
            if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return ERR;
            rc = enqueue_step(d);
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
        rc = cudaGraphLaunch(d->exec, c->stream) == cudaSuccess ? OK : ERR;
    }
    if (rc == OK) d->pos += 1;
    return rc;
}

// One step from host memory to host memory in one call (the reference's decode loop hands the
// engine a host embedding row and reads host results back, moe.rs:1862-1870, 2429-2442): the
// row goes to pinned staging, then one graph launch runs the host -> device copy, the step and
// the device -> host copy of the output, and the call waits for it. Replacing three enqueues
// and a wait by one launch and a wait keeps the GPU's idle time between synchronous steps to
// the launch latency of one graph.
// Copies one row between pinned host memory (read or written by the kernel over PCIe through its
// device mapping) and device memory; a kernel node beside the step's kernels in place of a copy
// engine node, whose hand-over to and from the compute engine costs more than the row's PCIe time.
__global__ void k_row_copy(float4 *__restrict__ dst, const float4 *__restrict__ src, int n4) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) dst[i] = src[i];
}

int moearc_x_decoder_step_host(moearc_x_decoder *d, const float *x, float *y) {
    if (!d || !x || !y) return ERR;
    if ((unsigned)d->pos >= d->cfg.n_ctx) return ERR_ARG;
    moearc_ctx *c = d->c;
    const size_t bytes = sizeof(float) * d->cfg.n_embd;
    if (!d->pin_in) {
        void *pi = nullptr, *po = nullptr;
        if (cudaMallocHost(&pi, bytes) != cudaSuccess || cudaMallocHost(&po, bytes) != cudaSuccess) {
            cudaGetLastError();
            if (pi) cudaFreeHost(pi);
            return ERR;
        }
        d->host_allocs.push_back(pi);
        d->host_allocs.push_back(po);
        d->pin_in = static_cast<float *>(pi);
        d->pin_out = static_cast<float *>(po);
        void *di = nullptr, *dout = nullptr;
        if (cudaHostGetDevicePointer(&di, pi, 0) != cudaSuccess || cudaHostGetDevicePointer(&dout, po, 0) != cudaSuccess) {
            cudaGetLastError();
            d->pin_in = d->pin_out = nullptr;
            return ERR;
        }
        d->pin_in_dev = static_cast<float *>(di);
        d->pin_out_dev = static_cast<float *>(dout);
    }
    // the previous call waited for its graph, so the staging rows are free
    std::memcpy(d->pin_in, x, bytes);
    // rows of whole float4s (n_embd is a multiple of 64) copied by kernels; a copy engine otherwise
    const bool rows4 = d->cfg.n_embd % 4 == 0;
    const int n4 = (int)(d->cfg.n_embd / 4);
    const unsigned nb = (unsigned)((n4 + 255) / 256);
    auto enqueue = [&]() -> int {
        if (rows4) {
            k_row_copy<<<nb, 256, 0, c->stream>>>(reinterpret_cast<float4 *>(d->in),
                                                   reinterpret_cast<const float4 *>(d->pin_in_dev), n4);
            if (cudaPeekAtLastError() != cudaSuccess) return ERR;
        } else if (cudaMemcpyAsync(d->in, d->pin_in, bytes, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) {
            return ERR;
        }
        const int r = enqueue_step(d);
        if (r) return r;
        if (rows4) {
            k_row_copy<<<nb, 256, 0, c->stream>>>(reinterpret_cast<float4 *>(d->pin_out_dev),
                                                   reinterpret_cast<const float4 *>(d->out), n4);
            return cudaPeekAtLastError() == cudaSuccess ? OK : ERR;
        }
        return cudaMemcpyAsync(d->pin_out, d->out, bytes, cudaMemcpyDeviceToHost, c->stream) == cudaSuccess ? OK : ERR;
    };
    int rc = OK;
    if (!d->use_graph) {
        rc = enqueue();
    } else {
        if (!d->exec_io) {
            if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return ERR;
            rc = enqueue();
            cudaGraph_t g = nullptr;
            const cudaError_t e = cudaStreamEndCapture(c->stream, &g);
            if (rc || e != cudaSuccess) {
                if (g) cudaGraphDestroy(g);
                cudaGetLastError();
                return rc ? rc : ERR;
            }
            d->graph_io = g;
            if (cudaGraphInstantiate(&d->exec_io, g, 0) != cudaSuccess) {
                cudaGetLastError();
                return ERR;
            }
        }
        rc = cudaGraphLaunch(d->exec_io, c->stream) == cudaSuccess ? OK : ERR;
    }
    if (rc == OK) d->pos += 1;
    if (cudaStreamSynchronize(c->stream) != cudaSuccess) return ERR;
    if (rc == OK) std::memcpy(y, d->pin_out, bytes);
    return rc;
}

// One step, not graphed, with an event after every kernel; ms[k] receives the total device
// time of kernel kind k (0 qkv, 1 attention, 2 o-proj, 3 MoE route, 4 MoE gate-up, 5 MoE down,
// 6 final norm, 7 expert fetch) and counts[k] how many launches of that kind ran (kinds >= n
// are left out).
int moearc_x_decoder_profile(moearc_x_decoder *d, float *ms, int *counts, int n) {
    if (!d || !ms || n < 7) return ERR;
    if ((unsigned)d->pos >= d->cfg.n_ctx) return ERR_ARG;
    step_marks pm;
    int rc = enqueue_step(d, &pm);
    if (cudaStreamSynchronize(d->c->stream) != cudaSuccess) rc = ERR;
    for (int k = 0; k < n; ++k) {
        ms[k] = 0.f;
        if (counts) counts[k] = 0;
    }
    for (size_t i = 1; i < pm.ev.size(); ++i) {
        float t = 0.f;
        cudaEventElapsedTime(&t, pm.ev[i - 1], pm.ev[i]);
        const int k = pm.kind[i];
        if (k >= 0 && k < n) {
            ms[k] += t;
            if (counts) counts[k] += 1;
        }
    }
    for (auto e : pm.ev) cudaEventDestroy(e);
    if (rc == OK) d->pos += 1;
    return rc;
}

// Device pointers of one block's tensors, for inspection: 0 attn_norm, 1 ffn_norm, 2 sinks,
// 3 router, 4 K pool, 5 V pool, 6 page table, 7 packed Q/K/V, 8 packed O, 9 packed gate-up,
// 10 packed down; 11 output norm (layer ignored); 12/13 the step kernel's expert ids and gating
// weights of the last step; 14 the chain's expert-kernel spans of the last step (u64
// [2 kernels][CTA][start, wait over, end] in ns, while kernel spans are on); 15/16 the QK-norm
// weights; 17 the packed output head (layer ignored). `bytes` receives the size.
void *moearc_x_decoder_tensor(moearc_x_decoder *d, int which, unsigned layer, unsigned long *bytes) {
    if (!d || (which != 11 && which != 17 && layer >= d->cfg.n_layer)) return nullptr;
    const auto &g = d->cfg;
    const size_t H = g.n_embd;
    const size_t bb = (g.expert_type == T_MXFP4) ? 17 : 18;
    const size_t bank = (size_t)g.n_expert * g.n_ff * g.n_embd / 32 * bb;
    unsigned long n = 0;
    void *p = nullptr;
    if (which == 11) {
        p = d->output_norm;
        n = H * 4;
    } else if (which == 17) {
        p = d->w_out;
        n = p ? (unsigned long)g.n_vocab * H * 2 : 0;
    } else {
        auto &b = d->L[layer];
        switch (which) {
        case 0: p = b.attn_norm; n = H * 4; break;
        case 1: p = b.ffn_norm; n = H * 4; break;
        case 2: p = b.sinks; n = b.sinks ? g.n_head * 4 : 0; break;
        case 3: p = b.router; n = (unsigned long)g.n_expert * H * 4; break;
        case 4: p = b.k_pages; n = b.pool_tokens * d->Dkv * 2; break;
        case 5: p = b.v_pages; n = b.pool_tokens * d->Dkv * 2; break;
        case 6: p = (void *)b.table; n = (g.n_ctx + PAGE_TOKENS - 1) / PAGE_TOKENS * 4; break;
        case 7: p = b.wqkv; n = (unsigned long)d->n_qkv * H * 2; break;
        case 8: p = b.wo; n = H * d->Dq * 2; break;
        case 9:
        case 10: {
            // the tc layout for resident blocks of a tc decoder, else the fragment layout
            const bool tcl = d->tc && layer >= g.n_offload;
            moearc_x_moe_desc md{g.n_embd, g.n_ff, g.n_expert, g.n_expert_used, g.gating, g.act, g.alpha, g.limit,
                                 g.expert_type, 1};
            p = which == 9 ? b.gateup : b.down;
            n = tcl ? moearc_x_moe_tc_bytes(&md, which - 9) : (which == 9 ? 2 * bank : bank);
            break;
        }
        case 12: p = d->step ? static_cast<unsigned *>(step_buffer(d->step, 0)) + (size_t)layer * g.n_expert_used : nullptr;
                 n = p ? g.n_expert_used * 4 : 0; break;
        case 13: p = d->step ? static_cast<float *>(step_buffer(d->step, 1)) + (size_t)layer * g.n_expert_used : nullptr;
                 n = p ? g.n_expert_used * 4 : 0; break;
        case 14: p = d->spans ? d->spans + (size_t)layer * 2 * d->span_cta * 3 : nullptr;
                 n = p ? (unsigned long)2 * d->span_cta * 3 * 8 : 0; break;
        case 15: p = b.q_norm; n = p ? g.head_dim * 4 : 0; break;
        case 16: p = b.k_norm; n = p ? g.head_dim * 4 : 0; break;
        default: return nullptr;
        }
    }
    if (bytes) *bytes = n;
    return p;
}

// The seed the decoder generated tensor `kind` of block `layer` from (kinds: 0 attn_norm,
// 1 ffn_norm, 2 wq, 3 wk, 4 wv, 5 wo, 6 sinks, 7 router, 8 gate, 9 up, 10 down,
// 11 output_norm, 12/13 K/V fill, 14/15 QK-norm q/k, 16 output head), so a checker can
// regenerate the GGUF-layout tensors.
unsigned long long moearc_x_decoder_seed(moearc_x_decoder *d, int kind, unsigned layer, unsigned long long base) {
    (void)d;
    return tensor_seed(base, kind, (int)layer);
}

}  // extern "C"
