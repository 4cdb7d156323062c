// step.cuh — the whole batch-1 decode step of the synthetic decoder as one persistent kernel.
//
// The chained decode step launches seven kernels per block (Q/K/V, attention, O, router,
// gate-up, down, and the final norm once). Each launch pays a fixed chain — start, wait for its
// predecessor, read its inputs, reduce its outputs — of several microseconds, which at batch 1
// costs more than the block's weight bytes take to stream (moe.rs:1862-2443 is the sequence both
// follow). Here one cooperative launch runs every block: one CTA of 16 warps per SM, the
// phases of a block separated by grid barriers, and every warp streaming its share of each
// phase's weights through its own ring of bulk copies. The ring runs ahead across phase and block
// boundaries — a warp issues the next phase's weights as soon as a stage is free and their
// addresses are known (the dense weights always, an expert's once the block's routing is) — so
// the weights of the phase after a barrier are already in shared memory when the barrier opens.
//
// Phases of block l (all CTAs; "barrier" = grid barrier):
//   QKV   residual h (the previous block's combine, summed by every CTA), RMSNorm, the CTA's
//         share of the Q/K/V tiles; per-CTA partial sums per tile-row to global memory; barrier
//   ATT   CTA u < n_kv_heads x n_splits takes key split u: its warps 0-3 sum the head's q/k/v
//         partials, apply RoPE, the last split writes the step's K/V into the paged cache, then
//         split-K flash decode on the tensor cores; the last split of a head merges; barrier
//   O     the CTA's share of the O tiles (warps 4-15) against the attention output; barrier
//   ROUTE every CTA forms h + O and its RMSNorm (the MoE input) itself; router rows, one per
//         CTA, sliced over its warps; barrier
//   GU    every CTA takes the top-k of the logits (the routing is then known: expert weights
//         may stream), whole (expert, tile-row) segments of gate and up per CTA, SwiGLU on the
//         CTA's own sums, the activation's tensor-core fragments to global memory; barrier
//   DN    whole (expert, tile-row) segments of down per CTA, the activation fragments copied
//         into each stage beside its weights; unweighted expert outputs to global memory; barrier
// The router-order combine (sum over m of w_m o_m, an fmaf chain, plus the residual) is done by
// the next block's QKV phase (or the final norm) in every CTA.
//
// Every sum has a fixed order (warps in index order inside a CTA, CTAs in index order across),
// so a step is deterministic. Every wait is bounded: a grid barrier gives up after the launch's
// limit, raises STATUS_WAIT_TIMEOUT and an abort word that makes every later barrier return at
// once; bulk-copy waits are bounded as everywhere else; a CTA drains its copies before it exits.
#pragma once

#include "common.cuh"

namespace moearc {

// One block's tensors as the step kernel reads them (device pointers).
struct step_layer {
    const float *attn_norm, *ffn_norm, *sinks, *router;
    const uint8_t *wqkv, *wo;       // packed bf16 tiles (dense.cuh)
    const uint8_t *gateup, *down;   // packed expert banks (moearc_x_moe_pack)
    uint16_t *k_pages, *v_pages;    // bf16 [page][slot][kv_head][head_dim]
    const unsigned *table;          // logical page -> physical page
    int window;                     // keys a windowed block attends to, 0 = all
};

struct step_shape {
    int n_layer, H, n_head, n_kv, head_dim, E, K, I, gating, act, wtype;
    float alpha, limit, eps;
    const double *rope_freq;  // head_dim / 2 angle multipliers (device)
    double mscale;
};

struct step_plan;

// The plan for `grid` CTAs (one per SM), or null when the shape is outside what the step kernel
// serves (head_dim 64, experts resident, every phase's per-warp share within its limits) or
// memory runs out. `layers` is copied to the device.
step_plan *step_create(moearc_ctx *c, const step_shape &s, const step_layer *layers);
void step_destroy(step_plan *p);
// Enqueue one step on the context stream: h0 = in, out = RMSNorm(h) * out_norm, *pos += 1.
int step_run(step_plan *p, const float *in, float *out, const float *out_norm, int *pos);
// Reads and clears the status word (0, or STATUS_WAIT_TIMEOUT when a wait gave up).
int step_status(step_plan *p);
// The next step's barrier limit (ns) and a count of phantom arrivals its first barrier waits
// for in addition to the CTAs' (0 in normal use: a test makes the barrier run out with 1).
void step_set_wait(step_plan *p, unsigned long long limit_ns, unsigned phantom);
// Per-phase timestamps of the following steps: (layer, phase 0-5, point 0-3, CTA) in ns of
// %globaltimer into a device buffer of step_trace_words() u64 (null: off).
size_t step_trace_words(step_plan *p);
void step_set_trace(step_plan *p, unsigned long long *buf);
// Device pointers: 0 the expert ids [n_layer][K] (u32) and 1 their gating weights [n_layer][K]
// of the last step.
void *step_buffer(step_plan *p, int which);

}  // namespace moearc
