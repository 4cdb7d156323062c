// host_experts.hpp — expert FFNs computed on the host cores, beside the GPU.
//
// The reference sends part of an offloaded block's routed experts to a CPU worker pool while the
// device streams the rest (crates/moearc-engine/src/host_experts.rs:624-761 submit/sync,
// moe.rs:2169-2211 the split, 2389-2420 the fold). Here the pool reads the same packed banks the
// GPU fetches from (moearc_x_moe_pack layout, in pinned host memory), so an offloaded block keeps
// one copy of its experts: 16-row tile-rows are the unit of work, decoded from the tensor-core
// fragment order with AVX2 where the CPU has it.
#pragma once

#include <cstddef>
#include <cstdint>

namespace moearc {

struct host_shape {
    int H, I;        // n_embd, n_ff (multiples of 64)
    int wtype;       // 39 MXFP4 or 2 Q4_0
    int act;         // 0 SwiGLU, 1 SwiGLU-OAI(alpha, limit)
    float alpha, limit;
};

struct host_pool;

// A pool of worker threads (n_threads <= 0: MOEARC_HOST_THREADS, else the online cores - 1).
host_pool *host_pool_create(int n_threads);
void host_pool_destroy(host_pool *p);
int host_pool_threads(const host_pool *p);

// Publish one job and return without waiting: out = sum over i (in order) of weights[i] *
// down_e . act(gate_e . x, up_e . x), e = ids[i], n <= 32. gu and dn are the whole packed banks
// (expert e at e * the packed bytes per expert). The pool copies ids, weights and x; the banks
// must stay valid until host_sync returns. 0, or a negative moearc status (a job pending: sync
// it first).
int host_submit(host_pool *p, const host_shape &s, const uint8_t *gu, const uint8_t *dn, const unsigned *ids,
                const float *weights, unsigned n, const float *x);
// Work on the pending job beside the pool until it is done, then write its sum into out (H
// floats; zeros for a job of no experts).
int host_sync(host_pool *p, float *out);
// jobs, experts, busy ns (the pool's threads inside jobs), wait ns (sync waiting for others)
void host_stats(const host_pool *p, unsigned long long out[4]);
void host_reset_stats(host_pool *p);

// Bytes of one expert's packed gate-up (which 0) or down (which 1) bank; 0 on a bad shape.
size_t host_packed_bytes(const host_shape &s, int which);

}  // namespace moearc
