/*
 * moearc.h — the C ABI of libmoearc_b200.so, a B200 (sm_100a) implementation of MoEArc's
 * mixture-of-experts decode hot path.
 *
 * The first half is the reference's own operator ABI, symbol for symbol: every function
 * declared in crates/moearc-kernels/src/ffi.rs:19-263 (defined in kernels.cpp:734-1922) with
 * the same name, the same argument meaning and the same return codes, so the reference's Rust
 * crate links against this library unchanged. Each declaration cites the ffi.rs lines it
 * replaces. The second half (moearc_x_*) holds extensions the reference does not have.
 *
 * Return codes (ffi.rs:8-10): 0 success; -1 a device failure or a null argument; -2 an
 * argument out of range (unsupported type, a shape that is not whole blocks, k or n_mat above
 * 32, an empty key span, n_heads not a multiple of n_kv_heads, head_dim above 1024).
 *
 * Ordering (kernels.cpp:804-828): every context owns one in-order CUDA stream. Kernels return
 * 0 for "accepted", not "completed"; a device fault surfaces at moearc_sync or at the next
 * device-to-host copy. `unsigned long` is 64 bits (LP64), as in the reference's c_ulong.
 *
 * Type ids are GGUF's (reference.rs:21-40): F32 0, F16 1, Q4_0 2, Q8_0 8, Q4_K 12, Q5_K 13,
 * Q6_K 14, BF16 30, MXFP4 39. Every one expands (dequant, embed_rows) and multiplies
 * (matvec_q, matvec_q_batched): the reference's seven plus Q4_0 and BF16. The fused MoE paths
 * take MXFP4 and Q4_0 experts. KV caches may be F32, F16 or BF16.
 */
#ifndef MOEARC_H
#define MOEARC_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct moearc_ctx moearc_ctx; /* ffi.rs:14-17 MoearcCtx, opaque */

/* ---- lifecycle, profiling, memory (ffi.rs:20-66) --------------------------------------- */
moearc_ctx *moearc_ctx_create(void);                                        /* ffi.rs:20 */
void moearc_ctx_destroy(moearc_ctx *c);                                     /* ffi.rs:21 */
int moearc_profile_events_enabled(moearc_ctx *c);                           /* ffi.rs:22 */
int moearc_profile_events_reset(moearc_ctx *c);                             /* ffi.rs:23 */
int moearc_profile_events_report(moearc_ctx *c, char *out, unsigned long cap); /* ffi.rs:24-28 */
int moearc_sync(moearc_ctx *c);                                             /* ffi.rs:29 */
int moearc_zero(moearc_ctx *c, float *dst, unsigned long n);                /* ffi.rs:30 */
int moearc_device_name(moearc_ctx *c, char *out, unsigned long cap);        /* ffi.rs:31 */
void *moearc_alloc_device(moearc_ctx *c, unsigned long bytes);              /* ffi.rs:32 */
void moearc_free_device(moearc_ctx *c, void *p);                            /* ffi.rs:33 */
int moearc_copy_h2d(moearc_ctx *c, void *dst, const void *src, unsigned long bytes);       /* :34-39 */
int moearc_copy_h2d_async(moearc_ctx *c, void *dst, const void *src, unsigned long bytes); /* :40-45 */
int moearc_copy_d2h(moearc_ctx *c, void *dst, const void *src, unsigned long bytes);       /* :46-51 */
/* ffi.rs:52-59: dst[i] = pool[idx[i]] for count slots of slot_bytes; idx is a HOST array. */
int moearc_gather_experts(moearc_ctx *c, void *dst, const void *pool, const unsigned int *idx,
                          unsigned int count, unsigned long slot_bytes);

/* ---- dequantisation and matvecs (ffi.rs:61-117) ---------------------------------------- */
/* ffi.rs:61-67: nblocks blocks of type_id -> nblocks*block_elems floats. */
int moearc_dequant(moearc_ctx *c, unsigned int type_id, float *dst, const void *src,
                   unsigned long nblocks);
/* ffi.rs:68-76: out[r] = sum_c W[r,c] x[c], W rows in GGUF block layout. */
int moearc_matvec_q(moearc_ctx *c, unsigned int type_id, float *out, const void *w,
                    const float *x, unsigned long n_rows, unsigned long n_cols);
/* ffi.rs:77-88: n_mat <= 32 matrices of one shape; matrix m writes out[m*n_rows ...] and
 * reads x + m*x_stride (x_stride 0 shares one x). w is a HOST array of device pointers,
 * copied into the launch by value. */
int moearc_matvec_q_batched(moearc_ctx *c, unsigned int type_id, float *out,
                            const void *const *w, unsigned int n_mat, const float *x,
                            unsigned long x_stride, unsigned long n_rows, unsigned long n_cols);
/* ffi.rs:89-96: out[i] = sum over m ascending of weights[m]*parts[m*n+i] (weights on device). */
int moearc_moe_combine(moearc_ctx *c, float *out, const float *parts, const float *weights,
                       unsigned int n_mat, unsigned long n);
/* ffi.rs:97-104: f32 rows. Fixed order: lane l of a warp folds columns 4l+128i..+3 with fma,
 * then an xor butterfly 16,8,4,2,1 — reproducible bit for bit on the host. */
int moearc_matvec_f32(moearc_ctx *c, float *out, const float *w, const float *x,
                      unsigned long n_rows, unsigned long n_cols);

/* ---- normalisation and activations (ffi.rs:105-181) ------------------------------------ */
int moearc_rmsnorm(moearc_ctx *c, float *out, const float *x, const float *weight,
                   unsigned long n_rows, unsigned long n_cols, float eps);  /* ffi.rs:105-113 */
int moearc_silu(moearc_ctx *c, float *out, const float *x, unsigned long n); /* ffi.rs:114-119 */
int moearc_swiglu(moearc_ctx *c, float *out, const float *gate, const float *up,
                  unsigned long n);                                          /* ffi.rs:120-126 */
int moearc_swiglu_halves(moearc_ctx *c, float *out, const float *gu, unsigned long n); /* :127-132 */
int moearc_swiglu_oai(moearc_ctx *c, float *out, const float *gate, const float *up,
                      unsigned long n, float alpha, float limit);            /* ffi.rs:133-141 */
int moearc_swiglu_oai_halves(moearc_ctx *c, float *out, const float *gu, unsigned long n,
                             float alpha, float limit);                      /* ffi.rs:142-149 */
/* ffi.rs:150-157: out[m*n_rows+r] += bias[idx[m]*n_rows+r]; idx is a HOST array (<= 32). */
int moearc_add_bias_id(moearc_ctx *c, float *out, const float *bias, const unsigned int *idx,
                       unsigned int n_mat, unsigned long n_rows);
int moearc_softmax(moearc_ctx *c, float *out, const float *x, const float *mask,
                   unsigned long n_rows, unsigned long n_cols, float scale); /* ffi.rs:158-166 */
int moearc_add(moearc_ctx *c, float *out, const float *a, const float *b, unsigned long n); /* :167-173 */
int moearc_mul(moearc_ctx *c, float *out, const float *a, const float *b, unsigned long n); /* :174-180 */
int moearc_axpy(moearc_ctx *c, float *out, const float *x, float alpha, unsigned long n);   /* :181-187 */
int moearc_quantize_f16(moearc_ctx *c, void *dst, const float *src, unsigned long n);      /* :188-193 */
/* ffi.rs:194-202: gather + dequantise n_tokens rows; token_ids on the device. */
int moearc_embed_rows(moearc_ctx *c, unsigned int type_id, float *out, const void *table,
                      const unsigned int *token_ids, unsigned long n_tokens,
                      unsigned long n_embd);

/* ---- paged KV cache and decode attention (ffi.rs:203-238) ------------------------------ */
/* ffi.rs:203-216: write one token's K and V at (page_id, slot); layout
 * [page][slot][kv_head][head_dim]; kv_type F32, F16 or BF16 (30, an extension). */
int moearc_kv_append(moearc_ctx *c, void *k_pages, void *v_pages, const float *k,
                     const float *v, unsigned int page_id, unsigned int slot,
                     unsigned long n_kv_heads, unsigned long head_dim, unsigned long page_tokens,
                     unsigned int kv_type);
/* ffi.rs:217-238: single-query attention over logical keys [kv_begin, n_kv) through
 * block_table (device), GQA, optional per-head sinks (device, may be NULL). Split-K over the
 * span; bf16/f16 caches with group <= 8 and head_dim 64/128 run on tensor cores. */
int moearc_attn_decode(moearc_ctx *c, float *out, const float *q, const void *k_pages,
                       const void *v_pages, const unsigned int *block_table, const float *sinks,
                       unsigned long n_heads, unsigned long n_kv_heads, unsigned long head_dim,
                       unsigned long kv_begin, unsigned long n_kv, unsigned long page_tokens,
                       float scale, unsigned int kv_type);
/* ffi.rs:239-254: RoPE over [n_tokens][n_heads][head_dim] with the YaRN ramp; pos on the
 * device; neox selects (i, i+n_dims/2) pairs. */
int moearc_rope(moearc_ctx *c, float *dst, const float *src, const int *pos,
                unsigned long n_tokens, unsigned long n_heads, unsigned long head_dim,
                unsigned long n_dims, float freq_base, float freq_scale, float ext_factor,
                float attn_factor, float corr_lo, float corr_hi, int neox);
/* ffi.rs:255-264: k rounds of argmax over logits (lower id wins a tie); gating 0 softmax,
 * 1 softmax renormalised over k (sum clamped to 2^-14), 2 softmax of the k selected. */
int moearc_topk_router(moearc_ctx *c, unsigned int *idx, float *weights, const float *logits,
                       unsigned long n_tokens, unsigned long n_expert, unsigned int k,
                       unsigned int gating);

/* ======================================================================================= */
/* Extensions (no counterpart in ffi.rs)                                                    */
/* ======================================================================================= */

/* The context's compute stream (a cudaStream_t), for callers that order their own work. */
void *moearc_x_stream(moearc_ctx *c);
/* Device timing on the context's stream: start records an event, stop records a second one,
 * waits for it and writes the elapsed milliseconds. */
int moearc_x_timer_start(moearc_ctx *c);
int moearc_x_timer_stop(moearc_ctx *c, float *ms);
/* Page-locked host memory (for full-rate, overlappable copies) and its release. */
void *moearc_x_host_alloc(unsigned long bytes);
void moearc_x_host_free(void *p);
/* Device-to-host copy enqueued on the context's stream without waiting. */
int moearc_x_copy_d2h_async(moearc_ctx *c, void *dst, const void *src, unsigned long bytes);
/* Number of streaming multiprocessors of the context's device. */
int moearc_x_sm_count(moearc_ctx *c);
/* f32 -> bf16, round to nearest even. */
int moearc_x_quantize_bf16(moearc_ctx *c, void *dst, const float *src, unsigned long n);
/* Fill dst with n deterministic synthetic values (SplitMix64 stream `seed`, counter-based):
 * kind 0 = normal(0, sigma) as f32, 1 = normal(0, sigma) as bf16, 2 = MXFP4 blocks (n blocks,
 * e8m0 exponent uniform in [lo, hi]), 3 = Q4_0 blocks (n blocks, |normal(0, sigma)| scales),
 * 4 = 1 + normal(0, sigma) as f32 (norm weights). */
int moearc_x_synth(moearc_ctx *c, void *dst, unsigned long n, unsigned int kind,
                   unsigned long long seed, float sigma, int lo, int hi);

/* ---- fused MoE decode (moe.cu) ----------------------------------------------------------- */
/* The MoE block of crates/moearc-engine/src/moe.rs:2074-2427 (router -> top-k -> gate/up ->
 * activation -> down -> weighted combine -> residual) as three kernels with no host readback:
 * the router's choice stays on the device. Replaces the host-driven sequence moe.rs issues
 * through moearc_matvec_f32, moearc_topk_router, moearc_matvec_q_batched (x2),
 * moearc_swiglu*_halves and moearc_moe_combine. Expert banks are first repacked
 * (moearc_x_moe_pack) into tensor-core fragment order; bytes per block are unchanged. */
typedef struct moearc_x_moe moearc_x_moe;
typedef struct {
    unsigned int n_embd;     /* H, a multiple of 64 */
    unsigned int n_ff;       /* I, expert intermediate, a multiple of 64 */
    unsigned int n_expert;   /* E <= 1024 */
    unsigned int k;          /* experts per token <= 32 */
    unsigned int gating;     /* 0 softmax, 1 softmax renormalised, 2 softmax after top-k */
    unsigned int act;        /* 0 SwiGLU, 1 SwiGLU-OAI(alpha, limit) */
    float alpha, limit;
    unsigned int wtype;      /* 39 MXFP4 or 2 Q4_0 */
    unsigned int max_tokens; /* tokens per forward call */
} moearc_x_moe_desc;
/* NULL on an unsupported shape or a failed allocation. */
moearc_x_moe *moearc_x_moe_create(moearc_ctx *c, const moearc_x_moe_desc *d);
void moearc_x_moe_destroy(moearc_x_moe *m);
/* Bytes of one expert's packed gate-up (which = 0) or down (which = 1) bank. */
unsigned long moearc_x_moe_packed_bytes(const moearc_x_moe_desc *d, int which);
/* Repack n_expert experts from GGUF layout (gate/up: n_expert x [n_ff x n_embd], down:
 * n_expert x [n_embd x n_ff], each expert contiguous, device memory) into the two packed banks
 * (16-byte aligned device memory). */
int moearc_x_moe_pack(moearc_x_moe *m, const void *gate, const void *up, const void *down,
                      unsigned int n_expert, void *gateup_packed, void *down_packed);
/* out[t] = residual[t] (if not NULL) + MoE(x[t]) for t < n_tokens; x, router_w (E x H f32),
 * router_b (E, may be NULL), residual and out are device pointers; x and router_w 16-byte
 * aligned. The router GEMV folds in the fixed order of moearc_matvec_f32. */
int moearc_x_moe_forward(moearc_x_moe *m, const float *x, unsigned int n_tokens,
                         const float *router_w, const float *router_b, const void *gateup_packed,
                         const void *down_packed, const float *residual, float *out);
/* Device pointers to the last call's internals: 0 expert ids [T x k] (u32), 1 router weights
 * [T x k], 2 activations [column x n_ff] (column order: experts ascending, tokens ascending
 * within an expert), 3 router logits [T x E], 4 the int slot tables. */
void *moearc_x_moe_buffer(moearc_x_moe *m, int which);
/* Reads and clears the device status word: 0, or bit 1 = a bounded wait gave up. */
int moearc_x_moe_status(moearc_x_moe *m);
/* Per-expert biases for the following forward calls (moe.rs:2310-2331, 2362-2372, gpt-oss):
 * gate_up_bias f32 [2 n_expert][n_ff] (expert e's gate bias at row e, its up bias at row
 * n_expert + e), added after the expert matvecs and before the activation; down_bias f32
 * [n_expert][n_embd], added to each expert's output inside the router weighting. Device
 * pointers (NULL: none), kept until the next call; moearc_add_bias_id's semantics fused into the
 * decode kernels. */
int moearc_x_moe_set_bias(moearc_x_moe *m, const float *gate_up_bias, const float *down_bias);
/* The decode-path expert kernels' wait for one another's partial sums (ns; 0 = the default
 * 0.2 s); phantom 1 makes every such wait run out (testing the bounded wait). No reference
 * counterpart. */
int moearc_x_moe_set_wait(moearc_x_moe *m, unsigned long long poll_ns, int phantom);
/* ---- one token on the block-scaled FP4 tensor cores (xtc.cu; no reference counterpart) ----
 * MXFP4 experts in the tensor-core ("tc") layout: per expert, the gate-up bank in tiles of 64
 * gate rows and the 64 up rows of the same features, the down bank in tiles of 128 output rows,
 * each tile in k-steps of 64 elements (E2M1 codes two per byte, 32-byte swizzle) with their E8M0
 * scales laid out for tcgen05.cp; tcgen05.mma kind::mxf4.block_scale.block32 reads them as stored.
 * The activation enters as 16 E2M1 digits per element (each digit an exact part of the value;
 * together within 2e-8 of each 32-element block's largest magnitude), so the result keeps the f32
 * check-mode bound of the fragment path. Same semantics, biases and status as moearc_x_moe_forward.
 * Bytes of the whole tc-layout gate-up (which = 0) or down (1) bank of d->n_expert experts; 0
 * when the shape has none (MXFP4, n_embd and n_ff multiples of 64). */
unsigned long moearc_x_moe_tc_bytes(const moearc_x_moe_desc *d, int which);
/* 1 when the layer can run the tc path (k <= 8 and the shape above), else 0. */
int moearc_x_moe_has_tc(moearc_x_moe *m);
/* Repack GGUF-layout MXFP4 banks (as moearc_x_moe_pack) into the tc layout. */
int moearc_x_moe_pack_tc(moearc_x_moe *m, const void *gate, const void *up, const void *down,
                         unsigned int n_expert, void *gateup_tc, void *down_tc);
/* moearc_x_moe_forward for n_tokens <= 1 on tc-layout banks (-2 for more tokens or a layer
 * without the tc path). */
int moearc_x_moe_forward_tc(moearc_x_moe *m, const float *x, unsigned int n_tokens, const float *router_w,
                            const float *router_b, const void *gateup_tc, const void *down_tc,
                            const float *residual, float *out);

/* ---- expert FFNs on the host cores (host_experts.cpp; no GPU needed) ---------------------
 * The reference's HostExecutor (crates/moearc-engine/src/host_experts.rs:423-761): a pool of
 * worker threads that computes a token's FFN through a few experts on the CPU while the device
 * works, phase A (gate, up, activation) then phase B (down), the experts folded in router order
 * by the syncing thread (dst = 0; dst += w * part). The banks are the packed ones
 * (moearc_x_moe_pack layout) in host memory, so an offloaded block keeps one copy of its
 * experts; rows are decoded with AVX2 + FMA + F16C when the CPU has them (MOEARC_HOST_SCALAR=1
 * at create: the portable kernel). */
typedef struct moearc_x_host_pool moearc_x_host_pool;
/* host_experts.rs:445-456 HostExecutor::new: n_threads <= 0 takes MOEARC_HOST_THREADS, else the
 * online cores - 1. NULL when threads cannot start. */
moearc_x_host_pool *moearc_x_host_pool_create(int n_threads);
void moearc_x_host_pool_destroy(moearc_x_host_pool *p);
int moearc_x_host_pool_threads(const moearc_x_host_pool *p);
/* host_experts.rs:624-714 submit: publish out = sum over i < n of weights[i] *
 * down_e . act(gate_e . x, up_e . x), e = experts[i] (n <= 32; the shape, act, alpha, limit and
 * wtype from d), and return without waiting. The pool copies experts, weights and x; the banks
 * (every expert, HOST pointers) stay in use until sync returns. -1 while a job is pending or on
 * NULL, -2 on a shape the pool does not serve (n_embd, n_ff multiples of 64; MXFP4 or Q4_0). */
int moearc_x_host_submit(moearc_x_host_pool *p, const moearc_x_moe_desc *d, const void *gateup_packed,
                         const void *down_packed, const unsigned int *experts, const float *weights,
                         unsigned int n, const float *x);
/* host_experts.rs:717-761 sync: work on the pending job beside the workers, wait for it, write
 * its sum (n_embd floats) to out. -1 with no job pending. */
int moearc_x_host_sync(moearc_x_host_pool *p, float *out);
/* submit + sync. */
int moearc_x_host_ffn(moearc_x_host_pool *p, const moearc_x_moe_desc *d, const void *gateup_packed,
                      const void *down_packed, const unsigned int *experts, const float *weights,
                      unsigned int n, const float *x, float *out);
/* host_experts.rs:604-611 HostStats: out4 = jobs, experts, ns the threads spent inside jobs, ns
 * sync waited for the workers. */
void moearc_x_host_stats(const moearc_x_host_pool *p, unsigned long long *out4);
/* moearc_x_moe_pack on the host: the same packed bytes from GGUF-layout banks in host memory. */
int moearc_x_moe_pack_host(const moearc_x_moe_desc *d, const void *gate, const void *up, const void *down,
                           unsigned int n_expert, void *gateup_packed, void *down_packed);

/* ---- MoE prefill on tcgen05 (prefill.cu; no counterpart in the reference, whose engine
 * decodes one token at a time through matvec kernels, crates/moearc-engine/src/moe.rs:2074-2427)
 * The same MoE block for many tokens per call: router logits in the fixed fold order of
 * moearc_matvec_f32 (bit-exact routing), top-k as moearc_topk_router, then the expert FFN as
 * grouped GEMMs on the fifth-generation tensor cores (TMA operands, TMEM accumulators) with bf16
 * activations and f32 accumulation, SwiGLU fused into the gate-up epilogue, and the combine in
 * router order. d->max_tokens bounds n_tokens per call; scratch for that many tokens and the
 * bf16 expansion of one block's experts is allocated at create. NULL for n_embd > 3584 or
 * shapes the decode path also refuses. */
typedef struct moearc_x_prefill moearc_x_prefill;
moearc_x_prefill *moearc_x_prefill_create(moearc_ctx *c, const moearc_x_moe_desc *d);
void moearc_x_prefill_destroy(moearc_x_prefill *p);
/* Expand one block's packed banks (moearc_x_moe_pack layout, device) into the object's bf16
 * weight matrices; later forward calls use them until the next load. */
int moearc_x_prefill_load(moearc_x_prefill *p, const void *gateup_packed, const void *down_packed);
/* The MXFP8 perf mode (MXFP4 experts only): the packed banks expanded once to E4M3 elements (each
 * E2M1 value exactly) with their E8M0 block scales, and following forward calls run the
 * block-scaled FP8 GEMMs (tcgen05.mma kind::mxf8f6f4) on activations quantised to MXFP8 per 32
 * along K (scale 2^X, X the smallest exponent keeping the block within E4M3's 448; elements round
 * to nearest even) — the expert rows before gate-up and the SwiGLU output before down. Routing
 * is unchanged (bit-exact). -2 for Q4_0 experts. The expert-parallel steps
 * (moearc_x_prefill_route / _experts*) refuse this form; any other load leaves it. */
int moearc_x_prefill_load8(moearc_x_prefill *p, const void *gateup_packed, const void *down_packed);
/* Per-expert biases for the following forward calls, as moearc_x_moe_set_bias but indexed by the
 * object's weight blocks (the expert id after moearc_x_prefill_load; the list position after
 * moearc_x_prefill_load_list): gate_up_bias f32 [2E][n_ff] (gate of block w at row w, up at
 * E + w), added before the activation in the gate-up GEMM's epilogue; down_bias f32
 * [E][n_embd], added to each expert row in the down GEMM's epilogue (inside the weighting).
 * Device pointers (NULL: none), kept until the next call. */
int moearc_x_prefill_set_bias(moearc_x_prefill *p, const float *gate_up_bias, const float *down_bias);
/* out[t] = residual[t] (if not NULL) + MoE(x[t]) for t < n_tokens; x is bf16 [n_tokens][n_embd]
 * (16-byte aligned), router_w f32 [E][n_embd] (16-byte aligned), router_b [E] or NULL; out f32. */
int moearc_x_prefill_forward(moearc_x_prefill *p, const unsigned short *x, unsigned int n_tokens,
                             const float *router_w, const float *router_b, const float *residual,
                             float *out);
/* Device pointers to the last call's internals: 0 expert ids [T x k] (u32), 1 gating weights
 * [T x k], 2 logits [T x E], 3 per-expert counts [E] (int), 4 expanded gate-up weights
 * [E][2][n_ff][n_embd] (bf16), 5 expanded down weights [E][n_embd][n_ff] (bf16), 6 activations
 * in expert order [T k][n_embd] (bf16), 7 SwiGLU outputs [T k][n_ff] (bf16), 8 down rows
 * [T k][n_embd] (f32), 9 row of each (token, choice) [T k] (int), 10 segment offsets [E + 1]. */
void *moearc_x_prefill_buffer(moearc_x_prefill *p, int which);
/* Reads and clears the device status word: 0, or bit 0 = a pipeline wait gave up. */
int moearc_x_prefill_status(moearc_x_prefill *p);
/* Experts [e_first, e_first + n) only, into the object's weight slots 0 .. n-1 (the experts a
 * rank owns under expert parallelism); moearc_x_prefill_load is the range [0, E). */
int moearc_x_prefill_load_range(moearc_x_prefill *p, const void *gateup_packed, const void *down_packed,
                                unsigned int e_first, unsigned int n);
/* Expert experts[i] into weight slot i, i < n (host array of distinct expert ids): the experts a
 * rank owns under a placement other than contiguous ranges. */
int moearc_x_prefill_load_list(moearc_x_prefill *p, const void *gateup_packed, const void *down_packed,
                               const int *experts, unsigned int n);
/* The 4-bit form of the same experts (all, or experts[i] -> slot i): the packed banks are
 * repacked into chunks of 128 rows x 64 columns that one bulk copy moves, and the GEMMs expand
 * them in shared memory as they go, a quarter of the weight bytes of the bf16 form. This form
 * computes in f16 (weights, activations, SwiGLU outputs): -2 when the weights' scaled values do
 * not fit f16 exactly (MXFP4 e8m0 exponents outside [105, 140], or Q4_0 8|d| > 65504), leaving
 * the previous form in place. The last successful load picks the form. */
int moearc_x_prefill_load4(moearc_x_prefill *p, const void *gateup_packed, const void *down_packed);
int moearc_x_prefill_load4_list(moearc_x_prefill *p, const void *gateup_packed, const void *down_packed,
                                const int *experts, unsigned int n);
/* Row order of the route step: expert e's rows form segment pos[e] (host array, a permutation of
 * 0 .. E-1); buffers 3 and 10 are then indexed by position. Identity at create, which
 * moearc_x_prefill_forward requires (-2 otherwise). Under expert parallelism the positions are
 * owner-major, so each rank's experts are one contiguous range of rows. */
int moearc_x_prefill_set_order(moearc_x_prefill *p, const int *pos);
/* The three parts of moearc_x_prefill_forward, for expert parallelism:
 * route: routing and grouping of n_tokens; the activations are then in expert order (buffer 6:
 *   rows of expert e at [offsets[e], offsets[e+1]), buffer 10), counts in buffer 3.
 * experts: the expert FFN over n_rows rows of rows_in (bf16 [n_rows][n_embd]) given as n_seg
 *   consecutive segments, segment s holding seg_counts[s] rows of the loaded expert slot
 *   seg_expert[s] (host arrays, n_seg <= 1024, counts summing to n_rows); y_out (f32
 *   [n_rows][n_embd]) gets one row per input row in the same order; act_scratch is bf16
 *   [n_rows][n_ff]. -2 on inconsistent segments.
 * combine: out[t] = residual[t] (if not NULL) + sum_m w[t,m] y[row(t,m)] for the tokens of the
 *   last route call, y_rows f32 [n_tokens k][n_embd] in that call's expert order. */
int moearc_x_prefill_route(moearc_x_prefill *p, const unsigned short *x, unsigned int n_tokens,
                           const float *router_w, const float *router_b);
int moearc_x_prefill_experts(moearc_x_prefill *p, const unsigned short *rows_in, unsigned int n_rows,
                             const int *seg_counts, const int *seg_expert, unsigned int n_seg,
                             unsigned short *act_scratch, float *y_out);
int moearc_x_prefill_combine(moearc_x_prefill *p, const float *y_rows, unsigned int n_tokens,
                             const float *residual, float *out);
/* Expert parallelism over peer memory (no collective library): route_begin routes and counts
 * (buffer 3 per position); after the caller has all-gathered every rank's counts,
 * route_dispatch stores each row straight into the receive buffer of the rank owning its
 * position (dst_rows[r], starting at row dst_base[r]; host arrays of n_ranks, n_ranks *
 * n_local == E); after a barrier, experts_to runs the expert FFN on the received segments and
 * stores segment s's result rows straight to seg_dst[s] (the source rank's y buffer at the rows
 * its combine reads); after another barrier, combine. Both dispatch and experts_to return once
 * their stores are done. Pointers may be local or opened with moearc_x_ipc_open. */
int moearc_x_prefill_route_begin(moearc_x_prefill *p, const unsigned short *x, unsigned int n_tokens,
                                 const float *router_w, const float *router_b);
int moearc_x_prefill_route_dispatch(moearc_x_prefill *p, void *const *dst_rows, const int *dst_base,
                                    unsigned int n_ranks, unsigned int n_local);
int moearc_x_prefill_experts_to(moearc_x_prefill *p, const unsigned short *rows_in, unsigned int n_rows,
                                const int *seg_counts, const int *seg_expert, unsigned int n_seg,
                                unsigned short *act_scratch, float *const *seg_dst);
/* CUDA IPC for the exchange buffers: the 64-byte handle of a cudaMalloc'd allocation (its start),
 * its mapping in another process on the node, and the mapping's release. */
int moearc_x_ipc_handle(const void *ptr, void *handle);
int moearc_x_ipc_open(const void *handle, void **ptr);
int moearc_x_ipc_close(void *ptr);
/* moearc_x_prefill_forward with an event between its kernels, waited for: ms[i] = device time of
 * kernel i (0 router logits, 1 top-k, 2 scan, 3 scatter, 4 gate-up GEMM, 5 down GEMM, 6 combine);
 * n >= 7. */
int moearc_x_prefill_profile(moearc_x_prefill *p, const unsigned short *x, unsigned int n_tokens,
                             const float *router_w, const float *router_b, const float *residual,
                             float *out, float *ms, int n);

/* ---- expert parallelism over NCCL (ep.cu; the reference has none: its engine serves one GPU) --
 * The prefill MoE block with its experts split over n_ranks GPUs, one process (or thread) per GPU
 * and an NCCL communicator between them, passed as an opaque ncclComm_t (void *). Each rank's
 * moearc_x_prefill object holds its own experts (moearc_x_prefill_load_range / _load_list) and
 * routes in owner-major order (moearc_x_prefill_set_order, rank r's experts at positions
 * r * n_local .. (r + 1) * n_local - 1). moearc_x_ep_forward then routes the rank's tokens,
 * all-gathers the per-position counts (ncclAllGather), plans the exchange on the host (its one
 * synchronisation: NCCL's point-to-point sizes are host arguments), sends each rank's rows and
 * receives its own (one ncclSend / ncclRecv group), runs the grouped GEMMs on the received
 * (source, expert) segments, returns the result rows (a second group) and combines in router
 * order, all on the context stream. The output is bit-identical to the single-GPU block's.
 * NCCL is resolved at run time: the process's, if loaded with global symbols, else libnccl.so.2.
 * unique_id / comm_init / comm_destroy wrap ncclGetUniqueId (128 bytes) / ncclCommInitRank /
 * ncclCommDestroy for hosts without their own NCCL. max_rows bounds the rows a rank receives
 * (-2 from forward past it). */
typedef struct moearc_x_ep moearc_x_ep;
int moearc_x_ep_unique_id(void *id128);
int moearc_x_ep_comm_init(moearc_ctx *c, void **comm, int n_ranks, const void *id128, int rank);
int moearc_x_ep_comm_destroy(void *comm);
moearc_x_ep *moearc_x_ep_create(moearc_ctx *c, moearc_x_prefill *p, const moearc_x_moe_desc *d, void *nccl_comm,
                               int rank, int n_ranks, unsigned int max_rows);
void moearc_x_ep_destroy(moearc_x_ep *ep);
int moearc_x_ep_forward(moearc_x_ep *ep, const unsigned short *x, unsigned int n_tokens, const float *router_w,
                        const float *router_b, const float *residual, float *out);
/* The last forward's counts of every rank ([n_ranks][n_expert] by position, host) and the rows
 * this rank received. */
int moearc_x_ep_counts(moearc_x_ep *ep, int *counts_all);
unsigned int moearc_x_ep_received(moearc_x_ep *ep);

/* ---- synthetic decoder (decoder.cu) ----------------------------------------------------- */
/* One decode step of a routed-MoE transformer (crates/moearc-engine/src/moe.rs:1862-2443,
 * Model::decode) with random, seeded weights generated on the device: per block RMSNorm,
 * Q/K/V (bf16), NeoX RoPE with the YaRN ramp, paged bf16 KV (pages of 32 tokens; blocks with
 * l % swa_pattern < swa_pattern - 1 use a window of n_swa keys in a cyclic ring), decode
 * attention with optional sinks, O projection, and the fused MoE FFN; then a final RMSNorm.
 * There is no token embedding or output head: the step reads an n_embd vector from
 * moearc_x_decoder_input and writes the normalised final state to moearc_x_decoder_output. */
typedef struct moearc_x_decoder moearc_x_decoder;
typedef struct {
    unsigned int n_layer, n_embd, n_head, n_head_kv, head_dim; /* head_dim 64 or 128 */
    unsigned int n_expert, n_expert_used, n_ff;
    unsigned int expert_type;                 /* 39 MXFP4 or 2 Q4_0 */
    unsigned int gating, act;                 /* as moearc_x_moe_desc */
    float alpha, limit;
    unsigned int n_swa, swa_pattern;          /* window (0: none) and pattern */
    float rope_base, rope_freq_scale, rope_ext_factor, rope_attn_factor, rope_corr_lo, rope_corr_hi;
    float rms_eps;
    unsigned int has_sinks;
    unsigned int n_ctx;                       /* positions the KV cache holds */
    unsigned long long seed;
    /* Blocks 0 .. n_offload-1 keep their packed expert banks in pinned, device-mapped host
     * memory (the -ncmoe mirror, moe.rs:1179-1299); each step fetches the routed experts of
     * such a block over PCIe into device slots, with no host round trip. 0: all resident. */
    unsigned int n_offload;
    /* Residency cache of each offloaded block (the reference's ExpertCache, cache.rs:177, in
     * place of pure streaming): n_cache device slots per block keep fetched experts across
     * steps, so an expert routed again is not fetched again; a miss takes the least recently
     * used slot the step does not need. 0: no cache (one slot per routed expert, refilled every
     * step); otherwise at least n_expert_used and at most n_expert. */
    unsigned int n_cache;
    /* QK-norm (moe.rs:1961-1985, the qwen3moe form): q and k normalised per head over head_dim
     * channels with one head_dim-wide weight per block, before RoPE. */
    unsigned int has_qk_norm;
    /* The output head (moe.rs:2434-2437): logits = W_out . rmsnorm(h) with W_out bf16
     * [n_vocab][n_embd] (n_vocab a multiple of 16), after every step; 0 = none. */
    unsigned int n_vocab;
    /* Layout of the resident blocks' expert banks: 0 = the tensor-core layout (moearc_x_moe_pack_tc)
     * where the shape has one (MXFP4 experts, n_embd and n_ff multiples of 64), decoded by the
     * block-scaled FP4 tensor-core kernels; 1 = the fragment layout (moearc_x_moe_pack) everywhere,
     * which the persistent step kernel needs. Offloaded blocks always keep the fragment layout.
     * The batched decoder reads it as 0 = experts at 4 bits, 1 = their bf16 expansion. */
    unsigned int expert_layout;
} moearc_x_decoder_cfg;
moearc_x_decoder *moearc_x_decoder_create(moearc_ctx *c, const moearc_x_decoder_cfg *cfg);
void moearc_x_decoder_destroy(moearc_x_decoder *d);
void *moearc_x_decoder_input(moearc_x_decoder *d);
/* Device pointer of the last step's logits (n_vocab f32), or NULL without an output head. */
void *moearc_x_decoder_logits(moearc_x_decoder *d);
void *moearc_x_decoder_output(moearc_x_decoder *d);  /* device, n_embd f32 */
int moearc_x_decoder_pos(moearc_x_decoder *d);       /* the next position to decode */
int moearc_x_decoder_set_pos(moearc_x_decoder *d, unsigned int pos);
/* Fill every KV page with synthetic bf16 N(0, 0.02) and set the position to depth. */
int moearc_x_decoder_fill_kv(moearc_x_decoder *d, unsigned int depth, unsigned long long seed);
/* Decode one token at the current position, enqueued on the context's stream; the first call
 * captures the step as a CUDA graph (unless disabled) and later calls replay it. */
int moearc_x_decoder_step(moearc_x_decoder *d);
/* One token from host memory to host memory (the reference's decode loop takes a host embedding
 * row and returns host results, moe.rs:1862-1870, 2429-2442): x and y are n_embd f32 in any host
 * memory. The call copies x to pinned staging, launches the step with its two copies as one
 * graph (unless graphs are disabled), waits for it and writes the step's output to y. The first
 * call allocates the pinned staging and captures that graph. */
int moearc_x_decoder_step_host(moearc_x_decoder *d, const float *x, float *y);
int moearc_x_decoder_use_graph(moearc_x_decoder *d, int on);
/* Reads and clears the device status words of the decoder's kernels: 0, or nonzero when a
 * bounded wait gave up (the step's output is then invalid). No reference counterpart: the
 * reference's decode loop has no device-side waits. */
int moearc_x_decoder_status(moearc_x_decoder *d);
/* Experts fetched over PCIe since create by the offloaded blocks' residency caches (0 without a
 * cache); synchronises the stream. No reference counterpart. */
unsigned long long moearc_x_decoder_fetched(moearc_x_decoder *d);
/* One step without the graph and with an event after every kernel: ms[k] gets the device time
 * of kernel kind k (0 Q/K/V, 1 attention, 2 O projection, 3 MoE route, 4 MoE gate-up, 5 MoE
 * down, 6 final norm, 7 expert fetch of an offloaded block) summed over the blocks, counts[k]
 * the launches; n >= 7 (kinds >= n are not reported). */
int moearc_x_decoder_profile(moearc_x_decoder *d, float *ms, int *counts, int n);
/* Host execution of part of the offloaded blocks' experts (moe.rs:2169-2211 the split,
 * 2389-2420 the fold; HostPolicy host_experts.rs:91-127): kind 0 off, 1 the first
 * ceil(misses x fraction) of a block's misses in router order, 2 the misses beyond the first
 * `over`; a miss is a routed expert the block's residency cache does not hold (without a cache,
 * every routed expert). Those experts are computed by a pool of n_threads host threads
 * (moearc_x_host_pool_create's rule for <= 0) from the block's pinned packed banks while the device
 * streams the others; a cache admits only the device's share. Needs n_offload > 0 (-2
 * otherwise). The split and the answer pass through a mailbox in pinned memory that a host
 * thread polls (no host function in the step's graph). Synchronises the stream; the next step
 * re-captures its graph. */
int moearc_x_decoder_host_experts(moearc_x_decoder *d, int kind, float fraction, unsigned int over,
                                  int n_threads);
/* The fold's wait for the host's answer: limit_ns (0: the default 2 s), after which the step
 * raises the status (STATUS bit 1) and leaves the host's share out; hold = 1 makes the host
 * thread ignore new jobs (for testing that the wait runs out), 0 resumes. No reference
 * counterpart (its sync waits without a limit, host_experts.rs:717-745). Synchronises the stream. */
int moearc_x_decoder_host_wait(moearc_x_decoder *d, unsigned long long limit_ns, int hold);
/* The host pool's counters since create (moearc_x_host_stats); zeros without a pool.
 * Synchronises the stream. */
int moearc_x_decoder_host_stats(moearc_x_decoder *d, unsigned long long *out4);
/* Device pointer (and size) of one block's tensor: 0 attn_norm, 1 ffn_norm, 2 sinks,
 * 3 router, 4 K pool, 5 V pool, 6 page table, 7 packed Q/K/V, 8 packed O, 9 packed gate-up,
 * 10 packed down, 11 output norm; with the persistent step kernel, 12 the block's expert ids
 * of the last step (k u32, router order) and 13 their gating weights (k f32); with kernel spans
 * on, 14 the kernel chain's expert-kernel timestamps of the last step (u64 [2 kernels: gate-up,
 * down][CTA][start, dependency wait over, end], ns of %globaltimer); 15 / 16 the QK-norm
 * weights (head_dim f32, with has_qk_norm); 17 the packed bf16 output head (layer ignored, with
 * n_vocab). For an offloaded block, 9 and 10 are device-visible pointers of the pinned host
 * banks; for a resident block of a decoder with expert_layout 0 on a shape that has one, they are
 * in the tc layout (moearc_x_moe_pack_tc). */
void *moearc_x_decoder_tensor(moearc_x_decoder *d, int which, unsigned int layer, unsigned long *bytes);
/* Turn on (1) or off (0) the expert kernels' per-CTA timestamps in the kernel chain (tensor 14),
 * so their duration can be read from inside a graphed step. Synchronises the stream; the next
 * step re-captures its graph. No reference counterpart. */
int moearc_x_decoder_kernel_spans(moearc_x_decoder *d, int on);
/* The seed tensor `kind` of block `layer` was generated from, given the model seed. */
unsigned long long moearc_x_decoder_seed(moearc_x_decoder *d, int kind, unsigned int layer,
                                         unsigned long long base);
/* ---- the decode step as one persistent kernel (no reference counterpart) ----------------
 * Resident-expert decoders with head_dim 64 (the gpt-oss family) can run the whole step as one
 * cooperative launch: a CTA per SM, the phases of every block separated by grid barriers, each
 * warp streaming its share of the weights through a ring of bulk copies that runs ahead across
 * phase boundaries. The chain of per-block kernels is the default (MOEARC_STEP_KERNEL=1 at
 * create, or use_step_kernel, selects the persistent kernel). */
/* 1 when the shape has the persistent kernel. */
int moearc_x_decoder_has_step_kernel(moearc_x_decoder *d);
/* 1 when steps run the persistent kernel, 0 when they run the kernel chain. */
int moearc_x_decoder_uses_step_kernel(moearc_x_decoder *d);
/* Choose the persistent kernel (on, when the shape has one; -2 otherwise) or the chain. */
int moearc_x_decoder_use_step_kernel(moearc_x_decoder *d, int on);
/* The decode kernels' wait limits (ns; 0 = the default 0.2 s): the persistent kernel's grid
 * barriers and the chain's expert kernels' waits for one another's partial sums. phantom 1
 * makes them run out, for testing the bounded waits: the persistent kernel's first barrier
 * waits for one arrival beyond the CTAs', the expert kernels' finishing warps never see their
 * partials; the step then sets the status word and returns, its output invalid (reading the
 * status restores the partial buffers). Synchronises the stream; the next step re-captures
 * its graph. */
int moearc_x_decoder_set_wait(moearc_x_decoder *d, unsigned long long limit_ns, unsigned int phantom);
/* Phase timestamps of the persistent kernel: with a device buffer of trace_words u64 set,
 * every following step writes %globaltimer (ns) at four points of each phase of each block in
 * each CTA: word ((layer * 6 + phase) * 4 + point) * n_cta + cta; phases 0 Q/K/V, 1 attention,
 * 2 O projection, 3 router, 4 expert gate-up, 5 expert down; points 0 start (the grid barrier
 * opened), 1 inputs ready, 2 the CTA's warp 0 done with its share, 3 end. NULL turns it off.
 * Synchronises the stream; the next step re-captures its graph. */
unsigned long moearc_x_decoder_trace_words(moearc_x_decoder *d);
int moearc_x_decoder_set_trace(moearc_x_decoder *d, void *device_buffer);

/* ---- batched decoder (batch.cu; no counterpart in the reference, whose engine decodes one
 * sequence) ---------------------------------------------------------------------------------
 * n_batch independent sequences, one token each per step, through the decoder of cfg (same
 * weights as moearc_x_decoder_create would generate from it): bf16 activations into tcgen05
 * GEMMs for Q/K/V and O, RoPE and paged bf16 KV per sequence, one batched decode-attention launch,
 * and the prefill MoE block with the router on the f32 activations; QK-norm with has_qk_norm. The
 * experts stay at 4 bits (the prefill object's 4-bit form, f16 tiles expanded in shared memory)
 * with expert_layout 0, or are expanded to bf16 once at create with expert_layout 1. Requires
 * n_swa == 0, no sinks, n_offload == 0, n_vocab == 0; NULL otherwise. */
typedef struct moearc_x_batch_decoder moearc_x_batch_decoder;
moearc_x_batch_decoder *moearc_x_batch_decoder_create(moearc_ctx *c, const moearc_x_decoder_cfg *cfg,
                                                      unsigned int n_batch);
/* Expert parallelism for the batched decoder (configs[4] over n_ranks GPUs; no reference
 * counterpart): every rank decodes its own n_batch streams (attention and projections local) and
 * holds experts rank * n_expert / n_ranks .. of every block, at 4 bits (expert_layout 0 only). Per
 * block the ranks' routed rows are all-gathered, each owner runs its experts over every rank's
 * rows, the results return in one grouped exchange and each rank combines its own tokens — all
 * on comm (an ncclComm_t of the n_ranks ranks, e.g. from moearc_x_ep_comm_init) with fixed sizes,
 * inside the captured step graph. Every rank must step together. NULL if n_expert % n_ranks. */
moearc_x_batch_decoder *moearc_x_batch_decoder_create_ep(moearc_ctx *c, const moearc_x_decoder_cfg *cfg,
                                                         unsigned int n_batch, void *comm, int rank, int n_ranks);
void moearc_x_batch_decoder_destroy(moearc_x_batch_decoder *d);
void *moearc_x_batch_decoder_input(moearc_x_batch_decoder *d);   /* device, n_batch x n_embd f32 */
void *moearc_x_batch_decoder_output(moearc_x_batch_decoder *d);  /* device, n_batch x n_embd f32 */
/* Every sequence at position pos; with fill, every KV page first gets synthetic bf16 N(0, 0.02). */
int moearc_x_batch_decoder_set_pos(moearc_x_batch_decoder *d, unsigned int pos, int fill,
                                   unsigned long long seed);
/* One token for every sequence; the first call captures the step as a CUDA graph. */
int moearc_x_batch_decoder_step(moearc_x_batch_decoder *d);
/* Reads and clears the status words: 0, or nonzero when a bounded wait gave up. */
int moearc_x_batch_decoder_status(moearc_x_batch_decoder *d);
/* Device pointer to block `layer`'s expert choice of the last step, n_batch x k u32 in router
 * order (NULL for a layer out of range). */
void *moearc_x_batch_decoder_routing(moearc_x_batch_decoder *d, unsigned int layer);

/* ---- GGUF model files (no counterpart in the reference's ABI) -------------------------------
 * A read-only view of a GGUF v2/v3 file, replacing the reference's Rust reader
 * (crates/moearc-model/src/gguf.rs:166-279, the header parse with its plausibility checks) and
 * its expert addressing (crates/moearc-model/src/tensors.rs:237-289, slice_last_dim). The file
 * is mapped, not read: a tensor's bytes are a pointer into the mapping, valid until close, and
 * can go straight to moearc_copy_h2d / moearc_x_moe_pack. Every count and length in the header
 * is checked against the file size before it is used; a malformed file is refused at open. */
typedef struct moearc_x_gguf moearc_x_gguf;
typedef struct {
    unsigned int n_dims;                /* 1..4 */
    unsigned long long dims[4];         /* fastest-varying first, as stored */
    unsigned int type_id;               /* ggml type id: F32 0, F16 1, Q4_0 2, Q8_0 8, BF16 30, MXFP4 39 ... */
    unsigned long long offset;          /* of the tensor's first byte, from the start of the file */
    unsigned long long nbytes;          /* elements / block size x block bytes */
    const void *data;                   /* in the mapping */
} moearc_x_gguf_tensor;
/* NULL on any failure; moearc_x_gguf_last_error() then names it. */
moearc_x_gguf *moearc_x_gguf_open(const char *path);
void moearc_x_gguf_close(moearc_x_gguf *g);
/* The calling thread's message for its last failed moearc_x_gguf_* call ("" if none). */
const char *moearc_x_gguf_last_error(void);
unsigned int moearc_x_gguf_version(moearc_x_gguf *g);
unsigned long long moearc_x_gguf_alignment(moearc_x_gguf *g);
unsigned long long moearc_x_gguf_n_tensors(moearc_x_gguf *g);
/* Metadata: 0, or -2 when the key is absent or holds another kind of value. Integer keys of any
 * width (and bools) read as u64 when non-negative; f32 and f64 keys read as double; strings
 * are returned NUL-terminated, valid until close. */
int moearc_x_gguf_key_u64(moearc_x_gguf *g, const char *key, unsigned long long *out);
int moearc_x_gguf_key_f64(moearc_x_gguf *g, const char *key, double *out);
int moearc_x_gguf_key_str(moearc_x_gguf *g, const char *key, const char **out);
/* Tensor by name, or by index (name through *name); -2 when absent. */
int moearc_x_gguf_find(moearc_x_gguf *g, const char *name, moearc_x_gguf_tensor *out);
int moearc_x_gguf_tensor_at(moearc_x_gguf *g, unsigned long long i, moearc_x_gguf_tensor *out, const char **name);
/* Slice `index` of a stacked tensor along its last dimension (one expert of a
 * blk.N.ffn_{gate,up,down}_exps.weight bank): the n_dims - 1 inner dimensions, at a byte
 * stride of inner elements / block size x block bytes. -2 when the tensor is absent or rank 1,
 * the index is out of range, the inner elements are not whole blocks, or the slices do not
 * tile the tensor exactly. */
int moearc_x_gguf_slice_last(moearc_x_gguf *g, const char *name, unsigned long long index,
                             moearc_x_gguf_tensor *out);

/* ---- tensor-core peaks (mma_peak.cu; no reference counterpart) ---------------------------
 * Dense throughput of one MMA kind measured with the library's own tcgen05 loop (one CTA per
 * SM, 128 x 256 MMAs from shared memory into TMEM, timed by the slowest SM): kind 0 kind::f16
 * bf16, 1 kind::mxf8f6f4 E4M3 x E4M3, 2 kind::mxf4 E2M1 x E2M1, 3 kind::mxf8f6f4 E4M3 x E2M1
 * (block-scaled kinds with E8M0 scales per 32). iters MMAs per SM (1 .. 2^20); TFLOP/s into
 * *tflops. Synchronises the stream. */
int moearc_x_mma_peak(moearc_ctx *c, int kind, int iters, double *tflops);

/* ---- decode attention without allocation (no counterpart in the reference) ----------------
 * Same arguments, result and return codes as moearc_attn_decode, but the split-K partials live
 * in a fixed per-device array of MOEARC_X_ATTN_STATIC_SCRATCH_BYTES compiled into the library,
 * so no call allocates device or host memory. It serves hosts that may not allocate while they
 * decode (a fixed memory budget, or a neighbouring thread capturing a CUDA graph).
 * - Returns -2 when the partials for the split count the call picks,
 *   n_heads x n_splits x (head_dim + 2) x 4 bytes, exceed that size (2 MiB: e.g. 64 heads of
 *   128 over 8 KV heads needs 1.2 MiB on a 148-SM B200); nothing is enqueued then.
 * - The first call on a device looks the array's address up (cudaGetSymbolAddress, with that
 *   device made current for the lookup); make that first call before any stream capture.
 * - There is one array per device: calls that may overlap on a device (two streams, two
 *   contexts, two threads) race on it. Serialise them. Nothing in it needs to start at zero. */
#define MOEARC_X_ATTN_STATIC_SCRATCH_BYTES (2ul << 20)
int moearc_x_attn_decode_static(moearc_ctx *c, float *out, const float *q, const void *k_pages,
                                const void *v_pages, const unsigned int *block_table, const float *sinks,
                                unsigned long n_heads, unsigned long n_kv_heads, unsigned long head_dim,
                                unsigned long kv_begin, unsigned long n_kv, unsigned long page_tokens,
                                float scale, unsigned int kv_type);

#ifdef __cplusplus
}
#endif
#endif
