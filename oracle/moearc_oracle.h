/*
 * moearc_oracle.h — CPU oracle for the MoE decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the shipped library links, loads or calls this code.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs may
 * use it, and only as the checker or as the timed CPU baseline — never as the thing measured
 * on the GPU or as a fallback for it.
 *
 * What it is: a plain-C restatement of MoEArc's executable specification,
 * crates/moearc-kernels/src/reference.rs (the "CPU twin" every SYCL kernel is checked against),
 * plus the composition of the MoE block from crates/moearc-engine/src/moe.rs:2074-2427 and the
 * attention block from moe.rs:1936-2072. Each function names the reference lines it follows.
 *
 * Pinning: the reference is Rust (rustc/cargo are not installed here) and its kernels are SYCL
 * (icpx is not installed), so the reference cannot be compiled or run in this container. The
 * oracle is pinned instead against every known-answer test the reference's own test files hold
 * for this path (reference.rs:879-930, kernels_gpu.rs:406-467, forward_pass_gpu.rs:676/747),
 * read as text and restated in tests/test_oracle_kat.py, and against hand-computed blocks for
 * the formats the reference never tested (MXFP4, Q4_0, bf16). Q4_0 and bf16 have no code at
 * all in the reference (only a type id, crates/moearc-model/src/quant.rs:54 and :100), so their
 * parity is pinned only by this build's own known-answer tests.
 *
 * Accuracy convention (reference.rs:12-14): reductions accumulate in double where ggml uses
 * ggml_float, and in float where ggml uses float. Build with -ffp-contract=off: the functions
 * whose name ends in _gpu_order emulate a fixed float evaluation order bit for bit, and a
 * compiler-contracted multiply-add would break that.
 */
#ifndef MOEARC_ORACLE_H
#define MOEARC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF type ids (reference.rs:21-40; crates/moearc-model/src/quant.rs:51-107). */
enum {
    OR_F32 = 0,
    OR_F16 = 1,
    OR_Q4_0 = 2,
    OR_Q8_0 = 8,
    OR_Q4_K = 12,
    OR_Q5_K = 13,
    OR_Q6_K = 14,
    OR_BF16 = 30,
    OR_MXFP4 = 39
};

/* Router gatings (reference.rs:516-533). */
enum { OR_GATING_SOFTMAX = 0, OR_GATING_SOFTMAX_NORM = 1, OR_GATING_SOFTMAX_AFTER_TOPK = 2 };

/* ---- scalar formats ------------------------------------------------------------------ */
float or_f16_to_f32(uint16_t h);              /* reference.rs:123-149 */
uint16_t or_f32_to_f16(float f);              /* reference.rs:647-691 (RNE, NaN kept) */
float or_bf16_to_f32(uint16_t h);             /* bf16 = upper half of binary32 */
uint16_t or_f32_to_bf16(float f);             /* RNE, NaN kept quiet; no reference code */
float or_e8m0_half(uint8_t x);                /* reference.rs:66-70 */
extern const int8_t OR_KVALUES_MXFP4[16];     /* reference.rs:56 */

/* ---- block formats -------------------------------------------------------------------- */
int or_block_bytes(unsigned type_id);         /* reference.rs:78-89; 0 if unsupported */
int or_block_elems(unsigned type_id);         /* reference.rs:93-100 */
/* reference.rs:168-192. Returns 0, or -2 for an unsupported type. */
int or_dequant(unsigned type_id, const uint8_t *src, size_t nblocks, float *dst);

/* ---- matvecs -------------------------------------------------------------------------- */
/* reference.rs:305-320: dequantise the row, accumulate in double. */
int or_matvec_q(unsigned type_id, const uint8_t *w, const float *x, size_t n_rows, size_t n_cols,
                float *out);
/* reference.rs:323-335. */
void or_matvec_f32(const float *w, const float *x, size_t n_rows, size_t n_cols, float *out);
/* The device router GEMV's fixed float order, emulated bit for bit: lane l of a 32-lane warp
 * folds columns 4l+128i .. 4l+128i+3 in that order with fmaf, then the 32 partials are combined
 * by the xor butterfly 16,8,4,2,1. moearc_matvec_f32 on the device computes exactly this. */
void or_matvec_f32_gpu_order(const float *w, const float *x, size_t n_rows, size_t n_cols,
                             float *out);

/* ---- elementwise / rows --------------------------------------------------------------- */
void or_rmsnorm(const float *x, const float *weight, size_t n_rows, size_t n_cols, float eps,
                float *out);                  /* reference.rs:338-361 */
void or_silu(const float *x, size_t n, float *out);                       /* :363-366 */
void or_swiglu(const float *g, const float *u, size_t n, float *out);     /* :369-372 */
void or_swiglu_oai(const float *g, const float *u, size_t n, float alpha, float limit,
                   float *out);               /* reference.rs:386-396 */
void or_softmax_ext(const float *x, const float *mask, size_t n_rows, size_t n_cols, float scale,
                    float *out);              /* reference.rs:407-433 */
void or_add(const float *a, const float *b, size_t n, float *out);       /* :694-697 */
void or_mul(const float *a, const float *b, size_t n, float *out);       /* :700-703 */
void or_axpy(float *out, const float *x, float alpha, size_t n);         /* :706-711 */
/* kernels.cpp:1220-1235: out[i] = sum over m ascending of w[m]*parts[m*n+i], from 0.0f, each
 * step one fused multiply-add (the device kernel's rounding, emulated exactly). */
void or_moe_combine(const float *parts, const float *w, unsigned n_mat, size_t n, float *out);
/* kernels.cpp:1654-1670: out[m*n_rows+r] += bias[idx[m]*n_rows+r]. */
void or_add_bias_id(float *out, const float *bias, const uint32_t *idx, unsigned n_mat,
                    size_t n_rows);
/* reference.rs:714-724. */
int or_embed_rows(unsigned type_id, const uint8_t *table, const uint32_t *ids, size_t n_tokens,
                  size_t n_embd, float *out);

/* ---- RoPE ----------------------------------------------------------------------------- */
/* reference.rs:468-508: iterated angle table (theta *= theta_scale), plain RoPE. */
void or_rope(const float *src, const int32_t *pos, size_t n_tokens, size_t n_heads,
             size_t head_dim, size_t n_dims, float freq_base, int neox, float *out);
/* kernels.cpp:1399-1472: closed-form angle with the YaRN ramp, in double. */
void or_rope_ext(const float *src, const int32_t *pos, size_t n_tokens, size_t n_heads,
                 size_t head_dim, size_t n_dims, float freq_base, float freq_scale,
                 float ext_factor, float attn_factor, float corr_lo, float corr_hi, int neox,
                 float *out);

/* ---- router --------------------------------------------------------------------------- */
/* reference.rs:599-639. Stable descending order, lower expert id first on a tie. */
int or_topk_router(const float *logits, size_t n_tokens, size_t n_expert, unsigned k,
                   unsigned gating, uint32_t *idx, float *w);

/* ---- paged KV + attention ------------------------------------------------------------- */
/* reference.rs:767-777: ((page*page_tokens + slot)*n_kv_heads + head)*head_dim + d. */
size_t or_kv_index(uint32_t page, uint32_t slot, size_t head, size_t d, size_t n_kv_heads,
                   size_t head_dim, size_t page_tokens);
/* reference.rs:754-759 + kernels.cpp:427-440: the value a cache of kv_type actually holds. */
float or_kv_store(float v, unsigned kv_type);
/* reference.rs:781-802, generalised to the three cache types (F32 0, F16 1, BF16 30). The
 * pools hold raw elements of kv_type. */
int or_kv_append(void *k_pages, void *v_pages, const float *k, const float *v, uint32_t page,
                 uint32_t slot, size_t n_kv_heads, size_t head_dim, size_t page_tokens,
                 unsigned kv_type);
/* reference.rs:821-873 (two-pass, double) over pools of kv_type, plus the attention sink of
 * kernels.cpp:1856-1880: a per-head extra logit that joins the max and the denominator and
 * carries no value. sinks may be NULL. */
int or_attn_decode(const float *q, const void *k_pages, const void *v_pages,
                   const uint32_t *block_table, const float *sinks, size_t n_heads,
                   size_t n_kv_heads, size_t head_dim, size_t kv_begin, size_t n_kv,
                   size_t page_tokens, float scale, unsigned kv_type, float *out);

/* ---- the MoE FFN of one token (moe.rs:2074-2427) -------------------------------------- */
typedef struct {
    size_t n_embd;          /* H */
    size_t n_ff;            /* I, expert intermediate */
    size_t n_expert;        /* E */
    unsigned k;             /* experts used */
    unsigned gating;        /* OR_GATING_* */
    unsigned act;           /* 0 = SwiGLU, 1 = SwiGLU-OAI */
    float alpha, limit;     /* OAI constants, moe.rs:494 */
    unsigned wtype;         /* expert weight type (OR_MXFP4, OR_Q4_0, ...) */
    int router_gpu_order;   /* 1: logits by or_matvec_f32_gpu_order, 0: by or_matvec_f32 */
} or_moe_cfg;

/* One token: logits = router_w . x (+ router_b, before the top-k), top-k, then for each chosen
 * expert in router order: g = gate_e . x (+gb), u = up_e . x (+ub), a = act(g,u),
 * o = down_e . a (+db); out = sum over the k experts, m ascending, of w_m * o_m.
 * gate/up/down are banks of n_expert matrices in GGUF row layout, each expert's bytes
 * contiguous (crates/moearc-model/src/tensors.rs:237-289). Biases may be NULL. idx/w may be
 * NULL; otherwise they receive the router's choice. */
int or_moe_ffn_token(const or_moe_cfg *c, const float *x, const float *router_w,
                     const float *router_b, const uint8_t *gate, const uint8_t *up,
                     const uint8_t *down, const float *gate_b, const float *up_b,
                     const float *down_b, float *out, uint32_t *idx, float *w);

/* MXFP8 quantisation per 32 values (scale 2^X, X the smallest with max|x| / 2^X <= 448; E4M3
 * round to nearest even), dequantised: the declared arithmetic of the build's FP8 prefill mode. */
void or_mx8_quantize(const float *x, size_t n, float *out);
/* or_moe_ffn_token with that quantisation applied to x before gate/up and to the activation
 * before down (routing on x unquantised). */
int or_moe_ffn_token_mx8(const or_moe_cfg *c, const float *x, const float *router_w,
                         const float *router_b, const uint8_t *gate, const uint8_t *up,
                         const uint8_t *down, const float *gate_b, const float *up_b,
                         const float *down_b, float *out, uint32_t *idx, float *w);

/* ---- synthetic inputs (SplitMix64, tests/common/mod.rs:11-38) ------------------------- */
uint64_t or_splitmix64(uint64_t *state);
/* MXFP4 blocks: nibbles uniform over 16 codes, e8m0 = 127+e with e uniform in [e_lo, e_hi]. */
void or_synth_mxfp4(uint64_t seed, size_t nblocks, int e_lo, int e_hi, uint8_t *dst);
/* Q4_0 blocks: nibbles uniform, d = f16(|N(0, sigma)|). */
void or_synth_q4_0(uint64_t seed, size_t nblocks, double sigma, uint8_t *dst);
/* n normal draws N(0, sigma) by Box-Muller in double, rounded to float. */
void or_synth_normal_f32(uint64_t seed, size_t n, double sigma, float *dst);
/* n normal draws N(0, sigma) rounded to bf16 (RNE). */
void or_synth_normal_bf16(uint64_t seed, size_t n, double sigma, uint16_t *dst);

#ifdef __cplusplus
}
#endif
#endif
