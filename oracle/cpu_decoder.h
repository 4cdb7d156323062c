/*
 * cpu_decoder.h — one decode step of the synthetic gpt-oss / Qwen3-MoE shaped decoder on the
 * CPU. TEST / BENCH INFRASTRUCTURE ONLY.
 *
 * The step is the per-block kernel sequence of crates/moearc-engine/src/moe.rs:1935-2427:
 *   x = rmsnorm(h, attn_norm); q,k,v = W x; [per-head rmsnorm of q, k: QK-norm, moe.rs:1961-1985];
 *   rope(q), rope(k) (NeoX, moe.rs:1987-2012);
 *   kv_append at the layer's (page, slot); attention over [kv_begin, n_kv) with sinks;
 *   h += Wo . attn; x = rmsnorm(h, ffn_norm); h += moe_ffn(x)
 * and a final rmsnorm (moe.rs:2429-2433). Blocks l with l % swa_pattern < swa_pattern - 1
 * attend through a window of n_swa keys (moe.rs:687-699).
 *
 * Two engines share the sequence: pool == NULL runs the scalar oracle (double accumulation,
 * reference.rs semantics) and is the parity checker; a pool runs the restated CPU path
 * (host_experts.c) and is the timed CPU baseline.
 */
#ifndef MOEARC_CPU_DECODER_H
#define MOEARC_CPU_DECODER_H

#include <stddef.h>
#include <stdint.h>

#include "host_experts.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    size_t n_layer, n_embd, n_head, n_head_kv, head_dim, n_expert, n_ff;
    unsigned k, gating, act, wtype, kv_type;
    float alpha, limit, eps;
    size_t n_swa, swa_pattern, page_tokens;
    float rope_base, freq_scale, ext_factor, attn_factor, corr_lo, corr_hi;
    unsigned qk_norm; /* 1: q and k normalised per head (head_dim-wide weights) before RoPE */
} cd_cfg;

typedef struct {
    const float *attn_norm, *ffn_norm;      /* [H] */
    const uint16_t *wq, *wk, *wv, *wo;      /* bf16, rows of H (wo: rows of n_head*head_dim) */
    const float *sinks;                     /* [n_head] or NULL */
    const float *router;                    /* [E x H] f32 */
    const uint8_t *gate, *up, *down;        /* expert banks, GGUF layout, wtype */
    void *k_pages, *v_pages;                /* this layer's KV pool, kv_type elements */
    const uint32_t *table;                  /* logical page -> physical page */
    const float *q_norm, *k_norm;           /* [head_dim] QK-norm weights (qk_norm) or NULL */
} cd_layer;

/* Decode the token whose input hidden state is h_in (n_embd floats) at position pos; writes
 * the normalised final hidden state to out. If idx_out is not NULL it receives the router's
 * choice, n_layer * k ids. Returns 0 or a negative error. */
int cd_step(const cd_cfg *c, const cd_layer *layers, const float *output_norm, const float *h_in,
            size_t pos, hx_pool *pool, float *out, uint32_t *idx_out);

/* cd_step without the pool, also recording per layer in margin_out (n_layer floats) the gap
 * between the k-th and the (k+1)-th largest router logit: how close that routing is to a tie. */
int cd_step_margins(const cd_cfg *c, const cd_layer *layers, const float *output_norm,
                    const float *h_in, size_t pos, float *out, uint32_t *idx_out, float *margin_out);

/* The same sequence over layers [l0, l1) only, from h (updated in place), with no final
 * norm: the bounded sample the bench times. */
int cd_layers(const cd_cfg *c, const cd_layer *layers, size_t l0, size_t l1, float *h,
              size_t pos, hx_pool *pool, uint32_t *idx_out);

/* The output head (moe.rs:2434-2437): logits = W_out . x, W_out bf16 [n_vocab][n_embd], x the
 * normalised final hidden state (cd_step's out). */
int cd_logits(const cd_cfg *c, const uint16_t *w_out, size_t n_vocab, const float *x, float *logits);

#ifdef __cplusplus
}
#endif
#endif
