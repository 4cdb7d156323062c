/*
 * cpu_decoder.c — CPU decode step of the synthetic decoder (see cpu_decoder.h).
 * TEST / BENCH INFRASTRUCTURE ONLY.
 */
#include "cpu_decoder.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "moearc_oracle.h"

static int is_swa(const cd_cfg *c, size_t l) {
    return c->n_swa > 0 && c->swa_pattern > 0 && (l % c->swa_pattern) < c->swa_pattern - 1;
}

static int mv(hx_pool *pool, unsigned t, const void *w, const float *x, size_t rows, size_t cols,
              float *out) {
    if (pool) return hx_matvec(pool, t, (const uint8_t *)w, x, rows, cols, out);
    if (t == OR_F32) {
        or_matvec_f32((const float *)w, x, rows, cols, out);
        return 0;
    }
    return or_matvec_q(t, (const uint8_t *)w, x, rows, cols, out);
}

/* The gap between the k-th and the (k+1)-th largest router logit (0 when E <= k): how far the
 * routing is from a tie, so a test can tell a near-tie flip from a routing error. */
static float topk_margin(const float *logits, size_t E, unsigned k) {
    if (E <= k) return 0.f;
    float kth = -INFINITY, next = -INFINITY;
    /* k + 1 rounds of "largest value not above the previous, counted with multiplicity" */
    unsigned seen = 0;
    float prev = INFINITY;
    while (seen <= k) {
        float m = -INFINITY;
        for (size_t e = 0; e < E; ++e)
            if (logits[e] < prev && logits[e] > m) m = logits[e];
        unsigned cnt = 0;
        for (size_t e = 0; e < E; ++e) cnt += logits[e] == m;
        if (cnt == 0) break;
        for (unsigned i = 0; i < cnt && seen <= k; ++i, ++seen) {
            if (seen == k - 1) kth = m;
            if (seen == k) next = m;
        }
        prev = m;
    }
    return kth - next;
}

static int layers_impl(const cd_cfg *c, const cd_layer *L, size_t l0, size_t l1, float *h, size_t pos,
                       hx_pool *pool, uint32_t *idx_out, float *margin_out) {
    const size_t H = c->n_embd, Dq = c->n_head * c->head_dim, Dkv = c->n_head_kv * c->head_dim;
    const size_t E = c->n_expert;
    float *x = (float *)malloc(sizeof(float) * H);
    float *q = (float *)malloc(sizeof(float) * Dq);
    float *qr = (float *)malloc(sizeof(float) * Dq);
    float *k = (float *)malloc(sizeof(float) * Dkv);
    float *kr = (float *)malloc(sizeof(float) * Dkv);
    float *v = (float *)malloc(sizeof(float) * Dkv);
    float *att = (float *)malloc(sizeof(float) * Dq);
    float *proj = (float *)malloc(sizeof(float) * H);
    float *ffn = (float *)malloc(sizeof(float) * H);
    float *logits = (float *)malloc(sizeof(float) * E);
    const int32_t p32 = (int32_t)pos;
    const size_t n_kv = pos + 1;
    const size_t slot = pos % c->page_tokens;
    int rc = 0;

    or_moe_cfg mc = {H, c->n_ff, E, c->k, c->gating, c->act, c->alpha, c->limit, c->wtype, 0};

    for (size_t l = l0; l < l1 && !rc; ++l) {
        const cd_layer *b = &L[l];
        /* ---- attention (moe.rs:1936-2072) ---- */
        or_rmsnorm(h, b->attn_norm, 1, H, c->eps, x);
        if ((rc = mv(pool, OR_BF16, b->wq, x, Dq, H, q))) break;
        if ((rc = mv(pool, OR_BF16, b->wk, x, Dkv, H, k))) break;
        if ((rc = mv(pool, OR_BF16, b->wv, x, Dkv, H, v))) break;
        if (c->qk_norm) {
            /* QK-norm per head over head_dim channels, one weight row broadcast across heads
             * (moe.rs:1969-1981, the qwen3moe spelling) */
            if (!b->q_norm || !b->k_norm) {
                rc = -2;
                break;
            }
            or_rmsnorm(q, b->q_norm, c->n_head, c->head_dim, c->eps, q);
            or_rmsnorm(k, b->k_norm, c->n_head_kv, c->head_dim, c->eps, k);
        }
        or_rope_ext(q, &p32, 1, c->n_head, c->head_dim, c->head_dim, c->rope_base, c->freq_scale,
                    c->ext_factor, c->attn_factor, c->corr_lo, c->corr_hi, 1, qr);
        or_rope_ext(k, &p32, 1, c->n_head_kv, c->head_dim, c->head_dim, c->rope_base,
                    c->freq_scale, c->ext_factor, c->attn_factor, c->corr_lo, c->corr_hi, 1, kr);
        const uint32_t page = b->table[pos / c->page_tokens];
        if ((rc = or_kv_append(b->k_pages, b->v_pages, kr, v, page, (uint32_t)slot, c->n_head_kv,
                               c->head_dim, c->page_tokens, c->kv_type)))
            break;
        const size_t kv_begin = (is_swa(c, l) && n_kv > c->n_swa) ? n_kv - c->n_swa : 0;
        const float scale = 1.0f / sqrtf((float)c->head_dim);
        if ((rc = or_attn_decode(qr, b->k_pages, b->v_pages, b->table, b->sinks, c->n_head,
                                 c->n_head_kv, c->head_dim, kv_begin, n_kv, c->page_tokens, scale,
                                 c->kv_type, att)))
            break;
        if ((rc = mv(pool, OR_BF16, b->wo, att, H, Dq, proj))) break;
        or_add(h, proj, H, h);
        /* ---- MoE FFN (moe.rs:2074-2427) ---- */
        or_rmsnorm(h, b->ffn_norm, 1, H, c->eps, x);
        if (pool) {
            uint32_t idx[HX_MAX_EXPERTS];
            float w[HX_MAX_EXPERTS];
            const uint8_t *g[HX_MAX_EXPERTS], *u[HX_MAX_EXPERTS], *d[HX_MAX_EXPERTS];
            if ((rc = mv(pool, OR_F32, b->router, x, E, H, logits))) break;
            if ((rc = or_topk_router(logits, 1, E, c->k, c->gating, idx, w))) break;
            const int bb = or_block_bytes(c->wtype);
            const size_t gb = c->n_ff * (H / 32) * (size_t)bb, db = H * (c->n_ff / 32) * (size_t)bb;
            for (unsigned m = 0; m < c->k; ++m) {
                g[m] = b->gate + idx[m] * gb;
                u[m] = b->up + idx[m] * gb;
                d[m] = b->down + idx[m] * db;
            }
            if ((rc = hx_ffn(pool, c->wtype, H, c->n_ff, c->k, g, u, d, w, x, (int)c->act,
                             c->alpha, c->limit, ffn)))
                break;
            if (idx_out) memcpy(idx_out + l * c->k, idx, sizeof(uint32_t) * c->k);
        } else {
            if (margin_out) {
                or_matvec_f32(b->router, x, E, H, logits);
                margin_out[l] = topk_margin(logits, E, c->k);
            }
            if ((rc = or_moe_ffn_token(&mc, x, b->router, NULL, b->gate, b->up, b->down, NULL,
                                       NULL, NULL, ffn, idx_out ? idx_out + l * c->k : NULL,
                                       NULL)))
                break;
        }
        or_add(h, ffn, H, h);
    }
    free(x);
    free(q);
    free(qr);
    free(k);
    free(kr);
    free(v);
    free(att);
    free(proj);
    free(ffn);
    free(logits);
    return rc;
}

int cd_layers(const cd_cfg *c, const cd_layer *L, size_t l0, size_t l1, float *h, size_t pos,
              hx_pool *pool, uint32_t *idx_out) {
    return layers_impl(c, L, l0, l1, h, pos, pool, idx_out, NULL);
}

int cd_step_margins(const cd_cfg *c, const cd_layer *layers, const float *output_norm,
                    const float *h_in, size_t pos, float *out, uint32_t *idx_out, float *margin_out) {
    float *h = (float *)malloc(sizeof(float) * c->n_embd);
    memcpy(h, h_in, sizeof(float) * c->n_embd);
    int rc = layers_impl(c, layers, 0, c->n_layer, h, pos, NULL, idx_out, margin_out);
    if (!rc) or_rmsnorm(h, output_norm, 1, c->n_embd, c->eps, out);
    free(h);
    return rc;
}

int cd_step(const cd_cfg *c, const cd_layer *layers, const float *output_norm, const float *h_in,
            size_t pos, hx_pool *pool, float *out, uint32_t *idx_out) {
    float *h = (float *)malloc(sizeof(float) * c->n_embd);
    memcpy(h, h_in, sizeof(float) * c->n_embd);
    int rc = layers_impl(c, layers, 0, c->n_layer, h, pos, pool, idx_out, NULL);
    if (!rc) or_rmsnorm(h, output_norm, 1, c->n_embd, c->eps, out);
    free(h);
    return rc;
}

int cd_logits(const cd_cfg *c, const uint16_t *w_out, size_t n_vocab, const float *x, float *logits) {
    if (!c || !w_out || !x || !logits) return -1;
    return or_matvec_q(OR_BF16, (const uint8_t *)w_out, x, n_vocab, c->n_embd, logits);
}
