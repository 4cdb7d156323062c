/*
 * host_experts.h — the reference's CPU expert path, restated (see host_experts.c).
 * TEST / BENCH INFRASTRUCTURE ONLY: the shipped library never links or calls this.
 */
#ifndef MOEARC_HOST_EXPERTS_H
#define MOEARC_HOST_EXPERTS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HX_MAX_EXPERTS 32

typedef struct hx_pool hx_pool;

/* nproc - 1, or MOEARC_HOST_THREADS (host_experts.rs:451-456). */
int hx_default_threads(void);
hx_pool *hx_create(int n_threads);
void hx_destroy(hx_pool *p);
int hx_threads(const hx_pool *p);

/* One token through n_exp experts: out = sum over e (router order) of weights[e] *
 * down_e . act(gate_e . x, up_e . x). Banks are GGUF row layout, MXFP4 or Q4_0.
 * act: 0 SwiGLU, 1 SwiGLU-OAI(alpha, limit). Returns 0, -1 (null), -2 (bad argument). */
int hx_ffn(hx_pool *p, unsigned wtype, size_t n_embd, size_t n_ff, unsigned n_exp,
           const uint8_t *const *gate, const uint8_t *const *up, const uint8_t *const *down,
           const float *weights, const float *x, int act, float alpha, float limit, float *out);

/* out = W . x over the pool; W is n_rows rows of MXFP4, Q4_0, BF16 or F32. */
int hx_matvec(hx_pool *p, unsigned wtype, const uint8_t *w, const float *x, size_t n_rows,
              size_t n_cols, float *out);

#ifdef __cplusplus
}
#endif
#endif
