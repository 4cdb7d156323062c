/*
 * host_experts.c — restatement of MoEArc's CPU expert path, for the timed CPU baseline.
 *
 * TEST / BENCH INFRASTRUCTURE ONLY. This is the reference's own CPU implementation of the MoE
 * FFN (crates/moearc-engine/src/host_experts.rs), restated in C because no Rust toolchain is
 * available: a pool of n-1 worker threads pinned from core 1 (host_experts.rs:445-456,
 * 928-940), an epoch fork-join handshake (submit 624-714, worker 786-825, sync 717-761), two
 * phases per job — phase A computes gate and up fused straight into the activation, the last
 * finisher releases phase B, phase B computes the down rows (run_job 827-923) — and the
 * combine in router order on the calling thread (sync 746-760).
 *
 * The row kernels follow host_experts.rs term for term: dot_mxfp4 keeps two accumulators per
 * 32-block, one per nibble half, and scales their sum once per block (1088-1103); the row
 * bodies are compiled twice, once for the baseline target and once with AVX2+FMA, and chosen
 * at run time (1186-1235). Q4_0 has no CPU kernel in the reference; dot_q4_0 below is written
 * in the same style and is labelled a restatement. bf16/f32 rows (the dense projections the
 * CPU decoder needs) use eight independent accumulators, the reference's own device for
 * letting the compiler vectorise a float sum (host_experts.rs:1019-1025).
 */
#define _GNU_SOURCE
#include "host_experts.h"

#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include "moearc_oracle.h"

/* ---- row kernels ---------------------------------------------------------------------- */

static inline float e8m0_half(uint8_t x) {
    uint32_t bits = (x < 2) ? (0x00200000u << x) : ((uint32_t)(x - 1) << 23);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline float ld_f16(const uint8_t *p) { return or_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

#define ROW_KERNELS(SUFFIX, ATTR)                                                              \
    ATTR static float dot_mxfp4##SUFFIX(const uint8_t *w, const float *x, size_t nb) {         \
        float acc = 0.0f;                                                                      \
        for (size_t b = 0; b < nb; ++b) {                                                      \
            const uint8_t *blk = w + b * 17;                                                   \
            const float d = e8m0_half(blk[0]);                                                 \
            const float *xs = x + b * 32;                                                      \
            float lo = 0.0f, hi = 0.0f;                                                        \
            for (int l = 0; l < 16; ++l) {                                                     \
                const uint8_t byte = blk[1 + l];                                               \
                lo += (float)OR_KVALUES_MXFP4[byte & 0x0F] * xs[l];                            \
                hi += (float)OR_KVALUES_MXFP4[byte >> 4] * xs[l + 16];                         \
            }                                                                                  \
            acc += d * (lo + hi);                                                              \
        }                                                                                      \
        return acc;                                                                            \
    }                                                                                          \
    ATTR static float dot_q4_0##SUFFIX(const uint8_t *w, const float *x, size_t nb) {          \
        float acc = 0.0f;                                                                      \
        for (size_t b = 0; b < nb; ++b) {                                                      \
            const uint8_t *blk = w + b * 18;                                                   \
            const float d = ld_f16(blk);                                                       \
            const float *xs = x + b * 32;                                                      \
            float lo = 0.0f, hi = 0.0f;                                                        \
            for (int l = 0; l < 16; ++l) {                                                     \
                const uint8_t byte = blk[2 + l];                                               \
                lo += (float)((int)(byte & 0x0F) - 8) * xs[l];                                 \
                hi += (float)((int)(byte >> 4) - 8) * xs[l + 16];                              \
            }                                                                                  \
            acc += d * (lo + hi);                                                              \
        }                                                                                      \
        return acc;                                                                            \
    }                                                                                          \
    ATTR static float dot_bf16##SUFFIX(const uint8_t *w, const float *x, size_t n) {           \
        const uint16_t *h = (const uint16_t *)w;                                               \
        float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};                                                 \
        size_t c = 0;                                                                          \
        for (; c + 8 <= n; c += 8)                                                             \
            for (int l = 0; l < 8; ++l) {                                                      \
                uint32_t bits = (uint32_t)h[c + l] << 16;                                      \
                float wv;                                                                      \
                memcpy(&wv, &bits, 4);                                                         \
                a[l] += wv * x[c + l];                                                         \
            }                                                                                  \
        float s = 0.0f;                                                                        \
        for (int l = 0; l < 8; ++l) s += a[l];                                                 \
        for (; c < n; ++c) {                                                                   \
            uint32_t bits = (uint32_t)h[c] << 16;                                              \
            float wv;                                                                          \
            memcpy(&wv, &bits, 4);                                                             \
            s += wv * x[c];                                                                    \
        }                                                                                      \
        return s;                                                                              \
    }                                                                                          \
    ATTR static float dot_f32##SUFFIX(const uint8_t *w, const float *x, size_t n) {            \
        const float *f = (const float *)w;                                                     \
        float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};                                                 \
        size_t c = 0;                                                                          \
        for (; c + 8 <= n; c += 8)                                                             \
            for (int l = 0; l < 8; ++l) a[l] += f[c + l] * x[c + l];                           \
        float s = 0.0f;                                                                        \
        for (int l = 0; l < 8; ++l) s += a[l];                                                 \
        for (; c < n; ++c) s += f[c] * x[c];                                                   \
        return s;                                                                              \
    }                                                                                          \
    ATTR static float dot_row##SUFFIX(unsigned t, const uint8_t *row, const float *x,          \
                                      size_t n_cols) {                                         \
        switch (t) {                                                                           \
        case OR_MXFP4: return dot_mxfp4##SUFFIX(row, x, n_cols / 32);                          \
        case OR_Q4_0: return dot_q4_0##SUFFIX(row, x, n_cols / 32);                            \
        case OR_BF16: return dot_bf16##SUFFIX(row, x, n_cols);                                 \
        case OR_F32: return dot_f32##SUFFIX(row, x, n_cols);                                   \
        default: return NAN; /* unreachable: hx_* refuse other types up front */              \
        }                                                                                      \
    }                                                                                          \
    ATTR static void swiglu_rows##SUFFIX(unsigned t, const uint8_t *g, const uint8_t *u,       \
                                         size_t rb, const float *x, size_t n_cols, size_t r0,  \
                                         size_t r1, float *act, int activation, float alpha,   \
                                         float limit) {                                        \
        for (size_t r = r0; r < r1; ++r) {                                                     \
            const float gv = dot_row##SUFFIX(t, g + r * rb, x, n_cols);                        \
            const float uv = dot_row##SUFFIX(t, u + r * rb, x, n_cols);                        \
            if (activation == 1) {                                                             \
                const float xg = fminf(gv, limit);                                             \
                float yu = uv < -limit ? -limit : (uv > limit ? limit : uv);                   \
                act[r - r0] = (xg / (1.0f + expf(alpha * -xg))) * (yu + 1.0f);                 \
            } else {                                                                           \
                act[r - r0] = (gv / (1.0f + expf(-gv))) * uv;                                  \
            }                                                                                  \
        }                                                                                      \
    }                                                                                          \
    ATTR static void matvec_rows##SUFFIX(unsigned t, const uint8_t *w, size_t rb,              \
                                         const float *x, size_t n_cols, size_t r0, size_t r1,  \
                                         float *out) {                                         \
        for (size_t r = r0; r < r1; ++r) out[r - r0] = dot_row##SUFFIX(t, w + r * rb, x, n_cols); \
    }

ROW_KERNELS(_base, )
ROW_KERNELS(_avx2, __attribute__((target("avx2,fma"))))

static int have_avx2(void) {
    static int cached = -1;
    if (cached < 0) {
        __builtin_cpu_init();
        cached = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
    }
    return cached;
}

static void swiglu_rows(unsigned t, const uint8_t *g, const uint8_t *u, size_t rb, const float *x,
                        size_t n_cols, size_t r0, size_t r1, float *act, int a, float al,
                        float li) {
    if (have_avx2()) swiglu_rows_avx2(t, g, u, rb, x, n_cols, r0, r1, act, a, al, li);
    else swiglu_rows_base(t, g, u, rb, x, n_cols, r0, r1, act, a, al, li);
}

static void matvec_rows(unsigned t, const uint8_t *w, size_t rb, const float *x, size_t n_cols,
                        size_t r0, size_t r1, float *out) {
    if (have_avx2()) matvec_rows_avx2(t, w, rb, x, n_cols, r0, r1, out);
    else matvec_rows_base(t, w, rb, x, n_cols, r0, r1, out);
}

static size_t row_bytes(unsigned t, size_t n_cols) {
    switch (t) {
    case OR_MXFP4: return n_cols / 32 * 17;
    case OR_Q4_0: return n_cols / 32 * 18;
    case OR_BF16: return n_cols * 2;
    case OR_F32: return n_cols * 4;
    default: return 0;
    }
}

/* ---- the pool ------------------------------------------------------------------------- */

enum { JOB_FFN = 1, JOB_MATVEC = 2 };

struct hx_pool {
    int n_threads;
    pthread_t *threads;
    atomic_int stop;
    atomic_ulong epoch;
    atomic_ulong *acks;
    pthread_mutex_t mu;
    pthread_cond_t cv;
    /* the job in flight, written by the submitter before the epoch bump */
    int kind;
    unsigned wtype;
    size_t n_embd, n_ff, n_exp;
    const uint8_t *banks[HX_MAX_EXPERTS][3];
    const float *x;
    int act;
    float alpha, limit;
    size_t chunk_a, chunks_a, chunk_b, chunks_b;
    atomic_size_t cursor_a, cursor_b, done_a;
    atomic_int gate_b;
    float *act_buf; /* [HX_MAX_EXPERTS * n_ff] */
    float *out_buf; /* [HX_MAX_EXPERTS * n_embd] */
    size_t cap_ff, cap_embd;
    /* JOB_MATVEC */
    const uint8_t *mv_w;
    float *mv_out;
    size_t mv_rows, mv_cols;
};

static void pin_to_core(int core) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    cpu_set_t set;
    CPU_ZERO(&set);
    CPU_SET(core % n, &set);
    pthread_setaffinity_np(pthread_self(), sizeof(set), &set); /* best effort */
}

static void run_job(hx_pool *p) {
    if (p->kind == JOB_MATVEC) {
        const size_t rb = row_bytes(p->wtype, p->mv_cols);
        for (;;) {
            const size_t i = atomic_fetch_add_explicit(&p->cursor_a, 1, memory_order_relaxed);
            if (i >= p->chunks_a) break;
            const size_t r0 = i * p->chunk_a;
            size_t r1 = r0 + p->chunk_a;
            if (r1 > p->mv_rows) r1 = p->mv_rows;
            matvec_rows(p->wtype, p->mv_w, rb, p->x, p->mv_cols, r0, r1, p->mv_out + r0);
        }
        return;
    }
    const size_t total_a = p->n_exp * p->chunks_a, total_b = p->n_exp * p->chunks_b;
    const size_t rb_a = row_bytes(p->wtype, p->n_embd), rb_b = row_bytes(p->wtype, p->n_ff);
    /* phase A: gate and up, fused into the activation */
    for (;;) {
        const size_t i = atomic_fetch_add_explicit(&p->cursor_a, 1, memory_order_relaxed);
        if (i >= total_a) break;
        const size_t e = i / p->chunks_a, c = i % p->chunks_a;
        const size_t r0 = c * p->chunk_a;
        size_t r1 = r0 + p->chunk_a;
        if (r1 > p->n_ff) r1 = p->n_ff;
        swiglu_rows(p->wtype, p->banks[e][0], p->banks[e][1], rb_a, p->x, p->n_embd, r0, r1,
                    p->act_buf + e * p->n_ff + r0, p->act, p->alpha, p->limit);
        if (atomic_fetch_add_explicit(&p->done_a, 1, memory_order_acq_rel) + 1 == total_a)
            atomic_store_explicit(&p->gate_b, 1, memory_order_release);
    }
    /* the barrier: every activation row exists before any down row reads it */
    while (!atomic_load_explicit(&p->gate_b, memory_order_acquire)) {
        if (atomic_load_explicit(&p->stop, memory_order_relaxed)) return;
        __builtin_ia32_pause();
    }
    /* phase B: the down projection */
    for (;;) {
        const size_t i = atomic_fetch_add_explicit(&p->cursor_b, 1, memory_order_relaxed);
        if (i >= total_b) break;
        const size_t e = i / p->chunks_b, c = i % p->chunks_b;
        const size_t r0 = c * p->chunk_b;
        size_t r1 = r0 + p->chunk_b;
        if (r1 > p->n_embd) r1 = p->n_embd;
        matvec_rows(p->wtype, p->banks[e][2], rb_b, p->act_buf + e * p->n_ff, p->n_ff, r0, r1,
                    p->out_buf + e * p->n_embd + r0);
    }
}

typedef struct {
    hx_pool *p;
    int id;
} worker_arg;

static void *worker(void *arg) {
    worker_arg *wa = (worker_arg *)arg;
    hx_pool *p = wa->p;
    const int id = wa->id;
    free(wa);
    pin_to_core(id + 1); /* core 0 is left to the submitting thread */
    unsigned long seen = 0;
    for (;;) {
        unsigned long spins = 0;
        for (;;) {
            const unsigned long e = atomic_load_explicit(&p->epoch, memory_order_acquire);
            if (e != seen) {
                seen = e;
                break;
            }
            if (atomic_load_explicit(&p->stop, memory_order_relaxed)) return NULL;
            if (++spins > 2000000ul) {
                pthread_mutex_lock(&p->mu);
                if (atomic_load_explicit(&p->epoch, memory_order_acquire) == seen &&
                    !atomic_load_explicit(&p->stop, memory_order_relaxed)) {
                    struct timespec ts;
                    clock_gettime(CLOCK_REALTIME, &ts);
                    ts.tv_nsec += 50 * 1000 * 1000;
                    if (ts.tv_nsec >= 1000000000) {
                        ts.tv_sec += 1;
                        ts.tv_nsec -= 1000000000;
                    }
                    pthread_cond_timedwait(&p->cv, &p->mu, &ts);
                }
                pthread_mutex_unlock(&p->mu);
                spins = 0;
            } else {
                __builtin_ia32_pause();
            }
        }
        if (atomic_load_explicit(&p->stop, memory_order_relaxed)) return NULL;
        run_job(p);
        atomic_store_explicit(&p->acks[id], seen, memory_order_release);
    }
}

int hx_default_threads(void) {
    const char *env = getenv("MOEARC_HOST_THREADS");
    if (env && atoi(env) > 0) return atoi(env);
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 1 ? (int)(n - 1) : 1;
}

hx_pool *hx_create(int n_threads) {
    if (n_threads <= 0) n_threads = hx_default_threads();
    hx_pool *p = (hx_pool *)calloc(1, sizeof(hx_pool));
    if (!p) return NULL;
    p->n_threads = n_threads;
    p->threads = (pthread_t *)calloc((size_t)n_threads, sizeof(pthread_t));
    p->acks = (atomic_ulong *)calloc((size_t)n_threads, sizeof(atomic_ulong));
    pthread_mutex_init(&p->mu, NULL);
    pthread_cond_init(&p->cv, NULL);
    atomic_init(&p->stop, 0);
    atomic_init(&p->epoch, 0);
    for (int i = 0; i < n_threads; ++i) {
        worker_arg *wa = (worker_arg *)malloc(sizeof(worker_arg));
        wa->p = p;
        wa->id = i;
        pthread_create(&p->threads[i], NULL, worker, wa);
    }
    return p;
}

void hx_destroy(hx_pool *p) {
    if (!p) return;
    atomic_store_explicit(&p->stop, 1, memory_order_release);
    atomic_fetch_add_explicit(&p->epoch, 1, memory_order_release);
    pthread_mutex_lock(&p->mu);
    pthread_cond_broadcast(&p->cv);
    pthread_mutex_unlock(&p->mu);
    for (int i = 0; i < p->n_threads; ++i) pthread_join(p->threads[i], NULL);
    free(p->threads);
    free((void *)p->acks);
    free(p->act_buf);
    free(p->out_buf);
    pthread_mutex_destroy(&p->mu);
    pthread_cond_destroy(&p->cv);
    free(p);
}

int hx_threads(const hx_pool *p) { return p ? p->n_threads : 0; }

/* Publish the job, wake the workers, and wait for every acknowledgement. */
static void fork_join(hx_pool *p) {
    atomic_store_explicit(&p->cursor_a, 0, memory_order_relaxed);
    atomic_store_explicit(&p->cursor_b, 0, memory_order_relaxed);
    atomic_store_explicit(&p->done_a, 0, memory_order_relaxed);
    atomic_store_explicit(&p->gate_b, 0, memory_order_relaxed);
    const unsigned long ep = atomic_fetch_add_explicit(&p->epoch, 1, memory_order_release) + 1;
    pthread_mutex_lock(&p->mu);
    pthread_cond_broadcast(&p->cv);
    pthread_mutex_unlock(&p->mu);
    for (int i = 0; i < p->n_threads; ++i)
        while (atomic_load_explicit(&p->acks[i], memory_order_acquire) < ep) __builtin_ia32_pause();
}

/* Rows per task: a couple of tasks per thread, at least 16 rows, at most one expert's rows
 * (host_experts.rs:677-682, 771-774). */
static size_t chunk_for(size_t total_rows, size_t target, size_t rows_per_expert) {
    size_t c = (total_rows + target - 1) / (target ? target : 1);
    if (c < 16) c = 16;
    if (c > rows_per_expert) c = rows_per_expert;
    return c ? c : 1;
}

int hx_ffn(hx_pool *p, unsigned wtype, size_t n_embd, size_t n_ff, unsigned n_exp,
           const uint8_t *const *gate, const uint8_t *const *up, const uint8_t *const *down,
           const float *weights, const float *x, int act, float alpha, float limit, float *out) {
    if (!p || !x || !out) return -1;
    if (n_exp > HX_MAX_EXPERTS) return -2;
    if (wtype != OR_MXFP4 && wtype != OR_Q4_0) return -2;
    if (n_embd % 32 || n_ff % 32) return -2;
    if (p->cap_ff < n_ff || p->cap_embd < n_embd) {
        free(p->act_buf);
        free(p->out_buf);
        p->act_buf = (float *)malloc(sizeof(float) * HX_MAX_EXPERTS * n_ff);
        p->out_buf = (float *)malloc(sizeof(float) * HX_MAX_EXPERTS * n_embd);
        p->cap_ff = n_ff;
        p->cap_embd = n_embd;
    }
    p->kind = JOB_FFN;
    p->wtype = wtype;
    p->n_embd = n_embd;
    p->n_ff = n_ff;
    p->n_exp = n_exp;
    for (unsigned e = 0; e < n_exp; ++e) {
        p->banks[e][0] = gate[e];
        p->banks[e][1] = up[e];
        p->banks[e][2] = down[e];
    }
    p->x = x;
    p->act = act;
    p->alpha = alpha;
    p->limit = limit;
    const size_t target = (size_t)p->n_threads * 2;
    p->chunk_a = chunk_for(n_exp * n_ff, target, n_ff);
    p->chunk_b = chunk_for(n_exp * n_embd, target, n_embd);
    p->chunks_a = (n_ff + p->chunk_a - 1) / p->chunk_a;
    p->chunks_b = (n_embd + p->chunk_b - 1) / p->chunk_b;
    if (n_exp) fork_join(p);
    /* The combine, in router order, on the calling thread (host_experts.rs:746-760). */
    for (size_t i = 0; i < n_embd; ++i) out[i] = 0.0f;
    for (unsigned e = 0; e < n_exp; ++e) {
        const float *part = p->out_buf + (size_t)e * n_embd;
        for (size_t i = 0; i < n_embd; ++i) out[i] += weights[e] * part[i];
    }
    return 0;
}

int hx_matvec(hx_pool *p, unsigned wtype, const uint8_t *w, const float *x, size_t n_rows,
              size_t n_cols, float *out) {
    if (!p || !w || !x || !out) return -1;
    if (!row_bytes(wtype, n_cols)) return -2;
    if ((wtype == OR_MXFP4 || wtype == OR_Q4_0) && n_cols % 32) return -2;
    p->kind = JOB_MATVEC;
    p->wtype = wtype;
    p->mv_w = w;
    p->mv_out = out;
    p->mv_rows = n_rows;
    p->mv_cols = n_cols;
    p->x = x;
    p->chunk_a = chunk_for(n_rows, (size_t)p->n_threads * 2, n_rows);
    p->chunks_a = (n_rows + p->chunk_a - 1) / p->chunk_a;
    if (n_rows) fork_join(p);
    return 0;
}
