/*
 * moearc_oracle.c — CPU restatement of MoEArc's CPU twin for the MoE decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see moearc_oracle.h). Written from the reference's stated
 * semantics; every function names the lines of crates/moearc-kernels/src/reference.rs or
 * crates/moearc-kernels/kernels.cpp whose arithmetic it restates. Compile with
 * -ffp-contract=off so that float expressions round exactly as written.
 */
#include "moearc_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>
#include <unistd.h>

/* ---- row-parallel loops ------------------------------------------------------------------
 * Large matvecs and attention spread their rows (heads) over host threads. Rows are
 * independent and each keeps its own sequential sum, so the split changes no result; it only
 * makes full-size parity checks finish in seconds. Calls below 2^20 multiply-adds stay on the
 * calling thread. MOEARC_ORACLE_THREADS caps the count. */
typedef void (*or_rows_fn)(void *arg, size_t r0, size_t r1, int tid);

struct or_chunk {
    or_rows_fn fn;
    void *arg;
    size_t r0, r1;
    int tid;
};

static void *or_chunk_run(void *p) {
    struct or_chunk *c = (struct or_chunk *)p;
    c->fn(c->arg, c->r0, c->r1, c->tid);
    return NULL;
}

static int or_threads(size_t work) {
    if (work < ((size_t)1 << 20)) return 1;
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    const char *e = getenv("MOEARC_ORACLE_THREADS");
    if (e && atoi(e) > 0) n = atoi(e);
    return n < 1 ? 1 : (n > 64 ? 64 : (int)n);
}

/* fn over [0, n) in nt contiguous chunks (chunk i on thread i; thread 0 is the caller). */
static void or_parallel(size_t n, int nt, or_rows_fn fn, void *arg) {
    if (nt > (int)n) nt = n ? (int)n : 1;
    if (nt <= 1) {
        fn(arg, 0, n, 0);
        return;
    }
    struct or_chunk ch[64];
    pthread_t th[64];
    int started[64] = {0};
    for (int i = 0; i < nt; ++i) {
        ch[i] = (struct or_chunk){fn, arg, n * (size_t)i / (size_t)nt, n * (size_t)(i + 1) / (size_t)nt, i};
        if (i > 0) started[i] = pthread_create(&th[i], NULL, or_chunk_run, &ch[i]) == 0;
    }
    fn(arg, ch[0].r0, ch[0].r1, 0);
    for (int i = 1; i < nt; ++i) {
        if (started[i]) pthread_join(th[i], NULL);
        else fn(arg, ch[i].r0, ch[i].r1, 0); /* no thread: run it here (buffer 0 is free now) */
    }
}

/* ====================================================================================== */
/* scalar formats                                                                          */
/* ====================================================================================== */

static inline float bits_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static inline uint32_t f32_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

/* binary16 -> binary32, exact (reference.rs:123-149). Subnormal halves are renormalised by
 * shifting the mantissa up until its implicit bit appears. */
float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int shift = 0;
            while (!(m & 0x400u)) {
                m <<= 1;
                ++shift;
            }
            m &= 0x3FFu;
            /* value = 1.m * 2^(-14 - shift) */
            bits = sign | ((uint32_t)(127 - 14 - shift) << 23) | (m << 13);
        }
    } else if (e == 0x1F) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + (127 - 15)) << 23) | (m << 13);
    }
    return bits_f32(bits);
}

/* binary32 -> binary16, round to nearest even, subnormals rounded, overflow to infinity,
 * NaN stays NaN (reference.rs:647-691). */
uint16_t or_f32_to_f16(float f) {
    uint32_t x = f32_bits(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t e32 = (x >> 23) & 0xFFu;
    uint32_t mant = x & 0x7FFFFFu;
    if (e32 == 0xFF) {
        return (uint16_t)(sign | 0x7C00u | (mant ? (0x0200u | (mant >> 13)) : 0u));
    }
    int e = (int)e32 - 127 + 15;
    if (e >= 0x1F) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t full = mant | 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t t = full >> shift;
        uint32_t rem = full & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (t & 1u))) ++t; /* a carry lands in the exponent */
        return (uint16_t)(sign | t);
    }
    uint32_t t = mant >> 13;
    uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (t & 1u))) {
        ++t;
        if (t == 0x400u) {
            t = 0;
            ++e;
            if (e >= 0x1F) return (uint16_t)(sign | 0x7C00u);
        }
    }
    return (uint16_t)(sign | ((uint32_t)e << 10) | t);
}

float or_bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

/* bf16 is the top half of binary32. Round to nearest even on the discarded half; a NaN keeps
 * its sign and top payload bits and is forced quiet so it cannot collapse to infinity. */
uint16_t or_f32_to_bf16(float f) {
    uint32_t x = f32_bits(f);
    if ((x & 0x7F800000u) == 0x7F800000u && (x & 0x7FFFFFu)) {
        return (uint16_t)((x >> 16) | 0x0040u);
    }
    uint32_t lsb = (x >> 16) & 1u;
    return (uint16_t)((x + 0x7FFFu + lsb) >> 16);
}

/* ggml_e8m0_to_fp32_half: 2^(x-128). Exponent bytes 0 and 1 give subnormal floats and take
 * their own arm (reference.rs:66-70). */
float or_e8m0_half(uint8_t x) {
    uint32_t bits = (x < 2) ? (0x00200000u << x) : ((uint32_t)(x - 1) << 23);
    return bits_f32(bits);
}

/* E2M1 values doubled so the table is integral; the halved scale above undoes the doubling
 * (reference.rs:51-56). Index 8 is negative zero. */
const int8_t OR_KVALUES_MXFP4[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

/* ====================================================================================== */
/* block formats                                                                           */
/* ====================================================================================== */

int or_block_bytes(unsigned t) {
    switch (t) {
    case OR_F32: return 4;
    case OR_F16: return 2;
    case OR_BF16: return 2;
    case OR_Q4_0: return 18;  /* f16 delta + 16 bytes of nibble pairs */
    case OR_Q8_0: return 34;  /* f16 delta + 32 signed bytes */
    case OR_MXFP4: return 17; /* e8m0 byte + 16 bytes of nibble pairs */
    case OR_Q4_K: return 144; /* d, dmin, 12 scale bytes, 128 nibble bytes (reference.rs:74-89) */
    case OR_Q5_K: return 176; /* as Q4_K plus 32 high-bit bytes */
    case OR_Q6_K: return 210; /* 128 low nibbles, 64 high-pair bytes, 16 int8 scales, d */
    default: return 0;
    }
}

int or_block_elems(unsigned t) {
    switch (t) {
    case OR_F32:
    case OR_F16:
    case OR_BF16: return 1;
    case OR_Q4_0:
    case OR_Q8_0:
    case OR_MXFP4: return 32;
    case OR_Q4_K:
    case OR_Q5_K:
    case OR_Q6_K: return 256; /* QK_K super-blocks (reference.rs:42, 93-100) */
    default: return 0;
    }
}

static inline float ld_f16(const uint8_t *p) { return or_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* The 6-bit scale and min of sub-block j of a Q4_K / Q5_K super-block from its 12 packed
 * bytes (ggml's get_scale_min_k4, reference.rs:154-160): sub-blocks 0-3 keep theirs in the
 * low six bits of bytes j and j+4; 4-7 take four bits from bytes j+4 and the top two of bytes
 * j-4 and j. */
static void scale_min_k4(const uint8_t *q, int j, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* A Q4_K (hb = 0) or Q5_K (hb = 1) super-block (reference.rs:218-276): four 64-element runs,
 * each two 32-element sub-blocks sharing the run's 32 nibble bytes (low nibbles first); an
 * element is (d * scale) * q - (dmin * min), with Q5_K adding 16 to q when its bit in the
 * run's high-bit plane is set. */
static void dequant_kq45(const uint8_t *b, float *y, int hb) {
    const float d = ld_f16(b), dmin = ld_f16(b + 2);
    const uint8_t *scales = b + 4;
    const uint8_t *qh = b + 16;
    const uint8_t *qs = b + (hb ? 48 : 16);
    for (int run = 0; run < 4; ++run) {
        for (int half = 0; half < 2; ++half) {
            uint8_t sc, m;
            scale_min_k4(scales, 2 * run + half, &sc, &m);
            const float d1 = d * (float)sc, m1 = dmin * (float)m;
            const uint8_t bit = (uint8_t)(1u << (2 * run + half));
            for (int l = 0; l < 32; ++l) {
                const uint8_t byte = qs[32 * run + l];
                int q = half ? (byte >> 4) : (byte & 0xF);
                if (hb && (qh[l] & bit)) q += 16;
                y[64 * run + 32 * half + l] = d1 * (float)q - m1;
            }
        }
    }
}

/* A Q6_K super-block (reference.rs:278-300): two 128-element halves; element l of quarter k of
 * a half takes four low bits from byte l (k even) or l + 32 (k odd) of the half's 64 low-nibble
 * bytes (low nibble for k < 2, high for k >= 2) and two high bits from bits 2k..2k+1 of byte l
 * of the half's 32 high bytes; q - 32 is scaled by d times int8 scale 2k + l/16 of the half. */
static void dequant_q6k(const uint8_t *b, float *y) {
    const float d = ld_f16(b + 208);
    for (int n = 0; n < 2; ++n) {
        const uint8_t *ql = b + 64 * n, *qh = b + 128 + 32 * n;
        const int8_t *sc = (const int8_t *)(b + 192 + 8 * n);
        for (int k = 0; k < 4; ++k)
            for (int l = 0; l < 32; ++l) {
                const uint8_t lo = ql[l + 32 * (k & 1)];
                const int q = (((k >= 2) ? (lo >> 4) : (lo & 0xF)) | (((qh[l] >> (2 * k)) & 3) << 4)) - 32;
                y[128 * n + 32 * k + l] = d * (float)sc[2 * k + l / 16] * (float)q;
            }
    }
}

/* One block of each format. The nibble formats share one rule: byte j's low nibble is element
 * j and its high nibble is element j+16 — the two halves of the block, not an adjacent pair
 * (reference.rs:202-216 for MXFP4; ggml's dequantize_row_q4_0 for Q4_0). */
static void dequant_block(unsigned t, const uint8_t *b, float *y) {
    switch (t) {
    case OR_F32: memcpy(y, b, 4); break;
    case OR_F16: y[0] = ld_f16(b); break;
    case OR_BF16: y[0] = or_bf16_to_f32((uint16_t)(b[0] | (b[1] << 8))); break;
    case OR_Q8_0: {
        const float d = ld_f16(b);
        for (int j = 0; j < 32; ++j) y[j] = (float)(int8_t)b[2 + j] * d;
        break;
    }
    case OR_Q4_0: {
        const float d = ld_f16(b);
        for (int j = 0; j < 16; ++j) {
            const int lo = (b[2 + j] & 0x0F) - 8;
            const int hi = (b[2 + j] >> 4) - 8;
            y[j] = (float)lo * d;
            y[j + 16] = (float)hi * d;
        }
        break;
    }
    case OR_MXFP4: {
        const float d = or_e8m0_half(b[0]);
        for (int j = 0; j < 16; ++j) {
            y[j] = (float)OR_KVALUES_MXFP4[b[1 + j] & 0x0F] * d;
            y[j + 16] = (float)OR_KVALUES_MXFP4[b[1 + j] >> 4] * d;
        }
        break;
    }
    case OR_Q4_K: dequant_kq45(b, y, 0); break;
    case OR_Q5_K: dequant_kq45(b, y, 1); break;
    case OR_Q6_K: dequant_q6k(b, y); break;
    default: break;
    }
}

int or_dequant(unsigned t, const uint8_t *src, size_t nblocks, float *dst) {
    const int bb = or_block_bytes(t);
    const int be = or_block_elems(t);
    if (!bb) return -2;
    for (size_t i = 0; i < nblocks; ++i) dequant_block(t, src + i * (size_t)bb, dst + i * (size_t)be);
    return 0;
}

/* ====================================================================================== */
/* matvecs                                                                                 */
/* ====================================================================================== */

struct mvq_arg {
    unsigned t;
    int bb;
    size_t nb, n_cols;
    const uint8_t *w;
    const float *x;
    float *out, *rows;
};

static void mvq_rows(void *p, size_t r0, size_t r1, int tid) {
    const struct mvq_arg *a = (const struct mvq_arg *)p;
    float *row = a->rows + (size_t)tid * a->n_cols;
    for (size_t r = r0; r < r1; ++r) {
        or_dequant(a->t, a->w + r * a->nb * (size_t)a->bb, a->nb, row);
        double acc = 0.0;
        for (size_t c = 0; c < a->n_cols; ++c) acc += (double)row[c] * (double)a->x[c];
        a->out[r] = (float)acc;
    }
}

int or_matvec_q(unsigned t, const uint8_t *w, const float *x, size_t n_rows, size_t n_cols,
                float *out) {
    const int bb = or_block_bytes(t);
    const int be = or_block_elems(t);
    if (!bb) return -2;
    if (n_cols % (size_t)be) return -2;
    const int nt = or_threads(n_rows * n_cols);
    float *rows = (float *)malloc((size_t)nt * n_cols * sizeof(float));
    if (!rows) return -1;
    struct mvq_arg a = {t, bb, n_cols / (size_t)be, n_cols, w, x, out, rows};
    or_parallel(n_rows, nt, mvq_rows, &a);
    free(rows);
    return 0;
}

struct mvf_arg {
    const float *w, *x;
    size_t n_cols;
    float *out;
};

static void mvf_rows(void *p, size_t r0, size_t r1, int tid) {
    const struct mvf_arg *a = (const struct mvf_arg *)p;
    (void)tid;
    for (size_t r = r0; r < r1; ++r) {
        double acc = 0.0;
        for (size_t c = 0; c < a->n_cols; ++c) acc += (double)a->w[r * a->n_cols + c] * (double)a->x[c];
        a->out[r] = (float)acc;
    }
}

void or_matvec_f32(const float *w, const float *x, size_t n_rows, size_t n_cols, float *out) {
    struct mvf_arg a = {w, x, n_cols, out};
    or_parallel(n_rows, or_threads(n_rows * n_cols), mvf_rows, &a);
}

void or_matvec_f32_gpu_order(const float *w, const float *x, size_t n_rows, size_t n_cols,
                             float *out) {
    const size_t n4 = (n_cols + 3) / 4;
    for (size_t r = 0; r < n_rows; ++r) {
        const float *wr = w + r * n_cols;
        float p[32];
        for (int l = 0; l < 32; ++l) {
            float acc = 0.0f;
            for (size_t c4 = (size_t)l; c4 < n4; c4 += 32) {
                for (size_t t = 0; t < 4; ++t) {
                    const size_t c = 4 * c4 + t;
                    if (c < n_cols) acc = fmaf(wr[c], x[c], acc);
                }
            }
            p[l] = acc;
        }
        for (int off = 16; off >= 1; off >>= 1) {
            float q[32];
            for (int l = 0; l < 32; ++l) q[l] = p[l] + p[l ^ off];
            memcpy(p, q, sizeof(p));
        }
        out[r] = p[0];
    }
}

/* ====================================================================================== */
/* elementwise / rows                                                                      */
/* ====================================================================================== */

void or_rmsnorm(const float *x, const float *weight, size_t n_rows, size_t n_cols, float eps,
                float *out) {
    for (size_t r = 0; r < n_rows; ++r) {
        const float *row = x + r * n_cols;
        double sum = 0.0;
        for (size_t c = 0; c < n_cols; ++c) sum += (double)row[c] * (double)row[c];
        const float mean = (float)(sum / (double)n_cols);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (size_t c = 0; c < n_cols; ++c) {
            const float s = row[c] * scale;
            out[r * n_cols + c] = weight ? s * weight[c] : s;
        }
    }
}

void or_silu(const float *x, size_t n, float *out) {
    for (size_t i = 0; i < n; ++i) out[i] = x[i] / (1.0f + expf(-x[i]));
}

void or_swiglu(const float *g, const float *u, size_t n, float *out) {
    for (size_t i = 0; i < n; ++i) out[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
}

/* x = min(g, limit) (above only), y = clamp(u, -limit, limit), out = x*sigmoid(alpha*x)*(y+1). */
void or_swiglu_oai(const float *g, const float *u, size_t n, float alpha, float limit,
                   float *out) {
    for (size_t i = 0; i < n; ++i) {
        const float xg = fminf(g[i], limit);
        float yu = u[i];
        if (yu < -limit) yu = -limit;
        if (yu > limit) yu = limit;
        out[i] = (xg / (1.0f + expf(alpha * -xg))) * (yu + 1.0f);
    }
}

void or_softmax_ext(const float *x, const float *mask, size_t n_rows, size_t n_cols, float scale,
                    float *out) {
    for (size_t r = 0; r < n_rows; ++r) {
        const size_t lo = r * n_cols;
        float mx = -INFINITY;
        for (size_t c = 0; c < n_cols; ++c) {
            const float a = x[lo + c] * scale + (mask ? mask[lo + c] : 0.0f);
            mx = fmaxf(mx, a);
        }
        double sum = 0.0;
        for (size_t c = 0; c < n_cols; ++c) {
            const float a = x[lo + c] * scale + (mask ? mask[lo + c] : 0.0f);
            sum += (double)expf(a - mx);
        }
        /* A fully masked row comes back as zeros, not NaN (reference.rs:424-427). */
        const double denom = sum > (double)FLT_MIN ? sum : (double)FLT_MIN;
        for (size_t c = 0; c < n_cols; ++c) {
            const float a = x[lo + c] * scale + (mask ? mask[lo + c] : 0.0f);
            out[lo + c] = (float)((double)expf(a - mx) / denom);
        }
    }
}

void or_add(const float *a, const float *b, size_t n, float *out) {
    for (size_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}
void or_mul(const float *a, const float *b, size_t n, float *out) {
    for (size_t i = 0; i < n; ++i) out[i] = a[i] * b[i];
}
void or_axpy(float *out, const float *x, float alpha, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] += alpha * x[i];
}

void or_moe_combine(const float *parts, const float *w, unsigned n_mat, size_t n, float *out) {
    for (size_t i = 0; i < n; ++i) {
        float acc = 0.0f;
        for (unsigned m = 0; m < n_mat; ++m) acc = fmaf(w[m], parts[(size_t)m * n + i], acc);
        out[i] = acc;
    }
}

void or_add_bias_id(float *out, const float *bias, const uint32_t *idx, unsigned n_mat,
                    size_t n_rows) {
    for (unsigned m = 0; m < n_mat; ++m)
        for (size_t r = 0; r < n_rows; ++r) out[(size_t)m * n_rows + r] += bias[(size_t)idx[m] * n_rows + r];
}

int or_embed_rows(unsigned t, const uint8_t *table, const uint32_t *ids, size_t n_tokens,
                  size_t n_embd, float *out) {
    const int bb = or_block_bytes(t);
    const int be = or_block_elems(t);
    if (!bb || n_embd % (size_t)be) return -2;
    const size_t row_bytes = n_embd / (size_t)be * (size_t)bb;
    for (size_t i = 0; i < n_tokens; ++i)
        or_dequant(t, table + (size_t)ids[i] * row_bytes, n_embd / (size_t)be, out + i * n_embd);
    return 0;
}

/* ====================================================================================== */
/* RoPE                                                                                    */
/* ====================================================================================== */

void or_rope(const float *src, const int32_t *pos, size_t n_tokens, size_t n_heads,
             size_t head_dim, size_t n_dims, float freq_base, int neox, float *out) {
    const float theta_scale = powf(freq_base, -2.0f / (float)n_dims);
    const size_t half = n_dims / 2;
    float *cs = (float *)malloc(sizeof(float) * half * 2);
    memcpy(out, src, sizeof(float) * n_tokens * n_heads * head_dim);
    for (size_t t = 0; t < n_tokens; ++t) {
        float theta = (float)pos[t];
        for (size_t p = 0; p < half; ++p) {
            cs[2 * p] = cosf(theta);
            cs[2 * p + 1] = sinf(theta);
            theta *= theta_scale;
        }
        for (size_t h = 0; h < n_heads; ++h) {
            const size_t base = (t * n_heads + h) * head_dim;
            for (size_t p = 0; p < half; ++p) {
                const size_t lo = neox ? p : 2 * p;
                const size_t hi = neox ? p + half : 2 * p + 1;
                const float x0 = src[base + lo], x1 = src[base + hi];
                const float ct = cs[2 * p], st = cs[2 * p + 1];
                out[base + lo] = x0 * ct - x1 * st;
                out[base + hi] = x0 * st + x1 * ct;
            }
        }
    }
    free(cs);
}

void or_rope_ext(const float *src, const int32_t *pos, size_t n_tokens, size_t n_heads,
                 size_t head_dim, size_t n_dims, float freq_base, float freq_scale,
                 float ext_factor, float attn_factor, float corr_lo, float corr_hi, int neox,
                 float *out) {
    const double theta_scale = pow((double)freq_base, -2.0 / (double)n_dims);
    const size_t half = n_dims / 2;
    memcpy(out, src, sizeof(float) * n_tokens * n_heads * head_dim);
    for (size_t t = 0; t < n_tokens; ++t) {
        for (size_t p = 0; p < half; ++p) {
            const size_t i0 = 2 * p;
            const double theta_extrap = (double)pos[t] * pow(theta_scale, (double)i0 / 2.0);
            double theta = (double)freq_scale * theta_extrap;
            double mscale = attn_factor;
            if (ext_factor != 0.0f) {
                const double den = fmax(0.001, (double)corr_hi - (double)corr_lo);
                const double y = ((double)(i0 / 2) - (double)corr_lo) / den;
                const double ramp = 1.0 - fmin(1.0, fmax(0.0, y));
                const double mix = ramp * (double)ext_factor;
                theta = theta * (1.0 - mix) + theta_extrap * mix;
                mscale *= 1.0 + 0.1 * log(1.0 / (double)freq_scale);
            }
            const double ct = cos(theta) * mscale, st = sin(theta) * mscale;
            for (size_t h = 0; h < n_heads; ++h) {
                const size_t base = (t * n_heads + h) * head_dim;
                const size_t lo = neox ? p : 2 * p;
                const size_t hi = neox ? p + half : 2 * p + 1;
                const double x0 = src[base + lo], x1 = src[base + hi];
                out[base + lo] = (float)(x0 * ct - x1 * st);
                out[base + hi] = (float)(x0 * st + x1 * ct);
            }
        }
    }
}

/* ====================================================================================== */
/* router                                                                                  */
/* ====================================================================================== */

/* Insertion sort of expert ids by logit, descending; equal logits keep ascending id order
 * (the stable sort of reference.rs:613-617). */
static void order_desc(const float *row, size_t n, uint32_t *order) {
    for (size_t i = 0; i < n; ++i) order[i] = (uint32_t)i;
    for (size_t i = 1; i < n; ++i) {
        const uint32_t v = order[i];
        size_t j = i;
        while (j > 0 && row[order[j - 1]] < row[v]) {
            order[j] = order[j - 1];
            --j;
        }
        order[j] = v;
    }
}

int or_topk_router(const float *logits, size_t n_tokens, size_t n_expert, unsigned k,
                   unsigned gating, uint32_t *idx, float *w) {
    if (k == 0 || k > n_expert || gating > 2) return -2;
    float *probs = (float *)malloc(sizeof(float) * n_expert);
    uint32_t *order = (uint32_t *)malloc(sizeof(uint32_t) * n_expert);
    float sel[1024];
    float sw[1024];
    for (size_t t = 0; t < n_tokens; ++t) {
        const float *row = logits + t * n_expert;
        order_desc(row, n_expert, order);
        for (unsigned r = 0; r < k; ++r) idx[t * k + r] = order[r];
        if (gating == OR_GATING_SOFTMAX_AFTER_TOPK) {
            /* A softmax over the k selected logits, not a restriction of the full one. */
            for (unsigned r = 0; r < k; ++r) sel[r] = row[order[r]];
            or_softmax_ext(sel, NULL, 1, k, 1.0f, sw);
            for (unsigned r = 0; r < k; ++r) w[t * k + r] = sw[r];
            continue;
        }
        or_softmax_ext(row, NULL, 1, n_expert, 1.0f, probs);
        float sum = 0.0f;
        for (unsigned r = 0; r < k; ++r) {
            w[t * k + r] = probs[order[r]];
            sum += w[t * k + r];
        }
        if (gating == OR_GATING_SOFTMAX_NORM) {
            const float clamp = 6.103515625e-5f; /* 2^-14, the smallest normal f16 */
            if (sum < clamp) sum = clamp;
            for (unsigned r = 0; r < k; ++r) w[t * k + r] /= sum;
        }
    }
    free(probs);
    free(order);
    return 0;
}

/* ====================================================================================== */
/* paged KV + attention                                                                    */
/* ====================================================================================== */

size_t or_kv_index(uint32_t page, uint32_t slot, size_t head, size_t d, size_t n_kv_heads,
                   size_t head_dim, size_t page_tokens) {
    return (((size_t)page * page_tokens + slot) * n_kv_heads + head) * head_dim + d;
}

float or_kv_store(float v, unsigned t) {
    if (t == OR_F16) return or_f16_to_f32(or_f32_to_f16(v));
    if (t == OR_BF16) return or_bf16_to_f32(or_f32_to_bf16(v));
    return v;
}

static inline float kv_get(const void *base, size_t i, unsigned t) {
    if (t == OR_F16) return or_f16_to_f32(((const uint16_t *)base)[i]);
    if (t == OR_BF16) return or_bf16_to_f32(((const uint16_t *)base)[i]);
    return ((const float *)base)[i];
}

static inline void kv_put(void *base, size_t i, float v, unsigned t) {
    if (t == OR_F16) ((uint16_t *)base)[i] = or_f32_to_f16(v);
    else if (t == OR_BF16) ((uint16_t *)base)[i] = or_f32_to_bf16(v);
    else ((float *)base)[i] = v;
}

int or_kv_append(void *k_pages, void *v_pages, const float *k, const float *v, uint32_t page,
                 uint32_t slot, size_t n_kv_heads, size_t head_dim, size_t page_tokens,
                 unsigned t) {
    if (t != OR_F32 && t != OR_F16 && t != OR_BF16) return -2;
    if (page_tokens == 0 || slot >= page_tokens) return -2;
    for (size_t h = 0; h < n_kv_heads; ++h)
        for (size_t d = 0; d < head_dim; ++d) {
            const size_t i = or_kv_index(page, slot, h, d, n_kv_heads, head_dim, page_tokens);
            kv_put(k_pages, i, k[h * head_dim + d], t);
            kv_put(v_pages, i, v[h * head_dim + d], t);
        }
    return 0;
}

struct attn_arg {
    const float *q;
    const void *k_pages, *v_pages;
    const uint32_t *block_table;
    const float *sinks;
    size_t group, n_kv_heads, head_dim, kv_begin, span, page_tokens;
    float scale;
    unsigned t;
    float *out;
    double *scs;
};

/* Heads h0 .. h1-1 (reference.rs:821-873, the sink seeding of kernels.cpp:1856-1880). */
static void attn_heads(void *p, size_t h0, size_t h1, int tid) {
    const struct attn_arg *a = (const struct attn_arg *)p;
    const size_t span = a->span, head_dim = a->head_dim, page_tokens = a->page_tokens;
    double *sc = a->scs + span * (size_t)tid;
    for (size_t h = h0; h < h1; ++h) {
        const size_t kvh = h / a->group;
        const float *qh = a->q + h * head_dim;
        double mx = a->sinks ? (double)a->sinks[h] : -INFINITY;
        for (size_t i = 0; i < span; ++i) {
            const size_t j = a->kv_begin + i;
            const uint32_t page = a->block_table[j / page_tokens];
            const uint32_t slot = (uint32_t)(j % page_tokens);
            const size_t base = or_kv_index(page, slot, kvh, 0, a->n_kv_heads, head_dim, page_tokens);
            double dot = 0.0;
            for (size_t d = 0; d < head_dim; ++d) dot += (double)qh[d] * (double)kv_get(a->k_pages, base + d, a->t);
            sc[i] = dot * (double)a->scale;
            if (sc[i] > mx) mx = sc[i];
        }
        double denom = a->sinks ? exp((double)a->sinks[h] - mx) : 0.0;
        for (size_t i = 0; i < span; ++i) {
            sc[i] = exp(sc[i] - mx);
            denom += sc[i];
        }
        for (size_t d = 0; d < head_dim; ++d) {
            double acc = 0.0;
            for (size_t i = 0; i < span; ++i) {
                const size_t j = a->kv_begin + i;
                const uint32_t page = a->block_table[j / page_tokens];
                const uint32_t slot = (uint32_t)(j % page_tokens);
                const size_t base = or_kv_index(page, slot, kvh, 0, a->n_kv_heads, head_dim, page_tokens);
                acc += sc[i] * (double)kv_get(a->v_pages, base + d, a->t);
            }
            a->out[h * head_dim + d] = (float)(acc / denom);
        }
    }
}

int or_attn_decode(const float *q, const void *k_pages, const void *v_pages,
                   const uint32_t *block_table, const float *sinks, size_t n_heads,
                   size_t n_kv_heads, size_t head_dim, size_t kv_begin, size_t n_kv,
                   size_t page_tokens, float scale, unsigned t, float *out) {
    if (n_heads == 0 || n_kv_heads == 0 || head_dim == 0 || n_kv == 0 || page_tokens == 0)
        return -2;
    if (n_heads % n_kv_heads) return -2;
    if (kv_begin >= n_kv) return -2;
    const size_t span = n_kv - kv_begin;
    const int nt = or_threads(n_heads * span * head_dim);
    double *scs = (double *)malloc(sizeof(double) * span * (size_t)nt);
    if (!scs) return -1;
    struct attn_arg a = {q, k_pages, v_pages, block_table, sinks, n_heads / n_kv_heads, n_kv_heads,
                         head_dim, kv_begin, span, page_tokens, scale, t, out, scs};
    or_parallel(n_heads, nt, attn_heads, &a);
    free(scs);
    return 0;
}

/* ====================================================================================== */
/* one token's MoE FFN                                                                     */
/* ====================================================================================== */

/* ---- MXFP8 activation quantisation (the prefill perf mode's declared arithmetic) ----------
 * Not in the reference (its engine has no FP8 path): the declared quantisation of the build's
 * MXFP8 prefill mode, restated from the OCP MX format — per 32 consecutive values one E8M0 scale
 * 2^X, X the smallest integer with max|x| / 2^X <= 448 (E4M3's largest finite), the elements
 * E4M3 (1 sign, 4 exponent bits of bias 7, 3 mantissa bits, subnormals down to 2^-9) rounded to
 * nearest even. Returns the dequantised values. */
static float e4m3_rne(float v) {
    const float a = fabsf(v);
    if (a == 0.0f) return v;
    int e;
    frexpf(a, &e); /* a = f * 2^e, f in [0.5, 1) */
    int E = e - 1; /* a = (2f) * 2^E, 2f in [1, 2) */
    if (E < -6) E = -6; /* subnormals: a quantum of 2^-9 */
    const double q = ldexp(1.0, E - 3);
    const double r = (double)a / q; /* in units of the quantum */
    double n = floor(r);
    const double frac = r - n;
    if (frac > 0.5 || (frac == 0.5 && fmod(n, 2.0) != 0.0)) n += 1.0;
    double out = n * q;
    if (out > 448.0) out = 448.0;
    return v < 0 ? (float)-out : (float)out;
}

void or_mx8_quantize(const float *x, size_t n, float *out) {
    for (size_t b = 0; b < n; b += 32) {
        const size_t m = n - b < 32 ? n - b : 32;
        float amax = 0.0f;
        for (size_t i = 0; i < m; ++i) amax = fmaxf(amax, fabsf(x[b + i]));
        int X = 0;
        if (amax > 0.0f) {
            uint32_t bits;
            memcpy(&bits, &amax, 4);
            X = (int)((bits >> 23) & 0xFF) - 127 - 8 + ((bits & 0x7FFFFF) > 0x600000u ? 1 : 0);
            if (X < -127) X = -127;
        }
        for (size_t i = 0; i < m; ++i) out[b + i] = ldexpf(e4m3_rne(ldexpf(x[b + i], -X)), X);
    }
}

int or_moe_ffn_token(const or_moe_cfg *c, const float *x, const float *router_w,
                     const float *router_b, const uint8_t *gate, const uint8_t *up,
                     const uint8_t *down, const float *gate_b, const float *up_b,
                     const float *down_b, float *out, uint32_t *idx_out, float *w_out) {
    const int bb = or_block_bytes(c->wtype);
    const int be = or_block_elems(c->wtype);
    if (!bb || c->n_embd % (size_t)be || c->n_ff % (size_t)be || c->k > 32) return -2;
    const size_t H = c->n_embd, I = c->n_ff, E = c->n_expert;
    const size_t gate_bytes = I * (H / (size_t)be) * (size_t)bb; /* one expert's gate / up */
    const size_t down_bytes = H * (I / (size_t)be) * (size_t)bb; /* one expert's down */
    float *logits = (float *)malloc(sizeof(float) * E);
    float *g = (float *)malloc(sizeof(float) * I);
    float *u = (float *)malloc(sizeof(float) * I);
    float *a = (float *)malloc(sizeof(float) * I);
    float *o = (float *)malloc(sizeof(float) * H * c->k);
    double *acc = (double *)calloc(H, sizeof(double));
    uint32_t idx[32];
    float w[32];
    int rc = 0;

    if (c->router_gpu_order) or_matvec_f32_gpu_order(router_w, x, E, H, logits);
    else or_matvec_f32(router_w, x, E, H, logits);
    /* The router bias goes on before the top-k, so it changes which experts run
     * (moe.rs:2084-2089). */
    if (router_b) or_add(logits, router_b, E, logits);
    rc = or_topk_router(logits, 1, E, c->k, c->gating, idx, w);
    if (rc) goto done;

    for (unsigned m = 0; m < c->k; ++m) {
        const size_t e = idx[m];
        or_matvec_q(c->wtype, gate + e * gate_bytes, x, I, H, g);
        or_matvec_q(c->wtype, up + e * gate_bytes, x, I, H, u);
        /* Per-expert biases before the activation (moe.rs:2310-2331). */
        if (gate_b) or_add(g, gate_b + e * I, I, g);
        if (up_b) or_add(u, up_b + e * I, I, u);
        if (c->act == 1) or_swiglu_oai(g, u, I, c->alpha, c->limit, a);
        else or_swiglu(g, u, I, a);
        or_matvec_q(c->wtype, down + e * down_bytes, a, H, I, o + m * H);
        /* The down bias sits inside the router's weighting (moe.rs:2362-2372). */
        if (down_b) or_add(o + m * H, down_b + e * H, H, o + m * H);
    }
    /* Combine in router order (moe.rs:2374-2386), on the higher-precision side. */
    for (unsigned m = 0; m < c->k; ++m)
        for (size_t i = 0; i < H; ++i) acc[i] += (double)w[m] * (double)o[m * H + i];
    for (size_t i = 0; i < H; ++i) out[i] = (float)acc[i];
    if (idx_out) memcpy(idx_out, idx, sizeof(uint32_t) * c->k);
    if (w_out) memcpy(w_out, w, sizeof(float) * c->k);
done:
    free(logits);
    free(g);
    free(u);
    free(a);
    free(o);
    free(acc);
    return rc;
}

int or_moe_ffn_token_mx8(const or_moe_cfg *c, const float *x, const float *router_w,
                     const float *router_b, const uint8_t *gate, const uint8_t *up,
                     const uint8_t *down, const float *gate_b, const float *up_b,
                     const float *down_b, float *out, uint32_t *idx_out, float *w_out) {
    const int bb = or_block_bytes(c->wtype);
    const int be = or_block_elems(c->wtype);
    if (!bb || c->n_embd % (size_t)be || c->n_ff % (size_t)be || c->k > 32) return -2;
    const size_t H = c->n_embd, I = c->n_ff, E = c->n_expert;
    const size_t gate_bytes = I * (H / (size_t)be) * (size_t)bb; /* one expert's gate / up */
    const size_t down_bytes = H * (I / (size_t)be) * (size_t)bb; /* one expert's down */
    float *logits = (float *)malloc(sizeof(float) * E);
    float *g = (float *)malloc(sizeof(float) * I);
    float *u = (float *)malloc(sizeof(float) * I);
    float *a = (float *)malloc(sizeof(float) * I);
    float *o = (float *)malloc(sizeof(float) * H * c->k);
    float *xq = (float *)malloc(sizeof(float) * H);
    float *aq = (float *)malloc(sizeof(float) * I);
    double *acc = (double *)calloc(H, sizeof(double));
    uint32_t idx[32];
    float w[32];
    int rc = 0;

    if (c->router_gpu_order) or_matvec_f32_gpu_order(router_w, x, E, H, logits);
    else or_matvec_f32(router_w, x, E, H, logits);
    /* The router bias goes on before the top-k, so it changes which experts run
     * (moe.rs:2084-2089). */
    if (router_b) or_add(logits, router_b, E, logits);
    rc = or_topk_router(logits, 1, E, c->k, c->gating, idx, w);
    if (rc) goto done;

    or_mx8_quantize(x, H, xq); /* the routing above saw x itself */
    for (unsigned m = 0; m < c->k; ++m) {
        const size_t e = idx[m];
        or_matvec_q(c->wtype, gate + e * gate_bytes, xq, I, H, g);
        or_matvec_q(c->wtype, up + e * gate_bytes, xq, I, H, u);
        /* Per-expert biases before the activation (moe.rs:2310-2331). */
        if (gate_b) or_add(g, gate_b + e * I, I, g);
        if (up_b) or_add(u, up_b + e * I, I, u);
        if (c->act == 1) or_swiglu_oai(g, u, I, c->alpha, c->limit, a);
        else or_swiglu(g, u, I, a);
        or_mx8_quantize(a, I, aq);
        or_matvec_q(c->wtype, down + e * down_bytes, aq, H, I, o + m * H);
        /* The down bias sits inside the router's weighting (moe.rs:2362-2372). */
        if (down_b) or_add(o + m * H, down_b + e * H, H, o + m * H);
    }
    /* Combine in router order (moe.rs:2374-2386), on the higher-precision side. */
    for (unsigned m = 0; m < c->k; ++m)
        for (size_t i = 0; i < H; ++i) acc[i] += (double)w[m] * (double)o[m * H + i];
    for (size_t i = 0; i < H; ++i) out[i] = (float)acc[i];
    if (idx_out) memcpy(idx_out, idx, sizeof(uint32_t) * c->k);
    if (w_out) memcpy(w_out, w, sizeof(float) * c->k);
done:
    free(logits);
    free(g);
    free(u);
    free(a);
    free(o);
    free(xq);
    free(aq);
    free(acc);
    return rc;
}

/* ====================================================================================== */
/* synthetic inputs                                                                        */
/* ====================================================================================== */

/* SplitMix64, tests/common/mod.rs:18-24. */
uint64_t or_splitmix64(uint64_t *s) {
    *s += 0x9E3779B97F4A7C15ull;
    uint64_t z = *s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Counter-based draw: the value a SplitMix64 stream seeded with `seed` yields at position i.
 * The device generator computes the same function, so integer-derived synthetic bytes
 * (MXFP4 and Q4_0 payloads) are identical on host and device. */
static inline uint64_t draw(uint64_t seed, uint64_t i) {
    uint64_t s = seed + i * 0x9E3779B97F4A7C15ull;
    return or_splitmix64(&s);
}

void or_synth_mxfp4(uint64_t seed, size_t nblocks, int e_lo, int e_hi, uint8_t *dst) {
    const uint64_t span = (uint64_t)(e_hi - e_lo + 1);
    for (size_t b = 0; b < nblocks; ++b) {
        uint8_t *p = dst + b * 17;
        const uint64_t r0 = draw(seed, 3 * b), r1 = draw(seed, 3 * b + 1), r2 = draw(seed, 3 * b + 2);
        p[0] = (uint8_t)(127 + e_lo + (int)(r0 % span));
        for (int j = 0; j < 8; ++j) {
            p[1 + j] = (uint8_t)(r1 >> (8 * j));
            p[9 + j] = (uint8_t)(r2 >> (8 * j));
        }
    }
}

static inline double unit_open(uint64_t r) { return ((double)(r >> 11) + 1.0) * 0x1.0p-53; } /* (0,1] */
static inline double unit_half(uint64_t r) { return (double)(r >> 11) * 0x1.0p-53; }        /* [0,1) */

void or_synth_q4_0(uint64_t seed, size_t nblocks, double sigma, uint8_t *dst) {
    for (size_t b = 0; b < nblocks; ++b) {
        uint8_t *p = dst + b * 18;
        const uint64_t r0 = draw(seed, 3 * b), r1 = draw(seed, 3 * b + 1), r2 = draw(seed, 3 * b + 2);
        const double u1 = ((double)(r0 >> 32) + 1.0) * 0x1.0p-32;
        const double u2 = (double)(r0 & 0xFFFFFFFFu) * 0x1.0p-32;
        const double z = sqrt(-2.0 * log(u1)) * cos(2.0 * M_PI * u2);
        const uint16_t d = or_f32_to_f16((float)fabs(z * sigma));
        p[0] = (uint8_t)d;
        p[1] = (uint8_t)(d >> 8);
        for (int j = 0; j < 8; ++j) {
            p[2 + j] = (uint8_t)(r1 >> (8 * j));
            p[10 + j] = (uint8_t)(r2 >> (8 * j));
        }
    }
}

/* Box-Muller: pair i uses draws 2i and 2i+1; element 2i takes the cosine branch, 2i+1 the
 * sine branch. */
static double normal_at(uint64_t seed, size_t i) {
    const uint64_t a = draw(seed, 2 * (i / 2)), b = draw(seed, 2 * (i / 2) + 1);
    const double r = sqrt(-2.0 * log(unit_open(a)));
    const double th = 2.0 * M_PI * unit_half(b);
    return (i & 1) ? r * sin(th) : r * cos(th);
}

void or_synth_normal_f32(uint64_t seed, size_t n, double sigma, float *dst) {
    for (size_t i = 0; i < n; ++i) dst[i] = (float)(normal_at(seed, i) * sigma);
}

void or_synth_normal_bf16(uint64_t seed, size_t n, double sigma, uint16_t *dst) {
    for (size_t i = 0; i < n; ++i) dst[i] = or_f32_to_bf16((float)(normal_at(seed, i) * sigma));
}
