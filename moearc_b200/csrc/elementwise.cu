// elementwise.cu — RMSNorm, activations, softmax, residual ops, the MoE combine, per-expert
// bias and RoPE (kernels.cpp:1220-1472, 1590-1735).
#include <cmath>

#include "common.cuh"

using namespace moearc;

namespace {

unsigned grid_1d(moearc_ctx *c, size_t n, unsigned th = 256) {
    size_t g = (n + th - 1) / th;
    const size_t cap = (size_t)c->sm_count * 16;
    return (unsigned)(g < cap ? (g ? g : 1) : cap);
}

#define GRID_STRIDE(i, n) \
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (n); i += (size_t)gridDim.x * blockDim.x)

__device__ __forceinline__ float silu1(float v) { return v / (1.0f + expf(-v)); }

// ggml_swiglu_oai (kernels.cpp:1609-1613): gate clamped above only, up clamped both ways,
// alpha-scaled sigmoid, +1 on the up branch.
__device__ __forceinline__ float swiglu_oai1(float g, float u, float alpha, float limit) {
    const float x = fminf(g, limit);
    const float y = fminf(fmaxf(u, -limit), limit);
    return (x / (1.0f + expf(alpha * (-x)))) * (y + 1.0f);
}

__global__ void k_silu(float *o, const float *x, size_t n) { GRID_STRIDE(i, n) o[i] = silu1(x[i]); }
__global__ void k_swiglu(float *o, const float *g, const float *u, size_t n) {
    GRID_STRIDE(i, n) o[i] = silu1(g[i]) * u[i];
}
__global__ void k_swiglu_oai(float *o, const float *g, const float *u, size_t n, float a, float l) {
    GRID_STRIDE(i, n) o[i] = swiglu_oai1(g[i], u[i], a, l);
}
__global__ void k_add(float *o, const float *a, const float *b, size_t n) { GRID_STRIDE(i, n) o[i] = a[i] + b[i]; }
__global__ void k_mul(float *o, const float *a, const float *b, size_t n) { GRID_STRIDE(i, n) o[i] = a[i] * b[i]; }
__global__ void k_axpy(float *o, const float *x, float alpha, size_t n) { GRID_STRIDE(i, n) o[i] = fmaf(alpha, x[i], o[i]); }
__global__ void k_zero(float *o, size_t n) { GRID_STRIDE(i, n) o[i] = 0.0f; }

// out[i] = sum over m ascending of w[m] * parts[m*n + i], from 0, one fma per step
// (kernels.cpp:1220-1235): the same order as a zero followed by m axpys.
__global__ void k_combine(float *o, const float *parts, const float *w, unsigned k, size_t n) {
    GRID_STRIDE(i, n) {
        float acc = 0.0f;
        for (unsigned m = 0; m < k; ++m) acc = fmaf(w[m], parts[(size_t)m * n + i], acc);
        o[i] = acc;
    }
}

struct idx_table {
    unsigned i[MAX_BATCHED_MATS];
};
__global__ void k_add_bias_id(float *o, const float *bias, idx_table t, size_t n_rows, size_t n) {
    GRID_STRIDE(g, n) {
        const size_t m = g / n_rows, r = g - m * n_rows;
        o[g] += bias[(size_t)t.i[m] * n_rows + r];
    }
}

template <int TH>
__device__ __forceinline__ float block_sum(float v, float *sh) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) sh[w] = v;
    __syncthreads();
    float t = (threadIdx.x < TH / 32) ? sh[threadIdx.x] : 0.f;
    if (w == 0) t = warp_sum(t);
    if (threadIdx.x == 0) sh[0] = t;
    __syncthreads();
    const float r = sh[0];
    __syncthreads();
    return r;
}
template <int TH>
__device__ __forceinline__ float block_max(float v, float *sh) {
    v = warp_max(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) sh[w] = v;
    __syncthreads();
    float t = (threadIdx.x < TH / 32) ? sh[threadIdx.x] : -INFINITY;
    if (w == 0) t = warp_max(t);
    if (threadIdx.x == 0) sh[0] = t;
    __syncthreads();
    const float r = sh[0];
    __syncthreads();
    return r;
}

// RMSNorm (kernels.cpp:1246-1275): f32 sum of squares, y = x / sqrt(mean + eps) * w.
template <int TH>
__global__ void __launch_bounds__(TH) k_rmsnorm(float *out, const float *x, const float *w, size_t n_cols, float eps) {
    __shared__ float sh[32];
    const float *xr = x + blockIdx.x * n_cols;
    float *orow = out + blockIdx.x * n_cols;
    float ss = 0.f;
    for (size_t i = threadIdx.x; i < n_cols; i += TH) ss = fmaf(xr[i], xr[i], ss);
    ss = block_sum<TH>(ss, sh);
    const float scale = 1.0f / sqrtf(ss / (float)n_cols + eps);
    for (size_t i = threadIdx.x; i < n_cols; i += TH) {
        const float v = xr[i] * scale;
        orow[i] = w ? v * w[i] : v;
    }
}

// softmax(x * scale + mask), max-subtracted, a fully masked row comes back as zeros
// (kernels.cpp:1343-1379).
template <int TH>
__global__ void __launch_bounds__(TH) k_softmax(float *out, const float *x, const float *mask, size_t n_cols, float scale) {
    __shared__ float sh[32];
    const size_t base = blockIdx.x * n_cols;
    float mx = -3.402823466e+38f;
    for (size_t i = threadIdx.x; i < n_cols; i += TH)
        mx = fmaxf(mx, x[base + i] * scale + (mask ? mask[base + i] : 0.f));
    mx = block_max<TH>(mx, sh);
    float s = 0.f;
    for (size_t i = threadIdx.x; i < n_cols; i += TH)
        s += expf(x[base + i] * scale + (mask ? mask[base + i] : 0.f) - mx);
    s = block_sum<TH>(s, sh);
    const float inv = 1.0f / fmaxf(s, 1.175494351e-38f);
    for (size_t i = threadIdx.x; i < n_cols; i += TH)
        out[base + i] = expf(x[base + i] * scale + (mask ? mask[base + i] : 0.f) - mx) * inv;
}

// RoPE (kernels.cpp:1399-1472) with the angle in double: pos * theta_scale^(i0/2), the YaRN
// ramp, then cos/sin rounded once to float. The reference kernel's f32 angle loses
// |pos| * 2^-24 radians; this one does not. One thread owns a rotated pair (both of its
// outputs) or one pass-through channel, so dst may alias src.
__global__ void k_rope(float *dst, const float *src, const int *pos, size_t n_tokens, size_t n_heads,
                       size_t head_dim, size_t n_dims, double theta_scale, float freq_scale,
                       float ext_factor, float attn_factor, float corr_lo, float corr_hi, int neox) {
    const size_t half = n_dims / 2;
    const size_t per_head = half + (head_dim - n_dims);
    const size_t n = n_tokens * n_heads * per_head;
    GRID_STRIDE(g, n) {
        const size_t u = g % per_head;
        const size_t th = g / per_head;  // t * n_heads + h
        const size_t t = th / n_heads;
        const float *s = src + th * head_dim;
        float *o = dst + th * head_dim;
        if (u >= half) {
            const size_t d = n_dims + (u - half);
            o[d] = s[d];
            continue;
        }
        const size_t lo = neox ? u : 2 * u;
        const size_t hi = neox ? u + half : 2 * u + 1;
        const size_t i0 = 2 * u;
        const double theta_extrap = (double)pos[t] * pow(theta_scale, (double)i0 / 2.0);
        double theta = (double)freq_scale * theta_extrap;
        double mscale = attn_factor;
        if (ext_factor != 0.0f) {
            const double y = ((double)(i0 / 2) - (double)corr_lo) / fmax(0.001, (double)corr_hi - (double)corr_lo);
            const double ramp = 1.0 - fmin(1.0, fmax(0.0, y));
            const double mix = ramp * (double)ext_factor;
            theta = theta * (1.0 - mix) + theta_extrap * mix;
            mscale *= 1.0 + 0.1 * log(1.0 / (double)freq_scale);
        }
        double sn, cs;
        sincos(theta, &sn, &cs);
        cs *= mscale;
        sn *= mscale;
        const double x0 = s[lo], x1 = s[hi];
        o[lo] = (float)(x0 * cs - x1 * sn);
        o[hi] = (float)(x0 * sn + x1 * cs);
    }
}

}  // namespace

extern "C" {

int moearc_rmsnorm(moearc_ctx *c, float *out, const float *x, const float *weight,
                   unsigned long n_rows, unsigned long n_cols, float eps) {
    if (!c || !out || !x) return ERR;
    if (n_cols == 0) return ERR_ARG;
    if (n_rows == 0) return OK;
    launch_scope ls(c, "rmsnorm", n_rows, 1);
    if (n_cols >= 1024) k_rmsnorm<256><<<(unsigned)n_rows, 256, 0, c->stream>>>(out, x, weight, n_cols, eps);
    else k_rmsnorm<64><<<(unsigned)n_rows, 64, 0, c->stream>>>(out, x, weight, n_cols, eps);
    return ls.finish();
}

int moearc_silu(moearc_ctx *c, float *out, const float *x, unsigned long n) {
    if (!c || !out || !x) return ERR;
    if (n == 0) return OK;
    launch_scope ls(c, "silu", n, 1);
    k_silu<<<grid_1d(c, n), 256, 0, c->stream>>>(out, x, n);
    return ls.finish();
}

int moearc_swiglu(moearc_ctx *c, float *out, const float *gate, const float *up, unsigned long n) {
    if (!c || !out || !gate || !up) return ERR;
    if (n == 0) return OK;
    launch_scope ls(c, "swiglu", n, 1);
    k_swiglu<<<grid_1d(c, n), 256, 0, c->stream>>>(out, gate, up, n);
    return ls.finish();
}

// kernels.cpp:1304-1323: the gate is the first half of gu, the up the second.
int moearc_swiglu_halves(moearc_ctx *c, float *out, const float *gu, unsigned long n) {
    if (!c || !out || !gu) return ERR;
    if (n == 0) return OK;
    launch_scope ls(c, "swiglu_halves", n, 1);
    k_swiglu<<<grid_1d(c, n), 256, 0, c->stream>>>(out, gu, gu + n, n);
    return ls.finish();
}

int moearc_swiglu_oai(moearc_ctx *c, float *out, const float *gate, const float *up,
                      unsigned long n, float alpha, float limit) {
    if (!c || !out || !gate || !up) return ERR;
    if (n == 0) return OK;
    launch_scope ls(c, "swiglu_oai", n, 1);
    k_swiglu_oai<<<grid_1d(c, n), 256, 0, c->stream>>>(out, gate, up, n, alpha, limit);
    return ls.finish();
}

int moearc_swiglu_oai_halves(moearc_ctx *c, float *out, const float *gu, unsigned long n,
                             float alpha, float limit) {
    if (!c || !out || !gu) return ERR;
    if (n == 0) return OK;
    launch_scope ls(c, "swiglu_oai_halves", n, 1);
    k_swiglu_oai<<<grid_1d(c, n), 256, 0, c->stream>>>(out, gu, gu + n, n, alpha, limit);
    return ls.finish();
}

int moearc_softmax(moearc_ctx *c, float *out, const float *x, const float *mask,
                   unsigned long n_rows, unsigned long n_cols, float scale) {
    if (!c || !out || !x) return ERR;
    if (n_cols == 0) return ERR_ARG;
    if (n_rows == 0) return OK;
    launch_scope ls(c, "softmax", n_rows, 1);
    k_softmax<128><<<(unsigned)n_rows, 128, 0, c->stream>>>(out, x, mask, n_cols, scale);
    return ls.finish();
}

int moearc_add(moearc_ctx *c, float *out, const float *a, const float *b, unsigned long n) {
    if (!c || !out || !a || !b) return ERR;
    if (n == 0) return OK;
    launch_scope ls(c, "add", n, 1);
    k_add<<<grid_1d(c, n), 256, 0, c->stream>>>(out, a, b, n);
    return ls.finish();
}

int moearc_mul(moearc_ctx *c, float *out, const float *a, const float *b, unsigned long n) {
    if (!c || !out || !a || !b) return ERR;
    if (n == 0) return OK;
    launch_scope ls(c, "mul", n, 1);
    k_mul<<<grid_1d(c, n), 256, 0, c->stream>>>(out, a, b, n);
    return ls.finish();
}

int moearc_axpy(moearc_ctx *c, float *out, const float *x, float alpha, unsigned long n) {
    if (!c || !out || !x) return ERR;
    if (n == 0) return OK;
    launch_scope ls(c, "axpy", n, 1);
    k_axpy<<<grid_1d(c, n), 256, 0, c->stream>>>(out, x, alpha, n);
    return ls.finish();
}

int moearc_zero(moearc_ctx *c, float *dst, unsigned long n) {
    if (!c || !dst) return ERR;
    if (n == 0) return OK;
    launch_scope ls(c, "zero", n, 1);
    k_zero<<<grid_1d(c, n), 256, 0, c->stream>>>(dst, n);
    return ls.finish();
}

int moearc_moe_combine(moearc_ctx *c, float *out, const float *parts, const float *weights,
                       unsigned int n_mat, unsigned long n) {
    if (!c || !out || !parts || !weights) return ERR;
    if (n == 0) return OK;
    if (n_mat > (unsigned)MAX_BATCHED_MATS) return ERR_ARG;
    launch_scope ls(c, "moe_combine", n, n_mat);
    k_combine<<<grid_1d(c, n), 256, 0, c->stream>>>(out, parts, weights, n_mat, n);
    return ls.finish();
}

int moearc_add_bias_id(moearc_ctx *c, float *out, const float *bias, const unsigned int *idx,
                       unsigned int n_mat, unsigned long n_rows) {
    if (!c || !out || !bias || !idx) return ERR;
    if (n_mat == 0 || n_rows == 0) return OK;
    if (n_mat > (unsigned)MAX_BATCHED_MATS) return ERR_ARG;
    idx_table t{};
    for (unsigned i = 0; i < n_mat; ++i) t.i[i] = idx[i];
    const size_t n = (size_t)n_mat * n_rows;
    launch_scope ls(c, "add_bias_id", n_rows, n_mat);
    k_add_bias_id<<<grid_1d(c, n), 256, 0, c->stream>>>(out, bias, t, n_rows, n);
    return ls.finish();
}

int moearc_rope(moearc_ctx *c, float *dst, const float *src, const int *pos,
                unsigned long n_tokens, unsigned long n_heads, unsigned long head_dim,
                unsigned long n_dims, float freq_base, float freq_scale, float ext_factor,
                float attn_factor, float corr_lo, float corr_hi, int neox) {
    if (!c || !dst || !src || !pos) return ERR;
    if (n_dims == 0 || n_dims % 2 != 0 || n_dims > head_dim) return ERR_ARG;
    if (n_tokens == 0 || n_heads == 0) return OK;
    const double theta_scale = std::pow((double)freq_base, -2.0 / (double)n_dims);
    const size_t n = (size_t)n_tokens * n_heads * (n_dims / 2 + (head_dim - n_dims));
    launch_scope ls(c, "rope", n_heads, (unsigned)n_tokens);
    k_rope<<<grid_1d(c, n), 256, 0, c->stream>>>(dst, src, pos, n_tokens, n_heads, head_dim, n_dims,
                                                 theta_scale, freq_scale, ext_factor, attn_factor,
                                                 corr_lo, corr_hi, neox);
    return ls.finish();
}

}  // extern "C"
